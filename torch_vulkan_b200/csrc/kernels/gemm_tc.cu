// Tensor-core GEMM for sm_100a: tcgen05.mma with TMEM accumulators, operands staged by TMA.
//
// Serves b2_gemm for bf16/f16 (the reference's cooperative-matrix kernel
// vkrt/shaders/mm_coop.comp.in:96-209, 64x64x32 tiles, no double buffering) and b2_int8_gemm,
// the int8-weight linear with the dequantisation fused into the mainloop (new: the reference
// dequantises in a separate pass, vkrt/shaders/dq8.comp.in, then runs the GEMM).
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A and B tiles (128B-swizzled, K- or MN-major) into an S-stage ring
//   warp 1      allocates TMEM; one lane issues tcgen05.mma 128xBNx16 into a double-buffered
//               fp32 accumulator (2*BN TMEM columns) and commits stages / accumulators to mbarriers
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, alpha/beta/bias, round, store to HBM,
//               overlapped with the next tile's mainloop through the second accumulator
//   warps 6..9  (int8 only) dequant: int8 tile (TMA, unswizzled) * scale -> bf16 (RNE) written
//               straight into the swizzled UMMA layout of the B stage, bit-identical to
//               b2_dequant_int8; the bf16 weight never reaches HBM
// Every mbarrier wait is bounded (tc::kWaitLimitNs); on expiry the kernel records an error code,
// drains its own TMA copies (bounded) and frees TMEM before returning.
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace b2 {

bool int8_gemv_applies(const b2_int8_gemm_args* a);  // int8_gemv.cu
int int8_gemv_launch(const b2_int8_gemm_args* a, cudaStream_t st);

// ---- driver entry point for tensor-map encoding (no -lcuda needed) ------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
    (void)cudaGetLastError();
  });
  return fn;
}

// Encodes a 1..5-D tiled tensor map. dims/strides: innermost first; strides in bytes for dims
// 1.. (dim 0 is contiguous). Returns false if the driver rejects it.
bool make_tmap(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle sw) {
  EncodeTiledFn f = encode_fn();
  if (!f) return false;
  if (rank < 1 || rank > 5) return false;
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = f(m, dt, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

constexpr int BM = 128, BK = 64;  // one UMMA M-tile; a CTA tile stacks MSUB of them

struct TcParams {
  int64_t M, N, K, batch;
  int m_tiles, n_tiles, k_blocks;
  int a_mn, b_mn;  // operand is MN-major (else K-major)
  int a3d, b3d;    // tensor map has a batch dimension
  void* c;
  int64_t c_sb, c_sm, c_sn;
  const void* bias;
  int64_t bias_sb, bias_sm, bias_sn;
  int has_bias;
  float alpha, beta;
  int* err;
  // int8 dequant of B
  const void* scale;
  int scale_layout;
  int64_t scale_nb;   // columns of the block-64 scale matrix
  int64_t deq_rows;   // rows of q (output features N of the linear)
  // split-K: work item t covers tile t % tiles and K blocks [split * kps, split * kps + kps) with
  // split = t / tiles; its fp32 partial goes to partial[split][M][N] (no alpha / bias) and
  // gemm_splitk_reduce forms C. ksplit == 1: the epilogue writes C directly.
  int ksplit, kps;
  float* partial;
  // c_tma: C is written through the tensor map tmC (32-column x 32-row boxes, 64 B swizzle) from a
  // per-warp shared-memory staging tile; c3d: that map has a batch dimension
  int c_tma, c3d;
  // fused activation epilogue (bf16 output written through tmC, no split-K):
  //   EPI_GELU:     C = h = acc + bias, and aux = gelu_tanh(h) (both bf16; gelu of the rounded h)
  //   EPI_GELU_BWD: C = bf16(acc) * gelu_tanh'(aux) (aux = the forward's h)
  int epi;
  void* aux;
  int64_t aux_ld;
  // int8 LoRA side path: one extra 64-wide K block after the k_blocks of the weight, whose A tile is
  // the [M, r] activation-side operand (tensor map tmH) and whose B tile the dequant warps copy from
  // lora_b ([N, r] forward, [r, K] transposed); k_total = k_blocks + (lora_r > 0)
  const void* lora_b;
  int64_t lora_b_ld;
  int lora_r, k_total;
  // split-K reduced inside a thread-block cluster (bf16 kernel, 128-column tiles): kcl > 1 CTAs of a
  // cluster each take one K slice of the same tile, leave their fp32 partial tile in shared memory and
  // sum a share of its rows across the cluster through distributed shared memory; no workspace and no
  // second kernel (the partial/gemm_splitk_reduce form above needs both)
  int kcl;
};

enum : int { EPI_NONE = 0, EPI_GELU = 1, EPI_GELU_BWD = 2 };

// GELU with the tanh approximation (Hendrycks & Gimpel 2016): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))),
// tanh from the hardware approximation (relative error ~2^-11, below a bf16 ulp).
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kGeluK0 = 0.7978845608028654f, kGeluK1 = 0.044715f;
__device__ __forceinline__ float gelu_tanh(float x) {
  const float t = tanh_fast(kGeluK0 * (x + kGeluK1 * x * x * x));
  return 0.5f * x * (1.f + t);
}
__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float t = tanh_fast(kGeluK0 * (x + kGeluK1 * x * x * x));
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * kGeluK0 * (1.f + 3.f * kGeluK1 * x * x);
}
__device__ __forceinline__ float bf16_round(float v) { return bf16_bits_to_f32(f32_to_bf16_bits(v)); }

// CG = CTAs per MMA: 1, or 2 for a cluster pair (cta_group::2) whose MMAs are M = 256 with each CTA
// staging its own 128-row A halves and half (BN / 2 rows) of the B tile; the pair covers 2 * BMT x BN.
template <int BN, int DEQ, int MSUB, int CG = 1>
struct Cfg {
  static constexpr int BMT = BM * MSUB;             // rows of the CTA tile (this CTA's share of a pair)
  static constexpr int BNC = BN / CG;               // B rows (output columns) this CTA stages
  static constexpr int A_BYTES = BMT * BK * 2;
  static constexpr int B_BYTES = BNC * BK * 2;
  static constexpr int R_BYTES = DEQ ? BNC * BK : 0;  // raw int8 tile
  // bf16: a TMA stage holds A and B. int8: three rings. A stages (released by the MMAs), raw int8
  // tiles (released by the dequant warps as soon as they have converted one, so those loads run
  // ahead of the MMAs) and NB dequantised bf16 B tiles (released by the MMAs).
  static constexpr int STAGE = A_BYTES + (DEQ ? 0 : B_BYTES);
  // epilogue: per warp one staging buffer (32 rows x 32 16-bit columns) and the tile's bias row
  static constexpr int EPI_BYTES = 4 * 2048 + 4 * 512;
  // int8: the dequant warps form DQG groups that take alternate K blocks, so that one group's waits,
  // proxy fence and barrier arrivals overlap the other group's conversion (one group converting every
  // K block left the MMA waiting on the slowest warp's per-block latency); two groups need four B
  // buffers and four raw tiles, which every shape whose A ring keeps three stages affords
  static constexpr int DQG = (DEQ && (224 * 1024 - 4 * B_BYTES - 4 * R_BYTES - EPI_BYTES) / STAGE >= 3) ? 2 : 1;
  static constexpr int NB = DEQ ? 2 * DQG : 0;  // int8: depth of the dequantised B ring (DEQ = 0: the bf16 path)
  static constexpr int NR = !DEQ ? 0 : DQG == 2 ? 4 : (R_BYTES >= 11264 ? 3 : 4);  // int8: depth of the raw ring
  static_assert(CG == 1 || (DEQ && BNC % 8 == 0), "CTA pairs: int8 kernels, B halves of whole 8-row groups");
  static constexpr int BUDGET = 224 * 1024 - NB * B_BYTES - NR * R_BYTES - EPI_BYTES;
  static constexpr int STAGES = BUDGET / STAGE > 8 ? 8 : BUDGET / STAGE;
  static constexpr int OFF_R = STAGES * STAGE;       // int8: the raw ring
  static constexpr int OFF_B = OFF_R + NR * R_BYTES;  // int8: the B ring
  // int8 dequant warps run pure ALU work; they take warp ids 6-8, 10-12, 14-15 so that none shares
  // a scheduler (warp id % 4) with the MMA-issuing warp 1, whose issue slots they would otherwise
  // take (warps 9 and 13 idle).
  static constexpr int DEQ_WARPS = DEQ ? 8 : 0;
  static constexpr int THREADS = DEQ ? 16 * 32 : 6 * 32;
  static constexpr int R_WARP = 13;  // int8: lane 0 of this otherwise idle warp loads the raw ring
  static constexpr int OFF_EPI = OFF_B + NB * B_BYTES;
  static constexpr int SMEM = OFF_EPI + EPI_BYTES + 1024 + 512;
  static_assert(SMEM <= 232448, "GEMM stages exceed the 227 KB shared-memory limit");
  static_assert(STAGES >= 2, "GEMM needs at least two TMA stages");
  static constexpr uint32_t SUB_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;  // per M sub-tile
  static constexpr uint32_t ACC_COLS = MSUB * SUB_COLS;  // one accumulator (all M sub-tiles)
  static constexpr int NACC = 2 * ACC_COLS <= 512 ? 2 : 1;  // double-buffered when it fits
  static constexpr uint32_t TMEM_COLS = NACC * ACC_COLS;   // (a power of two)
  static_assert(TMEM_COLS <= 512, "accumulators exceed TMEM");
  static_assert(BN % 16 == 0 && BN <= 256, "UMMA N must be a multiple of 16 up to 256");
};

__device__ __forceinline__ uint32_t pack_out(float lo, float hi, bool bf16) {
  if (bf16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int BN, bool BF16, int DEQ, int MSUB, int CG>
__global__ void __launch_bounds__(Cfg<BN, DEQ, MSUB, CG>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmH, TcParams p) {
  using C = Cfg<BN, DEQ, MSUB, CG>;
  constexpr int BNC = C::BNC;
  constexpr int S = C::STAGES;
  constexpr int NDQ = C::DEQ_WARPS * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int NB = C::NB > 0 ? C::NB : 1;
  constexpr int NACC = C::NACC;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_EPI + C::EPI_BYTES);
  uint64_t* full = bars;                // [S]  TMA landed
  uint64_t* empty = bars + S;           // [S]  MMA done reading the stage
  uint64_t* tfull = bars + 2 * S;       // [2]  accumulator ready
  uint64_t* tempty = bars + 2 * S + 2;  // [2]  accumulator drained
  uint64_t* bready = bars + 2 * S + 4;       // [NB] (int8) B buffer dequantised
  uint64_t* bfree = bars + 2 * S + 4 + NB;   // [NB] (int8) MMAs reading the B buffer done
  constexpr int NR = C::NR > 0 ? C::NR : 1;
  uint64_t* rfull = bars + 2 * S + 4 + 2 * NB;        // [NR] (int8) raw tile landed
  uint64_t* rempty = bars + 2 * S + 4 + 2 * NB + NR;  // [NR] (int8) raw tile converted
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4 + 2 * NB + 2 * NR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_tiles = p.m_tiles * p.n_tiles * (int)p.batch;
  const int total_work = total_tiles * p.ksplit;
  // CTA pairs: rank 0 (the leader) issues the MMAs and owns the barriers that gather both CTAs' work;
  // both CTAs of a pair walk the same work items (pair index = blockIdx.x / CG)
  const uint32_t rank = CG == 2 ? tc::cluster_ctarank() : 0u;
  const int unit0 = (int)blockIdx.x / CG, nunits = (int)gridDim.x / CG;
  // cluster split-K: CTA `krank` of cluster c takes the single work item (split krank, tile c)
  const bool kc = DEQ == 0 && CG == 1 && BN == 128 && MSUB == 1 && p.kcl > 1;
  const uint32_t krank = kc ? tc::cluster_ctarank() : 0u;
  const int w0 = kc ? (int)krank * total_tiles + (int)blockIdx.x / p.kcl : unit0;
  const int wstep = kc ? total_work : nunits;
  // leader-side barrier addresses as seen from this CTA (its own shared::cta addresses when CG == 1)
  auto leader_bar = [&](uint64_t* bar) -> uint32_t {
    return CG == 2 ? tc::mapa_shared(tc::smem_u32(bar), 0u) : tc::smem_u32(bar);
  };
  auto wait_bar = [&](uint64_t* bar, uint32_t parity) -> bool { return tc::mbar_wait(bar, parity, p.err); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      // one arrival per dequant warp (of both CTAs of a pair)
      tc::mbar_init(&bready[i], C::DEQ_WARPS > 0 ? C::DEQ_WARPS / C::DQG * CG : 1);
      tc::mbar_init(&bfree[i], 1);
    }
    for (int i = 0; i < NR; ++i) {
      tc::mbar_init(&rfull[i], 1);
      tc::mbar_init(&rempty[i], C::DEQ_WARPS > 0 ? C::DEQ_WARPS / C::DQG : 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&tfull[i], 1);
      tc::mbar_init(&tempty[i], CG == 2 ? 4 * CG : 128);  // pairs: one arrival per epilogue warp
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (CG == 2) tc::cluster_sync();  // both CTAs' barriers initialised before any cross-CTA arrival
  if (warp == 1) {
    if (CG == 2) {
      tc::tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
      tc::tmem_relinquish();
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  auto k_range = [&](int t, int& kb0, int& kb1) {
    kb0 = (t / total_tiles) * p.kps;
    kb1 = kb0 + p.kps < p.k_total ? kb0 + p.kps : p.k_total;
  };
  auto tile_coords = [&](int t, int& m0, int& n0, int& b) {
    t %= total_tiles;
    int per_b = p.m_tiles * p.n_tiles;
    b = t / per_b;
    int r = t - b * per_b;
    int mt = r % p.m_tiles, nt = r / p.m_tiles;
    m0 = mt * C::BMT * CG;  // first row of the (pair) tile; this CTA's rows start at m0 + rank * BMT
    n0 = nt * BN;
  };

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------------------
    if (lane == 0) {
      tc::tma_prefetch_desc(&tmA);
      tc::tma_prefetch_desc(&tmB);
      if (p.lora_r) tc::tma_prefetch_desc(&tmH);
      if (p.c_tma) tc::tma_prefetch_desc(&tmC);
      int stage = 0;
      uint32_t phase = 0;
      int issued[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      bool ok = true;
      const uint32_t full0 = leader_bar(&full[0]);  // the leader's full[s] is full0 + 8 * s
      for (int t = w0; t < total_work && ok; t += wstep) {
        int m0, n0, b, kb0, kb1;
        tile_coords(t, m0, n0, b);
        k_range(t, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bar(&empty[stage], phase ^ 1) || *abort_flag) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE;
          uint8_t* sb = sa + C::A_BYTES;
          const int k0 = kb * BK;
          if (CG == 2) {
            // this CTA's BMT rows of A land in its own shared memory and count on the leader's full
            // barrier, which the leader arms for both CTAs' bytes
            if (rank == 0) tc::mbar_arrive_expect_tx(&full[stage], (uint32_t)(C::STAGE * CG));
            if (kb < p.k_blocks) tc::tma_load_2d_pair(sa, &tmA, full0 + 8u * (uint32_t)stage, k0, m0 + (int)rank * C::BMT);
            else tc::tma_load_2d_pair(sa, &tmH, full0 + 8u * (uint32_t)stage, 0, m0 + (int)rank * C::BMT);
            issued[stage] += 1;
            if (++stage == S) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          const uint32_t bytes = C::STAGE;
          tc::mbar_arrive_expect_tx(&full[stage], bytes);
          if (kb >= p.k_blocks) {  // the LoRA block: A = the [M, r] side-path operand (K-major)
            tc::tma_load_2d(sa, &tmH, &full[stage], 0, m0);
          } else if (!p.a_mn) {  // one box of BMT rows x 64 k
            if (p.a3d) tc::tma_load_3d(sa, &tmA, &full[stage], k0, m0, b);
            else tc::tma_load_2d(sa, &tmA, &full[stage], k0, m0);
          } else {  // BMT/64 boxes of 64 m x 64 k
#pragma unroll
            for (int j = 0; j < C::BMT / 64; ++j) {
              if (p.a3d) tc::tma_load_3d(sa + j * 8192, &tmA, &full[stage], m0 + 64 * j, k0, b);
              else tc::tma_load_2d(sa + j * 8192, &tmA, &full[stage], m0 + 64 * j, k0);
            }
          }
          if (DEQ) {
            // the raw int8 W tiles have their own ring and producer
          } else if (!p.b_mn) {
            if (p.b3d) tc::tma_load_3d(sb, &tmB, &full[stage], k0, n0, b);
            else tc::tma_load_2d(sb, &tmB, &full[stage], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              if (p.b3d) tc::tma_load_3d(sb + j * 8192, &tmB, &full[stage], n0 + 64 * j, k0, b);
              else tc::tma_load_2d(sb + j * 8192, &tmB, &full[stage], n0 + 64 * j, k0);
            }
          }
          issued[stage] += 1;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && rank == 0) {
        // Drain: every issued load completes on its stage's full barrier. Stage s saw issued[s]
        // arms, so its phase count is issued[s]; wait (bounded) for the last one.
        for (int s = 0; s < S; ++s)
          if (issued[s] > 0) tc::mbar_wait(&full[s], (uint32_t)((issued[s] - 1) & 1), nullptr);
      }
      if (ok && CG == 2) {
        // pairs: the leader's last MMA commits arrive on this CTA's empty barriers; wait for them
        // before the CTA can leave, so no arrival reaches a CTA that has exited
        for (int s = 0; s < S; ++s)
          if (issued[s] > 0) wait_bar(&empty[s], (uint32_t)((issued[s] - 1) & 1));
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer ---------------------------------------------
    // (pairs: only the leader issues; the peer's warp 1 only allocates and frees its TMEM)
    if (lane == 0 && rank == 0) {
      // pairs: M = 256 per MMA (128 rows from each CTA), N = BN (BN / 2 B rows from each CTA)
      constexpr uint32_t IDESC_BASE = tc::idesc_f16(BM * CG, BN, BF16, false, false);
      const uint32_t idesc = IDESC_BASE | ((uint32_t)p.a_mn << 15) | ((uint32_t)p.b_mn << 16);
      // K-major: +32 B per 16-element K step inside the 128 B swizzle row (LBO unused);
      // MN-major: +16 rows of 128 B per step, LBO = distance between 64-element MN chunks.
      const uint32_t a_step = p.a_mn ? 2048u : 32u, b_step = p.b_mn ? 2048u : 32u;
      const uint32_t a_lbo = p.a_mn ? 8192u : 16u, b_lbo = p.b_mn ? 8192u : 16u;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      int gk = 0;  // K blocks consumed so far (B ring position)
      bool ok = true;
      for (int t = w0; t < total_work && ok; t += wstep, ++it) {
        int kb0, kb1;
        k_range(t, kb0, kb1);
        const int acc = it % NACC;
        if (!wait_bar(&tempty[acc], ((it / NACC) & 1) ^ 1) || *abort_flag) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t d = tbase + (uint32_t)(acc * C::ACC_COLS);
        for (int kb = kb0; kb < kb1; ++kb) {
          const int bb = gk % NB;
          if (!wait_bar(&full[stage], phase) || (DEQ && !wait_bar(&bready[bb], (uint32_t)((gk / NB) & 1)))) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          uint8_t* sa = smem + stage * C::STAGE;
          uint8_t* sb = DEQ ? smem + C::OFF_B + bb * C::B_BYTES : sa + C::A_BYTES;
          const tc::SDesc ad0 = tc::sdesc_parts(tc::smem_u32(sa), a_lbo, 1024);
          const tc::SDesc bd0 = tc::sdesc_parts(tc::smem_u32(sb), b_lbo, 1024);
          const uint32_t acc0 = kb > kb0 ? 1u : 0u;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t bd = tc::sdesc_at(bd0, k * b_step);
#pragma unroll
            for (int ms = 0; ms < MSUB; ++ms) {  // M sub-tile ms at +ms*16 KB (K-major rows / MN-major chunks)
              if (CG == 2)
                tc::mma_f16_ss_pair(d + ms * C::SUB_COLS, tc::sdesc_at(ad0, ms * 16384 + k * a_step), bd, idesc,
                                    k > 0 ? 1u : acc0);
              else
                tc::mma_f16_ss(d + ms * C::SUB_COLS, tc::sdesc_at(ad0, ms * 16384 + k * a_step), bd, idesc,
                               k > 0 ? 1u : acc0);
            }
          }
          if (CG == 2) {  // release the stage and the B buffer in both CTAs
            tc::mma_commit_pair(&empty[stage], (uint16_t)3);
            tc::mma_commit_pair(&bfree[bb], (uint16_t)3);
          } else {
            tc::mma_commit(&empty[stage]);
            if (DEQ) tc::mma_commit(&bfree[bb]);
          }
          ++gk;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (CG == 2) tc::mma_commit_pair(&tfull[acc], (uint16_t)3);
        else tc::mma_commit(&tfull[acc]);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp < 6) {
    // ------------------------------- epilogue -----------------------------------------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint8_t* stg = smem + C::OFF_EPI + (warp - 2) * 2048;  // this warp's staging buffer
    int it = 0;
    using OutT = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    // a bias that is one row broadcast over M (addmm's usual form) is copied to shared memory per
    // tile before the accumulator is ready, so that its load latency overlaps the mainloop
    OutT* bsm = reinterpret_cast<OutT*>(smem + C::OFF_EPI + 4 * 2048 + (warp - 2) * 512);
    const bool bias_row = p.has_bias && p.bias_sm == 0 && (p.batch == 1 || p.bias_sb == 0) && p.bias_sn == 1 &&
                          (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0;
    const uint32_t tempty0 = leader_bar(&tempty[0]);  // pairs: the leader's tempty[a] is tempty0 + 8 * a
    for (int t = w0; t < total_work; t += wstep, ++it) {
      const int acc = it % NACC;
      int m0, n0, b;
      tile_coords(t, m0, n0, b);
      m0 += (int)rank * C::BMT;  // pairs: this CTA's TMEM holds its own BMT rows of the pair tile
      if (kc) {
        // cluster split-K: this CTA's fp32 partial tile goes into the stage ring, idle now that the
        // CTA's single work item is done ([BMT rows][BN + 4] floats, 16-byte aligned rows);
        // the cluster sums it after the final CTA barrier
        if (!wait_bar(&tfull[acc], (it / NACC) & 1) || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        float* red = reinterpret_cast<float*>(smem);
        const int ncols = (int)(p.N - n0 < BN ? p.N - n0 : BN);
        for (int cc = 0; cc < ncols; cc += 32) {  // warp-uniform
          uint32_t r[32];
          __syncwarp();
          tc::tmem_ld32(tbase + (uint32_t)(acc * C::ACC_COLS + cc) + ((uint32_t)(q * 32) << 16), r);
          tc::tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(red + (q * 32 + lane) * (BN + 4) + cc);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                                 __uint_as_float(r[4 * j + 3]));
        }
        continue;
      }
      if (bias_row) {
        const OutT* bsrc = (const OutT*)p.bias + n0;
        for (int c = lane; c < BN / 8; c += 32) {
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (n0 + c * 8 + 8 <= p.N) {
            v = *reinterpret_cast<const uint4*>(bsrc + c * 8);
          } else {
            OutT* h = reinterpret_cast<OutT*>(&v);
            for (int e = 0; e < 8; ++e)
              if (n0 + c * 8 + e < p.N) h[e] = bsrc[c * 8 + e];
          }
          *reinterpret_cast<uint4*>(bsm + c * 8) = v;
        }
        __syncwarp();
      }
      if (!wait_bar(&tfull[acc], (it / NACC) & 1) || *abort_flag) {
        *abort_flag = 1;
        break;
      }
      tc::tc_fence_after();
#pragma unroll 1
      for (int ms = 0; ms < MSUB; ++ms) {
        const int64_t row = m0 + ms * BM + q * 32 + lane;
        const bool row_ok = row < p.M;
        OutT* crow = (OutT*)p.c + b * p.c_sb + row * p.c_sm;
        const OutT* brow = (const OutT*)p.bias + b * p.bias_sb + row * p.bias_sm;
        // one chunk of W (32 or 16) accumulator columns: TMEM -> registers -> C (or the split-K partial)
        auto chunk = [&](auto wc, int cc) {
          constexpr int W = decltype(wc)::value;
          uint32_t r[W];
          __syncwarp();
          const uint32_t taddr = tbase + (uint32_t)(acc * C::ACC_COLS + ms * C::SUB_COLS + cc) + ((uint32_t)(q * 32) << 16);
          if constexpr (W == 32) tc::tmem_ld32(taddr, r);
          else tc::tmem_ld16(taddr, r);
          tc::tmem_wait_ld();
          const int64_t col0 = n0 + cc;
          if (col0 >= p.N) return;  // warp-uniform
          if constexpr (W == 32) {
            if (p.c_tma == 2) {
              // fp32 split-K partial: two 32-row x 16-column boxes through the staging tile
              const int32_t r0 = (int32_t)(m0 + ms * BM + q * 32);
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                if (lane == 0) tc::bulk_wait_read0();
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  *reinterpret_cast<uint4*>(stg + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                      make_uint4(r[16 * hh + 4 * j], r[16 * hh + 4 * j + 1], r[16 * hh + 4 * j + 2], r[16 * hh + 4 * j + 3]);
                tc::fence_async_shared();
                __syncwarp();
                if (lane == 0) {
                  tc::tma_store_3d(&tmC, stg, (int32_t)(col0 + 16 * hh), r0, t / total_tiles);
                  tc::bulk_commit();
                }
              }
              return;
            }
            if (p.c_tma == 1 && !p.partial) {
              // bias / alpha in registers, bf16 row into the swizzled staging tile, one TMA store
              // of the warp's 32 x 32 box (rows past M and columns past N are clipped by the store)
              // in place: r[j] holds the fp32 bits of alpha * acc + beta * bias
#pragma unroll
              for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(p.alpha * __uint_as_float(r[j]));
              if (bias_row) {
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                  const uint4 raw = reinterpret_cast<const uint4*>(bsm + cc)[q4];
                  const OutT* h = reinterpret_cast<const OutT*>(&raw);
#pragma unroll
                  for (int e = 0; e < 8; ++e)
                    r[8 * q4 + e] = __float_as_uint(__uint_as_float(r[8 * q4 + e]) + p.beta * to_f32(h[e]));
                }
              } else if (p.has_bias && row_ok) {
                const OutT* bp = brow + col0 * p.bias_sn;
                if (p.bias_sn == 1 && col0 + 32 <= p.N && (reinterpret_cast<uintptr_t>(bp) & 15) == 0) {
#pragma unroll
                  for (int q4 = 0; q4 < 4; ++q4) {
                    const uint4 raw = reinterpret_cast<const uint4*>(bp)[q4];
                    const OutT* h = reinterpret_cast<const OutT*>(&raw);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                      r[8 * q4 + e] = __float_as_uint(__uint_as_float(r[8 * q4 + e]) + p.beta * to_f32(h[e]));
                  }
                } else {
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    if (col0 + j < p.N)
                      r[j] = __float_as_uint(__uint_as_float(r[j]) + p.beta * to_f32(brow[(col0 + j) * p.bias_sn]));
                }
              }
              if (p.epi != EPI_NONE && row_ok) {
                // fused GELU: each lane's 32 columns of its row are 64 contiguous bytes of aux
                OutT* arow = (OutT*)p.aux + row * p.aux_ld + col0;
                const bool full = col0 + 32 <= p.N && (reinterpret_cast<uintptr_t>(arow) & 15) == 0;
                if (p.epi == EPI_GELU) {  // aux = gelu(h) of the bf16-rounded h the main output holds
                  uint32_t a[16];
#pragma unroll
                  for (int j = 0; j < 16; ++j)
                    a[j] = pack_out(gelu_tanh(bf16_round(__uint_as_float(r[2 * j]))),
                                    gelu_tanh(bf16_round(__uint_as_float(r[2 * j + 1]))), BF16);
                  if (full) {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                      reinterpret_cast<uint4*>(arow)[j] = make_uint4(a[4 * j], a[4 * j + 1], a[4 * j + 2], a[4 * j + 3]);
                  } else {
                    const OutT* ah = reinterpret_cast<const OutT*>(a);
                    for (int j = 0; j < 32 && col0 + j < p.N; ++j) arow[j] = ah[j];
                  }
                } else {  // EPI_GELU_BWD: dh = bf16(da) * gelu'(h), h read from aux
                  float hv[32];
                  if (full) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                      const uint4 raw = reinterpret_cast<const uint4*>(arow)[j];
                      const OutT* hh = reinterpret_cast<const OutT*>(&raw);
#pragma unroll
                      for (int e = 0; e < 8; ++e) hv[8 * j + e] = to_f32(hh[e]);
                    }
                  } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) hv[j] = col0 + j < p.N ? to_f32(arow[j]) : 0.f;
                  }
#pragma unroll
                  for (int j = 0; j < 32; ++j)
                    r[j] = __float_as_uint(bf16_round(__uint_as_float(r[j])) * gelu_tanh_grad(hv[j]));
                }
              }
              uint8_t* buf = stg;
              if (lane == 0) tc::bulk_wait_read0();  // the previous chunk's store has read the buffer
              __syncwarp();
              uint8_t* rowp = buf + lane * 64;
#pragma unroll
              for (int j = 0; j < 4; ++j)  // 64 B swizzle: 16 B chunk j of row r at (j ^ ((r >> 1) & 3))
                *reinterpret_cast<uint4*>(rowp + ((j ^ ((lane >> 1) & 3)) << 4)) =
                    make_uint4(pack_out(__uint_as_float(r[8 * j]), __uint_as_float(r[8 * j + 1]), BF16),
                               pack_out(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]), BF16),
                               pack_out(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]), BF16),
                               pack_out(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]), BF16));
              tc::fence_async_shared();
              __syncwarp();
              if (lane == 0) {
                const int32_t r0 = (int32_t)(m0 + ms * BM + q * 32);
                if (p.c3d) tc::tma_store_3d(&tmC, buf, (int32_t)col0, r0, b);
                else tc::tma_store_2d(&tmC, buf, (int32_t)col0, r0);
                tc::bulk_commit();
              }
              return;
            }
          }
          if (!row_ok) return;
          if (p.partial) {  // split-K partial tile, fp32 [split][M][N]
            float* prow = p.partial + ((int64_t)(t / total_tiles) * p.M + row) * p.N + col0;
            if (col0 + W <= p.N && (p.N & 3) == 0) {
#pragma unroll
              for (int j = 0; j < W / 4; ++j)
                reinterpret_cast<float4*>(prow)[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            } else {
              for (int j = 0; j < W && col0 + j < p.N; ++j) prow[j] = __uint_as_float(r[j]);
            }
            return;
          }
          float v[W];
#pragma unroll
          for (int j = 0; j < W; ++j) v[j] = p.alpha * __uint_as_float(r[j]);
          if (bias_row) {
#pragma unroll
            for (int q4 = 0; q4 < W / 8; ++q4) {
              const uint4 raw = reinterpret_cast<const uint4*>(bsm + cc)[q4];
              const OutT* h = reinterpret_cast<const OutT*>(&raw);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[8 * q4 + e] += p.beta * to_f32(h[e]);
            }
          } else if (p.has_bias) {
            const OutT* bp = brow + col0 * p.bias_sn;
            if (p.bias_sn == 1 && col0 + W <= p.N && (reinterpret_cast<uintptr_t>(bp) & 15) == 0) {
              // a contiguous bias row segment (addmm with a full-matrix or broadcast-row bias): 16 B loads
#pragma unroll
              for (int q4 = 0; q4 < W / 8; ++q4) {
                const uint4 raw = reinterpret_cast<const uint4*>(bp)[q4];
                const OutT* h = reinterpret_cast<const OutT*>(&raw);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[8 * q4 + e] += p.beta * to_f32(h[e]);
              }
            } else {
#pragma unroll
              for (int j = 0; j < W; ++j)
                if (col0 + j < p.N) v[j] += p.beta * to_f32(brow[(col0 + j) * p.bias_sn]);
            }
          }
          const bool vec = (p.c_sn == 1) && (col0 + W <= p.N) && ((reinterpret_cast<uintptr_t>(crow + col0) & 15) == 0);
          if (vec) {
            uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
            for (int j = 0; j < W / 8; ++j)
              dst[j] = make_uint4(pack_out(v[8 * j], v[8 * j + 1], BF16), pack_out(v[8 * j + 2], v[8 * j + 3], BF16),
                                  pack_out(v[8 * j + 4], v[8 * j + 5], BF16), pack_out(v[8 * j + 6], v[8 * j + 7], BF16));
          } else {
#pragma unroll
            for (int j = 0; j < W; ++j)
              if (col0 + j < p.N) crow[(col0 + j) * p.c_sn] = from_f32<OutT>(v[j]);
          }
        };
#pragma unroll 1
        for (int ch = 0; ch < BN / 32; ++ch) chunk(std::integral_constant<int, 32>{}, ch * 32);
        if constexpr (BN % 32 != 0) chunk(std::integral_constant<int, 16>{}, (BN / 32) * 32);
      }
      tc::tc_fence_before();
      if (CG == 2) {  // one arrival per warp on the leader's barrier, after every lane's TMEM reads
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cluster(tempty0 + 8u * (uint32_t)acc);
      } else {
        tc::mbar_arrive(&tempty[acc]);
      }
    }
    if (lane == 0) tc::bulk_wait0();  // every C store of this warp complete before the CTA exits
  } else if (DEQ && warp == C::R_WARP) {
    // ------------------------------- int8 raw-tile producer ----------------------------------
    if (lane == 0) {
      int rs = 0;
      uint32_t rph = 0;
      int issued[4] = {0, 0, 0, 0};
      bool ok = true;
      for (int t = w0; t < total_work && ok; t += wstep) {
        int m0, n0, b, kb0, kb1;
        tile_coords(t, m0, n0, b);
        k_range(t, kb0, kb1);
        n0 += (int)rank * BNC;  // pairs: this CTA stages B rows [n0 + rank * BN/2, + BN/2)
        for (int kb = kb0; kb < kb1 && kb < p.k_blocks; ++kb) {  // (the LoRA block has no int8 tile)
          if (!tc::mbar_wait(&rempty[rs], rph ^ 1, p.err) || *abort_flag) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          uint8_t* sr = smem + C::OFF_R + rs * C::R_BYTES;
          tc::mbar_arrive_expect_tx(&rfull[rs], (uint32_t)C::R_BYTES);
          // raw int8 W tile: forward box {64 (k), BNC (n)}; transposed box {BNC (k_feat), 64 (n_feat)}
          if (!p.b_mn) tc::tma_load_2d(sr, &tmB, &rfull[rs], kb * BK, n0);
          else tc::tma_load_2d(sr, &tmB, &rfull[rs], n0, kb * BK);
          issued[rs] += 1;
          if (++rs == NR) {
            rs = 0;
            rph ^= 1;
          }
        }
      }
      if (!ok)
        for (int r = 0; r < NR; ++r)
          if (issued[r] > 0) tc::mbar_wait(&rfull[r], (uint32_t)((issued[r] - 1) & 1), nullptr);
    }
  } else if (DEQ && (warp & 3) != 1) {
    // ------------------------------- int8 dequant -------------------------------------------
    const int dw = warp - 6 - (warp > 9 ? 1 : 0) - (warp > 13 ? 1 : 0);  // 0 .. 7
    constexpr int DQG = C::DQG;
    constexpr int NDQG = (NDQ > 0 ? NDQ : DQG) / DQG;  // threads of one group
    const int grp = dw / (C::DEQ_WARPS / DQG);          // this warp's group: K blocks gk with gk % DQG == grp
    const int dt = (dw % (C::DEQ_WARPS / DQG)) * 32 + lane;  // 0 .. NDQG-1
    int gk = 0;  // K blocks staged so far (B ring position)
    int gr = 0;  // int8 tiles converted so far (raw ring position; the LoRA block has none)
    constexpr int FIPT = (BNC * 4 + NDQG - 1) / NDQG;  // forward items per thread
    float fsc[FIPT];
    constexpr int IPT = (64 * (BNC / 16) + NDQG - 1) / NDQG;  // transposed items per thread
    float sc[IPT];
    const uint32_t bready0 = leader_bar(&bready[0]);  // pairs: the leader's bready[i] is bready0 + 8 * i
    bool ok = true;
    for (int t = w0; t < total_work && ok; t += wstep) {
      int m0, n0, b, kb0, kb1;
      tile_coords(t, m0, n0, b);
      k_range(t, kb0, kb1);
      n0 += (int)rank * BNC;  // pairs: this CTA dequantises B rows [n0 + rank * BN/2, + BN/2)
      for (int kb = kb0; kb < kb1; ++kb) {
        const bool lora_blk = kb >= p.k_blocks;
        const bool mine = DQG == 1 || gk % DQG == grp;
        // forward scales, loaded before the waits so that their latency overlaps them: block-64
        // scales change with the K block, per-row scales are loaded once per tile (by every group)
        if (!p.b_mn && !lora_blk && ((p.scale_layout == 0 && mine) || (p.scale_layout != 0 && kb == kb0))) {
#pragma unroll
          for (int u = 0; u < FIPT; ++u) {  // every scale load in flight before the first is used
            const int i = dt + u * NDQG;
            const int64_t gn = (int64_t)n0 + (i >> 2);
            fsc[u] = 0.f;
            if (i < BNC * 4 && gn < p.deq_rows)
              fsc[u] = p.scale_layout == 0
                           ? bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(p.scale)[gn * p.scale_nb + kb])
                           : reinterpret_cast<const float*>(p.scale)[gn];
          }
        }
        if (!mine) {  // the other group's K block
          ++gk;
          if (!lora_blk) ++gr;
          continue;
        }
        const int rs = gr % NR;
        if (p.b_mn && !lora_blk) {
          // transposed form: the scale of reduction row nf = kb * 64 + i, loaded before the waits
#pragma unroll
          for (int u = 0; u < IPT; ++u) {  // every scale load in flight before the first is used
            const int e = dt + u * NDQG;
            const int i = e / (BNC / 16), qd = e % (BNC / 16);
            const int64_t nf = (int64_t)kb * BK + i;   // n_feat (the reduction index)
            const int64_t kf = (int64_t)n0 + qd * 16;  // first k_feat of the 16
            sc[u] = 0.f;
            if (e < 64 * (BNC / 16) && nf < p.deq_rows)
              sc[u] = p.scale_layout == 0
                          ? bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(p.scale)[nf * p.scale_nb + (kf >> 6)])
                          : reinterpret_cast<const float*>(p.scale)[nf];
          }
        }
        if (!lora_blk && (!tc::mbar_wait(&rfull[rs], (uint32_t)((gr / NR) & 1), p.err) || *abort_flag)) {
          ok = false;
          break;
        }
        const int bb = gk % NB;
        if (!wait_bar(&bfree[bb], (uint32_t)(((gk / NB) & 1) ^ 1))) {
          ok = false;
          break;
        }
        uint8_t* sb = smem + C::OFF_B + bb * C::B_BYTES;
        const uint8_t* sr = smem + C::OFF_R + rs * C::R_BYTES;
        if (lora_blk) {
          // the LoRA block: the bf16 side-path weight copied (rows beyond r as zeros) into the same
          // swizzled layout the dequantised tiles use; forward: lora_b [N, r], row n of the B tile is
          // lora_b row n0 + n; transposed: lora_b [r, K], reduction row i of the tile is lora_b row i
          const __nv_bfloat16* lb = reinterpret_cast<const __nv_bfloat16*>(p.lora_b);
          if (!p.b_mn) {
            for (int e = dt; e < BNC * 8; e += NDQG) {
              const int n = e >> 3, c = e & 7;  // 16 B chunk c = k 8c..8c+7 of row n
              const int64_t gn = (int64_t)n0 + n;
              uint4 v = make_uint4(0u, 0u, 0u, 0u);
              if (c * 8 < p.lora_r && gn < p.N) v = *reinterpret_cast<const uint4*>(lb + gn * p.lora_b_ld + c * 8);
              *reinterpret_cast<uint4*>(sb + n * 128 + ((c ^ (n & 7)) << 4)) = v;
            }
          } else {
            for (int e = dt; e < 64 * (BNC / 8); e += NDQG) {
              const int i = e / (BNC / 8), g8 = e % (BNC / 8);  // reduction row i, output columns 8*g8..
              const int64_t col = (int64_t)n0 + g8 * 8;
              uint4 v = make_uint4(0u, 0u, 0u, 0u);
              if (i < p.lora_r && col < p.N) v = *reinterpret_cast<const uint4*>(lb + (int64_t)i * p.lora_b_ld + col);
              const int chunk = (g8 * 8) >> 6, g0 = ((g8 * 8) & 63) >> 3;
              *reinterpret_cast<uint4*>(sb + chunk * 8192 + i * 128 + ((g0 ^ (i & 7)) << 4)) = v;
            }
          }
        } else if (!p.b_mn) {
          // forward: raw [BNC rows n][64 bytes k]; B stage K-major SW128: row n at n*128 B,
          // 16 B chunk c (k 8c..8c+7) at ((c ^ (n & 7)) * 16).
#pragma unroll
          for (int u = 0; u < FIPT; ++u) {
            const int i = dt + u * NDQG;
            if (i >= BNC * 4) break;
            const int n = i >> 2, j = i & 3;  // 16 int8 = k 16j..16j+15
            const float s = fsc[u];
            const int4 raw = *reinterpret_cast<const int4*>(sr + n * 64 + j * 16);
            uint32_t w[8];
            dequant16(raw, s, w);
            uint8_t* rowp = sb + n * 128;
            const int c0 = 2 * j, c1 = 2 * j + 1;
            *reinterpret_cast<uint4*>(rowp + ((c0 ^ (n & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(rowp + ((c1 ^ (n & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
          }
        } else {
          // backward: raw [64 rows i (n_feat)][BNC bytes (k_feat = n_gemm)]; B stage MN-major SW128:
          // chunk j = n_gemm/64 at j*8192, row i at i*128, 16 B granule g at ((g ^ (i & 7)) * 16).
#pragma unroll
          for (int u = 0; u < IPT; ++u) {
            const int e = dt + u * NDQG;
            if (e >= 64 * (BNC / 16)) break;
            const int i = e / (BNC / 16), qd = e % (BNC / 16);
            const float s = sc[u];
            const int4 raw = *reinterpret_cast<const int4*>(sr + i * BNC + qd * 16);
            uint32_t w[8];
            dequant16(raw, s, w);
            const int chunk = (qd * 16) >> 6, g0 = ((qd * 16) & 63) >> 3;
            uint8_t* rowp = sb + chunk * 8192 + i * 128;
            *reinterpret_cast<uint4*>(rowp + ((g0 ^ (i & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(rowp + (((g0 + 1) ^ (i & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
          }
        }
        // every thread's B stores visible to the tensor core's (async proxy) reads; the raw tile and
        // the B buffer are signalled once per warp
        tc::fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          if (!lora_blk) tc::mbar_arrive(&rempty[rs]);
          if (CG == 2) tc::mbar_arrive_cluster(bready0 + 8u * (uint32_t)bb);
          else tc::mbar_arrive(&bready[bb]);
        }
        ++gk;
        if (!lora_blk) ++gr;
      }
    }
    if (ok && CG == 2 && dw == 0 && lane == 0) {
      // pairs: the leader's last commits arrive on this CTA's bfree barriers; wait for them before
      // the CTA can leave
      for (int i = 0; i < NB && i < gk; ++i) {
        const int last = gk - 1 - ((gk - 1 - i) % NB);  // the last use of buffer i
        wait_bar(&bfree[i], (uint32_t)((last / NB) & 1));
      }
    }
  }

  // Warps 0 and 1 reach here diverged (lane 0 ran the producer / MMA role): reconverge each warp
  // before the CTA barrier, which is an aligned barrier and must be executed by whole warps.
  __syncwarp();
  tc::tc_fence_before();
  __syncthreads();
  // pairs: neither CTA frees its TMEM or leaves while the other may still arrive on its barriers
  if (CG == 2) tc::cluster_sync();
  if (kc) {
    // every CTA's partial tile is in its shared memory (barrier.cluster arrive.release / wait.acquire);
    // CTA krank sums rows [krank * rows, (krank + 1) * rows) over the kcl partials in rank order
    // (deterministic) through distributed shared memory and writes them to C with alpha and the bias
    tc::cluster_sync();
    if (warp >= 2 && warp < 6 && !*abort_flag) {
      using OutT = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      int m0, n0, b;
      tile_coords(w0, m0, n0, b);
      const int ncols = (int)(p.N - n0 < BN ? p.N - n0 : BN);
      const int rows = (C::BMT + p.kcl - 1) / p.kcl;
      const int r0 = (int)krank * rows, r1 = r0 + rows < C::BMT ? r0 + rows : C::BMT;
      uint32_t src[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) src[k] = tc::mapa_shared(tc::smem_u32(smem), (uint32_t)(k < p.kcl ? k : 0));
      // thread = (row, 4 columns): eight 16-byte loads (one per cluster rank) in flight at once
      const int nc4 = (ncols + 3) >> 2;
      for (int e = (int)threadIdx.x - 64; e < (r1 - r0) * nc4; e += 128) {
        const int rr = r0 + e / nc4, col = (e - (e / nc4) * nc4) * 4;
        const int64_t row = m0 + rr;
        if (row >= p.M) continue;
        const uint32_t off = (uint32_t)((rr * (BN + 4) + col) * 4);
        float4 part[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k < p.kcl) part[k] = tc::ld_shared_cluster_v4(src[k] + off);
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k < p.kcl) sum[0] += part[k].x, sum[1] += part[k].y, sum[2] += part[k].z, sum[3] += part[k].w;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (col + j >= ncols) break;
          float v = p.alpha * sum[j];
          if (p.has_bias) v += p.beta * to_f32(((const OutT*)p.bias)[row * p.bias_sm + (n0 + col + j) * p.bias_sn]);
          OutT o;
          if constexpr (BF16) o = __float2bfloat16_rn(v);
          else o = __float2half_rn(v);
          ((OutT*)p.c)[row * p.c_sm + (n0 + col + j) * p.c_sn] = o;
        }
      }
    }
    tc::cluster_sync();  // no CTA leaves while another may still read its partial
  }
  if (warp == 1) {
    __syncwarp();
    tc::tc_fence_after();
    if (CG == 2) tc::tmem_dealloc_pair(tbase, C::TMEM_COLS);
    else tc::tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// ---- host side ----------------------------------------------------------------------------------

bool tma_ok_stride(int64_t s_elems, int esz) { return ((s_elems * esz) % 16) == 0; }

template <int BN, bool BF16, int DEQ, int MSUB, int CG = 1>
int launch_kernel(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc_, const TcParams& p, cudaStream_t st,
                  const char* name, const CUtensorMap* th = nullptr) {
  CUtensorMap th0;  // the LoRA operand's map (unused without a side path)
  if (!th) {
    memset(&th0, 0, sizeof(th0));
    th = &th0;
  }
  using C = Cfg<BN, DEQ, MSUB, CG>;
  auto kern = gemm_tc_kernel<BN, BF16, DEQ, MSUB, CG>;
  static int max_pairs = 0;  // set once per process (single device per process)
  static bool attr_set = false;
  if (!attr_set) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                            "cudaFuncSetAttribute(gemm_tc)"))
      return rc;
    if (CG == 2) {
      // persistent grid: as many CTA pairs as the GPU can hold at once (one CTA per SM)
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * device_info().sm_count);
      cfg.blockDim = dim3(C::THREADS);
      cfg.dynamicSmemBytes = C::SMEM;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2, at[0].val.clusterDim.y = 1, at[0].val.clusterDim.z = 1;
      cfg.attrs = at, cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = device_info().sm_count / 2;
      }
      max_pairs = n;
    }
    attr_set = true;
  }
  const int tiles = p.m_tiles * p.n_tiles * (int)p.batch * p.ksplit;
  if (CG == 1 && p.kcl > 1) {
    // cluster split-K: one CTA per (tile, K slice), the kcl slices of a tile in one cluster
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)tiles);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)p.kcl, at[0].val.clusterDim.y = 1, at[0].val.clusterDim.z = 1;
    cfg.attrs = at, cfg.numAttrs = 1;
    cudaError_t e;
    {
      LaunchScope ls("gemm_tc_bn128_kcluster", st);
      e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc_, *th, p);
    }
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail_cuda(e, "gemm_tc_bn128_kcluster");
    }
    return after_launch("gemm_tc_bn128_kcluster");
  }
  if (CG == 2) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * std::min(tiles, max_pairs)));
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2, at[0].val.clusterDim.y = 1, at[0].val.clusterDim.z = 1;
    cfg.attrs = at, cfg.numAttrs = 1;
    cudaError_t e;
    {
      LaunchScope ls(name, st);
      e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc_, *th, p);
    }
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail_cuda(e, name);
    }
    return after_launch(name);
  }
  int grid = std::min(tiles, device_info().sm_count);
  LaunchScope ls(name, st);
  kern<<<grid, C::THREADS, C::SMEM, st>>>(ta, tb, tc_, *th, p);
  return after_launch(name);
}

// C = alpha * sum_s partial[s] + beta * bias, converted to the output type with C's strides.
template <typename OutT>
__global__ void __launch_bounds__(256) gemm_splitk_reduce(const float* __restrict__ part, int ksplit, int64_t M,
                                                          int64_t N, OutT* __restrict__ c, int64_t c_sm, int64_t c_sn,
                                                          const OutT* __restrict__ bias, int64_t bias_sm,
                                                          int64_t bias_sn, float alpha, float beta) {
  const int64_t total = M * N;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if ((N & 3) == 0) {
    // four consecutive columns of one row per thread, the partial loads of four slices in flight at once
    for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < total; i += stride * 4) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      int s = 0;
      for (; s + 4 <= ksplit; s += 4) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const float4*>(part + (int64_t)(s + u) * total + i);
#pragma unroll
        for (int u = 0; u < 4; ++u) acc.x += v[u].x, acc.y += v[u].y, acc.z += v[u].z, acc.w += v[u].w;
      }
      for (; s < ksplit; ++s) {
        const float4 v = *reinterpret_cast<const float4*>(part + (int64_t)s * total + i);
        acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
      }
      const int64_t m = i / N, n = i % N;
      const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = alpha * a4[e];
        if (bias) v += beta * to_f32(bias[m * bias_sm + (n + e) * bias_sn]);
        c[m * c_sm + (n + e) * c_sn] = from_f32<OutT>(v);
      }
    }
    return;
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    float acc = 0.f;
    for (int s = 0; s < ksplit; ++s) acc += part[(int64_t)s * total + i];
    const int64_t m = i / N, n = i % N;
    float v = alpha * acc;
    if (bias) v += beta * to_f32(bias[m * bias_sm + n * bias_sn]);
    c[m * c_sm + n * c_sn] = from_f32<OutT>(v);
  }
}

// Split-K plan: GEMMs with too few output tiles to fill the GPU but a long reduction (the LoRA
// projections: N or M = 16, K = 2048..4096) give each SM a slice of K instead.
void splitk_plan(int64_t tiles, int k_blocks, int& ksplit, int& kps) {
  const int sms = device_info().sm_count > 0 ? device_info().sm_count : 148;
  ksplit = 1, kps = k_blocks;
  if (tiles * 2 > sms || k_blocks < 8) return;
  int want = (int)std::min<int64_t>(sms / tiles, k_blocks / 4);  // at least 4 K blocks per slice
  if (want < 2) return;
  kps = (k_blocks + want - 1) / want;
  ksplit = (k_blocks + kps - 1) / kps;
}

// Wave-quantisation aware choice among 128x128, 128x256 and 256x256 CTA tiles, each weighted by its
// measured per-SM rate (wider tiles need less operand bandwidth per FLOP).
struct TileChoice {
  int bn, msub;
};
TileChoice pick_tile(int64_t M, int64_t N, int64_t batch) {
  const int sms = device_info().sm_count > 0 ? device_info().sm_count : 148;
  static const int forced = [] {  // B2_GEMM_TILE=<bn>x<msub> pins the tile (measurement sweeps)
    const char* e = getenv("B2_GEMM_TILE");
    int bn = 0, ms = 0;
    return (e && sscanf(e, "%dx%d", &bn, &ms) == 2) ? bn * 10 + ms : 0;
  }();
  struct Opt {
    int bn, msub;
    double eff;
  };
  const Opt opts[] = {{256, 2, 1.1}, {256, 1, 1.0}, {128, 1, 0.65}};
  TileChoice best{256, 1};
  double best_score = -1.0;
  for (const Opt& o : opts) {
    const int64_t tiles = ((M + BM * o.msub - 1) / (BM * o.msub)) * ((N + o.bn - 1) / o.bn) * batch;
    const int64_t waves = (tiles + sms - 1) / sms;
    double score = (double)M * N * batch / ((double)waves * sms * BM * o.msub * o.bn) * o.eff;
    if (forced) score = forced == o.bn * 10 + o.msub ? 1e9 : -1.0;
    if (score > best_score) best_score = score, best = TileChoice{o.bn, o.msub};
  }
  return best;
}

// How many clusters of ks CTAs of the bf16 128x128 kernel the GPU holds at once (cached per ks).
int kcluster_capacity(int ks) {
  static int cap[9] = {0};
  if (ks < 2 || ks > 8) return 0;
  if (cap[ks] == 0) {
    using C = Cfg<128, 0, 1, 1>;
    auto kern = gemm_tc_kernel<128, true, 0, 1, 1>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(ks * 64));
      cfg.blockDim = dim3(C::THREADS);
      cfg.dynamicSmemBytes = C::SMEM;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = (unsigned)ks, at[0].val.clusterDim.y = 1, at[0].val.clusterDim.z = 1;
      cfg.attrs = at, cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    (void)cudaGetLastError();
    cap[ks] = n > 0 ? n : -1;
  }
  return cap[ks] > 0 ? cap[ks] : 0;
}

// Split-K reduced inside a cluster (TcParams::kcl; B2_GEMM_KCLUSTER=0 turns it off): GEMMs with few
// 128x128 output tiles and a long K (the LoRA down-projections and weight gradients: N or M = 16-64) whose
// splitk_plan split fits a portable cluster (<= 8) take it as clusters of K slices that sum their tile
// through distributed shared memory, without a workspace or a second kernel. Measured against the
// workspace + gemm_splitk_reduce form (graphs of back-to-back calls): 1024x2048x48 8.85 -> 7.73 us,
// 4096x2048x48 10.8 -> 10.2, 4096x8192x16 21.6 -> 20.5, 6144x1024x48 (MN-major A, 48 clusters of 3)
// 10.4 -> 10.6; in the DiT step (graphed, A/B twice each) configs[3] block 0.781 -> 0.776 ms, configs[4]
// stack 65.37 -> 65.26 ms.
bool kcluster_plan(const b2_gemm_args* a, const TileChoice& t, int& ks, int& kps) {
  static const bool on = [] {
    const char* e = getenv("B2_GEMM_KCLUSTER");
    return !(e && e[0] == '0');
  }();
  ks = 1, kps = 0;
  if (!on || a->batch != 1 || t.bn != 128 || t.msub != 1 || a->K <= 0) return false;
  const int64_t tiles = ((a->M + BM - 1) / BM) * ((a->N + 127) / 128);
  const int k_blocks = (int)((a->K + BK - 1) / BK);
  splitk_plan(tiles, k_blocks, ks, kps);
  // a split wider than a cluster would have to be capped, losing the parallelism the split is for
  if (ks <= 1 || ks > 8 || tiles * ks > (int64_t)device_info().sm_count) return false;
  // every cluster must be resident at once: clusters of ks CTAs of ~210 KB each are placed inside one
  // GPC, and a split whose clusters need a second wave (measured: 48 clusters of 3, 16 of 8) runs at
  // half speed, so those keep the workspace form
  return tiles <= kcluster_capacity(ks);
}

// Tensor map for the output C (16-bit, unit column stride): boxes of 32 columns x 32 rows with the
// 64 B swizzle the epilogue's staging tiles use. Sets p.c_tma / p.c3d; leaves them 0 (direct
// stores) when C's layout cannot be described (strided columns, unaligned rows) or the GEMM writes
// split-K partials.
void setup_cmap(CUtensorMap* tm, CUtensorMapDataType dt, TcParams& p) {
  p.c_tma = 0, p.c3d = 0;
  if (p.kcl > 1) return;  // cluster split-K writes C from the reduction, without a tensor map
  if (p.ksplit > 1) {
    // split-K: the map describes the fp32 partials [ksplit][M][N] instead (32-row x 16-column boxes)
    if (p.batch != 1 || (p.N % 4) || ((uintptr_t)p.partial & 15)) return;
    uint64_t dims[3] = {(uint64_t)p.N, (uint64_t)p.M, (uint64_t)p.ksplit};
    uint64_t strides[2] = {(uint64_t)p.N * 4, (uint64_t)p.N * p.M * 4};
    uint32_t box[3] = {16, 32, 1};
    if (make_tmap(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, p.partial, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B))
      p.c_tma = 2;
    return;
  }
  if (p.c_sn != 1 || ((uintptr_t)p.c & 15)) return;
  if (p.M > 1 && (p.c_sm * 2) % 16) return;
  const bool b3 = p.batch > 1;
  if (b3 && (p.c_sb == 0 || (p.c_sb * 2) % 16)) return;
  uint64_t dims[3] = {(uint64_t)p.N, (uint64_t)p.M, (uint64_t)p.batch};
  uint64_t strides[2] = {(uint64_t)(p.M > 1 ? p.c_sm : ((p.N + 7) / 8) * 8) * 2, (uint64_t)p.c_sb * 2};
  uint32_t box[3] = {32, 32, 1};
  if (!make_tmap(tm, dt, b3 ? 3 : 2, p.c, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B)) return;
  p.c_tma = 1, p.c3d = b3 ? 1 : 0;
}

}  // namespace

bool gemm_tc_eligible(const b2_gemm_args* a) {
  if (a->dtype != B2_BF16 && a->dtype != B2_F16) return false;
  if (!device_info().tcgen05 || !encode_fn()) return false;
  if (a->K <= 0 || a->M <= 0 || a->N <= 0) return false;
  const int e = 2;
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (!al(a->a) || !al(a->b)) return false;
  // A: K-major (a_sk == 1) or M-major (a_sm == 1); the other stride must be a 16-byte multiple
  bool a_k = a->a_sk == 1 && (a->M == 1 || tma_ok_stride(a->a_sm, e));
  bool a_m = !a_k && a->a_sm == 1 && (a->K == 1 || tma_ok_stride(a->a_sk, e));
  bool b_k = a->b_sk == 1 && (a->N == 1 || tma_ok_stride(a->b_sn, e));
  bool b_n = !b_k && a->b_sn == 1 && (a->K == 1 || tma_ok_stride(a->b_sk, e));
  if (!(a_k || a_m) || !(b_k || b_n)) return false;
  if (a->batch > 1) {
    if (a->a_sb != 0 && !tma_ok_stride(a->a_sb, e)) return false;
    if (a->b_sb != 0 && !tma_ok_stride(a->b_sb, e)) return false;
  }
  // TMA dims/strides must fit the encoder's 32-bit box coordinates
  if (a->M >= (1ll << 31) || a->N >= (1ll << 31) || a->K >= (1ll << 31)) return false;
  return true;
}

int gemm_tc_launch(const b2_gemm_args* a, cudaStream_t st) {
  const bool bf16 = a->dtype == B2_BF16;
  const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const TileChoice tc_ = pick_tile(a->M, a->N, a->batch);
  const int BN = tc_.bn, BMT = BM * tc_.msub;
  TcParams p{};
  p.M = a->M, p.N = a->N, p.K = a->K, p.batch = a->batch;
  p.m_tiles = (int)((a->M + BMT - 1) / BMT);
  p.n_tiles = (int)((a->N + BN - 1) / BN);
  p.k_blocks = (int)((a->K + BK - 1) / BK);
  p.k_total = p.k_blocks;
  p.a_mn = !(a->a_sk == 1 && (a->M == 1 || tma_ok_stride(a->a_sm, 2)));
  p.b_mn = !(a->b_sk == 1 && (a->N == 1 || tma_ok_stride(a->b_sn, 2)));
  p.a3d = a->batch > 1 && a->a_sb != 0;
  p.b3d = a->batch > 1 && a->b_sb != 0;
  p.c = a->c, p.c_sb = a->c_sb, p.c_sm = a->c_sm, p.c_sn = a->c_sn;
  p.bias = a->bias, p.has_bias = a->has_bias && a->bias != nullptr;
  p.bias_sb = a->bias_sb, p.bias_sm = a->bias_sm, p.bias_sn = a->bias_sn;
  p.alpha = a->alpha, p.beta = a->beta;
  p.err = device_error_ptr();
  p.ksplit = 1, p.kps = p.k_blocks;
  p.kcl = 0;
  int kcl_ks, kcl_kps;
  if (kcluster_plan(a, tc_, kcl_ks, kcl_kps)) {
    p.ksplit = kcl_ks, p.kps = kcl_kps, p.kcl = kcl_ks;
  } else if (a->batch == 1 && a->workspace) {
    int ks, kps;
    splitk_plan((int64_t)p.m_tiles * p.n_tiles, p.k_blocks, ks, kps);
    if (ks > 1 && (uint64_t)a->workspace_bytes >= (uint64_t)ks * a->M * a->N * sizeof(float) &&
        ((uintptr_t)a->workspace & 15) == 0)
      p.ksplit = ks, p.kps = kps, p.partial = (float*)a->workspace;
  }
  CUtensorMap tcm;
  memset(&tcm, 0, sizeof(tcm));
  setup_cmap(&tcm, dt, p);

  CUtensorMap ta, tb;
  {
    uint64_t dims[3], strides[2];
    uint32_t box[3];
    int rank = p.a3d ? 3 : 2;
    if (!p.a_mn) {
      dims[0] = a->K, dims[1] = a->M, strides[0] = (uint64_t)(a->M == 1 ? a->K : a->a_sm) * 2;
      box[0] = 64, box[1] = (uint32_t)BMT;
    } else {
      dims[0] = a->M, dims[1] = a->K, strides[0] = (uint64_t)(a->K == 1 ? a->M : a->a_sk) * 2;
      box[0] = 64, box[1] = 64;
    }
    if (strides[0] == 0 || strides[0] % 16) strides[0] = ((dims[0] * 2 + 15) / 16) * 16;
    dims[2] = a->batch, strides[1] = (uint64_t)a->a_sb * 2, box[2] = 1;
    if (!make_tmap(&ta, dt, rank, a->a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(B2_ERR_ARG, "gemm_tc: tensor map for A rejected");
  }
  {
    uint64_t dims[3], strides[2];
    uint32_t box[3];
    int rank = p.b3d ? 3 : 2;
    if (!p.b_mn) {
      dims[0] = a->K, dims[1] = a->N, strides[0] = (uint64_t)(a->N == 1 ? a->K : a->b_sn) * 2;
      box[0] = 64, box[1] = BN;
    } else {
      dims[0] = a->N, dims[1] = a->K, strides[0] = (uint64_t)(a->K == 1 ? a->N : a->b_sk) * 2;
      box[0] = 64, box[1] = 64;
    }
    if (strides[0] == 0 || strides[0] % 16) strides[0] = ((dims[0] * 2 + 15) / 16) * 16;
    dims[2] = a->batch, strides[1] = (uint64_t)a->b_sb * 2, box[2] = 1;
    if (!make_tmap(&tb, dt, rank, a->b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(B2_ERR_ARG, "gemm_tc: tensor map for B rejected");
  }
  int rc;
  if (BN == 256 && tc_.msub == 2)
    rc = bf16 ? launch_kernel<256, true, 0, 2>(ta, tb, tcm, p, st, "gemm_tc_256x256")
              : launch_kernel<256, false, 0, 2>(ta, tb, tcm, p, st, "gemm_tc_256x256");
  else if (BN == 256)
    rc = bf16 ? launch_kernel<256, true, 0, 1>(ta, tb, tcm, p, st, "gemm_tc_bn256")
              : launch_kernel<256, false, 0, 1>(ta, tb, tcm, p, st, "gemm_tc_bn256");
  else
    rc = bf16 ? launch_kernel<128, true, 0, 1>(ta, tb, tcm, p, st, "gemm_tc_bn128")
              : launch_kernel<128, false, 0, 1>(ta, tb, tcm, p, st, "gemm_tc_bn128");
  if (rc || p.ksplit == 1 || p.kcl > 1) return rc;
  const int64_t total = a->M * a->N;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)device_info().sm_count * 8);
  LaunchScope ls("gemm_splitk_reduce", st);
  const void* bias = p.has_bias ? a->bias : nullptr;
  if (bf16)
    gemm_splitk_reduce<__nv_bfloat16><<<grid, 256, 0, st>>>(p.partial, p.ksplit, a->M, a->N, (__nv_bfloat16*)a->c, a->c_sm,
                                                            a->c_sn, (const __nv_bfloat16*)bias, a->bias_sm, a->bias_sn,
                                                            a->alpha, a->beta);
  else
    gemm_splitk_reduce<__half><<<grid, 256, 0, st>>>(p.partial, p.ksplit, a->M, a->N, (__half*)a->c, a->c_sm, a->c_sn,
                                                     (const __half*)bias, a->bias_sm, a->bias_sn, a->alpha, a->beta);
  return after_launch("gemm_splitk_reduce");
}

uint64_t gemm_tc_workspace_bytes(const b2_gemm_args* a) {
  if (a->batch != 1 || a->K == 0 || !gemm_tc_eligible(a)) return 0;
  const TileChoice t = pick_tile(a->M, a->N, a->batch);
  int ks_c, kps_c;
  if (kcluster_plan(a, t, ks_c, kps_c)) return 0;  // reduced inside the cluster: no scratch
  const int64_t BMT = BM * t.msub;
  int ks, kps;
  splitk_plan(((a->M + BMT - 1) / BMT) * ((a->N + t.bn - 1) / t.bn), (int)((a->K + BK - 1) / BK), ks, kps);
  return ks > 1 ? (uint64_t)ks * a->M * a->N * sizeof(float) : 0;
}

// int8 launch plan. The dequant work per FLOP is 1/(2*rows of the CTA tile), so two stacked M=128
// UMMA tiles (256 rows) halve it; among the shapes the kernel supports, take the one with the best
// wave-quantised SM utilisation, weighted by how well the dequant warps keep up. The 176-wide tile
// (forward only: the transposed form dequantises 64-column chunks) puts M = 1024, N = 6144 on
// 140 CTAs, one wave. GEMMs with too few 256x256 tiles to fill the GPU and a long reduction (K >= 4096:
// the DiT block's fc2 forward and fc1 dX at M = 1024) split it instead when the caller gives a
// workspace: each work item is a 256x256 tile over a K slice of >= 8 blocks whose fp32 partial is
// TMA-stored and summed (with the bias) by gemm_splitk_reduce. With K = 2048 the partial traffic and
// the second kernel cost more than the split gains (measured 30 -> 45 us at 1024x2048x2048).
struct Int8Plan {
  int bn, msub, ksplit, kps, cg;
};
Int8Plan int8_plan(const b2_int8_gemm_args* a) {
  // cg = 2: a CTA pair (cta_group::2) shares each MMA, every CTA staging and dequantising only half of
  // the B tile, which halves the dequant work and the B operand bytes per CTA; pair tiles are
  // 2 * 128 * msub rows by bn columns and use half as many units of GPU capacity (one per pair).
  // eff: measured relative per-SM rate of each shape (pairs: estimated from their shared-memory bytes
  // per K block until measured, B2_INT8_CG=1|2 pins the choice for sweeps). The 256 x 128 pair tile
  // (0.75) takes the M = 1024, N = 2048 and M = 512, N = 4096 shapes of the DiT block, where 256 x 256
  // pairs leave half the SMs idle: measured 32.2 -> 25.2 us forward, 37.8 -> 27.5 us dX at K = 2048.
  struct Choice { int bn, msub, cg; double eff; };
  const Choice fwd_opts[] = {{256, 2, 2, 1.55}, {176, 2, 2, 1.45}, {256, 1, 2, 1.3}, {128, 2, 2, 1.25},
                             {256, 2, 1, 1.15}, {176, 2, 1, 1.08}, {128, 2, 1, 1.0},  {96, 2, 1, 0.97},
                             {256, 1, 1, 0.85}, {128, 1, 2, 0.75},  {128, 1, 1, 0.55}};
  const Choice dx_opts[] = {{256, 2, 2, 1.55}, {256, 1, 2, 1.3}, {128, 2, 2, 1.25}, {256, 2, 1, 1.15},
                            {128, 2, 1, 1.0},  {256, 1, 1, 0.85}, {128, 1, 2, 0.75},  {128, 1, 1, 0.55}};
  const int sms = device_info().sm_count > 0 ? device_info().sm_count : 148;
  const int64_t out_cols = a->transpose_w ? a->K : a->N;
  const int64_t red = a->transpose_w ? a->N : a->K;
  const int k_blocks = (int)((red + BK - 1) / BK);
  static const int forced = [] {  // B2_INT8_TILE=<bn>x<msub> pins the tile (measurement sweeps)
    const char* e = getenv("B2_INT8_TILE");
    int bn = 0, ms = 0;
    return (e && sscanf(e, "%dx%d", &bn, &ms) == 2) ? bn * 10 + ms : 0;
  }();
  static const int forced_cg = [] {
    const char* e = getenv("B2_INT8_CG");
    return (e && (e[0] == '1' || e[0] == '2')) ? e[0] - '0' : 0;
  }();
  Int8Plan best{0, 0, 1, k_blocks, 1};
  double best_score = -1.0;
  const int nopts = a->transpose_w ? 8 : 11;
  for (int i = 0; i < nopts; ++i) {
    const Choice c = a->transpose_w ? dx_opts[i] : fwd_opts[i];
    if (forced_cg && c.cg != forced_cg) continue;
    if (a->epilogue && c.bn % 32) continue;  // fused epilogues run on whole 32-column chunks
    const int64_t rows = 128 * c.msub * c.cg, cap = sms / c.cg;
    const int64_t tiles = ((a->M + rows - 1) / rows) * ((out_cols + c.bn - 1) / c.bn);
    const int64_t waves = (tiles + cap - 1) / cap;
    double score = (double)a->M * out_cols / ((double)waves * cap * rows * c.bn) * c.eff;
    if (forced) score = (forced == c.bn * 10 + c.msub) ? 1e9 * c.eff : -1.0;
    if (score > best_score) best_score = score, best = Int8Plan{c.bn, c.msub, 1, k_blocks, c.cg};
  }
  if (best.bn == 0) best = Int8Plan{128, 2, 1, k_blocks, 1};
  // split-K over 256x256 tiles (CTA pairs: 512x256) when too few tiles fill the GPU and K is long
  if (!forced && !a->epilogue && !a->lora_r && a->workspace_bytes > 0 && k_blocks >= 64) {
    for (int cg = 1; cg <= 2; ++cg) {
      if (forced_cg && cg != forced_cg) continue;
      const int64_t rows = 256 * cg, cap = sms / cg;
      const double eff = cg == 2 ? 1.55 : 1.15;
      const int64_t tiles = ((a->M + rows - 1) / rows) * ((out_cols + 255) / 256);
      if (tiles * 2 > cap) continue;
      const int want = (int)std::min<int64_t>(cap / tiles, k_blocks / 8);
      if (want < 2) continue;
      const int kps = (k_blocks + want - 1) / want;
      const int ks = (k_blocks + kps - 1) / kps;
      const int64_t units = tiles * ks;
      const int64_t waves = (units + cap - 1) / cap;
      const double score = (double)a->M * out_cols / ((double)waves * cap * rows * 256) * ks * eff * 0.8;
      const uint64_t need = (uint64_t)ks * a->M * out_cols * sizeof(float);
      if (score > best_score && (uint64_t)a->workspace_bytes >= need)
        best_score = score, best = Int8Plan{256, 2, ks, kps, cg};
    }
  }
  return best;
}

}  // namespace b2

using namespace b2;

// ---- fused int8-weight linear -------------------------------------------------------------------
extern "C" int b2_int8_gemm(const b2_int8_gemm_args* a, b2_stream_t stream) {
  if (!a) return fail(B2_ERR_ARG, "int8_gemm: null args");
  if (int rc = ensure_init()) return rc;
  if (a->M < 0 || a->N < 0 || a->K < 0) return fail(B2_ERR_ARG, "int8_gemm: negative size");
  if (a->scale_layout != 0 && a->scale_layout != 1) return fail(B2_ERR_ARG, "int8_gemm: scale_layout must be 0 or 1");
  const int64_t out_cols = a->transpose_w ? a->K : a->N;
  const int64_t red = a->transpose_w ? a->N : a->K;  // reduction length
  if (a->M == 0 || out_cols == 0) return 0;
  if (!a->x || !a->q || !a->scale || !a->out) return fail(B2_ERR_ARG, "int8_gemm: null pointer");
  if (!device_info().tcgen05 || !encode_fn()) return fail(B2_ERR_ARG, "int8_gemm: requires an sm_100a device");
  if (red == 0) return fail(B2_ERR_ARG, "int8_gemm: empty reduction");
  if (((uintptr_t)a->x & 15) || ((uintptr_t)a->q & 15) || a->x_ld % 8 || a->K % 16)
    return fail(B2_ERR_ARG, "int8_gemm: x and q must be 16-byte aligned, x_ld a multiple of 8 and K of 16");
  if (a->transpose_w && a->bias) return fail(B2_ERR_ARG, "int8_gemm: bias is only supported in the forward form");
  if (a->epilogue < 0 || a->epilogue > 2 || (a->epilogue == 1 && a->transpose_w) || (a->epilogue == 2 && !a->transpose_w))
    return fail(B2_ERR_ARG, "int8_gemm: epilogue 1 (GELU) needs the forward form, 2 (GELU backward) the transposed form");
  if (a->epilogue && (!a->aux || ((uintptr_t)a->aux & 15) || a->aux_ld < out_cols || a->aux_ld % 8))
    return fail(B2_ERR_ARG, "int8_gemm: the GELU epilogue needs a 16-byte aligned bf16 aux with aux_ld >= out_cols, a multiple of 8");
  if (a->lora_r && (a->lora_r < 8 || a->lora_r > 64 || a->lora_r % 8 || !a->lora_h || !a->lora_b ||
                    ((uintptr_t)a->lora_h & 15) || ((uintptr_t)a->lora_b & 15) || a->lora_h_ld < a->lora_r ||
                    a->lora_h_ld % 8 || a->lora_b_ld % 8 || a->lora_b_ld < (a->transpose_w ? a->K : a->lora_r)))
    return fail(B2_ERR_ARG, "int8_gemm: LoRA operands need 8 <= r <= 64 (a multiple of 8), 16-byte aligned bf16 rows and "
                            "leading dims that are multiples of 8");
  cudaStream_t st = (cudaStream_t)stream;
  if (a->workspace && ((uintptr_t)a->workspace & 15)) return fail(B2_ERR_ARG, "int8_gemm: workspace must be 16-byte aligned");
  if (int8_gemv_applies(a)) return int8_gemv_launch(a, st);  // a few rows of x: the weight-stream kernel
  b2_int8_gemm_args aa = *a;
  if (!aa.workspace) aa.workspace_bytes = 0;
  const Int8Plan best = int8_plan(&aa);
  const int BN = best.bn, BMT = 128 * best.msub, BNC = best.bn / best.cg;
  TcParams p{};
  p.M = a->M, p.N = out_cols, p.K = red, p.batch = 1;
  p.m_tiles = (int)((a->M + BMT * best.cg - 1) / (BMT * best.cg));
  p.n_tiles = (int)((out_cols + BN - 1) / BN);
  p.k_blocks = (int)((red + BK - 1) / BK);
  p.a_mn = 0;
  p.b_mn = a->transpose_w ? 1 : 0;
  p.c = a->out, p.c_sm = a->out_ld, p.c_sn = 1, p.c_sb = 0;
  p.bias = a->bias, p.has_bias = a->bias != nullptr, p.bias_sn = 1;
  p.alpha = 1.f, p.beta = 1.f;
  p.err = device_error_ptr();
  p.scale = a->scale, p.scale_layout = a->scale_layout, p.scale_nb = (a->K + 63) / 64, p.deq_rows = a->N;
  p.ksplit = best.ksplit, p.kps = best.kps;
  if (p.ksplit > 1) p.partial = (float*)a->workspace;
  // the LoRA side path: one more K block (the plan never splits K when there is one)
  p.lora_r = a->lora_r, p.lora_b = a->lora_b, p.lora_b_ld = a->lora_b_ld;
  p.k_total = p.k_blocks + (a->lora_r ? 1 : 0);
  if (a->lora_r) p.kps = p.k_total;
  CUtensorMap th;
  memset(&th, 0, sizeof(th));
  if (a->lora_r) {  // [M, r] bf16, read as 64-wide boxes (columns past r are filled with zeros)
    uint64_t dims[2] = {(uint64_t)a->lora_r, (uint64_t)a->M}, strides[1] = {(uint64_t)a->lora_h_ld * 2};
    uint32_t box[2] = {64, (uint32_t)BMT};
    if (!make_tmap(&th, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->lora_h, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(B2_ERR_ARG, "int8_gemm: tensor map for the LoRA operand rejected");
  }
  CUtensorMap tcm;
  memset(&tcm, 0, sizeof(tcm));
  setup_cmap(&tcm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p);
  p.epi = a->epilogue, p.aux = a->aux, p.aux_ld = a->aux_ld;
  if (p.epi && p.c_tma != 1)
    return fail(B2_ERR_ARG, "int8_gemm: the GELU epilogue needs an output a tensor map can describe (16-byte rows)");
  CUtensorMap ta, tb;
  {
    uint64_t dims[2] = {(uint64_t)red, (uint64_t)a->M}, strides[1] = {(uint64_t)a->x_ld * 2};
    uint32_t box[2] = {64, (uint32_t)BMT};
    if (!make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a->x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(B2_ERR_ARG, "int8_gemm: tensor map for x rejected");
  }
  {
    uint64_t dims[2] = {(uint64_t)a->K, (uint64_t)a->N}, strides[1] = {(uint64_t)a->K};
    uint32_t box[2];
    if (!a->transpose_w) box[0] = 64, box[1] = (uint32_t)BNC;  // each CTA of a pair loads its half
    else box[0] = (uint32_t)BNC, box[1] = 64;
    if (!make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, a->q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return fail(B2_ERR_ARG, "int8_gemm: tensor map for q rejected");
  }
  const char* name = a->transpose_w ? "int8_gemm_dx" : "int8_gemm_fwd";
  int rc;
  if (best.cg == 2) {
    const char* pname = a->transpose_w ? "int8_gemm_dx_pair" : "int8_gemm_fwd_pair";
    if (best.msub == 2 && BN == 256) rc = launch_kernel<256, true, 2, 2, 2>(ta, tb, tcm, p, st, pname, &th);
    else if (best.msub == 2 && BN == 176) rc = launch_kernel<176, true, 2, 2, 2>(ta, tb, tcm, p, st, pname, &th);
    else if (best.msub == 2) rc = launch_kernel<128, true, 2, 2, 2>(ta, tb, tcm, p, st, pname, &th);
    else if (BN == 128) rc = launch_kernel<128, true, 2, 1, 2>(ta, tb, tcm, p, st, pname, &th);
    else rc = launch_kernel<256, true, 2, 1, 2>(ta, tb, tcm, p, st, pname, &th);
  } else if (best.msub == 2 && BN == 256) rc = launch_kernel<256, true, 2, 2>(ta, tb, tcm, p, st, name, &th);
  else if (best.msub == 2 && BN == 176) rc = launch_kernel<176, true, 2, 2>(ta, tb, tcm, p, st, name, &th);
  else if (best.msub == 2 && BN == 128) rc = launch_kernel<128, true, 2, 2>(ta, tb, tcm, p, st, name, &th);
  else if (best.msub == 2 && BN == 96) rc = launch_kernel<96, true, 2, 2>(ta, tb, tcm, p, st, name, &th);
  else if (BN == 256) rc = launch_kernel<256, true, 2, 1>(ta, tb, tcm, p, st, name, &th);
  else rc = launch_kernel<128, true, 2, 1>(ta, tb, tcm, p, st, name, &th);
  if (rc || p.ksplit == 1) return rc;
  const int64_t total = a->M * out_cols;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, (int64_t)device_info().sm_count * 8);
  LaunchScope ls("int8_gemm_splitk_reduce", st);
  gemm_splitk_reduce<__nv_bfloat16><<<grid, 256, 0, st>>>(p.partial, p.ksplit, a->M, out_cols, (__nv_bfloat16*)a->out,
                                                          a->out_ld, 1, (const __nv_bfloat16*)a->bias, 0, 1, 1.f, 1.f);
  return after_launch("int8_gemm_splitk_reduce");
}

extern "C" uint64_t b2_int8_gemm_workspace_bytes(const b2_int8_gemm_args* a) {
  if (!a || a->M <= 0 || a->N <= 0 || a->K <= 0 || !device_info().tcgen05 || int8_gemv_applies(a)) return 0;
  b2_int8_gemm_args q = *a;
  q.workspace = nullptr, q.workspace_bytes = INT64_MAX;  // the plan a large enough workspace gets
  const Int8Plan pl = int8_plan(&q);
  const int64_t out_cols = a->transpose_w ? a->K : a->N;
  return pl.ksplit > 1 ? (uint64_t)pl.ksplit * a->M * out_cols * sizeof(float) : 0;
}
