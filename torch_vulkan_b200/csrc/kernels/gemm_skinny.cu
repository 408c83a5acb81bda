// Skinny GEMM: C[M, N] = alpha * A[M, K] @ B[K, N] + beta * bias with one output dimension <= 64 (the
// LoRA projections and weight gradients of a DiT block: x A^T, dY B, x^T dH, dY^T H at rank 16-64).
//
// These GEMMs carry 0.1-1 GFLOP and are bound by latency, not by the tensor cores: the tcgen05 kernel
// spends most of their time in its prologue and epilogue and needs a split-K workspace and a second
// reduction kernel to find parallelism. Here one CTA of eight warps owns BM rows of C and the whole
// reduction: each warp streams every eighth 32-wide K block of A and B into its own double-buffered
// shared-memory slice with 16-byte cp.async (zero-filled past the edges), feeds mma.sync m16n8k16 from
// ldmatrix (.trans for M-major A and N-major B), and the eight partial tiles are summed through shared
// memory by the CTA before alpha / bias / the dtype conversion. One launch, no workspace. The narrow
// dimension may be M instead (C^T = B^T A^T is computed then). Same contract as b2_gemm (strides in
// elements, fp32 accumulate).
#include <type_traits>

#include "common.cuh"

namespace b2 {
namespace {

constexpr int kKB = 32;       // K elements per block (two k16 MMA steps)
constexpr int kWarps = 8;     // warps per CTA, each taking every eighth K block
constexpr int kPad = 8;       // elements of padding per staged row (16 bytes: conflict-free ldmatrix)

struct SkParams {
  const void* a;
  const void* b;
  void* c;
  const void* bias;
  int64_t M, N, K;
  int64_t a_sm, a_sk, b_sk, b_sn, c_sm, c_sn, bias_sm, bias_sn;
  float alpha, beta;
  int has_bias;
  int a_kmajor, b_kmajor;  // A rows / B columns contiguous along K (else M- / N-contiguous)
};

template <int BM, int NP>
struct SkCfg {
  // per-warp stage: A as [BM][KB + pad] (K-major) or [KB][BM + pad] (M-major), B as [NP][KB + pad]
  // (K-major) or [KB][NP + pad] (N-major); elements
  static constexpr int A_ELEMS = BM * (kKB + kPad) > kKB * (BM + kPad) ? BM * (kKB + kPad) : kKB * (BM + kPad);
  static constexpr int B_ELEMS = NP * (kKB + kPad) > kKB * (NP + kPad) ? NP * (kKB + kPad) : kKB * (NP + kPad);
  static constexpr int STAGE_BYTES = (A_ELEMS + B_ELEMS) * 2;
  // K blocks in flight per warp: four when eight warps' rings fit in 200 KB, else three
  static constexpr int STAGES = kWarps * 4 * STAGE_BYTES <= 200 * 1024 ? 4 : 3;
  static constexpr int WARP_BYTES = STAGES * STAGE_BYTES;
  static constexpr int RED_BYTES = kWarps * BM * NP * 4;
  static constexpr int SMEM = kWarps * WARP_BYTES > RED_BYTES ? kWarps * WARP_BYTES : RED_BYTES;
  static_assert(STAGE_BYTES % 16 == 0, "stages must keep 16-byte alignment");
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
template <bool BF16>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ float to_float(T v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(v);
  else return __half2float(v);
}
template <typename T>
__device__ __forceinline__ T from_float(float v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(v);
  else return __float2half_rn(v);
}

template <typename T, int BM, int NP>
__global__ void __launch_bounds__(kWarps * 32) gemm_skinny_kernel(SkParams p) {
  using C = SkCfg<BM, NP>;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int MT = BM / 16, NT = NP / 8;
  extern __shared__ __align__(128) uint8_t sk_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const T* A = (const T*)p.a;
  const T* B = (const T*)p.b;
  uint8_t* wbase = sk_smem + warp * C::WARP_BYTES;
  const int nkb = (int)((p.K + kKB - 1) / kKB);

  // stage `st` of this warp: K block kb of A (BM x KB) and B (KB x NP), 16-byte chunks, zero past the edges
  auto load = [&](int st, int kb) {
    T* sa = reinterpret_cast<T*>(wbase + st * C::STAGE_BYTES);
    T* sb = sa + C::A_ELEMS;
    const int64_t k0 = (int64_t)kb * kKB;
    if (p.a_kmajor) {  // [BM][KB + pad]: row m, chunk c of 8 k
      for (int i = lane; i < BM * (kKB / 8); i += 32) {
        const int m = i / (kKB / 8), c = i % (kKB / 8);
        const int64_t gm = m0 + m, gk = k0 + c * 8;
        const bool ok = gm < p.M && gk < p.K;
        cp_async16(smem_u32(sa + m * (kKB + kPad) + c * 8), ok ? A + gm * p.a_sm + gk : A, ok);
      }
    } else {  // [KB][BM + pad]: row k, chunk c of 8 m
      for (int i = lane; i < kKB * (BM / 8); i += 32) {
        const int k = i / (BM / 8), c = i % (BM / 8);
        const int64_t gm = m0 + c * 8, gk = k0 + k;
        const bool ok = gm < p.M && gk < p.K;
        cp_async16(smem_u32(sa + k * (BM + kPad) + c * 8), ok ? A + gk * p.a_sk + gm : A, ok);
      }
    }
    if (p.b_kmajor) {  // [NP][KB + pad]: row n, chunk c of 8 k
      for (int i = lane; i < NP * (kKB / 8); i += 32) {
        const int n = i / (kKB / 8), c = i % (kKB / 8);
        const int64_t gk = k0 + c * 8;
        const bool ok = n < p.N && gk < p.K;
        cp_async16(smem_u32(sb + n * (kKB + kPad) + c * 8), ok ? B + (int64_t)n * p.b_sn + gk : B, ok);
      }
    } else {  // [KB][NP + pad]: row k, chunk c of 8 n
      for (int i = lane; i < kKB * (NP / 8); i += 32) {
        const int k = i / (NP / 8), c = i % (NP / 8);
        const int64_t gk = k0 + k;
        const bool ok = c * 8 < p.N && gk < p.K;
        cp_async16(smem_u32(sb + k * (NP + kPad) + c * 8), ok ? B + gk * p.b_sk + c * 8 : B, ok);
      }
    }
    cp_async_commit();
  };

  float acc[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;

  const int mi = lane >> 3, r8 = lane & 7;  // ldmatrix: matrix index and row within it
  constexpr int S = C::STAGES;
  // this warp's K blocks are warp, warp + 8, ...; block i of them lands in stage i % S, S - 1 ahead of use
  // (an empty group is committed where there is no block, so the wait count stays uniform)
#pragma unroll
  for (int i = 0; i < S - 1; ++i) {
    const int kb = warp + i * kWarps;
    if (kb < nkb) load(i, kb);
    else cp_async_commit();
  }
  for (int i = 0, kb = warp; kb < nkb; ++i, kb += kWarps) {
    cp_async_wait<S - 2>();
    __syncwarp();
    const int st = i % S;
    const T* sa = reinterpret_cast<const T*>(wbase + st * C::STAGE_BYTES);
    const T* sb = sa + C::A_ELEMS;
#pragma unroll
    for (int ks = 0; ks < kKB / 16; ++ks) {
      uint32_t af[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        if (p.a_kmajor)  // lanes 0-15: rows 0-15 at k 0; lanes 16-31: rows 0-15 at k 8
          ldsm_x4(smem_u32(sa + (mt * 16 + (lane & 15)) * (kKB + kPad) + ks * 16 + (lane >> 4) * 8), af[mt][0],
                  af[mt][1], af[mt][2], af[mt][3]);
        else  // matrix mi: m block (mi & 1) * 8, k block (mi >> 1) * 8, stored k-major rows
          ldsm_x4_t(smem_u32(sa + (ks * 16 + (mi >> 1) * 8 + r8) * (BM + kPad) + mt * 16 + (mi & 1) * 8), af[mt][0],
                    af[mt][1], af[mt][2], af[mt][3]);
      }
#pragma unroll
      for (int j = 0; j < NP / 16; ++j) {  // n tiles 2j and 2j + 1
        uint32_t b0, b1, b2, b3;
        if (p.b_kmajor)  // matrix mi: n block (mi >> 1) * 8, k block (mi & 1) * 8
          ldsm_x4(smem_u32(sb + (j * 16 + (mi >> 1) * 8 + r8) * (kKB + kPad) + ks * 16 + (mi & 1) * 8), b0, b1, b2, b3);
        else  // stored [k][n]: matrix mi rows k = (mi & 1) * 8 + r, columns n = (mi >> 1) * 8
          ldsm_x4_t(smem_u32(sb + (ks * 16 + (mi & 1) * 8 + r8) * (NP + kPad) + j * 16 + (mi >> 1) * 8), b0, b1, b2, b3);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma16816<BF16>(acc[mt][2 * j], af[mt], b0, b1);
          mma16816<BF16>(acc[mt][2 * j + 1], af[mt], b2, b3);
        }
      }
    }
    __syncwarp();  // every lane is done reading this stage before it is refilled
    const int kn = kb + (S - 1) * kWarps;  // into the stage read in the previous iteration
    if (kn < nkb) load((i + S - 1) % S, kn);
    else cp_async_commit();
  }
  cp_async_wait<0>();

  // the eight warps' partial tiles are summed through shared memory (the stages are idle now)
  __syncthreads();
  float* red = reinterpret_cast<float*>(sk_smem);
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float* r0 = red + ((int64_t)warp * BM + mt * 16 + g) * NP + nt * 8 + 2 * t;
      *reinterpret_cast<float2*>(r0) = make_float2(acc[mt][nt][0], acc[mt][nt][1]);
      *reinterpret_cast<float2*>(r0 + 8 * NP) = make_float2(acc[mt][nt][2], acc[mt][nt][3]);
    }
  __syncthreads();
  for (int e = threadIdx.x; e < BM * NP; e += kWarps * 32) {
    const int row = e / NP, col = e - (e / NP) * NP;
    const int64_t gm = m0 + row;
    if (gm >= p.M || col >= p.N) continue;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w * BM * NP + e];
    float v = p.alpha * s;
    if (p.has_bias) v += p.beta * to_float(((const T*)p.bias)[gm * p.bias_sm + col * p.bias_sn]);
    ((T*)p.c)[gm * p.c_sm + col * p.c_sn] = from_float<T>(v);
  }
}

template <typename T, int BM, int NP>
int launch_skinny(const SkParams& p, cudaStream_t st) {
  using C = SkCfg<BM, NP>;
  auto kern = gemm_skinny_kernel<T, BM, NP>;
  static bool attr = false;
  if (!attr) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                            "cudaFuncSetAttribute(gemm_skinny)"))
      return rc;
    attr = true;
  }
  const unsigned grid = (unsigned)((p.M + BM - 1) / BM);
  {
    LaunchScope ls("gemm_skinny", st);
    kern<<<grid, kWarps * 32, C::SMEM, st>>>(p);
  }
  return after_launch("gemm_skinny");
}

template <typename T, int BM>
int launch_skinny_np(const SkParams& p, cudaStream_t st) {
  const int np = (int)((p.N + 15) / 16 * 16);
  switch (np) {
    case 16: return launch_skinny<T, BM, 16>(p, st);
    case 32: return launch_skinny<T, BM, 32>(p, st);
    case 48: return launch_skinny<T, BM, 48>(p, st);
    default: return launch_skinny<T, BM, 64>(p, st);
  }
}

// The problem with its narrow dimension as N: C^T = B^T A^T when M is the narrow one.
bool normalise(const b2_gemm_args* a, SkParams& p) {
  const bool swap = a->N > 64 || (a->M <= 64 && a->M < a->N);
  p = SkParams{};
  p.K = a->K;
  p.alpha = a->alpha, p.beta = a->beta;
  p.has_bias = a->has_bias && a->bias != nullptr;
  p.bias = a->bias;
  p.c = a->c;
  if (!swap) {
    p.a = a->a, p.b = a->b, p.M = a->M, p.N = a->N;
    p.a_sm = a->a_sm, p.a_sk = a->a_sk, p.b_sk = a->b_sk, p.b_sn = a->b_sn;
    p.c_sm = a->c_sm, p.c_sn = a->c_sn, p.bias_sm = a->bias_sm, p.bias_sn = a->bias_sn;
  } else {
    p.a = a->b, p.b = a->a, p.M = a->N, p.N = a->M;
    p.a_sm = a->b_sn, p.a_sk = a->b_sk, p.b_sk = a->a_sk, p.b_sn = a->a_sm;
    p.c_sm = a->c_sn, p.c_sn = a->c_sm, p.bias_sm = a->bias_sn, p.bias_sn = a->bias_sm;
  }
  if (p.N > 64 || p.N % 8 != 0 || p.N <= 0 || p.M <= 0) return false;
  auto al = [](const void* q) { return ((uintptr_t)q & 15) == 0; };
  if (!al(p.a) || !al(p.b)) return false;
  // A: rows contiguous along K, or columns contiguous along M, with 16-byte aligned rows / columns
  if (p.a_sk == 1 && (p.M == 1 || p.a_sm % 8 == 0) && p.K % 8 == 0) p.a_kmajor = 1;
  else if (p.a_sm == 1 && p.a_sk % 8 == 0 && p.M % 8 == 0) p.a_kmajor = 0;
  else return false;
  if (p.b_sk == 1 && p.b_sn % 8 == 0 && p.K % 8 == 0) p.b_kmajor = 1;
  else if (p.b_sn == 1 && p.b_sk % 8 == 0) p.b_kmajor = 0;
  else return false;
  return true;
}

}  // namespace

// Taken for bf16/f16 GEMMs whose narrow dimension is <= 64 (a multiple of 8), with 256 <= K <= 1024 and a
// wide dimension of at most 2048: there it beats the tcgen05 kernel's split-K form (graphs of back-to-back
// calls: 2048x1024x48 with M-major A 8.7 -> 6.5 us). Every CTA re-reads all of B through cp.async, whose
// outstanding requests per SM cap it near 30 GB/s per SM whatever the pipeline depth (two and three K
// blocks in flight per warp measured the same), so longer reductions and wider outputs stay on the TMA-fed
// tcgen05 kernel (1024x6144x48 10.5 us there, 26 us here; 4096x2048x48 10.8 against 13.2).
// B2_GEMM_SKINNY=0 never takes it, =1 takes it for every supported layout up to K x 64 x 2 <= 1.5 MB.
bool gemm_skinny_applies(const b2_gemm_args* a) {
  static const int pinned = [] {
    const char* e = getenv("B2_GEMM_SKINNY");
    return e && (e[0] == '0' || e[0] == '1') ? e[0] - '0' : -1;
  }();
  if (pinned == 0 || a->batch != 1 || (a->dtype != B2_BF16 && a->dtype != B2_F16) || a->K < 256) return false;
  if (a->M > 64 && a->N > 64) return false;
  SkParams p;
  if (!normalise(a, p)) return false;
  const int64_t np = (p.N + 15) / 16 * 16;
  if (pinned == 1) return p.K * np * 2 <= (int64_t)(3u << 19) && p.M <= (1 << 20);
  return p.K <= 1024 && p.M <= 2048;
}

int gemm_skinny_launch(const b2_gemm_args* a, cudaStream_t st) {
  SkParams p;
  if (!normalise(a, p)) return fail(B2_ERR_ARG, "gemm_skinny: layout not supported");
  const bool wide = p.M > 2048;  // 32-row CTAs once 16-row ones would exceed two per SM
  if (a->dtype == B2_BF16)
    return wide ? launch_skinny_np<__nv_bfloat16, 32>(p, st) : launch_skinny_np<__nv_bfloat16, 16>(p, st);
  return wide ? launch_skinny_np<__half, 32>(p, st) : launch_skinny_np<__half, 16>(p, st);
}

}  // namespace b2
