// Tensor-core fused attention for sm_100a (tcgen05 + TMEM + TMA), bf16/f16, head dim 64 or 128.
//
// Replaces the reference's cooperative-matrix kernels vkrt/shaders/attn_coop.comp.in (fwd 158-211,
// dK/dV 213-259, dQ 261-301) and the delta pass attn.comp.in:210-240. Same equations
// (FlashAttention-2): forward online softmax with lse = m + log(l); backward
// P = exp(scale*S - lse), dS = P*(dP - delta), dV = P^T dO, dK = scale dS^T Q, dQ = scale dS K.
// B200 design:
//  forward  one CTA per (128-query tile, batch*head). warp 0 TMA (Q once, K/V ring), warp 1 issues
//           S = Q K^T into a double-buffered TMEM tile and O += P V into a TMEM accumulator, warps
//           2..5 (one thread per query row) run the online softmax from tcgen05.ld'ed S, write P
//           (bf16, 128B-swizzled) to shared memory for the PV MMA, and rescale O in TMEM only when the
//           running max grows by more than 2^8 (lazy rescaling); the epilogue normalises O from TMEM.
//  backward delta = rowsum(O*dO) pre-pass; then one CTA per (128-key tile, batch*head) keeps K, V in
//           shared memory and dK, dV in TMEM while it walks 64-query tiles: S^T = K Q^T and
//           dP^T = V dO^T on the tensor cores, P^T / dS^T in registers (thread = key row), then
//           dV += P^T dO, dK += dS^T Q and dQ^T = K^T dS^T (all tcgen05); dQ partials are added into an
//           fp32 workspace tile by tile with bulk reductions (cp.reduce.async.bulk, done in L2) and
//           converted at the end.
// Every mbarrier wait is bounded; on expiry the kernel records an error code and unwinds.
#include <cuda.h>
#include <cstdlib>
#include <cstring>

#include <type_traits>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace b2 {

bool make_tmap(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle sw);  // gemm_tc.cu
int attn_delta_launch(const b2_attn_args* a, cudaStream_t st);                              // attn_simt.cu

namespace {

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool bf16) {
  if (bf16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

struct AttnTcParams {
  int64_t B, H, Sq, Sk;
  float scale_log2;  // scale * log2(e)
  float scale;
  void* o;
  int64_t o_s[3];
  float* lse;
  int* err;
  // backward
  const float* delta;
  float* dq_acc;  // fp32 [B*H, Sq, D]
  void* dk;
  void* dv;
  int64_t dk_s[3], dv_s[3];
  // fused dQ (dS-to-L2 form, all key-tile CTAs resident at once): per-(b, h) count of key-tile CTAs whose
  // dS^T tiles are stored, zeroed by the prep kernel; nullptr: dQ comes from a GEMM after the kernel
  int* dsready;
};

// ==================================================================================================
// forward: two softmax warpgroups split the KV blocks (even / odd), each with its own TMEM S and O
// ==================================================================================================
// CG = 2: a cluster pair of CTAs shares every MMA (tcgen05 cta_group::2, M = 256 query rows, 128 per
// CTA): each CTA stages its own Q rows but only half of each K block (64 keys) and half of each V block
// (64 of the 128 head-dim columns), which halves the per-CTA K/V traffic into shared memory and the
// B-operand reads of both MMAs. The leader (even CTA) issues the MMAs for both.
template <int D, int CG = 1>
struct FwdCfg {
  static constexpr int BQ = 128, BKV = 128;
  static constexpr int DCH = D / 64;                 // 64-element chunks along D
  static constexpr int KROWS = BKV / CG;              // keys of a K block this CTA stages
  static constexpr int VCH = DCH / CG;                // 64-column V chunks this CTA stages
  static_assert(CG == 1 || D == 128, "CTA pairs split V by 64-column chunks: D = 128");
  static constexpr int Q_BYTES = BQ * D * 2;
  static constexpr int K_BYTES = KROWS * D * 2;
  static constexpr int V_BYTES = BKV * 64 * VCH * 2;
  static constexpr int NS = CG == 2 ? 4 : 3;          // K / V ring depth
  static constexpr int OFF_Q = 0;                     // also the (m, l) exchange area of the epilogue
  static constexpr int OFF_K = OFF_Q + Q_BYTES;       // NS stages
  static constexpr int OFF_V = OFF_K + NS * K_BYTES;  // NS stages
  static constexpr int OFF_BAR = OFF_V + NS * V_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static_assert(SMEM <= 232448, "forward tile set exceeds the 227 KB shared-memory limit");
  static_assert(Q_BYTES >= 2 * BQ * 8, "exchange area");
  static constexpr int THREADS = 320;
  // TMEM columns: S0 [0,128) S1 [128,256) O0 [256,256+D) O1 [384,384+D); P_g (bf16 pairs) overwrites
  // the first 64 columns of S_g once the softmax has read S_g into registers
  static constexpr uint32_t T_S = 0, T_O = 256, TMEM_COLS = 512;
};

template <int D, bool BF16, int CG>
__global__ void __launch_bounds__(320, 1)
    attn_fwd_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, AttnTcParams p) {
  using C = FwdCfg<D, CG>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  constexpr int NS = C::NS;
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;             // [NS] K of block j in stage j % NS
  uint64_t* k_empty = k_full + NS;        // [NS]
  uint64_t* v_full = k_empty + NS;        // [NS]
  uint64_t* v_empty = v_full + NS;        // [NS]
  uint64_t* s_full = v_empty + NS;        // [2] S of block j into S[j&1]
  uint64_t* p_full = s_full + 2;          // [2] P of block j into TMEM over S[j&1] (count 128)
  uint64_t* o_upd = p_full + 2;           // [2] PV of block j into O[j&1] done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_upd + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(o_upd + 3);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // pairs: CTA rank r of the cluster takes query rows [q0, q0 + 128) of the pair's 256
  const uint32_t rank = CG == 2 ? tc::cluster_ctarank() : 0u;
  const int q0 = (int)(blockIdx.x / CG) * C::BQ * CG + (int)rank * C::BQ;
  const int bh = blockIdx.y;
  const int b = bh / (int)p.H, h = bh % (int)p.H;
  const int nblk = (int)((p.Sk + C::BKV - 1) / C::BKV);
  // the leader's copy of a barrier (the barrier itself for single CTAs)
  auto leader_bar = [&](uint64_t* bar) -> uint32_t {
    return CG == 2 ? tc::mapa_shared(tc::smem_u32(bar), 0u) : tc::smem_u32(bar);
  };

  if (threadIdx.x == 0) {
    tc::mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      tc::mbar_init(&k_full[i], 1);
      tc::mbar_init(&k_empty[i], 1);
      tc::mbar_init(&v_full[i], 1);
      tc::mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&p_full[i], CG == 2 ? 4 * CG : 128);  // pairs: one arrival per softmax warp
      tc::mbar_init(&o_upd[i], 1);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (CG == 2) tc::cluster_sync();  // both CTAs' barriers initialised before any cross-CTA arrival
  // the previous kernel on the stream must be done before any global or tensor memory is touched;
  // TMEM is allocated only after this wait, so a waiting CTA never holds columns another CTA needs
  tc::pdl_wait();
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
  tc::pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: Q once, then K_j / V_j into NS-stage rings ----------------
      // pairs: every load lands in this CTA's shared memory and completes on the leader's barrier,
      // which the leader arms for both CTAs' bytes
      bool ok = true;
      if (rank == 0) tc::mbar_arrive_expect_tx(q_full, C::Q_BYTES * CG);
      for (int c = 0; c < C::DCH; ++c) {
        if (CG == 2) tc::tma_load_4d_pair(smem + C::OFF_Q + c * (C::BQ * 128), &tmQ, leader_bar(q_full), c * 64, q0, h, b);
        else tc::tma_load_4d(smem + C::OFF_Q + c * (C::BQ * 128), &tmQ, q_full, c * 64, q0, h, b);
      }
      int issued_k[NS] = {}, issued_v[NS] = {};
      for (int j = 0; j < nblk && ok; ++j) {
        const int s = j % NS;
        const uint32_t ph = (uint32_t)((j / NS) & 1);
        if (!tc::mbar_wait(&k_empty[s], ph ^ 1, p.err) || *abort_flag) { ok = false; break; }
        if (rank == 0) tc::mbar_arrive_expect_tx(&k_full[s], C::K_BYTES * CG);
        for (int c = 0; c < C::DCH; ++c) {  // this CTA's keys of block j, all D columns
          uint8_t* dst = smem + C::OFF_K + s * C::K_BYTES + c * (C::KROWS * 128);
          const int krow = j * C::BKV + (int)rank * C::KROWS;
          if (CG == 2) tc::tma_load_4d_pair(dst, &tmK, leader_bar(&k_full[s]), c * 64, krow, h, b);
          else tc::tma_load_4d(dst, &tmK, &k_full[s], c * 64, krow, h, b);
        }
        issued_k[s]++;
        if (!tc::mbar_wait(&v_empty[s], ph ^ 1, p.err) || *abort_flag) { ok = false; break; }
        if (rank == 0) tc::mbar_arrive_expect_tx(&v_full[s], C::V_BYTES * CG);
        for (int c = 0; c < C::VCH; ++c) {  // all keys of block j, this CTA's 64-column V chunks
          uint8_t* dst = smem + C::OFF_V + s * C::V_BYTES + c * (C::BKV * 128);
          const int vcol = ((int)rank * C::VCH + c) * 64;
          if (CG == 2) tc::tma_load_4d_pair(dst, &tmV, leader_bar(&v_full[s]), vcol, j * C::BKV, h, b);
          else tc::tma_load_4d(dst, &tmV, &v_full[s], vcol, j * C::BKV, h, b);
        }
        issued_v[s]++;
      }
      if (ok && CG == 2) {
        // pairs: the leader's last commits arrive on this CTA's empty barriers; wait for them before
        // the CTA can leave
        for (int s = 0; s < NS; ++s) {
          if (issued_k[s]) tc::mbar_wait(&k_empty[s], (uint32_t)((issued_k[s] - 1) & 1), p.err);
          if (issued_v[s]) tc::mbar_wait(&v_empty[s], (uint32_t)((issued_v[s] - 1) & 1), p.err);
        }
      }
      if (!ok && rank == 0) {
        *abort_flag = 1;
        tc::mbar_wait(q_full, 0, nullptr);
        for (int s = 0; s < NS; ++s) {
          if (issued_k[s]) tc::mbar_wait(&k_full[s], (uint32_t)((issued_k[s] - 1) & 1), nullptr);
          if (issued_v[s]) tc::mbar_wait(&v_full[s], (uint32_t)((issued_v[s] - 1) & 1), nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (pairs: the leader only) ----------------
      // S_j = Q K_j^T into S[j&1]; once the softmax has replaced S_j by P_j (bf16, in TMEM),
      // O[j&1] += P_j V_j with A read from TMEM, then S_j+2 into the same columns: tcgen05.mma from
      // one thread executes in order, so S_j+2 cannot overwrite P_j before PV_j has read it.
      constexpr uint32_t IDESC_S = tc::idesc_f16(128 * CG, C::BKV, BF16, false, false);  // Q K^T: both K-major
      constexpr uint32_t IDESC_O = tc::idesc_f16(128 * CG, D, BF16, false, true);        // P V: V is MN-major
      const tc::SDesc qd = tc::sdesc_parts(tc::smem_u32(smem + C::OFF_Q), 16, 1024);
      bool ok = tc::mbar_wait(q_full, 0, p.err);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1, ks = j % NS;
        if (!tc::mbar_wait(&k_full[ks], (uint32_t)((j / NS) & 1), p.err)) return false;
        tc::tc_fence_after();
        const tc::SDesc kd = tc::sdesc_parts(tc::smem_u32(smem + C::OFF_K + ks * C::K_BYTES), 16, 1024);
        const uint32_t dst = tbase + C::T_S + s * 128;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t qoff = (k >> 2) * (C::BQ * 128) + (k & 3) * 32, koff = (k >> 2) * (C::KROWS * 128) + (k & 3) * 32;
          if (CG == 2) tc::mma_f16_ss_pair(dst, tc::sdesc_at(qd, qoff), tc::sdesc_at(kd, koff), IDESC_S, k > 0 ? 1u : 0u);
          else tc::mma_f16_ss(dst, tc::sdesc_at(qd, qoff), tc::sdesc_at(kd, koff), IDESC_S, k > 0 ? 1u : 0u);
        }
        if (CG == 2) {  // the S tile is ready in both CTAs; both CTAs' K stages are free
          tc::mma_commit_pair(&s_full[s], (uint16_t)3);
          tc::mma_commit_pair(&k_empty[ks], (uint16_t)3);
        } else {
          tc::mma_commit(&s_full[s]);
          tc::mma_commit(&k_empty[ks]);
        }
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nblk > 1) ok = issue_s(1);
      for (int j = 0; j < nblk && ok; ++j) {
        const int s = j & 1, ks = j % NS;
        if (!tc::mbar_wait(&p_full[s], (uint32_t)((j >> 1) & 1), p.err) ||
            !tc::mbar_wait(&v_full[ks], (uint32_t)((j / NS) & 1), p.err)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const tc::SDesc vd = tc::sdesc_parts(tc::smem_u32(smem + C::OFF_V + ks * C::V_BYTES), C::BKV * 128, 1024);
        const uint32_t o_dst = tbase + C::T_O + s * 128, p_src = tbase + C::T_S + s * 128;
        const uint32_t acc0 = j >= 2 ? 1u : 0u;
#pragma unroll
        for (int k = 0; k < C::BKV / 16; ++k) {
          if (CG == 2) tc::mma_f16_ts_pair(o_dst, p_src + k * 8, tc::sdesc_at(vd, k * 2048), IDESC_O, k > 0 ? 1u : acc0);
          else tc::mma_f16_ts(o_dst, p_src + k * 8, tc::sdesc_at(vd, k * 2048), IDESC_O, k > 0 ? 1u : acc0);
        }
        if (CG == 2) {
          tc::mma_commit_pair(&o_upd[s], (uint16_t)3);
          tc::mma_commit_pair(&v_empty[ks], (uint16_t)3);
        } else {
          tc::mma_commit(&o_upd[s]);
          tc::mma_commit(&v_empty[ks]);
        }
        if (j + 2 < nblk && !issue_s(j + 2)) ok = false;
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ---------------- softmax warpgroups: g = 0 takes even KV blocks, g = 1 odd ones ----------------
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row inside the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t t_s = tbase + C::T_S + g * 128, t_o = tbase + C::T_O + g * 128;
    const float2 sl2 = make_float2(p.scale_log2, p.scale_log2);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    int kb = 0;  // blocks processed by this warpgroup
    for (int j = g; j < nblk; j += 2, ++kb) {
      // S_j complete implies PV_j-2 of this group complete (issued before it, in-order execution)
      if (!tc::mbar_wait(&s_full[g], (uint32_t)(kb & 1), p.err) || *abort_flag) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      uint32_t sr[128];
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::tmem_ld32(t_s + c * 32 + lane_off, sr + 32 * c);
      tc::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) tc::reg_fence32(sr + 32 * c);
      const int64_t rem = p.Sk - (int64_t)j * C::BKV;
      if (rem < C::BKV) {  // ragged last block: keys past the end contribute exp2(-inf) = 0
#pragma unroll
        for (int e = 0; e < 128; ++e)
          if (e >= (int)rem) sr[e] = __float_as_uint(-INFINITY);
      }
      float mx8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx8[e] = __uint_as_float(sr[e]);
#pragma unroll
      for (int e = 8; e < 128; ++e) mx8[e & 7] = fmaxf(mx8[e & 7], __uint_as_float(sr[e]));
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float m_blk = mx * p.scale_log2;
      // lazy rescale: keep the old max unless the new one is more than 2^8 larger
      const bool need = (m == -INFINITY) || (m_blk > m + 8.f);
      float alpha = 1.f;
      if (need) {
        const float m_new = fmaxf(m, m_blk);
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_new);
        m = m_new;
      }
      if (kb > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < D / 16; ++c) {  // 16 columns at a time: the S row is still in registers
          uint32_t orow[16];
          tc::tmem_ld16(t_o + c * 16 + lane_off, orow);
          tc::tmem_wait_ld();
          tc::reg_fence16(orow);
#pragma unroll
          for (int e = 0; e < 16; ++e) orow[e] = __float_as_uint(__uint_as_float(orow[e]) * alpha);
          tc::tmem_st16(t_o + c * 16 + lane_off, orow);
        }
      }
      // P = exp2(s * scale_log2 - m) as 16-bit pairs, 64 keys at a time into TMEM columns [0, 64)
      // of this group's S tile: the A operand of the PV MMA
      const float2 nm = make_float2(-m, -m);
      float2 rs4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c = hh * 64 + 2 * i;
          const float2 x = __ffma2_rn(make_float2(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sl2, nm);
          const float2 e2 = make_float2(ex2(x.x), ex2(x.y));
          rs4[i & 3] = __fadd2_rn(rs4[i & 3], e2);
          w[i] = pack2(e2.x, e2.y, BF16);
        }
        tc::tmem_st32(t_s + hh * 32 + lane_off, w);
      }
      const float2 rs2 = __fadd2_rn(__fadd2_rn(rs4[0], rs4[1]), __fadd2_rn(rs4[2], rs4[3]));
      l = l * alpha + (rs2.x + rs2.y);
      tc::tmem_wait_st();
      tc::tc_fence_before();
      if (CG == 2) {  // one arrival per warp on the leader's barrier, after every lane's TMEM stores
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cluster(leader_bar(&p_full[g]));
      } else {
        tc::mbar_arrive(&p_full[g]);
      }
    }
    // ---------------- epilogue: combine the two groups, O / l -> global, lse ----------------
    // Each group's last PV completing implies every S MMA (hence every read of Q) is done, so the
    // (m, l) exchange can use the Q tile.
    const int nb0 = (nblk + 1) / 2, nb1 = nblk / 2;
    if (ok && kb > 0 && !tc::mbar_wait(&o_upd[g], (uint32_t)((kb - 1) & 1), p.err)) ok = false;
    float2* x0p = reinterpret_cast<float2*>(smem + C::OFF_Q);
    float2* x1p = x0p + C::BQ;
    tc::named_bar_sync(1, 256);  // both groups past their last PV before the Q tile is overwritten
    (g ? x1p : x0p)[r] = make_float2(m, l);
    tc::named_bar_sync(1, 256);
    if (ok && !*abort_flag) {
      tc::tc_fence_after();
      const float2 x0 = x0p[r], x1 = x1p[r];
      const float M = fmaxf(x0.x, x1.x);
      const float a0 = nb0 > 0 ? ex2(x0.x - M) : 0.f;
      const float a1 = nb1 > 0 ? ex2(x1.x - M) : 0.f;
      const float L = x0.y * a0 + x1.y * a1;
      const float s0 = a0 / L, s1 = a1 / L;
      const int64_t qrow = q0 + r;
      // O rows go through a per-warp staging tile in the (now idle) K ring: 32 rows x 32 columns per
      // box, 64-byte swizzle, one TMA store each (rows past Sq are clipped by the store)
      uint8_t* stg = smem + C::OFF_K + (warp - 2) * (D / 64) * 2048;
#pragma unroll
      for (int cc = 0; cc < D / 64; ++cc) {
        const int c = g * (D / 64) + cc;  // this group's 32-column chunks
        uint32_t o0[32], o1[32];
        __syncwarp();
        tc::tmem_ld32(tbase + C::T_O + c * 32 + lane_off, o0);
        if (nb1 > 0) tc::tmem_ld32(tbase + C::T_O + 128 + c * 32 + lane_off, o1);
        tc::tmem_wait_ld();
        tc::reg_fence32(o0);
        if (nb1 > 0) tc::reg_fence32(o1);
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float v0 = __uint_as_float(o0[2 * e]) * s0, v1 = __uint_as_float(o0[2 * e + 1]) * s0;
          if (nb1 > 0) {
            v0 += __uint_as_float(o1[2 * e]) * s1;
            v1 += __uint_as_float(o1[2 * e + 1]) * s1;
          }
          w[e] = pack2(v0, v1, BF16);
        }
        uint8_t* buf = stg + cc * 2048;
#pragma unroll
        for (int e = 0; e < 4; ++e)  // 16 B chunk e of row `lane` at (e ^ ((lane >> 1) & 3))
          *reinterpret_cast<uint4*>(buf + lane * 64 + ((e ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        tc::fence_async_shared();
        __syncwarp();
        if (lane == 0 && q0 + quarter * 32 < p.Sq) {  // boxes wholly past Sq (ragged last tile or pair) are skipped
          tc::tma_store_4d(&tmO, buf, c * 32, (int32_t)(q0 + quarter * 32), h, b);
          tc::bulk_commit();
        }
      }
      if (lane == 0) tc::bulk_wait0();
      if (g == 0 && qrow < p.Sq) p.lse[(int64_t)bh * p.Sq + qrow] = (M + __log2f(L)) * 0.6931471805599453f;
    } else {
      *abort_flag = 1;
    }
  }

  // Warps 0 and 1 reach here diverged (lane 0 ran the producer / MMA role): reconverge each warp
  // before the CTA barrier, which is an aligned barrier and must be executed by whole warps.
  __syncwarp();
  tc::tc_fence_before();
  __syncthreads();
  // pairs: neither CTA frees its TMEM or leaves while the other may still arrive on its barriers
  if (CG == 2) tc::cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc::tc_fence_after();
    if (CG == 2) tc::tmem_dealloc_pair(tbase, C::TMEM_COLS);
    else tc::tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// ---- tensor maps over [B, H, S, D] with arbitrary (b, h, s) strides -----------------------------
bool make_bhsd_map(CUtensorMap* m, const void* base, const int64_t* s3, int64_t B, int64_t H, int64_t S, int64_t D,
                   bool bf16, uint32_t box_rows, uint32_t box_inner = 64,
                   CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B) {
  uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  uint64_t strides[3] = {(uint64_t)s3[2] * 2, (uint64_t)s3[1] * 2, (uint64_t)s3[0] * 2};
  // size-1 dims: any valid stride
  if (S == 1) strides[0] = (uint64_t)D * 2;
  if (H == 1) strides[1] = strides[0] * (uint64_t)S;
  if (B == 1) strides[2] = strides[1] * (uint64_t)H;
  uint32_t box[4] = {box_inner, box_rows, 1, 1};
  return make_tmap(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, base, dims,
                   strides, box, sw);
}

bool strides_ok(const int64_t* s3, int64_t B, int64_t H, int64_t S) {
  auto ok = [](int64_t v) { return v > 0 && (v * 2) % 16 == 0; };
  return (S == 1 || ok(s3[2])) && (H == 1 || ok(s3[1])) && (B == 1 || ok(s3[0]));
}

}  // namespace

bool attn_tc_eligible(const b2_attn_args* a) {
  if (a->dtype != B2_BF16 && a->dtype != B2_F16) return false;
  if (a->D != 64 && a->D != 128) return false;
  if (!device_info().tcgen05) return false;
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (!al(a->q) || !al(a->k) || !al(a->v) || !al(a->o)) return false;
  if (!strides_ok(a->q_s, a->B, a->H, a->Sq) || !strides_ok(a->k_s, a->B, a->H, a->Sk) ||
      !strides_ok(a->v_s, a->B, a->H, a->Sk))
    return false;
  if ((a->o_s[2] % 8) || (a->o_s[1] % 8) || (a->o_s[0] % 8)) return false;  // 16-byte vector stores of O rows
  if (a->Sq >= (1ll << 31) || a->Sk >= (1ll << 31) || a->B * a->H > 65535) return false;
  return true;
}

template <int D, bool BF16, int CG>
int launch_fwd(const b2_attn_args* a, cudaStream_t st) {
  using C = FwdCfg<D, CG>;
  auto kern = attn_fwd_tc<D, BF16, CG>;
  static bool attr = false;
  if (!attr) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM),
                            "attn_fwd_tc attr"))
      return rc;
    attr = true;
  }
  CUtensorMap tq, tk, tv, to;
  if (!make_bhsd_map(&tq, a->q, a->q_s, a->B, a->H, a->Sq, D, BF16, 128) ||
      !make_bhsd_map(&tk, a->k, a->k_s, a->B, a->H, a->Sk, D, BF16, C::KROWS) ||
      !make_bhsd_map(&tv, a->v, a->v_s, a->B, a->H, a->Sk, D, BF16, 128) ||
      !make_bhsd_map(&to, a->o, a->o_s, a->B, a->H, a->Sq, D, BF16, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    return fail(B2_ERR_ARG, "attn_tc: tensor map rejected");
  AttnTcParams p{};
  p.B = a->B, p.H = a->H, p.Sq = a->Sq, p.Sk = a->Sk;
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.o = a->o;
  for (int i = 0; i < 3; ++i) p.o_s[i] = a->o_s[i];
  p.lse = a->lse;
  p.err = device_error_ptr();
  if (CG == 1) {
    dim3 grid((unsigned)((a->Sq + 127) / 128), (unsigned)(a->B * a->H));
    return launch_pdl("attn_fwd_tc", kern, grid, dim3(C::THREADS), C::SMEM, st, tq, tk, tv, to, p);
  }
  // CTA pairs: clusters of two along x, each pair over 256 query rows; programmatic dependent launch
  // as for single CTAs (outside stream capture)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(((a->Sq + 255) / 256) * 2), (unsigned)(a->B * a->H));
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2, at[0].val.clusterDim.y = 1, at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
    (void)cudaGetLastError();
    cs = cudaStreamCaptureStatusActive;
  }
  cfg.attrs = at;
  cfg.numAttrs = (pdl_enabled() && cs == cudaStreamCaptureStatusNone) ? 2 : 1;
  cudaError_t e;
  {
    LaunchScope ls("attn_fwd_tc_pair", st);
    e = cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, to, p);
  }
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail_cuda(e, "attn_fwd_tc_pair");
  }
  return after_launch("attn_fwd_tc_pair");
}

int attn_tc_fwd(const b2_attn_args* a, cudaStream_t st) {
  const bool bf16 = a->dtype == B2_BF16;
  // CTA pairs need D = 128 (V splits into two 64-column halves) and at least two query tiles. They are
  // opt-in (B2_ATTN_FWD_PAIRS=1): measured at B1 H16 S1024 D128 the pair form takes 21.3 us per forward
  // against 19.9 us for single CTAs (the softmax hand-off, not operand bandwidth, bounds this kernel)
  static const bool pairs_on = [] {
    const char* e = getenv("B2_ATTN_FWD_PAIRS");
    return e && e[0] == '1';
  }();
  if (a->D == 128 && a->Sq > 128 && pairs_on) return bf16 ? launch_fwd<128, true, 2>(a, st) : launch_fwd<128, false, 2>(a, st);
  if (a->D == 128) return bf16 ? launch_fwd<128, true, 1>(a, st) : launch_fwd<128, false, 1>(a, st);
  return bf16 ? launch_fwd<64, true, 1>(a, st) : launch_fwd<64, false, 1>(a, st);
}

int attn_simt_bwd_dispatch(const b2_attn_args* a, cudaStream_t st);  // attn_simt.cu

namespace {

// Bounded wait until the global counter reaches `target` (acquire at GPU scope); false (with the error
// word set) after the wait limit.
__device__ __forceinline__ bool wait_count(const int* ctr, int target, int* err) {
  uint64_t t0 = tc::globaltimer();
  for (;;) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if (tc::globaltimer() - t0 > tc::kWaitLimitNs) {
      if (err) atomicExch(err, tc::kErrMbarTimeout);
      return false;
    }
    __nanosleep(128);
  }
}

// ==================================================================================================
// backward (D = 128): one CTA per (128-key tile, batch*head), walking 64-query tiles; two compute
// warpgroups split each tile's 64 query columns (elementwise work needs no cross-group reduction)
// ==================================================================================================
struct BwdCfg {
  static constexpr int D = 128, BKV = 128, BQ = 64;
  static constexpr int KV_BYTES = BKV * D * 2;        // K or V tile, 32 KB
  static constexpr int QT_BYTES = BQ * D * 2;         // Q or dO tile, 16 KB
  static constexpr int PT_BYTES = BKV * BQ * 2;       // P^T or dS^T tile, 16 KB
  static constexpr int LD_BYTES = BQ * 8;             // (lse*log2e, delta) per query
  static constexpr int QS = 3;                        // Q / dO / (lse, delta) prefetch depth
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + KV_BYTES;
  static constexpr int OFF_Q = OFF_V + KV_BYTES;       // QS stages
  static constexpr int OFF_DO = OFF_Q + QS * QT_BYTES;  // QS stages
  static constexpr int OFF_DS = OFF_DO + QS * QT_BYTES;  // dS^T, 2 buffers (B operand of dQ^T)
  static constexpr int OFF_LD = OFF_DS + 2 * PT_BYTES;  // QS stages
  // dQ^T tile staging (fp32): two 128-row x 32-float boxes in the 128-byte swizzled TMA layout
  static constexpr int OFF_BAR = OFF_LD + QS * LD_BYTES;  // 256 bytes in the alignment gap before the staging tile
  static constexpr int OFF_STG = (OFF_BAR + 256 + 1023) / 1024 * 1024;
  static constexpr int STG_BYTES = D * BQ * 4;
  static constexpr int SMEM = OFF_STG + STG_BYTES + 1024;
  static_assert(SMEM <= 232448, "backward tile set exceeds the 227 KB shared-memory limit");
  static constexpr int NG = 4;                 // element-wise warpgroups, each owning BQ / NG query columns
  static constexpr int QPG = BQ / NG;          // 16
  static constexpr int NEW = 128 * NG;         // element-wise threads
  static constexpr int THREADS = 64 + NEW;
  // TMEM columns: S^T [0,64) dP^T [64,128) dQ^T [128,192) P^T [192,224) dS^T [224,256) (bf16 pairs,
  // A operands of dV / dK) dV [256,384) dK [384,512)
  static constexpr uint32_t T_S = 0, T_DP = 64, T_DQ = 128, T_PT = 192, T_DST = 224, T_DV = 256, T_DK = 384,
                            TMEM_COLS = 512;
};

// DSOUT = false: dQ^T_i = K^T dS^T_i is a fifth MMA per tile, added into an fp32 accumulator in L2.
// DSOUT = true (dS fits in L2): the dS^T tile in shared memory is stored by TMA to a bf16 [bh][Sk][sq_pad]
// buffer (tmDQ then maps that buffer) and one tensor-core GEMM dQ = scale * dS K follows the kernel.
template <bool DSOUT>
__global__ void __launch_bounds__(BwdCfg::THREADS, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ CUtensorMap tmDK,
                       const __grid_constant__ CUtensorMap tmDV, const __grid_constant__ CUtensorMap tmDQO,
                       AttnTcParams p, const float2* __restrict__ lsed, int64_t sq_pad) {
  using C = BwdCfg;
  constexpr bool BF16 = true;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  constexpr int QS = C::QS;
  uint64_t* kv_full = bar + 0;
  uint64_t* sdp_full = bar + 1;   // S^T_i and dP^T_i in TMEM
  uint64_t* pds_full = bar + 2;   // [2] P^T_i / dS^T_i written (count 256)
  uint64_t* pds_empty = bar + 4;  // [2] MMAs reading P^T_i / dS^T_i done
  uint64_t* dq_full = bar + 6;    // dQ^T_i in TMEM
  uint64_t* dq_empty = bar + 7;   // dQ^T_i drained (count 256)
  uint64_t* dkv_full = bar + 8;   // final dK, dV in TMEM
  uint64_t* sdp_empty = bar + 9;  // S^T_i / dP^T_i loaded into registers (count 256)
  uint64_t* q_full = bar + 10;    // [QS] Q_i, dO_i, (lse, delta)_i landed
  uint64_t* q_empty = bar + 10 + QS;  // [QS] all MMAs reading Q_i / dO_i done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 10 + 2 * QS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + 11 + 2 * QS);
  uint64_t* stg_full = bar + 12 + 2 * QS;  // dQ^T staging tile written (count 256)
  uint64_t* stg_free = bar + 13 + 2 * QS;  // the bulk reduction of the previous tile has read it
  uint64_t* ptm_empty = bar + 14 + 2 * QS;  // dV / dK MMAs of the previous tile read P^T / dS^T in TMEM
  // fused dQ (second phase): a 3-stage ring of (dS^T, K) blocks over the idle tile regions, the accumulator
  uint64_t* p2_full = bar + 15 + 2 * QS;     // [3] dS^T and K block landed
  uint64_t* p2_empty = bar + 18 + 2 * QS;    // [3] MMAs reading the block done
  uint64_t* p2_acc = bar + 21 + 2 * QS;      // dQ tile complete in TMEM
  uint64_t* p2_drained = bar + 22 + 2 * QS;  // dQ tile read out of TMEM (count NEW)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = blockIdx.x * C::BKV;
  const int bh = blockIdx.y;
  const int b = bh / (int)p.H, h = bh % (int)p.H;
  const int ntile = (int)((p.Sq + C::BQ - 1) / C::BQ);

  if (threadIdx.x == 0) {
    tc::mbar_init(kv_full, 1);
    for (int i = 0; i < QS; ++i) {
      tc::mbar_init(&q_full[i], 1);
      tc::mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&pds_full[i], C::NEW);
      tc::mbar_init(&pds_empty[i], 1);
    }
    tc::mbar_init(sdp_full, 1);
    tc::mbar_init(dq_full, 1);
    tc::mbar_init(dq_empty, C::NEW);
    tc::mbar_init(dkv_full, 1);
    tc::mbar_init(sdp_empty, C::NEW);
    tc::mbar_init(stg_full, C::NEW);
    tc::mbar_init(stg_free, 1);
    tc::mbar_init(ptm_empty, 1);
    for (int i = 0; i < 3; ++i) {
      tc::mbar_init(&p2_full[i], 1);
      tc::mbar_init(&p2_empty[i], 1);
    }
    tc::mbar_init(p2_acc, 1);
    tc::mbar_init(p2_drained, C::NEW);
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  // the previous kernel on the stream must be done before any global or tensor memory is touched;
  // TMEM is allocated only after this wait, so a waiting CTA never holds columns another CTA needs
  tc::pdl_wait();
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  tc::pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: K, V once; Q_i, dO_i, (lse, delta)_i into a 2-stage ring ----------------
      tc::mbar_arrive_expect_tx(kv_full, 2 * C::KV_BYTES);
      for (int c = 0; c < 2; ++c) {
        tc::tma_load_4d(smem + C::OFF_K + c * (C::BKV * 128), &tmK, kv_full, c * 64, k0, h, b);
        tc::tma_load_4d(smem + C::OFF_V + c * (C::BKV * 128), &tmV, kv_full, c * 64, k0, h, b);
      }
      int issued[QS] = {};
      bool ok = true;
      for (int i = 0; i < ntile; ++i) {
        const int s = i % QS;
        if (!tc::mbar_wait(&q_empty[s], ((uint32_t)(i / QS) & 1) ^ 1, p.err) || *abort_flag) {
          ok = false;
          break;
        }
        tc::mbar_arrive_expect_tx(&q_full[s], 2 * C::QT_BYTES + C::LD_BYTES);
        for (int c = 0; c < 2; ++c) {
          tc::tma_load_4d(smem + C::OFF_Q + s * C::QT_BYTES + c * (C::BQ * 128), &tmQ, &q_full[s], c * 64, i * C::BQ, h, b);
          tc::tma_load_4d(smem + C::OFF_DO + s * C::QT_BYTES + c * (C::BQ * 128), &tmDO, &q_full[s], c * 64, i * C::BQ, h, b);
        }
        tc::bulk_load(smem + C::OFF_LD + s * C::LD_BYTES, lsed + (int64_t)bh * sq_pad + (int64_t)i * C::BQ, C::LD_BYTES,
                      &q_full[s]);
        issued[s]++;
      }
      if (!ok) {
        *abort_flag = 1;
        tc::mbar_wait(kv_full, 0, nullptr);
        for (int s = 0; s < QS; ++s)
          if (issued[s]) tc::mbar_wait(&q_full[s], (uint32_t)((issued[s] - 1) & 1), nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t IDESC_SDP = tc::idesc_f16(128, C::BQ, BF16, false, false);  // K Q^T, V dO^T: K-major
      constexpr uint32_t IDESC_KV = tc::idesc_f16(128, C::D, BF16, false, true);     // P^T dO, dS^T Q: B MN-major
      constexpr uint32_t IDESC_DQ = tc::idesc_f16(128, C::BQ, BF16, true, true);     // K^T dS^T: A, B MN-major
      const uint32_t k_addr = tc::smem_u32(smem + C::OFF_K), v_addr = tc::smem_u32(smem + C::OFF_V);
      const tc::SDesc kd = tc::sdesc_parts(k_addr, 16, 1024), vd = tc::sdesc_parts(v_addr, 16, 1024);
      const tc::SDesc ktd = tc::sdesc_parts(k_addr, C::BKV * 128, 1024);  // K^T view (MN-major A of dQ^T)
      bool ok = tc::mbar_wait(kv_full, 0, p.err);
      auto issue_sdp = [&](int i) -> bool {
        const int s = i % QS;
        if (!tc::mbar_wait(&q_full[s], (uint32_t)((i / QS) & 1), p.err)) return false;
        tc::tc_fence_after();
        const tc::SDesc qd = tc::sdesc_parts(tc::smem_u32(smem + C::OFF_Q + s * C::QT_BYTES), 16, 1024);
        const tc::SDesc dod = tc::sdesc_parts(tc::smem_u32(smem + C::OFF_DO + s * C::QT_BYTES), 16, 1024);
#pragma unroll
        for (int k = 0; k < C::D / 16; ++k) {
          const uint32_t ka = (k >> 2) * (C::BKV * 128) + (k & 3) * 32;
          const uint32_t qa = (k >> 2) * (C::BQ * 128) + (k & 3) * 32;
          tc::mma_f16_ss(tbase + C::T_S, tc::sdesc_at(kd, ka), tc::sdesc_at(qd, qa), IDESC_SDP, k > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < C::D / 16; ++k) {
          const uint32_t ka = (k >> 2) * (C::BKV * 128) + (k & 3) * 32;
          const uint32_t qa = (k >> 2) * (C::BQ * 128) + (k & 3) * 32;
          tc::mma_f16_ss(tbase + C::T_DP, tc::sdesc_at(vd, ka), tc::sdesc_at(dod, qa), IDESC_SDP, k > 0 ? 1u : 0u);
        }
        tc::mma_commit(sdp_full);
        return true;
      };
      if (ok) ok = issue_sdp(0);
      for (int i = 0; i < ntile && ok; ++i) {
        const int s = i & 1;         // P^T / dS^T buffer
        const int qs = i % QS;       // Q / dO stage
        const uint32_t ph = (uint32_t)((i >> 1) & 1);
        // as soon as S^T_i / dP^T_i are in registers, the next tile's scores can go into TMEM
        if (!tc::mbar_wait(sdp_empty, (uint32_t)(i & 1), p.err)) { ok = false; break; }
        tc::tc_fence_after();
        if (i + 1 < ntile && !issue_sdp(i + 1)) { ok = false; break; }
        if (!tc::mbar_wait(&pds_full[s], ph, p.err)) { ok = false; break; }
        tc::tc_fence_after();
        const tc::SDesc qmd = tc::sdesc_parts(tc::smem_u32(smem + C::OFF_Q + qs * C::QT_BYTES), C::BQ * 128, 1024);
        const tc::SDesc domd = tc::sdesc_parts(tc::smem_u32(smem + C::OFF_DO + qs * C::QT_BYTES), C::BQ * 128, 1024);
        const tc::SDesc dsd = tc::sdesc_parts(tc::smem_u32(smem + C::OFF_DS + s * C::PT_BYTES), 8192, 1024);
        const uint32_t acc0 = i > 0 ? 1u : 0u;
        // dV += P^T dO ; dK += dS^T Q   (M = 128 keys, N = D, K = 64 queries; A from TMEM)
#pragma unroll
        for (int k = 0; k < C::BQ / 16; ++k)
          tc::mma_f16_ts(tbase + C::T_DV, tbase + C::T_PT + k * 8, tc::sdesc_at(domd, k * 2048), IDESC_KV, k > 0 ? 1u : acc0);
#pragma unroll
        for (int k = 0; k < C::BQ / 16; ++k)
          tc::mma_f16_ts(tbase + C::T_DK, tbase + C::T_DST + k * 8, tc::sdesc_at(qmd, k * 2048), IDESC_KV, k > 0 ? 1u : acc0);
        tc::mma_commit(&q_empty[qs]);
        tc::mma_commit(ptm_empty);
        if constexpr (!DSOUT) {
          // dQ^T = K^T dS^T (M = D, N = 64 queries, K = 128 keys) once the previous dQ^T was drained
          if (i > 0 && !tc::mbar_wait(dq_empty, (uint32_t)((i - 1) & 1), p.err)) { ok = false; break; }
          tc::tc_fence_after();
#pragma unroll
          for (int k = 0; k < C::BKV / 16; ++k)
            tc::mma_f16_ss(tbase + C::T_DQ, tc::sdesc_at(ktd, k * 2048), tc::sdesc_at(dsd, k * 2048), IDESC_DQ, k > 0 ? 1u : 0u);
          tc::mma_commit(dq_full);
          tc::mma_commit(&pds_empty[s]);
        }
      }
      if (ok) tc::mma_commit(dkv_full);
      else *abort_flag = 1;
    }
  } else {
    // ---------------- warps 2..: P^T / dS^T, dQ drain, dK/dV epilogue ----------------
    // thread = key row r (TMEM lane; also d for dQ^T); group g owns query columns [16g, 16g+16).
    // NG groups of 4 warps keep enough independent work in flight to hide TMEM / MUFU latency.
    constexpr int QPG = C::QPG;
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    // dQ^T_i (fp32, [d][64 queries]) leaves TMEM through a shared-memory staging tile and is added to
    // the accumulator tile [bh][i][d][64] by two TMA reductions performed in L2 (one per 32-query
    // box), issued by thread ew == 0: no per-thread atomics. The scale is applied at conversion.
    const int ew = threadIdx.x - 64;  // 0 .. NEW-1
    uint8_t* stg = smem + C::OFF_STG;
    const int64_t ntq = sq_pad / C::BQ;
    auto drain_dq = [&](int i) -> bool {
      if (!tc::mbar_wait(dq_full, (uint32_t)(i & 1), p.err)) return false;
      tc::tc_fence_after();
      uint32_t v[QPG];
      __syncwarp();
      tc::tmem_ld16(tbase + C::T_DQ + g * QPG + lane_off, v);
      tc::tmem_wait_ld();
      tc::reg_fence16(v);
      tc::tc_fence_before();
      tc::mbar_arrive(dq_empty);
      if (i > 0) {
        if (ew == 0) {
          tc::bulk_wait_read0();
          tc::mbar_arrive(stg_free);
        }
        if (!tc::mbar_wait(stg_free, (uint32_t)((i - 1) & 1), p.err)) return false;
      }
      // box g/2 (32 queries), row d = r: 4 16-byte chunks at their 128-byte-swizzle positions
      uint8_t* row = stg + (g >> 1) * (C::D * 128) + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int cc = (g & 1) * 4 + c;
        *reinterpret_cast<uint4*>(row + ((cc ^ (r & 7)) << 4)) = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
      }
      tc::fence_async_shared();
      tc::mbar_arrive(stg_full);
      if (ew == 0) {
        if (!tc::mbar_wait(stg_full, (uint32_t)(i & 1), p.err)) return false;
        const int32_t y = (int32_t)(((int64_t)bh * ntq + i) * C::D);
        tc::tma_reduce_add_2d(&tmDQ, stg, 0, y);
        tc::tma_reduce_add_2d(&tmDQ, stg + C::D * 128, 32, y);
        tc::bulk_commit();
      }
      return true;
    };
    for (int i = 0; i < ntile; ++i) {
      const int s = i & 1, qs = i % QS;
      if (!tc::mbar_wait(sdp_full, (uint32_t)(i & 1), p.err) || !tc::mbar_wait(&q_full[qs], (uint32_t)((i / QS) & 1), p.err) ||
          *abort_flag) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      uint32_t sv[QPG], dp[QPG];
      __syncwarp();
      tc::tmem_ld16(tbase + C::T_S + g * QPG + lane_off, sv);
      tc::tmem_ld16(tbase + C::T_DP + g * QPG + lane_off, dp);
      tc::tmem_wait_ld();
      tc::reg_fence16(sv);
      tc::reg_fence16(dp);
      tc::tc_fence_before();
      tc::mbar_arrive(sdp_empty);
      // (lse * log2e, delta) of two queries per 16-byte load; padding rows hold (+inf, 0)
      const float4* ld = reinterpret_cast<const float4*>(smem + C::OFF_LD + qs * C::LD_BYTES) + g * (QPG / 2);
      uint32_t wp[QPG / 2], wd[QPG / 2];
#pragma unroll
      for (int e = 0; e < QPG / 2; ++e) {
        const float4 L = ld[e];
        const float p0 = ex2(fmaf(__uint_as_float(sv[2 * e]), p.scale_log2, -L.x));
        const float p1 = ex2(fmaf(__uint_as_float(sv[2 * e + 1]), p.scale_log2, -L.z));
        const float2 ds = __fmul2_rn(make_float2(p0, p1), __fadd2_rn(make_float2(__uint_as_float(dp[2 * e]),
                                                                                 __uint_as_float(dp[2 * e + 1])),
                                                                     make_float2(-L.y, -L.w)));
        wp[e] = pack2(p0, p1, BF16);
        wd[e] = pack2(ds.x, ds.y, BF16);
      }
      // P^T / dS^T in TMEM were read by the dV / dK MMAs of tile i-1
      if (i >= 1 && !tc::mbar_wait(ptm_empty, (uint32_t)((i - 1) & 1), p.err)) { ok = false; break; }
      tc::tc_fence_after();
      tc::tmem_st8(tbase + C::T_PT + g * (QPG / 2) + lane_off, wp);
      tc::tmem_st8(tbase + C::T_DST + g * (QPG / 2) + lane_off, wd);
      // dS^T buffer s in shared memory was last read by the dQ^T MMA of tile i-2
      if (i >= 2 && !tc::mbar_wait(&pds_empty[s], (uint32_t)(((i - 2) >> 1) & 1), p.err)) { ok = false; break; }
      uint8_t* dst = smem + C::OFF_DS + s * C::PT_BYTES + r * 128;
#pragma unroll
      for (int q2 = 0; q2 < QPG / 8; ++q2) {  // granules of 8 queries, 128-byte swizzled rows
        const int gr = g * (QPG / 8) + q2;
        *reinterpret_cast<uint4*>(dst + ((gr ^ (r & 7)) << 4)) =
            make_uint4(wd[4 * q2], wd[4 * q2 + 1], wd[4 * q2 + 2], wd[4 * q2 + 3]);
      }
      tc::tmem_wait_st();
      tc::fence_async_shared();
      tc::tc_fence_before();
      if constexpr (DSOUT) {
        // stg_full before pds_full: a thread can reach tile i+1's stg_full arrival only after the dV / dK
        // MMAs of tile i, i.e. after every thread's pds_full (and so stg_full) arrival for tile i
        tc::mbar_arrive(stg_full);
        tc::mbar_arrive(&pds_full[s]);
        if (ew == 0) {
          if (!tc::mbar_wait(stg_full, (uint32_t)(i & 1), p.err)) { ok = false; break; }
          tc::tma_store_3d(&tmDQ, smem + C::OFF_DS + s * C::PT_BYTES, i * C::BQ, k0, bh);
          tc::bulk_commit();
          // the store of tile i-1 has read its buffer: the dS^T of tile i+1 may be written there
          tc::bulk_wait_read1();
          if (i > 0) tc::mbar_arrive(&pds_empty[s ^ 1]);
        }
      } else {
        tc::mbar_arrive(&pds_full[s]);
        if (i > 0 && !drain_dq(i - 1)) { ok = false; break; }
      }
    }
    if constexpr (!DSOUT) {
      if (ok && ntile > 0) ok = drain_dq(ntile - 1);
    }
    if (ew == 0) tc::bulk_wait0();
    if (DSOUT && p.dsready != nullptr && ew == 0) {
      // this CTA's dS^T stores are complete: publish them to the other CTAs of the head (whose TMA
      // loads read them in the second phase); also on the error path, so that nobody waits for it
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence();
      atomicAdd(&p.dsready[bh], 1);
    }
    // ---------------- dK, dV epilogue: group g writes d columns [32g, 32g+32) ----------------
    if (ok && tc::mbar_wait(dkv_full, 0, p.err)) {
      tc::tc_fence_after();
      // rows go through a per-warp staging tile in the (now idle) Q / dO rings: 32 rows x 32 columns
      // per box, 64-byte swizzle, one TMA store each (rows past Sk are clipped by the store)
      uint8_t* estg = smem + C::OFF_Q + (warp - 2) * 4096;
      for (int which = 0; which < 2; ++which) {  // 0: dV, 1: dK (times scale)
        void* base = which ? p.dk : p.dv;
        const float mul = which ? p.scale : 1.f;
        const uint32_t tcol = which ? C::T_DK : C::T_DV;
        uint32_t v[32];
        __syncwarp();
        tc::tmem_ld32(tbase + tcol + g * 32 + lane_off, v);
        tc::tmem_wait_ld();
        tc::reg_fence32(v);
        if (base) {
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            w[e] = pack2(__uint_as_float(v[2 * e]) * mul, __uint_as_float(v[2 * e + 1]) * mul, BF16);
          uint8_t* buf = estg + which * 2048;
#pragma unroll
          for (int e = 0; e < 4; ++e)  // 16 B chunk e of row `lane` at (e ^ ((lane >> 1) & 3))
            *reinterpret_cast<uint4*>(buf + lane * 64 + ((e ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
          tc::fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            tc::tma_store_4d(which ? &tmDK : &tmDV, buf, g * 32, (int32_t)(k0 + quarter * 32), h, b);
            tc::bulk_commit();
          }
        }
      }
      if (lane == 0) tc::bulk_wait0();
    } else {
      *abort_flag = 1;
    }
  }

  // Warps 0 and 1 reach here diverged (lane 0 ran the producer / MMA role): reconverge each warp
  // before the CTA barrier, which is an aligned barrier and must be executed by whole warps.
  __syncwarp();
  tc::tc_fence_before();
  __syncthreads();

  if constexpr (DSOUT) if (p.dsready != nullptr) {
    // ---------------- second phase: dQ = scale * dS K for this CTA's 128-query tiles ----------------
    // Every CTA of the grid is resident (cooperative launch), so the wait for the other key tiles of
    // the head ends. Query tiles qt = blockIdx.x, blockIdx.x + nkt, ... of the head; the reduction runs
    // over its nkt 128-key blocks: A = dS (M-major, read through the dS^T buffer in L2), B = K (N-major),
    // both TMA-loaded in 64-element-wide boxes into a 3-stage ring of 64 KB stages laid over the idle
    // K / V / Q / dO / dS^T regions; the accumulator reuses dV's TMEM columns (drained above).
    constexpr int P2S = 3;
    constexpr int P2_STAGE = 65536;
    static_assert(P2S * P2_STAGE <= C::OFF_LD, "second-phase ring overlaps the (lse, delta) ring");
    const int nkt = (int)gridDim.x;
    const int nqt = (int)((p.Sq + 127) / 128);
    if (warp == 0) {
      if (lane == 0) {
        bool ok = !*abort_flag && wait_count(&p.dsready[bh], nkt, p.err);
        asm volatile("fence.proxy.async.global;" ::: "memory");  // the TMA loads below see those stores
        int st = 0, issued[P2S] = {0, 0, 0};
        uint32_t ph = 0;
        for (int qt = (int)blockIdx.x; qt < nqt && ok; qt += nkt) {
          for (int kb = 0; kb < nkt; ++kb) {
            if (!tc::mbar_wait(&p2_empty[st], ph ^ 1, p.err) || *abort_flag) {
              ok = false;
              break;
            }
            uint8_t* sa = smem + st * P2_STAGE;
            tc::mbar_arrive_expect_tx(&p2_full[st], P2_STAGE);
            tc::tma_load_3d(sa, &tmDQ, &p2_full[st], qt * 128, kb * C::BKV, bh);
            tc::tma_load_3d(sa + 16384, &tmDQ, &p2_full[st], qt * 128 + 64, kb * C::BKV, bh);
            tc::tma_load_4d(sa + 32768, &tmK, &p2_full[st], 0, kb * C::BKV, h, b);
            tc::tma_load_4d(sa + 49152, &tmK, &p2_full[st], 64, kb * C::BKV, h, b);
            issued[st]++;
            if (++st == P2S) st = 0, ph ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          for (int i = 0; i < P2S; ++i)
            if (issued[i]) tc::mbar_wait(&p2_full[i], (uint32_t)((issued[i] - 1) & 1), nullptr);
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t IDESC_P2 = tc::idesc_f16(128, 128, BF16, true, true);  // A, B MN-major
        int st = 0, tcount = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int qt = (int)blockIdx.x; qt < nqt && ok; qt += nkt, ++tcount) {
          if (tcount > 0 && !tc::mbar_wait(p2_drained, (uint32_t)((tcount - 1) & 1), p.err)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          for (int kb = 0; kb < nkt; ++kb) {
            if (!tc::mbar_wait(&p2_full[st], ph, p.err) || *abort_flag) {
              ok = false;
              break;
            }
            tc::tc_fence_after();
            const uint32_t sa = tc::smem_u32(smem + st * P2_STAGE);
            const tc::SDesc ad = tc::sdesc_parts(sa, 16384, 1024);          // dS: two 64-query chunks
            const tc::SDesc bd = tc::sdesc_parts(sa + 32768, 16384, 1024);  // K: two 64-column chunks
#pragma unroll
            for (int k = 0; k < C::BKV / 16; ++k)
              tc::mma_f16_ss(tbase + C::T_DV, tc::sdesc_at(ad, k * 2048), tc::sdesc_at(bd, k * 2048), IDESC_P2,
                             (kb > 0 || k > 0) ? 1u : 0u);
            tc::mma_commit(&p2_empty[st]);
            if (++st == P2S) st = 0, ph ^= 1;
          }
          if (ok) tc::mma_commit(p2_acc);
        }
        if (!ok) *abort_flag = 1;
      }
    } else {
      // warp (group g, quarter): 32 query rows x 32 d columns per tile, through a per-warp 2 KB staging
      // box in the idle dQ^T staging region and one TMA store (boxes wholly past Sq are skipped)
      const int g = (warp - 2) >> 2, quarter = warp & 3;
      const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
      uint8_t* buf = smem + C::OFF_STG + (warp - 2) * 2048;
      int tcount = 0;
      for (int qt = (int)blockIdx.x; qt < nqt; qt += nkt, ++tcount) {
        if (!tc::mbar_wait(p2_acc, (uint32_t)(tcount & 1), p.err) || *abort_flag) {
          *abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        uint32_t v[32];
        __syncwarp();
        tc::tmem_ld32(tbase + C::T_DV + g * 32 + lane_off, v);
        tc::tmem_wait_ld();
        tc::reg_fence32(v);
        tc::tc_fence_before();
        tc::mbar_arrive(p2_drained);
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          w[e] = pack2(__uint_as_float(v[2 * e]) * p.scale, __uint_as_float(v[2 * e + 1]) * p.scale, BF16);
        if (lane == 0) tc::bulk_wait_read0();  // the previous tile's store has read the staging box
        __syncwarp();
#pragma unroll
        for (int e = 0; e < 4; ++e)
          *reinterpret_cast<uint4*>(buf + lane * 64 + ((e ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
        tc::fence_async_shared();
        __syncwarp();
        const int64_t r0 = (int64_t)qt * 128 + quarter * 32;
        if (lane == 0 && r0 < p.Sq) {
          tc::tma_store_4d(&tmDQO, buf, g * 32, (int32_t)r0, h, b);
          tc::bulk_commit();
        }
      }
      if (lane == 0) tc::bulk_wait0();
    }
    __syncwarp();
    tc::tc_fence_before();
    __syncthreads();
  }

  if (warp == 1) {
    __syncwarp();
    tc::tc_fence_after();
    tc::tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// Pre-pass, one block per (64-query tile, batch*head): lsed[bh][q] = (lse*log2e, rowsum(O*dO)) with
// (+inf, 0) for padding rows, and zero the tile of the fp32 dQ accumulator [bh][q/64][d][64].
__global__ void __launch_bounds__(256) attn_bwd_prep(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ d_o,
                                                     const float* __restrict__ lse, float2* __restrict__ lsed,
                                                     float* __restrict__ dq_acc, int* __restrict__ dsready, int64_t H,
                                                     int64_t Sq, int64_t sq_pad, int64_t o0, int64_t o1, int64_t o2,
                                                     int64_t g0, int64_t g1, int64_t g2) {
  tc::pdl_wait();
  tc::pdl_trigger();
  const int64_t bh = blockIdx.y, b = bh / H, h = bh % H;
  if (dsready && blockIdx.x == 0 && blockIdx.z == 0 && threadIdx.x == 0) dsready[bh] = 0;  // fused-dQ counter
  const int64_t q0 = (int64_t)blockIdx.x * 64;
  if (blockIdx.z == 1) {  // the zeroing blocks run beside the delta blocks
    float4* acc = reinterpret_cast<float4*>(dq_acc + (bh * (sq_pad / 64) + blockIdx.x) * (128 * 64));
#pragma unroll
    for (int it = 0; it < 8; ++it) acc[threadIdx.x + it * 256] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  // thread = (row, quarter of the 128-wide row): 4 x 16-byte loads of O and of dO, all in flight at once
  const int row = threadIdx.x >> 2, qtr = threadIdx.x & 3;
  const int64_t q = q0 + row;
  float s = 0.f;
  if (q < Sq) {
    const uint4* op = reinterpret_cast<const uint4*>(o + b * o0 + h * o1 + q * o2) + qtr * 4;
    const uint4* gp = reinterpret_cast<const uint4*>(d_o + b * g0 + h * g1 + q * g2) + qtr * 4;
    uint4 a[4], c[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) a[e] = __ldg(op + e), c[e] = __ldg(gp + e);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a[e]);
      const __nv_bfloat162* c2 = reinterpret_cast<const __nv_bfloat162*>(&c[e]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 x = __bfloat1622float2(a2[k]), y = __bfloat1622float2(c2[k]);
        s += x.x * y.x + x.y * y.y;
      }
    }
  }
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  if (qtr == 0)
    lsed[bh * sq_pad + q] = q < Sq ? make_float2(lse[bh * Sq + q] * 1.4426950408889634f, s) : make_float2(INFINITY, 0.f);
}

// dq[b,h,q,:] = bf16(dq_acc[bh][:][q]), one block per (64-query tile, batch*head), transposed through
// shared memory so both the fp32 reads and the bf16 writes are 16-byte and coalesced.
__global__ void __launch_bounds__(256) attn_dq_convert(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dq,
                                                       int64_t H, int64_t Sq, int64_t sq_pad, int64_t s0, int64_t s1,
                                                       int64_t s2, float scale) {
  __shared__ float t[128][33];
  tc::pdl_wait();
  tc::pdl_trigger();
  const int64_t bh = blockIdx.y, b = bh / H, h = bh % H;
  const int half = blockIdx.x & 1;
  const int64_t q0 = (int64_t)(blockIdx.x >> 1) * 64 + half * 32;
  const float* tile = dq_acc + (bh * (sq_pad / 64) + (blockIdx.x >> 1)) * (128 * 64) + half * 32;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int e = threadIdx.x + it * 256;  // 128 d-rows x 8 float4
    const int d = e >> 3, j = (e & 7) * 4;
    float4 v = *reinterpret_cast<const float4*>(tile + d * 64 + j);
    t[d][j] = v.x * scale, t[d][j + 1] = v.y * scale, t[d][j + 2] = v.z * scale, t[d][j + 3] = v.w * scale;
  }
  __syncthreads();
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int e = threadIdx.x + it * 256;  // 32 rows x 16 chunks of 8 d
    const int j = e >> 4, d0 = (e & 15) * 8;
    const int64_t q = q0 + j;
    if (q >= Sq) continue;
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = pack2(t[d0 + 2 * k][j], t[d0 + 2 * k + 1][j], true);
    *reinterpret_cast<uint4*>(dq + b * s0 + h * s1 + q * s2 + d0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace

bool attn_tc_bwd_eligible(const b2_attn_args* a) {
  if (!attn_tc_eligible(a) || a->D != 128 || a->dtype != B2_BF16) return false;
  if (!strides_ok(a->do_s, a->B, a->H, a->Sq) || ((uintptr_t)a->d_o & 15)) return false;
  if (a->B * a->H * ((a->Sq + 63) / 64 * 64) * 2 >= (1ll << 31)) return false;  // dQ accumulator rows fit int32
  if ((a->do_s[2] % 8) || (a->do_s[1] % 8) || (a->do_s[0] % 8)) return false;
  auto al = [](const void* p) { return p == nullptr || ((uintptr_t)p & 15) == 0; };
  if (!al(a->dk) || !al(a->dv) || !al(a->dq)) return false;
  for (int i = 0; i < 3; ++i)
    if ((a->dk && a->dk_s[i] % 8) || (a->dv && a->dv_s[i] % 8) || (a->dq && a->dq_s[i] % 8)) return false;
  return true;
}

// dS^T [B*H][Sk][sq_pad] bf16 stays in L2 between the backward kernel and the dQ GEMM up to this size
constexpr uint64_t kDsOutMaxBytes = 64ull << 20;

// The dS-out form pays a separate GEMM launch (~10 us at B1 H16 S1024) to take the dQ^T MMA and its fp32
// traffic out of the key-tile CTAs. Measured (graphs of back-to-back fwd+bwd, B1 H16 D128): it wins when
// those CTAs fill at most half the GPU (Sq x Sk = 1024 x 512: 50.0 -> 47.8 us; 4096 x 512: 168 -> 154 us)
// and loses when they fill it (1024 x 1024: 54.5 -> 56.9 us; 2048 x 2048: even).
// B2_ATTN_BWD_DSOUT=0 / =1 pins the form (A/B measurements and the tests of both forms).
// When every key-tile CTA fits on the GPU at once (one CTA per SM), the dQ GEMM runs inside the backward
// kernel instead, as a second phase after the CTAs of a head have stored their dS^T tiles (cooperative
// launch: all CTAs resident, so the wait for the head's other CTAs ends); B2_ATTN_BWD_FUSEDQ=0 keeps the
// separate GEMM.
bool attn_bwd_fusedq(const b2_attn_args* a) {
  static const bool off = [] {
    const char* e = getenv("B2_ATTN_BWD_FUSEDQ");
    return e && e[0] == '0';
  }();
  const int64_t key_ctas = a->B * a->H * ((a->Sk + 127) / 128);
  return !off && device_info().coop_launch && key_ctas <= (int64_t)device_info().sm_count;
}

bool attn_bwd_dsout(const b2_attn_args* a) {
  static const int pinned = [] {
    const char* e = getenv("B2_ATTN_BWD_DSOUT");
    return e && (e[0] == '0' || e[0] == '1') ? e[0] - '0' : -1;
  }();
  const int64_t sq_pad = (a->Sq + 63) / 64 * 64;
  if (pinned == 0 || a->dq == nullptr ||
      (uint64_t)(a->B * a->H) * (uint64_t)a->Sk * (uint64_t)sq_pad * 2 > kDsOutMaxBytes)
    return false;
  if (pinned == 1 || attn_bwd_fusedq(a)) return true;
  const int64_t key_ctas = a->B * a->H * ((a->Sk + 127) / 128);
  return 2 * key_ctas <= (int64_t)device_info().sm_count;
}

// workspace = (dS^T bf16 [B*H][Sk][sq_pad] and, after the (lse, delta) pairs, one int per (b, h) for the
// fused form, when attn_bwd_dsout; else the fp32 dQ accumulator [B*H][sq_pad/64][D][64]) with
// (lse*log2e, delta) [B*H][sq_pad] after it
uint64_t attn_bwd_ws_bytes(const b2_attn_args* a) {
  if (!attn_tc_bwd_eligible(a)) return 0;
  const int64_t sq_pad = (a->Sq + 63) / 64 * 64;
  const bool ds = attn_bwd_dsout(a);
  const uint64_t per_q = ds ? (uint64_t)a->Sk * 2 + 8 : (uint64_t)(a->D * 4 + 8);
  const uint64_t extra = ds ? ((uint64_t)(a->B * a->H) * 4 + 15) / 16 * 16 : 0;
  return (uint64_t)(a->B * a->H) * (uint64_t)sq_pad * per_q + extra;
}

template <bool DSOUT>
int set_bwd_smem_attr() {
  static bool attr = false;
  if (!attr) {
    if (int rc = check_cuda(cudaFuncSetAttribute(attn_bwd_tc_kernel<DSOUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 BwdCfg::SMEM),
                            "attn_bwd_tc attr"))
      return rc;
    attr = true;
  }
  return 0;
}

int attn_tc_bwd(const b2_attn_args* a, cudaStream_t st) {
  if (!attn_tc_bwd_eligible(a)) return attn_simt_bwd_dispatch(a, st);
  if (!a->workspace || ((uintptr_t)a->workspace & 15))
    return fail(B2_ERR_ARG, "attn_bwd: a 16-byte aligned workspace of b2_attn_bwd_workspace_bytes() is required");
  using C = BwdCfg;
  const bool dsout = attn_bwd_dsout(a);
  if (int rc = dsout ? set_bwd_smem_attr<true>() : set_bwd_smem_attr<false>()) return rc;
  const int64_t BH = a->B * a->H;
  const int64_t sq_pad = (a->Sq + 63) / 64 * 64;
  float* dq_acc = (float*)a->workspace;                                 // !dsout
  __nv_bfloat16* ds_t = (__nv_bfloat16*)a->workspace;                   // dsout
  float2* lsed = dsout ? reinterpret_cast<float2*>(ds_t + BH * a->Sk * sq_pad)
                       : reinterpret_cast<float2*>(dq_acc + BH * a->D * sq_pad);
  const bool fused = dsout && attn_bwd_fusedq(a);
  int* dsready = fused ? reinterpret_cast<int*>(lsed + BH * sq_pad) : nullptr;
  {
    // z = 1: (lse, delta) blocks only; z = 2 adds the blocks that zero the dQ accumulator
    dim3 grid((unsigned)(sq_pad / 64), (unsigned)BH, dsout ? 1u : 2u);
    if (int rc = launch_pdl("attn_bwd_prep", attn_bwd_prep, grid, dim3(256), 0, st, (const __nv_bfloat16*)a->o,
                            (const __nv_bfloat16*)a->d_o, (const float*)a->lse, lsed, dq_acc, dsready, (int64_t)a->H,
                            (int64_t)a->Sq, sq_pad, a->o_s[0], a->o_s[1], a->o_s[2], a->do_s[0], a->do_s[1],
                            a->do_s[2]))
      return rc;
  }
  CUtensorMap tq, tk, tv, tdo, tdq;
  if (dsout) {
    // dS^T as [BH][Sk][sq_pad] bf16, written in 64-query x 128-key boxes (the swizzled shared-memory tile)
    const uint64_t dims[3] = {(uint64_t)sq_pad, (uint64_t)a->Sk, (uint64_t)BH};
    const uint64_t strides[2] = {(uint64_t)sq_pad * 2, (uint64_t)a->Sk * (uint64_t)sq_pad * 2};
    const uint32_t box[3] = {64, 128, 1};
    if (!make_tmap(&tdq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ds_t, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(B2_ERR_ARG, "attn_bwd_tc: dS tensor map rejected");
  } else {
    // dQ accumulator as [B*H*sq_pad/64*D rows][64 fp32], reduced into in 128 x 32 boxes
    const uint64_t dims[2] = {64, (uint64_t)(BH * (sq_pad / 64) * 128)};
    const uint64_t strides[1] = {256};
    const uint32_t box[2] = {32, 128};
    if (!make_tmap(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dq_acc, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(B2_ERR_ARG, "attn_bwd_tc: dQ accumulator tensor map rejected");
  }
  if (!make_bhsd_map(&tq, a->q, a->q_s, a->B, a->H, a->Sq, 128, true, 64) ||
      !make_bhsd_map(&tk, a->k, a->k_s, a->B, a->H, a->Sk, 128, true, 128) ||
      !make_bhsd_map(&tv, a->v, a->v_s, a->B, a->H, a->Sk, 128, true, 128) ||
      !make_bhsd_map(&tdo, a->d_o, a->do_s, a->B, a->H, a->Sq, 128, true, 64))
    return fail(B2_ERR_ARG, "attn_bwd_tc: tensor map rejected");
  // dK / dV (when requested) are written by TMA stores of 32 x 32 boxes
  CUtensorMap tdk, tdv, tdqo;
  memset(&tdk, 0, sizeof(tdk));
  memset(&tdv, 0, sizeof(tdv));
  memset(&tdqo, 0, sizeof(tdqo));
  if ((a->dk && !make_bhsd_map(&tdk, a->dk, a->dk_s, a->B, a->H, a->Sk, 128, true, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) ||
      (a->dv && !make_bhsd_map(&tdv, a->dv, a->dv_s, a->B, a->H, a->Sk, 128, true, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)) ||
      (fused && !make_bhsd_map(&tdqo, a->dq, a->dq_s, a->B, a->H, a->Sq, 128, true, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B)))
    return fail(B2_ERR_ARG, "attn_bwd_tc: dK / dV / dQ tensor map rejected");
  AttnTcParams p{};
  p.B = a->B, p.H = a->H, p.Sq = a->Sq, p.Sk = a->Sk;
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.lse = a->lse;
  p.dq_acc = dq_acc;
  p.dk = a->dk, p.dv = a->dv;
  for (int i = 0; i < 3; ++i) p.dk_s[i] = a->dk_s[i], p.dv_s[i] = a->dv_s[i];
  p.err = device_error_ptr();
  p.dsready = dsready;
  if (fused) {
    // all CTAs resident at once (the second phase waits for the head's other key tiles)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a->Sk + 127) / 128), (unsigned)BH);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at, cfg.numAttrs = 1;
    cudaError_t e;
    {
      LaunchScope ls("attn_bwd_tc_fusedq", st);
      e = cudaLaunchKernelEx(&cfg, attn_bwd_tc_kernel<true>, tq, tk, tv, tdo, tdq, tdk, tdv, tdqo, p,
                             (const float2*)lsed, sq_pad);
    }
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return fail_cuda(e, "attn_bwd_tc_fusedq");
    }
    return after_launch("attn_bwd_tc_fusedq");
  }
  {
    dim3 grid((unsigned)((a->Sk + 127) / 128), (unsigned)BH);
    int rc = dsout ? launch_pdl("attn_bwd_tc", attn_bwd_tc_kernel<true>, grid, dim3(C::THREADS), C::SMEM, st, tq, tk, tv,
                                tdo, tdq, tdk, tdv, tdqo, p, (const float2*)lsed, sq_pad)
                   : launch_pdl("attn_bwd_tc", attn_bwd_tc_kernel<false>, grid, dim3(C::THREADS), C::SMEM, st, tq, tk, tv,
                                tdo, tdq, tdk, tdv, tdqo, p, (const float2*)lsed, sq_pad);
    if (rc) return rc;
  }
  if (dsout) {
    // dQ[b, h] = scale * dS[b, h] K[b, h]: A = dS (Sq x Sk) read through dS^T (M-major), B = K (Sk x D,
    // N-major), one batched tensor-core GEMM over the heads of each batch entry
    for (int64_t b = 0; b < a->B; ++b) {
      b2_gemm_args g{};
      g.a = ds_t + b * a->H * a->Sk * sq_pad;
      g.b = (const __nv_bfloat16*)a->k + b * a->k_s[0];
      g.c = (__nv_bfloat16*)a->dq + b * a->dq_s[0];
      g.M = a->Sq, g.N = a->D, g.K = a->Sk, g.batch = a->H;
      g.a_sb = a->Sk * sq_pad, g.a_sm = 1, g.a_sk = sq_pad;
      g.b_sb = a->k_s[1], g.b_sk = a->k_s[2], g.b_sn = 1;
      g.c_sb = a->dq_s[1], g.c_sm = a->dq_s[2], g.c_sn = 1;
      g.alpha = a->scale, g.beta = 0.f;
      g.dtype = B2_BF16;
      if (int rc = b2_gemm(&g, st)) return rc;
    }
  } else if (a->dq) {
    dim3 grid((unsigned)(sq_pad / 32), (unsigned)BH);
    if (int rc = launch_pdl("attn_dq_convert", attn_dq_convert, grid, dim3(256), 0, st, (const float*)dq_acc,
                            (__nv_bfloat16*)a->dq, (int64_t)a->H, (int64_t)a->Sq, sq_pad, a->dq_s[0], a->dq_s[1],
                            a->dq_s[2], a->scale))
      return rc;
  }
  return 0;
}

}  // namespace b2

extern "C" uint64_t b2_attn_bwd_workspace_bytes(const b2_attn_args* a) { return a ? b2::attn_bwd_ws_bytes(a) : 0; }
