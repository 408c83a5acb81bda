// Strided SIMT flash attention (fp32 math): the general path of b2_attn_fwd / b2_attn_bwd for fp32
// inputs and for head dims / layouts the tensor-core kernels do not take (D not a multiple of 16,
// unaligned views).
//
// Algorithm = the reference's scalar kernels vkrt/shaders/attn.comp.in: MODE 0 forward with online
// softmax (256-313), MODE 3 delta = rowsum(O*dO) (210-240), MODE 1 dK/dV (315-362), MODE 2 dQ
// (364-394); lse is the natural-log logsumexp. Layout: a block of 4 warps owns 16 query (or key)
// rows, K/V (or Q/dO) tiles of 32 rows are staged in shared memory as fp32; lane j scores row j of
// the tile, lane d owns output columns d, d+32, d+64, d+96.
#include "common.cuh"

namespace b2 {

int attn_tc_fwd(const b2_attn_args* a, cudaStream_t st);  // attn_tc.cu
int attn_tc_bwd(const b2_attn_args* a, cudaStream_t st);
bool attn_tc_eligible(const b2_attn_args* a);

namespace {

constexpr int TILE = 32;       // keys (queries) per shared-memory tile
constexpr int ROWS_PER_WARP = 4;
constexpr int WARPS = 4;
constexpr int ROWS = ROWS_PER_WARP * WARPS;  // rows per block
constexpr int DMAX = 128;
constexpr int DP = DMAX + 1;  // padded smem row

template <typename T>
__device__ __forceinline__ const T* row_ptr(const void* base, const int64_t* s, int64_t b, int64_t h, int64_t i) {
  return (const T*)base + b * s[0] + h * s[1] + i * s[2];
}

template <typename T>
__global__ void __launch_bounds__(128) attn_fwd_simt(b2_attn_args p) {
  __shared__ float Ks[TILE][DP], Vs[TILE][DP];
  __shared__ float Qs[ROWS][DMAX];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int64_t q0 = (int64_t)blockIdx.x * ROWS;
  const int D = (int)p.D;
  for (int e = threadIdx.x; e < ROWS * DMAX; e += blockDim.x) {
    int r = e / DMAX, d = e % DMAX;
    int64_t qi = q0 + r;
    Qs[r][d] = (qi < p.Sq && d < D) ? to_f32(row_ptr<T>(p.q, p.q_s, b, h, qi)[d]) * p.scale : 0.f;
  }
  float m[ROWS_PER_WARP], l[ROWS_PER_WARP], o[ROWS_PER_WARP][4];
#pragma unroll
  for (int r = 0; r < ROWS_PER_WARP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[r][i] = 0.f;
  }
  for (int64_t k0 = 0; k0 < p.Sk; k0 += TILE) {
    __syncthreads();
    for (int e = threadIdx.x; e < TILE * DMAX; e += blockDim.x) {
      int j = e / DMAX, d = e % DMAX;
      int64_t kj = k0 + j;
      bool ok = kj < p.Sk && d < D;
      Ks[j][d] = ok ? to_f32(row_ptr<T>(p.k, p.k_s, b, h, kj)[d]) : 0.f;
      Vs[j][d] = ok ? to_f32(row_ptr<T>(p.v, p.v_s, b, h, kj)[d]) : 0.f;
    }
    __syncthreads();
    const bool kvalid = (k0 + lane) < p.Sk;
#pragma unroll
    for (int r = 0; r < ROWS_PER_WARP; ++r) {
      const int qr = warp * ROWS_PER_WARP + r;
      float s = 0.f;
      for (int d = 0; d < D; ++d) s += Qs[qr][d] * Ks[lane][d];
      s = kvalid ? s : -INFINITY;
      float mn = fmaxf(m[r], warp_max(s));
      float alpha = (m[r] == -INFINITY) ? 0.f : expf(m[r] - mn);
      float pj = kvalid ? expf(s - mn) : 0.f;
      l[r] = l[r] * alpha + warp_sum(pj);
      m[r] = mn;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[r][i] *= alpha;
      for (int j = 0; j < TILE; ++j) {
        float pb = __shfl_sync(0xffffffffu, pj, j);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[r][i] += pb * Vs[j][lane + 32 * i];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS_PER_WARP; ++r) {
    const int64_t qi = q0 + warp * ROWS_PER_WARP + r;
    if (qi >= p.Sq) continue;
    T* orow = (T*)p.o + b * p.o_s[0] + h * p.o_s[1] + qi * p.o_s[2];
    const float inv = 1.f / l[r];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < D) orow[lane + 32 * i] = from_f32<T>(o[r][i] * inv);
    if (lane == 0) p.lse[bh * p.Sq + qi] = m[r] + logf(l[r]);
  }
}

// delta[bh, i] = sum_d O[i,d] * dO[i,d]; one warp per row.
template <typename T>
__global__ void attn_delta(b2_attn_args p) {
  const int64_t rows = p.B * p.H * p.Sq;
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    int64_t bh = r / p.Sq, i = r % p.Sq, b = bh / p.H, h = bh % p.H;
    const T* orow = (const T*)p.o + b * p.o_s[0] + h * p.o_s[1] + i * p.o_s[2];
    const T* grow = (const T*)p.d_o + b * p.do_s[0] + h * p.do_s[1] + i * p.do_s[2];
    float s = 0.f;
    for (int d = lane; d < p.D; d += 32) s += to_f32(orow[d]) * to_f32(grow[d]);
    s = warp_sum(s);
    if (lane == 0) p.delta[r] = s;
  }
}

template <typename T>
__global__ void __launch_bounds__(128) attn_dq_simt(b2_attn_args p) {
  extern __shared__ float smf[];
  float(*Ks)[DP] = reinterpret_cast<float(*)[DP]>(smf);
  float(*Vs)[DP] = reinterpret_cast<float(*)[DP]>(smf + TILE * DP);
  float(*Qs)[DMAX] = reinterpret_cast<float(*)[DMAX]>(smf + 2 * TILE * DP);
  float(*Gs)[DMAX] = reinterpret_cast<float(*)[DMAX]>(smf + 2 * TILE * DP + ROWS * DMAX);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int64_t q0 = (int64_t)blockIdx.x * ROWS;
  const int D = (int)p.D;
  for (int e = threadIdx.x; e < ROWS * DMAX; e += blockDim.x) {
    int r = e / DMAX, d = e % DMAX;
    int64_t qi = q0 + r;
    bool ok = qi < p.Sq && d < D;
    Qs[r][d] = ok ? to_f32(row_ptr<T>(p.q, p.q_s, b, h, qi)[d]) : 0.f;
    Gs[r][d] = ok ? to_f32(row_ptr<T>(p.d_o, p.do_s, b, h, qi)[d]) : 0.f;
  }
  float lse[ROWS_PER_WARP], dl[ROWS_PER_WARP], acc[ROWS_PER_WARP][4];
#pragma unroll
  for (int r = 0; r < ROWS_PER_WARP; ++r) {
    int64_t qi = q0 + warp * ROWS_PER_WARP + r;
    lse[r] = qi < p.Sq ? p.lse[bh * p.Sq + qi] : 0.f;
    dl[r] = qi < p.Sq ? p.delta[bh * p.Sq + qi] : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[r][i] = 0.f;
  }
  for (int64_t k0 = 0; k0 < p.Sk; k0 += TILE) {
    __syncthreads();
    for (int e = threadIdx.x; e < TILE * DMAX; e += blockDim.x) {
      int j = e / DMAX, d = e % DMAX;
      int64_t kj = k0 + j;
      bool ok = kj < p.Sk && d < D;
      Ks[j][d] = ok ? to_f32(row_ptr<T>(p.k, p.k_s, b, h, kj)[d]) : 0.f;
      Vs[j][d] = ok ? to_f32(row_ptr<T>(p.v, p.v_s, b, h, kj)[d]) : 0.f;
    }
    __syncthreads();
    const bool kvalid = (k0 + lane) < p.Sk;
#pragma unroll
    for (int r = 0; r < ROWS_PER_WARP; ++r) {
      const int qr = warp * ROWS_PER_WARP + r;
      float s = 0.f, dp = 0.f;
      for (int d = 0; d < D; ++d) {
        s += Qs[qr][d] * Ks[lane][d];
        dp += Gs[qr][d] * Vs[lane][d];
      }
      float pj = kvalid ? expf(s * p.scale - lse[r]) : 0.f;
      float ds = pj * (dp - dl[r]);
      for (int j = 0; j < TILE; ++j) {
        float db = __shfl_sync(0xffffffffu, ds, j);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[r][i] += db * Ks[j][lane + 32 * i];
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS_PER_WARP; ++r) {
    const int64_t qi = q0 + warp * ROWS_PER_WARP + r;
    if (qi >= p.Sq) continue;
    T* out = (T*)p.dq + b * p.dq_s[0] + h * p.dq_s[1] + qi * p.dq_s[2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < D) out[lane + 32 * i] = from_f32<T>(acc[r][i] * p.scale);
  }
}

template <typename T>
__global__ void __launch_bounds__(128) attn_dkdv_simt(b2_attn_args p) {
  extern __shared__ float smf[];
  float(*Qs)[DP] = reinterpret_cast<float(*)[DP]>(smf);
  float(*Gs)[DP] = reinterpret_cast<float(*)[DP]>(smf + TILE * DP);
  float(*Ks)[DMAX] = reinterpret_cast<float(*)[DMAX]>(smf + 2 * TILE * DP);
  float(*Vs)[DMAX] = reinterpret_cast<float(*)[DMAX]>(smf + 2 * TILE * DP + ROWS * DMAX);
  float* Ls = smf + 2 * TILE * DP + 2 * ROWS * DMAX;
  float* Dl = Ls + TILE;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int64_t k0 = (int64_t)blockIdx.x * ROWS;
  const int D = (int)p.D;
  for (int e = threadIdx.x; e < ROWS * DMAX; e += blockDim.x) {
    int r = e / DMAX, d = e % DMAX;
    int64_t kj = k0 + r;
    bool ok = kj < p.Sk && d < D;
    Ks[r][d] = ok ? to_f32(row_ptr<T>(p.k, p.k_s, b, h, kj)[d]) : 0.f;
    Vs[r][d] = ok ? to_f32(row_ptr<T>(p.v, p.v_s, b, h, kj)[d]) : 0.f;
  }
  float dk[ROWS_PER_WARP][4], dv[ROWS_PER_WARP][4];
#pragma unroll
  for (int r = 0; r < ROWS_PER_WARP; ++r)
#pragma unroll
    for (int i = 0; i < 4; ++i) dk[r][i] = dv[r][i] = 0.f;
  for (int64_t q0 = 0; q0 < p.Sq; q0 += TILE) {
    __syncthreads();
    for (int e = threadIdx.x; e < TILE * DMAX; e += blockDim.x) {
      int j = e / DMAX, d = e % DMAX;
      int64_t qi = q0 + j;
      bool ok = qi < p.Sq && d < D;
      Qs[j][d] = ok ? to_f32(row_ptr<T>(p.q, p.q_s, b, h, qi)[d]) : 0.f;
      Gs[j][d] = ok ? to_f32(row_ptr<T>(p.d_o, p.do_s, b, h, qi)[d]) : 0.f;
    }
    if (threadIdx.x < TILE) {
      int64_t qi = q0 + threadIdx.x;
      Ls[threadIdx.x] = qi < p.Sq ? p.lse[bh * p.Sq + qi] : 0.f;
      Dl[threadIdx.x] = qi < p.Sq ? p.delta[bh * p.Sq + qi] : 0.f;
    }
    __syncthreads();
    const bool qvalid = (q0 + lane) < p.Sq;
#pragma unroll
    for (int r = 0; r < ROWS_PER_WARP; ++r) {
      const int kr = warp * ROWS_PER_WARP + r;
      float s = 0.f, dp = 0.f;
      for (int d = 0; d < D; ++d) {
        s += Qs[lane][d] * Ks[kr][d];
        dp += Gs[lane][d] * Vs[kr][d];
      }
      float pj = qvalid ? expf(s * p.scale - Ls[lane]) : 0.f;
      float ds = pj * (dp - Dl[lane]);
      for (int j = 0; j < TILE; ++j) {
        float pb = __shfl_sync(0xffffffffu, pj, j);
        float db = __shfl_sync(0xffffffffu, ds, j);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dv[r][i] += pb * Gs[j][lane + 32 * i];
          dk[r][i] += db * Qs[j][lane + 32 * i];
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS_PER_WARP; ++r) {
    const int64_t kj = k0 + warp * ROWS_PER_WARP + r;
    if (kj >= p.Sk) continue;
    T* ok_ = (T*)p.dk + b * p.dk_s[0] + h * p.dk_s[1] + kj * p.dk_s[2];
    T* ov = (T*)p.dv + b * p.dv_s[0] + h * p.dv_s[1] + kj * p.dv_s[2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < D) {
        if (p.dk) ok_[lane + 32 * i] = from_f32<T>(dk[r][i] * p.scale);
        if (p.dv) ov[lane + 32 * i] = from_f32<T>(dv[r][i]);
      }
  }
}

template <typename T>
int simt_fwd(const b2_attn_args* a, cudaStream_t st) {
  dim3 grid((unsigned)((a->Sq + ROWS - 1) / ROWS), (unsigned)(a->B * a->H));
  LaunchScope ls("attn_fwd_simt", st);
  attn_fwd_simt<T><<<grid, 128, 0, st>>>(*a);
  return after_launch("b2_attn_fwd(simt)");
}

template <typename T>
int launch_delta(const b2_attn_args* a, cudaStream_t st) {
  LaunchScope ls("attn_delta", st);
  int grid = grid_for(a->B * a->H * a->Sq * 32, 256, 8);
  attn_delta<T><<<grid, 256, 0, st>>>(*a);
  return after_launch("attn_delta");
}

constexpr int kDqSmem = (2 * TILE * DP + 2 * ROWS * DMAX) * 4;
constexpr int kDkdvSmem = (2 * TILE * DP + 2 * ROWS * DMAX + 2 * TILE) * 4;

template <typename T>
int simt_bwd(const b2_attn_args* a, cudaStream_t st) {
  static bool attrs = false;
  if (!attrs) {
    if (int rc = check_cuda(cudaFuncSetAttribute(attn_dq_simt<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDqSmem),
                            "attn_dq_simt attr"))
      return rc;
    if (int rc = check_cuda(
            cudaFuncSetAttribute(attn_dkdv_simt<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDkdvSmem),
            "attn_dkdv_simt attr"))
      return rc;
    attrs = true;
  }
  if (int rc = launch_delta<T>(a, st)) return rc;
  if (a->dk || a->dv) {
    dim3 grid((unsigned)((a->Sk + ROWS - 1) / ROWS), (unsigned)(a->B * a->H));
    LaunchScope ls("attn_dkdv_simt", st);
    attn_dkdv_simt<T><<<grid, 128, kDkdvSmem, st>>>(*a);
  }
  if (a->dq) {
    dim3 grid((unsigned)((a->Sq + ROWS - 1) / ROWS), (unsigned)(a->B * a->H));
    LaunchScope ls("attn_dq_simt", st);
    attn_dq_simt<T><<<grid, 128, kDqSmem, st>>>(*a);
  }
  return after_launch("b2_attn_bwd(simt)");
}

int check_args(const b2_attn_args* a, bool bwd) {
  if (!a) return fail(B2_ERR_ARG, "attn: null args");
  if (a->B < 0 || a->H < 0 || a->Sq < 0 || a->Sk < 0 || a->D < 1 || a->D > 128)
    return fail(B2_ERR_ARG, "attn: need B,H,Sq,Sk >= 0 and 1 <= D <= 128");
  if (a->B * a->H > 65535 * 64) return fail(B2_ERR_ARG, "attn: B*H too large");
  if (!a->q || !a->k || !a->v || !a->o || !a->lse) return fail(B2_ERR_ARG, "attn: null pointer");
  if (bwd && (!a->d_o || !a->delta)) return fail(B2_ERR_ARG, "attn_bwd: null dO or delta");
  if (a->dtype != B2_F32 && a->dtype != B2_BF16 && a->dtype != B2_F16)
    return fail(B2_ERR_ARG, "attn: dtype must be F32, BF16 or F16");
  return 0;
}

}  // namespace

// SIMT backward, also used by attn_tc.cu for cases its kernels do not take.
int attn_simt_bwd_dispatch(const b2_attn_args* a, cudaStream_t st) {
  switch (a->dtype) {
    case B2_F32: return simt_bwd<float>(a, st);
    case B2_BF16: return simt_bwd<__nv_bfloat16>(a, st);
    default: return simt_bwd<__half>(a, st);
  }
}

// Entry points shared with attn_tc.cu for its delta pre-pass.
int attn_delta_launch(const b2_attn_args* a, cudaStream_t st) {
  switch (a->dtype) {
    case B2_F32: return launch_delta<float>(a, st);
    case B2_BF16: return launch_delta<__nv_bfloat16>(a, st);
    default: return launch_delta<__half>(a, st);
  }
}

}  // namespace b2

using namespace b2;

extern "C" int b2_attn_path(const b2_attn_args* a) {
  if (!a || a->force_simt) return 0;
  return attn_tc_eligible(a) ? 1 : 0;
}

extern "C" int b2_attn_fwd(const b2_attn_args* a, b2_stream_t stream) {
  if (int rc = check_args(a, false)) return rc;
  if (int rc = ensure_init()) return rc;
  if (a->B == 0 || a->H == 0 || a->Sq == 0) return 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (a->Sk == 0) return fail(B2_ERR_ARG, "attn: Sk == 0");
  if (!a->force_simt && attn_tc_eligible(a)) return attn_tc_fwd(a, st);
  switch (a->dtype) {
    case B2_F32: return simt_fwd<float>(a, st);
    case B2_BF16: return simt_fwd<__nv_bfloat16>(a, st);
    default: return simt_fwd<__half>(a, st);
  }
}

extern "C" int b2_attn_bwd(const b2_attn_args* a, b2_stream_t stream) {
  if (int rc = check_args(a, true)) return rc;
  if (int rc = ensure_init()) return rc;
  if (a->B == 0 || a->H == 0 || a->Sq == 0 || a->Sk == 0) return 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (!a->force_simt && attn_tc_eligible(a)) return attn_tc_bwd(a, st);
  switch (a->dtype) {
    case B2_F32: return simt_bwd<float>(a, st);
    case B2_BF16: return simt_bwd<__nv_bfloat16>(a, st);
    default: return simt_bwd<__half>(a, st);
  }
}
