// Row kernels: softmax forward/backward and LayerNorm forward/backward.
//
// Semantics follow the reference kernels vkrt/shaders/softmax.comp.in:20-51 and ln.comp.in:25-84
// (fp32 math, fp32 mean/rstd, `safe` rows of all -inf give 0). B200 design: the reference runs one
// 256-thread workgroup per row with 3 global passes and scalar 2-byte loads; here a group of
// GROUP threads (a warp for short rows, 256 threads for long rows) owns a row, reads it ONCE with
// 16-byte vector loads into registers, reduces with warp shuffles, and writes it once — the
// ideal HBM traffic of one read and one write per element. LayerNorm weight/bias gradients are a
// two-stage column reduction (per-row-group partials, then a column sum) instead of the
// reference's one-thread-per-column loop over all rows (ln.comp.in:27-38).
#include <mutex>
#include <string>

#include "common.cuh"

namespace b2 {
namespace {

// ---- vector load/store of V elements as fp32 ----------------------------------------------------
template <typename T, int V>
struct VecIO {
  static __device__ __forceinline__ void load(const T* p, float* o) {
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = to_f32(p[i]);
  }
  static __device__ __forceinline__ void store(T* p, const float* v) {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = from_f32<T>(v[i]);
  }
};
template <>
struct VecIO<float, 4> {
  static __device__ __forceinline__ void load(const float* p, float* o) {
    float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x, o[1] = v.y, o[2] = v.z, o[3] = v.w;
  }
  static __device__ __forceinline__ void store(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <typename T>
struct VecIO16 {  // 8 x 16-bit
  static __device__ __forceinline__ void load(const T* p, float* o) {
    uint4 r = *reinterpret_cast<const uint4*>(p);
    const T* h = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = to_f32(h[i]);
  }
  static __device__ __forceinline__ void store(T* p, const float* v) {
    uint4 r;
    T* h = reinterpret_cast<T*>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(v[i]);
    *reinterpret_cast<uint4*>(p) = r;
  }
};
template <>
struct VecIO<__nv_bfloat16, 8> : VecIO16<__nv_bfloat16> {};
template <>
struct VecIO<__half, 8> : VecIO16<__half> {};

// A vector kept in its stored form until it is needed, so that a load can stay in flight across
// other work (16-byte vectors: one uint4; otherwise converted on load).
template <typename T, int V>
struct RawVec {
  float v[V];
  __device__ __forceinline__ void load(const T* p) { VecIO<T, V>::load(p, v); }
  __device__ __forceinline__ void get(float* o) const {
#pragma unroll
    for (int i = 0; i < V; ++i) o[i] = v[i];
  }
};
template <typename T>
struct RawVec16 {
  uint4 r;
  __device__ __forceinline__ void load(const T* p) { r = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void get(float* o) const {
    const T* h = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = to_f32(h[i]);
  }
};
template <>
struct RawVec<__nv_bfloat16, 8> : RawVec16<__nv_bfloat16> {};
template <>
struct RawVec<__half, 8> : RawVec16<__half> {};
template <>
struct RawVec<float, 4> {
  float4 r;
  __device__ __forceinline__ void load(const float* p) { r = *reinterpret_cast<const float4*>(p); }
  __device__ __forceinline__ void get(float* o) const { o[0] = r.x, o[1] = r.y, o[2] = r.z, o[3] = r.w; }
};

template <int GROUP>
__device__ __forceinline__ float group_sum(float v, float* red) {
  if (GROUP == 32) return warp_sum(v);
  return block_sum(v, red);
}
template <int GROUP>
__device__ __forceinline__ float group_max(float v, float* red) {
  if (GROUP == 32) return warp_max(v);
  return block_max(v, red);
}

// ================================== softmax ======================================================

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Contiguous rows (inner == 1), a row held in registers: R <= GROUP * V * NCH.
template <typename TI, typename TO, int GROUP, int V, int NCH>
__global__ void __launch_bounds__(256) softmax_fwd_reg(const TI* __restrict__ x, TO* __restrict__ y, int64_t rows,
                                                       int64_t R, int safe) {
  __shared__ float red[32];
  const int rpb = blockDim.x / GROUP;
  const int t = threadIdx.x % GROUP;
  for (int64_t row = (int64_t)blockIdx.x * rpb + threadIdx.x / GROUP; row - threadIdx.x / GROUP < rows;
       row += (int64_t)gridDim.x * rpb) {
    const bool active = row < rows;  // block-wide groups must all reach the reductions
    const TI* xr = x + row * R;
    float v[NCH][V];
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (active && idx < R) {
        VecIO<TI, V>::load(xr + idx, v[c]);
#pragma unroll
        for (int i = 0; i < V; ++i) m = fmaxf(m, v[c][i]);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) v[c][i] = -INFINITY;
      }
    }
    m = group_max<GROUP>(m, red);
    const bool all_masked = (m == -INFINITY);
    // exp(v - m) = 2^(v*log2e - m*log2e): one FMA and one ex2.approx per element (relative error
    // ~2^-22, far below the output types' rounding)
    const float mm2 = all_masked ? 0.f : m * 1.4426950408889634f;
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int i = 0; i < V; ++i) {
        v[c][i] = fast_ex2(fmaf(v[c][i], 1.4426950408889634f, -mm2));
        s += v[c][i];
      }
    s = group_sum<GROUP>(s, red);
    const float inv = (safe && all_masked) ? 0.f : 1.f / s;
    if (!active) continue;
    TO* yr = y + row * R;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (idx < R) {
        float o[V];
#pragma unroll
        for (int i = 0; i < V; ++i) o[i] = (safe && all_masked) ? 0.f : (all_masked ? NAN : v[c][i] * inv);
        VecIO<TO, V>::store(yr + idx, o);
      }
    }
  }
}

template <typename TI, typename TO, int GROUP, int V, int NCH>
__global__ void __launch_bounds__(256, 2) softmax_bwd_reg(const TI* __restrict__ yv, const TI* __restrict__ g,
                                                       TO* __restrict__ dx, int64_t rows, int64_t R) {
  // persistent row groups (two blocks per SM): the next row's y and g are loaded, and stay in flight,
  // while the current row is reduced and written
  __shared__ float red[32];
  const int rpb = blockDim.x / GROUP;
  const int t = threadIdx.x % GROUP;
  const int64_t stride = (int64_t)gridDim.x * rpb;
  RawVec<TI, V> ny[NCH], ng[NCH];
  int64_t row = (int64_t)blockIdx.x * rpb + threadIdx.x / GROUP;
  auto fetch = [&](int64_t r) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (r < rows && idx < R) {
        ny[c].load(yv + r * R + idx);
        ng[c].load(g + r * R + idx);
      }
    }
  };
  fetch(row);
  for (; row - threadIdx.x / GROUP < rows; row += stride) {
    const bool active = row < rows;
    float a[NCH][V], b[NCH][V];
    float d = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (active && idx < R) {
        ny[c].get(a[c]);
        ng[c].get(b[c]);
#pragma unroll
        for (int i = 0; i < V; ++i) d += a[c][i] * b[c][i];
      }
    }
    fetch(row + stride);
    d = group_sum<GROUP>(d, red);
    if (!active) continue;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (idx < R) {
        float o[V];
#pragma unroll
        for (int i = 0; i < V; ++i) o[i] = a[c][i] * (b[c][i] - d);
        VecIO<TO, V>::store(dx + row * R + idx, o);
      }
    }
  }
}

// Any [outer, R, inner] layout: one thread per (outer, inner) column walks the R axis
// (online max/sum, then a write pass). Coalesced along `inner`; used for inner > 1 and huge R.
template <typename TI, typename TO>
__global__ void softmax_fwd_cols(const TI* __restrict__ x, TO* __restrict__ y, int64_t outer, int64_t R,
                                 int64_t inner, int safe) {
  int64_t ncol = outer * inner;
  for (int64_t col = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; col < ncol; col += (int64_t)gridDim.x * blockDim.x) {
    int64_t o = col / inner, i = col - o * inner;
    const TI* xp = x + o * R * inner + i;
    TO* yp = y + o * R * inner + i;
    float m = -INFINITY, s = 0.f;
    for (int64_t r = 0; r < R; ++r) {
      float v = to_f32(xp[r * inner]);
      if (v > m) {
        s = s * expf(m - v) + 1.f;
        m = v;
      } else {
        s += expf(v - m);
      }
    }
    bool all_masked = (m == -INFINITY);
    float inv = 1.f / s;
    for (int64_t r = 0; r < R; ++r) {
      float v = to_f32(xp[r * inner]);
      float o2 = (safe && all_masked) ? 0.f : (all_masked ? NAN : expf(v - m) * inv);
      yp[r * inner] = from_f32<TO>(o2);
    }
  }
}

template <typename TI, typename TO>
__global__ void softmax_bwd_cols(const TI* __restrict__ yv, const TI* __restrict__ g, TO* __restrict__ dx,
                                 int64_t outer, int64_t R, int64_t inner) {
  int64_t ncol = outer * inner;
  for (int64_t col = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; col < ncol; col += (int64_t)gridDim.x * blockDim.x) {
    int64_t o = col / inner, i = col - o * inner;
    int64_t base = o * R * inner + i;
    float d = 0.f;
    for (int64_t r = 0; r < R; ++r) d += to_f32(yv[base + r * inner]) * to_f32(g[base + r * inner]);
    for (int64_t r = 0; r < R; ++r) {
      float a = to_f32(yv[base + r * inner]);
      dx[base + r * inner] = from_f32<TO>(a * (to_f32(g[base + r * inner]) - d));
    }
  }
}

// Block-per-row for long contiguous rows that do not fit in registers: online max/sum pass, then
// a write pass (the row is re-read from L2).
template <typename TI, typename TO>
__global__ void __launch_bounds__(256) softmax_fwd_long(const TI* __restrict__ x, TO* __restrict__ y, int64_t rows,
                                                        int64_t R, int safe) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const TI* xr = x + row * R;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < R; i += blockDim.x) m = fmaxf(m, to_f32(xr[i]));
    m = block_max(m, red);
    bool all_masked = (m == -INFINITY);
    float mm = all_masked ? 0.f : m;
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < R; i += blockDim.x) s += expf(to_f32(xr[i]) - mm);
    s = block_sum(s, red);
    float inv = 1.f / s;
    for (int64_t i = threadIdx.x; i < R; i += blockDim.x) {
      float o = (safe && all_masked) ? 0.f : (all_masked ? NAN : expf(to_f32(xr[i]) - mm) * inv);
      y[row * R + i] = from_f32<TO>(o);
    }
    __syncthreads();
  }
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(256) softmax_bwd_long(const TI* __restrict__ yv, const TI* __restrict__ g,
                                                        TO* __restrict__ dx, int64_t rows, int64_t R) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    float d = 0.f;
    for (int64_t i = threadIdx.x; i < R; i += blockDim.x) d += to_f32(yv[row * R + i]) * to_f32(g[row * R + i]);
    d = block_sum(d, red);
    for (int64_t i = threadIdx.x; i < R; i += blockDim.x)
      dx[row * R + i] = from_f32<TO>(to_f32(yv[row * R + i]) * (to_f32(g[row * R + i]) - d));
    __syncthreads();
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

template <typename TI, typename TO, int GROUP, int V, int NCH>
void launch_softmax_reg(const b2_softmax_args* a, cudaStream_t st, bool fwd) {
  const int threads = 256;
  const int rpb = threads / GROUP;
  // backward: persistent row groups with the next row prefetched; rows of 4+ vectors per lane keep
  // enough bytes in flight at two blocks per SM, shorter rows need more resident blocks
  const int bwd_per_sm = NCH * V * (int)sizeof(TI) >= 64 ? 2 : (NCH * V * (int)sizeof(TI) >= 32 ? 4 : 8);
  int grid = grid_for((a->outer + rpb - 1) / rpb, 1, fwd ? 16 : bwd_per_sm);
  if (fwd)
    softmax_fwd_reg<TI, TO, GROUP, V, NCH><<<grid, threads, 0, st>>>((const TI*)a->x, (TO*)a->out, a->outer, a->R, a->safe);
  else
    softmax_bwd_reg<TI, TO, GROUP, V, NCH><<<grid, threads, 0, st>>>((const TI*)a->y, (const TI*)a->g, (TO*)a->out, a->outer, a->R);
}

// Picks the register-resident variant for a contiguous row of R elements; returns false if R is
// too long for registers.
template <typename TI, typename TO>
bool softmax_reg_dispatch(const b2_softmax_args* a, cudaStream_t st, bool fwd) {
  constexpr int VI = sizeof(TI) == 4 ? 4 : 8;
  constexpr int VO = sizeof(TO) == 4 ? 4 : 8;
  constexpr int V = VI < VO ? VI : VO;  // elements per 16-byte access of the narrower side... both must divide R
  const void* ptrs[3] = {fwd ? a->x : a->y, a->out, fwd ? nullptr : a->g};
  bool vec = (a->R % V == 0);
  for (const void* p : ptrs)
    if (p && !aligned16(p)) vec = false;
  const int64_t R = a->R;
  if (vec) {
    if (R <= 32 * V * 1) return launch_softmax_reg<TI, TO, 32, V, 1>(a, st, fwd), true;
    if (R <= 32 * V * 2) return launch_softmax_reg<TI, TO, 32, V, 2>(a, st, fwd), true;
    if (R <= 32 * V * 4) return launch_softmax_reg<TI, TO, 32, V, 4>(a, st, fwd), true;
    if (R <= 256 * V * 2) return launch_softmax_reg<TI, TO, 256, V, 2>(a, st, fwd), true;
    if (R <= 256 * V * 4) return launch_softmax_reg<TI, TO, 256, V, 4>(a, st, fwd), true;
    if (R <= 256 * V * 8) return launch_softmax_reg<TI, TO, 256, V, 8>(a, st, fwd), true;
    return false;
  }
  if (R <= 32 * 1) return launch_softmax_reg<TI, TO, 32, 1, 1>(a, st, fwd), true;
  if (R <= 32 * 4) return launch_softmax_reg<TI, TO, 32, 1, 4>(a, st, fwd), true;
  if (R <= 32 * 16) return launch_softmax_reg<TI, TO, 32, 1, 16>(a, st, fwd), true;
  if (R <= 256 * 8) return launch_softmax_reg<TI, TO, 256, 1, 8>(a, st, fwd), true;
  if (R <= 256 * 32) return launch_softmax_reg<TI, TO, 256, 1, 32>(a, st, fwd), true;
  return false;
}

template <typename TI, typename TO>
int softmax_run(const b2_softmax_args* a, cudaStream_t st, bool fwd) {
  if (a->inner == 1) {
    LaunchScope ls(fwd ? "softmax_fwd_rows" : "softmax_bwd_rows", st);
    if (!softmax_reg_dispatch<TI, TO>(a, st, fwd)) {
      int grid = grid_for(a->outer, 1, 8);
      if (fwd)
        softmax_fwd_long<TI, TO><<<grid, 256, 0, st>>>((const TI*)a->x, (TO*)a->out, a->outer, a->R, a->safe);
      else
        softmax_bwd_long<TI, TO><<<grid, 256, 0, st>>>((const TI*)a->y, (const TI*)a->g, (TO*)a->out, a->outer, a->R);
    }
  } else {
    LaunchScope ls(fwd ? "softmax_fwd_cols" : "softmax_bwd_cols", st);
    int grid = grid_for(a->outer * a->inner, 256, 8);
    if (fwd)
      softmax_fwd_cols<TI, TO><<<grid, 256, 0, st>>>((const TI*)a->x, (TO*)a->out, a->outer, a->R, a->inner, a->safe);
    else
      softmax_bwd_cols<TI, TO><<<grid, 256, 0, st>>>((const TI*)a->y, (const TI*)a->g, (TO*)a->out, a->outer, a->R,
                                                     a->inner);
  }
  return after_launch(fwd ? "b2_softmax_fwd" : "b2_softmax_bwd");
}

template <typename TI>
int softmax_out(const b2_softmax_args* a, cudaStream_t st, bool fwd) {
  switch (a->out_dtype) {
    case B2_F32: return softmax_run<TI, float>(a, st, fwd);
    case B2_BF16: return softmax_run<TI, __nv_bfloat16>(a, st, fwd);
    case B2_F16: return softmax_run<TI, __half>(a, st, fwd);
    default: return fail(B2_ERR_ARG, "softmax: out_dtype must be F32, BF16 or F16");
  }
}

int softmax_entry(const b2_softmax_args* a, b2_stream_t stream, bool fwd) {
  if (!a) return fail(B2_ERR_ARG, "softmax: null args");
  if (int rc = ensure_init()) return rc;
  if (a->outer < 0 || a->R < 0 || a->inner < 0) return fail(B2_ERR_ARG, "softmax: negative size");
  if (a->outer == 0 || a->R == 0 || a->inner == 0) return 0;
  if (!a->out || (fwd ? !a->x : (!a->y || !a->g))) return fail(B2_ERR_ARG, "softmax: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->in_dtype) {
    case B2_F32: return softmax_out<float>(a, st, fwd);
    case B2_BF16: return softmax_out<__nv_bfloat16>(a, st, fwd);
    case B2_F16: return softmax_out<__half>(a, st, fwd);
    default: return fail(B2_ERR_ARG, "softmax: in_dtype must be F32, BF16 or F16");
  }
}

// ================================== layer norm ===================================================

// Two sums in one pass of the group reduction (`red` holds >= 64 floats).
template <int GROUP>
__device__ __forceinline__ void group_sum2(float& a, float& b, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  if (GROUP == 32) return;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, g0 = (threadIdx.x / GROUP) * (GROUP / 32);
  __syncthreads();
  if (lane == 0) red[w] = a, red[32 + w] = b;
  __syncthreads();
  a = red[g0], b = red[32 + g0];
#pragma unroll
  for (int i = 1; i < GROUP / 32; ++i) a += red[g0 + i], b += red[32 + g0 + i];
}

template <typename T, int GROUP, int V, int NCH>
__global__ void __launch_bounds__(256) ln_fwd_reg(const T* __restrict__ x, const T* __restrict__ w,
                                                  const T* __restrict__ b, T* __restrict__ y, float* __restrict__ mean,
                                                  float* __restrict__ rstd, int64_t rows, int64_t D, float eps) {
  __shared__ float red[32];
  const int rpb = blockDim.x / GROUP;
  const int t = threadIdx.x % GROUP;
  const float invD = 1.f / (float)D;
  // rows of up to two chunks per thread keep this thread's weight and bias columns in registers, loaded
  // once before the first row, so no load sits between a row's reductions and its stores
  constexpr bool HOIST = NCH <= 2;
  float wh[HOIST ? NCH : 1][V], bh[HOIST ? NCH : 1][V];
  if constexpr (HOIST) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t idx = ((int64_t)c * GROUP + t) * V;
#pragma unroll
      for (int i = 0; i < V; ++i) wh[c][i] = 1.f, bh[c][i] = 0.f;
      if (idx < D) {
        if (w) VecIO<T, V>::load(w + idx, wh[c]);
        if (b) VecIO<T, V>::load(b + idx, bh[c]);
      }
    }
  }
  for (int64_t row = (int64_t)blockIdx.x * rpb + threadIdx.x / GROUP; row - threadIdx.x / GROUP < rows;
       row += (int64_t)gridDim.x * rpb) {
    const bool active = row < rows;
    float v[NCH][V];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (active && idx < D) {
        VecIO<T, V>::load(x + row * D + idx, v[c]);
#pragma unroll
        for (int i = 0; i < V; ++i) s += v[c][i];
      }
    }
    const float mu = group_sum<GROUP>(s, red) * invD;
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (active && idx < D)
#pragma unroll
        for (int i = 0; i < V; ++i) {
          float d = v[c][i] - mu;
          q += d * d;
        }
    }
    const float rs = rsqrtf(group_sum<GROUP>(q, red) * invD + eps);
    if (!active) continue;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (idx < D) {
        float o[V];
        if constexpr (HOIST) {
#pragma unroll
          for (int i = 0; i < V; ++i) o[i] = fmaf((v[c][i] - mu) * rs, wh[c][i], bh[c][i]);
        } else {
          float wv[V], bv[V];
          if (w) VecIO<T, V>::load(w + idx, wv);
          if (b) VecIO<T, V>::load(b + idx, bv);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            float r = (v[c][i] - mu) * rs;
            if (w) r *= wv[i];
            if (b) r += bv[i];
            o[i] = r;
          }
        }
        VecIO<T, V>::store(y + row * D + idx, o);
      }
    }
    if (t == 0) {
      mean[row] = mu;
      rstd[row] = rs;
    }
  }
}

// Backward. Each row group computes dx for its rows; when `part` is non-null it also accumulates
// per-column partial sums of g*xhat and g over the rows it visits and writes them to
// part[(slot) * 2D + {0, D} + col], slot = blockIdx.x * rows_per_block + group.
template <typename T, int GROUP, int V, int NCH>
__global__ void __launch_bounds__(256) ln_bwd_reg(const T* __restrict__ x, const T* __restrict__ w,
                                                  const T* __restrict__ g, const float* __restrict__ mean,
                                                  const float* __restrict__ rstd, T* __restrict__ dx,
                                                  float* __restrict__ part, int64_t rows, int64_t D) {
  __shared__ float red[64];
  const int rpb = blockDim.x / GROUP;
  const int t = threadIdx.x % GROUP;
  const float invD = 1.f / (float)D;
  const int64_t stride = (int64_t)gridDim.x * rpb;
  float pdw[NCH][V], pdb[NCH][V], wv[NCH][V];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int64_t idx = ((int64_t)c * GROUP + t) * V;
#pragma unroll
    for (int i = 0; i < V; ++i) pdw[c][i] = pdb[c][i] = 0.f, wv[c][i] = 1.f;
    if (w && idx < D) VecIO<T, V>::load(w + idx, wv[c]);
  }
  // the next row's x and g are loaded (and stay in flight) while the current row is reduced
  RawVec<T, V> nx[NCH], ng[NCH];
  float nmu = 0.f, nrs = 0.f;
  int64_t row = (int64_t)blockIdx.x * rpb + threadIdx.x / GROUP;
  auto fetch = [&](int64_t r) {
    if (r < rows) nmu = mean[r], nrs = rstd[r];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (r < rows && idx < D) {
        nx[c].load(x + r * D + idx);
        ng[c].load(g + r * D + idx);
      }
    }
  };
  fetch(row);
  for (; row - threadIdx.x / GROUP < rows; row += stride) {
    const bool active = row < rows;
    float xh[NCH][V], gw[NCH][V];
    float s1 = 0.f, s2 = 0.f;
    const float mu = nmu, rs = nrs;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (active && idx < D) {
        float gv[V];
        nx[c].get(xh[c]);
        ng[c].get(gv);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          xh[c][i] = (xh[c][i] - mu) * rs;
          gw[c][i] = gv[i] * wv[c][i];
          s1 += gw[c][i];
          s2 += gw[c][i] * xh[c][i];
          pdw[c][i] += gv[i] * xh[c][i];
          pdb[c][i] += gv[i];
        }
      }
    }
    fetch(row + stride);
    group_sum2<GROUP>(s1, s2, red);
    s1 *= invD, s2 *= invD;
    if (!active || !dx) continue;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (idx < D) {
        float o[V];
#pragma unroll
        for (int i = 0; i < V; ++i) o[i] = rs * (gw[c][i] - s1 - xh[c][i] * s2);
        VecIO<T, V>::store(dx + row * D + idx, o);
      }
    }
  }
  // the weight-gradient reduction (launched as a programmatic dependent) may start its prologue; its
  // griddepcontrol.wait still sees every partial written below
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (part) {
    int64_t slot = (int64_t)blockIdx.x * rpb + threadIdx.x / GROUP;
    float* pw = part + slot * 2 * D;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      int64_t idx = ((int64_t)c * GROUP + t) * V;
      if (idx < D)
#pragma unroll
        for (int i = 0; i < V; ++i) {
          pw[idx + i] = pdw[c][i];
          pw[D + idx + i] = pdb[c][i];
        }
    }
  }
}

// Column sum of the partials: dw[d] = sum_s part[s][d], db[d] = sum_s part[s][D + d].
// blockDim = (8, 32): x over 8 consecutive columns (32-byte sectors per slot), y over the slots; 8
// columns per block spread the partials (L2-resident: the backward kernel just wrote them) over
// D / 8 blocks, and the 32 slot lanes are combined through shared memory.
constexpr int kWgradCols = 8;
template <typename T>
__global__ void __launch_bounds__(256) ln_wgrad_reduce(const float* __restrict__ part, int64_t nslots, int64_t D,
                                                       T* __restrict__ dw, T* __restrict__ db) {
  __shared__ float sw[32][kWgradCols + 1], sb[32][kWgradCols + 1];
  const int64_t col = (int64_t)blockIdx.x * kWgradCols + threadIdx.x;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the partials of the preceding backward kernel
  float aw0 = 0.f, ab0 = 0.f, aw1 = 0.f, ab1 = 0.f;
  if (col < D) {
    const float* pc = part + col;
    int64_t s = threadIdx.y;
    // eight slots per thread per pass, all sixteen loads issued before the first add
    for (; s + 7 * 32 < nslots; s += 8 * 32) {
      float lw[8], lb[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        lw[u] = pc[(s + 32 * u) * 2 * D];
        lb[u] = pc[(s + 32 * u) * 2 * D + D];
      }
#pragma unroll
      for (int u = 0; u < 8; u += 2) {
        aw0 += lw[u], ab0 += lb[u];
        aw1 += lw[u + 1], ab1 += lb[u + 1];
      }
    }
    for (; s < nslots; s += 32) {
      aw0 += pc[s * 2 * D];
      ab0 += pc[s * 2 * D + D];
    }
  }
  sw[threadIdx.y][threadIdx.x] = aw0 + aw1;
  sb[threadIdx.y][threadIdx.x] = ab0 + ab1;
  __syncthreads();
  for (int k = 16; k > 0; k >>= 1) {
    if (threadIdx.y < k) {
      sw[threadIdx.y][threadIdx.x] += sw[threadIdx.y + k][threadIdx.x];
      sb[threadIdx.y][threadIdx.x] += sb[threadIdx.y + k][threadIdx.x];
    }
    __syncthreads();
  }
  if (threadIdx.y == 0 && col < D) {
    if (dw) dw[col] = from_f32<T>(sw[0][threadIdx.x]);
    if (db) db[col] = from_f32<T>(sb[0][threadIdx.x]);
  }
}

// Rows too long for registers: block per row, re-reading the row (L2-resident) per pass.
template <typename T>
__global__ void __launch_bounds__(256) ln_fwd_long(const T* __restrict__ x, const T* __restrict__ w,
                                                   const T* __restrict__ b, T* __restrict__ y, float* __restrict__ mean,
                                                   float* __restrict__ rstd, int64_t rows, int64_t D, float eps) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * D;
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) s += to_f32(xr[i]);
    float mu = block_sum(s, red) / (float)D;
    float q = 0.f;
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
      float d = to_f32(xr[i]) - mu;
      q += d * d;
    }
    float rs = rsqrtf(block_sum(q, red) / (float)D + eps);
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
      float r = (to_f32(xr[i]) - mu) * rs;
      if (w) r *= to_f32(w[i]);
      if (b) r += to_f32(b[i]);
      y[row * D + i] = from_f32<T>(r);
    }
    if (threadIdx.x == 0) {
      mean[row] = mu;
      rstd[row] = rs;
    }
    __syncthreads();
  }
}

template <typename T>
__global__ void __launch_bounds__(256) ln_bwd_long(const T* __restrict__ x, const T* __restrict__ w,
                                                   const T* __restrict__ g, const float* __restrict__ mean,
                                                   const float* __restrict__ rstd, T* __restrict__ dx, int64_t rows,
                                                   int64_t D) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    float mu = mean[row], rs = rstd[row];
    float s1 = 0.f, s2 = 0.f;
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
      float gw = to_f32(g[row * D + i]) * (w ? to_f32(w[i]) : 1.f);
      float xh = (to_f32(x[row * D + i]) - mu) * rs;
      s1 += gw;
      s2 += gw * xh;
    }
    s1 = block_sum(s1, red) / (float)D;
    s2 = block_sum(s2, red) / (float)D;
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
      float gw = to_f32(g[row * D + i]) * (w ? to_f32(w[i]) : 1.f);
      float xh = (to_f32(x[row * D + i]) - mu) * rs;
      dx[row * D + i] = from_f32<T>(rs * (gw - s1 - xh * s2));
    }
    __syncthreads();
  }
}

// Column-parallel partials for long rows: slot = blockIdx.y chunk of rows, x over columns.
template <typename T>
__global__ void ln_wgrad_part_long(const T* __restrict__ x, const T* __restrict__ g, const float* __restrict__ mean,
                                   const float* __restrict__ rstd, float* __restrict__ part, int64_t rows, int64_t D,
                                   int64_t rows_per_slot) {
  int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= D) return;
  int64_t r0 = (int64_t)blockIdx.y * rows_per_slot, r1 = min(rows, r0 + rows_per_slot);
  float aw = 0.f, ab = 0.f;
  for (int64_t r = r0; r < r1; ++r) {
    float gv = to_f32(g[r * D + col]);
    aw += gv * (to_f32(x[r * D + col]) - mean[r]) * rstd[r];
    ab += gv;
  }
  part[(int64_t)blockIdx.y * 2 * D + col] = aw;
  part[(int64_t)blockIdx.y * 2 * D + D + col] = ab;
}

// Launch plan shared by the workspace query and the launch.
struct LnPlan {
  int kind;      // 0 = register kernel, 1 = long-row kernels
  int group, v, nch;
  int grid;
  int64_t nslots;  // partial slots (rows of the workspace)
};

LnPlan ln_plan(const b2_layernorm_args* a, bool fwd) {
  LnPlan p{};
  const int V = dtype_size(a->dtype) == 4 ? 4 : 8;
  bool vec = (a->D % V == 0);
  const void* ptrs[] = {a->x, a->w, a->b, a->y, a->g, a->dx};
  for (const void* q : ptrs)
    if (q && ((uintptr_t)q & 15)) vec = false;
  const int64_t D = a->D;
  const int vv = vec ? V : 1;
  p.v = vv;
  p.kind = 0;
  if (vec) {
    if (D <= 32 * V) p.group = 32, p.nch = 1;
    else if (D <= 32 * V * 2) p.group = 32, p.nch = 2;
    else if (D <= 32 * V * 4) p.group = 32, p.nch = 4;
    else if (D <= 256 * V) p.group = 256, p.nch = 1;
    else if (D <= 256 * V * 2) p.group = 256, p.nch = 2;
    else if (D <= 256 * V * 4) p.group = 256, p.nch = 4;
    else p.kind = 1;
  } else {
    if (D <= 32) p.group = 32, p.nch = 1;
    else if (D <= 32 * 4) p.group = 32, p.nch = 4;
    else if (D <= 32 * 16) p.group = 32, p.nch = 16;
    else if (D <= 256 * 8) p.group = 256, p.nch = 8;
    else if (D <= 256 * 16) p.group = 256, p.nch = 16;
    else p.kind = 1;
  }
  const int sms = device_info().sm_count > 0 ? device_info().sm_count : 148;
  if (p.kind == 0) {
    const int rpb = 256 / p.group;
    int64_t blocks = (a->rows + rpb - 1) / rpb;
    // forward: enough blocks to fill the GPU. backward: two blocks per SM walking several rows with
    // the next row prefetched, which keeps the weight-gradient partial slots (and their reduction) few
    // (forward with a 256-thread group per row: up to eight rows per SM at once, so a [1024, 2048] input is
    // read in a single wave of loads)
    int64_t cap = fwd ? (int64_t)sms * (p.group == 256 ? 8 : 4) : (p.group == 32 ? (int64_t)sms / 2 : (int64_t)sms * 2);
    p.grid = (int)std::max<int64_t>(1, std::min(blocks, cap));
    p.nslots = (int64_t)p.grid * rpb;
  } else {
    p.grid = (int)std::max<int64_t>(1, std::min<int64_t>(a->rows, (int64_t)sms * 4));
    p.nslots = std::min<int64_t>(a->rows, 256);
  }
  return p;
}

template <typename T, int GROUP, int V, int NCH>
void ln_launch_reg(const b2_layernorm_args* a, const LnPlan& p, cudaStream_t st, bool fwd, float* part) {
  if (fwd)
    ln_fwd_reg<T, GROUP, V, NCH><<<p.grid, 256, 0, st>>>((const T*)a->x, (const T*)a->w, (const T*)a->b, (T*)a->y,
                                                          a->mean, a->rstd, a->rows, a->D, a->eps);
  else
    ln_bwd_reg<T, GROUP, V, NCH><<<p.grid, 256, 0, st>>>((const T*)a->x, (const T*)a->w, (const T*)a->g, a->mean,
                                                          a->rstd, (T*)a->dx, part, a->rows, a->D);
}

template <typename T, int V>
void ln_reg_switch(const b2_layernorm_args* a, const LnPlan& p, cudaStream_t st, bool fwd, float* part) {
  if (p.group == 32) {
    if (p.nch == 1) return ln_launch_reg<T, 32, V, 1>(a, p, st, fwd, part);
    if (p.nch == 2) return ln_launch_reg<T, 32, V, 2>(a, p, st, fwd, part);
    if (p.nch == 4) return ln_launch_reg<T, 32, V, 4>(a, p, st, fwd, part);
    if (p.nch == 16) return ln_launch_reg<T, 32, V, 16>(a, p, st, fwd, part);
  } else {
    if (p.nch == 1) return ln_launch_reg<T, 256, V, 1>(a, p, st, fwd, part);
    if (p.nch == 2) return ln_launch_reg<T, 256, V, 2>(a, p, st, fwd, part);
    if (p.nch == 4) return ln_launch_reg<T, 256, V, 4>(a, p, st, fwd, part);
    if (p.nch == 8) return ln_launch_reg<T, 256, V, 8>(a, p, st, fwd, part);
    if (p.nch == 16) return ln_launch_reg<T, 256, V, 16>(a, p, st, fwd, part);
  }
}

template <typename T>
int ln_run(const b2_layernorm_args* a, cudaStream_t st, bool fwd) {
  LnPlan p = ln_plan(a, fwd);
  constexpr int VV = sizeof(T) == 4 ? 4 : 8;
  const bool want_w = !fwd && (a->dw || a->db);
  float* part = want_w ? (float*)a->workspace : nullptr;
  if (want_w && !part) return fail(B2_ERR_ARG, "layernorm_bwd: workspace required for dw/db");
  {
    LaunchScope ls(fwd ? "layernorm_fwd" : "layernorm_bwd", st);
    if (p.kind == 0) {
      if (p.v == 1)
        ln_reg_switch<T, 1>(a, p, st, fwd, part);
      else
        ln_reg_switch<T, VV>(a, p, st, fwd, part);
    } else if (fwd) {
      ln_fwd_long<T><<<p.grid, 256, 0, st>>>((const T*)a->x, (const T*)a->w, (const T*)a->b, (T*)a->y, a->mean,
                                             a->rstd, a->rows, a->D, a->eps);
    } else {
      if (a->dx)
        ln_bwd_long<T><<<p.grid, 256, 0, st>>>((const T*)a->x, (const T*)a->w, (const T*)a->g, a->mean, a->rstd,
                                               (T*)a->dx, a->rows, a->D);
      if (want_w) {
        int64_t rps = (a->rows + p.nslots - 1) / p.nslots;
        dim3 grid((unsigned)((a->D + 255) / 256), (unsigned)p.nslots);
        ln_wgrad_part_long<T><<<grid, 256, 0, st>>>((const T*)a->x, (const T*)a->g, a->mean, a->rstd, part, a->rows,
                                                     a->D, rps);
      }
    }
  }
  if (want_w) {
    if (int rc = launch_pdl("layernorm_wgrad_reduce", ln_wgrad_reduce<T>,
                            dim3((unsigned)((a->D + kWgradCols - 1) / kWgradCols)), dim3(kWgradCols, 32),
                            0, st, (const float*)part, p.nslots, a->D, (T*)a->dw, (T*)a->db))
      return rc;
  }
  return after_launch(fwd ? "b2_layernorm_fwd" : "b2_layernorm_bwd");
}

int ln_entry(const b2_layernorm_args* a, b2_stream_t stream, bool fwd) {
  if (!a) return fail(B2_ERR_ARG, "layernorm: null args");
  if (int rc = ensure_init()) return rc;
  if (a->rows < 0 || a->D < 0) return fail(B2_ERR_ARG, "layernorm: negative size");
  if (a->rows == 0 || a->D == 0) return 0;
  if (!a->x || !a->mean || !a->rstd) return fail(B2_ERR_ARG, "layernorm: null pointer");
  if (fwd && !a->y) return fail(B2_ERR_ARG, "layernorm_fwd: null output");
  if (!fwd && !a->g) return fail(B2_ERR_ARG, "layernorm_bwd: null grad");
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->dtype) {
    case B2_F32: return ln_run<float>(a, st, fwd);
    case B2_BF16: return ln_run<__nv_bfloat16>(a, st, fwd);
    case B2_F16: return ln_run<__half>(a, st, fwd);
    default: return fail(B2_ERR_ARG, "layernorm: dtype must be F32, BF16 or F16");
  }
}

// ---- allocation-free LayerNorm backward ---------------------------------------------------------
// Some callers cannot allocate device memory in the middle of a step: a host framework that owns
// every byte of VRAM through its own allocator or a fixed budget, or an FFI caller that only holds the
// tensors. For them the weight/bias-gradient partials live in this file-scope array instead of a
// caller-provided workspace. It is 2 MiB (512 Ki floats); every GPU that loads the library keeps it
// until the process exits. Host code must not pass the symbol itself to a kernel (on the host it is
// only a stand-in): its device address is looked up once per device with cudaGetSymbolAddress.
constexpr int64_t kLnNoAllocScratchFloats = 512 * 1024;
static __device__ __align__(256) float g_ln_noalloc_scratch[kLnNoAllocScratchFloats];

std::mutex g_ln_noalloc_mu;
void* g_ln_noalloc_ptr[256];  // per device ordinal

// Device address of g_ln_noalloc_scratch on the current device (resolved on first use).
int ln_noalloc_scratch(float** out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "layernorm_bwd_noalloc: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 256) return fail(B2_ERR_ARG, "layernorm_bwd_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> g(g_ln_noalloc_mu);
  if (!g_ln_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_ln_noalloc_scratch), "layernorm_bwd_noalloc: cudaGetSymbolAddress"))
      return rc;
    g_ln_noalloc_ptr[dev] = p;
  }
  *out = (float*)g_ln_noalloc_ptr[dev];
  return 0;
}

// The LayerNorm backward launch sequence for an explicit plan whose partial slots fit `part`.
template <typename T>
int ln_bwd_planned(const b2_layernorm_args* a, const LnPlan& p, float* part, cudaStream_t st) {
  constexpr int VV = sizeof(T) == 4 ? 4 : 8;
  const bool want_w = a->dw || a->db;
  float* pw = want_w ? part : nullptr;
  {
    LaunchScope ls("layernorm_bwd_noalloc", st);
    if (p.kind == 0) {
      if (p.v == 1)
        ln_reg_switch<T, 1>(a, p, st, false, pw);
      else
        ln_reg_switch<T, VV>(a, p, st, false, pw);
    } else {
      if (a->dx)
        ln_bwd_long<T><<<p.grid, 256, 0, st>>>((const T*)a->x, (const T*)a->w, (const T*)a->g, a->mean, a->rstd,
                                               (T*)a->dx, a->rows, a->D);
      if (want_w) {
        int64_t rps = (a->rows + p.nslots - 1) / p.nslots;
        dim3 grid((unsigned)((a->D + 255) / 256), (unsigned)p.nslots);
        ln_wgrad_part_long<T><<<grid, 256, 0, st>>>((const T*)a->x, (const T*)a->g, a->mean, a->rstd, pw, a->rows, a->D,
                                                     rps);
      }
    }
  }
  if (want_w) {
    LaunchScope ls("layernorm_wgrad_reduce_noalloc", st);
    dim3 block(kWgradCols, 32);
    ln_wgrad_reduce<T><<<(unsigned)((a->D + kWgradCols - 1) / kWgradCols), block, 0, st>>>(pw, p.nslots, a->D, (T*)a->dw,
                                                                                             (T*)a->db);
  }
  return after_launch("b2_layernorm_bwd_noalloc");
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" {
int b2_softmax_fwd(const b2_softmax_args* a, b2_stream_t s) { return softmax_entry(a, s, true); }
int b2_softmax_bwd(const b2_softmax_args* a, b2_stream_t s) { return softmax_entry(a, s, false); }
int b2_layernorm_fwd(const b2_layernorm_args* a, b2_stream_t s) { return ln_entry(a, s, true); }
int b2_layernorm_bwd(const b2_layernorm_args* a, b2_stream_t s) { return ln_entry(a, s, false); }
int b2_layernorm_bwd_noalloc(const b2_layernorm_args* a, b2_stream_t stream) {
  if (!a) return fail(B2_ERR_ARG, "layernorm_bwd_noalloc: null args");
  if (int rc = ensure_init()) return rc;
  if (a->rows < 0 || a->D < 0) return fail(B2_ERR_ARG, "layernorm_bwd_noalloc: negative size");
  if (a->rows == 0 || a->D == 0) return 0;
  if (!a->x || !a->mean || !a->rstd || !a->g) return fail(B2_ERR_ARG, "layernorm_bwd_noalloc: null pointer");
  // each partial slot holds 2*D floats (weight and bias columns); at least one slot must fit
  const int64_t max_slots = kLnNoAllocScratchFloats / (2 * a->D);
  if ((a->dw || a->db) && max_slots < 1)
    return fail(B2_ERR_ARG, "layernorm_bwd_noalloc: D = " + std::to_string(a->D) + " exceeds the static scratch (D <= " +
                                std::to_string(kLnNoAllocScratchFloats / 2) + ")");
  LnPlan p = ln_plan(a, false);
  if (a->dw || a->db) {
    if (p.kind == 0) {
      const int rpb = 256 / p.group;
      if (max_slots < rpb)
        return fail(B2_ERR_ARG, "layernorm_bwd_noalloc: D too large for the static scratch with this row layout");
      if ((int64_t)p.grid * rpb > max_slots) p.grid = (int)(max_slots / rpb);
      p.nslots = (int64_t)p.grid * rpb;
    } else if (p.nslots > max_slots) {
      p.nslots = max_slots;
    }
  }
  float* part = nullptr;
  if (int rc = ln_noalloc_scratch(&part)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->dtype) {
    case B2_F32: return ln_bwd_planned<float>(a, p, part, st);
    case B2_BF16: return ln_bwd_planned<__nv_bfloat16>(a, p, part, st);
    case B2_F16: return ln_bwd_planned<__half>(a, p, part, st);
    default: return fail(B2_ERR_ARG, "layernorm_bwd_noalloc: dtype must be F32, BF16 or F16");
  }
}
uint64_t b2_layernorm_bwd_workspace_bytes(const b2_layernorm_args* a) {
  if (!a || a->rows <= 0 || a->D <= 0) return 0;
  if (ensure_init()) return 0;
  LnPlan p = ln_plan(a, false);
  return (uint64_t)p.nslots * 2 * (uint64_t)a->D * sizeof(float);
}
}
