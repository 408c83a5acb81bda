// Optimizer elementwise kernels: addcmul / addcdiv / lerp (b2_ew_ternary) and a multi-tensor
// AdamW step (b2_adamw_step).
//
// Expressions follow the reference's generated kernels (tools/gen_shaders.py:83-92, dispatched by
// try_ternary csrc/ops_ew.cpp:405-430): fp32 math, one rounding to the tensor dtype. lerp uses the
// two-branch form of PyTorch's CPU kernel (the reference's CPU fallback), which is exact at weight 1.
// B200 layout: contiguous same-shape operands take a 16-byte vectorised grid-stride path;
// broadcast or strided operands a generic path with up to 8 dims of strides (the reference merges
// to 4, ops_ew.cpp:76-129).
#include "common.cuh"

namespace b2 {
namespace {

__device__ __forceinline__ float ternary(int op, float x, float a, float b, float v) {
  if (op == 0) return x + v * a * b;
  if (op == 1) return x + v * a / b;
  float d = a - x;  // lerp(self=x, end=a, weight=v)
  return fabsf(v) < 0.5f ? x + v * d : a - d * (1.f - v);
}

struct Strides8 {
  int64_t sizes[B2_EW_MAX_DIMS];
  int64_t s[4][B2_EW_MAX_DIMS];  // out, x, t1, t2
  int ndim;
};

template <typename T>
__global__ void ew_generic(T* out, const T* x, const T* t1, const T* t2, Strides8 st, int64_t n, int op, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, o[4] = {0, 0, 0, 0};
    for (int d = st.ndim - 1; d >= 0; --d) {
      int64_t idx = rem % st.sizes[d];
      rem /= st.sizes[d];
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] += idx * st.s[k][d];
    }
    float b = (op == 2) ? 0.f : to_f32(t2[o[3]]);
    out[o[0]] = from_f32<T>(ternary(op, to_f32(x[o[1]]), to_f32(t1[o[2]]), b, v));
  }
}

template <typename T, int V>
__global__ void ew_contig(T* __restrict__ out, const T* x, const T* __restrict__ t1, const T* __restrict__ t2,
                          int64_t n, int op, float v) {
  const int64_t nv = n / V;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    T xv[V], av[V], bv[V], ov[V];
    *reinterpret_cast<uint4*>(xv) = reinterpret_cast<const uint4*>(x)[i];
    *reinterpret_cast<uint4*>(av) = reinterpret_cast<const uint4*>(t1)[i];
    if (op != 2) *reinterpret_cast<uint4*>(bv) = reinterpret_cast<const uint4*>(t2)[i];
#pragma unroll
    for (int k = 0; k < V; ++k)
      ov[k] = from_f32<T>(ternary(op, to_f32(xv[k]), to_f32(av[k]), op != 2 ? to_f32(bv[k]) : 0.f, v));
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<uint4*>(ov);
  }
  // tail
  for (int64_t i = nv * V + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = from_f32<T>(ternary(op, to_f32(x[i]), to_f32(t1[i]), op != 2 ? to_f32(t2[i]) : 0.f, v));
}

// [rows, C] operands whose rows are either contiguous (row stride C) or one broadcast row (row
// stride 0), C contiguous: the residual update x + g * branch with g a per-channel vector.
template <typename T, int V>
__global__ void ew_rows(T* __restrict__ out, const T* x, const T* __restrict__ t1, const T* __restrict__ t2,
                        int64_t rows, int64_t C, int64_t xs, int64_t s1, int64_t s2, int op, float v) {
  const int64_t cv = C / V, nv = rows * cv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cv, c = (i - r * cv) * V;
    T xv[V], av[V], bv[V], ov[V];
    *reinterpret_cast<uint4*>(xv) = *reinterpret_cast<const uint4*>(x + r * xs + c);
    *reinterpret_cast<uint4*>(av) = *reinterpret_cast<const uint4*>(t1 + r * s1 + c);
    if (op != 2) *reinterpret_cast<uint4*>(bv) = *reinterpret_cast<const uint4*>(t2 + r * s2 + c);
#pragma unroll
    for (int k = 0; k < V; ++k)
      ov[k] = from_f32<T>(ternary(op, to_f32(xv[k]), to_f32(av[k]), op != 2 ? to_f32(bv[k]) : 0.f, v));
    *reinterpret_cast<uint4*>(out + r * C + c) = *reinterpret_cast<uint4*>(ov);
  }
}

// Row stride of an operand that is either contiguous over `sizes` or one broadcast row: C or 0;
// -1 otherwise.
int64_t row_stride(const b2_ew_args* a, const int64_t* s) {
  const int nd = a->ndim;
  const int64_t C = a->sizes[nd - 1];
  if (C > 1 && s[nd - 1] != 1) return -1;
  bool contig = true, bcast = true;
  int64_t expect = C;
  for (int d = nd - 2; d >= 0; --d) {
    if (a->sizes[d] != 1) {
      if (s[d] != expect) contig = false;
      if (s[d] != 0) bcast = false;
    }
    expect *= a->sizes[d];
  }
  return contig ? C : bcast ? 0 : -1;
}

template <typename T>
int ew_run(const b2_ew_args* a, cudaStream_t st) {
  int64_t n = 1;
  for (int d = 0; d < a->ndim; ++d) n *= a->sizes[d];
  if (n == 0) return 0;
  // contiguous and identical layouts?
  bool contig = true;
  int64_t expect = 1;
  for (int d = a->ndim - 1; d >= 0; --d) {
    if (a->sizes[d] != 1) {
      if (a->out_s[d] != expect || a->x_s[d] != expect || a->t1_s[d] != expect || (a->op != 2 && a->t2_s[d] != expect))
        contig = false;
    }
    expect *= a->sizes[d];
  }
  constexpr int V = 16 / sizeof(T);
  bool al = ((uintptr_t)a->out | (uintptr_t)a->x | (uintptr_t)a->t1 | (a->op != 2 ? (uintptr_t)a->t2 : 0)) % 16 == 0;
  LaunchScope ls(a->op == 0 ? "ew_addcmul" : a->op == 1 ? "ew_addcdiv" : "ew_lerp", st);
  const int64_t C = a->ndim > 0 ? a->sizes[a->ndim - 1] : 1;
  const int64_t rs_out = a->ndim > 0 ? row_stride(a, a->out_s) : -1, rs_x = a->ndim > 0 ? row_stride(a, a->x_s) : -1;
  const int64_t rs1 = a->ndim > 0 ? row_stride(a, a->t1_s) : -1;
  const int64_t rs2 = (a->ndim > 0 && a->op != 2) ? row_stride(a, a->t2_s) : 0;
  if (contig && al) {
    int grid = grid_for(n / V + 1, 256, 8);
    ew_contig<T, V><<<grid, 256, 0, st>>>((T*)a->out, (const T*)a->x, (const T*)a->t1, (const T*)a->t2, n, a->op, a->value);
  } else if (al && C % V == 0 && rs_out == C && rs_x >= 0 && rs1 >= 0 && rs2 >= 0) {
    const int64_t rows = n / C;
    int grid = grid_for(n / V, 256, 8);
    ew_rows<T, V><<<grid, 256, 0, st>>>((T*)a->out, (const T*)a->x, (const T*)a->t1, (const T*)a->t2, rows, C, rs_x, rs1,
                                        rs2, a->op, a->value);
  } else {
    Strides8 s{};
    s.ndim = a->ndim;
    for (int d = 0; d < a->ndim; ++d) {
      s.sizes[d] = a->sizes[d];
      s.s[0][d] = a->out_s[d];
      s.s[1][d] = a->x_s[d];
      s.s[2][d] = a->t1_s[d];
      s.s[3][d] = a->t2_s[d];
    }
    int grid = grid_for(n, 256, 8);
    ew_generic<T><<<grid, 256, 0, st>>>((T*)a->out, (const T*)a->x, (const T*)a->t1, (const T*)a->t2, s, n, a->op, a->value);
  }
  return after_launch("b2_ew_ternary");
}

// ---- multi-tensor AdamW -------------------------------------------------------------------------
constexpr int kAdamChunk = 48;
struct AdamList {
  void* p[kAdamChunk];
  const void* g[kAdamChunk];
  void* m[kAdamChunk];
  void* v[kAdamChunk];
  int64_t n[kAdamChunk];
};

template <typename T>
__global__ void adamw_multi(AdamList L, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2) {
  const int t = blockIdx.y;
  const int64_t n = L.n[t];
  T* P = (T*)L.p[t];
  const T* G = (const T*)L.g[t];
  T* M = (T*)L.m[t];
  T* Vv = (T*)L.v[t];
  const float step_size = lr / bc1;
  const float bc2_sqrt = sqrtf(bc2);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    // the exact sequence of torch.optim.AdamW(foreach=False), each step rounded to T like the
    // separate in-place ops would be
    float p = to_f32(P[i]), g = to_f32(G[i]), m = to_f32(M[i]), v = to_f32(Vv[i]);
    p = to_f32(from_f32<T>(p * (1.f - lr * wd)));
    m = to_f32(from_f32<T>(ternary(2, m, g, 0.f, 1.f - b1)));
    v = to_f32(from_f32<T>(v * b2));
    v = to_f32(from_f32<T>(v + (1.f - b2) * g * g));
    float denom = to_f32(from_f32<T>(to_f32(from_f32<T>(sqrtf(v))) / bc2_sqrt));
    denom = to_f32(from_f32<T>(denom + eps));
    p = p + (-step_size) * m / denom;
    P[i] = from_f32<T>(p);
    M[i] = from_f32<T>(m);
    Vv[i] = from_f32<T>(v);
  }
}

template <typename T>
int adamw_run(const b2_adamw_args* a, cudaStream_t st) {
  for (int base = 0; base < a->n; base += kAdamChunk) {
    AdamList L{};
    int cnt = std::min(kAdamChunk, a->n - base);
    int64_t mx = 0;
    for (int i = 0; i < cnt; ++i) {
      L.p[i] = a->param[base + i];
      L.g[i] = a->grad[base + i];
      L.m[i] = a->exp_avg[base + i];
      L.v[i] = a->exp_avg_sq[base + i];
      L.n[i] = a->numel[base + i];
      mx = std::max(mx, L.n[i]);
    }
    if (mx == 0) continue;
    dim3 grid((unsigned)std::min<int64_t>((mx + 255) / 256, 64), (unsigned)cnt);
    LaunchScope ls("adamw_multi_tensor", st);
    adamw_multi<T><<<grid, 256, 0, st>>>(L, a->lr, a->beta1, a->beta2, a->eps, a->weight_decay, a->bias_correction1,
                                         a->bias_correction2);
  }
  return after_launch("b2_adamw_step");
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" int b2_ew_ternary(const b2_ew_args* a, b2_stream_t stream) {
  if (!a) return fail(B2_ERR_ARG, "ew_ternary: null args");
  if (int rc = ensure_init()) return rc;
  if (a->ndim < 0 || a->ndim > B2_EW_MAX_DIMS) return fail(B2_ERR_ARG, "ew_ternary: ndim must be 0..8");
  if (a->op < 0 || a->op > 2) return fail(B2_ERR_ARG, "ew_ternary: op must be 0 (addcmul), 1 (addcdiv) or 2 (lerp)");
  if (!a->out || !a->x || !a->t1 || (a->op != 2 && !a->t2)) return fail(B2_ERR_ARG, "ew_ternary: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->dtype) {
    case B2_F32: return ew_run<float>(a, st);
    case B2_BF16: return ew_run<__nv_bfloat16>(a, st);
    case B2_F16: return ew_run<__half>(a, st);
    default: return fail(B2_ERR_ARG, "ew_ternary: dtype must be F32, BF16 or F16");
  }
}

extern "C" int b2_adamw_step(const b2_adamw_args* a, b2_stream_t stream) {
  if (!a) return fail(B2_ERR_ARG, "adamw: null args");
  if (int rc = ensure_init()) return rc;
  if (a->n < 0) return fail(B2_ERR_ARG, "adamw: negative tensor count");
  if (a->n == 0) return 0;
  if (!a->param || !a->grad || !a->exp_avg || !a->exp_avg_sq || !a->numel) return fail(B2_ERR_ARG, "adamw: null list");
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->dtype) {
    case B2_F32: return adamw_run<float>(a, st);
    case B2_BF16: return adamw_run<__nv_bfloat16>(a, st);
    default: return fail(B2_ERR_ARG, "adamw: dtype must be F32 or BF16");
  }
}
