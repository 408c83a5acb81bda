// Mean-squared-error loss of the DiT LoRA step (b2_mse_loss_fwd / b2_mse_loss_bwd), the arithmetic of
// F.mse_loss(x.float(), t.float()) read straight from the 16-bit tensors: fp32 differences and sums, no
// fp32 copies of the operands, and a fixed summation order so that the loss is the same bits on every
// run (per-block partial sums, then one block adds them in block order).
#include "common.cuh"

namespace b2 {
namespace {

constexpr int kMseThreads = 256;
constexpr int kMseMaxBlocks = 1024;

// V elements per step: 16 bytes at a time (8 x 16-bit, 4 x fp32) when n and the pointers allow it, else 1
template <typename T, int V>
__device__ __forceinline__ void load_v(const T* p, float* f) {
  if constexpr (V == 1) {
    f[0] = to_f32(*p);
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < V; ++i) f[i] = to_f32(h[i]);
  }
}

template <typename T, int V>
__global__ void __launch_bounds__(kMseThreads) mse_partial(const T* __restrict__ x, const T* __restrict__ t, int64_t n,
                                                           float* __restrict__ partial) {
  __shared__ float red[kMseThreads / 32];
  float s = 0.f;
  for (int64_t i = (blockIdx.x * (int64_t)kMseThreads + threadIdx.x) * V; i < n; i += (int64_t)gridDim.x * kMseThreads * V) {
    float a[V], b[V];
    load_v<T, V>(x + i, a);
    load_v<T, V>(t + i, b);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float d = a[j] - b[j];
      s = fmaf(d, d, s);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.f;
#pragma unroll
    for (int w = 0; w < kMseThreads / 32; ++w) b += red[w];
    partial[blockIdx.x] = b;
  }
}

__global__ void __launch_bounds__(kMseThreads) mse_final(const float* __restrict__ partial, int nparts, float inv_n,
                                                         float* __restrict__ loss) {
  __shared__ float red[kMseThreads];
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += kMseThreads) s += partial[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int k = kMseThreads / 2; k > 0; k >>= 1) {
    if (threadIdx.x < k) red[threadIdx.x] += red[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = red[0] * inv_n;
}

template <typename T, int V>
__global__ void __launch_bounds__(kMseThreads) mse_grad(const T* __restrict__ x, const T* __restrict__ t, int64_t n,
                                                        const float* __restrict__ grad_loss, float two_over_n,
                                                        T* __restrict__ gx) {
  const float k = *grad_loss * two_over_n;
  for (int64_t i = (blockIdx.x * (int64_t)kMseThreads + threadIdx.x) * V; i < n; i += (int64_t)gridDim.x * kMseThreads * V) {
    float a[V], b[V];
    load_v<T, V>(x + i, a);
    load_v<T, V>(t + i, b);
    if constexpr (V == 1) {
      gx[i] = from_f32<T>((a[0] - b[0]) * k);
    } else {
      uint4 u;
      T* h = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int j = 0; j < V; ++j) h[j] = from_f32<T>((a[j] - b[j]) * k);
      *reinterpret_cast<uint4*>(gx + i) = u;
    }
  }
}

// 16-byte steps need n a multiple of the step and 16-byte aligned tensors
template <typename T>
constexpr int vec_of() {
  return 16 / (int)sizeof(T);
}
bool vec_ok(const b2_mse_args* a, int v, bool bwd) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  return a->n % v == 0 && al(a->x) && al(a->t) && (!bwd || al(a->grad_x));
}

int mse_blocks(int64_t n) {
  const int64_t want = (n + kMseThreads * 8 - 1) / (kMseThreads * 8);  // about eight elements per thread
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, std::min<int64_t>(kMseMaxBlocks, device_info().sm_count * 8)));
}

int mse_check(const b2_mse_args* a, bool fwd) {
  if (!a) return fail(B2_ERR_ARG, "mse_loss: null args");
  if (int rc = ensure_init()) return rc;
  if (a->n < 0) return fail(B2_ERR_ARG, "mse_loss: negative n");
  if (a->dtype != B2_F32 && a->dtype != B2_BF16 && a->dtype != B2_F16)
    return fail(B2_ERR_ARG, "mse_loss: dtype must be F32, BF16 or F16");
  if (a->n > 0 && (!a->x || !a->t)) return fail(B2_ERR_ARG, "mse_loss: null input");
  if (fwd && (!a->loss || (a->n > 0 && !a->partial))) return fail(B2_ERR_ARG, "mse_loss: null loss or scratch");
  if (!fwd && a->n > 0 && (!a->grad_x || !a->grad_loss)) return fail(B2_ERR_ARG, "mse_loss: null gradient");
  return 0;
}

template <typename T>
int mse_fwd_run(const b2_mse_args* a, cudaStream_t st) {
  const int blocks = mse_blocks(a->n);
  {
    LaunchScope ls("mse_partial", st);
    constexpr int V = vec_of<T>();
    if (vec_ok(a, V, false))
      mse_partial<T, V><<<blocks, kMseThreads, 0, st>>>((const T*)a->x, (const T*)a->t, a->n, a->partial);
    else
      mse_partial<T, 1><<<blocks, kMseThreads, 0, st>>>((const T*)a->x, (const T*)a->t, a->n, a->partial);
  }
  {
    LaunchScope ls("mse_final", st);
    mse_final<<<1, kMseThreads, 0, st>>>(a->partial, blocks, 1.f / (float)a->n, a->loss);
  }
  return after_launch("b2_mse_loss_fwd");
}

template <typename T>
int mse_bwd_run(const b2_mse_args* a, cudaStream_t st) {
  LaunchScope ls("mse_grad", st);
  constexpr int V = vec_of<T>();
  if (vec_ok(a, V, true))
    mse_grad<T, V><<<mse_blocks(a->n), kMseThreads, 0, st>>>((const T*)a->x, (const T*)a->t, a->n, a->grad_loss,
                                                             2.f / (float)a->n, (T*)a->grad_x);
  else
    mse_grad<T, 1><<<mse_blocks(a->n), kMseThreads, 0, st>>>((const T*)a->x, (const T*)a->t, a->n, a->grad_loss,
                                                             2.f / (float)a->n, (T*)a->grad_x);
  return after_launch("b2_mse_loss_bwd");
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" uint64_t b2_mse_loss_workspace_bytes(int64_t n) {
  if (n <= 0 || ensure_init()) return 0;
  return (uint64_t)mse_blocks(n) * sizeof(float);
}

extern "C" int b2_mse_loss_fwd(const b2_mse_args* a, b2_stream_t stream) {
  if (int rc = mse_check(a, true)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // the mean over no elements is NaN, as F.mse_loss gives (all-ones bytes are a NaN)
  if (a->n == 0) return check_cuda(cudaMemsetAsync(a->loss, 0xff, sizeof(float), st), "mse_loss");
  switch (a->dtype) {
    case B2_BF16: return mse_fwd_run<__nv_bfloat16>(a, st);
    case B2_F16: return mse_fwd_run<__half>(a, st);
    default: return mse_fwd_run<float>(a, st);
  }
}

extern "C" int b2_mse_loss_bwd(const b2_mse_args* a, b2_stream_t stream) {
  if (int rc = mse_check(a, false)) return rc;
  if (a->n == 0) return 0;
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->dtype) {
    case B2_BF16: return mse_bwd_run<__nv_bfloat16>(a, st);
    case B2_F16: return mse_bwd_run<__half>(a, st);
    default: return mse_bwd_run<float>(a, st);
  }
}
