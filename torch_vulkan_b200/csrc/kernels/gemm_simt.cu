// Strided SIMT GEMM: the general path of b2_gemm for fp32/fp64 and for bf16/f16 layouts the TMA
// tensor-core kernel cannot address (odd strides, unaligned views).
//
// Same contract as the reference's tiled kernel vkrt/shaders/mm.comp.in:46-155 (64x64 tile, any
// non-negative strides, alpha/beta/broadcast bias, fp32 accumulate) with fp64 accumulate for
// fp64 inputs. 256 threads compute a 64x64 tile, 4x4 outputs each, from a double-buffered
// shared-memory K slice of 16.
#include "common.cuh"

namespace b2 {

int gemm_tc_launch(const b2_gemm_args* a, cudaStream_t st);  // gemm_tc.cu
bool gemm_tc_eligible(const b2_gemm_args* a);
bool gemm_skinny_applies(const b2_gemm_args* a);                // gemm_skinny.cu
int gemm_skinny_launch(const b2_gemm_args* a, cudaStream_t st);
uint64_t gemm_tc_workspace_bytes(const b2_gemm_args* a);  // gemm_tc.cu

namespace {

template <typename T>
struct AccOf {
  using type = float;
};
template <>
struct AccOf<double> {
  using type = double;
};

template <typename T>
__device__ __forceinline__ typename AccOf<T>::type to_acc(T v) {
  return (typename AccOf<T>::type)to_f32(v);
}
template <>
__device__ __forceinline__ double to_acc<double>(double v) {
  return v;
}
template <typename T>
__device__ __forceinline__ T from_acc(typename AccOf<T>::type v) {
  return from_f32<T>((float)v);
}
template <>
__device__ __forceinline__ double from_acc<double>(double v) {
  return v;
}

constexpr int BM = 64, BN = 64, BK = 16;

template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(b2_gemm_args p) {
  using Acc = typename AccOf<T>::type;
  __shared__ Acc As[2][BK][BM + 4];
  __shared__ Acc Bs[2][BK][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int64_t bz = blockIdx.z;
  const T* A = (const T*)p.a + bz * p.a_sb;
  const T* B = (const T*)p.b + bz * p.b_sb;
  Acc acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0;

  auto load = [&](int buf, int64_t k0) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      int e = tid + r * 256;  // 0..1023 over a 64x16 tile
      // A tile: m = e % 64, k = e / 64 (consecutive threads walk m: coalesced when a_sm == 1)
      int mm = e % BM, kk = e / BM;
      int64_t gm = m0 + mm, gk = k0 + kk;
      As[buf][kk][mm] = (gm < p.M && gk < p.K) ? to_acc<T>(A[gm * p.a_sm + gk * p.a_sk]) : (Acc)0;
      int nn = e % BN, kb = e / BN;
      int64_t gn = n0 + nn, gkb = k0 + kb;
      Bs[buf][kb][nn] = (gn < p.N && gkb < p.K) ? to_acc<T>(B[gkb * p.b_sk + gn * p.b_sn]) : (Acc)0;
    }
  };
  int buf = 0;
  load(0, 0);
  __syncthreads();
  for (int64_t k0 = 0; k0 < p.K; k0 += BK) {
    if (k0 + BK < p.K) load(buf ^ 1, k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      Acc av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[buf][kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[buf][kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
    }
    __syncthreads();
    buf ^= 1;
  }
  T* C = (T*)p.c + bz * p.c_sb;
  const T* bias = (const T*)p.bias;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t gm = m0 + ty * 4 + i;
    if (gm >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t gn = n0 + tx * 4 + j;
      if (gn >= p.N) continue;
      Acc r = (Acc)p.alpha * acc[i][j];
      if (p.has_bias) r += (Acc)p.beta * to_acc<T>(bias[bz * p.bias_sb + gm * p.bias_sm + gn * p.bias_sn]);
      C[gm * p.c_sm + gn * p.c_sn] = from_acc<T>(r);
    }
  }
}

template <typename T>
int simt_launch(const b2_gemm_args* a, cudaStream_t st) {
  dim3 grid((unsigned)((a->N + BN - 1) / BN), (unsigned)((a->M + BM - 1) / BM), (unsigned)a->batch);
  LaunchScope ls("gemm_simt", st);
  gemm_simt_kernel<T><<<grid, 256, 0, st>>>(*a);
  return after_launch("b2_gemm(simt)");
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" uint64_t b2_gemm_workspace_bytes(const b2_gemm_args* a) {
  if (!a || a->force_simt || ensure_init()) return 0;
  if (a->K > 0 && gemm_skinny_applies(a)) return 0;
  return a->K > 0 ? gemm_tc_workspace_bytes(a) : 0;
}

extern "C" int b2_gemm_path(const b2_gemm_args* a) {
  if (!a || a->force_simt) return 0;
  if (a->K > 0 && gemm_skinny_applies(a)) return 2;
  return gemm_tc_eligible(a) ? 1 : 0;
}

extern "C" int b2_gemm(const b2_gemm_args* a, b2_stream_t stream) {
  if (!a) return fail(B2_ERR_ARG, "gemm: null args");
  if (int rc = ensure_init()) return rc;
  if (a->M < 0 || a->N < 0 || a->K < 0 || a->batch < 0) return fail(B2_ERR_ARG, "gemm: negative size");
  if (a->M == 0 || a->N == 0 || a->batch == 0) return 0;
  if (a->batch > 65535) return fail(B2_ERR_ARG, "gemm: batch > 65535");
  const int64_t st[] = {a->a_sb, a->a_sm, a->a_sk, a->b_sb, a->b_sk, a->b_sn, a->c_sb, a->c_sm, a->c_sn};
  for (int64_t s : st)
    if (s < 0) return fail(B2_ERR_ARG, "gemm: negative stride");
  if (!a->c || (a->K > 0 && (!a->a || !a->b))) return fail(B2_ERR_ARG, "gemm: null pointer");
  if (a->has_bias && !a->bias) return fail(B2_ERR_ARG, "gemm: has_bias with null bias");
  cudaStream_t s = (cudaStream_t)stream;
  if (!a->force_simt && a->K > 0 && gemm_skinny_applies(a)) return gemm_skinny_launch(a, s);
  if (!a->force_simt && a->K > 0 && gemm_tc_eligible(a)) return gemm_tc_launch(a, s);
  switch (a->dtype) {
    case B2_F32: return simt_launch<float>(a, s);
    case B2_BF16: return simt_launch<__nv_bfloat16>(a, s);
    case B2_F16: return simt_launch<__half>(a, s);
    case B2_F64: return simt_launch<double>(a, s);
    default: return fail(B2_ERR_ARG, "gemm: dtype must be F32, BF16, F16 or F64");
  }
}
