// b2_int8_gemm's forward form for a few rows of x (M <= 8): the DiT block's adaLN modulation
// (one conditioning vector per sample against an int8 [18432, 2048] weight) and batch-1 decode shapes.
// A tensor-core tile is 128 rows tall, so at M = 1 it would spend 127/128 of its MMA work and all of
// its per-tile set-up on padding; this path is a weight stream instead: each warp walks whole rows n of
// q with 16-byte loads (four in flight per lane), dequantises them exactly as the GEMM's mainloop does
// (bf16(float(q) * scale), bit-identical to b2_dequant_int8) and accumulates x . w in fp32 for every
// row m of x from shared memory; a warp reduction, + bias, one bf16 rounding. The bound is HBM: the
// int8 weight is read once (N * K bytes).
#include <cstdlib>

#include "common.cuh"

namespace b2 {
namespace {

constexpr int kGvThreads = 256;
constexpr int kGvWarps = kGvThreads / 32;
constexpr int kGvLoads = 4;                       // 16-byte weight loads in flight per lane
constexpr int kGvMaxSmem = 96 * 1024;            // x staged as fp32: M * K * 4 bytes at most
constexpr int kGvMaxRows = 8;

__device__ __forceinline__ int4 ld_stream(const int8_t* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// x is staged chunk-transposed: the 16 values of 16-column chunk c are four float4 pieces, piece j of
// every chunk stored contiguously (index j * chunks + c), so that the 32 lanes of a warp, reading
// piece j of 32 consecutive chunks, touch 512 consecutive bytes (no bank conflicts).
template <int MR>
__global__ void __launch_bounds__(kGvThreads) int8_gemv_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_ld, int M,
                                                              const int8_t* __restrict__ q, const void* __restrict__ scale,
                                                              int scale_layout, const __nv_bfloat16* __restrict__ bias,
                                                              __nv_bfloat16* __restrict__ out, int64_t out_ld, int64_t N,
                                                              int64_t K) {
  extern __shared__ float4 xs[];  // [MR][4][chunks]
  const int64_t chunks = K / 16;
  for (int64_t i = threadIdx.x; i < (int64_t)MR * chunks * 4; i += kGvThreads) {
    const int m = (int)(i / (chunks * 4));
    const int64_t r = i - (int64_t)m * chunks * 4;  // r = c * 4 + j: four consecutive columns of x
    const int64_t c = r >> 2;
    const int j = (int)(r & 3);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m < M) {
      const __nv_bfloat16* xp = x + (int64_t)m * x_ld + c * 16 + j * 4;
      v = make_float4(__bfloat162float(xp[0]), __bfloat162float(xp[1]), __bfloat162float(xp[2]), __bfloat162float(xp[3]));
    }
    xs[(int64_t)m * chunks * 4 + (int64_t)j * chunks + c] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nb = (K + 63) / 64;  // scale_layout 0: one bf16 scale per 64 columns
  for (int64_t n = (int64_t)blockIdx.x * kGvWarps + warp; n < N; n += (int64_t)gridDim.x * kGvWarps) {
    const int8_t* qr = q + n * K;
    const float srow = scale_layout == 1 ? static_cast<const float*>(scale)[n] : 0.f;
    float acc[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[m] = 0.f;
    for (int64_t c0 = lane; c0 < chunks; c0 += 32 * kGvLoads) {
      int4 raw[kGvLoads];
#pragma unroll
      for (int u = 0; u < kGvLoads; ++u) {
        const int64_t c = c0 + u * 32;
        raw[u] = c < chunks ? ld_stream(qr + c * 16) : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kGvLoads; ++u) {
        const int64_t c = c0 + u * 32;
        if (c >= chunks) break;
        const float s = scale_layout == 1
                            ? srow
                            : __bfloat162float(static_cast<const __nv_bfloat16*>(scale)[n * nb + (c >> 2)]);
        uint32_t w[8];
        dequant16(raw[u], s, w);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          const float4* xm = xs + (int64_t)m * chunks * 4 + c;
          float a = acc[m];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 xv = xm[(int64_t)j * chunks];
            const uint32_t w0 = w[2 * j], w1 = w[2 * j + 1];
            a = fmaf(xv.x, __uint_as_float(w0 << 16), a);
            a = fmaf(xv.y, __uint_as_float(w0 & 0xffff0000u), a);
            a = fmaf(xv.z, __uint_as_float(w1 << 16), a);
            a = fmaf(xv.w, __uint_as_float(w1 & 0xffff0000u), a);
          }
          acc[m] = a;
        }
      }
    }
    const float b = bias ? __bfloat162float(bias[n]) : 0.f;
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      float a = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0 && m < M) out[(int64_t)m * out_ld + n] = Num<__nv_bfloat16>::from_f(a + b);
    }
  }
}

template <int MR>
int gemv_run(const b2_int8_gemm_args* a, cudaStream_t st) {
  auto kern = int8_gemv_kernel<MR>;
  const int smem = (int)(MR * a->K * 4);
  static bool attr = false;  // one device per process
  if (!attr) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGvMaxSmem),
                            "cudaFuncSetAttribute(int8_gemv)"))
      return rc;
    attr = true;
  }
  const int sms = device_info().sm_count > 0 ? device_info().sm_count : 148;
  const int per_sm = std::max(1, std::min(8, (int)((228 * 1024) / (smem + 1024))));
  const int64_t want = (a->N + kGvWarps - 1) / kGvWarps;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * std::min(per_sm, 4)));
  LaunchScope ls("int8_gemv", st);
  kern<<<blocks, kGvThreads, smem, st>>>((const __nv_bfloat16*)a->x, a->x_ld, (int)a->M, a->q, a->scale, a->scale_layout,
                                        (const __nv_bfloat16*)a->bias, (__nv_bfloat16*)a->out, a->out_ld, a->N, a->K);
  return after_launch("b2_int8_gemm (gemv)");
}

int gemv_rows(int64_t m) { return m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8; }

}  // namespace

// B2_INT8_GEMV=0 turns the path off (measurement sweeps); the tensor-core GEMM then takes these shapes
bool int8_gemv_applies(const b2_int8_gemm_args* a) {
  static const bool off = [] {
    const char* e = getenv("B2_INT8_GEMV");
    return e && e[0] == '0';
  }();
  return !off && !a->transpose_w && !a->epilogue && !a->lora_r && a->M >= 1 && a->M <= kGvMaxRows &&
         gemv_rows(a->M) * a->K * 4 <= kGvMaxSmem && a->out_ld >= a->N;
}

int int8_gemv_launch(const b2_int8_gemm_args* a, cudaStream_t st) {
  switch (gemv_rows(a->M)) {
    case 1: return gemv_run<1>(a, st);
    case 2: return gemv_run<2>(a, st);
    case 4: return gemv_run<4>(a, st);
    default: return gemv_run<8>(a, st);
  }
}

}  // namespace b2
