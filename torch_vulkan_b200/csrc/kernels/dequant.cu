// Weight-only int8 dequantisation (b2_dequant_int8).
//
// Same arithmetic as the reference kernel vkrt/shaders/dq8.comp.in:27-62 and its pure-PyTorch
// reference torch_vulkan/__init__.py:203-205: out = round(float(q) * float(scale)), one fp32 multiply,
// one round-to-nearest-even. B200 layout: one thread dequantises 16 int8 (one 16-byte load) and
// writes 16 outputs with 16-byte stores; a grid-stride loop over a grid sized to the SM count.
#include "common.cuh"

namespace b2 {
namespace {

template <typename OutT>
struct Store16;

template <>
struct Store16<float> {
  static __device__ __forceinline__ void run(float* out, const float* v) {
    float4* o = reinterpret_cast<float4*>(out);
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
};
template <>
struct Store16<__nv_bfloat16> {
  static __device__ __forceinline__ void run(__nv_bfloat16* out, const float* v) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      w[i] = (uint32_t)f32_to_bf16_bits(v[2 * i]) | ((uint32_t)f32_to_bf16_bits(v[2 * i + 1]) << 16);
    uint4* o = reinterpret_cast<uint4*>(out);
    o[0] = make_uint4(w[0], w[1], w[2], w[3]);
    o[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
};
template <>
struct Store16<__half> {
  static __device__ __forceinline__ void run(__half* out, const float* v) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      __half a = __float2half_rn(v[2 * i]), b = __float2half_rn(v[2 * i + 1]);
      w[i] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
    }
    uint4* o = reinterpret_cast<uint4*>(out);
    o[0] = make_uint4(w[0], w[1], w[2], w[3]);
    o[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
};

__device__ __forceinline__ float load_scale(const void* scale, int layout, int64_t r, int64_t c, int64_t nb) {
  if (layout == 0) return bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(scale)[r * nb + (c >> 6)]);
  return reinterpret_cast<const float*>(scale)[r];
}

// 16 consecutive int8 of one row per thread; requires cols % 16 == 0 and aligned rows.
template <typename OutT>
__global__ void dequant_vec16(const int8_t* __restrict__ q, const void* __restrict__ scale, OutT* __restrict__ out,
                              int64_t rows, int64_t cols, int64_t q_ld, int layout) {
  const int64_t chunks_per_row = cols >> 4;
  const int64_t total = rows * chunks_per_row;
  const int64_t nb = (cols + 63) >> 6;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / chunks_per_row;
    int64_t c = (i - r * chunks_per_row) << 4;
    int4 raw = __ldg(reinterpret_cast<const int4*>(q + r * q_ld + c));
    const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
    float s = load_scale(scale, layout, r, c, nb);  // a 16-aligned chunk never crosses a 64-block
    float v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = (float)b[k] * s;
    Store16<OutT>::run(out + r * cols + c, v);
  }
}

template <typename OutT>
__global__ void dequant_scalar(const int8_t* __restrict__ q, const void* __restrict__ scale, OutT* __restrict__ out,
                               int64_t rows, int64_t cols, int64_t q_ld, int layout) {
  const int64_t total = rows * cols;
  const int64_t nb = (cols + 63) >> 6;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / cols, c = i - r * cols;
    float v = (float)q[r * q_ld + c] * load_scale(scale, layout, r, c, nb);
    out[i] = from_f32<OutT>(v);
  }
}

template <typename OutT>
int launch(const b2_dequant_args* a, cudaStream_t st) {
  const bool vec = (a->cols % 16 == 0) && (a->q_ld % 16 == 0) && ((uintptr_t)a->q % 16 == 0) &&
                   ((uintptr_t)a->out % 16 == 0);
  const int threads = 256;
  if (vec) {
    LaunchScope ls("dequant_int8_vec16", st);
    int grid = grid_for(a->rows * (a->cols / 16), threads, 8);
    dequant_vec16<OutT><<<grid, threads, 0, st>>>(a->q, a->scale, (OutT*)a->out, a->rows, a->cols, a->q_ld,
                                                  a->scale_layout);
  } else {
    LaunchScope ls("dequant_int8_scalar", st);
    int grid = grid_for(a->rows * a->cols, threads, 8);
    dequant_scalar<OutT><<<grid, threads, 0, st>>>(a->q, a->scale, (OutT*)a->out, a->rows, a->cols, a->q_ld,
                                                   a->scale_layout);
  }
  return after_launch("b2_dequant_int8");
}

}  // namespace
}  // namespace b2

using namespace b2;

extern "C" int b2_dequant_int8(const b2_dequant_args* a, b2_stream_t stream) {
  if (!a) return fail(B2_ERR_ARG, "dequant_int8: null args");
  if (int rc = ensure_init()) return rc;
  if (a->rows < 0 || a->cols < 0 || a->q_ld < a->cols) return fail(B2_ERR_ARG, "dequant_int8: bad shape");
  if (a->scale_layout != 0 && a->scale_layout != 1) return fail(B2_ERR_ARG, "dequant_int8: scale_layout must be 0 or 1");
  if (a->rows == 0 || a->cols == 0) return 0;
  if (!a->q || !a->scale || !a->out) return fail(B2_ERR_ARG, "dequant_int8: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->out_dtype) {
    case B2_F32: return launch<float>(a, st);
    case B2_BF16: return launch<__nv_bfloat16>(a, st);
    case B2_F16: return launch<__half>(a, st);
    default: return fail(B2_ERR_ARG, "dequant_int8: out_dtype must be F32, BF16 or F16");
  }
}
