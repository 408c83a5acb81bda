// Device helpers shared by the kernels of libb2rt.so.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>

#include "../runtime/b2_internal.h"

namespace b2 {

// fp32 -> bf16 bits with round-to-nearest-even and canonical NaN 0x7FC0: the same bit pattern as
// torch's CPU conversion (c10::BFloat16) and the reference shader's f2bf
// (vkrt/shaders/types.glsl:45-50). Standard RNE bit trick: add 0x7FFF plus the lsb of the kept half.
__host__ __device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
#ifdef __CUDA_ARCH__
  uint32_t u = __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
#endif
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

template <typename T>
struct Num;

template <>
struct Num<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <>
struct Num<double> {
  static __device__ __forceinline__ double to_f(double v) { return v; }
  static __device__ __forceinline__ double from_f(double v) { return v; }
};
template <>
struct Num<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) {
    uint16_t b = f32_to_bf16_bits(v);
    return *reinterpret_cast<__nv_bfloat16*>(&b);
  }
};
template <>
struct Num<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  return (float)Num<T>::to_f(v);
}
template <typename T>
__device__ __forceinline__ T from_f32(float v) {
  return Num<T>::from_f(v);
}
template <>
__device__ __forceinline__ double from_f32<double>(float v) {
  return (double)v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 and <= 1024. `red` has >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float r = lane < nw ? red[lane] : 0.f;
  return warp_sum(r);
}
__device__ __forceinline__ float block_max(float v, float* red) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float r = lane < nw ? red[lane] : -INFINITY;
  return warp_max(r);
}

inline int grid_for(int64_t work_items, int per_block, int max_blocks_per_sm = 8) {
  int64_t blocks = (work_items + per_block - 1) / per_block;
  int sms = device_info().sm_count > 0 ? device_info().sm_count : 148;
  int64_t cap = (int64_t)sms * max_blocks_per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

// 16 int8 * scale -> 8 words of packed bf16 (one fp32 multiply and one round-to-nearest-even each,
// the same bits as b2_dequant_int8 for every finite product). The exact int8 -> fp32 step and the
// scale multiply run as packed two-lane fp32 operations (each lane rounds exactly as the scalar op).
__device__ __forceinline__ void dequant16(const int4& raw, float s, uint32_t* w) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(&raw);
  const float2 ss = make_float2(s, s);
  const float2 bias = make_float2(-8388736.f, -8388736.f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t u = r[i] ^ 0x80808080u;
    float2 lo = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)));
    float2 hi = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                            __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)));
    lo = __fmul2_rn(__fadd2_rn(lo, bias), ss);
    hi = __fmul2_rn(__fadd2_rn(hi, bias), ss);
    __nv_bfloat162 blo = __floats2bfloat162_rn(lo.x, lo.y);
    __nv_bfloat162 bhi = __floats2bfloat162_rn(hi.x, hi.y);
    w[2 * i] = *reinterpret_cast<uint32_t*>(&blo);
    w[2 * i + 1] = *reinterpret_cast<uint32_t*>(&bhi);
  }
}

}  // namespace b2
