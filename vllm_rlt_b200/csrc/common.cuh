// Shared device helpers for the B200 (sm_100a) paged-KV kernels.
//
// Element types are passed across the C ABI as an integer code (RLT_F32,
// RLT_F16, RLT_BF16). Every kernel moves K/V through 16-byte vectors; the
// helpers below convert one 16-byte vector into fp32 lanes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rlt_b200.h"

namespace rlt {

constexpr unsigned kFullMask = 0xffffffffu;

// Status bits a kernel may OR into the caller's status word. They report
// caller bugs (metadata that points outside the pool) without faulting: the
// offending page or row is skipped and the bit is raised.
constexpr int32_t kStatusBadLength = 1;   // context length < 0 or > table width * page
constexpr int32_t kStatusBadBlock = 2;    // block id outside [0, num_blocks)
constexpr int32_t kStatusBadOffset = 4;   // in-page offset outside [0, page)
constexpr int32_t kStatusBadSlot = 8;     // descriptor slot / depth outside the resident tables
constexpr int32_t kStatusBadSequence = 16;  // packed-prefill sequence metadata inconsistent
constexpr int32_t kStatusTimeout = 32;      // a bounded wait gave up (the call's output is void)

// Inter-CTA hand-off through global memory (gpu scope).
__device__ __forceinline__ int ld_acquire_gpu(const int* ptr) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* ptr, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

__device__ __forceinline__ void raise_status(int32_t* status, int32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

template <typename T>
struct Vec16 {
  static constexpr int kElems = 16 / sizeof(T);
};

// Streaming 16-byte load of data that is read once (K/V pages).
__device__ __forceinline__ uint4 ld_stream(const void* ptr) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(ptr));
  return r;
}

__device__ __forceinline__ uint4 ld_vec(const void* ptr) {
  return *reinterpret_cast<const uint4*>(ptr);
}

__device__ __forceinline__ void st_vec(void* ptr, uint4 v) {
  *reinterpret_cast<uint4*>(ptr) = v;
}

// Base-2 exponential: the hardware approximation (MUFU.EX2), relative
// error about 2^-22, flushes denormals; ex2(-inf) = +0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- 16-byte vector <-> fp32 conversion -----------------------------------

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& r, float* f);

template <>
__device__ __forceinline__ void unpack16<float>(const uint4& r, float* f) {
  f[0] = __uint_as_float(r.x);
  f[1] = __uint_as_float(r.y);
  f[2] = __uint_as_float(r.z);
  f[3] = __uint_as_float(r.w);
}

// bf16 -> fp32 is exact: the bf16 bits are the top half of the fp32 bits.
__device__ __forceinline__ void bf16x2_to_f32(uint32_t w, float& lo, float& hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xffff0000u);
}

template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& r, float* f) {
  bf16x2_to_f32(r.x, f[0], f[1]);
  bf16x2_to_f32(r.y, f[2], f[3]);
  bf16x2_to_f32(r.z, f[4], f[5]);
  bf16x2_to_f32(r.w, f[6], f[7]);
}

__device__ __forceinline__ void f16x2_to_f32(uint32_t w, float& lo, float& hi) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  float2 f = __half22float2(h);
  lo = f.x;
  hi = f.y;
}

template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& r, float* f) {
  f16x2_to_f32(r.x, f[0], f[1]);
  f16x2_to_f32(r.y, f[2], f[3]);
  f16x2_to_f32(r.z, f[4], f[5]);
  f16x2_to_f32(r.w, f[6], f[7]);
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f);

template <>
__device__ __forceinline__ uint4 pack16<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}

// Round-to-nearest-even, the rounding of torch's .to(bfloat16/float16).
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* f) {
  uint4 r;
  __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
  __nv_bfloat162 c = __floats2bfloat162_rn(f[4], f[5]);
  __nv_bfloat162 d = __floats2bfloat162_rn(f[6], f[7]);
  r.x = *reinterpret_cast<uint32_t*>(&a);
  r.y = *reinterpret_cast<uint32_t*>(&b);
  r.z = *reinterpret_cast<uint32_t*>(&c);
  r.w = *reinterpret_cast<uint32_t*>(&d);
  return r;
}

template <>
__device__ __forceinline__ uint4 pack16<__half>(const float* f) {
  uint4 r;
  __half2 a = __floats2half2_rn(f[0], f[1]);
  __half2 b = __floats2half2_rn(f[2], f[3]);
  __half2 c = __floats2half2_rn(f[4], f[5]);
  __half2 d = __floats2half2_rn(f[6], f[7]);
  r.x = *reinterpret_cast<uint32_t*>(&a);
  r.y = *reinterpret_cast<uint32_t*>(&b);
  r.z = *reinterpret_cast<uint32_t*>(&c);
  r.w = *reinterpret_cast<uint32_t*>(&d);
  return r;
}

// Scalar element <-> fp32 for the generic (any head_dim) paths.
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

inline int launch_status(cudaError_t err) {
  return err == cudaSuccess ? RLT_OK : static_cast<int>(err);
}

}  // namespace rlt
