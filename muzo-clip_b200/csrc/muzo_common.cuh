// Shared device helpers for the MuZO-Clip sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "muzo_b200.h"

namespace muzo {

// Records the CUDA error of the last failed call so the C ABI can report it.
void set_last_cuda_error(cudaError_t err);

#define MUZO_CUDA_CHECK(expr)                                   \
  do {                                                          \
    cudaError_t err__ = (expr);                                 \
    if (err__ != cudaSuccess) {                                 \
      ::muzo::set_last_cuda_error(err__);                       \
      return MUZO_ERR_CUDA;                                     \
    }                                                           \
  } while (0)

// Checks the launch that was just enqueued.
inline int launch_status() {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return MUZO_ERR_CUDA;
  }
  return MUZO_OK;
}

// Number of SMs of the current device (cached per device ordinal).
int device_sm_count();

// ------------------------------------------------------------------ element conversions

__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dtype) {
  if (dtype == MUZO_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == MUZO_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_elem(void* p, int64_t i, int dtype, float v) {
  if (dtype == MUZO_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == MUZO_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// Round an fp32 value to `dtype` and back (the value torch holds after `.to(dtype)`).
__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == MUZO_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == MUZO_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Two values rounded to bf16 and back through one packed conversion: the same round-to-nearest-
// even result as two bf16r calls, on the ALU pipe instead of one conversion each on the XU pipe.
__device__ __forceinline__ void bf16r2(float& a, float& b) {
  const uint32_t p = pack_bf16(a, b);
  a = bf16_lo(p);
  b = bf16_hi(p);
}

// Pairwise round_to.
__device__ __forceinline__ void round2_to(float& a, float& b, int dtype) {
  if (dtype == MUZO_BF16) {
    bf16r2(a, b);
  } else if (dtype == MUZO_F16) {
    const __half2 h = __floats2half2_rn(a, b);
    a = __low2float(h);
    b = __high2float(h);
  }
}

__device__ __forceinline__ float half_lo(uint32_t packed) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(packed & 0xffffu)));
}
__device__ __forceinline__ float half_hi(uint32_t packed) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(packed >> 16)));
}
__device__ __forceinline__ uint32_t pack_half(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Load 8 consecutive elements of `dtype` starting at element i (16-byte aligned for 16-bit types,
// 32-byte for fp32) into fp32 registers.
__device__ __forceinline__ void load8(const void* base, int64_t i, int dtype, float (&v)[8]) {
  if (dtype == MUZO_F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + i);
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (dtype == MUZO_BF16) { v[2 * q] = bf16_lo(w[q]); v[2 * q + 1] = bf16_hi(w[q]); }
      else { v[2 * q] = half_lo(w[q]); v[2 * q + 1] = half_hi(w[q]); }
    }
  }
}

// Store 8 fp32 values rounded to `dtype` at element i (same alignment rule as load8).
__device__ __forceinline__ void store8(void* base, int64_t i, int dtype, const float (&v)[8]) {
  if (dtype == MUZO_F32) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u;
    if (dtype == MUZO_BF16) {
      u.x = pack_bf16(v[0], v[1]); u.y = pack_bf16(v[2], v[3]);
      u.z = pack_bf16(v[4], v[5]); u.w = pack_bf16(v[6], v[7]);
    } else {
      u.x = pack_half(v[0], v[1]); u.y = pack_half(v[2], v[3]);
      u.z = pack_half(v[4], v[5]); u.w = pack_half(v[6], v[7]);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base) + i) = u;
  }
}

// ------------------------------------------------------------------ segment tables

// Locates the segment holding global work item `item`: binary search the first time, then a
// forward walk (items are visited in increasing order by every thread).
__device__ __forceinline__ int find_segment(const muzo_segment* segs, int nsegs, int64_t item) {
  int lo = 0, hi = nsegs - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (segs[mid].item_begin <= item) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ int advance_segment(const muzo_segment* segs, int nsegs, int cur,
                                               int64_t item) {
  while (cur + 1 < nsegs && segs[cur + 1].item_begin <= item) ++cur;
  return cur;
}

// Warp-level fp64 sum.
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kElemThreads = 256;  // block size of the element-wise kernels

// Grid of the persistent element-wise kernels: `per_sm` CTAs per SM, capped by the work.
inline int elem_grid(int64_t total_items, int per_sm) {
  int64_t want = (total_items + kElemThreads - 1) / kElemThreads;
  int64_t cap = static_cast<int64_t>(device_sm_count()) * per_sm;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return static_cast<int>(want);
}

}  // namespace muzo
