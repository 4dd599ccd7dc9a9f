// Shared device helpers for the verify-round kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "specdec_b200.h"

namespace sd {

// ---------------------------------------------------------------------------
// dtype handling
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bits16_to_float(uint32_t b, int dtype) {
  if (dtype == SD_DTYPE_BF16) return __uint_as_float(b << 16);
  return __half2float(__ushort_as_half((unsigned short)b));
}

__device__ __forceinline__ float load_logit(const void* base, int dtype, int64_t idx) {
  if (dtype == SD_DTYPE_F32) return __ldg(reinterpret_cast<const float*>(base) + idx);
  uint32_t b = __ldg(reinterpret_cast<const unsigned short*>(base) + idx);
  return bits16_to_float(b, dtype);
}

// Order-preserving 32-bit key of a float; -0 and +0 share the key of +0 so that
// equal values always form one tie class.
__device__ __forceinline__ uint32_t fkey(float f) {
  uint32_t b = __float_as_uint(f);
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Order-preserving 16-bit key of a bf16 / fp16 bit pattern, and its inverse.
__device__ __forceinline__ uint32_t key16(uint32_t raw) {
  return (raw & 0x8000u) ? (~raw & 0xFFFFu) : (raw | 0x8000u);
}
__device__ __forceinline__ uint32_t raw16(uint32_t key) {
  return (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
}

// ---------------------------------------------------------------------------
// arithmetic contract shared with the oracle:
//   d = fl(x / T), e = expf(fl(d - m)), p = fl(e * inv_s), p' = fl(p / zf)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float scaled_logit(float x, float T) { return __fdiv_rn(x, T); }
__device__ __forceinline__ float softmax_num(float x, float T, float m) {
  return expf(__fsub_rn(scaled_logit(x, T), m));
}
__device__ __forceinline__ float prob_of(float x, float T, float m, float inv_s) {
  return __fmul_rn(softmax_num(x, T, m), inv_s);
}

// ---------------------------------------------------------------------------
// block-wide reductions / scans (blockDim.x multiple of 32, <= 1024)
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    T w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_min(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    T w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w < v ? w : v;
  }
  return v;
}

// Inclusive warp scan.
template <typename T>
__device__ __forceinline__ T warp_incl_scan(T v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T w = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += w;
  }
  return v;
}

// All threads get the block total.  `red` needs blockDim.x/32 slots.
template <typename T>
__device__ __forceinline__ T block_sum(T v, T* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  T t = lane < nw ? red[lane] : T(0);
  return warp_sum(t);
}

template <typename T>
__device__ __forceinline__ T block_max(T v, T* red, T lowest) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  T t = lane < nw ? red[lane] : lowest;
  return warp_max(t);
}

template <typename T>
__device__ __forceinline__ T block_min(T v, T* red, T highest) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_min(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  T t = lane < nw ? red[lane] : highest;
  return warp_min(t);
}

// Exclusive scan across the block in thread order; returns this thread's
// exclusive prefix and writes the block total to *total.
template <typename T>
__device__ __forceinline__ T block_excl_scan(T v, T* red, T* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  T inc = warp_incl_scan(v);
  __syncthreads();
  if (lane == 31) red[wid] = inc;
  __syncthreads();
  if (wid == 0) {
    T w = lane < nw ? red[lane] : T(0);
    T wi = warp_incl_scan(w);
    if (lane < nw) red[lane] = wi - w;     // exclusive warp offsets
    if (lane == nw - 1) red[32] = wi;      // total
  }
  __syncthreads();
  *total = red[32];
  return red[wid] + inc - v;
}

}  // namespace sd
