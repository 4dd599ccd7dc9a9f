// The decoder layers' RMSNorm and gated-MLP activation around the verify
// round's forwards (sm_100a, bf16).
//
// transformers' Qwen3RMSNorm / LlamaRMSNorm.forward is about eight small
// kernels per call (cast, square, mean, add, rsqrt, multiply, cast, weight);
// Qwen3MLP / LlamaMLP.forward runs the gate and up GEMMs, the SiLU and the
// product.  Both appear twice per decoder layer in every draft and verify
// forward of the reference's engine (specdec/engine.py:245-274 call the HF
// models), where launches, not bytes, set their cost.  Here each is one
// launch with transformers' bf16 arithmetic in the same order:
//   rmsnorm:  y = rn(w * rn(x * rsqrt(mean(x^2) + eps)))   (x^2 summed in f32)
//   silu_mul: y = rn(rn(g / (1 + exp(-g))) * u)
// The float32 sum of squares is reduced in another order than torch's, so a
// normalised value can land one bf16 ulp apart.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "specdec_b200.h"

namespace sd {

constexpr int NORM_THREADS = 256;

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One CTA per row of H elements; the row is read twice (the second time from
// L1 / L2).  Rows are `x_rs` / `out_rs` elements apart.
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(
    const __nv_bfloat16* x, int64_t x_rs, const __nv_bfloat16* __restrict__ w, float eps,
    __nv_bfloat16* out, int64_t out_rs, int H) {     // out may be x: each element has one owner
  __shared__ float red[NORM_THREADS / 32];
  const int64_t r = blockIdx.x;
  const __nv_bfloat16* xr = x + r * x_rs;
  __nv_bfloat16* yr = out + r * out_rs;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += NORM_THREADS) {
    const float v = __bfloat162float(xr[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    ss = lane < NORM_THREADS / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[0] = ss;
  }
  __syncthreads();
  const float rs = rsqrtf(__fdiv_rn(red[0], (float)H) + eps);
  for (int i = threadIdx.x; i < H; i += NORM_THREADS)
    yr[i] = __float2bfloat16_rn(__bfloat162float(w[i]) * bfr(__bfloat162float(xr[i]) * rs));
}

// The residual add fused in front of the norm (a decoder layer's
// "residual = residual + h; h = norm(residual)"):
//   s = rn(x + res) -> res_out,  out = rn(w * rn(s * rsqrt(mean(s^2) + eps)))
// The sum is kept in registers between the passes (up to ADD_NORM_PER
// elements per thread).
constexpr int ADD_NORM_PER = 32;
__global__ void __launch_bounds__(NORM_THREADS) add_rmsnorm_kernel(
    const __nv_bfloat16* x, int64_t x_rs, const __nv_bfloat16* res, int64_t res_rs,
    const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* out, int64_t out_rs,
    __nv_bfloat16* res_out, int64_t ro_rs, int H) {   // outputs may alias inputs: one owner each
  __shared__ float red[NORM_THREADS / 32];
  const int64_t r = blockIdx.x;
  float sv[ADD_NORM_PER];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < ADD_NORM_PER; ++k) {
    const int i = threadIdx.x + k * NORM_THREADS;
    sv[k] = 0.f;
    if (i < H) {
      sv[k] = bfr(__bfloat162float(x[r * x_rs + i]) + __bfloat162float(res[r * res_rs + i]));
      ss = fmaf(sv[k], sv[k], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    ss = lane < NORM_THREADS / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[0] = ss;
  }
  __syncthreads();
  const float rs = rsqrtf(__fdiv_rn(red[0], (float)H) + eps);
#pragma unroll
  for (int k = 0; k < ADD_NORM_PER; ++k) {
    const int i = threadIdx.x + k * NORM_THREADS;
    if (i < H) {
      res_out[r * ro_rs + i] = __float2bfloat16_rn(sv[k]);
      out[r * out_rs + i] = __float2bfloat16_rn(__bfloat162float(w[i]) * bfr(sv[k] * rs));
    }
  }
}

// Vector forms for the usual widths (H = 256 VPL, rows 16-byte aligned): one
// warp per row, the row in registers (VPL 16-byte units per lane, unit u of
// lane l at element 8 (l + 32 u)), one read, one warp reduction.  `res`
// non-null: the residual add first (res_out = rn(x + res)).
constexpr int NORM_ROWS_PER_CTA = 4;

__device__ __forceinline__ void bf8_to_f(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 v = __bfloat1622float2(h[e]);
    f[2 * e] = v.x;
    f[2 * e + 1] = v.y;
  }
}
__device__ __forceinline__ uint4 f_to_bf8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
  return u;
}

template <int VPL>
__global__ void __launch_bounds__(32 * NORM_ROWS_PER_CTA) rmsnorm_vec_kernel(
    const __nv_bfloat16* x, int64_t x_rs, const __nv_bfloat16* res, int64_t res_rs,
    const __nv_bfloat16* __restrict__ w, float eps, __nv_bfloat16* out, int64_t out_rs,
    __nv_bfloat16* res_out, int64_t ro_rs, int rows) {
  constexpr int H = 256 * VPL;
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * NORM_ROWS_PER_CTA + (threadIdx.x >> 5);
  if (r >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + r * x_rs);
  uint4 u[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) u[k] = xr[lane + 32 * k];
  if (res != nullptr) {
    const uint4* rr = reinterpret_cast<const uint4*>(res + r * res_rs);
    uint4* ro = reinterpret_cast<uint4*>(res_out + r * ro_rs);
    uint4 v[VPL];
#pragma unroll
    for (int k = 0; k < VPL; ++k) v[k] = rr[lane + 32 * k];
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      float a[8], c[8];
      bf8_to_f(u[k], a);
      bf8_to_f(v[k], c);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] += c[e];
      u[k] = f_to_bf8(a);                             // s = rn(x + res)
      ro[lane + 32 * k] = u[k];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    float a[8];
    bf8_to_f(u[k], a);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(a[e], a[e], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rs = rsqrtf(__fdiv_rn(ss, (float)H) + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(out + r * out_rs);
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    float a[8], g[8];
    bf8_to_f(u[k], a);
    bf8_to_f(__ldg(wr + lane + 32 * k), g);
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] = g[e] * bfr(a[e] * rs);
    yr[lane + 32 * k] = f_to_bf8(a);
  }
}

// The vector kernel for this width and alignment, else nullptr.
typedef void (*NormVecFn)(const __nv_bfloat16*, int64_t, const __nv_bfloat16*, int64_t,
                          const __nv_bfloat16*, float, __nv_bfloat16*, int64_t, __nv_bfloat16*,
                          int64_t, int);
static NormVecFn norm_vec_for(int H, const void* const* ptrs, int nptr, const int64_t* rs,
                              int nrs) {
  for (int i = 0; i < nptr; ++i)
    if (ptrs[i] && (reinterpret_cast<uintptr_t>(ptrs[i]) & 15)) return nullptr;
  for (int i = 0; i < nrs; ++i)
    if (rs[i] % 8) return nullptr;
  switch (H) {
    case 512: return rmsnorm_vec_kernel<2>;
    case 1024: return rmsnorm_vec_kernel<4>;
    case 2048: return rmsnorm_vec_kernel<8>;
    case 3072: return rmsnorm_vec_kernel<12>;
    case 4096: return rmsnorm_vec_kernel<16>;
    default: return nullptr;
  }
}

// out[r, i] = silu(gu[r, i]) * gu[r, I + i], one thread per output element
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int64_t gu_rs,
                                __nv_bfloat16* __restrict__ out, int64_t out_rs, int I,
                                int64_t total) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= total) return;
  const int64_t r = e / I;
  const int i = (int)(e - r * I);
  const float g = __bfloat162float(gu[r * gu_rs + i]);
  const float u = __bfloat162float(gu[r * gu_rs + I + i]);
  const float s = bfr(g / (1.0f + expf(-g)));
  out[r * out_rs + i] = __float2bfloat16_rn(s * u);
}

}  // namespace sd

extern "C" {

int sd_rmsnorm(const void* x, int64_t x_rs, const void* w, float eps, void* out, int64_t out_rs,
               int rows, int H, void* stream) {
  if (!x || !w || !out || rows < 0 || H <= 0) return SD_EINVAL;
  if (rows == 0) return SD_OK;
  {
    const void* ptrs[3] = {x, w, out};
    const int64_t rs[2] = {x_rs, out_rs};
    sd::NormVecFn f = sd::norm_vec_for(H, ptrs, 3, rs, 2);
    if (f) {
      const unsigned grid = (unsigned)((rows + sd::NORM_ROWS_PER_CTA - 1) / sd::NORM_ROWS_PER_CTA);
      f<<<grid, 32 * sd::NORM_ROWS_PER_CTA, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
          static_cast<const __nv_bfloat16*>(x), x_rs, nullptr, 0,
          static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(out), out_rs,
          nullptr, 0, rows);
      return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
    }
  }
  sd::rmsnorm_kernel<<<(unsigned)rows, sd::NORM_THREADS, 0,
                       reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), x_rs, static_cast<const __nv_bfloat16*>(w), eps,
      static_cast<__nv_bfloat16*>(out), out_rs, H);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

int sd_add_rmsnorm(const void* x, int64_t x_rs, const void* res, int64_t res_rs, const void* w,
                   float eps, void* out, int64_t out_rs, void* res_out, int64_t ro_rs, int rows,
                   int H, void* stream) {
  if (!x || !res || !w || !out || !res_out || rows < 0 || H <= 0) return SD_EINVAL;
  if (H > sd::ADD_NORM_PER * sd::NORM_THREADS) return SD_ENOTSUP;
  if (rows == 0) return SD_OK;
  {
    const void* ptrs[5] = {x, res, w, out, res_out};
    const int64_t rs[4] = {x_rs, res_rs, out_rs, ro_rs};
    sd::NormVecFn f = sd::norm_vec_for(H, ptrs, 5, rs, 4);
    if (f) {
      const unsigned grid = (unsigned)((rows + sd::NORM_ROWS_PER_CTA - 1) / sd::NORM_ROWS_PER_CTA);
      f<<<grid, 32 * sd::NORM_ROWS_PER_CTA, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
          static_cast<const __nv_bfloat16*>(x), x_rs, static_cast<const __nv_bfloat16*>(res),
          res_rs, static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(out),
          out_rs, static_cast<__nv_bfloat16*>(res_out), ro_rs, rows);
      return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
    }
  }
  sd::add_rmsnorm_kernel<<<(unsigned)rows, sd::NORM_THREADS, 0,
                           reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), x_rs, static_cast<const __nv_bfloat16*>(res), res_rs,
      static_cast<const __nv_bfloat16*>(w), eps, static_cast<__nv_bfloat16*>(out), out_rs,
      static_cast<__nv_bfloat16*>(res_out), ro_rs, H);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

int sd_silu_mul(const void* gu, int64_t gu_rs, void* out, int64_t out_rs, int rows, int I,
                void* stream) {
  if (!gu || !out || rows < 0 || I <= 0) return SD_EINVAL;
  const int64_t total = (int64_t)rows * I;
  if (total == 0) return SD_OK;
  const int64_t grid = (total + 255) / 256;
  if (grid > 0x7FFFFFFF) return SD_ENOTSUP;
  sd::silu_mul_kernel<<<(unsigned)grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gu), gu_rs, static_cast<__nv_bfloat16*>(out), out_rs, I,
      total);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

}  // extern "C"
