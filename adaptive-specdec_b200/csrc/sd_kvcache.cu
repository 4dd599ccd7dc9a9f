// Ragged KV cache bookkeeping on the device (sm_100a).
//
// Reference: specdec/kvcache.py.  There the per-row lengths live on the CPU
// and are mirrored to the GPU after every advance / rollback (kvcache.py:
// 165-190), and _RaggedLayer.update scatters the new K/V rows at
// lengths[b] + j (kvcache.py:61-74).  Here the lengths are device-resident:
// advance, rollback and the verify-round commit are one tiny kernel each (O(1)
// per row, no data movement, no host synchronisation), and the append writes
// each row's new tokens at its own offset with 16-byte copies.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "specdec_b200.h"

namespace sd {

// Where a layer's K / V rows live: the contiguous [B, H, C, D] cache
// (bt == nullptr) or a pool of pages [npages, H, SD_KV_PAGE, D] with row b's
// slot s in page bt[b * bt_stride + s / SD_KV_PAGE] (-1: no page assigned).
struct KvLayout {
  const int32_t* bt;
  int bt_stride, npages;
};

// Row index (in rows of D elements) of slot s of row b, head h; -1 when a
// paged row has no page there (the write is skipped and *err gets bit 1).
__device__ __forceinline__ int64_t kv_slot(const KvLayout& lay, int b, int h, int H, int C,
                                           int64_t s) {
  if (lay.bt == nullptr) return ((int64_t)b * H + h) * C + s;
  const int pg = lay.bt[(int64_t)b * lay.bt_stride + (s / SD_KV_PAGE)];
  if (pg < 0 || pg >= lay.npages) return -1;
  return ((int64_t)pg * H + h) * SD_KV_PAGE + (s % SD_KV_PAGE);
}

// ---- fused post-projection step of an attention layer ------------------------
// Per (row b, position l, head) vector of D elements, one warp: the head's
// RMSNorm (q and k, when a weight is given), the rotary embedding with that
// position's (cos, sin) (q and k), then q to q_out [B, Hq, L, D] and k, v
// into the ragged cache at slot lengths[b] + l.  It does in one launch what
// transformers' Qwen3Attention.forward does between the projections and the
// attention (modeling_qwen3.py: q_norm / k_norm, apply_rotary_pos_emb, and the
// cache update, specdec/kvcache.py:61-74 in the reference), with the same
// bf16 tensor arithmetic: the sum of squares in float32 (in a warp reduction
// order, where torch's differs: a normalised value can land one bf16 ulp
// apart), x * rsqrt(mean + eps) in float32 rounded to bf16, times the weight
// rounded to bf16; rope = rn(rn(x * cos) + rn(rotate_half(x) * sin)).
struct QkvArgs {
  const __nv_bfloat16* q; int64_t q_rs;      // [B * L rows, Hq * D], row stride
  const __nv_bfloat16* k; int64_t k_rs;      // [B * L rows, Hkv * D]
  const __nv_bfloat16* v; int64_t v_rs;
  const __nv_bfloat16* qw;                   // [D] or null: no norm
  const __nv_bfloat16* kw;
  float eps;
  const __nv_bfloat16* cos; const __nv_bfloat16* sin;   // [B, L, D], strides (cs_bs, cs_ls, 1)
  int64_t cs_bs, cs_ls;
  __nv_bfloat16* kc; __nv_bfloat16* vc;      // [B, Hkv, C, D]
  const int64_t* lengths;
  __nv_bfloat16* q_out;                      // [B, Hq, L, D]
  int B, L, Hq, Hkv, D, C;
  int* err;
  KvLayout lay;
};

constexpr int QKV_WARPS = 8;
constexpr int QKV_DMAX = 256;

__device__ __forceinline__ float bf16_rn(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__global__ void __launch_bounds__(QKV_WARPS * 32) qkv_rope_append_kernel(QkvArgs a) {
  __shared__ float buf[QKV_WARPS][QKV_DMAX];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  const int nh = a.Hq + 2 * a.Hkv;
  const int64_t w = (int64_t)blockIdx.x * QKV_WARPS + wl;
  if (w >= (int64_t)a.B * a.L * nh) return;
  const int hv = (int)(w % nh);
  const int64_t r = w / nh;                  // b * L + l
  const int l = (int)(r % a.L), b = (int)(r / a.L);
  const int D = a.D;
  const __nv_bfloat16* src;
  const __nv_bfloat16* nw = nullptr;
  __nv_bfloat16* dst;
  bool rope = true;
  if (hv < a.Hq) {
    src = a.q + r * a.q_rs + (int64_t)hv * D;
    nw = a.qw;
    dst = a.q_out + (((int64_t)b * a.Hq + hv) * a.L + l) * D;
  } else {
    const int64_t len = a.lengths[b];
    if (len < 0 || len + a.L > a.C) {        // the row's slots would pass the capacity
      if (lane == 0 && l == 0 && hv == a.Hq && a.err) atomicOr(a.err, 1);
      return;
    }
    const int h = hv < a.Hq + a.Hkv ? hv - a.Hq : hv - a.Hq - a.Hkv;
    const int64_t row = kv_slot(a.lay, b, h, a.Hkv, a.C, len + l);
    if (row < 0) {
      if (lane == 0 && a.err) atomicOr(a.err, 2);
      return;
    }
    const int64_t slot = row * D;
    if (hv < a.Hq + a.Hkv) {
      src = a.k + r * a.k_rs + (int64_t)h * D;
      nw = a.kw;
      dst = a.kc + slot;
    } else {
      src = a.v + r * a.v_rs + (int64_t)h * D;
      rope = false;
      dst = a.vc + slot;
    }
  }
  float* x = buf[wl];
  float ss = 0.f;
  for (int i = lane; i < D; i += 32) {
    const float xv = __bfloat162float(src[i]);
    x[i] = xv;
    ss = fmaf(xv, xv, ss);
  }
  if (nw != nullptr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rs = rsqrtf(__fdiv_rn(ss, (float)D) + a.eps);
    for (int i = lane; i < D; i += 32)
      x[i] = bf16_rn(__bfloat162float(nw[i]) * bf16_rn(x[i] * rs));
  }
  __syncwarp();
  const int half = D >> 1;
  const __nv_bfloat16* cp = a.cos + (int64_t)b * a.cs_bs + (int64_t)l * a.cs_ls;
  const __nv_bfloat16* sp = a.sin + (int64_t)b * a.cs_bs + (int64_t)l * a.cs_ls;
  for (int i = lane; i < D; i += 32) {
    float o = x[i];
    if (rope) {
      const float rot = i < half ? -x[i + half] : x[i - half];
      o = bf16_rn(bf16_rn(x[i] * __bfloat162float(cp[i])) + bf16_rn(rot * __bfloat162float(sp[i])));
    }
    dst[i] = __float2bfloat16_rn(o);
  }
}

__global__ void lengths_update_kernel(int64_t* lengths, const int64_t* delta, int64_t q, int sign,
                                      int B, int64_t capacity, int* err) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t d = delta ? delta[b] : q;
  const int64_t nl = lengths[b] + (sign >= 0 ? d : -d);
  if (nl < 0 || nl > capacity) {
    if (err) atomicOr(err, 1);
    return;
  }
  lengths[b] = nl;
}

__global__ void commit_kernel(int64_t* lengths, const int64_t* n_acc, int k, int B, int* err) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t a = n_acc[b];
  const int64_t nl = lengths[b] - ((int64_t)k - a);
  if (a < 0 || a > k || nl < 0) {
    if (err) atomicOr(err, 1);
    return;
  }
  lengths[b] = nl;
}

// One thread per 16-byte unit of one (b, h, j) row; `upr` units per row.
__global__ void append_vec_kernel(uint4* __restrict__ kc, uint4* __restrict__ vc,
                                  const char* __restrict__ nk, const char* __restrict__ nv,
                                  int64_t nbs, int64_t nhs, int64_t nqs, int esz,
                                  const int64_t* __restrict__ lengths, int B, int H, int C, int q,
                                  int upr, int64_t total, int* err, KvLayout lay) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int u = (int)(i % upr);
  int64_t r = i / upr;
  const int j = (int)(r % q); r /= q;
  const int h = (int)(r % H);
  const int b = (int)(r / H);
  const int64_t L = lengths[b];
  if (L < 0 || L + q > C) {
    if (u == 0 && j == 0 && h == 0 && err) atomicOr(err, 1);
    return;
  }
  const int64_t row = kv_slot(lay, b, h, H, C, L + j);
  if (row < 0) {
    if (u == 0 && err) atomicOr(err, 2);
    return;
  }
  const int64_t src = (b * nbs + h * nhs + j * nqs) * esz;        // bytes
  const int64_t dst = row * upr;                                   // uint4 units
  kc[dst + u] = *reinterpret_cast<const uint4*>(nk + src + 16 * (int64_t)u);
  vc[dst + u] = *reinterpret_cast<const uint4*>(nv + src + 16 * (int64_t)u);
}

// Element-wise fallback for rows that are not 16-byte aligned.
__global__ void append_elem_kernel(char* kc, char* vc, const char* nk, const char* nv, int64_t nbs,
                                   int64_t nhs, int64_t nqs, int esz, const int64_t* lengths, int B,
                                   int H, int C, int D, int q, int64_t total, int* err,
                                   KvLayout lay) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % D);
  int64_t r = i / D;
  const int j = (int)(r % q); r /= q;
  const int h = (int)(r % H);
  const int b = (int)(r / H);
  const int64_t L = lengths[b];
  if (L < 0 || L + q > C) {
    if (d == 0 && j == 0 && h == 0 && err) atomicOr(err, 1);
    return;
  }
  const int64_t row = kv_slot(lay, b, h, H, C, L + j);
  if (row < 0) {
    if (d == 0 && err) atomicOr(err, 2);
    return;
  }
  const int64_t src = (b * nbs + h * nhs + j * nqs + d) * esz;
  const int64_t dst = (row * D + d) * esz;
  for (int e = 0; e < esz; ++e) {
    kc[dst + e] = nk[src + e];
    vc[dst + e] = nv[src + e];
  }
}

}  // namespace sd

using namespace sd;

extern "C" {

int sd_kv_lengths_update(int64_t* lengths, const int64_t* delta, int64_t q, int sign, int B,
                         int64_t capacity, int* err, void* stream) {
  if (!lengths || B < 0 || capacity < 0) return SD_EINVAL;
  if (B == 0) return SD_OK;
  lengths_update_kernel<<<(B + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      lengths, delta, q, sign, B, capacity, err);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

int sd_kv_commit(int64_t* lengths, const int64_t* n_acc, int k, int B, int* err, void* stream) {
  if (!lengths || !n_acc || B < 0 || k < 0) return SD_EINVAL;
  if (B == 0) return SD_OK;
  commit_kernel<<<(B + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      lengths, n_acc, k, B, err);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

int sd_qkv_norm_rope_append(const void* q, int64_t q_rs, const void* k, int64_t k_rs,
                            const void* v, int64_t v_rs, const void* q_norm_w,
                            const void* k_norm_w, float eps, const void* cos, const void* sin,
                            int64_t cs_bs, int64_t cs_ls, void* kcache, void* vcache,
                            const int32_t* block_table, int bt_stride, int npages,
                            const int64_t* lengths, int B, int L, int Hq, int Hkv, int D, int C,
                            void* q_out, int* err, void* stream) {
  if (!q || !k || !v || !cos || !sin || !kcache || !vcache || !lengths || !q_out) return SD_EINVAL;
  if (block_table && (bt_stride <= 0 || npages <= 0 || (int64_t)bt_stride * SD_KV_PAGE < C))
    return SD_EINVAL;
  if (B < 0 || L < 0 || Hq <= 0 || Hkv <= 0 || C <= 0 || D <= 0) return SD_EINVAL;
  if (D % 2 || D > sd::QKV_DMAX) return SD_ENOTSUP;
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr)) return SD_EINVAL;
  if (B == 0 || L == 0) return SD_OK;
  sd::QkvArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q); a.q_rs = q_rs;
  a.k = static_cast<const __nv_bfloat16*>(k); a.k_rs = k_rs;
  a.v = static_cast<const __nv_bfloat16*>(v); a.v_rs = v_rs;
  a.qw = static_cast<const __nv_bfloat16*>(q_norm_w);
  a.kw = static_cast<const __nv_bfloat16*>(k_norm_w);
  a.eps = eps;
  a.cos = static_cast<const __nv_bfloat16*>(cos); a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.cs_bs = cs_bs; a.cs_ls = cs_ls;
  a.kc = static_cast<__nv_bfloat16*>(kcache); a.vc = static_cast<__nv_bfloat16*>(vcache);
  a.lengths = lengths;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.B = B; a.L = L; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.C = C;
  a.err = err;
  a.lay = sd::KvLayout{block_table, bt_stride, npages};
  const int64_t nwarp = (int64_t)B * L * (Hq + 2 * Hkv);
  const int64_t grid = (nwarp + sd::QKV_WARPS - 1) / sd::QKV_WARPS;
  if (grid > 0x7FFFFFFF) return SD_ENOTSUP;
  sd::qkv_rope_append_kernel<<<(unsigned)grid, sd::QKV_WARPS * 32, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

}  // extern "C"

namespace sd {
static int kv_append(void* kcache, void* vcache, const void* new_k, const void* new_v, int64_t nbs,
                     int64_t nhs, int64_t nqs, const int64_t* lengths, int B, int H, int C, int D,
                     int q, int dtype, int* err, KvLayout lay, void* stream) {
  if (!kcache || !vcache || !new_k || !new_v || !lengths) return SD_EINVAL;
  if (B < 0 || H <= 0 || C <= 0 || D <= 0 || q < 0) return SD_EINVAL;
  if (dtype != SD_DTYPE_F32 && dtype != SD_DTYPE_F16 && dtype != SD_DTYPE_BF16) return SD_EINVAL;
  if (B == 0 || q == 0) return SD_OK;
  const int esz = dtype == SD_DTYPE_F32 ? 4 : 2;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = (D * esz) % 16 == 0 && ((nbs * esz) % 16 == 0) && ((nhs * esz) % 16 == 0) &&
                   ((nqs * esz) % 16 == 0) &&
                   ((reinterpret_cast<uintptr_t>(new_k) | reinterpret_cast<uintptr_t>(new_v) |
                     reinterpret_cast<uintptr_t>(kcache) | reinterpret_cast<uintptr_t>(vcache)) %
                    16) == 0;
  if (vec) {
    const int upr = D * esz / 16;
    const int64_t total = (int64_t)B * H * q * upr;
    append_vec_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<uint4*>(kcache), reinterpret_cast<uint4*>(vcache),
        reinterpret_cast<const char*>(new_k), reinterpret_cast<const char*>(new_v), nbs, nhs, nqs,
        esz, lengths, B, H, C, q, upr, total, err, lay);
  } else {
    const int64_t total = (int64_t)B * H * q * D;
    append_elem_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<char*>(kcache), reinterpret_cast<char*>(vcache),
        reinterpret_cast<const char*>(new_k), reinterpret_cast<const char*>(new_v), nbs, nhs, nqs,
        esz, lengths, B, H, C, D, q, total, err, lay);
  }
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}
}  // namespace sd

extern "C" {

int sd_kv_append(void* kcache, void* vcache, const void* new_k, const void* new_v, int64_t nbs,
                 int64_t nhs, int64_t nqs, const int64_t* lengths, int B, int H, int C, int D,
                 int q, int dtype, int* err, void* stream) {
  return sd::kv_append(kcache, vcache, new_k, new_v, nbs, nhs, nqs, lengths, B, H, C, D, q, dtype,
                       err, sd::KvLayout{nullptr, 0, 0}, stream);
}

int sd_kv_append_paged(void* kpool, void* vpool, const void* new_k, const void* new_v,
                       int64_t nbs, int64_t nhs, int64_t nqs, const int32_t* block_table,
                       int bt_stride, int npages, const int64_t* lengths, int B, int H, int D,
                       int q, int dtype, int* err, void* stream) {
  if (!block_table || bt_stride <= 0 || npages <= 0) return SD_EINVAL;
  if ((int64_t)bt_stride * SD_KV_PAGE > 0x7FFFFFFF) return SD_ENOTSUP;
  return sd::kv_append(kpool, vpool, new_k, new_v, nbs, nhs, nqs, lengths, B, H,
                       bt_stride * SD_KV_PAGE, D, q, dtype, err,
                       sd::KvLayout{block_table, bt_stride, npages}, stream);
}

}  // extern "C"
