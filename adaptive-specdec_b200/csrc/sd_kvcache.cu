// Ragged KV cache bookkeeping on the device (sm_100a).
//
// Reference: specdec/kvcache.py.  There the per-row lengths live on the CPU
// and are mirrored to the GPU after every advance / rollback (kvcache.py:
// 165-190), and _RaggedLayer.update scatters the new K/V rows at
// lengths[b] + j (kvcache.py:61-74).  Here the lengths are device-resident:
// advance, rollback and the verify-round commit are one tiny kernel each (O(1)
// per row, no data movement, no host synchronisation), and the append writes
// each row's new tokens at its own offset with 16-byte copies.
#include <cuda_runtime.h>
#include <stdint.h>

#include "specdec_b200.h"

namespace sd {

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
                                  int upr, int64_t total, int* err) {
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
  const int64_t src = (b * nbs + h * nhs + j * nqs) * esz;        // bytes
  const int64_t dst = (((int64_t)b * H + h) * C + (L + j)) * upr;  // uint4 units
  kc[dst + u] = *reinterpret_cast<const uint4*>(nk + src + 16 * (int64_t)u);
  vc[dst + u] = *reinterpret_cast<const uint4*>(nv + src + 16 * (int64_t)u);
}

// Element-wise fallback for rows that are not 16-byte aligned.
__global__ void append_elem_kernel(char* kc, char* vc, const char* nk, const char* nv, int64_t nbs,
                                   int64_t nhs, int64_t nqs, int esz, const int64_t* lengths, int B,
                                   int H, int C, int D, int q, int64_t total, int* err) {
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
  const int64_t src = (b * nbs + h * nhs + j * nqs + d) * esz;
  const int64_t dst = ((((int64_t)b * H + h) * C + (L + j)) * D + d) * esz;
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

int sd_kv_append(void* kcache, void* vcache, const void* new_k, const void* new_v, int64_t nbs,
                 int64_t nhs, int64_t nqs, const int64_t* lengths, int B, int H, int C, int D,
                 int q, int dtype, int* err, void* stream) {
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
        esz, lengths, B, H, C, q, upr, total, err);
  } else {
    const int64_t total = (int64_t)B * H * q * D;
    append_elem_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<char*>(kcache), reinterpret_cast<char*>(vcache),
        reinterpret_cast<const char*>(new_k), reinterpret_cast<const char*>(new_v), nbs, nhs, nqs,
        esz, lengths, B, H, C, D, q, total, err);
  }
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

}  // extern "C"
