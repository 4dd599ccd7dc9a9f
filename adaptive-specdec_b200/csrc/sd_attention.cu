// Verify attention over the ragged KV cache (sm_100a).
//
// Reference: the HF Qwen3 attention at specdec/engine.py:274 reads
// _RaggedLayer.update's [B, Hkv, max_len+q, D] view (specdec/kvcache.py:61-74)
// with the additive mask s <= lengths[b] + j (and s < valid[b] during a
// right-padded prefill) from RaggedCache.attn_mask (kvcache.py:138-162).
// Here each row reads only its own live keys: row b, query j attends to cache
// slots [0, min(lengths[b] + j + 1, valid[b])).
//
// Work decomposition: one CTA per (row, kv head, key split).  The CTA holds the
// R = qlen * (Hq / Hkv) query rows that share the kv head (grouped-query), so
// every K/V element is read from HBM once per split.  Splits write partial
// (max, sum, acc) to the workspace; a combine kernel merges them.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "specdec_b200.h"

namespace sd {

constexpr int AT = 256;          // threads
constexpr int KT = 32;           // keys per tile
constexpr int RMAX = 64;         // query rows per CTA (qlen * group)
constexpr int DMAX = 128;        // head dim supported by this kernel
constexpr int SPLIT_KEYS = 1024; // keys per split

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16(x);
}

struct AttnParams {
  const void* q; int64_t qbs, qhs, qqs;
  const void* k; const void* v;
  const int64_t* lengths; const int64_t* valid;
  int B, Hq, Hkv, D, C, qlen, group, R, nsplit, nrc;
  float scale;
  void* out; int64_t obs, oqs, ohs;
  float* part_acc;   // [B, Hkv, nsplit, R, D]
  float* part_ml;    // [B, Hkv, nsplit, R, 2]
};

__device__ __forceinline__ int row_limit(const AttnParams& P, int b, int j) {
  int64_t lim = P.lengths[b] + j + 1;
  if (P.valid && P.valid[b] < lim) lim = P.valid[b];
  if (lim > P.C) lim = P.C;
  return lim > 0 ? (int)lim : 0;
}

template <typename T>
struct AttnSmem {
  T qs[RMAX][DMAX + 2];
  T ks[KT][DMAX + 2];
  T vs[KT][DMAX];
  float ps[RMAX][KT + 1];
  float m_s[RMAX], l_s[RMAX], a_s[RMAX];
  int lim_s[RMAX];
};

template <typename T>
__global__ void __launch_bounds__(AT) attn_split_kernel(AttnParams P) {
  extern __shared__ __align__(16) unsigned char attn_smem[];
  AttnSmem<T>& S = *reinterpret_cast<AttnSmem<T>*>(attn_smem);
  auto& qs = S.qs; auto& ks = S.ks; auto& vs = S.vs; auto& ps = S.ps;
  auto& m_s = S.m_s; auto& l_s = S.l_s; auto& a_s = S.a_s; auto& lim_s = S.lim_s;
  const T* Q = reinterpret_cast<const T*>(P.q);
  const int split = blockIdx.x % P.nsplit;
  const int rc = (blockIdx.x / P.nsplit) % P.nrc;
  const int bh = blockIdx.x / (P.nsplit * P.nrc);
  const int h = bh % P.Hkv, b = bh / P.Hkv;
  const int t = threadIdx.x, D = P.D;
  const int r0 = rc * RMAX, R = min(RMAX, P.R - r0);
  // local row r <-> global row r0 + r = j * group + g  (query j, head h*group+g)
  int kmax = 0;
  for (int r = 0; r < R; ++r) kmax = max(kmax, row_limit(P, b, (r0 + r) / P.group));
  const int s0 = split * SPLIT_KEYS, s1 = min(kmax, s0 + SPLIT_KEYS);
  for (int i = t; i < R * D; i += AT) {
    const int r = i / D, d = i % D;
    const int j = (r0 + r) / P.group, hq = h * P.group + (r0 + r) % P.group;
    qs[r][d] = Q[b * P.qbs + hq * P.qhs + j * P.qqs + d];
  }
  for (int r = t; r < RMAX; r += AT) {
    m_s[r] = -INFINITY;
    l_s[r] = 0.f;
    lim_s[r] = r < R ? row_limit(P, b, (r0 + r) / P.group) : 0;
  }
  // accumulators: thread owns (r, d) pairs i = t, t+AT, ...
  constexpr int NA = RMAX * DMAX / AT;
  float acc[NA];
#pragma unroll
  for (int i = 0; i < NA; ++i) acc[i] = 0.f;
  __syncthreads();
  const T* kb = reinterpret_cast<const T*>(P.k) + ((int64_t)b * P.Hkv + h) * P.C * D;
  const T* vb = reinterpret_cast<const T*>(P.v) + ((int64_t)b * P.Hkv + h) * P.C * D;
  for (int kt = s0; kt < s1; kt += KT) {
    const int nk = min(KT, s1 - kt);
    for (int i = t; i < KT * D; i += AT) {
      const int kk = i / D, d = i % D;
      const bool in = kk < nk;
      ks[kk][d] = in ? kb[(int64_t)(kt + kk) * D + d] : from_f<T>(0.f);
      vs[kk][d] = in ? vb[(int64_t)(kt + kk) * D + d] : from_f<T>(0.f);
    }
    __syncthreads();
    for (int i = t; i < R * KT; i += AT) {
      const int r = i / KT, kk = i % KT;
      float sc = -INFINITY;
      if (kk < nk && kt + kk < lim_s[r]) {
        float a = 0.f;
        for (int d = 0; d < D; ++d)
          a = fmaf(to_f<T>(qs[r][d]), to_f<T>(ks[kk][d]), a);
        sc = a * P.scale;
      }
      ps[r][kk] = sc;
    }
    __syncthreads();
    // online softmax per row (one warp per row, rows strided over warps)
    const int lane = t & 31, w = t >> 5;
    for (int r = w; r < R; r += AT / 32) {
      const float sc = ps[r][lane];
      float mx = sc;
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = m_s[r];
      const float mnew = fmaxf(mold, mx);
      const float p = (sc == -INFINITY) ? 0.f : __expf(sc - mnew);
      float sum = p;
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      ps[r][lane] = p;
      if (lane == 0) {
        const float alpha = (mold == -INFINITY) ? 0.f : __expf(mold - mnew);
        a_s[r] = (mnew == -INFINITY) ? 1.f : alpha;
        l_s[r] = l_s[r] * a_s[r] + sum;
        m_s[r] = mnew;
      }
    }
    __syncthreads();
#pragma unroll
    for (int ii = 0; ii < NA; ++ii) {
      const int i = t + ii * AT;
      const int r = i / D, d = i % D;
      if (r < R) {
        float a = acc[ii] * a_s[r];
        for (int kk = 0; kk < nk; ++kk) a = fmaf(ps[r][kk], to_f<T>(vs[kk][d]), a);
        acc[ii] = a;
      }
    }
    __syncthreads();
  }
  const int64_t pbase = (((int64_t)b * P.Hkv + h) * P.nsplit + split) * P.R + r0;
#pragma unroll
  for (int ii = 0; ii < NA; ++ii) {
    const int i = t + ii * AT;
    const int r = i / D, d = i % D;
    if (r < R) P.part_acc[(pbase + r) * D + d] = acc[ii];
  }
  for (int r = t; r < R; r += AT) {
    P.part_ml[(pbase + r) * 2 + 0] = m_s[r];
    P.part_ml[(pbase + r) * 2 + 1] = l_s[r];
  }
}

template <typename T>
__global__ void __launch_bounds__(AT) attn_combine_kernel(AttnParams P) {
  const int bh = blockIdx.x;
  const int h = bh % P.Hkv, b = bh / P.Hkv;
  const int D = P.D, R = P.R;
  for (int i = threadIdx.x; i < R * D; i += AT) {
    const int r = i / D, d = i % D;
    const int64_t base = ((int64_t)b * P.Hkv + h) * P.nsplit * R;
    float m = -INFINITY;
    for (int s = 0; s < P.nsplit; ++s) m = fmaxf(m, P.part_ml[(base + (int64_t)s * R + r) * 2]);
    float l = 0.f, a = 0.f;
    if (m != -INFINITY) {
      for (int s = 0; s < P.nsplit; ++s) {
        const int64_t o = base + (int64_t)s * R + r;
        const float ms = P.part_ml[o * 2];
        if (ms == -INFINITY) continue;
        const float w = __expf(ms - m);
        l += w * P.part_ml[o * 2 + 1];
        a += w * P.part_acc[o * D + d];
      }
    }
    const int j = r / P.group, hq = h * P.group + r % P.group;
    const float y = l > 0.f ? a / l : 0.f;
    reinterpret_cast<T*>(P.out)[b * P.obs + j * P.oqs + hq * P.ohs + d] = from_f<T>(y);
  }
}

static int nsplit_for(int C, int qlen) {
  const int maxkeys = C + qlen;
  return (maxkeys + SPLIT_KEYS - 1) / SPLIT_KEYS;
}

}  // namespace sd

using namespace sd;

extern "C" {

size_t sd_verify_attn_workspace_bytes(int B, int Hq, int Hkv, int D, int C, int qlen) {
  if (B <= 0 || Hkv <= 0 || Hq % Hkv) return 0;
  const int R = qlen * (Hq / Hkv);
  const size_t ns = (size_t)nsplit_for(C, qlen);
  return (size_t)B * Hkv * ns * R * (D + 2) * sizeof(float) + 256;
}

int sd_verify_attn(const void* q, int64_t qbs, int64_t qhs, int64_t qqs, const void* kcache,
                   const void* vcache, const int64_t* lengths, const int64_t* valid, int B, int Hq,
                   int Hkv, int D, int C, int qlen, float scale, void* out, int64_t obs,
                   int64_t oqs, int64_t ohs, int dtype, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (dtype != SD_DTYPE_BF16 && dtype != SD_DTYPE_F32) return SD_ENOTSUP;
  if (!q || !kcache || !vcache || !lengths || !out) return SD_EINVAL;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || qlen <= 0 || C <= 0) return SD_EINVAL;
  if (D > DMAX || D % 2) return SD_ENOTSUP;
  if (workspace_bytes < sd_verify_attn_workspace_bytes(B, Hq, Hkv, D, C, qlen) || !workspace)
    return SD_ENOSPC;
  AttnParams P;
  P.q = q; P.qbs = qbs; P.qhs = qhs; P.qqs = qqs;
  P.k = kcache;
  P.v = vcache;
  P.lengths = lengths; P.valid = valid;
  P.B = B; P.Hq = Hq; P.Hkv = Hkv; P.D = D; P.C = C; P.qlen = qlen; P.group = Hq / Hkv;
  P.R = qlen * P.group; P.nsplit = nsplit_for(C, qlen); P.scale = scale;
  P.nrc = (P.R + RMAX - 1) / RMAX;
  P.out = out; P.obs = obs; P.oqs = oqs; P.ohs = ohs;
  float* ws = reinterpret_cast<float*>(workspace);
  P.part_acc = ws;
  P.part_ml = ws + (size_t)B * Hkv * P.nsplit * P.R * D;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)(B * Hkv * P.nrc * P.nsplit);
  if (dtype == SD_DTYPE_BF16) {
    const size_t sm = sizeof(AttnSmem<__nv_bfloat16>);
    cudaFuncSetAttribute(attn_split_kernel<__nv_bfloat16>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    attn_split_kernel<__nv_bfloat16><<<grid, AT, sm, st>>>(P);
    attn_combine_kernel<__nv_bfloat16><<<B * Hkv, AT, 0, st>>>(P);
  } else {
    const size_t sm = sizeof(AttnSmem<float>);
    cudaFuncSetAttribute(attn_split_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sm);
    attn_split_kernel<float><<<grid, AT, sm, st>>>(P);
    attn_combine_kernel<float><<<B * Hkv, AT, 0, st>>>(P);
  }
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

}  // extern "C"
