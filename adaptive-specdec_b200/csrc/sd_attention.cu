// Verify attention over the ragged KV cache (sm_100a).
//
// Reference: the HF Qwen3 attention at specdec/engine.py:274 reads
// _RaggedLayer.update's [B, Hkv, max_len+q, D] view (specdec/kvcache.py:61-74)
// with the additive mask s <= lengths[b] + j (and s < valid[b] during a
// right-padded prefill) from RaggedCache.attn_mask (kvcache.py:138-162).
// Here each row reads only its own live keys: row b, query j attends to cache
// slots [0, min(lengths[b] + j + 1, valid[b])).
//
// A CTA holds the R = qlen * (Hq / Hkv) query rows that share a kv head
// (grouped-query), so every live K/V element is read from HBM once.  bf16 with
// head_dim 128 runs on the tensor cores (attn_plan_kernel + the persistent
// attn_mma_kernel, which merges its own partials); other shapes and fp32 run
// on the CUDA cores (attn_split_kernel, one CTA per (row, kv head, key
// split), then attn_combine_kernel).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>

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
  int* split_done;   // [B, Hkv] pieces finished (tensor-core path; zeroed per call)
  int* rowpre;       // [B + 1] exclusive prefix of 64-key tiles per row (tensor-core path)
  int* rowkmax;      // [B] live-key bound of each row (tensor-core path)
  int npiece;        // partial slots per (row, kv head) on the tensor-core path
  int out_vec4;      // out is 8-byte aligned and its strides are multiples of 4 elements
  int tile_keys;     // keys per tile of the tensor-core schedule (plan kernel)
  int seg_ovh;       // schedule cost of a (row, kv head) beyond its tiles, in tiles
  int* status;       // sticky: bit 0 = a bounded wait of the tcgen05 kernel gave up
  // paged caches: k / v are pools [npages, Hkv, SD_KV_PAGE, D] and row b's key
  // s sits in page bt[b * bt_stride + s / SD_KV_PAGE]; bt == nullptr: the
  // contiguous [B, Hkv, C, D] layout
  const int32_t* bt;
  int bt_stride, npages;
};

// Offset, in rows of D elements, of key s of row b and kv head h.  A page
// index outside the pool reads page 0 (the caller's block table is wrong, but
// nothing is read out of bounds).
__device__ __forceinline__ int64_t kv_row(const AttnParams& P, int b, int h, int s) {
  if (P.bt == nullptr) return ((int64_t)b * P.Hkv + h) * P.C + s;
  int pg = __ldg(P.bt + (int64_t)b * P.bt_stride + (s / SD_KV_PAGE));
  if ((unsigned)pg >= (unsigned)P.npages) pg = 0;
  return ((int64_t)pg * P.Hkv + h) * SD_KV_PAGE + (s % SD_KV_PAGE);
}

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
  const T* kb = reinterpret_cast<const T*>(P.k);
  const T* vb = reinterpret_cast<const T*>(P.v);
  for (int kt = s0; kt < s1; kt += KT) {
    const int nk = min(KT, s1 - kt);
    for (int i = t; i < KT * D; i += AT) {
      const int kk = i / D, d = i % D;
      const bool in = kk < nk;
      const int64_t e = in ? kv_row(P, b, h, kt + kk) * D + d : 0;
      ks[kk][d] = in ? kb[e] : from_f<T>(0.f);
      vs[kk][d] = in ? vb[e] : from_f<T>(0.f);
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

// Merge of the splits: one CTA per (row, kv head, query row), one thread per
// head-dim element (blockDim.x = D).
template <typename T>
__global__ void attn_combine_kernel(AttnParams P) {
  const int r = blockIdx.x % P.R, bh = blockIdx.x / P.R;
  const int h = bh % P.Hkv, b = bh / P.Hkv;
  const int d = threadIdx.x;
  const int64_t base = ((int64_t)b * P.Hkv + h) * P.nsplit * P.R + r;
  float m = -INFINITY;
  for (int sp = 0; sp < P.nsplit; ++sp) m = fmaxf(m, P.part_ml[(base + (int64_t)sp * P.R) * 2]);
  float l = 0.f, a = 0.f;
  if (m != -INFINITY) {
    for (int sp = 0; sp < P.nsplit; ++sp) {
      const int64_t o = base + (int64_t)sp * P.R;
      const float ms = P.part_ml[o * 2];
      if (ms == -INFINITY) continue;
      const float w = __expf(ms - m);
      l += w * P.part_ml[o * 2 + 1];
      a += w * P.part_acc[o * P.D + d];
    }
  }
  const int j = r / P.group, hq = h * P.group + r % P.group;
  const float y = l > 0.f ? a / l : 0.f;
  reinterpret_cast<T*>(P.out)[b * P.obs + j * P.oqs + hq * P.ohs + d] = from_f<T>(y);
}

// ---------------------------------------------------------------------------
// Tensor-core path (bf16, head_dim 128, R = qlen * group <= 32 query rows)
// ---------------------------------------------------------------------------
// One CTA per (row, kv head, split of SPLIT_KEYS keys), 4 warps.  Per tile of
// 64 keys each warp takes 16 keys and computes S^T = K Q^T (keys on the M
// side, the <= 32 query rows of the kv head on N, so only N pads), the online
// softmax per query row in base 2, and O^T += V^T P^T with P^T moved into the
// B-operand layout by a register transpose.  K / V tiles are double-buffered
// in shared memory by cp.async with a 16-byte-chunk XOR swizzle (conflict-free
// ldmatrix).  The four warps' (max, sum, O) merge in shared memory.  A row
// whose live keys fit one split writes its output directly; otherwise each
// split leaves a partial (max, sum, O) in the workspace and the split that
// finishes last for its (row, kv head), found by an atomic counter, merges
// them while they are still in L2 — no separate combine launch.
constexpr int MT_KEYS = 64;              // keys per tile (16 per warp)
constexpr int MT_MIN_SHARE = SPLIT_KEYS / MT_KEYS;  // fewest tiles per CTA
constexpr float MT_HEADROOM = 8.f;       // lazy-rescale headroom of the running max (base 2)
constexpr int MT_THREADS = 128;
constexpr int MT_D = 128;

struct MmaSmem {
  union {
    struct {
      __nv_bfloat16 k[2][MT_KEYS * MT_D];
      __nv_bfloat16 v[2][MT_KEYS * MT_D];
    } kv;
    float o[4][32][MT_D];                // per-warp O (rows x d) for the merge
  } u;
  __nv_bfloat16 q[32 * MT_D];
  float ms[4][32], ls[4][32];
  int last;                              // this CTA finished its (row, kv head) last
  int seg_b;                             // row of the CTA's first tile
};

// byte offset of 16-byte chunk c of row r in a swizzled [rows][128] bf16 tile
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)(r * (MT_D * 2) + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool in) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
               :: "r"(dst), "l"(src), "r"(in ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

__device__ __forceinline__ void ldm_x4(uint32_t addr, uint32_t& a0, uint32_t& a1, uint32_t& a2,
                                       uint32_t& a3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3) : "r"(addr));
}
__device__ __forceinline__ void ldm_x4_t(uint32_t addr, uint32_t& a0, uint32_t& a1, uint32_t& a2,
                                         uint32_t& a3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3) : "r"(addr));
}
__device__ __forceinline__ void ldm_x2(uint32_t addr, uint32_t& b0, uint32_t& b1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(b0), "=r"(b1) : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}
// D = A (16x16, row) * B (16x8, col) + D, bf16 in, fp32 accumulate
__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
               "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Merge with every load issued up front (128 threads; `scratch` holds
// 2 * R * np floats of shared memory): (max, sum) of every (row, piece) in
// one pass, per-row weights in shared memory, then each thread (head-dim
// element t) pulls all its partial O values at once.  About three memory
// round trips instead of one per row and pass.
__device__ __noinline__ void merge_pieces_wide(const AttnParams& P, int b, int h, int np, int t,
                                               float* scratch, __nv_bfloat16* out,
                                               void (*sync)()) {
  const int R = P.R;
  const int64_t base0 = ((int64_t)b * P.Hkv + h) * P.npiece * R;
  float* ms = scratch;                                 // [R][np] max (natural log units)
  float* wl = scratch + R * np;                        // [R][np] sum, then weight / L
  for (int i = t; i < R * np; i += 128) {
    const int r = i / np, sp = i - r * np;
    const int64_t o = (base0 + (int64_t)sp * R + r) * 2;
    ms[i] = __ldcg(&P.part_ml[o]);
    wl[i] = __ldcg(&P.part_ml[o + 1]);
  }
  sync();
  if (t < R) {
    float m = -INFINITY;
    for (int sp = 0; sp < np; ++sp) m = fmaxf(m, ms[t * np + sp]);
    float L = 0.f;
    for (int sp = 0; sp < np; ++sp) {
      const float mv = ms[t * np + sp];
      const float f = (m == -INFINITY || mv == -INFINITY) ? 0.f : __expf(mv - m);
      ms[t * np + sp] = f;
      L += f * wl[t * np + sp];
    }
    const float il = L > 0.f ? 1.f / L : 0.f;
    for (int sp = 0; sp < np; ++sp) wl[t * np + sp] = ms[t * np + sp] * il;
  }
  sync();
  const int d = t;
  for (int r0 = 0; r0 < R; r0 += 8) {                  // 8 rows x np pieces of loads in flight
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int sp = 0; sp < np; ++sp) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int r = r0 + q;
        if (r < R)
          acc[q] += wl[r * np + sp] *
                    __ldcg(&P.part_acc[(base0 + (int64_t)sp * R + r) * MT_D + d]);
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int r = r0 + q;
      if (r < R) {
        const int j = r / P.group, hq = h * P.group + r % P.group;
        out[b * P.obs + j * P.oqs + hq * P.ohs + d] = __float2bfloat16(acc[q]);
      }
    }
  }
}

// Merge the partials (max, sum, O) of a (row, kv head)'s pieces into the
// output: one warp per query row; lanes own pieces for (max, sum), then four
// head-dim elements each for O (float4), eight pieces' loads in flight.
__device__ __noinline__ void merge_pieces(const AttnParams& P, int b, int h, int np, int w,
                                          int lane, __nv_bfloat16* out) {
  const int R = P.R;
  const int64_t base0 = ((int64_t)b * P.Hkv + h) * P.npiece * R;
  for (int r = w; r < R; r += MT_THREADS / 32) {
    float mx = -INFINITY, ll = 0.f, ms0 = -INFINITY;
    for (int c0 = 0; c0 < np; c0 += 32) {              // per lane, online over its pieces
      const int sp = c0 + lane;
      if (sp < np) {
        const float ms = __ldcg(&P.part_ml[(base0 + (int64_t)sp * R + r) * 2]);
        const float lv = __ldcg(&P.part_ml[(base0 + (int64_t)sp * R + r) * 2 + 1]);
        if (c0 == 0) ms0 = ms;
        if (ms != -INFINITY) {
          const float mn = fmaxf(mx, ms);
          ll = (mx == -INFINITY ? 0.f : ll * __expf(mx - mn)) + lv * __expf(ms - mn);
          mx = mn;
        }
      }
    }
    float gm = mx;
#pragma unroll
    for (int o = 16; o; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
    float L = mx == -INFINITY ? 0.f : ll * __expf(mx - gm);
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (L > 0.f) {
      for (int c0 = 0; c0 < np; c0 += 32) {
        const int sp = c0 + lane;
        float ms = ms0;
        if (c0 > 0) ms = sp < np ? __ldcg(&P.part_ml[(base0 + (int64_t)sp * R + r) * 2]) : -INFINITY;
        const float f = (sp < np && ms != -INFINITY) ? __expf(ms - gm) : 0.f;
        const int n = min(32, np - c0);
        for (int i0 = 0; i0 < n; i0 += 8) {
          float4 v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            v[u] = i0 + u < n ? __ldcg(reinterpret_cast<const float4*>(
                                    P.part_acc + (base0 + (int64_t)(c0 + i0 + u) * R + r) * MT_D) +
                                lane)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float fu = __shfl_sync(0xffffffffu, f, (i0 + u) & 31);
            a.x += fu * v[u].x; a.y += fu * v[u].y; a.z += fu * v[u].z; a.w += fu * v[u].w;
          }
        }
      }
    }
    const float il = L > 0.f ? 1.f / L : 0.f;
    const int j = r / P.group, hq = h * P.group + r % P.group;
    const __nv_bfloat162 y0 = __floats2bfloat162_rn(a.x * il, a.y * il);
    const __nv_bfloat162 y1 = __floats2bfloat162_rn(a.z * il, a.w * il);
    __nv_bfloat16* dst = out + b * P.obs + j * P.oqs + hq * P.ohs + 4 * lane;
    if (P.out_vec4) {
      uint2 pk;
      pk.x = *reinterpret_cast<const uint32_t*>(&y0);
      pk.y = *reinterpret_cast<const uint32_t*>(&y1);
      *reinterpret_cast<uint2*>(dst) = pk;
    } else {
      dst[0] = y0.x; dst[1] = y0.y; dst[2] = y1.x; dst[3] = y1.y;
    }
  }
}

// One CTA for the whole call: per row b the live-key bound kmax_b (the
// largest limit over its queries), the exclusive prefix of its 64-key tile
// counts (rowpre[B] = tiles per kv head summed over rows), the split counters
// zeroed, and a zero output for rows without a live key.
__global__ void __launch_bounds__(1024) attn_plan_kernel(AttnParams P) {
  __shared__ int wsum[32];
  __shared__ int carry, nzero;
  __shared__ int zrow[1024];                           // rows of this chunk without a live key
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  if (t == 0) {
    carry = 0;
    *P.status = 0;
  }
  for (int i = t; i < P.B * P.Hkv; i += 1024) P.split_done[i] = 0;
  __syncthreads();
  for (int b0 = 0; b0 < P.B; b0 += 1024) {
    const int b = b0 + t;
    if (t == 0) nzero = 0;
    int km = 0;
    if (b < P.B) {
      km = row_limit(P, b, P.qlen - 1);                // the limit grows with the query index
      P.rowkmax[b] = km;
    }
    int tiles = (km + P.tile_keys - 1) / P.tile_keys;
    if (tiles > 0) tiles += P.seg_ovh;                 // fixed per-(row, kv head) cost
    int x = tiles;                                     // inclusive scan within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int s = wsum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      wsum[lane] = s;
    }
    __syncthreads();
    const int excl = carry + (w ? wsum[w - 1] : 0) + x - tiles;
    if (b < P.B) {
      P.rowpre[b] = excl;
      if (km == 0) zrow[atomicAdd(&nzero, 1)] = b;
    }
    __syncthreads();
    if (t == 1023) carry = excl + tiles;
    // rows without a live key get a zero output (no CTA of the main kernel visits them)
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(P.out);
    for (int z = 0; z < nzero; ++z) {
      const int bz = zrow[z];
      for (int idx = t; idx < P.Hq * P.qlen * MT_D; idx += 1024) {
        const int d = idx % MT_D, jh = idx / MT_D, j = jh % P.qlen, hq = jh / P.qlen;
        out[bz * P.obs + j * P.oqs + hq * P.ohs + d] = __float2bfloat16(0.f);
      }
    }
    __syncthreads();
  }
  if (t == 0) P.rowpre[P.B] = carry;
}

// Persistent, stream-K style: the 64-key tiles of every (row, kv head) are laid
// end to end (row-major, kv head inner) and each CTA takes one contiguous run
// of `share` tiles, so every CTA streams the same number of K/V bytes whatever
// the row lengths.  A run crosses (row, kv head) boundaries as segments; a
// (row, kv head) covered by one CTA writes its output directly, otherwise
// each piece leaves a partial and the piece that finishes last merges them.
template <int NT>
__global__ void __launch_bounds__(MT_THREADS, NT <= 3 ? 3 : 2)
attn_mma_kernel(const __grid_constant__ AttnParams P) {
  extern __shared__ __align__(128) unsigned char mma_smem[];
  MmaSmem& S = *reinterpret_cast<MmaSmem*>(mma_smem);
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int R = P.R, Hkv = P.Hkv;
  const int total = P.rowpre[P.B] * Hkv;
  const int share = max(MT_MIN_SHARE, (total + (int)gridDim.x - 1) / (int)gridDim.x);
  const int t0 = (int)blockIdx.x * share;
  if (t0 >= total) return;
  const int t1 = min(total, t0 + share);
  for (int b = t; b < P.B; b += MT_THREADS)            // the row holding tile t0
    if (P.rowpre[b] * Hkv <= t0 && t0 < P.rowpre[b + 1] * Hkv) S.seg_b = b;
  __syncthreads();
  int b = S.seg_b;
  int tb = P.rowpre[b + 1] - P.rowpre[b];              // tiles per kv head in row b
  int h = (t0 - P.rowpre[b] * Hkv) / tb;
  int off = (t0 - P.rowpre[b] * Hkv) % tb;
  int tt = t0;
  const __nv_bfloat16* Q = reinterpret_cast<const __nv_bfloat16*>(P.q);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(P.out);
  const float sl2 = P.scale * 1.4426950408889634f;
  const int krow0 = 16 * w;                            // this warp's keys within a tile
  while (true) {
    const int nseg = min(tb - off, t1 - tt);           // tiles of this segment
    const int s0 = off * MT_KEYS, s1 = min(P.rowkmax[b], (off + nseg) * MT_KEYS);
    const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(P.k);
    const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(P.v);
    auto load_tile = [&](int tile, int buf) {
      const int key0 = s0 + tile * MT_KEYS;
      const uint32_t kd = smem_addr(S.u.kv.k[buf]), vd = smem_addr(S.u.kv.v[buf]);
      for (int i = t; i < MT_KEYS * 16; i += MT_THREADS) {
        const int kk = i >> 4, c = i & 15;
        const bool in = key0 + kk < s1;
        const int64_t row = kv_row(P, b, h, in ? key0 + kk : s0);   // valid when nothing is read
        cp_async16(kd + sw_off(kk, c), kb + row * MT_D + 8 * c, in);
        cp_async16(vd + sw_off(kk, c), vb + row * MT_D + 8 * c, in);
      }
      cp_async_commit();
    };
    load_tile(0, 0);
    if (nseg > 1) load_tile(1, 1);
    // the kv head's query rows r = j * group + g (zero rows up to 8 * NT)
    for (int i = t; i < 32 * 16; i += MT_THREADS) {
      const int r = i >> 4, c = i & 15;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < R) {
        const int j = r / P.group, hq = h * P.group + r % P.group;
        v = *reinterpret_cast<const uint4*>(Q + b * P.qbs + hq * P.qhs + j * P.qqs + 8 * c);
      }
      *reinterpret_cast<uint4*>(reinterpret_cast<char*>(S.q) + sw_off(r, c)) = v;
    }
    __syncthreads();
    const uint32_t qbase = smem_addr(S.q);
    // this thread's query-row columns r = 8 nt + 2 (lane % 4) + e
    float mrow[NT][2], lrow[NT][2];
    int lim[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = 8 * nt + 2 * (lane & 3) + e;
        mrow[nt][e] = -INFINITY;
        lrow[nt][e] = 0.f;
        lim[nt][e] = r < R ? min(row_limit(P, b, r / P.group), s1) : 0;
      }
    float o[8][NT][4];
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;
    for (int tile = 0; tile < nseg; ++tile) {
      const int buf = tile & 1;
      if (tile + 1 < nseg) cp_async_wait<1>(); else cp_async_wait<0>();
      __syncthreads();
      const uint32_t kbase = smem_addr(S.u.kv.k[buf]), vbase = smem_addr(S.u.kv.v[buf]);
      // S^T = K Q^T for the warp's 16 keys
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldm_x4(kbase + sw_off(krow0 + (lane & 15), 2 * ks + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          uint32_t q0, q1;                             // Q fragments, re-read from shared memory
          ldm_x2(qbase + sw_off(8 * nt + (lane & 7), 2 * ks + ((lane >> 3) & 1)), q0, q1);
          mma16816(sc[nt], a0, a1, a2, a3, q0, q1);
        }
      }
      // online softmax per query row (base 2), over the warp's keys
      const int kg = s0 + tile * MT_KEYS + krow0 + (lane >> 2);
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int le = lim[nt][e];
          const float sa = kg < le ? sc[nt][e] * sl2 : -INFINITY;
          const float sb = kg + 8 < le ? sc[nt][2 + e] * sl2 : -INFINITY;
          // lazy rescale: the reference max m of a query row moves only when a
          // score exceeds it by more than MT_HEADROOM (base 2), so the common
          // tile needs no cross-lane max; p = 2^(s - m) stays below 2^MT_HEADROOM
          float mx = fmaxf(sa, sb);
          if (__any_sync(0xffffffffu, mx > mrow[nt][e] + MT_HEADROOM)) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mold = mrow[nt][e];
            const float mnew = fmaxf(mold, mx);
            const float alpha =
                mnew == -INFINITY ? 1.f : (mold == -INFINITY ? 0.f : ex2f(mold - mnew));
            lrow[nt][e] *= alpha;
            mrow[nt][e] = mnew;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
              o[mt][nt][e] *= alpha;
              o[mt][nt][2 + e] *= alpha;
            }
          }
          const float pa = sa == -INFINITY ? 0.f : ex2f(sa - mrow[nt][e]);
          const float pbv = sb == -INFINITY ? 0.f : ex2f(sb - mrow[nt][e]);
          lrow[nt][e] += pa + pbv;
          sc[nt][e] = pa;
          sc[nt][2 + e] = pbv;
        }
        // P^T (keys x rows) into the B-operand layout
        pb[nt][0] = movm_t(pack_bf16(sc[nt][0], sc[nt][1]));
        pb[nt][1] = movm_t(pack_bf16(sc[nt][2], sc[nt][3]));
      }
      // O^T += V^T P^T over the head dimension (8 m-tiles of 16)
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldm_x4_t(vbase + sw_off(krow0 + (lane & 7) + ((lane >> 4) << 3), 2 * mt + ((lane >> 3) & 1)),
                 a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816(o[mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
      }
      __syncthreads();                                 // the buffer is refilled next
      if (tile + 2 < nseg) load_tile(tile + 2, buf);
    }
    // row sums over the lanes that share a column; merge the four warps
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float l = lrow[nt][e];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        lrow[nt][e] = l;
      }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = 8 * nt + 2 * (lane & 3) + e;
        if (lane < 4) { S.ms[w][r] = mrow[nt][e]; S.ls[w][r] = lrow[nt][e]; }
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          S.u.o[w][r][16 * mt + (lane >> 2)] = o[mt][nt][e];
          S.u.o[w][r][16 * mt + (lane >> 2) + 8] = o[mt][nt][2 + e];
        }
      }
    __syncthreads();
    const int bh = b * Hkv + h;
    const int Tb = P.rowpre[b] * Hkv + h * tb;         // first tile of this (row, kv head)
    const int cfirst = Tb / share;
    const int npieces = (Tb + tb - 1) / share - cfirst + 1;
    const int64_t pbase = ((int64_t)bh * P.npiece + ((int)blockIdx.x - cfirst)) * R;
    for (int idx = t; idx < R * MT_D; idx += MT_THREADS) {
      const int r = idx >> 7, d = idx & (MT_D - 1);
      float m = -INFINITY;
#pragma unroll
      for (int q = 0; q < 4; ++q) m = fmaxf(m, S.ms[q][r]);
      float acc = 0.f, l = 0.f;
      if (m != -INFINITY) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (S.ms[q][r] == -INFINITY) continue;
          const float f = ex2f(S.ms[q][r] - m);
          acc += f * S.u.o[q][r][d];
          l += f * S.ls[q][r];
        }
      }
      if (npieces == 1) {                              // the only piece: final output
        const int j = r / P.group, hq = h * P.group + r % P.group;
        out[b * P.obs + j * P.oqs + hq * P.ohs + d] = __float2bfloat16(l > 0.f ? acc / l : 0.f);
        continue;
      }
      P.part_acc[(pbase + r) * MT_D + d] = acc;
      if (d == 0) {
        P.part_ml[(pbase + r) * 2] = m == -INFINITY ? -INFINITY : m * 0.6931471805599453f;
        P.part_ml[(pbase + r) * 2 + 1] = l;
      }
    }
    if (npieces > 1) {
      __threadfence();
      __syncthreads();
      if (t == 0) S.last = atomicAdd(&P.split_done[bh], 1) == npieces - 1;
      __syncthreads();
      if (S.last) {
        __threadfence();
        merge_pieces(P, b, h, npieces, w, lane, out);
      }
    }
    tt += nseg;
    if (tt >= t1) break;
    off = 0;
    if (++h == Hkv) {
      h = 0;
      do { ++b; } while (P.rowpre[b + 1] == P.rowpre[b]);
      tb = P.rowpre[b + 1] - P.rowpre[b];
    }
    __syncthreads();                                   // merge area and Q are rewritten next
  }
}

// ---------------------------------------------------------------------------
// tcgen05 path (bf16, head_dim 128, R <= 32 query rows per kv head)
// ---------------------------------------------------------------------------
// Same stream-K schedule as attn_mma_kernel, with 128-key tiles.  Per tile:
//   S^T[128 keys, 32] = K_tile[128, 128 d] . Q^T        (tcgen05.mma, M=128 N=32,
//                        A = K tile K-major, B = Q K-major, both 128B-swizzled;
//                        accumulator in TMEM, double-buffered)
//   softmax: thread t of the 4 softmax warps owns key t (TMEM lane t): 32
//            scores in registers, lazy reference max per query row (moved
//            only when a score passes it by TC_HEADROOM, a CTA-wide vote),
//            p = 2^(s - m) written to shared memory as P^T (MN-major, 16 B
//            per thread and row group)
//   O^T[128 d, 32] += V^T[128 d, 128 keys] . P^T       (tcgen05.mma, A = the V
//                        tile MN-major 128B-swizzled, B = P^T MN-major; O in
//                        TMEM for the whole segment)
// K / V tiles arrive by TMA (2D tensor maps over the caches viewed as
// [B * Hkv * C, 128], 64-column boxes, 128B swizzle, no multicast) into a
// TC_NST-stage ring.  Warp roles: 0-3 softmax + epilogue (TMEM lane quarter
// = warp), 4 TMA producer, 5 MMA issuer (one elected thread each).  Every
// wait is bounded; on expiry the CTA records SD attention error bit 0 and
// drains.
constexpr int TC_KEYS = 128;             // keys per tile
static_assert(TC_KEYS == SD_KV_PAGE, "a K/V tile of the tcgen05 kernel is one cache page");
constexpr int TC_N = 32;                 // query rows per kv head (padded)
constexpr int TC_NST = 3;                // K/V ring stages
constexpr int TC_THREADS = 192;
constexpr int TC_MIN_SHARE = SPLIT_KEYS / TC_KEYS;
constexpr float TC_HEADROOM = 8.f;
// Schedule cost of starting a (row, kv head) segment, in tiles: its Q,
// first-tile max, epilogue and barriers take about as long as this many
// tiles, so CTAs that cover many short rows get fewer tiles.  The schedule
// lays these virtual tiles in front of each (row, kv head)'s real ones.
constexpr int TC_OVH = 6;
constexpr uint32_t TC_TMEM_COLS = 128;   // S0, S1, O0, O1 (32 columns each)
constexpr long long TC_WAIT = 1LL << 31; // cycles (~1 s) before a wait gives up

struct TcSmem {
  alignas(1024) unsigned char k[TC_NST][2][TC_KEYS * 128];   // [stage][64-col box][128 rows x 128 B]
  alignas(1024) unsigned char v[TC_NST][2][TC_KEYS * 128];
  alignas(1024) unsigned char q[2][2][TC_N * 128];           // Q per segment parity, 2 boxes
  alignas(1024) unsigned char p[2][4 * 2048];                // P^T, MN-major, double-buffered
  alignas(8) unsigned long long full[TC_NST], empty[TC_NST];
  alignas(8) unsigned long long sfull[2], sfree[2], pfull[2];
  // oready[g & 1]: GEMM2 of tile g done.  Two barriers so that every wait on
  // one sees at most two of its phases outstanding (a tile's sfull commit
  // already covers the GEMM2 two tiles back).
  alignas(8) unsigned long long oready[2], qfull, fin;
  float red[4][TC_N];                                        // cross-warp row reductions
  uint32_t tmem;
  int seg_b;
  int abort_;
  int last;
};
static_assert(sizeof(TcSmem) + 1024 <= 227 * 1024, "tcgen05 attention shared memory");

__device__ __forceinline__ uint32_t tc_sw128(int row, int col) {  // element offset in a 64-col box
  return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                            uint32_t layout) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)(layout & 7) << 61);
}
// kind::f16 instruction descriptor: bf16 A and B, f32 D, M x N, majors
__host__ __device__ constexpr uint32_t tc_idesc(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, int acc) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
               " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
               :: "r"(d), "l"(a), "l"(b), "r"(id), "r"(acc) : "memory");
}
__device__ __forceinline__ void tc_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tc_bar_init(unsigned long long* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_addr(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void tc_arrive(unsigned long long* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}"
               :: "r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tc_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// Has the phase of parity `par` completed?  (non-blocking)
__device__ __forceinline__ bool tc_test(unsigned long long* bar, uint32_t par) {
  uint32_t done;
  asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
               " selp.u32 %0, 1, 0, p;\n}" : "=r"(done) : "r"(smem_addr(bar)), "r"(par)
               : "memory");
  return done != 0;
}
// Bounded wait for the phase of parity `par`; false (and the CTA's abort
// flag set) on expiry or when another thread already gave up.
__device__ __forceinline__ bool tc_wait(unsigned long long* bar, uint32_t par, int* abort_) {
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}" : "=r"(done) : "r"(smem_addr(bar)), "r"(par)
                 : "memory");
    if (done) return true;
    if (*reinterpret_cast<volatile int*>(abort_) || clock64() - t0 > TC_WAIT) {
      *reinterpret_cast<volatile int*>(abort_) = 1;
      return false;
    }
  }
}
__device__ __forceinline__ void tc_tma_2d(void* dst, const void* tmap, int x, int y,
                                          unsigned long long* bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
               " [%0], [%1, {%2, %3}], [%4];"
               :: "r"(smem_addr(dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
               : "memory");
}
#define TC_LD32(r, addr)                                                                        \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,"    \
               "%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,"  \
               "%30,%31}, [%32];"                                                               \
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),        \
                 "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),     \
                 "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), \
                 "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), \
                 "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), \
                 "=r"(r[30]), "=r"(r[31])                                                      \
               : "r"(addr) : "memory")
#define TC_ST32(addr, r)                                                                        \
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,"  \
               "%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,"  \
               "%30,%31,%32};"                                                                  \
               :: "r"(addr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), \
                 "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),\
                 "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),       \
                 "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),       \
                 "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]),       \
                 "r"(r[31]) : "memory")
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// barrier of the four softmax warps
__device__ __forceinline__ void tc_sbar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool tc_sbar_or(bool p) {
  int r;
  asm volatile("{\n .reg .pred a, b;\n setp.ne.b32 a, %1, 0;\n"
               " bar.red.or.pred b, 1, 128, a;\n selp.s32 %0, 1, 0, b;\n}"
               : "=r"(r) : "r"((int)p) : "memory");
  return r != 0;
}

// The CTA's run of tiles as (row, kv head) segments, walked identically by
// every role.
struct TcSeg {
  int b, h, tb, off, tt, t1, ncost, nseg, s0, s1;   // tb, off, ncost: schedule units
};
__device__ __forceinline__ void tc_seg_init(TcSeg& g, const AttnParams& P, int b0, int t0, int t1) {
  g.b = b0;
  g.tb = P.rowpre[b0 + 1] - P.rowpre[b0];
  g.h = (t0 - P.rowpre[b0] * P.Hkv) / g.tb;
  g.off = (t0 - P.rowpre[b0] * P.Hkv) % g.tb;
  g.tt = t0;
  g.t1 = t1;
}
__device__ __forceinline__ void tc_seg_bounds(TcSeg& g, const AttnParams& P) {
  g.ncost = min(g.tb - g.off, g.t1 - g.tt);
  const int r0 = max(g.off, TC_OVH) - TC_OVH;          // real tiles: units past the virtual ones
  const int r1 = g.off + g.ncost - TC_OVH;
  g.nseg = max(r1 - r0, 0);
  g.s0 = r0 * TC_KEYS;
  g.s1 = min(P.rowkmax[g.b], r1 * TC_KEYS);
}
// advance past the current segment; false when the run is over
__device__ __forceinline__ bool tc_seg_next(TcSeg& g, const AttnParams& P) {
  g.tt += g.ncost;
  if (g.tt >= g.t1) return false;
  g.off = 0;
  if (++g.h == P.Hkv) {
    g.h = 0;
    do { ++g.b; } while (P.rowpre[g.b + 1] == P.rowpre[g.b]);
    g.tb = P.rowpre[g.b + 1] - P.rowpre[g.b];
  }
  return true;
}
// the current or next segment that holds real tiles; false when none is left
__device__ __forceinline__ bool tc_seg_real(TcSeg& g, const AttnParams& P) {
  tc_seg_bounds(g, P);
  while (g.nseg == 0) {
    if (!tc_seg_next(g, P)) return false;
    tc_seg_bounds(g, P);
  }
  return true;
}

template <int NTG>                                    // 8-row groups of real query rows
__global__ void __launch_bounds__(TC_THREADS, 1)
attn_tc_kernel(const __grid_constant__ AttnParams P, const __grid_constant__ CUtensorMap tmk,
               const __grid_constant__ CUtensorMap tmv) {
  constexpr int RN = 8 * NTG;                          // rows the softmax computes (<= TC_N)
  extern __shared__ __align__(1024) unsigned char tc_raw[];
  const uint32_t pad = (1024u - (smem_addr(tc_raw) & 1023u)) & 1023u;  // swizzle atoms: 1024 B
  TcSmem& S = *reinterpret_cast<TcSmem*>(tc_raw + pad);
  const int t = threadIdx.x, w = t >> 5, lane = t & 31;
  const int R = P.R, Hkv = P.Hkv;
  const int total = P.rowpre[P.B] * Hkv;
  const int share = max(TC_MIN_SHARE, (total + (int)gridDim.x - 1) / (int)gridDim.x);
  const int t0 = (int)blockIdx.x * share;
  if (t0 >= total) return;                             // no work for this CTA (uniform)
  const int t1 = min(total, t0 + share);
  for (int b = t; b < P.B; b += TC_THREADS)
    if (P.rowpre[b] * Hkv <= t0 && t0 < P.rowpre[b + 1] * Hkv) S.seg_b = b;
  if (t == 0) {
    for (int i = 0; i < TC_NST; ++i) {
      tc_bar_init(&S.full[i], 1);
      tc_bar_init(&S.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc_bar_init(&S.sfull[i], 1);
      tc_bar_init(&S.sfree[i], 128);
      tc_bar_init(&S.pfull[i], 128);
    }
    tc_bar_init(&S.oready[0], 1);
    tc_bar_init(&S.oready[1], 1);
    tc_bar_init(&S.qfull, 128);
    tc_bar_init(&S.fin, 1);
    S.abort_ = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (w == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_addr(&S.tmem)), "r"(TC_TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = S.tmem;
  TcSeg g;
  tc_seg_init(g, P, S.seg_b, t0, t1);

  if (w == 4) {
    // ---------------- TMA producer
    if (lane == 0) {
      uint32_t gi = 0;
      bool ok = true;
      do {
        tc_seg_bounds(g, P);
        const int row0 = P.bt ? 0 : (g.b * Hkv + g.h) * P.C + g.s0;
        for (int i = 0; i < g.nseg && ok; ++i, ++gi) {
          const int st = (int)(gi % TC_NST);
          if (gi >= (uint32_t)TC_NST)
            ok = tc_wait(&S.empty[st], ((gi / TC_NST) - 1) & 1u, &S.abort_);
          if (!ok) break;
          tc_expect_tx(&S.full[st], 4u * TC_KEYS * 128u);
          // a tile is one page of a paged cache (segments start on tile bounds)
          const int y = P.bt ? (int)kv_row(P, g.b, g.h, g.s0 + i * TC_KEYS) : row0 + i * TC_KEYS;
          tc_tma_2d(S.k[st][0], &tmk, 0, y, &S.full[st]);
          tc_tma_2d(S.k[st][1], &tmk, 64, y, &S.full[st]);
          tc_tma_2d(S.v[st][0], &tmv, 0, y, &S.full[st]);
          tc_tma_2d(S.v[st][1], &tmv, 64, y, &S.full[st]);
        }
      } while (ok && tc_seg_next(g, P));
      if (!ok) {
        // let the copies already issued land before the CTA leaves
        for (uint32_t q = gi > (uint32_t)TC_NST ? gi - TC_NST : 0u; q < gi; ++q) {
          int dummy = 0;
          tc_wait(&S.full[q % TC_NST], (q / TC_NST) & 1u, &dummy);
        }
      }
    }
  } else if (w == 5) {
    // ---------------- MMA issuer: two in-order queues polled together, the
    // GEMM1s (S^T of tile a: needs its K/V stage loaded, its S buffer read
    // out, and for a segment's first tile that segment's Q) and the GEMM2s
    // (O^T += V^T P^T of tile c: needs its P), so that neither waits behind
    // the other's unrelated dependency
    if (lane == 0) {
      constexpr uint32_t ID1 = tc_idesc(128, TC_N, 0, 0);   // S^T = K . Q^T
      constexpr uint32_t ID2 = tc_idesc(128, TC_N, 1, 1);   // O^T += V^T . P^T
      uint32_t ntot = 0;                               // real tiles of the run
      {
        TcSeg gw = g;
        bool more = tc_seg_real(gw, P);
        while (more) {
          ntot += (uint32_t)gw.nseg;
          more = tc_seg_next(gw, P) && tc_seg_real(gw, P);
        }
      }
      TcSeg ga = g, gc = g;
      tc_seg_real(ga, P);
      tc_seg_real(gc, P);
      int ia = 0, ic = 0;
      uint32_t a = 0, c = 0, sa = 0, sc = 0;             // tiles and segments of the two heads
      long long idle0 = clock64();
      while (c < ntot) {
        bool progressed = false;
        // GEMM1(a) only after GEMM2(a - 2) was issued: its sfull commit then
        // covers that GEMM2, so the softmax may rewrite P buffer a & 1 and
        // every oready wait sees at most two phases outstanding
        if (a < ntot && a < c + 2) {
          const int st = (int)(a % TC_NST), sb = (int)(a & 1u);
          const bool ready = tc_test(&S.full[st], (a / TC_NST) & 1u) &&
                             (a < 2 || tc_test(&S.sfree[sb], ((a >> 1) - 1) & 1u)) &&
                             (ia != 0 || tc_test(&S.qfull, sa & 1u));
          if (ready) {
            tc_fence_after();
            const uint32_t ka0 = smem_addr(S.k[st][0]), ka1 = smem_addr(S.k[st][1]);
            const uint32_t qa0 = smem_addr(S.q[sa & 1u][0]), qa1 = smem_addr(S.q[sa & 1u][1]);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint32_t ko = (uint32_t)(ks & 3) * 32u;
              tc_mma(tm + (uint32_t)sb * 32u, tc_desc((ks < 4 ? ka0 : ka1) + ko, 16, 1024, 2),
                     tc_desc((ks < 4 ? qa0 : qa1) + ko, 16, 1024, 2), ID1, ks > 0 ? 1 : 0);
            }
            tc_commit(&S.sfull[sb]);
            ++a;
            if (++ia == ga.nseg) {
              ia = 0;
              ++sa;
              if (tc_seg_next(ga, P)) tc_seg_real(ga, P);
            }
            progressed = true;
          }
        }
        if (c < a) {
          const int st = (int)(c % TC_NST), pb = (int)(c & 1u);
          if (tc_test(&S.pfull[pb], (c >> 1) & 1u)) {
            tc_fence_after();
            const uint32_t va = smem_addr(S.v[st][0]), pa = smem_addr(S.p[pb]);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)
              tc_mma(tm + 64u + 32u * (sc & 1u), tc_desc(va + ks * 2048, 16384, 1024, 2),
                     tc_desc(pa + ks * 256, 128, 2048, 0), ID2, (ic > 0 || ks > 0) ? 1 : 0);
            tc_commit(&S.empty[st]);
            tc_commit(&S.oready[c & 1u]);
            ++c;
            if (++ic == gc.nseg) {
              ic = 0;
              ++sc;
              if (tc_seg_next(gc, P)) tc_seg_real(gc, P);
            }
            progressed = true;
          }
        }
        if (progressed) {
          idle0 = clock64();
        } else if (*reinterpret_cast<volatile int*>(&S.abort_) || clock64() - idle0 > TC_WAIT) {
          *reinterpret_cast<volatile int*>(&S.abort_) = 1;
          break;
        }
      }
      // every MMA this thread issued has finished before the CTA leaves
      // (TMEM is released after this)
      tc_commit(&S.fin);
      int dummy = 0;
      tc_wait(&S.fin, 0u, &dummy);
    }
  } else {
    // ---------------- softmax + epilogue warps (thread t: key t of a tile,
    // head-dim element t of O; TMEM lane quarter = warp)
    const uint32_t lrow = (uint32_t)(32 * w) << 16;
    const float sl2 = P.scale * 1.4426950408889634f;
    const __nv_bfloat16* Qg = reinterpret_cast<const __nv_bfloat16*>(P.q);
    if (NTG < TC_N / 8) {                              // row groups past RN stay 0 in P^T
      for (int i = t; i < 2 * 4 * 2048 / 16; i += 128)
        reinterpret_cast<uint4*>(&S.p[0][0])[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(P.out);
    // Q of a (row, kv head) into the swizzled B-operand tile of its segment
    // parity; rows >= R are 0
    auto write_q = [&](int qb, int qh, uint32_t qs) {
      for (int i = t; i < TC_N * 16; i += 128) {
        const int r = i >> 4, c = i & 15;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < R) {
          const int j = r / P.group, hq = qh * P.group + r % P.group;
          v = *reinterpret_cast<const uint4*>(Qg + qb * P.qbs + hq * P.qhs + j * P.qqs + 8 * c);
        }
        *reinterpret_cast<uint4*>(S.q[qs & 1u][c >> 3] + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_arrive(&S.qfull);
    };
    uint32_t gi = 0, seg = 0;
    bool run = true;
    bool more = tc_seg_real(g, P);
    if (more) write_q(g.b, g.h, 0u);
    while (more) {
      const int b = g.b, h = g.h;
      const uint32_t ocol = 64u + 32u * (seg & 1u);     // this segment's O buffer
      // per query row: live-key limit within this segment, reference max, partial sum
      int lim[RN];
      float m[RN], mc[RN], l[RN];
      int lim_min = g.s1;
      // the row's length and cap once (row_limit per query row would repeat
      // the global loads, serialised, at every segment start)
      const int64_t lenb = __ldg(P.lengths + b);
      const int64_t capb = min(P.valid ? __ldg(P.valid + b) : (int64_t)P.C, (int64_t)P.C);
#pragma unroll
      for (int r = 0; r < RN; ++r) {
        const int64_t lj = min(lenb + r / P.group + 1, capb);
        lim[r] = r < R ? (int)min(max(lj, (int64_t)0), (int64_t)g.s1) : 0;
        if (r < R) lim_min = min(lim_min, lim[r]);
        m[r] = -INFINITY;
        mc[r] = -1e30f;                                // m clamped: 2^(-inf - mc) = 0
        l[r] = 0.f;
      }
      for (int i = 0; i < g.nseg; ++i, ++gi) {
        const int sb = (int)(gi & 1u);
        const bool ok = tc_wait(&S.sfull[sb], (gi >> 1) & 1u, &S.abort_);
        uint32_t sr[TC_N];
        tc_fence_after();
        TC_LD32(sr, tm + lrow + (uint32_t)sb * 32u);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        tc_fence_before();
        tc_arrive(&S.sfree[sb]);
        const int key = g.s0 + i * TC_KEYS + t;
        // every row sees every key of the tile except near a row's limit
        const bool whole = g.s0 + (i + 1) * TC_KEYS <= lim_min;
        float sc[RN];
        bool exceed = false;
#pragma unroll
        for (int r = 0; r < RN; ++r) {
          const float v = __uint_as_float(sr[r]) * sl2;
          sc[r] = (whole || key < lim[r]) ? v : -INFINITY;
          exceed |= sc[r] > m[r] + TC_HEADROOM;
        }
        if (tc_sbar_or(exceed || !ok)) {
          if (tc_sbar_or(!ok)) { run = false; break; }   // a wait gave up: all leave together
          // move the reference max of every row to the tile's maximum
#pragma unroll
          for (int r = 0; r < RN; ++r) {
            float mx = sc[r];
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) S.red[w][r] = mx;
          }
          tc_sbar();
          float alpha[RN];
#pragma unroll
          for (int r = 0; r < RN; ++r) {
            const float mt = fmaxf(fmaxf(S.red[0][r], S.red[1][r]), fmaxf(S.red[2][r], S.red[3][r]));
            const float mn = fmaxf(m[r], mt);
            alpha[r] = mn == -INFINITY ? 1.f : (m[r] == -INFINITY ? 0.f : ex2f(m[r] - mn));
            m[r] = mn;
            mc[r] = fmaxf(mn, -1e30f);
            l[r] *= alpha[r];
          }
          if (i > 0) {
            // O holds this segment's earlier tiles: wait for the last GEMM into
            // it (GEMM2 of tile gi - 1), then rescale every row in TMEM
            const bool ok2 = tc_wait(&S.oready[(gi - 1) & 1u], ((gi - 1) >> 1) & 1u, &S.abort_);
            (void)ok2;
            tc_fence_after();
            uint32_t o[TC_N];
            TC_LD32(o, tm + lrow + ocol);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int r = 0; r < RN; ++r) o[r] = __float_as_uint(__uint_as_float(o[r]) * alpha[r]);
            TC_ST32(tm + lrow + ocol, o);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
          }
          tc_sbar();                                   // S.red free again; O rescaled by all
        }
        // p = 2^(s - m) into P^T (MN-major: 16 B per row group of 8)
        unsigned char* pb = S.p[sb];
#pragma unroll
        for (int gr = 0; gr < NTG; ++gr) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int r = 8 * gr + e;
            pv[e] = ex2f(sc[r] - mc[r]);
            l[r] += pv[e];
          }
          uint4 pk;
          pk.x = pack_bf16(pv[0], pv[1]); pk.y = pack_bf16(pv[2], pv[3]);
          pk.z = pack_bf16(pv[4], pv[5]); pk.w = pack_bf16(pv[6], pv[7]);
          *reinterpret_cast<uint4*>(pb + gr * 2048 + (t >> 3) * 128 + (t & 7) * 16) = pk;
        }
        if (key >= g.s1) {
          // past the live window the tile holds other cache slots (maybe never
          // written: NaN would survive 0 * x): zero this key's V row
          const int st = (int)(gi % TC_NST);
          uint4* v0 = reinterpret_cast<uint4*>(S.v[st][0] + t * 128);
          uint4* v1 = reinterpret_cast<uint4*>(S.v[st][1] + t * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            v0[c] = make_uint4(0u, 0u, 0u, 0u);
            v1[c] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        tc_arrive(&S.pfull[sb]);
        if (i == 0) {
          // the next segment's Q, early: its buffer's last reader (the previous
          // segment's GEMM1s) finished before this tile's S arrived, and the
          // global loads overlap this segment's tiles
          TcSeg gn = g;
          if (tc_seg_next(gn, P) && tc_seg_real(gn, P)) write_q(gn.b, gn.h, seg + 1u);
        }
      }
      if (!run) break;
      // ---- segment epilogue: O^T (lane = head-dim element t), row sums, output
      const bool ok = tc_wait(&S.oready[(gi - 1) & 1u], ((gi - 1) >> 1) & 1u, &S.abort_);
      if (tc_sbar_or(!ok)) break;
      tc_fence_after();
      uint32_t o[TC_N];
      TC_LD32(o, tm + lrow + ocol);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      tc_fence_before();
#pragma unroll
      for (int r = 0; r < RN; ++r) {
        float sum = l[r];
#pragma unroll
        for (int q = 16; q; q >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, q);
        if (lane == 0) S.red[w][r] = sum;
      }
      tc_sbar();
      const int bh = b * Hkv + h;
      const int Tb = P.rowpre[b] * Hkv + h * g.tb;     // first tile of this (row, kv head)
      const int cfirst = (Tb + TC_OVH) / share;         // CTAs holding its real tiles
      const int npieces = (Tb + g.tb - 1) / share - cfirst + 1;
      const int64_t pbase = ((int64_t)bh * P.npiece + ((int)blockIdx.x - cfirst)) * R;
      const int d = t;
#pragma unroll
      for (int r = 0; r < RN; ++r) {
        if (r >= R) continue;
        const float L = (S.red[0][r] + S.red[1][r]) + (S.red[2][r] + S.red[3][r]);
        const float acc = __uint_as_float(o[r]);
        if (npieces == 1) {
          const int j = r / P.group, hq = h * P.group + r % P.group;
          out[b * P.obs + j * P.oqs + hq * P.ohs + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
        } else {
          P.part_acc[(pbase + r) * MT_D + d] = acc;
          if (d == 0) {
            P.part_ml[(pbase + r) * 2] = m[r] == -INFINITY ? -INFINITY : m[r] * 0.6931471805599453f;
            P.part_ml[(pbase + r) * 2 + 1] = L;
          }
        }
      }
      if (npieces > 1) {
        __threadfence();
        tc_sbar();
        if (t == 0) S.last = atomicAdd(&P.split_done[bh], 1) == npieces - 1;
        tc_sbar();
        if (S.last) {
          __threadfence();
          if (2 * R * npieces * (int)sizeof(float) <= (int)sizeof(S.p))
            merge_pieces_wide(P, b, h, npieces, t, reinterpret_cast<float*>(&S.p[0][0]), out,
                              tc_sbar);
          else
            merge_pieces(P, b, h, npieces, w, lane, out);
        }
      }
      tc_sbar();                                       // S.red and S.last reused next segment
      ++seg;
      more = tc_seg_next(g, P) && tc_seg_real(g, P);
    }
  }
  // ---------------- teardown: TMEM back once every role is done with it
  tc_fence_before();
  __syncthreads();
  if (w == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :: "r"(tm), "r"(TC_TMEM_COLS) : "memory");
  }
  if (t == 0 && S.abort_) atomicOr(P.status, 1);
}

static int nsplit_for(int C, int qlen) {
  const int maxkeys = C + qlen;
  return (maxkeys + SPLIT_KEYS - 1) / SPLIT_KEYS;
}

// Persistent grid of the tensor-core kernel: SMs x resident CTAs, looked up
// once per device.
template <int NT>
static int launch_mma(const AttnParams& P, cudaStream_t st) {
  static std::atomic<int> grid_of[SD_MAX_DEVICES];
  const int sm = (int)sizeof(MmaSmem);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SD_ELAUNCH;
  if (cudaFuncSetAttribute(attn_mma_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm) !=
      cudaSuccess)
    return SD_ELAUNCH;
  int g = dev < SD_MAX_DEVICES ? grid_of[dev].load() : 0;
  if (g == 0) {
    int nsm = 0, occ = 0;
    if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, attn_mma_kernel<NT>, MT_THREADS, sm) !=
            cudaSuccess)
      return SD_ELAUNCH;
    g = nsm * (occ > 0 ? occ : 1);
    if (dev < SD_MAX_DEVICES) grid_of[dev].store(g);
  }
  attn_mma_kernel<NT><<<g, MT_THREADS, sm, st>>>(P);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library)
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::atomic<void*> fn{nullptr};
  void* f = fn.load();
  if (f == nullptr) {
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) !=
            cudaSuccess || qr != cudaDriverEntryPointSuccess || f == nullptr)
      return nullptr;
    fn.store(f);
  }
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
}

// 2D map over a [B, Hkv, C, 128] bf16 cache viewed as [B * Hkv * C, 128]:
// boxes of 128 rows x 64 columns (128 B), 128-byte swizzle, zero fill
static bool cache_map(CUtensorMap* map, const void* base, int64_t rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)MT_D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)MT_D * 2};
  const cuuint32_t box[2] = {64u, (cuuint32_t)TC_KEYS};
  const cuuint32_t estr[2] = {1u, 1u};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int NTG>
static int launch_tc_ntg(const AttnParams& P, const CUtensorMap& mk, const CUtensorMap& mv,
                         int nsm, cudaStream_t st) {
  const int sm = (int)sizeof(TcSmem) + 1024;         // + room to align to 1024 B
  if (cudaFuncSetAttribute(attn_tc_kernel<NTG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           sm) != cudaSuccess)
    return SD_ELAUNCH;
  attn_tc_kernel<NTG><<<nsm, TC_THREADS, sm, st>>>(P, mk, mv);
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

static int launch_tc(const AttnParams& P, cudaStream_t st) {
  const int64_t rows = P.bt ? (int64_t)P.npages * P.Hkv * SD_KV_PAGE : (int64_t)P.B * P.Hkv * P.C;
  if (rows >= (int64_t)1 << 31) return SD_ENOTSUP;
  CUtensorMap mk, mv;
  if (!cache_map(&mk, P.k, rows) || !cache_map(&mv, P.v, rows)) return SD_ENOTSUP;
  int dev = 0, nsm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return SD_ELAUNCH;
  switch ((P.R + 7) / 8) {
    case 1: return launch_tc_ntg<1>(P, mk, mv, nsm, st);
    case 2: return launch_tc_ntg<2>(P, mk, mv, nsm, st);
    case 3: return launch_tc_ntg<3>(P, mk, mv, nsm, st);
    default: return launch_tc_ntg<4>(P, mk, mv, nsm, st);
  }
}

// Which kernel takes the tensor-core shapes: tcgen05 (default) or the
// mma.sync kernel (SD_ATTN_KERNEL=mma, kept for comparison).
static bool use_tcgen05() {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("SD_ATTN_KERNEL");
    mode = (e && e[0] == 'm') ? 0 : 1;
  }
  return mode == 1;
}

}  // namespace sd

using namespace sd;

extern "C" {

size_t sd_verify_attn_workspace_bytes(int B, int Hq, int Hkv, int D, int C, int qlen) {
  if (B <= 0 || Hkv <= 0 || Hq % Hkv) return 0;
  const int R = qlen * (Hq / Hkv);
  const size_t np = (size_t)nsplit_for(C, qlen) + 1;   // pieces per (row, kv head), either path
  return (size_t)B * Hkv * np * R * (D + 2) * sizeof(float) +
         ((size_t)B * Hkv + 2 * (size_t)B + 2) * sizeof(int) + 256;
}

}  // extern "C"

namespace sd {
static int verify_attn(const void* q, int64_t qbs, int64_t qhs, int64_t qqs, const void* kcache,
                       const void* vcache, const int32_t* bt, int bt_stride, int npages,
                       const int64_t* lengths, const int64_t* valid, int B, int Hq, int Hkv, int D,
                       int C, int qlen, float scale, void* out, int64_t obs, int64_t oqs,
                       int64_t ohs, int dtype, void* workspace, size_t workspace_bytes,
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
  P.out_vec4 = (reinterpret_cast<uintptr_t>(out) & 7) == 0 && obs % 4 == 0 && oqs % 4 == 0 &&
               ohs % 4 == 0;
  float* ws = reinterpret_cast<float*>(workspace);
  P.part_acc = ws;
  P.npiece = P.nsplit + 1;
  P.part_ml = ws + (size_t)B * Hkv * P.npiece * P.R * D;
  P.split_done = reinterpret_cast<int*>(P.part_ml + (size_t)B * Hkv * P.npiece * P.R * 2);
  P.rowpre = P.split_done + (size_t)B * Hkv;
  P.rowkmax = P.rowpre + B + 1;
  P.status = P.rowkmax + B;
  P.tile_keys = MT_KEYS;
  P.seg_ovh = 0;
  P.bt = bt; P.bt_stride = bt_stride; P.npages = npages;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // tensor-core path: bf16, head_dim 128, <= 32 query rows per kv head,
  // 16-byte aligned rows
  const bool mma_ok = dtype == SD_DTYPE_BF16 && D == MT_D && P.R <= 32 &&
                      (reinterpret_cast<uintptr_t>(q) & 15) == 0 && qbs % 8 == 0 &&
                      qhs % 8 == 0 && qqs % 8 == 0 &&
                      (reinterpret_cast<uintptr_t>(kcache) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(vcache) & 15) == 0;
  if (mma_ok && use_tcgen05()) {
    P.nrc = 1;
    P.tile_keys = TC_KEYS;
    P.seg_ovh = TC_OVH;
    attn_plan_kernel<<<1, 1024, 0, st>>>(P);
    if (cudaGetLastError() != cudaSuccess) return SD_ELAUNCH;
    return launch_tc(P, st);
  }
  if (mma_ok) {
    P.nrc = 1;
    attn_plan_kernel<<<1, 1024, 0, st>>>(P);
    switch ((P.R + 7) / 8) {
      case 1: return launch_mma<1>(P, st);
      case 2: return launch_mma<2>(P, st);
      case 3: return launch_mma<3>(P, st);
      default: return launch_mma<4>(P, st);
    }
  }
  const unsigned grid = (unsigned)(B * Hkv * P.nrc * P.nsplit);
  if (dtype == SD_DTYPE_BF16) {
    const size_t sm = sizeof(AttnSmem<__nv_bfloat16>);
    cudaFuncSetAttribute(attn_split_kernel<__nv_bfloat16>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    attn_split_kernel<__nv_bfloat16><<<grid, AT, sm, st>>>(P);
    attn_combine_kernel<__nv_bfloat16><<<B * Hkv * P.R, D, 0, st>>>(P);
  } else {
    const size_t sm = sizeof(AttnSmem<float>);
    cudaFuncSetAttribute(attn_split_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sm);
    attn_split_kernel<float><<<grid, AT, sm, st>>>(P);
    attn_combine_kernel<float><<<B * Hkv * P.R, D, 0, st>>>(P);
  }
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}
}  // namespace sd

extern "C" {

int sd_verify_attn(const void* q, int64_t qbs, int64_t qhs, int64_t qqs, const void* kcache,
                   const void* vcache, const int64_t* lengths, const int64_t* valid, int B, int Hq,
                   int Hkv, int D, int C, int qlen, float scale, void* out, int64_t obs,
                   int64_t oqs, int64_t ohs, int dtype, void* workspace, size_t workspace_bytes,
                   void* stream) {
  return sd::verify_attn(q, qbs, qhs, qqs, kcache, vcache, nullptr, 0, 0, lengths, valid, B, Hq,
                         Hkv, D, C, qlen, scale, out, obs, oqs, ohs, dtype, workspace,
                         workspace_bytes, stream);
}

int sd_verify_attn_paged(const void* q, int64_t qbs, int64_t qhs, int64_t qqs, const void* kpool,
                         const void* vpool, const int32_t* block_table, int bt_stride, int npages,
                         const int64_t* lengths, const int64_t* valid, int B, int Hq, int Hkv,
                         int D, int qlen, float scale, void* out, int64_t obs, int64_t oqs,
                         int64_t ohs, int dtype, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (!block_table || bt_stride <= 0 || npages <= 0) return SD_EINVAL;
  if ((int64_t)bt_stride * SD_KV_PAGE > 0x7FFFFFFF) return SD_ENOTSUP;
  return sd::verify_attn(q, qbs, qhs, qqs, kpool, vpool, block_table, bt_stride, npages, lengths,
                         valid, B, Hq, Hkv, D, bt_stride * SD_KV_PAGE, qlen, scale, out, obs, oqs,
                         ohs, dtype, workspace, workspace_bytes, stream);
}

}  // extern "C"
