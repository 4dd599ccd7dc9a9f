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

#include <atomic>

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
  if (t == 0) carry = 0;
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
    const int tiles = (km + MT_KEYS - 1) / MT_KEYS;
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
    const __nv_bfloat16* kb = reinterpret_cast<const __nv_bfloat16*>(P.k) +
                              ((int64_t)b * Hkv + h) * P.C * MT_D;
    const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(P.v) +
                              ((int64_t)b * Hkv + h) * P.C * MT_D;
    auto load_tile = [&](int tile, int buf) {
      const int key0 = s0 + tile * MT_KEYS;
      const uint32_t kd = smem_addr(S.u.kv.k[buf]), vd = smem_addr(S.u.kv.v[buf]);
      for (int i = t; i < MT_KEYS * 16; i += MT_THREADS) {
        const int kk = i >> 4, c = i & 15;
        const bool in = key0 + kk < s1;
        const int64_t row = in ? key0 + kk : s0;       // a valid address when nothing is read
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

}  // namespace sd

using namespace sd;

extern "C" {

size_t sd_verify_attn_workspace_bytes(int B, int Hq, int Hkv, int D, int C, int qlen) {
  if (B <= 0 || Hkv <= 0 || Hq % Hkv) return 0;
  const int R = qlen * (Hq / Hkv);
  const size_t np = (size_t)nsplit_for(C, qlen) + 1;   // pieces per (row, kv head), either path
  return (size_t)B * Hkv * np * R * (D + 2) * sizeof(float) +
         ((size_t)B * Hkv + 2 * (size_t)B + 1) * sizeof(int) + 256;
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
  P.out_vec4 = (reinterpret_cast<uintptr_t>(out) & 7) == 0 && obs % 4 == 0 && oqs % 4 == 0 &&
               ohs % 4 == 0;
  float* ws = reinterpret_cast<float*>(workspace);
  P.part_acc = ws;
  P.npiece = P.nsplit + 1;
  P.part_ml = ws + (size_t)B * Hkv * P.npiece * P.R * D;
  P.split_done = reinterpret_cast<int*>(P.part_ml + (size_t)B * Hkv * P.npiece * P.R * 2);
  P.rowpre = P.split_done + (size_t)B * Hkv;
  P.rowkmax = P.rowpre + B + 1;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // tensor-core path: bf16, head_dim 128, <= 32 query rows per kv head,
  // 16-byte aligned rows
  const bool mma_ok = dtype == SD_DTYPE_BF16 && D == MT_D && P.R <= 32 &&
                      (reinterpret_cast<uintptr_t>(q) & 15) == 0 && qbs % 8 == 0 &&
                      qhs % 8 == 0 && qqs % 8 == 0 &&
                      (reinterpret_cast<uintptr_t>(kcache) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(vcache) & 15) == 0;
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

}  // extern "C"
