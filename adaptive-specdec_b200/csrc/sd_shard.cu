// Vocabulary-sharded verify round (sm_100a): the SPMD form of the fused
// verify-sample for a vocab-parallel LM head.
//
// Every rank holds the columns [v_start[r], v_start[r+1]) of every target and
// draft logits vector.  The arithmetic is the single-device contract of
// specdec/sampling.py:42-67 and specdec/engine.py:282-303 as restated by the
// fused kernel: d = fl(x / T), e = expf(fl(d - m)) with m the GLOBAL maximum,
// p = fl(e * fl(1 / S)), top-p over (p desc, index asc) with the cumulative
// mass in float64, p' = fl(p / max(fl(Z), 1e-12)), the accept test
// u < min(1, fl(p'(x) / max(q'(x), 1e-10))), and the inverse-CDF draw from the
// residual max(fl(p' - q'), 0) (or p' itself for the bonus / degenerate case)
// in vocabulary order with float64 prefix sums.
//
// Messages between the phases (the caller runs the collectives):
//   P1  -> all_gather : per vector (shard max of d, d at the probe token if
//                       this shard holds it)                       8 B
//   P2  -> all_reduce : per vector (S of the shard, 128-bin e-mass histogram
//                       of depth -t in 1/8 base-2 units)           1032 B
//   P3  -> all_gather : per vector (shard mass of the bins above the
//                       boundary, boundary elements (p, index))    1040 B
//   P4  -> all_gather : per row (shard residual mass, shard p' mass) 16 B
//   P5  -> all_reduce : per row drawn token id or -1 (max)          8 B
//   greedy P1 -> all_reduce(max): per target vector (argmax key)    8 B
// Only the top-p boundary bins are sorted, across all shards; every other
// decision is a sum or a maximum over shards.
#include <cuda_runtime.h>
#include <stdint.h>

#include "sd_common.cuh"

namespace sd {
namespace shard {

constexpr int NT = 256;                   // threads per CTA
constexpr int PSPLIT = 8;                 // CTAs per row of the per-row phases (P4b, P5)
constexpr int NB = 128;                   // depth bins
constexpr float BPU = 8.f;                // bins per base-2 unit (window 16 units)
constexpr int CAP = SD_SHARD_BOUNDARY_CAP;
constexpr int SORT_MAX = SD_SHARD_MAX_RANKS * CAP;   // boundary entries sorted per vector
constexpr double DELTA = 1e-5;            // bound on the error of the binned p-masses
constexpr int F_FALLBACK = 1;             // message flag: this round needs full vectors

struct Msg1 { float m; float dx; };
struct Msg3 {
  double pre;                   // mass of this shard's elements above the boundary bins
  int n;                        // boundary elements of this shard (may exceed CAP)
  int flags;
  unsigned long long e[CAP];    // (fkey(p) << 32) | (~index)
};
static_assert(sizeof(Msg3) == 16 + 8 * CAP, "Msg3 layout");

// per-vector state kept between phases
struct Vec {
  float m, dx, inv_s, zf;
  int lo, hi;                   // bins < lo kept; lo..hi decided by the cut; > hi dropped
  int flags, pad;
  unsigned long long cut;       // smallest kept key inside lo..hi
  double S;
};
struct Row {
  int n_acc, pick, all_acc, pad;
};

struct Geo {
  int B, k, per, nvec, Vr, v0, V, rank, nranks, dtype;
  float T, top_p;
  bool truncate;
};

__device__ __forceinline__ int depth_bin(float t) {        // t = fl(d - m) <= 0
  const float y = __fmul_rn(-t, BPU * 1.4426950408889634f);
  return y < (float)NB ? (int)y : NB;                       // NB: below the window
}
__device__ __forceinline__ unsigned long long pkey(float p, int64_t j) {
  return ((unsigned long long)fkey(p) << 32) | (0xFFFFFFFFull - (unsigned long long)j);
}
__device__ __forceinline__ float pkey_val(unsigned long long k) {
  const uint32_t u = (uint32_t)(k >> 32);
  const uint32_t b = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  return __uint_as_float(b);
}

__device__ __forceinline__ const void* vec_base(const sd_shard_args& a, const Geo& g, int v,
                                                int* b_out, int* set_out, int* pos_out) {
  const int b = v / g.per, l = v - b * g.per;
  const int set = l <= g.k ? 0 : 1;
  const int pos = set ? l - (g.k + 1) : l;
  *b_out = b; *set_out = set; *pos_out = pos;
  const int esz = g.dtype == SD_DTYPE_F32 ? 4 : 2;
  const char* base = reinterpret_cast<const char*>(set ? a.drf : a.tgt);
  const int64_t off = set ? (b * a.drf_bs + pos * a.drf_ps) : (b * a.tgt_bs + pos * a.tgt_ps);
  return base + off * esz;
}
// global vocabulary id of the probe token of vector (set, pos), or -1
__device__ __forceinline__ int64_t probe_of(const sd_shard_args& a, const Geo& g, int b, int pos) {
  if (pos >= g.k) return -1;
  return a.xs[b * a.xs_bs + pos];
}
__device__ __forceinline__ int owner_of(const sd_shard_args& a, int64_t x) {
  int r = 0;
  while (r + 1 < a.nranks && x >= a.v_start[r + 1]) ++r;
  return r;
}

// p' of an element with scaled logit d under the vector's state (the kept
// predicate: bins above lo, the cut inside lo..hi, nothing below hi)
__device__ __forceinline__ float pprime(const Vec& s, float d, int64_t j) {
  const float t = __fsub_rn(d, s.m);
  const float e = expf(t);
  const float p = __fmul_rn(e, s.inv_s);
  const int bin = depth_bin(t);
  const bool kept = bin < s.lo || (bin <= s.hi && pkey(p, j) >= s.cut);
  return kept ? __fdiv_rn(p, s.zf) : 0.f;
}

// Calls f(j, x_j) for every element j of [j0, j1) of a logits slice (bf16,
// fp16 or fp32), a block's threads striding over it: scalar elements up to
// the first 16-byte boundary, then 16-byte units (8 or 4 elements per load),
// then the scalar tail.  The order of the calls is unspecified.
template <typename F>
__device__ __forceinline__ void slice_range_for_each(const void* x, int dtype, int j0, int j1,
                                                     F&& f) {
  if (j1 <= j0) return;
  const int esz = dtype == SD_DTYPE_F32 ? 4 : 2;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(x) + (uintptr_t)j0 * esz;
  int head = (int)(((16u - (uint32_t)(a0 & 15u)) & 15u) / (uint32_t)esz);
  if ((a0 & (uintptr_t)(esz - 1)) != 0 || head > j1 - j0) head = j1 - j0;   // (elements are aligned)
  const int epu = 16 / esz;
  const int nunits = (j1 - j0 - head) / epu;
  const int b0 = j0 + head, tail0 = b0 + nunits * epu;
  for (int j = j0 + threadIdx.x; j < b0; j += NT) f(j, load_logit(x, dtype, j));
  const uint4* body = reinterpret_cast<const uint4*>(static_cast<const char*>(x) + (size_t)b0 * esz);
  if (esz == 4) {
    for (int u = threadIdx.x; u < nunits; u += NT) {
      const uint4 w = __ldg(body + u);
      const int j = b0 + u * 4;
      f(j, __uint_as_float(w.x));
      f(j + 1, __uint_as_float(w.y));
      f(j + 2, __uint_as_float(w.z));
      f(j + 3, __uint_as_float(w.w));
    }
  } else {
    for (int u = threadIdx.x; u < nunits; u += NT) {
      const uint4 w = __ldg(body + u);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
      const int j = b0 + u * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) f(j + e, bits16_to_float((ww[e >> 1] >> (16 * (e & 1))) & 0xFFFFu, dtype));
    }
  }
  for (int j = tail0 + threadIdx.x; j < j1; j += NT) f(j, load_logit(x, dtype, j));
}
template <typename F>
__device__ __forceinline__ void slice_for_each(const void* x, int dtype, int n, F&& f) {
  slice_range_for_each(x, dtype, 0, n, f);
}

// The same over [j0, j1) of two slices read in step, f(j, a_j, b_j): 16-byte
// units when both slices sit at the same offset modulo 16 bytes (rows of a
// contiguous slice tensor do when the slice width times the element size is a
// multiple of 16: even_split's default boundaries give that), element by
// element otherwise.
template <typename F>
__device__ __forceinline__ void slice2_range_for_each(const void* xa, const void* xb, int dtype,
                                                      int j0, int j1, F&& f) {
  if (j1 <= j0) return;
  const int esz = dtype == SD_DTYPE_F32 ? 4 : 2;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(xa) + (uintptr_t)j0 * esz;
  const uintptr_t c0 = reinterpret_cast<uintptr_t>(xb) + (uintptr_t)j0 * esz;
  if ((a0 & 15u) != (c0 & 15u) || (a0 & (uintptr_t)(esz - 1)) != 0) {
    for (int j = j0 + threadIdx.x; j < j1; j += NT)
      f(j, load_logit(xa, dtype, j), load_logit(xb, dtype, j));
    return;
  }
  int head = (int)(((16u - (uint32_t)(a0 & 15u)) & 15u) / (uint32_t)esz);
  if (head > j1 - j0) head = j1 - j0;
  const int epu = 16 / esz;
  const int nunits = (j1 - j0 - head) / epu;
  const int b0 = j0 + head, tail0 = b0 + nunits * epu;
  for (int j = j0 + threadIdx.x; j < b0; j += NT)
    f(j, load_logit(xa, dtype, j), load_logit(xb, dtype, j));
  const uint4* ba = reinterpret_cast<const uint4*>(static_cast<const char*>(xa) + (size_t)b0 * esz);
  const uint4* bb = reinterpret_cast<const uint4*>(static_cast<const char*>(xb) + (size_t)b0 * esz);
  for (int u = threadIdx.x; u < nunits; u += NT) {
    const uint4 wa = __ldg(ba + u), wb = __ldg(bb + u);
    const uint32_t va[4] = {wa.x, wa.y, wa.z, wa.w}, vb[4] = {wb.x, wb.y, wb.z, wb.w};
    const int j = b0 + u * epu;
    if (esz == 4) {
#pragma unroll
      for (int e = 0; e < 4; ++e) f(j + e, __uint_as_float(va[e]), __uint_as_float(vb[e]));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int sh = 16 * (e & 1);
        f(j + e, bits16_to_float((va[e >> 1] >> sh) & 0xFFFFu, dtype),
          bits16_to_float((vb[e >> 1] >> sh) & 0xFFFFu, dtype));
      }
    }
  }
  for (int j = tail0 + threadIdx.x; j < j1; j += NT)
    f(j, load_logit(xa, dtype, j), load_logit(xb, dtype, j));
}

// ---- P1: shard maximum of d and the probe's d ------------------------------
__global__ void __launch_bounds__(NT) p1_kernel(const sd_shard_args a, Geo g, Msg1* send) {
  __shared__ float red[32];
  const int v = blockIdx.x;
  int b, set, pos;
  const void* x = vec_base(a, g, v, &b, &set, &pos);
  // max_j fl(x_j / T) = fl(max_j x_j / T): dividing by T > 0 and rounding are
  // monotone, so one division after the maximum of the logits
  float mx = -INFINITY;
  slice_for_each(x, g.dtype, g.Vr, [&](int, float xv) { mx = fmaxf(mx, xv); });
  mx = block_max(mx, red, -INFINITY);
  mx = scaled_logit(mx, g.T);
  if (threadIdx.x == 0) {
    const int64_t xp = probe_of(a, g, b, pos);
    float dx = __int_as_float(0x7FC00000);             // NaN: not held here
    if (xp >= g.v0 && xp < g.v0 + g.Vr) dx = scaled_logit(load_logit(x, g.dtype, xp - g.v0), g.T);
    send[v].m = mx;
    send[v].dx = dx;
  }
}

// ---- P2: global m; shard S and the depth histogram ---------------------------
__global__ void __launch_bounds__(NT) p2_kernel(const sd_shard_args a, Geo g, const Msg1* recv,
                                                Vec* st, double* send) {
  __shared__ double bins[NB];
  __shared__ double red[33];
  const int v = blockIdx.x;
  int b, set, pos;
  const void* x = vec_base(a, g, v, &b, &set, &pos);
  float m = -INFINITY;
  for (int r = 0; r < g.nranks; ++r) m = fmaxf(m, recv[(size_t)r * g.nvec + v].m);
  for (int i = threadIdx.x; i < NB; i += NT) bins[i] = 0.0;
  __syncthreads();
  double s = 0.0;
  slice_for_each(x, g.dtype, g.Vr, [&](int, float xv) {
    const float t = __fsub_rn(scaled_logit(xv, g.T), m);
    const float e = expf(t);
    s += (double)e;
    if (g.truncate) {
      const int bin = depth_bin(t);
      if (bin < NB) atomicAdd(&bins[bin], (double)e);
    }
  });
  s = block_sum(s, red);
  __syncthreads();
  double* out = send + (size_t)v * (1 + NB);
  if (threadIdx.x == 0) {
    out[0] = s;
    const int64_t xp = probe_of(a, g, b, pos);
    st[v].m = m;
    st[v].dx = xp >= 0 && xp < g.V ? recv[(size_t)owner_of(a, xp) * g.nvec + v].dx
                                   : __int_as_float(0x7FC00000);
  }
  for (int i = threadIdx.x; i < NB; i += NT) out[1 + i] = bins[i];
}

// ---- P3: S, the boundary bins, the shard's pre-kept mass and boundary list ---
__global__ void __launch_bounds__(NT) p3_kernel(const sd_shard_args a, Geo g, const double* recv,
                                                Vec* st, Msg3* send) {
  __shared__ double red[33];
  __shared__ int cnt, lo_s, hi_s, fl_s;
  __shared__ float inv_s_s;
  const int v = blockIdx.x;
  int b, set, pos;
  const void* x = vec_base(a, g, v, &b, &set, &pos);
  const double* in = recv + (size_t)v * (1 + NB);
  const float m = st[v].m;
  if (threadIdx.x == 0) {
    const double S = in[0];
    const float inv_s = __double2float_rn(1.0 / S);
    int lo = NB + 1, hi = NB, fl = 0;                  // no truncation: everything kept
    if (g.truncate) {
      const double tp = (double)g.top_p;
      double A = 0.0;
      int lo_b = -1, hi_b = -1;
      for (int i = 0; i < NB; ++i) {
        const double mb = in[1 + i] * (double)inv_s;
        if (lo_b < 0 && A + mb > tp - DELTA) lo_b = i;
        if (A < tp + DELTA) hi_b = i;
        A += mb;
      }
      if (A < tp + DELTA || lo_b < 0 || hi_b >= NB - 1) {
        fl = F_FALLBACK;                               // boundary not inside the window
        lo = 0; hi = -1;
      } else {
        lo = lo_b > 0 ? lo_b - 1 : 0;                  // one bin of margin on each side:
        hi = hi_b + 1;                                 // p ties across a bin edge stay together
      }
    }
    st[v].S = S;
    st[v].inv_s = inv_s;
    st[v].lo = lo;
    st[v].hi = hi;
    st[v].flags = fl;
    inv_s_s = inv_s; lo_s = lo; hi_s = hi; fl_s = fl; cnt = 0;
  }
  __syncthreads();
  const float inv_s = inv_s_s;
  const int lo = lo_s, hi = hi_s;
  Msg3& o = send[v];
  double pre = 0.0;
  slice_for_each(x, g.dtype, g.Vr, [&](int j, float xv) {
    const float t = __fsub_rn(scaled_logit(xv, g.T), m);
    const int bin = depth_bin(t);
    if (bin < lo) {
      pre += (double)__fmul_rn(expf(t), inv_s);
    } else if (bin <= hi) {
      const float p = __fmul_rn(expf(t), inv_s);
      const int i = atomicAdd(&cnt, 1);
      if (i < CAP) o.e[i] = pkey(p, (int64_t)g.v0 + j);
    }
  });
  pre = block_sum(pre, red);
  __syncthreads();
  if (threadIdx.x == 0) {
    o.pre = pre;
    o.n = cnt;
    o.flags = fl_s | (cnt > CAP ? F_FALLBACK : 0);
  }
}

// ---- P4a: per vector, the cut inside the boundary bins and the kept mass ----
__global__ void __launch_bounds__(NT) p4a_kernel(Geo g, const Msg3* recv, Vec* st,
                                                 uint32_t* status) {
  __shared__ unsigned long long key[SORT_MAX];
  __shared__ int ntot_s;
  const int v = blockIdx.x;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int r = 0; r < g.nranks; ++r) n += min(recv[(size_t)r * g.nvec + v].n, CAP);
    ntot_s = n;
  }
  __syncthreads();
  const int ntot = ntot_s;
  int N = 1;
  while (N < ntot) N <<= 1;
  // gather every shard's boundary entries (rank order), pad with the smallest key
  for (int i = threadIdx.x; i < N; i += NT) key[i] = 0ull;
  __syncthreads();
  {
    int off = 0;
    for (int r = 0; r < g.nranks; ++r) {
      const Msg3& m = recv[(size_t)r * g.nvec + v];
      const int n = min(m.n, CAP);
      for (int i = threadIdx.x; i < n; i += NT) key[off + i] = m.e[i];
      off += n;
    }
  }
  __syncthreads();
  for (int k2 = 2; k2 <= N; k2 <<= 1)                  // bitonic sort, descending
    for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
      for (int i = threadIdx.x; i < N; i += NT) {
        const int ixj = i ^ j2;
        if (ixj > i) {
          const unsigned long long x = key[i], y = key[ixj];
          const bool desc = (i & k2) == 0;
          if (desc ? (x < y) : (x > y)) { key[i] = y; key[ixj] = x; }
        }
      }
      __syncthreads();
    }
  if (threadIdx.x == 0) {
    Vec& s = st[v];
    double pre = 0.0;
    int fl = s.flags;
    for (int r = 0; r < g.nranks; ++r) {
      pre += recv[(size_t)r * g.nvec + v].pre;
      fl |= recv[(size_t)r * g.nvec + v].flags;
    }
    double Z = pre;
    unsigned long long cut = ~0ull;                    // nothing of lo..hi kept yet
    if (g.truncate && !(fl & F_FALLBACK)) {
      // the reference's rule on the sorted boundary entries: keep while
      // fl32(fl32(cum) - p) < top_p, cum in float64; keep[0] when no bin lies above
      double cum = pre;
      for (int i = 0; i < ntot; ++i) {
        const float p = pkey_val(key[i]);
        cum += (double)p;
        const float c = __fsub_rn(__double2float_rn(cum), p);
        if (c < g.top_p || (i == 0 && s.lo == 0)) {
          cut = key[i];
          Z += (double)p;
        } else {
          break;
        }
      }
    }
    float zf = __double2float_rn(Z);
    if (zf < 1e-12f) zf = 1e-12f;
    s.cut = cut;
    s.zf = zf;
    s.flags = fl;
    if (fl & F_FALLBACK) atomicOr(status, (uint32_t)SD_SHARD_STATUS_FALLBACK);
  }
}

// ---- P4b: per row, the accept test and the shard's residual mass ------------
__global__ void __launch_bounds__(NT) p4b_kernel(const sd_shard_args a, Geo g, const Vec* st,
                                                 Row* rows, double* psum) {
  __shared__ double red[33];
  __shared__ int pick_s, all_s;
  const int b = blockIdx.x, part = blockIdx.y;         // part: 1/PSPLIT of the slice
  if (threadIdx.x == 0) {                              // engine.py:286-294 (every part; part 0 writes)
    bool alive = a.alive ? a.alive[b] != 0 : true;
    int n = 0;
    for (int i = 0; i < g.k; ++i) {
      const Vec& sp = st[b * g.per + i];
      const Vec& sq = st[b * g.per + g.k + 1 + i];
      const int64_t x = a.xs[b * a.xs_bs + i];
      const bool in = x >= 0 && x < g.V;
      const float px = in ? pprime(sp, sp.dx, x) : 0.f;
      const float qx = in ? pprime(sq, sq.dx, x) : 0.f;
      const float ratio = __fdiv_rn(px, fmaxf(qx, 1e-10f));
      const float thr = fminf(ratio, 1.f);
      const bool ok = alive && n == i && a.u_acc[b * a.u_bs + i] < thr;
      n += ok ? 1 : 0;
      alive = alive && ok;
    }
    const int all_acc = n == g.k;
    const int pick = min(n, g.k - 1);
    if (part == 0) {
      rows[b].n_acc = n;
      rows[b].pick = pick;
      rows[b].all_acc = all_acc;
    }
    pick_s = pick;
    all_s = all_acc;
  }
  __syncthreads();
  const int all_acc = all_s, pick = pick_s;
  const int vp = b * g.per + (all_acc ? g.k : pick);
  const int vq = b * g.per + g.k + 1 + pick;
  int bb, set, pos;
  const void* xp = vec_base(a, g, vp, &bb, &set, &pos);
  const void* xq = vec_base(a, g, vq, &bb, &set, &pos);
  const Vec sp = st[vp], sq = st[vq];
  double R = 0.0, Pm = 0.0;
  const int seg = (g.Vr + PSPLIT - 1) / PSPLIT;
  const int j1 = min(g.Vr, (part + 1) * seg);
  if (all_acc) {                                       // the bonus draw: p alone
    slice_range_for_each(xp, g.dtype, part * seg, j1, [&](int j, float xv) {
      const float pj = pprime(sp, scaled_logit(xv, g.T), (int64_t)g.v0 + j);
      R += (double)pj;
      Pm += (double)pj;
    });
  } else {
    slice2_range_for_each(xp, xq, g.dtype, part * seg, j1, [&](int j, float xpv, float xqv) {
      const int64_t gj = (int64_t)g.v0 + j;
      const float pj = pprime(sp, scaled_logit(xpv, g.T), gj);
      const float qj = pprime(sq, scaled_logit(xqv, g.T), gj);
      R += (double)fmaxf(__fsub_rn(pj, qj), 0.f);
      Pm += (double)pj;
    });
  }
  R = block_sum(R, red);
  __syncthreads();
  Pm = block_sum(Pm, red);
  if (threadIdx.x == 0) {                              // this part's sums, in its own slot
    psum[((size_t)b * PSPLIT + part) * 2] = R;
    psum[((size_t)b * PSPLIT + part) * 2 + 1] = Pm;
  }
}

// P4c: per row, the shard's (R, Pm) as the parts' sums added in part order,
// so the totals every rank agrees on are reproducible from run to run (and
// are the sums of the part masses that P5 walks).
__global__ void p4c_kernel(Geo g, const double* psum, double* send) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= g.B) return;
  double R = 0.0, Pm = 0.0;
  for (int p = 0; p < PSPLIT; ++p) {
    R += psum[((size_t)b * PSPLIT + p) * 2];
    Pm += psum[((size_t)b * PSPLIT + p) * 2 + 1];
  }
  send[2 * b] = R;
  send[2 * b + 1] = Pm;
}

// ---- P5: per row, the shard that holds the draw walks its slice -------------
// The row's draw state on this shard (every thread computes it): mode 1 when
// this shard's prefix interval holds t = u * total, 2 when nobody's does (t
// at or past the total: every shard offers its last nonzero index), 0 when
// another shard holds it; the offset of this shard's prefix; and the two
// vectors whose masses are drawn from.
struct Draw {
  int mode, all_acc, degen;
  double base, t;
  const void* xp;
  const void* xq;
  Vec sp, sq;
};
__device__ __forceinline__ Draw draw_state(const sd_shard_args& a, const Geo& g, const double* recv,
                                           const Vec* st, const Row* rows, int b) {
  Draw d;
  d.all_acc = rows[b].all_acc;
  double Rt = 0.0;
  for (int r = 0; r < g.nranks; ++r) Rt += recv[(size_t)r * 2 * g.B + 2 * b];
  // engine.py:297-303 / sampling.py:85-89: a residual of (near) zero mass
  // falls back to p; the bonus draw uses p itself
  d.degen = !d.all_acc && __double2float_rn(Rt) <= 1e-9f;
  const int use = (d.all_acc || d.degen) ? 1 : 0;
  double total = 0.0, before = 0.0;
  for (int r = 0; r < g.nranks; ++r) {
    const double w = recv[(size_t)r * 2 * g.B + 2 * b + use];
    if (r < g.rank) before += w;
    total += w;
  }
  const double mine = recv[(size_t)g.rank * 2 * g.B + 2 * b + use];
  d.t = (double)a.u_res[b] * total;
  d.mode = (d.t >= total) ? 2 : ((mine > 0.0 && before <= d.t && d.t < before + mine) ? 1 : 0);
  d.base = before;
  const int pick = rows[b].pick;
  const int vp = b * g.per + (d.all_acc ? g.k : pick);
  const int vq = b * g.per + g.k + 1 + pick;
  int bb, set, pos;
  d.xp = vec_base(a, g, vp, &bb, &set, &pos);
  d.xq = vec_base(a, g, vq, &bb, &set, &pos);
  d.sp = st[vp];
  d.sq = st[vq];
  return d;
}
__device__ __forceinline__ float draw_mass(const Draw& d, const Geo& g, int j) {
  const int64_t gj = (int64_t)g.v0 + j;
  const float pj = pprime(d.sp, scaled_logit(load_logit(d.xp, g.dtype, j), g.T), gj);
  if (d.all_acc || d.degen) return pj;
  const float qj = pprime(d.sq, scaled_logit(load_logit(d.xq, g.dtype, j), g.T), gj);
  return fmaxf(__fsub_rn(pj, qj), 0.f);
}

// P5a: grid (B, PSPLIT).  Part p of the slice: its float64 mass and its last
// index of nonzero mass (-1: none), for the walk of P5b.
__global__ void __launch_bounds__(NT) p5a_kernel(const sd_shard_args a, Geo g, const double* recv,
                                                 const Vec* st, const Row* rows, double* segm,
                                                 int* segl) {
  __shared__ double red[33];
  __shared__ int lred[32];
  const int b = blockIdx.x, part = blockIdx.y;
  const Draw d = draw_state(a, g, recv, st, rows, b);
  if (d.mode == 0) return;
  const int seg = (g.Vr + PSPLIT - 1) / PSPLIT;
  const int j1 = min(g.Vr, (part + 1) * seg);
  double m = 0.0;
  int last = -1;
  if (d.all_acc || d.degen) {                          // p alone
    slice_range_for_each(d.xp, g.dtype, part * seg, j1, [&](int j, float xv) {
      const float r = pprime(d.sp, scaled_logit(xv, g.T), (int64_t)g.v0 + j);
      m += (double)r;
      if (r > 0.f) last = max(last, j);
    });
  } else {
    slice2_range_for_each(d.xp, d.xq, g.dtype, part * seg, j1, [&](int j, float xpv, float xqv) {
      const int64_t gj = (int64_t)g.v0 + j;
      const float r = fmaxf(__fsub_rn(pprime(d.sp, scaled_logit(xpv, g.T), gj),
                                      pprime(d.sq, scaled_logit(xqv, g.T), gj)), 0.f);
      m += (double)r;
      if (r > 0.f) last = max(last, j);
    });
  }
  m = block_sum(m, red);
  last = block_max(last, lred, -1);
  if (threadIdx.x == 0) {
    segm[b * PSPLIT + part] = m;
    segl[b * PSPLIT + part] = last;
  }
}

// P5b: grid B.  The parts' masses in order locate the part holding the
// crossing; within it (and after it, should float64 rounding carry the
// crossing over) the smallest j with base + sum_{i <= j} r_i > t, a float64
// prefix in chunks of NT; no crossing: the last element of nonzero mass, as
// the reference's inverse CDF falls back to.
__global__ void __launch_bounds__(NT) p5b_kernel(const sd_shard_args a, Geo g, const double* recv,
                                                 const Vec* st, const Row* rows,
                                                 const double* segm, const int* segl,
                                                 int64_t* send) {
  __shared__ double red[33];
  __shared__ int found;
  const int b = blockIdx.x;
  const Draw d = draw_state(a, g, recv, st, rows, b);
  if (d.mode == 0) {
    if (threadIdx.x == 0) send[b] = -1;
    return;
  }
  int best = 0x7FFFFFFF;
  if (d.mode == 1) {
    const int seg = (g.Vr + PSPLIT - 1) / PSPLIT;
    double run = d.base;
    int p0 = PSPLIT;
    for (int p = 0; p < PSPLIT; ++p) {                 // same order in every thread
      const double m = segm[b * PSPLIT + p];
      if (run + m > d.t) { p0 = p; break; }
      run += m;
    }
    if (threadIdx.x == 0) found = 0x7FFFFFFF;
    __syncthreads();
    if (p0 < PSPLIT) {
      for (int c0 = p0 * seg; c0 < g.Vr; c0 += NT) {
        const int j = c0 + threadIdx.x;
        const double r = j < g.Vr ? (double)draw_mass(d, g, j) : 0.0;
        double tot;
        const double ex = block_excl_scan(r, red, &tot);
        if (r > 0.0 && run + ex + r > d.t) atomicMin(&found, j);
        __syncthreads();
        if (found != 0x7FFFFFFF) break;
        run += tot;
      }
    }
    best = found;
  }
  if (threadIdx.x == 0) {
    if (best == 0x7FFFFFFF) {
      best = -1;
      for (int p = 0; p < PSPLIT; ++p) best = max(best, segl[b * PSPLIT + p]);
    }
    send[b] = best >= 0 ? (int64_t)g.v0 + best : -1;
  }
}

// ---- P6: outputs ------------------------------------------------------------
__global__ void p6_kernel(const sd_shard_args a, Geo g, const int64_t* recv, const Row* rows) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= g.B) return;
  a.n_acc[b] = rows[b].n_acc;
  a.y[b] = recv[b];
}

// ---- greedy: per target vector the shard argmax, then the decision ----------
// key = (fkey(x) << 31) | (0x7FFFFFFF - j): the int64 maximum over shards is
// the largest value at its first index (every NaN, whatever its sign bit, takes
// the largest key, as in the fused argmax)
__global__ void __launch_bounds__(NT) g1_kernel(const sd_shard_args a, Geo g, int64_t* send) {
  __shared__ unsigned long long red[32];
  const int v = blockIdx.x;                            // b * (k + 1) + i
  const int b = v / (g.k + 1), i = v - b * (g.k + 1);
  const char* x = reinterpret_cast<const char*>(a.tgt) +
                  (b * a.tgt_bs + i * a.tgt_ps) * (g.dtype == SD_DTYPE_F32 ? 4 : 2);
  unsigned long long best = 0ull;
  slice_for_each(x, g.dtype, g.Vr, [&](int j, float xv) {
    const unsigned long long kk =
        ((unsigned long long)(xv != xv ? 0xFFFFFFFFu : fkey(xv)) << 31) |
        (unsigned long long)(0x7FFFFFFF - (g.v0 + j));
    best = kk > best ? kk : best;
  });
  best = block_max(best, red, 0ull);
  if (threadIdx.x == 0) send[v] = (int64_t)best;
}

__global__ void g6_kernel(const sd_shard_args a, Geo g, const int64_t* recv) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= g.B) return;
  const int k1 = g.k + 1;
  auto amax = [&](int i) -> int64_t {
    return (int64_t)(0x7FFFFFFF - (int)(recv[b * k1 + i] & 0x7FFFFFFF));
  };
  bool alive = a.alive ? a.alive[b] != 0 : true;
  int n = 0;
  for (int i = 0; i < g.k; ++i) {                      // accept iff x_i is the target argmax
    const bool ok = alive && n == i && a.xs[b * a.xs_bs + i] == amax(i);
    n += ok ? 1 : 0;
    alive = alive && ok;
  }
  a.n_acc[b] = n;
  a.y[b] = amax(n);
}

}  // namespace shard
}  // namespace sd

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using namespace sd::shard;

namespace {

constexpr size_t STATUS_BYTES = 256;

size_t vec_bytes(int B, int k) { return (size_t)B * (2 * k + 1) * sizeof(Vec); }
size_t row_bytes(int B) { return (size_t)B * sizeof(Row); }
// P5's part masses [B, PSPLIT] and last indices [B, PSPLIT], then P4's part
// sums [B, PSPLIT, 2] (offset B * PSPLIT * 12 bytes: a multiple of 8)
size_t seg_bytes(int B) {
  return ((size_t)B * PSPLIT * (sizeof(double) + sizeof(int) + 2 * sizeof(double)) + 255) &
         ~(size_t)255;
}

int check_args(const sd_shard_args* a, Geo* g) {
  if (!a) return SD_EINVAL;
  if (a->B <= 0 || a->k < 1 || a->V <= 0 || a->nranks < 1 || a->nranks > SD_SHARD_MAX_RANKS ||
      a->rank < 0 || a->rank >= a->nranks)
    return SD_EINVAL;
  if (a->dtype != SD_DTYPE_BF16 && a->dtype != SD_DTYPE_F16 && a->dtype != SD_DTYPE_F32)
    return SD_ENOTSUP;
  if (a->v_start[0] != 0 || a->v_start[a->nranks] != a->V) return SD_EINVAL;
  for (int r = 0; r < a->nranks; ++r)
    if (a->v_start[r + 1] < a->v_start[r]) return SD_EINVAL;
  const bool greedy = !(a->temperature > 0.f);
  if (!greedy && a->top_k != 0) return SD_ENOTSUP;
  if (!a->tgt || !a->xs || !a->n_acc || !a->y || (!greedy && (!a->drf || !a->u_acc || !a->u_res)))
    return SD_EINVAL;
  if (!a->workspace || a->workspace_bytes < sd_shard_workspace_bytes(a->B, a->k, a->nranks))
    return SD_ENOSPC;
  g->B = a->B; g->k = a->k; g->per = 2 * a->k + 1; g->nvec = a->B * g->per;
  g->v0 = a->v_start[a->rank]; g->Vr = a->v_start[a->rank + 1] - g->v0; g->V = a->V;
  g->rank = a->rank; g->nranks = a->nranks; g->dtype = a->dtype;
  g->T = a->temperature; g->top_p = a->top_p;
  g->truncate = a->top_p > 0.f && a->top_p < 1.f;
  return SD_OK;
}

int launched() { return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH; }

}  // namespace

extern "C" {

size_t sd_shard_workspace_bytes(int B, int k, int nranks) {
  if (B <= 0 || k < 1 || nranks < 1) return 0;
  return STATUS_BYTES + vec_bytes(B, k) + ((row_bytes(B) + 255) & ~(size_t)255) + seg_bytes(B);
}

size_t sd_shard_send_bytes(int B, int k, int nranks, int greedy, int phase) {
  if (B <= 0 || k < 1 || nranks < 1) return 0;
  const size_t nvec = (size_t)B * (2 * k + 1);
  if (greedy) return phase == 1 ? (size_t)B * (k + 1) * sizeof(int64_t) : 0;
  switch (phase) {
    case 1: return nvec * sizeof(Msg1);
    case 2: return nvec * (1 + NB) * sizeof(double);
    case 3: return nvec * sizeof(Msg3);
    case 4: return (size_t)B * 2 * sizeof(double);
    case 5: return (size_t)B * sizeof(int64_t);
    default: return 0;
  }
}

int sd_shard_phase(const sd_shard_args* args, int phase, const void* recv, void* send,
                   void* stream) {
  Geo g;
  const int rc = check_args(args, &g);
  if (rc != SD_OK) return rc;
  const sd_shard_args& a = *args;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(a.workspace);
  uint32_t* status = reinterpret_cast<uint32_t*>(ws);
  Vec* vs = reinterpret_cast<Vec*>(ws + STATUS_BYTES);
  Row* rows = reinterpret_cast<Row*>(ws + STATUS_BYTES + vec_bytes(g.B, g.k));
  char* segw = ws + STATUS_BYTES + vec_bytes(g.B, g.k) + ((row_bytes(g.B) + 255) & ~(size_t)255);
  double* segm = reinterpret_cast<double*>(segw);                 // [B, PSPLIT]
  int* segl = reinterpret_cast<int*>(segw + (size_t)g.B * PSPLIT * sizeof(double));
  double* psum = reinterpret_cast<double*>(segw + (size_t)g.B * PSPLIT * (sizeof(double) + sizeof(int)));
  const bool greedy = !(a.temperature > 0.f);
  if (phase < 1 || phase > 6) return SD_EINVAL;
  if (phase > 1 && !recv) return SD_EINVAL;
  if (phase < 6 && !greedy && !send) return SD_EINVAL;
  if (greedy) {
    if (phase == 1) {
      if (!send) return SD_EINVAL;
      if (cudaMemsetAsync(status, 0, sizeof(uint32_t), st) != cudaSuccess) return SD_ELAUNCH;
      g1_kernel<<<g.B * (g.k + 1), NT, 0, st>>>(a, g, reinterpret_cast<int64_t*>(send));
      return launched();
    }
    if (phase == 6) {
      g6_kernel<<<(g.B + 127) / 128, 128, 0, st>>>(a, g, reinterpret_cast<const int64_t*>(recv));
      return launched();
    }
    return SD_EINVAL;                                  // greedy has phases 1 and 6 only
  }
  switch (phase) {
    case 1:
      if (cudaMemsetAsync(status, 0, sizeof(uint32_t), st) != cudaSuccess) return SD_ELAUNCH;
      p1_kernel<<<g.nvec, NT, 0, st>>>(a, g, reinterpret_cast<Msg1*>(send));
      break;
    case 2:
      p2_kernel<<<g.nvec, NT, 0, st>>>(a, g, reinterpret_cast<const Msg1*>(recv), vs,
                                       reinterpret_cast<double*>(send));
      break;
    case 3:
      p3_kernel<<<g.nvec, NT, 0, st>>>(a, g, reinterpret_cast<const double*>(recv), vs,
                                       reinterpret_cast<Msg3*>(send));
      break;
    case 4:
      p4a_kernel<<<g.nvec, NT, 0, st>>>(g, reinterpret_cast<const Msg3*>(recv), vs, status);
      p4b_kernel<<<dim3(g.B, PSPLIT), NT, 0, st>>>(a, g, vs, rows, psum);
      p4c_kernel<<<(g.B + 127) / 128, 128, 0, st>>>(g, psum, reinterpret_cast<double*>(send));
      break;
    case 5:
      p5a_kernel<<<dim3(g.B, PSPLIT), NT, 0, st>>>(a, g, reinterpret_cast<const double*>(recv), vs,
                                                   rows, segm, segl);
      p5b_kernel<<<g.B, NT, 0, st>>>(a, g, reinterpret_cast<const double*>(recv), vs, rows, segm,
                                     segl, reinterpret_cast<int64_t*>(send));
      break;
    case 6:
      p6_kernel<<<(g.B + 127) / 128, 128, 0, st>>>(a, g, reinterpret_cast<const int64_t*>(recv),
                                                   rows);
      break;
  }
  return launched();
}

}  // extern "C"
