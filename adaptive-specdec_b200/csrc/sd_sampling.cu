// Verify-round sampling kernels for B200 (sm_100a).
//
// Reference path replaced: specdec/sampling.py:34-95 (to_probs, residual_probs,
// gather_prob, sample_from_probs) and the accept / residual / bonus block of
// specdec/engine.py:282-303.
//
// Design
// ------
// * bf16 / fp16 logits at any vocabulary size (the verify round's case): a
//   persistent stats kernel reads every logits element exactly once and
//   produces, per vector, the softmax normaliser, the top-k / top-p kept set
//   and the probe probability, without sorting the vocabulary (see the stats
//   kernel section below).  An exact 65,536-bin count histogram of the
//   vector's 16-bit values backs it up for the rare vectors the list cannot
//   decide.  The CTA that finishes a row's last vector performs that row's
//   accept test and its residual / bonus draw.
// * fp32 / any dtype with V <= SMALLV_MAX: one CTA per vector computes every
//   probability, sorts (p desc, index asc) with a bitonic sort in shared memory
//   and materialises the final probabilities in the workspace.
// * greedy (T <= 0): only the target argmax is needed; the draft logits are
//   never read.
// * the finish kernel (small-V, fp32 and histogram paths) runs per (row,
//   vocabulary chunk): it decides the accepted prefix from the per-vector
//   probe probabilities p_i(x_i), q_i(x_i), sums the residual (or bonus) mass
//   of its chunk, and the last chunk of a row to finish performs the
//   inverse-CDF draw.  No CTA ever waits on another CTA.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "sd_common.cuh"

namespace sd {

constexpr int HIST_WORDS = 32768;       // 65536 16-bit counters (exact fallback)
constexpr int NCORR_MAX = 96;           // counter-wrap corrections per vector
constexpr int SMALLV_MAX = 2048;        // small-vocabulary exact path
constexpr int ST = 512;                 // threads of the small-V kernel
constexpr int FT = 512;                 // threads of the finish / probs kernels
constexpr int NCH_MAX = 64;             // vocabulary chunks per row in finish
constexpr int AM_UPT = 8;               // argmax: 16-byte units per thread per pass, loaded at once
constexpr int AM_FT = 256;              // argmax: threads per block (several blocks per SM)

constexpr uint32_t NO_CUT = 0x7FFFFFFFu;

struct VecStats {
  float m;          // max of fl(x / T)
  float inv_s;      // fl(1 / S)
  float zf;         // max(fl(Z), 1e-12): kept mass after top-k / top-p
  float probe_p;    // final probability of the probe token (0 if no probe)
  uint32_t kth;     // top-k: keep fkey(x) >= kth
  uint32_t vstar;   // top-p boundary class (fkey); keys > vstar kept
  int32_t idx_cut;  // members of the vstar class with index <= idx_cut kept
  int32_t argmax;   // greedy: first index of the maximum
  int32_t flags;    // bit0: histogram overflow path taken; bit1: correction table full
  int32_t n_keep;   // kept members of the boundary class (diagnostics)
  int32_t fb_why;   // FB_* reason when the histogram path ran, else 0
  int32_t pad;
};
static_assert(sizeof(VecStats) == 48, "VecStats layout");

// Two logits tensors addressed as one list of vectors, row-major:
// vector v -> row b = v / (npos0 + npos1), then set 0 positions, then set 1.
struct VecSet {
  const void* base[2];
  int64_t bs[2], ps[2];
  int npos[2];
  const int64_t* probe;      // probe token ids [rows, probe_bs]
  int64_t probe_bs;
  int probe_npos[2];         // positions < probe_npos[s] have a probe
  int nrows;
};

__device__ __forceinline__ void vec_locate(const VecSet& vs, int v, int* set, int* row, int* pos) {
  const int per = vs.npos[0] + vs.npos[1];
  const int b = v / per, l = v - b * per;
  *row = b;
  if (l < vs.npos[0]) { *set = 0; *pos = l; } else { *set = 1; *pos = l - vs.npos[0]; }
}

__device__ __forceinline__ const void* vec_ptr(const VecSet& vs, int set, int row, int pos, int dtype) {
  const int esz = dtype == SD_DTYPE_F32 ? 4 : 2;
  const char* p = reinterpret_cast<const char*>(vs.base[set]);
  return p + (row * vs.bs[set] + pos * vs.ps[set]) * esz;
}

__device__ __forceinline__ int64_t vec_probe(const VecSet& vs, int set, int row, int pos) {
  if (vs.probe == nullptr || pos >= vs.probe_npos[set]) return -1;
  return vs.probe[row * vs.probe_bs + pos];
}

// ---------------------------------------------------------------------------
// stats kernel (bf16 / fp16): persistent, one CTA per SM, three warp roles
// ---------------------------------------------------------------------------
// Warp 0 (producer) streams each vector's 16-byte-aligned body into a ring of
// NSLOT shared-memory slots with cp.async.bulk (mbarrier completion, bounded
// waits).  Warps 1..NSW (streaming) read every element once from the ring:
// each lane sums 2^(x c2 - Rc2) over its elements below the list threshold
// (the vector's running maximum minus W_LIST base-2 units) against a
// per-vector reference Rc2, and lists the elements at or above it itself,
// re-reading them from the slot: a list entry is (order key, vocabulary
// index).  The NCW finalize warps take a finished vector (its list, the
// streaming warps' partial sums, its maximum) while the next one streams.
// They compute S exactly (the bulk mass plus expf over the listed elements,
// float64), place the listed elements in coarse depth bins, sort only the
// bins that can hold the top-k / top-p boundary by (value desc, index asc) --
// the order of the reference's sort with ties broken by index -- and apply
// the reference's element-wise rules there: top-k (keep p >= k-th value),
// top-p (keep while fl32(cum - p) < top_p, cum in float64), renormalisation.
// The kept set is described by its last element L in that order: j is kept
// iff value_j > value_L or (value_j == value_L and j <= index_L).  Every
// element at or above M - W_LIST is listed, so the rules are exact when the
// boundary falls there; otherwise (boundary deeper, list overflow, top-k
// beyond the list) the vector is recomputed exactly from a 65,536-bin count
// histogram of all its elements read again from global memory
// (VecStats.fb_why records why).  Two vectors are in flight per CTA (two
// hand-over sets).
//
// The CTA that finishes the last vector of a row then performs that row's
// accept test and its residual / bonus draw (finalize warps).  Outside the
// nucleus of p the residual max(p - q, 0) is zero, so the draw only walks p's
// kept elements in index order (q gathered at those indices).
constexpr int NSW = 19;                  // streaming warps
constexpr int ST_N = NSW * 32;           // streaming threads
constexpr int ST0 = 32;                  // first streaming thread (warp 0 produces)
constexpr int NCW = 4;                   // finalize warps
constexpr int CT = NCW * 32;             // finalize threads
constexpr int FIN0 = ST0 + ST_N;         // first finalize thread
constexpr int HT = FIN0 + CT;            // threads per CTA
constexpr int GRID_MAX = 160;            // bound on the persistent grid (fallback buffers)
constexpr int GPS = 4;                   // 16-byte units per streaming lane per ring slot
constexpr int SLOT = GPS * 16 * ST_N;    // bytes per ring slot (30 KB)
constexpr int NSLOT = 3;
constexpr long long WAIT_CYCLES = 1LL << 32;   // ~2 s at 2 GHz: bound on every wait
constexpr int LIST_CAP = 3072;           // listed elements per vector
static_assert(LIST_CAP < 65536, "list-path counts pack into 16 bits");
constexpr int NUC_MAX = 1024;            // kept elements stored per vector for the draw
constexpr float W_LIST = 12.f;           // list window, base-2 units below the maximum

static_assert(FIN0 % 32 == 0, "finalize warps start on a warp boundary");

constexpr int F_FALLBACK = 1;            // exact full-histogram path taken
// why the list path handed a vector to the histogram path (VecStats.fb_why)
constexpr int FB_LIST = 2;               // more listed elements than LIST_CAP
constexpr int FB_SELECT = 3;             // more selected elements than SEL_CAP
constexpr int FB_BOUNDARY = 4;           // top-p / top-k boundary outside the sorted part
constexpr int F_INEXACT = 2;             // that path's correction table overflowed
constexpr int F_LISTED = 4;              // kept elements stored in the workspace
constexpr int F_ALLKEPT = 8;             // no truncation: every element kept
constexpr int F_DEFER = 16;              // handed to the fallback kernel (not yet computed)


constexpr int SEL_CAP = 1024;            // entries sorted per vector
constexpr int RANK_MAX = 512;            // row draw by direct prefix sums up to this many kept
constexpr int NBIN = 49;                 // coarse depth bins: 4 per base-2 unit, + overflow
constexpr int NBIN_PAD = 64;             // two bins per lane of one warp
static_assert((unsigned long long)LIST_CAP << 20 <= 0xFFFFFFFFull,
              "a bin's 20-bit mass parts sum below 2^32");

// Finalize-warp scratch of the list path.
struct ListBuf {
  float ecache[LIST_CAP];                // exact softmax numerator of each window key
  unsigned long long sel[SEL_CAP];       // entries selected for sorting
  float p[SEL_CAP];
  // depth-bin mass in 2^-40 fixed point as 2^20 * binhi + binlo (each part
  // sums at most LIST_CAP terms below 2^20), and count
  uint32_t binhi[NBIN_PAD];
  uint32_t binlo[NBIN_PAD];
  uint32_t bincnt[NBIN_PAD];
  uint8_t bin8[LIST_CAP];                // depth bin of each window key (NBIN_PAD: outside)
};

// What the streaming warps hand to the finalize warps for one vector (two
// of these alternate).
struct VecHand {
  unsigned long long key[LIST_CAP];      // (fkey(value) << 32) | ~index
  double wbulk[NSW];                     // per streaming warp: sum of 2^(y - (wrc2 - Rc2))
  float wrc2[NSW];                       // per streaming warp: its common offset (-inf: none)
  uint32_t gkey;                         // fkey of the vector's running maximum
  int nkey;                              // listed elements
};

// The exact fallback's counters reuse the ring and hand-over memory once the
// CTA has streamed all its vectors.
struct FbScratch {
  uint32_t hist[HIST_WORDS];             // 65,536 16-bit counters, indexed by raw value
  uint32_t corr_raw[NCORR_MAX];          // counters that wrapped: +65536 per entry
  int32_t corr_add[NCORR_MAX];
};

struct HistSmem {
  union {
    struct {
      alignas(128) unsigned char ring[NSLOT][SLOT];
      VecHand hand[2];
    } st;
    FbScratch fb;
  } w;
  union {
    ListBuf l;
  } u;
  double dred[40];
  uint32_t ured[40];
  float fred[40];
  alignas(8) unsigned long long full[NSLOT];
  alignas(8) unsigned long long empty[NSLOT];
  alignas(8) unsigned long long streamed[2];   // the streaming warps finished a vector
  alignas(8) unsigned long long freed[2];      // the finalize warps released its hand-over
  int ncorr;
  int corr_full;
  uint32_t npre_nsel;  // list path: kept elements above the sorted part (low 16 bits) and
                       // elements selected for sorting (high 16 bits)
  int fb_why;          // FB_* reason of the last hand-over to the histogram path
  int abort_flag;
  int fin_skip;        // finalize warps: skip the work of this vector (after an abort)
  uint32_t keyk16;
  uint32_t vstar16;
  int n_keep;
  int vcount;
  double z;
  int32_t idx_cut;
  int found_cut;
  int last_row;
  int sc_n;
  int sc_L;
  long long sc_y;
  double sc_pre;
};

static_assert(sizeof(HistSmem) <= 227 * 1024, "stats kernel shared memory");

// Index of this thread within the finalize warps.
__device__ __forceinline__ int ftid() { return (int)threadIdx.x - FIN0; }

// barrier of the finalize warps
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 2, %0;" :: "n"(CT) : "memory"); }
// barrier of the streaming warps
__device__ __forceinline__ void sbar() { asm volatile("bar.sync 1, %0;" :: "n"(ST_N) : "memory"); }
static_assert(CT % 32 == 0 && ST_N % 32 == 0, "named barrier thread counts");
static_assert(RANK_MAX % CT == 0, "finalize loops split evenly over CT threads");

template <typename T>
__device__ __forceinline__ T c_sum(T v, T* red) {
  const int lane = threadIdx.x & 31, wid = ftid() >> 5;
  v = warp_sum(v);
  cbar();
  if (lane == 0) red[wid] = v;
  cbar();
  T t = lane < NCW ? red[lane] : T(0);
  return warp_sum(t);
}

template <typename T>
__device__ __forceinline__ T c_max(T v, T* red, T lowest) {
  const int lane = threadIdx.x & 31, wid = ftid() >> 5;
  v = warp_max(v);
  cbar();
  if (lane == 0) red[wid] = v;
  cbar();
  T t = lane < NCW ? red[lane] : lowest;
  return warp_max(t);
}

template <typename T>
__device__ __forceinline__ T c_excl_scan(T v, T* red, T* total) {
  const int lane = threadIdx.x & 31, wid = ftid() >> 5;
  T inc = warp_incl_scan(v);
  cbar();
  if (lane == 31) red[wid] = inc;
  cbar();
  if (wid == 0) {
    T w = lane < NCW ? red[lane] : T(0);
    T wi = warp_incl_scan(w);
    if (lane < NCW) red[lane] = wi - w;
    if (lane == NCW - 1) red[32] = wi;
  }
  cbar();
  *total = red[32];
  return red[wid] + inc - v;
}

// ---- mbarrier / bulk-copy primitives --------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(unsigned long long* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_u32(b)), "r"(bytes) : "memory");
}
// Bounded wait for the phase of parity `parity` to complete.  Returns false
// (and raises the CTA's abort flag) after WAIT_CYCLES or when another thread
// already aborted.
__device__ __forceinline__ bool mbar_wait(unsigned long long* b, uint32_t parity, int* abort_flag) {
  const uint32_t a = smem_u32(b);
  const long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(a), "r"(parity) : "memory");
    if (ok) return true;
    if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
    if (clock64() - t0 > WAIT_CYCLES) {
      *reinterpret_cast<volatile int*>(abort_flag) = 1;
      return false;
    }
  }
}
// Non-blocking: has the phase of parity `parity` completed?
__device__ __forceinline__ bool mbar_test(unsigned long long* b, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
               " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         unsigned long long* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Vector geometry shared by producer and consumers: ragged head elements up to
// the first 16-byte boundary, a body of whole 16-byte units split into ring
// chunks, ragged tail elements.
struct VecGeom {
  int head, nunits, tail0, nchunk;
  __device__ VecGeom(const void* p, int V) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    head = (int)(((16u - (uint32_t)(a & 15u)) & 15u) >> 1);
    if (head > V) head = V;
    nunits = (V - head) >> 3;
    tail0 = head + (nunits << 3);
    nchunk = (nunits * 16 + SLOT - 1) / SLOT;
  }
};

// inverse of fkey for finite non-NaN keys
__device__ __forceinline__ float fkey_value(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(b);
}
__device__ __forceinline__ unsigned long long list_key(float x, uint32_t idx) {
  return ((unsigned long long)fkey(x) << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t list_idx(unsigned long long k) {
  return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
}
__device__ __forceinline__ float list_val(unsigned long long k) {
  return fkey_value((uint32_t)(k >> 32));
}

// Bitonic sort of key[0..N) (N a power of two, <= LIST_CAP), consumer threads.
__device__ void bitonic_sort(unsigned long long* key, int N, bool descending) {
  for (int k2 = 2; k2 <= N; k2 <<= 1) {
    for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
      for (int i = ftid(); i < N; i += CT) {
        const int ixj = i ^ j2;
        if (ixj > i) {
          const unsigned long long a = key[i], b = key[ixj];
          const bool up = ((i & k2) == 0) == descending;
          if (up ? (a < b) : (a > b)) { key[i] = b; key[ixj] = a; }
        }
      }
      cbar();
    }
  }
}

// ---- exact full-histogram path (fallback) ---------------------------------
struct StatsParams {
  VecSet vs;
  int dtype, V, nvec;
  float T, top_p;
  int top_k;
  VecStats* stats;
  unsigned long long* nuc;   // [nvec, NUC_MAX] kept elements (list keys)
  int* row_ctr;              // [rows] vectors finished per row (zeroed before launch)
  int* status;               // device status word: bit0 = a bounded wait timed out
  // fused row finish (top-p / top-k modes)
  int fused, k;
  const float* u_acc; int64_t u_bs;
  const float* u_res;
  const uint8_t* alive;
  int64_t* n_acc; int64_t* y; float* px; float* qx; float* y_prob;
  // draft distributions given as probabilities (null: computed from the draft
  // logits of set 1): row b, position i at qprob + b q_bs + i q_ps, [V] fp32
  const float* qprob; int64_t q_bs, q_ps;
};

// q at element j of the draft distribution of row `row`, position `n`: the
// caller's probability row when given, else from the draft vector's stats.
__device__ __forceinline__ float q_at(const StatsParams& P, const VecStats& stq, const void* xq,
                                      int row, int n, int64_t j);

// q(x_i) of the accept test of row `row`, position i.
__device__ __forceinline__ float q_probe(const StatsParams& P, int row, int i) {
  const int npos0 = P.vs.npos[0], npos = P.vs.npos[0] + P.vs.npos[1];
  if (P.qprob) {
    const int64_t x = P.vs.probe[row * P.vs.probe_bs + i];
    return __ldg(P.qprob + row * P.q_bs + i * P.q_ps + x);
  }
  return __ldcg(&P.stats[(int64_t)row * npos + npos0 + i].probe_p);
}

// ---- streaming ---------------------------------------------------------------

struct Stream {
  float Rc2;      // exponent offset of the bulk sum: y(x) = x c2 - Rc2 (-inf until set)
  float m;        // this lane's running max (logit units)
  float xt;       // list threshold: a value of the input type <= m - wlist
  uint32_t xt2;   // xt twice, packed in the input type
  float eY;       // 2^y(xt): the bulk term of an element clamped to xt
  double bulk;    // sum of 2^y(x) over the unlisted elements
};

// Append `key` for the lanes with `pred` set: one shared atomic per warp.
__device__ __forceinline__ void warp_append(int* counter, unsigned long long* buf, int cap,
                                            bool pred, unsigned long long key) {
  const unsigned mask = __ballot_sync(0xffffffffu, pred);
  if (!mask) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(mask) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(counter, __popc(mask));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (pred) {
    const int slot = base + __popc(mask & ((1u << lane) - 1u));
    if (slot < cap) buf[slot] = key;
  }
}

// low / high element of a packed pair as float
template <int DT>
__device__ __forceinline__ float lo16(uint32_t w) {
  if (DT == SD_DTYPE_BF16) return __uint_as_float(w << 16);
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
}
template <int DT>
__device__ __forceinline__ float hi16(uint32_t w) {
  if (DT == SD_DTYPE_BF16) return __uint_as_float(w & 0xFFFF0000u);
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
// packed pair of -inf
template <int DT>
__device__ __forceinline__ constexpr uint32_t neg_inf2() {
  return DT == SD_DTYPE_BF16 ? 0xFF80FF80u : 0xFC00FC00u;
}
// element-wise max of two packed pairs
template <int DT>
__device__ __forceinline__ uint32_t pmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  if (DT == SD_DTYPE_BF16) asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// (y0, y1) = (x0, x1) * c + (d0, d1) on the paired FP32 pipe (each an IEEE fma)
__device__ __forceinline__ void fma2(float& y0, float& y1, float x0, float x1, float c, float d0,
                                     float d1) {
  asm("{\n .reg .b64 A, B, C, D;\n mov.b64 A, {%2, %3};\n mov.b64 B, {%4, %4};\n"
      " mov.b64 C, {%5, %6};\n fma.rn.f32x2 D, A, B, C;\n mov.b64 {%0, %1}, D;\n}"
      : "=f"(y0), "=f"(y1) : "f"(x0), "f"(x1), "f"(c), "f"(d0), "f"(d1));
}
// (a0, a1) += (b0, b1)
__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  asm("{\n .reg .b64 A, B, D;\n mov.b64 A, {%0, %1};\n mov.b64 B, {%2, %3};\n"
      " add.rn.f32x2 D, A, B;\n mov.b64 {%0, %1}, D;\n}"
      : "+f"(a0), "+f"(a1) : "f"(b0), "f"(b1));
}

// Base-2 exponent of an element relative to the bulk reference,
// y(x) = x (c2h + c2l) - Rc2 with c2h + c2l = log2(e) / T to ~2^-48 and
// c2h, c2l > 0.  Monotone non-decreasing in x (a composition of two fmas with
// positive multipliers), so x >= thr implies y(x) >= y(thr); y(-inf) = -inf.
__device__ __forceinline__ float yof(float x, float c2h, float c2l, float Rc2) {
  return fmaf(x, c2h, fmaf(x, c2l, -Rc2));
}
__device__ __forceinline__ void yof2(float& y0, float& y1, float x0, float x1, float c2h,
                                     float c2l, float Rc2) {
  float i0, i1;
  fma2(i0, i1, x0, x1, c2l, -Rc2, -Rc2);
  fma2(y0, y1, x0, x1, c2h, i0, i1);
}

// Largest finite value of the input type at or below f (the lowest finite
// value below that), so that a -inf element is never at or above it.
template <int DT>
__device__ __forceinline__ uint32_t round_down16(float f) {
  if (DT == SD_DTYPE_BF16) {
    const uint32_t h = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rd(f));
    return h == 0xFF80u ? 0xFF7Fu : h;
  }
  const uint32_t h = (uint32_t)__half_as_ushort(__float2half_rd(f));
  return h == 0xFC00u ? 0xFBFFu : h;
}
template <int DT>
__device__ __forceinline__ float val16(uint32_t h) {
  if (DT == SD_DTYPE_BF16) return __uint_as_float(h << 16);
  return __half2float(__ushort_as_half((unsigned short)h));
}

// List threshold of a lane from its running max: xt = the largest value of
// the input type at or below m - wlist, so every element at or above the
// vector's final M - wlist is at or above it.  The clamped term 2^y(xt) bounds
// every bulk term; the bulk reference moves up when it would exceed 2^64.
template <int DT>
__device__ __forceinline__ void set_thr(Stream& st, float c2h, float c2l, float wlist) {
  const uint32_t h = round_down16<DT>(st.m - wlist);
  st.xt2 = h | (h << 16);
  st.xt = val16<DT>(h);
  float Y = yof(st.xt, c2h, c2l, st.Rc2);
  if (Y > 64.f) {
    const float nr = st.Rc2 + (Y - 32.f);
    st.bulk *= exp2((double)st.Rc2 - (double)nr);
    st.Rc2 = nr;
    Y = yof(st.xt, c2h, c2l, nr);
  }
  st.eY = ex2_approx(Y);
}

// Raise this lane's running max (list threshold follows).
template <int DT>
__device__ __forceinline__ void raise_m(Stream& st, float mn, float c2h, float c2l, float wlist) {
  st.m = mn;
  set_thr<DT>(st, c2h, c2l, wlist);
}

// Fix the bulk reference of a lane that has none yet (its first finite element).
template <int DT>
__device__ __forceinline__ void set_ref(Stream& st, float r, float c2h, float c2l, float wlist) {
  st.Rc2 = r * c2h;
  st.m = fmaxf(st.m, r);
  set_thr<DT>(st, c2h, c2l, wlist);
}

// Lane maximum of 4G packed words.
template <int DT, int G>
__device__ __forceinline__ float lane_max(const uint32_t* w, uint32_t* pm1) {
  uint32_t pm[2 * G];
#pragma unroll
  for (int i = 0; i < 2 * G; ++i) pm1[i] = pm[i] = pmax2<DT>(w[2 * i], w[2 * i + 1]);
#pragma unroll
  for (int n = 2 * G; n > 1; n >>= 1) {
#pragma unroll
    for (int i = 0; i < n / 2; ++i) pm[i] = pmax2<DT>(pm[i], pm[i + n / 2]);
  }
  return fmaxf(lo16<DT>(pm[0]), hi16<DT>(pm[0]));
}

// element-wise min of two packed pairs
template <int DT>
__device__ __forceinline__ uint32_t pmin2(uint32_t a, uint32_t b) {
  uint32_t r;
  if (DT == SD_DTYPE_BF16) asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("min.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// 2^y summed over the elements of 4G packed words, each first clamped to the
// list threshold xt (packed pair xt2): an element at or above xt adds exactly
// 2^y(xt), which the caller takes back out when it lists the element.  No
// per-element test or select: one packed min per pair.
template <int DT, int G>
__device__ __forceinline__ float bulk_words(const uint32_t* w, float c2h, float c2l, float Rc2,
                                            uint32_t xt2) {
  float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
#pragma unroll
  for (int i = 0; i < 4 * G; ++i) {
    const uint32_t c = pmin2<DT>(w[i], xt2);
    float y0, y1;
    yof2(y0, y1, lo16<DT>(c), hi16<DT>(c), c2h, c2l, Rc2);
    const float e0 = ex2_approx(y0);
    const float e1 = ex2_approx(y1);
    if (i & 1) add2(b2, b3, e0, e1); else add2(b0, b1, e0, e1);
  }
  return (b0 + b2) + (b1 + b3);
}

// Bit mask of the elements of 16 packed words at or above the threshold pair
// xt2: word i's low element at bit i, its high element at bit 16 + i.
template <int DT>
__device__ __forceinline__ uint32_t ge_mask16(const uint32_t* w, uint32_t xt2) {
  uint32_t m = 0u;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t g;                                       // 0xFFFF per half where w >= xt
    if (DT == SD_DTYPE_BF16) asm("set.ge.u32.bf16x2 %0, %1, %2;" : "=r"(g) : "r"(w[i]), "r"(xt2));
    else asm("set.ge.u32.f16x2 %0, %1, %2;" : "=r"(g) : "r"(w[i]), "r"(xt2));
    m |= g & (0x00010001u << i);
  }
  return m;
}

// One pass over 4G packed words per lane; groups without data hold -inf
// pairs.  Called by whole streaming warps.  RING: the words are streaming
// thread st's 16-byte units st + q * ST_N (q < 4) of ring slot `slot`, whose
// first element has vocabulary index jbase.  A lane whose maximum reaches its
// threshold lists its elements at or above it (a packed compare per word,
// then one shared atomic for all of them, each element read again from the
// slot) and takes their clamped terms back out of its bulk sum.  Otherwise
// (the < 16 ragged elements, one per lane in the low half of w[0], index jr)
// the lane's element is listed the same way.
template <int DT, int G, bool RING>
__device__ __forceinline__ void stream_words(HistSmem& s, VecHand& H, Stream& st,
                                             const uint32_t* w, int slot, uint32_t jbase,
                                             uint32_t jr, float c2h, float c2l, float wlist) {
  static_assert(!RING || G == 4, "16 packed words per lane and slot");
  // The bulk sum and the lane maximum are independent (straight-line code the
  // compiler interleaves); a lane without a reference yet discards the sum.
  const bool had_ref = st.Rc2 != -INFINITY;
  const float b = bulk_words<DT, G>(w, c2h, c2l, st.Rc2, st.xt2);
  uint32_t pm1[2 * G];
  const float gm = lane_max<DT, G>(w, pm1);
  if (had_ref) {
    st.bulk += (double)b;
  } else if (gm > -INFINITY) {                        // rare: the lane's first finite element
    set_ref<DT>(st, gm, c2h, c2l, wlist);
    atomicMax(&H.gkey, fkey(gm));
    st.bulk += (double)bulk_words<DT, G>(w, c2h, c2l, st.Rc2, st.xt2);
  }
  if (st.Rc2 != -INFINITY) {
    if (gm >= st.xt) {                                // rare: elements to list
      if (RING) {
        uint32_t hm = ge_mask16<DT>(w, st.xt2);
        const int cnt = __popc(hm);
        int o = atomicAdd(&H.nkey, cnt);
        st.bulk -= (double)cnt * (double)st.eY;
        const uint32_t* ring32 = reinterpret_cast<const uint32_t*>(s.w.st.ring[slot]);
        const int tl = (int)threadIdx.x - ST0;
        while (hm) {
          const int bit = __ffs(hm) - 1;
          hm &= hm - 1u;
          const int i = bit & 15, h = bit >> 4;
          const int unit = tl + (i >> 2) * ST_N;
          float xv = gm;                              // the only element at or above xt
          if (cnt > 1) {
            const uint32_t ww = ring32[unit * 4 + (i & 3)];
            xv = h ? hi16<DT>(ww) : lo16<DT>(ww);
          }
          if (o < LIST_CAP)
            H.key[o] = list_key(xv, jbase + 8u * (uint32_t)unit + 2u * (uint32_t)(i & 3) + (uint32_t)h);
          ++o;
        }
      } else {                                        // the lane's only element
        const int o = atomicAdd(&H.nkey, 1);
        if (o < LIST_CAP) H.key[o] = list_key(lo16<DT>(w[0]), jr);
        st.bulk -= (double)st.eY;
      }
    }
  }
  // The lane's running max never exceeds the published vector max: it only
  // rises from the published value (sync_max), the seed (published), or its
  // own elements, published here as they raise it.
  if (gm > st.m) {
    raise_m<DT>(st, gm, c2h, c2l, wlist);
    atomicMax(&H.gkey, fkey(gm));
  }
}

// Start of a ring slot: adopt the vector's running max if it is ahead.
template <int DT>
__device__ __forceinline__ void sync_max(VecHand& H, Stream& st, float c2h, float c2l,
                                         float wlist) {
  const uint32_t gk = *reinterpret_cast<volatile uint32_t*>(&H.gkey);
  const float gv = fkey_value(gk);
  if (st.Rc2 != -INFINITY && gv > st.m) raise_m<DT>(st, gv, c2h, c2l, wlist);
}

// Probability of element j of a vector under its stats (the kept predicate
// and p' = fl(fl(e * inv_s) / zf)).
__device__ __forceinline__ float stats_prob(const VecStats& st, const void* x, int dtype, float T,
                                            int64_t j) {
  const float xv = load_logit(x, dtype, j);
  const uint32_t kx = fkey(xv);
  const bool kept = kx >= st.kth && (kx > st.vstar || (kx == st.vstar && j <= (int64_t)st.idx_cut));
  if (!kept) return 0.f;
  return __fdiv_rn(prob_of(xv, T, st.m, st.inv_s), st.zf);
}

__device__ __forceinline__ float q_at(const StatsParams& P, const VecStats& stq, const void* xq,
                                      int row, int n, int64_t j) {
  if (P.qprob) return __ldg(P.qprob + row * P.q_bs + n * P.q_ps + j);
  return stats_prob(stq, xq, P.dtype, P.T, j);
}

__device__ __forceinline__ VecStats load_stats_cg(const VecStats* p) {
  VecStats o;
  const int4* src = reinterpret_cast<const int4*>(p);
  int4* dst = reinterpret_cast<int4*>(&o);
  dst[0] = __ldcg(src);
  dst[1] = __ldcg(src + 1);
  dst[2] = __ldcg(src + 2);
  return o;
}

// List-based exact computation (see the section comment).  Returns true when
// the vector needs the exact full-histogram path.
__device__ __forceinline__ int depth_bin(float M, float xv, float c2) {
  return min(NBIN - 1, (int)((M - xv) * c2 * 4.f));
}

// Descending sort of one key per lane across a warp (bitonic network).
__device__ __forceinline__ unsigned long long warp_sort_desc(unsigned long long key) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k2 = 2; k2 <= 32; k2 <<= 1) {
#pragma unroll
    for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, j2);
      const bool lower = (lane & j2) == 0;
      const bool desc = (lane & k2) == 0;             // this half of the merge sorts descending
      const bool take_max = lower == desc;
      key = take_max ? (o > key ? o : key) : (o < key ? o : key);
    }
  }
  return key;
}

// p' of element j (logit xv) under `o`: the kept predicate and fl(fl(e * inv_s) / zf).
__device__ __forceinline__ float stats_prob_x(const VecStats& o, float xv, float T, int64_t j) {
  const uint32_t kx = fkey(xv);
  const bool kept = kx >= o.kth && (kx > o.vstar || (kx == o.vstar && j <= (int64_t)o.idx_cut));
  return kept ? __fdiv_rn(prob_of(xv, T, o.m, o.inv_s), o.zf) : 0.f;
}

__device__ __forceinline__ bool fallback_why(HistSmem& s, int why) {
  if (ftid() == 0) s.fb_why = why;
  return true;
}

__device__ bool finalize_list(HistSmem& s, VecHand& H, const StatsParams& P, int v,
                              const uint16_t* x, int64_t probe, float c2, float wlist) {
  const int t = ftid(), lane = t & 31;
  const int V = P.V;
  const bool topk_on = P.top_k > 0 && P.top_k < V;
  const bool topp_on = P.top_p > 0.0f && P.top_p < 1.0f;
  const bool all_kept = !topk_on && !topp_on;
  const float tp32 = P.top_p;
  const int nl = H.nkey;
  if (nl > LIST_CAP || nl < 1) return fallback_why(s, FB_LIST);
  // the probe's logit, requested now so that its latency overlaps the list work
  const bool has_probe = probe >= 0 && probe < V;
  float xprobe = 0.f;
  if (t == 0 && has_probe) xprobe = bits16_to_float(__ldg(x + probe), P.dtype);
  const float M = fkey_value(H.gkey);                   // every element raised gkey
  const float m = scaled_logit(M, P.T);
  const float wlow = M - wlist;
  if (t < NBIN_PAD) { s.u.l.binhi[t] = 0u; s.u.l.binlo[t] = 0u; s.u.l.bincnt[t] = 0u; }
  if (t == 0) s.npre_nsel = 0u;
  cbar();
  // exact softmax numerators of the listed elements of the window (at or
  // above M - W_LIST) and their depth bins below the maximum (4 bins per
  // base-2 unit), each bin's mass and count added with 32-bit shared atomics.
  // The streaming warps' bulk sums are relative to their offsets wrc2 (terms
  // 2^(x c2 - wrc2)); the listed terms are exp(x / T - m).
  double es = 0.0;
  if (t < NSW && H.wbulk[t] > 0.0 && H.wrc2[t] != -INFINITY)
    es = H.wbulk[t] * exp2((double)H.wrc2[t] - (double)m * 1.4426950408889634);
  // keys below the window only add to S: the ex2 form of the bulk sum
  const float mc2 = (float)((double)m * 1.4426950408889634);
  for (int i = t; i < nl; i += CT) {
    const float xv = list_val(H.key[i]);
    float e;
    int bin = NBIN_PAD;
    if (!(xv >= wlow)) {
      e = ex2_approx(fmaf(xv, c2, -mc2));
    } else {
      e = softmax_num(xv, P.T, m);                      // <= 1: xv <= M
      s.u.l.ecache[i] = e;
      bin = depth_bin(M, xv, c2);
      if (!all_kept) {
        const unsigned long long f = __float2ull_rn(e * 0x1p40f);
        atomicAdd(&s.u.l.binhi[bin], (unsigned)(f >> 20));
        atomicAdd(&s.u.l.binlo[bin], (unsigned)(f & 0xFFFFFull));
        atomicAdd(&s.u.l.bincnt[bin], 1u);
      }
    }
    s.u.l.bin8[i] = (uint8_t)bin;
    es += (double)e;
  }
  const double S = c_sum<double>(es, s.dred);            // (its barriers publish bin8, ecache)
  const float inv_s = __double2float_rn(1.0 / S);
  int L = -1;                                            // last kept, sorted-part index
  float kth_x = -INFINITY;
  double z = 0.0;
  int npre = 0;                                          // kept elements above the sorted part
  if (!all_kept) {
    if (t < 32) {
      // Bins, lane l owning 2l and 2l+1.  bstar: the shallowest bin holding
      // top_p of the mass (with 1e-4 slack) and top_k elements, plus the next
      // occupied bin, so the first dropped element is sorted.  bL: the first
      // bin where the top-p or top-k boundary can lie; every element of the
      // bins before it is kept (its exclusive mass is below top_p by the
      // slack and it ranks within top_k), in any order.
      const unsigned long long f0 =
          ((unsigned long long)s.u.l.binhi[2 * lane] << 20) + s.u.l.binlo[2 * lane];
      const unsigned long long f1 =
          ((unsigned long long)s.u.l.binhi[2 * lane + 1] << 20) + s.u.l.binlo[2 * lane + 1];
      const int c0 = (int)s.u.l.bincnt[2 * lane], c1 = (int)s.u.l.bincnt[2 * lane + 1];
      const unsigned long long fi = warp_incl_scan<unsigned long long>(f0 + f1);
      const int ci = warp_incl_scan<int>(c0 + c1);
      const unsigned long long fe = fi - f0 - f1;
      const int ce = ci - c0 - c1;
      // thresholds in fixed point (the bins hold at most 2^52)
      const double hi_d = topp_on ? (double)tp32 * S * (1.0 + 1e-4) * 0x1p40 : 0.0;
      const double lo_d = (double)tp32 * S * (1.0 - 1e-4) * 0x1p40;
      const unsigned long long hi_t = hi_d >= 0x1p60 ? ~0ull : (unsigned long long)ceil(hi_d);
      const unsigned long long lo_t = lo_d >= 0x1p60 ? ~0ull : (unsigned long long)ceil(lo_d);
      const bool ok0 = fe + f0 >= hi_t && (!topk_on || ce + c0 >= P.top_k);
      const bool ok1 = fi >= hi_t && (!topk_on || ci >= P.top_k);
      const unsigned okm = __ballot_sync(0xffffffffu, ok0 || ok1);
      int bstar = NBIN - 1;
      if (okm) {
        const int fl = __ffs(okm) - 1;
        bstar = 2 * fl + (__shfl_sync(0xffffffffu, ok0, fl) ? 0 : 1);
      }
      const unsigned n0 = __ballot_sync(0xffffffffu, c0 > 0 && 2 * lane > bstar);
      const unsigned n1 = __ballot_sync(0xffffffffu, c1 > 0 && 2 * lane + 1 > bstar);
      int nb = NBIN_PAD;
      if (n0) nb = min(nb, 2 * (__ffs(n0) - 1));
      if (n1) nb = min(nb, 2 * (__ffs(n1) - 1) + 1);
      if (nb < NBIN) bstar = nb;
      // first bin reaching the lower mass bound / holding the top_k-th element
      int bL = NBIN_PAD;
      auto first_bin = [&](bool a0, bool a1) {
        const unsigned mm = __ballot_sync(0xffffffffu, a0 || a1);
        if (!mm) return NBIN_PAD;
        const int fl = __ffs(mm) - 1;
        return 2 * fl + (__shfl_sync(0xffffffffu, a0, fl) ? 0 : 1);
      };
      if (topp_on) bL = min(bL, first_bin(fe + f0 >= lo_t, fi >= lo_t));
      if (topk_on) bL = min(bL, first_bin(ce + c0 >= P.top_k, ci >= P.top_k));
      if (bL > bstar) bL = bstar;
      if (lane == 0) {
        s.ured[37] = (uint32_t)bstar;
        s.ured[36] = nb >= NBIN;
        s.ured[35] = (uint32_t)bL;
      }
    }
    cbar();
    const int bstar = (int)s.ured[37];
    const bool whole = s.ured[36] != 0u;
    const int bL = (int)s.ured[35];
    // all of the window sorted and its mass clear of top_p: every element of
    // it is kept, the next one (outside) is the first dropped
    const double tp_clear = (double)tp32 + 2e-6;
    unsigned long long* nuc = P.nuc != nullptr ? P.nuc + (int64_t)v * NUC_MAX : nullptr;
    double zp = 0.0;
    for (int base = 0; base < nl; base += CT) {
      const int i = base + t;
      const bool in = i < nl;
      const unsigned long long key = in ? H.key[i] : 0ull;
      const int bin = in ? (int)s.u.l.bin8[i] : NBIN_PAD;
      const bool pre = bin < bL;
      const bool sel = bin >= bL && bin <= bstar;
      if (pre) zp += (double)__fmul_rn(s.u.l.ecache[i], inv_s);
      // kept for sure: straight into the stored kept set (order is free
      // there); boundary bins: to be sorted.  One shared atomic per warp for
      // both counts (each below 2^16: at most LIST_CAP elements).
      const unsigned pm = __ballot_sync(0xffffffffu, pre);
      const unsigned sm = __ballot_sync(0xffffffffu, sel);
      if (pm | sm) {
        const int leader = __ffs(pm | sm) - 1;
        uint32_t b0 = 0u;
        if (lane == leader)
          b0 = atomicAdd(&s.npre_nsel, (uint32_t)__popc(pm) | ((uint32_t)__popc(sm) << 16));
        b0 = __shfl_sync(0xffffffffu, b0, leader);
        const unsigned lt = (1u << lane) - 1u;
        if (pre) {
          const int o = (int)(b0 & 0xFFFFu) + __popc(pm & lt);
          if (nuc != nullptr && o < NUC_MAX) nuc[o] = key;
        }
        if (sel) {
          const int o = (int)(b0 >> 16) + __popc(sm & lt);
          if (o < SEL_CAP) s.u.l.sel[o] = key;
        }
      }
    }
    const double zpre = c_sum<double>(zp, s.dred);     // (its barriers publish nsel, npre)
    npre = (int)(s.npre_nsel & 0xFFFFu);
    const int nsel = (int)(s.npre_nsel >> 16);
    if (nsel > SEL_CAP || nsel < 1) return fallback_why(s, FB_SELECT);
    if (nsel <= 32) {
      // one warp: register sort, shuffle scans
      if (t < 32) {
        unsigned long long key = lane < nsel ? s.u.l.sel[lane] : 0ull;
        key = warp_sort_desc(key);
        s.u.l.sel[lane] = key;
        const bool valid = lane < nsel;
        const float xv = valid ? list_val(key) : 0.f;
        const float p = valid ? __fmul_rn(softmax_num(xv, P.T, m), inv_s) : 0.f;
        int n_eff = nsel, Lw = -1;
        bool exact = false;
        float kx = -INFINITY;
        if (topk_on) {
          const int kl = P.top_k - 1 - npre;
          if (kl < 0 || kl >= nsel) {
            exact = true;
          } else {
            kx = __shfl_sync(0xffffffffu, xv, kl);
            n_eff = __popc(__ballot_sync(0xffffffffu, valid && xv >= kx));
          }
        }
        Lw = n_eff - 1;
        if (!exact && topp_on) {
          const double incl = zpre + warp_incl_scan<double>(lane < n_eff ? (double)p : 0.0);
          const float cl = __fsub_rn(__double2float_rn(incl), p);
          const unsigned dm = __ballot_sync(0xffffffffu,
                                            lane < n_eff && npre + lane > 0 && !(cl < tp32));
          const double last = __shfl_sync(0xffffffffu, incl, n_eff - 1);
          if (dm) {
            const int D = __ffs(dm) - 1;
            if (D == 0) exact = true;                    // boundary above the sorted part
            else Lw = D - 1;
          } else if (!topk_on && !(whole && last >= tp_clear)) {
            exact = true;                                // boundary deeper
          }
        }
        const double zs = zpre + warp_sum<double>(lane <= Lw ? (double)p : 0.0);
        if (lane == 0) { s.sc_L = exact ? -1 : Lw; s.z = zs; s.fred[39] = kx; }
      }
      cbar();
      if (s.sc_L < 0) return fallback_why(s, FB_BOUNDARY);
      L = s.sc_L;
      kth_x = s.fred[39];
      z = s.z;
    } else {
      int N = 1;
      while (N < nsel) N <<= 1;
      for (int i = nsel + t; i < N; i += CT) s.u.l.sel[i] = 0ull;
      cbar();
      bitonic_sort(s.u.l.sel, N, true);
      for (int i = t; i < nsel; i += CT)
        s.u.l.p[i] = __fmul_rn(softmax_num(list_val(s.u.l.sel[i]), P.T, m), inv_s);
      cbar();
      int n_eff = nsel;
      if (topk_on) {
        const int kl = P.top_k - 1 - npre;
        if (kl < 0 || kl >= nsel) return fallback_why(s, FB_BOUNDARY);
        kth_x = list_val(s.u.l.sel[kl]);
        int c = 0;
        for (int i = t; i < nsel; i += CT) c += list_val(s.u.l.sel[i]) >= kth_x;
        n_eff = c_sum<int>(c, reinterpret_cast<int*>(s.ured));
      }
      if (topp_on) {
        if (t == 0) s.sc_L = 0x7FFFFFFF;
        cbar();
        double carry = zpre;
        for (int base = 0; base < n_eff; base += CT) {
          const int i = base + t;
          const float p = i < n_eff ? s.u.l.p[i] : 0.f;
          double tot;
          const double pre = c_excl_scan<double>((double)p, s.dred, &tot);
          if (i < n_eff && npre + i > 0) {
            const float cl = __fsub_rn(__double2float_rn(carry + pre + (double)p), p);
            if (!(cl < tp32)) atomicMin(&s.sc_L, i);
          }
          carry += tot;
          cbar();
          if (s.sc_L != 0x7FFFFFFF) break;
        }
        const int D = s.sc_L;
        if (D == 0) return fallback_why(s, FB_BOUNDARY);   // boundary above the sorted part
        if (D != 0x7FFFFFFF) L = D - 1;
        else if (topk_on || (whole && carry >= tp_clear)) L = n_eff - 1;
        else return fallback_why(s, FB_BOUNDARY);         // boundary below the sorted part
      } else {
        L = n_eff - 1;
      }
      double zs = 0.0;
      for (int i = t; i <= L; i += CT) zs += (double)s.u.l.p[i];
      z = zpre + c_sum<double>(zs, s.dred);
    }
  } else {
    z = S * (double)inv_s;
  }
  const float zf = fmaxf(__double2float_rn(z), 1e-12f);
  const int nkept = npre + L + 1;
  const bool listed = P.nuc != nullptr && !all_kept && nkept <= NUC_MAX;
  if (listed) {
    unsigned long long* dst = P.nuc + (int64_t)v * NUC_MAX + npre;
    for (int i = t; i <= L; i += CT) dst[i] = s.u.l.sel[i];
  }
  if (t == 0) {
    VecStats o;
    o.m = m;
    o.inv_s = inv_s;
    o.zf = zf;
    o.kth = topk_on ? fkey(kth_x) : 0u;
    o.vstar = all_kept ? 0u : (uint32_t)(s.u.l.sel[L] >> 32);
    o.idx_cut = all_kept ? (int32_t)NO_CUT : (int32_t)list_idx(s.u.l.sel[L]);
    o.argmax = -1;
    o.flags = (all_kept ? F_ALLKEPT : 0) | (listed ? F_LISTED : 0);
    o.n_keep = all_kept ? -1 : nkept;
    o.fb_why = 0;
    o.pad = 0;
    o.probe_p = has_probe ? stats_prob_x(o, xprobe, P.T, probe) : 0.f;
    P.stats[v] = o;
  }
  cbar();
  return false;
}

// The row's accept test and its residual / bonus draw (consumer threads of the
// CTA that finished the row's last vector).
__device__ void finish_row(HistSmem& s, const StatsParams& P, int row) {
  const int t = ftid();
  const int npos0 = P.vs.npos[0], npos = P.vs.npos[0] + P.vs.npos[1];
  const int vrow = row * npos;
  const int k = P.k;
  __threadfence();
  if (t < 32) {
    // accepted prefix: one lane per draft position
    const int lane = t;
    int n = k;
    for (int base = 0; base < k; base += 32) {
      const int i = base + lane;
      bool acc = false;
      if (i < k) {
        const float pxi = __ldcg(&P.stats[vrow + i].probe_p);
        const float qxi = q_probe(P, row, i);
        const float thr = fminf(__fdiv_rn(pxi, fmaxf(qxi, 1e-10f)), 1.0f);
        if (P.px) P.px[row * k + i] = pxi;
        if (P.qx) P.qx[row * k + i] = qxi;
        acc = P.u_acc[row * P.u_bs + i] < thr;
      }
      const unsigned rm = __ballot_sync(0xffffffffu, i < k && !acc);
      if (rm && n == k) n = base + __ffs(rm) - 1;
    }
    if (P.alive && P.alive[row] == 0) n = 0;
    if (lane == 0) s.sc_n = n;
  }
  cbar();
  const int n = s.sc_n;
  const bool resid = n < k;
  const int ppos = resid ? n : k;
  const VecStats stp = load_stats_cg(P.stats + vrow + ppos);
  VecStats stq = stp;
  const void* xp = vec_ptr(P.vs, 0, row, ppos, P.dtype);
  const void* xq = xp;
  if (resid && !P.qprob) {
    stq = load_stats_cg(P.stats + vrow + npos0 + n);
    xq = vec_ptr(P.vs, 1, row, n, P.dtype);
  }
  const double u = (double)P.u_res[row];
  if ((stp.flags & F_LISTED) && stp.n_keep <= 32) {
    // p's kept set fits one warp: values come with the stored keys, q is
    // gathered at those indices, register sort into vocabulary order
    if (t < 32) {
      const int lane = t;
      const int cnt = stp.n_keep;
      const bool valid = lane < cnt;
      const unsigned long long key =
          valid ? __ldcg(P.nuc + (int64_t)(vrow + ppos) * NUC_MAX + lane) : 0ull;
      int jj = valid ? (int)list_idx(key) : 0x7FFFFFFF;
      float pp = valid ? __fdiv_rn(prob_of(list_val(key), P.T, stp.m, stp.inv_s), stp.zf) : 0.f;
      float rr = pp;
      if (resid && valid && pp != 0.f)
        rr = fmaxf(__fsub_rn(pp, q_at(P, stq, xq, row, n, jj)), 0.f);
#pragma unroll
      for (int k2 = 2; k2 <= 32; k2 <<= 1) {
#pragma unroll
        for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
          const int oj = __shfl_xor_sync(0xffffffffu, jj, j2);
          const float orr = __shfl_xor_sync(0xffffffffu, rr, j2);
          const float opp = __shfl_xor_sync(0xffffffffu, pp, j2);
          const bool take_min = ((lane & j2) == 0) == ((lane & k2) == 0);
          if (take_min ? (oj < jj) : (oj > jj)) { jj = oj; rr = orr; pp = opp; }
        }
      }
      double R = warp_sum<double>((double)rr);
      if (resid && __double2float_rn(R) <= 1e-9f) {         // sampling.py:86-89: fall back to p
        rr = pp;
        R = warp_sum<double>((double)pp);
      }
      const double tgt = u * R;
      const double pre = warp_incl_scan<double>((double)rr) - (double)rr;
      const unsigned hm =
          __ballot_sync(0xffffffffu, lane < cnt && pre <= tgt && pre + (double)rr > tgt);
      int ly = 0;
      if (hm) {
        ly = __ffs(hm) - 1;
      } else {
        const unsigned pm = __ballot_sync(0xffffffffu, lane < cnt && rr > 0.f);
        if (pm) ly = 31 - __clz(pm);
      }
      const int yy = __shfl_sync(0xffffffffu, jj, ly);
      const float ypp = __shfl_sync(0xffffffffu, pp, ly);
      if (lane == 0) {
        if (P.n_acc) P.n_acc[row] = n;
        P.y[row] = yy;
        if (P.y_prob) P.y_prob[row] = ypp;
        P.row_ctr[row] = 0;
      }
    }
    cbar();
    return;
  }
  if (t == 0) s.sc_y = -1;
  cbar();
  if ((stp.flags & F_LISTED) && stp.n_keep <= RANK_MAX) {
    // p's kept set (values from the stored keys, q gathered at their
    // indices); each element's exclusive prefix in vocabulary order is summed
    // directly over the set (no sort): the draw is the element whose
    // [prefix, prefix + r) holds u * R
    constexpr int PER = RANK_MAX / CT;
    const int cnt = stp.n_keep;
    const unsigned long long* src = P.nuc + (int64_t)(vrow + ppos) * NUC_MAX;
    float* ra = s.u.l.p;                       // r, then p at RANK_MAX
    double rs = 0.0, ps = 0.0;
    uint32_t jmine[PER];
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int i = t + q * CT;
      jmine[q] = 0xFFFFFFFFu;
      if (i < cnt) {
        const unsigned long long key = __ldcg(src + i);
        const uint32_t j = list_idx(key);
        const float pj = __fdiv_rn(prob_of(list_val(key), P.T, stp.m, stp.inv_s), stp.zf);
        float r = pj;
        if (resid && pj != 0.f)
          r = fmaxf(__fsub_rn(pj, q_at(P, stq, xq, row, n, (int64_t)j)), 0.f);
        s.u.l.sel[i] = j;
        ra[i] = r;
        ra[RANK_MAX + i] = pj;
        rs += (double)r;
        ps += (double)pj;
        jmine[q] = j;
      }
    }
    if (t == 0) { s.ured[29] = 0xFFFFFFFFu; s.ured[30] = 0xFFFFFFFFu; s.ured[31] = 0u; }
    double R = c_sum<double>(rs, s.dred);
    const double Pm = c_sum<double>(ps, s.dred);
    const bool use_p = !resid || __double2float_rn(R) <= 1e-9f;   // sampling.py:86-89
    if (use_p) { R = Pm; ra += RANK_MAX; }
    const double tgt = u * R;
#pragma unroll
    for (int q = 0; q < PER; ++q) {
      const int i = t + q * CT;
      if (i < cnt) {
        const uint32_t j = jmine[q];
        double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
        int k = 0;
        for (; k + 4 <= cnt; k += 4) {
          if ((uint32_t)s.u.l.sel[k] < j) a0 += (double)ra[k];
          if ((uint32_t)s.u.l.sel[k + 1] < j) a1 += (double)ra[k + 1];
          if ((uint32_t)s.u.l.sel[k + 2] < j) a2 += (double)ra[k + 2];
          if ((uint32_t)s.u.l.sel[k + 3] < j) a3 += (double)ra[k + 3];
        }
        for (; k < cnt; ++k)
          if ((uint32_t)s.u.l.sel[k] < j) a0 += (double)ra[k];
        const double pre = (a0 + a1) + (a2 + a3);
        const float r = ra[i];
        if (pre <= tgt && pre + (double)r > tgt) atomicMin(&s.ured[30], j);
        if (r > 0.f) atomicMax(&s.ured[31], j + 1u);
        atomicMin(&s.ured[29], j);
      }
    }
    cbar();
    if (t == 0)
      s.sc_y = s.ured[30] != 0xFFFFFFFFu ? (long long)s.ured[30]
               : s.ured[31] > 0u ? (long long)(s.ured[31] - 1u) : (long long)s.ured[29];
  } else if (stp.flags & F_LISTED) {
    const int cnt = stp.n_keep;
    int N = 1;
    while (N < cnt) N <<= 1;
    const unsigned long long* src = P.nuc + (int64_t)(vrow + ppos) * NUC_MAX;
    for (int i = t; i < N; i += CT)
      s.u.l.sel[i] = i < cnt ? (unsigned long long)list_idx(__ldcg(src + i)) : ~0ull;
    cbar();
    bitonic_sort(s.u.l.sel, N, false);        // kept elements in vocabulary order
    double rs = 0.0;
    for (int i = t; i < cnt; i += CT) {
      const int64_t j = (int64_t)s.u.l.sel[i];
      const float pj = stats_prob(stp, xp, P.dtype, P.T, j);
      float r = pj;
      if (resid && pj != 0.f) r = fmaxf(__fsub_rn(pj, q_at(P, stq, xq, row, n, j)), 0.f);
      s.u.l.p[i] = r;
      rs += (double)r;
    }
    double R = c_sum<double>(rs, s.dred);
    if (resid && __double2float_rn(R) <= 1e-9f) {        // sampling.py:86-89: fall back to p
      rs = 0.0;
      for (int i = t; i < cnt; i += CT) {
        const float pj = stats_prob(stp, xp, P.dtype, P.T, (int64_t)s.u.l.sel[i]);
        s.u.l.p[i] = pj;
        rs += (double)pj;
      }
      R = c_sum<double>(rs, s.dred);
    }
    const double tgt = u * R;
    double carry = 0.0;
    for (int base = 0; base < cnt; base += CT) {
      const int i = base + t;
      const float r = i < cnt ? s.u.l.p[i] : 0.f;
      double tot;
      const double pre = c_excl_scan<double>((double)r, s.dred, &tot);
      if (i < cnt && carry + pre <= tgt && carry + pre + (double)r > tgt)
        s.sc_y = (long long)s.u.l.sel[i];
      carry += tot;
      cbar();
      if (s.sc_y >= 0) break;
    }
    if (t == 0 && s.sc_y < 0) {
      for (int i = cnt - 1; i >= 0; --i)
        if (s.u.l.p[i] > 0.f) { s.sc_y = (long long)s.u.l.sel[i]; break; }
      if (s.sc_y < 0) s.sc_y = (long long)s.u.l.sel[0];
    }
  } else {
    // kept set not listed: two ordered passes over the whole vocabulary
    constexpr int PT = 8;
    double rs = 0.0, ps = 0.0;
    for (int j = t; j < P.V; j += CT) {
      const float pj = stats_prob(stp, xp, P.dtype, P.T, j);
      ps += (double)pj;
      if (resid && pj != 0.f) rs += (double)fmaxf(__fsub_rn(pj, q_at(P, stq, xq, row, n, j)), 0.f);
    }
    double R = c_sum<double>(rs, s.dred);
    const double Pm = c_sum<double>(ps, s.dred);
    const bool use_p = !resid || __double2float_rn(R) <= 1e-9f;
    if (use_p) R = Pm;
    const double tgt = u * R;
    double carry = 0.0;
    for (int base = 0; base < P.V; base += CT * PT) {
      const int j0 = base + t * PT;
      float r[PT];
      double ls = 0.0;
#pragma unroll
      for (int e = 0; e < PT; ++e) {
        const int j = j0 + e;
        float v = 0.f;
        if (j < P.V) {
          v = stats_prob(stp, xp, P.dtype, P.T, j);
          if (!use_p && v != 0.f) v = fmaxf(__fsub_rn(v, q_at(P, stq, xq, row, n, j)), 0.f);
        }
        r[e] = v;
        ls += (double)v;
      }
      double tot;
      const double pre = c_excl_scan<double>(ls, s.dred, &tot);
      if (carry + pre <= tgt && carry + pre + ls > tgt) {
        double run = carry + pre;
#pragma unroll
        for (int e = 0; e < PT; ++e) {
          run += (double)r[e];
          if (run > tgt) { s.sc_y = j0 + e; break; }
        }
      }
      carry += tot;
      cbar();
      if (s.sc_y >= 0) break;
    }
    if (t == 0 && s.sc_y < 0) {
      for (int j = P.V - 1; j >= 0; --j) {
        float v = stats_prob(stp, xp, P.dtype, P.T, j);
        if (!use_p && v != 0.f) v = fmaxf(__fsub_rn(v, q_at(P, stq, xq, row, n, j)), 0.f);
        if (v > 0.f) { s.sc_y = j; break; }
      }
      if (s.sc_y < 0) s.sc_y = 0;
    }
  }
  cbar();
  if (t == 0) {
    const int64_t yy = s.sc_y;
    if (P.n_acc) P.n_acc[row] = n;
    P.y[row] = yy;
    if (P.y_prob) P.y_prob[row] = stats_prob(stp, xp, P.dtype, P.T, yy);
    P.row_ctr[row] = 0;
  }
  cbar();
}

// ---------------------------------------------------------------------------
// exact fallback (bf16 / fp16): vectors the list path cannot decide
// ---------------------------------------------------------------------------
// The finalize warps defer a vector (VecStats.flags F_DEFER) when its list
// overflows or the top-k / top-p boundary lies below the list window: flat
// distributions, high temperatures, top-p near 1.  Once the CTA has streamed
// all its vectors, all its threads take its deferred vectors one at a time
// and compute them exactly from a 65,536-bin count histogram of the vector's
// 16-bit values in shared memory (the ring's memory)
// (two 16-bit counters per word, a counter that wraps is logged as a +65536
// correction): every element of one value has the same probability, so the
// normaliser, the top-k value and the top-p boundary follow from per-value
// counts, walked in descending value order with each thread owning 64
// consecutive values and one block scan carrying the mass across threads.
// Within the boundary value, the kept members are the first ones in
// vocabulary order (the stable-sort tie policy): the n-th is found by one
// counting pass over the vector.  The CTA that completes a row then performs
// the row's accept test and draw with all its threads: two ordered passes
// over the pick vector's vocabulary (each thread a contiguous slice, block
// scans in between).


__device__ __forceinline__ void fb_corr(HistSmem& s, FbScratch& h, uint32_t raw, int add) {
  const int i = atomicAdd(&s.ncorr, 1);
  if (i < NCORR_MAX) { h.corr_raw[i] = raw; h.corr_add[i] = add; }
  else s.corr_full = 1;
}

// Count one 16-bit pattern; a wrap of its 16-bit counter (the returned old
// word shows it) is logged as a correction.
__device__ __forceinline__ void fb_count(HistSmem& s, FbScratch& h, uint32_t raw) {
  const uint32_t inc = 1u << ((raw & 1u) << 4);
  const uint32_t old = atomicAdd(&h.hist[raw >> 1], inc);
  if ((raw & 1u) == 0u) {
    if ((old & 0xFFFFu) == 0xFFFFu) {        // low counter wrapped, carried into high
      fb_corr(s, h, raw, 65536);
      fb_corr(s, h, raw + 1, -1);
      if ((old >> 16) == 0xFFFFu) fb_corr(s, h, raw + 1, 65536);
    }
  } else if ((old >> 16) == 0xFFFFu) {      // high counter wrapped out of the word
    fb_corr(s, h, raw, 65536);
  }
}

// Count one 16-bit pattern without reading the counter back (a reduction,
// no round trip); a wrap shows up afterwards as a total below V.
__device__ __forceinline__ void fb_count_fast(FbScratch& h, uint32_t raw) {
  atomicAdd(&h.hist[raw >> 1], 1u << ((raw & 1u) << 4));
}

// Elements of 16-bit value `raw` (-0 counted with +0, its key being +0's).
__device__ __forceinline__ uint32_t fb_get(const FbScratch& h, uint32_t raw, int ncorr) {
  uint32_t c = (h.hist[raw >> 1] >> ((raw & 1u) << 4)) & 0xFFFFu;
  for (int i = 0; i < ncorr; ++i)
    if (h.corr_raw[i] == raw) c += (uint32_t)h.corr_add[i];
  if (raw == 0u) {
    c += (h.hist[0x8000u >> 1] >> ((0x8000u & 1u) << 4)) & 0xFFFFu;
    for (int i = 0; i < ncorr; ++i)
      if (h.corr_raw[i] == 0x8000u) c += (uint32_t)h.corr_add[i];
  }
  return c;
}
__device__ __forceinline__ uint32_t fb_count_key(const FbScratch& h, uint32_t key, int ncorr) {
  const uint32_t raw = raw16(key);
  return raw == 0x8000u ? 0u : fb_get(h, raw, ncorr);   // -0 lives in +0's class
}

// Keys are visited in chunks of NT consecutive keys, descending: in chunk c
// thread t holds key 65535 - NT c - t (none past the last key), so
// neighbouring threads read neighbouring counters (no bank conflicts) and
// thread order is descending key order within a chunk.
template <int NT>
__device__ __forceinline__ uint32_t fb_chunk_count(const FbScratch& h, int c, int t, int ncorr,
                                                   uint32_t* key) {
  const int i = NT * c + t;
  *key = 65535u - (uint32_t)i;
  return i < 65536 ? fb_count_key(h, *key, ncorr) : 0u;
}

// Exact stats of vector v (all NT threads of the CTA).
template <int NT>
__device__ void fb_vector(HistSmem& s, FbScratch& h, const StatsParams& P, int v,
                          const uint16_t* x, int64_t probe, int fb_why) {
  const int t = threadIdx.x;
  const int V = P.V;
  const bool topk_on = P.top_k > 0 && P.top_k < V;
  const bool topp_on = P.top_p > 0.0f && P.top_p < 1.0f;
  const float tp32 = P.top_p;
  // A: the histogram (16-byte loads, neighbouring threads on neighbouring
  // units, two loads in flight per thread); counters are incremented without
  // reading them back, and a wrap (more than 65,535 equal values) is caught
  // by the total and recounted with checked increments
  constexpr int NCH = (65536 + NT - 1) / NT;
  static_assert(NCH <= 128, "chunk mask");
  const VecGeom gm(x, V);
  const uint4* body = reinterpret_cast<const uint4*>(x + gm.head);
  uint4* h4 = reinterpret_cast<uint4*>(h.hist);
  uint32_t occ[4];
  uint32_t kmax = 0u;
  for (int pass = 0; pass < 2; ++pass) {
    for (int i = t; i < HIST_WORDS / 4; i += NT) h4[i] = make_uint4(0, 0, 0, 0);
    if (t == 0) { s.ncorr = 0; s.corr_full = 0; }
    __syncthreads();
    for (int u = t; u < gm.nunits; u += 2 * NT) {
      const uint4 q0 = __ldg(body + u);
      const bool two = u + NT < gm.nunits;
      const uint4 q1 = two ? __ldg(body + u + NT) : make_uint4(0, 0, 0, 0);
      const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < 4 || two) {
          if (pass == 0) { fb_count_fast(h, w[i] & 0xFFFFu); fb_count_fast(h, w[i] >> 16); }
          else { fb_count(s, h, w[i] & 0xFFFFu); fb_count(s, h, w[i] >> 16); }
        }
      }
    }
    uint32_t rr = 0xFFFFFFFFu;
    if (t < gm.head) rr = __ldg(x + t);
    else if (t < gm.head + V - gm.tail0) rr = __ldg(x + gm.tail0 + (t - gm.head));
    if (rr != 0xFFFFFFFFu) { if (pass == 0) fb_count_fast(h, rr); else fb_count(s, h, rr); }
    if (t < 4) s.ured[34 + t] = 0u;
    __syncthreads();
    // B: populated chunks (one OR reduction), the maximum, the total
    const int ncorr = min(s.ncorr, NCORR_MAX);
    uint32_t lmask[4] = {0u, 0u, 0u, 0u};
    uint32_t cnt = 0u;
    kmax = 0u;
    for (int c = 0; c < NCH; ++c) {
      uint32_t key;
      const uint32_t n = fb_chunk_count<NT>(h, c, t, ncorr, &key);
      if (n) {
        if (kmax == 0u) kmax = key;                   // this thread's largest populated key
        lmask[c >> 5] |= 1u << (c & 31);
        cnt += n;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t m4 = __reduce_or_sync(0xffffffffu, lmask[i]);
      if ((t & 31) == 0 && m4) atomicOr(&s.ured[34 + i], m4);
    }
    const uint32_t total = block_sum<uint32_t>(cnt, s.ured);   // (its barriers publish the mask)
#pragma unroll
    for (int i = 0; i < 4; ++i) occ[i] = s.ured[34 + i];
    if (total == (uint32_t)V) break;                  // (uniform) no counter wrapped
  }
  const int ncorr = min(s.ncorr, NCORR_MAX);
  const int flags = F_FALLBACK | (s.corr_full ? F_INEXACT : 0);
  const uint32_t maxkey = block_max<uint32_t>(kmax, s.ured, 0u);
  const float m = scaled_logit(bits16_to_float(raw16(maxkey), P.dtype), P.T);
  // C: the normaliser
  double es = 0.0;
  for (int c = 0; c < NCH; ++c) {
    if (!(occ[c >> 5] >> (c & 31) & 1u)) continue;
    uint32_t key;
    const uint32_t n = fb_chunk_count<NT>(h, c, t, ncorr, &key);
    if (n) es += (double)n * (double)softmax_num(bits16_to_float(raw16(key), P.dtype), P.T, m);
  }
  const double S = block_sum<double>(es, s.dred);
  const float inv_s = __double2float_rn(1.0 / S);
  // D: top-k: the key of the top_k-th element in descending order
  uint32_t keyk = 0u;
  if (topk_on) {
    uint32_t carry = 0u;
    for (int c = 0; c < NCH; ++c) {
      if (!(occ[c >> 5] >> (c & 31) & 1u)) continue;
      uint32_t key;
      const uint32_t n = fb_chunk_count<NT>(h, c, t, ncorr, &key);
      uint32_t tot;
      const uint32_t pre = carry + block_excl_scan<uint32_t>(n, s.ured, &tot);
      if (t == 0) s.ured[37] = 0u;
      __syncthreads();
      if (n && pre < (uint32_t)P.top_k && pre + n >= (uint32_t)P.top_k) s.ured[37] = key;
      __syncthreads();
      keyk = s.ured[37];
      carry += tot;
      if (keyk != 0u || carry >= (uint32_t)P.top_k) break;   // (uniform)
    }
  }
  // E: top-p: walk the kept candidates (keys >= keyk) in descending order
  // with the float64 running mass; the boundary class is the first whose
  // last member is dropped (keep while fl32(cum - p) < top_p)
  uint32_t vstar = 0xFFFFFFFFu;
  int nkeep = 0, vcount = 0;
  double z = 0.0;
  {
    double carry = 0.0;
    if (t == 0) s.ured[38] = 0xFFFFFFFFu;
    __syncthreads();
    for (int c = 0; c < NCH; ++c) {
      if (!(occ[c >> 5] >> (c & 31) & 1u)) continue;
      uint32_t key;
      uint32_t n = fb_chunk_count<NT>(h, c, t, ncorr, &key);
      if (key < keyk) n = 0u;
      const float p = n ? prob_of(bits16_to_float(raw16(key), P.dtype), P.T, m, inv_s) : 0.f;
      const double mine = (double)n * (double)p;
      double tot;
      const double pre = carry + block_excl_scan<double>(mine, s.dred, &tot);
      bool cand = false;
      if (topp_on && n) {
        const float cl = __fsub_rn(__double2float_rn(pre + mine), p);
        cand = !(cl < tp32);
      }
      if (cand) atomicMin(&s.ured[38], (uint32_t)t);   // lowest thread = highest key
      __syncthreads();
      if (s.ured[38] != 0xFFFFFFFFu) {                  // (uniform) the boundary is here
        if ((uint32_t)t == s.ured[38]) {
          int lo = 0, hi = (int)n;                      // largest k with keep(j) for all j < k
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            const float cl = __fsub_rn(__double2float_rn(pre + (double)(mid + 1) * (double)p), p);
            if (cl < tp32) lo = mid + 1; else hi = mid;
          }
          int nk = lo;
          if (nk == 0 && key == maxkey) nk = 1;         // the first sorted entry is always kept
          s.ured[39] = key;
          s.ured[36] = (uint32_t)nk;
          s.sc_n = (int)n;
          s.dred[39] = pre + (double)nk * (double)p;
        }
        __syncthreads();
        vstar = s.ured[39];
        nkeep = (int)s.ured[36];
        vcount = s.sc_n;
        z = s.dred[39];
        break;
      }
      carry += tot;
    }
    if (vstar == 0xFFFFFFFFu) z = carry;
    __syncthreads();
  }
  const float zf = fmaxf(__double2float_rn(z), 1e-12f);
  // F: the nkeep-th member (vocabulary order) of the boundary class, tile by
  // tile (NT groups of 32 consecutive elements per tile)
  int32_t idx_cut = (int32_t)NO_CUT;
  if (vstar != 0xFFFFFFFFu) {
    if (nkeep == 0) {
      idx_cut = -1;
    } else if (nkeep < vcount) {
      const uint32_t r0 = raw16(vstar);
      const bool zero_cls = r0 == 0u;
      if (t == 0) s.ured[37] = (uint32_t)NO_CUT;
      uint32_t carry = 0u;
      for (int base = 0; base < V; base += 32 * NT) {
        const int j0 = base + 32 * t;
        uint32_t c = 0u;
#pragma unroll 8
        for (int e = 0; e < 32; ++e) {
          const int j = j0 + e;
          if (j < V) {
            const uint32_t r = __ldg(x + j);
            c += (r == r0) || (zero_cls && r == 0x8000u);
          }
        }
        uint32_t tot;
        const uint32_t pc = carry + block_excl_scan<uint32_t>(c, s.ured, &tot);
        if (pc < (uint32_t)nkeep && pc + c >= (uint32_t)nkeep) {
          uint32_t rr = pc;
          for (int e = 0; e < 32; ++e) {
            const int j = j0 + e;
            if (j < V) {
              const uint32_t r = __ldg(x + j);
              if ((r == r0) || (zero_cls && r == 0x8000u)) {
                if (++rr == (uint32_t)nkeep) { s.ured[37] = (uint32_t)j; break; }
              }
            }
          }
        }
        carry += tot;
        __syncthreads();
        if (carry >= (uint32_t)nkeep) break;            // (uniform)
      }
      idx_cut = (int32_t)s.ured[37];
    }
  }
  if (t == 0) {
    VecStats o;
    o.m = m;
    o.inv_s = inv_s;
    o.zf = zf;
    o.kth = topk_on ? fkey(bits16_to_float(raw16(keyk), P.dtype)) : 0u;
    o.vstar = vstar == 0xFFFFFFFFu ? 0u : fkey(bits16_to_float(raw16(vstar), P.dtype));
    o.idx_cut = vstar == 0xFFFFFFFFu ? (int32_t)NO_CUT : idx_cut;
    o.argmax = -1;
    o.flags = flags | ((!topp_on && !topk_on) ? F_ALLKEPT : 0);
    o.n_keep = -1;
    o.fb_why = fb_why;
    o.pad = 0;
    float pp = 0.f;
    if (probe >= 0 && probe < V) {
      const float xv = bits16_to_float(__ldg(x + probe), P.dtype);
      const uint32_t kx = fkey(xv);
      const bool kept = kx >= o.kth &&
                        (kx > o.vstar || (kx == o.vstar && probe <= (int64_t)o.idx_cut));
      if (kept) pp = __fdiv_rn(prob_of(xv, P.T, m, inv_s), zf);
    }
    o.probe_p = pp;
    P.stats[v] = o;
  }
  __syncthreads();
}

// The row's accept test and its residual / bonus draw by inverse CDF over the
// whole vocabulary, in vocabulary order (all NT threads; reference
// engine.py:282-303).  Tiles of NT groups of 8 consecutive elements:
// neighbouring threads read neighbouring logits, one block scan per tile
// carries the running mass.  Valid for any pair of stats records.
template <int NT>
__device__ void fb_finish_row(HistSmem& s, const StatsParams& P, int row) {
  const int t = threadIdx.x;
  const int npos0 = P.vs.npos[0], npos = P.vs.npos[0] + P.vs.npos[1];
  const int vrow = row * npos;
  const int k = P.k;
  const int V = P.V;
  if (t < 32) {
    // accepted prefix: one lane per draft position
    const int lane = t;
    int n = k;
    for (int base = 0; base < k; base += 32) {
      const int i = base + lane;
      bool acc = false;
      if (i < k) {
        const float pxi = __ldcg(&P.stats[vrow + i].probe_p);
        const float qxi = q_probe(P, row, i);
        const float thr = fminf(__fdiv_rn(pxi, fmaxf(qxi, 1e-10f)), 1.0f);
        if (P.px) P.px[row * k + i] = pxi;
        if (P.qx) P.qx[row * k + i] = qxi;
        acc = P.u_acc[row * P.u_bs + i] < thr;
      }
      const unsigned rm = __ballot_sync(0xffffffffu, i < k && !acc);
      if (rm && n == k) n = base + __ffs(rm) - 1;
    }
    if (P.alive && P.alive[row] == 0) n = 0;
    if (lane == 0) { s.sc_n = n; s.sc_y = -1; }
  }
  __syncthreads();
  const int n = s.sc_n;
  const bool resid = n < k;
  const int ppos = resid ? n : k;
  const VecStats stp = load_stats_cg(P.stats + vrow + ppos);
  VecStats stq = stp;
  const void* xp = vec_ptr(P.vs, 0, row, ppos, P.dtype);
  const void* xq = xp;
  if (resid && !P.qprob) {
    stq = load_stats_cg(P.stats + vrow + npos0 + n);
    xq = vec_ptr(P.vs, 1, row, n, P.dtype);
  }
  // pass 1: per tile (NT groups of 8 consecutive elements) the residual mass
  // and the kept mass of p, summed per warp into shared memory (the
  // histogram's memory), and the last index with mass of each
  constexpr int NW = NT / 32;
  double* tsum = reinterpret_cast<double*>(&s.w);          // [tiles][NW][2]
  static_assert(((1 << 21) / (8 * NT) + 1) * NW * 2 * sizeof(double) <= sizeof(s.w),
                "tile sums of the largest vocabulary fit the ring's memory");
  const int ntile = (V + 8 * NT - 1) / (8 * NT);
  double rs = 0.0, ps = 0.0;
  int last_r = -1, last_p = -1;
  for (int ti = 0; ti < ntile; ++ti) {
    const int base = ti * 8 * NT;
    double tr = 0.0, tpm = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = base + 8 * t + e;
      if (j < V) {
        const float pj = stats_prob(stp, xp, P.dtype, P.T, j);
        tpm += (double)pj;
        if (pj > 0.f) last_p = j;
        if (resid && pj != 0.f) {
          const float r = fmaxf(__fsub_rn(pj, q_at(P, stq, xq, row, n, j)), 0.f);
          tr += (double)r;
          if (r > 0.f) last_r = j;
        }
      }
    }
    rs += tr;
    ps += tpm;
    tr = warp_sum(tr);
    tpm = warp_sum(tpm);
    if ((t & 31) == 0) {
      tsum[(ti * NW + (t >> 5)) * 2] = tr;
      tsum[(ti * NW + (t >> 5)) * 2 + 1] = tpm;
    }
  }
  const double R = block_sum<double>(rs, s.dred);
  const double Pm = block_sum<double>(ps, s.dred);     // (its barriers publish tsum)
  const bool use_p = !resid || __double2float_rn(R) <= 1e-9f;   // sampling.py:86-89
  const double tgt = (double)P.u_res[row] * (use_p ? Pm : R);
  const int lastv = block_max<int>(use_p ? last_p : last_r, reinterpret_cast<int*>(s.ured), -1);
  // pass 2: the tile holding the crossing from the tile sums (thread 0, in
  // tile order), then that tile alone, recomputed
  if (t == 0) {
    double carry = 0.0;
    int hit = -1;
    double hit_carry = 0.0;
    for (int ti = 0; ti < ntile && hit < 0; ++ti) {
      double tt = 0.0;
      for (int w = 0; w < NW; ++w) tt += tsum[(ti * NW + w) * 2 + (use_p ? 1 : 0)];
      if (carry <= tgt && carry + tt > tgt) { hit = ti; hit_carry = carry; }
      carry += tt;
    }
    s.ured[38] = (uint32_t)hit;
    s.dred[39] = hit_carry;
  }
  __syncthreads();
  const int hit = (int)s.ured[38];
  const double hit_carry = s.dred[39];
  if (hit >= 0) {                                     // (uniform)
    const int base = hit * 8 * NT;
    float vals[8];
    double ls = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = base + 8 * t + e;
      float val = 0.f;
      if (j < V) {
        val = stats_prob(stp, xp, P.dtype, P.T, j);
        if (!use_p && val != 0.f)
          val = fmaxf(__fsub_rn(val, q_at(P, stq, xq, row, n, j)), 0.f);
      }
      vals[e] = val;
      ls += (double)val;
    }
    double tot;
    const double pre = hit_carry + block_excl_scan<double>(ls, s.dred, &tot);
    if (pre <= tgt && pre + ls > tgt) {
      double run = pre;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        run += (double)vals[e];
        if (run > tgt) { s.sc_y = base + 8 * t + e; break; }
      }
    }
    __syncthreads();
  }
  if (t == 0) {
    long long yy = s.sc_y;
    if (yy < 0) yy = lastv >= 0 ? lastv : 0;         // rounding put the crossing past the end
    if (P.n_acc) P.n_acc[row] = n;
    P.y[row] = yy;
    if (P.y_prob) P.y_prob[row] = stats_prob(stp, xp, P.dtype, P.T, yy);
    P.row_ctr[row] = 0;
  }
  __syncthreads();
}

template <int DT>
__global__ void __launch_bounds__(HT, 1) hist_stats_kernel(StatsParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  HistSmem& s = *reinterpret_cast<HistSmem*>(smem_raw);
  // a row-draw pass launched as this grid's programmatic dependent may start
  // its blocks as CTAs of this grid exit; it waits for the whole grid before
  // it reads any stats
  asm volatile("griddepcontrol.launch_dependents;");
  const int V = P.V;
  // log2(e) / T as c2 + c2l, c2 rounded down so that c2l > 0: y(x) is then
  // monotone and y(-inf) = -inf (a negative c2l would give -inf + inf)
  const double c2d = 1.4426950408889634 / (double)P.T;
  const float c2 = __double2float_rd(c2d);
  const float c2l = fmaxf((float)(c2d - (double)c2), __int_as_float(1));
  const float wlist = W_LIST / c2;                      // list window in logit units
  const int npos = P.vs.npos[0] + P.vs.npos[1];

  if (threadIdx.x == 0) {
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], NSW);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.streamed[i], NSW);
      mbar_init(&s.freed[i], 1);
      s.w.st.hand[i].nkey = 0;
      s.w.st.hand[i].gkey = 0u;
    }
    s.abort_flag = 0;
    s.fb_why = 0;
    s.ncorr = 0;
    s.corr_full = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (threadIdx.x == 0) {
    // ---------------- producer warp (lane 0): ring refills
    bool ok = true;
    uint32_t g = 0, issued = 0;
    for (int v = blockIdx.x; v < P.nvec; v += gridDim.x) {
      int set, row, pos;
      vec_locate(P.vs, v, &set, &row, &pos);
      const uint16_t* x = reinterpret_cast<const uint16_t*>(vec_ptr(P.vs, set, row, pos, P.dtype));
      const VecGeom gm(x, V);
      const char* body = reinterpret_cast<const char*>(x + gm.head);
      for (int c = 0; c < gm.nchunk; ++c, ++g) {
        const int sl = g % NSLOT;
        if (g >= NSLOT)
          ok = ok && mbar_wait(&s.empty[sl], ((g - NSLOT) / NSLOT) & 1u, &s.abort_flag);
        if (ok) {
          const uint32_t bytes = (uint32_t)min(SLOT, gm.nunits * 16 - c * SLOT);
          mbar_expect_tx(&s.full[sl], bytes);
          bulk_g2s(s.w.st.ring[sl], body + (size_t)c * SLOT, bytes, &s.full[sl]);
          issued = g + 1;
        }
      }
    }
    if (!ok) {
      // after an abort, let the copies already issued land before the CTA exits
      for (uint32_t gg = issued > (uint32_t)NSLOT ? issued - NSLOT : 0u; gg < issued; ++gg) {
        int dummy = 0;
        mbar_wait(&s.full[gg % NSLOT], (gg / NSLOT) & 1u, &dummy);
      }
      atomicOr(P.status, 1);
    }
  } else if (threadIdx.x < ST0) {
    // producer warp, lanes 1-31: nothing to do until the fallback phase
  }

  else if (threadIdx.x < FIN0) {
    // ---------------- streaming warps
    const int t = threadIdx.x - ST0;
    const int lane = t & 31, wl = t >> 5;
    uint32_t g = 0;
    int vl = 0;
    for (int v = blockIdx.x; v < P.nvec; v += gridDim.x, ++vl) {
      VecHand& H = s.w.st.hand[vl & 1];
      if (vl >= 2)                                   // wait until the finalize warps release it
        __all_sync(0xffffffffu, mbar_wait(&s.freed[vl & 1], ((vl >> 1) - 1) & 1, &s.abort_flag));
      int set, row, pos;
      vec_locate(P.vs, v, &set, &row, &pos);
      const uint16_t* x = reinterpret_cast<const uint16_t*>(vec_ptr(P.vs, set, row, pos, P.dtype));
      const VecGeom gm(x, V);
      Stream st;
      st.Rc2 = -INFINITY; st.m = -INFINITY; st.xt = INFINITY; st.xt2 = 0u; st.eY = 0.f;
      st.bulk = 0.0;
      for (int c = 0; c < gm.nchunk; ++c, ++g) {
        const int sl = g % NSLOT;
        const bool okw = __all_sync(0xffffffffu, mbar_wait(&s.full[sl], (g / NSLOT) & 1u, &s.abort_flag));
        const int units = okw ? min(SLOT, gm.nunits * 16 - c * SLOT) >> 4 : 0;
        const uint4* u4 = reinterpret_cast<const uint4*>(s.w.st.ring[sl]);
        uint32_t w[4 * GPS];
#pragma unroll
        for (int q = 0; q < GPS; ++q) {
          const int u = t + q * ST_N;
          const uint32_t n2 = neg_inf2<DT>();
          const uint4 w4 = u < units ? u4[u] : make_uint4(n2, n2, n2, n2);
          w[4 * q] = w4.x; w[4 * q + 1] = w4.y; w[4 * q + 2] = w4.z; w[4 * q + 3] = w4.w;
        }
        if (c == 0) {
          // the maximum of the chunks already in the ring (no waiting for the
          // later ones): bulk reference of every lane and the first list
          // threshold
          uint32_t pm1[2 * GPS];
          float lm = lane_max<DT, GPS>(w, pm1);
          const int nseed = min(NSLOT, gm.nchunk);
#pragma unroll 1
          for (int i = 1; i < nseed; ++i) {
            const uint32_t gi = g + (uint32_t)i;
            const bool oki = __all_sync(0xffffffffu, mbar_test(&s.full[gi % NSLOT], (gi / NSLOT) & 1u));
            if (oki) {
              const int ui = min(SLOT, gm.nunits * 16 - i * SLOT) >> 4;
              const uint4* wi4 = reinterpret_cast<const uint4*>(s.w.st.ring[gi % NSLOT]);
              uint32_t wi[4 * GPS];
#pragma unroll
              for (int q = 0; q < GPS; ++q) {
                const int u = t + q * ST_N;
                const uint32_t n2 = neg_inf2<DT>();
                const uint4 w4 = u < ui ? wi4[u] : make_uint4(n2, n2, n2, n2);
                wi[4 * q] = w4.x; wi[4 * q + 1] = w4.y; wi[4 * q + 2] = w4.z; wi[4 * q + 3] = w4.w;
              }
              lm = fmaxf(lm, lane_max<DT, GPS>(wi, pm1));
            }
          }
          const uint32_t wk = __reduce_max_sync(0xffffffffu, fkey(lm));
          if (lane == 0) atomicMax(&H.gkey, wk);
          sbar();
          const float r = fkey_value(*reinterpret_cast<volatile uint32_t*>(&H.gkey));
          if (r > -INFINITY) set_ref<DT>(st, r, c2, c2l, wlist);
        }
        if (okw) {
          sync_max<DT>(H, st, c2, c2l, wlist);
          stream_words<DT, GPS, true>(s, H, st, w, sl, (uint32_t)(gm.head + c * (SLOT / 2)), 0u,
                                      c2, c2l, wlist);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.empty[sl]);
      }
      // ragged head / tail elements (< 16 of them), first streaming warp
      const int nrag = gm.head + (V - gm.tail0);
      if (wl == 0 && nrag > 0) {
        const bool valid = lane < nrag;
        const int j = !valid ? 0 : (lane < gm.head ? lane : gm.tail0 + (lane - gm.head));
        constexpr uint32_t NEG16 = neg_inf2<DT>() & 0xFFFFu;
        const uint32_t lo = valid ? (uint32_t)__ldg(x + j) : NEG16;
        const uint32_t wv[4] = {lo | (NEG16 << 16), neg_inf2<DT>(), neg_inf2<DT>(), neg_inf2<DT>()};
        stream_words<DT, 1, false>(s, H, st, wv, 0, 0u, (uint32_t)j, c2, c2l, wlist);
      }
      // the warp's bulk sum, relative to the largest offset among its lanes
      float wr = st.Rc2;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) wr = fmaxf(wr, __shfl_xor_sync(0xffffffffu, wr, o));
      double b = 0.0;
      if (st.Rc2 != -INFINITY && st.bulk > 0.0) b = st.bulk * exp2((double)st.Rc2 - (double)wr);
      b = warp_sum(b);
      if (lane == 0) {
        H.wbulk[wl] = b;
        H.wrc2[wl] = wr;
        mbar_arrive(&s.streamed[vl & 1]);
      }
    }
  } else {

  // ---------------- finalize warps: list -> stats -> row draw, one vector
  // behind the streaming warps
  const int t = ftid();
  int vl = 0;
  for (int v = blockIdx.x; v < P.nvec; v += gridDim.x, ++vl) {
    VecHand& H = s.w.st.hand[vl & 1];
    const uint32_t par = (vl >> 1) & 1;
    if (!mbar_wait(&s.streamed[vl & 1], par, &s.abort_flag)) s.abort_flag = 1;
    cbar();
    if (t == 0) s.fin_skip = *reinterpret_cast<volatile int*>(&s.abort_flag);
    cbar();
    if (!s.fin_skip) {
      int set, row, pos;
      vec_locate(P.vs, v, &set, &row, &pos);
      const uint16_t* x = reinterpret_cast<const uint16_t*>(vec_ptr(P.vs, set, row, pos, P.dtype));
      const int64_t probe = vec_probe(P.vs, set, row, pos);
      // a vector the list cannot decide is deferred to this CTA's fallback
      // phase, which also counts it toward its row
      const bool deferred = finalize_list(s, H, P, v, x, probe, c2, wlist);
      if (deferred && t == 0) {
        VecStats o = {};
        o.flags = F_DEFER;
        o.fb_why = s.fb_why;
        P.stats[v] = o;
      }
      // row bookkeeping: the CTA that completes a row draws for it
      if (P.fused && !deferred) {
        __threadfence();
        cbar();
        if (t == 0) s.last_row = atomicAdd(&P.row_ctr[row], 1) == npos - 1;
        cbar();
        if (s.last_row) finish_row(s, P, row);
      }
    }
    cbar();
    if (t == 0) {
      H.nkey = 0;
      H.gkey = 0u;
      mbar_arrive(&s.freed[vl & 1]);
    }
  }
    if (t == 0 && s.abort_flag) atomicOr(P.status, 1);
  }

  // ---------------- fallback phase: every warp of the CTA, after all its
  // vectors streamed (the ring and hand-over memory is free now)
  __syncthreads();
  if (!*reinterpret_cast<volatile int*>(&s.abort_flag)) {
    for (int v = blockIdx.x; v < P.nvec; v += gridDim.x) {
      const VecStats* sv = P.stats + v;
      if (!(*reinterpret_cast<const volatile int*>(&sv->flags) & F_DEFER)) continue;
      int set, row, pos;
      vec_locate(P.vs, v, &set, &row, &pos);
      const uint16_t* x = reinterpret_cast<const uint16_t*>(vec_ptr(P.vs, set, row, pos, P.dtype));
      fb_vector<HT>(s, s.w.fb, P, v, x, vec_probe(P.vs, set, row, pos),
                    *reinterpret_cast<const volatile int*>(&sv->fb_why));
      if (P.fused) {
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s.last_row = atomicAdd(&P.row_ctr[row], 1) == npos - 1;
        __syncthreads();
        if (s.last_row) fb_finish_row<HT>(s, P, row);
      }
    }
  }
}

// Inverse-CDF draw over p's kept entries when they are listed (up to NUC_MAX
// of them), on all NT threads: each entry's weight (r = (p - q)+ for a
// residual draw, p for the bonus draw, and p again when the residual mass is
// <= 1e-9, sampling.py:86-89), the entries put in vocabulary order by a
// bitonic sort of (index, position) pairs, one block scan of the weights in
// that order, and the entry whose [prefix, prefix + w) holds u * R.  When
// rounding leaves no such entry: the last one with a positive weight, else the
// first (reference engine.py:294-303).
template <int NT>
__device__ void row_draw_listed(HistSmem& s, const StatsParams& P, int row, int n, int ppos,
                                bool resid, const VecStats& stp, const VecStats& stq,
                                const void* xp, const void* xq) {
  const int t = threadIdx.x;
  const int npos = P.vs.npos[0] + P.vs.npos[1];
  const int cnt = stp.n_keep;
  int N = 1;
  while (N < cnt) N <<= 1;                              // <= NUC_MAX <= SEL_CAP
  const unsigned long long* src = P.nuc + (int64_t)(row * npos + ppos) * NUC_MAX;
  float* rr = s.u.l.p;                                  // weight r of entry i
  float* pv = s.u.l.ecache;                             // p of entry i
  double rs = 0.0, ps = 0.0;
  for (int i = t; i < N; i += NT) {
    unsigned long long sk = ~0ull;
    if (i < cnt) {
      const unsigned long long key = __ldcg(src + i);
      const uint32_t j = list_idx(key);
      const float pj = __fdiv_rn(prob_of(list_val(key), P.T, stp.m, stp.inv_s), stp.zf);
      float r = pj;
      if (resid && pj != 0.f)
        r = fmaxf(__fsub_rn(pj, q_at(P, stq, xq, row, n, (int64_t)j)), 0.f);
      rr[i] = r;
      pv[i] = pj;
      rs += (double)r;
      ps += (double)pj;
      sk = ((unsigned long long)j << 32) | (uint32_t)i;
    }
    s.u.l.sel[i] = sk;
  }
  const double R0 = block_sum<double>(rs, s.dred);
  const double Pm = block_sum<double>(ps, s.dred);
  const bool use_p = !resid || __double2float_rn(R0) <= 1e-9f;
  const float* wv = use_p ? pv : rr;
  const double tgt = (double)P.u_res[row] * (use_p ? Pm : R0);
  // ascending (index, position): vocabulary order
  for (int k2 = 2; k2 <= N; k2 <<= 1) {
    for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
      for (int i = t; i < N; i += NT) {
        const int ixj = i ^ j2;
        if (ixj > i) {
          const unsigned long long a = s.u.l.sel[i], b = s.u.l.sel[ixj];
          if (((i & k2) == 0) ? (a > b) : (a < b)) { s.u.l.sel[i] = b; s.u.l.sel[ixj] = a; }
        }
      }
      __syncthreads();
    }
  }
  // each thread E consecutive entries; block scan of their sums
  const int E = (N + NT - 1) / NT;
  double loc = 0.0;
  for (int e = 0; e < E; ++e) {
    const int i = t * E + e;
    if (i < cnt) loc += (double)wv[(uint32_t)s.u.l.sel[i]];
  }
  // (index << 32 | position) of the crossing entry and of the last entry
  // with a positive weight
  unsigned long long* pick = reinterpret_cast<unsigned long long*>(&s.sc_pre);
  unsigned long long* last = reinterpret_cast<unsigned long long*>(&s.sc_y);   // + 1; 0: none
  if (t == 0) { pick[0] = ~0ull; *last = 0ull; }
  double tot;
  double run = block_excl_scan<double>(loc, s.dred, &tot);
  for (int e = 0; e < E; ++e) {
    const int i = t * E + e;
    if (i < cnt) {
      const unsigned long long sk = s.u.l.sel[i];
      const float w = wv[(uint32_t)sk];
      if (run <= tgt && run + (double)w > tgt) atomicMin(pick, sk);
      if (w > 0.f) atomicMax(last, sk + 1ull);
      run += (double)w;
    }
  }
  __syncthreads();
  if (t == 0) {
    const unsigned long long sk = pick[0] != ~0ull ? pick[0]
                                  : *last > 0ull ? *last - 1ull : s.u.l.sel[0];
    if (P.n_acc) P.n_acc[row] = n;
    P.y[row] = (int64_t)(sk >> 32);
    if (P.y_prob) P.y_prob[row] = pv[(uint32_t)sk];   // = p at the drawn index
  }
}

// Row draws of a truncated sampling call, after the stats kernel: one CTA per
// row (the stats kernel's thread layout and shared memory), launched as its
// programmatic dependent so the launch overlaps the stats kernel's tail.
// Warp 0 takes the accept test (the accepted prefix n, and p(x_i), q(x_i));
// the draw then follows the kept set of the pick vector: at most 32 listed
// entries, one warp (finish_row); more listed entries, all threads
// (row_draw_listed); a kept set that is not listed (the exact fallback's
// vectors), all threads over the whole vocabulary (fb_finish_row).
__global__ void __launch_bounds__(HT, 1) row_draw_kernel(StatsParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  HistSmem& s = *reinterpret_cast<HistSmem*>(smem_raw);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x;
  const int npos0 = P.vs.npos[0], npos = P.vs.npos[0] + P.vs.npos[1];
  const int vrow = row * npos;
  const int k = P.k;
  // the row's stats records, all in one round trip (npos * 48 bytes)
  VecStats* rst = reinterpret_cast<VecStats*>(s.u.l.ecache);
  {
    const int* src = reinterpret_cast<const int*>(P.stats + vrow);
    int* dst = reinterpret_cast<int*>(rst);
    for (int i = threadIdx.x; i < npos * 12; i += HT) dst[i] = __ldcg(src + i);
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // accepted prefix: one lane per draft position (engine.py:286-293)
    const int lane = threadIdx.x;
    int n = k;
    for (int base = 0; base < k; base += 32) {
      const int i = base + lane;
      bool acc = false;
      if (i < k) {
        const float pxi = rst[i].probe_p;
        const float qxi = P.qprob ? q_probe(P, row, i) : rst[npos0 + i].probe_p;
        const float thr = fminf(__fdiv_rn(pxi, fmaxf(qxi, 1e-10f)), 1.0f);
        if (P.px) P.px[row * k + i] = pxi;
        if (P.qx) P.qx[row * k + i] = qxi;
        acc = P.u_acc[row * P.u_bs + i] < thr;
      }
      const unsigned rm = __ballot_sync(0xffffffffu, i < k && !acc);
      if (rm && n == k) n = base + __ffs(rm) - 1;
    }
    if (P.alive && P.alive[row] == 0) n = 0;
    if (lane == 0) s.sc_n = n;
  }
  __syncthreads();
  const int n = s.sc_n;
  const bool resid = n < k;
  const int ppos = resid ? n : k;
  const VecStats stp = rst[ppos];
  const VecStats stq = resid && !P.qprob ? rst[npos0 + n] : stp;
  __syncthreads();                                    // rst is overwritten below
  if (!(stp.flags & F_LISTED)) {
    fb_finish_row<HT>(s, P, row);
    return;
  }
  if (stp.n_keep <= 32) {
    if (threadIdx.x >= FIN0) finish_row(s, P, row);
    return;
  }
  const void* xp = vec_ptr(P.vs, 0, row, ppos, P.dtype);
  const void* xq = resid && !P.qprob ? vec_ptr(P.vs, 1, row, n, P.dtype) : xp;
  row_draw_listed<HT>(s, P, row, n, ppos, resid, stp, stq, xp, xq);
}

// ---------------------------------------------------------------------------
// small-vocabulary exact kernel: materialises the final probabilities
// ---------------------------------------------------------------------------
struct SmallParams {
  VecSet vs;
  int dtype, V, nvec;
  float T, top_p;
  int top_k;
  VecStats* stats;
  float* mat;          // [nvec, V]
  int* zero_ctr;
  int n_ctr;
};

__global__ void __launch_bounds__(ST) small_stats_kernel(SmallParams P) {
  __shared__ float pv[SMALLV_MAX];
  __shared__ unsigned long long sk[SMALLV_MAX];
  __shared__ double dred[40];
  __shared__ float fred[40];
  const int v = blockIdx.x, t = threadIdx.x, V = P.V;
  for (int i = v * ST + t; i < P.n_ctr; i += gridDim.x * ST) P.zero_ctr[i] = 0;
  int set, row, pos;
  vec_locate(P.vs, v, &set, &row, &pos);
  const void* x = vec_ptr(P.vs, set, row, pos, P.dtype);
  const int64_t probe = vec_probe(P.vs, set, row, pos);
  float* out = P.mat + (int64_t)v * V;

  float lmax = -INFINITY;
  for (int j = t; j < V; j += ST) {
    const float d = scaled_logit(load_logit(x, P.dtype, j), P.T);
    pv[j] = d;
    lmax = fmaxf(lmax, d);
  }
  const float m = block_max<float>(lmax, fred, -INFINITY);
  double es = 0.0;
  for (int j = t; j < V; j += ST) {
    const float e = expf(__fsub_rn(pv[j], m));
    pv[j] = e;
    es += (double)e;
  }
  const double S = block_sum<double>(es, dred);
  const float inv_s = __double2float_rn(1.0 / S);
  int N = 1;
  while (N < V) N <<= 1;
  for (int j = t; j < N; j += ST) {
    if (j < V) {
      const float p = __fmul_rn(pv[j], inv_s);
      pv[j] = p;
      sk[j] = ((unsigned long long)fkey(p) << 32) | (0xFFFFFFFFu - (uint32_t)j);
    } else {
      sk[j] = 0ull;
    }
  }
  __syncthreads();
  const bool topk_on = P.top_k > 0 && P.top_k < V;
  const bool topp_on = P.top_p > 0.0f && P.top_p < 1.0f;
  if (topk_on || topp_on) {
    // bitonic sort, descending
    for (int k2 = 2; k2 <= N; k2 <<= 1) {
      for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
        for (int i = t; i < N; i += ST) {
          const int ixj = i ^ j2;
          if (ixj > i) {
            const unsigned long long a = sk[i], b = sk[ixj];
            const bool desc = (i & k2) == 0;
            if (desc ? (a < b) : (a > b)) { sk[i] = b; sk[ixj] = a; }
          }
        }
        __syncthreads();
      }
    }
    // sorted entries: p = pv[idx]; top-k: keep p >= p of entry top_k-1
    float kth = 0.f;
    if (topk_on) kth = pv[0xFFFFFFFFu - (uint32_t)(sk[P.top_k - 1] & 0xFFFFFFFFu)];
    __syncthreads();
    if (topk_on) {
      for (int j = t; j < V; j += ST)
        if (pv[j] < kth) pv[j] = 0.f;
      __syncthreads();
    }
    if (topp_on) {
      // float64 running sum in sorted order, processed in tiles of ST
      const float tp32 = P.top_p;
      double carry = 0.0;
      for (int base = 0; base < V; base += ST) {
        const int i = base + t;
        uint32_t idx = 0;
        float p = 0.f;
        if (i < V) { idx = 0xFFFFFFFFu - (uint32_t)(sk[i] & 0xFFFFFFFFu); p = pv[idx]; }
        double tot;
        const double pre = block_excl_scan<double>((double)p, dred, &tot);
        bool keep = true;
        if (i < V) {
          const float cum = __double2float_rn(carry + pre + (double)p);
          keep = __fsub_rn(cum, p) < tp32 || i == 0;
        }
        __syncthreads();
        if (i < V && !keep) pv[idx] = -pv[idx] - 1.0f;   // mark dropped, keep value
        carry += tot;
        __syncthreads();
      }
      for (int j = t; j < V; j += ST)
        if (pv[j] < 0.f) pv[j] = 0.f;
      __syncthreads();
    }
  }
  double zs = 0.0;
  for (int j = t; j < V; j += ST) zs += (double)pv[j];
  const double Z = block_sum<double>(zs, dred);
  const float zf = fmaxf(__double2float_rn(Z), 1e-12f);
  for (int j = t; j < V; j += ST) out[j] = __fdiv_rn(pv[j], zf);
  __syncthreads();
  if (t == 0) {
    VecStats st;
    st.m = m; st.inv_s = inv_s; st.zf = zf;
    st.kth = 0; st.vstar = 0; st.idx_cut = (int32_t)NO_CUT; st.argmax = -1;
    st.flags = 0; st.n_keep = -1; st.fb_why = 0; st.pad = 0;
    st.probe_p = (probe >= 0 && probe < V) ? out[probe] : 0.f;
    P.stats[v] = st;
  }
}

// ---------------------------------------------------------------------------
// greedy: argmax per target vector, then the accept / emit decision per row
// ---------------------------------------------------------------------------
struct ArgmaxParams {
  VecSet vs;           // set 0 only
  int dtype, V, nvec, nch, cu;   // f32: nch blocks per vector, cu 16-byte units per block
  // 16-bit: chunk units, chunks (key slots) per vector, launched warps
  int ch;
  uint32_t cpv, nwarps;
  unsigned long long* partial;   // f32: [nvec, nch] block keys; 16-bit: [nvec, cpv] chunk keys
  int* vec_counter;              // f32: [nvec], zeroed by the launch
  int* row_counter;              // f32: [rows], zeroed by the launch
  VecStats* stats;
  // row decision (verify mode: k >= 1; draft mode: k == 0)
  int k;
  const int64_t* xs; int64_t xs_bs;
  const float* u_acc; int64_t u_bs;
  const uint8_t* alive;
  int64_t* n_acc; int64_t* y; float* px; float* qx;
};

// One thread, once vector v's argmax `am` is known: its stats entry, then, if
// it completes its row (and the call decides rows: k >= 0), the row's accept
// count and emitted token.
__device__ __forceinline__ void argmax_vector_done(const ArgmaxParams& P, int v, int row, int am) {
  VecStats st;
  st.m = 0.f; st.inv_s = 1.f; st.zf = 1.f; st.probe_p = 0.f;
  st.kth = 0; st.vstar = 0; st.idx_cut = (int32_t)NO_CUT; st.argmax = am;
  st.flags = 0; st.n_keep = -1; st.fb_why = 0; st.pad = 0;
  P.stats[v] = st;
  __threadfence();
  const int per = P.vs.npos[0];
  if (P.k < 0 || atomicAdd(&P.row_counter[row], 1) != per - 1) return;
  __threadfence();
  P.row_counter[row] = 0;
  const volatile VecStats* vst = P.stats + (int64_t)row * per;
  if (P.k == 0) {
    P.y[row] = vst[0].argmax;
    if (P.qx) P.qx[row] = 1.0f;
    return;
  }
  // p_i(x_i) is 1 iff x_i is the target argmax; the ratio is then >= 1
  // whatever q is, so the test is u < 1 (engine.py:290-292 with one-hot p).
  int n = 0;
  bool alive = P.alive ? P.alive[row] != 0 : true;
  for (int i = 0; i < P.k; ++i) {
    const int64_t xi = P.xs[row * P.xs_bs + i];
    const float pxi = (xi == (int64_t)vst[i].argmax) ? 1.f : 0.f;
    if (P.px) P.px[row * P.k + i] = pxi;
    if (P.qx) P.qx[row * P.k + i] = nanf("");
    const float thr = pxi > 0.f ? 1.f : 0.f;
    if (alive && n == i && P.u_acc[row * P.u_bs + i] < thr) ++n; else alive = false;
  }
  P.n_acc[row] = n;
  P.y[row] = vst[n].argmax;     // residual and bonus are both one-hot at argmax p_n
}

// Argmax key of element j: larger value first, then smaller index.  Every NaN,
// whatever its sign bit (bf16 conversions of a float NaN give 0xFFFF), takes
// the largest key: NaN counts as the maximum and the first NaN wins.
template <int DT>
__device__ __forceinline__ unsigned long long argmax_key(float x, int j) {
  const uint32_t k = x != x ? 0xFFFFFFFFu : fkey(x);
  return ((unsigned long long)k << 32) | (0xFFFFFFFFu - (uint32_t)j);
}

// Element-wise max of two packed 16-bit pairs, NaN propagating.
template <int DT>
__device__ __forceinline__ uint32_t pmax2_nan(uint32_t a, uint32_t b) {
  uint32_t r;
  if (DT == SD_DTYPE_BF16) asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Argmax (first index of the maximum, NaN counting as the largest value) of a
// vector, used for fp32 logits (bf16 / fp16 go through argmax16_kernel):
// block c of the vector reads 16-byte units [c cu, (c+1) cu) of its aligned
// body with vectorised loads (block 0 also the unaligned head, the last block
// the tail).  Each pass issues a thread's AM_UPT loads at once, keys every
// unit by its maximum (the 16-bit branch keys one packed max of its eight
// elements), takes the warp's largest key once, and builds per-element keys
// only in the units that reach it (ties included: the first index among
// equal values is decided by the element keys).
template <int DT>
__global__ void __launch_bounds__(AM_FT) argmax_kernel(ArgmaxParams P) {
  __shared__ unsigned long long ured[40];
  __shared__ int last;
  constexpr int ESZ = DT == SD_DTYPE_F32 ? 4 : 2;
  constexpr int EPU = 16 / ESZ;
  const int c = blockIdx.x % P.nch, v = blockIdx.x / P.nch, t = threadIdx.x;
  const int V = P.V;
  int set, row, pos;
  vec_locate(P.vs, v, &set, &row, &pos);
  const char* xb = reinterpret_cast<const char*>(vec_ptr(P.vs, set, row, pos, DT));
  int head = (int)(((16u - (uint32_t)(reinterpret_cast<uintptr_t>(xb) & 15u)) & 15u) / ESZ);
  if (head > V) head = V;
  const int nunits = (V - head) / EPU;
  const int tail0 = head + nunits * EPU;
  unsigned long long best = 0ull;
  if (c == 0 && t < head) best = argmax_key<DT>(load_logit(xb, DT, t), t);
  if (c == P.nch - 1 && t < V - tail0) {
    const unsigned long long kk = argmax_key<DT>(load_logit(xb, DT, tail0 + t), tail0 + t);
    best = kk > best ? kk : best;
  }
  const uint4* body = reinterpret_cast<const uint4*>(xb + (size_t)head * ESZ);
  const int u1 = min((c + 1) * P.cu, nunits);
  for (int base = c * P.cu; base < u1; base += AM_UPT * AM_FT) {      // block-uniform
    uint4 w[AM_UPT];
    uint32_t mk[AM_UPT];
#pragma unroll
    for (int i = 0; i < AM_UPT; ++i) {
      const int u = base + t + i * AM_FT;
      w[i] = u < u1 ? __ldg(body + u) : make_uint4(0u, 0u, 0u, 0u);
    }
    uint32_t lm = (uint32_t)(best >> 32);
#pragma unroll
    for (int i = 0; i < AM_UPT; ++i) {
      uint32_t k = 0u;                                  // 0: no data
      if (base + t + i * AM_FT < u1) {
        if (DT == SD_DTYPE_F32) {
          const float a = __uint_as_float(w[i].x), b2 = __uint_as_float(w[i].y);
          const float c2v = __uint_as_float(w[i].z), d = __uint_as_float(w[i].w);
          const bool nan = a != a || b2 != b2 || c2v != c2v || d != d;
          k = nan ? 0xFFFFFFFFu : fkey(fmaxf(fmaxf(a, b2), fmaxf(c2v, d)));
        } else {
          const uint32_t m = pmax2_nan<DT>(pmax2_nan<DT>(w[i].x, w[i].y), pmax2_nan<DT>(w[i].z, w[i].w));
          const float lo = lo16<DT>(m), hi = hi16<DT>(m);
          k = (lo != lo || hi != hi) ? 0xFFFFFFFFu : fkey(fmaxf(lo, hi));
        }
      }
      mk[i] = k;
      lm = k > lm ? k : lm;
    }
    const uint32_t wthr = __reduce_max_sync(0xffffffffu, lm);
#pragma unroll
    for (int i = 0; i < AM_UPT; ++i) {
      if (mk[i] != 0u && mk[i] >= wthr) {              // may hold (or tie) the maximum
        const int j0 = head + (base + t + i * AM_FT) * EPU;
        const uint32_t ww[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
        for (int e = 0; e < EPU; ++e) {
          float xv;
          if (DT == SD_DTYPE_F32) xv = __uint_as_float(ww[e]);
          else xv = (e & 1) ? hi16<DT>(ww[e >> 1]) : lo16<DT>(ww[e >> 1]);
          const unsigned long long kk = argmax_key<DT>(xv, j0 + e);
          best = kk > best ? kk : best;
        }
      }
    }
  }
  best = block_max<unsigned long long>(best, ured, 0ull);
  if (t == 0) {
    P.partial[(int64_t)v * P.nch + c] = best;
    __threadfence();
    last = atomicAdd(&P.vec_counter[v], 1) == P.nch - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (t == 0) {
    unsigned long long b = 0ull;
    for (int i = 0; i < P.nch; ++i) {
      const unsigned long long w = *((volatile unsigned long long*)&P.partial[(int64_t)v * P.nch + i]);
      b = w > b ? w : b;
    }
    P.vec_counter[v] = 0;
    argmax_vector_done(P, v, row, (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFu)));
  }
}

// Order-preserving 16-bit key of one bf16 / fp16 element: every NaN, whatever
// its sign, is the largest key (0xFFFF) and -0 keys as +0.  Keys are >= 1.
template <int DT>
__device__ __forceinline__ uint32_t elem_key16(uint32_t h) {
  constexpr uint32_t INF = DT == SD_DTYPE_BF16 ? 0x7F80u : 0x7C00u;
  h &= 0xFFFFu;
  if ((h & 0x7FFFu) > INF) return 0xFFFFu;
  if (h == 0x8000u) h = 0u;
  return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}

// 16-byte streaming load, not kept in L1 (every byte is read once).
__device__ __forceinline__ uint4 ld_stream16(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

constexpr int AM16_WARPS = AM_FT / 32;     // warps per block
constexpr int AM16_BLOCKS_PER_SM = 2;      // 16 resident warps per SM
constexpr int AM16_UPT = 16;               // 16-byte loads per lane per chunk (one pass)
constexpr int AM16_PER_MAX = 65;           // vectors per row (k + 1 <= 65)
constexpr int AM16_SLOTS_MAX = 512;        // chunks per vector (V <= 2^21 at 512 units)
constexpr int AM16_CHUNK_COST = 128;       // a chunk's fixed cost, in units of streaming

// One warp per row: per vector the largest key over its chunks' slots, then
// either its stats entry (k < 0, to_probs) or the row's accept count and
// emitted token (k >= 0).  The decision's inputs are loaded first, so their latency overlaps
// the keys' loads.  Every lane takes part.
__device__ __forceinline__ void argmax16_row_done(const ArgmaxParams& P, int row, int lane,
                                                  unsigned long long* red) {
  const int per = P.vs.npos[0];
  const int k = P.k;
  int64_t xq[3];
  float uq[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int i = lane + 32 * j;
    xq[j] = (k > 0 && i < k) ? P.xs[row * P.xs_bs + i] : -1;
    uq[j] = (k > 0 && i < k) ? P.u_acc[row * P.u_bs + i] : 2.f;
  }
  const bool alive_row = (k > 0 && P.alive) ? P.alive[row] != 0 : true;
  // the inputs above are the caller's; the keys below come from pass 1
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t cpv = P.cpv;
  const uint32_t v0 = (uint32_t)row * per;
  for (int p = lane; p < per; p += 32) red[p] = 0ull;
  __syncwarp();
  // the row's keys are contiguous: 8 loads per lane in flight at once
  const unsigned long long* keys = P.partial + (size_t)v0 * cpv;
  const uint32_t nk = (uint32_t)per * cpv;
  for (uint32_t f0 = 0; f0 < nk; f0 += 32 * 8) {
    unsigned long long kk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t f = f0 + lane + 32 * i;
      kk[i] = f < nk ? __ldcg(keys + f) : 0ull;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t f = f0 + lane + 32 * i;
      if (f < nk) atomicMax(red + f / cpv, kk[i]);
    }
  }
  __syncwarp();
  if (k < 0) {                         // to_probs: the stats records are the output
    for (int p = lane; p < per; p += 32) {
      VecStats st;
      st.m = 0.f; st.inv_s = 1.f; st.zf = 1.f; st.probe_p = 0.f;
      st.kth = 0; st.vstar = 0; st.idx_cut = (int32_t)NO_CUT;
      st.argmax = (int32_t)(0xFFFFFFFFu - (uint32_t)red[p]);
      st.flags = 0; st.n_keep = -1; st.fb_why = 0; st.pad = 0;
      P.stats[v0 + p] = st;
    }
    return;
  }
  if (k == 0) {
    if (lane == 0) {
      P.y[row] = (int64_t)(0xFFFFFFFFu - (uint32_t)red[0]);
      if (P.qx) P.qx[row] = 1.0f;
    }
    return;
  }
  // p_i(x_i) is 1 iff x_i is the target argmax; the ratio is then >= 1
  // whatever q is, so the test is u < 1 (engine.py:290-292 with one-hot p).
  int n = 0;
  bool run = alive_row;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int i0 = 32 * j, i = i0 + lane;
    if (i0 >= k) break;                                     // warp-uniform
    bool ok = false;
    if (i < k) {
      const int64_t am = (int64_t)(0xFFFFFFFFu - (uint32_t)red[i]);
      const float pxi = xq[j] == am ? 1.f : 0.f;
      if (P.px) P.px[row * k + i] = pxi;
      if (P.qx) P.qx[row * k + i] = nanf("");
      ok = uq[j] < (pxi > 0.f ? 1.f : 0.f);
    }
    const unsigned m = __ballot_sync(0xffffffffu, ok);
    if (run) {
      const int lim = min(32, k - i0);
      const unsigned full = lim == 32 ? 0xffffffffu : ((1u << lim) - 1u);
      if ((m & full) == full) n += lim;
      else { n += __ffs(~m) - 1; run = false; }
    }
  }
  if (lane == 0) {
    P.n_acc[row] = n;
    P.y[row] = (int64_t)(0xFFFFFFFFu - (uint32_t)red[n]);   // residual and bonus: argmax p_n
  }
}

// Where chunk c lies: vector v = c / cpv, chunk j = c mod cpv covering
// vector-local 16-byte units [a, b) of the vector's aligned body (b clipped
// to the body), and for the vector's first chunk the head / tail elements.
struct Am16Chunk {
  const char* xb;                  // the vector's first element
  const uint4* body;               // its 16-byte-aligned body
  int a, b;                        // units of this chunk
  int head, tail0;                 // unaligned head [0, head), tail [tail0, V)
  uint32_t v, j;
  int row;
};

template <int DT>
__device__ __forceinline__ Am16Chunk am16_chunk(const ArgmaxParams& P, uint32_t c) {
  Am16Chunk q;
  q.v = c / P.cpv;
  q.j = c - q.v * P.cpv;
  int set, pos;
  vec_locate(P.vs, (int)q.v, &set, &q.row, &pos);
  q.xb = reinterpret_cast<const char*>(vec_ptr(P.vs, set, q.row, pos, DT));
  const int V = P.V;
  int head = (int)(((16u - (uint32_t)(reinterpret_cast<uintptr_t>(q.xb) & 15u)) & 15u) >> 1);
  if (head > V) head = V;
  const int nunits = (V - head) >> 3;
  q.head = head;
  q.tail0 = head + nunits * 8;
  q.body = reinterpret_cast<const uint4*>(q.xb + (size_t)head * 2);
  q.a = (int)q.j * P.ch;
  q.b = min(q.a + P.ch, nunits);
  return q;
}

// Issues a chunk's loads: AM16_UPT 16-byte units per lane, and (first chunk
// of a vector) lane l < 8 the head element l, lane 8 + t the tail element t.
__device__ __forceinline__ void am16_issue(const Am16Chunk& q, int V, int lane,
                                           uint4 (&w)[AM16_UPT], uint32_t& ends) {
#pragma unroll
  for (int i = 0; i < AM16_UPT; ++i) {
    const int u = q.a + lane + 32 * i;
    w[i] = u < q.b ? ld_stream16(q.body + u) : make_uint4(0u, 0u, 0u, 0u);
  }
  ends = 0xFFFFFFFFu;                                       // no element
  if (q.j == 0) {
    const uint16_t* x16 = reinterpret_cast<const uint16_t*>(q.xb);
    if (lane < q.head) ends = x16[lane];
    else if (lane >= 8 && lane - 8 < V - q.tail0) ends = x16[q.tail0 + lane - 8];
  }
}

// Argmax of bf16 / fp16 vectors, pass 1 of 2 (first index of the maximum,
// NaN counting as the largest value, -0 equal to +0): persistent and
// warp-granular.  Each vector is cut into cpv chunks of ch 16-byte units
// (ch <= 32 * AM16_UPT: one load per lane and unit group, all issued at
// once); chunk c goes to warp c mod nwarps, so the warps sweep memory
// together, round after round, and a warp's next loads go out right after
// its current chunk's key is stored.  Per unit a lane takes one packed
// NaN-propagating maximum of its eight elements (a NaN comes out as the
// canonical positive NaN), keys it with -0 merged into +0, and keeps the
// first of its units reaching its best key with that unit's data; the
// chunk's key (value key, then the complement of the index) is resolved
// inside the lanes' winning units from registers and stored to slot j of the
// vector.  No fences, counters or atomics: pass 2 (argmax16_rows_kernel)
// reads the keys after this kernel ends.
template <int DT>
__global__ void __launch_bounds__(AM_FT, AM16_BLOCKS_PER_SM) argmax16_kernel(ArgmaxParams P) {
  const int lane = threadIdx.x & 31;
  const uint32_t gw = blockIdx.x * AM16_WARPS + (threadIdx.x >> 5);
  const uint32_t nchunks = (uint32_t)P.nvec * P.cpv;
  // pass 2 may launch now: its blocks load their own inputs, then wait for
  // this grid to finish (griddepcontrol.wait) before reading the keys
  asm volatile("griddepcontrol.launch_dependents;");
  uint32_t c = gw;
  if (c >= nchunks) return;
  uint4 w[AM16_UPT];
  uint32_t ends;
  Am16Chunk q = am16_chunk<DT>(P, c);
  am16_issue(q, P.V, lane, w, ends);
  for (;;) {
    uint32_t bk = 0u;                                       // 0: no unit yet
    int bu = -1;
    uint4 bw = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int i = 0; i < AM16_UPT; ++i) {
      const int u = q.a + lane + 32 * i;
      const uint32_t m = pmax2_nan<DT>(pmax2_nan<DT>(w[i].x, w[i].y),
                                       pmax2_nan<DT>(w[i].z, w[i].w));
      const uint32_t k2 = m ^ (((m >> 15) & 0x00010001u) * 0x7FFFu) ^ 0x80008000u;
      uint32_t k = max(k2 & 0xFFFFu, k2 >> 16);
      k += (k == 0x7FFFu);                                  // -0 -> +0
      if (u < q.b && k > bk) { bk = k; bu = u; bw = w[i]; }
    }
    unsigned long long best = 0ull;
    if (bu >= 0) {
      const uint32_t ww[4] = {bw.x, bw.y, bw.z, bw.w};
      int e = 7;
#pragma unroll
      for (int i = 7; i >= 0; --i)
        if (elem_key16<DT>((i & 1) ? ww[i >> 1] >> 16 : ww[i >> 1]) == bk) e = i;
      best = ((unsigned long long)bk << 32) | (0xFFFFFFFFu - (uint32_t)(q.head + bu * 8 + e));
    }
    if (ends != 0xFFFFFFFFu) {
      const int jx = lane < 8 ? lane : q.tail0 + lane - 8;
      const unsigned long long kk = ((unsigned long long)elem_key16<DT>(ends) << 32) |
                                    (0xFFFFFFFFu - (uint32_t)jx);
      best = kk > best ? kk : best;
    }
    const uint32_t hi = (uint32_t)(best >> 32);
    const uint32_t mh = __reduce_max_sync(0xffffffffu, hi);
    const uint32_t ml = __reduce_max_sync(0xffffffffu, hi == mh ? (uint32_t)best : 0u);
    if (lane == 0) P.partial[(size_t)q.v * P.cpv + q.j] = ((unsigned long long)mh << 32) | ml;
    c += P.nwarps;
    if (c >= nchunks) break;
    q = am16_chunk<DT>(P, c);
    am16_issue(q, P.V, lane, w, ends);
  }
}

// Pass 2: one warp per row reduces its vectors' chunk keys and finishes the
// row (argmax16_row_done).  Launched as a programmatic dependent of pass 1:
// it may start while pass 1 runs and waits for it before reading the keys.
__global__ void __launch_bounds__(AM_FT) argmax16_rows_kernel(ArgmaxParams P) {
  __shared__ unsigned long long red_all[AM16_WARPS][AM16_PER_MAX];
  const int row = blockIdx.x * AM16_WARPS + (threadIdx.x >> 5);
  if (row >= P.vs.nrows) return;
  argmax16_row_done(P, row, threadIdx.x & 31, red_all[threadIdx.x >> 5]);
}

// ---------------------------------------------------------------------------
// finish: accept decision, residual / bonus mass per chunk, inverse-CDF draw
// ---------------------------------------------------------------------------
struct FinishParams {
  VecSet vs;           // set 0: target [rows, k+1]; set 1: draft [rows, k]
  int dtype, V, k, nch, chunk;
  float T;
  const VecStats* stats;
  const float* mat;    // materialised probabilities [nvec, V] or nullptr
  const float* u_acc; int64_t u_bs;
  const float* u_res;
  const uint8_t* alive;
  int64_t* n_acc; int64_t* y; float* px; float* qx; float* y_prob;
  double* partial;     // [rows, nch, 2]
  int* counter;        // [rows]
};

struct SelVec {
  const void* x;       // logits (hist mode)
  const float* mat;    // materialised probabilities (small mode)
  VecStats st;
};

__device__ __forceinline__ float final_prob(const SelVec& s, int dtype, float T, int j) {
  if (s.mat) return s.mat[j];
  const float xv = load_logit(s.x, dtype, j);
  const uint32_t kx = fkey(xv);
  const bool kept = kx >= s.st.kth &&
                    (kx > s.st.vstar || (kx == s.st.vstar && j <= s.st.idx_cut));
  if (!kept) return 0.f;
  return __fdiv_rn(prob_of(xv, T, s.st.m, s.st.inv_s), s.st.zf);
}

// mass of element j of the distribution the row draws from
__device__ __forceinline__ float draw_mass(const SelVec& p, const SelVec& q, bool resid, bool use_p,
                                           int dtype, float T, int j) {
  const float pj = final_prob(p, dtype, T, j);
  if (!resid || use_p || pj == 0.f) return pj;
  const float qj = final_prob(q, dtype, T, j);
  return fmaxf(__fsub_rn(pj, qj), 0.f);
}

__global__ void __launch_bounds__(FT) finish_kernel(FinishParams P) {
  __shared__ double dred[40];
  __shared__ int s_n, s_last;
  __shared__ int64_t s_y;
  const int c = blockIdx.x % P.nch, b = blockIdx.x / P.nch, t = threadIdx.x;
  const int npos = P.vs.npos[0] + P.vs.npos[1];
  const int vrow = b * npos;
  if (t == 0) {
    int n = 0;
    bool alive = P.alive ? P.alive[b] != 0 : true;
    for (int i = 0; i < P.k; ++i) {
      const float pxi = P.stats[vrow + i].probe_p;
      const float qxi = P.stats[vrow + P.vs.npos[0] + i].probe_p;
      const float thr = fminf(__fdiv_rn(pxi, fmaxf(qxi, 1e-10f)), 1.0f);
      if (c == 0) {
        if (P.px) P.px[b * P.k + i] = pxi;
        if (P.qx) P.qx[b * P.k + i] = qxi;
      }
      if (alive && n == i && P.u_acc[b * P.u_bs + i] < thr) ++n; else alive = false;
    }
    s_n = n;
  }
  __syncthreads();
  const int n = s_n;
  const bool resid = n < P.k;
  const int ppos = resid ? n : P.k;            // pick = min(n, k-1) when resid
  SelVec ps, qs;
  ps.st = P.stats[vrow + ppos];
  ps.x = vec_ptr(P.vs, 0, b, ppos, P.dtype);
  ps.mat = P.mat ? P.mat + (int64_t)(vrow + ppos) * P.V : nullptr;
  if (resid) {
    qs.st = P.stats[vrow + P.vs.npos[0] + n];
    qs.x = vec_ptr(P.vs, 1, b, n, P.dtype);
    qs.mat = P.mat ? P.mat + (int64_t)(vrow + P.vs.npos[0] + n) * P.V : nullptr;
  } else {
    qs = ps;
  }
  const int j0 = c * P.chunk, j1 = min(P.V, j0 + P.chunk);
  double sr = 0.0, sp = 0.0;
  for (int j = j0 + t; j < j1; j += FT) {
    const float pj = final_prob(ps, P.dtype, P.T, j);
    sp += (double)pj;
    if (resid && pj != 0.f) sr += (double)fmaxf(__fsub_rn(pj, final_prob(qs, P.dtype, P.T, j)), 0.f);
  }
  sr = block_sum<double>(sr, dred);
  sp = block_sum<double>(sp, dred);
  if (t == 0) {
    double* part = P.partial + ((int64_t)b * P.nch + c) * 2;
    part[0] = sr;
    part[1] = sp;
    __threadfence();
    s_last = atomicAdd(&P.counter[b], 1) == P.nch - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ---- last CTA of the row: totals in chunk order, locate the chunk, scan it
  __shared__ double s_pre, s_tot;
  __shared__ int s_cstar, s_usep;
  if (t == 0) {
    const volatile double* part = P.partial + (int64_t)b * P.nch * 2;
    double R = 0.0, Pm = 0.0;
    for (int i = 0; i < P.nch; ++i) { R += part[2 * i]; Pm += part[2 * i + 1]; }
    const bool use_p = !resid || (__double2float_rn(R) <= 1e-9f);   // sampling.py:86-89
    const double tot = use_p ? Pm : R;
    const double target = (double)P.u_res[b] * tot;
    double pre = 0.0, prelast = 0.0;
    int cstar = -1, lastnz = 0;
    for (int i = 0; i < P.nch; ++i) {
      const double w = use_p ? part[2 * i + 1] : part[2 * i];
      if (w > 0.0) { lastnz = i; prelast = pre; }
      if (cstar < 0 && pre + w > target) { cstar = i; s_pre = pre; }
      pre += w;
    }
    if (cstar < 0) { cstar = lastnz; s_pre = prelast; }
    s_cstar = cstar;
    s_usep = use_p;
    s_tot = tot;
    P.counter[b] = 0;
  }
  __syncthreads();
  const bool use_p = s_usep;
  const double tgt = (double)P.u_res[b] * s_tot;
  const int cs = s_cstar;
  const int k0 = cs * P.chunk, k1 = min(P.V, k0 + P.chunk);
  const int len = k1 - k0;
  const int sub = (len + FT - 1) / FT;
  const int a0 = k0 + min(len, t * sub), a1 = k0 + min(len, (t + 1) * sub);
  double ls = 0.0;
  for (int j = a0; j < a1; ++j) ls += (double)draw_mass(ps, qs, resid, use_p, P.dtype, P.T, j);
  double ctot;
  const double pre = s_pre + block_excl_scan<double>(ls, dred, &ctot);
  if (t == 0) s_y = -1;
  __syncthreads();
  if (a0 < a1 && pre <= tgt && pre + ls > tgt) {
    double run = pre;
    for (int j = a0; j < a1; ++j) {
      run += (double)draw_mass(ps, qs, resid, use_p, P.dtype, P.T, j);
      if (run > tgt) { s_y = j; break; }
    }
  }
  __syncthreads();
  if (t == 0 && s_y < 0) {
    // rounding put the crossing past this chunk: last element with mass
    for (int j = k1 - 1; j >= k0; --j)
      if (draw_mass(ps, qs, resid, use_p, P.dtype, P.T, j) > 0.f) { s_y = j; break; }
    if (s_y < 0) s_y = k0;
  }
  __syncthreads();
  if (t == 0) {
    if (P.n_acc) P.n_acc[b] = n;
    P.y[b] = s_y;
    if (P.y_prob) P.y_prob[b] = final_prob(ps, P.dtype, P.T, (int)s_y);
  }
}

// ---------------------------------------------------------------------------
// probs writer (to_probs API)
// ---------------------------------------------------------------------------
struct ProbsParams {
  VecSet vs;
  int dtype, V, nch, chunk, greedy;
  float T;
  const VecStats* stats;
  const float* mat;
  float* out; int64_t out_stride;
};

__global__ void __launch_bounds__(FT) probs_kernel(ProbsParams P) {
  const int c = blockIdx.x % P.nch, v = blockIdx.x / P.nch, t = threadIdx.x;
  int set, row, pos;
  vec_locate(P.vs, v, &set, &row, &pos);
  SelVec s;
  s.st = P.stats[v];
  s.x = vec_ptr(P.vs, set, row, pos, P.dtype);
  s.mat = P.mat ? P.mat + (int64_t)v * P.V : nullptr;
  float* o = P.out + (int64_t)v * P.out_stride;
  const int j0 = c * P.chunk, j1 = min(P.V, j0 + P.chunk);
  for (int j = j0 + t; j < j1; j += FT)
    o[j] = P.greedy ? (j == s.st.argmax ? 1.f : 0.f) : final_prob(s, P.dtype, P.T, j);
}

// ---------------------------------------------------------------------------
// fp32-probability utilities: residual_probs, sample_from_probs, gather_prob
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(FT) residual_kernel(const float* p, const float* q, int V, float* out) {
  __shared__ double dred[40];
  const int r = blockIdx.x, t = threadIdx.x;
  const float* pr = p + (int64_t)r * V;
  const float* qr = q + (int64_t)r * V;
  float* o = out + (int64_t)r * V;
  double s = 0.0, sp = 0.0;
  for (int j = t; j < V; j += FT) {
    s += (double)fmaxf(__fsub_rn(pr[j], qr[j]), 0.f);
    sp += (double)pr[j];
  }
  s = block_sum<double>(s, dred);
  sp = block_sum<double>(sp, dred);
  const bool deg = __double2float_rn(s) <= 1e-9f;
  const float tot = fmaxf(__double2float_rn(deg ? sp : s), 1e-12f);
  for (int j = t; j < V; j += FT) {
    const float rj = deg ? pr[j] : fmaxf(__fsub_rn(pr[j], qr[j]), 0.f);
    o[j] = __fdiv_rn(rj, tot);
  }
}

__global__ void __launch_bounds__(FT) sample_probs_kernel(const float* probs, int V, const float* u,
                                                          int64_t* out) {
  __shared__ double dred[40];
  __shared__ int64_t s_y;
  const int r = blockIdx.x, t = threadIdx.x;
  const float* pr = probs + (int64_t)r * V;
  const int sub = (V + FT - 1) / FT;
  const int a0 = min(V, t * sub), a1 = min(V, (t + 1) * sub);
  double ls = 0.0;
  for (int j = a0; j < a1; ++j) ls += (double)pr[j];
  double tot;
  const double pre = block_excl_scan<double>(ls, dred, &tot);
  const double tgt = (double)u[r] * tot;
  if (t == 0) s_y = -1;
  __syncthreads();
  if (a0 < a1 && pre <= tgt && pre + ls > tgt) {
    double run = pre;
    for (int j = a0; j < a1; ++j) {
      run += (double)pr[j];
      if (run > tgt) { s_y = j; break; }
    }
  }
  __syncthreads();
  if (t == 0) {
    if (s_y < 0) {
      for (int j = V - 1; j >= 0; --j)
        if (pr[j] > 0.f) { s_y = j; break; }
      if (s_y < 0) s_y = V - 1;
    }
    out[r] = s_y;
  }
}

__global__ void gather_kernel(const float* probs, int n, int V, const int64_t* ids, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const int64_t j = ids[i];
    out[i] = (j >= 0 && j < V) ? probs[(int64_t)i * V + j] : nanf("");
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int g_num_sms[64];
static bool g_attr_set[64];

static int device_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!g_num_sms[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms[dev] = n > 0 ? n : 148;
  }
  if (!g_attr_set[dev]) {
    cudaFuncSetAttribute(hist_stats_kernel<SD_DTYPE_BF16>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(HistSmem));
    cudaFuncSetAttribute(hist_stats_kernel<SD_DTYPE_F16>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(HistSmem));
    cudaFuncSetAttribute(row_draw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sizeof(HistSmem));
    g_attr_set[dev] = true;
  }
  return g_num_sms[dev];
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct WsLayout {
  size_t status, stats, partial, counter, vcounter, rcounter, apartial, mat, nuc, total;
};

// Argmax geometry: blocks per vector and 16-byte units per block (a multiple
// of AM_FT, at most NCH_MAX blocks).
struct ArgmaxGeom {
  int nch, cu;
};
static ArgmaxGeom argmax_geom(int V, int dtype) {
  const int epu = dtype == SD_DTYPE_F32 ? 4 : 8;
  const int units = V / epu + 1;
  ArgmaxGeom g;
  g.cu = AM_UPT * AM_FT;
  g.nch = (units + g.cu - 1) / g.cu;
  if (g.nch > NCH_MAX) {
    g.nch = NCH_MAX;
    g.cu = ((units + g.nch - 1) / g.nch + AM_FT - 1) / AM_FT * AM_FT;
  }
  return g;
}

static int nch_for(int V) {
  int n = (V + 4095) / 4096;
  return n < 1 ? 1 : (n > NCH_MAX ? NCH_MAX : n);
}

static bool use_small(int V, int dtype) { return V <= SMALLV_MAX || dtype == SD_DTYPE_F32; }

static WsLayout ws_layout(int n_rows, int n_vec, int V, bool small) {
  WsLayout L;
  size_t off = 0;
  L.status = off; off = 256;      // sticky device status word, same place for every shape
  L.stats = off; off = align256(off + (size_t)n_vec * sizeof(VecStats));
  L.partial = off; off = align256(off + (size_t)n_rows * NCH_MAX * 2 * sizeof(double));
  L.counter = off; off = align256(off + (size_t)n_rows * sizeof(int));
  L.vcounter = off; off = align256(off + (size_t)n_vec * sizeof(int));
  L.rcounter = off; off = align256(off + (size_t)n_rows * sizeof(int));
  // keys: f32, NCH_MAX blocks per vector; 16-bit, one per chunk of >= 256 units
  const size_t nkey = std::max<size_t>(NCH_MAX, ((size_t)V / 8 + 255) / 256);
  L.apartial = off; off = align256(off + (size_t)n_vec * nkey * sizeof(unsigned long long));
  L.mat = off; off = align256(off + (small ? (size_t)n_vec * V * sizeof(float) : 0));
  L.nuc = off; off = align256(off + (small ? 0 : (size_t)n_vec * NUC_MAX * sizeof(unsigned long long)));
  L.total = off;
  return L;
}

static int check_launch() {
  return cudaGetLastError() == cudaSuccess ? SD_OK : SD_ELAUNCH;
}

// argmax16_kernel geometry: the grid fills every SM (fewer warps for small
// inputs); the chunk size ch (a multiple of 32 units, at most 32 * AM16_UPT,
// at least 32 * AM16_UPT / 2 unless a vector is shorter, at most
// AM16_SLOTS_MAX chunks per vector) minimises rounds * (ch + AM16_CHUNK_COST),
// the time of the round-robin sweep with each chunk's fixed cost (its load
// latency and key publishing) counted as AM16_CHUNK_COST units; the larger
// chunk wins ties.
struct Am16Geom {
  int ch, cpv, grid;
};
static int am16_geom(int V, int nvec, Am16Geom* g) {
  const int64_t nu = V / 8 > 0 ? V / 8 : 1;
  if ((int64_t)nvec * nu > INT32_MAX / 2) return SD_ENOTSUP;
  const int64_t full = (int64_t)device_sms() * AM16_BLOCKS_PER_SM * AM16_WARPS;
  const int64_t cmax = 32 * AM16_UPT;
  int64_t best_t = -1, best_ch = cmax;
  for (int64_t ch = cmax; ch >= cmax / 2; ch -= 32) {
    const int64_t cpv = (nu + ch - 1) / ch;
    if (cpv > AM16_SLOTS_MAX) break;
    const int64_t nch = (int64_t)nvec * cpv;
    const int64_t t = (nch + full - 1) / full * (std::min(ch, nu) + AM16_CHUNK_COST);
    if (best_t < 0 || t < best_t) { best_t = t; best_ch = ch; }
  }
  if (best_t < 0) return SD_ENOTSUP;        // V above 8 * AM16_SLOTS_MAX * 32 * AM16_UPT
  const int64_t cpv = (nu + best_ch - 1) / best_ch;
  const int64_t nwarps = std::min<int64_t>(full, (int64_t)nvec * cpv);
  g->ch = (int)best_ch;
  g->cpv = (int)cpv;
  g->grid = (int)((nwarps + AM16_WARPS - 1) / AM16_WARPS);
  return SD_OK;
}

// f32 logits: zero the two counter arrays, then argmax_kernel over (vector,
// chunk) blocks.  16-bit logits: argmax16_kernel (chunk keys into P.partial,
// nvec * cpv of them), then argmax16_rows_kernel.
static int launch_argmax(ArgmaxParams P, cudaStream_t st) {
  if (P.dtype == SD_DTYPE_F32) {
    if (cudaMemsetAsync(P.vec_counter, 0, (size_t)P.nvec * sizeof(int), st) != cudaSuccess ||
        cudaMemsetAsync(P.row_counter, 0, (size_t)P.vs.nrows * sizeof(int), st) != cudaSuccess)
      return SD_ELAUNCH;
    argmax_kernel<SD_DTYPE_F32><<<P.nch * P.nvec, AM_FT, 0, st>>>(P);
    return check_launch();
  }
  if (P.vs.npos[0] > AM16_PER_MAX) return SD_EINVAL;
  Am16Geom g;
  if (int rc = am16_geom(P.V, P.nvec, &g)) return rc;
  P.ch = g.ch;
  P.cpv = (uint32_t)g.cpv;
  P.nwarps = (uint32_t)g.grid * AM16_WARPS;
  if (P.dtype == SD_DTYPE_BF16) argmax16_kernel<SD_DTYPE_BF16><<<g.grid, AM_FT, 0, st>>>(P);
  else argmax16_kernel<SD_DTYPE_F16><<<g.grid, AM_FT, 0, st>>>(P);
  if (int rc = check_launch()) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((P.vs.nrows + AM16_WARPS - 1) / AM16_WARPS));
  cfg.blockDim = dim3(AM_FT);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, argmax16_rows_kernel, P) != cudaSuccess) return SD_ELAUNCH;
  return check_launch();
}


// What a verify / draft call draws (to_probs passes none).
struct DrawSpec {
  int k;
  const float* u_acc; int64_t u_bs;
  const float* u_res;
  const uint8_t* alive;
  int64_t* n_acc; int64_t* y; float* px; float* qx; float* y_prob;
  const float* qprob; int64_t q_bs, q_ps;     // draft distributions as probabilities, or null
};

// Non-greedy path: stats for every vector of `vs`, then (if `draw`) each
// row's accept test and draw.  Histogram-path truncated sampling draws inside
// the stats kernel; otherwise a finish kernel follows.
static int run_sampling(const VecSet& vs, int nvec, int dtype, int V, float T, float top_p,
                        int top_k, const WsLayout& L, char* ws, cudaStream_t st,
                        const DrawSpec* draw) {
  VecStats* stats = reinterpret_cast<VecStats*>(ws + L.stats);
  const bool small = use_small(V, dtype);
  const int rows = vs.nrows;
  bool need_finish = draw != nullptr;
  if (small) {
    if (V > SMALLV_MAX) return SD_ENOTSUP;
    SmallParams P;
    P.vs = vs; P.dtype = dtype; P.V = V; P.nvec = nvec; P.T = T; P.top_p = top_p;
    P.top_k = top_k; P.stats = stats; P.mat = reinterpret_cast<float*>(ws + L.mat);
    P.zero_ctr = reinterpret_cast<int*>(ws + L.counter); P.n_ctr = rows;
    small_stats_kernel<<<nvec, ST, 0, st>>>(P);
    if (int rc = check_launch()) return rc;
  } else {
    const bool truncated = (top_p > 0.0f && top_p < 1.0f) || (top_k > 0 && top_k < V);
    // rows drawn by row_draw_kernel (always when the draft distributions come
    // as probabilities: finish_kernel reads them from draft stats)
    const bool rowpass = draw != nullptr && (truncated || draw->qprob != nullptr);
    StatsParams P = {};
    P.vs = vs; P.dtype = dtype; P.V = V; P.nvec = nvec; P.T = T; P.top_p = top_p;
    P.top_k = top_k; P.stats = stats;
    P.nuc = draw ? reinterpret_cast<unsigned long long*>(ws + L.nuc) : nullptr;
    P.row_ctr = reinterpret_cast<int*>(ws + L.rcounter);
    P.status = reinterpret_cast<int*>(ws + L.status);
    P.fused = false;
    if (rowpass) {
      P.k = draw->k; P.u_acc = draw->u_acc; P.u_bs = draw->u_bs; P.u_res = draw->u_res;
      P.alive = draw->alive; P.n_acc = draw->n_acc; P.y = draw->y; P.px = draw->px;
      P.qx = draw->qx; P.y_prob = draw->y_prob;
      P.qprob = draw->qprob; P.q_bs = draw->q_bs; P.q_ps = draw->q_ps;
    }
    const int nsm = device_sms();
    int grid = nsm;
    if (grid > GRID_MAX) grid = GRID_MAX;
    if (grid > nvec) grid = nvec;
    if (dtype == SD_DTYPE_BF16)
      hist_stats_kernel<SD_DTYPE_BF16><<<grid, HT, sizeof(HistSmem), st>>>(P);
    else
      hist_stats_kernel<SD_DTYPE_F16><<<grid, HT, sizeof(HistSmem), st>>>(P);
    if (int rc = check_launch()) return rc;
    if (rowpass) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)rows);
      cfg.blockDim = dim3(HT);
      cfg.dynamicSmemBytes = sizeof(HistSmem);
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaLaunchKernelEx(&cfg, row_draw_kernel, P) != cudaSuccess) return SD_ELAUNCH;
      if (int rc = check_launch()) return rc;
    }

    need_finish = draw != nullptr && !rowpass;
    if (need_finish &&
        cudaMemsetAsync(ws + L.counter, 0, (size_t)rows * sizeof(int), st) != cudaSuccess)
      return SD_ELAUNCH;
  }
  if (!need_finish) return SD_OK;
  FinishParams F;
  F.vs = vs; F.dtype = dtype; F.V = V; F.k = draw->k;
  F.nch = nch_for(V); F.chunk = (V + F.nch - 1) / F.nch;
  F.T = T;
  F.stats = stats;
  F.mat = small ? reinterpret_cast<const float*>(ws + L.mat) : nullptr;
  F.u_acc = draw->u_acc; F.u_bs = draw->u_bs; F.u_res = draw->u_res; F.alive = draw->alive;
  F.n_acc = draw->n_acc; F.y = draw->y; F.px = draw->px; F.qx = draw->qx; F.y_prob = draw->y_prob;
  F.partial = reinterpret_cast<double*>(ws + L.partial);
  F.counter = reinterpret_cast<int*>(ws + L.counter);
  finish_kernel<<<F.nch * rows, FT, 0, st>>>(F);
  return check_launch();
}

// Greedy verify round over caller-provided buffers: argmax of every target
// vector, then per row the accepted prefix and the emitted token.
static int launch_greedy_verify(const void* tgt, int64_t tgt_bs, int64_t tgt_ps, int dtype,
                                const int64_t* xs, int64_t xs_bs, const float* u_acc,
                                int64_t u_bs, const uint8_t* alive, int B, int k, int V,
                                int64_t* n_acc, int64_t* y, float* px, float* qx,
                                VecStats* stats, unsigned long long* partial, int* vcounter,
                                int* rcounter, cudaStream_t st) {
  const int nvec = B * (k + 1);
  VecSet vs = {};
  vs.base[0] = tgt; vs.bs[0] = tgt_bs; vs.ps[0] = tgt_ps; vs.npos[0] = k + 1;
  vs.npos[1] = 0; vs.nrows = B;
  ArgmaxParams P;
  P.vs = vs; P.dtype = dtype; P.V = V; P.nvec = nvec;
  const ArgmaxGeom ag = argmax_geom(V, dtype);
  P.nch = ag.nch; P.cu = ag.cu;
  P.partial = partial;
  P.vec_counter = vcounter;
  P.row_counter = rcounter;
  P.stats = stats;
  P.k = k; P.xs = xs; P.xs_bs = xs_bs; P.u_acc = u_acc; P.u_bs = u_bs; P.alive = alive;
  P.n_acc = n_acc; P.y = y; P.px = px; P.qx = qx;
  return launch_argmax(P, st);
}

// Fixed device scratch of sd_verify_greedy_static (one copy per device, in
// this library's module): stats, the counters and the per-vector keys.
static __device__ __align__(256) unsigned char g_static_scratch[SD_STATIC_SCRATCH_BYTES];

struct StaticLayout {
  size_t stats, vcounter, rcounter, partial, total;
};
static StaticLayout static_layout(int B, int nvec, int nslot) {
  StaticLayout L;
  size_t off = 0;
  L.stats = off; off = align256(off + (size_t)nvec * sizeof(VecStats));
  L.vcounter = off; off = align256(off + (size_t)nvec * sizeof(int));
  L.rcounter = off; off = align256(off + (size_t)B * sizeof(int));
  L.partial = off; off = align256(off + (size_t)nvec * nslot * sizeof(unsigned long long));
  L.total = off;
  return L;
}

// Address of g_static_scratch on the current device, looked up once per device.
static std::mutex g_static_mu;
static void* g_static_ptr[SD_MAX_DEVICES];

static int static_scratch(char** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= SD_MAX_DEVICES) return SD_ELAUNCH;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || p == nullptr) return SD_ELAUNCH;
    g_static_ptr[dev] = p;
  }
  *out = reinterpret_cast<char*>(g_static_ptr[dev]);
  return SD_OK;
}

static int validate_common(int dtype, int V, float T) {
  if (dtype != SD_DTYPE_F32 && dtype != SD_DTYPE_F16 && dtype != SD_DTYPE_BF16) return SD_EINVAL;
  if (V <= 0 || V > (1 << 21)) return SD_EINVAL;
  if (!(T == T)) return SD_EINVAL;
  return SD_OK;
}

}  // namespace sd

using namespace sd;

extern "C" {

int sd_version(void) { return 1; }

size_t sd_sampling_workspace_bytes(int n_rows, int n_vec, int V, int dtype) {
  return ws_layout(n_rows, n_vec, V, use_small(V, dtype)).total;
}

int sd_verify_sample(const void* tgt, int64_t tgt_bs, int64_t tgt_ps,
                     const void* drf, int64_t drf_bs, int64_t drf_ps, int dtype,
                     const int64_t* xs, int64_t xs_bs, const float* u_acc, int64_t u_bs,
                     const float* u_res, const uint8_t* alive,
                     int B, int k, int V, float temperature, float top_p, int top_k,
                     int64_t* n_acc, int64_t* y, float* px, float* qx,
                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate_common(dtype, V, temperature);
  if (rc) return rc;
  if (B <= 0 || k < 1 || k > 64 || !tgt || !xs || !u_acc || !u_res || !n_acc || !y || !workspace)
    return SD_EINVAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool greedy = !(temperature > 0.0f);
  char* ws = reinterpret_cast<char*>(workspace);
  if (greedy) {
    const int nvec = B * (k + 1);
    WsLayout L = ws_layout(B, nvec, V, use_small(V, dtype));
    if (workspace_bytes < L.total) return SD_ENOSPC;
    return launch_greedy_verify(tgt, tgt_bs, tgt_ps, dtype, xs, xs_bs, u_acc, u_bs, alive, B, k, V,
                                n_acc, y, px, qx, reinterpret_cast<VecStats*>(ws + L.stats),
                                reinterpret_cast<unsigned long long*>(ws + L.apartial),
                                reinterpret_cast<int*>(ws + L.vcounter),
                                reinterpret_cast<int*>(ws + L.rcounter), st);
  }
  if (!drf) return SD_EINVAL;
  const int nvec = B * (2 * k + 1);
  WsLayout L = ws_layout(B, nvec, V, use_small(V, dtype));
  if (workspace_bytes < L.total) return SD_ENOSPC;
  VecSet vs = {};
  vs.base[0] = tgt; vs.bs[0] = tgt_bs; vs.ps[0] = tgt_ps; vs.npos[0] = k + 1;
  vs.base[1] = drf; vs.bs[1] = drf_bs; vs.ps[1] = drf_ps; vs.npos[1] = k;
  vs.probe = xs; vs.probe_bs = xs_bs; vs.probe_npos[0] = k; vs.probe_npos[1] = k;
  vs.nrows = B;
  DrawSpec d = {k, u_acc, u_bs, u_res, alive, n_acc, y, px, qx, nullptr, nullptr, 0, 0};
  return run_sampling(vs, nvec, dtype, V, temperature, top_p, top_k, L, ws, st, &d);
}

int sd_verify_sample_qprobs(const void* tgt, int64_t tgt_bs, int64_t tgt_ps, int dtype,
                            const float* qprobs, int64_t q_bs, int64_t q_ps,
                            const int64_t* xs, int64_t xs_bs, const float* u_acc, int64_t u_bs,
                            const float* u_res, const uint8_t* alive,
                            int B, int k, int V, float temperature, float top_p, int top_k,
                            int64_t* n_acc, int64_t* y, float* px, float* qx,
                            void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate_common(dtype, V, temperature);
  if (rc) return rc;
  if (B <= 0 || k < 1 || k > 64 || !tgt || !xs || !u_acc || !u_res || !n_acc || !y || !workspace)
    return SD_EINVAL;
  const bool greedy = !(temperature > 0.0f);
  if (greedy)                       // one-hot p: q plays no part (sd_verify_sample's greedy path)
    return sd_verify_sample(tgt, tgt_bs, tgt_ps, nullptr, 0, 0, dtype, xs, xs_bs, u_acc, u_bs,
                            u_res, alive, B, k, V, temperature, top_p, top_k, n_acc, y, px, qx,
                            workspace, workspace_bytes, stream);
  if (!qprobs) return SD_EINVAL;
  if (use_small(V, dtype)) return SD_ENOTSUP;       // the list kernels: bf16 / fp16, V > 2048
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(workspace);
  const int nvec = B * (k + 1);
  WsLayout L = ws_layout(B, nvec, V, false);
  if (workspace_bytes < L.total) return SD_ENOSPC;
  VecSet vs = {};
  vs.base[0] = tgt; vs.bs[0] = tgt_bs; vs.ps[0] = tgt_ps; vs.npos[0] = k + 1; vs.npos[1] = 0;
  vs.probe = xs; vs.probe_bs = xs_bs; vs.probe_npos[0] = k; vs.probe_npos[1] = 0;
  vs.nrows = B;
  DrawSpec d = {k, u_acc, u_bs, u_res, alive, n_acc, y, px, qx, nullptr, qprobs, q_bs, q_ps};
  return run_sampling(vs, nvec, dtype, V, temperature, top_p, top_k, L, ws, st, &d);
}

int sd_verify_greedy_static(const void* tgt, int64_t tgt_bs, int64_t tgt_ps, int dtype,
                            const int64_t* xs, int64_t xs_bs, const float* u_acc, int64_t u_bs,
                            const uint8_t* alive, int B, int k, int V, int64_t* n_acc,
                            int64_t* y, float* px, float* qx, void* stream) {
  int rc = validate_common(dtype, V, 0.0f);
  if (rc) return rc;
  if (B <= 0 || k < 1 || k > 64 || !tgt || !xs || !u_acc || !n_acc || !y) return SD_EINVAL;
  // per vector: f32, one key per chunk block; 16-bit, one per warp slot
  int nslot = 0;
  if (dtype == SD_DTYPE_F32) {
    nslot = argmax_geom(V, dtype).nch;
  } else {
    Am16Geom g;
    if ((rc = am16_geom(V, B * (k + 1), &g))) return rc;
    nslot = g.cpv;
  }
  const StaticLayout L = static_layout(B, B * (k + 1), nslot);
  if (L.total > SD_STATIC_SCRATCH_BYTES) return SD_ENOSPC;
  char* ws = nullptr;
  if ((rc = static_scratch(&ws))) return rc;
  return launch_greedy_verify(tgt, tgt_bs, tgt_ps, dtype, xs, xs_bs, u_acc, u_bs, alive, B, k, V,
                              n_acc, y, px, qx, reinterpret_cast<VecStats*>(ws + L.stats),
                              reinterpret_cast<unsigned long long*>(ws + L.partial),
                              reinterpret_cast<int*>(ws + L.vcounter),
                              reinterpret_cast<int*>(ws + L.rcounter),
                              reinterpret_cast<cudaStream_t>(stream));
}

int sd_draft_sample(const void* logits, int64_t row_stride, int dtype, int B, int V,
                    const float* u, float temperature, float top_p, int top_k,
                    int64_t* x, float* qx, void* workspace, size_t workspace_bytes,
                    void* stream) {
  int rc = validate_common(dtype, V, temperature);
  if (rc) return rc;
  if (B <= 0 || !logits || !u || !x || !workspace) return SD_EINVAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(workspace);
  VecSet vs = {};
  vs.base[0] = logits; vs.bs[0] = row_stride; vs.ps[0] = 0; vs.npos[0] = 1; vs.npos[1] = 0;
  vs.nrows = B;
  if (!(temperature > 0.0f)) {
    WsLayout L = ws_layout(B, B, V, use_small(V, dtype));
    if (workspace_bytes < L.total) return SD_ENOSPC;
    ArgmaxParams P;
    P.vs = vs; P.dtype = dtype; P.V = V; P.nvec = B;
    const ArgmaxGeom ag = argmax_geom(V, dtype);
    P.nch = ag.nch; P.cu = ag.cu;
    P.partial = reinterpret_cast<unsigned long long*>(ws + L.apartial);
    P.vec_counter = reinterpret_cast<int*>(ws + L.vcounter);
    P.row_counter = reinterpret_cast<int*>(ws + L.rcounter);
    P.stats = reinterpret_cast<VecStats*>(ws + L.stats);
    P.k = 0; P.xs = nullptr; P.xs_bs = 0; P.u_acc = nullptr; P.u_bs = 0; P.alive = nullptr;
    P.n_acc = nullptr; P.y = x; P.px = nullptr; P.qx = qx;
    return launch_argmax(P, st);
  }
  WsLayout L = ws_layout(B, B, V, use_small(V, dtype));
  if (workspace_bytes < L.total) return SD_ENOSPC;
  DrawSpec d = {0, nullptr, 0, u, nullptr, nullptr, x, nullptr, nullptr, qx, nullptr, 0, 0};
  return run_sampling(vs, B, dtype, V, temperature, top_p, top_k, L, ws, st, &d);
}

int sd_to_probs(const void* logits, int64_t row_stride, int dtype, int n_rows, int V,
                float temperature, float top_p, int top_k, float* out, int64_t out_stride,
                void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate_common(dtype, V, temperature);
  if (rc) return rc;
  if (n_rows < 0 || !logits || !out || !workspace) return SD_EINVAL;
  if (n_rows == 0) return SD_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(workspace);
  VecSet vs = {};
  vs.base[0] = logits; vs.bs[0] = row_stride; vs.ps[0] = 0; vs.npos[0] = 1; vs.npos[1] = 0;
  vs.nrows = n_rows;
  const bool greedy = !(temperature > 0.0f);
  const bool small = !greedy && use_small(V, dtype);
  WsLayout L = ws_layout(n_rows, n_rows, V, use_small(V, dtype));
  if (workspace_bytes < L.total) return SD_ENOSPC;
  ProbsParams P;
  P.vs = vs; P.dtype = dtype; P.V = V; P.nch = nch_for(V); P.chunk = (V + P.nch - 1) / P.nch;
  P.greedy = greedy; P.T = temperature;
  P.stats = reinterpret_cast<const VecStats*>(ws + L.stats);
  P.mat = small ? reinterpret_cast<const float*>(ws + L.mat) : nullptr;
  P.out = out; P.out_stride = out_stride;
  if (greedy) {
    ArgmaxParams A;
    A.vs = vs; A.dtype = dtype; A.V = V; A.nvec = n_rows;
    const ArgmaxGeom ag = argmax_geom(V, dtype);
    A.nch = ag.nch; A.cu = ag.cu;
    A.partial = reinterpret_cast<unsigned long long*>(ws + L.apartial);
    A.vec_counter = reinterpret_cast<int*>(ws + L.vcounter);
    A.row_counter = reinterpret_cast<int*>(ws + L.rcounter);
    A.stats = reinterpret_cast<VecStats*>(ws + L.stats);
    A.k = -1;   // stats only: no per-row decision
    A.xs = nullptr; A.xs_bs = 0; A.u_acc = nullptr; A.u_bs = 0; A.alive = nullptr;
    A.n_acc = nullptr; A.y = nullptr; A.px = nullptr; A.qx = nullptr;
    if ((rc = launch_argmax(A, st))) return rc;
  } else {
    rc = run_sampling(vs, n_rows, dtype, V, temperature, top_p, top_k, L, ws, st, nullptr);
    if (rc) return rc;
  }
  probs_kernel<<<P.nch * n_rows, FT, 0, st>>>(P);
  return check_launch();
}

int sd_residual_probs(const float* p, const float* q, int n_rows, int V, float* out, void* stream) {
  if (n_rows < 0 || V <= 0 || !p || !q || !out) return SD_EINVAL;
  if (n_rows == 0) return SD_OK;
  residual_kernel<<<n_rows, FT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p, q, V, out);
  return check_launch();
}

int sd_sample_from_probs(const float* probs, int n_rows, int V, const float* u, int64_t* out,
                         void* stream) {
  if (n_rows < 0 || V <= 0 || !probs || !u || !out) return SD_EINVAL;
  if (n_rows == 0) return SD_OK;
  sample_probs_kernel<<<n_rows, FT, 0, reinterpret_cast<cudaStream_t>(stream)>>>(probs, V, u, out);
  return check_launch();
}

int sd_gather_prob(const float* probs, int n_rows, int V, const int64_t* ids, float* out,
                   void* stream) {
  if (n_rows < 0 || V <= 0 || !probs || !ids || !out) return SD_EINVAL;
  if (n_rows == 0) return SD_OK;
  gather_kernel<<<(n_rows + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      probs, n_rows, V, ids, out);
  return check_launch();
}

}  // extern "C"
