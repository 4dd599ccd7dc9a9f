/*
 * specdec_b200 -- C ABI of the B200-native verify-round kernels.
 *
 * Conventions (all entry points):
 *   - plain device pointers and sizes; the caller owns every buffer, including
 *     the workspace, and the library allocates nothing;
 *   - all work is enqueued on `stream` (a cudaStream_t passed as void*), no
 *     host synchronisation;
 *   - return 0 on success or a negative errno-style code (SD_E*) for bad
 *     shapes, unsupported configurations, a too-small workspace or a failed
 *     launch;
 *   - token ids are int64 (torch.long, as the reference uses);
 *   - logits rows are contiguous along the vocabulary; other dimensions are
 *     addressed by element strides.
 *
 * Uniforms are passed in as arrays so that every draw is a deterministic
 * function of its inputs: the draw from a distribution r over the vocabulary
 * is the smallest index j whose running float64 sum of r exceeds u * sum(r).
 */
#ifndef SPECDEC_B200_H_
#define SPECDEC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SD_OK 0
#define SD_EINVAL (-22)    /* bad shape / argument */
#define SD_ENOTSUP (-95)   /* configuration not supported by these kernels */
#define SD_ENOSPC (-28)    /* workspace too small */
#define SD_ERANGE (-34)    /* length would leave [0, capacity] */
#define SD_ELAUNCH (-5)    /* CUDA launch error */

#define SD_DTYPE_F32 0
#define SD_DTYPE_F16 1
#define SD_DTYPE_BF16 2

/* Tokens per page of a paged KV cache (one K/V tile of the tcgen05 verify
 * attention).  A paged layer is a pool [npages, H, SD_KV_PAGE, D] per K and
 * V; row b's slot s lives in page block_table[b * bt_stride + s / SD_KV_PAGE]
 * (int32, -1 = no page assigned), so a row's capacity is
 * bt_stride * SD_KV_PAGE. */
#define SD_KV_PAGE 128

/* Library version and build information, for the loaders' sanity checks. */
int sd_version(void);

/* Workspace bytes needed by sd_verify_sample / sd_draft_sample / sd_to_probs
 * for n_vec logits vectors of width V split over n_rows rows.  A workspace
 * needs no initialisation (each call zeroes the counters it uses; the greedy
 * calls use none) and may be reused by later calls of any shape on the same
 * stream; calls that overlap on the GPU need separate workspaces. */
size_t sd_sampling_workspace_bytes(int n_rows, int n_vec, int V, int dtype);

/* The first 4 bytes of a sampling workspace hold a sticky device status word:
 * bit 0 is set when a kernel's bounded wait on its own copy pipeline timed out
 * (the affected outputs are then invalid).  Kernels only ever set bits; the
 * caller reads it at its convenience and clears it. */
#define SD_STATUS_WAIT_TIMEOUT 1

/*
 * Fused verify round: to_probs on every target/draft vector, the accept test
 * u < min(1, p(x)/max(q(x),1e-10)) with prefix-alive semantics, and the
 * residual draw from norm((p-q)+) at the first rejection, or the bonus draw
 * from p_k when every draft token was accepted.
 *
 * Replaces reference specdec/engine.py:282-303 (the k+1 to_probs calls, the
 * accept loop and the two sample_from_probs calls) and, inside it,
 * specdec/sampling.py:34-95 (to_probs, residual_probs, gather_prob).
 *
 *   tgt    [B, k+1, V] logits, element strides (tgt_bs, tgt_ps, 1)
 *   drf    [B, k,   V] logits, element strides (drf_bs, drf_ps, 1); unused
 *          (may be NULL) when temperature <= 0 (greedy reads the target only)
 *   xs     [B, k] int64 draft tokens, row stride xs_bs
 *   u_acc  [B, k] float uniforms for the accept tests, row stride u_bs
 *   u_res  [B] float uniform for the residual / bonus draw
 *   alive  [B] uint8 or NULL (NULL = all rows alive; the reference's ~done)
 *   n_acc  [B] int64 out: accepted draft tokens per row
 *   y      [B] int64 out: the emitted token (residual or bonus draw)
 *   px, qx [B, k] float out or NULL: p_i(x_i) and q_i(x_i)
 */
int sd_verify_sample(const void* tgt, int64_t tgt_bs, int64_t tgt_ps,
                     const void* drf, int64_t drf_bs, int64_t drf_ps, int dtype,
                     const int64_t* xs, int64_t xs_bs, const float* u_acc, int64_t u_bs,
                     const float* u_res, const uint8_t* alive,
                     int B, int k, int V, float temperature, float top_p, int top_k,
                     int64_t* n_acc, int64_t* y, float* px, float* qx,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * The verify round of sd_verify_sample with the draft distributions given as
 * probabilities instead of draft logits: what a serving engine's rejection
 * sampler holds (vLLM's RejectionSampler.forward receives draft_probs
 * [num_tokens, V] fp32, vllm/v1/sample/rejection_sampler.py:87-95, built
 * from the draws its drafter made).  Same accept test, residual and bonus
 * draws as sd_verify_sample (reference specdec/engine.py:282-303), with
 * q_i = qprobs[b, i, :] used as given (no temperature, top-p or top-k on it);
 * to_probs (temperature, top-p, top-k) applies to the target logits only.
 *
 *   qprobs [B, k, V] fp32, element strides (q_bs, q_ps, 1)
 *   other arguments as sd_verify_sample (drf is not taken)
 *
 * temperature <= 0 is the greedy round (qprobs unused).  Sampling needs
 * bf16 / fp16 target logits with V > 2048 (SD_ENOTSUP otherwise).
 */
int sd_verify_sample_qprobs(const void* tgt, int64_t tgt_bs, int64_t tgt_ps, int dtype,
                            const float* qprobs, int64_t q_bs, int64_t q_ps,
                            const int64_t* xs, int64_t xs_bs, const float* u_acc, int64_t u_bs,
                            const float* u_res, const uint8_t* alive,
                            int B, int k, int V, float temperature, float top_p, int top_k,
                            int64_t* n_acc, int64_t* y, float* px, float* qx,
                            void* workspace, size_t workspace_bytes, void* stream);

/*
 * No counterpart in the reference (added entry point), for callers that may
 * not allocate device memory: a serving framework that reserves nearly all
 * of the GPU for its own KV-cache pool up front and forbids other
 * allocations (cudaMalloc can also synchronise the device in the middle of
 * a decode step), or a host that binds the C ABI and only ever holds
 * pointers it was handed.  The greedy verify
 * round of sd_verify_sample (temperature <= 0: u_res, draft logits, top-p and
 * top-k unused; same arguments, results and error codes otherwise) with no
 * workspace argument: its scratch is a fixed SD_STATIC_SCRATCH_BYTES device
 * array inside this library, one per device, whose address is looked up once
 * per device (cudaGetSymbolAddress) on the first call there.  The call
 * allocates no memory.  Returns SD_ENOSPC when the shape needs more scratch
 * than that (about B*(k+1)*(52 + 8*chunks) bytes; chunks = the vector's
 * 16-byte units / 256..512, 43 at V = 151936).
 * Calls that overlap on one device (other streams, other host threads) share
 * the scratch and race: serialise them.  The first call on a device does the
 * one-time set-up (the symbol lookup); make it before any stream capture.
 */
#define SD_STATIC_SCRATCH_BYTES (1u << 20)
#define SD_MAX_DEVICES 64
int sd_verify_greedy_static(const void* tgt, int64_t tgt_bs, int64_t tgt_ps, int dtype,
                            const int64_t* xs, int64_t xs_bs, const float* u_acc, int64_t u_bs,
                            const uint8_t* alive, int B, int k, int V, int64_t* n_acc,
                            int64_t* y, float* px, float* qx, void* stream);

/*
 * One draft step: x[b] ~ to_probs(logits[b]) drawn by inverse CDF with u[b],
 * and qx[b] = q(x[b]).  Replaces reference specdec/engine.py:250-251 and 256
 * (to_probs, sample_from_probs, gather_prob for the confidence product).
 *   logits [B, V], row stride row_stride; x [B] int64; qx [B] float or NULL.
 */
int sd_draft_sample(const void* logits, int64_t row_stride, int dtype, int B, int V,
                    const float* u, float temperature, float top_p, int top_k,
                    int64_t* x, float* qx, void* workspace, size_t workspace_bytes,
                    void* stream);

/*
 * to_probs: logits [n_rows, V] (row stride row_stride) -> fp32 probabilities
 * [n_rows, V] (row stride out_stride).  Replaces specdec/sampling.py:34-67.
 */
int sd_to_probs(const void* logits, int64_t row_stride, int dtype, int n_rows, int V,
                float temperature, float top_p, int top_k, float* out, int64_t out_stride,
                void* workspace, size_t workspace_bytes, void* stream);

/* residual_probs: norm((p-q)+) row-wise, p falling back when the positive
 * part sums to <= 1e-9.  Replaces specdec/sampling.py:77-90.  fp32 [n, V]. */
int sd_residual_probs(const float* p, const float* q, int n_rows, int V, float* out,
                      void* stream);

/* sample_from_probs with given uniforms: out[i] = inverse-CDF draw of row i.
 * Replaces specdec/sampling.py:70-74 (torch.multinomial). */
int sd_sample_from_probs(const float* probs, int n_rows, int V, const float* u,
                         int64_t* out, void* stream);

/* gather_prob: out[i] = probs[i, ids[i]].  Replaces specdec/sampling.py:93-95. */
int sd_gather_prob(const float* probs, int n_rows, int V, const int64_t* ids, float* out,
                   void* stream);

/* ---- ragged KV cache (reference specdec/kvcache.py) --------------------- */

/*
 * lengths[b] += delta[b] (delta NULL: += q for every row).  Any row leaving
 * [0, capacity] is left unchanged and sets *err (device int) to 1.
 * Replaces RaggedCache.advance / rollback / set_lengths bookkeeping
 * (specdec/kvcache.py:165-190) with device-resident lengths: O(1), no data
 * movement, no host sync.  `sign` is +1 (advance) or -1 (rollback).
 */
int sd_kv_lengths_update(int64_t* lengths, const int64_t* delta, int64_t q, int sign,
                         int B, int64_t capacity, int* err, void* stream);

/*
 * Commit a verify round: lengths[b] -= k - n_acc[b] (drops the rejected tail).
 * Replaces the rollback at specdec/engine.py:309-312 without the host copy.
 */
int sd_kv_commit(int64_t* lengths, const int64_t* n_acc, int k, int B, int* err,
                 void* stream);

/*
 * Append q new tokens per row at each row's own offset:
 *   cache[b, h, lengths[b] + j, :] = new[b, h, j, :]   for j < q
 * for the K and V caches of one layer ([B, H, C, D] contiguous) from
 * new_k / new_v ([B, H, q, D] with element strides (nbs, nhs, nqs, 1)).
 * Replaces the scatter in _RaggedLayer.update (specdec/kvcache.py:61-74).
 * Rows whose write would pass `capacity` are skipped and set *err.
 */
int sd_kv_append(void* kcache, void* vcache, const void* new_k, const void* new_v,
                 int64_t nbs, int64_t nhs, int64_t nqs, const int64_t* lengths,
                 int B, int H, int C, int D, int q, int dtype, int* err, void* stream);

/*
 * sd_kv_append into a paged layer (pools and block table as SD_KV_PAGE
 * describes).  A slot whose page is not assigned (-1) is not written and
 * sets bit 1 of *err; rows past bt_stride * SD_KV_PAGE set bit 0.
 */
int sd_kv_append_paged(void* kpool, void* vpool, const void* new_k, const void* new_v,
                       int64_t nbs, int64_t nhs, int64_t nqs, const int32_t* block_table,
                       int bt_stride, int npages, const int64_t* lengths, int B, int H, int D,
                       int q, int dtype, int* err, void* stream);

/*
 * The fused step between an attention layer's QKV projections and its
 * attention, for bf16 Qwen3 / Llama-style layers: per row b, position
 * l < L and head, the head's RMSNorm on q and k (weights q_norm_w / k_norm_w
 * [D], eps; both null: no norm), the rotary embedding with (cos, sin)
 * [B, L, D] (element strides (cs_bs, cs_ls, 1)) on q and k, then
 *   q_out[b, h, l, :]             = q'      ([B, Hq, L, D] contiguous)
 *   kcache[b, h, lengths[b] + l]  = k',  vcache[...] = v
 * (caches [B, Hkv, C, D]).  q, k, v are the projections' outputs, rows
 * b * L + l with element strides q_rs / k_rs / v_rs and heads of D contiguous
 * elements.  Replaces transformers' q_norm / k_norm and apply_rotary_pos_emb
 * in Qwen3Attention.forward and the cache update of _RaggedLayer.update
 * (reference specdec/kvcache.py:61-74): one launch instead of a dozen
 * elementwise kernels and the append.  Same arithmetic on bf16 tensors, but
 * for the float32 sum of squares' order (a normalised value may differ by one
 * bf16 ulp).  Rows whose slots would pass C are not written and set bit 0
 * of *err.  block_table non-NULL: kcache / vcache are page pools
 * (SD_KV_PAGE), C <= bt_stride * SD_KV_PAGE, and a slot without a page is
 * not written and sets bit 1.
 */
int sd_qkv_norm_rope_append(const void* q, int64_t q_rs, const void* k, int64_t k_rs,
                            const void* v, int64_t v_rs, const void* q_norm_w,
                            const void* k_norm_w, float eps, const void* cos, const void* sin,
                            int64_t cs_bs, int64_t cs_ls, void* kcache, void* vcache,
                            const int32_t* block_table, int bt_stride, int npages,
                            const int64_t* lengths, int B, int L, int Hq, int Hkv, int D, int C,
                            void* q_out, int* err, void* stream);

/*
 * The decoder layers' RMSNorm as one launch (bf16): for each of `rows` rows
 * of H elements (x rows x_rs elements apart, out rows out_rs apart)
 *   out = rn(w * rn(x * rsqrt(mean(x^2) + eps)))
 * transformers' Qwen3RMSNorm / LlamaRMSNorm arithmetic (the float32 sum of
 * squares in another order: a value may differ by one bf16 ulp).  In place
 * (out == x) is allowed.
 */
int sd_rmsnorm(const void* x, int64_t x_rs, const void* w, float eps, void* out, int64_t out_rs,
               int rows, int H, void* stream);

/*
 * A decoder layer's residual add and the norm after it as one launch (bf16):
 *   res_out = rn(x + res);  out = sd_rmsnorm(res_out)
 * (transformers' "residual = residual + hidden_states" then
 * post_attention_layernorm).  H <= 8192.  Outputs may alias the inputs.
 */
int sd_add_rmsnorm(const void* x, int64_t x_rs, const void* res, int64_t res_rs, const void* w,
                   float eps, void* out, int64_t out_rs, void* res_out, int64_t ro_rs, int rows,
                   int H, void* stream);

/*
 * The gated MLP's activation as one launch (bf16): gu rows hold [gate | up]
 * (2 I elements, rows gu_rs apart);
 *   out[r, i] = rn(rn(silu(gate[r, i])) * up[r, i])
 * as transformers' act_fn(gate_proj(x)) * up_proj(x) with SiLU.
 */
int sd_silu_mul(const void* gu, int64_t gu_rs, void* out, int64_t out_rs, int rows, int I,
                void* stream);

/*
 * Verify attention over the ragged cache (after the append of this forward):
 * query j of row b (position lengths[b] + j) attends to cache slots
 * s <= lengths[b] + j, i.e. the reference mask s <= len[b] + j
 * (specdec/kvcache.py:138-162) with SDPA (HF Qwen3 attention at
 * specdec/engine.py:274), grouped-query: query head h reads kv head
 * h / (Hq/Hkv).  `lengths` are the lengths BEFORE this forward's advance.
 *   q   [B, Hq, qlen, D] (strides qbs, qhs, qqs, 1)
 *   k/v [B, Hkv, C, D] contiguous
 *   out [B, qlen, Hq, D] (strides obs, oqs, ohs, 1)
 *   valid [B] int64 or NULL: optional cap s < valid[b] (right-padded prefill)
 *   dtype SD_DTYPE_BF16 (the Qwen3 path) or SD_DTYPE_F32; fp32 accumulation.
 */
int sd_verify_attn(const void* q, int64_t qbs, int64_t qhs, int64_t qqs,
                   const void* kcache, const void* vcache, const int64_t* lengths,
                   const int64_t* valid, int B, int Hq, int Hkv, int D, int C, int qlen,
                   float scale, void* out, int64_t obs, int64_t oqs, int64_t ohs, int dtype,
                   void* workspace, size_t workspace_bytes, void* stream);

size_t sd_verify_attn_workspace_bytes(int B, int Hq, int Hkv, int D, int C, int qlen);

/*
 * sd_verify_attn over a paged cache: kpool / vpool [npages, Hkv, SD_KV_PAGE,
 * D] and the rows' block table [B, bt_stride] (SD_KV_PAGE above).  Same
 * masking and arithmetic; the row capacity C is bt_stride * SD_KV_PAGE (size
 * the workspace with it).  A page index outside [0, npages) reads page 0.
 * The reference keeps one capacity-padded buffer per layer
 * (specdec/kvcache.py:98-116); pages let rows of very different lengths
 * share one pool.
 */
int sd_verify_attn_paged(const void* q, int64_t qbs, int64_t qhs, int64_t qqs,
                         const void* kpool, const void* vpool, const int32_t* block_table,
                         int bt_stride, int npages, const int64_t* lengths, const int64_t* valid,
                         int B, int Hq, int Hkv, int D, int qlen, float scale, void* out,
                         int64_t obs, int64_t oqs, int64_t ohs, int dtype, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * Vocabulary-sharded verify round: the SPMD form of sd_verify_sample for a
 * vocab-parallel LM head.  Rank r holds columns [v_start[r], v_start[r+1]) of
 * every target and draft logits vector; every rank ends with the n_acc and y
 * that sd_verify_sample gives on the full vectors (same arithmetic, same
 * exemptions).  The reference verifies on one device only; this replaces
 * specdec/engine.py:282-303 when the logits arrive vocab-sharded.
 *
 * The round is a fixed sequence of local phases; between two phases the
 * caller runs one collective over all ranks on the phase's send buffer
 * (sd_shard_send_bytes) and passes the result as the next phase's recv:
 *
 *   temperature > 0:  P1 -> all_gather -> P2 -> all_reduce(sum, float64)
 *                     -> P3 -> all_gather -> P4 -> all_gather
 *                     -> P5 -> all_reduce(max, int64) -> P6
 *   temperature <= 0: P1 -> all_reduce(max, int64) -> P6
 *
 * all_gather concatenates the ranks' buffers in rank order.  What crosses
 * the ranks: P1 each shard's maximum and the draft tokens' logits; P2 the
 * shard's softmax normaliser and a 128-bin depth histogram of its mass
 * (16 base-2 units below the global maximum); P3 the shard's mass above the
 * top-p boundary bins and its elements inside them (at most
 * SD_SHARD_BOUNDARY_CAP per vector); P4 the shard's residual mass per row;
 * P5 the drawn token from the shard that holds it.  Greedy needs only the
 * per-shard argmax.  top_k must be 0 (SD_ENOTSUP otherwise).
 *
 * When the top-p boundary lies deeper than the histogram window or a shard
 * holds more boundary elements than the cap, the round cannot be decided
 * from these messages: P6 then sets SD_SHARD_STATUS_FALLBACK in the status
 * word (the first 4 bytes of the workspace, identical on every rank) and
 * the caller re-runs the round on gathered full vectors.
 */
#define SD_SHARD_MAX_RANKS 16
#define SD_SHARD_BOUNDARY_CAP 128
#define SD_SHARD_STATUS_FALLBACK 2
typedef struct sd_shard_args {
  const void* tgt;              /* [B, k+1, Vr] local slice, element strides (tgt_bs, tgt_ps, 1) */
  int64_t tgt_bs, tgt_ps;
  const void* drf;              /* [B, k, Vr] local slice (unused when temperature <= 0) */
  int64_t drf_bs, drf_ps;
  int dtype;                    /* SD_DTYPE_BF16 or SD_DTYPE_F16 */
  const int64_t* xs;            /* [B, k] draft tokens, global vocabulary ids */
  int64_t xs_bs;
  const float* u_acc;           /* [B, k] */
  int64_t u_bs;
  const float* u_res;           /* [B] */
  const uint8_t* alive;         /* [B] or NULL */
  int B, k, V, rank, nranks;
  int v_start[SD_SHARD_MAX_RANKS + 1];   /* v_start[0] = 0, v_start[nranks] = V */
  float temperature, top_p;
  int top_k;
  int64_t* n_acc;               /* [B] out (written by P6) */
  int64_t* y;                   /* [B] out (written by P6) */
  void* workspace;
  size_t workspace_bytes;
} sd_shard_args;

size_t sd_shard_workspace_bytes(int B, int k, int nranks);
/* Bytes this rank contributes to the collective that follows phase `phase`
 * (1..5); the collective's result is nranks times that for an all_gather and
 * the same size for an all_reduce.  0 when no collective follows. */
size_t sd_shard_send_bytes(int B, int k, int nranks, int greedy, int phase);
/* Run local phase `phase` (1..6).  recv: the previous collective's result
 * (NULL for P1); send: this phase's send buffer (NULL for P6). */
int sd_shard_phase(const sd_shard_args* args, int phase, const void* recv, void* send,
                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPECDEC_B200_H_ */
