/*
 * sgsa_b200 -- C ABI of the B200 (sm_100a) SGSA layer forward.
 *
 * Every entry point takes raw device pointers, plain integer shapes and a
 * cudaStream_t (passed as void*), returns an int status (SGSA_OK == 0, a
 * negative SGSA_ERR_* otherwise) and never aborts or traps.  The library keeps
 * no pointers between calls and allocates nothing: outputs and workspaces are
 * owned by the caller, sized with the *_workspace_size queries.  The library
 * holds, per device, cached kernel attributes, the device watchdog words
 * (sgsa_watchdog_status) and the no-allocation entry point's scratch array, and
 * per host thread and device the side stream of sgsa_layer_fwd.
 *
 * Tensor layouts follow the reference (row-major, contiguous):
 *   q, k, v, sparse_k, sparse_v, o     [B, T, H, D]          dtype
 *   beta, gamma, alpha                 [B, T, H]             dtype
 *   initial_state, final_state         [B, H, D, D]          float32, S[d_k][d_v]
 *   iq, ik (indexer)                   [B, T, H, DI]         dtype
 *   mix                                [B, T, H, D] or [B, T, H]   dtype
 *   top-k indices                      [B, H, T, K]          int32, ascending, -1 padded
 * dtype is SGSA_DTYPE_F32 or SGSA_DTYPE_BF16 for all floating inputs of a call.
 */
#ifndef SGSA_B200_H_
#define SGSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SGSA_OK = 0,
    SGSA_ERR_SHAPE = -1,       /* bad or unsupported shape */
    SGSA_ERR_DTYPE = -2,       /* unsupported dtype */
    SGSA_ERR_NULL = -3,        /* required pointer is NULL */
    SGSA_ERR_WORKSPACE = -4,   /* workspace too small or misaligned */
    SGSA_ERR_LAUNCH = -5,      /* CUDA launch / runtime error */
    SGSA_ERR_UNSUPPORTED = -6, /* valid request this build does not implement */
    SGSA_ERR_DEVICE = -7       /* current device is not sm_100 */
};

enum { SGSA_DTYPE_F32 = 0, SGSA_DTYPE_BF16 = 1 };

/* Flags of sgsa_chunk_fwd. */
enum {
    SGSA_FLAG_HAS_SPARSE = 1,   /* sparse_k/sparse_v/alpha given: 2 virtual samples per token */
    SGSA_FLAG_HAS_INIT = 2,     /* initial_state given */
    SGSA_FLAG_STORE_FINAL = 4,  /* write final_state */
    SGSA_FLAG_OUT_F32 = 8,      /* o is float32 regardless of dtype */
    /* Tensor-core path only (bf16, D == 128, no sparse write): */
    SGSA_FLAG_TRANSITION = 16,  /* v taken as zero and o not written: final_state = M initial_state,
                                   M the product of the chunk transitions (sequence-parallel pass) */
    SGSA_FLAG_REUSE_PREP = 32   /* the workspace holds the per-chunk operands of these same inputs
                                   from a previous call: only the scan runs */
};

/* Human-readable text of a status code (static storage). */
const char *sgsa_status_string(int status);

/* Last CUDA error text seen by this thread (static storage, "" if none). */
const char *sgsa_last_error(void);

/* Library version, e.g. 1000 for 0.1.0. */
int sgsa_version(void);

/* Number of kernels this library has launched in this process (all devices and
 * threads).  No reference counterpart: it lets a benchmark count its launches. */
unsigned long long sgsa_kernel_launches(void);

/*
 * Synchronises `stream`, returns and clears the device watchdog word: 0 when
 * every bounded wait inside the tensor-core kernels completed, else a bitmask
 * of the waits that gave up (their results are then invalid).  No reference
 * counterpart: the reference's Triton kernels have no device-side waits.
 */
int sgsa_watchdog_status(void *stream);

/*
 * Exercises the watchdog path: launches one thread that waits, with at most
 * spin_limit polls (1 .. 2^20), on a barrier nothing arrives at.  The wait gives
 * up and the kernel returns; the next sgsa_watchdog_status on `stream` then
 * reports bit 0x80.  No reference counterpart (test support).
 */
int sgsa_watchdog_selftest(unsigned int spin_limit, void *stream);

/*
 * Bounds-checked debug build (libsgsa_b200_check.so, the same sources compiled
 * with -DSGSA_CHECK): kernels test the invariants of their index arithmetic --
 * caller-supplied gather and decode indices within [-1, T), the indexer's
 * candidate lists within their capacity, exactly top_k collected indices, each
 * inside its row, a threshold record for every attended row -- record a violated
 * one as a bit (0x1 gather index, 0x2 decode index, 0x10 candidate capacity,
 * 0x20 collect count, 0x40 collected index, 0x100 threshold record) and skip the
 * access it guards.  Synchronises the device and stores the OR of the bits in
 * *word (cleared when reset != 0).  The release build returns
 * SGSA_ERR_UNSUPPORTED.  No reference counterpart (a stand-in for running the
 * kernels under a memory checker).
 */
int sgsa_check_status(unsigned int *word, int reset);

/*
 * Chunked SGSA / gated-delta-rule forward.
 * Replaces chunk_sgsa (modelings/sgsa_ops/chunk.py:104-148) and its forward
 * chunk_sgsa_fwd (modelings/sgsa_ops/chunk_fwd.py:12-131), with the semantics of
 * naive_recurrent_sgsa (modelings/sgsa_ops/naive.py:39-55): no query scale,
 * o_t = S_t^T q_t.  d_k == d_v == D, D in {32, 64, 128}; chunk_size == 64.
 * sparse_k/sparse_v/alpha may be NULL unless SGSA_FLAG_HAS_SPARSE is set.
 * bf16 with D == 128 runs on the tensor cores, the sparse write included (its
 * two samples per token as 2T interleaved rows); the workspace size covers
 * that layout and the CUDA-core one, since it does not take the dtype.  Flag
 * bits outside SGSA_FLAG_* are ignored.
 */
size_t sgsa_chunk_fwd_workspace_size(int B, int T, int H, int D, int flags);
int sgsa_chunk_fwd(const void *q, const void *k, const void *v, const void *beta,
                   const void *gamma, const void *sparse_k, const void *sparse_v,
                   const void *alpha, const float *initial_state, void *o,
                   float *final_state, int B, int T, int H, int D, int dtype, int chunk_size,
                   int flags, void *workspace, size_t workspace_bytes, void *stream);

/*
 * Same as sgsa_chunk_fwd, but for callers that cannot allocate device memory
 * when they run (a fixed memory plan, a locked allocator, a plugin that only
 * receives its inputs and outputs).  No reference counterpart: the
 * reference's op allocates its temporaries through torch.  The workspace is a
 * 64 MiB scratch array built into the library and held on every GPU that
 * loads it; a problem whose sgsa_chunk_fwd_workspace_size exceeds 64 MiB is
 * rejected with SGSA_ERR_WORKSPACE.  The first call on each device looks up
 * the array's device address, so make it before any stream capture.  All
 * calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  SGSA_FLAG_REUSE_PREP is refused with
 * SGSA_ERR_UNSUPPORTED, since the shared array may hold another caller's
 * operands.  A cudaDeviceReset invalidates the cached address: do not call
 * this entry point after one.  The call allocates and frees nothing.
 */
int sgsa_chunk_fwd_noalloc(const void *q, const void *k, const void *v, const void *beta,
                           const void *gamma, const void *sparse_k, const void *sparse_v,
                           const void *alpha, const float *initial_state, void *o,
                           float *final_state, int B, int T, int H, int D, int dtype,
                           int chunk_size, int flags, void *stream);

/*
 * Causal per-head top-k indexer: s_tj = iq_t . ik_j for j <= t; row t keeps the
 * min(top_k, t+1) largest, ties to the lowest j, written ascending and padded
 * with -1.  Replaces the selection of TopKSparseKVReuseAttention.forward
 * (modelings/hybrid_dense_delta_topk.py:344-349) and
 * SparseRetriever._masked_topk (modelings/modeling_sgsa.py:144-165).
 * DI in {32, 64, 128}; bf16 scores run on tcgen05 when DI % 64 == 0.
 */
int sgsa_indexer_topk(const void *iq, const void *ik, int32_t *indices, int B, int T, int H,
                      int DI, int top_k, int dtype, void *stream);

/*
 * Test support for the tensor-core indexer (bf16, DI 64 or 128, T <= 4096): the
 * call of sgsa_indexer_topk that also writes the fp32 scores its selection ran on,
 * scores[B,H,T,T] (row t: columns j <= t; rows t < top_k, which keep every
 * column, may be left unwritten).  Selecting top_k on those very scores with the
 * rule of modelings/modeling_sgsa.py:155-164 (ties to the lowest index) must
 * give `indices` bit for bit.
 */
int sgsa_indexer_topk_scores(const void *iq, const void *ik, int32_t *indices, float *scores,
                             int B, int T, int H, int DI, int top_k, void *stream);

/*
 * Test support: counters of the tensor-core indexer on the current device since
 * the last reset -- rows that needed the refine pass, rows that restarted with
 * the plain radix select, plain-radix candidate passes, rows whose k-th score
 * was an exact tie (counts[0..3]).  Synchronises the device.  No reference
 * counterpart.
 */
int sgsa_indexer_stats(unsigned long long *counts, int reset);

/*
 * Row-wise top-k of a float32 score matrix [R, S] where row r considers
 * columns [0, valid[r]).  Same selection rule and output format as
 * sgsa_indexer_topk; it exists so that the select can be checked bit-exactly
 * on identical scores (the rule of modelings/modeling_sgsa.py:155-164).
 */
int sgsa_topk_select(const float *scores, const int32_t *valid, int32_t *indices, int R, int S,
                     int top_k, void *stream);

/*
 * Sparse attention over selected rows plus the gate:
 *   o_s = sum_{j in I_t} softmax_j(q_t . k_j * scale) v_j     (fp32)
 *   out = mix * o_s + (1 - mix) * o_delta
 * Replaces modelings/hybrid_dense_delta_topk.py:350-356 and :389-390.
 * o_delta is float32 [B,T,H,D] (NULL: out = o_s).  mix_per_channel selects
 * the [B,T,H,D] (1) or [B,T,H] (0) mix layout; mix may be NULL with o_delta.
 * out has the call's dtype.  idx_heads == H: indices [B,H,T,K]; idx_heads == 1:
 * one index set per token shared by all heads, indices [B,1,T,K].
 */
int sgsa_sparse_attn_mix(const void *q, const void *k, const void *v, const int32_t *indices,
                         const float *o_delta, const void *mix, void *out, int B, int T, int H,
                         int D, int top_k, int idx_heads, float scale, int mix_per_channel,
                         int dtype, void *stream);

/*
 * The indexer of sgsa_indexer_topk (bf16, DI == 64 or 128) that also writes,
 * per query row, the exact selection as a threshold record
 * thresholds[B,H,T][4] = {prefix, mask, cut, 1}: column j <= t is selected iff
 * (key(s_tj) & mask) > prefix, or == prefix and j <= cut, where key() is the
 * order-preserving 32-bit image of the fp32 score.  indices may be NULL.
 * q_tiles (NULL: all) lists the 128-query tiles to compute, heaviest first;
 * rows of other tiles are left untouched (sequence-parallel ranks split them).
 * Replaces the selection of modelings/hybrid_dense_delta_topk.py:344-349.
 */
int sgsa_indexer_thresholds(const void *iq, const void *ik, int32_t *indices,
                            uint32_t *thresholds, const int32_t *q_tiles, int n_tiles, int B,
                            int T, int H, int DI, int top_k, void *stream);

/*
 * Sparse attention + gate over the rows selected by threshold records from
 * sgsa_indexer_thresholds, computed on the tensor cores over the causal
 * prefix (bf16 inputs, D == 128, DI == 64).  Same result as
 * sgsa_sparse_attn_mix on the equivalent index rows.  out is bf16, or float32
 * with out_f32; q_tiles as for sgsa_indexer_thresholds.  idx_heads == 1: iq, ik
 * [B,T,1,DI] and thresholds [B,1,T,4] are shared by all heads (the DeepSeek-style
 * shared indexer of modelings/deepseek_v3_2.py:435-487, an option: it changes the
 * selection semantics from per-head to per-token).
 * norm_scratch (optional, 8*B*H bytes, 4-byte aligned): with it the call first
 * takes max|q|, max|k| per (b,h) and, where their product bounds the scores
 * tightly enough, runs the softmax against that fixed bound (no running maximum).
 * Replaces modelings/hybrid_dense_delta_topk.py:343-356 and :389-390.
 */
int sgsa_sparse_attn_thresholds(const void *q, const void *k, const void *v, const void *iq,
                                const void *ik, const uint32_t *thresholds,
                                const int32_t *q_tiles, int n_tiles, const float *o_delta,
                                const void *mix, void *out, int B, int T, int H, int D, int DI,
                                int idx_heads, float scale, int mix_per_channel, int out_f32,
                                void *norm_scratch, void *stream);

/*
 * Test support for the tensor-core attention (bf16, D 128, DI 64, T <= 4096,
 * per-head indexer): runs sgsa_sparse_attn_thresholds (out float32, no gate, the
 * running-maximum softmax) and also writes the indexer scores it recomputed for
 * its selection, scores[B,H,T,T] (row t: columns j <= t).  They must equal, bit
 * for bit, the scores sgsa_indexer_topk_scores reports for the same iq, ik -- the
 * attention's selection is then exactly the indexer's.  No reference counterpart.
 */
int sgsa_sparse_attn_index_scores(const void *q, const void *k, const void *v, const void *iq,
                                  const void *ik, const uint32_t *thresholds, float *out,
                                  float *scores, int B, int T, int H, void *stream);

/*
 * Retrieval of the sparse-write SGSA block: k_hat, v_hat [B,T,H,D] (dtype) are
 * the softmax(q_t . k_j * scale)-weighted sums of the selected k and v rows.
 * Replaces the aggregation of SparseRetriever._token_only
 * (modelings/modeling_sgsa.py:113-142); with indices from sgsa_indexer_topk on
 * iq = q, ik = k it is the retriever's token path, and (k_hat, v_hat) are the
 * sparse_k / sparse_v of sgsa_chunk_fwd (modelings/modeling_sgsa.py:546-609).
 */
int sgsa_sparse_retrieve(const void *q, const void *k, const void *v, const int32_t *indices,
                         void *k_hat, void *v_hat, int B, int T, int H, int D, int top_k,
                         int idx_heads, float scale, int dtype, void *stream);

/*
 * The gate alone: out = mix * o_s + (1 - mix) * o_delta over `rows` rows of D
 * (o_s, o_delta float32; mix [rows, D] or [rows]; out in dtype).  The mix of
 * modelings/hybrid_dense_delta_topk.py:389-390, used where the two branch
 * outputs are produced on different ranks.
 */
int sgsa_gate_mix(const float *o_s, const float *o_delta, const void *mix, void *out,
                  long long rows, int D, int mix_per_channel, int dtype, void *stream);

/*
 * The composite layer forward: chunked delta stage (no sparse write),
 * indexer top-k, sparse attention and gate, in one stream-ordered call.
 * Replaces the core of SGSAStateLayer.forward (modelings/modeling_sgsa.py:522-619)
 * with the top-k attention and gate of modelings/hybrid_dense_delta_topk.py:343-390.
 * indices may be NULL.  final_state may be NULL.
 * iq, ik are [B,T,idx_heads,DI] with idx_heads == H (per-head selection) or 1
 * (one selection per token shared by all heads).
 * The workspace depends on the path the call takes: bf16 with D == 128 and
 * DI == 64 runs the tensor-core indexer and attention and keeps 16-byte
 * selection records per row; every other case keeps B*idx_heads*T*top_k int32
 * index rows.  The delta stage's per-chunk operands are capped at 1.25 GiB:
 * beyond that the stage runs in groups of (batch, head) pairs that reuse them.
 * The delta stage runs on a non-blocking side stream with a fork and a join
 * event, created on the first call of each host thread on each device and
 * reused by that thread's later calls; the call joins it back into `stream`
 * before the attention (which applies the gate), so the call is stream-ordered
 * as a whole.
 */
size_t sgsa_layer_fwd_workspace_size(int B, int T, int H, int D, int DI, int idx_heads,
                                     int top_k, int dtype);
int sgsa_layer_fwd(const void *q, const void *k, const void *v, const void *beta,
                   const void *gamma, const void *iq, const void *ik, const void *mix,
                   const float *initial_state, void *out, float *final_state, int32_t *indices,
                   int B, int T, int H, int D, int DI, int idx_heads, int top_k,
                   int mix_per_channel, int dtype, void *workspace, size_t workspace_bytes,
                   void *stream);

/*
 * Token-by-token SGSA recurrence (forward): the semantics of
 * naive_recurrent_sgsa (modelings/sgsa_ops/naive.py:39-55).  Replaces the
 * forward of fused_recurrent_sgsa (modelings/sgsa_ops/recurrent.py:138-175,
 * Triton kernel recurrent_fwd_triton.py:19-87).  Same arguments and flags as
 * sgsa_chunk_fwd without the workspace; D in {32, 64, 128}.  With T = 1 it is
 * the decode step of the delta stage (state read and written once).
 */
int sgsa_recurrent_fwd(const void *q, const void *k, const void *v, const void *beta,
                       const void *gamma, const void *sparse_k, const void *sparse_v,
                       const void *alpha, const float *initial_state, void *o,
                       float *final_state, int B, int T, int H, int D, int dtype, int flags,
                       void *stream);

/*
 * Decode cache append: row `pos` of k_cache / v_cache [B,Tc,H,D] and ik_cache
 * [B,Tc,H,DI] from this token's k, v [B,H,D] and ik [B,H,DI] (same dtype as the
 * caches), every batch row in one launch.  Replaces the per-step key/value cache
 * growth of the reference's decode (torch.cat of the past and new rows,
 * modelings/hybrid_dense_delta_topk.py:226-230); here the caches are allocated
 * once at their full length.  All pointers 16-byte aligned; 0 <= pos < Tc.
 */
int sgsa_decode_append(void *k_cache, void *v_cache, void *ik_cache, const void *k,
                       const void *v, const void *ik, int B, int Tc, int H, int D, int DI,
                       int pos, int dtype, void *stream);

/*
 * Decode-time indexer: for each (b, h), the top-k of iq[b,h] . ik_cache[b,j,h]
 * over the cache positions j < n (the current token included), ties to the
 * lowest j, ascending, -1 padded.  iq [B,H,DI]; ik_cache [B,Tc,H,DI] (Tc the
 * allocated cache length, n <= Tc and n <= 55296).  The decode form of the
 * selection of modelings/hybrid_dense_delta_topk.py:343-349, which the
 * reference re-scores against the whole cache at every step (:343-349 with
 * the cache of :226-230).
 */
int sgsa_decode_topk(const void *iq, const void *ik_cache, int32_t *indices, int B, int H,
                     int Tc, int n, int DI, int top_k, int dtype, void *stream);

/*
 * Decode-time sparse attention + gate for one query per (b, h) over its
 * selected cache rows (modelings/hybrid_dense_delta_topk.py:350-356, :389-390).
 * q, o_delta (float32), mix, out: [B,H,D] (mix may be [B,H]); k_cache,
 * v_cache [B,Tc,H,D]; indices [B,H,K] as written by sgsa_decode_topk.
 */
int sgsa_decode_attn_mix(const void *q, const void *k_cache, const void *v_cache,
                         const int32_t *indices, const float *o_delta, const void *mix, void *out,
                         int B, int H, int Tc, int D, int top_k, float scale, int mix_per_channel,
                         int dtype, void *stream);

/* ---- Hybrid model (the layers around the SGSA layer; 16-byte aligned rows) ---- */

/* out = weight * x / sqrt(mean(x^2) + eps) per row of N (N % 8 == 0).
 * Replaces RMSNorm.forward (modelings/hybrid_dense_delta_topk.py:97-106). */
int sgsa_rmsnorm(const void *x, const void *weight, void *out, long long rows, int N, float eps,
                 int dtype, void *stream);

/* out [rows, I] = silu(gate_up[:, :I]) * gate_up[:, I:]  (I % 8 == 0).
 * Replaces the activation of SwiGLUMLP.forward (modelings/hybrid_dense_delta_topk.py:117-119). */
int sgsa_swiglu(const void *gate_up, void *out, long long rows, int I, int dtype, void *stream);

/* qkv [B*T, 3*H*D] -> q, k rotated by RoPE and v, all [B, T, H, D].  cos_sin float32
 * [pos0 + T, D/2, 2] holds (cos, sin) of position t and frequency theta^(-2j/D).
 * Replaces _apply_rope on q and k (modelings/hybrid_dense_delta_topk.py:127-151, :210-211). */
int sgsa_rope_qkv(const void *qkv, const float *cos_sin, void *q, void *k, void *v, int B, int T,
                  int H, int D, int pos0, int dtype, void *stream);

/* Epilogue of an SGSA layer's fused input projection proj [rows, ld] whose column
 * blocks are q | k | v | mix (H*D each) | iq | ik (H*DI each) | beta | gamma (H each):
 * q, k l2-normalised per head, mix = sigmoid, beta = max(sigmoid, 1e-4), gamma =
 * sigmoid (SGSAStateLayer, modelings/modeling_sgsa.py:538-539; mix gate of
 * modelings/hybrid_dense_delta_topk.py:389).  Outputs [rows, H, *]. */
int sgsa_layer_proj(const void *proj, int ld, void *q, void *k, void *v, void *mix, void *iq,
                    void *ik, void *beta, void *gamma, long long rows, int H, int D, int DI,
                    int dtype, void *stream);

/* out [rows, N] = table[ids]; ids outside [0, vocab) give zero rows.
 * Replaces embed_tokens (modelings/hybrid_dense_delta_topk.py:447). */
int sgsa_embed(const int64_t *ids, const void *table, void *out, long long rows, int N, int vocab,
               int dtype, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SGSA_B200_H_ */
