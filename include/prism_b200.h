/*
 * prism_b200 — C ABI of the B200 (sm_100a) ReAttention recall scorer.
 *
 * The scorer is the hot path of Prism-Test's ReAttention method
 * (RUSH-Intelligence/Prism-Test, eval_harness/): inverse-RoPE un-rotation of the
 * cached keys, position-agnostic q·K^T per GQA head, exact per-query top-k,
 * sorted like torch.topk. Every entry point takes plain device pointers, sizes
 * and a cudaStream_t passed as void*; nothing allocates except where noted, no
 * entry point synchronises the stream unless its comment says so, and results
 * are written asynchronously on the given stream.
 *
 * Return value of every int function: PRISM_OK (0) or a negative PRISM_E_*
 * code; prism_last_error() returns a message for the calling thread's last
 * failure.
 */
#ifndef PRISM_B200_H_
#define PRISM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define PRISM_API __attribute__((visibility("default")))
#else
#define PRISM_API
#endif

#define PRISM_ABI_VERSION 1

/* element types of q and k */
#define PRISM_DTYPE_BF16 0
#define PRISM_DTYPE_FP16 1

/* selection modes */
#define PRISM_MODE_EXACT 0    /* exact top-k of the fp32 scores (torch.topk semantics) */
#define PRISM_MODE_BLOCKMAX 1 /* per-128-key-block maxima, top-1 / top-4 (Triton kernel semantics) */
#define PRISM_MODE_EXACT_STREAM 2 /* exact, without a score matrix (prefill chunks; see below) */

/* status codes */
#define PRISM_OK 0
#define PRISM_E_INVALID (-1)       /* bad argument (shape, stride, alignment, range) */
#define PRISM_E_UNSUPPORTED (-2)   /* valid request outside what the kernels implement */
#define PRISM_E_WORKSPACE (-3)     /* workspace missing or too small */
#define PRISM_E_CUDA (-4)          /* a CUDA runtime call failed */
#define PRISM_E_DEVICE_STATUS (-5) /* a kernel reported a device-side error */

/*
 * Fused un-rotate + score + top-k.
 *
 * Replaces eval_harness/kernels/einsum_topk.py:164-225 (einsum_topk_func,
 * re-exported by eval_harness/kernels/__init__.py:12-15 and called from
 * eval_harness/attention_methods/reattention.py:483) and, with inv_freq given,
 * also ReAttentionMethod._unrotate_keys (reattention.py:743-793) in front of it.
 * With mode PRISM_MODE_EXACT the result equals ReAttentionMethod._dense_topk
 * (reattention.py:486-498): scores = einsum("bhqd,bhmd->bhqm", q, repeat_kv(k))
 * in fp32, then topk(topk, dim=-1).
 *
 *   q          [B, Hq, Sq, D] elements of `dtype`; q_strides[4] in elements,
 *              q_strides[3] must be 1.
 *   k          [B, Hkv, Sk, D] elements of `dtype`; k_strides[3] == 1 and
 *              k_strides[2] == D (key rows contiguous), base and k_strides[0..1]
 *              16-byte aligned. Hq % Hkv == 0; q head h reads kv head h / (Hq/Hkv).
 *   D          must be 128.
 *   inv_freq   [D/2] fp32 device pointer or NULL. When given, k holds RoPE-rotated
 *              keys (HF rotate_half layout) of absolute positions pos_offset + j
 *              and is un-rotated with angle fp32(position) * inv_freq[i].
 *              pos_offset + Sk must be below 2^22.
 *   causal_offset  >= 0: key j is visible to query row s iff j <= causal_offset + s
 *              (invisible keys score -inf); < 0: no mask.
 *   topk       1 <= topk <= Sk, and topk <= 16384 (exact mode);
 *              topk in {1, 4} with Sq % 128 == 0 and Sk % 128 == 0 (blockmax mode).
 *   mode       PRISM_MODE_EXACT, PRISM_MODE_BLOCKMAX or PRISM_MODE_EXACT_STREAM.
 *              The streaming path gives the exact-mode result without writing
 *              the B*Hq*Sq x Sk score matrix: per-row thresholds from a strided
 *              key sample, the keys at or above them, a selection per row, and
 *              an exact recompute of any row the threshold missed. Exact mode
 *              takes it by itself when Sq >= 128, Sk >= 8192, topk <= 4096 and
 *              the score matrix would be 2 GiB or more; it needs at least 128
 *              query rows per KV head, 16-byte aligned query rows and
 *              topk <= 4096 (PRISM_E_UNSUPPORTED otherwise), and, for RoPE'd
 *              keys, prism_einsum_topk_rope_workspace_size() bytes of workspace.
 *   index_base added to every output index (global index of key 0 of this shard).
 *   out_idx    [B, Hq, Sq, topk] int32, contiguous. Sorted by descending score,
 *              ties by ascending index.
 *   out_scores [B, Hq, Sq, topk] fp32, contiguous, or NULL.
 *   workspace  device memory of at least prism_einsum_topk_workspace_size() bytes.
 *              RoPE'd keys with at least 128 query rows per KV head (prefill
 *              chunks) are scored on the tensor cores from un-rotated copies of
 *              the keys kept in the workspace: give
 *              prism_einsum_topk_rope_workspace_size() bytes (the score-matrix
 *              path falls back to the CUDA-core scorers with less; the streaming
 *              path returns PRISM_E_WORKSPACE).
 *   stream     cudaStream_t.
 */
PRISM_API int prism_einsum_topk(const void* q, const void* k, const float* inv_freq, int dtype,
                      int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                      const int64_t* q_strides, const int64_t* k_strides, int64_t pos_offset,
                      int64_t causal_offset, int32_t topk, int32_t mode, int64_t index_base,
                      int32_t* out_idx, float* out_scores, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Workspace bytes prism_einsum_topk needs for this shape (0 on invalid input). */
PRISM_API size_t prism_einsum_topk_workspace_size(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk,
                                        int32_t topk, int32_t mode);

/* recall weightings of prism_einsum_topk_weighted (the reference's recall_type) */
#define PRISM_RECALL_QK 0   /* "qk": unweighted, the same as prism_einsum_topk */
#define PRISM_RECALL_QKV 1  /* "qkv": key j scaled by ||v_j||_1 */
#define PRISM_RECALL_QKV2 2 /* "qkv2": key j scaled by ||v_j||_2 */

/*
 * prism_einsum_topk with the value-norm recall weighting: the score of key j
 * is multiplied by the L1 (PRISM_RECALL_QKV) or L2 (PRISM_RECALL_QKV2) norm of
 * value row j of the same KV head, computed in fp32 and rounded to `dtype`.
 *
 * Replaces ReAttentionMethod._apply_recall_weight
 * (eval_harness/attention_methods/reattention.py:822-842, applied at :358 and
 * in reattention_exact.py:547) — raw_k * values.norm(p, dim=-1, keepdim=True),
 * a bf16/fp16 norm — followed by the selection prism_einsum_topk replaces.
 * Scaling the raw key by a scalar and scaling its score by it are the same
 * product; the weighting runs after scoring, on the score matrix.
 *
 *   v          [B, Hkv, Sk, Dv] elements of `dtype`: the value rows of the
 *              same keys (the middle slice k covers). v_strides[3] == 1;
 *              base and v_strides[0..2] 16-byte aligned; Dv % 8 == 0,
 *              8 <= Dv <= 1024.
 *   recall_weight  PRISM_RECALL_QK, PRISM_RECALL_QKV or PRISM_RECALL_QKV2
 *              (with PRISM_RECALL_QK, v and v_strides are ignored).
 *   workspace  at least prism_einsum_topk_weighted_workspace_size() bytes
 *              (prism_einsum_topk's plus B * Hkv * Sk fp32 weights).
 * Every other argument and the outputs are those of prism_einsum_topk;
 * out_scores holds the weighted scores. A masked (-inf) score stays -inf.
 */
PRISM_API size_t prism_einsum_topk_weighted_workspace_size(int64_t B, int64_t Hq, int64_t Hkv,
                                                           int64_t Sq, int64_t Sk, int32_t topk,
                                                           int32_t mode, int32_t recall_weight);
/*
 * Workspace bytes for a call with RoPE'd keys (inv_freq != NULL), to
 * prism_einsum_topk (recall_weight PRISM_RECALL_QK) or prism_einsum_topk_weighted:
 * the size above plus, when the call has at least 128 query rows per KV head,
 * B * Hkv * Sk * 512 bytes for the keys un-rotated once into two 16-bit planes
 * (hi + lo within 2^-17 of the fp32 un-rotated key) that the tcgen05 scorer reads.
 */
PRISM_API size_t prism_einsum_topk_rope_workspace_size(int64_t B, int64_t Hq, int64_t Hkv,
                                                       int64_t Sq, int64_t Sk, int32_t topk,
                                                       int32_t mode, int32_t recall_weight);
PRISM_API int prism_einsum_topk_weighted(const void* q, const void* k, const void* v,
                                         const float* inv_freq, int dtype, int64_t B, int64_t Hq,
                                         int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                                         int64_t Dv, const int64_t* q_strides,
                                         const int64_t* k_strides, const int64_t* v_strides,
                                         int64_t pos_offset, int64_t causal_offset,
                                         int32_t recall_weight, int32_t topk, int32_t mode,
                                         int64_t index_base, int32_t* out_idx, float* out_scores,
                                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * Attention over the selected view: the step after the recall selection in the
 * exact method. Replaces ReAttentionExactMethod._chunk_attention's gather of
 * the [global | recalled | local] view from the raw cache, its RoPE of keys and
 * queries at their positions (eval_harness/attention_methods/
 * reattention_exact.py:453-508) and the eager path of _attend (:650-661):
 * softmax(q k^T * scale) v in fp32, keys at absolute positions above a query's
 * masked, a query that sees no key giving zeros (the reference's nan_to_num).
 *
 *   q          [B, Hq, Sq, D] raw (pre-RoPE) queries of `dtype`, q_strides in
 *              elements, q_strides[3] == 1, other strides multiples of 4.
 *   k, v       [B, Hkv, S, D] raw cache; rows contiguous (strides[2] == D,
 *              strides[3] == 1), base and strides 8-byte aligned.
 *   key_pos    int64 [nsel] device array: absolute positions of the view (its
 *              order is the view's order). A position outside [0, S) is skipped
 *              and reported in the status word (prism_read_status).
 *   q_pos      int64 [Sq] device array: absolute positions of the query rows.
 *   inv_freq   [D/2] fp32 or NULL (no rotation).
 *   pe_original  1: RoPE at the absolute positions; 0: keys at 0 .. nsel-1 and
 *              query row i at nsel - Sq + i (the contiguous re-rotation).
 *   D          must be 128.
 *   out        [B, Hq, Sq, D] contiguous, `dtype`.
 *   workspace  prism_sparse_attention_workspace_size(B, Hq, Sq, nsel) bytes
 *              (256-aligned): the status block, the per-split partial softmax
 *              states and a table of the view's RoPE angles.
 */
PRISM_API int prism_sparse_attention(const void* q, const void* k, const void* v,
                                     const int64_t* key_pos, int64_t nsel, const int64_t* q_pos,
                                     const float* inv_freq, int32_t pe_original, float scale,
                                     int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                                     int64_t S, int64_t D, const int64_t* q_strides,
                                     const int64_t* k_strides, const int64_t* v_strides, void* out,
                                     void* workspace, size_t workspace_bytes, void* stream);
PRISM_API size_t prism_sparse_attention_workspace_size(int64_t B, int64_t Hq, int64_t Sq,
                                                       int64_t nsel);

/*
 * Exact top-k over candidate lists: for each of `rows` rows, picks the topk
 * largest of n (score, index) pairs laid out with row stride ld (ld % 4 == 0,
 * 16-byte aligned rows) and writes them sorted like prism_einsum_topk.
 * This is the device merge of the sequence-sharded path: the candidates are the
 * per-rank top-k lists after an all-gather, indices already global. It has no
 * single reference counterpart; it reproduces torch.topk over the union of the
 * shards (reattention.py:497) and the sorted merge of
 * eval_harness/kernels/bitonic_merge_wrapper.py:36-52 for any width.
 * `workspace` holds prism_topk_merge_workspace_size(rows, n) bytes of device
 * memory (16-byte aligned) for the per-row candidate buffers.
 */
PRISM_API int prism_topk_merge(const float* cand_scores, const int32_t* cand_idx, int64_t rows,
                               int64_t n, int64_t ld, int32_t topk, int32_t* out_idx,
                               float* out_scores, void* workspace, size_t workspace_bytes,
                               void* stream);

/* Workspace bytes prism_topk_merge needs (0 on invalid input). */
PRISM_API size_t prism_topk_merge_workspace_size(int64_t rows, int64_t n);

/*
 * Top-k of the union of `nruns` sorted runs, the merge of the sequence-sharded
 * path when every rank contributes its own prism_einsum_topk result.
 *   runs     int32 [nruns, 2, rows, run_len]: per run a plane of fp32 score bits
 *            and a plane of int32 global indices, each row sorted by descending
 *            score then ascending index, as prism_einsum_topk returns them (an
 *            all-gather of the ranks' [out_scores; out_idx] buffers lays them
 *            out so). Indices must be distinct across runs.
 *   1 <= nruns <= 16, 1 <= topk <= run_len, topk <= 16384.
 *   out_idx / out_scores [rows, topk] as prism_topk_merge.
 * No workspace. Replaces the same reference merge as prism_topk_merge
 * (bitonic_merge_wrapper.py:36-52, torch.topk over the union, reattention.py:497)
 * for inputs that are already sorted runs.
 */
PRISM_API int prism_topk_merge_runs(const int32_t* runs, int32_t nruns, int64_t rows,
                                    int64_t run_len, int32_t topk, int32_t* out_idx,
                                    float* out_scores, void* stream);

/*
 * Peer exchange of the sequence-sharded path over NVLink. It has no counterpart
 * in the reference (which is single-GPU); with prism_peer_merge it replaces the
 * all-gather of the ranks' local top-k runs plus prism_topk_merge_runs, i.e. the
 * torch.topk over the union (reattention.py:497) of a sequence split over GPUs.
 * One process per GPU. Every rank owns one exchange buffer of
 * prism_peer_buffer_bytes(rows, topk) bytes: a PRISM_PEER_HEADER_BYTES header
 * (its first int32 is the status word prism_read_status reads), then the rank's
 * run, int32 [2, rows, topk] (fp32 score bits, global indices) at offset
 * PRISM_PEER_HEADER_BYTES, laid out as prism_einsum_topk's out_scores / out_idx.
 *   prism_peer_alloc   cudaMalloc + zero + an IPC handle (PRISM_IPC_HANDLE_BYTES)
 *                      to hand to the other ranks (any host transport).
 *   prism_peer_open    maps another rank's buffer from its handle;
 *                      prism_peer_close unmaps it, prism_peer_free frees one's own.
 * A step on every rank, on one stream, in the same order on all ranks:
 *   1. write the local top-k into the own buffer's run;
 *   2. prism_peer_publish: advances the rank's step counter and marks its run
 *      ready in every rank's header (one warp, release stores over NVLink);
 *   3. prism_peer_merge: waits until every rank's run of the step is ready, merges
 *      the runs straight from the peers' memory into out_idx / out_scores
 *      [rows, topk] (same result as prism_topk_merge_runs), then tells every rank
 *      its run was read; with wait_acks != 0 its last CTA also waits until every
 *      rank has read this rank's run, so step 1 of the next step may overwrite it.
 *   prism_peer_wait_acks: on the device, waits until every rank has read this
 *      rank's run of the current step — step 1's guard when the previous merge ran
 *      with wait_acks = 0 (as prism_sharded_topk's does).
 * bufs is a HOST array of the world buffers as mapped in this process (the own
 * one at bufs[rank]), each 256-byte aligned; world <= PRISM_PEER_MAX_RANKS.
 * Steps are counted on the device, so the calls can be captured in a CUDA graph.
 * Every wait gives up after timeout_ns (<= 0: 2 s) and sets status 1; the
 * exchange must then be rebuilt (new buffers on every rank).
 */
#define PRISM_IPC_HANDLE_BYTES 64
#define PRISM_PEER_HEADER_BYTES 512
#define PRISM_PEER_MAX_RANKS 16
PRISM_API size_t prism_peer_buffer_bytes(int64_t rows, int32_t topk);
PRISM_API int prism_peer_alloc(size_t bytes, void** buf, void* ipc_handle);
PRISM_API int prism_peer_open(const void* ipc_handle, void** buf);
PRISM_API int prism_peer_close(void* buf);
PRISM_API int prism_peer_free(void* buf);
PRISM_API int prism_peer_publish(void* const* bufs, int32_t world, int32_t rank, void* stream);
PRISM_API int prism_peer_merge(void* const* bufs, int32_t world, int32_t rank, int64_t rows,
                               int32_t topk, int32_t wait_acks, int64_t timeout_ns,
                               int32_t* out_idx, float* out_scores, void* stream);
PRISM_API int prism_peer_wait_acks(void* const* bufs, int32_t world, int32_t rank, int64_t timeout_ns,
                                   void* stream);
/*
 * One step of the sequence-sharded recall as a single call — the composition the
 * reference's single-GPU _dense_topk (eval_harness/attention_methods/
 * reattention.py:486-498) becomes when the key cache is split over the GPUs of
 * one node: this rank's exact local top-k of its key slice (prism_einsum_topk
 * with pos_offset = index_base = shard_start, written into its exchange run),
 * then prism_peer_publish, then prism_peer_merge into out_idx / out_scores
 * ([B, Hq, Sq, topk] int32 global indices / fp32 scores, the same on every rank).
 *   k_shard     this rank's keys [B, Hkv, Sk_shard, 128], first key at absolute
 *               position / global index shard_start; Sk_shard >= topk
 *   exchange_bufs  every rank's exchange buffer of
 *               prism_peer_buffer_bytes(B * Hq * Sq, topk) bytes, as mapped here
 *               (prism_peer_alloc on each rank, the IPC handles exchanged by the
 *               caller, prism_peer_open of the other ranks' handles)
 *   wait_acks   1: before the call rewrites this rank's run, it waits (on the
 *               device, while its scorer runs) until every rank has acknowledged
 *               reading the run of the previous step; the merge then only sends
 *               this rank's acknowledgements. 0: the caller guarantees that no rank
 *               rewrites its run before all ranks have read it.
 *   timeout_ns  bound of every device-side wait (<= 0: 2 s)
 *   workspace   prism_einsum_topk_workspace_size(B, Hq, Sq, Sk_shard, topk,
 *               PRISM_MODE_EXACT) bytes, 256-byte aligned (with inv_freq:
 *               prism_einsum_topk_rope_workspace_size(B, Hq, Hkv, Sq, Sk_shard, topk,
 *               PRISM_MODE_EXACT, PRISM_RECALL_QK))
 * Every rank makes the call for the same step, with the same shapes, in the same
 * order relative to its other exchange calls.
 */
PRISM_API int prism_sharded_topk(const void* q, const void* k_shard, const float* inv_freq, int dtype,
                                 int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk_shard,
                                 int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                                 int64_t shard_start, int32_t topk, void* const* exchange_bufs,
                                 int32_t world, int32_t rank, int32_t wait_acks, int64_t timeout_ns,
                                 int32_t* out_idx, float* out_scores, void* workspace,
                                 size_t workspace_bytes, void* stream);

/*
 * Measurement of this rank's peer merges (device time, %globaltimer): out[0] the
 * number of merges since the last reset, out[1..3] the nanoseconds they spent in
 * total waiting for the ranks' runs to be published (from the merge's start),
 * merging, and waiting for the other ranks' acknowledgements. Synchronises
 * `stream`; reset != 0 zeroes the sums afterwards. No reference counterpart.
 */
PRISM_API int prism_peer_read_timings(void* own_buf, uint64_t* out4, int32_t reset, void* stream);

/*
 * prism_topk_merge without a workspace, for callers that cannot allocate device
 * memory (no cudaMalloc / cudaFree / allocating library call anywhere in the
 * call). It has no counterpart in the reference. Same arguments, kernel and
 * results as prism_topk_merge; the per-row candidate buffers live in one static
 * device array of PRISM_NOALLOC_SCRATCH_BYTES per device, so the request must
 * satisfy rows * min(n, 16384) * 8 <= PRISM_NOALLOC_SCRATCH_BYTES (e.g. 64 rows
 * of any length); larger requests return PRISM_E_WORKSPACE. Only requests of
 * fewer than 64 rows write the scratch (one 4-CTA cluster per row, exact path);
 * 64 rows or more run one CTA per row with its candidates in shared memory, but
 * the same size rule applies to them.
 *   - The first call on a device, made with that device current, looks the
 *     scratch address up (cudaGetSymbolAddress) and caches it; make that first
 *     call before any stream capture starts on the device. The cached address
 *     does not survive cudaDeviceReset of that device: do not call this entry
 *     point on a device after resetting it in the same process.
 *   - Nothing in the scratch needs to start at zero.
 *   - All calls on one device share the scratch: calls whose executions overlap
 *     (different streams, concurrent host threads) race and give wrong results.
 *     Calls on one stream are serialised and safe.
 *   - Not counted by the measurement aids below.
 */
#define PRISM_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20) /* 8 MiB */
PRISM_API int prism_topk_merge_noalloc(const float* cand_scores, const int32_t* cand_idx,
                                       int64_t rows, int64_t n, int64_t ld, int32_t topk,
                                       int32_t* out_idx, float* out_scores, void* stream);

/*
 * Post-selection of the recall path, on the device: the sorted, deduplicated
 * union of the selected middle positions, each widened into a span. Replaces
 * ReAttentionMethod._global_unique + _expand_spans
 * (eval_harness/attention_methods/reattention.py:844-874; span_mode
 * PRISM_SPAN_CENTERED) and the span expansion of
 * eval_harness/attention_methods/reattention_exact.py:571-585 (PRISM_SPAN_FLOOR).
 *   topk_idx     int32 [n_idx] middle-relative indices (e.g. the flattened
 *                prism_einsum_topk output); entries outside [0, n_mid) are ignored.
 *   recall_clip  < 0: keep every selected position; otherwise keep the recall_clip
 *                most frequently selected (ties toward lower positions; torch.topk
 *                leaves them unspecified); at most 16384.
 *   span_size    >= 0. CENTERED: offsets [-(s/2), (s+1)/2), s = 0 keeps the position.
 *                FLOOR: offsets [floor(-s/2), (s+1)/2) (one more before the position
 *                for odd s), s = 0 keeps nothing.
 *   out_pos      int32 [n_mid]: the result in ascending order, clamped to [0, n_mid).
 *   out_count    int32 device scalar: number of positions written.
 *   workspace    prism_post_select_workspace_size(n_mid, recall_clip) bytes, 256-byte aligned.
 */
#define PRISM_SPAN_CENTERED 0
#define PRISM_SPAN_FLOOR 1
PRISM_API int prism_post_select(const int32_t* topk_idx, int64_t n_idx, int64_t n_mid,
                                int32_t recall_clip, int32_t span_size, int32_t span_mode,
                                int32_t* out_pos, int32_t* out_count, void* workspace,
                                size_t workspace_bytes, void* stream);

/* Workspace bytes prism_post_select needs (0 on invalid input). */
PRISM_API size_t prism_post_select_workspace_size(int64_t n_mid, int32_t recall_clip);

/*
 * Reads the device status word kept at the start of `workspace` (synchronises
 * `stream`), stores it in *status_out and resets it to 0. A non-zero value means
 * a kernel gave up on a bounded wait (1), rejected an access (2) or ran out of
 * candidate space (3) since the previous read.
 */
PRISM_API int prism_read_status(void* workspace, int* status_out, void* stream);

/*
 * Measurement aids (no reference counterpart; used by bench.py). While
 * profiling is on, every kernel launch of the library on any stream is
 * bracketed by a pair of CUDA events taken from a pool of `capacity` pairs
 * (launches beyond the pool are counted but not timed). prism_profile_read
 * synchronises those events and returns, for one kernel kind, the number of
 * timed launches and their summed device duration. prism_launch_count counts
 * every kernel launch of the library since it was loaded. Process-global;
 * call from one host thread.
 */
#define PRISM_KERNEL_SCORE 0  /* decode scorer (un-rotate + q·K^T) */
#define PRISM_KERNEL_SELECT 1 /* exact top-k selection of a score matrix */
#define PRISM_KERNEL_MERGE 2  /* top-k merge of gathered shard candidates */
#define PRISM_KERNEL_WEIGHT 3 /* value-row norms of the weighted recall */
#define PRISM_KERNEL_SCALE 4  /* weighting of the score matrix by those norms */
#define PRISM_KERNEL_THRESHOLD 5 /* sampled per-row thresholds of the streaming prefill path */
#define PRISM_KERNEL_ATTN 6   /* attention over the selected view */
#define PRISM_KERNEL_UNROTATE 7 /* RoPE'd keys un-rotated into planes for the tensor-core scorer */
PRISM_API int prism_profile_start(int32_t capacity);
PRISM_API int prism_profile_stop(void);
PRISM_API int prism_profile_read(int32_t kernel, int64_t* launches, double* total_ms);
PRISM_API int64_t prism_launch_count(void);

/* Message describing the calling thread's most recent failure ("" if none). */
PRISM_API const char* prism_last_error(void);

/* PRISM_ABI_VERSION of the loaded library. */
PRISM_API int prism_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PRISM_B200_H_ */
