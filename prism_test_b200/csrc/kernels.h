// Internal launch interface shared by the .cu files of the extension.
// (The public C-ABI lives in include/prism_b200.h.)
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace prism {

enum DType : int { kBF16 = 0, kFP16 = 1 };

// --- decode scorer (CUDA cores; few query rows per KV head) ----------------
struct DecodeArgs {
  const void* q;            // [B, Hq, Sq, 128], innermost stride 1
  const void* k;            // [B, Hkv, Sk, 128], rows contiguous (stride(-2) == 128)
  const float* inv_freq;    // [64] or nullptr (keys already un-rotated)
  int B, Hq, Hkv, G;        // G = Hq / Hkv
  int Sq;                   // full query length (row indexing)
  int s0, sq_n;             // this launch scores query rows [s0, s0 + sq_n)
  int Sk;
  int64_t q_sb, q_sh, q_ss; // q strides in elements
  int64_t k_sb, k_sh;       // k strides in elements
  int64_t pos_offset;       // absolute position of key 0 (RoPE)
  int causal;               // 1: key j visible to query s iff j <= causal_offset + s
  int64_t causal_offset;
  float* scores;            // [B*Hq*Sq, ld] fp32 workspace
  int64_t ld;
  int ntiles;
  int* status;
  unsigned int* work;       // nullptr, or B work counters, zero at launch (dynamic slice claims)
  void* planes;             // RoPE'd keys on the tcgen05 scorer: the un-rotated keys as 16-bit
                            // hi / lo planes (rope_planes_bytes), or nullptr
};

// rows (Hq * sq_n) resident per CTA must not exceed this
constexpr int kDecodeMaxRows = 128;

cudaError_t launch_decode_scores(const DecodeArgs& a, int dtype, int num_sms,
                                 cudaStream_t stream);

// Head-pair tensor-core path: bf16, <= 4 query rows per KV head, Hkv in {2, 4, 8}.
bool decode_hp_supported(const DecodeArgs& a, int dtype);
cudaError_t launch_decode_scores_hp(const DecodeArgs& a, int num_sms, cudaStream_t stream);

// Register tensor-core (mma.sync TF32) path: <= 16 query rows per KV head,
// Hkv in {2, 4, 8}.
bool decode_mma_supported(const DecodeArgs& a);
cudaError_t launch_decode_scores_mma(const DecodeArgs& a, int dtype, int num_sms,
                                     cudaStream_t stream);

// Tensor-core path with the query rows as the MMA's M dimension: up to
// 256 / Hkv rows per KV head, Hkv in {2, 4, 8}.
bool decode_wide_supported(const DecodeArgs& a);
cudaError_t launch_decode_scores_wide(const DecodeArgs& a, int dtype, int num_sms,
                                      cudaStream_t stream);
// The same scorer for the streaming top-k (no score matrix): a threshold sample
// (the scores of every kWideSampleStride-th stage of 128 / Hkv positions, into
// a.scores as [rows, a.ld] with a.ld >= wide_sample_cols), and the candidate pass
// (keys at or above thr[row] appended to the rows' lists).
constexpr int kWideSampleStride = 16;
int64_t wide_sample_cols(int Hkv, int64_t Sk);
cudaError_t launch_wide_sample(const DecodeArgs& a, int dtype, int num_sms, cudaStream_t stream);
cudaError_t launch_wide_candidates(const DecodeArgs& a, int dtype, const float* thr, uint32_t* counts,
                                   uint64_t* cand, int64_t cap, int num_sms, cudaStream_t stream);
// The same three modes on the tensor cores (score_wide_tc.cu): Hkv in {2, 4}, at
// most 64 query rows per KV head, 16-byte aligned score rows; same outputs.
bool wide_tc_supported(const DecodeArgs& a);
cudaError_t launch_wide_tc_scores(const DecodeArgs& a, int dtype, int num_sms, cudaStream_t stream);
cudaError_t launch_wide_tc_sample(const DecodeArgs& a, int dtype, int num_sms, cudaStream_t stream);
cudaError_t launch_wide_tc_candidates(const DecodeArgs& a, int dtype, const float* thr, uint32_t* counts,
                                      uint64_t* cand, int64_t cap, uint64_t* seg, uint32_t* segn,
                                      int num_sms, cudaStream_t stream);

// CUDA-core path for <= 4 query rows per KV head, Hkv in {1, 2, 4, 8, 16}.
bool decode_g4_supported(const DecodeArgs& a);
cudaError_t launch_decode_scores_g4(const DecodeArgs& a, int dtype, int num_sms,
                                    cudaStream_t stream);

// Tensor-core (tcgen05) scorer for raw keys (inv_freq == nullptr) and at least
// kPrefillMinRows query rows per KV head; q rows 16-byte aligned.
constexpr int kPrefillMinRows = 128;
// RoPE'd keys take it through un-rotated planes (a.planes, written by
// launch_unrotate_planes): [nb, Hkv, 2, Sk, 128] of the keys' dtype, hi then lo,
// hi + lo = the fp32 un-rotated key within 2^-17 relative; nb = B, or 1 when the
// keys are shared across the batch (k_sb == 0).
bool prefill_tc_supported(const DecodeArgs& a);
cudaError_t launch_prefill_scores_tc(const DecodeArgs& a, int dtype, cudaStream_t stream);
size_t rope_planes_bytes(int64_t B, int64_t Hkv, int64_t Sk);
cudaError_t launch_unrotate_planes(const DecodeArgs& a, int dtype, int num_sms, cudaStream_t stream);

// Streaming prefill top-k (no score matrix): per-row thresholds from a strided
// key sample (every kSampleStride-th key), then the candidates >= threshold,
// then an exact selection per row with an exact recompute of rows whose
// candidates fell outside [min(k, visible keys), cap].
constexpr int kSampleStride = 16;
cudaError_t launch_prefill_threshold_tc(const DecodeArgs& a, int dtype, int topk, float* thr,
                                        cudaStream_t stream);
cudaError_t launch_prefill_candidates_tc(const DecodeArgs& a, int dtype, const float* thr,
                                         uint32_t* counts, uint64_t* cand, int64_t cap,
                                         cudaStream_t stream);
int64_t prefill_cand_cap(int64_t Sk, int topk);
// nfall: rows the exact fallback can take per call (< 0: the prefill default, 64)
size_t prefill_stream_workspace_bytes(int64_t rows, int64_t Sk, int topk, int64_t nfall = -1);
// The streaming path in three phases on one workspace `ws` of
// prefill_stream_workspace_bytes(rows, Sk, topk) bytes (256-aligned):
// thresholds (one tcgen05 launch), candidates (one tcgen05 launch), selection
// (the per-row select and the exact fallback: four launches).
cudaError_t prefill_stream_threshold(const DecodeArgs& a, int dtype, int topk, void* ws,
                                     cudaStream_t stream);
cudaError_t prefill_stream_candidates(const DecodeArgs& a, int dtype, int topk, void* ws,
                                      cudaStream_t stream);
// seg / segn: candidate segments (the queries-as-M tensor-core pass) appended to the
// rows' lists first.
cudaError_t prefill_stream_select(const DecodeArgs& a, int dtype, int topk, int64_t index_base,
                                  int32_t* out_idx, float* out_scores, void* ws,
                                  cudaStream_t stream, int64_t nfall = -1, const uint64_t* seg = nullptr,
                                  const uint32_t* segn = nullptr);
// The streaming workspace's thresholds, candidate counts [rows, 2], candidate
// lists [rows, cap] and fallback flags (two ints), for other candidate producers.
struct StreamBuffers {
  float* thr;
  uint32_t* counts;
  uint64_t* cand;
  int64_t cap;
  int* flags;
};
StreamBuffers stream_buffers(int64_t rows, int64_t Sk, int topk, void* ws, int64_t nfall);

// Streaming top-k on the queries-as-M scorer (many query rows per KV head, RoPE'd
// keys allowed): a threshold sample, per-row thresholds, the candidate pass and
// the streaming selection with its exact fallback. `ws` is
// wide_stream_workspace_bytes(rows, Sk, topk) bytes, 256-byte aligned.
size_t wide_stream_workspace_bytes(int64_t rows, int64_t Sk, int topk);
// Candidate segments of the tensor-core candidate pass: CTA c's epilogue group g
// appends row r's candidates to segment (r, 2 c + g) of kWideSegCap entries without
// atomics (beyond that, to the row's list through its counter); the streaming
// selection appends the segments to the rows' lists before it reads them.
constexpr int kWideMaxSegs = 512;   // 2 per CTA of a batch row
constexpr int kWideSegCap = 64;
struct WideStreamPtrs {
  StreamBuffers sb;
  float* S;      // the threshold sample [rows, ld_s]
  int64_t ld_s;
  uint64_t* seg;   // [rows, kWideMaxSegs, kWideSegCap]
  uint32_t* segn;  // [rows, kWideMaxSegs] entries in each segment (zero before the pass)
};
WideStreamPtrs wide_stream_ptrs(const DecodeArgs& a, int topk, void* ws);
// phases: the sample and the thresholds (also clears the counts and flags), the
// candidate pass; then prefill_stream_select on the same workspace
cudaError_t wide_stream_threshold(const DecodeArgs& a, int dtype, int topk, void* ws, int num_sms,
                                  cudaStream_t stream);
cudaError_t wide_stream_candidates(const DecodeArgs& a, int dtype, int topk, void* ws, int num_sms,
                                   cudaStream_t stream);
// the streaming selection on the wide path's workspace (segments included; every row
// can take the exact fallback)
cudaError_t wide_stream_select(const DecodeArgs& a, int dtype, int topk, int64_t index_base, int32_t* out_idx,
                               float* out_scores, void* ws, cudaStream_t stream);

// --- exact per-row top-k selection over a score matrix ----------------------
struct SelectArgs {
  const float* scores;      // [rows, ld]
  const int32_t* idx_in;    // [rows, ld] or nullptr (index = column)
  int64_t rows;
  int64_t n;                // valid columns per row
  int64_t ld;
  int k;                    // 1 <= k <= min(n, kSelectMaxK)
  int64_t index_base;       // added to column indices (ignored when idx_in given)
  int32_t* out_idx;         // [rows, k]
  float* out_scores;        // [rows, k] or nullptr
  int* status;
  const int* rows_dyn;      // nullptr, or a device count: rows >= *rows_dyn are skipped
};
constexpr int kSelectMaxK = 16384;

// Candidate buffer the cluster select kernel needs (cand_ws); with cand_ws ==
// nullptr the general one-block-per-row kernel runs instead.
int64_t select_cand_cap(int64_t n);
size_t select_workspace_bytes(int64_t rows, int64_t n);
cudaError_t launch_select_topk(const SelectArgs& a, void* cand_ws, cudaStream_t stream);

// Top-k of the union of nruns sorted runs, run r an int32 [2, rows, run_len]
// buffer (fp32 score bits, int32 indices), run_len >= k, k <= 16384. The first
// form takes the runs back to back ([nruns, 2, rows, run_len]).
cudaError_t launch_merge_runs(const int32_t* runs, int nruns, int64_t rows, int64_t run_len, int k,
                              int32_t* out_idx, float* out_scores, cudaStream_t stream);

// --- peer exchange of the sequence-sharded path (NVLink, peer-mapped memory) ----
// Every rank owns one exchange buffer: this header, then its run [2, rows, topk]
// at kPeerHeaderBytes. Every rank maps every other rank's buffer.
constexpr int kPeerMaxRanks = 16;
constexpr size_t kPeerHeaderBytes = 512;
struct PeerHeader {
  int32_t status;               // kStatus* of this rank's exchange kernels (first word)
  uint32_t done;                // merge CTAs of the current step that finished reading
  uint64_t step;                // this rank's exchange step (advanced by the publish)
  uint64_t ready[kPeerMaxRanks];  // ready[r] == s: rank r's run of step s is complete
  uint64_t ack[kPeerMaxRanks];    // ack[r] == s: rank r has read this rank's run of step s
  // measurement (%globaltimer ns): the current merge's start and the end of its
  // ready waits (merge CTA 0), and sums over the merges since the last reset of
  // the time spent waiting for the ranks' runs, merging, and waiting for the acks
  uint64_t t_start, t_ready;
  uint64_t wait_ns, merge_ns, ack_ns, merges;
};
static_assert(sizeof(PeerHeader) <= kPeerHeaderBytes, "peer header too large");
constexpr int kMergeRunsMax = 16;
struct RunSet {
  const int32_t* run[kMergeRunsMax];
};
struct PeerSync {
  PeerHeader* self;                 // nullptr: a plain merge, no exchange
  PeerHeader* peer[kPeerMaxRanks];  // every rank's header, as mapped here
  int rank;
  int wait_acks;                    // the merge's last CTA waits for every rank's ack
  int64_t timeout_ns;               // bound of every wait
};
cudaError_t launch_merge_runs(const RunSet& rs, int nruns, int64_t rows, int64_t run_len, int k,
                              int32_t* out_idx, float* out_scores, const PeerSync& sync,
                              cudaStream_t stream);
cudaError_t launch_peer_publish(const PeerSync& sync, int world, cudaStream_t stream);
// Waits until every rank acknowledged this rank's run of the current step (see
// select_topk.cu); launched before a local top-k that rewrites the run.
cudaError_t launch_peer_wait_acks(const PeerSync& sync, int world, cudaStream_t stream);

// Post-selection: sorted union of the selected middle positions (optionally the
// recall_clip most frequent), each widened to [p + lo, p + hi) and clamped to
// [0, n_mid). out_pos holds up to n_mid positions, out_count the number written.
size_t post_select_workspace_bytes(int64_t n_mid, int32_t recall_clip);
cudaError_t launch_post_select(const int32_t* idx, int64_t n_idx, int64_t n_mid, int32_t recall_clip,
                               int lo, int hi, int32_t* out_pos, int32_t* out_count, void* workspace,
                               int num_sms, cudaStream_t stream);

// Block-maximum top-1 / top-4 (the reference Triton kernels' selection); a.k in
// {1, 4}, a.n % 128 == 0.
cudaError_t launch_select_blockmax(const SelectArgs& a, cudaStream_t stream);

// Value-norm weighting of a score matrix in place: scores[(b, hq, s), j] *=
// dtype-rounded ||v[b, hq / G, j, :]||_p, p in {1, 2}. Value rows: unit stride,
// row/head/batch strides and base 16-byte aligned, Dv % 8 == 0.
// launch_value_norms writes w [B * Hkv, ld] (weight_workspace_bytes, 16-byte
// aligned); launch_scale_scores then scales the scores [rows, ld] by it.
struct WeightArgs {
  const void* v;
  int64_t v_sb, v_sh, v_ss;  // element strides of batch, KV head, key
  int Dv;
  int p;
  int B, Hq, Hkv, G, Sq;
  int64_t Sk;
  float* scores;
  int64_t ld;
  float* w;
  int* status;  // device status word (bounded waits report kStatusTimeout)
};
size_t weight_workspace_bytes(int64_t B, int64_t Hkv, int64_t Sk);
cudaError_t launch_value_norms(const WeightArgs& a, int dtype, int num_sms, cudaStream_t stream);
cudaError_t launch_scale_scores(const WeightArgs& a, int num_sms, cudaStream_t stream);

// Attention over a selected view (sparse_attn.cu): gathered keys/values at the
// view's absolute positions key_pos[nsel], RoPE at the view's positions (if
// inv_freq), causal by absolute position, fp32 softmax; split over the view.
constexpr int kSparseMaxSplits = 128;
struct SparseAttnArgs {
  const void* q;          // [B, Hq, Sq, 128]
  const void* k;          // [B, Hkv, S, 128], rows contiguous
  const void* v;          // [B, Hkv, S, 128], rows contiguous
  const int64_t* key_pos; // [nsel] absolute positions of the view (< S)
  const int64_t* q_pos;   // [Sq] absolute positions of the query rows
  const float* inv_freq;  // [64] or nullptr (no rotation)
  int pe_original;        // RoPE at absolute positions (1) or at 0 .. nsel-1 with the queries last (0)
  float scale;
  int B, Hq, Hkv, G, Sq;
  int64_t S, nsel;
  int64_t q_sb, q_sh, q_ss, k_sb, k_sh, v_sb, v_sh;
  void* out;              // [B, Hq, Sq, 128] contiguous, dtype of q
  int* status;
  float* part_m;          // workspace (set by the launcher)
  float* part_l;
  float* part_acc;
  const float2* table;    // [nsel][64] (cos, sin) of the view's RoPE angles (launcher)
  const float* qrot;      // [B * Hq * Sq][128] rotated, scaled fp32 queries (launcher, with RoPE)
};
size_t sparse_attn_workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t nsel);
cudaError_t launch_sparse_attn(SparseAttnArgs a, int dtype, void* ws, int num_sms,
                               cudaStream_t stream);

// Sets the message prism_last_error() returns for the calling thread.
void set_last_error(const char* msg);

}  // namespace prism
