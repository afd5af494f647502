// C-ABI entry points (include/prism_b200.h): argument checking, workspace
// layout and kernel orchestration on the caller's stream.
#include <algorithm>
#include <cstddef>
#include <atomic>
#include <vector>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/prism_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PRISM_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

constexpr size_t kStatusBytes = 256;  // status word + padding, keeps scores 256-B aligned
constexpr size_t kWorkOffset = 64;    // decode scorer work counters inside the status block
constexpr int64_t kMaxWorkCounters = (kStatusBytes - kWorkOffset) / 4;
constexpr int64_t kMaxPosition = int64_t(1) << 22;

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

int num_sms_current_device() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n;
}

// ---- measurement aids ----------------------------------------------------------
std::atomic<int64_t> g_launches{0};
struct ProfRec {
  int kernel;
  cudaEvent_t start, stop;
};
std::vector<cudaEvent_t> g_prof_pool;  // 2 * capacity events
std::vector<ProfRec> g_prof_recs;
bool g_prof_on = false;
size_t g_prof_next = 0;
int64_t g_prof_untimed[8] = {0, 0, 0, 0, 0, 0, 0, 0};

// Runs `launch` (which enqueues one kernel on `stream`), counting it and, while
// profiling is on, bracketing it with a pair of events from the pool.
template <typename F>
cudaError_t launch_counted(int kernel, cudaStream_t stream, F&& launch) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (!g_prof_on) return launch();
  if (g_prof_next + 2 > g_prof_pool.size()) {
    ++g_prof_untimed[kernel];
    return launch();
  }
  cudaEvent_t a = g_prof_pool[g_prof_next], b = g_prof_pool[g_prof_next + 1];
  g_prof_next += 2;
  cudaError_t e = cudaEventRecord(a, stream);
  if (e != cudaSuccess) return e;
  e = launch();
  if (e != cudaSuccess) return e;
  e = cudaEventRecord(b, stream);
  if (e == cudaSuccess) g_prof_recs.push_back(ProfRec{kernel, a, b});
  return e;
}

// status block | fp32 scores [rows, ld] | select candidates [rows, cap] u64
size_t scores_bytes(int64_t rows, int64_t Sk) {
  return size_t(rows) * size_t(round_up(Sk, 4)) * sizeof(float);
}
size_t exact_workspace(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk) {
  const int64_t rows = B * Hq * Sq;
  return kStatusBytes + round_up(int64_t(scores_bytes(rows, Sk)), 256) +
         prism::select_workspace_bytes(rows, Sk);
}
// Exact mode switches to the streaming prefill path (no score matrix) when the
// matrix would reach 2 GiB on a prefill-shaped call; PRISM_MODE_EXACT_STREAM
// asks for it at any size.
constexpr int64_t kStreamMinTopk = 4096;  // streaming path: topk <= this
bool auto_stream(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk, int32_t topk) {
  const double bytes = double(B) * double(Hq) * double(Sq) * double(round_up(Sk, 4)) * 4.0;
  return Sq >= prism::kPrefillMinRows && topk <= kStreamMinTopk && Sk >= 8192 &&
         bytes >= double(int64_t(1) << 31);
}
bool use_stream(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk, int32_t topk, int32_t mode) {
  return mode == PRISM_MODE_EXACT_STREAM ||
         (mode == PRISM_MODE_EXACT && auto_stream(B, Hq, Sq, Sk, topk));
}
size_t stream_workspace(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk, int32_t topk) {
  return kStatusBytes + prism::prefill_stream_workspace_bytes(B * Hq * Sq, Sk, topk);
}
// Exact mode on the queries-as-M scorer streams its top-k (thresholded candidates,
// no score matrix) for long contexts shared by many query rows.
bool wide_stream_shape(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk, int32_t topk) {
  return Sq >= 2 && B * Hq * Sq >= 64 && Sk >= 32768 && topk <= 4096 && int64_t(topk) * 16 <= Sk;
}
size_t wide_stream_workspace(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk, int32_t topk) {
  return kStatusBytes + prism::wide_stream_workspace_bytes(B * Hq * Sq, Sk, topk);
}
// the value-norm weights of the weighted call follow, 256-byte aligned
size_t weights_offset(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk) {
  return size_t(round_up(int64_t(exact_workspace(B, Hq, Sq, Sk)), 256));
}
// RoPE'd keys reach the tcgen05 scorer (>= kPrefillMinRows query rows per KV head)
// through un-rotated hi / lo key planes placed after the rest of the workspace
bool rope_planes_shape(int64_t Hq, int64_t Hkv, int64_t Sq) {
  return Hkv > 0 && Hq % Hkv == 0 && (Hq / Hkv) * Sq >= prism::kPrefillMinRows;
}

}  // namespace

namespace prism {
void set_last_error(const char* msg) { g_last_error = msg; }
}  // namespace prism

extern "C" {

int prism_abi_version(void) { return PRISM_ABI_VERSION; }

const char* prism_last_error(void) { return g_last_error.c_str(); }

size_t prism_einsum_topk_workspace_size(int64_t B, int64_t Hq, int64_t Sq, int64_t Sk,
                                        int32_t topk, int32_t mode) {
  if (B <= 0 || Hq <= 0 || Sq <= 0 || Sk <= 0) return 0;
  if (mode != PRISM_MODE_EXACT && mode != PRISM_MODE_BLOCKMAX && mode != PRISM_MODE_EXACT_STREAM)
    return 0;
  if (use_stream(B, Hq, Sq, Sk, topk, mode)) {
    if (topk < 1 || topk > kStreamMinTopk) return 0;
    return stream_workspace(B, Hq, Sq, Sk, topk);
  }
  const size_t ex = exact_workspace(B, Hq, Sq, Sk);
  if (mode == PRISM_MODE_EXACT && topk >= 1 && wide_stream_shape(B, Hq, Sq, Sk, topk))
    return std::max(ex, wide_stream_workspace(B, Hq, Sq, Sk, topk));
  return ex;
}

}  // extern "C"

namespace {

// Shared body of prism_einsum_topk and prism_einsum_topk_weighted: `weight`
// (already validated) scales the score matrix between scoring and selection.
// `acks` (the sharded call): the outputs are this rank's exchange run, so the
// kernels that write them first wait until every rank has read the previous
// step's run — on the score-matrix paths right before the selection (the wait
// overlaps the scorer), on the streaming paths before the first kernel.
int einsum_topk_impl(const void* q, const void* k, const float* inv_freq, int dtype, int64_t B,
                     int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                     const int64_t* q_strides, const int64_t* k_strides, int64_t pos_offset,
                     int64_t causal_offset, int32_t topk, int32_t mode, int64_t index_base,
                     int32_t* out_idx, float* out_scores, void* workspace,
                     size_t workspace_bytes, void* stream_ptr, const prism::WeightArgs* weight,
                     const prism::PeerSync* acks = nullptr, int acks_world = 0) {
  if (!q || !k || !out_idx || !q_strides || !k_strides)
    return fail(PRISM_E_INVALID, "null pointer argument");
  if (dtype != PRISM_DTYPE_BF16 && dtype != PRISM_DTYPE_FP16)
    return fail(PRISM_E_INVALID, "dtype must be PRISM_DTYPE_BF16 or PRISM_DTYPE_FP16");
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Sk <= 0)
    return fail(PRISM_E_INVALID, "all of B, Hq, Hkv, Sq, Sk must be positive");
  if (Hq % Hkv != 0) return fail(PRISM_E_INVALID, "num_heads must be divisible by num_heads_k");
  if (D != prism::kHeadDim) return fail(PRISM_E_UNSUPPORTED, "head_dim must be 128, got %lld", (long long)D);
  if (q_strides[3] != 1 || k_strides[3] != 1)
    return fail(PRISM_E_INVALID, "q and k must have unit stride in the last dimension");
  if (k_strides[2] != D)
    return fail(PRISM_E_INVALID, "key rows must be contiguous (k.stride(-2) == head_dim)");
  if ((reinterpret_cast<uintptr_t>(k) & 15u) != 0 || (k_strides[0] * 2) % 16 != 0 ||
      (k_strides[1] * 2) % 16 != 0)
    return fail(PRISM_E_INVALID, "k base and batch/head strides must be 16-byte aligned");
  if (mode != PRISM_MODE_EXACT && mode != PRISM_MODE_BLOCKMAX && mode != PRISM_MODE_EXACT_STREAM)
    return fail(PRISM_E_INVALID, "unknown mode %d", mode);
  if (mode == PRISM_MODE_BLOCKMAX && topk != 1 && topk != 4)
    return fail(PRISM_E_INVALID, "blockmax mode supports topk 1 or 4, got %d", topk);
  if (mode == PRISM_MODE_BLOCKMAX && Sk % 128 != 0)
    return fail(PRISM_E_INVALID, "blockmax mode needs Sk %% 128 == 0, got %lld", (long long)Sk);
  if (topk < 1 || int64_t(topk) > Sk)
    return fail(PRISM_E_INVALID, "topk must satisfy 1 <= topk <= Sk (topk=%d, Sk=%lld)", topk,
                (long long)Sk);
  if (topk > prism::kSelectMaxK)
    return fail(PRISM_E_UNSUPPORTED, "topk above %d is not supported", prism::kSelectMaxK);
  if (inv_freq && (pos_offset < 0 || pos_offset + Sk > kMaxPosition))
    return fail(PRISM_E_UNSUPPORTED, "RoPE positions must lie in [0, 2^22)");
  if (index_base < 0 || index_base + Sk - 1 > INT32_MAX)
    return fail(PRISM_E_INVALID, "index_base + Sk must fit in int32");
  if (Sk > INT32_MAX || B * Hq * Sq > (int64_t(1) << 31))
    return fail(PRISM_E_UNSUPPORTED, "problem too large");
  if (Hq > prism::kDecodeMaxRows)
    return fail(PRISM_E_UNSUPPORTED, "more than %d query heads", prism::kDecodeMaxRows);

  const bool streaming = use_stream(B, Hq, Sq, Sk, topk, mode);
  if (streaming) {
    if (topk > kStreamMinTopk)
      return fail(PRISM_E_UNSUPPORTED, "the streaming prefill path takes topk <= %lld, got %d",
                  (long long)kStreamMinTopk, topk);
    if (weight)
      return fail(PRISM_E_UNSUPPORTED, "value-weighted recall is not available on the streaming "
                                       "prefill path");
    if ((Hq / Hkv) * Sq < prism::kPrefillMinRows)
      return fail(PRISM_E_UNSUPPORTED, "the streaming prefill path needs at least %d query rows "
                                       "per KV head", prism::kPrefillMinRows);
    if ((reinterpret_cast<uintptr_t>(q) & 15u) != 0 || q_strides[0] % 8 || q_strides[1] % 8 ||
        q_strides[2] % 8)
      return fail(PRISM_E_INVALID, "the streaming prefill path needs 16-byte aligned query rows");
  }
  const size_t need = streaming ? stream_workspace(B, Hq, Sq, Sk, topk)
                      : weight ? weights_offset(B, Hq, Sq, Sk) + prism::weight_workspace_bytes(B, Hkv, Sk)
                               : exact_workspace(B, Hq, Sq, Sk);
  if (!workspace || workspace_bytes < need)
    return fail(PRISM_E_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(PRISM_E_INVALID, "workspace must be 256-byte aligned");
  // RoPE'd keys on the tcgen05 scorer: the un-rotated planes after `need`. The
  // streaming path requires them; the score-matrix path uses the CUDA-core scorers
  // when the workspace has no room for them.
  const size_t planes_off = size_t(round_up(int64_t(need), 256));
  const size_t planes_end = planes_off + prism::rope_planes_bytes(B, Hkv, Sk);
  const bool want_planes = inv_freq != nullptr && rope_planes_shape(Hq, Hkv, Sq);
  if (streaming && inv_freq != nullptr && workspace_bytes < planes_end)
    return fail(PRISM_E_WORKSPACE,
                "RoPE'd keys on the streaming path need %zu bytes of workspace "
                "(prism_einsum_topk_rope_workspace_size), got %zu",
                planes_end, workspace_bytes);
  const bool use_planes = want_planes && workspace_bytes >= planes_end;

  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  float* scores = reinterpret_cast<float*>(ws + kStatusBytes);
  const int64_t ld = round_up(Sk, 4);
  // the status block holds the status word and, from byte kWorkOffset, the decode
  // scorer's work counters (one per batch row); one memset clears what is used
  const bool dyn_work = !streaming && B <= kMaxWorkCounters;
  cudaError_t e = cudaMemsetAsync(status, 0, dyn_work ? kWorkOffset + size_t(B) * 4 : sizeof(int), stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(status)");

  const int nsm = num_sms_current_device();
  // ---- value norms (streams V once) ------------------------------------------------
  prism::WeightArgs wa{};
  if (weight) {
    wa = *weight;
    wa.B = int(B);
    wa.Hq = int(Hq);
    wa.Hkv = int(Hkv);
    wa.G = int(Hq / Hkv);
    wa.Sq = int(Sq);
    wa.Sk = Sk;
    wa.scores = scores;
    wa.ld = ld;
    wa.w = reinterpret_cast<float*>(ws + weights_offset(B, Hq, Sq, Sk));
    wa.status = status;
    e = launch_counted(PRISM_KERNEL_WEIGHT, stream,
                       [&] { return prism::launch_value_norms(wa, dtype, nsm, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "value norm kernel launch");
  }

  // ---- scoring ----------------------------------------------------------------------
  prism::DecodeArgs a{};
  a.q = q;
  a.k = k;
  a.inv_freq = inv_freq;
  a.B = int(B);
  a.Hq = int(Hq);
  a.Hkv = int(Hkv);
  a.G = int(Hq / Hkv);
  a.Sq = int(Sq);
  a.s0 = 0;
  a.sq_n = int(Sq);
  a.Sk = int(Sk);
  a.q_sb = q_strides[0];
  a.q_sh = q_strides[1];
  a.q_ss = q_strides[2];
  a.k_sb = k_strides[0];
  a.k_sh = k_strides[1];
  a.pos_offset = pos_offset;
  a.causal = causal_offset >= 0 ? 1 : 0;
  a.causal_offset = causal_offset;
  a.scores = scores;
  a.ld = ld;
  a.ntiles = int((Sk + 127) / 128);
  a.status = status;
  a.planes = use_planes ? static_cast<void*>(ws + planes_off) : nullptr;
  auto unrotate = [&]() -> cudaError_t {
    return launch_counted(PRISM_KERNEL_UNROTATE, stream,
                          [&] { return prism::launch_unrotate_planes(a, dtype, nsm, stream); });
  };
  // specialised kernels take every query row of a KV head in one launch:
  // tensor-core tiles (keys as M for <= 16 rows per KV head, queries as M up
  // to 256 / Hkv rows), CUDA cores for <= 4
  auto wait_acks = [&]() -> cudaError_t {
    if (acks == nullptr) return cudaSuccess;
    return launch_counted(PRISM_KERNEL_MERGE, stream,
                          [&] { return prism::launch_peer_wait_acks(*acks, acks_world, stream); });
  };
  if (streaming) {  // thresholds, candidates, per-row selection + exact fallback
    e = wait_acks();
    if (e != cudaSuccess) return cuda_fail(e, "peer ack wait launch");
    if (a.planes != nullptr) {
      e = unrotate();
      if (e != cudaSuccess) return cuda_fail(e, "key un-rotation launch");
    }
    void* pws = ws + kStatusBytes;
    e = launch_counted(PRISM_KERNEL_THRESHOLD, stream,
                       [&] { return prism::prefill_stream_threshold(a, dtype, topk, pws, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "prefill threshold launch");
    e = launch_counted(PRISM_KERNEL_SCORE, stream,
                       [&] { return prism::prefill_stream_candidates(a, dtype, topk, pws, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "prefill candidate launch");
    e = launch_counted(PRISM_KERNEL_SELECT, stream, [&] {
      return prism::prefill_stream_select(a, dtype, topk, index_base, out_idx, out_scores, pws,
                                          stream);
    });
    if (e != cudaSuccess) return cuda_fail(e, "prefill select launch");
    g_launches.fetch_add(3, std::memory_order_relaxed);  // the select phase launches 4 kernels
    return PRISM_OK;
  }
  // the queries-as-M scorer on a long shared context: streaming top-k
  if (mode == PRISM_MODE_EXACT && !weight && wide_stream_shape(B, Hq, Sq, Sk, topk) &&
      !prism::decode_hp_supported(a, dtype) && !prism::decode_mma_supported(a) &&
      prism::decode_wide_supported(a)) {
    if (workspace_bytes < wide_stream_workspace(B, Hq, Sq, Sk, topk))
      return fail(PRISM_E_WORKSPACE, "workspace needs %zu bytes, got %zu",
                  wide_stream_workspace(B, Hq, Sq, Sk, topk), workspace_bytes);
    e = wait_acks();
    if (e != cudaSuccess) return cuda_fail(e, "peer ack wait launch");
    void* pws = ws + kStatusBytes;
    e = launch_counted(PRISM_KERNEL_THRESHOLD, stream,
                       [&] { return prism::wide_stream_threshold(a, dtype, topk, pws, nsm, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "wide threshold launch");
    e = launch_counted(PRISM_KERNEL_SCORE, stream,
                       [&] { return prism::wide_stream_candidates(a, dtype, topk, pws, nsm, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "wide candidate launch");
    e = launch_counted(PRISM_KERNEL_SELECT, stream, [&] {
      return prism::wide_stream_select(a, dtype, topk, index_base, out_idx, out_scores, pws, stream);
    });
    if (e != cudaSuccess) return cuda_fail(e, "wide stream select launch");
    g_launches.fetch_add(4, std::memory_order_relaxed);  // sample + thresholds, select phase of 4
    return PRISM_OK;
  }
  if (prism::decode_hp_supported(a, dtype)) {
    a.work = dyn_work ? reinterpret_cast<unsigned int*>(ws + kWorkOffset) : nullptr;
    e = launch_counted(PRISM_KERNEL_SCORE, stream,
                       [&] { return prism::launch_decode_scores_hp(a, nsm, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "decode score kernel launch");
  } else if (prism::decode_mma_supported(a)) {
    e = launch_counted(PRISM_KERNEL_SCORE, stream,
                       [&] { return prism::launch_decode_scores_mma(a, dtype, nsm, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "decode score kernel launch");
  } else if (prism::decode_wide_supported(a)) {
    e = launch_counted(PRISM_KERNEL_SCORE, stream, [&] {
      return prism::wide_tc_supported(a) ? prism::launch_wide_tc_scores(a, dtype, nsm, stream)
                                         : prism::launch_decode_scores_wide(a, dtype, nsm, stream);
    });
    if (e != cudaSuccess) return cuda_fail(e, "decode score kernel launch");
  } else if (prism::prefill_tc_supported(a)) {
    if (a.planes != nullptr) {
      e = unrotate();
      if (e != cudaSuccess) return cuda_fail(e, "key un-rotation launch");
    }
    e = launch_counted(PRISM_KERNEL_SCORE, stream,
                       [&] { return prism::launch_prefill_scores_tc(a, dtype, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "prefill score kernel launch");
  } else if (prism::decode_g4_supported(a)) {
    e = launch_counted(PRISM_KERNEL_SCORE, stream,
                       [&] { return prism::launch_decode_scores_g4(a, dtype, nsm, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "decode score kernel launch");
  } else {
    // general kernel: the query rows of one batch row resident per CTA, so the
    // query positions are taken in chunks of at most 128 / Hq
    const int sq_chunk = int(std::max<int64_t>(1, prism::kDecodeMaxRows / Hq));
    for (int64_t s0 = 0; s0 < Sq; s0 += sq_chunk) {
      prism::DecodeArgs ac = a;
      ac.s0 = int(s0);
      ac.sq_n = int(std::min<int64_t>(sq_chunk, Sq - s0));
      e = launch_counted(PRISM_KERNEL_SCORE, stream,
                         [&] { return prism::launch_decode_scores(ac, dtype, nsm, stream); });
      if (e != cudaSuccess) return cuda_fail(e, "decode score kernel launch");
    }
  }

  // ---- value-norm weighting of the score matrix ----------------------------------------
  // (a separate pass: loading the weights inside the issue-bound scorer's
  // epilogue was measured slower than re-reading the scores here)
  if (weight) {
    e = launch_counted(PRISM_KERNEL_SCALE, stream,
                       [&] { return prism::launch_scale_scores(wa, nsm, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "score weighting kernel launch");
  }

  // ---- selection ------------------------------------------------------------------
  prism::SelectArgs s{};
  s.scores = scores;
  s.idx_in = nullptr;
  s.rows = B * Hq * Sq;
  s.n = Sk;
  s.ld = ld;
  s.k = topk;
  s.index_base = index_base;
  s.out_idx = out_idx;
  s.out_scores = out_scores;
  s.status = status;
  void* cand_ws = ws + kStatusBytes + round_up(int64_t(scores_bytes(B * Hq * Sq, Sk)), 256);
  e = wait_acks();
  if (e != cudaSuccess) return cuda_fail(e, "peer ack wait launch");
  if (mode == PRISM_MODE_BLOCKMAX) {
    e = launch_counted(PRISM_KERNEL_SELECT, stream,
                       [&] { return prism::launch_select_blockmax(s, stream); });
    if (e != cudaSuccess) return cuda_fail(e, "blockmax select kernel launch");
    return PRISM_OK;
  }
  e = launch_counted(PRISM_KERNEL_SELECT, stream,
                     [&] { return prism::launch_select_topk(s, cand_ws, stream); });
  if (e != cudaSuccess) return cuda_fail(e, "select kernel launch");
  return PRISM_OK;
}

}  // namespace

extern "C" {

int prism_einsum_topk(const void* q, const void* k, const float* inv_freq, int dtype, int64_t B,
                      int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                      const int64_t* q_strides, const int64_t* k_strides, int64_t pos_offset,
                      int64_t causal_offset, int32_t topk, int32_t mode, int64_t index_base,
                      int32_t* out_idx, float* out_scores, void* workspace,
                      size_t workspace_bytes, void* stream_ptr) {
  g_last_error.clear();
  return einsum_topk_impl(q, k, inv_freq, dtype, B, Hq, Hkv, Sq, Sk, D, q_strides, k_strides,
                          pos_offset, causal_offset, topk, mode, index_base, out_idx, out_scores,
                          workspace, workspace_bytes, stream_ptr, nullptr);
}

size_t prism_einsum_topk_weighted_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                                                 int64_t Sk, int32_t topk, int32_t mode,
                                                 int32_t recall_weight) {
  const size_t base = prism_einsum_topk_workspace_size(B, Hq, Sq, Sk, topk, mode);
  if (base == 0 || Hkv <= 0) return 0;
  if (recall_weight == PRISM_RECALL_QK) return base;
  if (recall_weight != PRISM_RECALL_QKV && recall_weight != PRISM_RECALL_QKV2) return 0;
  return weights_offset(B, Hq, Sq, Sk) + prism::weight_workspace_bytes(B, Hkv, Sk);
}

size_t prism_einsum_topk_rope_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                                             int64_t Sk, int32_t topk, int32_t mode,
                                             int32_t recall_weight) {
  const size_t base =
      prism_einsum_topk_weighted_workspace_size(B, Hq, Hkv, Sq, Sk, topk, mode, recall_weight);
  if (base == 0 || !rope_planes_shape(Hq, Hkv, Sq)) return base;
  return size_t(round_up(int64_t(base), 256)) + prism::rope_planes_bytes(B, Hkv, Sk);
}

int prism_einsum_topk_weighted(const void* q, const void* k, const void* v, const float* inv_freq,
                               int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                               int64_t Sk, int64_t D, int64_t Dv, const int64_t* q_strides,
                               const int64_t* k_strides, const int64_t* v_strides,
                               int64_t pos_offset, int64_t causal_offset, int32_t recall_weight,
                               int32_t topk, int32_t mode, int64_t index_base, int32_t* out_idx,
                               float* out_scores, void* workspace, size_t workspace_bytes,
                               void* stream_ptr) {
  g_last_error.clear();
  if (recall_weight != PRISM_RECALL_QK && recall_weight != PRISM_RECALL_QKV &&
      recall_weight != PRISM_RECALL_QKV2)
    return fail(PRISM_E_INVALID, "unknown recall_weight %d", recall_weight);
  if (recall_weight == PRISM_RECALL_QK)
    return einsum_topk_impl(q, k, inv_freq, dtype, B, Hq, Hkv, Sq, Sk, D, q_strides, k_strides,
                            pos_offset, causal_offset, topk, mode, index_base, out_idx,
                            out_scores, workspace, workspace_bytes, stream_ptr, nullptr);
  if (!v || !v_strides) return fail(PRISM_E_INVALID, "null values pointer or strides");
  if (Dv <= 0 || Dv % 8 != 0 || Dv > 1024)
    return fail(PRISM_E_UNSUPPORTED, "value head_dim must be a multiple of 8 in [8, 1024], got %lld",
                (long long)Dv);
  if (v_strides[3] != 1) return fail(PRISM_E_INVALID, "values must have unit stride in the last dimension");
  if ((reinterpret_cast<uintptr_t>(v) & 15u) != 0 || (v_strides[0] * 2) % 16 != 0 ||
      (v_strides[1] * 2) % 16 != 0 || (v_strides[2] * 2) % 16 != 0)
    return fail(PRISM_E_INVALID, "values base and batch/head/key strides must be 16-byte aligned");
  prism::WeightArgs wa{};
  wa.v = v;
  wa.v_sb = v_strides[0];
  wa.v_sh = v_strides[1];
  wa.v_ss = v_strides[2];
  wa.Dv = int(Dv);
  wa.p = recall_weight == PRISM_RECALL_QKV ? 1 : 2;
  return einsum_topk_impl(q, k, inv_freq, dtype, B, Hq, Hkv, Sq, Sk, D, q_strides, k_strides,
                          pos_offset, causal_offset, topk, mode, index_base, out_idx, out_scores,
                          workspace, workspace_bytes, stream_ptr, &wa);
}

size_t prism_sparse_attention_workspace_size(int64_t B, int64_t Hq, int64_t Sq, int64_t nsel) {
  if (B <= 0 || Hq <= 0 || Sq <= 0 || nsel <= 0) return 0;
  return kStatusBytes + prism::sparse_attn_workspace_bytes(B, Hq, Sq, nsel);
}

int prism_sparse_attention(const void* q, const void* k, const void* v, const int64_t* key_pos,
                           int64_t nsel, const int64_t* q_pos, const float* inv_freq,
                           int32_t pe_original, float scale, int dtype, int64_t B, int64_t Hq,
                           int64_t Hkv, int64_t Sq, int64_t S, int64_t D,
                           const int64_t* q_strides, const int64_t* k_strides,
                           const int64_t* v_strides, void* out, void* workspace,
                           size_t workspace_bytes, void* stream_ptr) {
  g_last_error.clear();
  if (!q || !k || !v || !key_pos || !q_pos || !out || !q_strides || !k_strides || !v_strides)
    return fail(PRISM_E_INVALID, "null pointer argument");
  if (dtype != PRISM_DTYPE_BF16 && dtype != PRISM_DTYPE_FP16)
    return fail(PRISM_E_INVALID, "dtype must be PRISM_DTYPE_BF16 or PRISM_DTYPE_FP16");
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || S <= 0 || nsel <= 0)
    return fail(PRISM_E_INVALID, "all of B, Hq, Hkv, Sq, S, nsel must be positive");
  if (Hq % Hkv != 0) return fail(PRISM_E_INVALID, "num_heads must be divisible by num_heads_k");
  if (D != prism::kHeadDim) return fail(PRISM_E_UNSUPPORTED, "head_dim must be 128, got %lld", (long long)D);
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1)
    return fail(PRISM_E_INVALID, "q, k and v must have unit stride in the last dimension");
  if (k_strides[2] != D || v_strides[2] != D)
    return fail(PRISM_E_INVALID, "key and value rows must be contiguous (stride(-2) == head_dim)");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v)) & 7u)
    return fail(PRISM_E_INVALID, "q, k and v must be 8-byte aligned");
  for (int i = 0; i < 3; ++i)
    if (q_strides[i] % 4 || k_strides[i] % 4 || v_strides[i] % 4)
      return fail(PRISM_E_INVALID, "q, k and v strides must be multiples of 4 elements");
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0)
    return fail(PRISM_E_INVALID, "out must be 16-byte aligned");
  const size_t need = prism_sparse_attention_workspace_size(B, Hq, Sq, nsel);
  if (!workspace || workspace_bytes < need)
    return fail(PRISM_E_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(PRISM_E_INVALID, "workspace must be 256-byte aligned");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* status = reinterpret_cast<int*>(ws);
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(status)");
  prism::SparseAttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.key_pos = key_pos;
  a.q_pos = q_pos;
  a.inv_freq = inv_freq;
  a.pe_original = pe_original ? 1 : 0;
  a.scale = scale;
  a.B = int(B);
  a.Hq = int(Hq);
  a.Hkv = int(Hkv);
  a.G = int(Hq / Hkv);
  a.Sq = int(Sq);
  a.S = S;
  a.nsel = nsel;
  a.q_sb = q_strides[0];
  a.q_sh = q_strides[1];
  a.q_ss = q_strides[2];
  a.k_sb = k_strides[0];
  a.k_sh = k_strides[1];
  a.v_sb = v_strides[0];
  a.v_sh = v_strides[1];
  a.out = out;
  a.status = status;
  const int nsm = num_sms_current_device();
  e = launch_counted(PRISM_KERNEL_ATTN, stream, [&] {
    return prism::launch_sparse_attn(a, dtype, ws + kStatusBytes, nsm, stream);
  });
  if (e != cudaSuccess) return cuda_fail(e, "sparse attention launch");
  g_launches.fetch_add(inv_freq ? 2 : 1, std::memory_order_relaxed);  // table, partial, combine
  return PRISM_OK;
}

size_t prism_topk_merge_workspace_size(int64_t rows, int64_t n) {
  if (rows < 0 || n <= 0) return 0;
  return prism::select_workspace_bytes(rows, n);
}

int prism_topk_merge(const float* cand_scores, const int32_t* cand_idx, int64_t rows, int64_t n,
                     int64_t ld, int32_t topk, int32_t* out_idx, float* out_scores,
                     void* workspace, size_t workspace_bytes, void* stream_ptr) {
  g_last_error.clear();
  if (!cand_scores || !cand_idx || !out_idx) return fail(PRISM_E_INVALID, "null pointer argument");
  if (rows < 0 || n <= 0 || ld < n || ld % 4 != 0)
    return fail(PRISM_E_INVALID, "need rows >= 0, n > 0, ld >= n and ld %% 4 == 0");
  if ((reinterpret_cast<uintptr_t>(cand_scores) & 15u) || (reinterpret_cast<uintptr_t>(cand_idx) & 15u))
    return fail(PRISM_E_INVALID, "candidate arrays must be 16-byte aligned");
  if (topk < 1 || int64_t(topk) > n) return fail(PRISM_E_INVALID, "topk must satisfy 1 <= topk <= n");
  if (topk > prism::kSelectMaxK)
    return fail(PRISM_E_UNSUPPORTED, "topk above %d is not supported", prism::kSelectMaxK);
  prism::SelectArgs s{};
  s.scores = cand_scores;
  s.idx_in = cand_idx;
  s.rows = rows;
  s.n = n;
  s.ld = ld;
  s.k = topk;
  s.index_base = 0;
  s.out_idx = out_idx;
  s.out_scores = out_scores;
  s.status = nullptr;
  const size_t need = prism::select_workspace_bytes(rows, n);
  if (!workspace || workspace_bytes < need)
    return fail(PRISM_E_WORKSPACE, "merge workspace needs %zu bytes, got %zu", need, workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) & 15u)
    return fail(PRISM_E_INVALID, "merge workspace must be 16-byte aligned");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaError_t e = launch_counted(PRISM_KERNEL_MERGE, stream,
                                 [&] { return prism::launch_select_topk(s, workspace, stream); });
  if (e != cudaSuccess) return cuda_fail(e, "merge kernel launch");
  return PRISM_OK;
}

int prism_topk_merge_runs(const int32_t* runs, int32_t nruns, int64_t rows, int64_t run_len,
                          int32_t topk, int32_t* out_idx, float* out_scores, void* stream_ptr) {
  g_last_error.clear();
  if (!runs || !out_idx) return fail(PRISM_E_INVALID, "null pointer argument");
  if (nruns < 1 || nruns > 16) return fail(PRISM_E_UNSUPPORTED, "1 to 16 runs are supported, got %d", nruns);
  if (rows < 0 || run_len < 1) return fail(PRISM_E_INVALID, "need rows >= 0 and run_len >= 1");
  if (topk < 1 || int64_t(topk) > run_len)
    return fail(PRISM_E_INVALID, "topk must satisfy 1 <= topk <= run_len");
  if (topk > prism::kSelectMaxK)
    return fail(PRISM_E_UNSUPPORTED, "topk above %d is not supported", prism::kSelectMaxK);
  if (reinterpret_cast<uintptr_t>(runs) & 3u) return fail(PRISM_E_INVALID, "runs must be 4-byte aligned");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaError_t e = launch_counted(PRISM_KERNEL_MERGE, stream, [&] {
    return prism::launch_merge_runs(runs, nruns, rows, run_len, topk, out_idx, out_scores, stream);
  });
  if (e != cudaSuccess) return cuda_fail(e, "run merge kernel launch");
  return PRISM_OK;
}

size_t prism_post_select_workspace_size(int64_t n_mid, int32_t recall_clip) {
  if (n_mid <= 0) return 0;
  return prism::post_select_workspace_bytes(n_mid, recall_clip);
}

int prism_post_select(const int32_t* topk_idx, int64_t n_idx, int64_t n_mid, int32_t recall_clip,
                      int32_t span_size, int32_t span_mode, int32_t* out_pos, int32_t* out_count,
                      void* workspace, size_t workspace_bytes, void* stream_ptr) {
  g_last_error.clear();
  if ((!topk_idx && n_idx > 0) || !out_pos || !out_count)
    return fail(PRISM_E_INVALID, "null pointer argument");
  if (n_idx < 0 || n_mid <= 0 || n_mid > INT32_MAX)
    return fail(PRISM_E_INVALID, "need n_idx >= 0 and 0 < n_mid <= INT32_MAX");
  if (span_size < 0) return fail(PRISM_E_INVALID, "span_size must be >= 0");
  if (span_mode != PRISM_SPAN_CENTERED && span_mode != PRISM_SPAN_FLOOR)
    return fail(PRISM_E_INVALID, "unknown span_mode %d", span_mode);
  const int32_t clip = recall_clip < 0 || int64_t(recall_clip) >= n_mid ? -1 : recall_clip;
  if (clip > prism::kSelectMaxK)
    return fail(PRISM_E_UNSUPPORTED, "recall_clip above %d is not supported", prism::kSelectMaxK);
  const size_t need = prism::post_select_workspace_bytes(n_mid, clip);
  if (!workspace || workspace_bytes < need)
    return fail(PRISM_E_WORKSPACE, "post-select workspace needs %zu bytes, got %zu", need, workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(PRISM_E_INVALID, "workspace must be 256-byte aligned");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  // offsets [lo, hi): centered = [-(s/2), (s+1)/2) and s = 0 keeps the position;
  // floor = [floor(-s/2), (s+1)/2), empty for s = 0
  int lo, hi;
  if (span_mode == PRISM_SPAN_CENTERED) {
    lo = span_size > 0 ? -(span_size / 2) : 0;
    hi = span_size > 0 ? (span_size + 1) / 2 : 1;
  } else {
    lo = -((span_size + 1) / 2);
    hi = (span_size + 1) / 2;
  }
  if (clip == 0 || lo >= hi) {
    cudaError_t e = cudaMemsetAsync(out_count, 0, sizeof(int32_t), stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(out_count)");
    return PRISM_OK;
  }
  const int nsm = num_sms_current_device();
  cudaError_t e = launch_counted(PRISM_KERNEL_SELECT, stream, [&] {
    return prism::launch_post_select(topk_idx, n_idx, n_mid, clip, lo, hi, out_pos, out_count,
                                     workspace, nsm, stream);
  });
  if (e != cudaSuccess) return cuda_fail(e, "post-select kernel launch");
  return PRISM_OK;
}

int prism_profile_start(int32_t capacity) {
  g_last_error.clear();
  if (capacity < 0) return fail(PRISM_E_INVALID, "capacity must be >= 0");
  const size_t want = size_t(capacity) * 2;
  while (g_prof_pool.size() < want) {
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreate(&ev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
    g_prof_pool.push_back(ev);
  }
  g_prof_recs.clear();
  g_prof_next = 0;
  for (int64_t& u : g_prof_untimed) u = 0;
  g_prof_on = capacity > 0;
  return PRISM_OK;
}

int prism_profile_stop(void) {
  g_prof_on = false;
  return PRISM_OK;
}

int prism_profile_read(int32_t kernel, int64_t* launches, double* total_ms) {
  g_last_error.clear();
  if (!launches || !total_ms || kernel < 0 || kernel > PRISM_KERNEL_UNROTATE)
    return fail(PRISM_E_INVALID, "bad kernel id or null output");
  int64_t n = 0;
  double ms = 0.0;
  for (const ProfRec& r : g_prof_recs) {
    if (r.kernel != kernel) continue;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize");
    float t = 0.f;
    e = cudaEventElapsedTime(&t, r.start, r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime");
    ms += t;
    ++n;
  }
  *launches = n;
  *total_ms = ms;
  return PRISM_OK;
}

int64_t prism_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

// ---- peer exchange of the sequence-sharded path -------------------------------------
static_assert(PRISM_PEER_HEADER_BYTES == prism::kPeerHeaderBytes, "peer header size");
static_assert(PRISM_PEER_MAX_RANKS == prism::kPeerMaxRanks, "peer rank limit");

size_t prism_peer_buffer_bytes(int64_t rows, int32_t topk) {
  if (rows < 1 || topk < 1) return 0;
  return prism::kPeerHeaderBytes + size_t(rows) * size_t(topk) * 2 * sizeof(int32_t);
}

int prism_peer_alloc(size_t bytes, void** buf, void* ipc_handle) {
  g_last_error.clear();
  if (!buf || !ipc_handle) return fail(PRISM_E_INVALID, "null pointer argument");
  if (bytes < prism::kPeerHeaderBytes) return fail(PRISM_E_INVALID, "buffer smaller than its header");
  static_assert(sizeof(cudaIpcMemHandle_t) == PRISM_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "allocating the exchange buffer");
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "preparing the exchange buffer");
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *buf = p;
  return PRISM_OK;
}

int prism_peer_open(const void* ipc_handle, void** buf) {
  g_last_error.clear();
  if (!buf || !ipc_handle) return fail(PRISM_E_INVALID, "null pointer argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "mapping a peer's exchange buffer");
  *buf = p;
  return PRISM_OK;
}

int prism_peer_close(void* buf) {
  g_last_error.clear();
  if (!buf) return fail(PRISM_E_INVALID, "null pointer argument");
  cudaError_t e = cudaIpcCloseMemHandle(buf);
  if (e != cudaSuccess) return cuda_fail(e, "unmapping a peer's exchange buffer");
  return PRISM_OK;
}

int prism_peer_free(void* buf) {
  g_last_error.clear();
  if (!buf) return fail(PRISM_E_INVALID, "null pointer argument");
  cudaError_t e = cudaFree(buf);
  if (e != cudaSuccess) return cuda_fail(e, "freeing the exchange buffer");
  return PRISM_OK;
}

}  // extern "C"

namespace {
int peer_sync(void* const* bufs, int32_t world, int32_t rank, prism::PeerSync& sync) {
  if (!bufs) return fail(PRISM_E_INVALID, "null pointer argument");
  if (world < 1 || world > prism::kPeerMaxRanks)
    return fail(PRISM_E_UNSUPPORTED, "1 to %d ranks are supported, got %d", prism::kPeerMaxRanks, world);
  if (rank < 0 || rank >= world) return fail(PRISM_E_INVALID, "rank %d outside [0, %d)", rank, world);
  sync = prism::PeerSync{};
  for (int r = 0; r < world; ++r) {
    if (!bufs[r]) return fail(PRISM_E_INVALID, "null exchange buffer of rank %d", r);
    if (reinterpret_cast<uintptr_t>(bufs[r]) & 255u)
      return fail(PRISM_E_INVALID, "exchange buffer of rank %d is not 256-byte aligned", r);
    sync.peer[r] = static_cast<prism::PeerHeader*>(bufs[r]);
  }
  sync.self = sync.peer[rank];
  sync.rank = rank;
  return PRISM_OK;
}
}  // namespace

extern "C" {

int prism_peer_publish(void* const* bufs, int32_t world, int32_t rank, void* stream_ptr) {
  g_last_error.clear();
  prism::PeerSync sync;
  const int rc = peer_sync(bufs, world, rank, sync);
  if (rc != PRISM_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaError_t e = launch_counted(PRISM_KERNEL_MERGE, stream, [&] {
    return prism::launch_peer_publish(sync, world, stream);
  });
  if (e != cudaSuccess) return cuda_fail(e, "publish kernel launch");
  return PRISM_OK;
}

int prism_peer_wait_acks(void* const* bufs, int32_t world, int32_t rank, int64_t timeout_ns,
                         void* stream_ptr) {
  g_last_error.clear();
  prism::PeerSync sync;
  const int rc = peer_sync(bufs, world, rank, sync);
  if (rc != PRISM_OK) return rc;
  sync.timeout_ns = timeout_ns > 0 ? timeout_ns : int64_t(prism::kWaitTimeoutNs);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaError_t e = launch_counted(PRISM_KERNEL_MERGE, stream, [&] {
    return prism::launch_peer_wait_acks(sync, world, stream);
  });
  if (e != cudaSuccess) return cuda_fail(e, "ack wait kernel launch");
  return PRISM_OK;
}

int prism_peer_merge(void* const* bufs, int32_t world, int32_t rank, int64_t rows, int32_t topk,
                     int32_t wait_acks, int64_t timeout_ns, int32_t* out_idx, float* out_scores,
                     void* stream_ptr) {
  g_last_error.clear();
  prism::PeerSync sync;
  const int rc = peer_sync(bufs, world, rank, sync);
  if (rc != PRISM_OK) return rc;
  if (!out_idx) return fail(PRISM_E_INVALID, "null pointer argument");
  if (rows < 1 || topk < 1) return fail(PRISM_E_INVALID, "need rows >= 1 and topk >= 1");
  if (topk > prism::kSelectMaxK)
    return fail(PRISM_E_UNSUPPORTED, "topk above %d is not supported", prism::kSelectMaxK);
  sync.wait_acks = wait_acks != 0;
  sync.timeout_ns = timeout_ns > 0 ? timeout_ns : int64_t(prism::kWaitTimeoutNs);
  prism::RunSet rs{};
  for (int r = 0; r < world; ++r)
    rs.run[r] = reinterpret_cast<const int32_t*>(static_cast<const uint8_t*>(bufs[r]) + prism::kPeerHeaderBytes);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaError_t e = launch_counted(PRISM_KERNEL_MERGE, stream, [&] {
    return prism::launch_merge_runs(rs, world, rows, topk, topk, out_idx, out_scores, sync, stream);
  });
  if (e != cudaSuccess) return cuda_fail(e, "peer merge kernel launch");
  return PRISM_OK;
}

int prism_sharded_topk(const void* q, const void* k_shard, const float* inv_freq, int dtype, int64_t B,
                       int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk_shard, int64_t D,
                       const int64_t* q_strides, const int64_t* k_strides, int64_t shard_start,
                       int32_t topk, void* const* exchange_bufs, int32_t world, int32_t rank,
                       int32_t wait_acks, int64_t timeout_ns, int32_t* out_idx, float* out_scores,
                       void* workspace, size_t workspace_bytes, void* stream_ptr) {
  g_last_error.clear();
  prism::PeerSync sync;
  int rc = peer_sync(exchange_bufs, world, rank, sync);
  if (rc != PRISM_OK) return rc;
  if (!out_idx) return fail(PRISM_E_INVALID, "null pointer argument");
  if (B <= 0 || Hq <= 0 || Sq <= 0 || topk < 1)
    return fail(PRISM_E_INVALID, "all of B, Hq, Sq and topk must be positive");
  if (Sk_shard < topk)
    return fail(PRISM_E_UNSUPPORTED, "every shard must hold at least topk keys (Sk_shard=%lld, topk=%d)",
                (long long)Sk_shard, topk);
  if (shard_start < 0) return fail(PRISM_E_INVALID, "shard_start must be >= 0");
  const int64_t rows = B * Hq * Sq;
  // this rank's run in its exchange buffer: [2, rows, topk] (score bits, indices)
  uint8_t* run = static_cast<uint8_t*>(exchange_bufs[rank]) + prism::kPeerHeaderBytes;
  float* run_scores = reinterpret_cast<float*>(run);
  int32_t* run_idx = reinterpret_cast<int32_t*>(run) + rows * topk;
  sync.timeout_ns = timeout_ns > 0 ? timeout_ns : int64_t(prism::kWaitTimeoutNs);
  rc = einsum_topk_impl(q, k_shard, inv_freq, dtype, B, Hq, Hkv, Sq, Sk_shard, D, q_strides, k_strides,
                        shard_start, -1, topk, PRISM_MODE_EXACT, shard_start, run_idx, run_scores,
                        workspace, workspace_bytes, stream_ptr, nullptr, wait_acks ? &sync : nullptr,
                        world);
  if (rc != PRISM_OK) return rc;
  rc = prism_peer_publish(exchange_bufs, world, rank, stream_ptr);
  if (rc != PRISM_OK) return rc;
  // the merge sends its acknowledgements; the next call waits for the others' before
  // it rewrites the run, while its scorer runs
  return prism_peer_merge(exchange_bufs, world, rank, rows, topk, 0, timeout_ns, out_idx,
                          out_scores, stream_ptr);
}

int prism_peer_read_timings(void* own_buf, uint64_t* out4, int32_t reset, void* stream_ptr) {
  g_last_error.clear();
  if (!own_buf || !out4) return fail(PRISM_E_INVALID, "null pointer argument");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  auto* h = static_cast<prism::PeerHeader*>(own_buf);
  uint64_t host[4] = {0, 0, 0, 0};
  static_assert(offsetof(prism::PeerHeader, merge_ns) == offsetof(prism::PeerHeader, wait_ns) + 8 &&
                    offsetof(prism::PeerHeader, ack_ns) == offsetof(prism::PeerHeader, wait_ns) + 16 &&
                    offsetof(prism::PeerHeader, merges) == offsetof(prism::PeerHeader, wait_ns) + 24,
                "timing sums are contiguous");
  cudaError_t e = cudaMemcpyAsync(host, &h->wait_ns, sizeof(host), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "reading the exchange timings");
  out4[0] = host[3];
  out4[1] = host[0];
  out4[2] = host[1];
  out4[3] = host[2];
  if (reset) {
    e = cudaMemsetAsync(&h->wait_ns, 0, sizeof(host), stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "resetting the exchange timings");
  }
  return PRISM_OK;
}

int prism_read_status(void* workspace, int* status_out, void* stream_ptr) {
  g_last_error.clear();
  if (!workspace || !status_out) return fail(PRISM_E_INVALID, "null pointer argument");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, workspace, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "reading the status word");
  *status_out = host;
  if (host != 0) {
    e = cudaMemsetAsync(workspace, 0, sizeof(int), stream);
    if (e != cudaSuccess) return cuda_fail(e, "resetting the status word");
  }
  return PRISM_OK;
}

}  // extern "C"
