// prism_topk_merge_noalloc: the candidate merge of prism_topk_merge for callers
// that must not allocate device memory (declared in include/prism_b200.h).
//
// Some callers cannot call cudaMalloc or hand the library a workspace: code that
// runs under a fixed device-memory budget owned by another allocator, or on a
// path where cudaMalloc's implicit device synchronisation is not acceptable.
// This entry point runs the same selection kernel as prism_topk_merge, but its
// per-row candidate buffers live in one file-scope device array of fixed size,
// so a call allocates nothing: no cudaMalloc, no cudaFree, no allocating
// library routine.
//
// Set-up: the first call on each device (with that device current) looks the
// array's address up once with cudaGetSymbolAddress and caches it. That first
// call may make the CUDA runtime load this module on the device, so make it
// before any stream capture is started on that device, e.g. once at start-up.
// The cached address belongs to the device's current context: after a
// cudaDeviceReset of that device it is stale, so the entry point must not be
// called on a device that was reset in the same process.
//
// Only requests of fewer than 64 rows write the scratch (one 4-CTA cluster per
// row; its exact path appends each row's candidates to the row's slice). From 64
// rows on, one CTA per row keeps its candidates in shared memory; the size rule
// below is applied to every request all the same.
//
// Nothing in the scratch has to start at zero: the selection kernel counts its
// candidate slots in shared memory and writes every slot before reading it.
//
// One scratch array per device is shared by every call on that device: calls
// whose executions overlap (different streams, or several host threads
// launching concurrently) race on it and give wrong results. Calls issued on
// one stream run one after another and are safe.
#include <cstdio>
#include <mutex>

#include "../../include/prism_b200.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = PRISM_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_merge_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Records the message prism_last_error() returns and passes the code through.
int noalloc_fail(int code, const char* msg, const char* detail = nullptr) {
  char buf[320];
  snprintf(buf, sizeof(buf), "prism_topk_merge_noalloc: %s%s%s", msg, detail ? ": " : "",
           detail ? detail : "");
  prism::set_last_error(buf);
  return code;
}

// Device address of g_merge_scratch on the current device, looked up on the
// first call for that device.
cudaError_t scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_merge_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

int prism_topk_merge_noalloc(const float* cand_scores, const int32_t* cand_idx, int64_t rows,
                             int64_t n, int64_t ld, int32_t topk, int32_t* out_idx,
                             float* out_scores, void* stream_ptr) {
  prism::set_last_error("");
  if (!cand_scores || !cand_idx || !out_idx)
    return noalloc_fail(PRISM_E_INVALID, "null pointer argument");
  if (rows < 0 || n <= 0 || ld < n || ld % 4 != 0)
    return noalloc_fail(PRISM_E_INVALID, "need rows >= 0, n > 0, ld >= n and ld % 4 == 0");
  if ((reinterpret_cast<uintptr_t>(cand_scores) & 15u) ||
      (reinterpret_cast<uintptr_t>(cand_idx) & 15u))
    return noalloc_fail(PRISM_E_INVALID, "candidate arrays must be 16-byte aligned");
  if (topk < 1 || int64_t(topk) > n)
    return noalloc_fail(PRISM_E_INVALID, "topk must satisfy 1 <= topk <= n");
  if (topk > prism::kSelectMaxK)
    return noalloc_fail(PRISM_E_UNSUPPORTED, "topk above 16384 is not supported");
  const size_t need = prism::select_workspace_bytes(rows, n);
  if (need > kScratchBytes) {
    char detail[128];
    snprintf(detail, sizeof(detail), "rows * min(n, 16384) * 8 = %zu bytes, limit %zu bytes", need,
             kScratchBytes);
    return noalloc_fail(PRISM_E_WORKSPACE, "request exceeds the static merge scratch", detail);
  }
  if (rows == 0) return PRISM_OK;

  void* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess)
    return noalloc_fail(PRISM_E_CUDA, "cudaGetSymbolAddress(merge scratch)", cudaGetErrorString(e));

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
  e = prism::launch_select_topk(s, scratch, static_cast<cudaStream_t>(stream_ptr));
  if (e != cudaSuccess)
    return noalloc_fail(PRISM_E_CUDA, "merge kernel launch", cudaGetErrorString(e));
  return PRISM_OK;
}

}  // extern "C"
