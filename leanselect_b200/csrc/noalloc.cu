// ls_select_pages_noalloc: page selection for callers that cannot allocate
// device memory.
//
// ls_select_pages needs a scratch workspace (the pooled page scores of every
// (group, row)) that its caller allocates.  Some callers have no allocator to
// draw from: a plain C or C++ host that links only this library and runs
// inside a process whose device-memory budget belongs to another runtime, or
// a caller on a latency-critical path that must not call cudaMalloc, which
// can synchronise the whole device.  For them this entry point uses a
// fixed scratch buffer compiled into the library instead.
//
// The buffer is a file-scope __device__ array of kScratchBytes (16 MiB).
// Every GPU that loads the library holds its own copy until the process
// exits.  A host pointer to the array's name is not a device address, so the
// device address is looked up with cudaGetSymbolAddress, once per device,
// with that device current, on the first call made on it; make that first
// call before any stream capture.
//
// All calls on a device share the one buffer and it keeps the last call's
// contents.  Nothing in it has to start at zero: the scoring kernel writes
// every page score the top-k kernel later reads, within the same call.
// Calls that overlap on the GPU (issued to different streams, or from
// different host threads without ordering) would overwrite each other's
// scores: serialise them.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace ls {
namespace {

constexpr size_t kScratchBytes = size_t{16} << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_select_scratch[kScratchBytes / sizeof(float)];

std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of this device's scratch array (looked up on first use).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_host_error(LS_ERR_CUDA, cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices)
    return set_host_error(LS_ERR_UNSUPPORTED, "device ordinal beyond the scratch table");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_select_scratch);
    if (err != cudaSuccess) return set_host_error(LS_ERR_CUDA, cudaGetErrorString(err));
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
  return LS_OK;
}

}  // namespace
}  // namespace ls

extern "C" int ls_select_pages_noalloc(
    const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks, const int32_t* cu_seqlens_q,
    const int32_t* cu_seqlens_c, int32_t batch, int32_t max_seqlen_q, int64_t total_q,
    int64_t total_c, int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t width,
    int32_t take, int32_t init_blocks, int32_t local_blocks, int32_t block_size,
    int32_t kernel_stride, int32_t* topk_idx, int32_t* status, void* stream) {
  const size_t need = ls_select_pages_workspace_bytes(total_q, num_kv_heads, max_seqlen_q);
  if (need > ls::kScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "ls_select_pages_noalloc needs %zu bytes of scratch but its built-in buffer holds "
             "%zu; call ls_select_pages with a caller-provided workspace",
             need, ls::kScratchBytes);
    return ls::set_host_error(LS_ERR_UNSUPPORTED, msg);
  }
  void* scratch = nullptr;
  const int rc = ls::scratch_address(&scratch);
  if (rc != LS_OK) return rc;
  return ls_select_pages(q, wq_t, ks, cu_seqlens_q, cu_seqlens_c, batch, max_seqlen_q, total_q,
                         total_c, num_heads, num_kv_heads, head_dim, width, take, init_blocks,
                         local_blocks, block_size, kernel_stride, topk_idx, scratch,
                         ls::kScratchBytes, status, stream);
}
