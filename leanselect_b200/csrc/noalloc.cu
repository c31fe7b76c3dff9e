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
// exits.  A host pointer to the array's name is not a device address, so
// every call looks the device address up with cudaGetSymbolAddress on the
// current device.  The first such lookup on a device loads the library's
// device code there, so make the first call on each device before any
// stream capture; later lookups are host-side, and looking the address up
// on every call (rather than caching it) keeps it valid across a
// cudaDeviceReset.
//
// All calls on a device share the one buffer and it keeps the last call's
// contents.  Nothing in it has to start at zero: the scoring kernel writes
// every page score the top-k kernel later reads, within the same call.
// Calls that overlap on the GPU (issued to different streams, or from
// different host threads without ordering) would overwrite each other's
// scores: serialise them.
#include <cstdio>

#include "common.cuh"
#include "launch.h"

namespace ls {
namespace {

constexpr size_t kScratchBytes = size_t{16} << 20;

static __device__ __align__(256) uint16_t g_select_scratch[kScratchBytes / sizeof(uint16_t)];

// Device address of the current device's scratch array.
int scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&p, g_select_scratch);
  if (err != cudaSuccess) return set_host_error(LS_ERR_CUDA, cudaGetErrorString(err));
  *out = p;
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
  // The same argument checks as ls_select_pages first, so a malformed call
  // gets the same error code; then the built-in buffer's size limit.
  int rc = ls::check_select_args(q, wq_t, ks, cu_seqlens_q, cu_seqlens_c, batch, max_seqlen_q,
                                 total_q, total_c, num_heads, num_kv_heads, head_dim, width, take,
                                 init_blocks, local_blocks, block_size, kernel_stride, topk_idx);
  if (rc != LS_OK) return rc;
  const size_t need = ls_select_pages_workspace_bytes(total_q, num_kv_heads, max_seqlen_q);
  if (need > ls::kScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "ls_select_pages_noalloc needs %zu bytes of scratch but its built-in buffer holds "
             "%zu; call ls_select_pages with a caller-provided workspace",
             need, ls::kScratchBytes);
    return ls::set_host_error(LS_ERR_UNSUPPORTED, msg);
  }
  if (total_q == 0 || take == 0) return LS_OK;
  void* scratch = nullptr;
  rc = ls::scratch_address(&scratch);
  if (rc != LS_OK) return rc;
  return ls_select_pages(q, wq_t, ks, cu_seqlens_q, cu_seqlens_c, batch, max_seqlen_q, total_q,
                         total_c, num_heads, num_kv_heads, head_dim, width, take, init_blocks,
                         local_blocks, block_size, kernel_stride, topk_idx, scratch,
                         ls::kScratchBytes, status, stream);
}
