// extern "C" entry points of libleanselect_b200.so: argument validation,
// TMA descriptor construction and kernel launches.  See
// include/leanselect_b200.h for the contract of each function.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace ls {

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(LS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) ==
            cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

}  // namespace

bool make_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                        uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows) {
  auto encode = get_encode_fn();
  if (encode == nullptr) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t elem_strides[2] = {1, 1};
  const CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                              dims, strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return res == CUDA_SUCCESS;
}

int set_host_error(int code, const char* message) { return fail(code, "%s", message); }

}  // namespace ls

using namespace ls;

#define LS_REQUIRE(cond, ...)                                   \
  do {                                                          \
    if (!(cond)) return fail(LS_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define LS_REQUIRE_ALIGNED(ptr)                                                          \
  do {                                                                                   \
    if (!aligned16(ptr)) return fail(LS_ERR_ALIGNMENT, "%s is not 16-byte aligned", #ptr); \
  } while (0)

extern "C" {

const char* ls_status_string(int code) {
  switch (code) {
    case LS_OK: return "LS_OK";
    case LS_ERR_INVALID_ARGUMENT: return "LS_ERR_INVALID_ARGUMENT";
    case LS_ERR_UNSUPPORTED: return "LS_ERR_UNSUPPORTED";
    case LS_ERR_ALIGNMENT: return "LS_ERR_ALIGNMENT";
    case LS_ERR_CUDA: return "LS_ERR_CUDA";
    default: return "LS_ERR_UNKNOWN";
  }
}

const char* ls_last_error(void) { return g_last_error; }

const char* ls_version(void) { return "leanselect_b200 0.1.0 sm_100a"; }

int ls_fold_weights(const float* head_mix, const float* kv_head_mix, const float* q_proj,
                    const float* k_proj, int32_t num_heads, int32_t num_kv_heads,
                    int32_t head_dim, int32_t router_heads, int32_t router_dim,
                    float* q_fused_f32, float* kv_fused_f32, uint16_t* q_fused_bf16,
                    uint16_t* kv_fused_bf16, uint16_t* wq_t, uint16_t* wk_t, void* stream) {
  LS_REQUIRE(head_mix && kv_head_mix && q_proj && k_proj, "null selector parameter");
  LS_REQUIRE(num_heads > 0 && num_kv_heads > 0 && head_dim > 0 && router_heads > 0 &&
                 router_dim > 0,
             "all selector dimensions must be positive");
  LS_REQUIRE(router_heads <= num_heads, "router_heads cannot exceed num_heads");
  LS_REQUIRE(num_heads % num_kv_heads == 0, "num_heads must be divisible by num_kv_heads");
  const cudaError_t err = launch_fold_weights(
      head_mix, kv_head_mix, q_proj, k_proj, num_heads, num_kv_heads, head_dim, router_heads,
      router_dim, q_fused_f32, kv_fused_f32, q_fused_bf16, kv_fused_bf16, wq_t, wk_t,
      static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "fold_weights launch");
}

int ls_compressed_seqlens(const int32_t* cu_seqlens_k, int32_t batch, int32_t kernel_size,
                          int32_t kernel_stride, int32_t* cu_seqlens_c, int32_t* status,
                          void* stream) {
  LS_REQUIRE(cu_seqlens_k && cu_seqlens_c, "null cu_seqlens");
  LS_REQUIRE(batch >= 1, "batch must be >= 1");
  LS_REQUIRE(kernel_size > 0 && kernel_stride > 0, "compression geometry must be positive");
  const cudaError_t err = launch_compressed_seqlens(cu_seqlens_k, batch, kernel_size,
                                                    kernel_stride, cu_seqlens_c, status,
                                                    static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "compressed_seqlens launch");
}

int ls_compress_keys(const uint16_t* k, const int32_t* cu_seqlens_k, int32_t batch,
                     int64_t total_k, int32_t num_kv_heads, int32_t head_dim,
                     int32_t kernel_size, int32_t kernel_stride, uint16_t* k_compressed,
                     int32_t* cu_seqlens_c, int64_t total_c, int32_t* status, void* stream) {
  LS_REQUIRE(k && cu_seqlens_k && cu_seqlens_c, "null argument");
  LS_REQUIRE(batch >= 1 && total_k >= 0 && total_c >= 0, "bad sizes");
  LS_REQUIRE(total_c == 0 || k_compressed, "null k_compressed");
  LS_REQUIRE(num_kv_heads > 0 && head_dim > 0, "bad head geometry");
  LS_REQUIRE(kernel_size > 0 && kernel_stride > 0, "compression geometry must be positive");
  if (kernel_size % kernel_stride != 0)
    return fail(LS_ERR_UNSUPPORTED, "kernel_size must be a multiple of kernel_stride");
  const int runs = kernel_size / kernel_stride;
  if (runs != 1 && runs != 2 && runs != 4)
    return fail(LS_ERR_UNSUPPORTED, "kernel_size/kernel_stride must be 1, 2 or 4");
  if (kernel_size / compress_run_length(kernel_stride) > 64)
    return fail(LS_ERR_UNSUPPORTED, "kernel_size must be at most 64 runs of 16 keys");
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (row % 8 != 0 || row > 2048)
    return fail(LS_ERR_UNSUPPORTED, "num_kv_heads*head_dim must be a multiple of 8 and <= 2048");
  LS_REQUIRE_ALIGNED(k);
  LS_REQUIRE_ALIGNED(k_compressed);
  LS_REQUIRE(total_c <= total_k / kernel_stride + batch, "total_c exceeds the possible atom count");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err =
      launch_compressed_seqlens(cu_seqlens_k, batch, kernel_size, kernel_stride, cu_seqlens_c,
                                status, s);
  if (err != cudaSuccess) return cuda_fail(err, "compressed_seqlens launch");
  err = launch_compress_keys(k, cu_seqlens_k, cu_seqlens_c, batch, total_k, total_c, num_kv_heads,
                             head_dim, kernel_size, kernel_stride, k_compressed, status, s);
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "compress_keys launch");
}

int ls_compress_keys_dual(const uint16_t* k, const int32_t* cu_seqlens_k, int32_t batch,
                          int32_t max_seqlen_k, int64_t total_k, int32_t num_kv_heads,
                          int32_t head_dim, uint16_t* k_compressed, int32_t* cu_seqlens_c,
                          int64_t total_c, uint16_t* k_compressed2, int32_t* cu_seqlens_c2,
                          int64_t total_c2, int32_t* status, void* stream) {
  LS_REQUIRE(k && cu_seqlens_k && cu_seqlens_c && cu_seqlens_c2, "null argument");
  LS_REQUIRE(batch >= 1 && batch <= 65535 && total_k >= 0 && total_c >= 0 && total_c2 >= 0 &&
                 max_seqlen_k >= 0,
             "bad sizes");
  LS_REQUIRE(total_c == 0 || k_compressed, "null k_compressed");
  LS_REQUIRE(total_c2 == 0 || k_compressed2, "null k_compressed2");
  LS_REQUIRE(num_kv_heads > 0 && head_dim > 0, "bad head geometry");
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (row % 8 != 0 || row > 2048)
    return fail(LS_ERR_UNSUPPORTED, "num_kv_heads*head_dim must be a multiple of 8 and <= 2048");
  LS_REQUIRE_ALIGNED(k);
  LS_REQUIRE_ALIGNED(k_compressed);
  LS_REQUIRE_ALIGNED(k_compressed2);
  LS_REQUIRE(total_c <= total_k / 16 + batch && total_c2 <= total_k / 64 + batch,
             "atom totals exceed the possible counts");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = launch_compressed_seqlens(cu_seqlens_k, batch, 32, 16, cu_seqlens_c, status, s);
  if (err == cudaSuccess)
    err = launch_compressed_seqlens(cu_seqlens_k, batch, 128, 64, cu_seqlens_c2, status, s);
  const int max_atoms = max_seqlen_k >= 32 ? (max_seqlen_k - 32) / 16 + 1 : 0;
  if (err == cudaSuccess && total_c > 0)
    err = launch_compress_keys_dual(k, cu_seqlens_k, cu_seqlens_c, cu_seqlens_c2, batch, max_atoms,
                                    total_k, num_kv_heads, head_dim, k_compressed, k_compressed2,
                                    status, s);
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "compress_keys_dual launch");
}

int ls_project_atom_keys(const uint16_t* kc, int64_t total_c, int32_t num_kv_heads,
                         int32_t head_dim, const uint16_t* wk_t, int32_t width, uint16_t* ks,
                         void* stream) {
  LS_REQUIRE(total_c >= 0 && total_c < (int64_t{1} << 31), "bad total_c");
  if (total_c == 0) return LS_OK;
  LS_REQUIRE(kc && wk_t && ks, "null argument");
  LS_REQUIRE(num_kv_heads > 0, "bad num_kv_heads");
  if (head_dim != 128 || width != 128)
    return fail(LS_ERR_UNSUPPORTED, "head_dim and selector width must be 128");
  LS_REQUIRE_ALIGNED(kc);
  LS_REQUIRE_ALIGNED(wk_t);
  LS_REQUIRE_ALIGNED(ks);
  // The tcgen05 projection GEMM with one "head" per group: rows are atoms,
  // Kc [total_c, G*D] plays the queries and wk_t [G*F, D] the folded weight.
  ScoreArgs a{};
  const uint64_t row = static_cast<uint64_t>(num_kv_heads) * 128;
  if (!make_tensor_map_2d(&a.tm_q, kc, static_cast<uint64_t>(total_c), row, row * 2, 64, 128))
    return fail(LS_ERR_CUDA, "cuTensorMapEncodeTiled failed for kc");
  if (!make_tensor_map_2d(&a.tm_w, wk_t, row, 128, 256, 64, 128))
    return fail(LS_ERR_CUDA, "cuTensorMapEncodeTiled failed for wk_t");
  a.tm_ks = a.tm_w;  // unused by the projection
  a.num_groups = num_kv_heads;
  a.hg = 1;
  a.total_q = total_c;
  a.cu_q = nullptr;
  a.cu_c = nullptr;
  a.batch = 1;
  a.max_seqlen_q = static_cast<int>(total_c);
  a.qs_out = ks;
  a.status = nullptr;
  const cudaError_t err = launch_score(kModeProject, a, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "project_atom_keys launch");
}

namespace {

int check_score_common(const uint16_t* q, const uint16_t* wq_t, int64_t total_q,
                       int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                       int32_t width) {
  LS_REQUIRE(q && wq_t, "null q or wq_t");
  LS_REQUIRE(total_q >= 0 && total_q < (int64_t{1} << 31), "total_q out of range");
  LS_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
             "num_heads must be a positive multiple of num_kv_heads");
  LS_REQUIRE(total_q * num_kv_heads < (int64_t{1} << 31), "num_kv_heads * total_q out of range");
  if (head_dim != 128 || width != 128)
    return fail(LS_ERR_UNSUPPORTED, "head_dim and selector width must be 128");
  const int hg = num_heads / num_kv_heads;
  if (hg != 8 && hg != 16) return fail(LS_ERR_UNSUPPORTED, "heads per group must be 8 or 16");
  LS_REQUIRE_ALIGNED(q);
  LS_REQUIRE_ALIGNED(wq_t);
  return LS_OK;
}

int build_score_args(ScoreArgs* a, const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                     int64_t total_q, int64_t total_c, int32_t num_heads, int32_t num_kv_heads) {
  const int hg = num_heads / num_kv_heads;
  const uint64_t hd = static_cast<uint64_t>(num_heads) * 128;
  if (!make_tensor_map_2d(&a->tm_q, q, static_cast<uint64_t>(std::max<int64_t>(total_q, 1)), hd,
                          hd * 2, 64, 128))
    return fail(LS_ERR_CUDA, "cuTensorMapEncodeTiled failed for q");
  if (!make_tensor_map_2d(&a->tm_w, wq_t, static_cast<uint64_t>(num_kv_heads) * 128,
                          static_cast<uint64_t>(hg) * 128, static_cast<uint64_t>(hg) * 256, 64, 128))
    return fail(LS_ERR_CUDA, "cuTensorMapEncodeTiled failed for wq_t");
  const void* ks_base = (ks != nullptr && total_c > 0) ? static_cast<const void*>(ks) : wq_t;
  const uint64_t ks_rows = (ks != nullptr && total_c > 0)
                               ? static_cast<uint64_t>(num_kv_heads) * static_cast<uint64_t>(total_c)
                               : 128;
  if (!make_tensor_map_2d(&a->tm_ks, ks_base, ks_rows, 128, 256, 64, 128))
    return fail(LS_ERR_CUDA, "cuTensorMapEncodeTiled failed for ks");
  a->num_groups = num_kv_heads;
  a->hg = hg;
  a->total_q = total_q;
  a->total_c = total_c;
  return LS_OK;
}

}  // namespace

int ls_project_queries(const uint16_t* q, int64_t total_q, int32_t num_heads,
                       int32_t num_kv_heads, int32_t head_dim, const uint16_t* wq_t,
                       int32_t width, uint16_t* qs, int32_t* status, void* stream) {
  int rc = check_score_common(q, wq_t, total_q, num_heads, num_kv_heads, head_dim, width);
  if (rc != LS_OK) return rc;
  if (total_q == 0) return LS_OK;
  LS_REQUIRE(qs, "null qs");
  LS_REQUIRE_ALIGNED(qs);
  ScoreArgs a{};
  rc = build_score_args(&a, q, wq_t, nullptr, total_q, 0, num_heads, num_kv_heads);
  if (rc != LS_OK) return rc;
  // Projection is row-local: with null cu_seqlens the kernel treats all
  // total_q rows as one sequence.
  a.cu_q = nullptr;
  a.cu_c = nullptr;
  a.batch = 1;
  a.max_seqlen_q = static_cast<int>(total_q);
  a.qs_out = qs;
  a.status = status;
  const cudaError_t err = launch_score(kModeProject, a, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "project_queries launch");
}

int ls_score_pages(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                   const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c, int32_t batch,
                   int32_t max_seqlen_q, int64_t total_q, int64_t total_c, int32_t num_heads,
                   int32_t num_kv_heads, int32_t head_dim, int32_t width, int32_t block_size,
                   int32_t kernel_stride, float* page_scores, int32_t* status, void* stream) {
  int rc = check_score_common(q, wq_t, total_q, num_heads, num_kv_heads, head_dim, width);
  if (rc != LS_OK) return rc;
  LS_REQUIRE(cu_seqlens_q && cu_seqlens_c, "null cu_seqlens");
  LS_REQUIRE(batch >= 1 && max_seqlen_q >= 0 && total_c >= 0, "bad sizes");
  if (block_size != 64 || kernel_stride != 16)
    return fail(LS_ERR_UNSUPPORTED, "block_size must be 64 and kernel_stride 16");
  if (total_q == 0 || max_seqlen_q == 0) return LS_OK;
  LS_REQUIRE(page_scores, "null page_scores");
  LS_REQUIRE(total_c == 0 || ks, "null ks");
  if (ks) LS_REQUIRE_ALIGNED(ks);
  ScoreArgs a{};
  rc = build_score_args(&a, q, wq_t, ks, total_q, total_c, num_heads, num_kv_heads);
  if (rc != LS_OK) return rc;
  a.cu_q = cu_seqlens_q;
  a.cu_c = cu_seqlens_c;
  a.batch = batch;
  a.max_seqlen_q = max_seqlen_q;
  a.max_pages = (max_seqlen_q + 63) / 64;
  a.page_scores = page_scores;
  a.status = status;
  const cudaError_t err = launch_score(kModeScore, a, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "score_pages launch");
}

int ls_score_pages_single(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                          int64_t total_q, int64_t total_c, int32_t seq_len, int32_t num_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t width,
                          int32_t block_size, int32_t kernel_stride, float* page_scores,
                          int32_t* status, void* stream) {
  int rc = check_score_common(q, wq_t, total_q, num_heads, num_kv_heads, head_dim, width);
  if (rc != LS_OK) return rc;
  LS_REQUIRE(total_c >= 0 && seq_len >= 0, "bad sizes");
  if (block_size != 64 || kernel_stride != 16)
    return fail(LS_ERR_UNSUPPORTED, "block_size must be 64 and kernel_stride 16");
  if (seq_len > 65536 * 64)
    return fail(LS_ERR_UNSUPPORTED, "sequences longer than 4M tokens are not supported");
  if (total_q == 0 || seq_len == 0) return LS_OK;
  LS_REQUIRE(page_scores, "null page_scores");
  LS_REQUIRE(total_c == 0 || ks, "null ks");
  if (ks) LS_REQUIRE_ALIGNED(ks);
  ScoreArgs a{};
  rc = build_score_args(&a, q, wq_t, ks, total_q, total_c, num_heads, num_kv_heads);
  if (rc != LS_OK) return rc;
  // One sequence: all total_q rows, all total_c atoms, ceil(seq_len/64) pages.
  a.cu_q = nullptr;
  a.cu_c = nullptr;
  a.batch = 1;
  a.max_seqlen_q = static_cast<int>(total_q);
  a.seq_len = seq_len;
  a.max_pages = (seq_len + 63) / 64;
  a.page_scores = page_scores;
  a.status = status;
  const cudaError_t err = launch_score(kModeScore, a, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "score_pages_single launch");
}

int ls_atom_scores(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                   const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c, int32_t batch,
                   int32_t max_seqlen_q, int64_t total_q, int64_t total_c, int32_t num_heads,
                   int32_t num_kv_heads, int32_t head_dim, int32_t width, int32_t max_atoms,
                   uint16_t* atom_scores, int32_t* status, void* stream) {
  int rc = check_score_common(q, wq_t, total_q, num_heads, num_kv_heads, head_dim, width);
  if (rc != LS_OK) return rc;
  LS_REQUIRE(cu_seqlens_q && cu_seqlens_c, "null cu_seqlens");
  LS_REQUIRE(batch >= 1 && max_seqlen_q >= 0 && total_c >= 0 && max_atoms >= 0, "bad sizes");
  if (total_q == 0 || max_seqlen_q == 0 || max_atoms == 0) return LS_OK;
  LS_REQUIRE(atom_scores, "null atom_scores");
  LS_REQUIRE(total_c == 0 || ks, "null ks");
  if (ks) LS_REQUIRE_ALIGNED(ks);
  LS_REQUIRE_ALIGNED(atom_scores);
  ScoreArgs a{};
  rc = build_score_args(&a, q, wq_t, ks, total_q, total_c, num_heads, num_kv_heads);
  if (rc != LS_OK) return rc;
  a.cu_q = cu_seqlens_q;
  a.cu_c = cu_seqlens_c;
  a.batch = batch;
  a.max_seqlen_q = max_seqlen_q;
  a.max_atoms = max_atoms;
  a.atom_out = atom_scores;
  a.status = status;
  const cudaError_t err = launch_score(kModeAtoms, a, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "atom_scores launch");
}

size_t ls_select_pages_workspace_bytes(int64_t total_q, int32_t num_kv_heads,
                                       int32_t max_seqlen_q) {
  if (total_q <= 0 || num_kv_heads <= 0 || max_seqlen_q <= 0) return 0;
  return select_workspace_bytes(total_q * num_kv_heads, (max_seqlen_q + 63) / 64);
}

}  // extern "C"

namespace ls {

int check_select_args(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                      const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c, int32_t batch,
                      int32_t max_seqlen_q, int64_t total_q, int64_t total_c, int32_t num_heads,
                      int32_t num_kv_heads, int32_t head_dim, int32_t width, int32_t take,
                      int32_t init_blocks, int32_t local_blocks, int32_t block_size,
                      int32_t kernel_stride, const int32_t* topk_idx) {
  int rc = check_score_common(q, wq_t, total_q, num_heads, num_kv_heads, head_dim, width);
  if (rc != LS_OK) return rc;
  LS_REQUIRE(cu_seqlens_q && cu_seqlens_c, "null cu_seqlens");
  LS_REQUIRE(batch >= 1 && max_seqlen_q >= 0 && total_c >= 0, "bad sizes");
  LS_REQUIRE(take >= 0 && init_blocks >= 0 && local_blocks >= 0, "negative budget");
  if (block_size != 64 || kernel_stride != 16)
    return fail(LS_ERR_UNSUPPORTED, "block_size must be 64 and kernel_stride 16");
  if (take > LS_MAX_TOPK) return fail(LS_ERR_UNSUPPORTED, "take exceeds LS_MAX_TOPK");
  if (max_seqlen_q > 65536 * 64)
    return fail(LS_ERR_UNSUPPORTED, "sequences longer than 4M tokens are not supported");
  if (total_q == 0 || take == 0) return LS_OK;
  LS_REQUIRE(topk_idx, "null topk_idx");
  LS_REQUIRE(total_c == 0 || ks, "null ks");
  if (ks) LS_REQUIRE_ALIGNED(ks);
  return LS_OK;
}

}  // namespace ls

extern "C" {

int ls_select_pages(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                    const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c, int32_t batch,
                    int32_t max_seqlen_q, int64_t total_q, int64_t total_c, int32_t num_heads,
                    int32_t num_kv_heads, int32_t head_dim, int32_t width, int32_t take,
                    int32_t init_blocks, int32_t local_blocks, int32_t block_size,
                    int32_t kernel_stride, int32_t* topk_idx, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = check_select_args(q, wq_t, ks, cu_seqlens_q, cu_seqlens_c, batch, max_seqlen_q,
                             total_q, total_c, num_heads, num_kv_heads, head_dim, width, take,
                             init_blocks, local_blocks, block_size, kernel_stride, topk_idx);
  if (rc != LS_OK) return rc;
  if (total_q == 0 || take == 0) return LS_OK;
  const size_t need = ls_select_pages_workspace_bytes(total_q, num_kv_heads, max_seqlen_q);
  LS_REQUIRE(workspace && workspace_bytes >= need, "workspace too small: %zu < %zu bytes",
             workspace_bytes, need);
  LS_REQUIRE_ALIGNED(workspace);
  ScoreArgs a{};
  rc = build_score_args(&a, q, wq_t, ks, total_q, total_c, num_heads, num_kv_heads);
  if (rc != LS_OK) return rc;
  a.workspace = static_cast<uint16_t*>(workspace);
  a.cu_q = cu_seqlens_q;
  a.cu_c = cu_seqlens_c;
  a.batch = batch;
  a.max_seqlen_q = max_seqlen_q;
  a.take = take;
  a.init_blocks = init_blocks;
  a.local_blocks = local_blocks;
  a.max_pages = (max_seqlen_q + 63) / 64;
  a.topk_idx = topk_idx;
  a.status = status;
  const cudaError_t err = launch_score(kModeSelect, a, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "select_pages launch");
}

namespace {
size_t align256(size_t n) { return (n + 255) & ~size_t{255}; }
}  // namespace

size_t ls_uniform_select_workspace_bytes(int64_t total_q, int64_t total_c, int32_t num_heads,
                                         int32_t num_kv_heads, int32_t max_seqlen_q) {
  if (total_q <= 0 || total_c < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_seqlen_q <= 0)
    return 0;
  const size_t weights = sizeof(uint16_t) * static_cast<size_t>(num_heads) * 128 * 128;
  const size_t keys = sizeof(uint16_t) * static_cast<size_t>(num_kv_heads) *
                      static_cast<size_t>(std::max<int64_t>(total_c, 1)) * 128;
  return align256(weights) + align256(keys) +
         ls_select_pages_workspace_bytes(total_q, num_kv_heads, max_seqlen_q);
}

int ls_uniform_select_pages(const uint16_t* q, const uint16_t* kc, const int32_t* cu_seqlens_q,
                            const int32_t* cu_seqlens_c, int32_t batch, int32_t max_seqlen_q,
                            int64_t total_q, int64_t total_c, int32_t num_heads,
                            int32_t num_kv_heads, int32_t head_dim, int32_t take,
                            int32_t init_blocks, int32_t local_blocks, int32_t block_size,
                            int32_t kernel_stride, float softmax_scale, int32_t* topk_idx,
                            void* workspace, size_t workspace_bytes, int32_t* status,
                            void* stream) {
  LS_REQUIRE(q && cu_seqlens_q && cu_seqlens_c, "null argument");
  LS_REQUIRE(total_q >= 0 && total_q < (int64_t{1} << 31), "total_q out of range");
  LS_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
             "num_heads must be a positive multiple of num_kv_heads");
  LS_REQUIRE(total_q * num_kv_heads < (int64_t{1} << 31), "num_kv_heads * total_q out of range");
  if (head_dim != 128) return fail(LS_ERR_UNSUPPORTED, "head_dim must be 128");
  const int hg = num_heads / num_kv_heads;
  if (hg != 8 && hg != 16) return fail(LS_ERR_UNSUPPORTED, "heads per group must be 8 or 16");
  LS_REQUIRE(batch >= 1 && max_seqlen_q >= 0 && total_c >= 0, "bad sizes");
  LS_REQUIRE(take >= 0 && init_blocks >= 0 && local_blocks >= 0, "negative budget");
  LS_REQUIRE(softmax_scale >= 0.f, "negative softmax_scale");
  if (block_size != 64 || kernel_stride != 16)
    return fail(LS_ERR_UNSUPPORTED, "block_size must be 64 and kernel_stride 16");
  if (take > LS_MAX_TOPK) return fail(LS_ERR_UNSUPPORTED, "take exceeds LS_MAX_TOPK");
  if (max_seqlen_q > 65536 * 64)
    return fail(LS_ERR_UNSUPPORTED, "sequences longer than 4M tokens are not supported");
  LS_REQUIRE_ALIGNED(q);
  if (total_q == 0 || take == 0) return LS_OK;
  LS_REQUIRE(topk_idx, "null topk_idx");
  LS_REQUIRE(total_c == 0 || kc, "null kc");
  if (kc) LS_REQUIRE_ALIGNED(kc);
  const size_t need = ls_uniform_select_workspace_bytes(total_q, total_c, num_heads,
                                                        num_kv_heads, max_seqlen_q);
  LS_REQUIRE(workspace && workspace_bytes >= need, "workspace too small: %zu < %zu bytes",
             workspace_bytes, need);
  LS_REQUIRE_ALIGNED(workspace);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  uint16_t* wq_t = reinterpret_cast<uint16_t*>(base);
  base += align256(sizeof(uint16_t) * static_cast<size_t>(num_heads) * 128 * 128);
  uint16_t* ks = reinterpret_cast<uint16_t*>(base);
  base += align256(sizeof(uint16_t) * static_cast<size_t>(num_kv_heads) *
                   static_cast<size_t>(std::max<int64_t>(total_c, 1)) * 128);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = launch_uniform_prep(kc, total_c, num_kv_heads, hg, wq_t, ks, st);
  if (err != cudaSuccess) return cuda_fail(err, "uniform prep launch");
  ScoreArgs a{};
  int rc = build_score_args(&a, q, wq_t, ks, total_q, total_c, num_heads, num_kv_heads);
  if (rc != LS_OK) return rc;
  a.workspace = reinterpret_cast<uint16_t*>(base);
  a.cu_q = cu_seqlens_q;
  a.cu_c = cu_seqlens_c;
  a.batch = batch;
  a.max_seqlen_q = max_seqlen_q;
  a.take = take;
  a.init_blocks = init_blocks;
  a.local_blocks = local_blocks;
  a.max_pages = (max_seqlen_q + 63) / 64;
  a.topk_idx = topk_idx;
  a.status = status;
  a.uniform = 1;
  a.score_scale = softmax_scale > 0.f ? softmax_scale : 0.08838834764831845f;  // 128^-0.5
  err = launch_score(kModeSelect, a, st);
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "uniform select launch");
}

int ls_select_pages_chunk(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                          int64_t chunk_q, int32_t q_position, int32_t seq_len, int64_t total_c,
                          int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t width,
                          int32_t take, int32_t init_blocks, int32_t local_blocks,
                          int32_t block_size, int32_t kernel_stride, int32_t* topk_idx,
                          void* workspace, size_t workspace_bytes, int32_t* status,
                          void* stream) {
  int rc = check_score_common(q, wq_t, chunk_q, num_heads, num_kv_heads, head_dim, width);
  if (rc != LS_OK) return rc;
  LS_REQUIRE(q_position >= 0 && seq_len >= 0 && total_c >= 0, "bad sizes");
  LS_REQUIRE(q_position + chunk_q <= seq_len, "query chunk extends past the sequence");
  LS_REQUIRE(take >= 0 && init_blocks >= 0 && local_blocks >= 0, "negative budget");
  if (block_size != 64 || kernel_stride != 16)
    return fail(LS_ERR_UNSUPPORTED, "block_size must be 64 and kernel_stride 16");
  if (take > LS_MAX_TOPK) return fail(LS_ERR_UNSUPPORTED, "take exceeds LS_MAX_TOPK");
  if (seq_len > 65536 * 64)
    return fail(LS_ERR_UNSUPPORTED, "sequences longer than 4M tokens are not supported");
  if (chunk_q == 0 || take == 0) return LS_OK;
  LS_REQUIRE(topk_idx, "null topk_idx");
  LS_REQUIRE(total_c == 0 || ks, "null ks");
  if (ks) LS_REQUIRE_ALIGNED(ks);
  const size_t need = ls_select_pages_workspace_bytes(chunk_q, num_kv_heads, seq_len);
  LS_REQUIRE(workspace && workspace_bytes >= need, "workspace too small: %zu < %zu bytes",
             workspace_bytes, need);
  LS_REQUIRE_ALIGNED(workspace);
  ScoreArgs a{};
  rc = build_score_args(&a, q, wq_t, ks, chunk_q, total_c, num_heads, num_kv_heads);
  if (rc != LS_OK) return rc;
  a.cu_q = nullptr;
  a.cu_c = nullptr;
  a.batch = 1;
  a.max_seqlen_q = static_cast<int>(chunk_q);
  a.take = take;
  a.init_blocks = init_blocks;
  a.local_blocks = local_blocks;
  a.max_pages = (seq_len + 63) / 64;
  a.pos_offset = q_position;
  a.seq_len = seq_len;
  a.topk_idx = topk_idx;
  a.workspace = static_cast<uint16_t*>(workspace);
  a.status = status;
  const cudaError_t err = launch_score(kModeSelect, a, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "select_pages_chunk launch");
}

namespace {

int sparse_attn_impl(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                     const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t batch,
                     int32_t max_seqlen_q, int32_t max_seqlen_k, int64_t total_q, int64_t total_k,
                     int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                     const int32_t* topk_idx, int32_t topk, int32_t block_size,
                     float softmax_scale, int32_t causal, uint16_t* out, float* lse,
                     int32_t* status, void* stream, bool gather_only, int32_t splits = 1,
                     void* workspace = nullptr, size_t workspace_bytes = 0) {
  LS_REQUIRE(q && k && v && cu_seqlens_q && cu_seqlens_k && (out || gather_only),
             "null argument");
  LS_REQUIRE(splits >= 1 && splits <= LS_MAX_ATTN_SPLITS, "splits must lie in [1, 64]");
  LS_REQUIRE(batch >= 1 && total_q >= 0 && total_k >= 0, "bad sizes");
  LS_REQUIRE(total_q < (int64_t{1} << 31) && total_k < (int64_t{1} << 31), "totals out of range");
  LS_REQUIRE(max_seqlen_q >= 0 && max_seqlen_k >= 0, "bad max_seqlen");
  LS_REQUIRE(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
             "num_heads must be a positive multiple of num_kv_heads");
  LS_REQUIRE(topk >= 0, "negative topk");
  if (head_dim != 128) return fail(LS_ERR_UNSUPPORTED, "head_dim must be 128");
  const int hg = num_heads / num_kv_heads;
  if (hg != 8 && hg != 16) return fail(LS_ERR_UNSUPPORTED, "heads per group must be 8 or 16");
  if (block_size != 64) return fail(LS_ERR_UNSUPPORTED, "block_size must be 64");
  if (topk > LS_MAX_TOPK) return fail(LS_ERR_UNSUPPORTED, "topk exceeds LS_MAX_TOPK");
  LS_REQUIRE(topk == 0 || topk_idx, "null topk_idx");
  LS_REQUIRE_ALIGNED(q);
  LS_REQUIRE_ALIGNED(k);
  LS_REQUIRE_ALIGNED(v);
  if (out) LS_REQUIRE_ALIGNED(out);
  if (total_q == 0) return LS_OK;
  LS_REQUIRE(total_q * num_kv_heads * splits < (int64_t{1} << 31), "too many CTAs");
  AttnArgs a{};
  a.splits = splits;
  if (splits > 1) {
    const size_t need = ls_sparse_attn_split_workspace_bytes(total_q, num_heads, splits);
    LS_REQUIRE(workspace, "null workspace");
    LS_REQUIRE_ALIGNED(workspace);
    LS_REQUIRE(workspace_bytes >= need, "workspace too small");
    const int64_t rows = total_q * num_heads;
    a.part_o = static_cast<float*>(workspace);
    a.part_ml = a.part_o + static_cast<int64_t>(splits) * rows * 128;
  }
  const uint64_t row = static_cast<uint64_t>(num_kv_heads) * 128;
  const uint64_t rows = static_cast<uint64_t>(std::max<int64_t>(total_k, 1));
  if (!make_tensor_map_2d(&a.tm_k, k, rows, row, row * 2, 64, 64))
    return fail(LS_ERR_CUDA, "cuTensorMapEncodeTiled failed for k");
  if (!make_tensor_map_2d(&a.tm_v, v, rows, row, row * 2, 64, 64))
    return fail(LS_ERR_CUDA, "cuTensorMapEncodeTiled failed for v");
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(static_cast<float>(head_dim));
  a.q = q;
  a.cu_q = cu_seqlens_q;
  a.cu_k = cu_seqlens_k;
  a.topk_idx = topk_idx;
  a.batch = batch;
  a.num_heads = num_heads;
  a.num_groups = num_kv_heads;
  a.topk = topk;
  a.causal = causal;
  a.scale = scale;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.total_q = total_q;
  a.total_k = total_k;
  a.out = out;
  a.lse = lse;
  a.status = status;
  a.order = 1;  // group-major: resident CTAs share one group's K/V in L2
  cudaError_t err = gather_only
                        ? launch_sparse_attn_gather_only(a, static_cast<cudaStream_t>(stream))
                        : launch_sparse_attn(a, static_cast<cudaStream_t>(stream));
  if (err == cudaSuccess && !gather_only && splits > 1)
    err = launch_sparse_attn_merge(a, static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "sparse_attn launch");
}

}  // namespace

int ls_sparse_attn(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                   const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t batch,
                   int32_t max_seqlen_q, int32_t max_seqlen_k, int64_t total_q, int64_t total_k,
                   int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                   const int32_t* topk_idx, int32_t topk, int32_t block_size,
                   float softmax_scale, int32_t causal, uint16_t* out, float* lse,
                   int32_t* status, void* stream) {
  return sparse_attn_impl(q, k, v, cu_seqlens_q, cu_seqlens_k, batch, max_seqlen_q, max_seqlen_k,
                          total_q, total_k, num_heads, num_kv_heads, head_dim, topk_idx, topk,
                          block_size, softmax_scale, causal, out, lse, status, stream, false);
}

size_t ls_sparse_attn_split_workspace_bytes(int64_t total_q, int32_t num_heads, int32_t splits) {
  if (total_q <= 0 || num_heads <= 0 || splits <= 1) return 0;
  return static_cast<size_t>(splits) * static_cast<size_t>(total_q) *
         static_cast<size_t>(num_heads) * (128 + 2) * sizeof(float);
}

int ls_sparse_attn_split(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t batch,
                         int32_t max_seqlen_q, int32_t max_seqlen_k, int64_t total_q,
                         int64_t total_k, int32_t num_heads, int32_t num_kv_heads,
                         int32_t head_dim, const int32_t* topk_idx, int32_t topk,
                         int32_t block_size, float softmax_scale, int32_t causal, int32_t splits,
                         void* workspace, size_t workspace_bytes, uint16_t* out, float* lse,
                         int32_t* status, void* stream) {
  return sparse_attn_impl(q, k, v, cu_seqlens_q, cu_seqlens_k, batch, max_seqlen_q, max_seqlen_k,
                          total_q, total_k, num_heads, num_kv_heads, head_dim, topk_idx, topk,
                          block_size, softmax_scale, causal, out, lse, status, stream, false,
                          splits, workspace, workspace_bytes);
}

int ls_wait_timeout_probe(int32_t* status, int32_t* done, uint64_t timeout_ns, void* stream) {
  LS_REQUIRE(status && done, "null status or done");
  LS_REQUIRE(timeout_ns >= 1000 && timeout_ns <= LS_WAIT_TIMEOUT_NS,
             "timeout_ns must lie in [1 us, 2 s]");
  const cudaError_t err = launch_wait_probe(status, done, timeout_ns,
                                            static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? LS_OK : cuda_fail(err, "wait probe launch");
}

int ls_sparse_attn_gather_only(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                               const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                               int32_t batch, int32_t max_seqlen_q, int32_t max_seqlen_k,
                               int64_t total_q, int64_t total_k, int32_t num_heads,
                               int32_t num_kv_heads, int32_t head_dim, const int32_t* topk_idx,
                               int32_t topk, int32_t block_size, int32_t causal, int32_t* status,
                               void* stream) {
  return sparse_attn_impl(q, k, v, cu_seqlens_q, cu_seqlens_k, batch, max_seqlen_q, max_seqlen_k,
                          total_q, total_k, num_heads, num_kv_heads, head_dim, topk_idx, topk,
                          block_size, 0.f, causal, nullptr, nullptr, status, stream, true);
}

}  // extern "C"
