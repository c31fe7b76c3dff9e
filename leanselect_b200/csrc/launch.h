// Internal launcher declarations shared by the kernels and the C ABI layer.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace ls {

cudaError_t launch_fold_weights(const float* head_mix, const float* kv_head_mix,
                                const float* q_proj, const float* k_proj, int H, int G, int D,
                                int R, int r, float* q_f32, float* kv_f32, uint16_t* q_bf16,
                                uint16_t* kv_bf16, uint16_t* wq_t, uint16_t* wk_t,
                                cudaStream_t stream);

cudaError_t launch_compressed_seqlens(const int32_t* cu_k, int batch, int kernel_size,
                                      int kernel_stride, int32_t* cu_c, int32_t* status,
                                      cudaStream_t stream);

// Keys summed per run when compressing with stride `kernel_stride`: 16 when
// 16 divides the stride, else the stride (the summation order of the
// compression kernels and of the oracle).
inline int compress_run_length(int kernel_stride) {
  return kernel_stride % 16 == 0 ? 16 : kernel_stride;
}

cudaError_t launch_compress_keys(const uint16_t* k, const int32_t* cu_k, const int32_t* cu_c,
                                 int batch, int64_t total_k, int64_t total_c, int G, int D,
                                 int kernel_size, int kernel_stride, uint16_t* kc,
                                 int32_t* status, cudaStream_t stream);

// compress_k (32/16) and compress_k2 (128/64) in one pass over K.
cudaError_t launch_compress_keys_dual(const uint16_t* k, const int32_t* cu_k, const int32_t* cu_c,
                                      const int32_t* cu_c2, int batch, int max_atoms,
                                      int64_t total_k, int G, int D, uint16_t* kc, uint16_t* kc2,
                                      int32_t* status, cudaStream_t stream);

// Score/select kernel family (score_select.cu).
enum ScoreMode { kModeProject = 0, kModeScore = 1, kModeSelect = 2, kModeAtoms = 3 };

struct ScoreArgs {
  CUtensorMap tm_q;    // Q as [total_q, H*D] bf16, box {64, 128}, 128B swizzle
  CUtensorMap tm_w;    // WqT as [G*F, Hg*D] bf16, box {64, 128}
  CUtensorMap tm_ks;   // Ks as [G*total_c, F] bf16, box {64, 128}
  const int32_t* cu_q;
  const int32_t* cu_c;
  int batch;
  int num_groups;
  int hg;              // query heads per group
  int max_seqlen_q;
  int64_t total_q;
  int64_t total_c;
  int take;            // output width of topk_idx
  int init_blocks;
  int local_blocks;
  int max_pages;       // ceil(max_seqlen_q / 64): width of page_scores
  int pos_offset;      // chunk mode: position of query row 0 inside its sequence
  int seq_len;         // chunk mode: length of the whole sequence (0 = rows are the sequence)
  int32_t* topk_idx;   // kModeSelect
  uint16_t* workspace; // kModeSelect: pooled page scores [G, total_q, round8(max_pages)] bf16
  uint16_t* atom_out;  // kModeAtoms: raw atom scores [G, total_q, max_atoms] bf16
  int max_atoms;       // kModeAtoms: row length of atom_out
  float* page_scores;  // kModeScore
  uint16_t* qs_out;    // kModeProject: [G, total_q, F] bf16
  int32_t* status;
  // kModeSelect, uniform method (ops/uniform.py): atoms after the query are
  // hidden, pooled scores are rounded as bf16(bf16(s) * score_scale), rows
  // of sequences without atoms keep their forced pages, and page q_page+1
  // competes for a slot that it then leaves empty.
  int uniform;
  float score_scale;
};

cudaError_t launch_score(int mode, const ScoreArgs& args, cudaStream_t stream);

// Uniform method inputs (prep.cu): the mean-of-group-heads projection as a
// folded weight wq_t [G, D, Hg*D] (1/Hg on the diagonal of each head block)
// and Kc [total_c, G, D] re-laid out as Ks [G, total_c, D].
cudaError_t launch_uniform_prep(const uint16_t* kc, int64_t total_c, int num_kv_heads, int hg,
                                uint16_t* wq_t, uint16_t* ks, cudaStream_t stream);

// Bytes of selection workspace for `rows` = G * query rows and `max_pages`:
// one bf16 page score per (row, page), rows padded to 8 pages (16 bytes).
size_t select_workspace_bytes(int64_t rows, int max_pages);

// Sparse attention (sparse_attn.cu).
struct AttnArgs {
  CUtensorMap tm_k;    // K as [total_k, G*D] bf16, box {64, 64}, 128B swizzle
  CUtensorMap tm_v;    // V, same geometry
  const uint16_t* q;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t* topk_idx;
  int batch;
  int num_heads;
  int num_groups;
  int topk;
  int causal;
  float scale_log2;    // softmax_scale * log2(e)
  float scale;         // softmax_scale
  int64_t total_q;
  int64_t total_k;
  uint16_t* out;
  float* lse;
  int32_t* status;
  int order;           // CTA order: 0 token-major (groups interleaved), 1 group-major
  // Split pages (decode): each (token, group) row's sorted page list is cut
  // into `splits` contiguous slices, one CTA each; the CTAs write normalised
  // partial outputs and (row max in log2 units, row sum), which
  // launch_sparse_attn_merge combines.  splits == 1: no workspace, the CTA
  // writes `out` (and `lse`) itself.
  int splits;
  float* part_o;       // [splits, total_q * num_heads, 128]
  float* part_ml;      // [splits, total_q * num_heads, 2]
};

cudaError_t launch_sparse_attn(const AttnArgs& args, cudaStream_t stream);

// Combines the split partial results of a launch_sparse_attn with
// args.splits > 1 into `out` (and `lse`).
cudaError_t launch_sparse_attn_merge(const AttnArgs& args, cudaStream_t stream);

// The attention launch's data movement alone: same grid, page lists, TMA
// boxes and shared-memory ring, consumers release each stage unread and
// nothing is written.  Its duration is the L2 -> shared-memory gather time
// the attention kernel cannot beat (a measured roofline for it).
cudaError_t launch_sparse_attn_gather_only(const AttnArgs& args, cudaStream_t stream);

// Host-side argument checks of ls_select_pages other than its workspace
// (shared with ls_select_pages_noalloc); LS_OK or the LS_ERR_* code it sets.
int check_select_args(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                      const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c, int32_t batch,
                      int32_t max_seqlen_q, int64_t total_q, int64_t total_c, int32_t num_heads,
                      int32_t num_kv_heads, int32_t head_dim, int32_t width, int32_t take,
                      int32_t init_blocks, int32_t local_blocks, int32_t block_size,
                      int32_t kernel_stride, const int32_t* topk_idx);

// The bounded-wait test hook (waitprobe.cu).
cudaError_t launch_wait_probe(int32_t* status, int32_t* done, uint64_t timeout_ns,
                              cudaStream_t stream);

// Records `message` as the calling thread's ls_last_error() text; returns `code`.
int set_host_error(int code, const char* message);

// Builds a 2-D bf16 tensor map (row-major [rows, cols], 128B swizzle).
// Returns false if the driver entry point is unavailable or encoding fails.
bool make_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                        uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows);

}  // namespace ls
