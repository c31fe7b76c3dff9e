/*
 * leanselect_b200.h -- C ABI of the B200 (sm_100a) LeanSelect prefill path.
 *
 * Four stages of LeanSelect's long-context prefill are exposed here:
 *   key compression -> selector scoring (folded head mix) -> per-group top-T
 *   page selection with forced sink/local pages -> block-sparse causal
 *   attention over the selected 64-token pages.
 *
 * Conventions shared by every entry point
 *   - All tensor pointers are DEVICE pointers on the current CUDA device;
 *     bf16 tensors are passed as `uint16_t*` bit patterns.  Layouts are
 *     row-major with the shapes given per argument.  cu_seqlens arrays are
 *     int32 prefix sums of length batch+1 (the reference's varlen packing).
 *   - Host scalars (batch, totals, maxima) are what the caller already knows;
 *     the library never synchronises the stream to read device data.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call
 *     is stream-ordered, stateless apart from cached tensor-map builders, and
 *     reentrant across streams and threads.
 *   - The caller allocates every buffer.  The library never allocates or
 *     frees device memory on these paths.
 *   - Return value: LS_OK or an LS_ERR_* code.  Argument and capability
 *     checks happen on the host before anything is launched, so an error
 *     return means nothing was enqueued.  `status` (nullable, device int32)
 *     accumulates LS_DEVERR_* bits raised inside kernels (bad indices, a
 *     bounded wait that expired); kernels never trap.
 *
 * Reference interfaces (paths relative to the LeanSelect repository).
 */
#ifndef LEANSELECT_B200_H_
#define LEANSELECT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Host-side return codes. */
#define LS_OK 0
#define LS_ERR_INVALID_ARGUMENT 1 /* null pointer, bad shape, inconsistent sizes */
#define LS_ERR_UNSUPPORTED 2      /* valid but not compiled (e.g. head_dim != 128) */
#define LS_ERR_ALIGNMENT 3        /* a pointer or stride is not 16-byte aligned */
#define LS_ERR_CUDA 4             /* a CUDA runtime/driver call failed */

/* Device-side status bits (OR-ed into *status). */
#define LS_DEVERR_TIMEOUT 0x1          /* a bounded wait expired; outputs are invalid */
#define LS_DEVERR_PAGE_INDEX 0x2       /* a topk_idx entry >= number of key pages (ignored) */
#define LS_DEVERR_SEQLENS 0x4          /* cu_seqlens not monotone or beyond the totals */

/* Largest per-row page budget T accepted by ls_select_pages/ls_sparse_attn. */
#define LS_MAX_TOPK 128

/* Most page-list slices per row accepted by ls_sparse_attn_split. */
#define LS_MAX_ATTN_SPLITS 64

/* Human-readable name of an LS_ERR_* code. */
const char* ls_status_string(int code);

/* Text of the last host-side error raised on the calling thread. */
const char* ls_last_error(void);

/* Library build identity: "leanselect_b200 <version> sm_100a". */
const char* ls_version(void);

/*
 * ls_fold_weights -- replaces LeanSelectSelector.fused_weights
 * (leanselect/selector.py:144-158).
 *
 * q_fused[h, d, rho*r + j]  = head_mix[h, rho]    * q_proj[rho, d, j]
 * kv_fused[g, d, rho*r + j] = kv_head_mix[g, rho] * k_proj[rho, d, j]
 * Inputs are fp32 (the selector is kept in fp32, models/__init__.py:178-181).
 * Outputs (each nullable):
 *   q_fused_f32 [H, D, F], kv_fused_f32 [G, D, F]   fp32, reference layout
 *   q_fused_bf16 [H, D, F], kv_fused_bf16 [G, D, F] bf16, reference layout
 *   wq_t [G, F, Hg*D], wk_t [G, F, D]               bf16, kernel (K-major) layout
 * with F = R*r and Hg = H/G.
 */
int ls_fold_weights(const float* head_mix, const float* kv_head_mix, const float* q_proj,
                    const float* k_proj, int32_t num_heads, int32_t num_kv_heads,
                    int32_t head_dim, int32_t router_heads, int32_t router_dim,
                    float* q_fused_f32, float* kv_fused_f32, uint16_t* q_fused_bf16,
                    uint16_t* kv_fused_bf16, uint16_t* wq_t, uint16_t* wk_t, void* stream);

/*
 * ls_compressed_seqlens -- replaces the cu_seqlens_compressed half of
 * calc_chunks_with_stride (leanselect/models/minicpm.py:710-750).
 * cu_seqlens_c[b+1] = cu_seqlens_c[b] + (n_b >= kernel_size ? (n_b - kernel_size)/kernel_stride + 1 : 0).
 */
int ls_compressed_seqlens(const int32_t* cu_seqlens_k, int32_t batch, int32_t kernel_size,
                          int32_t kernel_stride, int32_t* cu_seqlens_c, int32_t* status,
                          void* stream);

/*
 * ls_compress_keys -- replaces CompressK.forward (leanselect/models/minicpm.py:1169-1185)
 * (same math as pages.compress_keys_mean, leanselect/pages.py:84-101).
 *
 * k [total_k, G, D] bf16 -> k_compressed [total_c, G, D] bf16 and
 * cu_seqlens_c [batch+1].  Atom i of sequence b is the mean of keys
 * [16 i, 16 i + 32) of that sequence (kernel_size/kernel_stride in general,
 * kernel_size a multiple of kernel_stride), summed in fp32 as runs of 16
 * keys (of kernel_stride keys when 16 does not divide it), the run sums
 * added in order, then scaled and rounded to bf16.  total_c must equal the
 * value implied by cu_seqlens_k (the caller computes it, as the reference
 * does on the host); G*D must be a multiple of 8 and at most 2048.
 */
int ls_compress_keys(const uint16_t* k, const int32_t* cu_seqlens_k, int32_t batch,
                     int64_t total_k, int32_t num_kv_heads, int32_t head_dim,
                     int32_t kernel_size, int32_t kernel_stride, uint16_t* k_compressed,
                     int32_t* cu_seqlens_c, int64_t total_c, int32_t* status, void* stream);

/*
 * ls_compress_keys_dual -- both compressions of a prefill in one pass over
 * K: the compress_k (kernel 32, stride 16) and compress_k2 (kernel 128,
 * stride 64) calls of MiniCPMInfLLMv2Attention.get_compress_k
 * (leanselect/models/minicpm.py:2785-2792).  Outputs equal, bit for bit,
 * ls_compress_keys with (32, 16) and with (128, 64): every window is summed
 * as 16-key runs in fp32, the run sums added in order, scaled and rounded to
 * bf16.  k [total_k, G, D] bf16 -> k_compressed [total_c, G, D] +
 * cu_seqlens_c, k_compressed2 [total_c2, G, D] + cu_seqlens_c2; the totals
 * are those cu_seqlens_k implies (the caller computes them, as the
 * reference does on the host); max_seqlen_k bounds the sequences' lengths.
 */
int ls_compress_keys_dual(const uint16_t* k, const int32_t* cu_seqlens_k, int32_t batch,
                          int32_t max_seqlen_k, int64_t total_k, int32_t num_kv_heads,
                          int32_t head_dim, uint16_t* k_compressed, int32_t* cu_seqlens_c,
                          int64_t total_c, uint16_t* k_compressed2, int32_t* cu_seqlens_c2,
                          int64_t total_c2, int32_t* status, void* stream);

/*
 * ls_project_atom_keys -- replaces LeanSelectSelector.project_atom_keys
 * (leanselect/selector.py:179-190).
 * kc [total_c, G, D] bf16, wk_t [G, F, D] bf16 -> ks [G, total_c, F] bf16
 * (fp32 accumulation, one rounding to bf16 as the reference's bf16 einsum).
 */
int ls_project_atom_keys(const uint16_t* kc, int64_t total_c, int32_t num_kv_heads,
                         int32_t head_dim, const uint16_t* wk_t, int32_t width, uint16_t* ks,
                         void* stream);

/*
 * ls_project_queries -- replaces LeanSelectSelector.project_queries
 * (leanselect/selector.py:160-177); tcgen05 GEMM.
 * q [total_q, H, D] bf16, wq_t [G, F, Hg*D] bf16 -> qs [G, total_q, F] bf16.
 * Requires D == 128, F == 128, Hg in {8, 16}.
 */
int ls_project_queries(const uint16_t* q, int64_t total_q, int32_t num_heads,
                       int32_t num_kv_heads, int32_t head_dim, const uint16_t* wq_t,
                       int32_t width, uint16_t* qs, int32_t* status, void* stream);

/*
 * ls_score_pages -- replaces LeanSelectSelector.score_pages
 * (leanselect/selector.py:192-214) with pool_atoms_to_pages(reduce="max")
 * (leanselect/pages.py:146-187), for a packed batch.
 *
 * Page scores [G, total_q, max_pages] fp32, max_pages = ceil(max_seqlen_q/block):
 * row t of sequence b holds the max over atoms [4p-1, 4p+4) of Qs[t]·Ks[a]
 * for p < P_b (no causal mask, as the reference) and -inf for p >= P_b.
 * Atom scores are rounded to bf16 as the reference's bf16 einsum rounds
 * them (selector.py:203-207), so every value is a bf16 number; these are
 * the scores ls_select_pages ranks.
 * q is the post-RoPE query; ks comes from ls_project_atom_keys.  Requires
 * block_size == 64, kernel_stride == 16.
 */
int ls_score_pages(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                   const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c, int32_t batch,
                   int32_t max_seqlen_q, int64_t total_q, int64_t total_c, int32_t num_heads,
                   int32_t num_kv_heads, int32_t head_dim, int32_t width, int32_t block_size,
                   int32_t kernel_stride, float* page_scores, int32_t* status, void* stream);

/*
 * ls_score_pages_single -- LeanSelectSelector.score_pages for one sequence
 * with the reference's own seq_len argument (leanselect/selector.py:192-214):
 * q [total_q, H, D] are any query rows, ks [G, total_c, F] the sequence's
 * atoms, and the output has ceil(seq_len/64) pages per row whatever
 * total_q is: page p pools atoms [4p-1, 4p+4) that exist (no causal mask),
 * pages with no atom are -inf.  Values as ls_score_pages (bf16 numbers in
 * fp32).  page_scores [G, total_q, ceil(seq_len/64)] fp32.
 */
int ls_score_pages_single(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                          int64_t total_q, int64_t total_c, int32_t seq_len, int32_t num_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t width,
                          int32_t block_size, int32_t kernel_stride, float* page_scores,
                          int32_t* status, void* stream);

/*
 * ls_atom_scores -- replaces NOSA's LlamaSdpaAttention._leanselect_atom_scores
 * (leanselect/models/nosa.py:1822-1853): raw LeanSelect atom scores
 * Qs[t]·Ks[a] for every (group, query row, atom of its sequence), no causal
 * mask, as bf16 [G, total_q, max_atoms] (max_atoms = the batch's largest atom
 * count; entries past a sequence's atoms are -inf), fed to NOSA's
 * compressed_attention as precomputed scores.  Requires D == 128, F == 128.
 */
int ls_atom_scores(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                   const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c, int32_t batch,
                   int32_t max_seqlen_q, int64_t total_q, int64_t total_c, int32_t num_heads,
                   int32_t num_kv_heads, int32_t head_dim, int32_t width, int32_t max_atoms,
                   uint16_t* atom_scores, int32_t* status, void* stream);

/*
 * ls_select_pages_workspace_bytes -- bytes of scratch ls_select_pages needs:
 * the pooled page scores of every (group, query row), bf16, rows padded to
 * 8 pages: 2 * G * total_q * round_up(ceil(max_seqlen_q / 64), 8).
 */
size_t ls_select_pages_workspace_bytes(int64_t total_q, int32_t num_kv_heads,
                                       int32_t max_seqlen_q);

/*
 * ls_select_pages -- replaces the selection loop of
 * MiniCPMInfLLMv2Attention._lightweight_compressed_attention
 * (leanselect/models/minicpm.py:3093-3141).
 *
 * Two kernels: a tcgen05 kernel computes the Q projection, the atom scores
 * and the page max-pool for every (group, row, candidate page) into
 * `workspace` as bf16 (the rounding of the reference's bf16 einsum,
 * selector.py:203-207); a warp-per-row radix select then picks the pages.
 *
 * topk_idx [G, total_q, take] int32, take = min(topk, max_pages) as in the
 * reference (minicpm.py:3096-3104).  Row t of sequence b holds
 * min(take, P_b) pages -- the forced pages (p < init_blocks, and
 * p in [t/64 - local_blocks, t/64]) and the best-scoring visible non-forced
 * pages, in ascending page order -- then -1.  Ties are broken toward the
 * lower page index (the reference uses torch.topk, whose order and
 * tie-break are unspecified).  Rows of sequences without atoms are all -1
 * (minicpm.py:3115-3116).  `workspace` must hold
 * ls_select_pages_workspace_bytes(total_q, G, max_seqlen_q) bytes.
 * Requires take <= LS_MAX_TOPK, block_size == 64, kernel_stride == 16.
 */
int ls_select_pages(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                    const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c, int32_t batch,
                    int32_t max_seqlen_q, int64_t total_q, int64_t total_c, int32_t num_heads,
                    int32_t num_kv_heads, int32_t head_dim, int32_t width, int32_t take,
                    int32_t init_blocks, int32_t local_blocks, int32_t block_size,
                    int32_t kernel_stride, int32_t* topk_idx, void* workspace,
                    size_t workspace_bytes, int32_t* status, void* stream);

/*
 * ls_select_pages_noalloc -- ls_select_pages for callers that cannot
 * allocate device memory (no counterpart in the reference, whose PyTorch
 * code always allocates through its caching allocator).  Same arguments
 * minus the workspace: scratch comes from a 16 MiB buffer compiled into the
 * library (one per GPU, held until the process exits), so requests with
 * ls_select_pages_workspace_bytes(total_q, G, max_seqlen_q) above 16 MiB
 * (e.g. one 2-group sequence longer than 16384 tokens) return
 * LS_ERR_UNSUPPORTED, after the same argument checks as ls_select_pages.
 * Each call looks up the buffer's device address on the current device;
 * the first lookup on a device loads the library's device code there, so
 * make the first call on each device before any stream capture.  Calls
 * share the buffer: calls that overlap on the GPU race, so serialise them.
 */
int ls_select_pages_noalloc(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                            const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_c,
                            int32_t batch, int32_t max_seqlen_q, int64_t total_q,
                            int64_t total_c, int32_t num_heads, int32_t num_kv_heads,
                            int32_t head_dim, int32_t width, int32_t take, int32_t init_blocks,
                            int32_t local_blocks, int32_t block_size, int32_t kernel_stride,
                            int32_t* topk_idx, int32_t* status, void* stream);

/*
 * ls_compress_keys_f32 -- ls_compress_keys for fp32 keys: CompressK.forward
 * on fp32 tensors (leanselect/models/minicpm.py:1169-1185), whose output
 * stays fp32.  k [total_k, G, D] fp32 -> k_compressed [total_c, G, D] fp32.
 * Each window is summed as kernel_size/kernel_stride runs of kernel_stride
 * keys (in order), the run sums added and the total scaled by
 * 1/kernel_size.  G*D must be a multiple of 4.
 */
int ls_compress_keys_f32(const float* k, const int32_t* cu_seqlens_k, int32_t batch,
                         int64_t total_k, int32_t num_kv_heads, int32_t head_dim,
                         int32_t kernel_size, int32_t kernel_stride, float* k_compressed,
                         int32_t* cu_seqlens_c, int64_t total_c, int32_t* status, void* stream);

/*
 * ls_select_pages_f32 -- ls_select_pages for fp32 inputs: the reference's
 * selection run on fp32 tensors (benchmark config 0), where the fused
 * weights, projections and scores are fp32 einsums (selector.py:144-214)
 * and the masking / top-k block is that of minicpm.py:3093-3141.  q
 * [total_q, H, D] fp32, q_fused [H, D, F] and kv_fused [G, D, F] fp32 (the
 * reference layout of ls_fold_weights), kc [total_c, G, D] fp32.  Output
 * and conventions as ls_select_pages (ascending pages, ties to the lower
 * page, -1 padding).  SIMT fp32 kernels; `workspace` (256-byte aligned)
 * holds ls_select_pages_f32_workspace_bytes(...) bytes: Qs and Ks fp32 and
 * one fp32 score per (group, row, page).  Requires D == F == 128,
 * block_size == 64, kernel_stride == 16, take <= LS_MAX_TOPK.
 */
size_t ls_select_pages_f32_workspace_bytes(int64_t total_q, int64_t total_c, int32_t num_kv_heads,
                                           int32_t max_seqlen_q);
int ls_select_pages_f32(const float* q, const float* q_fused, const float* kc,
                        const float* kv_fused, const int32_t* cu_seqlens_q,
                        const int32_t* cu_seqlens_c, int32_t batch, int32_t max_seqlen_q,
                        int64_t total_q, int64_t total_c, int32_t num_heads, int32_t num_kv_heads,
                        int32_t head_dim, int32_t width, int32_t take, int32_t init_blocks,
                        int32_t local_blocks, int32_t block_size, int32_t kernel_stride,
                        int32_t* topk_idx, void* workspace, size_t workspace_bytes,
                        int32_t* status, void* stream);

/*
 * ls_uniform_select_pages -- replaces uniform_prefill_topk_idx
 * (leanselect/ops/uniform.py:185-320), the uniform-method selection that
 * MiniCPMInfLLMv2Attention._lightweight_compressed_attention dispatches to
 * when selection_method == "uniform" (minicpm.py:3073-3087).  Scores are
 * mean(group query heads) . Kc * softmax_scale (0 = head_dim^-0.5), kept
 * in bf16 like the reference's bf16 matmul (head_mix.py:21-77); atoms after
 * the query are hidden, pages max-pooled, sink + local pages forced, and
 * the top `take` = min(topk, max pages) taken over all pages, a pick of
 * page q_page+1 leaving its slot -1 (uniform.py:68-112).  kc is the
 * compressed-key tensor [total_c, G, D] bf16 itself.  Rows are written sink
 * pages, selected pages, local pages -- ascending -- then -1 (the
 * reference orders by score; the sets are the same).  `workspace` holds
 * ls_uniform_select_workspace_bytes(...) bytes.  The reference rejects query
 * lengths <= 1 on the host; this entry point does not look at them.
 */
size_t ls_uniform_select_workspace_bytes(int64_t total_q, int64_t total_c, int32_t num_heads,
                                         int32_t num_kv_heads, int32_t max_seqlen_q);
int ls_uniform_select_pages(const uint16_t* q, const uint16_t* kc, const int32_t* cu_seqlens_q,
                            const int32_t* cu_seqlens_c, int32_t batch, int32_t max_seqlen_q,
                            int64_t total_q, int64_t total_c, int32_t num_heads,
                            int32_t num_kv_heads, int32_t head_dim, int32_t take,
                            int32_t init_blocks, int32_t local_blocks, int32_t block_size,
                            int32_t kernel_stride, float softmax_scale, int32_t* topk_idx,
                            void* workspace, size_t workspace_bytes, int32_t* status,
                            void* stream);

/*
 * ls_select_pages_chunk -- ls_select_pages for a slice of ONE sequence, used
 * by the sequence-parallel prefill (no reference counterpart: the reference
 * prefill runs on one GPU).  q holds chunk_q query rows at positions
 * [q_position, q_position + chunk_q) of a sequence of seq_len tokens whose
 * total_c atoms are all of ks [G, total_c, F].  Visibility, forced pages and
 * the output width `take` follow ls_select_pages with P = ceil(seq_len/64);
 * `workspace` holds ls_select_pages_workspace_bytes(chunk_q, G, seq_len) bytes.
 */
int ls_select_pages_chunk(const uint16_t* q, const uint16_t* wq_t, const uint16_t* ks,
                          int64_t chunk_q, int32_t q_position, int32_t seq_len, int64_t total_c,
                          int32_t num_heads, int32_t num_kv_heads, int32_t head_dim, int32_t width,
                          int32_t take, int32_t init_blocks, int32_t local_blocks,
                          int32_t block_size, int32_t kernel_stride, int32_t* topk_idx,
                          void* workspace, size_t workspace_bytes, int32_t* status,
                          void* stream);

/*
 * ls_sparse_attn -- replaces infllmv2_attn_varlen_func(..., topk_idx=)
 * (called at leanselect/models/minicpm.py:3229-3243; InfLLM-v2 varlen_fwd
 * with a block mask, third_party/infllmv2/paper1.patch).
 *
 * For packed query t of sequence b and head h (group g = h / (H/G)):
 *   out[t, h] = softmax_k(scale * q[t,h]·k[k,g]) v[k,g]
 * over keys k of sequence b lying in a page listed in topk_idx[g, t, :]
 * (entries < 0 are empty, duplicates count once) and, with causal != 0, at
 * relative position <= t_rel + (N_k - N_q).  Rows with no key output zeros
 * (lse = +inf).  q [total_q, H, D], k/v [total_k, G, D], out [total_q, H, D]
 * bf16; lse [H, total_q] fp32 (nullable); scale <= 0 selects D^-0.5.
 * Requires D == 128, H/G in {8, 16}, block_size == 64, topk <= LS_MAX_TOPK.
 * When the status word reports LS_DEVERR_TIMEOUT, the rows whose CTA gave
 * up are left unwritten in out and lse (their contents are undefined).
 */
int ls_sparse_attn(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                   const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t batch,
                   int32_t max_seqlen_q, int32_t max_seqlen_k, int64_t total_q, int64_t total_k,
                   int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                   const int32_t* topk_idx, int32_t topk, int32_t block_size,
                   float softmax_scale, int32_t causal, uint16_t* out, float* lse,
                   int32_t* status, void* stream);

/*
 * ls_sparse_attn_split -- ls_sparse_attn for few query rows, such as a decode
 * step (the same infllmv2_attn_varlen_func call with max_seqlen_q == 1 and
 * causal == 0, minicpm.py:3229-3243).  One CTA per (token, group) leaves
 * most of the GPU idle when there are few tokens; here each row's sorted,
 * de-duplicated page list is cut into `splits` contiguous slices (1 ..
 * LS_MAX_ATTN_SPLITS), one CTA each, and a second kernel combines the
 * slices' partial softmax results (each slice's output weighted by its share
 * of the row's exponential mass).  Same arguments and results as
 * ls_sparse_attn up to fp32 summation order; `workspace` holds
 * ls_sparse_attn_split_workspace_bytes(total_q, H, splits) bytes
 * (16-byte aligned; unused when splits == 1).
 */
size_t ls_sparse_attn_split_workspace_bytes(int64_t total_q, int32_t num_heads, int32_t splits);
int ls_sparse_attn_split(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k, int32_t batch,
                         int32_t max_seqlen_q, int32_t max_seqlen_k, int64_t total_q,
                         int64_t total_k, int32_t num_heads, int32_t num_kv_heads,
                         int32_t head_dim, const int32_t* topk_idx, int32_t topk,
                         int32_t block_size, float softmax_scale, int32_t causal, int32_t splits,
                         void* workspace, size_t workspace_bytes, uint16_t* out, float* lse,
                         int32_t* status, void* stream);

/*
 * ls_sparse_attn_gather_only -- measurement twin of ls_sparse_attn (no
 * reference counterpart).  Runs the same grid over the same page lists and
 * moves the same K/V pages from L2 into shared memory through the same TMA
 * ring, but computes and writes nothing: its duration is the gather time
 * that bounds ls_sparse_attn on the caller's inputs (the kernel's measured
 * roofline).  Arguments as ls_sparse_attn without scale and outputs.
 */
int ls_sparse_attn_gather_only(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                               const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                               int32_t batch, int32_t max_seqlen_q, int32_t max_seqlen_k,
                               int64_t total_q, int64_t total_k, int32_t num_heads,
                               int32_t num_kv_heads, int32_t head_dim, const int32_t* topk_idx,
                               int32_t topk, int32_t block_size, int32_t causal, int32_t* status,
                               void* stream);

/*
 * ls_wait_timeout_probe -- test hook for the bounded waits (no reference
 * counterpart).  Launches one CTA that allocates tensor memory and waits on
 * an mbarrier that nothing completes, for timeout_ns (1 us .. 2 s), then
 * unwinds the way every kernel of this library does when a wait expires:
 * LS_DEVERR_TIMEOUT is OR-ed into *status (device int32), the other warps
 * leave through the CTA's abort flag, the tensor memory is released and the
 * kernel returns, writing 1 to *done (device int32).  The context stays
 * usable; nothing traps.
 */
int ls_wait_timeout_probe(int32_t* status, int32_t* done, uint64_t timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LEANSELECT_B200_H_ */
