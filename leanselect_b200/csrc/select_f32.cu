// The selection path on fp32 inputs (benchmark config 0).
//
// The reference computes LeanSelect's selection in the dtype of its inputs:
// fp32 keys are compressed in fp32 (CompressK, minicpm.py:1169-1185), the
// selector's fused weights stay fp32 (selector.py:144-158) and the
// projections and scores are fp32 einsums (selector.py:160-214).  Rounding
// such inputs to bf16 changes which pages win in a sizeable share of rows,
// so fp32 inputs take this path: SIMT fp32 kernels (fp32 FMA accumulation;
// tf32 tensor-core products would round the operands to 10 mantissa bits).
//
//   compress_keys_f32_kernel  mean of each 32/16 window, fp32
//   project_f32_kernel        Qs = Q x q_fused, Ks = Kc x kv_fused per group
//   score_f32_kernel          Qs x Ks^T for the causally reachable atom tiles,
//                             max-pooled into pages (window 5, stride 4, pad 1)
//   topk_f32_kernel           visibility, forced pages and the exact top-T'
//                             (range radix on 32-bit order-preserving keys)
//
// It is the exactness path, not the fast one: the bf16 path of
// score_select.cu serves the model.
#include <algorithm>
#include <cmath>
#include <cstdio>

#include "common.cuh"
#include "launch.h"
#include "topk_rows.cuh"

namespace ls {
namespace {

// ---------------------------------------------------------------------------
// Compression: one thread per (atom, 4 channels), runs of `run_len` keys
// summed in order, the run sums added, scaled by 1/kernel_size (the oracle's
// order).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) compress_keys_f32_kernel(
    const float4* __restrict__ k, const int32_t* __restrict__ cu_k, const int32_t* __restrict__ cu_c,
    int batch, int64_t total_k, int64_t total_c, int vecs_per_row, int runs, int run_len,
    int stride, float inv_kernel, float4* __restrict__ kc, int32_t* status) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t atom = gid / vecs_per_row;
  const int vec = static_cast<int>(gid % vecs_per_row);
  if (atom >= total_c) return;
  const int b = find_sequence(cu_c, batch, atom);
  const int64_t local = atom - __ldg(cu_c + b);
  const int64_t tok0 = __ldg(cu_k + b) + local * stride;
  if (tok0 + static_cast<int64_t>(runs) * run_len > total_k) {
    report(status, LS_DEVERR_SEQLENS);
    return;
  }
  const float4* src = k + tok0 * vecs_per_row + vec;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < runs; ++j) {
    float4 run = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int t = 0; t < run_len; ++t) {
      const float4 u = __ldg(src + (static_cast<int64_t>(j) * run_len + t) * vecs_per_row);
      run.x += u.x;
      run.y += u.y;
      run.z += u.z;
      run.w += u.w;
    }
    acc.x += run.x;
    acc.y += run.y;
    acc.z += run.z;
    acc.w += run.w;
  }
  kc[atom * vecs_per_row + vec] =
      make_float4(acc.x * inv_kernel, acc.y * inv_kernel, acc.z * inv_kernel, acc.w * inv_kernel);
}

// ---------------------------------------------------------------------------
// Projection: out[g, row, f] = sum_k a[row * lda + g * K + k] * w[(g * K + k) * 128 + f].
// A CTA computes 64 rows x 128 outputs, a thread 4 rows x 8 outputs, in
// K-chunks of 16 staged in shared memory.
// ---------------------------------------------------------------------------
constexpr int kPRows = 64;
constexpr int kPK = 16;

__global__ void __launch_bounds__(256) project_f32_kernel(const float* __restrict__ a, int64_t rows,
                                                          int64_t lda, int K,
                                                          const float* __restrict__ w,
                                                          float* __restrict__ out) {
  __shared__ __align__(16) float a_s[kPK][kPRows];
  __shared__ __align__(16) float w_s[kPK][128];
  const int g = blockIdx.y;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kPRows;
  const int tr = threadIdx.x >> 4, tf = threadIdx.x & 15;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += kPK) {
    for (int i = threadIdx.x; i < kPK * kPRows; i += 256) {
      const int r = i / kPK, kk = i % kPK;
      a_s[kk][r] = row0 + r < rows ? a[(row0 + r) * lda + static_cast<int64_t>(g) * K + k0 + kk] : 0.f;
    }
    for (int i = threadIdx.x; i < kPK * 128; i += 256) {
      const int kk = i / 128, f = i % 128;
      w_s[kk][f] = w[(static_cast<int64_t>(g) * K + k0 + kk) * 128 + f];
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kPK; ++kk) {
      const float4 av = *reinterpret_cast<const float4*>(&a_s[kk][tr * 4]);
      const float4 w0 = *reinterpret_cast<const float4*>(&w_s[kk][tf * 8]);
      const float4 w1 = *reinterpret_cast<const float4*>(&w_s[kk][tf * 8 + 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w};
      const float wr[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(ar[i], wr[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = row0 + tr * 4 + i;
    if (r < rows) {
      float* dst = out + (static_cast<int64_t>(g) * rows + r) * 128 + tf * 8;
      *reinterpret_cast<float4*>(dst) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
    }
  }
}

// ---------------------------------------------------------------------------
// Scores: one CTA per (64 query rows of one sequence, group).  For each tile
// of 128 atoms up to the causal limit of the tile's last row it computes the
// 64 x 128 fp32 scores (F-chunks of 32 staged in shared memory, a thread 4
// rows x 8 atoms), parks them in shared memory and max-pools them into 32
// pages per row; page p's window is atoms [4p-1, 4p+4), so a row carries its
// last atom into the next tile.
// ---------------------------------------------------------------------------
constexpr int kSRows = 64;
constexpr int kSAtoms = 128;
constexpr int kSF = 32;

struct ScoreF32Smem {
  float q[kSF][kSRows];
  float k[kSF][kSAtoms];
  float s[kSRows][kSAtoms + 1];
  float carry[kSRows];
};

__global__ void __launch_bounds__(256) score_f32_kernel(const __grid_constant__ ScoreArgs args,
                                                        const float* __restrict__ qs,
                                                        const float* __restrict__ ks,
                                                        float* __restrict__ ws) {
  extern __shared__ __align__(16) uint8_t score_f32_smem[];
  ScoreF32Smem* sm = reinterpret_cast<ScoreF32Smem*>(score_f32_smem);
  const int tiles_max = (args.max_seqlen_q + kSRows - 1) / kSRows;
  const int64_t bid = blockIdx.x;
  const int g = static_cast<int>(bid % args.num_groups);
  const int b = static_cast<int>((bid / args.num_groups) % args.batch);
  const int tile = tiles_max - 1 - static_cast<int>(bid / (static_cast<int64_t>(args.num_groups) * args.batch));
  const int64_t q0 = args.cu_q ? __ldg(args.cu_q + b) : 0;
  const int n = args.cu_q ? static_cast<int>(__ldg(args.cu_q + b + 1) - q0) : args.max_seqlen_q;
  if (n > args.max_seqlen_q) {
    if (tile == 0 && threadIdx.x == 0) report(args.status, LS_DEVERR_SEQLENS);
    return;
  }
  const int row0 = tile * kSRows;
  if (row0 >= n) return;
  const int rows = min(kSRows, n - row0);
  const int64_t c0 = args.cu_c ? __ldg(args.cu_c + b) : 0;
  const int atoms = args.cu_c ? static_cast<int>(__ldg(args.cu_c + b + 1) - c0)
                              : static_cast<int>(args.total_c);
  // Candidates of the tile's last row are pages p <= qp_max - local - 1, whose
  // windows end at atom 4p + 3 < 4 (qp_max - local).
  const int qp_max = (args.pos_offset + row0 + rows - 1) / 64;
  const int needed = max(0, min(atoms, 4 * (qp_max - args.local_blocks)));
  const int atom_tiles = (needed + kSAtoms - 1) / kSAtoms;
  if (atom_tiles == 0) return;
  const int tr = threadIdx.x >> 4, ta = threadIdx.x & 15;
  if (threadIdx.x < kSRows) sm->carry[threadIdx.x] = -INFINITY;
  for (int j = 0; j < atom_tiles; ++j) {
    const int a0 = j * kSAtoms;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[i][c] = 0.f;
    for (int f0 = 0; f0 < 128; f0 += kSF) {
      __syncthreads();
      for (int i = threadIdx.x; i < kSF * kSRows; i += 256) {
        const int r = i / kSF, f = i % kSF;
        sm->q[f][r] = r < rows ? qs[(static_cast<int64_t>(g) * args.total_q + q0 + row0 + r) * 128 + f0 + f]
                               : 0.f;
      }
      for (int i = threadIdx.x; i < kSF * kSAtoms; i += 256) {
        const int a = i / kSF, f = i % kSF;
        sm->k[f][a] = a0 + a < atoms
                          ? ks[(static_cast<int64_t>(g) * args.total_c + c0 + a0 + a) * 128 + f0 + f]
                          : 0.f;
      }
      __syncthreads();
#pragma unroll 8
      for (int f = 0; f < kSF; ++f) {
        const float4 qv = *reinterpret_cast<const float4*>(&sm->q[f][tr * 4]);
        const float4 k0 = *reinterpret_cast<const float4*>(&sm->k[f][ta * 8]);
        const float4 k1 = *reinterpret_cast<const float4*>(&sm->k[f][ta * 8 + 4]);
        const float qr[4] = {qv.x, qv.y, qv.z, qv.w};
        const float kr[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 8; ++c) acc[i][c] = fmaf(qr[i], kr[c], acc[i][c]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        sm->s[tr * 4 + i][ta * 8 + c] = a0 + ta * 8 + c < atoms ? acc[i][c] : -INFINITY;
    __syncthreads();
    // Pool: 64 rows x 32 pages, 8 per thread.
    for (int i = threadIdx.x; i < kSRows * 32; i += 256) {
      const int r = i >> 5, pl = i & 31;
      const float* srow = sm->s[r];
      const float first = pl == 0 ? sm->carry[r] : srow[4 * pl - 1];
      const float v = fmaxf(fmaxf(first, fmaxf(srow[4 * pl], srow[4 * pl + 1])),
                            fmaxf(srow[4 * pl + 2], srow[4 * pl + 3]));
      const int p = j * 32 + pl;
      if (r < rows && p < args.max_pages)
        ws[(static_cast<int64_t>(g) * args.total_q + q0 + row0 + r) * args.max_pages + p] = v;
    }
    __syncthreads();
    if (threadIdx.x < kSRows) sm->carry[threadIdx.x] = sm->s[threadIdx.x][kSAtoms - 1];
  }
}

// ---------------------------------------------------------------------------
// Top-T' per (group, row), one warp per row, exact over the workspace row.
// ---------------------------------------------------------------------------
// Order-preserving key of an fp32 score; -inf and NaN map to 0 (never picked),
// -0 and +0 share a key.
__device__ __forceinline__ uint32_t f32_key(float x) {
  uint32_t u = __float_as_uint(x);
  u = u == 0x80000000u ? 0u : u;
  const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (k <= 0x007FFFFFu || k > 0xFF800000u) ? 0u : k;
}

struct F32RowKeys {
  const float* p;
  __device__ __forceinline__ uint32_t operator()(int i) const { return f32_key(__ldg(p + i)); }
};

constexpr int kTopkF32Warps = 8;

__global__ void __launch_bounds__(kTopkF32Warps * 32) topk_f32_kernel(const __grid_constant__ ScoreArgs args,
                                                                      const float* __restrict__ ws) {
  __shared__ uint32_t hist_all[kTopkF32Warps][256];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t* hist = hist_all[warp];
  const uint32_t total_q = static_cast<uint32_t>(args.total_q);
  const uint32_t rows_total = static_cast<uint32_t>(args.num_groups) * total_q;
  for (uint32_t r = blockIdx.x * kTopkF32Warps + warp; r < rows_total;
       r += gridDim.x * kTopkF32Warps) {
    int32_t* out;
    int64_t ws_row;
    bool empty;
    int m_all = 0, cap = 0, future = -1, n_init = 0, take_b = 0, local0 = 0, n_local = 0;
    row_geometry(args, r, total_q, &out, &ws_row, &empty, &m_all, &cap, &future, &n_init, &take_b,
                 &local0, &n_local);
    if (empty) {
      for (int k = lane; k < args.take; k += 32) out[k] = -1;
      continue;
    }
    const int sinks_out = min(n_init, take_b);
    for (int k = lane; k < sinks_out; k += 32) out[k] = k;
    int k_out = sinks_out;
    if (cap > 0) {
      const F32RowKeys keys{ws + ws_row + n_init};
      int finite = 0;
      for (int i = lane; i < m_all; i += 32) finite += keys(i) != 0u;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) finite += __shfl_xor_sync(0xffffffffu, finite, o);
      int need = cap;
      // With no more finite candidates than slots every finite one is taken:
      // threshold at the lowest possible key, all ties taken.
      const uint32_t thr = finite <= cap ? 1u : radix_threshold(keys, m_all, need, hist, lane);
      if (finite <= cap) need = m_all;
      k_out = emit_threshold(keys, Identity{}, m_all, thr, need, future, n_init, out, k_out, lane);
    }
    const int local_out = max(0, min(n_local, take_b - k_out));
    for (int k = lane; k < local_out; k += 32) out[k_out + k] = local0 + k;
    k_out += local_out;
    for (int k = k_out + lane; k < args.take; k += 32) out[k] = -1;
  }
}

size_t align256(size_t n) { return (n + 255) & ~size_t{255}; }

int fail(int code, const char* what) { return set_host_error(code, what); }

}  // namespace
}  // namespace ls

using namespace ls;

extern "C" {

int ls_compress_keys_f32(const float* k, const int32_t* cu_seqlens_k, int32_t batch,
                         int64_t total_k, int32_t num_kv_heads, int32_t head_dim,
                         int32_t kernel_size, int32_t kernel_stride, float* k_compressed,
                         int32_t* cu_seqlens_c, int64_t total_c, int32_t* status, void* stream) {
  if (!k || !cu_seqlens_k || !cu_seqlens_c) return fail(LS_ERR_INVALID_ARGUMENT, "null argument");
  if (batch < 1 || total_k < 0 || total_c < 0) return fail(LS_ERR_INVALID_ARGUMENT, "bad sizes");
  if (total_c > 0 && !k_compressed) return fail(LS_ERR_INVALID_ARGUMENT, "null k_compressed");
  if (num_kv_heads <= 0 || head_dim <= 0) return fail(LS_ERR_INVALID_ARGUMENT, "bad head geometry");
  if (kernel_size <= 0 || kernel_stride <= 0 || kernel_size % kernel_stride != 0)
    return fail(LS_ERR_UNSUPPORTED, "kernel_size must be a positive multiple of kernel_stride");
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (row % 4 != 0) return fail(LS_ERR_UNSUPPORTED, "num_kv_heads*head_dim must be a multiple of 4");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(k_compressed)) & 15u)
    return fail(LS_ERR_ALIGNMENT, "k or k_compressed is not 16-byte aligned");
  if (total_c > total_k / kernel_stride + batch)
    return fail(LS_ERR_INVALID_ARGUMENT, "total_c exceeds the possible atom count");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err =
      launch_compressed_seqlens(cu_seqlens_k, batch, kernel_size, kernel_stride, cu_seqlens_c,
                                status, s);
  if (err == cudaSuccess && total_c > 0) {
    const int vecs = static_cast<int>(row / 4);
    const int64_t threads = total_c * vecs;
    compress_keys_f32_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(
        reinterpret_cast<const float4*>(k), cu_seqlens_k, cu_seqlens_c, batch, total_k, total_c,
        vecs, kernel_size / compress_run_length(kernel_stride), compress_run_length(kernel_stride),
        kernel_stride, 1.0f / static_cast<float>(kernel_size),
        reinterpret_cast<float4*>(k_compressed), status);
    err = cudaGetLastError();
  }
  return err == cudaSuccess ? LS_OK : fail(LS_ERR_CUDA, cudaGetErrorString(err));
}

size_t ls_select_pages_f32_workspace_bytes(int64_t total_q, int64_t total_c, int32_t num_kv_heads,
                                           int32_t max_seqlen_q) {
  if (total_q <= 0 || total_c < 0 || num_kv_heads <= 0 || max_seqlen_q <= 0) return 0;
  const size_t g = static_cast<size_t>(num_kv_heads);
  const size_t pages = static_cast<size_t>(((max_seqlen_q + 63) / 64 + 7) & ~7);
  return align256(sizeof(float) * g * static_cast<size_t>(total_q) * 128) +
         align256(sizeof(float) * g * static_cast<size_t>(std::max<int64_t>(total_c, 1)) * 128) +
         sizeof(float) * g * static_cast<size_t>(total_q) * pages;
}

int ls_select_pages_f32(const float* q, const float* q_fused, const float* kc,
                        const float* kv_fused, const int32_t* cu_seqlens_q,
                        const int32_t* cu_seqlens_c, int32_t batch, int32_t max_seqlen_q,
                        int64_t total_q, int64_t total_c, int32_t num_heads, int32_t num_kv_heads,
                        int32_t head_dim, int32_t width, int32_t take, int32_t init_blocks,
                        int32_t local_blocks, int32_t block_size, int32_t kernel_stride,
                        int32_t* topk_idx, void* workspace, size_t workspace_bytes,
                        int32_t* status, void* stream) {
  if (!q || !q_fused || !kv_fused || !cu_seqlens_q || !cu_seqlens_c)
    return fail(LS_ERR_INVALID_ARGUMENT, "null argument");
  if (total_q < 0 || total_c < 0 || batch < 1 || max_seqlen_q < 0)
    return fail(LS_ERR_INVALID_ARGUMENT, "bad sizes");
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0)
    return fail(LS_ERR_INVALID_ARGUMENT, "num_heads must be a positive multiple of num_kv_heads");
  if (total_q * num_kv_heads >= (int64_t{1} << 31))
    return fail(LS_ERR_INVALID_ARGUMENT, "num_kv_heads * total_q out of range");
  if (take < 0 || init_blocks < 0 || local_blocks < 0)
    return fail(LS_ERR_INVALID_ARGUMENT, "negative budget");
  if (head_dim != 128 || width != 128)
    return fail(LS_ERR_UNSUPPORTED, "head_dim and selector width must be 128");
  if (block_size != 64 || kernel_stride != 16)
    return fail(LS_ERR_UNSUPPORTED, "block_size must be 64 and kernel_stride 16");
  if (take > LS_MAX_TOPK) return fail(LS_ERR_UNSUPPORTED, "take exceeds LS_MAX_TOPK");
  if (max_seqlen_q > 65536 * 64)
    return fail(LS_ERR_UNSUPPORTED, "sequences longer than 4M tokens are not supported");
  if (total_q == 0 || take == 0) return LS_OK;
  if (!topk_idx) return fail(LS_ERR_INVALID_ARGUMENT, "null topk_idx");
  if (total_c > 0 && !kc) return fail(LS_ERR_INVALID_ARGUMENT, "null kc");
  const size_t need = ls_select_pages_f32_workspace_bytes(total_q, total_c, num_kv_heads,
                                                          max_seqlen_q);
  if (!workspace || workspace_bytes < need)
    return fail(LS_ERR_INVALID_ARGUMENT, "workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(LS_ERR_ALIGNMENT, "workspace is not 256-byte aligned");
  const int G = num_kv_heads, hg = num_heads / num_kv_heads;
  uint8_t* base = static_cast<uint8_t*>(workspace);
  float* qs = reinterpret_cast<float*>(base);
  base += align256(sizeof(float) * G * static_cast<size_t>(total_q) * 128);
  float* ks = reinterpret_cast<float*>(base);
  base += align256(sizeof(float) * G * static_cast<size_t>(std::max<int64_t>(total_c, 1)) * 128);
  float* pages = reinterpret_cast<float*>(base);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Qs[g] = Q[:, g*Hg*D : (g+1)*Hg*D] x q_fused[g*Hg : (g+1)*Hg] viewed as [Hg*D, F].
  project_f32_kernel<<<dim3(static_cast<unsigned>((total_q + kPRows - 1) / kPRows), G), 256, 0, s>>>(
      q, total_q, static_cast<int64_t>(num_heads) * 128, hg * 128, q_fused, qs);
  cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess && total_c > 0) {
    project_f32_kernel<<<dim3(static_cast<unsigned>((total_c + kPRows - 1) / kPRows), G), 256, 0, s>>>(
        kc, total_c, static_cast<int64_t>(G) * 128, 128, kv_fused, ks);
    err = cudaGetLastError();
  }
  ScoreArgs a{};
  a.cu_q = cu_seqlens_q;
  a.cu_c = cu_seqlens_c;
  a.batch = batch;
  a.num_groups = G;
  a.hg = hg;
  a.max_seqlen_q = max_seqlen_q;
  a.total_q = total_q;
  a.total_c = total_c;
  a.take = take;
  a.init_blocks = init_blocks;
  a.local_blocks = local_blocks;
  a.max_pages = (((max_seqlen_q + 63) / 64) + 7) & ~7;
  a.topk_idx = topk_idx;
  a.status = status;
  if (err == cudaSuccess) {
    const int tiles_max = (max_seqlen_q + kSRows - 1) / kSRows;
    const int64_t grid = static_cast<int64_t>(tiles_max) * batch * G;
    err = cudaFuncSetAttribute(score_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(sizeof(ScoreF32Smem)));
    if (err == cudaSuccess && grid > 0 && total_c > 0) {
      score_f32_kernel<<<static_cast<unsigned>(grid), 256, sizeof(ScoreF32Smem), s>>>(a, qs, ks,
                                                                                      pages);
      err = cudaGetLastError();
    }
  }
  if (err == cudaSuccess) {
    const int64_t rows = static_cast<int64_t>(G) * total_q;
    const int64_t blocks = std::min<int64_t>((rows + kTopkF32Warps - 1) / kTopkF32Warps, 148 * 8);
    topk_f32_kernel<<<static_cast<unsigned>(blocks), kTopkF32Warps * 32, 0, s>>>(a, pages);
    err = cudaGetLastError();
  }
  return err == cudaSuccess ? LS_OK : fail(LS_ERR_CUDA, cudaGetErrorString(err));
}

}  // extern "C"
