// Streaming kernels of the selection path: selector weight folding, the
// compressed cu_seqlens, key compression (a1) and the atom-key projection (a4).
//
// These are HBM- or launch-bound SIMT kernels; the GEMM-shaped work lives in
// score_select.cu.
#include "common.cuh"
#include "launch.h"

#include <algorithm>

namespace ls {

// ---------------------------------------------------------------------------
// Weight folding (selector.py:144-158)
// ---------------------------------------------------------------------------

__global__ void fold_weights_kernel(const float* __restrict__ head_mix,
                                    const float* __restrict__ kv_head_mix,
                                    const float* __restrict__ q_proj,
                                    const float* __restrict__ k_proj, int H, int G, int D, int R,
                                    int r, float* q_f32, float* kv_f32, __nv_bfloat16* q_bf16,
                                    __nv_bfloat16* kv_bf16, __nv_bfloat16* wq_t,
                                    __nv_bfloat16* wk_t) {
  const int F = R * r;
  const int Hg = H / G;
  const int64_t nq = static_cast<int64_t>(H) * D * F;
  const int64_t nk = static_cast<int64_t>(G) * D * F;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nq + nk;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (i < nq) {
      // q_fused[h, d, f], f = rho * r + j
      const int f = static_cast<int>(i % F);
      const int d = static_cast<int>((i / F) % D);
      const int h = static_cast<int>(i / (static_cast<int64_t>(F) * D));
      const int rho = f / r, j = f % r;
      const float w = head_mix[h * R + rho] * q_proj[(static_cast<int64_t>(rho) * D + d) * r + j];
      if (q_f32) q_f32[i] = w;
      const __nv_bfloat16 wb = __float2bfloat16_rn(w);
      if (q_bf16) q_bf16[i] = wb;
      if (wq_t) {
        const int g = h / Hg, s = h % Hg;
        wq_t[(static_cast<int64_t>(g) * F + f) * (Hg * D) + s * D + d] = wb;
      }
    } else {
      const int64_t k = i - nq;
      const int f = static_cast<int>(k % F);
      const int d = static_cast<int>((k / F) % D);
      const int g = static_cast<int>(k / (static_cast<int64_t>(F) * D));
      const int rho = f / r, j = f % r;
      const float w =
          kv_head_mix[g * R + rho] * k_proj[(static_cast<int64_t>(rho) * D + d) * r + j];
      if (kv_f32) kv_f32[k] = w;
      const __nv_bfloat16 wb = __float2bfloat16_rn(w);
      if (kv_bf16) kv_bf16[k] = wb;
      if (wk_t) wk_t[(static_cast<int64_t>(g) * F + f) * D + d] = wb;
    }
  }
}

// ---------------------------------------------------------------------------
// Compressed cu_seqlens (minicpm.py:710-750)
// ---------------------------------------------------------------------------

__global__ void compressed_seqlens_kernel(const int32_t* __restrict__ cu_k, int batch,
                                          int kernel_size, int kernel_stride,
                                          int32_t* __restrict__ cu_c, int32_t* status) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) {
    carry = 0;
    cu_c[0] = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int base = 0; base < batch; base += blockDim.x) {
    const int b = base + threadIdx.x;
    int32_t count = 0;
    if (b < batch) {
      const int32_t n = cu_k[b + 1] - cu_k[b];
      if (n < 0) report(status, LS_DEVERR_SEQLENS);
      count = n >= kernel_size ? (n - kernel_size) / kernel_stride + 1 : 0;
    }
    int32_t incl = count;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int nw = blockDim.x >> 5;
      int32_t w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t v = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += v;
      }
      if (lane < nw) warp_sums[lane] = w;
    }
    __syncthreads();
    const int32_t prefix = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + incl;
    if (b < batch) cu_c[b + 1] = prefix;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = prefix;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Key compression (CompressK.forward, minicpm.py:1169-1185)
// ---------------------------------------------------------------------------
//
// One thread per (packed atom, 16-byte vector of 8 channels).  Consecutive
// threads cover one key row (512 bytes for G*D = 256), so every load is a
// fully coalesced row.  A thread sums its window as runs of `run_len` keys
// (16 when 16 divides the stride, each run sequentially in fp32), adds the
// run sums in order, scales by 1/kernel_size and rounds to bf16 -- the
// oracle's order, so results match it bit for bit.  Each key is read by
// several atoms; the later reads of a run hit L2.

__global__ void __launch_bounds__(256) compress_keys_kernel(
    const uint4* __restrict__ k, const int32_t* __restrict__ cu_k, const int32_t* __restrict__ cu_c,
    int batch, int64_t total_k, int64_t total_c, int vecs_per_row, int runs, int run_len,
    int stride, float inv_kernel, uint4* __restrict__ kc, int32_t* status) {
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
  const uint4* src = k + tok0 * vecs_per_row + vec;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.f;
  for (int j = 0; j < runs; ++j) {
    float run[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) run[c] = 0.f;
#pragma unroll 4
    for (int t = 0; t < run_len; ++t) {
      const uint4 u = __ldg(src + (static_cast<int64_t>(j) * run_len + t) * vecs_per_row);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float2 f = __bfloat1622float2(h[c]);
        run[2 * c] += f.x;
        run[2 * c + 1] += f.y;
      }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] += run[c];
  }
  uint4 out;
  out.x = pack_bf16x2(acc[0] * inv_kernel, acc[1] * inv_kernel);
  out.y = pack_bf16x2(acc[2] * inv_kernel, acc[3] * inv_kernel);
  out.z = pack_bf16x2(acc[4] * inv_kernel, acc[5] * inv_kernel);
  out.w = pack_bf16x2(acc[6] * inv_kernel, acc[7] * inv_kernel);
  kc[atom * vecs_per_row + vec] = out;
}

// ---------------------------------------------------------------------------
// Uniform method inputs (ops/uniform.py, pages.py:62-71)
// ---------------------------------------------------------------------------

// One pass of 16-byte vectors: the first `w_vecs` write the mean-query
// weight wq_t[g, f, s*D + d] = (d == f) / Hg, the rest copy Kc[a, g, :] to
// Ks[g, a, :].  With Hg a power of two, Q x wq_t is the exact group mean
// before its bf16 rounding, which is how the reference's bf16 mean rounds.
__global__ void __launch_bounds__(256) uniform_prep_kernel(const uint4* __restrict__ kc,
                                                           int64_t total_c, int G, int hg,
                                                           uint4* __restrict__ wq_t,
                                                           uint4* __restrict__ ks) {
  constexpr int D = 128, V = D / 8;
  const int64_t w_vecs = static_cast<int64_t>(G) * D * hg * V;
  const int64_t k_vecs = total_c * G * V;
  const uint16_t inv = __bfloat16_as_ushort(__float2bfloat16_rn(1.0f / static_cast<float>(hg)));
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < w_vecs + k_vecs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (i < w_vecs) {
      const int f = static_cast<int>((i / (static_cast<int64_t>(hg) * V)) % D);
      const int d0 = static_cast<int>(i % V) * 8;  // d of the vector's first element
      uint32_t w[4] = {0u, 0u, 0u, 0u};
      if (f >= d0 && f < d0 + 8) {
        const int e = f - d0;
        w[e >> 1] = static_cast<uint32_t>(inv) << (16 * (e & 1));
      }
      wq_t[i] = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      const int64_t j = i - w_vecs;
      const int c = static_cast<int>(j % V);
      const int64_t ag = j / V;  // a * G + g
      const int64_t a = ag / G;
      const int g = static_cast<int>(ag % G);
      ks[(static_cast<int64_t>(g) * total_c + a) * V + c] = kc[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

cudaError_t launch_uniform_prep(const uint16_t* kc, int64_t total_c, int num_kv_heads, int hg,
                                uint16_t* wq_t, uint16_t* ks, cudaStream_t stream) {
  const int64_t vecs = (static_cast<int64_t>(num_kv_heads) * 128 * hg + total_c * num_kv_heads) * 16;
  const int blocks = static_cast<int>(std::min<int64_t>((vecs + 255) / 256, 148 * 8));
  uniform_prep_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const uint4*>(kc), total_c,
                                                  num_kv_heads, hg, reinterpret_cast<uint4*>(wq_t),
                                                  reinterpret_cast<uint4*>(ks));
  return cudaGetLastError();
}

cudaError_t launch_fold_weights(const float* head_mix, const float* kv_head_mix,
                                const float* q_proj, const float* k_proj, int H, int G, int D,
                                int R, int r, float* q_f32, float* kv_f32, uint16_t* q_bf16,
                                uint16_t* kv_bf16, uint16_t* wq_t, uint16_t* wk_t,
                                cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(H + G) * D * R * r;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
  fold_weights_kernel<<<blocks, 256, 0, stream>>>(
      head_mix, kv_head_mix, q_proj, k_proj, H, G, D, R, r, q_f32, kv_f32,
      reinterpret_cast<__nv_bfloat16*>(q_bf16), reinterpret_cast<__nv_bfloat16*>(kv_bf16),
      reinterpret_cast<__nv_bfloat16*>(wq_t), reinterpret_cast<__nv_bfloat16*>(wk_t));
  return cudaGetLastError();
}

cudaError_t launch_compressed_seqlens(const int32_t* cu_k, int batch, int kernel_size,
                                      int kernel_stride, int32_t* cu_c, int32_t* status,
                                      cudaStream_t stream) {
  compressed_seqlens_kernel<<<1, 1024, 0, stream>>>(cu_k, batch, kernel_size, kernel_stride,
                                                     cu_c, status);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Both compressions of a prefill in one pass over K (get_compress_k,
// minicpm.py:2774-2810: compress_k with kernel 32 / stride 16 and compress_k2
// with kernel 128 / stride 64)
// ---------------------------------------------------------------------------
//
// A CTA takes 8 consecutive 64-key blocks of one sequence and 16 of the
// 16-byte vectors of a key row (256 bytes).  Phase 1: every thread sums
// 16-key runs of one vector (each run sequentially in fp32, 16 loads in
// flight), the 32 runs of the CTA's blocks plus the next block's first 4,
// into shared memory.  Phase 2: the 32/16 atom a is runs a and a+1 added,
// the 128/64 atom b is runs 4b .. 4b+7 added in order, both scaled and
// rounded to bf16 -- the order of compress_keys_kernel for both geometries,
// so either compressor gives the same bits.  K is read 1.125 times, where
// two separate compressions read it three times.
constexpr int kDualBlocks = 8;                   // 64-key blocks per CTA
constexpr int kDualVecs = 16;                    // 16-byte vectors per CTA
constexpr int kDualRuns = 4 * kDualBlocks + 4;   // + the next block's first 4 runs

__global__ void __launch_bounds__(256) compress_keys_dual_kernel(
    const uint4* __restrict__ k, const int32_t* __restrict__ cu_k, const int32_t* __restrict__ cu_c,
    const int32_t* __restrict__ cu_c2, int64_t total_k, int vecs_per_row,
    uint4* __restrict__ kc, uint4* __restrict__ kc2, int32_t* status) {
  __shared__ float4 runs[kDualRuns][kDualVecs][2];  // 18 KB: 8 fp32 sums per (run, vector)
  const int b = blockIdx.y;
  const int blk0 = static_cast<int>(blockIdx.x) * kDualBlocks;
  const int vec0 = static_cast<int>(blockIdx.z) * kDualVecs;
  const int64_t k0 = __ldg(cu_k + b), k1 = __ldg(cu_k + b + 1);
  const int64_t c0 = __ldg(cu_c + b), c20 = __ldg(cu_c2 + b);
  const int atoms = static_cast<int>(__ldg(cu_c + b + 1) - c0);
  const int atoms2 = static_cast<int>(__ldg(cu_c2 + b + 1) - c20);
  // A 128/64 atom b needs keys [64b, 64b+128), so it implies the 32/16 atom 4b.
  if (4 * blk0 >= atoms) return;
  if (k1 > total_k || k1 < k0) {
    if (threadIdx.x == 0) report(status, LS_DEVERR_SEQLENS);
    return;
  }
  const int64_t n_runs = (k1 - k0) / 16;  // complete 16-key runs of the sequence
  const int r0 = 4 * blk0;
  for (int item = threadIdx.x; item < kDualRuns * kDualVecs; item += blockDim.x) {
    const int rr = item / kDualVecs, v = item % kDualVecs;
    float run[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) run[c] = 0.f;
    if (r0 + rr < n_runs && vec0 + v < vecs_per_row) {
      const uint4* src = k + (k0 + 16 * static_cast<int64_t>(r0 + rr)) * vecs_per_row + vec0 + v;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const uint4 u = __ldg(src + static_cast<int64_t>(t) * vecs_per_row);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 f = __bfloat1622float2(h[c]);
          run[2 * c] += f.x;
          run[2 * c + 1] += f.y;
        }
      }
    }
    runs[rr][v][0] = make_float4(run[0], run[1], run[2], run[3]);
    runs[rr][v][1] = make_float4(run[4], run[5], run[6], run[7]);
  }
  __syncthreads();
  // 32/16 atoms r0 + i: runs i and i + 1.
  for (int item = threadIdx.x; item < 4 * kDualBlocks * kDualVecs; item += blockDim.x) {
    const int i = item / kDualVecs, v = item % kDualVecs;
    const int a = r0 + i;
    if (a >= atoms || vec0 + v >= vecs_per_row) continue;
    const float4 p0 = runs[i][v][0], p1 = runs[i][v][1];
    const float4 n0 = runs[i + 1][v][0], n1 = runs[i + 1][v][1];
    const float s = 1.f / 32.f;
    uint4 out;
    out.x = pack_bf16x2(((0.f + p0.x) + n0.x) * s, ((0.f + p0.y) + n0.y) * s);
    out.y = pack_bf16x2(((0.f + p0.z) + n0.z) * s, ((0.f + p0.w) + n0.w) * s);
    out.z = pack_bf16x2(((0.f + p1.x) + n1.x) * s, ((0.f + p1.y) + n1.y) * s);
    out.w = pack_bf16x2(((0.f + p1.z) + n1.z) * s, ((0.f + p1.w) + n1.w) * s);
    kc[(c0 + a) * vecs_per_row + vec0 + v] = out;
  }
  // 128/64 atoms blk0 + j: runs 4j .. 4j + 7 in order.
  for (int item = threadIdx.x; item < kDualBlocks * kDualVecs; item += blockDim.x) {
    const int j = item / kDualVecs, v = item % kDualVecs;
    if (blk0 + j >= atoms2 || vec0 + v >= vecs_per_row) continue;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 x0 = runs[4 * j + q][v][0], x1 = runs[4 * j + q][v][1];
      acc[0] += x0.x;
      acc[1] += x0.y;
      acc[2] += x0.z;
      acc[3] += x0.w;
      acc[4] += x1.x;
      acc[5] += x1.y;
      acc[6] += x1.z;
      acc[7] += x1.w;
    }
    const float s = 1.f / 128.f;
    uint4 out;
    out.x = pack_bf16x2(acc[0] * s, acc[1] * s);
    out.y = pack_bf16x2(acc[2] * s, acc[3] * s);
    out.z = pack_bf16x2(acc[4] * s, acc[5] * s);
    out.w = pack_bf16x2(acc[6] * s, acc[7] * s);
    kc2[(c20 + blk0 + j) * vecs_per_row + vec0 + v] = out;
  }
}

cudaError_t launch_compress_keys_dual(const uint16_t* k, const int32_t* cu_k, const int32_t* cu_c,
                                      const int32_t* cu_c2, int batch, int max_atoms,
                                      int64_t total_k, int G, int D, uint16_t* kc, uint16_t* kc2,
                                      int32_t* status, cudaStream_t stream) {
  if (max_atoms <= 0) return cudaSuccess;
  const int vecs = G * D / 8;
  const int blocks64 = (max_atoms + 3) / 4;
  const dim3 grid(static_cast<unsigned>((blocks64 + kDualBlocks - 1) / kDualBlocks),
                  static_cast<unsigned>(batch),
                  static_cast<unsigned>((vecs + kDualVecs - 1) / kDualVecs));
  compress_keys_dual_kernel<<<grid, 256, 0, stream>>>(
      reinterpret_cast<const uint4*>(k), cu_k, cu_c, cu_c2, total_k, vecs,
      reinterpret_cast<uint4*>(kc), reinterpret_cast<uint4*>(kc2), status);
  return cudaGetLastError();
}

cudaError_t launch_compress_keys(const uint16_t* k, const int32_t* cu_k, const int32_t* cu_c,
                                 int batch, int64_t total_k, int64_t total_c, int G, int D,
                                 int kernel_size, int kernel_stride, uint16_t* kc,
                                 int32_t* status, cudaStream_t stream) {
  if (total_c == 0) return cudaSuccess;
  const int vecs = G * D / 8;
  const int64_t threads = total_c * vecs;
  const int64_t blocks = (threads + 255) / 256;
  const int run_len = compress_run_length(kernel_stride);
  compress_keys_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      reinterpret_cast<const uint4*>(k), cu_k, cu_c, batch, total_k, total_c, vecs,
      kernel_size / run_len, run_len, kernel_stride, 1.0f / static_cast<float>(kernel_size),
      reinterpret_cast<uint4*>(kc), status);
  return cudaGetLastError();
}

}  // namespace ls
