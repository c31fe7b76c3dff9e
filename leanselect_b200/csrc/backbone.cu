// Fused elementwise kernels for the MiniCPM-shaped benchmark host model.
//
// These are not part of the LeanSelect hot path; they replace chains of
// PyTorch elementwise launches around the cuBLAS projections of the host
// model (RMSNorm, LongRoPE + q/k/v split, SiLU-gated product), each a single
// HBM pass with fp32 math.
#include "common.cuh"
#include "launch.h"
#include "../../include/leanselect_b200_backbone.h"

namespace ls {
namespace {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float2 t = __bfloat1622float2(h[c]);
    f[2 * c] = t.x;
    f[2 * c + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

// y = x * rsqrt(mean(x^2) + eps) * w, one CTA (256 threads) per row, fp32 math
// (the reference's rms_layernorm, minicpm.py:772-798).
template <int VPT>
__global__ void __launch_bounds__(256) rms_norm_kernel(const uint4* __restrict__ x,
                                                       const uint4* __restrict__ w, float eps,
                                                       int vecs, uint4* __restrict__ y) {
  const int64_t row = blockIdx.x;
  const uint4* xr = x + row * vecs;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c < vecs) {
      unpack8(__ldg(xr + c), v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[i][e], v[i][e], ss);
    }
  }
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) total += red[i];
  const float inv = rsqrtf(total / static_cast<float>(vecs * 8) + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c < vecs) {
      float wf[8];
      unpack8(__ldg(w + c), wf);
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[i][e] * inv * wf[e];
      y[row * vecs + c] = pack8(o);
    }
  }
}

// Rotary embedding (rotate_half convention, minicpm.py:1027-1069) applied to
// q and k of a fused [N, (H + 2G) * D] projection, writing contiguous
// q [N, H, D], k [N, G, D] and v [N, G, D].  cos/sin are computed in fp32 from
// the position and the per-frequency inverse wavelength (already divided by
// the LongRoPE factor) and scaled by `scaling`.
__global__ void __launch_bounds__(256) rope_split_kernel(
    const uint4* __restrict__ qkv, const int64_t* __restrict__ positions,
    const float* __restrict__ inv_freq, float scaling, int64_t n, int H, int G,
    uint4* __restrict__ q, uint4* __restrict__ k, uint4* __restrict__ v) {
  // D = 128: a head row is 16 vectors; thread handles vector c (dims 8c..8c+7)
  // of the first half together with vector c+8 of the second half.
  const int heads = H + 2 * G;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = n * heads * 8;
  if (gid >= total) return;
  const int c = static_cast<int>(gid & 7);
  const int head = static_cast<int>((gid >> 3) % heads);
  const int64_t t = gid / (8 * heads);
  const uint4* src = qkv + (t * heads + head) * 16;
  if (head >= H + G) {  // v: plain copy
    uint4* dst = v + (t * G + (head - H - G)) * 16;
    dst[c] = __ldg(src + c);
    dst[c + 8] = __ldg(src + c + 8);
    return;
  }
  float x1[8], x2[8];
  unpack8(__ldg(src + c), x1);
  unpack8(__ldg(src + c + 8), x2);
  const float pos = static_cast<float>(__ldg(positions + t));
  float o1[8], o2[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float sn, cs;
    sincosf(pos * __ldg(inv_freq + 8 * c + e), &sn, &cs);
    cs *= scaling;
    sn *= scaling;
    o1[e] = x1[e] * cs - x2[e] * sn;
    o2[e] = x2[e] * cs + x1[e] * sn;
  }
  uint4* dst = head < H ? q + (t * H + head) * 16 : k + (t * G + (head - H)) * 16;
  dst[c] = pack8(o1);
  dst[c + 8] = pack8(o2);
}

// out[t, i] = silu(gu[t, i]) * gu[t, I + i], fp32 math.
__global__ void __launch_bounds__(256) silu_mul_kernel(const uint4* __restrict__ gu, int64_t n,
                                                       int ivecs, uint4* __restrict__ out) {
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= n * ivecs) return;
  const int64_t t = gid / ivecs;
  const int c = static_cast<int>(gid % ivecs);
  float a[8], b[8], o[8];
  unpack8(__ldg(gu + t * 2 * ivecs + c), a);
  unpack8(__ldg(gu + t * 2 * ivecs + ivecs + c), b);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = a[e] / (1.f + __expf(-a[e])) * b[e];
  out[gid] = pack8(o);
}

}  // namespace
}  // namespace ls

extern "C" {

int ls_bb_rms_norm(const uint16_t* x, const uint16_t* weight, int64_t rows, int32_t hidden,
                   float eps, uint16_t* out, void* stream) {
  if (!x || !weight || !out || rows < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > 8 * 256 * 4)
    return LS_ERR_INVALID_ARGUMENT;
  if (rows == 0) return LS_OK;
  const int vecs = hidden / 8;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  const uint4* wv = reinterpret_cast<const uint4*>(weight);
  uint4* yv = reinterpret_cast<uint4*>(out);
  if (vecs <= 256)
    ls::rms_norm_kernel<1><<<static_cast<unsigned>(rows), 256, 0, s>>>(xv, wv, eps, vecs, yv);
  else if (vecs <= 512)
    ls::rms_norm_kernel<2><<<static_cast<unsigned>(rows), 256, 0, s>>>(xv, wv, eps, vecs, yv);
  else
    ls::rms_norm_kernel<4><<<static_cast<unsigned>(rows), 256, 0, s>>>(xv, wv, eps, vecs, yv);
  return cudaGetLastError() == cudaSuccess ? LS_OK : LS_ERR_CUDA;
}

int ls_bb_rope_split(const uint16_t* qkv, const int64_t* positions, const float* inv_freq,
                     float scaling, int64_t tokens, int32_t num_heads, int32_t num_kv_heads,
                     int32_t head_dim, uint16_t* q, uint16_t* k, uint16_t* v, void* stream) {
  if (!qkv || !positions || !inv_freq || !q || !k || !v || tokens < 0) return LS_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return LS_ERR_UNSUPPORTED;
  if (tokens == 0) return LS_OK;
  const int64_t threads = tokens * (num_heads + 2 * num_kv_heads) * 8;
  ls::rope_split_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0,
                          static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(qkv), positions, inv_freq, scaling, tokens, num_heads,
      num_kv_heads, reinterpret_cast<uint4*>(q), reinterpret_cast<uint4*>(k),
      reinterpret_cast<uint4*>(v));
  return cudaGetLastError() == cudaSuccess ? LS_OK : LS_ERR_CUDA;
}

int ls_bb_silu_mul(const uint16_t* gate_up, int64_t tokens, int32_t intermediate, uint16_t* out,
                   void* stream) {
  if (!gate_up || !out || tokens < 0 || intermediate <= 0 || intermediate % 8 != 0)
    return LS_ERR_INVALID_ARGUMENT;
  if (tokens == 0) return LS_OK;
  const int ivecs = intermediate / 8;
  const int64_t threads = tokens * ivecs;
  ls::silu_mul_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(gate_up), tokens, ivecs, reinterpret_cast<uint4*>(out));
  return cudaGetLastError() == cudaSuccess ? LS_OK : LS_ERR_CUDA;
}

}  // extern "C"
