// Block-sparse causal attention over per-token page lists (stage 2, a9).
//
// Replaces infllmv2_attn_varlen_func(..., topk_idx=) (minicpm.py:3229-3243).
// LeanSelect picks pages per query token, and on the benchmark inputs a
// page shared by 8 neighbouring tokens is read by only 1.4 of them on
// average, so a tensor-core tile that spans several tokens would compute
// mostly masked products.  This kernel therefore works per (token, KV
// group): the Hg query heads of the group form the 16 rows of an m16n8k16
// tile and the keys of the token's own pages form the columns, so every
// product computed is a product the token needs.
//
// CTA = one (packed token, group); 5 warps:
//   warp 4      TMA producer: streams each selected page's K and V
//               (64 keys x 128 dims each, two 128B-swizzled boxes apiece)
//               through a 3-stage shared-memory ring (32 KB per stage);
//   warps 0..3  consumers: warp w owns keys 16w..16w+15 of every page and
//               keeps its own online softmax (m, l, O[16 x 128] in registers);
//               the four partial results are merged at the end.
// The page list is loaded once, invalid entries dropped, sorted and
// de-duplicated by one warp (bitonic network over 128 slots; a list that is
// already strictly ascending, as the selection kernels write it, is not
// sorted).  Its loads and the Q rows' are issued before anything else in the
// CTA, so their latency overlaps the sequence lookup.
//
// For few query rows (a decode step) the page list of each row can be cut
// into `splits` slices, one CTA each (AttnArgs::splits); the slices write
// partial results that attn_merge_kernel combines.
#include "common.cuh"
#include "launch.h"

namespace ls {
namespace {

constexpr int kStages = 3;
constexpr int kBoxBytes = 64 * 128;            // 64 keys x 64 dims bf16
constexpr int kStageBytes = 4 * kBoxBytes;     // K half0, K half1, V half0, V half1
constexpr int kThreads = 160;
constexpr int kMaxT = LS_MAX_TOPK;
constexpr int32_t kSentinel = 0x7FFFFFFF;
constexpr float kRescaleSlack = 8.f;  // log2 units: exponentials stay below 256

struct AttnSmem {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int abort_flag;
  int n_pages;
  int32_t pages[kMaxT];
  float m_part[4][16];
  float l_part[4][16];
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128B-swizzled box.
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Sorts 128 keys held as v[r] at position 32*r + lane, ascending.
__device__ __forceinline__ void warp_bitonic_sort128(int32_t (&v)[4], int lane) {
#pragma unroll
  for (int k = 2; k <= 128; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
        const int rj = j >> 5;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if ((r & rj) == 0) {
            const int pos = 32 * r + lane;
            const bool up = (pos & k) == 0;
            const int32_t a = v[r], b = v[r | rj];
            const bool swap = up ? (a > b) : (a < b);
            v[r] = swap ? b : a;
            v[r | rj] = swap ? a : b;
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int pos = 32 * r + lane;
          const int32_t other = __shfl_xor_sync(0xffffffffu, v[r], j);
          const bool up = (pos & k) == 0;
          const bool lower = (lane & j) == 0;
          const int32_t lo = min(v[r], other), hi = max(v[r], other);
          v[r] = (lower == up) ? lo : hi;
        }
      }
    }
  }
}

template <int HG, bool kGatherOnly>
__global__ void __launch_bounds__(kThreads, 2) sparse_attn_kernel(const __grid_constant__ AttnArgs args) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint8_t* q_smem = stages + kStages * kStageBytes;  // [16 rows x 256 B], swizzled chunks
  AttnSmem* sm = reinterpret_cast<AttnSmem*>(q_smem + 16 * 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool group_major = args.order == 1;
  // Slice `split` of the row's page list (the whole list when splits == 1);
  // a row's slices are neighbouring CTAs.
  const int split = static_cast<int>(blockIdx.x % static_cast<uint32_t>(args.splits));
  const int64_t item = blockIdx.x / static_cast<uint32_t>(args.splits);
  const int64_t t = group_major ? item % args.total_q : item / args.num_groups;
  const int g = group_major ? static_cast<int>(item / args.total_q)
                            : static_cast<int>(item % args.num_groups);
  // The page list and the Q rows depend only on (t, g): their loads are
  // issued first, so their latency overlaps the sequence lookup below.
  int32_t praw[4];
  uint4 qraw[8];
  if (warp == 0) {
    const int32_t* row = args.topk_idx + (static_cast<int64_t>(g) * args.total_q + t) * args.topk;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int pos = 32 * r + lane;
      praw[r] = pos < args.topk ? __ldg(row + pos) : -1;
    }
  } else if (warp == 1) {
    const uint4* src = reinterpret_cast<const uint4*>(args.q + (t * args.num_heads + g * HG) * 128);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = lane + 32 * k;
      const int r = i >> 4, c = i & 15;
      qraw[k] = r < HG ? __ldg(src + r * 16 + c) : make_uint4(0, 0, 0, 0);
    }
  }
  const int b = find_sequence(args.cu_q, args.batch, t);
  const int64_t q_start = __ldg(args.cu_q + b);
  const int64_t k_start = __ldg(args.cu_k + b);
  const int nq = static_cast<int>(__ldg(args.cu_q + b + 1) - q_start);
  const int nk = static_cast<int>(__ldg(args.cu_k + b + 1) - k_start);
  const int t_rel = static_cast<int>(t - q_start);
  const int t_lim = args.causal ? min(nk - 1, t_rel + (nk - nq)) : nk - 1;
  const int n_kpages = (nk + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm->full[s], 1);
      mbar_init(&sm->empty[s], 4);
    }
    sm->abort_flag = 0;
    fence_barrier_init();
  }

  if (warp == 0) {
    // Page list: drop empty/out-of-range/fully-masked entries, sort, de-duplicate.
    int32_t v[4];
    bool bad_index = false;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int32_t p = praw[r];
      if (p >= n_kpages) bad_index = true;
      v[r] = (p >= 0 && p < n_kpages && p * 64 <= t_lim) ? p : kSentinel;
    }
    if (__any_sync(0xffffffffu, bad_index) && lane == 0) report(args.status, LS_DEVERR_PAGE_INDEX);
    // Strictly ascending valid entries followed by sentinels (the lists the
    // selection kernels write) need no sort.
    bool ordered = true;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      int32_t next = __shfl_down_sync(0xffffffffu, v[r], 1);
      const int32_t next_row = __shfl_sync(0xffffffffu, v[r < 3 ? r + 1 : r], 0);
      if (lane == 31) next = r < 3 ? next_row : kSentinel;
      ordered = ordered && (v[r] < next || next == kSentinel);
    }
    if (!__all_sync(0xffffffffu, ordered)) warp_bitonic_sort128(v, lane);
    int base = 0;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      int32_t prev = __shfl_up_sync(0xffffffffu, v[r], 1);
      const int32_t prev_reg = r > 0 ? __shfl_sync(0xffffffffu, v[r - 1], 31) : -1;
      if (lane == 0) prev = prev_reg;
      const bool keep = v[r] != kSentinel && v[r] != prev;
      const uint32_t mask = __ballot_sync(0xffffffffu, keep);
      if (keep) sm->pages[base + __popc(mask & ((1u << lane) - 1))] = v[r];
      base += __popc(mask);
    }
    if (lane == 0) sm->n_pages = base;
  } else if (warp == 1) {
    // Q rows of this group (HG heads, padded to 16 rows with zeros), swizzled.
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = lane + 32 * k;
      const int r = i >> 4, c = i & 15;
      *reinterpret_cast<uint4*>(q_smem + r * 256 + (((c & 7) ^ (r & 7)) | (c & 8)) * 16) = qraw[k];
    }
  }
  __syncthreads();
  const int page_lo = static_cast<int>(static_cast<int64_t>(split) * sm->n_pages / args.splits);
  const int n_pages =
      static_cast<int>(static_cast<int64_t>(split + 1) * sm->n_pages / args.splits) - page_lo;
  const int32_t* pages = sm->pages + page_lo;
  volatile int* abort_flag = &sm->abort_flag;

  if (warp == 4) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&args.tm_k);
      tma_prefetch_desc(&args.tm_v);
      int i = 0;
      bool ok = true;
      for (; i < n_pages; ++i) {
        const int s = i % kStages;
        ok = mbar_wait(&sm->empty[s], ((i / kStages) & 1) ^ 1, args.status, abort_flag);
        if (!ok) break;
        uint8_t* st = stages + s * kStageBytes;
        const int32_t y = static_cast<int32_t>(k_start + static_cast<int64_t>(pages[i]) * 64);
        const int32_t x = g * 128;
        mbar_arrive_expect_tx(&sm->full[s], kStageBytes);
        tma_load_2d(st, &args.tm_k, &sm->full[s], x, y);
        tma_load_2d(st + kBoxBytes, &args.tm_k, &sm->full[s], x + 64, y);
        tma_load_2d(st + 2 * kBoxBytes, &args.tm_v, &sm->full[s], x, y);
        tma_load_2d(st + 3 * kBoxBytes, &args.tm_v, &sm->full[s], x + 64, y);
      }
      if (!ok) {
        for (int k = max(0, i - kStages); k < i; ++k)
          mbar_wait(&sm->full[k % kStages], (k / kStages) & 1, nullptr, nullptr);
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  if constexpr (kGatherOnly) {
    for (int i = 0; i < n_pages; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&sm->full[s], (i / kStages) & 1, args.status, abort_flag)) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm->empty[s]);
    }
    return;
  }
  // Q fragments for the 8 k-steps (rows = heads, k = dims).
  uint32_t qa[8][4];
  {
    const uint32_t qbase = smem_u32(q_smem);
    const int mat = lane >> 3, r8 = lane & 7;
    const int row = (mat & 1) * 8 + r8;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = 2 * kk + (mat >> 1);  // 16-byte chunk index 0..15 in the 256-byte row
      const uint32_t addr = qbase + row * 256 + ((((c & 7) ^ (row & 7)) | (c & 8)) << 4);
      ldsm_x4(addr, qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
    }
  }

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float mu0 = 0.f, mu1 = 0.f;                // m with -inf read as 0
  float th0 = -INFINITY, th1 = -INFINITY;    // (m + slack) in raw score units
  const float sl2 = args.scale_log2;         // > 0
  const int key_base = warp * 16;
  bool ok = true;

  for (int i = 0; i < n_pages; ++i) {
    const int s = i % kStages;
    ok = mbar_wait(&sm->full[s], (i / kStages) & 1, args.status, abort_flag);
    if (!ok) break;
    const uint32_t st = smem_u32(stages + s * kStageBytes);
    // ---- S = Q K^T for keys key_base .. key_base+15 of this page.  The
    // head dimension is split over two accumulator sets (dims 0-63, 64-127)
    // so four independent MMA chains are in flight.
    float sc[2][4], sh[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
      sh[n][0] = sh[n][1] = sh[n][2] = sh[n][3] = 0.f;
    }
    {
      const int mat = lane >> 3, r8 = lane & 7;
      const int key = key_base + (mat >> 1) * 8 + r8;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int chunk = 2 * kk + (mat & 1);  // 16-byte chunk inside each 64-dim box
        uint32_t b0, b1, b2, b3, c0, c1, c2, c3;
        ldsm_x4(st + sw128(key, chunk), b0, b1, b2, b3);
        ldsm_x4(st + kBoxBytes + sw128(key, chunk), c0, c1, c2, c3);
        mma_bf16_16816(sc[0], qa[kk], b0, b1);
        mma_bf16_16816(sc[1], qa[kk], b2, b3);
        mma_bf16_16816(sh[0], qa[kk + 4], c0, c1);
        mma_bf16_16816(sh[1], qa[kk + 4], c2, c3);
      }
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[n][e] += sh[n][e];
    }
    // ---- causal / length mask (only pages that reach past t_lim)
    const int page_key0 = pages[i] * 64 + key_base;
    if (page_key0 + 15 > t_lim) {
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = page_key0 + n * 8 + (lane & 3) * 2 + (e & 1);
          if (key > t_lim) sc[n][e] = -INFINITY;
        }
    }
    // ---- online softmax (log2 domain) with a lazily raised reference max:
    // m0/m1 only move when a score exceeds them by more than kRescaleSlack,
    // so exponentials stay below 2^kRescaleSlack and the O rescale is rare.
    // Most pages raise nothing: each thread tests its own raw scores against
    // the rows' thresholds, and only a page on which some score passes one
    // pays for the quad max (a row's scores sit in four lanes) and the
    // rescale.  (Near a threshold the raw test and the scaled one may
    // disagree; either way the exponentials stay far from overflow.)
    const float rx0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    const float rx1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
    if (__any_sync(0xffffffffu, rx0 > th0 || rx1 > th1)) {
      float mx0 = rx0 * sl2, mx1 = rx1 * sl2;
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const bool grow0 = mx0 > m0 + kRescaleSlack, grow1 = mx1 > m1 + kRescaleSlack;
      const float a0 = grow0 ? ex2(m0 - mx0) : 1.f;
      const float a1 = grow1 ? ex2(m1 - mx1) : 1.f;
      if (grow0) {
        m0 = mx0;
        mu0 = m0;
        th0 = (m0 + kRescaleSlack) / sl2;
      }
      if (grow1) {
        m1 = mx1;
        mu1 = m1;
        th1 = (m1 + kRescaleSlack) / sl2;
      }
      l0 *= a0;
      l1 *= a1;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= a0;
        o[j][1] *= a0;
        o[j][2] *= a1;
        o[j][3] *= a1;
      }
    }
    float p[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      p[n][0] = ex2(fmaf(sc[n][0], sl2, -mu0));
      p[n][1] = ex2(fmaf(sc[n][1], sl2, -mu0));
      p[n][2] = ex2(fmaf(sc[n][2], sl2, -mu1));
      p[n][3] = ex2(fmaf(sc[n][3], sl2, -mu1));
    }
    l0 += (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]);
    l1 += (p[0][2] + p[0][3]) + (p[1][2] + p[1][3]);
    uint32_t pa[4];
    pa[0] = pack_bf16x2(p[0][0], p[0][1]);
    pa[1] = pack_bf16x2(p[0][2], p[0][3]);
    pa[2] = pack_bf16x2(p[1][0], p[1][1]);
    pa[3] = pack_bf16x2(p[1][2], p[1][3]);
    // ---- O += P V for the same 16 keys.
    {
      const int mat = lane >> 3, r8 = lane & 7;
      const int key = key_base + (mat & 1) * 8 + r8;
      const uint32_t vbase = st + 2 * kBoxBytes;
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const int dim0 = 8 * j + (mat >> 1) * 8;
        const uint32_t addr = vbase + (dim0 >> 6) * kBoxBytes + sw128(key, (dim0 & 63) >> 3);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(addr, b0, b1, b2, b3);
        mma_bf16_16816(o[j], pa, b0, b1);
        mma_bf16_16816(o[j + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm->empty[s]);
  }

  // ---- merge the four warps' partial softmax states
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const int r0 = lane >> 2, r1 = r0 + 8;
  if ((lane & 3) == 0) {
    sm->m_part[warp][r0] = m0;
    sm->m_part[warp][r1] = m1;
    sm->l_part[warp][r0] = l0;
    sm->l_part[warp][r1] = l1;
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  // A wait that gave up leaves the row unwritten: copies the producer issued
  // may still be landing in the stage memory the merge below would reuse.
  // Every consumer warp has either set or seen the flag before the barrier.
  if (*abort_flag) return;
  float mt0 = -INFINITY, mt1 = -INFINITY;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    mt0 = fmaxf(mt0, sm->m_part[w][r0]);
    mt1 = fmaxf(mt1, sm->m_part[w][r1]);
  }
  const float mv0 = mt0 == -INFINITY ? 0.f : mt0;
  const float mv1 = mt1 == -INFINITY ? 0.f : mt1;
  float lt0 = 0.f, lt1 = 0.f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    lt0 += sm->l_part[w][r0] * ex2(sm->m_part[w][r0] - mv0);
    lt1 += sm->l_part[w][r1] * ex2(sm->m_part[w][r1] - mv1);
  }
  const float f0 = (lt0 > 0.f ? ex2(m0 - mv0) / lt0 : 0.f);
  const float f1 = (lt1 > 0.f ? ex2(m1 - mv1) / lt1 : 0.f);
  // Stage memory is idle once every page was consumed: sum partial O there.
  float* acc = reinterpret_cast<float*>(stages);  // [4 warps][16 rows][128 dims]
  {
    float* mine = acc + warp * 16 * 128;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int col = 8 * j + (lane & 3) * 2;
      *reinterpret_cast<float2*>(&mine[r0 * 128 + col]) = make_float2(o[j][0] * f0, o[j][1] * f0);
      *reinterpret_cast<float2*>(&mine[r1 * 128 + col]) = make_float2(o[j][2] * f1, o[j][3] * f1);
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  {
    // 128 threads x 16 outputs: thread -> (row, 16 consecutive dims).
    const int row = threadIdx.x >> 3;
    const int col0 = (threadIdx.x & 7) * 16;
    if (row < HG) {
      float sum[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) sum[c] = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int c = 0; c < 16; c += 4) {
          const float4 x = *reinterpret_cast<const float4*>(&acc[(w * 16 + row) * 128 + col0 + c]);
          sum[c] += x.x;
          sum[c + 1] += x.y;
          sum[c + 2] += x.z;
          sum[c + 3] += x.w;
        }
      // Row max (log2 units) and row sum of this CTA's pages.
      float mt = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) mt = fmaxf(mt, sm->m_part[w][row]);
      const float mu = mt == -INFINITY ? 0.f : mt;
      float lt = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) lt += sm->l_part[w][row] * ex2(sm->m_part[w][row] - mu);
      const int64_t orow = t * args.num_heads + g * HG + row;
      if (args.splits > 1) {
        // Partial result of this slice: normalised output, max and sum.
        const int64_t prow = static_cast<int64_t>(split) * args.total_q * args.num_heads + orow;
        float4* po = reinterpret_cast<float4*>(args.part_o + prow * 128 + col0);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          po[c] = make_float4(sum[4 * c], sum[4 * c + 1], sum[4 * c + 2], sum[4 * c + 3]);
        if ((threadIdx.x & 7) == 0)
          *reinterpret_cast<float2*>(args.part_ml + prow * 2) = make_float2(mt, lt);
      } else {
        uint4 packed[2];
        uint32_t* pw = reinterpret_cast<uint32_t*>(packed);
#pragma unroll
        for (int c = 0; c < 8; ++c) pw[c] = pack_bf16x2(sum[2 * c], sum[2 * c + 1]);
        uint4* dst = reinterpret_cast<uint4*>(args.out + orow * 128 + col0);
        dst[0] = packed[0];
        dst[1] = packed[1];
        if (args.lse != nullptr && (threadIdx.x & 7) == 0)
          args.lse[static_cast<int64_t>(g * HG + row) * args.total_q + t] =
              lt > 0.f ? (mt + __log2f(lt)) * 0.69314718055994531f : INFINITY;
      }
    }
  }
}

size_t attn_smem_bytes() { return 1024 + kStages * kStageBytes + 16 * 256 + sizeof(AttnSmem); }

// One warp per (token, head) row: weights each slice's normalised output by
// its share of the row's softmax mass, l_s * 2^(m_s - max m), and writes the
// bf16 row (zeros when no slice saw a page) and its log-sum-exp.  Lane l
// reads the max and sum of slices l and l + 32 at once; the slices' outputs
// are then summed with several loads in flight.
__global__ void __launch_bounds__(256) attn_merge_kernel(const __grid_constant__ AttnArgs args) {
  const int64_t rows = args.total_q * args.num_heads;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int splits = args.splits;  // 2 .. 64
  float2 ml_a = make_float2(-INFINITY, 0.f), ml_b = make_float2(-INFINITY, 0.f);
  if (lane < splits) ml_a = *reinterpret_cast<const float2*>(args.part_ml + (lane * rows + r) * 2);
  if (lane + 32 < splits)
    ml_b = *reinterpret_cast<const float2*>(args.part_ml + ((lane + 32) * rows + r) * 2);
  float mx = fmaxf(ml_a.y > 0.f ? ml_a.x : -INFINITY, ml_b.y > 0.f ? ml_b.x : -INFINITY);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float w_a = ml_a.y > 0.f ? ml_a.y * ex2(ml_a.x - mx) : 0.f;
  const float w_b = ml_b.y > 0.f ? ml_b.y * ex2(ml_b.x - mx) : 0.f;
  float wsum = w_a + w_b;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* po = reinterpret_cast<const float4*>(args.part_o + r * 128) + lane;
  const int64_t stride4 = rows * 32;  // float4 per slice
#pragma unroll 8
  for (int s = 0; s < splits; ++s) {
    const float w = __shfl_sync(0xffffffffu, s < 32 ? w_a : w_b, s & 31);
    if (w > 0.f) {
      const float4 o = po[s * stride4];
      acc.x = fmaf(w, o.x, acc.x);
      acc.y = fmaf(w, o.y, acc.y);
      acc.z = fmaf(w, o.z, acc.z);
      acc.w = fmaf(w, o.w, acc.w);
    }
  }
  const float f = wsum > 0.f ? 1.f / wsum : 0.f;
  uint2 packed;
  packed.x = pack_bf16x2(acc.x * f, acc.y * f);
  packed.y = pack_bf16x2(acc.z * f, acc.w * f);
  reinterpret_cast<uint2*>(args.out + r * 128)[lane] = packed;
  if (args.lse != nullptr && lane == 0) {
    const int64_t t = r / args.num_heads;
    const int h = static_cast<int>(r % args.num_heads);
    args.lse[static_cast<int64_t>(h) * args.total_q + t] =
        wsum > 0.f ? (mx + __log2f(wsum)) * 0.69314718055994531f : INFINITY;
  }
}


}  // namespace

template <bool kGatherOnly>
cudaError_t launch_attn(const AttnArgs& args, cudaStream_t stream) {
  if (args.splits < 1) return cudaErrorInvalidValue;
  const int64_t grid = args.total_q * args.num_groups * args.splits;
  if (grid == 0) return cudaSuccess;
  const size_t smem = attn_smem_bytes();
  const int hg = args.num_heads / args.num_groups;
  cudaError_t err;
  if (hg == 16) {
    err = cudaFuncSetAttribute(sparse_attn_kernel<16, kGatherOnly>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    sparse_attn_kernel<16, kGatherOnly><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(args);
  } else if (hg == 8) {
    err = cudaFuncSetAttribute(sparse_attn_kernel<8, kGatherOnly>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    sparse_attn_kernel<8, kGatherOnly><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(args);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_sparse_attn(const AttnArgs& args, cudaStream_t stream) {
  return launch_attn<false>(args, stream);
}

cudaError_t launch_sparse_attn_gather_only(const AttnArgs& args, cudaStream_t stream) {
  AttnArgs a = args;
  a.splits = 1;
  return launch_attn<true>(a, stream);
}

cudaError_t launch_sparse_attn_merge(const AttnArgs& args, cudaStream_t stream) {
  const int64_t rows = args.total_q * args.num_heads;
  if (rows == 0) return cudaSuccess;
  attn_merge_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(args);
  return cudaGetLastError();
}

}  // namespace ls
