// Row geometry of the page selection (top-k) kernels.
#pragma once

#include "common.cuh"
#include "launch.h"

namespace ls {

// Output row, workspace row and candidate geometry of (group, query) row r
// = g * total_q + q_row of a select-mode launch (minicpm.py:3121-3138).
// Candidate i is page n_init + i for i < m (pages n_init .. lo-1); for the
// uniform method candidate m is page qp+1, which the score kernel stored in
// the workspace slot n_init + m.  `cap` is how many candidates the row
// selects.  `empty` rows stay all -1.
__device__ __forceinline__ void row_geometry(const ScoreArgs& args, uint32_t r, uint32_t total_q,
                                             int32_t** out, int64_t* ws_row, bool* empty,
                                             int* m_all, int* cap, int* future, int* n_init,
                                             int* take_b, int* local0, int* n_local) {
  const int64_t q_row = r % total_q;
  *out = args.topk_idx + static_cast<int64_t>(r) * args.take;
  *ws_row = static_cast<int64_t>(r) * args.max_pages;
  *empty = false;
  int b = 0, n;
  int64_t q0 = 0;
  if (args.cu_q) {
    b = find_sequence(args.cu_q, args.batch, q_row);
    q0 = __ldg(args.cu_q + b);
    n = static_cast<int>(__ldg(args.cu_q + b + 1) - q0);
    if (n > args.max_seqlen_q) {  // reported by the score kernel; the row stays empty
      *empty = true;
      return;
    }
  } else {
    n = args.max_seqlen_q;
  }
  const int atoms = args.cu_c ? static_cast<int>(__ldg(args.cu_c + b + 1) - __ldg(args.cu_c + b))
                              : static_cast<int>(args.total_c);
  const int pos = args.pos_offset + static_cast<int>(q_row - q0);
  const int pages = ((args.seq_len > 0 ? args.seq_len : n) + 63) / 64;
  const int qp = pos / 64;
  *take_b = min(args.take, pages);
  *n_init = min(args.init_blocks, qp + 1);               // sink pages 0 .. n_init-1
  const int lo = max(0, qp - args.local_blocks);          // local pages lo .. qp
  *local0 = max(lo, *n_init);
  *n_local = qp - *local0 + 1;                            // local pages that are not sinks
  int m = max(0, lo - *n_init);                           // candidates n_init .. lo-1
  int slots = *take_b - (*n_init + *n_local);
  // Uniform method: page qp+1 is scored too (its first window atom may be
  // visible) and competes as candidate m, or as a forced sink; either way
  // a slot it wins stays -1 (uniform.py:100-106).  Rows of sequences
  // without atoms keep their forced pages (head_mix.py:150-170).
  *future = -1;
  if (args.uniform) {
    if (atoms <= 0) m = 0;
    slots -= max(0, min(args.init_blocks, pages) - (qp + 1));  // future sinks
    if (atoms > 0 && qp + 1 < pages && qp + 1 >= args.init_blocks) *future = m;
  } else if (atoms <= 0) {
    // The reference leaves rows of sequences without atoms at -1 (minicpm.py:3115-3116).
    *empty = true;
    return;
  }
  *m_all = m + (*future >= 0 ? 1 : 0);
  *cap = max(0, min(slots, *m_all));
}

// Exclusive prefix sum over the warp; returns it and sets `total`.
__device__ __forceinline__ int warp_excl_scan(int v, int lane, int& total) {
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  total = __shfl_sync(0xffffffffu, incl, 31);
  return incl - v;
}

// Exact threshold of the `need` largest nonzero keys among keys(0 ..
// count-1), need >= 1.  A histogram over the keys' own range: 256 bins of
// width 2^shift from the smallest key, so one pass is exact when the keys
// span fewer than 256 values; otherwise the next pass splits the bin that
// holds the threshold into 256 again (16-bit keys: at most 2 passes, 32-bit
// keys: at most 4).  Returns the threshold key;
// `need` becomes the number of keys equal to it that belong to the
// selection (the lowest indices win).
// `kmin`/`kmax` bound the nonzero keys (any bounds that hold are fine).
template <class Keys>
__device__ uint32_t radix_threshold_in(const Keys& keys, int count, int& need, uint32_t* hist,
                                       int lane, uint32_t kmin, uint32_t kmax) {
  const uint32_t range = kmax - kmin;
  int shift = range > 255u ? (32 - __clz(range)) - 8 : 0;  // (range >> shift) < 256
  uint32_t lo = kmin;        // keys of the current pass: [lo, lo + width)
  uint64_t width = uint64_t{256} << shift;
#pragma unroll 1
  while (true) {
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[lane + 32 * j] = 0;
    __syncwarp();
    for (int i = lane; i < count; i += 32) {
      const uint32_t key = keys(i);
      if (key != 0u && key >= lo && static_cast<uint64_t>(key - lo) < width)
        atomicAdd(&hist[(key - lo) >> shift], 1u);
    }
    __syncwarp();
    // Lane l owns bins 255-8l .. 248-8l (descending).
    uint32_t c[8];
    uint32_t lane_sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = hist[255 - 8 * lane - j];
      lane_sum += c[j];
    }
    uint32_t incl = lane_sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const uint32_t excl = incl - lane_sum;
    const bool here = excl < static_cast<uint32_t>(need) && incl >= static_cast<uint32_t>(need);
    const uint32_t owner_mask = __ballot_sync(0xffffffffu, here);
    const int owner = __ffs(owner_mask) - 1;
    int bin = 0;
    uint32_t above = 0;
    if (here) {
      uint32_t cum = excl;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (cum + c[j] >= static_cast<uint32_t>(need)) {
          bin = 255 - 8 * lane - j;
          above = cum;
          break;
        }
        cum += c[j];
      }
    }
    bin = __shfl_sync(0xffffffffu, bin, owner);
    above = __shfl_sync(0xffffffffu, above, owner);
    need -= static_cast<int>(above);
    __syncwarp();
    lo += static_cast<uint32_t>(bin) << shift;
    if (shift == 0) return lo;
    width = uint64_t{1} << shift;   // the bin's keys, split into 256 again
    shift = max(0, shift - 8);
  }
}

// radix_threshold_in with the keys' own bounds, found by one pass.
template <class Keys>
__device__ uint32_t radix_threshold(const Keys& keys, int count, int& need, uint32_t* hist,
                                    int lane) {
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  for (int i = lane; i < count; i += 32) {
    const uint32_t key = keys(i);
    if (key != 0u) {
      kmin = min(kmin, key);
      kmax = max(kmax, key);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
  }
  return radix_threshold_in(keys, count, need, hist, lane, kmin, kmax);
}

// Writes, in index order, the entries among keys(0 .. count-1) above `thr`
// plus the first `ties` equal to it, as page numbers `index(j) + base`;
// candidate `skip` is selected but not written.  Returns the next output
// position.
template <class Keys, class Index>
__device__ int emit_threshold(const Keys& keys, const Index& index, int count, uint32_t thr,
                              int ties, int skip, int base, int32_t* out, int k_out, int lane) {
  int ties_seen = 0;
  for (int b0 = 0; b0 < count; b0 += 32) {
    const int j = b0 + lane;
    const uint32_t key = j < count ? keys(j) : 0u;
    const bool tie = key == thr && key != 0u;
    const uint32_t tie_mask = __ballot_sync(0xffffffffu, tie);
    const int tie_rank = ties_seen + __popc(tie_mask & ((1u << lane) - 1));
    ties_seen += __popc(tie_mask);
    bool take = key > thr || (tie && tie_rank < ties);
    const int i = j < count ? index(j) : -1;
    if (i == skip) take = false;  // the slot page qp+1 won stays empty
    const uint32_t take_mask = __ballot_sync(0xffffffffu, take);
    if (take) out[k_out + __popc(take_mask & ((1u << lane) - 1))] = base + i;
    k_out += __popc(take_mask);
  }
  return k_out;
}

struct Identity {
  __device__ __forceinline__ int operator()(int j) const { return j; }
};
}  // namespace ls
