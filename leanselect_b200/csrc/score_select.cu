// Selector scoring and page selection on the 5th-generation tensor cores.
//
// One CTA owns a tile of 128 query rows of one sequence and one KV group.
//
//   Phase A  Qs = Q_tile[128, Hg*D] x WqT_g[F, Hg*D]^T            (a3, selector.py:160-177)
//            TMA streams 64-wide K blocks of Q and WqT through a 3-stage ring,
//            one thread issues tcgen05.mma (M=128, N=128, K=16) into TMEM.
//            The epilogue warps round Qs to bf16 (the reference's bf16 einsum
//            output) and store it back to shared memory as the A operand of
//            phase B (128B-swizzled K-major, the layout TMA would write).
//   Phase B  for each tile of 128 atoms: S = Qs x Ks_tile^T        (a5, selector.py:203-207)
//            into one of two TMEM accumulators (double buffered), while the
//            epilogue warps drain the other: each thread owns one query row,
//            max-pools atoms into pages (window 5, stride 4, pad 1; a6,
//            pages.py:146-187) and either writes the page scores (score
//            mode) or feeds visible non-forced pages into a per-row min-heap
//            of the best T' pages in shared memory (select mode; a7,
//            minicpm.py:3124-3141).  Only atom tiles that can reach a
//            candidate page are computed: the atom loop stops at the causal
//            limit of the tile's last row.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer and TMEM
// owner, warps 2-5 epilogue (warp w reads TMEM lanes 32*(w%4) .. +31).
#include "common.cuh"
#include "launch.h"

namespace ls {
namespace {

constexpr int kRows = 128;
constexpr int kWidth = 128;          // F
constexpr int kStages = 3;
constexpr int kHalfBytes = 128 * 128;        // [128 rows x 64 bf16]
constexpr int kStageBytes = 2 * kHalfBytes;  // A+B (phase A) or one Ks tile (phase B)
constexpr int kQsBytes = 2 * kHalfBytes;
constexpr int kHeapCap = LS_MAX_TOPK;
constexpr int kHeapBytes = kHeapCap * kRows * (4 + 2);
constexpr int kThreads = 192;
constexpr uint32_t kIdesc = umma_idesc_bf16(128, 128);

struct Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t qs_full;
  uint64_t qs_ready;
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

__host__ __device__ constexpr size_t smem_bytes(int mode) {
  return 1024  // alignment slack
         + static_cast<size_t>(kStages) * kStageBytes + (mode == kModeProject ? 0 : kQsBytes) +
         (mode == kModeSelect ? kHeapBytes : 0) + sizeof(Barriers);
}

struct TileInfo {
  int g, b, tile;
  int64_t q0;       // first packed query row of the sequence
  int n;            // sequence length
  int row0;         // first row of the tile inside the sequence
  int rows;         // valid rows in the tile
  int64_t c0;       // first packed atom of the sequence
  int atoms;        // atoms of the sequence
  int pages;        // pages of the sequence
  int pos0;         // position of row 0 inside the sequence (chunk mode), else 0
  int atom_tiles;   // atom tiles the tile needs
  bool prologue;    // whether Qs is computed at all
};

__device__ __forceinline__ bool worse(float sa, uint32_t pa, float sb, uint32_t pb) {
  return sa < sb || (sa == sb && pa > pb);
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) score_kernel(const __grid_constant__ ScoreArgs args) {
  const int tiles_max = (args.max_seqlen_q + kRows - 1) / kRows;
  TileInfo ti;
  {
    const int64_t i = blockIdx.x;
    ti.g = static_cast<int>(i % args.num_groups);
    ti.b = static_cast<int>((i / args.num_groups) % args.batch);
    ti.tile = tiles_max - 1 - static_cast<int>(i / (static_cast<int64_t>(args.num_groups) * args.batch));
    // Null cu_seqlens (projection only): all rows form one sequence.
    ti.q0 = args.cu_q ? __ldg(args.cu_q + ti.b) : 0;
    ti.n = args.cu_q ? static_cast<int>(__ldg(args.cu_q + ti.b + 1) - ti.q0) : args.max_seqlen_q;
    ti.row0 = ti.tile * kRows;
    if (ti.row0 >= ti.n) return;  // whole CTA exits before touching barriers or TMEM
    ti.rows = min(kRows, ti.n - ti.row0);
    // Null cu_seqlens_c: one sequence whose atoms are all total_c rows of Ks.
    ti.c0 = args.cu_c ? __ldg(args.cu_c + ti.b) : 0;
    ti.atoms = args.cu_c ? static_cast<int>(__ldg(args.cu_c + ti.b + 1) - ti.c0)
                         : static_cast<int>(args.total_c);
    // Chunk mode: the rows are a slice [pos_offset, pos_offset + n) of a
    // sequence of seq_len tokens (sequence-parallel prefill).
    ti.pos0 = args.pos_offset;
    ti.pages = ((args.seq_len > 0 ? args.seq_len : ti.n) + 63) / 64;
    int needed_atoms = 0;
    if (MODE == kModeScore) {
      needed_atoms = ti.atoms;
    } else if (MODE == kModeSelect) {
      // Candidates of the last row are pages p <= qp_max - local - 1, whose
      // windows end at atom 4p + 3 < 4 (qp_max - local).
      const int qp_max = (ti.pos0 + ti.row0 + ti.rows - 1) / 64;
      needed_atoms = max(0, min(ti.atoms, 4 * (qp_max - args.local_blocks)));
    }
    ti.atom_tiles = (needed_atoms + kRows - 1) / kRows;
    ti.prologue = (MODE == kModeProject) || ti.atom_tiles > 0;
  }

  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint8_t* qs_smem = stages + kStages * kStageBytes;
  uint8_t* heap_base = qs_smem + (MODE == kModeProject ? 0 : kQsBytes);
  float* heap_s = reinterpret_cast<float*>(heap_base);
  uint16_t* heap_p = reinterpret_cast<uint16_t*>(heap_base + kHeapCap * kRows * 4);
  Barriers* bars = reinterpret_cast<Barriers*>(heap_base + (MODE == kModeSelect ? kHeapBytes : 0));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->qs_full, 1);
    mbar_init(&bars->qs_ready, 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_empty[s], 128);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  const uint32_t tmem_cols = MODE == kModeProject ? 128 : 512;
  if (warp == 1) tmem_alloc(&bars->tmem_base, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tmem_qs = tmem;          // columns [0, 128)
  const uint32_t tmem_s = tmem + 128;     // columns [128, 384): two 128-column buffers
  volatile int* abort_flag = &bars->abort_flag;
  int32_t* status = args.status;

  const int kd = args.hg * 128;           // K extent of phase A (Hg * D)
  const int nkb = kd / 64;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (elect_one()) {
      tma_prefetch_desc(&args.tm_q);
      tma_prefetch_desc(&args.tm_w);
      if (MODE != kModeProject) tma_prefetch_desc(&args.tm_ks);
      int it = 0;
      bool ok = true;
      if (ti.prologue) {
        const int32_t qrow = static_cast<int32_t>(ti.q0 + ti.row0);
        for (int kb = 0; kb < nkb && ok; ++kb, ++it) {
          const int s = it % kStages;
          ok = mbar_wait(&bars->empty[s], ((it / kStages) & 1) ^ 1, status, abort_flag);
          if (!ok) break;
          uint8_t* st = stages + s * kStageBytes;
          mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
          tma_load_2d(st, &args.tm_q, &bars->full[s], ti.g * kd + kb * 64, qrow);
          tma_load_2d(st + kHalfBytes, &args.tm_w, &bars->full[s], kb * 64, ti.g * kWidth);
        }
      }
      if (MODE != kModeProject) {
        for (int j = 0; j < ti.atom_tiles && ok; ++j, ++it) {
          const int s = it % kStages;
          ok = mbar_wait(&bars->empty[s], ((it / kStages) & 1) ^ 1, status, abort_flag);
          if (!ok) break;
          uint8_t* st = stages + s * kStageBytes;
          const int32_t arow =
              static_cast<int32_t>(ti.g * args.total_c + ti.c0 + static_cast<int64_t>(j) * kRows);
          mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
          tma_load_2d(st, &args.tm_ks, &bars->full[s], 0, arow);
          tma_load_2d(st + kHalfBytes, &args.tm_ks, &bars->full[s], 64, arow);
        }
      }
      if (!ok) {
        // Let copies already in flight land before the CTA releases its memory.
        for (int k = max(0, it - kStages); k < it; ++k)
          mbar_wait(&bars->full[k % kStages], (k / kStages) & 1, nullptr, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      if (ti.prologue) {
        for (int kb = 0; kb < nkb && ok; ++kb, ++it) {
          const int s = it % kStages;
          ok = mbar_wait(&bars->full[s], (it / kStages) & 1, status, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a = smem_u32(stages + s * kStageBytes);
          const uint32_t b = a + kHalfBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_ss(tmem_qs, umma_desc_sw128(a + kk * 32), umma_desc_sw128(b + kk * 32),
                         kIdesc, (kb | kk) != 0);
          umma_commit(&bars->empty[s]);
        }
        umma_commit(&bars->qs_full);
      }
      if (MODE != kModeProject && ok && ti.atom_tiles > 0) {
        ok = mbar_wait(&bars->qs_ready, 0, status, abort_flag);
        tc_fence_after();
        const uint32_t qa = smem_u32(qs_smem);
        for (int j = 0; j < ti.atom_tiles && ok; ++j, ++it) {
          const int s = it % kStages;
          const int buf = j & 1;
          ok = mbar_wait(&bars->full[s], (it / kStages) & 1, status, abort_flag);
          if (ok) ok = mbar_wait(&bars->s_empty[buf], ((j >> 1) & 1) ^ 1, status, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t kb_addr = smem_u32(stages + s * kStageBytes);
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16_ss(tmem_s + buf * 128, umma_desc_sw128(qa + h * kHalfBytes + kk * 32),
                           umma_desc_sw128(kb_addr + h * kHalfBytes + kk * 32), kIdesc,
                           (h | kk) != 0);
          umma_commit(&bars->empty[s]);
          umma_commit(&bars->s_full[buf]);
        }
      }
      // All MMAs issued by this thread must retire before TMEM is released.
      umma_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, nullptr, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const bool valid = row < ti.rows;
    const int t_rel = ti.pos0 + ti.row0 + row;       // position inside the sequence
    const int64_t q_row = ti.q0 + ti.row0 + row;     // packed row
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    bool ok = true;

    // Per-row selection geometry (minicpm.py:3121-3138).
    const int qp = t_rel / 64;
    const int take_b = min(args.take, ti.pages);
    const int n_init = min(args.init_blocks, qp + 1);      // visible sink pages 0 .. n_init-1
    const int lo = max(0, qp - args.local_blocks);          // local pages lo .. qp
    const int overlap = max(0, n_init - lo);
    const int n_forced = n_init + (qp - lo + 1) - overlap;
    const int n_cand = max(0, lo - n_init);                 // visible non-forced pages n_init .. lo-1
    const int cap = max(0, min(take_b - n_forced, n_cand));
    int hsize = 0;

    if (ti.prologue) {
      ok = mbar_wait(&bars->qs_full, 0, status, abort_flag);
      tc_fence_after();
      if (ok) {
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          float v[32];
          tmem_ld32(tmem_qs + lane_base + q * 32, v);
          uint4 packed[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            packed[c].x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
            packed[c].y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
            packed[c].z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
            packed[c].w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
          }
          if (MODE == kModeProject) {
            if (valid) {
              uint4* dst = reinterpret_cast<uint4*>(
                  args.qs_out + (static_cast<int64_t>(ti.g) * args.total_q + q_row) * kWidth + q * 32);
#pragma unroll
              for (int c = 0; c < 4; ++c) dst[c] = packed[c];
            }
          } else {
            uint8_t* half = qs_smem + (q >> 1) * kHalfBytes + row * 128;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int chunk = (q & 1) * 4 + c;
              *reinterpret_cast<uint4*>(half + ((chunk ^ (row & 7)) << 4)) = packed[c];
            }
          }
        }
      }
      if (MODE != kModeProject) {
        fence_proxy_async_smem();
        mbar_arrive(&bars->qs_ready);
      }
    }

    if (MODE != kModeProject) {
      float carry = -INFINITY;  // score of the last atom of the previous tile
      const int last_atom = ti.atoms - 1;
      for (int j = 0; j < ti.atom_tiles && ok; ++j) {
        const int buf = j & 1;
        ok = mbar_wait(&bars->s_full[buf], (j >> 1) & 1, status, abort_flag);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          float v[32];
          tmem_ld32(tmem_s + buf * 128 + lane_base + q * 32, v);
          const int a_base = j * 128 + q * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (a_base + i > last_atom) v[i] = -INFINITY;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float m = i == 0 ? carry : v[4 * i - 1];
            m = fmaxf(m, fmaxf(fmaxf(v[4 * i], v[4 * i + 1]), fmaxf(v[4 * i + 2], v[4 * i + 3])));
            const int p = j * 32 + q * 8 + i;
            if (MODE == kModeScore) {
              if (valid && p < args.max_pages)
                args.page_scores[(static_cast<int64_t>(ti.g) * args.total_q + q_row) * args.max_pages + p] =
                    p < ti.pages ? m : -INFINITY;
            } else {
              // Candidate: visible, not forced, finite.
              if (valid && p >= n_init && p < lo && m > -INFINITY && cap > 0) {
                if (hsize < cap) {
                  int k = hsize++;
                  while (k > 0) {
                    const int parent = (k - 1) >> 1;
                    const float ps = heap_s[parent * kRows + row];
                    const uint32_t pp = heap_p[parent * kRows + row];
                    if (!worse(m, p, ps, pp)) break;
                    heap_s[k * kRows + row] = ps;
                    heap_p[k * kRows + row] = static_cast<uint16_t>(pp);
                    k = parent;
                  }
                  heap_s[k * kRows + row] = m;
                  heap_p[k * kRows + row] = static_cast<uint16_t>(p);
                } else if (m > heap_s[row]) {
                  int k = 0;
                  while (true) {
                    const int l = 2 * k + 1;
                    if (l >= hsize) break;
                    int c = l;
                    float cs = heap_s[l * kRows + row];
                    uint32_t cp = heap_p[l * kRows + row];
                    if (l + 1 < hsize) {
                      const float rs = heap_s[(l + 1) * kRows + row];
                      const uint32_t rp = heap_p[(l + 1) * kRows + row];
                      if (worse(rs, rp, cs, cp)) { c = l + 1; cs = rs; cp = rp; }
                    }
                    if (!worse(cs, cp, m, p)) break;
                    heap_s[k * kRows + row] = cs;
                    heap_p[k * kRows + row] = static_cast<uint16_t>(cp);
                    k = c;
                  }
                  heap_s[k * kRows + row] = m;
                  heap_p[k * kRows + row] = static_cast<uint16_t>(p);
                }
              }
            }
          }
          carry = v[31];
        }
        tc_fence_before();
        mbar_arrive(&bars->s_empty[buf]);
      }
      if (MODE == kModeScore && valid) {
        // Pages past the last computed tile: only page 32*tiles can still see an atom.
        for (int p = ti.atom_tiles * 32; p < args.max_pages; ++p)
          args.page_scores[(static_cast<int64_t>(ti.g) * args.total_q + q_row) * args.max_pages + p] =
              (p == ti.atom_tiles * 32 && p < ti.pages) ? carry : -INFINITY;
      }
      if (MODE == kModeSelect && valid) {
        int32_t* out = args.topk_idx + (static_cast<int64_t>(ti.g) * args.total_q + q_row) * args.take;
        int k = 0;
        if (ti.atoms > 0) {
          // Forced pages first (sink pages, then local pages), lowest index first.
          for (int p = 0; p < n_init && k < take_b; ++p) out[k++] = p;
          for (int p = max(lo, n_init); p <= qp && k < take_b; ++p) out[k++] = p;
          for (int i = 0; i < hsize; ++i) out[k++] = heap_p[i * kRows + row];
        }
        for (; k < args.take; ++k) out[k] = -1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

}  // namespace

cudaError_t launch_score(int mode, const ScoreArgs& args, cudaStream_t stream) {
  const int tiles_max = (args.max_seqlen_q + kRows - 1) / kRows;
  const int64_t grid = static_cast<int64_t>(tiles_max) * args.batch * args.num_groups;
  if (grid == 0) return cudaSuccess;
  const size_t smem = smem_bytes(mode);
  cudaError_t err = cudaSuccess;
  switch (mode) {
    case kModeProject:
      err = cudaFuncSetAttribute(score_kernel<kModeProject>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return err;
      score_kernel<kModeProject><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(args);
      break;
    case kModeScore:
      err = cudaFuncSetAttribute(score_kernel<kModeScore>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return err;
      score_kernel<kModeScore><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(args);
      break;
    case kModeSelect:
      err = cudaFuncSetAttribute(score_kernel<kModeSelect>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return err;
      score_kernel<kModeSelect><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(args);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

size_t score_smem_bytes(int mode) { return smem_bytes(mode); }

}  // namespace ls
