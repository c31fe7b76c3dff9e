// Selector scoring and page selection on the 5th-generation tensor cores.
//
// score_kernel: one CTA owns a tile of 128 query rows of one sequence and one
// KV group.
//
//   Phase A  Qs = Q_tile[128, Hg*D] x WqT_g[F, Hg*D]^T            (a3, selector.py:160-177)
//            TMA streams 64-wide K blocks of Q and WqT through a 2-stage ring,
//            one thread issues tcgen05.mma (M=128, N=128, K=16) into TMEM.
//            The epilogue warps round Qs to bf16 (the reference's bf16 einsum
//            output) and store it back to shared memory as the A operand of
//            phase B (128B-swizzled K-major, the layout TMA would write).
//   Phase B  for each tile of 128 atoms: S = Qs x Ks_tile^T        (a5, selector.py:203-207)
//            into one of two TMEM accumulators (double buffered; buffer 0
//            reuses the drained Qs columns), while the epilogue warps drain
//            the other: each thread owns one query row and max-pools atoms
//            into pages (window 5, stride 4, pad 1; a6, pages.py:146-187),
//            32 pages per atom tile, written as fp32 either to the caller's
//            page-score output (score mode) or to the selection workspace
//            (select mode); atom mode instead writes the raw bf16 atom
//            scores (NOSA's precomputed scores).  In select mode only the atom
//            tiles that can reach a candidate page of the tile's last row are
//            computed.
//
// topk_kernel (select mode, a7 minicpm.py:3124-3141): one warp per (group,
// query row) reads the row's candidate pages (visible, not forced) from the
// workspace and finds the best T' = min(take_b, P_b) - forced by an exact
// MSB-first radix select on order-preserving 32-bit keys (4 passes of 8
// bits, histograms in shared memory), breaking ties toward the lower page.
// It writes sink pages, selected pages and local pages -- ascending -- then
// -1 padding.
//
// Warp roles of score_kernel (192 threads): warp 0 TMA producer, warp 1 MMA
// issuer and TMEM owner, warps 2-5 epilogue (warp w reads TMEM lanes
// 32*(w%4) .. +31).  Two CTAs fit on an SM (shared memory and 256 TMEM
// columns each), so one CTA's phase A overlaps another's phase B.
#include <algorithm>

#include "common.cuh"
#include "launch.h"
#include "topk_rows.cuh"

namespace ls {
namespace {

constexpr int kRows = 128;
constexpr int kWidth = 128;          // F
constexpr int kStages = 2;
constexpr int kHalfBytes = 128 * 128;        // [128 rows x 64 bf16]
constexpr int kStageBytes = 2 * kHalfBytes;  // A+B (phase A) or one Ks tile (phase B)
constexpr int kQsBytes = 2 * kHalfBytes;
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

constexpr int kStoreStageBytes = 4 * 32 * 8 * 4;  // per epilogue warp: 32 rows x 8 pages fp32

__host__ __device__ constexpr size_t smem_bytes(int mode) {
  return 1024  // alignment slack
         + static_cast<size_t>(kStages) * kStageBytes + (mode == kModeProject ? 0 : kQsBytes) +
         sizeof(Barriers) + 16 + kStoreStageBytes;
}

struct TileInfo {
  int g, b, tile;
  int64_t q0;       // first packed query row of the sequence
  int n;            // query rows of the sequence
  int row0;         // first row of the tile inside the sequence
  int rows;         // valid rows in the tile
  int64_t c0;       // first packed atom of the sequence
  int atoms;        // atoms of the sequence
  int pages;        // pages of the sequence
  int pos0;         // position of row 0 inside the sequence (chunk mode), else 0
  int atom_tiles;   // atom tiles the tile needs
  bool prologue;    // whether Qs is computed at all
};

// Uniform method page score: the reference's bf16 matmul output times the
// softmax scale, rounded to bf16 again (head_mix.py:47-53, bf16 inputs).
// Pooling commutes with this monotone map, so it is applied per page.
__device__ __forceinline__ float uniform_score(float s, float scale) {
  const float r = __bfloat162float(__float2bfloat16_rn(s));
  return __bfloat162float(__float2bfloat16_rn(r * scale));
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 2) score_kernel(const __grid_constant__ ScoreArgs args) {
  const int tiles_max = (args.max_seqlen_q + kRows - 1) / kRows;
  TileInfo ti;
  {
    const int64_t i = blockIdx.x;
    ti.g = static_cast<int>(i % args.num_groups);
    ti.b = static_cast<int>((i / args.num_groups) % args.batch);
    ti.tile = tiles_max - 1 - static_cast<int>(i / (static_cast<int64_t>(args.num_groups) * args.batch));
    // Null cu_seqlens (projection, chunk mode): all rows form one sequence.
    ti.q0 = args.cu_q ? __ldg(args.cu_q + ti.b) : 0;
    ti.n = args.cu_q ? static_cast<int>(__ldg(args.cu_q + ti.b + 1) - ti.q0) : args.max_seqlen_q;
    ti.row0 = ti.tile * kRows;
    if (ti.n > args.max_seqlen_q) {
      // max_seqlen_q sizes the workspace rows: a longer sequence is a caller error.
      if (ti.tile == 0 && threadIdx.x == 0) report(args.status, LS_DEVERR_SEQLENS);
      return;
    }
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
    if (MODE == kModeScore || MODE == kModeAtoms) {
      needed_atoms = ti.atoms;
    } else if (MODE == kModeSelect) {
      // Candidates of the last row are pages p <= qp_max - local - 1, whose
      // windows end at atom 4p + 3 < 4 (qp_max - local).  Uniform method:
      // also page qp_max + 1, whose only visible atom is 4 qp_max + 3.
      const int qp_max = (ti.pos0 + ti.row0 + ti.rows - 1) / 64;
      needed_atoms = args.uniform ? min(ti.atoms, 4 * qp_max + 4)
                                  : max(0, min(ti.atoms, 4 * (qp_max - args.local_blocks)));
    }
    ti.atom_tiles = (needed_atoms + kRows - 1) / kRows;
    ti.prologue = (MODE == kModeProject) || ti.atom_tiles > 0;
  }
  // Select mode: a tile without candidate pages has nothing to score
  // (such rows have no candidates, so the top-k kernel reads nothing).
  // Score mode: a sequence without atoms scores -inf everywhere.
  if (!ti.prologue) {
    if (MODE == kModeAtoms) {
      const int64_t count = static_cast<int64_t>(ti.rows) * args.max_atoms;
      for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
        const int64_t q_row = ti.q0 + ti.row0 + i / args.max_atoms;
        args.atom_out[(static_cast<int64_t>(ti.g) * args.total_q + q_row) * args.max_atoms +
                      i % args.max_atoms] = 0xFF80u;  // bf16 -inf
      }
    }
    if (MODE == kModeScore) {
      const int64_t count = static_cast<int64_t>(ti.rows) * args.max_pages;
      for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
        const int64_t q_row = ti.q0 + ti.row0 + i / args.max_pages;
        args.page_scores[(static_cast<int64_t>(ti.g) * args.total_q + q_row) * args.max_pages +
                         i % args.max_pages] = -INFINITY;
      }
    }
    return;
  }

  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stages = smem;
  uint8_t* qs_smem = stages + kStages * kStageBytes;
  Barriers* bars =
      reinterpret_cast<Barriers*>(qs_smem + (MODE == kModeProject ? 0 : kQsBytes));
  // Page-score staging: each epilogue warp turns its 32 rows x 8 pages into
  // row-contiguous 32-byte stores.
  float* store_stage = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(bars + 1) + 15) & ~static_cast<uintptr_t>(15));

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
  const uint32_t tmem_cols = MODE == kModeProject ? 128 : 256;
  if (warp == 1) tmem_alloc(&bars->tmem_base, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tmem_qs = tmem;  // columns [0, 128); reused as S buffer 0 in phase B
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
      if (MODE != kModeProject && ok) {
        // Qs has been drained from TMEM and stored to shared memory.
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
              umma_bf16_ss(tmem + buf * 128, umma_desc_sw128(qa + h * kHalfBytes + kk * 32),
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
    const int64_t q_row = ti.q0 + ti.row0 + row;     // packed row
    const int pos = ti.pos0 + ti.row0 + row;          // position inside the sequence
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    bool ok = mbar_wait(&bars->qs_full, 0, status, abort_flag);
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
      tc_fence_before();
      fence_proxy_async_smem();
      mbar_arrive(&bars->qs_ready);

      // Score mode: fp32 page scores of the caller.  Select mode: bf16 page
      // scores in the workspace (rows padded to a multiple of 8 pages).
      float* out_row = MODE == kModeScore
                           ? args.page_scores +
                                 (static_cast<int64_t>(ti.g) * args.total_q + q_row) * args.max_pages
                           : nullptr;
      uint16_t* ws_row = MODE == kModeSelect
                             ? args.workspace +
                                   (static_cast<int64_t>(ti.g) * args.total_q + q_row) * args.max_pages
                             : nullptr;
      uint16_t* atom_row = MODE == kModeAtoms
                               ? args.atom_out +
                                     (static_cast<int64_t>(ti.g) * args.total_q + q_row) * args.max_atoms
                               : nullptr;
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
          tmem_ld32(tmem + buf * 128 + lane_base + q * 32, v);
          const int a_base = j * 128 + q * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (a_base + i > last_atom) v[i] = -INFINITY;
          if (MODE == kModeSelect && args.uniform) {
            // Atom a starts at token 16 a and is visible iff 16 a <= pos (pages.py:199-219).
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (16 * (a_base + i) > pos) v[i] = -INFINITY;
          }
          if constexpr (MODE == kModeAtoms) {
            // Raw atom scores, rounded to bf16 (the reference's bf16 einsum
            // output).  Rows lie max_atoms elements apart, of any parity, so
            // each half of the warp's 32 rows x 32 atoms is staged in shared
            // memory and written back as contiguous 32-byte row segments, two
            // rows per store instruction (not 32 rows of 2 bytes).
            uint16_t* st16 = reinterpret_cast<uint16_t*>(store_stage + quad * 256);
            const int64_t row_base = static_cast<int64_t>(ti.g) * args.total_q + ti.q0 + ti.row0 +
                                     quad * 32;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int a0 = a_base + 16 * h;
              if (a0 >= args.max_atoms) break;  // the same for the whole warp
              uint4 u0, u1;
              u0.x = pack_bf16x2(v[16 * h + 0], v[16 * h + 1]);
              u0.y = pack_bf16x2(v[16 * h + 2], v[16 * h + 3]);
              u0.z = pack_bf16x2(v[16 * h + 4], v[16 * h + 5]);
              u0.w = pack_bf16x2(v[16 * h + 6], v[16 * h + 7]);
              u1.x = pack_bf16x2(v[16 * h + 8], v[16 * h + 9]);
              u1.y = pack_bf16x2(v[16 * h + 10], v[16 * h + 11]);
              u1.z = pack_bf16x2(v[16 * h + 12], v[16 * h + 13]);
              u1.w = pack_bf16x2(v[16 * h + 14], v[16 * h + 15]);
              reinterpret_cast<uint4*>(st16 + lane * 16)[0] = u0;
              reinterpret_cast<uint4*>(st16 + lane * 16)[1] = u1;
              __syncwarp();
              const int col = lane & 15;
#pragma unroll 4
              for (int rr = 0; rr < 32; rr += 2) {
                const int r = rr + (lane >> 4);
                if (quad * 32 + r < ti.rows && a0 + col < args.max_atoms)
                  args.atom_out[(row_base + r) * args.max_atoms + a0 + col] = st16[r * 16 + col];
              }
              __syncwarp();
            }
          } else {
            // Page p of this block pools atoms [4p-1, 4p+4): its first atom is
            // the previous block's last one (carry).  The reference rounds the
            // atom scores to bf16 (its bf16 einsum output, selector.py:203-207)
            // before pooling; rounding is monotone, so rounding the pooled
            // maximum once gives the same value.
            float pg[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float m = i == 0 ? carry : v[4 * i - 1];
              pg[i] = fmaxf(m, fmaxf(fmaxf(v[4 * i], v[4 * i + 1]), fmaxf(v[4 * i + 2], v[4 * i + 3])));
            }
            carry = v[31];
            const int p0 = j * 32 + q * 8;
            if constexpr (MODE == kModeSelect) {
              // Uniform method: bf16(bf16(s) * scale) is already a bf16 value.
              if (args.uniform) {
#pragma unroll
                for (int i = 0; i < 8; ++i) pg[i] = uniform_score(pg[i], args.score_scale);
              }
              if (valid && p0 < args.max_pages) {
                uint4 u;
                u.x = pack_bf16x2(pg[0], pg[1]);
                u.y = pack_bf16x2(pg[2], pg[3]);
                u.z = pack_bf16x2(pg[4], pg[5]);
                u.w = pack_bf16x2(pg[6], pg[7]);
                *reinterpret_cast<uint4*>(ws_row + p0) = u;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) pg[i] = __bfloat162float(__float2bfloat16_rn(pg[i]));
              if (valid && p0 < args.max_pages) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  if (p0 + i >= ti.pages) pg[i] = -INFINITY;
              }
              if ((args.max_pages & 7) == 0) {
                // Rows of a multiple of 8 pages: stage the warp's 32 x 8 block
                // in shared memory and write it back as 32-byte row segments,
                // two lanes per row.
                if (valid && p0 < args.max_pages) {
                  float* st = store_stage + quad * 256;
                  *reinterpret_cast<float4*>(st + lane * 8) = make_float4(pg[0], pg[1], pg[2], pg[3]);
                  *reinterpret_cast<float4*>(st + lane * 8 + 4) = make_float4(pg[4], pg[5], pg[6], pg[7]);
                }
                if (p0 < args.max_pages) {
                  __syncwarp();
                  const float* st = store_stage + quad * 256;
                  float* wbase = args.page_scores +
                                 (static_cast<int64_t>(ti.g) * args.total_q + ti.q0 + ti.row0 +
                                  quad * 32) * args.max_pages + p0;
#pragma unroll
                  for (int i = 0; i < 2; ++i) {
                    const int c = lane + 32 * i;  // row c / 2, half c % 2
                    const int r = c >> 1;
                    if (quad * 32 + r < ti.rows)
                      *reinterpret_cast<float4*>(wbase + static_cast<int64_t>(r) * args.max_pages +
                                                 4 * (c & 1)) =
                          *reinterpret_cast<const float4*>(st + r * 8 + 4 * (c & 1));
                  }
                  __syncwarp();
                }
              } else if (valid && p0 < args.max_pages) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  if (p0 + i < args.max_pages) out_row[p0 + i] = pg[i];
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&bars->s_empty[buf]);
      }
      if (MODE == kModeAtoms && valid && ok) {
        for (int a = ti.atom_tiles * 128; a < args.max_atoms; ++a) atom_row[a] = 0xFF80u;
      }
      if (MODE == kModeScore && valid && ok) {
        // Pages past the last computed tile: only page 32*tiles can still see
        // an atom (the last one, carried).
        const float tail = __bfloat162float(__float2bfloat16_rn(carry));
        for (int p = ti.atom_tiles * 32; p < args.max_pages; ++p)
          out_row[p] = (p == ti.atom_tiles * 32 && p < ti.pages) ? tail : -INFINITY;
      }
      if (MODE == kModeSelect && valid && ok) {
        // Candidate pages past the last computed tile (up to the row's last
        // candidate): only page 32*tiles can still see an atom (the carried one).
        const int qp = pos / 64;
        const int end = args.uniform ? min(args.max_pages, qp + 2)
                                     : min(args.max_pages, qp - args.local_blocks);
        const float tail = args.uniform ? uniform_score(carry, args.score_scale) : carry;
        const uint16_t tail_bits = __bfloat16_as_ushort(__float2bfloat16_rn(tail));
        for (int p = ti.atom_tiles * 32; p < end; ++p)
          ws_row[p] = (p == ti.atom_tiles * 32 && p < ti.pages) ? tail_bits : uint16_t{0xFF80u};
        if (args.uniform && qp + 1 < ti.pages && qp + 1 < args.max_pages) {
          // Page qp+1 competes as the candidate after the last regular one:
          // move its score into that slot (the first non-sink local page,
          // whose own score is never read; the same thread wrote both).
          const int slot = max(max(0, qp - args.local_blocks), min(args.init_blocks, qp + 1));
          ws_row[slot] = ws_row[qp + 1];
        }
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

// ---------------------------------------------------------------------------
// Top-T' page selection per (group, row)
// ---------------------------------------------------------------------------

constexpr int kTopkWarps = 4;
constexpr int kTopkBlocksPerSm = 7;        // 7 x 4 warps x 7.2 KB of shared memory per SM
constexpr int kRowCap = 2048;              // candidates a warp stages in shared memory
constexpr int kRowChunks = kRowCap / 8 + 1;  // 16-byte chunks, +1 for a misaligned start
constexpr int kKeptCap = 512;              // candidates kept above the estimated cut

struct TopkWarpSmem {
  uint4 row[kRowChunks];        // the row's candidate scores (bf16), 16-byte aligned copy
  uint32_t hist[256];           // radix histogram
  uint32_t kept[kKeptCap];      // candidates at or above the cut, in candidate order:
                                // key << 16 | candidate index
};

constexpr size_t topk_smem_bytes() { return kTopkWarps * sizeof(TopkWarpSmem); }

// Order-preserving 16-bit key of a bf16 score; -inf and NaN map to 0 (never
// picked).  Finite scores map to 0x0080 .. 0xFF7F and +inf to 0xFF80; -0
// and +0 share a key (they compare equal, so they tie).
__device__ __forceinline__ uint32_t bf16_key(uint32_t b) {
  b = b == 0x8000u ? 0u : b;
  const uint32_t k = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  return (k <= 0x7Fu || k > 0xFF80u) ? 0u : k;
}

__device__ __forceinline__ float bf16_value(uint32_t b) { return __uint_as_float(b << 16); }

__device__ __forceinline__ uint32_t chunk_bits(const uint4& v, int e) {
  const uint32_t w = e < 2 ? v.x : e < 4 ? v.y : e < 6 ? v.z : v.w;
  return (e & 1) ? (w >> 16) : (w & 0xFFFFu);
}

// A row's candidates as 16-byte chunks: candidate i is element off + i of
// the chunk sequence (the copy starts at the 8-page boundary below the first
// candidate).  Either the warp's shared-memory copy or the workspace row.
struct SmemChunks {
  const uint4* p;
  __device__ __forceinline__ uint4 chunk(int c) const { return p[c]; }
  __device__ __forceinline__ uint32_t bits(int e) const {
    return reinterpret_cast<const uint16_t*>(p)[e];
  }
};
struct GlobalChunks {
  const uint4* p;
  __device__ __forceinline__ uint4 chunk(int c) const { return __ldg(p + c); }
  __device__ __forceinline__ uint32_t bits(int e) const {
    return __ldg(reinterpret_cast<const unsigned short*>(p) + e);
  }
};

template <class Src>
struct ChunkKeys {        // key of candidate i
  Src src;
  int off;
  __device__ __forceinline__ uint32_t operator()(int i) const { return bf16_key(src.bits(off + i)); }
};
struct KeptKeys {         // entry j of the warp's kept buffer
  const uint32_t* k;
  __device__ __forceinline__ uint32_t operator()(int j) const { return k[j] >> 16; }
};

struct KeptIndex {
  const uint32_t* k;
  __device__ __forceinline__ int operator()(int j) const { return static_cast<int>(k[j] & 0xFFFFu); }
};

__device__ __forceinline__ __nv_bfloat162 as_bf162(uint32_t w) {
  return *reinterpret_cast<const __nv_bfloat162*>(&w);
}

// Flags (bit e) of the candidates of a 16-byte chunk whose score is >= cut:
// two bf16 compares per instruction; NaN never passes.
__device__ __forceinline__ uint32_t chunk_ge_flags(const uint4& v, __nv_bfloat162 cut) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t flags = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t mk = __hge2_mask(as_bf162(w[j]), cut);   // 0xFFFF per passing half
    flags |= ((mk & 1u) | ((mk >> 15) & 2u)) << (2 * j);
  }
  return flags;
}

// One pass over candidates 0 .. m-1 in rounds of 64 chunks (lane l takes
// chunks base + 2l and base + 2l + 1, sixteen consecutive candidates): the
// candidates whose score is >= `cut` are handed to `emit(pos, bits, i)`
// with consecutive positions in candidate order (`bits(e)` of the source
// re-reads a passing score).  Returns how many there were.
template <class Src, class Emit>
__device__ int compact_ge(const Src& src, int off, int m, __nv_bfloat162 cut, const Emit& emit,
                          int lane) {
  const int nch = (off + m + 7) >> 3;
  int total = 0;
  for (int base = 0; base < nch; base += 64) {
    const int c = base + 2 * lane;
    uint32_t flags = 0;  // bit e: candidate 8c - off + e passes
    if (c < nch) flags = chunk_ge_flags(src.chunk(c), cut);
    if (c + 1 < nch) flags |= chunk_ge_flags(src.chunk(c + 1), cut) << 8;
    const int first = 8 * c - off;  // candidate index of bit 0
    if (first < 0) flags &= 0xFFFFu << (-first);
    if (first + 16 > m) flags &= m - first <= 0 ? 0u : (0xFFFFu >> (16 - (m - first)));
    int round_total;
    int pos = total + warp_excl_scan(__popc(flags), lane, round_total);
    while (flags) {
      const int e = __ffs(flags) - 1;
      flags &= flags - 1;
      emit(pos++, src.bits(8 * c + e), first + e);
    }
    total += round_total;
  }
  return total;
}

// Selects the top `cap` of the m candidates of one row (ties to the lower
// candidate index) and writes their pages (n_init + i) to out[k_out ...] in
// ascending order.  Returns the next output position.
//
// Candidates at or above a cut estimated from a 1/8 sample (every 8th
// round of chunks; the normal quantile at the sample's mean and spread,
// aiming at ~2.5x the needed count) go to the warp's kept buffer in one
// pass; the exact radix select then runs over those.  When
// the estimate kept too few or too many, the exact radix runs over the
// whole row, read from the workspace (`row`).  `release()` is called once
// `src` will not be read again (its shared-memory copy may then be reused).
template <class Src, class Release>
__device__ int select_row(const Src& src, const GlobalChunks& row, int off, int m, int cap, int skip,
                          int n_init, int32_t* out, int k_out, TopkWarpSmem* ws,
                          const Release& release, int lane) {
  if (cap <= 0 || m <= 0) return k_out;
  // Every finite candidate selected: the skipped one (always the last) is
  // left out of the range, so it takes no output position.
  const __nv_bfloat162 finite2 = as_bf162(0xFF7FFF7Fu);  // lowest finite bf16, twice
  const int m_out = skip >= 0 ? skip : m;
  const auto write_out = [&](int pos, uint32_t, int i) { out[k_out + pos] = n_init + i; };
  if (cap >= m) {
    k_out += compact_ge(src, off, m_out, finite2, write_out, lane);
    __syncwarp();
    release();
    return k_out;
  }
  // ---- 1/8 sample (the first 256 candidates of every 2048): how many were
  // sampled, and the mean and spread of the finite ones.
  const int nch = (off + m + 7) >> 3;
  float s1 = 0.f, s2 = 0.f;
  int sampled = 0, finite_s = 0;
  for (int base = 0; base < nch; base += 256) {
    const int c = base + lane;
    if (c < nch) {
      const uint4 v = src.chunk(c);
      const int first = 8 * c - off;
      const bool full = first >= 0 && first + 8 <= m;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (full || (first + e >= 0 && first + e < m)) {
          ++sampled;
          const float x = bf16_value(chunk_bits(v, e));
          if (fabsf(x) < INFINITY) {  // NaN and infinities are left out
            ++finite_s;
            s1 += x;
            s2 = fmaf(x, x, s2);
          }
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sampled += __shfl_xor_sync(0xffffffffu, sampled, o);
    finite_s += __shfl_xor_sync(0xffffffffu, finite_s, o);
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  // The cut: the normal quantile, at the sample's mean and spread, above
  // which ~2.5x the needed count of candidates lies.  It is only an
  // estimate: whatever it keeps is searched exactly below, and a row where it
  // kept too few (< cap) or too many (> kKeptCap) is searched whole.  On the
  // benchmark's synthetic rows it keeps 1.1x - 2.7x of cap (1st - 99th
  // percentile), and no row of a 128K-token layer is searched whole.
  float cut = -INFINITY;
  if (finite_s > 1) {
    const float keep = 2.5f * static_cast<float>(cap) * static_cast<float>(sampled) /
                       (static_cast<float>(m) * static_cast<float>(finite_s));
    if (keep < 1.f) {
      const float mean = s1 / static_cast<float>(finite_s);
      const float var = fmaxf(0.f, s2 / static_cast<float>(finite_s) - mean * mean);
      cut = mean + normcdfinvf(1.f - keep) * sqrtf(var);
    }
  }
  // ---- one pass: keep the candidates at or above the cut, in candidate order.
  // A bf16 score is >= cut iff it is >= cut rounded up to bf16.
  const uint32_t cut_bits =
      cut > -INFINITY ? static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_ru(cut)))
                      : 0xFF7Fu;
  // Kept keys are >= the cut's key; their maximum is tracked on the way.
  uint32_t kept_max = 0u;
  const int kept = compact_ge(
      src, off, m, as_bf162(cut_bits | (cut_bits << 16)),
      [&](int pos, uint32_t bits, int i) {
        const uint32_t key = bf16_key(bits);
        kept_max = max(kept_max, key);
        if (pos < kKeptCap) ws->kept[pos] = key << 16 | static_cast<uint32_t>(i);
      },
      lane);
  __syncwarp();
  release();
  int need = cap;
  if (kept >= cap && kept <= kKeptCap) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kept_max = max(kept_max, __shfl_xor_sync(0xffffffffu, kept_max, o));
    const KeptKeys kk{ws->kept};
    const uint32_t thr = radix_threshold_in(kk, kept, need, ws->hist, lane,
                                            max(1u, bf16_key(cut_bits)), kept_max);
    return emit_threshold(kk, KeptIndex{ws->kept}, kept, thr, need, skip, n_init, out, k_out, lane);
  }
  // ---- exact radix over the whole row (the estimate kept too few or too many).
  const ChunkKeys<GlobalChunks> row_keys{row, off};
  int finite = 0;
  for (int i = lane; i < m; i += 32) finite += row_keys(i) != 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) finite += __shfl_xor_sync(0xffffffffu, finite, o);
  if (finite <= cap) return k_out + compact_ge(row, off, m_out, finite2, write_out, lane);
  const uint32_t thr = radix_threshold(row_keys, m, need, ws->hist, lane);
  return emit_threshold(row_keys, Identity{}, m, thr, need, skip, n_init, out, k_out, lane);
}

// Geometry of one (group, query) row of the top-k kernel (minicpm.py:3121-3138).
struct RowPlan {
  bool valid;           // a row to process
  bool empty;           // the row stays all -1 (bad seqlens, or no atoms outside uniform)
  int32_t* out;
  int64_t ws_row;       // element offset of the row in the workspace
  const uint4* row4;    // the candidates' 16-byte chunks in the workspace (bf16 rows)
  int off, nch;         // candidate i is element off + i of nch chunks
  int m_all, cap, future, n_init, take_b, local0, n_local;
  bool staged;          // copied into the warp's shared memory
};

__device__ __forceinline__ RowPlan plan_row(const ScoreArgs& args, uint32_t r, uint32_t total_q,
                                            uint32_t rows_total) {
  RowPlan p{};
  p.valid = r < rows_total;
  if (!p.valid) return p;
  row_geometry(args, r, total_q, &p.out, &p.ws_row, &p.empty, &p.m_all, &p.cap, &p.future,
               &p.n_init, &p.take_b, &p.local0, &p.n_local);
  if (p.empty) return p;
  // Chunks start at the 8-page boundary below the first candidate (rows are
  // 16-byte aligned).
  p.off = p.n_init & 7;
  p.row4 = reinterpret_cast<const uint4*>(args.workspace + p.ws_row) + (p.n_init >> 3);
  p.nch = (p.off + p.m_all + 7) >> 3;
  p.staged = p.cap > 0 && p.nch <= kRowChunks;
  return p;
}

// Starts the asynchronous 16-byte copies of a staged row into the warp's
// shared memory (no registers held, all of a lane's copies in flight).
__device__ __forceinline__ void stage_row(const RowPlan& p, TopkWarpSmem* ws, int lane) {
  if (!p.valid || !p.staged) return;
  for (int c = lane; c < p.nch; c += 32) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(ws->row + c)),
                 "l"(p.row4 + c)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Top-T' of each (group, query) row, one warp per row.  A row's candidate
// scores are bf16 values of the workspace; rows of at most kRowCap
// candidates are copied into the warp's shared memory, longer rows are read
// from the workspace.  The copy of a warp's next row starts as soon as the
// current row's copy is no longer read (after its filtering pass), so it
// overlaps the exact selection and the output of the current row.  The
// result is the same on every path: the T' largest scores, ties to the
// lower page.
__global__ void __launch_bounds__(kTopkWarps * 32, kTopkBlocksPerSm) topk_kernel(const __grid_constant__ ScoreArgs args) {
  extern __shared__ __align__(16) uint8_t topk_smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  TopkWarpSmem* ws = reinterpret_cast<TopkWarpSmem*>(topk_smem_raw) + warp;
  // Rows r = g * total_q + q_row with G * total_q < 2^31 (host checks), so
  // 32-bit unsigned arithmetic indexes them without wrapping.
  const uint32_t total_q = static_cast<uint32_t>(args.total_q);
  const uint32_t rows_total = static_cast<uint32_t>(args.num_groups) * total_q;
  const uint32_t stride = gridDim.x * kTopkWarps;
  uint32_t r = blockIdx.x * kTopkWarps + warp;
  RowPlan cur = plan_row(args, r, total_q, rows_total);
  stage_row(cur, ws, lane);
  while (cur.valid) {
    const RowPlan nxt = plan_row(args, r + stride, total_q, rows_total);
    bool next_staged = false;
    const auto release = [&]() {
      if (!next_staged) {
        next_staged = true;
        stage_row(nxt, ws, lane);
      }
    };
    int32_t* out = cur.out;
    if (cur.empty) {
      for (int k = lane; k < args.take; k += 32) out[k] = -1;
    } else {
      const int sinks_out = min(cur.n_init, cur.take_b);
      for (int k = lane; k < sinks_out; k += 32) out[k] = k;
      int k_out = sinks_out;
      if (cur.cap > 0) {
        const GlobalChunks row{cur.row4};
        if (cur.staged) {
          asm volatile("cp.async.wait_all;" ::: "memory");
          __syncwarp();
          k_out = select_row(SmemChunks{ws->row}, row, cur.off, cur.m_all, cur.cap, cur.future,
                             cur.n_init, out, k_out, ws, release, lane);
        } else {
          k_out = select_row(row, row, cur.off, cur.m_all, cur.cap, cur.future, cur.n_init, out,
                             k_out, ws, release, lane);
        }
        __syncwarp();
      }
      // Local pages (those that are not sinks), then padding.
      const int local_out = max(0, min(cur.n_local, cur.take_b - k_out));
      for (int k = lane; k < local_out; k += 32) out[k_out + k] = cur.local0 + k;
      k_out += local_out;
      for (int k = k_out + lane; k < args.take; k += 32) out[k] = -1;
    }
    __syncwarp();
    release();
    cur = nxt;
    r += stride;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

}  // namespace

size_t select_workspace_bytes(int64_t rows, int max_pages) {
  return sizeof(uint16_t) * static_cast<size_t>(rows) * static_cast<size_t>((max_pages + 7) & ~7);
}

cudaError_t launch_score(int mode, const ScoreArgs& args_in, cudaStream_t stream) {
  ScoreArgs args = args_in;
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
    case kModeAtoms:
      err = cudaFuncSetAttribute(score_kernel<kModeAtoms>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return err;
      score_kernel<kModeAtoms><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(args);
      break;
    case kModeSelect: {
      // Workspace rows are padded to a multiple of 8 pages (32-byte aligned stores).
      args.max_pages = (args.max_pages + 7) & ~7;
      err = cudaFuncSetAttribute(score_kernel<kModeSelect>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return err;
      score_kernel<kModeSelect><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(args);
      err = cudaGetLastError();
      if (err != cudaSuccess) return err;
      const int64_t rows = static_cast<int64_t>(args.num_groups) * args.total_q;
      const int64_t blocks =
          std::min<int64_t>((rows + kTopkWarps - 1) / kTopkWarps, 148 * kTopkBlocksPerSm * 4);
      err = cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(topk_smem_bytes()));
      if (err != cudaSuccess) return err;
      topk_kernel<<<static_cast<unsigned>(blocks), kTopkWarps * 32, topk_smem_bytes(), stream>>>(args);
      break;
    }
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace ls
