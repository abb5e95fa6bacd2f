// dsa_indexer_sm100.cu — the DSA top-k indexer on sm_100a
// (definition dsa_topk_indexer_fp8_h64_d128_topk2048_ps64), the operator
// that produces sparse_indices for the attention kernel.
//
// For batch row b with seq_len sl (reference: methodology/reference/
// topk_kernel_naive.cu:65-111):
//   final[pos] = sum_h weights[b][h] * relu(q[b][h] . K[pos]),  pos < sl,
//   K[pos] = fp8 key row * its fp32 scale, read through block_table[b],
// and topk_indices[b] = the min(2048, sl) positions with the largest final,
// largest first (equal scores: lower position first), as slot ids
// block_table[b][pos >> 6] * 64 + (pos & 63); the rest -1.
//
// Two kernels:
//   score   two CTAs per SM, each over a contiguous range of the call's
//           128-position tiles (two pages) that hold positions: its share of
//           them, equal or from the plan calibrated on the previous calls
//           (see PlanState).  Warp 0 loads pages with TMA (a page is 64 rows
//           of 128 fp8 + 64 fp32 scales = 8448 bytes; the tensor map views the
//           cache as rows of 128 bytes, 66 per page, so the 64 data rows land
//           128-byte-swizzled for the tensor cores), looking up 32 tiles' page
//           ids at a time; warps 1-2 issue tcgen05.mma kind::f8f6f4 (e4m3 x
//           e4m3, M=128 positions, N=64 heads, K=32) for alternate tiles into
//           two TMEM accumulators; two groups of 4 warps (one TMEM lane = one
//           position per thread) apply scale, relu and the head weights and
//           write the position's final score (fp32) to the workspace.
//           HBM-bound: 132 bytes per position.
//   topk    a cluster of two CTAs (1024 threads each) per batch row: each
//           loads half the row's order-preserving keys into shared memory and
//           counts them into 2048 linear value bins between the row's smallest
//           and largest score (reduced by the score kernel); the halves' counts
//           are combined through distributed shared memory to find the bin of
//           the k-th key; the keys above it go to per-bin buckets and the
//           threshold bin's keys to a candidate list, both in CTA 0's shared
//           memory, where the candidates are ranked directly and each bucket
//           in place, writing the slot ids in order.  Rows over the direct-
//           ranking limits, and rows too long for shared memory, take a
//           single-CTA routine (radix passes, ordered gather, bitonic sort).
//           With a plan, one more CTA (cluster) past the rows turns the score
//           CTAs' logged run times into the next call's plan.

// Every wait is bounded (DSA_DEVICE_ERR_TIMEOUT on expiry).  A block-table
// entry outside [0, num_pages) for a page inside seq_len, or a seq_len larger
// than the table holds, is reported as DSA_DEVICE_ERR_BAD_INDEX; such
// positions score -inf and are never returned as slots.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cooperative_groups.h>

#include <cstdlib>
#include <mutex>

#include "dsa_common.cuh"
#include "dsa_sm100_ptx.cuh"

namespace dsa {
namespace indexer {

using namespace ptx;

constexpr int kHeads = 64;
constexpr int kDim = 128;
constexpr int kPageRows = 64;
constexpr int kPageBytes = 8448;
constexpr int kPageDataBytes = 8192;
constexpr int kRowsPerPage = kPageBytes / 128;   // 66 rows of 128 bytes in the tensor-map view
constexpr int kTileRows = 128;                   // positions per tile = two pages
constexpr int kTopk = 2048;

constexpr int kStages = 4;   // per CTA; two CTAs share an SM (two independent load pipelines)
// MMA warp m and epilogue group m take the tiles with n % 2 == m.  With an even
// stage count every use of a stage belongs to the same warp and group, so a
// parity wait on its full barrier always refers to that warp's previous phase;
// with an odd count the other warp's phase may still be pending and the
// parity test would pass early.
static_assert(kStages % 2 == 0, "stages must alternate with the MMA warps and epilogue groups");
constexpr uint32_t kStageBytes = kTileRows * kDim;   // 16 KB of fp8 keys
constexpr uint32_t kQBytes = kHeads * kDim;          // 8 KB of fp8 queries

constexpr uint32_t kScaleBytes = 2 * kPageRows * 4;   // the two pages' fp32 scales
constexpr uint32_t kOffStage = 0;
constexpr uint32_t kOffQ = kOffStage + kStages * kStageBytes;
constexpr uint32_t kOffScale = kOffQ + 2 * kQBytes;             // float [kStages][2][64]
constexpr uint32_t kOffW = kOffScale + kStages * kScaleBytes;   // float [2 groups][2][64] head weights
constexpr uint32_t kOffBar = kOffW + 4 * kHeads * 4;
enum : int {
  B_FULL = 0,
  B_EMPTY = B_FULL + kStages,
  B_Q_FULL = B_EMPTY + kStages,   // 2
  B_Q_EMPTY = B_Q_FULL + 2,       // 2
  B_D_FULL = B_Q_EMPTY + 2,       // 2
  B_D_EMPTY = B_D_FULL + 2,       // 2
  B_DONE = B_D_EMPTY + 2,         // 2: one per MMA warp
  B_COUNT = B_DONE + 2
};
constexpr uint32_t kOffMisc = kOffBar + B_COUNT * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 32 + 1024;   // misc: TMEM slot, abort flag, the CTA's tile range
static_assert(kOffQ % 1024 == 0 && kStageBytes % 1024 == 0, "swizzle atoms need 1 KB");

constexpr int kThreads = 352;   // warp 0 TMA, warps 1-2 MMA (warp 1 owns TMEM), warps 3-6 and 7-10 epilogue
constexpr uint32_t kEpiThreads = 128;   // one epilogue group: 4 warps, one per TMEM lane quarter
constexpr uint32_t kTmemCols = 128;   // two 64-column accumulators

// 128-byte-swizzled K-major operand descriptor (rows of 128 bytes, 8-row
// groups 1024 bytes apart).
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t(kDescHi) << 32) | uint64_t((1u << 16) | ((saddr & 0x3FFFFu) >> 4));
}
// Instruction descriptor, kind::f8f6f4: fp32 D (bits 4-5 = 1), A and B e4m3
// (format 0 in bits 7-9 and 10-12), both K-major, N >> 3 in bits 17-22, M >> 4
// in bits 24-28.
constexpr uint32_t kIdescF8 = (1u << 4) | (uint32_t(kHeads >> 3) << 17) | (uint32_t(kTileRows >> 4) << 24);

__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Order-preserving key: a larger float gives a larger unsigned key (-inf lowest
// of the ordinary values); -0 and +0 compare equal, so they share a key.
__device__ __forceinline__ uint32_t ordered_key(float x) {
  const uint32_t u = x == 0.f ? 0u : __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Score-kernel work split and its calibrated plan.  The roles skip a row's
// tiles past its length, so the CTAs split the call's ACTIVE tiles (those with
// positions): CTA g takes the active tiles between the cumulative fractions
// frac[g] and frac[g + 1] of their total, mapped to tile indices through the
// rows' active-tile prefix of the call (for full rows this is the equal split
// of the tile indices).  The fractions are g / grid, or a plan: equal shares
// still end at different times (CTAs over many short rows pay a query load,
// head weights and key-range atomics per row; on equal work the CTAs' rates
// differ by up to a quarter, the same CTAs slow from one call to the next),
// and the top-k kernel can start only once the slowest has ended.  So each
// score CTA logs its active tiles and
// its start and end times, and after the score grid the top-k grid's last CTA
// turns the log into the next call's fractions: each CTA's share in
// proportion to its measured rate (offset by how late it started), blended
// half and half with its current share so that noise is damped (taken whole
// after a call on g / grid).  Fractions carry over between calls of any shape
// with the same grid.  Any partition gives the same scores; the split changes
// only which CTA computes which tile.
constexpr uint32_t kPlanMagic = 0x4E414C50u;   // "PLAN"
constexpr uint32_t kPlanOne = 1u << 31;        // fraction 1
constexpr uint32_t kPlanUsed = 0x80000000u;    // log flag: the CTA's fractions came from a plan
constexpr int64_t kPlanMaxRows = kStageBytes / 4;   // rows' seq_lens staged in the first pipeline stage
struct PlanState {
  uint32_t magic, pad0, grid, pad1;
  uint32_t frac[kIndexerPlanMaxGrid + 4];   // CTA g: active tiles [frac[g], frac[g + 1]) x total / kPlanOne
  // per score CTA: x = tiles | kPlanUsed, y / z = start / end (low 32 bits
  // of %globaltimer, ns), w = active tiles
  uint4 log[kIndexerPlanMaxGrid];
};
static_assert(sizeof(PlanState) == kIndexerPlanBytes, "plan state layout");

struct ScoreParams {
  const uint8_t* cache;          // [num_pages, 8448]
  const float* weights;          // [B, 64]
  const int32_t* seq_lens;       // [B]
  const int32_t* block_table;    // [B, max_pages]
  float* scores;                 // [B, max_pages * 64]
  // [B][2]: max of the ordered keys of the row's scores and max of their
  // complements (= ~min); 0 = none.  The top-k kernel reads and clears them.
  uint32_t* row_keys;
  uint32_t* err_word;
  PlanState* plan;               // null: no calibrated plan, nothing logged
  int split_active;              // split the active tiles (rows <= kPlanMaxRows), else the tile indices
  int64_t batch;
  int64_t max_pages;
  int64_t num_pages;
  int64_t tiles_per_row;         // ceil(max_pages / 2)
  int64_t total_tiles;           // batch * tiles_per_row
  int grid;
};

struct Ctx {
  uint32_t sbase;
  uint32_t tmem;
  volatile uint32_t* abort;
  uint64_t timeout_ns;     // pipeline waits
  uint64_t drain_ns;       // waits for this CTA's own copies / MMAs after an abort
  int64_t t_begin, t_end;
};

__device__ __forceinline__ uint32_t bar(const Ctx& c, int b) { return c.sbase + kOffBar + 8u * uint32_t(b); }

// Bounded wait used only to drain this CTA's own copies / MMAs before exit.
__device__ __forceinline__ void drain_wait(uint32_t b, uint32_t parity, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(b, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) return;
  }
}

__device__ __forceinline__ int64_t range_begin(const ScoreParams& p, int64_t g) {
  return plan_div(g * p.total_tiles, p.grid);
}

// Positions of a row that the score kernel covers: seq_len clamped to what the
// table can hold (a larger seq_len is a bad index).
__device__ __forceinline__ int clamp_len(const ScoreParams& p, int sl) {
  const int64_t cap = p.max_pages * kPageRows;
  return sl <= 0 ? 0 : int(sl > cap ? cap : sl);
}
__device__ __forceinline__ int row_len(const ScoreParams& p, int64_t b) { return clamp_len(p, __ldg(p.seq_lens + b)); }

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Walks the plan's tiles as (row b, tile k of the row) without a division per
// tile; `sl` is row b's length, reloaded only when the row changes.
struct TileWalk {
  int64_t t, b, k;
  int sl;
  __device__ TileWalk(const ScoreParams& p, int64_t t0) : t(t0) {
    b = t0 / p.tiles_per_row;
    k = t0 - b * p.tiles_per_row;
    sl = b < p.batch ? row_len(p, b) : 0;
  }
  __device__ void next(const ScoreParams& p) {
    ++t;
    if (++k == p.tiles_per_row) {
      k = 0;
      ++b;
      if (b < p.batch) sl = row_len(p, b);
    }
  }
  // a row's tiles with positions come first: from the first one without, the
  // rest of the row is skipped (the following next() enters the next row)
  __device__ void skip_row(const ScoreParams& p) {
    t += p.tiles_per_row - 1 - k;
    k = p.tiles_per_row - 1;
  }
};

// Warp 0, before any copy: this CTA's tile range [tb, te) (see PlanState).
// The rows' seq_lens are copied (cp.async, one round trip for all rows) to
// `len_s` (the first pipeline stage, not yet in use; the load warp's first
// lookups read them there too); each lane sums the active tiles of a
// contiguous segment of rows, a warp scan gives the segments' prefixes, and
// each fraction's target maps to the last row whose prefix is <= the target
// plus the target's offset in that row.  With more rows than kPlanMaxRows,
// the equal split of the tile indices.
__device__ __forceinline__ uint32_t active_tiles(const ScoreParams& p, int32_t seq_len) {
  return uint32_t((clamp_len(p, seq_len) + kTileRows - 1) / kTileRows);
}

__device__ void cta_range(const ScoreParams& p, int32_t* len_s, int64_t& tb, int64_t& te, uint32_t& planned) {
  const int lane = threadIdx.x & 31;
  const int64_t g = blockIdx.x;
  planned = 0u;
  if (!p.split_active) {
    tb = range_begin(p, g);
    te = range_begin(p, g + 1);
    return;
  }
  const int64_t B = p.batch;
  uint4 h = make_uint4(0u, 0u, 0u, 0u);
  uint32_t f0 = 0u, f1 = 0u;
  if (lane == 0 && p.plan != nullptr) {   // loaded together with the rows' lengths below
    h = __ldcg(reinterpret_cast<const uint4*>(p.plan));
    f0 = __ldcg(p.plan->frac + g);
    f1 = __ldcg(p.plan->frac + g + 1);
  }
  for (int64_t r = lane; r < B; r += 32) cp_async4(smem_u32(len_s + r), p.seq_lens + r);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();
  const int64_t seg = (B + 31) / 32;
  const int64_t r0 = min(B, lane * seg), r1 = min(B, r0 + seg);
  uint32_t sum = 0u;
  for (int64_t r = r0; r < r1; ++r) sum += active_tiles(p, len_s[r]);
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
  const bool use = __shfl_sync(0xffffffffu, h.x == kPlanMagic && h.z == uint32_t(p.grid) && f0 <= f1 &&
                                                f1 <= kPlanOne, 0);
  f0 = __shfl_sync(0xffffffffu, f0, 0);
  f1 = __shfl_sync(0xffffffffu, f1, 0);
  uint32_t a0, a1;
  if (use) {
    a0 = uint32_t((uint64_t(total) * f0) >> 31);
    a1 = uint32_t((uint64_t(total) * f1) >> 31);
    planned = kPlanUsed;
  } else {
    a0 = uint32_t(uint64_t(total) * uint64_t(g) / uint64_t(p.grid));
    a1 = uint32_t(uint64_t(total) * uint64_t(g + 1) / uint64_t(p.grid));
  }
  int32_t lo0 = -1, lo1 = -1;
  uint32_t p0 = 0u, p1 = 0u, pr = incl - sum;
  for (int64_t r = r0; r < r1; ++r) {
    if (pr <= a0) {
      lo0 = int32_t(r);
      p0 = pr;
    }
    if (pr <= a1) {
      lo1 = int32_t(r);
      p1 = pr;
    }
    pr += active_tiles(p, len_s[r]);
  }
  // row 0's prefix is 0 <= any target, so both rows exist; one lane holds each
  const int32_t m0 = __reduce_max_sync(0xffffffffu, lo0), m1 = __reduce_max_sync(0xffffffffu, lo1);
  const uint32_t q0 = __shfl_sync(0xffffffffu, p0, __ffs(__ballot_sync(0xffffffffu, lo0 == m0)) - 1);
  const uint32_t q1 = __shfl_sync(0xffffffffu, p1, __ffs(__ballot_sync(0xffffffffu, lo1 == m1)) - 1);
  tb = int64_t(m0) * p.tiles_per_row + int64_t(a0 - q0);
  te = int64_t(m1) * p.tiles_per_row + int64_t(a1 - q1);
}

// ---------------------------------------------------------------- TMA warp
// The whole warp walks the tiles 32 at a time: lane l looks up tile t0 + l
// (its row, whether it has positions, its two page ids) with independent
// loads, then lane 0 issues the 32 tiles' TMA loads in order, taking the page
// ids from the lanes by shuffle -- no dependent global load per tile.
// Returns the number of tiles with positions (loaded) of the CTA's range.
// `len_s` (or null): the rows' lengths staged by cta_range in the first
// stage, read by the first lookups only (before the first copy).
__device__ int64_t load_warp(const Ctx& c, const ScoreParams& p, const CUtensorMap* tm_k, const CUtensorMap* tm_s,
                             const CUtensorMap* tm_q, const int32_t* len_s) {
  const int lane = threadIdx.x & 31;
  const uint64_t policy = l2_evict_first_policy();
  int64_t n = 0;
  int32_t prev_b = -1;
  int rows = 0;   // Q buffers loaded
  bool ok = true;
  uint32_t bad = 0;
  for (int64_t t0 = c.t_begin; t0 < c.t_end && ok;) {
    const int64_t t = t0 + lane;
    int32_t b = 0, pg0 = -1, pg1 = -1;
    bool act = false;
    if (t < c.t_end) {
      const int64_t bb = t / p.tiles_per_row, k = t - bb * p.tiles_per_row;
      b = int32_t(bb);
      const int sl = len_s != nullptr ? clamp_len(p, len_s[bb]) : row_len(p, bb);
      act = k * kTileRows < sl;
      if (act) {
        const int32_t* row_pages = p.block_table + bb * p.max_pages + 2 * k;
        pg0 = __ldg(row_pages);
        if ((2 * k + 1) * kPageRows < sl) pg1 = __ldg(row_pages + 1);
        else pg1 = -2;   // past the row's end: not a bad index
        if (pg0 < 0 || int64_t(pg0) >= p.num_pages) {
          bad = 1;
          pg0 = -1;
        }
        if (pg1 != -2 && (pg1 < 0 || int64_t(pg1) >= p.num_pages)) {
          bad = 1;
          pg1 = -1;
        }
      }
    }
    if (len_s != nullptr) {
      len_s = nullptr;
      fence_proxy_async_smem();   // the stage's generic-proxy reads end before its first copy
    }
    const int cnt = int(min(int64_t(32), c.t_end - t0));
    for (int j = 0; j < cnt && ok; ++j) {
      if (!__shfl_sync(0xffffffffu, act, j)) continue;
      const int32_t bj = __shfl_sync(0xffffffffu, b, j);
      const int32_t pages[2] = {__shfl_sync(0xffffffffu, pg0, j), __shfl_sync(0xffffffffu, pg1, j)};
      if (lane == 0) {
        if (bj != prev_b) {
          const int qb = rows & 1;
          if (rows >= 2)
            ok = mbar_wait(bar(c, B_Q_EMPTY + qb), uint32_t((rows >> 1) - 1) & 1u, c.abort, c.timeout_ns);
          if (ok) {
            mbar_arrive_expect_tx(bar(c, B_Q_FULL + qb), kQBytes);
            tma_load_2d(c.sbase + kOffQ + qb * kQBytes, tm_q, 0, bj * kHeads, bar(c, B_Q_FULL + qb));
          }
        }
        const int s = int(n % kStages);
        if (ok && n >= kStages)
          ok = mbar_wait(bar(c, B_EMPTY + s), uint32_t(n / kStages - 1) & 1u, c.abort, c.timeout_ns);
        if (ok) {
          mbar_arrive_expect_tx(bar(c, B_FULL + s), kStageBytes + kScaleBytes);
          for (int h = 0; h < 2; ++h) {
            // A page past the row's end or a bad one is loaded from row -66:
            // the tensor maps fill it with zeros (its positions are discarded,
            // or scored -inf by the top-k kernel).
            // The keys are read once: evicted from L2 first, so that the
            // scores the top-k kernel reads next stay there.
            const int row = pages[h] >= 0 ? pages[h] * kRowsPerPage : -kRowsPerPage;
            tma_load_2d_hint(c.sbase + kOffStage + s * kStageBytes + h * kPageDataBytes, tm_k, 0, row,
                             bar(c, B_FULL + s), policy);
            tma_load_2d_hint(c.sbase + kOffScale + s * kScaleBytes + h * (kScaleBytes / 2), tm_s, 0, row + kPageRows,
                             bar(c, B_FULL + s), policy);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (bj != prev_b) {
        ++rows;
        prev_b = bj;
      }
      ++n;
    }
    // the next 32 tiles; if the last one looked up has no positions, the rest
    // of its row has none either: continue at the next row
    const bool last_act = __shfl_sync(0xffffffffu, act, cnt - 1);
    const int32_t last_b = __shfl_sync(0xffffffffu, b, cnt - 1);
    t0 += cnt;
    if (!last_act) {
      const int64_t next_row = (int64_t(last_b) + 1) * p.tiles_per_row;
      t0 = next_row > t0 ? next_row : t0;
    }
  }
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    if (bad) report_error(p.err_word, DSA_DEVICE_ERR_BAD_INDEX);
    // every load must have landed before the CTA exits (also on an abort)
    if (n > 0) drain_wait(bar(c, B_FULL + int((n - 1) % kStages)), uint32_t((n - 1) / kStages) & 1u, c.drain_ns);
    if (rows > 0) drain_wait(bar(c, B_Q_FULL + ((rows - 1) & 1)), uint32_t((rows - 1) >> 1) & 1u, c.drain_ns);
  }
  return n;
}

// ---------------------------------------------------------------- MMA warp
// MMA warp m issues the tiles with n % 2 == m into TMEM accumulator m (one
// thread issues a tcgen05.mma only every ~150 ns, so two warps share the work).
__device__ void mma_warp(const Ctx& c, const ScoreParams& p, const int m) {
  int64_t n = 0, prev_b = -1;
  int rows = 0;
  bool ok = true;
  for (TileWalk tw(p, c.t_begin); tw.t < c.t_end && ok; tw.next(p)) {
    const int64_t b = tw.b, k = tw.k;
    const int sl = tw.sl;
    if (int64_t(k) * kTileRows >= sl) {
      tw.skip_row(p);
      continue;
    }
    if (b != prev_b) {
      if (rows > 0) mma_commit(bar(c, B_Q_EMPTY + ((rows - 1) & 1)));   // previous row's queries done (both warps)
      if (!(ok = mbar_wait(bar(c, B_Q_FULL + (rows & 1)), uint32_t(rows >> 1) & 1u, c.abort, c.timeout_ns))) break;
      ++rows;
      prev_b = b;
    }
    const int s = int(n % kStages), db = int(n & 1);
    if (db != m) {
      ++n;
      continue;
    }
    if (!(ok = mbar_wait(bar(c, B_FULL + s), uint32_t(n / kStages) & 1u, c.abort, c.timeout_ns))) break;
    if (n >= 2 && !(ok = mbar_wait(bar(c, B_D_EMPTY + db), uint32_t((n >> 1) - 1) & 1u, c.abort, c.timeout_ns)))
      break;
    tc_fence_after();
    const uint32_t a0 = c.sbase + kOffStage + s * kStageBytes;
    const uint32_t b0 = c.sbase + kOffQ + ((rows - 1) & 1) * kQBytes;
#pragma unroll
    for (int kk = 0; kk < kDim / 32; ++kk)
      mma_f8(c.tmem + 64u * db, desc_sw128(a0 + 32u * kk), desc_sw128(b0 + 32u * kk), kIdescF8, kk ? 1u : 0u);
    mma_commit(bar(c, B_EMPTY + s));
    mma_commit(bar(c, B_D_FULL + db));
    ++n;
  }
  mma_commit(bar(c, B_DONE + m));
  drain_wait(bar(c, B_DONE + m), 0u, c.drain_ns);
}

// ---------------------------------------------------------------- epilogue
// Two groups of 4 warps; group g takes the tiles with n % 2 == g (its own TMEM
// accumulator).  Thread r (TMEM lane r) owns position r of a tile:
// final = sum_h w[h] * relu(dot[h] * scale).  The stage is released once the
// MMA is done and the group has read its scales (stage barrier count 1 + 128).
__device__ void epilogue_warps(const Ctx& c, const ScoreParams& p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = (warp - 3) >> 2;          // group 0: warps 3-6, group 1: warps 7-10
  const int r = 32 * (warp & 3) + lane;
  const int gr = threadIdx.x - 96 - g * 128;   // 0..127 within the group
  const uint32_t t_lane = uint32_t(32 * (warp & 3)) << 16;
  int64_t n = 0, prev_b = -1;
  int rows = 0;
  bool ok = true;
  // the row's key range for the top-k kernel's value bins: lane-local maxima
  // of the keys and of their complements, reduced over the warp and added to
  // the row's global maxima when the warp moves to another row
  uint32_t key_max = 0u, key_not = 0u;
  auto flush_keys = [&](int64_t row) {
    const uint32_t m = __reduce_max_sync(0xffffffffu, key_max), mn = __reduce_max_sync(0xffffffffu, key_not);
    if (lane == 0 && m != 0u) {
      atomicMax(p.row_keys + 2 * row, m);
      atomicMax(p.row_keys + 2 * row + 1, mn);
    }
    key_max = 0u;
    key_not = 0u;
  };
  for (TileWalk tw(p, c.t_begin); tw.t < c.t_end && ok; tw.next(p)) {
    const int64_t b = tw.b, k = tw.k;
    const int sl = tw.sl;
    if (int64_t(k) * kTileRows >= sl) {
      tw.skip_row(p);
      continue;
    }
    if (b != prev_b) {
      // this row's head weights into the group's shared memory (double-buffered by row)
      named_barrier_sync(1 + g, kEpiThreads);   // the previous row's weights are no longer read
      if (gr < kHeads) {
        float* w = reinterpret_cast<float*>(
            __cvta_shared_to_generic(c.sbase + kOffW + (2 * g + (rows & 1)) * kHeads * 4));
        w[gr] = __ldg(p.weights + b * kHeads + gr);
      }
      named_barrier_sync(1 + g, kEpiThreads);
      flush_keys(prev_b);
      ++rows;
      prev_b = b;
    }
    const int s = int(n % kStages), db = int(n & 1);
    if (db != g) {
      ++n;
      continue;
    }
    // the stage cannot be refilled before this group arrives on its empty
    // barrier, so its full phase is unambiguous here
    bool got = mbar_wait(bar(c, B_FULL + s), uint32_t(n / kStages) & 1u, c.abort, c.timeout_ns);
    got = got && mbar_wait(bar(c, B_D_FULL + db), uint32_t(n >> 1) & 1u, c.abort, c.timeout_ns);
    if (!(ok = got)) break;
    tc_fence_after();
    const float scale =
        *reinterpret_cast<const float*>(__cvta_shared_to_generic(c.sbase + kOffScale + s * kScaleBytes + 4u * r));
    const float* w = reinterpret_cast<const float*>(
        __cvta_shared_to_generic(c.sbase + kOffW + (2 * g + ((rows - 1) & 1)) * kHeads * 4));
    // relu(dot * scale) = scale * relu(dot) for scale >= 0 and
    // scale * min(dot, 0) otherwise, so the scale leaves the head sum
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const bool pos_scale = scale >= 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float d[16];
      tmem_ld16(c.tmem + t_lane + 64u * db + 16u * q, d);
      tmem_wait_ld();
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const float v = pos_scale ? fmaxf(d[h], 0.f) : fminf(d[h], 0.f);
        acc[h & 3] = fmaf(v, w[16 * q + h], acc[h & 3]);
      }
    }
    tc_fence_before();
    mbar_arrive(bar(c, B_D_EMPTY + db));
    mbar_arrive(bar(c, B_EMPTY + s));
    const int64_t pos = int64_t(k) * kTileRows + r;
    if (pos < sl) {
      const float fin = scale * ((acc[0] + acc[1]) + (acc[2] + acc[3]));
      p.scores[b * (p.max_pages * kPageRows) + pos] = fin;
      const uint32_t key = ordered_key(fin);
      key_max = max(key_max, key);
      key_not = max(key_not, ~key);
    }
    ++n;
  }
  flush_keys(prev_b);
}

__global__ void __launch_bounds__(kThreads, 2)
    indexer_score_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_s,
                         const __grid_constant__ CUtensorMap tm_q, const ScoreParams p, const uint64_t timeout_ns) {
  // the top-k kernel may be scheduled while this grid runs; it waits for this
  // grid's completion (griddepcontrol.wait) before it reads anything
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Ctx c;
  c.sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  c.abort = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc + 4);
  c.timeout_ns = timeout_ns;
  c.drain_ns = drain_limit_ns(timeout_ns);
  int64_t* range_s = reinterpret_cast<int64_t*>(smem + kOffMisc + 16);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_k)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_q)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_s)) : "memory");
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(c, B_FULL + s), 1);
      mbar_init(bar(c, B_EMPTY + s), 1 + kEpiThreads);   // MMA done + scales read
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(bar(c, B_Q_FULL + k), 1);
      mbar_init(bar(c, B_Q_EMPTY + k), 2);   // both MMA warps
      mbar_init(bar(c, B_D_FULL + k), 1);
      mbar_init(bar(c, B_D_EMPTY + k), kEpiThreads);
    }
    mbar_init(bar(c, B_DONE), 1);
    mbar_init(bar(c, B_DONE + 1), 1);
    *c.abort = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  // launched with programmatic stream serialization: the setup above overlaps
  // the previous kernel on the stream; its outputs are read only after this
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // this CTA's tiles, from the plan left by the previous call's top-k grid
  // (complete once the wait returns) or the equal split of the active tiles
  uint32_t t_start = 0u, planned = 0u;
  if (warp == 0) {
    int64_t tb, te;
    cta_range(p, reinterpret_cast<int32_t*>(smem + kOffStage), tb, te, planned);
    if (threadIdx.x == 0) {
      range_s[0] = tb;
      range_s[1] = te;
      t_start = uint32_t(globaltimer_ns());
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  c.tmem = *tmem_slot;
  c.t_begin = range_s[0];
  c.t_end = range_s[1];
  int64_t active = 0;
  if (warp == 0) {
    active = load_warp(c, p, &tm_k, &tm_s, &tm_q,
                       p.split_active ? reinterpret_cast<const int32_t*>(smem + kOffStage) : nullptr);
  } else if (warp <= 2) {
    if ((threadIdx.x & 31) == 0) mma_warp(c, p, warp - 1);
    __syncwarp();
  } else {
    epilogue_warps(c, p);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (*c.abort) report_error(p.err_word, DSA_DEVICE_ERR_TIMEOUT);
    if (p.plan != nullptr)
      p.plan->log[blockIdx.x] =
          make_uint4(uint32_t(c.t_end - c.t_begin) | planned, t_start, uint32_t(globaltimer_ns()), uint32_t(active));
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(c.tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- top-k
constexpr int kTopkThreads = 1024;

// Exclusive prefix sum over the block's 1024 threads; returns the total in *total.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t s = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_sums[lane] = s;   // inclusive over warps
  }
  __syncthreads();
  const uint32_t before = (warp ? warp_sums[warp - 1] : 0u) + x - v;
  *total = warp_sums[31];
  __syncthreads();
  return before;
}

struct TopkParams {
  const float* scores;
  uint32_t* row_keys;    // [B][2], written by the score kernel (see ScoreParams)
  const int32_t* seq_lens;
  const int32_t* block_table;
  int32_t* out;          // [B, 2048]
  int64_t max_pages;
  int64_t num_pages;
  int64_t batch;         // rows; the CTAs past them (if plan) update the plan
  PlanState* plan;       // null: no plan update
  int plan_grid;         // the score launch's grid
};

// The plan update (see PlanState), by one CTA of kTopkThreads threads after
// the score grid is complete; thread g speaks for score CTA g.  `scratch` is
// 1 KB of shared memory.  Rates are active tiles per ns over each CTA's own
// run, clamped to [1/2, 2] x their mean; a CTA with no usable entry gets the
// mean rate and no start offset.  The ideal shares end all CTAs at one time T:
//   ideal_g = rate_g * (T - offset_g),  sum_g ideal_g = active tiles.
// The fractions come from an exclusive scan of integer weights, so they are
// monotone from 0 to kPlanOne.  Not inlined: it keeps the top-k kernels'
// register allocation to their own code; plain-value arguments keep it off the stack.
__device__ __noinline__ void update_plan(PlanState* ps, const int32_t* seq_lens, int64_t max_pages, int64_t B,
                                         int G, uint32_t* warp_sums, uint8_t* scratch) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* fred = reinterpret_cast<float*>(scratch);                 // [32][2]
  uint32_t* ured = reinterpret_cast<uint32_t*>(scratch + 256);     // [32][4]
  const int64_t cap = max_pages * kPageRows;
  // this call's active tiles, which the log must add up to
  uint32_t active = 0u;
  for (int64_t r0 = 0; r0 < B; r0 += kTopkThreads) {
    const int64_t r = r0 + tid;
    uint32_t act = 0u;
    if (r < B) {
      const int sl = seq_lens[r];
      const int64_t len = sl <= 0 ? 0 : (sl > cap ? cap : int64_t(sl));
      act = uint32_t((len + kTileRows - 1) / kTileRows);
    }
    uint32_t chunk = 0u;
    block_exclusive_scan(act, warp_sums, &chunk);
    active += chunk;
  }
  const bool mine = tid < G;
  const uint4 e = mine ? __ldcg(ps->log + tid) : make_uint4(0u, 0u, 0u, 0u);
  const uint32_t s_ref = __ldcg(&ps->log[0].y);
  const uint32_t dur = e.z - e.y;
  const int32_t off = int32_t(e.y - s_ref);
  const bool valid = mine && e.w > 0u && dur > 0u && dur < (1u << 30);
  const float rate = valid ? float(e.w) / float(dur) : 0.f;
  // pass 1: active total, valid count, earliest start, plan-used flag, rate sum
  {
    const uint32_t n = __reduce_add_sync(0xffffffffu, e.w);
    const uint32_t cnt = __reduce_add_sync(0xffffffffu, valid ? 1u : 0u);
    // offsets as order-preserving unsigned keys (int32 + 2^31)
    const uint32_t omin = __reduce_min_sync(0xffffffffu, valid ? uint32_t(off) ^ 0x80000000u : 0xffffffffu);
    const uint32_t used = __reduce_or_sync(0xffffffffu, e.x & kPlanUsed);
    float r = rate;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (lane == 0) {
      ured[4 * warp] = n;
      ured[4 * warp + 1] = cnt;
      ured[4 * warp + 2] = omin;
      ured[4 * warp + 3] = used;
      fred[2 * warp] = r;
    }
  }
  __syncthreads();
  uint32_t logged = 0u, cnt = 0u, omin = 0xffffffffu, used = 0u;
  float rsum = 0.f;
  for (int w = 0; w < kTopkThreads / 32; ++w) {
    logged += ured[4 * w];
    cnt += ured[4 * w + 1];
    omin = min(omin, ured[4 * w + 2]);
    used |= ured[4 * w + 3];
    rsum += fred[2 * w];
  }
  __syncthreads();
  if (logged != active || cnt == 0u) {   // an incomplete log (an aborted CTA) or nothing scored
    if (tid == 0) ps->magic = 0u;
    return;
  }
  const float mean = rsum / float(cnt);
  const float rc = mine ? (valid ? fminf(fmaxf(rate, 0.5f * mean), 2.f * mean) : mean) : 0.f;
  const float ofs = valid ? float(int32_t((uint32_t(off) ^ 0x80000000u) - omin)) : 0.f;
  // pass 2: sum of rates, sum of rate x offset
  {
    float a = rc, b = rc * ofs;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (lane == 0) {
      fred[2 * warp] = a;
      fred[2 * warp + 1] = b;
    }
  }
  __syncthreads();
  float ra = 0.f, rb = 0.f;
  for (int w = 0; w < kTopkThreads / 32; ++w) {
    ra += fred[2 * w];
    rb += fred[2 * w + 1];
  }
  const float t_end = (float(active) + rb) / ra;
  const float ideal = mine ? fmaxf(0.f, rc * (t_end - ofs)) : 0.f;
  const float share = used ? 0.5f * float(e.w) + 0.5f * ideal : ideal;
  const uint32_t wgt = mine ? uint32_t(share * (16777216.f / float(active)) + 0.5f) : 0u;
  uint32_t total = 0u;
  const uint32_t before = block_exclusive_scan(wgt, warp_sums, &total);
  if (total == 0u) {
    if (tid == 0) ps->magic = 0u;
    return;
  }
  if (mine) ps->frac[tid] = uint32_t((uint64_t(before) << 31) / total);
  if (tid == 0) {
    ps->frac[G] = kPlanOne;
    ps->grid = uint32_t(G);
    ps->magic = kPlanMagic;
  }
}

// Rows of up to kSmemKeys positions keep their keys in shared memory for all
// passes; longer rows read them from the scores in global memory (L2).
constexpr int kSmemKeys = 32768;
constexpr int kBins = 2048;
constexpr int kHistCopies = 8;   // privatised first-pass histograms, 4 warps each
constexpr int kRankCap = 1024;   // threshold-bin candidates ranked by direct comparison
constexpr int kBucketCap = 64;   // largest bucket ordered by direct comparison
constexpr uint32_t kKeyNegInf = 0x007fffffu;   // ordered_key(-inf)
constexpr uint32_t kTopkSmemBytes = 212992;

// Dynamic shared memory of the top-k kernel.  With the keys in shared memory:
// keys [32768] | sel [2048] u64 | candidates [8192] | 8 histograms of 2048
// 16-bit counts (two per word; a copy counts at most 4 warps x 32 keys a bin).
// Without: 8 histograms of 2048 32-bit counts | candidates [16384] | sel.
// Once merged, the histogram area holds the per-bin output offsets.
template <bool kKeysInSmem>
struct TopkLayout {
  static constexpr uint32_t kSel = 131072;
  static constexpr uint32_t kCand = kKeysInSmem ? 147456 : 65536;
  static constexpr int kCandCap = kKeysInSmem ? 8192 : 16384;
  static constexpr uint32_t kPriv = kKeysInSmem ? 180224 : 0;
  static constexpr int kPrivWords = kKeysInSmem ? kHistCopies * 1024 : kHistCopies * 2048;
  static_assert(kPriv + kPrivWords * 4 <= kTopkSmemBytes && kCand + kCandCap * 4 <= (kKeysInSmem ? kPriv : kSel),
                "top-k shared memory layout");
};

__device__ __forceinline__ float key_value(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

// Linear value bins between the row's smallest finite score lo and its
// largest: a monotone (non-decreasing) map of the ordered key, so a bin holds
// a contiguous key range and bins order like keys; -inf goes to bin 0.
struct LinearBins {
  float lo, scale;
  __device__ __forceinline__ uint32_t operator()(uint32_t key) const {
    // clamp to [0, 2047] (NaN from inf * 0 -> 0), round to an integer by
    // adding 2^23 and reading the low mantissa bits (monotone, like the value)
    float v = fminf(fmaxf(0.f, __fmul_rn(__fsub_rn(key_value(key), lo), scale)), float(kBins - 1));
    v = key <= kKeyNegInf ? 0.f : v;
    return __float_as_uint(__fadd_rn(v, 8388608.f)) & uint32_t(kBins - 1);
  }
};

__device__ __forceinline__ unsigned long long sel_entry(uint32_t key, uint32_t pos) {
  return (static_cast<unsigned long long>(~key) << 32) | pos;   // ascending = score descending, position ascending
}

// One CTA per batch row; k = min(2048, seq_len) positions are returned.
//  1. one pass over the row: every position's ordered key (kept in shared
//     memory when the row fits) counted into 2048 linear value bins between
//     the row's smallest and largest score (reduced by the score kernel);
//  2. from the histogram: the bin b1 holding the k-th largest key, the keys
//     in bins above it (all selected) and the per-bin output offsets;
//  3. keys above b1 are written to their bin's bucket of `sel`; the keys in
//     b1 become a candidate list in position order;
//  4. the candidates are ranked by (key, position) directly when there are at
//     most kRankCap of them, else narrowed by radix passes (11 bits at a time
//     below their common prefix) to the k-th key T, taking the keys equal to T
//     by lowest position;
//  5. output: each bucket is ordered by direct comparison and the slot ids are
//     written to their final places; rows with a bucket over kBucketCap take
//     a bitonic sort instead.
// Rows whose threshold bin overflows the candidate list run radix passes over
// the whole row (step 4 on every key) and the bitonic sort.
// The whole selection for batch row b by one CTA.  The row's key range comes
// from the score kernel's reduction (read and cleared here) or, when
// `given_range`, from the caller.
template <bool kKeysInSmem>
__device__ void topk_row(const TopkParams& p, const int64_t b, const uint32_t given_kmin, const uint32_t given_kmax,
                         const bool given_range) {
  using L = TopkLayout<kKeysInSmem>;
  extern __shared__ __align__(16) uint8_t topk_smem[];
  uint32_t* keys_s = reinterpret_cast<uint32_t*>(topk_smem);
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(topk_smem + L::kSel);
  uint32_t* cand = reinterpret_cast<uint32_t*>(topk_smem + L::kCand);
  uint32_t* priv = reinterpret_cast<uint32_t*>(topk_smem + L::kPriv);
  uint32_t* start = priv;   // after the merge: keys in bins above each bin
  __shared__ uint32_t hist[kBins];   // radix histograms; bucket fill counts
  __shared__ uint32_t warp_sums[32], warp_cnt[32];
  __shared__ uint32_t sh_bin, sh_need, sh_count, sh_kmin, sh_kmax, sh_maxb, sh_fill;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t cap = p.max_pages * kPageRows;
  int sl = p.seq_lens[b];
  sl = sl <= 0 ? 0 : int(sl > cap ? cap : sl);
  const float* sc = p.scores + b * cap;
  const float4* sc4 = reinterpret_cast<const float4*>(sc);   // scores rows are 16-byte aligned
  const int32_t* bt = p.block_table + b * p.max_pages;
  int32_t* out = p.out + b * kTopk;
  const int k = sl < kTopk ? sl : kTopk;
  if (k == 0) {
    for (int i = tid; i < kTopk; i += kTopkThreads) out[i] = -1;
    return;
  }
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int ng = (sl + 3) >> 2;   // groups of 4 positions

  // key of position i: a position on a page outside the pool scores -inf
  auto key_global = [&](int i) -> uint32_t {
    const int32_t page = __ldg(bt + (i >> 6));
    const bool ok = page >= 0 && int64_t(page) < p.num_pages;
    return ordered_key(ok ? sc[i] : -INFINITY);
  };
  auto key_of = [&](int i) -> uint32_t {
    if constexpr (kKeysInSmem) return keys_s[i];
    else return key_global(i);
  };
  auto keys4_from = [&](float4 v, int32_t page, uint32_t* kk) {
    const bool ok = page >= 0 && int64_t(page) < p.num_pages;
    kk[0] = ordered_key(ok ? v.x : -INFINITY);
    kk[1] = ordered_key(ok ? v.y : -INFINITY);
    kk[2] = ordered_key(ok ? v.z : -INFINITY);
    kk[3] = ordered_key(ok ? v.w : -INFINITY);
  };
  // keys of positions 4g .. 4g+3 (g < ng) after the load pass
  auto keys4 = [&](int g, uint32_t* kk) {
    if constexpr (kKeysInSmem) {
      const uint4 q = reinterpret_cast<const uint4*>(keys_s)[g];
      kk[0] = q.x;
      kk[1] = q.y;
      kk[2] = q.z;
      kk[3] = q.w;
    } else {
      keys4_from(__ldg(sc4 + g), __ldg(bt + (g >> 4)), kk);
    }
  };
  // The bin of the nb-bin histogram `count` (highest bin first) where the
  // running count reaches need_in: sh_bin, how many of it to take (sh_need)
  // and its count (sh_count).  Each thread owns two adjacent bins.
  auto select_bin = [&](int nb, uint32_t need_in, auto count) {
    const int j0 = 2 * tid, j1 = 2 * tid + 1;
    const uint32_t c0 = j0 < nb ? count(uint32_t(nb - 1 - j0)) : 0u;
    const uint32_t c1 = j1 < nb ? count(uint32_t(nb - 1 - j1)) : 0u;
    uint32_t total;
    const uint32_t before = block_exclusive_scan(c0 + c1, warp_sums, &total);
    if (j0 < nb && before < need_in && before + c0 >= need_in) {
      sh_bin = uint32_t(nb - 1 - j0);
      sh_need = need_in - before;
      sh_count = c0;
    }
    if (j1 < nb && before + c0 < need_in && before + c0 + c1 >= need_in) {
      sh_bin = uint32_t(nb - 1 - j1);
      sh_need = need_in - (before + c0);
      sh_count = c1;
    }
    __syncthreads();
  };

  uint32_t prefix = 0, prefix_mask = 0;
  uint32_t need = uint32_t(k);
  // radix pass over n positions (pos_at(i)) on bits [sh, sh + log2 nb):
  // narrows prefix/need to the bin holding the k-th key, returns its count
  auto refine = [&](int n, auto pos_at, int sh, int nb) -> uint32_t {
    for (int i = tid; i < nb; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kTopkThreads) {
      const uint32_t key = key_of(pos_at(i));
      if ((key & prefix_mask) == prefix) atomicAdd(&hist[(key >> sh) & uint32_t(nb - 1)], 1u);
    }
    __syncthreads();
    select_bin(nb, need, [&](uint32_t j) { return hist[j]; });
    prefix |= sh_bin << sh;
    prefix_mask |= uint32_t(nb - 1) << sh;
    need = sh_need;
    const uint32_t cnt = sh_count;
    __syncthreads();
    return cnt;
  };
  // radix passes below the bits that every key in scope shares
  auto refine_all = [&](int n, auto pos_at, uint32_t kmin, uint32_t kmax) -> uint32_t {
    const int lz = min(31, __clz(kmin ^ kmax));
    prefix_mask = lz == 0 ? 0u : ~0u << (32 - lz);
    prefix = kmax & prefix_mask;
    uint32_t m = uint32_t(n);
    for (int rem = 32 - lz; rem > 0;) {
      const int w = min(11, rem);
      rem -= w;
      m = refine(n, pos_at, rem, 1 << w);
    }
    return m;
  };

  // ---- 1. the row's key range (reduced by the score kernel; cleared here
  // for the next call), and one pass over the row: every position's ordered
  // key (kept in shared memory when the row fits) counted into a histogram of
  // 2048 linear value bins; each group of 4 warps counts into its own copy
  for (int i = tid; i < L::kPrivWords; i += kTopkThreads) priv[i] = 0;
  if (tid == 0) {
    if (given_range) {
      sh_kmax = given_kmax;
      sh_kmin = given_kmin;
    } else {
      sh_kmax = p.row_keys[2 * b];
      sh_kmin = ~p.row_keys[2 * b + 1];
      p.row_keys[2 * b] = 0u;
      p.row_keys[2 * b + 1] = 0u;
    }
    sh_maxb = 0u;
  }
  __syncthreads();
  LinearBins bins;
  {
    const uint32_t kmin = sh_kmin, kmax = sh_kmax;
    bins.lo = kmin <= kmax ? key_value(kmin) : 0.f;
    const float range = kmin <= kmax ? __fsub_rn(key_value(kmax), bins.lo) : 0.f;
    bins.scale = range > 0.f ? __fdiv_rn(float(kBins), range) : 0.f;
  }
  {
    const uint32_t copy = uint32_t(warp) >> 2;
    for (int g0 = 0; g0 < ng; g0 += 4 * kTopkThreads) {
      float4 v[4];
      int32_t pg[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int g = g0 + u * kTopkThreads + tid;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        pg[u] = -1;
        if (g < ng) {
          v[u] = __ldg(sc4 + g);
          pg[u] = __ldg(bt + (g >> 4));
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int g = g0 + u * kTopkThreads + tid;
        uint32_t kk[4];
        keys4_from(v[u], pg[u], kk);
        if constexpr (kKeysInSmem) {
          if (g < ng) reinterpret_cast<uint4*>(keys_s)[g] = make_uint4(kk[0], kk[1], kk[2], kk[3]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (4 * g + e < sl) {
            const uint32_t bin = bins(kk[e]);
            if constexpr (kKeysInSmem) atomicAdd(priv + (copy << 10) + (bin >> 1), 1u << ((bin & 1) << 4));
            else atomicAdd(priv + (copy << 11) + bin, 1u);
          }
        }
      }
    }
  }
  __syncthreads();
  uint32_t b1, c1, gt1;
  {
    auto merged = [&](uint32_t j) {
      uint32_t s = 0;
#pragma unroll
      for (int c = 0; c < kHistCopies; ++c) {
        if constexpr (kKeysInSmem) s += (priv[(c << 10) + (j >> 1)] >> ((j & 1) << 4)) & 0xffffu;
        else s += priv[(c << 11) + j];
      }
      return s;
    };
    const uint32_t j0 = uint32_t(kBins - 1 - 2 * tid), j1 = j0 - 1;   // this thread's bins, highest first
    const uint32_t n0 = merged(j0), n1 = merged(j1);
    uint32_t total;
    const uint32_t before = block_exclusive_scan(n0 + n1, warp_sums, &total);   // all merges are read
    start[j0] = before;
    start[j1] = before + n0;
    if (before < need && before + n0 >= need) {
      sh_bin = j0;
      sh_need = need - before;
      sh_count = n0;
    }
    if (before + n0 < need && before + n0 + n1 >= need) {
      sh_bin = j1;
      sh_need = need - (before + n0);
      sh_count = n1;
    }
    for (int i = tid; i < kBins; i += kTopkThreads) hist[i] = 0;
    __syncthreads();
    b1 = sh_bin;
    c1 = sh_count;
    need = sh_need;
    gt1 = uint32_t(k) - need;
    // largest bucket above b1
    uint32_t mb = (j0 > b1 ? n0 : 0u);
    mb = max(mb, j1 > b1 ? n1 : 0u);
    mb = __reduce_max_sync(0xffffffffu, mb);
    if (lane == 0 && mb) atomicMax(&sh_maxb, mb);
  }
  bool bucketed = false;   // sel holds the buckets above b1, then the best of b1 in order
  if (c1 <= uint32_t(L::kCandCap)) {
    // ---- 3. keys above b1 into their buckets, keys in b1 to the candidate
    // list (one atomic per warp and 128 positions that hold candidates)
    if (tid == 0) sh_fill = 0;
    __syncthreads();
    for (int g0 = 0; g0 < ng; g0 += kTopkThreads) {
      const int g = g0 + tid;
      uint32_t kk[4] = {0u, 0u, 0u, 0u};
      if (g < ng) keys4(g, kk);
      uint32_t mine = 0;
      bool is_c[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool valid = g < ng && 4 * g + e < sl;
        const uint32_t bn = bins(kk[e]);
        if (valid && bn > b1) sel[start[bn] + atomicAdd(&hist[bn], 1u)] = sel_entry(kk[e], uint32_t(4 * g + e));
        is_c[e] = valid && bn == b1;
        mine += is_c[e];
      }
      if (__any_sync(0xffffffffu, mine != 0)) {
        uint32_t incl = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        uint32_t base = 0;
        if (lane == 31) base = atomicAdd(&sh_fill, incl);
        uint32_t at = __shfl_sync(0xffffffffu, base, 31) + incl - mine;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (is_c[e]) cand[at++] = uint32_t(4 * g + e);
      }
    }
    __syncthreads();
    const int nc_total = int(c1);
    if (nc_total <= kRankCap) {
      // ---- 4a. the best `need` candidates by (key, position), in order
      for (int i = tid; i < nc_total; i += kTopkThreads) {
        const uint32_t pos = cand[i], key = key_of(int(pos));
        uint32_t r = 0;
        for (int j = 0; j < nc_total; ++j) {
          const uint32_t pj = cand[j], kj = key_of(int(pj));
          r += kj > key || (kj == key && pj < pos);
        }
        if (r < need) sel[gt1 + r] = sel_entry(key, pos);
      }
      bucketed = true;
    } else {
      // ---- 4b. radix passes over the candidates narrow the k-th key T;
      // the ordered gather over the whole row takes the ties by position
      auto cand_at = [&](int i) { return int(cand[i]); };
      if (tid == 0) {
        sh_kmin = 0xffffffffu;
        sh_kmax = 0u;
      }
      __syncthreads();
      uint32_t cmin = 0xffffffffu, cmax = 0u;
      for (int i = tid; i < nc_total; i += kTopkThreads) {
        const uint32_t key = key_of(cand_at(i));
        cmin = min(cmin, key);
        cmax = max(cmax, key);
      }
      cmin = __reduce_min_sync(0xffffffffu, cmin);
      cmax = __reduce_max_sync(0xffffffffu, cmax);
      if (lane == 0) {
        atomicMin(&sh_kmin, cmin);
        atomicMax(&sh_kmax, cmax);
      }
      __syncthreads();
      refine_all(nc_total, cand_at, sh_kmin, sh_kmax);
    }
  } else {
    // ---- the threshold bin overflows the candidate list: radix passes
    // over the whole row
    auto all_at = [](int i) { return i; };
    need = uint32_t(k);
    refine_all(sl, all_at, 0u, 0xffffffffu);
  }
  if (!bucketed) {
    // ordered gather: warp w owns a contiguous chunk; keys above T all go,
    // keys equal to T while fewer than `need` were taken before them
    const uint32_t T = prefix;
    const int chunk = ((sl + 31) / 32 + 31) & ~31;
    const int lo = min(sl, warp * chunk), hi = min(sl, lo + chunk);
    uint32_t gt = 0, eq = 0;
    for (int i = lo + lane; i < hi; i += 32) {
      const uint32_t key = key_of(i);
      gt += key > T;
      eq += key == T;
    }
    gt = __reduce_add_sync(0xffffffffu, gt);
    eq = __reduce_add_sync(0xffffffffu, eq);
    if (lane == 0) {
      warp_sums[warp] = gt;
      warp_cnt[warp] = eq;
    }
    __syncthreads();
    uint32_t g_off = 0, e_off = 0, gt_total = 0;
    for (int w = 0; w < 32; ++w) {
      if (w < warp) {
        g_off += warp_sums[w];
        e_off += warp_cnt[w];
      }
      gt_total += warp_sums[w];
    }
    for (int base = lo; base < hi; base += 32) {
      const int i = base + lane;
      const uint32_t key = i < hi ? key_of(i) : 0u;
      const bool g = i < hi && key > T, e = i < hi && key == T;
      const uint32_t gm = __ballot_sync(0xffffffffu, g), em = __ballot_sync(0xffffffffu, e);
      if (g) sel[g_off + __popc(gm & lt_mask)] = sel_entry(key, uint32_t(i));
      if (e) {
        const uint32_t r = e_off + __popc(em & lt_mask);
        if (r < need) sel[gt_total + r] = sel_entry(key, uint32_t(i));
      }
      g_off += __popc(gm);
      e_off += __popc(em);
    }
  }
  __syncthreads();

  // slot id of a selected entry; a position on a bad page (scored -inf) is none
  auto slot_of = [&](unsigned long long v) -> int32_t {
    const uint32_t pos = uint32_t(v & 0xffffffffu), key = ~uint32_t(v >> 32);
    const int32_t page = __ldg(bt + (pos >> 6));
    return key != kKeyNegInf && page >= 0 && int64_t(page) < p.num_pages ? page * kPageRows + int32_t(pos & 63)
                                                                          : -1;
  };
  for (int i = k + tid; i < kTopk; i += kTopkThreads) out[i] = -1;
  if (bucketed && sh_maxb <= uint32_t(kBucketCap)) {
    // ---- 5. rank each entry within its bucket; write its slot id in place
    // (entries from gt1 on are already in order)
    for (int i = tid; i < k; i += kTopkThreads) {
      const unsigned long long v = sel[i];
      uint32_t dst = uint32_t(i);
      if (uint32_t(i) < gt1) {
        const uint32_t bn = bins(~uint32_t(v >> 32));
        const uint32_t s1 = start[bn - 1];   // bn > b1 >= 0: the bucket ends where the next lower bin's starts
        dst = start[bn];
        for (uint32_t j = dst; j < s1; ++j) dst += sel[j] < v;
      }
      out[dst] = slot_of(v);
    }
    return;
  }
  // bitonic sort of sel (padding sorts last), ascending entries; thread t
  // holds elements 2t and 2t+1 in registers: strides up to 32 are exchanged
  // by shuffles within the warp, larger ones through shared memory
  for (int i = k + tid; i < kTopk; i += kTopkThreads) sel[i] = ~0ull;
  __syncthreads();
  ulonglong2 pair = reinterpret_cast<const ulonglong2*>(sel)[tid];
  unsigned long long a0 = pair.x, a1 = pair.y;
  for (int size = 2; size <= kTopk; size <<= 1) {
    int stride = size >> 1;
    if (stride >= 64) {
      reinterpret_cast<ulonglong2*>(sel)[tid] = make_ulonglong2(a0, a1);
      __syncthreads();
      for (; stride >= 64; stride >>= 1) {
        const int i = 2 * tid - (tid & (stride - 1));   // lower index of this thread's pair
        const int j = i + stride;
        const bool up = ((i & size) == 0);
        const unsigned long long x = sel[i], y = sel[j];
        if ((x > y) == up) {
          sel[i] = y;
          sel[j] = x;
        }
        __syncthreads();
      }
      pair = reinterpret_cast<const ulonglong2*>(sel)[tid];
      a0 = pair.x;
      a1 = pair.y;
    }
    const bool up = ((2 * tid) & size) == 0;
    for (; stride >= 2; stride >>= 1) {
      // element 2t+r pairs with element (2t+r)^stride, held by thread t^(stride/2)
      const bool keep_min = (((2 * tid) & stride) == 0) == up;
      const unsigned long long y0 = __shfl_xor_sync(0xffffffffu, a0, stride >> 1);
      const unsigned long long y1 = __shfl_xor_sync(0xffffffffu, a1, stride >> 1);
      a0 = keep_min ? (a0 < y0 ? a0 : y0) : (a0 < y0 ? y0 : a0);
      a1 = keep_min ? (a1 < y1 ? a1 : y1) : (a1 < y1 ? y1 : a1);
    }
    if ((a0 > a1) == up) {
      const unsigned long long x = a0;
      a0 = a1;
      a1 = x;
    }
  }
  if (2 * tid < k) out[2 * tid] = slot_of(a0);
  if (2 * tid + 1 < k) out[2 * tid + 1] = slot_of(a1);
}

template <bool kKeysInSmem>
__global__ void __launch_bounds__(kTopkThreads, 1) indexer_topk_kernel(const TopkParams p) {
  // launched as a programmatic dependent of the score kernel: its scores and
  // key ranges are complete and visible once this wait returns.  The next
  // kernel on the stream (the attention) may be scheduled from now on.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  if (blockIdx.x >= p.batch) {   // the CTA past the rows updates the score plan
    extern __shared__ __align__(16) uint8_t topk_smem[];
    __shared__ uint32_t plan_sums[32];
    update_plan(p.plan, p.seq_lens, p.max_pages, p.batch, p.plan_grid, plan_sums, topk_smem);
    return;
  }
  topk_row<kKeysInSmem>(p, blockIdx.x, 0u, 0u, false);
}

// Two CTAs (a cluster) per batch row, for rows that fit in shared memory.
// CTA r of the pair loads and histograms half the row (positions [0, h) and
// [h, sl), h a multiple of 4); the halves' per-bin counts are combined
// through distributed shared memory, so both CTAs find the same threshold bin
// and bucket offsets; both write their bucket entries and their threshold-bin
// candidates (key and position) straight into CTA 0's arrays, and CTA 0 ranks
// the candidates and the buckets and writes the row's slot ids.  A row whose
// threshold bin or largest bucket is over the direct-ranking limits is handed
// whole to CTA 0's single-CTA routine (topk_row), which re-reads its scores.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTopkThreads, 1)
    indexer_topk_pair_kernel(const TopkParams p) {
  using L = TopkLayout<true>;
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  extern __shared__ __align__(16) uint8_t topk_smem[];
  uint32_t* keys_s = reinterpret_cast<uint32_t*>(topk_smem);   // this CTA's half
  // each key's bin (16 bits), in the half of the key area this kernel leaves free
  uint16_t* bins_s = reinterpret_cast<uint16_t*>(topk_smem + kSmemKeys * 2);
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(topk_smem + L::kSel);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(topk_smem + L::kCand);   // key << 32 | pos
  uint32_t* priv = reinterpret_cast<uint32_t*>(topk_smem + L::kPriv);
  uint32_t* start = priv;   // after the merge: this half's output offset of each bin
  __shared__ uint32_t cnt[kBins];   // this half's per-bin counts, then its bucket cursors
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t sh_bin, sh_need, sh_count, sh_maxb, sh_fill;
  __shared__ int32_t bt_s[kSmemKeys / kPageRows];   // the row's block table
  static_assert(kRankCap * 8 <= L::kCandCap * 4, "candidate entries fit the candidate area");
  const int64_t b = blockIdx.x >> 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (b >= p.batch) {   // the cluster past the rows: its first CTA updates the score plan
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    if (rank == 0)
      update_plan(p.plan, p.seq_lens, p.max_pages, p.batch, p.plan_grid, warp_sums, topk_smem);
    return;
  }
  // shared-memory setup first: it overlaps the score grid's tail
  for (int i = tid; i < L::kPrivWords; i += kTopkThreads) priv[i] = 0;
  if (tid == 0) {
    sh_maxb = 0u;
    sh_fill = 0u;
  }
  // launched as a programmatic dependent of the score kernel: its scores and
  // key ranges are complete and visible once this wait returns
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");   // the next kernel may be scheduled
  const int64_t cap = p.max_pages * kPageRows;   // <= kSmemKeys on this path
  // the row's length, key range and block table, loaded together
  const uint32_t kmax = p.row_keys[2 * b], kmin = ~p.row_keys[2 * b + 1];
  int sl = p.seq_lens[b];
  const int32_t* bt = p.block_table + b * p.max_pages;
  if (tid < p.max_pages) bt_s[tid] = __ldg(bt + tid);
  sl = sl <= 0 ? 0 : int(sl > cap ? cap : sl);
  const int k = sl < kTopk ? sl : kTopk;
  int32_t* out = p.out + b * kTopk;
  if (k == 0) {   // both CTAs of the pair return here
    if (rank == 0)
      for (int i = tid; i < kTopk; i += kTopkThreads) out[i] = -1;
    return;
  }
  LinearBins bins;
  bins.lo = kmin <= kmax ? key_value(kmin) : 0.f;
  {
    const float range = kmin <= kmax ? __fsub_rn(key_value(kmax), bins.lo) : 0.f;
    bins.scale = range > 0.f ? __fdiv_rn(float(kBins), range) : 0.f;
  }
  const int h = min(sl, ((sl + 1) / 2 + 3) & ~3);
  const int lo = rank ? h : 0, n = rank ? sl - h : h;   // this CTA's positions [lo, lo + n)
  const int ng = (n + 3) >> 2;
  const float4* sc4 = reinterpret_cast<const float4*>(p.scores + b * cap + lo);   // lo % 4 == 0
  __syncthreads();   // histogram copies zeroed, block table in shared memory
  // ---- this half's keys and histogram (8 privatised 16-bit copies)
  {
    const uint32_t copy = uint32_t(warp) >> 2;
    for (int g0 = 0; g0 < ng; g0 += 4 * kTopkThreads) {
      float4 v[4];
      int32_t pg[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int g = g0 + u * kTopkThreads + tid;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        pg[u] = -1;
        if (g < ng) {
          v[u] = __ldg(sc4 + g);
          pg[u] = bt_s[(lo + 4 * g) >> 6];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int g = g0 + u * kTopkThreads + tid;
        const bool ok = pg[u] >= 0 && int64_t(pg[u]) < p.num_pages;
        const uint32_t kk[4] = {ordered_key(ok ? v[u].x : -INFINITY), ordered_key(ok ? v[u].y : -INFINITY),
                                ordered_key(ok ? v[u].z : -INFINITY), ordered_key(ok ? v[u].w : -INFINITY)};
        const uint32_t bn[4] = {bins(kk[0]), bins(kk[1]), bins(kk[2]), bins(kk[3])};
        if (g < ng) {
          reinterpret_cast<uint4*>(keys_s)[g] = make_uint4(kk[0], kk[1], kk[2], kk[3]);
          reinterpret_cast<uint2*>(bins_s)[g] = make_uint2(bn[0] | (bn[1] << 16), bn[2] | (bn[3] << 16));
        }
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (4 * g + e < n) atomicAdd(priv + (copy << 10) + (bn[e] >> 1), 1u << ((bn[e] & 1) << 4));
      }
    }
  }
  __syncthreads();
  const uint32_t j0 = uint32_t(kBins - 1 - 2 * tid), j1 = j0 - 1;   // this thread's bins, highest first
  {
    uint32_t m0 = 0, m1 = 0;
#pragma unroll
    for (int c = 0; c < kHistCopies; ++c) {
      m0 += (priv[(c << 10) + (j0 >> 1)] >> ((j0 & 1) << 4)) & 0xffffu;
      m1 += (priv[(c << 10) + (j1 >> 1)] >> ((j1 & 1) << 4)) & 0xffffu;
    }
    cnt[j0] = m0;
    cnt[j1] = m1;
  }
  cluster.sync();   // both halves' counts are complete
  if (rank == 0 && tid == 0) {   // both CTAs read the key range before the barrier above
    p.row_keys[2 * b] = 0u;      // cleared for the next call
    p.row_keys[2 * b + 1] = 0u;
  }
  const uint32_t* other = cluster.map_shared_rank(cnt, rank ^ 1u);
  const uint32_t mine0 = cnt[j0], mine1 = cnt[j1], oth0 = other[j0], oth1 = other[j1];
  const uint32_t n0 = mine0 + oth0, n1 = mine1 + oth1;
  uint32_t need = uint32_t(k);
  uint32_t total;
  const uint32_t before = block_exclusive_scan(n0 + n1, warp_sums, &total);   // all priv reads are done
  // this half's entries of a bin follow CTA 0's
  start[j0] = before + (rank ? oth0 : 0u);
  start[j1] = before + n0 + (rank ? oth1 : 0u);
  if (before < need && before + n0 >= need) {
    sh_bin = j0;
    sh_need = need - before;
    sh_count = n0;
  }
  if (before + n0 < need && before + n0 + n1 >= need) {
    sh_bin = j1;
    sh_need = need - (before + n0);
    sh_count = n1;
  }
  __syncthreads();
  const uint32_t b1 = sh_bin, c1 = sh_count;
  need = sh_need;
  const uint32_t gt1 = uint32_t(k) - need;
  {
    uint32_t mb = (j0 > b1 ? n0 : 0u);
    mb = max(mb, j1 > b1 ? n1 : 0u);
    mb = __reduce_max_sync(0xffffffffu, mb);
    if (lane == 0 && mb) atomicMax(&sh_maxb, mb);
  }
  // CTA 0's count of b1: where CTA 1's candidates start
  const uint32_t cbase = rank ? (b1 == j0 ? oth0 : 0u) + (b1 == j1 ? oth1 : 0u) : 0u;
  __shared__ uint32_t sh_cbase;
  if (rank == 1 && (b1 == j0 || b1 == j1)) sh_cbase = cbase;
  cluster.sync();   // the partner has read cnt[]; maxb and the candidate base are final
  const bool fast = c1 <= uint32_t(kRankCap) && sh_maxb <= uint32_t(kBucketCap);
  if (!fast) {
    if (rank == 0) topk_row<true>(p, b, kmin, kmax, true);
    return;
  }
  const uint32_t cand_base = rank ? sh_cbase : 0u;
  for (int i = tid; i < kBins; i += kTopkThreads) cnt[i] = 0;
  __syncthreads();
  // ---- this half's keys above b1 into their buckets and its b1 keys to the
  // candidates, both in CTA 0's shared memory
  // CTA 0 writes its own arrays directly, CTA 1 through distributed shared memory
  unsigned long long* sel0 = rank ? cluster.map_shared_rank(sel, 0u) : sel;
  unsigned long long* cand0 = rank ? cluster.map_shared_rank(cand, 0u) : cand;
  // the keys' stored bins are read first; a group of four whose bins are all
  // below b1 (most of them) needs neither its keys nor any work
  for (int g0 = 0; g0 < ng; g0 += kTopkThreads) {
    const int g = g0 + tid;
    uint32_t bins4[4] = {0u, 0u, 0u, 0u};
    bool any = false;
    if (g < ng) {
      const uint2 w2 = reinterpret_cast<const uint2*>(bins_s)[g];
      bins4[0] = w2.x & 0xffffu;
      bins4[1] = w2.x >> 16;
      bins4[2] = w2.y & 0xffffu;
      bins4[3] = w2.y >> 16;
      any = max(max(bins4[0], bins4[1]), max(bins4[2], bins4[3])) >= b1;
    }
    if (!__any_sync(0xffffffffu, any)) continue;
    uint32_t kk[4] = {0u, 0u, 0u, 0u};
    if (any) {
      const uint4 q = reinterpret_cast<const uint4*>(keys_s)[g];
      kk[0] = q.x;
      kk[1] = q.y;
      kk[2] = q.z;
      kk[3] = q.w;
    }
    uint32_t mine = 0;
    bool is_c[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool valid = any && 4 * g + e < n;
      const uint32_t bn = bins4[e];
      if (valid && bn > b1)
        sel0[start[bn] + atomicAdd(&cnt[bn], 1u)] = sel_entry(kk[e], uint32_t(lo + 4 * g + e));
      is_c[e] = valid && bn == b1;
      mine += is_c[e];
    }
    if (__any_sync(0xffffffffu, mine != 0)) {
      uint32_t incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      uint32_t base = 0;
      if (lane == 31) base = atomicAdd(&sh_fill, incl);
      uint32_t at = cand_base + __shfl_sync(0xffffffffu, base, 31) + incl - mine;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (is_c[e]) cand0[at++] = (static_cast<unsigned long long>(kk[e]) << 32) | uint32_t(lo + 4 * g + e);
    }
  }
  cluster.sync();   // every entry of both halves is in CTA 0's arrays
  if (rank != 0) return;
  // ---- CTA 0: the best `need` candidates by (key, position), in order
  for (int i = tid; i < int(c1); i += kTopkThreads) {
    const unsigned long long v = cand[i];
    const uint32_t key = uint32_t(v >> 32), pos = uint32_t(v);
    uint32_t r = 0;
    for (int j = 0; j < int(c1); ++j) {
      const unsigned long long w = cand[j];
      const uint32_t kj = uint32_t(w >> 32), pj = uint32_t(w);
      r += kj > key || (kj == key && pj < pos);
    }
    if (r < need) sel[gt1 + r] = sel_entry(key, pos);
  }
  __syncthreads();
  // ---- rank each bucket entry within its bucket; write slot ids in place
  for (int i = k + tid; i < kTopk; i += kTopkThreads) out[i] = -1;
  for (int i = tid; i < k; i += kTopkThreads) {
    const unsigned long long v = sel[i];
    uint32_t dst = uint32_t(i);
    if (uint32_t(i) < gt1) {
      const uint32_t bn = bins(~uint32_t(v >> 32));
      const uint32_t s1 = start[bn - 1];   // bn > b1 >= 0: the bucket ends where the next lower bin's starts
      dst = start[bn];
      for (uint32_t j = dst; j < s1; ++j) dst += sel[j] < v;
    }
    const uint32_t pos = uint32_t(v & 0xffffffffu), key = ~uint32_t(v >> 32);
    const int32_t page = bt_s[pos >> 6];
    out[dst] = key != kKeyNegInf && page >= 0 && int64_t(page) < p.num_pages ? page * kPageRows + int32_t(pos & 63)
                                                                             : -1;
  }
}

// ---------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
constexpr int kMaxDevices = 64;
std::once_flag g_attr_once[kMaxDevices];
cudaError_t g_attr_err[kMaxDevices];

bool encode_rows128(CUtensorMap* map, const void* base, uint64_t rows, uint32_t box_rows, bool swizzle) {
  const cuuint64_t dims[2] = {128, rows};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace indexer

// Launches the score and top-k kernels on `stream`; arguments were validated
// by the caller.  `scores` holds batch * max_pages * 64 floats.
cudaError_t launch_indexer(const uint8_t* q, const uint8_t* cache, const float* weights, const int32_t* seq_lens,
                           const int32_t* block_table, int64_t batch, int64_t max_pages, int64_t num_pages,
                           int32_t* out, float* scores, uint32_t* row_keys, uint32_t* err_word, void* plan_state,
                           int sms, cudaStream_t stream) {
  using namespace indexer;
  std::call_once(g_encode_once, []() {
    cudaDriverEntryPointQueryResult qr;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return cudaErrorNotSupported;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::call_once(g_attr_once[dev], [dev]() {
    g_attr_err[dev] = cudaFuncSetAttribute(indexer_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(kSmemBytes));
    if (g_attr_err[dev] == cudaSuccess)
      g_attr_err[dev] = cudaFuncSetAttribute(indexer_topk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(kTopkSmemBytes));
    if (g_attr_err[dev] == cudaSuccess)
      g_attr_err[dev] = cudaFuncSetAttribute(indexer_topk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(kTopkSmemBytes));
    if (g_attr_err[dev] == cudaSuccess)
      g_attr_err[dev] = cudaFuncSetAttribute(indexer_topk_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(kTopkSmemBytes));
  });
  if (g_attr_err[dev] != cudaSuccess) return g_attr_err[dev];
  // the key cache as rows of 128 bytes: 64 data rows (swizzled for the MMA)
  // and 2 scale rows (plain) per page; the queries as 64 rows per batch row
  CUtensorMap tm_k, tm_s, tm_q;
  if (!encode_rows128(&tm_k, cache, uint64_t(num_pages) * kRowsPerPage, kPageRows, true) ||
      !encode_rows128(&tm_s, cache, uint64_t(num_pages) * kRowsPerPage, 2, false) ||
      !encode_rows128(&tm_q, q, uint64_t(batch) * indexer::kHeads, indexer::kHeads, true))
    return cudaErrorInvalidValue;
  ScoreParams sp;
  sp.cache = cache;
  sp.weights = weights;
  sp.seq_lens = seq_lens;
  sp.block_table = block_table;
  sp.scores = scores;
  sp.row_keys = row_keys;
  sp.err_word = err_word;
  sp.batch = batch;
  sp.max_pages = max_pages;
  sp.num_pages = num_pages;
  sp.tiles_per_row = (max_pages + 1) / 2;
  sp.total_tiles = batch * sp.tiles_per_row;
  // two CTAs per SM: each CTA's load warp keeps at most 4 tiles in flight, and
  // two pipelines per SM read faster than one pipeline with 8 stages
  sp.grid = int(sp.total_tiles < 2 * sms ? sp.total_tiles : 2 * sms);
  // the split over active tiles keeps 32-bit counts and the rows' lengths in
  // a pipeline stage; the plan, one log entry per CTA
  sp.split_active = batch <= kPlanMaxRows && sp.total_tiles < (int64_t(1) << 31);
  const bool planned = plan_state != nullptr && sp.split_active && sp.grid <= kIndexerPlanMaxGrid;
  sp.plan = planned ? static_cast<PlanState*>(plan_state) : nullptr;
  // Both kernels are launched with programmatic stream serialization: each
  // grid's launch and setup overlap the previous kernel's tail, and each
  // waits (griddepcontrol.wait) for that kernel before it reads anything.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t scfg = {};
  scfg.gridDim = dim3(unsigned(sp.grid));
  scfg.blockDim = dim3(kThreads);
  scfg.dynamicSmemBytes = kSmemBytes;
  scfg.stream = stream;
  scfg.attrs = attr;
  scfg.numAttrs = 1;
  const uint64_t wait_ns = pipeline_wait_ns();
  if ((e = cudaLaunchKernelEx(&scfg, indexer_score_kernel, tm_k, tm_s, tm_q, sp, wait_ns)) != cudaSuccess) return e;
  TopkParams tp;
  tp.scores = scores;
  tp.row_keys = row_keys;
  tp.seq_lens = seq_lens;
  tp.block_table = block_table;
  tp.out = out;
  tp.max_pages = max_pages;
  tp.num_pages = num_pages;
  tp.batch = batch;
  tp.plan = sp.plan;
  tp.plan_grid = sp.grid;
  // with a plan, one more CTA (cluster) past the rows updates it
  const int64_t extra = planned ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(batch + extra));
  cfg.blockDim = dim3(kTopkThreads);
  cfg.dynamicSmemBytes = kTopkSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // rows that fit in shared memory: a cluster of two CTAs per row; longer rows
  // one CTA each, keys re-read from the L2-resident scores
  if (max_pages * kPageRows <= kSmemKeys) {
    cfg.gridDim = dim3(unsigned(2 * (batch + extra)));
    e = cudaLaunchKernelEx(&cfg, indexer_topk_pair_kernel, tp);
  } else {
    e = cudaLaunchKernelEx(&cfg, indexer_topk_kernel<false>, tp);
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace dsa
