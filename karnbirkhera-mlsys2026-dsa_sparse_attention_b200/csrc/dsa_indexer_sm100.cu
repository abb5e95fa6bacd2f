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
//   score   one persistent CTA per SM over a static plan of 128-position
//           tiles (two pages).  Warp 0 loads pages with TMA (a page is 64 rows
//           of 128 fp8 + 64 fp32 scales = 8448 bytes; the tensor map views the
//           cache as rows of 128 bytes, 66 per page, so the 64 data rows land
//           128-byte-swizzled for the tensor cores), warp 1 issues
//           tcgen05.mma kind::f8f6f4 (e4m3 x e4m3, M=128 positions, N=64
//           heads, K=32) into a double-buffered TMEM accumulator, warps 2-5
//           (one TMEM lane = one position per thread) apply scale, relu and
//           the head weights and write the position's final score (fp32) to
//           the workspace.  HBM-bound: 132 bytes per position.
//   topk    one CTA (1024 threads) per batch row: the row's order-preserving
//           keys into shared memory (rows up to 40960 positions), radix select
//           of the 2048th largest (11 + 11 + 10 bits, warp-aggregated shared
//           histograms), a position-ordered gather of the winners, a bitonic
//           sort (score descending, position ascending) and the translation to
//           slot ids.
//
// Every wait is bounded (DSA_DEVICE_ERR_TIMEOUT on expiry).  A block-table
// entry outside [0, num_pages) for a page inside seq_len, or a seq_len larger
// than the table holds, is reported as DSA_DEVICE_ERR_BAD_INDEX; such
// positions score -inf and are never returned as slots.
#include <cuda.h>
#include <cudaTypedefs.h>

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

constexpr int kStages = 6;
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
constexpr uint32_t kSmemBytes = kOffMisc + 16 + 1024;
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

struct ScoreParams {
  const uint8_t* cache;          // [num_pages, 8448]
  const float* weights;          // [B, 64]
  const int32_t* seq_lens;       // [B]
  const int32_t* block_table;    // [B, max_pages]
  float* scores;                 // [B, max_pages * 64]
  uint32_t* err_word;
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
  uint64_t timeout_ns;
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

// Positions of row b that the score kernel covers: seq_len clamped to what the
// table can hold (a larger seq_len is a bad index).
__device__ __forceinline__ int row_len(const ScoreParams& p, int64_t b) {
  const int sl = __ldg(p.seq_lens + b);
  const int64_t cap = p.max_pages * kPageRows;
  return sl <= 0 ? 0 : int(sl > cap ? cap : sl);
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
};

// ---------------------------------------------------------------- TMA warp
// The whole warp walks the tiles 32 at a time: lane l looks up tile t0 + l
// (its row, whether it has positions, its two page ids) with independent
// loads, then lane 0 issues the 32 tiles' TMA loads in order, taking the page
// ids from the lanes by shuffle -- no dependent global load per tile.
__device__ void load_warp(const Ctx& c, const ScoreParams& p, const CUtensorMap* tm_k, const CUtensorMap* tm_s,
                          const CUtensorMap* tm_q) {
  const int lane = threadIdx.x & 31;
  int64_t n = 0;
  int32_t prev_b = -1;
  int rows = 0;   // Q buffers loaded
  bool ok = true;
  uint32_t bad = 0;
  for (int64_t t0 = c.t_begin; t0 < c.t_end && ok; t0 += 32) {
    const int64_t t = t0 + lane;
    int32_t b = 0, pg0 = -1, pg1 = -1;
    bool act = false;
    if (t < c.t_end) {
      const int64_t bb = t / p.tiles_per_row, k = t - bb * p.tiles_per_row;
      b = int32_t(bb);
      const int sl = row_len(p, bb);
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
            const int row = pages[h] >= 0 ? pages[h] * kRowsPerPage : -kRowsPerPage;
            tma_load_2d(c.sbase + kOffStage + s * kStageBytes + h * kPageDataBytes, tm_k, 0, row, bar(c, B_FULL + s));
            tma_load_2d(c.sbase + kOffScale + s * kScaleBytes + h * (kScaleBytes / 2), tm_s, 0, row + kPageRows,
                        bar(c, B_FULL + s));
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
  }
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    if (bad) report_error(p.err_word, DSA_DEVICE_ERR_BAD_INDEX);
    // every load must have landed before the CTA exits (also on an abort)
    if (n > 0) drain_wait(bar(c, B_FULL + int((n - 1) % kStages)), uint32_t((n - 1) / kStages) & 1u, c.timeout_ns);
    if (rows > 0) drain_wait(bar(c, B_Q_FULL + ((rows - 1) & 1)), uint32_t((rows - 1) >> 1) & 1u, c.timeout_ns);
  }
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
    if (int64_t(k) * kTileRows >= sl) continue;
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
  drain_wait(bar(c, B_DONE + m), 0u, c.timeout_ns);
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
  for (TileWalk tw(p, c.t_begin); tw.t < c.t_end && ok; tw.next(p)) {
    const int64_t b = tw.b, k = tw.k;
    const int sl = tw.sl;
    if (int64_t(k) * kTileRows >= sl) continue;
    if (b != prev_b) {
      // this row's head weights into the group's shared memory (double-buffered by row)
      named_barrier_sync(1 + g, kEpiThreads);   // the previous row's weights are no longer read
      if (gr < kHeads) {
        float* w = reinterpret_cast<float*>(
            __cvta_shared_to_generic(c.sbase + kOffW + (2 * g + (rows & 1)) * kHeads * 4));
        w[gr] = __ldg(p.weights + b * kHeads + gr);
      }
      named_barrier_sync(1 + g, kEpiThreads);
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
    if (pos < sl) p.scores[b * (p.max_pages * kPageRows) + pos] = scale * ((acc[0] + acc[1]) + (acc[2] + acc[3]));
    ++n;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    indexer_score_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_s,
                         const __grid_constant__ CUtensorMap tm_q, const ScoreParams p, const uint64_t timeout_ns) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Ctx c;
  c.sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  c.abort = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc + 4);
  c.timeout_ns = timeout_ns;
  c.t_begin = range_begin(p, blockIdx.x);
  c.t_end = range_begin(p, int64_t(blockIdx.x) + 1);
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  c.tmem = *tmem_slot;
  if (warp == 0) {
    load_warp(c, p, &tm_k, &tm_s, &tm_q);
  } else if (warp <= 2) {
    if ((threadIdx.x & 31) == 0) mma_warp(c, p, warp - 1);
    __syncwarp();
  } else {
    epilogue_warps(c, p);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *c.abort) report_error(p.err_word, DSA_DEVICE_ERR_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(c.tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- top-k
constexpr int kTopkThreads = 1024;

// Order-preserving key: a larger float gives a larger unsigned key (-inf lowest
// of the ordinary values).
__device__ __forceinline__ uint32_t ordered_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

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
  const int32_t* seq_lens;
  const int32_t* block_table;
  int32_t* out;          // [B, 2048]
  int64_t max_pages;
  int64_t num_pages;
};

// Rows of up to kSmemKeys positions keep their keys in shared memory for all
// passes; longer rows read them from the scores in global memory (L2).
constexpr int kSmemKeys = 40960;
constexpr uint32_t kTopkSmemBytes = kSmemKeys * 4 + kTopk * 8;

template <bool kKeysInSmem>
__global__ void __launch_bounds__(kTopkThreads, 1) indexer_topk_kernel(const TopkParams p) {
  extern __shared__ __align__(16) uint8_t topk_smem[];
  uint32_t* keys_s = reinterpret_cast<uint32_t*>(topk_smem);
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(topk_smem + kSmemKeys * 4);
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t warp_sums[32];
  __shared__ uint32_t warp_gt[32], warp_eq[32];
  __shared__ uint32_t sh_prefix, sh_need;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t cap = p.max_pages * kPageRows;
  int sl = p.seq_lens[b];
  sl = sl <= 0 ? 0 : int(sl > cap ? cap : sl);
  const float* sc = p.scores + b * cap;
  const int32_t* bt = p.block_table + b * p.max_pages;
  int32_t* out = p.out + b * kTopk;
  const int k = sl < kTopk ? sl : kTopk;
  // key of position i: a position on a page outside the pool scores -inf
  auto key_global = [&](int i) -> uint32_t {
    const int32_t page = __ldg(bt + (i >> 6));
    const bool ok = page >= 0 && int64_t(page) < p.num_pages;
    return ordered_key(ok ? sc[i] : -INFINITY);
  };
  if constexpr (kKeysInSmem) {
    for (int i = tid; i < sl; i += kTopkThreads) keys_s[i] = key_global(i);
    __syncthreads();
  }
  auto key_of = [&](int i) -> uint32_t {
    if constexpr (kKeysInSmem) return keys_s[i];
    else return key_global(i);
  };

  // radix select: the k-th largest key T, and how many keys equal to T to take
  uint32_t prefix = 0, prefix_mask = 0;
  uint32_t need = uint32_t(k);
  if (sl > kTopk) {
    const int shifts[3] = {21, 10, 0};
    const int widths[3] = {11, 11, 10};
    for (int pass = 0; pass < 3; ++pass) {
      const int sh = shifts[pass], nb = 1 << widths[pass];
      for (int i = tid; i < nb; i += kTopkThreads) hist[i] = 0;
      __syncthreads();
      // warp-aggregated: a row's scores crowd into few high-order bins, so
      // lanes with the same bin add their count with one atomic
      for (int base = 0; base < sl; base += kTopkThreads) {
        const int i = base + tid;
        uint32_t bin = 0xffffffffu;
        if (i < sl) {
          const uint32_t key = key_of(i);
          if ((key & prefix_mask) == prefix) bin = (key >> sh) & uint32_t(nb - 1);
        }
        const uint32_t same = __match_any_sync(0xffffffffu, bin);
        if (bin != 0xffffffffu && lane == __ffs(same) - 1) atomicAdd(&hist[bin], __popc(same));
      }
      __syncthreads();
      // cumulative counts from the top bin; each thread owns two adjacent bins
      const int j0 = 2 * tid, j1 = 2 * tid + 1;
      const uint32_t c0 = j0 < nb ? hist[nb - 1 - j0] : 0u, c1 = j1 < nb ? hist[nb - 1 - j1] : 0u;
      uint32_t total;
      const uint32_t before = block_exclusive_scan(c0 + c1, warp_sums, &total);
      if (j0 < nb && before < need && before + c0 >= need) {
        sh_prefix = uint32_t(nb - 1 - j0);
        sh_need = need - before;
      }
      if (j1 < nb && before + c0 < need && before + c0 + c1 >= need) {
        sh_prefix = uint32_t(nb - 1 - j1);
        sh_need = need - (before + c0);
      }
      __syncthreads();
      prefix |= sh_prefix << sh;
      prefix_mask |= uint32_t(nb - 1) << sh;
      need = sh_need;
      __syncthreads();
    }
  }
  if (sl <= kTopk) {
    // every position is selected
    for (int i = tid; i < kTopk; i += kTopkThreads)
      sel[i] = i < sl ? (static_cast<unsigned long long>(~key_of(i)) << 32) | uint32_t(i) : ~0ull;
  } else {
    // gather in position order: warp w owns a contiguous chunk, its lanes read
    // consecutive positions; keys above T all go, keys equal to T while fewer
    // than `need` were taken before them
    const int chunk = ((sl + 31) / 32 + 31) & ~31;
    const int lo = warp * chunk, hi = min(sl, lo + chunk);
    uint32_t gt = 0, eq = 0;
    for (int i = lo + lane; i < hi; i += 32) {
      const uint32_t key = key_of(i);
      gt += key > prefix;
      eq += key == prefix;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      gt += __shfl_xor_sync(0xffffffffu, gt, o);
      eq += __shfl_xor_sync(0xffffffffu, eq, o);
    }
    if (lane == 0) {
      warp_gt[warp] = gt;
      warp_eq[warp] = eq;
    }
    __syncthreads();
    uint32_t g_off = 0, e_off = 0, gt_total = 0;
    for (int w = 0; w < 32; ++w) {
      if (w < warp) {
        g_off += warp_gt[w];
        e_off += warp_eq[w];
      }
      gt_total += warp_gt[w];
    }
    const uint32_t lt_mask = (1u << lane) - 1u;
    for (int base = lo; base < hi; base += 32) {
      const int i = base + lane;
      const uint32_t key = i < hi ? key_of(i) : 0u;
      const bool g = i < hi && key > prefix, e = i < hi && key == prefix;
      const uint32_t gm = __ballot_sync(0xffffffffu, g), em = __ballot_sync(0xffffffffu, e);
      const unsigned long long v = (static_cast<unsigned long long>(~key) << 32) | uint32_t(i);
      if (g) sel[g_off + __popc(gm & lt_mask)] = v;
      if (e) {
        const uint32_t r = e_off + __popc(em & lt_mask);
        if (r < need) sel[gt_total + r] = v;
      }
      g_off += __popc(gm);
      e_off += __popc(em);
    }
  }
  __syncthreads();
  // bitonic sort, ascending on (~key, position) = score descending, position ascending
  for (int size = 2; size <= kTopk; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
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
  }
  for (int i = tid; i < kTopk; i += kTopkThreads) {
    int32_t slot = -1;
    if (i < k) {
      const uint32_t pos = uint32_t(sel[i] & 0xffffffffu);
      const uint32_t key = ~uint32_t(sel[i] >> 32);
      const int32_t page = __ldg(bt + (pos >> 6));
      // a position on a bad page (scored -inf) is no slot
      if (key != ordered_key(-INFINITY) && page >= 0 && int64_t(page) < p.num_pages)
        slot = page * kPageRows + int32_t(pos & 63);
    }
    out[i] = slot;
  }
}

// ---------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
constexpr int kMaxDevices = 64;
std::once_flag g_attr_once[kMaxDevices];
cudaError_t g_attr_err[kMaxDevices];
uint64_t g_timeout_ns = 0;

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
                           int32_t* out, float* scores, uint32_t* err_word, int sms, cudaStream_t stream) {
  using namespace indexer;
  std::call_once(g_encode_once, []() {
    cudaDriverEntryPointQueryResult qr;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    const char* env = std::getenv("DSA_WAIT_TIMEOUT_MS");
    const long ms = env ? std::strtol(env, nullptr, 10) : 0;
    g_timeout_ns = uint64_t(ms > 0 ? ms : 2000) * 1000000ull;
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
  sp.err_word = err_word;
  sp.batch = batch;
  sp.max_pages = max_pages;
  sp.num_pages = num_pages;
  sp.tiles_per_row = (max_pages + 1) / 2;
  sp.total_tiles = batch * sp.tiles_per_row;
  sp.grid = int(sp.total_tiles < sms ? sp.total_tiles : sms);
  indexer_score_kernel<<<sp.grid, kThreads, kSmemBytes, stream>>>(tm_k, tm_s, tm_q, sp, g_timeout_ns);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  TopkParams tp;
  tp.scores = scores;
  tp.seq_lens = seq_lens;
  tp.block_table = block_table;
  tp.out = out;
  tp.max_pages = max_pages;
  tp.num_pages = num_pages;
  // rows that fit keep their keys in shared memory through every pass
  if (max_pages * kPageRows <= kSmemKeys)
    indexer_topk_kernel<true><<<int(batch), kTopkThreads, kTopkSmemBytes, stream>>>(tp);
  else
    indexer_topk_kernel<false><<<int(batch), kTopkThreads, kTopkSmemBytes, stream>>>(tp);
  return cudaGetLastError();
}

}  // namespace dsa
