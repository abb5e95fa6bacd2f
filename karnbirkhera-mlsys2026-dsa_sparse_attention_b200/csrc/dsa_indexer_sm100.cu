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
//   topk    one CTA (1024 threads) per batch row: radix select of the 2048th
//           largest score (11 + 11 + 10 bits of the order-preserving key,
//           histograms in shared memory), a position-ordered gather of the
//           winners, a bitonic sort (score descending, position ascending) and
//           the translation to slot ids.
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

constexpr uint32_t kOffStage = 0;
constexpr uint32_t kOffQ = kOffStage + kStages * kStageBytes;
constexpr uint32_t kOffW = kOffQ + 2 * kQBytes;                 // float [2][64] head weights
constexpr uint32_t kOffBar = kOffW + 2 * kHeads * 4;
enum : int {
  B_FULL = 0,
  B_EMPTY = B_FULL + kStages,
  B_Q_FULL = B_EMPTY + kStages,   // 2
  B_Q_EMPTY = B_Q_FULL + 2,       // 2
  B_D_FULL = B_Q_EMPTY + 2,       // 2
  B_D_EMPTY = B_D_FULL + 2,       // 2
  B_DONE = B_D_EMPTY + 2,
  B_COUNT
};
constexpr uint32_t kOffMisc = kOffBar + B_COUNT * 8;
constexpr uint32_t kSmemBytes = kOffMisc + 16 + 1024;
static_assert(kOffQ % 1024 == 0 && kStageBytes % 1024 == 0, "swizzle atoms need 1 KB");

constexpr int kThreads = 192;   // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr uint32_t kEpiThreads = 128;
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

// ---------------------------------------------------------------- TMA warp
__device__ void load_warp(const Ctx& c, const ScoreParams& p, const CUtensorMap* tm_k, const CUtensorMap* tm_q) {
  int64_t n = 0, prev_b = -1;
  int rows = 0;   // Q buffers loaded
  bool ok = true;
  uint32_t bad = 0;
  for (int64_t t = c.t_begin; t < c.t_end && ok; ++t) {
    const int64_t b = t / p.tiles_per_row, k = t % p.tiles_per_row;
    const int sl = row_len(p, b);
    if (int64_t(k) * kTileRows >= sl) continue;   // past the row's end: nothing to score
    if (b != prev_b) {
      const int qb = rows & 1;
      if (rows >= 2 && !(ok = mbar_wait(bar(c, B_Q_EMPTY + qb), uint32_t((rows >> 1) - 1) & 1u, c.abort, c.timeout_ns)))
        break;
      mbar_arrive_expect_tx(bar(c, B_Q_FULL + qb), kQBytes);
      tma_load_2d(c.sbase + kOffQ + qb * kQBytes, tm_q, 0, int(b * kHeads), bar(c, B_Q_FULL + qb));
      ++rows;
      prev_b = b;
    }
    const int s = int(n % kStages);
    if (n >= kStages && !(ok = mbar_wait(bar(c, B_EMPTY + s), uint32_t(n / kStages - 1) & 1u, c.abort, c.timeout_ns)))
      break;
    mbar_arrive_expect_tx(bar(c, B_FULL + s), kStageBytes);
    for (int h = 0; h < 2; ++h) {
      const int64_t pi = 2 * k + h;
      int32_t page = -1;
      if (pi * kPageRows < sl) {
        page = __ldg(p.block_table + b * p.max_pages + pi);
        if (page < 0 || int64_t(page) >= p.num_pages) {
          bad = 1;
          page = -1;
        }
      }
      // A page past the row's end or a bad one is loaded from row -66: the
      // tensor map fills it with zeros (its scores are discarded anyway).
      const int row = page >= 0 ? page * kRowsPerPage : -kRowsPerPage;
      tma_load_2d(c.sbase + kOffStage + s * kStageBytes + h * kPageDataBytes, tm_k, 0, row, bar(c, B_FULL + s));
    }
    ++n;
  }
  if (bad) report_error(p.err_word, DSA_DEVICE_ERR_BAD_INDEX);
  // every load must have landed before the CTA exits (also on an abort)
  if (n > 0) drain_wait(bar(c, B_FULL + int((n - 1) % kStages)), uint32_t((n - 1) / kStages) & 1u, c.timeout_ns);
  if (rows > 0) drain_wait(bar(c, B_Q_FULL + ((rows - 1) & 1)), uint32_t((rows - 1) >> 1) & 1u, c.timeout_ns);
}

// ---------------------------------------------------------------- MMA warp
__device__ void mma_warp(const Ctx& c, const ScoreParams& p) {
  int64_t n = 0, prev_b = -1;
  int rows = 0;
  bool ok = true;
  for (int64_t t = c.t_begin; t < c.t_end && ok; ++t) {
    const int64_t b = t / p.tiles_per_row, k = t % p.tiles_per_row;
    const int sl = row_len(p, b);
    if (int64_t(k) * kTileRows >= sl) continue;
    if (b != prev_b) {
      if (rows > 0) mma_commit(bar(c, B_Q_EMPTY + ((rows - 1) & 1)));   // previous row's queries done
      if (!(ok = mbar_wait(bar(c, B_Q_FULL + (rows & 1)), uint32_t(rows >> 1) & 1u, c.abort, c.timeout_ns))) break;
      ++rows;
      prev_b = b;
    }
    const int s = int(n % kStages), db = int(n & 1);
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
  mma_commit(bar(c, B_DONE));
  drain_wait(bar(c, B_DONE), 0u, c.timeout_ns);
}

// ---------------------------------------------------------------- epilogue
// Thread r (TMEM lane r) owns position r of each tile.
__device__ void epilogue_warps(const Ctx& c, const ScoreParams& p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = 32 * (warp & 3) + lane;
  const uint32_t t_lane = uint32_t(32 * (warp & 3)) << 16;
  const int er = threadIdx.x - 64;   // 0..127: weight loader index
  int64_t n = 0, prev_b = -1;
  int rows = 0;
  bool ok = true;
  for (int64_t t = c.t_begin; t < c.t_end && ok; ++t) {
    const int64_t b = t / p.tiles_per_row, k = t % p.tiles_per_row;
    const int sl = row_len(p, b);
    if (int64_t(k) * kTileRows >= sl) continue;
    if (b != prev_b) {
      // this row's head weights into shared memory (double-buffered by row)
      named_barrier_sync(1, kEpiThreads);   // the previous row's weights are no longer read
      const int wb = rows & 1;
      if (er < kHeads) {
        float* w = reinterpret_cast<float*>(__cvta_shared_to_generic(c.sbase + kOffW + wb * kHeads * 4));
        w[er] = __ldg(p.weights + b * kHeads + er);
      }
      named_barrier_sync(1, kEpiThreads);
      ++rows;
      prev_b = b;
    }
    const int64_t pos = int64_t(k) * kTileRows + r;
    // this position's scale and page validity, fetched while the MMA runs
    const int64_t pi = pos >> 6;
    float scale = 0.f;
    bool valid = pos < sl;
    if (valid) {
      const int32_t page = __ldg(p.block_table + b * p.max_pages + pi);
      valid = page >= 0 && int64_t(page) < p.num_pages;
      if (valid)
        scale = __ldg(reinterpret_cast<const float*>(p.cache + int64_t(page) * kPageBytes + kPageDataBytes) + (pos & 63));
    }
    const int db = int(n & 1);
    if (!(ok = mbar_wait(bar(c, B_D_FULL + db), uint32_t(n >> 1) & 1u, c.abort, c.timeout_ns))) break;
    tc_fence_after();
    const float* w = reinterpret_cast<const float*>(__cvta_shared_to_generic(c.sbase + kOffW + ((rows - 1) & 1) * kHeads * 4));
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float d[16];
      tmem_ld16(c.tmem + t_lane + 64u * db + 16u * q, d);
      tmem_wait_ld();
#pragma unroll
      for (int h = 0; h < 16; ++h) acc = fmaf(fmaxf(d[h] * scale, 0.f), w[16 * q + h], acc);
    }
    tc_fence_before();
    mbar_arrive(bar(c, B_D_EMPTY + db));
    if (pos < sl) p.scores[b * (p.max_pages * kPageRows) + pos] = valid ? acc : -INFINITY;
    ++n;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    indexer_score_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_q,
                         const ScoreParams p, const uint64_t timeout_ns) {
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
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(c, B_FULL + s), 1);
      mbar_init(bar(c, B_EMPTY + s), 1);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(bar(c, B_Q_FULL + k), 1);
      mbar_init(bar(c, B_Q_EMPTY + k), 1);
      mbar_init(bar(c, B_D_FULL + k), 1);
      mbar_init(bar(c, B_D_EMPTY + k), kEpiThreads);
    }
    mbar_init(bar(c, B_DONE), 1);
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
    if ((threadIdx.x & 31) == 0) load_warp(c, p, &tm_k, &tm_q);
    __syncwarp();
  } else if (warp == 1) {
    if ((threadIdx.x & 31) == 0) mma_warp(c, p);
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

__global__ void __launch_bounds__(kTopkThreads, 1) indexer_topk_kernel(const TopkParams p) {
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t warp_sums[32];
  __shared__ unsigned long long sel[kTopk];
  __shared__ uint32_t sh_prefix, sh_need;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t cap = p.max_pages * kPageRows;
  int sl = p.seq_lens[b];
  sl = sl <= 0 ? 0 : int(sl > cap ? cap : sl);
  const float* sc = p.scores + b * cap;
  int32_t* out = p.out + b * kTopk;
  const int k = sl < kTopk ? sl : kTopk;

  // radix select: find the k-th largest key T and how many keys equal to T to take
  uint32_t prefix = 0, prefix_mask = 0;
  uint32_t need = uint32_t(k);
  if (sl > kTopk) {
    const int shifts[3] = {21, 10, 0};
    const int widths[3] = {11, 11, 10};
    for (int pass = 0; pass < 3; ++pass) {
      const int sh = shifts[pass], nb = 1 << widths[pass];
      for (int i = tid; i < nb; i += kTopkThreads) hist[i] = 0;
      __syncthreads();
      for (int i = tid; i < sl; i += kTopkThreads) {
        const uint32_t key = ordered_key(sc[i]);
        if ((key & prefix_mask) == prefix) atomicAdd(&hist[(key >> sh) & uint32_t(nb - 1)], 1u);
      }
      __syncthreads();
      // suffix sums from the top bin: bin j holds count(bins >= j) after the scan
      // (each thread owns two adjacent bins of the 2048)
      const int j0 = 2 * tid, j1 = 2 * tid + 1;
      const uint32_t c0 = j0 < nb ? hist[nb - 1 - j0] : 0u, c1 = j1 < nb ? hist[nb - 1 - j1] : 0u;
      uint32_t total;
      const uint32_t before = block_exclusive_scan(c0 + c1, warp_sums, &total);
      // descending bins: cumulative count including bin (nb-1-j)
      const uint32_t incl0 = before + c0, incl1 = before + c0 + c1;
      if (j0 < nb && before < need && incl0 >= need) {
        sh_prefix = uint32_t(nb - 1 - j0);
        sh_need = need - before;
      }
      if (j1 < nb && before + c0 < need && incl1 >= need) {
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
  // gather: every key above the threshold, and the first `need` keys equal to
  // it in position order (each thread scans a contiguous chunk of positions)
  const int chunk = (sl + kTopkThreads - 1) / kTopkThreads;
  const int lo = tid * chunk, hi = min(sl, lo + chunk);
  uint32_t gt = 0, eq = 0;
  if (sl > kTopk) {
    for (int i = lo; i < hi; ++i) {
      const uint32_t key = ordered_key(sc[i]);
      gt += key > prefix;
      eq += key == prefix;
    }
  } else {
    gt = uint32_t(max(hi - lo, 0));   // every position is selected
  }
  uint32_t gt_total, eq_total;
  const uint32_t gt_off = block_exclusive_scan(gt, warp_sums, &gt_total);
  const uint32_t eq_off = block_exclusive_scan(eq, warp_sums, &eq_total);
  {
    uint32_t g = gt_off, e = eq_off;
    for (int i = lo; i < hi; ++i) {
      const uint32_t key = ordered_key(sc[i]);
      const unsigned long long v = (static_cast<unsigned long long>(~key) << 32) | uint32_t(i);
      if (sl <= kTopk || key > prefix) {
        sel[g++] = v;
      } else if (key == prefix && e < need) {
        sel[gt_total + e] = v;
        ++e;
      } else if (key == prefix) {
        ++e;
      }
    }
  }
  for (int i = k + tid; i < kTopk; i += kTopkThreads) sel[i] = ~0ull;   // padding sorts last
  __syncthreads();
  // bitonic sort, ascending on (~key, position) = score descending, position ascending
  for (int size = 2; size <= kTopk; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int i = 2 * tid - (tid & (stride - 1));   // lower index of this thread's pair
      const int j = i + stride;
      const bool up = ((i & size) == 0);
      const unsigned long long a = sel[i], bb = sel[j];
      if ((a > bb) == up) {
        sel[i] = bb;
        sel[j] = a;
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < kTopk; i += kTopkThreads) {
    int32_t slot = -1;
    if (i < k) {
      const uint32_t pos = uint32_t(sel[i] & 0xffffffffu);
      const uint32_t key = ~uint32_t(sel[i] >> 32);
      const int32_t page = p.block_table[b * p.max_pages + (pos >> 6)];
      // a position on a bad page scored -inf (key 0x007fffff); it is no slot
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

bool encode_rows128(CUtensorMap* map, const void* base, uint64_t rows, uint32_t box_rows) {
  const cuuint64_t dims[2] = {128, rows};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
  });
  if (g_attr_err[dev] != cudaSuccess) return g_attr_err[dev];
  CUtensorMap tm_k, tm_q;
  if (!encode_rows128(&tm_k, cache, uint64_t(num_pages) * kRowsPerPage, kPageRows) ||
      !encode_rows128(&tm_q, q, uint64_t(batch) * indexer::kHeads, indexer::kHeads))
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
  indexer_score_kernel<<<sp.grid, kThreads, kSmemBytes, stream>>>(tm_k, tm_q, sp, g_timeout_ns);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  TopkParams tp;
  tp.scores = scores;
  tp.seq_lens = seq_lens;
  tp.block_table = block_table;
  tp.out = out;
  tp.max_pages = max_pages;
  tp.num_pages = num_pages;
  indexer_topk_kernel<<<int(batch), kTopkThreads, 0, stream>>>(tp);
  return cudaGetLastError();
}

}  // namespace dsa
