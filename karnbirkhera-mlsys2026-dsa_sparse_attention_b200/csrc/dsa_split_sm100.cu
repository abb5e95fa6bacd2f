// dsa_split_sm100.cu — the split-KV kernel on the sm_100a tensor cores.
//
// One persistent CTA per SM walks its range of the static plan (dsa_common.cuh)
// one 128-slot block ("tile") at a time.  Per tile:
//   gather   4 producer warps copy the 128 selected rows with 16-byte
//            cp.async straight into the 128-byte-swizzled shared-memory layout
//            the tensor cores read: each ckv row (1024 B) as 8 chunks of 64
//            columns, each kpe row (128 B) as 1 chunk.  A warp instruction
//            covers 2 rows x 256 contiguous bytes (fully used 128-byte lines).
//            Padding (-1) and out-of-range slots are zero-filled (src-size 0)
//            without touching HBM.  (TMA tile::gather4 moves 128-byte rows at
//            about 1/3 of this rate on B200, so it is not used for the rows.)
//   logits   S^T[128 keys x 16 heads] = K[128 x 576] . Q^T  — 36 tcgen05.mma
//            (M=128, N=16, K=16), keys on M, the 16 heads on N, fp32 in TMEM.
//   softmax  4 warps, one TMEM lane (key) per thread: mask, scale to log2
//            units, per-head tile max across the 128 threads, exp2.  The
//            running reference max only moves when a head's max grows by more
//            than 8 (2^8 headroom in fp32), so the O accumulator is rescaled
//            in TMEM only on those rare tiles.
//   PV       O^T[512 dims x 16 heads] += V^T . P^T — the SAME ckv chunks read
//            as an MN-major operand (no second copy), P^T in bf16 from shared
//            memory; 4 accumulator blocks of 128 dims, 32 MMAs per tile.
//   epilogue when the CTA's segment of a token ends: O / l -> bf16 output and
//            base-2 lse, or (a token split over several CTAs) a ticket: over
//            a few CTAs the last segment to arrive merges the others' fp32
//            partial records with its own accumulator, the others write and
//            publish theirs; over many CTAs every segment publishes and the
//            CTAs whose ranges end inside the token share the merge.
//   indices  slot ids, or (second instantiation) positions translated
//            through a block table on the fly.
//
// Warp roles (384 threads): warps 0-3 gather, warps 4-5 issue the logits MMAs
// (warp 4 owns the TMEM allocation and loads Q with TMA), warps 6-7 the PV
// MMAs, warps 8-11 run softmax and the epilogue.
// A thread issues one tcgen05.mma per ~130 cycles, so each MMA stream is
// split over several issuing threads.
//
// Shared memory (bytes, 1024-aligned): Q 9x2 KB | kpe 2x16 KB | ckv slabs
// 5x32 KB (a slab = ckv columns [128j, 128j+128) of one tile) | P 2x4 KB |
// reduction scratch | mbarriers.  The 5-slab ring lets the next tile's kpe
// and first slab land while the current tile computes; the current tile's
// slabs are released one by one as its PV MMAs retire.
//
// Every wait is bounded (DSA_DEVICE_ERR_TIMEOUT on expiry); the kernel then
// drains its own copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>

#include <cooperative_groups.h>

#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "dsa_common.cuh"
#include "dsa_sm100_ptx.cuh"

namespace dsa {
namespace sm100 {

using namespace ptx;

constexpr int kProducerWarps = 4;
constexpr int kQkWarp0 = 4;       // warps 4,5 issue the logits MMAs; warp 4 owns the TMEM allocation
constexpr int kPvWarp0 = 6;       // warps 6,7 issue the PV MMAs
constexpr int kSoftmaxWarp0 = 8;
constexpr int kSetupWarp = kQkWarp0 + 1;   // its lane 0 initialises the barriers
constexpr int kThreads = 384;
constexpr uint32_t kProducerThreads = 128;
constexpr uint32_t kSoftmaxThreads = 128;

constexpr int kSlabs = 5;
constexpr uint32_t kChunkBytes = 128 * 128;      // 128 rows x 64 bf16 columns
constexpr uint32_t kSlabBytes = 2 * kChunkBytes;  // two chunks: columns 128j..128j+127
constexpr uint32_t kQChunkBytes = 16 * 128;      // 16 heads x 64 columns
constexpr uint32_t kQBytes = 9 * kQChunkBytes;
constexpr uint32_t kPBytes = 2 * 16 * 128;       // P^T: 16 heads x 128 keys as two 64-key chunks

constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffKpe = kOffQ + kQBytes;
constexpr uint32_t kOffSlab = kOffKpe + 2 * kChunkBytes;
constexpr uint32_t kOffP = kOffSlab + kSlabs * kSlabBytes;
constexpr uint32_t kOffRed = kOffP + 2 * kPBytes;              // float [2][4][16] tile max
constexpr uint32_t kOffRedL = kOffRed + 2 * 4 * 16 * 4;         // float [4][16] segment sums
constexpr uint32_t kOffMerge = kOffRedL + 4 * 16 * 4;          // merge scratch: weights [16][16], 1/L [16], records [16]
constexpr uint32_t kOffMergeRec = kOffMerge + (16 * 16 + 16) * 4;
constexpr uint32_t kOffTask = kOffMergeRec + 16 * 8;           // merges left for the end of the CTA [2]
constexpr uint32_t kOffBar = kOffTask + 2 * 64;

enum : int {
  B_Q_FULL = 0,
  B_Q_EMPTY,
  B_KPE_FULL,                    // 2
  B_KPE_EMPTY = B_KPE_FULL + 2,  // 2
  B_SLAB_FULL = B_KPE_EMPTY + 2,
  B_SLAB_EMPTY = B_SLAB_FULL + kSlabs,
  B_S_FULL = B_SLAB_EMPTY + kSlabs,
  B_S_EMPTY = B_S_FULL + 2,
  B_P_FULL = B_S_EMPTY + 2,
  B_P_EMPTY = B_P_FULL + 2,
  B_O_FULL = B_P_EMPTY + 2,
  B_O_EMPTY,
  B_DONE,                        // 4: one per MMA-issuing thread (2 logits, 2 PV)
  B_MERGE = B_DONE + 4,          // bulk copies of other segments' records into the slab ring
  B_STAGE_FULL,                  // 3: FP8 mode, staged fp8 slab landed (gather warps' copies)
  B_STAGE_EMPTY = B_STAGE_FULL + 3,  // 3: FP8 mode, staged slab converted (softmax warps)
  B_COUNT = B_STAGE_EMPTY + 3
};

constexpr uint32_t kOffMisc = kOffBar + B_COUNT * 8;   // tmem base, abort flag, merge flag
constexpr uint32_t kOffScale8 = (kOffMisc + 16 + 15) & ~15u;   // FP8 mode: staged row scales [3][128] fp32
constexpr uint32_t kSmemBytes = kOffScale8 + 3 * 128 * 4 + 1024;  // + slack for 1024-B alignment
static_assert(kOffSlab % 1024 == 0 && kOffKpe % 1024 == 0 && kOffP % 1024 == 0, "swizzle atoms need 1 KB");
static_assert(kSmemBytes <= 232448, "shared memory budget of one CTA");
constexpr int kMaxStaged = 4;   // other segments' records staged in shared memory by a merge
static_assert(kMaxStaged * kRecordBytes <= kSlabs * kSlabBytes, "merge staging of the records fits in the slab ring");
static_assert(16 * 512 * 2 <= 2 * 16384, "a merged bf16 output tile fits in the kpe ring");

// TMEM columns: S buffer b, partial q at 32 b + 16 q (two partial sums of the
// logits, one per issuing warp); O block j at 64 + 16 j.
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kTmemO = 64;

constexpr float kRescaleThreshold = 8.0f;   // log2 units

// Descriptor high words (stride byte offset 1024, fixed 0b001, 128-byte swizzle)
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
constexpr uint32_t kLboKMajor = 1u << 16;                      // unused for swizzled K-major; 16 B
constexpr uint32_t kLboPV = (kChunkBytes >> 4) << 16;           // MN-major: stride between 64-dim chunks

__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo_field) {
  return (uint64_t(kDescHi) << 32) | uint64_t(lbo_field | ((saddr & 0x3FFFFu) >> 4));
}

// A token split over more than kMaxStaged + 1 CTAs is merged by several of
// them at the end of their ranges (help_merge): slot 1 for the CTA's last
// segment, slot 0 for its first segment when that one arrived last.
struct HelpTask {
  int64_t t;          // the split token
  int64_t b_lo;       // its first CTA
  int32_t nseg;       // its segments (CTAs b_lo .. b_lo + nseg - 1)
  uint32_t pref;      // output chunks this CTA claims first
  uint32_t last;      // this segment arrived last: it completes the merge
  uint32_t pending;   // there is merge work at the end of the CTA
  int32_t helpers;    // CTAs of the token that end their ranges inside it
};
static_assert(sizeof(HelpTask) <= 64, "two merge tasks fit their shared-memory slot");

struct Ctx {
  uint32_t sbase;          // shared address of the aligned base
  uint32_t tmem;           // TMEM base address
  volatile uint32_t* abort;
  volatile uint32_t* merge_flag;
  float* red;
  float* red_l;
  uint8_t* merge;          // merge scratch: weights [16][16], 1/L [16], record addresses [16]
  HelpTask* task;          // [2]
  uint8_t* merge_stage;    // the slab ring, reused to stage records once a CTA has no tiles left
  uint8_t* merge_out;      // the kpe ring, reused for the merged bf16 output tile at the end
  uint8_t* scale8;         // FP8 mode: staged row scales [3][128]
  uint64_t timeout_ns;     // pipeline waits
  uint64_t drain_ns;       // waits for this CTA's own copies / MMAs after an abort
  int64_t g_begin, g_end;  // plan range of this CTA
};

__device__ __forceinline__ uint32_t bar_addr(const Ctx& c, int b) { return c.sbase + kOffBar + 8u * uint32_t(b); }

// Any thread of named barrier `id` (128 threads) has `v`.
template <int kId>
__device__ __forceinline__ bool group_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "n"(kId)
      : "memory");
  return r != 0;
}

// All threads of named barrier `id` (128 threads) agree on `ok`.
template <int kId>
__device__ __forceinline__ bool group_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(ok)), "n"(kId)
      : "memory");
  return r != 0;
}

// Wait used only while draining after an abort (ignores the abort flag).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) return;
  }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// -------------------------------------------------------------------------
// warps 0-3: gather producer (thread p = 0..127)
//   ckv slab: thread p copies 16 B piece (p & 7) of chunk (p >> 3) & 1 of rows
//             (p >> 4) + 8 e, e = 0..15  -> warp covers 2 rows x 256 B per copy
//   kpe:      piece (p & 7) of rows (p >> 4) + 8 (2 e + ((p >> 3) & 1)), e = 0..7
//   All rows of a thread share (row & 7) = p >> 4, so the swizzle XOR is fixed.
// -------------------------------------------------------------------------
// Index slots of block g that producer thread p gathers: rows (p >> 4) + 8 e.
__device__ __forceinline__ void load_slots(const SplitParams& prm, int64_t g, int p, int (&s)[16]) {
  const int32_t* row = prm.indices + (g / kBlocksPerToken) * kTopk + (g % kBlocksPerToken) * kBlockKeys + (p >> 4);
#pragma unroll
  for (int e = 0; e < 16; ++e) s[e] = __ldg(row + 8 * e);
}

// Page-table-native indexing: the block-table row of token t as an offset
// into block_table, or -1 when the row is outside the table (every position
// of such a token is then a bad index).
__device__ __forceinline__ int64_t row_base(const SplitParams& prm, int32_t row) {
  return (row >= 0 && int64_t(row) < prm.num_rows) ? int64_t(row) * prm.max_pages : -1;
}
__device__ __forceinline__ int32_t row_of(const SplitParams& prm, int64_t t) {
  return prm.seq_of_token ? __ldg(prm.seq_of_token + t) : int32_t(t);
}
// Page holding position `pos` (-1: padding, or outside the row / table).
__device__ __forceinline__ int32_t page_of(const SplitParams& prm, int64_t rbase, int32_t pos) {
  return (rbase >= 0 && pos >= 0 && int64_t(pos >> 6) < prm.max_pages) ? __ldg(prm.block_table + rbase + (pos >> 6))
                                                                          : -1;
}
__device__ __forceinline__ bool page_valid(const SplitParams& prm, int32_t page) {
  return page >= 0 && int64_t(page) * kPage < prm.num_slots;
}

// `raw` holds the index entries of the CTA's first block (loaded before the
// CTA's setup barrier, so their latency overlaps it): slot ids, or in paged
// mode positions, whose block-table row `first_row` was loaded alongside.
// Paged mode runs a two-stage prefetch: positions two blocks ahead, their
// pages one block ahead, so no dependent load stalls a tile's issue.
template <bool kPaged>
__device__ void producer(const Ctx& c, const SplitParams& prm, int (&raw)[16], int32_t first_row) {
  const int p = threadIdx.x;
  const uint32_t row0 = uint32_t(p >> 4);                 // 0..7
  const uint32_t piece = uint32_t(p & 7);
  const uint32_t half = uint32_t((p >> 3) & 1);           // slab: which 64-col chunk; kpe: odd/even row group
  const uint32_t swz = (piece ^ row0) << 4;
  const uint32_t sKpe = c.sbase + kOffKpe, sSlab = c.sbase + kOffSlab;
  const uint8_t* ckv = static_cast<const uint8_t*>(prm.ckv);
  const uint8_t* kpe = static_cast<const uint8_t*>(prm.kpe);

  int64_t i = 0, u = 0;
  bool ok = true;
  uint32_t bad = 0;
  // paged mode: pages of the current block, positions (and row) of the next
  int pg[16], raw_next[16];
  int32_t row_next = 0;
  if constexpr (kPaged) {
    if (c.g_begin < c.g_end) {
      const int64_t rb = row_base(prm, first_row);
#pragma unroll
      for (int e = 0; e < 16; ++e) pg[e] = page_of(prm, rb, raw[e]);
    }
    if (c.g_begin + 1 < c.g_end) {
      load_slots(prm, c.g_begin + 1, p, raw_next);
      row_next = row_of(prm, (c.g_begin + 1) / kBlocksPerToken);
    }
  }
  {
    for (int64_t blk = c.g_begin; blk < c.g_end && ok; ++blk, ++i) {
      int slot[16];
      uint32_t vmask = 0;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int v = raw[e];
        bool valid;
        if constexpr (kPaged) {
          valid = page_valid(prm, pg[e]);
          slot[e] = valid ? pg[e] * kPage + (v & (kPage - 1)) : 0;
        } else {
          valid = v >= 0 && int64_t(v) < prm.num_slots;
          slot[e] = valid ? v : 0;
        }
        bad |= (!valid && v != -1) ? 1u : 0u;
        vmask |= valid ? (1u << e) : 0u;
      }
      if constexpr (kPaged) {
        if (blk + 1 < c.g_end) {
          const int64_t rb = row_base(prm, row_next);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            pg[e] = page_of(prm, rb, raw_next[e]);
            raw[e] = raw_next[e];
          }
          if (blk + 2 < c.g_end) {
            load_slots(prm, blk + 2, p, raw_next);
            row_next = row_of(prm, (blk + 2) / kBlocksPerToken);
          }
        }
      } else {
        if (blk + 1 < c.g_end) load_slots(prm, blk + 1, p, raw);
      }

      const int kb = int(i & 1);
      if (i >= 2 && !(ok = group_all<3>(mbar_wait(bar_addr(c, B_KPE_EMPTY + kb), (uint32_t(i >> 1) & 1u) ^ 1u,
                                                    c.abort, c.timeout_ns))))
        break;
      {
        const uint32_t dst0 = sKpe + kb * kChunkBytes + swz;
#pragma unroll
        for (int e2 = 0; e2 < 8; ++e2) {
          const int e = 2 * e2 + int(half);
          const int s = half ? slot[2 * e2 + 1] : slot[2 * e2];
          const bool valid = (vmask >> e) & 1u;
          const uint32_t row = row0 + 8u * uint32_t(e);
          cp_async16(dst0 + row * 128u, kpe + int64_t(s) * (kKpe * 2) + piece * 16u, valid ? 16u : 0u);
        }
        cp_async_arrive_noinc(bar_addr(c, B_KPE_FULL + kb));
      }
#pragma unroll 1
      for (int j = 0; j < 4; ++j, ++u) {
        const int sl = int(u % kSlabs);
        if (u >= kSlabs && !(ok = group_all<3>(mbar_wait(bar_addr(c, B_SLAB_EMPTY + sl),
                                                          (uint32_t(u / kSlabs) & 1u) ^ 1u, c.abort, c.timeout_ns))))
          break;
        const uint32_t dst0 = sSlab + sl * kSlabBytes + half * kChunkBytes + swz;
        const uint8_t* src0 = ckv + 256 * j + 128 * half + 16 * piece;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint32_t row = row0 + 8u * uint32_t(e);
          cp_async16(dst0 + row * 128u, src0 + int64_t(slot[e]) * (kCkv * 2), ((vmask >> e) & 1u) ? 16u : 0u);
        }
        cp_async_arrive_noinc(bar_addr(c, B_SLAB_FULL + sl));
      }
    }
  }
  bad = __any_sync(0xffffffffu, bad);
  if (bad && (p & 31) == 0) report_error(prm.err_word, DSA_DEVICE_ERR_BAD_INDEX);
  // Every copy must land before the CTA exits (also on an abort).
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// -------------------------------------------------------------------------
// FP8 KV mode (prm.kv_fp8).
//   Copies (gather warps 0-3): thread p covers 16-byte piece q = p & 7 of
//   rows (p >> 3) + 16 e, e = 0..7 (a warp instruction covers 4 rows x 128
//   contiguous bytes).  Per tile the rope pieces (8 bf16 values) go to the
//   kpe buffer (single-buffered in this mode); per 128-column slab the fp8
//   pieces go to a 3-slot staging ring (the fifth slab's 32 KB and the kpe
//   ring's second 16 KB) and lane q copies the slab's scale of row
//   (p >> 3) + 16 q into the staged-scale array.
//   Conversion: before each tile's softmax the softmax warps (idle between
//   tiles) convert the tile's four staged slabs to bf16_rn(fp8 * scale) in the
//   128-byte-swizzled bf16 slab the logits and PV MMAs read (a 4-slab ring),
//   8 pieces per thread, loaded before they are converted so that their
//   latencies overlap.  The gather warps only copy, up to three slabs ahead.  (Splitting the rows between the gather and softmax
//   warps, or an L2 prefetch of the next tile's rows, measured slower: the
//   copies' latency with three 16 KB slabs in flight per SM is the limit.)
// -------------------------------------------------------------------------
constexpr int kRingFp8 = 4;                         // bf16 slabs in FP8 mode
constexpr int kStageSlots = 3;                      // staged fp8 slabs
constexpr uint32_t kStageBytes = 128 * 128;         // one fp8 slab: 128 rows x 128 e4m3
static_assert(2 * kStageBytes <= kSlabBytes && kStageBytes == kChunkBytes, "staging slots: fifth slab, kpe buffer 1");

// Index slots of block g that FP8 gather thread p copies: rows (p >> 3) + 16 e.
__device__ __forceinline__ void load_slots8(const SplitParams& prm, int64_t g, int p, int (&s)[8]) {
  const int32_t* row = prm.indices + (g / kBlocksPerToken) * kTopk + (g % kBlocksPerToken) * kBlockKeys + (p >> 3);
#pragma unroll
  for (int e = 0; e < 8; ++e) s[e] = __ldg(row + 16 * e);
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

// 2 e4m3 values (low byte first) -> 2 bf16 of value * s (low half first).
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint32_t two, float s) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two & 0xffffu), __NV_E4M3);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  const __nv_bfloat162 b = __floats2bfloat162_rn(f.x * s, f.y * s);
  return *reinterpret_cast<const uint32_t*>(&b);
}

// Softmax warps, FP8 mode: converts staged slab u into bf16 ring slot u % 4
// once the slab has landed and the slot is free (thread t covers piece t & 7
// of rows (t >> 3) + 16 e, e = 0..7; the 8 pieces and scales are loaded before
// they are converted so that their latencies overlap), then arrives on the
// slot's full and the staging slot's empty barrier.  Returns false if a wait
// gave up (the 128 threads agree).
__device__ __forceinline__ bool convert_slab_fp8(const Ctx& c, int64_t u, int t) {
  const uint32_t q = uint32_t(t & 7), rb = uint32_t(t >> 3), r7 = rb & 7u;   // rows rb + 16 e
  const uint32_t k0 = 2u * (q & 3u);
  const uint32_t sw0 = (k0 ^ r7) << 4, sw1 = ((k0 + 1u) ^ r7) << 4;
  const int st = int(u % kStageSlots), sl = int(u % kRingFp8);
  bool got = mbar_wait(bar_addr(c, B_STAGE_FULL + st), uint32_t(u / kStageSlots) & 1u, c.abort, c.timeout_ns);
  if (u >= kRingFp8)
    got = got && mbar_wait(bar_addr(c, B_SLAB_EMPTY + sl), (uint32_t(u / kRingFp8) & 1u) ^ 1u, c.abort, c.timeout_ns);
  if (!group_all<1>(got)) return false;
  uint8_t* const slabs = c.merge_stage;   // the slab ring (generic pointer into the shared window)
  const uint8_t* src = (st < 2 ? slabs + kRingFp8 * kSlabBytes + uint32_t(st) * kStageBytes
                               : c.merge_out + kChunkBytes) + rb * 128u + q * 16u;
  uint8_t* dst = slabs + uint32_t(sl) * kSlabBytes + (q >> 2) * kChunkBytes + rb * 128u;
  const float* scales = reinterpret_cast<const float*>(c.scale8) + st * 128 + rb;
  uint4 v[8];
  float sc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    v[e] = *reinterpret_cast<const uint4*>(src + e * 2048);
    sc[e] = scales[16 * e];
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float s = sc[e];
    uint4 lo, hi;
    lo.x = e4m3x2_to_bf16x2(v[e].x, s);
    lo.y = e4m3x2_to_bf16x2(v[e].x >> 16, s);
    lo.z = e4m3x2_to_bf16x2(v[e].y, s);
    lo.w = e4m3x2_to_bf16x2(v[e].y >> 16, s);
    hi.x = e4m3x2_to_bf16x2(v[e].z, s);
    hi.y = e4m3x2_to_bf16x2(v[e].z >> 16, s);
    hi.z = e4m3x2_to_bf16x2(v[e].w, s);
    hi.w = e4m3x2_to_bf16x2(v[e].w >> 16, s);
    uint8_t* row = dst + e * 2048;
    *reinterpret_cast<uint4*>(row + sw0) = lo;
    *reinterpret_cast<uint4*>(row + sw1) = hi;
  }
  mbar_arrive(bar_addr(c, B_SLAB_FULL + sl));
  mbar_arrive(bar_addr(c, B_STAGE_EMPTY + st));
  return true;
}

template <bool kPaged>
__device__ void producer_fp8(const Ctx& c, const SplitParams& prm, int (&raw)[8], int32_t first_row) {
  const int p = threadIdx.x;
  const uint32_t q = uint32_t(p & 7);
  const uint32_t rbase = uint32_t(p >> 3);   // rows rbase + 16 e all have (row & 7) == (rbase & 7)
  const uint32_t kpe_dst = c.sbase + kOffKpe + rbase * 128u + ((q ^ (rbase & 7u)) << 4);
  const uint32_t stage_off = rbase * 128u + q * 16u;
  const uint32_t scale_dst = c.sbase + kOffScale8 + (rbase + 16u * q) * 4u;   // row rbase + 16 q
  const uint8_t* kv = static_cast<const uint8_t*>(prm.kv_fp8);
  const int64_t nslabs = 4 * (c.g_end - c.g_begin);

  bool ok = true;
  uint32_t bad = 0;
  // copy stream: the tile being copied, its rows' slots and the next indices
  int64_t blk = c.g_begin - 1;
  int slot[8];
  uint32_t vmask = 0;
  int slot_q = 0;
  uint32_t valid_q = 0;
  int pg[8], raw_next[8];
  int32_t row_next = 0;
  if constexpr (kPaged) {
    if (c.g_begin < c.g_end) {
      const int64_t rb = row_base(prm, first_row);
#pragma unroll
      for (int e = 0; e < 8; ++e) pg[e] = page_of(prm, rb, raw[e]);
    }
    if (c.g_begin + 1 < c.g_end) {
      load_slots8(prm, c.g_begin + 1, p, raw_next);
      row_next = row_of(prm, (c.g_begin + 1) / kBlocksPerToken);
    }
  }
  // Copies slab u (and, at a tile's first slab, the tile's rope) into the staging ring.
  auto copy_slab = [&](int64_t u) -> bool {
    const int j = int(u & 3);
    if (j == 0) {
      ++blk;
      const int64_t ti = blk - c.g_begin;
      vmask = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int v = raw[e];
        bool valid;
        if constexpr (kPaged) {
          valid = page_valid(prm, pg[e]);
          slot[e] = valid ? pg[e] * kPage + (v & (kPage - 1)) : 0;
        } else {
          valid = v >= 0 && int64_t(v) < prm.num_slots;
          slot[e] = valid ? v : 0;
        }
        bad |= (!valid && v != -1) ? 1u : 0u;
        vmask |= valid ? (1u << e) : 0u;
      }
      if constexpr (kPaged) {
        if (blk + 1 < c.g_end) {
          const int64_t rb = row_base(prm, row_next);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            pg[e] = page_of(prm, rb, raw_next[e]);
            raw[e] = raw_next[e];
          }
          if (blk + 2 < c.g_end) {
            load_slots8(prm, blk + 2, p, raw_next);
            row_next = row_of(prm, (blk + 2) / kBlocksPerToken);
          }
        }
      } else {
        if (blk + 1 < c.g_end) load_slots8(prm, blk + 1, p, raw);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (uint32_t(e) == q) {
          slot_q = slot[e];
          valid_q = (vmask >> e) & 1u;
        }
      // rope: the single kpe buffer, free once the previous tile's rope MMAs retired
      if (ti >= 1 && !group_all<3>(mbar_wait(bar_addr(c, B_KPE_EMPTY), (uint32_t(ti) & 1u) ^ 1u, c.abort,
                                             c.timeout_ns)))
        return false;
      const uint8_t* src0 = kv + kFp8RopeOff + 16 * q;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        cp_async16(kpe_dst + uint32_t(e) * 2048u, src0 + int64_t(slot[e]) * kFp8RowBytes,
                   ((vmask >> e) & 1u) ? 16u : 0u);
      cp_async_arrive_noinc(bar_addr(c, B_KPE_FULL));
    }
    const int st = int(u % kStageSlots);
    if (u >= kStageSlots && !group_all<3>(mbar_wait(bar_addr(c, B_STAGE_EMPTY + st),
                                                    (uint32_t(u / kStageSlots) & 1u) ^ 1u, c.abort, c.timeout_ns)))
      return false;
    const uint32_t dst0 = (st < 2 ? c.sbase + kOffSlab + kRingFp8 * kSlabBytes + uint32_t(st) * kStageBytes
                                  : c.sbase + kOffKpe + kChunkBytes) + stage_off;
    const uint8_t* src0 = kv + 128 * j + 16 * q;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      cp_async16(dst0 + uint32_t(e) * 2048u, src0 + int64_t(slot[e]) * kFp8RowBytes, ((vmask >> e) & 1u) ? 16u : 0u);
    cp_async4(scale_dst + uint32_t(st) * 512u, kv + int64_t(slot_q) * kFp8RowBytes + kFp8ScaleOff + 4 * j,
              valid_q ? 4u : 0u);
    cp_async_arrive_noinc(bar_addr(c, B_STAGE_FULL + st));
    return true;
  };

  for (int64_t u = 0; u < nslabs && ok; ++u) ok = copy_slab(u);
  bad = __any_sync(0xffffffffu, bad);
  if (bad && (p & 31) == 0) report_error(prm.err_word, DSA_DEVICE_ERR_BAD_INDEX);
  // Every copy must land before the CTA exits (also on an abort).
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Softmax warps, FP8 mode: tile i's four staged slabs.
__device__ __forceinline__ bool convert_tile_fp8(const Ctx& c, int64_t i, int r) {
#pragma unroll 1
  for (int j = 0; j < 4; ++j)
    if (!convert_slab_fp8(c, 4 * i + j, r)) return false;
  return true;
}

// -------------------------------------------------------------------------
// warps 4,5 (lane 0): logits MMAs.  Issuer q accumulates the chunks c with
// c % 2 == q (ckv chunks 0..7; issuer 0 also the kpe chunk) into its own
// partial S^T, so the two halves of the 36 dependent MMAs run in parallel.
// (One thread issues a tcgen05.mma about every 130 cycles whatever the
// accumulator, so the issue is spread over warps.)
// -------------------------------------------------------------------------
template <int kRing, int kKpeRing>
__device__ void qk_issuer(const Ctx& c, const int q, const CUtensorMap* tm_qn, const CUtensorMap* tm_qp) {
  const uint32_t sQ = c.sbase + kOffQ, sKpe = c.sbase + kOffKpe, sSlab = c.sbase + kOffSlab;
  constexpr uint32_t idesc_qk = idesc_bf16_f32(128, 16, false, false);
  auto wait = [&](int b, uint32_t parity) { return mbar_wait(bar_addr(c, b), parity, c.abort, c.timeout_ns); };
  int64_t i = 0;
  int seg = 0;
  int last_q = -1;
  bool ok = true;
  for (int64_t gs = c.g_begin; gs < c.g_end && ok;) {
    const int64_t t = gs / kBlocksPerToken;
    const int64_t ge = min(c.g_end, (t + 1) * kBlocksPerToken);
    // Issuer 0 loads the segment's queries (Q^T, 16 heads x 576, 9 swizzled
    // 64-column chunks) once both issuers' MMAs of the previous segment are done.
    if (q == 0) {
      if (seg > 0 && !(ok = wait(B_Q_EMPTY, uint32_t(seg - 1) & 1u))) break;
      const uint32_t qb = bar_addr(c, B_Q_FULL);
      mbar_arrive_expect_tx(qb, kQBytes);
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) tma_load_2d(sQ + ch * kQChunkBytes, tm_qn, 64 * ch, int(t * kHeads), qb);
      tma_load_2d(sQ + 8 * kQChunkBytes, tm_qp, 0, int(t * kHeads), qb);
      last_q = seg;
    }
    if (!(ok = wait(B_Q_FULL, uint32_t(seg) & 1u))) break;
    for (int64_t blk = gs; blk < ge && ok; ++blk, ++i) {
      const int sb = int(i & 1);
      if (i >= 2 && !(ok = wait(B_S_EMPTY + sb, (uint32_t(i >> 1) & 1u) ^ 1u))) break;
      const uint32_t d = c.tmem + 32u * uint32_t(sb) + 16u * uint32_t(q);
      uint32_t acc = 0;
      if (q == 0) {
        const int kb = int(i % kKpeRing);
        if (!(ok = wait(B_KPE_FULL + kb, uint32_t(i / kKpeRing) & 1u))) break;
        fence_proxy_async_smem();   // cp.async data -> tensor-core reads
        tc_fence_after();
        const uint32_t a0 = sKpe + kb * kChunkBytes, b0 = sQ + 8 * kQChunkBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16(d, make_desc(a0 + 32 * kk, kLboKMajor), make_desc(b0 + 32 * kk, kLboKMajor), idesc_qk, acc);
          acc = 1;
        }
        mma_commit(bar_addr(c, B_KPE_EMPTY + kb));
      }
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
        const int64_t u = 4 * i + j;
        const int sl = int(u % kRing);
        if (!(ok = wait(B_SLAB_FULL + sl, uint32_t(u / kRing) & 1u))) break;
        fence_proxy_async_smem();
        tc_fence_after();
        const uint32_t a0 = sSlab + sl * kSlabBytes + uint32_t(q) * kChunkBytes;
        const uint32_t b0 = sQ + (2 * j + q) * kQChunkBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          mma_bf16(d, make_desc(a0 + 32 * kk, kLboKMajor), make_desc(b0 + 32 * kk, kLboKMajor), idesc_qk, acc);
          acc = 1;
        }
      }
      if (!ok) break;
      mma_commit(bar_addr(c, B_S_FULL + sb));
      if (blk + 1 == ge) mma_commit(bar_addr(c, B_Q_EMPTY));
    }
    ++seg;
    gs = ge;
  }
  mma_commit(bar_addr(c, B_DONE + q));
  drain_wait(bar_addr(c, B_DONE + q), 0u, c.drain_ns);
  // the last query load must have landed before the CTA exits (also on an abort)
  if (last_q >= 0) drain_wait(bar_addr(c, B_Q_FULL), uint32_t(last_q) & 1u, c.drain_ns);
}

// -------------------------------------------------------------------------
// warps 6,7 (lane 0): PV MMAs.  Issuer v owns O blocks j = 2v, 2v+1 (dims
// 128j .. 128j+127):  O^T[j] += V^T[tile, j] . P^T[tile], releasing slab j
// as soon as its 8 MMAs retire.  (Issuing the two blocks from two lanes of
// the warp was measured no faster: the lanes' MMAs issue one after another.)
// -------------------------------------------------------------------------
template <int kRing>
__device__ void pv_issuer(const Ctx& c, const int v) {
  const uint32_t sSlab = c.sbase + kOffSlab, sP = c.sbase + kOffP;
  constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 16, true, false);
  auto wait = [&](int b, uint32_t parity) { return mbar_wait(bar_addr(c, b), parity, c.abort, c.timeout_ns); };
  int64_t i = 0;
  int seg = 0;
  bool ok = true;
  for (int64_t gs = c.g_begin; gs < c.g_end && ok;) {
    const int64_t t = gs / kBlocksPerToken;
    const int64_t ge = min(c.g_end, (t + 1) * kBlocksPerToken);
    for (int64_t blk = gs; blk < ge && ok; ++blk, ++i) {
      const int pb = int(i & 1);
      const bool first = (blk == gs);
      if (!(ok = wait(B_P_FULL + pb, uint32_t(i >> 1) & 1u))) break;
      if (first && seg > 0 && !(ok = wait(B_O_EMPTY, uint32_t(seg - 1) & 1u))) break;
      fence_proxy_async_smem();
      tc_fence_after();
      const uint32_t b_base = sP + pb * kPBytes;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = 2 * v + jj;
        const int sl = int((4 * i + j) % kRing);
        const uint32_t a_base = sSlab + sl * kSlabBytes;
        const uint32_t d = c.tmem + kTmemO + 16u * j;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = make_desc(a_base + 2048u * kk, kLboPV);
          const uint64_t b = make_desc(b_base + (kk >> 2) * 2048u + (kk & 3) * 32u, kLboKMajor);
          mma_bf16(d, a, b, idesc_pv, (first && kk == 0) ? 0u : 1u);
        }
        mma_commit(bar_addr(c, B_SLAB_EMPTY + sl));
      }
      mma_commit(bar_addr(c, B_P_EMPTY + pb));
      if (blk + 1 == ge) mma_commit(bar_addr(c, B_O_FULL));
    }
    ++seg;
    gs = ge;
  }
  mma_commit(bar_addr(c, B_DONE + 2 + v));
  drain_wait(bar_addr(c, B_DONE + 2 + v), 0u, c.drain_ns);
}

// -------------------------------------------------------------------------
// warps 8..11: softmax + epilogue
// -------------------------------------------------------------------------
// 2^x with the hardware approximation (MUFU.EX2, ~2 ulp); 2^-inf = 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// log2(x) with the hardware approximation (MUFU.LG2).
__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Per-head max of 16 values over the 32 lanes of a warp in 16 shuffles: each
// step halves the heads a lane carries; lane l ends with head (l >> 1) & 15.
__device__ __forceinline__ float warp_head_max(const float (&v)[16], int lane) {
  float a[8], b[4], d[2];
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4, h2 = lane & 2;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float send = h16 ? v[k] : v[k + 8];
    const float keep = h16 ? v[k + 8] : v[k];
    a[k] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float send = h8 ? a[k] : a[k + 4];
    const float keep = h8 ? a[k + 4] : a[k];
    b[k] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const float send = h4 ? b[k] : b[k + 2];
    const float keep = h4 ? b[k + 2] : b[k];
    d[k] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  const float send = h2 ? d[0] : d[1];
  const float keep = h2 ? d[1] : d[0];
  float m = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 2));
  return fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
}

__device__ __forceinline__ float warp_head_sum(const float (&v)[16], int lane) {
  float a[8], b[4], d[2];
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4, h2 = lane & 2;
#pragma unroll
  for (int k = 0; k < 8; ++k) a[k] = (h16 ? v[k + 8] : v[k]) + __shfl_xor_sync(0xffffffffu, h16 ? v[k] : v[k + 8], 16);
#pragma unroll
  for (int k = 0; k < 4; ++k) b[k] = (h8 ? a[k + 4] : a[k]) + __shfl_xor_sync(0xffffffffu, h8 ? a[k] : a[k + 4], 8);
#pragma unroll
  for (int k = 0; k < 2; ++k) d[k] = (h4 ? b[k + 2] : b[k]) + __shfl_xor_sync(0xffffffffu, h4 ? b[k] : b[k + 2], 4);
  float s = (h2 ? d[1] : d[0]) + __shfl_xor_sync(0xffffffffu, h2 ? d[0] : d[1], 2);
  return s + __shfl_xor_sync(0xffffffffu, s, 1);
}

// Merge of a token split over CTAs b_lo .. b_lo+nseg-1 (the split-KV combine
// of the reference's last-arrival reduce, solution/cuda/kernel.cu:433-509, in
// the log2 domain):
//   M = max_s m_s,  w_s = 2^(m_s - M),  L = sum_s w_s l_s,
//   out = sum_s w_s o_s / L  (0 if L == 0),  lse = M + log2 L  (-inf if L == 0).
// Run by the 128 softmax threads of the last-arriving CTA after every other
// segment has published its record (whose address the caller has put in the
// scratch's record table); thread r owns dims 128 j + r (the TMEM
// lane layout of O), so a segment's 16 heads of one dim are 4 float4 loads
// (record o rows are chunk-swizzled, see record_chunk).  This CTA's own
// segment comes from TMEM (o) and registers (m_own, l_own).  Segments are
// always combined in index order, so the result does not depend on which CTA
// merges (bitwise deterministic).
// With `staged` (the CTA has no tiles left, so its slab and kpe rings are
// idle, and at most kMaxStaged other segments) the other records have been
// copied whole into the slab ring (stage_records), the 16 x 512 bf16 output
// tile is assembled in the kpe ring and leaves with one bulk store.
// Otherwise the records are read from global memory (L2) directly.
// Returns false if a wait gave up (the caller stops).
__device__ __forceinline__ bool merge_token(const Ctx& c, const SplitParams& prm, int64_t t, int64_t b_lo, int nseg,
                                            int r, const float (&m_own)[16], const float (&l_own)[16],
                                            uint32_t t_lane, bool staged) {
  float* w_s = reinterpret_cast<float*>(c.merge);   // weights [16 segments][16 heads]
  float* inv_s = w_s + 16 * 16;                      // 1/L per head
  const int self = int(blockIdx.x - b_lo);
  const float* stage = reinterpret_cast<const float*>(c.merge_stage);
  const float* const* rec_s = reinterpret_cast<const float* const*>(c.merge + (kOffMergeRec - kOffMerge));
  auto rec_of = [&](int sg) -> const float* { return rec_s[sg]; };
  // record of segment sg != self: its stage slot (segments in order, self skipped) or global memory
  auto src_of = [&](int sg) -> const float* {
    return staged ? stage + (sg < self ? sg : sg - 1) * kRecordFloats : rec_of(sg);
  };
  if (staged) {
    // A CTA stages at most once (only its last segment can), so the barrier's phase is 0.
    const uint32_t bar = bar_addr(c, B_MERGE);
    if (!group_all<2>(mbar_wait(bar, 0u, c.abort, c.timeout_ns))) {
      if (r == 0) drain_wait(bar, 0u, c.drain_ns);   // no copy may still write shared memory at exit
      return false;
    }
  }
  // Statistics: 8 lanes per head (head r / 8 of the 16, segments r % 8 and
  // r % 8 + 8), butterfly max and sum over the 8 lanes.
  {
    const int h = r >> 3, s0 = r & 7;
    float mo = -INFINITY, lo = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k)
      if (k == h) {
        mo = m_own[k];
        lo = l_own[k];
      }
    float ms[2], ls[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int sg = s0 + 8 * e;
      ms[e] = -INFINITY;
      ls[e] = 0.f;
      if (sg < nseg) {
        ms[e] = (sg == self) ? mo : src_of(sg)[h];
        ls[e] = (sg == self) ? lo : src_of(sg)[kHeads + h];
      }
    }
    float M = fmaxf(ms[0], ms[1]);
#pragma unroll
    for (int x = 1; x < 8; x <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
    float L = 0.f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int sg = s0 + 8 * e;
      const float w = (M == -INFINITY || sg >= nseg) ? 0.f : fast_exp2(ms[e] - M);
      if (sg < nseg) w_s[sg * 16 + h] = w;
      L += w * ls[e];
    }
#pragma unroll
    for (int x = 1; x < 8; x <<= 1) L += __shfl_xor_sync(0xffffffffu, L, x);
    if (s0 == 0) {
      inv_s[h] = L > 0.f ? 1.f / L : 0.f;
      prm.lse[t * kHeads + h] = L > 0.f ? M + fast_log2(L) : -INFINITY;
    }
  }
  named_barrier_sync(1, kSoftmaxThreads);
  const float4* w4 = reinterpret_cast<const float4*>(w_s);
  __nv_bfloat16* out_g = static_cast<__nv_bfloat16*>(prm.output) + t * (kHeads * kCkv);
  const uint32_t out_s = smem_u32(c.merge_out);
  // one segment's 16 heads of dim d, weighted, into acc
  auto accumulate = [&](int sg, int d, const float (&vo)[16], float (&acc)[16]) {
    float v[16];
    if (sg == self) {
#pragma unroll
      for (int h = 0; h < 16; ++h) v[h] = vo[h];
    } else {
      const float* row = src_of(sg) + 2 * kHeads + d * kHeads;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 x = *reinterpret_cast<const float4*>(row + 4 * record_chunk(d, q));
        v[4 * q] = x.x;
        v[4 * q + 1] = x.y;
        v[4 * q + 2] = x.z;
        v[4 * q + 3] = x.w;
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 w = w4[sg * 4 + q];
      acc[4 * q] += w.x * v[4 * q];
      acc[4 * q + 1] += w.y * v[4 * q + 1];
      acc[4 * q + 2] += w.z * v[4 * q + 2];
      acc[4 * q + 3] += w.w * v[4 * q + 3];
    }
  };
  // staged, nseg = N (2..kMaxStaged+1): the segments' data are selected, not branched on
  auto accumulate_n = [&](auto n_tag, int d, const float (&vo)[16], float (&acc)[16]) {
    constexpr int N = decltype(n_tag)::value;
#pragma unroll
    for (int sg = 0; sg < N; ++sg) {
      // (this CTA's own segment reads stage slot 0 and discards it)
      const float* row = stage + (sg < self ? sg : (sg > self ? sg - 1 : 0)) * kRecordFloats + 2 * kHeads + d * kHeads;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 x = *reinterpret_cast<const float4*>(row + 4 * record_chunk(d, q));
        const float4 w = w4[sg * 4 + q];
        acc[4 * q] += w.x * ((sg == self) ? vo[4 * q] : x.x);
        acc[4 * q + 1] += w.y * ((sg == self) ? vo[4 * q + 1] : x.y);
        acc[4 * q + 2] += w.z * ((sg == self) ? vo[4 * q + 2] : x.z);
        acc[4 * q + 3] += w.w * ((sg == self) ? vo[4 * q + 3] : x.w);
      }
    }
  };
#pragma unroll 1
  for (int j = 0; j < 4; ++j) {
    const int d = 128 * j + r;
    float vo[16], acc[16];
    tmem_ld16(c.tmem + t_lane + kTmemO + 16u * j, vo);
    tmem_wait_ld();
#pragma unroll
    for (int h = 0; h < 16; ++h) acc[h] = 0.f;
    if (staged) {
      switch (nseg) {   // fully unrolled per segment count: all loads issue together
        case 2: accumulate_n(std::integral_constant<int, 2>(), d, vo, acc); break;
        case 3: accumulate_n(std::integral_constant<int, 3>(), d, vo, acc); break;
        case 4: accumulate_n(std::integral_constant<int, 4>(), d, vo, acc); break;
        default: accumulate_n(std::integral_constant<int, 5>(), d, vo, acc); break;
      }
      uint16_t ob[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const __nv_bfloat16 b = __float2bfloat16_rn(acc[h] * inv_s[h]);
        ob[h] = *reinterpret_cast<const uint16_t*>(&b);
      }
#pragma unroll
      for (int h = 0; h < 16; ++h)
        asm volatile("st.shared.b16 [%0], %1;" ::"r"(out_s + 2u * uint32_t(h * kCkv + d)), "h"(ob[h]));
    } else {
      for (int sg = 0; sg < nseg; ++sg) accumulate(sg, d, vo, acc);
#pragma unroll
      for (int h = 0; h < 16; ++h) out_g[h * kCkv + d] = __float2bfloat16_rn(acc[h] * inv_s[h]);
    }
  }
  if (staged) {
    fence_proxy_async_smem();   // the tile, now read by the TMA engine
    named_barrier_sync(1, kSoftmaxThreads);
    if (r == 0) {
      bulk_store(out_g, out_s, uint32_t(kHeads * kCkv * 2));
      bulk_commit();
      bulk_wait_read_all();     // the kpe ring must not be left while the copy reads it
    }
  }
  named_barrier_sync(1, kSoftmaxThreads);   // scratch is reused by the next merge
  return true;
}

// Leader of a staged merge: copies each other segment's record into the slab
// ring (segments in order, self skipped) with one TMA bulk copy as soon as the
// segment's publication bit appears in the ticket counter, so that the copies
// of the records published early overlap the wait for the last one.  Bounded
// like wait_published.  B_MERGE (phase 0) completes once every issued copy has
// landed, also after a give-up, so that the caller can drain it.
__device__ __forceinline__ bool stage_records(const Ctx& c, const SplitParams& prm, const uint32_t* counter,
                                              uint32_t others, int self, int64_t b_lo, int64_t t) {
  const uint32_t bar = bar_addr(c, B_MERGE);
  const float* stage = reinterpret_cast<const float*>(c.merge_stage);
  uint32_t issued = 0;
  uint64_t t0 = 0;
  bool ok = true;
  for (uint32_t spins = 0;; ++spins) {
    const uint32_t fresh = (ld_acquire(counter) >> 16) & others & ~issued;
    if (fresh) {
      fence_proxy_async_global();   // the acquired records, now read by the TMA engine
      for (uint32_t m = fresh; m; m &= m - 1u) {
        const int sg = __ffs(int(m)) - 1;
        const float* src = prm.records + plan_record_slot(prm.plan, b_lo + sg, t) * kRecordFloats;
        mbar_expect_tx(bar, uint32_t(kRecordBytes));
        bulk_load(smem_u32(stage + (sg < self ? sg : sg - 1) * kRecordFloats), src, uint32_t(kRecordBytes), bar);
      }
      issued |= fresh;
      if (issued == others) break;
    }
    if (*c.abort) {
      ok = false;
      break;
    }
    if (spins == 0) {
      t0 = globaltimer_ns();
    } else if (globaltimer_ns() - t0 > c.timeout_ns) {
      *c.abort = 1u;
      ok = false;
      break;
    }
    __nanosleep(32);
  }
  mbar_arrive(bar);
  return ok;
}

// ---------------------------------------------------------------------------
// Merge of a token split over many CTAs (more than kMaxStaged + 1).  One CTA
// would have to pull every other record (32 KB each) into its SM; instead
// every segment publishes its record and the work is shared: the output is
// cut into kChunks chunks of 64 dims x 16 heads, and each CTA whose range
// ends inside the token (a "helper") waits for every record, claims its
// preferred chunks (c % helpers == its rank) on the token's claim word with
// atomicOr and writes them with all its threads, reading the records from L2.
// The segment that arrived last waits under the pipeline limit (every other
// segment has arrived, so it is running and publishes without waiting on
// anything) and then also claims and writes whatever is left; another helper
// waits at most kHelpWindowNs and otherwise leaves its chunks to it.  The
// combine is the one of merge_token, in segment order, so the result does not
// depend on which CTA writes a chunk (bitwise deterministic).
// ---------------------------------------------------------------------------
constexpr uint64_t kHelpWindowNs = 20000;

// Claims the chunks in `want` of token t on the token's claim word and writes
// those it wins (all kThreads threads of the CTA, whose slab ring is idle).
// Per chunk, every thread copies its share of the chunk's 4 KB of each record
// (and, with the first chunk, each record's statistics) into the ring with
// 16-byte cp.async, all at once, so the chunk arrives in about one L2 round
// trip; the sums then read shared memory.  The first wanted chunk is copied
// while the claim is in flight: the records are all published, and a chunk
// that another CTA wins is copied for nothing and not written.
__device__ void claim_and_merge(const Ctx& c, const SplitParams& prm, int64_t t, int64_t b_lo, int nseg,
                                uint32_t want, uint32_t* claim_word) {
  const int tid = threadIdx.x;
  float* w_s = reinterpret_cast<float*>(c.merge);                                     // [segment][head]
  float* inv_s = w_s + 256;                                                            // [head]
  const float** rec = reinterpret_cast<const float**>(c.merge + (kOffMergeRec - kOffMerge));
  volatile uint32_t* flag = c.merge_flag;
  uint8_t* const ring = c.merge_stage;
  const uint32_t ring_s = smem_u32(ring);
  constexpr uint32_t kStatOff = 0, kDataOff = 16 * 128;   // stats [16][128 B], then records' chunk [16][4 KB]
  if (tid < nseg) rec[tid] = prm.records + plan_record_slot(prm.plan, b_lo + tid, t) * kRecordFloats;
  __syncthreads();
  // 256 pieces of 16 B per record (its rows of chunk ch), then 8 per record of statistics
  auto stage = [&](int ch, bool stats) {
    const int pieces = nseg * 256 + (stats ? nseg * 8 : 0);
    for (int j = tid; j < pieces; j += kThreads) {
      if (j < nseg * 256) {
        const int sg = j >> 8, pc = j & 255;
        cp_async16(ring_s + kDataOff + uint32_t(sg) * 4096u + uint32_t(pc) * 16u,
                   rec[sg] + 2 * kHeads + ch * kChunkDims * kHeads + 4 * pc, 16u);
      } else {
        const int k = j - nseg * 256, sg = k >> 3, pc = k & 7;
        cp_async16(ring_s + kStatOff + uint32_t(sg) * 128u + uint32_t(pc) * 16u, rec[sg] + 4 * pc, 16u);
      }
    }
  };
  const int c0 = __ffs(int(want)) - 1;
  stage(c0, true);
  if (tid == 0) *flag = want & ~atomicOr(claim_word, want);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const uint32_t mine = *flag;
  if (mine == 0u) return;   // the caller's barrier follows before the flag is reused
  // statistics: thread (head h, segment lane s) for the first 256 threads;
  // max and sum over the 16 lanes of a head with shuffles
  if (tid < 256) {
    const int h = tid >> 4, sg = tid & 15;
    const float* st = reinterpret_cast<const float*>(ring + kStatOff + (sg < nseg ? sg : 0) * 128);
    const float m = sg < nseg ? st[h] : -INFINITY;
    float M = m;
#pragma unroll
    for (int x = 8; x >= 1; x >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
    const float w = (M == -INFINITY || sg >= nseg) ? 0.f : fast_exp2(m - M);
    w_s[sg * 16 + h] = w;
    float L = sg < nseg ? w * st[kHeads + h] : 0.f;
#pragma unroll
    for (int x = 8; x >= 1; x >>= 1) L += __shfl_xor_sync(0xffffffffu, L, x);
    if (sg == 0) {
      inv_s[h] = L > 0.f ? 1.f / L : 0.f;
      if (mine & 1u) prm.lse[t * kHeads + h] = L > 0.f ? M + fast_log2(L) : -INFINITY;
    }
  }
  __syncthreads();
  __nv_bfloat16* out_t = static_cast<__nv_bfloat16*>(prm.output) + t * (kHeads * kCkv);
  bool in_ring = true;   // chunk c0 is in the ring
#pragma unroll 1
  for (uint32_t left = mine; left; left &= left - 1u) {
    const int ch = __ffs(int(left)) - 1;
    if (!(in_ring && ch == c0)) {
      stage(ch, false);
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncthreads();
    }
    in_ring = false;
    // items: (dim, 4-head piece), consecutive threads on consecutive dims
    for (int i = tid; i < kChunkDims * 4; i += kThreads) {
      const int dl = i & 63, q = i >> 6;
      const int d = ch * kChunkDims + dl;
      const uint8_t* src = ring + kDataOff + uint32_t(dl) * 64u + 16u * uint32_t(record_chunk(d, q));
      float4 x[16];
#pragma unroll
      for (int sg = 0; sg < 16; ++sg)
        if (sg < nseg) x[sg] = *reinterpret_cast<const float4*>(src + uint32_t(sg) * 4096u);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sg = 0; sg < 16; ++sg)
        if (sg < nseg) {
          const float4 w = *reinterpret_cast<const float4*>(w_s + sg * 16 + 4 * q);
          acc.x += w.x * x[sg].x;
          acc.y += w.y * x[sg].y;
          acc.z += w.z * x[sg].z;
          acc.w += w.w * x[sg].w;
        }
      const float4 iv = *reinterpret_cast<const float4*>(inv_s + 4 * q);
      __nv_bfloat16* o = out_t + (4 * q) * kCkv + d;
      o[0] = __float2bfloat16_rn(acc.x * iv.x);
      o[kCkv] = __float2bfloat16_rn(acc.y * iv.y);
      o[2 * kCkv] = __float2bfloat16_rn(acc.z * iv.z);
      o[3 * kCkv] = __float2bfloat16_rn(acc.w * iv.w);
    }
    __syncthreads();   // the staged chunk is read: the next one may be copied over it
  }
}

// The merge work of a helper (all kThreads threads): wait for every record of
// the token, then claim and write chunks.  Returns false only when a wait of
// the last arrival gave up (the abort is raised).
__device__ bool help_merge(const Ctx& c, const SplitParams& prm, const HelpTask& task) {
  const int tid = threadIdx.x;
  uint32_t* word = prm.counters + 2 * (task.b_lo + 1);
  volatile uint32_t* flag = c.merge_flag;
  if (tid == 0) {
    const uint32_t all = (1u << task.nseg) - 1u;
    const uint64_t limit = task.last ? c.timeout_ns : min(c.timeout_ns, kHelpWindowNs);
    *flag = wait_published(word, all, c.abort, limit, task.last != 0u) ? 1u : 0u;
  }
  __syncthreads();
  const bool all_published = *flag != 0u;
  __syncthreads();                         // everyone has read the flag before it is reused
  if (!all_published) return task.last == 0u;   // a helper leaves its chunks to the last arrival
  // its preferred chunks
  if (task.pref) claim_and_merge(c, prm, task.t, task.b_lo, task.nseg, task.pref, word + 1);
  __syncthreads();                         // the flag and the scratch are reused
  if (task.last) {
    // then (the last arrival only) the chunks nobody has claimed yet
    if (tid == 0) *flag = ~ld_acquire(word + 1) & ((1u << kChunks) - 1u);
    __syncthreads();
    const uint32_t rest = *flag;
    __syncthreads();
    if (rest) claim_and_merge(c, prm, task.t, task.b_lo, task.nseg, rest, word + 1);
    __syncthreads();
  }
  return true;
}

// Runs a helper's merge work (help_merge), then closes the books on the
// token's counter pair: a helper that did not arrive last counts itself as
// finished (whether it wrote chunks or left them); the last arrival waits,
// bounded, until every other helper has finished — they are running, so they
// do within their window — and then resets the pair for the next call, when
// nothing touches it any more.
__device__ void finish_help(const Ctx& c, const SplitParams& prm, const HelpTask& task, bool is_helper) {
  const bool ok = help_merge(c, prm, task);
  if (threadIdx.x != 0) return;
  uint32_t* word = prm.counters + 2 * (task.b_lo + 1);
  if (!task.last) {
    atomicAdd(word + 1, 1u << 16);
    return;
  }
  if (!ok) return;   // the abort is raised; the error report makes the host clear the counters
  const uint32_t others = uint32_t(task.helpers - (is_helper ? 1 : 0));
  uint64_t t0 = 0;
  for (uint32_t spins = 0;; ++spins) {
    if ((ld_acquire(word + 1) >> 16) >= others) break;
    if (*c.abort) return;
    if (spins == 0) {
      t0 = globaltimer_ns();
    } else if (globaltimer_ns() - t0 > c.timeout_ns) {
      *c.abort = 1u;
      return;
    }
    __nanosleep(64);
  }
  word[0] = 0u;
  word[1] = 0u;
}

template <bool kPaged, bool kFp8>
__device__ void softmax_epilogue(const Ctx& c, const SplitParams& prm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wq = warp & 3;              // TMEM lanes 32*wq .. 32*wq+31 belong to this warp
  const int r = 32 * wq + lane;         // key row of a tile / dim row of an O block
  const int my_head = (lane >> 1) & 15; // head this lane holds after a warp reduction
  const uint32_t t_lane = uint32_t(32 * wq) << 16;
  const bool leader = (warp == kSoftmaxWarp0 && lane == 0);
  const uint32_t sP = c.sbase + kOffP;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(prm.output);
  // P^T store address pieces for key r: 64-key chunk, swizzled 16-B group, byte in group
  const uint32_t p_kc = uint32_t(r >> 6) * 2048u, p_grp = uint32_t((r & 63) >> 3), p_byte = uint32_t(r & 7) << 1;

  if (prm.hold != nullptr) {
    // test hook of the timeout path: a wait for a flag that nothing sets runs
    // out at the pipeline limit and raises the abort (the other roles' waits
    // then give up and drain)
    const bool got = leader ? wait_published(prm.hold, 1u, c.abort, c.timeout_ns) : true;
    if (!group_all<1>(got)) return;
  }
  int64_t i = 0;
  int seg = 0;
  bool ok = true;
  for (int64_t gs = c.g_begin; gs < c.g_end && ok;) {
    const int64_t t = gs / kBlocksPerToken;
    const int64_t ge = min(c.g_end, (t + 1) * kBlocksPerToken);
    const bool full = (gs == t * kBlocksPerToken) && (ge == (t + 1) * kBlocksPerToken);
    // CTAs b_lo .. b_lo+nseg-1 share a split token; computed here (64-bit
    // divisions) so that they are ready when the segment ends
    int64_t b_lo = full ? 0 : plan_owner(prm.plan, t * kBlocksPerToken);
    int64_t b_hi = full ? 0 : plan_owner(prm.plan, t * kBlocksPerToken + kBlocksPerToken - 1);
    asm volatile("" : "+l"(b_lo), "+l"(b_hi));
    const int nseg = int(b_hi - b_lo + 1);
    float m_run[16], l_part[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      m_run[h] = -INFINITY;
      l_part[h] = 0.f;
    }
    // Validity of this thread's key in each tile (the producer gathers the
    // same rows; a masked key gets logit -inf).  Slot mode: the slot id, one
    // tile ahead.  Paged mode: positions two tiles ahead, pages one ahead.
    const int32_t* key_row = prm.indices + t * kTopk + r;
    int32_t kidx_next = __ldg(key_row + (gs % kBlocksPerToken) * kBlockKeys);
    int64_t rbase = 0;
    int32_t pos_next = -1;
    if constexpr (kPaged) {
      rbase = row_base(prm, row_of(prm, t));
      kidx_next = page_of(prm, rbase, kidx_next);   // now the page of the first tile's key
      if (gs + 1 < ge) pos_next = __ldg(key_row + ((gs + 1) % kBlocksPerToken) * kBlockKeys);
    }
    for (int64_t blk = gs; blk < ge; ++blk, ++i) {
      const int32_t kidx = kidx_next;
      bool valid;
      if constexpr (kPaged) {
        valid = page_valid(prm, kidx);
        if (blk + 1 < ge) {
          kidx_next = page_of(prm, rbase, pos_next);
          if (blk + 2 < ge) pos_next = __ldg(key_row + ((blk + 2) % kBlocksPerToken) * kBlockKeys);
        }
      } else {
        if (blk + 1 < ge) kidx_next = __ldg(key_row + ((blk + 1) % kBlocksPerToken) * kBlockKeys);
        valid = kidx >= 0 && int64_t(kidx) < prm.num_slots;
      }
      if constexpr (kFp8) {
        if (!(ok = convert_tile_fp8(c, i, r))) break;
      }
      const int sb = int(i & 1);
      // A failed (timed-out) wait never skips a barrier: the thread carries on
      // with dummy data and the vote on the reduction barrier below stops all.
      const bool s_ok = mbar_wait(bar_addr(c, B_S_FULL + sb), uint32_t(i >> 1) & 1u, c.abort, c.timeout_ns);
      float x[16];
      if (s_ok) {
        float x1[16];
        tc_fence_after();
        tmem_ld16(c.tmem + t_lane + 32u * uint32_t(sb), x);
        tmem_ld16(c.tmem + t_lane + 32u * uint32_t(sb) + 16u, x1);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(bar_addr(c, B_S_EMPTY + sb));
#pragma unroll
        for (int h = 0; h < 16; ++h) x[h] += x1[h];
      }
#pragma unroll
      for (int h = 0; h < 16; ++h) x[h] = (valid && s_ok) ? x[h] * prm.scale_log2 : -INFINITY;
      // Fast path: while no key of the tile exceeds a head's reference max by
      // more than the threshold, p = 2^(x - m_run) stays below 2^8 and the
      // reference max is kept, so the tile max is not needed at all.  One vote
      // (which also catches a failed S wait) decides; otherwise the per-head
      // tile max is reduced over the 128 keys and the reference max moves.
      bool exceed = !s_ok;
#pragma unroll
      for (int h = 0; h < 16; ++h) exceed |= x[h] > m_run[h] + kRescaleThreshold;
      float alpha[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) alpha[h] = 1.f;
      bool any_rescale = false;
      if (group_any<1>(exceed)) {
        float* red = c.red + sb * 64;
        {
          const float wm = warp_head_max(x, lane);
          if ((lane & 1) == 0) red[wq * 16 + my_head] = wm;
        }
        if (!(ok = group_all<1>(s_ok))) break;   // also the barrier that publishes red[]
        float mx[16];
#pragma unroll
        for (int h = 0; h < 16; h += 4) {
          float4 a = *reinterpret_cast<const float4*>(red + h);
#pragma unroll
          for (int w = 1; w < 4; ++w) {
            const float4 b = *reinterpret_cast<const float4*>(red + w * 16 + h);
            a.x = fmaxf(a.x, b.x);
            a.y = fmaxf(a.y, b.y);
            a.z = fmaxf(a.z, b.z);
            a.w = fmaxf(a.w, b.w);
          }
          mx[h] = a.x;
          mx[h + 1] = a.y;
          mx[h + 2] = a.z;
          mx[h + 3] = a.w;
        }
        // branch-free: the reference max of a head moves when its tile max
        // exceeds it by more than the threshold (alpha scales O and l alike,
        // so its rounding cancels in O / l)
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const bool grow = mx[h] > m_run[h] + kRescaleThreshold;
          const bool scale = grow && (m_run[h] != -INFINITY);
          alpha[h] = scale ? fast_exp2(m_run[h] - mx[h]) : 1.f;
          any_rescale |= scale;
          m_run[h] = grow ? mx[h] : m_run[h];
          l_part[h] *= alpha[h];
        }
      }
      if (any_rescale) {
        // O holds the previous tiles of this segment: let their PV retire, then scale in place.
        if (!(ok = group_all<2>(mbar_wait(bar_addr(c, B_P_EMPTY + int((i - 1) & 1)), uint32_t((i - 1) >> 1) & 1u,
                                          c.abort, c.timeout_ns))))
          break;
        tc_fence_after();
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          float o[16];
          tmem_ld16(c.tmem + t_lane + kTmemO + 16u * j, o);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 16; ++h) o[h] *= alpha[h];
          tmem_st16(c.tmem + t_lane + kTmemO + 16u * j, o);
        }
        tmem_wait_st();
      }
      // P buffer sb is free once PV(i-2) retired; on a timeout the next vote stops the group
      if (i >= 2) mbar_wait(bar_addr(c, B_P_EMPTY + sb), (uint32_t(i >> 1) & 1u) ^ 1u, c.abort, c.timeout_ns);
      // P^T (bf16) into the K-major 128-byte-swizzled B operand: row = head, 64 keys per 128-byte row
      {
        const uint32_t base = sP + sb * kPBytes + p_kc;
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float pv = (m_run[h] == -INFINITY) ? 0.f : fast_exp2(x[h] - m_run[h]);
          l_part[h] += pv;
          const uint32_t hr = uint32_t(h & 7);
          const uint32_t addr = base + uint32_t(h >> 3) * 1024u + hr * 128u + (((p_grp ^ hr) << 4) | p_byte);
          const __nv_bfloat16 pb = __float2bfloat16_rn(pv);
          asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(*reinterpret_cast<const uint16_t*>(&pb)) : "memory");
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar_addr(c, B_P_FULL + sb));
    }
    if (!ok) break;

    // ---- segment epilogue ------------------------------------------------
    // A split token's segments take tickets on the token's state word (low 16
    // bits: arrivals, high 16 bits: one bit per published record), drawn now,
    // while PV of the last tile is still in flight.  Over at most
    // kMaxStaged + 1 CTAs, the last arrival merges straight from its TMEM
    // accumulator once the others have published their records; over more,
    // every segment publishes and the CTAs whose ranges end inside the token
    // share the merge at the end of their ranges (help_merge).
    uint32_t* counter = prm.counters + 2 * (b_lo + 1);   // plan_token_counter(prm.plan, t)
    const bool many = nseg - 1 > kMaxStaged;
    uint32_t ticket = 0;
    if (!full && leader && !prm.cluster_merge) ticket = atomicAdd(counter, 1u);
    {
      const float ws = warp_head_sum(l_part, lane);
      if ((lane & 1) == 0) c.red_l[wq * 16 + my_head] = ws;
    }
    named_barrier_sync(1, kSoftmaxThreads);
    float l_tot[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) l_tot[h] = c.red_l[h] + c.red_l[16 + h] + c.red_l[32 + h] + c.red_l[48 + h];
    named_barrier_sync(1, kSoftmaxThreads);   // red_l is rewritten by the next segment
    if (!(ok = group_all<2>(mbar_wait(bar_addr(c, B_O_FULL), uint32_t(seg) & 1u, c.abort, c.timeout_ns)))) break;
    tc_fence_after();
    if (prm.cluster_merge) {
      // The CTA's only segment: its statistics are kept for the merge through
      // distributed shared memory at the end of the CTA (cluster_merge_end).
      if (leader) {
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          c.red[h] = m_run[h];
          c.red[kHeads + h] = l_tot[h];
        }
      }
      break;
    }
    if (full) {
      if (leader) {
#pragma unroll
        for (int h = 0; h < 16; ++h) prm.lse[t * kHeads + h] = l_tot[h] > 0.f ? m_run[h] + log2f(l_tot[h]) : -INFINITY;
      }
      float inv_l[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) inv_l[h] = l_tot[h] > 0.f ? 1.f / l_tot[h] : 0.f;
#pragma unroll 1
      for (int j = 0; j < 4; ++j) {
        float o[16];
        tmem_ld16(c.tmem + t_lane + kTmemO + 16u * j, o);
        tmem_wait_ld();
        __nv_bfloat16* ot = out + t * (kHeads * kCkv) + 128 * j + r;
#pragma unroll
        for (int h = 0; h < 16; ++h) ot[h * kCkv] = __float2bfloat16_rn(o[h] * inv_l[h]);
      }
      tc_fence_before();
      mbar_arrive(bar_addr(c, B_O_EMPTY));
    } else {
      if (leader) *c.merge_flag = ((ticket & 0xffffu) + 1u == uint32_t(nseg)) ? 1u : 0u;
      named_barrier_sync(1, kSoftmaxThreads);
      const bool last = *c.merge_flag == 1u;
      named_barrier_sync(1, kSoftmaxThreads);   // the flag is read before the merger's leader reuses it
      if (last && !many) {
        // last arrival: every other segment has arrived, so it is running and
        // publishes without waiting on anything; wait (bounded) for that,
        // meanwhile fill the record table of the merge.  Staging needs the
        // idle rings of a CTA with no tiles left; the leader then copies each
        // record in as soon as it is published.
        if (r < nseg)
          reinterpret_cast<const float**>(c.merge + (kOffMergeRec - kOffMerge))[r] =
              prm.records + plan_record_slot(prm.plan, b_lo + r, t) * kRecordFloats;
        const bool staged = (ge == c.g_end);
        if (leader) {
          const int self = int(blockIdx.x - b_lo);
          const uint32_t others = ((1u << nseg) - 1u) & ~(1u << self);
          const bool got = staged ? stage_records(c, prm, counter, others, self, b_lo, t)
                                  : wait_published(counter, others, c.abort, c.timeout_ns);
          *c.merge_flag = got ? 1u : 0u;
        }
        named_barrier_sync(1, kSoftmaxThreads);   // the leader's acquire covers the CTA from here
        if (!(ok = (*c.merge_flag == 1u))) {
          if (staged && leader) drain_wait(bar_addr(c, B_MERGE), 0u, c.drain_ns);   // no copy may land after exit
          break;
        }
        if (!(ok = merge_token(c, prm, t, b_lo, nseg, r, m_run, l_tot, t_lane, staged))) break;
        tc_fence_before();
        mbar_arrive(bar_addr(c, B_O_EMPTY));
        if (leader) *counter = 0u;   // every other segment has published: ready for the next call
      } else {
        // With no tiles left the record is assembled in the idle slab ring and
        // leaves with one bulk store; otherwise each thread writes its dims.
        const bool staged = (ge == c.g_end);
        // own record slot: 2b for the CTA's first token, 2b+1 for its last (plan_record_slot)
        float* rec = prm.records + (2 * int64_t(blockIdx.x) + (t == c.g_begin / kBlocksPerToken ? 0 : 1)) * kRecordFloats;
        float* img = staged ? reinterpret_cast<float*>(c.merge_stage) : rec;
#pragma unroll 1
        for (int j = 0; j < 4; ++j) {
          float o[16];
          tmem_ld16(c.tmem + t_lane + kTmemO + 16u * j, o);
          tmem_wait_ld();
          const int d = 128 * j + r;
          float4* row = reinterpret_cast<float4*>(img + 2 * kHeads + d * kHeads);
          row[record_chunk(d, 0)] = make_float4(o[0], o[1], o[2], o[3]);
          row[record_chunk(d, 1)] = make_float4(o[4], o[5], o[6], o[7]);
          row[record_chunk(d, 2)] = make_float4(o[8], o[9], o[10], o[11]);
          row[record_chunk(d, 3)] = make_float4(o[12], o[13], o[14], o[15]);
        }
        tc_fence_before();
        mbar_arrive(bar_addr(c, B_O_EMPTY));
        if (leader) {
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            img[h] = m_run[h];
            img[kHeads + h] = l_tot[h];
          }
        }
        if (staged) fence_proxy_async_smem();   // the image, now read by the TMA engine
        // publish: the barrier orders every thread's record stores before the
        // leader's device-scope fence and count
        named_barrier_sync(1, kSoftmaxThreads);
        if (leader) {
          if (staged) {
            bulk_store(rec, smem_u32(img), uint32_t(kRecordBytes));
            bulk_commit();
            bulk_wait_all();
            fence_proxy_async_global();
          }
          red_release_add(counter, 1u << (16 + int(blockIdx.x - b_lo)));   // this segment's bit
          if (many && (staged || last)) {
            // merge work at the end of the CTA: a helper (segments 0 .. nseg-2
            // end their CTAs' ranges, the last one does when its CTA's range
            // ends with the token) claims its preferred chunks; the last
            // arrival also completes whatever is left
            const int sg = int(blockIdx.x - b_lo);
            const bool hi_helps = plan_range_begin(prm.plan, b_lo + nseg) == (t + 1) * kBlocksPerToken;
            const int helpers = nseg - 1 + (hi_helps ? 1 : 0);
            uint32_t pref = 0;
#pragma unroll
            for (int ch = 0; ch < kChunks; ++ch) pref |= (staged && ch % helpers == sg) ? (1u << ch) : 0u;
            HelpTask* tk = c.task + (staged ? 1 : 0);
            tk->t = t;
            tk->b_lo = b_lo;
            tk->nseg = nseg;
            tk->pref = pref;
            tk->last = last ? 1u : 0u;
            tk->helpers = helpers;
            tk->pending = 1u;
          }
        }
      }
    }
    ++seg;
    gs = ge;
  }
}

// ---------------------------------------------------------------------------
// Small batches: a token over the 16 CTAs of one thread-block cluster (one
// block per CTA; the launcher picks this when every token's cluster can be
// resident at once).  Each CTA's inbox is the fifth slab slot (O: 16
// segments x 32 dims x 16 heads fp32, 32 KB) and the second kpe buffer
// (statistics): with one tile per CTA the bf16 gather never uses them, so
// they may receive the others' data while this CTA still computes; the FP8
// gather stages rows there, so in that mode a cluster barrier first waits
// until every CTA of the token is past its tile.  At the end of the CTA,
// with every thread:
//   1. each CTA stores into every CTA's inbox its segment's statistics (m, l
//      per head), and into CTA k's inbox its O for dims 32 k .. 32 k + 31
//      (16 heads), read from TMEM by the warps of each TMEM lane quarter
//      taking (O block, head half) units; distributed-shared-memory stores,
//      so nothing waits on a round trip;
//   2. cluster barrier (release / acquire): every inbox is complete;
//   3. from its own inbox only: the token's statistics (the combine of
//      merge_token, segments = cluster ranks in order, so every CTA gets the
//      same weights; rank 0 writes lse) and output dims 32 k .. 32 k + 31.
// After step 2 no CTA touches another's memory, so each leaves on its own.
// The barriers are passed by every CTA, also after an abort (each CTA gets
// there once its own bounded waits have run out and its work has drained);
// an aborted CTA's data are not used (the call reports the timeout).
// ---------------------------------------------------------------------------
template <bool kFp8>
__device__ void cluster_merge_end(const Ctx& c, const SplitParams& prm) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = int(cl.block_rank());
  const int64_t t = int64_t(blockIdx.x) / kBlocksPerToken;
  const bool ok = *c.abort == 0u && c.g_begin < c.g_end;
  // inbox: statistics [16 segments][m 16 | l 16]; O [16 segments][32 dims][16 heads]
  float* inbox = reinterpret_cast<float*>(c.merge_out + kChunkBytes);
  float* in_o = reinterpret_cast<float*>(c.merge_stage + 4 * kSlabBytes);
  static_assert(kBlocksPerToken * 32 * kHeads * 4 == kSlabBytes, "a slab slot holds the O inbox");
  if constexpr (kFp8) cl.sync();   // the inbox is the FP8 staging area: every tile is done with it
  if (ok) {
    if (tid < kBlocksPerToken * 8) {   // 16 CTAs x 8 float4 of this segment's (m, l)
      const int k = tid >> 3, e = tid & 7;
      *reinterpret_cast<float4*>(cl.map_shared_rank(inbox, k) + rank * 2 * kHeads + 4 * e) =
          *reinterpret_cast<const float4*>(c.red + 4 * e);
    }
    // this warp's units u = grp, grp + 3, grp + 6 (< 8): loads issued together, one wait
    const int q4 = warp & 3, grp = warp >> 2;
    tc_fence_after();
    float v[3][8];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const int u = grp + 3 * i;
      if (u < 8)
        tmem_ld8(c.tmem + (uint32_t(32 * q4) << 16) + kTmemO + 16u * uint32_t(u >> 1) + 8u * uint32_t(u & 1), v[i]);
    }
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const int u = grp + 3 * i;
      if (u < 8) {
        const int j = u >> 1, hh = u & 1;
        const int k = 4 * j + q4;   // owner of dims 32 k .. 32 k + 31 (this lane: dim 32 k + lane)
        float* dst = cl.map_shared_rank(in_o, k) + (rank * 32 + lane) * kHeads + 8 * hh;
        *reinterpret_cast<float4*>(dst) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
      }
    }
  }
  tc_fence_before();   // this warp's TMEM reads, before the dealloc that follows
  cl.sync();
  if (!ok) return;
  float* w_s = reinterpret_cast<float*>(c.merge);   // weights [segment][head]
  float* inv_s = w_s + 256;                          // 1/L [head]
  if (tid < 256) {
    // thread (head h, segment s): max and sum over the 16 segment lanes
    const int h = tid >> 4, sg = tid & 15;
    const float m = inbox[sg * 2 * kHeads + h], l = inbox[sg * 2 * kHeads + kHeads + h];
    float M = m;
#pragma unroll
    for (int x = 8; x >= 1; x >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
    const float w = M == -INFINITY ? 0.f : fast_exp2(m - M);
    w_s[sg * 16 + h] = w;
    float L = w * l;
#pragma unroll
    for (int x = 8; x >= 1; x >>= 1) L += __shfl_xor_sync(0xffffffffu, L, x);
    if (sg == 0) {
      inv_s[h] = L > 0.f ? 1.f / L : 0.f;
      if (rank == 0) prm.lse[t * kHeads + h] = L > 0.f ? M + fast_log2(L) : -INFINITY;
    }
  }
  __syncthreads();
  if (tid < 128) {
    // thread (dim 32 rank + dl, heads 4 q .. 4 q + 3)
    const int dl = tid & 31, q = tid >> 5;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int sg = 0; sg < kBlocksPerToken; ++sg) {
      const float4 x = *reinterpret_cast<const float4*>(in_o + (sg * 32 + dl) * kHeads + 4 * q);
      const float4 w = *reinterpret_cast<const float4*>(w_s + sg * 16 + 4 * q);
      acc.x += w.x * x.x;
      acc.y += w.y * x.y;
      acc.z += w.z * x.z;
      acc.w += w.w * x.w;
    }
    const float4 iv = *reinterpret_cast<const float4*>(inv_s + 4 * q);
    __nv_bfloat16* o =
        static_cast<__nv_bfloat16*>(prm.output) + t * (kHeads * kCkv) + (4 * q) * kCkv + 32 * rank + dl;
    o[0] = __float2bfloat16_rn(acc.x * iv.x);
    o[kCkv] = __float2bfloat16_rn(acc.y * iv.y);
    o[2 * kCkv] = __float2bfloat16_rn(acc.z * iv.z);
    o[3 * kCkv] = __float2bfloat16_rn(acc.w * iv.w);
  }
}

template <bool kPaged, bool kFp8>
__global__ void __launch_bounds__(kThreads, 1)
    split_sm100_kernel(const __grid_constant__ CUtensorMap tm_qn, const __grid_constant__ CUtensorMap tm_qp,
                       const SplitParams prm, const uint64_t timeout_ns) {
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base, derived by pointer arithmetic on the shared array
  // so that the compiler keeps every access through it in the shared window
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Ctx c;
  c.sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  c.abort = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc + 4);
  c.red = reinterpret_cast<float*>(smem + kOffRed);
  c.red_l = reinterpret_cast<float*>(smem + kOffRedL);
  c.merge_flag = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc + 8);
  c.merge = smem + kOffMerge;
  c.task = reinterpret_cast<HelpTask*>(smem + kOffTask);
  c.merge_stage = smem + kOffSlab;
  c.merge_out = smem + kOffKpe;
  c.scale8 = smem + kOffScale8;
  c.timeout_ns = timeout_ns;
  c.drain_ns = drain_limit_ns(timeout_ns);
  c.g_begin = plan_range_begin(prm.plan, blockIdx.x);
  c.g_end = plan_range_begin(prm.plan, int64_t(blockIdx.x) + 1);
  const int warp = threadIdx.x >> 5;
  // Setup (barriers, TMEM) reads nothing a previous kernel writes, so it runs
  // before griddepcontrol.wait: launched with programmatic stream
  // serialization, the CTA gets here while the previous kernel on the stream
  // is still finishing.
  if (warp == kSetupWarp && (threadIdx.x & 31) == 0) {
    // the query tensor maps are needed by the first TMA loads: fetch them now
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_qn)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_qp)) : "memory");
    mbar_init(bar_addr(c, B_Q_FULL), 1);
    mbar_init(bar_addr(c, B_Q_EMPTY), 2);
    for (int k = 0; k < 2; ++k) {
      mbar_init(bar_addr(c, B_KPE_FULL + k), kProducerThreads);
      mbar_init(bar_addr(c, B_KPE_EMPTY + k), 1);
      mbar_init(bar_addr(c, B_S_FULL + k), 2);
      mbar_init(bar_addr(c, B_S_EMPTY + k), kSoftmaxThreads);
      mbar_init(bar_addr(c, B_P_FULL + k), kSoftmaxThreads);
      mbar_init(bar_addr(c, B_P_EMPTY + k), 2);
    }
    for (int s = 0; s < kSlabs; ++s) {
      mbar_init(bar_addr(c, B_SLAB_FULL + s), kFp8 ? kSoftmaxThreads : kProducerThreads);
      mbar_init(bar_addr(c, B_SLAB_EMPTY + s), 1);
    }
    mbar_init(bar_addr(c, B_O_FULL), 2);
    mbar_init(bar_addr(c, B_O_EMPTY), kSoftmaxThreads);
    for (int k = 0; k < 4; ++k) mbar_init(bar_addr(c, B_DONE + k), 1);
    mbar_init(bar_addr(c, B_MERGE), 1);
    for (int k = 0; k < kStageSlots; ++k) {
      mbar_init(bar_addr(c, B_STAGE_FULL + k), kProducerThreads);
      mbar_init(bar_addr(c, B_STAGE_EMPTY + k), kSoftmaxThreads);
    }
    *c.abort = 0u;
    c.task[0].pending = 0u;
    c.task[1].pending = 0u;
    fence_mbar_init();
  }
  if (warp == kQkWarp0) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  // L2 prefetches of the first block's index row and the first token's
  // queries.  They return nothing to the thread and L2 keeps device memory
  // coherent, so they may be issued before griddepcontrol.wait (a line that a
  // previous kernel still writes is updated in L2); the reads proper come
  // after the wait, from L2 instead of HBM.
  if (warp < kProducerWarps && c.g_begin < c.g_end) {
    const int p = threadIdx.x;   // 0..127
    const int64_t t0 = c.g_begin / kBlocksPerToken;
    const int32_t* row = prm.indices + t0 * kTopk + (c.g_begin % kBlocksPerToken) * kBlockKeys;   // 512 bytes
    if (p < 4) prefetch_l2(row + 32 * p);
    prefetch_l2(static_cast<const uint8_t*>(prm.q_nope) + t0 * (kHeads * kCkv * 2) + 128 * p);   // 16 KB
    if (p < 16) prefetch_l2(static_cast<const uint8_t*>(prm.q_pe) + t0 * (kHeads * kKpe * 2) + 128 * p);   // 2 KB
  }
  // Every input, the workspace's counters and records (a previous call's
  // merges reset them) and the outputs are touched only after this.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the gather's first index rows: in flight while the setup barrier completes
  int first_slots[16];
  int first_slots8[8];
  int32_t first_row = 0;
  if (warp < kProducerWarps && c.g_begin < c.g_end) {
    if constexpr (kFp8) load_slots8(prm, c.g_begin, threadIdx.x, first_slots8);
    else load_slots(prm, c.g_begin, threadIdx.x, first_slots);
    if constexpr (kPaged) first_row = row_of(prm, c.g_begin / kBlocksPerToken);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  c.tmem = *tmem_slot;

  constexpr int kRing = kFp8 ? kRingFp8 : kSlabs;
  if (warp < kProducerWarps) {
    if constexpr (kFp8) producer_fp8<kPaged>(c, prm, first_slots8, first_row);
    else producer<kPaged>(c, prm, first_slots, first_row);
  } else if (warp < kPvWarp0) {
    if ((threadIdx.x & 31) == 0) qk_issuer<kRing, kFp8 ? 1 : 2>(c, warp - kQkWarp0, &tm_qn, &tm_qp);
    __syncwarp();
  } else if (warp < kSoftmaxWarp0) {
    if ((threadIdx.x & 31) == 0) pv_issuer<kRing>(c, warp - kPvWarp0);
    __syncwarp();
  } else {
    softmax_epilogue<kPaged, kFp8>(c, prm);
  }

  tc_fence_before();
  __syncthreads();
  if (prm.cluster_merge) cluster_merge_end<kFp8>(c, prm);   // every thread of every CTA of the cluster
  if (warp == kQkWarp0) {
    tc_fence_after();
    tmem_dealloc(c.tmem, kTmemCols);   // the merges below read records, not TMEM
  }
  // Merges of tokens split over many CTAs, left for the end of the CTA, with
  // every thread of the CTA.
#pragma unroll 1
  for (int k = 1; k >= 0; --k)
    if (c.task[k].pending != 0u && *c.abort == 0u) finish_help(c, prm, c.task[k], k == 1);
  __syncthreads();
  if (threadIdx.x == 0 && *c.abort) report_error(prm.err_word, DSA_DEVICE_ERR_TIMEOUT);
}

// -------------------------------------------------------------------------
// host side
// -------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
constexpr int kMaxDevices = 64;
std::once_flag g_attr_once[kMaxDevices];
cudaError_t g_attr_err[kMaxDevices];
// Clusters of kBlocksPerToken CTAs of the split kernel that can be resident
// at once on each device (0: clusters are not used there).
int g_max_clusters[kMaxDevices];

bool encode_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace sm100

cudaError_t launch_split(const SplitParams& prm, cudaStream_t stream) {
  using namespace sm100;
  std::call_once(g_encode_once, []() {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return cudaErrorNotSupported;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::call_once(g_attr_once[dev], [dev]() {
    const void* kernels[] = {reinterpret_cast<const void*>(split_sm100_kernel<false, false>),
                             reinterpret_cast<const void*>(split_sm100_kernel<true, false>),
                             reinterpret_cast<const void*>(split_sm100_kernel<false, true>),
                             reinterpret_cast<const void*>(split_sm100_kernel<true, true>)};
    g_attr_err[dev] = cudaSuccess;
    for (const void* k : kernels)
      if (g_attr_err[dev] == cudaSuccess)
        g_attr_err[dev] = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
    // Clusters of 16 (beyond the portable 8) for the small-batch merge: the
    // fewest that every instantiation can keep resident at once; any failure
    // leaves cluster merges off on this device.
    int most = 1 << 30;
    for (const void* k : kernels) {
      int n = 0;
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(unsigned(kBlocksPerToken));
      q.blockDim = dim3(kThreads);
      q.dynamicSmemBytes = kSmemBytes;
      cudaLaunchAttribute a[1];
      a[0].id = cudaLaunchAttributeClusterDimension;
      a[0].val.clusterDim.x = unsigned(kBlocksPerToken);
      a[0].val.clusterDim.y = 1;
      a[0].val.clusterDim.z = 1;
      q.attrs = a;
      q.numAttrs = 1;
      if (cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
          cudaOccupancyMaxActiveClusters(&n, k, &q) != cudaSuccess)
        n = 0;
      most = n < most ? n : most;
    }
    cudaGetLastError();   // a refused query leaves no error behind
    g_max_clusters[dev] = most;
  });
  if (g_attr_err[dev] != cudaSuccess) return g_attr_err[dev];

  CUtensorMap tm_qn, tm_qp;
  const uint64_t qrows = uint64_t(prm.plan.total_blocks / kBlocksPerToken) * kHeads;
  if (!encode_2d(&tm_qn, prm.q_nope, kCkv, qrows, 64, 16) || !encode_2d(&tm_qp, prm.q_pe, kKpe, qrows, 64, 16))
    return cudaErrorInvalidValue;
  // Programmatic stream serialization: the CTAs may be scheduled and set up
  // while the previous kernel on the stream finishes; the kernel waits for it
  // (griddepcontrol.wait) before touching any data.
  // Small batches (one block per CTA, every token's cluster of 16 CTAs
  // resident at once): tokens are merged inside their cluster.
  SplitParams p = prm;
  const int64_t tokens = prm.plan.total_blocks / kBlocksPerToken;
  p.cluster_merge = (cluster_merge_enabled() && prm.plan.grid == prm.plan.total_blocks && tokens >= 1 &&
                     tokens <= g_max_clusters[dev])
                        ? 1
                        : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(prm.plan.grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = unsigned(kBlocksPerToken);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  const bool paged = prm.block_table != nullptr, fp8 = prm.kv_fp8 != nullptr;
  const uint64_t wait_ns = pipeline_wait_ns();
  auto launch = [&]() -> cudaError_t {
    cfg.numAttrs = p.cluster_merge ? 2 : 1;
    if (paged && fp8) return cudaLaunchKernelEx(&cfg, split_sm100_kernel<true, true>, tm_qn, tm_qp, p, wait_ns);
    if (paged) return cudaLaunchKernelEx(&cfg, split_sm100_kernel<true, false>, tm_qn, tm_qp, p, wait_ns);
    if (fp8) return cudaLaunchKernelEx(&cfg, split_sm100_kernel<false, true>, tm_qn, tm_qp, p, wait_ns);
    return cudaLaunchKernelEx(&cfg, split_sm100_kernel<false, false>, tm_qn, tm_qp, p, wait_ns);
  };
  e = launch();
  if (e != cudaSuccess && p.cluster_merge) {
    // a cluster launch refused at launch time: the same call through the workspace merge
    cudaGetLastError();
    p.cluster_merge = 0;
    e = launch();
  }
  return e;
}

}  // namespace dsa
