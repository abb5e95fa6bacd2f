// dsa_common.cuh — constants, the static work plan, the partial-record and
// workspace layouts and small device helpers of the split-KV kernel.
//
// Definition: dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64
// (reference constants: solution/cuda/kernel.cu:41-45).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "dsa_sparse_attention.h"   // found through -I include (flat in a packed solution)

namespace dsa {

constexpr int kHeads = DSA_NUM_HEADS;     // 16 query heads
constexpr int kCkv = DSA_CKV_DIM;         // 512 compressed-KV width (also the V width)
constexpr int kKpe = DSA_KPE_DIM;         // 64 rope-key width
constexpr int kQk = kCkv + kKpe;          // 576 contraction width of the logits
constexpr int kPage = DSA_PAGE_SIZE;      // 64 slots per page
constexpr int kTopk = DSA_TOPK;           // 2048 index slots per token

// Work unit: a "block" = 128 consecutive index slots of one token.  A token
// has kTopk / kBlockKeys = 16 blocks.  The gathered rows of one block are the
// M=128 operand of the logits contraction on the tensor cores.
constexpr int kBlockKeys = 128;
constexpr int kBlocksPerToken = kTopk / kBlockKeys;   // 16
static_assert(kTopk % kBlockKeys == 0, "blocks tile the index row");

constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------
// Static work plan.  The N*16 blocks are split into `grid` contiguous ranges of
// near-equal length (range b = [floor(b*T/G), floor((b+1)*T/G))).  A CTA walks
// its range token by token; the run of blocks it owns inside one token is a
// "segment".  A segment that covers all 16 blocks of its token writes the
// final output directly; any other segment writes a partial record, and the
// records are combined by the CTAs of the token at the end of their segments
// (see the split kernel).  CTA b owns at most two partial segments (its first
// and its last token), so records live at slots 2b and 2b+1.
// ---------------------------------------------------------------------------
struct Plan {
  int64_t total_blocks;  // T = num_tokens * 16
  int grid;              // G CTAs of the split kernel (<= SM count, <= T)
};

// floor(num / den) for 0 <= num < 2^38 and 1 <= den <= 2^28 (the plan's
// ranges: num_tokens <= 2^24, grid <= kMaxGrid).  On the device it is done in
// double precision, which is exact here: a non-integer quotient is at least
// 1/den (>= 2^-28) away from the next integer, far more than half an ulp of a
// quotient below 2^38 (<= 2^-15), so the rounded quotient floors correctly.
// (A 64-bit integer division is a long software sequence on the GPU.)
__host__ __device__ inline int64_t plan_div(int64_t num, int64_t den) {
#ifdef __CUDA_ARCH__
  return int64_t(floor(double(num) / double(den)));
#else
  return num / den;
#endif
}

__host__ __device__ inline int64_t plan_range_begin(const Plan& p, int64_t b) {
  return plan_div(b * p.total_blocks, p.grid);
}

// CTA owning global block g: the largest b with range_begin(b) <= g.
__host__ __device__ inline int64_t plan_owner(const Plan& p, int64_t g) {
  return plan_div((g + 1) * p.grid - 1, p.total_blocks);
}

// Record slot that CTA b uses for token t (t must intersect b's range).
__host__ __device__ inline int64_t plan_record_slot(const Plan& p, int64_t b, int64_t t) {
  const int64_t first_token = plan_range_begin(p, b) / kBlocksPerToken;
  return 2 * b + (t == first_token ? 0 : 1);
}

// True when token t is covered by more than one CTA (needs the merge).
__host__ __device__ inline bool plan_token_split(const Plan& p, int64_t t) {
  return plan_owner(p, t * kBlocksPerToken) !=
         plan_owner(p, t * kBlocksPerToken + kBlocksPerToken - 1);
}

// ---------------------------------------------------------------------------
// Partial record of one segment, fp32, relative to the segment's reference
// maximum m (log2 domain, logits pre-multiplied by sm_scale*log2(e)):
//   m[h]        reference max used for the exponentials (-inf if no valid key)
//   l[h]        sum_k 2^(x_k - m)
//   o[d][h]     sum_k 2^(x_k - m) * ckv_k[d]          (dim-major, the 16 heads of a dim contiguous)
// The 64-byte row o[d][*] is stored as four 16-byte chunks (heads 4q..4q+3)
// with chunk q at position record_chunk(d, q): a warp reading chunk q of 32
// consecutive dims from a shared-memory copy of the record then touches
// every bank once.  The record is one contiguous 32,896-byte block.
// ---------------------------------------------------------------------------
constexpr int kRecordFloats = 2 * kHeads + kHeads * kCkv;   // 8224 floats
constexpr size_t kRecordBytes = kRecordFloats * sizeof(float);

__host__ __device__ inline int record_chunk(int d, int q) { return q ^ ((d >> 1) & 3); }

struct RecordView {
  float* m;
  float* l;
  float* o;
};

__host__ __device__ inline RecordView record_at(float* base, int64_t slot) {
  float* r = base + slot * kRecordFloats;
  return RecordView{r, r + kHeads, r + 2 * kHeads};
}

// Workspace layout: [0,256) header (device error word at offset 0, a word
// that is never written at kHoldWordOffset), then a FIXED region of
// kMaxGrid pairs of uint32 merge counters (one pair per CTA boundary), then
// 2*grid records.  The counter region does not depend on the grid, so calls
// with different token counts never see each other's records as counters.
// Counters must start at zero (the workspace is zero-filled once); the CTA
// that completes a token resets its pair, so every call leaves them at zero
// again.
constexpr size_t kWorkspaceHeaderBytes = 256;
constexpr size_t kHoldWordOffset = 8;        // never written: the timeout-path test hook waits on it
constexpr int kMaxGrid = 1024;   // upper bound on split-kernel CTAs (one per SM)
constexpr size_t kWorkspaceCounterBytes = size_t(kMaxGrid) * 2 * sizeof(uint32_t);
constexpr size_t kWorkspaceRecordsOffset = kWorkspaceHeaderBytes + kWorkspaceCounterBytes;

// The top-k indexer's workspace ends (16-byte aligned) with the state of its
// calibrated score plan: a 16-byte header, kIndexerPlanMaxGrid + 4 range
// bounds and one 16-byte log entry per score CTA.
constexpr int kIndexerPlanMaxGrid = 1024;
constexpr size_t kIndexerPlanBytes = 16 + 4 * size_t(kIndexerPlanMaxGrid + 4) + 16 * size_t(kIndexerPlanMaxGrid);

__host__ __device__ constexpr size_t workspace_bytes_for_grid(int grid) {
  return kWorkspaceRecordsOffset + size_t(2) * size_t(grid) * kRecordBytes;
}

// A token split over CTAs b_lo..b_hi keeps its merge state in counter pair
// b_lo + 1 (the first CTA boundary inside the token, unique per split
// token):
//   word 0: the low 16 bits count the segments that arrived (their tickets),
//           the high 16 bits hold one bit per published record (bit
//           16 + b - b_lo; a token spans at most 16 CTAs, since every CTA
//           owns at least one block);
//   word 1: tokens merged by several CTAs only: the low 8 bits mark the
//           output chunks already claimed, the high 16 bits count the
//           helping CTAs that have finished.
__host__ __device__ inline int64_t plan_token_counter(const Plan& p, int64_t t) {
  return 2 * (plan_owner(p, t * kBlocksPerToken) + 1);
}

// Output chunks of a token merged by several CTAs: 64 dims x 16 heads each.
constexpr int kChunkDims = 64;
constexpr int kChunks = kCkv / kChunkDims;     // 8

// Arguments of the split-KV kernels (host-validated).
// FP8 KV row (one slot): ckv as e4m3 in [0, 512), the fp32 scale of ckv
// values [128 j, 128 j + 128) at 512 + 4 j, the bf16 rope values at 528.
// Dequantised ckv = bf16_rn(float(e4m3) * scale).
constexpr int kFp8RowBytes = 656;
constexpr int kFp8ScaleOff = 512;
constexpr int kFp8RopeOff = 528;

struct SplitParams {
  const void* q_nope;
  const void* q_pe;
  const void* ckv;
  const void* kpe;
  // FP8 KV cache (null: bf16 ckv / kpe above): rows of kFp8RowBytes per slot,
  // 512 e4m3 ckv values, 4 fp32 scales (one per 128 values), 64 bf16 rope values.
  const void* kv_fp8;
  const int32_t* indices;       // slot ids, or positions within a sequence when block_table is set
  // Page-table-native indexing (null block_table: `indices` are slot ids).
  // Token t reads row r = seq_of_token[t] (t itself when null) of
  // block_table [num_rows, max_pages]; position p maps to slot
  // block_table[r][p >> 6] * 64 + (p & 63).
  const int32_t* block_table;
  const int32_t* seq_of_token;
  int64_t num_rows;
  int64_t max_pages;
  void* output;
  float* lse;
  float* records;
  uint32_t* err_word;
  uint32_t* counters;      // per split token arrival counters (zero between calls)
  // Test hook of the timeout path (null in normal calls): the softmax warps of
  // every CTA first wait, under the pipeline limit, for this word (which
  // nothing sets) to become non-zero.
  const uint32_t* hold;
  int64_t num_slots;
  float scale_log2;  // sm_scale * log2(e)
  Plan plan;
  // Set by the launcher (1: one block per CTA and each token's 16 CTAs form
  // one thread-block cluster; the token is merged through distributed shared
  // memory at the end of the CTAs instead of through the workspace records).
  int32_t cluster_merge;
};

__device__ __forceinline__ void report_error(uint32_t* err_word, uint32_t bits) {
  atomicOr(err_word, bits);
}

// Wait limits.  Every pipeline wait of a kernel (a barrier another role or
// another CTA completes) gives up after the pipeline limit and raises the
// abort.  The waits that then drain a CTA's OWN copies, MMAs and bulk
// transfers before it frees TMEM and exits have a separate bound that is
// never shorter than kMinDrainWaitNs: those operations always complete, and
// leaving before they do would free TMEM or shared memory under them.
// pipeline_wait_ns() (host) is DSA_WAIT_TIMEOUT_MS (default 2000 ms) unless
// dsa_sparse_attention_set_wait_timeout_ns set another value.
constexpr uint64_t kMinDrainWaitNs = 2000000000ull;
__host__ __device__ inline uint64_t drain_limit_ns(uint64_t pipeline_ns) {
  return pipeline_ns > kMinDrainWaitNs ? pipeline_ns : kMinDrainWaitNs;
}
uint64_t pipeline_wait_ns();
// Whether small batches may be merged inside thread-block clusters (host;
// dsa_sparse_attention_set_cluster_merge).
bool cluster_merge_enabled();

}  // namespace dsa
