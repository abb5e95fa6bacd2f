/*
 * dsa_sparse_attention.h — C ABI of the B200 (sm_100a) DSA sparse MLA
 * attention operator for the definition
 * dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64.
 *
 * Plain pointers, sizes and status codes only: no torch, no CUDA types in the
 * signatures (a `void *stream` is a cudaStream_t, NULL = legacy default
 * stream of the current device).  Every entry point is safe to call from
 * several host threads on several devices at once.
 *
 * Tensor layouts (all row-major, contiguous, device memory of ONE device):
 *   q_nope          [num_tokens, 16, 512]   bf16
 *   q_pe            [num_tokens, 16, 64]    bf16
 *   ckv_cache       [num_pages, 64, 512]    bf16   (row r = slot r of the flat view)
 *   kpe_cache       [num_pages, 64, 64]     bf16
 *   sparse_indices  [num_tokens, 2048]      int32  slot id = page*64 + offset, -1 = padding
 *   output          [num_tokens, 16, 512]   bf16   (written)
 *   lse             [num_tokens, 16]        fp32   (written; BASE-2 log-sum-exp)
 * Every pointer must be 16-byte aligned.  A token whose indices are all -1
 * gets output 0 and lse -inf.
 */
#ifndef DSA_SPARSE_ATTENTION_H_
#define DSA_SPARSE_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSA_NUM_HEADS 16
#define DSA_CKV_DIM 512
#define DSA_KPE_DIM 64
#define DSA_PAGE_SIZE 64
#define DSA_TOPK 2048

/* Return codes of every entry point. */
typedef enum dsa_status {
  DSA_OK = 0,
  DSA_ERR_INVALID_ARGUMENT = 1,   /* NULL/misaligned pointer, negative or oversized count   */
  DSA_ERR_UNSUPPORTED_DEVICE = 2, /* current device is not compute capability 10.0 (B200)  */
  DSA_ERR_WORKSPACE_TOO_SMALL = 3,/* workspace_bytes < dsa_sparse_attention_workspace_size */
  DSA_ERR_CUDA = 4,               /* a CUDA runtime/driver call or a launch failed          */
  DSA_ERR_BAD_INDEX = 5,          /* device-reported: an index outside [-1, num_pages*64)   */
  DSA_ERR_DEVICE_TIMEOUT = 6      /* device-reported: a pipeline wait hit its time limit    */
} dsa_status;

/* Device-side error bits accumulated in the workspace (see read_errors). */
#define DSA_DEVICE_ERR_BAD_INDEX 0x1u
#define DSA_DEVICE_ERR_TIMEOUT 0x2u

/*
 * Bytes of device workspace dsa_sparse_attention_fwd needs for num_tokens
 * query tokens on the CURRENT device (it depends on the SM count).  The
 * workspace holds the split-KV partial records and a device error word.  It
 * must be zero-filled once when it is allocated; afterwards calls may reuse
 * it without clearing.  Calls that share one workspace must be ordered on
 * one stream.  Returns 0 if the device cannot be queried.
 * Replaces the reference's lazily grown process-global scratch and counters
 * (solution/cuda/kernel.cu:643-671), which were single-device and unchecked.
 */
size_t dsa_sparse_attention_workspace_size(int64_t num_tokens);

/*
 * Destination-passing forward pass: writes output and lse for every token.
 * Asynchronous on `stream`; returns DSA_OK once the kernels are enqueued.
 * num_tokens == 0 is a no-op.  Index errors and pipeline timeouts found on the
 * device are recorded in the workspace and reported by
 * dsa_sparse_attention_read_errors.
 * Replaces launch_sparse_attention_c (solution/cuda/kernel.cu:673-724) and
 * its pybind export (kernel.cu:726-729); the argument order is the same, with
 * sizes, workspace and stream made explicit.
 */
int dsa_sparse_attention_fwd(const void *q_nope, const void *q_pe,
                             const void *ckv_cache, const void *kpe_cache,
                             const int32_t *sparse_indices, int64_t num_tokens,
                             int64_t num_pages, float sm_scale, void *output,
                             float *lse, void *workspace,
                             size_t workspace_bytes, void *stream);

/*
 * Same computation as dsa_sparse_attention_fwd, plus timing: records
 * events[0] before the split-KV kernel and events[1] and events[2] after it
 * (three cudaEvent_t created by the caller; the partial-record merge runs
 * inside the same kernel, so events[2] - events[1] is zero).  Used by the
 * benchmark to time the kernel on its own stream.  No counterpart in the
 * reference.
 */
int dsa_sparse_attention_fwd_profiled(const void *q_nope, const void *q_pe,
                                      const void *ckv_cache,
                                      const void *kpe_cache,
                                      const int32_t *sparse_indices,
                                      int64_t num_tokens, int64_t num_pages,
                                      float sm_scale, void *output, float *lse,
                                      void *workspace, size_t workspace_bytes,
                                      void *stream, void *const *events);

/*
 * Page-table-native forward pass: the same computation as
 * dsa_sparse_attention_fwd, but the selected keys are given as positions
 * within each token's sequence and translated on the fly through a block
 * table, so no separate translation pass (and no index array round trip
 * through HBM) is needed.  Token t reads row r = seq_of_token[t] (t itself
 * when seq_of_token is NULL) of block_table [num_rows, max_num_pages] int32;
 * position p (positions [num_tokens, 2048] int32, -1 = padding) is the slot
 * block_table[r][p >> 6] * 64 + (p & 63).  A position outside the row, a row
 * outside the table or a table entry outside [0, num_pages) is a bad index:
 * treated as padding and reported like one.  Results are identical to
 * dsa_sparse_attention_fwd on the translated slot ids.
 * Replaces the reference's translate step, translate_indices_kernel with its
 * phys_idx = block_table row (methodology/reference/topk_kernel_naive.cu:52-62,
 * :96-109), followed by launch_sparse_attention_c (solution/cuda/kernel.cu:673).
 */
int dsa_sparse_attention_fwd_paged(const void *q_nope, const void *q_pe,
                                   const void *ckv_cache, const void *kpe_cache,
                                   const int32_t *block_table, int64_t num_rows,
                                   int64_t max_num_pages,
                                   const int32_t *seq_of_token,
                                   const int32_t *positions, int64_t num_tokens,
                                   int64_t num_pages, float sm_scale,
                                   void *output, float *lse, void *workspace,
                                   size_t workspace_bytes, void *stream);

/*
 * FP8 KV cache variant (no counterpart in the reference, which rejects FP8 KV
 * as outside its definition, methodology/optimization_log.md:1205).  The cache
 * is kv_cache_fp8 [num_pages, 64, 656] bytes, one 656-byte row per slot:
 *   bytes [0, 512)    ckv as fp8 e4m3,
 *   bytes [512, 528)  4 fp32 scales, scale j for ckv values [128 j, 128 j + 128),
 *   bytes [528, 656)  the 64 rope values (kpe) as bf16,
 * dequantised as ckv = bf16_rn(float(e4m3) * scale); everything else is
 * dsa_sparse_attention_fwd on the dequantised cache, bit for bit.  A key moves
 * 656 bytes instead of 1152.  Same workspace, errors and rules as
 * dsa_sparse_attention_fwd; kv_cache_fp8 must be 16-byte aligned.
 */
int dsa_sparse_attention_fwd_fp8(const void *q_nope, const void *q_pe,
                                 const void *kv_cache_fp8,
                                 const int32_t *sparse_indices,
                                 int64_t num_tokens, int64_t num_pages,
                                 float sm_scale, void *output, float *lse,
                                 void *workspace, size_t workspace_bytes,
                                 void *stream);

/* Page-table-native form of dsa_sparse_attention_fwd_fp8 (arguments as in
 * dsa_sparse_attention_fwd_paged). */
int dsa_sparse_attention_fwd_fp8_paged(
    const void *q_nope, const void *q_pe, const void *kv_cache_fp8,
    const int32_t *block_table, int64_t num_rows, int64_t max_num_pages,
    const int32_t *seq_of_token, const int32_t *positions, int64_t num_tokens,
    int64_t num_pages, float sm_scale, void *output, float *lse,
    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Synchronises `stream`, copies the workspace's device error word into
 * *device_flags (DSA_DEVICE_ERR_* bits, may be NULL), clears it, and returns
 * DSA_ERR_BAD_INDEX / DSA_ERR_DEVICE_TIMEOUT if a bit was set, else DSA_OK.
 * The reference has no device error reporting (its launch is unchecked,
 * kernel.cu:707); ATen's index_select in its naive kernel raises on a bad
 * index (methodology/checkpoints/kernel_naive.cu:54).
 */
int dsa_sparse_attention_read_errors(void *workspace, void *stream,
                                     uint32_t *device_flags);

/*
 * Forward pass for callers that cannot allocate device memory — for example
 * a serving process that hands every byte of the GPU to a fixed arena at
 * start-up, or a plugin host that does not let its plugins call cudaMalloc.
 * No counterpart in the reference.  Same arguments and results as
 * dsa_sparse_attention_fwd minus the workspace: the library keeps its own
 * scratch in a fixed 10.04 MiB device array that every GPU which loads the
 * library holds until the process exits, enough for a split grid of up to 160
 * CTAs (B200 has 148 SMs); on a device that would need more it returns
 * DSA_ERR_WORKSPACE_TOO_SMALL.  It calls no allocator.
 *  - The first call on each device looks up the array's device address (one
 *    cudaGetSymbolAddress with that device current; a failed lookup is tried
 *    again by the next call); make that first call before any stream capture.
 *  - Once its arguments have passed their checks, each call clears the
 *    array's counters and error word (one small memset on `stream`) and then
 *    reuses it, so calls whose work overlaps on the GPU (two streams, two
 *    threads) race on the same scratch: order them.  A rejected call does no
 *    device work.
 *  - Device-side findings (an out-of-range index, treated as padding; a
 *    pipeline wait that reached its time limit, leaving the output
 *    incomplete) are recorded in the error word of the library's array; read
 *    them with dsa_sparse_attention_noalloc_read_errors after the call and
 *    before the next no-alloc call on the device, which clears the word.
 */
int dsa_sparse_attention_fwd_noalloc(const void *q_nope, const void *q_pe,
                                     const void *ckv_cache,
                                     const void *kpe_cache,
                                     const int32_t *sparse_indices,
                                     int64_t num_tokens, int64_t num_pages,
                                     float sm_scale, void *output, float *lse,
                                     void *stream);

/*
 * dsa_sparse_attention_read_errors for the no-alloc calls on the current
 * device: synchronises `stream`, reads and clears the error word of the
 * library's array (after a timeout, its arrival counters too) and returns
 * DSA_ERR_DEVICE_TIMEOUT, DSA_ERR_BAD_INDEX or DSA_OK, with the raw bits in
 * *device_flags (may be null).  Allocates nothing.  No counterpart in the
 * reference.
 */
int dsa_sparse_attention_noalloc_read_errors(void *stream, uint32_t *device_flags);

/*
 * ---- DSA top-k indexer (definition dsa_topk_indexer_fp8_h64_d128_topk2048_ps64)
 * The operator upstream of the attention: for batch row b it scores every
 * position pos < seq_lens[b] of the row's sequence,
 *   final[pos] = sum_h weights[b][h] * relu(q[b][h] . K[pos]),
 * with q_index_fp8 [batch, 64, 128] fp8 e4m3 and K[pos] = the fp8 e4m3 key
 * row times its fp32 scale, read through block_table [batch, max_num_pages]
 * int32 from k_index_cache [num_pages] pages of 8448 bytes (64 rows of 128
 * fp8, then the 64 rows' fp32 scales); weights [batch, 64] fp32, seq_lens
 * [batch] int32.  topk_indices [batch, 2048] int32 receives the min(2048,
 * seq_len) best positions, largest score first (equal scores: lower
 * position first), as slot ids block_table[b][pos >> 6] * 64 + (pos & 63),
 * and -1 after them.  A block-table entry outside [0, num_pages) within
 * seq_len, or a seq_len beyond max_num_pages * 64, is a bad index: scored
 * -inf, never returned, reported through dsa_sparse_attention_read_errors on
 * this call's workspace.
 * The workspace (dsa_topk_indexer_workspace_size bytes) must be zero-filled
 * once when it is allocated; every call leaves it ready for the next.  Calls
 * that share one workspace must be ordered on one stream.
 * Replaces launch_topk_c (methodology/reference/topk_kernel_naive.cu:65-111),
 * same argument meaning with sizes, workspace and stream made explicit.
 */
size_t dsa_topk_indexer_workspace_size(int64_t batch, int64_t max_num_pages);

int dsa_topk_indexer_fwd(const void *q_index_fp8, const void *k_index_cache,
                         const float *weights, const int32_t *seq_lens,
                         const int32_t *block_table, int64_t batch,
                         int64_t max_num_pages, int64_t num_pages,
                         int32_t *topk_indices, void *workspace,
                         size_t workspace_bytes, void *stream);

/*
 * Bound, in nanoseconds, on every pipeline wait of the kernels launched after
 * this call, process-wide (0 = the default: DSA_WAIT_TIMEOUT_MS read from the
 * environment once, else 2000 ms).  A wait that reaches it makes its CTA stop,
 * drain its own copies and MMAs (those drain waits keep a separate bound of at
 * least 2 s), free its tensor memory and exit; the call then reports
 * DSA_ERR_DEVICE_TIMEOUT through dsa_sparse_attention_read_errors and its
 * outputs are incomplete.  No counterpart in the reference, whose waits spin
 * without a bound (solution/cuda/kernel.cu:105-116).  Returns DSA_OK.
 */
int dsa_sparse_attention_set_wait_timeout_ns(uint64_t pipeline_wait_ns);

/*
 * Test hook of the device-timeout path, process-wide, off by default; for
 * tests only.  While enabled (enable != 0), every CTA of the attention
 * launches that follow first waits for a word of the workspace header that
 * nothing ever sets; the wait runs out at the pipeline limit
 * (dsa_sparse_attention_set_wait_timeout_ns), the kernel drains and exits,
 * and dsa_sparse_attention_read_errors then reports DSA_ERR_DEVICE_TIMEOUT.
 * No counterpart in the reference.  Returns DSA_OK.
 */
int dsa_sparse_attention_test_hold(int enable);

/*
 * Small batches (one 128-slot block per CTA, every token's 16 CTAs able to be
 * resident as one thread-block cluster at once; on a B200, up to 7 tokens)
 * are merged inside the cluster through distributed shared memory instead of
 * through the workspace records.  Process-wide; on by default.  enable = 0
 * makes later launches use the workspace merge for every batch (the results
 * are bitwise the same; tests use this to cover both).  No counterpart in the
 * reference.  Returns DSA_OK.
 */
int dsa_sparse_attention_set_cluster_merge(int enable);

/*
 * The indexer's score kernel splits the call's active tiles (128 positions of
 * a row within its seq_len) over its CTAs by a plan kept in the workspace:
 * each call logs every CTA's tiles and run time, and the next call gives each
 * CTA a share in proportion to its measured rate (so that all end together).
 * Process-wide; on by default.  enable = 0 makes later launches take equal
 * shares and log nothing (the results are bitwise the same; tests use this to
 * cover both).  No counterpart in the reference.  Returns DSA_OK.
 */
int dsa_topk_indexer_set_calibrated_plan(int enable);

/* Human-readable name of a dsa_status value (static string). */
const char *dsa_status_string(int status);

/* ABI version of this library (major*1000 + minor). */
int dsa_sparse_attention_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DSA_SPARSE_ATTENTION_H_ */
