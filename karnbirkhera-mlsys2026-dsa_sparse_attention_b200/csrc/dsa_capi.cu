// dsa_capi.cu — the extern "C" boundary declared in include/dsa_sparse_attention.h.
//
// Host-side responsibilities of the reference launcher
// (solution/cuda/kernel.cu:631-724), redone for a multi-device process:
//   * argument validation (the reference checks only its split invariant,
//     kernel.cu:688-691) — every pointer must be device memory of the current
//     device and 16-byte aligned, counts must be in range;
//   * the split plan, sized from the device's real SM count (the reference
//     hard-codes 132, kernel.cu:634-641);
//   * caller-owned workspace instead of process-global lazily grown buffers
//     (kernel.cu:643-671);
//   * every CUDA call checked; status codes instead of silent failure.
#include <cuda_bf16.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "dsa_common.cuh"

namespace dsa {

cudaError_t launch_split(const SplitParams& prm, cudaStream_t stream);
cudaError_t launch_indexer(const uint8_t* q, const uint8_t* cache, const float* weights, const int32_t* seq_lens,
                           const int32_t* block_table, int64_t batch, int64_t max_pages, int64_t num_pages,
                           int32_t* out, float* scores, uint32_t* row_keys, uint32_t* err_word, void* plan_state,
                           int sms, cudaStream_t stream);

namespace {

constexpr int kMaxDevices = 64;
constexpr int64_t kMaxTokens = int64_t(1) << 24;

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
  cudaError_t err = cudaSuccess;
};

DeviceInfo g_info[kMaxDevices];
std::once_flag g_info_once[kMaxDevices];

const DeviceInfo* device_info(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(g_info_once[dev], [dev]() {
    DeviceInfo& d = g_info[dev];
    d.err = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (d.err == cudaSuccess) d.err = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    if (d.err == cudaSuccess) d.err = cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
  });
  return &g_info[dev];
}

Plan make_plan(int64_t num_tokens, int sms) {
  Plan p;
  p.total_blocks = num_tokens * kBlocksPerToken;
  p.grid = int(p.total_blocks < sms ? p.total_blocks : sms);
  return p;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// True when p is device (or managed) memory that the current device can use.
bool on_device(const void* p, int dev) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (a.type == cudaMemoryTypeManaged) return true;
  return a.type == cudaMemoryTypeDevice && a.device == dev;
}

}  // namespace

// Pipeline wait limit of the kernels: DSA_WAIT_TIMEOUT_MS (read once; default
// 2000 ms) unless dsa_sparse_attention_set_wait_timeout_ns set a value.
namespace {
std::atomic<uint64_t> g_wait_override_ns{0};
std::atomic<int> g_test_hold{0};
// Small-batch merges inside thread-block clusters (on unless switched off).
std::atomic<int> g_cluster_merge{1};
// The indexer's calibrated score plan (on unless switched off).
std::atomic<int> g_indexer_plan{1};
std::once_flag g_wait_env_once;
uint64_t g_wait_env_ns = 0;
}  // namespace

bool cluster_merge_enabled() { return g_cluster_merge.load(std::memory_order_relaxed) != 0; }

uint64_t pipeline_wait_ns() {
  const uint64_t o = g_wait_override_ns.load(std::memory_order_relaxed);
  if (o != 0) return o;
  std::call_once(g_wait_env_once, []() {
    const char* env = std::getenv("DSA_WAIT_TIMEOUT_MS");
    const long ms = env ? std::strtol(env, nullptr, 10) : 0;
    g_wait_env_ns = uint64_t(ms > 0 ? ms : 2000) * 1000000ull;
  });
  return g_wait_env_ns;
}

// Page-table-native indexing (dsa_sparse_attention_fwd_paged).
struct PagedIndex {
  const int32_t* block_table;
  int64_t num_rows;
  int64_t max_pages;
  const int32_t* seq_of_token;   // may be null: token t uses row t
};

namespace {
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
}  // namespace

// kv_fp8 non-null: FP8 KV rows (ckv and kpe unused, may be null).
// clear_bytes > 0: once every argument has passed its checks, the first
// clear_bytes of the workspace are zeroed on the stream before the launch
// (a call rejected by a check does no device work).
int fwd_impl_ex(const void* q_nope, const void* q_pe, const void* ckv, const void* kpe, const int32_t* idx,
                int64_t num_tokens, int64_t num_pages, float sm_scale, void* output, float* lse, void* workspace,
                size_t workspace_bytes, void* stream_ptr, void* const* events, const PagedIndex* paged,
                const void* kv_fp8 = nullptr, size_t clear_bytes = 0) {
  if (num_tokens < 0 || num_tokens > kMaxTokens) return DSA_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return DSA_OK;  // reference: kernel.cu:685
  if (num_pages <= 0 || num_pages > (int64_t(INT32_MAX) / kPage)) return DSA_ERR_INVALID_ARGUMENT;
  if (!(sm_scale == sm_scale)) return DSA_ERR_INVALID_ARGUMENT;  // NaN scale
  // in FP8 mode the cache pointer takes the ckv slot and kpe is not used
  const void* ptrs[] = {q_nope, q_pe, kv_fp8 ? kv_fp8 : ckv, kv_fp8 ? kv_fp8 : kpe, idx, output, lse, workspace};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return DSA_ERR_INVALID_ARGUMENT;
  if (paged != nullptr) {
    // positions are int32 and address pages through 64-slot pages
    if (paged->block_table == nullptr || !aligned4(paged->block_table) || paged->num_rows <= 0 ||
        paged->max_pages <= 0 || paged->max_pages > (int64_t(INT32_MAX) / kPage) ||
        paged->num_rows > (int64_t(1) << 40) / paged->max_pages)
      return DSA_ERR_INVALID_ARGUMENT;
    if (paged->seq_of_token != nullptr && !aligned4(paged->seq_of_token)) return DSA_ERR_INVALID_ARGUMENT;
  }

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSA_ERR_CUDA;
  const DeviceInfo* info = device_info(dev);
  if (info == nullptr || info->err != cudaSuccess) return DSA_ERR_CUDA;
  if (info->major != 10 || info->minor != 0 || info->sms > kMaxGrid) return DSA_ERR_UNSUPPORTED_DEVICE;
  for (const void* p : ptrs)
    if (!on_device(p, dev)) return DSA_ERR_INVALID_ARGUMENT;
  if (paged != nullptr) {
    if (!on_device(paged->block_table, dev)) return DSA_ERR_INVALID_ARGUMENT;
    if (paged->seq_of_token != nullptr && !on_device(paged->seq_of_token, dev)) return DSA_ERR_INVALID_ARGUMENT;
  }

  const Plan plan = make_plan(num_tokens, info->sms);
  if (workspace_bytes < workspace_bytes_for_grid(plan.grid)) return DSA_ERR_WORKSPACE_TOO_SMALL;

  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  SplitParams prm{};
  prm.q_nope = q_nope;
  prm.q_pe = q_pe;
  prm.ckv = kv_fp8 ? nullptr : ckv;
  prm.kpe = kv_fp8 ? nullptr : kpe;
  prm.kv_fp8 = kv_fp8;
  prm.indices = idx;
  prm.block_table = paged ? paged->block_table : nullptr;
  prm.seq_of_token = paged ? paged->seq_of_token : nullptr;
  prm.num_rows = paged ? paged->num_rows : 0;
  prm.max_pages = paged ? paged->max_pages : 0;
  prm.output = output;
  prm.lse = lse;
  prm.err_word = static_cast<uint32_t*>(workspace);
  prm.counters = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + kWorkspaceHeaderBytes);
  prm.hold = g_test_hold.load(std::memory_order_relaxed)
                 ? reinterpret_cast<const uint32_t*>(static_cast<uint8_t*>(workspace) + kHoldWordOffset)
                 : nullptr;
  prm.records = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWorkspaceRecordsOffset);
  prm.num_slots = num_pages * kPage;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.plan = plan;

  if (clear_bytes > 0 && cudaMemsetAsync(workspace, 0, clear_bytes, stream) != cudaSuccess) return DSA_ERR_CUDA;
  if (events && cudaEventRecord(static_cast<cudaEvent_t>(events[0]), stream) != cudaSuccess) return DSA_ERR_CUDA;
  if (launch_split(prm, stream) != cudaSuccess) return DSA_ERR_CUDA;
  if (events && cudaEventRecord(static_cast<cudaEvent_t>(events[1]), stream) != cudaSuccess) return DSA_ERR_CUDA;
  if (events && cudaEventRecord(static_cast<cudaEvent_t>(events[2]), stream) != cudaSuccess) return DSA_ERR_CUDA;
  return DSA_OK;
}

int fwd_impl(const void* q_nope, const void* q_pe, const void* ckv, const void* kpe, const int32_t* idx,
             int64_t num_tokens, int64_t num_pages, float sm_scale, void* output, float* lse, void* workspace,
             size_t workspace_bytes, void* stream_ptr, void* const* events) {
  return fwd_impl_ex(q_nope, q_pe, ckv, kpe, idx, num_tokens, num_pages, sm_scale, output, lse, workspace,
                     workspace_bytes, stream_ptr, events, nullptr);
}

}  // namespace dsa

extern "C" {

size_t dsa_sparse_attention_workspace_size(int64_t num_tokens) {
  if (num_tokens < 0 || num_tokens > dsa::kMaxTokens) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const dsa::DeviceInfo* info = dsa::device_info(dev);
  if (info == nullptr || info->err != cudaSuccess) return 0;
  const int64_t n = num_tokens > 0 ? num_tokens : 1;
  return dsa::workspace_bytes_for_grid(dsa::make_plan(n, info->sms).grid);
}

int dsa_sparse_attention_fwd(const void* q_nope, const void* q_pe, const void* ckv_cache, const void* kpe_cache,
                             const int32_t* sparse_indices, int64_t num_tokens, int64_t num_pages, float sm_scale,
                             void* output, float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  return dsa::fwd_impl(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, num_tokens, num_pages, sm_scale, output,
                       lse, workspace, workspace_bytes, stream, nullptr);
}

int dsa_sparse_attention_fwd_profiled(const void* q_nope, const void* q_pe, const void* ckv_cache,
                                      const void* kpe_cache, const int32_t* sparse_indices, int64_t num_tokens,
                                      int64_t num_pages, float sm_scale, void* output, float* lse, void* workspace,
                                      size_t workspace_bytes, void* stream, void* const* events) {
  if (events == nullptr || events[0] == nullptr || events[1] == nullptr || events[2] == nullptr)
    return DSA_ERR_INVALID_ARGUMENT;
  return dsa::fwd_impl(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, num_tokens, num_pages, sm_scale, output,
                       lse, workspace, workspace_bytes, stream, events);
}

int dsa_sparse_attention_fwd_paged(const void* q_nope, const void* q_pe, const void* ckv_cache,
                                   const void* kpe_cache, const int32_t* block_table, int64_t num_rows,
                                   int64_t max_num_pages, const int32_t* seq_of_token, const int32_t* positions,
                                   int64_t num_tokens, int64_t num_pages, float sm_scale, void* output, float* lse,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  const dsa::PagedIndex paged{block_table, num_rows, max_num_pages, seq_of_token};
  return dsa::fwd_impl_ex(q_nope, q_pe, ckv_cache, kpe_cache, positions, num_tokens, num_pages, sm_scale, output, lse,
                          workspace, workspace_bytes, stream, nullptr, &paged);
}

int dsa_sparse_attention_fwd_fp8(const void* q_nope, const void* q_pe, const void* kv_cache_fp8,
                                 const int32_t* sparse_indices, int64_t num_tokens, int64_t num_pages, float sm_scale,
                                 void* output, float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  if (kv_cache_fp8 == nullptr) return DSA_ERR_INVALID_ARGUMENT;
  return dsa::fwd_impl_ex(q_nope, q_pe, nullptr, nullptr, sparse_indices, num_tokens, num_pages, sm_scale, output, lse,
                          workspace, workspace_bytes, stream, nullptr, nullptr, kv_cache_fp8);
}

int dsa_sparse_attention_fwd_fp8_paged(const void* q_nope, const void* q_pe, const void* kv_cache_fp8,
                                       const int32_t* block_table, int64_t num_rows, int64_t max_num_pages,
                                       const int32_t* seq_of_token, const int32_t* positions, int64_t num_tokens,
                                       int64_t num_pages, float sm_scale, void* output, float* lse, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  if (kv_cache_fp8 == nullptr) return DSA_ERR_INVALID_ARGUMENT;
  const dsa::PagedIndex paged{block_table, num_rows, max_num_pages, seq_of_token};
  return dsa::fwd_impl_ex(q_nope, q_pe, nullptr, nullptr, positions, num_tokens, num_pages, sm_scale, output, lse,
                          workspace, workspace_bytes, stream, nullptr, &paged, kv_cache_fp8);
}

// ---------------------------------------------------------------- top-k indexer
namespace {
constexpr int64_t kIndexerMaxBatch = int64_t(1) << 20;
constexpr int64_t kIndexerPageBytes = 8448;

size_t indexer_row_keys_offset(int64_t batch, int64_t max_pages) {
  return dsa::kWorkspaceRecordsOffset + size_t(batch) * size_t(max_pages) * dsa::kPage * sizeof(float);
}

size_t indexer_plan_offset(int64_t batch, int64_t max_pages) {
  return (indexer_row_keys_offset(batch, max_pages) + size_t(batch) * 2 * sizeof(uint32_t) + 15) & ~size_t(15);
}

size_t indexer_workspace_bytes(int64_t batch, int64_t max_pages) {
  // same header as the attention workspace (error word, counters), then the
  // per-position scores [batch, max_pages * 64] fp32, then each row's key
  // range [batch][2] u32, then (16-byte aligned) the calibrated score plan
  return indexer_plan_offset(batch, max_pages) + dsa::kIndexerPlanBytes;
}
}  // namespace

size_t dsa_topk_indexer_workspace_size(int64_t batch, int64_t max_num_pages) {
  if (batch < 0 || batch > kIndexerMaxBatch || max_num_pages <= 0 || max_num_pages > (int64_t(INT32_MAX) / dsa::kPage))
    return 0;
  return indexer_workspace_bytes(batch > 0 ? batch : 1, max_num_pages);
}

int dsa_topk_indexer_fwd(const void* q_index_fp8, const void* k_index_cache, const float* weights,
                         const int32_t* seq_lens, const int32_t* block_table, int64_t batch, int64_t max_num_pages,
                         int64_t num_pages, int32_t* topk_indices, void* workspace, size_t workspace_bytes,
                         void* stream) {
  using namespace dsa;
  if (batch < 0 || batch > kIndexerMaxBatch) return DSA_ERR_INVALID_ARGUMENT;
  if (batch == 0) return DSA_OK;
  if (max_num_pages <= 0 || max_num_pages > (int64_t(INT32_MAX) / kPage)) return DSA_ERR_INVALID_ARGUMENT;
  // the key cache is addressed by the tensor map in rows of 128 bytes (66 per page, int32 coordinates)
  if (num_pages <= 0 || num_pages > (int64_t(INT32_MAX) / (kIndexerPageBytes / 128))) return DSA_ERR_INVALID_ARGUMENT;
  const void* p16[] = {q_index_fp8, k_index_cache, workspace};
  const void* p4[] = {weights, seq_lens, block_table, topk_indices};
  for (const void* p : p16)
    if (p == nullptr || !aligned16(p)) return DSA_ERR_INVALID_ARGUMENT;
  for (const void* p : p4)
    if (p == nullptr || !aligned4(p)) return DSA_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < indexer_workspace_bytes(batch, max_num_pages)) return DSA_ERR_WORKSPACE_TOO_SMALL;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSA_ERR_CUDA;
  const DeviceInfo* info = device_info(dev);
  if (info == nullptr || info->err != cudaSuccess) return DSA_ERR_CUDA;
  if (info->major != 10 || info->minor != 0) return DSA_ERR_UNSUPPORTED_DEVICE;
  for (const void* p : p16)
    if (!on_device(p, dev)) return DSA_ERR_INVALID_ARGUMENT;
  for (const void* p : p4)
    if (!on_device(p, dev)) return DSA_ERR_INVALID_ARGUMENT;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* row_keys = reinterpret_cast<uint32_t*>(ws + indexer_row_keys_offset(batch, max_num_pages));
  uint8_t* plan = ws + indexer_plan_offset(batch, max_num_pages);
  // Each call leaves the rows' key ranges cleared for the next; a workspace
  // first used, or used with another (batch, max_num_pages) layout, gets them
  // cleared here, with the plan's header (both regions move with the layout).
  {
    static std::mutex mu;
    static std::unordered_map<const void*, std::pair<int64_t, int64_t>> layouts;
    bool fresh;
    {
      std::lock_guard<std::mutex> lock(mu);
      auto it = layouts.find(workspace);
      fresh = it == layouts.end() || it->second != std::make_pair(batch, max_num_pages);
      layouts[workspace] = std::make_pair(batch, max_num_pages);
    }
    if (fresh && cudaMemsetAsync(row_keys, 0, size_t(plan + 16 - reinterpret_cast<uint8_t*>(row_keys)),
                                 static_cast<cudaStream_t>(stream)) != cudaSuccess)
      return DSA_ERR_CUDA;
  }
  if (launch_indexer(static_cast<const uint8_t*>(q_index_fp8), static_cast<const uint8_t*>(k_index_cache), weights,
                     seq_lens, block_table, batch, max_num_pages, num_pages, topk_indices,
                     reinterpret_cast<float*>(ws + kWorkspaceRecordsOffset), row_keys,
                     reinterpret_cast<uint32_t*>(ws), g_indexer_plan.load(std::memory_order_relaxed) ? plan : nullptr,
                     info->sms, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return DSA_ERR_CUDA;
  return DSA_OK;
}

int dsa_sparse_attention_read_errors(void* workspace, void* stream, uint32_t* device_flags) {
  if (workspace == nullptr || !dsa::aligned16(workspace)) return DSA_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t flags = 0;
  if (cudaMemcpyAsync(&flags, workspace, sizeof(flags), cudaMemcpyDeviceToHost, s) != cudaSuccess) return DSA_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return DSA_ERR_CUDA;
  if (flags != 0) {
    // after a timeout the per-token arrival counters may be left mid-count:
    // clear the header and every counter the largest plan can use
    const size_t n = (flags & DSA_DEVICE_ERR_TIMEOUT) ? dsa::kWorkspaceRecordsOffset
                                                      : sizeof(uint32_t);
    if (cudaMemsetAsync(workspace, 0, n, s) != cudaSuccess) return DSA_ERR_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return DSA_ERR_CUDA;
  }
  if (device_flags) *device_flags = flags;
  if (flags & DSA_DEVICE_ERR_TIMEOUT) return DSA_ERR_DEVICE_TIMEOUT;
  if (flags & DSA_DEVICE_ERR_BAD_INDEX) return DSA_ERR_BAD_INDEX;
  return DSA_OK;
}

const char* dsa_status_string(int status) {
  switch (status) {
    case DSA_OK: return "DSA_OK";
    case DSA_ERR_INVALID_ARGUMENT: return "DSA_ERR_INVALID_ARGUMENT";
    case DSA_ERR_UNSUPPORTED_DEVICE: return "DSA_ERR_UNSUPPORTED_DEVICE";
    case DSA_ERR_WORKSPACE_TOO_SMALL: return "DSA_ERR_WORKSPACE_TOO_SMALL";
    case DSA_ERR_CUDA: return "DSA_ERR_CUDA";
    case DSA_ERR_BAD_INDEX: return "DSA_ERR_BAD_INDEX";
    case DSA_ERR_DEVICE_TIMEOUT: return "DSA_ERR_DEVICE_TIMEOUT";
    default: return "DSA_ERR_UNKNOWN";
  }
}

int dsa_sparse_attention_set_wait_timeout_ns(uint64_t pipeline_wait_ns) {
  dsa::g_wait_override_ns.store(pipeline_wait_ns, std::memory_order_relaxed);
  return DSA_OK;
}

int dsa_sparse_attention_set_cluster_merge(int enable) {
  dsa::g_cluster_merge.store(enable ? 1 : 0, std::memory_order_relaxed);
  return DSA_OK;
}

int dsa_topk_indexer_set_calibrated_plan(int enable) {
  dsa::g_indexer_plan.store(enable ? 1 : 0, std::memory_order_relaxed);
  return DSA_OK;
}

int dsa_sparse_attention_test_hold(int enable) {
  dsa::g_test_hold.store(enable ? 1 : 0, std::memory_order_relaxed);
  return DSA_OK;
}

int dsa_sparse_attention_abi_version(void) { return 1004; }

}  // extern "C"
