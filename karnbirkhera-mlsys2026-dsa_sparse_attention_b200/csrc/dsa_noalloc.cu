// dsa_noalloc.cu — the forward pass for callers that cannot allocate device
// memory.
//
// dsa_sparse_attention_fwd needs a caller-provided workspace (partial records
// of tokens split over several CTAs, their arrival counters and the device
// error word).  Some callers cannot provide one: an inference server that
// carves all device memory out of a fixed arena at start-up and lets no
// component allocate afterwards, or a plugin host that forbids plugins to call
// cudaMalloc (the host owns the memory budget and accounts for every byte).  For them
// this file keeps the workspace in a file-scope __device__ array instead, of a
// fixed maximum size, that every GPU which loads the library holds until the
// process exits.  The kernel and the forward path are the ones
// dsa_sparse_attention_fwd uses; only the workspace pointer differs.
#include <cuda_runtime.h>

#include <mutex>

#include "dsa_common.cuh"

namespace dsa {

struct PagedIndex;
int fwd_impl_ex(const void* q_nope, const void* q_pe, const void* ckv, const void* kpe, const int32_t* idx,
                int64_t num_tokens, int64_t num_pages, float sm_scale, void* output, float* lse, void* workspace,
                size_t workspace_bytes, void* stream_ptr, void* const* events, const PagedIndex* paged,
                const void* kv_fp8, size_t clear_bytes);

namespace {

// Enough for a split grid of up to 160 CTAs (B200 has 148 SMs): 10.04 MiB.
constexpr int kNoAllocMaxGrid = 160;
constexpr size_t kNoAllocScratchBytes = workspace_bytes_for_grid(kNoAllocMaxGrid);

// In host code this name is only a host-side stand-in for the device array;
// its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu[kMaxDevices];
void* g_scratch_ptr[kMaxDevices];   // set once a lookup on that device succeeded

// Device address of the array on device `dev` (current), looked up on the
// first call that needs it; a failed lookup is not remembered, so a later
// call tries again.
void* scratch_on(int dev) {
  std::lock_guard<std::mutex> lock(g_mu[dev]);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
      cudaGetLastError();   // leave no sticky error behind for the caller
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace dsa

extern "C" int dsa_sparse_attention_fwd_noalloc(const void* q_nope, const void* q_pe, const void* ckv_cache,
                                                const void* kpe_cache, const int32_t* sparse_indices,
                                                int64_t num_tokens, int64_t num_pages, float sm_scale,
                                                void* output, float* lse, void* stream) {
  using namespace dsa;
  if (num_tokens < 0 || num_tokens > (int64_t(1) << 24)) return DSA_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return DSA_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return DSA_ERR_UNSUPPORTED_DEVICE;
  // The grid (and so the scratch this call needs) follows the device's SM count.
  const size_t need = dsa_sparse_attention_workspace_size(num_tokens);
  if (need == 0) return DSA_ERR_CUDA;
  if (need > kNoAllocScratchBytes) return DSA_ERR_WORKSPACE_TOO_SMALL;
  // With this device current: the device address of the array.
  void* scratch = scratch_on(dev);
  if (scratch == nullptr) return DSA_ERR_CUDA;
  // The error word and the arrival counters must start at zero; the array keeps
  // whatever the previous call left, so that part is cleared (one memset on
  // `stream`, issued only once every argument has passed its checks).
  return fwd_impl_ex(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, num_tokens, num_pages, sm_scale, output,
                     lse, scratch, kNoAllocScratchBytes, stream, nullptr, nullptr, nullptr, kWorkspaceRecordsOffset);
}

// The device findings of the no-alloc calls on the current device: the same
// read (and clear) as dsa_sparse_attention_read_errors, on the library's own
// array, which the caller cannot address.
extern "C" int dsa_sparse_attention_noalloc_read_errors(void* stream, uint32_t* device_flags) {
  using namespace dsa;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return DSA_ERR_UNSUPPORTED_DEVICE;
  void* scratch = scratch_on(dev);
  if (scratch == nullptr) return DSA_ERR_CUDA;
  return dsa_sparse_attention_read_errors(scratch, stream, device_flags);
}
