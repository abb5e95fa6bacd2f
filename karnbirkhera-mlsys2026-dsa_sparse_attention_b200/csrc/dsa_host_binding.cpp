// dsa_host_binding.cpp — a C++ fast path for the Python entry point
// launch_sparse_attention_c (the reference's launcher is C++ bound with
// pybind, solution/cuda/kernel.cu:673-729): the same argument checks as the
// Python layer, done on at::Tensor, then one call of the C ABI's
// dsa_sparse_attention_fwd on the current stream.  The C ABI function is
// handed over by address (set_fwd) from the library the package already
// loaded, so this module has no link dependency on it.
//
// fwd() returns the C ABI status (>= 0) or -1 when an argument check fails;
// the Python layer then runs its own checker, which raises with the message.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdint>

namespace {

using FwdFn = int (*)(const void*, const void*, const void*, const void*, const int32_t*, int64_t, int64_t, float,
                      void*, float*, void*, size_t, void*);
FwdFn g_fwd = nullptr;

constexpr int64_t kHeads = 16, kCkv = 512, kKpe = 64, kPage = 64, kTopk = 2048;

// CUDA, contiguous, 16-byte aligned, on device `dev` (-1: take this one's)
bool usable(const at::Tensor& t, int64_t& dev) {
  if (!t.defined() || !t.is_cuda() || !t.is_contiguous()) return false;
  if (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) return false;
  const int64_t d = t.get_device();
  if (dev < 0) dev = d;
  return d == dev;
}

bool shaped(const at::Tensor& t, at::ScalarType dt, std::initializer_list<int64_t> shape) {
  if (t.scalar_type() != dt || t.dim() != int64_t(shape.size())) return false;
  int64_t i = 0;
  for (int64_t s : shape)
    if (t.size(i++) != s) return false;
  return true;
}

int fwd(const at::Tensor& q_nope, const at::Tensor& q_pe, const at::Tensor& ckv, const at::Tensor& kpe,
        const at::Tensor& idx, double sm_scale, const at::Tensor& out, const at::Tensor& lse, const at::Tensor& ws) {
  if (g_fwd == nullptr) return -1;
  int64_t dev = -1;
  for (const at::Tensor* t : {&q_nope, &q_pe, &ckv, &kpe, &idx, &out, &lse})
    if (!usable(*t, dev)) return -1;
  if (q_nope.dim() != 3 || ckv.dim() != 3) return -1;
  const int64_t n = q_nope.size(0), p = ckv.size(0);
  if (!shaped(q_nope, at::kBFloat16, {n, kHeads, kCkv}) || !shaped(q_pe, at::kBFloat16, {n, kHeads, kKpe}) ||
      !shaped(ckv, at::kBFloat16, {p, kPage, kCkv}) || !shaped(kpe, at::kBFloat16, {p, kPage, kKpe}) ||
      !shaped(idx, at::kInt, {n, kTopk}) || !shaped(out, at::kBFloat16, {n, kHeads, kCkv}) ||
      !shaped(lse, at::kFloat, {n, kHeads}))
    return -1;
  if (n == 0) return 0;
  if (!ws.defined() || !ws.is_cuda() || ws.get_device() != dev) return -1;
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(dev));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(dev)).stream();
  return g_fwd(q_nope.data_ptr(), q_pe.data_ptr(), ckv.data_ptr(), kpe.data_ptr(),
               static_cast<const int32_t*>(idx.data_ptr()), n, p, static_cast<float>(sm_scale), out.data_ptr(),
               static_cast<float*>(lse.data_ptr()), ws.data_ptr(), static_cast<size_t>(ws.numel()), stream);
}

void set_fwd(uint64_t address) { g_fwd = reinterpret_cast<FwdFn>(static_cast<uintptr_t>(address)); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("fwd", &fwd, "launch_sparse_attention_c: checks, then dsa_sparse_attention_fwd on the current stream");
  m.def("set_fwd", &set_fwd, "address of the C ABI's dsa_sparse_attention_fwd");
}
