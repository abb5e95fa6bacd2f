// Force-included header used ONLY by oracle/build_ref.py when it compiles the
// reference's naive ATen kernel (methodology/checkpoints/kernel_naive.cu) as a
// CPU Python extension.  Test infrastructure, never shipped.
//
// kernel_naive.cu:31 opens an `at::cuda::CUDAGuard` on q_nope's device, which
// throws for CPU tensors.  Everything else in that file is plain ATen and runs
// on CPU unchanged.  This header pulls in the CUDA headers the file includes
// (so their include guards are already set), then renames the guard type to a
// no-op guard of our own.  No line of the reference source is altered.
#pragma once
#include <torch/extension.h>
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

namespace at {
namespace cuda {
struct OracleCpuDeviceGuard {
  explicit OracleCpuDeviceGuard(c10::Device) {}
};
}  // namespace cuda
}  // namespace at

#define CUDAGuard OracleCpuDeviceGuard
