// dsa_merge.cu — combines the partial records of tokens that the split-KV
// kernel spread over several CTAs, and writes their bf16 output and base-2 lse.
//
// Merge rule (the split-KV combine of the reference's fused last-arrival
// reduce, solution/cuda/kernel.cu:433-509, restated in the log2 domain):
//   M      = max_s m_s
//   w_s    = 2^(m_s - M)                  (0 for an empty segment)
//   L      = sum_s w_s * l_s
//   out    = sum_s w_s * o_s / L          (0 when L == 0)
//   lse    = M + log2(L)                  (-inf when L == 0)
//
// Grid: one CTA per CTA boundary b = 1..G-1 of the plan.  The CTA of the first
// boundary that falls strictly inside a token merges that token; every other
// CTA exits at once.  Launched with programmatic dependent launch so its launch
// overlaps the tail of the split kernel; griddepcontrol.wait orders its reads
// after the split kernel's writes.
#include <cuda_bf16.h>

#include "dsa_common.cuh"

namespace dsa {

constexpr int kMergeThreads = 256;
constexpr int kMaxSegments = kBlocksPerToken;  // a token's 16 blocks span at most 16 CTAs

__global__ __launch_bounds__(kMergeThreads) void merge_kernel(Plan plan, const float* __restrict__ records,
                                                              __nv_bfloat16* __restrict__ output,
                                                              float* __restrict__ lse) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t b = int64_t(blockIdx.x) + 1;
  const int64_t g = plan_range_begin(plan, b);
  if (g % kBlocksPerToken == 0) return;
  const int64_t t = g / kBlocksPerToken;
  if (b > 1) {
    const int64_t gp = plan_range_begin(plan, b - 1);
    if (gp / kBlocksPerToken == t && gp % kBlocksPerToken != 0) return;
  }
  const int64_t b_lo = plan_owner(plan, t * kBlocksPerToken);
  const int64_t b_hi = plan_owner(plan, t * kBlocksPerToken + kBlocksPerToken - 1);
  const int nseg = int(b_hi - b_lo + 1);

  __shared__ float w_s[kMaxSegments][kHeads];
  __shared__ float m_s[kMaxSegments][kHeads];
  __shared__ float l_s[kMaxSegments][kHeads];
  __shared__ float inv_l_s[kHeads];
  __shared__ const float* rec_s[kMaxSegments];
  const int tid = threadIdx.x;
  if (tid < nseg) rec_s[tid] = records + plan_record_slot(plan, b_lo + tid, t) * kRecordFloats;
  __syncthreads();
  // all (segment, head) statistics in one round of loads
  if (tid < nseg * kHeads) {
    const int s = tid / kHeads, h = tid % kHeads;
    m_s[s][h] = rec_s[s][h];
    l_s[s][h] = rec_s[s][kHeads + h];
  }
  __syncthreads();
  if (tid < kHeads) {
    const int h = tid;
    float M = -INFINITY;
    for (int s = 0; s < nseg; ++s) M = fmaxf(M, m_s[s][h]);
    float L = 0.f;
    for (int s = 0; s < nseg; ++s) {
      const float w = (M == -INFINITY) ? 0.f : exp2f(m_s[s][h] - M);
      w_s[s][h] = w;
      L += w * l_s[s][h];
    }
    inv_l_s[h] = (L > 0.f) ? 1.f / L : 0.f;
    lse[t * kHeads + h] = (L > 0.f) ? (M + log2f(L)) : -INFINITY;
  }
  __syncthreads();

  // 16*512 outputs as 2048 float4 groups; thread tid handles groups tid + 256k.
  __nv_bfloat16* out_t = output + t * (kHeads * kCkv);
  float4 acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
  for (int s = 0; s < nseg; ++s) {
    const float4* o = reinterpret_cast<const float4*>(rec_s[s] + 2 * kHeads);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int e = tid + k * kMergeThreads;  // float4 index; head = e / 128
      const float w = w_s[s][e / (kCkv / 4)];
      const float4 v = o[e];
      acc[k].x += w * v.x;
      acc[k].y += w * v.y;
      acc[k].z += w * v.z;
      acc[k].w += w * v.w;
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int e = tid + k * kMergeThreads;
    const float il = inv_l_s[e / (kCkv / 4)];
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc[k].x * il, acc[k].y * il);
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc[k].z * il, acc[k].w * il);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&lo);
    packed.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(out_t)[e] = packed;
  }
}

// Enqueue the merge after the split kernel on `stream`.  Nothing to do when
// the plan has a single CTA or every token is owned by one CTA (the kernel
// exits early for those boundaries anyway).
cudaError_t launch_merge(const Plan& plan, const float* records, __nv_bfloat16* output, float* lse,
                         cudaStream_t stream) {
  if (plan.grid <= 1) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(plan.grid - 1));
  cfg.blockDim = dim3(kMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, merge_kernel, plan, records, output, lse);
}

}  // namespace dsa
