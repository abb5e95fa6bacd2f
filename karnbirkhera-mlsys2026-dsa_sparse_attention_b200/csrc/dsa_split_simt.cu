// dsa_split_simt.cu — correctness-first split-KV kernel on CUDA cores.
//
// Same work plan, masking rules and partial-record format as the tcgen05
// kernel (dsa_split_sm100.cu); it exists as the first end-to-end path and as a
// GPU-side cross-check of the plan and merge logic.  One CTA of 256 threads
// per plan range; each 128-slot block is processed as two 64-row halves:
//   1. stage the half's indices in shared memory (validated: -1 or
//      [0, num_slots); anything else raises DSA_DEVICE_ERR_BAD_INDEX and is
//      treated as padding),
//   2. copy the 64 gathered rows (ckv 1024 B + kpe 128 B) with 16-byte loads,
//      zero rows for padding,
//   3. logits in fp32 (thread = head x 4 rows),
//   4. exact online softmax per head in the log2 domain,
//   5. o += p * ckv (thread = 2 output columns x 16 heads).
#include <cuda_bf16.h>

#include "dsa_common.cuh"

namespace dsa {

namespace simt {
constexpr int kThreads = 256;
constexpr int kRows = 64;                  // rows per half block
constexpr int kQStride = kQk + 4;          // fp32 elements per Q row (bank padding)
constexpr int kKStride = kQk + 8;          // bf16 elements per staged row (bank padding)
constexpr int kSStride = kRows + 1;

constexpr size_t kQBytes = size_t(kHeads) * kQStride * 4;
constexpr size_t kKBytes = size_t(kRows) * kKStride * 2;
constexpr size_t kSBytes = size_t(kHeads) * kSStride * 4;
constexpr size_t kPBytes = size_t(kRows) * kHeads * 4;
constexpr size_t kSmemBytes = kQBytes + kKBytes + kSBytes + kPBytes + 3 * kHeads * 4 + kRows * 4;
}  // namespace simt

__global__ __launch_bounds__(simt::kThreads, 1) void split_simt_kernel(SplitParams prm) {
  using namespace simt;
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ __align__(16) uint8_t smem[];
  float* q_s = reinterpret_cast<float*>(smem);
  __nv_bfloat16* k_s = reinterpret_cast<__nv_bfloat16*>(smem + kQBytes);
  float* s_s = reinterpret_cast<float*>(smem + kQBytes + kKBytes);
  float* p_s = reinterpret_cast<float*>(smem + kQBytes + kKBytes + kSBytes);
  float* m_s = p_s + kRows * kHeads;
  float* l_s = m_s + kHeads;
  float* a_s = l_s + kHeads;
  int* idx_s = reinterpret_cast<int*>(a_s + kHeads);

  const __nv_bfloat16* q_nope = static_cast<const __nv_bfloat16*>(prm.q_nope);
  const __nv_bfloat16* q_pe = static_cast<const __nv_bfloat16*>(prm.q_pe);
  const __nv_bfloat16* ckv = static_cast<const __nv_bfloat16*>(prm.ckv);
  const __nv_bfloat16* kpe = static_cast<const __nv_bfloat16*>(prm.kpe);
  __nv_bfloat16* output = static_cast<__nv_bfloat16*>(prm.output);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t g_begin = plan_range_begin(prm.plan, blockIdx.x);
  const int64_t g_end = plan_range_begin(prm.plan, int64_t(blockIdx.x) + 1);

  for (int64_t g = g_begin; g < g_end;) {
    const int64_t t = g / kBlocksPerToken;
    const int64_t seg_end = min(g_end, (t + 1) * kBlocksPerToken);
    const bool full = (g == t * kBlocksPerToken) && (seg_end == (t + 1) * kBlocksPerToken);

    // Q of token t -> fp32 shared memory.
    for (int e = tid; e < kHeads * kQk; e += kThreads) {
      const int h = e / kQk, d = e % kQk;
      const __nv_bfloat16 v = d < kCkv ? q_nope[(t * kHeads + h) * kCkv + d]
                                       : q_pe[(t * kHeads + h) * kKpe + (d - kCkv)];
      q_s[h * kQStride + d] = __bfloat162float(v);
    }
    if (tid < kHeads) {
      m_s[tid] = -INFINITY;
      l_s[tid] = 0.f;
    }
    float acc[kHeads][2];
#pragma unroll
    for (int h = 0; h < kHeads; ++h) acc[h][0] = acc[h][1] = 0.f;
    __syncthreads();

    for (int64_t blk = g; blk < seg_end; ++blk) {
      for (int half = 0; half < 2; ++half) {
        const int key0 = int(blk % kBlocksPerToken) * kBlockKeys + half * kRows;
        if (tid < kRows) {
          const int32_t v = prm.indices[t * kTopk + key0 + tid];
          const bool ok = v >= 0 && int64_t(v) < prm.num_slots;
          if (!ok && v != -1) report_error(prm.err_word, DSA_DEVICE_ERR_BAD_INDEX);
          idx_s[tid] = ok ? v : -1;
        }
        __syncthreads();
        // Gather: 64 rows x 72 16-byte chunks (64 ckv + 8 kpe).
        for (int c = tid; c < kRows * (kQk / 8); c += kThreads) {
          const int row = c / (kQk / 8), ch = c % (kQk / 8);
          const int32_t slot = idx_s[row];
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (slot >= 0) {
            const __nv_bfloat16* src = ch < kCkv / 8 ? ckv + int64_t(slot) * kCkv + ch * 8
                                                     : kpe + int64_t(slot) * kKpe + (ch - kCkv / 8) * 8;
            v = __ldg(reinterpret_cast<const uint4*>(src));
          }
          *reinterpret_cast<uint4*>(k_s + row * kKStride + ch * 8) = v;
        }
        __syncthreads();
        // Logits: thread -> head h, rows j0 + 16 m.
        {
          const int h = tid >> 4, j0 = tid & 15;
          const float* qh = q_s + h * kQStride;
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const int j = j0 + 16 * m;
            const __nv_bfloat162* kr = reinterpret_cast<const __nv_bfloat162*>(k_s + j * kKStride);
            float dot = 0.f;
#pragma unroll 8
            for (int d2 = 0; d2 < kQk / 2; ++d2) {
              const float2 kv = __bfloat1622float2(kr[d2]);
              dot = fmaf(qh[2 * d2], kv.x, dot);
              dot = fmaf(qh[2 * d2 + 1], kv.y, dot);
            }
            s_s[h * kSStride + j] = idx_s[j] >= 0 ? dot * prm.scale_log2 : -INFINITY;
          }
        }
        __syncthreads();
        // Online softmax: warp w owns heads 2w and 2w+1.
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int h = 2 * warp + hh;
          const float a = s_s[h * kSStride + lane];
          const float c = s_s[h * kSStride + lane + 32];
          float mx = fmaxf(a, c);
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
          const float m_old = m_s[h];
          const float m_new = fmaxf(m_old, mx);
          float pa = 0.f, pc = 0.f, alpha = 1.f;
          if (m_new != -INFINITY) {
            alpha = (m_old == -INFINITY) ? 0.f : exp2f(m_old - m_new);
            pa = exp2f(a - m_new);
            pc = exp2f(c - m_new);
          }
          p_s[lane * kHeads + h] = pa;
          p_s[(lane + 32) * kHeads + h] = pc;
          float sum = pa + pc;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
          __syncwarp();
          if (lane == 0) {
            l_s[h] = l_s[h] * alpha + sum;
            m_s[h] = m_new;
            a_s[h] = alpha;
          }
        }
        __syncthreads();
        // o += p * ckv: thread owns output columns 2*tid, 2*tid+1.
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          const float al = a_s[h];
          acc[h][0] *= al;
          acc[h][1] *= al;
        }
        for (int j = 0; j < kRows; ++j) {
          const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(k_s + j * kKStride + 2 * tid));
          const float4* pj = reinterpret_cast<const float4*>(p_s + j * kHeads);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const float4 p = pj[q4];
            acc[4 * q4 + 0][0] = fmaf(p.x, v.x, acc[4 * q4 + 0][0]);
            acc[4 * q4 + 0][1] = fmaf(p.x, v.y, acc[4 * q4 + 0][1]);
            acc[4 * q4 + 1][0] = fmaf(p.y, v.x, acc[4 * q4 + 1][0]);
            acc[4 * q4 + 1][1] = fmaf(p.y, v.y, acc[4 * q4 + 1][1]);
            acc[4 * q4 + 2][0] = fmaf(p.z, v.x, acc[4 * q4 + 2][0]);
            acc[4 * q4 + 2][1] = fmaf(p.z, v.y, acc[4 * q4 + 2][1]);
            acc[4 * q4 + 3][0] = fmaf(p.w, v.x, acc[4 * q4 + 3][0]);
            acc[4 * q4 + 3][1] = fmaf(p.w, v.y, acc[4 * q4 + 3][1]);
          }
        }
        __syncthreads();
      }
    }

    // Segment epilogue.
    if (full) {
      __nv_bfloat16* out_t = output + t * (kHeads * kCkv);
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        const float l = l_s[h];
        const float il = l > 0.f ? 1.f / l : 0.f;
        *reinterpret_cast<__nv_bfloat162*>(out_t + h * kCkv + 2 * tid) =
            __floats2bfloat162_rn(acc[h][0] * il, acc[h][1] * il);
      }
      if (tid < kHeads) {
        const float l = l_s[tid];
        prm.lse[t * kHeads + tid] = l > 0.f ? m_s[tid] + log2f(l) : -INFINITY;
      }
    } else {
      RecordView r = record_at(prm.records, plan_record_slot(prm.plan, blockIdx.x, t));
#pragma unroll
      for (int h = 0; h < kHeads; ++h)
        *reinterpret_cast<float2*>(r.o + h * kCkv + 2 * tid) = make_float2(acc[h][0], acc[h][1]);
      if (tid < kHeads) {
        r.m[tid] = m_s[tid];
        r.l[tid] = l_s[tid];
      }
    }
    __syncthreads();
    g = seg_end;
  }
}

cudaError_t launch_split_simt(const SplitParams& prm, cudaStream_t stream) {
  static_assert(simt::kSmemBytes <= 227 * 1024, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(split_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(simt::kSmemBytes));
  if (e != cudaSuccess) return e;
  split_simt_kernel<<<prm.plan.grid, simt::kThreads, simt::kSmemBytes, stream>>>(prm);
  return cudaGetLastError();
}

}  // namespace dsa
