// dsa_split_sm100.cu — the split-KV kernel on the sm_100a tensor cores.
//
// One persistent CTA per SM walks its range of the static plan (dsa_common.cuh)
// one 128-slot block ("tile") at a time.  Per tile:
//   gather   TMA tile::gather4 copies the 128 selected rows, 128 bytes per
//            row and request, into 128-byte-swizzled shared memory: the ckv
//            row (1024 B) as 8 chunks of 64 columns, the kpe row as 1 chunk.
//            Padding (-1) and out-of-range slots are sent to row `num_slots`,
//            which the tensor map zero-fills without touching HBM.
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
//            base-2 lse, or an fp32 partial record for the merge kernel.
//
// Warp roles (192 threads): warp 0 issues TMA (all 32 lanes, 4 rows each),
// warp 1 lane 0 issues tcgen05.mma/commit and owns the TMEM allocation,
// warps 2..5 run softmax and the epilogue.
//
// Shared memory (bytes, 1024-aligned): Q 9x2 KB | kpe 2x16 KB | ckv slabs
// 5x32 KB (a slab = ckv columns [128j, 128j+128) of one tile) | P 2x4 KB |
// reduction scratch | mbarriers.  The 5-slab ring lets the next tile's first
// slab and kpe land while the current tile computes; the current tile's slabs
// are released one by one as its PV MMAs retire.
//
// Every wait is bounded (DSA_DEVICE_ERR_TIMEOUT on expiry); the kernel then
// drains its own copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "dsa_common.cuh"
#include "dsa_sm100_ptx.cuh"

namespace dsa {
namespace sm100 {

using namespace ptx;

constexpr int kThreads = 192;
constexpr int kSoftmaxWarp0 = 2;
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
constexpr uint32_t kOffBar = kOffRedL + 4 * 16 * 4;

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
  B_DONE,
  B_COUNT
};

constexpr uint32_t kOffMisc = kOffBar + B_COUNT * 8;   // tmem base, abort flag
constexpr uint32_t kSmemBytes = kOffMisc + 16 + 1024;  // + slack for 1024-B alignment
static_assert(kOffSlab % 1024 == 0 && kOffKpe % 1024 == 0 && kOffP % 1024 == 0, "swizzle atoms need 1 KB");
static_assert(kSmemBytes <= 232448, "shared memory budget of one CTA");

constexpr uint32_t kTmemCols = 128;   // S[2] at columns 0/16, O blocks at 32 + 16 j
constexpr uint32_t kTmemO = 32;

constexpr float kRescaleThreshold = 8.0f;   // log2 units

struct Ctx {
  uint32_t sbase;          // shared address of the aligned base
  uint32_t tmem;           // TMEM base address
  volatile uint32_t* abort;
  float* red;
  float* red_l;
  uint64_t timeout_ns;
  int64_t g_begin, g_end;  // plan range of this CTA
};

__device__ __forceinline__ uint32_t bar_addr(const Ctx& c, int b) { return c.sbase + kOffBar + 8u * uint32_t(b); }

// All 128 softmax threads agree on `ok` (barrier 2 with an AND reduction).
__device__ __forceinline__ bool group_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(ok))
      : "memory");
  return r != 0;
}

// Producer waits: lane 0 polls, the whole warp follows its verdict.
__device__ __forceinline__ bool warp_wait(const Ctx& c, int b, uint32_t parity) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar_addr(c, b), parity, c.abort, c.timeout_ns);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Wait used only while draining after an abort (ignores the abort flag).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > timeout_ns) return;
  }
}

// -------------------------------------------------------------------------
// warp 0: TMA producer
// -------------------------------------------------------------------------
__device__ void producer(const Ctx& c, const SplitParams& prm, const CUtensorMap* tm_ckv, const CUtensorMap* tm_kpe,
                         const CUtensorMap* tm_qn, const CUtensorMap* tm_qp) {
  const int lane = threadIdx.x & 31;
  const uint32_t sQ = c.sbase + kOffQ, sKpe = c.sbase + kOffKpe, sSlab = c.sbase + kOffSlab;
  const int oob = int(prm.num_slots);   // first row past the tensor: zero-filled by TMA
  int64_t i = 0, u = 0;
  int seg = 0;
  bool ok = true;
  // index prefetch: lane l holds slots 4l..4l+3 of the next tile
  auto load_idx = [&](int64_t g) -> int4 {
    const int64_t t = g / kBlocksPerToken;
    const int32_t* row = prm.indices + t * kTopk + (g % kBlocksPerToken) * kBlockKeys + 4 * lane;
    return __ldg(reinterpret_cast<const int4*>(row));
  };
  int4 nxt = c.g_begin < c.g_end ? load_idx(c.g_begin) : make_int4(0, 0, 0, 0);
  uint32_t bad = 0;
  // last issue into each buffer (for the drain after an abort)
  int last_q = -1;
  int64_t last_kpe[2] = {-1, -1};
  int64_t last_slab[kSlabs] = {-1, -1, -1, -1, -1};
  for (int64_t gs = c.g_begin; gs < c.g_end && ok;) {
    const int64_t t = gs / kBlocksPerToken;
    const int64_t ge = min(c.g_end, (t + 1) * kBlocksPerToken);
    if (seg > 0 && !(ok = warp_wait(c, B_Q_EMPTY, uint32_t(seg - 1) & 1u))) break;
    if (lane == 0) {
      const uint32_t qb = bar_addr(c, B_Q_FULL);
      mbar_arrive_expect_tx(qb, kQBytes);
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) tma_load_2d(sQ + ch * kQChunkBytes, tm_qn, 64 * ch, int(t * kHeads), qb);
      tma_load_2d(sQ + 8 * kQChunkBytes, tm_qp, 0, int(t * kHeads), qb);
    }
    last_q = seg;
    __syncwarp();
    for (int64_t blk = gs; blk < ge && ok; ++blk, ++i) {
      const int4 cur = nxt;
      if (blk + 1 < c.g_end) nxt = load_idx(blk + 1);
      int4 rows;
      {
        const int v[4] = {cur.x, cur.y, cur.z, cur.w};
        int o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const bool valid = v[k] >= 0 && int64_t(v[k]) < prm.num_slots;
          bad |= (!valid && v[k] != -1) ? 1u : 0u;
          o[k] = valid ? v[k] : oob;
        }
        rows = make_int4(o[0], o[1], o[2], o[3]);
      }
      const int kb = int(i & 1);
      if (i >= 2 && !(ok = warp_wait(c, B_KPE_EMPTY + kb, (uint32_t(i >> 1) & 1u) ^ 1u))) break;
      if (lane == 0) mbar_arrive_expect_tx(bar_addr(c, B_KPE_FULL + kb), kChunkBytes);
      __syncwarp();
      tma_gather4(sKpe + kb * kChunkBytes + lane * 512u, tm_kpe, 0, rows, bar_addr(c, B_KPE_FULL + kb));
      last_kpe[kb] = i;
#pragma unroll 1
      for (int j = 0; j < 4; ++j, ++u) {
        const int slot = int(u % kSlabs);
        if (u >= kSlabs && !(ok = warp_wait(c, B_SLAB_EMPTY + slot, (uint32_t(u / kSlabs) & 1u) ^ 1u))) break;
        const uint32_t fb = bar_addr(c, B_SLAB_FULL + slot);
        if (lane == 0) mbar_arrive_expect_tx(fb, kSlabBytes);
        __syncwarp();
        const uint32_t dst = sSlab + slot * kSlabBytes + lane * 512u;
        tma_gather4(dst, tm_ckv, 128 * j, rows, fb);
        tma_gather4(dst + kChunkBytes, tm_ckv, 128 * j + 64, rows, fb);
        last_slab[slot] = u;
      }
    }
    ++seg;
    gs = ge;
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) report_error(prm.err_word, DSA_DEVICE_ERR_BAD_INDEX);
  // After an abort, every copy this warp issued must land before the CTA exits.
  if (lane == 0 && *c.abort) {
    const uint64_t to = c.timeout_ns;
    if (last_q >= 0) drain_wait(bar_addr(c, B_Q_FULL), uint32_t(last_q) & 1u, to);
    for (int kb = 0; kb < 2; ++kb)
      if (last_kpe[kb] >= 0) drain_wait(bar_addr(c, B_KPE_FULL + kb), uint32_t(last_kpe[kb] >> 1) & 1u, to);
    for (int s = 0; s < kSlabs; ++s)
      if (last_slab[s] >= 0) drain_wait(bar_addr(c, B_SLAB_FULL + s), uint32_t(last_slab[s] / kSlabs) & 1u, to);
  }
}

// -------------------------------------------------------------------------
// warp 1, lane 0: tcgen05.mma issuer
// -------------------------------------------------------------------------
struct PendingPV {
  int64_t i;
  int seg;
  bool first, last;
};

__device__ void mma_issuer(const Ctx& c) {
  const uint32_t sQ = c.sbase + kOffQ, sKpe = c.sbase + kOffKpe, sSlab = c.sbase + kOffSlab,
                 sP = c.sbase + kOffP;
  constexpr uint32_t idesc_qk = idesc_bf16_f32(128, 16, false, false);
  constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 16, true, false);
  bool ok = true;

  auto wait = [&](int b, uint32_t parity) -> bool {
    ok = mbar_wait(bar_addr(c, b), parity, c.abort, c.timeout_ns);
    return ok;
  };
  // logits MMAs of ckv slab j of tile i (columns 128j .. 128j+127)
  auto qk_slab = [&](int64_t i, int j) -> bool {
    const int64_t u = 4 * i + j;
    const int slot = int(u % kSlabs);
    if (!wait(B_SLAB_FULL + slot, uint32_t(u / kSlabs) & 1u)) return false;
    tc_fence_after();
    const uint32_t d = c.tmem + 16u * uint32_t(i & 1);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t a0 = sSlab + slot * kSlabBytes + half * kChunkBytes;
      const uint32_t b0 = sQ + (2 * j + half) * kQChunkBytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_bf16(d, smem_desc_sw128(a0 + 32 * kk, 16, 1024), smem_desc_sw128(b0 + 32 * kk, 16, 1024), idesc_qk, 1);
    }
    return true;
  };
  auto pv = [&](const PendingPV& p) -> bool {
    const int pb = int(p.i & 1);
    if (!wait(B_P_FULL + pb, uint32_t(p.i >> 1) & 1u)) return false;
    if (p.first && p.seg > 0 && !wait(B_O_EMPTY, uint32_t(p.seg - 1) & 1u)) return false;
    tc_fence_after();
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      const int slot = int((4 * p.i + j) % kSlabs);
      const uint32_t a0 = sSlab + slot * kSlabBytes;
      const uint32_t d = c.tmem + kTmemO + 16u * j;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t a = smem_desc_sw128(a0 + 2048u * kk, kChunkBytes, 1024);   // MN-major: LBO = chunk stride
        const uint64_t b = smem_desc_sw128(sP + pb * kPBytes + (kk >> 2) * 2048u + (kk & 3) * 32u, 16, 1024);
        mma_bf16(d, a, b, idesc_pv, (p.first && kk == 0) ? 0u : 1u);
      }
      mma_commit(bar_addr(c, B_SLAB_EMPTY + slot));
    }
    mma_commit(bar_addr(c, B_P_EMPTY + pb));
    if (p.last) mma_commit(bar_addr(c, B_O_FULL));
    return true;
  };

  int64_t i = 0;
  int seg = 0;
  PendingPV pend{0, 0, false, false};
  bool have_pend = false;
  for (int64_t gs = c.g_begin; gs < c.g_end && ok;) {
    const int64_t t = gs / kBlocksPerToken;
    const int64_t ge = min(c.g_end, (t + 1) * kBlocksPerToken);
    if (!wait(B_Q_FULL, uint32_t(seg) & 1u)) break;
    for (int64_t blk = gs; blk < ge; ++blk, ++i) {
      const int sb = int(i & 1);
      if (i >= 2 && !wait(B_S_EMPTY + sb, (uint32_t(i >> 1) & 1u) ^ 1u)) break;
      if (!wait(B_KPE_FULL + sb, uint32_t(i >> 1) & 1u)) break;
      tc_fence_after();
      {
        const uint32_t d = c.tmem + 16u * uint32_t(sb);
        const uint32_t a0 = sKpe + sb * kChunkBytes, b0 = sQ + 8 * kQChunkBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(d, smem_desc_sw128(a0 + 32 * kk, 16, 1024), smem_desc_sw128(b0 + 32 * kk, 16, 1024), idesc_qk,
                   kk > 0 ? 1u : 0u);
        mma_commit(bar_addr(c, B_KPE_EMPTY + sb));
      }
      if (!qk_slab(i, 0)) break;
      if (have_pend) {
        if (!pv(pend)) break;
        have_pend = false;
      }
      if (!qk_slab(i, 1) || !qk_slab(i, 2) || !qk_slab(i, 3)) break;
      mma_commit(bar_addr(c, B_S_FULL + sb));
      const bool last = (blk + 1 == ge);
      if (last) mma_commit(bar_addr(c, B_Q_EMPTY));
      pend = PendingPV{i, seg, blk == gs, last};
      have_pend = true;
    }
    ++seg;
    gs = ge;
  }
  if (ok && have_pend) pv(pend);
  // every MMA issued must retire before TMEM is freed
  mma_commit(bar_addr(c, B_DONE));
  drain_wait(bar_addr(c, B_DONE), 0u, c.timeout_ns);
}

// -------------------------------------------------------------------------
// warps 2..5: softmax + epilogue
// -------------------------------------------------------------------------
__device__ void softmax_epilogue(const Ctx& c, const SplitParams& prm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wq = warp & 3;              // TMEM lanes 32*wq .. 32*wq+31 belong to this warp
  const int r = 32 * wq + lane;         // key row of a tile / dim row of an O block
  const uint32_t t_lane = uint32_t(32 * wq) << 16;
  const bool leader = (warp == kSoftmaxWarp0 && lane == 0);
  const uint32_t sP = c.sbase + kOffP;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(prm.output);

  int64_t i = 0;
  int seg = 0;
  bool ok = true;
  for (int64_t gs = c.g_begin; gs < c.g_end && ok;) {
    const int64_t t = gs / kBlocksPerToken;
    const int64_t ge = min(c.g_end, (t + 1) * kBlocksPerToken);
    const bool full = (gs == t * kBlocksPerToken) && (ge == (t + 1) * kBlocksPerToken);
    float m_run[16], l_part[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      m_run[h] = -INFINITY;
      l_part[h] = 0.f;
    }
    for (int64_t blk = gs; blk < ge; ++blk, ++i) {
      const int32_t kidx = __ldg(prm.indices + t * kTopk + (blk % kBlocksPerToken) * kBlockKeys + r);
      const bool valid = kidx >= 0 && int64_t(kidx) < prm.num_slots;
      const int sb = int(i & 1);
      if (!(ok = group_all(mbar_wait(bar_addr(c, B_S_FULL + sb), uint32_t(i >> 1) & 1u, c.abort, c.timeout_ns))))
        break;
      tc_fence_after();
      float x[16];
      tmem_ld16(c.tmem + t_lane + 16u * uint32_t(sb), x);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar_addr(c, B_S_EMPTY + sb));
#pragma unroll
      for (int h = 0; h < 16; ++h) x[h] = valid ? x[h] * prm.scale_log2 : -INFINITY;
      // per-head max over the 128 keys of the tile
      float mx[16];
#pragma unroll
      for (int h = 0; h < 16; ++h) mx[h] = x[h];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int h = 0; h < 16; ++h) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
      float* red = c.red + sb * 64;
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < 16; h += 4) *reinterpret_cast<float4*>(red + wq * 16 + h) = make_float4(mx[h], mx[h + 1], mx[h + 2], mx[h + 3]);
      }
      named_barrier_sync(1, kSoftmaxThreads);
      float alpha[16];
      bool any_rescale = false;
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
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        alpha[h] = 1.f;
        if (mx[h] > m_run[h] + kRescaleThreshold) {
          if (m_run[h] != -INFINITY) {
            alpha[h] = exp2f(m_run[h] - mx[h]);
            any_rescale = true;
          }
          m_run[h] = mx[h];
        }
        l_part[h] *= alpha[h];
      }
      if (any_rescale) {
        // O holds the previous tiles of this segment: let their PV retire, then scale in place.
        if (!(ok = group_all(mbar_wait(bar_addr(c, B_P_EMPTY + int((i - 1) & 1)), uint32_t((i - 1) >> 1) & 1u,
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
      if (i >= 2 && !(ok = group_all(mbar_wait(bar_addr(c, B_P_EMPTY + sb), (uint32_t(i >> 1) & 1u) ^ 1u,
                                                c.abort, c.timeout_ns))))
        break;
      // P^T (bf16) into the K-major 128-byte-swizzled B operand: row = head, 64 keys per 128-byte row
      {
        const uint32_t kc = uint32_t(r >> 6), e = uint32_t(r & 63);
        const uint32_t base = sP + sb * kPBytes + kc * 2048u;
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          const float p = (m_run[h] == -INFINITY) ? 0.f : exp2f(x[h] - m_run[h]);
          l_part[h] += p;
          const uint32_t hr = uint32_t(h & 7);
          const uint32_t addr = base + uint32_t(h >> 3) * 1024u + hr * 128u + ((((e >> 3) ^ hr) << 4) | ((e & 7) << 1));
          const __nv_bfloat16 pb = __float2bfloat16_rn(p);
          asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(*reinterpret_cast<const uint16_t*>(&pb)) : "memory");
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar_addr(c, B_P_FULL + sb));
    }
    if (!ok) break;

    // ---- segment epilogue ------------------------------------------------
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int h = 0; h < 16; ++h) l_part[h] += __shfl_xor_sync(0xffffffffu, l_part[h], off);
    if (lane == 0) {
#pragma unroll
      for (int h = 0; h < 16; h += 4)
        *reinterpret_cast<float4*>(c.red_l + wq * 16 + h) = make_float4(l_part[h], l_part[h + 1], l_part[h + 2], l_part[h + 3]);
    }
    named_barrier_sync(1, kSoftmaxThreads);
    float l_tot[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) l_tot[h] = c.red_l[h] + c.red_l[16 + h] + c.red_l[32 + h] + c.red_l[48 + h];
    named_barrier_sync(1, kSoftmaxThreads);   // red_l is rewritten by the next segment
    if (!(ok = group_all(mbar_wait(bar_addr(c, B_O_FULL), uint32_t(seg) & 1u, c.abort, c.timeout_ns)))) break;
    tc_fence_after();
    RecordView rec{nullptr, nullptr, nullptr};
    if (!full) rec = record_at(prm.records, plan_record_slot(prm.plan, blockIdx.x, t));
    float inv_l[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) inv_l[h] = l_tot[h] > 0.f ? 1.f / l_tot[h] : 0.f;
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      float o[16];
      tmem_ld16(c.tmem + t_lane + kTmemO + 16u * j, o);
      tmem_wait_ld();
      const int d = 128 * j + r;
      if (full) {
        __nv_bfloat16* ot = out + t * (kHeads * kCkv) + d;
#pragma unroll
        for (int h = 0; h < 16; ++h) ot[h * kCkv] = __float2bfloat16_rn(o[h] * inv_l[h]);
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) rec.o[h * kCkv + d] = o[h];
      }
    }
    tc_fence_before();
    mbar_arrive(bar_addr(c, B_O_EMPTY));
    if (leader) {
      if (full) {
#pragma unroll
        for (int h = 0; h < 16; ++h) prm.lse[t * kHeads + h] = l_tot[h] > 0.f ? m_run[h] + log2f(l_tot[h]) : -INFINITY;
      } else {
#pragma unroll
        for (int h = 0; h < 16; ++h) {
          rec.m[h] = m_run[h];
          rec.l[h] = l_tot[h];
        }
      }
    }
    ++seg;
    gs = ge;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    split_sm100_kernel(const __grid_constant__ CUtensorMap tm_ckv, const __grid_constant__ CUtensorMap tm_kpe,
                       const __grid_constant__ CUtensorMap tm_qn, const __grid_constant__ CUtensorMap tm_qp,
                       const SplitParams prm, const uint64_t timeout_ns) {
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Ctx c;
  c.sbase = smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  c.abort = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc + 4);
  c.red = reinterpret_cast<float*>(smem + kOffRed);
  c.red_l = reinterpret_cast<float*>(smem + kOffRedL);
  c.timeout_ns = timeout_ns;
  c.g_begin = plan_range_begin(prm.plan, blockIdx.x);
  c.g_end = plan_range_begin(prm.plan, int64_t(blockIdx.x) + 1);
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    mbar_init(bar_addr(c, B_Q_FULL), 1);
    mbar_init(bar_addr(c, B_Q_EMPTY), 1);
    for (int k = 0; k < 2; ++k) {
      mbar_init(bar_addr(c, B_KPE_FULL + k), 1);
      mbar_init(bar_addr(c, B_KPE_EMPTY + k), 1);
      mbar_init(bar_addr(c, B_S_FULL + k), 1);
      mbar_init(bar_addr(c, B_S_EMPTY + k), kSoftmaxThreads);
      mbar_init(bar_addr(c, B_P_FULL + k), kSoftmaxThreads);
      mbar_init(bar_addr(c, B_P_EMPTY + k), 1);
    }
    for (int s = 0; s < kSlabs; ++s) {
      mbar_init(bar_addr(c, B_SLAB_FULL + s), 1);
      mbar_init(bar_addr(c, B_SLAB_EMPTY + s), 1);
    }
    mbar_init(bar_addr(c, B_O_FULL), 1);
    mbar_init(bar_addr(c, B_O_EMPTY), kSoftmaxThreads);
    mbar_init(bar_addr(c, B_DONE), 1);
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
    producer(c, prm, &tm_ckv, &tm_kpe, &tm_qn, &tm_qp);
  } else if (warp == 1) {
    if ((threadIdx.x & 31) == 0) mma_issuer(c);
    __syncwarp();
  } else {
    softmax_epilogue(c, prm);
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *c.abort) report_error(prm.err_word, DSA_DEVICE_ERR_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(c.tmem, kTmemCols);
  }
}

// -------------------------------------------------------------------------
// host side
// -------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
constexpr int kMaxDevices = 64;
std::once_flag g_attr_once[kMaxDevices];
cudaError_t g_attr_err[kMaxDevices];
uint64_t g_timeout_ns = 0;

bool encode_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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
    g_attr_err[dev] = cudaFuncSetAttribute(split_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           int(kSmemBytes));
  });
  if (g_attr_err[dev] != cudaSuccess) return g_attr_err[dev];

  CUtensorMap tm_ckv, tm_kpe, tm_qn, tm_qp;
  const uint64_t slots = uint64_t(prm.num_slots);
  const uint64_t qrows = uint64_t(prm.plan.total_blocks / kBlocksPerToken) * kHeads;
  if (!encode_2d(&tm_ckv, prm.ckv, kCkv, slots, 64, 1) || !encode_2d(&tm_kpe, prm.kpe, kKpe, slots, 64, 1) ||
      !encode_2d(&tm_qn, prm.q_nope, kCkv, qrows, 64, 16) || !encode_2d(&tm_qp, prm.q_pe, kKpe, qrows, 64, 16))
    return cudaErrorInvalidValue;
  split_sm100_kernel<<<prm.plan.grid, kThreads, kSmemBytes, stream>>>(tm_ckv, tm_kpe, tm_qn, tm_qp, prm,
                                                                       g_timeout_ns);
  return cudaGetLastError();
}

}  // namespace dsa
