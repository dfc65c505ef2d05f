// q4k_gemv.cu -- fused Q4_K x fp16 decode GEMV: y = W x (+ residual).
//
// Replaces the decode-time linears of the reference (encodeMPSMatrixMultiply
// on dequantized fp16 weights, MetalLM/Backend/Metal/MetalService.swift:
// 797-925, called from LlamaRunner.swift:563-609, 954-963, 1008-1034,
// 1059-1068, 1169-1178).  The packed 144-byte blocks are streamed from HBM
// once; no dequantized copy exists.
//
// Arithmetic.  For row r and sub-block j (32 elements) of block b:
//   sum_i W[r][i] x[i] = (d*sc_j) * sum_i q_i x_i  -  (dmin*m_j) * sum_i x_i
// sum_i x_i per sub-block is a property of x alone (computed once per CTA).
// sum_i q_i x_i runs on the tensor cores: a 4-bit quant masked into the low
// mantissa bits of a binary16 is the subnormal q * 2^-24 (bits 0-3) or
// 16 q * 2^-24 (bits 4-7), so one LOP3 turns two nibbles into an exact f16x2
// operand.  Products with x are exact in fp32 and accumulate in fp32; the
// two scales accumulate in separate MMA chains, combined as a + b/16, and
// the 2^24 is folded into d in the epilogue.
//
// MMA mapping (mma.sync.m16n8k16, A = quants [16 rows x 16 k], B = x):
// thread (g = lane/4, t = lane%4) owns, for each of its rows, the qs words
// 8t..8t+7 of a block, i.e. sub-blocks 2t and 2t+1.  Word w and w >> 8
// give, under mask 0x000F000F, the element pairs (e0,e4) and (e2,e6), and
// under 0x00F000F0 the pairs (e1,e5) and (e3,e7) scaled by 16: one MMA for
// each mask, the k order inside a chunk being that permutation.  B column n
// carries x of sub-block n only, so C[row][n] is the per-sub-block sum and
// lands in the thread that holds that sub-block's scale (C columns 2t,
// 2t+1).  x is staged once per CTA in shared memory in the permuted order
// [x0 x4 x2 x6 x1 x5 x3 x7] per 8-element group, so each MMA's B pair is two
// adjacent registers; threads whose B column does not match a word read a
// zero region instead.
//
// Work split.  A unit is one block column of a 32-row tile (4608 bytes); a
// segment is L consecutive units of one tile (L divides the blocks per row).
// Each CTA owns a contiguous range of segments in tile-major order, so every
// SM streams the same number of bytes (to one segment) whatever the shape.
// Inside a CTA, warps pull segments from a shared-memory queue.  Each warp
// streams its units through a ring of shared-memory stages, one TMA tensor
// copy per unit (a 32-row x 144-byte box of W viewed as a 2D byte tensor,
// L2 evict-first, rows past the end zero-filled by the TMA unit), each stage
// tracked by an mbarrier; waits are bounded by a %globaltimer budget and
// report a device error instead of hanging.  Each segment's 32 row sums go
// to a shared-memory slot; the warp that completes a tile's last segment
// sums the tile's slots in k order (deterministic) and stores y.  A tile
// shared with a neighbouring CTA leaves one partial per CTA in the context
// scratch and the last CTA to arrive (atomic counter) adds them in CTA
// order, stores y and re-zeroes the counter.  Those boundary tiles are
// queued first, so the cross-CTA exchange overlaps the interior work.
#include <cuda.h>

#include <algorithm>

#include "mlm_device.cuh"
#include "mlm_internal.h"

namespace mlm {

constexpr int kGemvMaxWarps = 12;                     // warps per CTA (upper bound)
constexpr int kGemvStages = 3;                        // smem stages per warp
constexpr int kTileRows = 32;                         // rows per tile
constexpr int kStageBytes = kTileRows * kBlockBytes;  // 4608
constexpr int kRing = 4;  // per-warp ring of (tile, block) entries: >= stages
static_assert(kGemvStages <= kRing, "ring must cover the units in flight");
constexpr unsigned long long kWaitBudgetNs = 200ull * 1000 * 1000;  // 200 ms

struct GemvArgs {
  const uint8_t *W;
  const __half *x;
  float *y;
  const float *residual;
  float *partials;  // [ctas][2][32]
  int *counters;    // [tiles]
  int *status;      // device-visible error word (0 = ok)
  unsigned long long nbs_magic;  // ceil(2^40 / nbs): s / nbs == (s * magic) >> 40
  int rows;
  int nb;      // blocks per row
  int L;       // units per segment
  int nbs;     // segments per tile
  int tiles;   // ceil(rows / 32)
  int nsegs;   // tiles * nbs
  int ctas;    // grid size
  int nslot;   // segment slots per CTA
  int ntile;   // tile counters per CTA (multiple of 4)
  uint32_t smem_bar;  // byte offset of the mbarriers
  uint32_t smem_x;    // byte offset of the x region
};

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Weights are read exactly once: copy them with an L2 evict-first policy so
// they do not push x, y and the KV cache out of L2.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// try_wait suspends the thread until the phase completes or the hint (ns)
// elapses, so a waiting warp does not spin on the issue slots
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(bar), "r"(phase), "r"(1000000u)
      : "memory");
  return done != 0;
}
// Bounded wait for a stage: gives up after kWaitBudgetNs and reports it.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t phase, int *status) {
  if (mbar_try_wait(bar, phase)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, phase)) {
    if (global_ns() - t0 > kWaitBudgetNs) {
      atomicExch(status, MLM_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// One unit (a 144-byte x 32-row box at byte column x, row y of W) into
// shared memory, completing on `bar`.
__device__ __forceinline__ void tma_unit(uint32_t dst, const CUtensorMap *tmap, int x, int y,
                                         uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(pol)
      : "memory");
}

// first segment of CTA c, and the CTA whose range holds segment s
// (all products stay below 2^31: checked on the host)
__device__ __forceinline__ int seg_begin(int c, const GemvArgs &p) {
  return (c * p.nsegs) / p.ctas;
}
__device__ __forceinline__ int cta_of_seg(int s, const GemvArgs &p) {
  return ((s + 1) * p.ctas - 1) / p.nsegs;
}
__device__ __forceinline__ int div_nbs(int s, const GemvArgs &p) {
  return (int)(((unsigned long long)(unsigned)s * p.nbs_magic) >> 40);
}

__global__ void __launch_bounds__(kGemvMaxWarps * 32, 1)
    q4k_gemv_kernel(const __grid_constant__ CUtensorMap tmap, GemvArgs p) {
  // TMA tensor destinations need 128-byte alignment: stages sit at multiples
  // of 4608 = 36 * 128 bytes from this base
  extern __shared__ __align__(1024) uint8_t smem[];
  const int nwarps = blockDim.x >> 5;
  uint4 *xzero = reinterpret_cast<uint4 *>(smem + p.smem_x);
  uint4 *xperm = xzero + 4;  // after 64 zero bytes
  float *xsum = reinterpret_cast<float *>(xperm + p.nb * 32);
  float *slots = xsum + p.nb * 8;                                  // [nslot][32]
  int *tile_done = reinterpret_cast<int *>(slots + p.nslot * 32);  // [ntile]
  // [warps][kRing] (tile, first block); 16-byte aligned: ntile is a multiple of 4
  int2 *ring = reinterpret_cast<int2 *>(tile_done + p.ntile);
  int *sched = reinterpret_cast<int *>(ring + nwarps * kRing);

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int c = blockIdx.x;

  // this warp's stages and their mbarriers
  const uint32_t my_stage_addr =
      (uint32_t)__cvta_generic_to_shared(smem + warp * kGemvStages * kStageBytes);
  const uint8_t *my_stages = smem + warp * kGemvStages * kStageBytes;
  const uint32_t my_bar = (uint32_t)__cvta_generic_to_shared(smem + p.smem_bar) +
                          warp * kGemvStages * 8;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kGemvStages; ++s) mbar_init(my_bar + 8 * s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  // this CTA's segments [sb0, sb1) and its boundary tiles
  const int sb0 = seg_begin(c, p), sb1 = seg_begin(c + 1, p);
  const int S = sb1 - sb0;
  const int t_first = div_nbs(sb0, p), t_last = div_nbs(sb1 - 1, p);
  const bool first_partial = (sb0 != t_first * p.nbs) || (sb1 < (t_first + 1) * p.nbs);
  const int nf = first_partial ? min(sb1, (t_first + 1) * p.nbs) - sb0 : 0;
  const int nl = (t_last != t_first && sb1 != (t_last + 1) * p.nbs) ? sb1 - t_last * p.nbs : 0;
  // queue order: first boundary tile, last boundary tile, interior tiles
  auto seg_of_queue = [&](int qi) -> int {
    if (qi < nf) return sb0 + qi;
    if (qi < nf + nl) return sb1 - nl + (qi - nf);
    return sb0 + qi - nl;
  };

  const uint64_t pol = evict_first_policy();

  // ---- producer state: segments are grabbed from the queue ----------------
  // The first kGemvStages-1 grabs of warp w are static (w, w + warps, ...),
  // so the prologue needs no shared counter; later grabs are dynamic.
  int grabs = 0;
  int ti = 0, bi = 0, iu = p.L;  // segment being issued (tile, first block), units issued
  bool issue_done = false;
  int ring_tail = 0;
  int st_in = 0;
  int pending = 0;  // units issued, not yet consumed

  auto issue_next = [&]() {
    if (issue_done) return;
    if (iu == p.L) {
      int qi;
      if (grabs < kGemvStages - 1) {
        qi = warp + grabs * nwarps;
      } else {
        if (lane == 0) qi = atomicAdd(sched, 1);
        qi = __shfl_sync(0xffffffffu, qi, 0);
      }
      ++grabs;
      if (qi >= S) {
        issue_done = true;
        return;
      }
      const int seg = seg_of_queue(qi);
      ti = div_nbs(seg, p);
      bi = (seg - ti * p.nbs) * p.L;
      if (lane == 0) ring[warp * kRing + (ring_tail & (kRing - 1))] = make_int2(ti, bi);
      ++ring_tail;
      iu = 0;
    }
    if (lane == 0) {
      const uint32_t bar = my_bar + 8 * st_in;
      mbar_expect_tx(bar, kStageBytes);
      tma_unit(my_stage_addr + st_in * kStageBytes, &tmap, (bi + iu) * kBlockBytes,
               ti * kTileRows, bar, pol);
    }
    st_in = (st_in + 1 == kGemvStages) ? 0 : st_in + 1;
    ++iu;
    ++pending;
  };

  // The first stages only read the weights, which no preceding kernel
  // writes: put them in flight before waiting on that kernel.
#pragma unroll
  for (int s = 0; s < kGemvStages - 1; ++s) issue_next();

  // Programmatic dependent launch: x, y and the split-K scratch may belong to
  // the previous kernel on the stream, so wait for it here.  Dependents may
  // start as soon as SMs free up.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");

  // ---- x -> shared memory, permuted, plus per-sub-block sums ---------------
  {
    const uint4 *xg = reinterpret_cast<const uint4 *>(p.x);
    const int ngroups = p.nb * 32;  // multiple of 32: whole warps stay converged
    constexpr int XB = 8;           // x loads in flight per thread
    if (threadIdx.x < 4) xzero[threadIdx.x] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < p.ntile; i += blockDim.x) tile_done[i] = 0;
    if (threadIdx.x == 0) *sched = (kGemvStages - 1) * nwarps;
    for (int base = threadIdx.x; base < ngroups; base += XB * blockDim.x) {
      uint4 xv[XB];
#pragma unroll
      for (int u = 0; u < XB; ++u) {
        const int i = base + u * blockDim.x;
        if (i < ngroups) xv[u] = __ldg(xg + i);
      }
#pragma unroll
      for (int u = 0; u < XB; ++u) {
        const int i = base + u * blockDim.x;
        if (i < ngroups) {
          const uint4 v = xv[u];
          uint4 o;
          o.x = __byte_perm(v.x, v.z, 0x5410);  // (x0, x4)
          o.y = __byte_perm(v.y, v.w, 0x5410);  // (x2, x6)
          o.z = __byte_perm(v.x, v.z, 0x7632);  // (x1, x5)
          o.w = __byte_perm(v.y, v.w, 0x7632);  // (x3, x7)
          xperm[i] = o;
          const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
          const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
          const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&v.z));
          const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&v.w));
          float sx = ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y));
          sx += __shfl_xor_sync(0xffffffffu, sx, 1);
          sx += __shfl_xor_sync(0xffffffffu, sx, 2);
          if ((i & 3) == 0) xsum[i >> 2] = sx;
        }
      }
    }
  }
  __syncthreads();

  // B operands: thread (g, t) carries x for words 0..3 of its slice when
  // g == 2t, for words 4..7 when g == 2t + 1, zeros otherwise.
  const int act = g - 2 * tig;
  const uint32_t xzero_addr = (uint32_t)__cvta_generic_to_shared(xzero);
  const uint32_t xperm_addr = (uint32_t)__cvta_generic_to_shared(xperm);
  const uint32_t x_lo_base = (act == 0) ? xperm_addr + 16 * (8 * tig) : xzero_addr;
  const uint32_t x_hi_base = (act == 1) ? xperm_addr + 16 * (8 * tig + 4) : xzero_addr;
  const uint32_t x_lo_step = (act == 0) ? 512u : 0u;  // per block column
  const uint32_t x_hi_step = (act == 1) ? 512u : 0u;

  // scale/min unpack of sub-blocks 2t, 2t+1 (get_scale_min_k4): one byte
  // permute gathers the two low-part bytes (and for sub-blocks 4..7 the two
  // bytes carrying the high bits), then masks finish the 6-bit values.
  const bool upper = tig >= 2;
  const uint32_t jb = 2 * (tig & 1);
  const uint32_t psel = upper ? ((jb + 4) | ((jb + 5) << 4) | (jb << 8) | ((jb + 1) << 12))
                              : (jb | ((jb + 1) << 4) | (jb << 8) | ((jb + 1) << 12));
  const uint32_t mA = upper ? 0x0F0Fu : 0x3F3Fu;
  const uint32_t mB = upper ? 0x3030u : 0u;
  const uint32_t shm = upper ? 4u : 0u;

  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // rows g, g+8, g+16, g+24 of the segment

  // The warp that completes a boundary tile's part of this CTA publishes it;
  // the last CTA to arrive adds the CTAs' parts in CTA order.
  auto boundary_finish = [&](int t, float s) {
    const int end = (t == t_first) ? 0 : 1;
    __stcg(p.partials + ((size_t)c * 2 + end) * kTileRows + lane, s);
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(p.counters + t, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    const int cf = cta_of_seg(t * p.nbs, p), cl = cta_of_seg((t + 1) * p.nbs - 1, p);
    if (old == cl - cf) {
      __threadfence();
      const int slot_cf = (seg_begin(cf, p) == t * p.nbs) ? 0 : 1;
      float tot = __ldcg(p.partials + ((size_t)cf * 2 + slot_cf) * kTileRows + lane);
      for (int cc = cf + 1; cc <= cl; ++cc)
        tot += __ldcg(p.partials + ((size_t)cc * 2) * kTileRows + lane);
      const int r = t * kTileRows + lane;
      if (r < p.rows) p.y[r] = tot + (p.residual ? p.residual[r] : 0.f);
      if (lane == 0) p.counters[t] = 0;
    }
  };

  auto finish_segment = [&](int t, int b0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
      acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);
    }
    const int k = t * p.nbs + b0 / p.L - sb0;
    if (tig == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) slots[k * kTileRows + g + 8 * i] = acc[i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = 0.f;
    __syncwarp();
    const int ks = max(sb0, t * p.nbs) - sb0;
    const int ke = min(sb1, (t + 1) * p.nbs) - sb0;
    int old = 0;
    if (lane == 0) {
      __threadfence_block();
      old = atomicAdd(tile_done + (t - t_first), 1);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == ke - ks - 1) {  // this warp completed the tile's part
      __threadfence_block();
      const volatile float *vs = slots;
      float s = 0.f;
      for (int k2 = ks; k2 < ke; ++k2) s += vs[k2 * kTileRows + lane];
      if (ks + sb0 == t * p.nbs && ke + sb0 == (t + 1) * p.nbs) {
        const int r = t * kTileRows + lane;
        if (r < p.rows) p.y[r] = s + (p.residual ? p.residual[r] : 0.f);
      } else {
        boundary_finish(t, s);
      }
    }
  };

  // ---- main loop: one unit per iteration ------------------------------------
  int ring_head = 0, cu = 0, st_out = 0;
  uint32_t phases = 0;  // bit s: parity of the next completion of stage s
  while (pending > 0) {
    issue_next();
    if (!mbar_wait_bounded(my_bar + 8 * st_out, (phases >> st_out) & 1, p.status)) break;
    phases ^= 1u << st_out;

    const int2 tb = ring[warp * kRing + (ring_head & (kRing - 1))];
    const int t = tb.x;
    const int b = tb.y + cu;
    const uint8_t *st = my_stages + st_out * kStageBytes;
    const uint32_t xlo = x_lo_base + b * x_lo_step;
    const uint32_t xhi = x_hi_base + b * x_hi_step;
    const float2 xs = *reinterpret_cast<const float2 *>(xsum + b * 8 + 2 * tig);

    // quants and headers of rows g, g+8, g+16, g+24
    uint32_t q[4][8];
    uint4 hd[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint8_t *r = st + (g + 8 * i) * kBlockBytes;
      hd[i] = *reinterpret_cast<const uint4 *>(r);
      *reinterpret_cast<uint4 *>(&q[i][0]) = *reinterpret_cast<const uint4 *>(r + 16 + 32 * tig);
      *reinterpret_cast<uint4 *>(&q[i][4]) = *reinterpret_cast<const uint4 *>(r + 32 + 32 * tig);
    }

    // [mt][chain]: chain 0 = mask 0x000F000F, chain 1 = mask 0x00F000F0 (x16).
    // Column 2t only collects words 0..3 and column 2t+1 words 4..7 (their B
    // columns), so one chain holds both sub-block sums.
    float cacc[2][2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int ch = 0; ch < 2; ++ch)
        cacc[mt][ch][0] = cacc[mt][ch][1] = cacc[mt][ch][2] = cacc[mt][ch][3] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint4 xb;
      const uint32_t xa = (j < 4) ? xlo + 16 * j : xhi + 16 * (j - 4);
      asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                   : "=r"(xb.x), "=r"(xb.y), "=r"(xb.z), "=r"(xb.w)
                   : "r"(xa));
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint32_t w0 = q[2 * mt][j], w1 = q[2 * mt + 1][j];
        const uint32_t t0 = w0 >> 8, t1 = w1 >> 8;
        const uint32_t M = 0x000F000Fu, M16 = 0x00F000F0u;
        mma_f16_16816(cacc[mt][0], w0 & M, w1 & M, t0 & M, t1 & M, xb.x, xb.y);
        mma_f16_16816(cacc[mt][1], w0 & M16, w1 & M16, t0 & M16, t1 & M16, xb.z, xb.w);
      }
    }

    // epilogue: scale the sub-block sums of columns 2t, 2t+1
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int mt = i >> 1, hr = i & 1;
      const uint4 h = hd[i];
      const float cs0 = fmaf(0.0625f, cacc[mt][1][2 * hr], cacc[mt][0][2 * hr]);
      const float cs1 = fmaf(0.0625f, cacc[mt][1][2 * hr + 1], cacc[mt][0][2 * hr + 1]);
      const uint32_t P = __byte_perm(h.y, h.w, psel);
      const uint32_t Q = __byte_perm(h.z, h.w, psel);
      const uint32_t scp = (P & mA) | ((P >> 18) & mB);
      const uint32_t mp = ((Q >> shm) & mA) | ((Q >> 18) & mB);
      const float D = half_bits_to_float(h.x) * 16777216.0f;  // d * 2^24
      const float Dm = half_bits_to_float(h.x >> 16);
      const float qs = (float)(scp & 0xFF) * cs0 + (float)(scp >> 8) * cs1;
      const float ms = (float)(mp & 0xFF) * xs.x + (float)(mp >> 8) * xs.y;
      acc[i] += D * qs - Dm * ms;
    }
    __syncwarp();  // stage fully read before it is refilled
    st_out = (st_out + 1 == kGemvStages) ? 0 : st_out + 1;
    --pending;
    if (++cu == p.L) {
      finish_segment(t, tb.y);
      ++ring_head;
      cu = 0;
    }
  }
  if (pending > 0) {
    // a stage wait ran out of budget: let the copies still in flight land
    // (bounded again) before this warp's shared memory is released
    for (int s = 0; s < kGemvStages && pending > 0; ++s, --pending) {
      if (!mbar_wait_bounded(my_bar + 8 * st_out, (phases >> st_out) & 1, p.status)) break;
      phases ^= 1u << st_out;
      st_out = (st_out + 1 == kGemvStages) ? 0 : st_out + 1;
    }
  }
}

// called once per context, with its device current
int gemv_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q4k_gemv_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ctx->max_smem_optin));
  return MLM_OK;
}

int gemv_max_ctas(int sm_count) { return sm_count; }

struct GemvPlan {
  int warps, L, nbs, nsegs, ctas, nslot, ntile;
  size_t smem;
  uint32_t smem_bar, smem_x;
};

// Smallest segment length (a divisor of the blocks per row) and the most
// warps whose shared-memory footprint fits.
static bool plan_gemv(int rows, int nb, int sm_count, size_t smem_max, GemvPlan &pl) {
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  for (int warps = kGemvMaxWarps; warps >= 4; --warps) {
    for (int L = 1; L <= nb; ++L) {
      if (nb % L) continue;
      const int nbs = nb / L;
      const long long nsegs = (long long)tiles * nbs;
      const int ctas = (int)std::min<long long>(sm_count, nsegs);
      if (nsegs * ctas >= (1LL << 31) || nsegs >= (1LL << 20)) continue;
      const int segmax = (int)((nsegs + ctas - 1) / ctas);
      // tile counters rounded to 16 bytes so the int2 ring after them is aligned
      const int ntile = ((segmax / nbs + 2) + 3) & ~3;
      const size_t smem_bar = (size_t)warps * kGemvStages * kStageBytes;
      const size_t smem_x = smem_bar + (((size_t)warps * kGemvStages * 8 + 15) & ~(size_t)15);
      const size_t smem = smem_x + 64 + (size_t)nb * 32 * 16 + (size_t)nb * 8 * 4 +
                          (size_t)segmax * kTileRows * 4 + (size_t)ntile * 4 +
                          (size_t)warps * kRing * sizeof(int2) + 16;
      if (smem <= smem_max && segmax <= 4096) {
        pl = {warps, L, nbs, (int)nsegs, ctas, segmax, ntile, smem, (uint32_t)smem_bar,
              (uint32_t)smem_x};
        return true;
      }
    }
  }
  return false;
}

// W viewed as a 2D byte tensor [rows][nb * 144]; box = one unit (144 bytes
// of 32 rows).  Rows past the end read as zeros.
static int encode_weight_map(mlm_ctx *ctx, const void *W, int rows, int nb, CUtensorMap *map) {
  using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return set_error(ctx, MLM_ERR_CUDA, "mlm_q4k_gemv: cuTensorMapEncodeTiled unavailable");
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  const cuuint64_t dims[2] = {(cuuint64_t)nb * kBlockBytes, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)nb * kBlockBytes};
  const cuuint32_t box[2] = {(cuuint32_t)kBlockBytes, (cuuint32_t)kTileRows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(W), dims,
                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ctx, MLM_ERR_CUDA, "mlm_q4k_gemv: tensor map encode failed (%d)", (int)r);
  return MLM_OK;
}

int gemv_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x, float *y,
                const float *residual, float *partials, int *counters, int max_ctas,
                int max_tiles, cudaStream_t stream) {
  const int nb = cols / kQK;
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  MLM_REQUIRE(ctx, tiles <= max_tiles, MLM_ERR_SHAPE,
              "mlm_q4k_gemv: %d rows exceed the %d-row scratch limit", rows,
              max_tiles * kTileRows);
  GemvPlan pl;
  const bool ok = plan_gemv(rows, nb, std::min(ctx->sm_count, max_ctas),
                            (size_t)ctx->max_smem_optin, pl);
  MLM_REQUIRE(ctx, ok, MLM_ERR_UNSUPPORTED,
              "mlm_q4k_gemv: rows=%d cols=%d does not fit the shared-memory plan", rows, cols);
  CUtensorMap tmap;
  int st = encode_weight_map(ctx, W, rows, nb, &tmap);
  if (st != MLM_OK) return st;
  GemvArgs a;
  a.W = reinterpret_cast<const uint8_t *>(W);
  a.x = reinterpret_cast<const __half *>(x);
  a.y = y;
  a.residual = residual;
  a.partials = partials;
  a.counters = counters;
  a.status = ctx->dev_status;
  a.nbs_magic = ((1ull << 40) + (unsigned long long)pl.nbs - 1) / (unsigned long long)pl.nbs;
  a.rows = rows;
  a.nb = nb;
  a.L = pl.L;
  a.nbs = pl.nbs;
  a.tiles = tiles;
  a.nsegs = pl.nsegs;
  a.ctas = pl.ctas;
  a.nslot = pl.nslot;
  a.ntile = pl.ntile;
  a.smem_bar = pl.smem_bar;
  a.smem_x = pl.smem_x;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.ctas);
  cfg.blockDim = dim3(pl.warps * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, q4k_gemv_kernel, tmap, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, MLM_ERR_CUDA, "mlm_q4k_gemv: launch failed: %s", cudaGetErrorString(e));
  }
  return MLM_OK;
}

int gemv_validate(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x, float *y) {
  MLM_REQUIRE(ctx, W && x && y, MLM_ERR_ARG, "mlm_q4k_gemv: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && cols > 0, MLM_ERR_SHAPE, "mlm_q4k_gemv: rows=%d cols=%d", rows,
              cols);
  MLM_REQUIRE(ctx, cols % kQK == 0, MLM_ERR_SHAPE,
              "mlm_q4k_gemv: cols=%d is not a multiple of the 256-element super-block", cols);
  MLM_REQUIRE(ctx, aligned16(W) && aligned16(x), MLM_ERR_ALIGN,
              "mlm_q4k_gemv: W and x must be 16-byte aligned");
  return MLM_OK;
}

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_q4k_gemv(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                            float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  int st = gemv_validate(ctx, W, rows, cols, x_f16, y);
  if (st != MLM_OK) return st;
  return gemv_launch(ctx, W, rows, cols, x_f16, y, residual, ctx->gemv_partials,
                     ctx->gemv_counters, ctx->gemv_max_ctas, ctx->gemv_max_tiles, ctx->stream);
}
