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
// Work split.  A unit is one block column of a 32-row tile (4608 bytes).
// Each CTA owns a contiguous range of units in tile-major order.  When a CTA
// count between half and all of the SMs divides the tiles without raising
// the most units a warp takes, every CTA owns whole tiles (no partial sum
// leaves a CTA); otherwise every SM gets a CTA and every SM streams the same
// number of bytes (to one unit).  The
// CTA walks its units boundary tiles first (the tiles it shares with its
// neighbours), so the cross-CTA exchange overlaps the interior work; each
// warp takes a contiguous run of that sequence and advances (tile, block)
// incrementally.  Units reach shared memory through a per-warp ring of
// stages, one TMA tensor copy per unit (a 32-row x 144-byte box of W viewed
// as a 2D byte tensor, L2 evict-first, rows past the end zero-filled by the
// TMA unit), each stage tracked by an mbarrier; waits are bounded by a
// %globaltimer budget and report a device error instead of hanging.  A warp
// keeps its row sums in registers across the consecutive units of a tile.
// A tile it covers alone is stored directly; a tile shared by several warps
// leaves one part per warp in shared memory, and the last warp to finish
// (shared-memory counter) adds the parts in warp order (deterministic).  A
// tile shared with a neighbouring CTA leaves one partial per CTA in the
// context scratch and the last CTA to arrive (atomic counter) adds them in
// CTA order, stores y and re-zeroes the counter.
#include <cuda.h>

#include <algorithm>

#include "mlm_internal.h"
#include "q4k_gemv_common.cuh"

namespace mlm {

#ifndef MLM_GEMV_WARPS
#define MLM_GEMV_WARPS 16
#endif
#ifndef MLM_GEMV_STAGES
#define MLM_GEMV_STAGES 2
#endif
#ifndef MLM_GEMV_MIN_BLOCKS
#define MLM_GEMV_MIN_BLOCKS 1  // resident CTAs per SM the register budget allows
#endif
constexpr int kGemvMaxWarps = MLM_GEMV_WARPS;          // warps per CTA (upper bound)
constexpr int kGemvStages = MLM_GEMV_STAGES;           // smem stages per warp
constexpr int kStageBytes = kTileRows * kBlockBytes;  // 4608

struct GemvArgs {
  const uint8_t *W;
  const __half *x;
  const float *x_scale;  // per 32-element sub-block of x (NULL: 1)
  const float *xa, *xb;  // fp32 sources of x in the kRmsNorm / kSwiGLU modes
  float eps;
  int x_mode;            // GemvInput::Mode
  float *y;
  const float *residual;
  float *partials;  // [ctas][2][32]
  int *counters;    // [tiles]
  __half *pair_h;   // gate/up pairing (GemvPair; NULL: off)
  float *pair_scale;
  int *pair_ctr;    // [rows / 64]
  int pair_tiles;   // tiles of the gate half: tile t pairs with t + pair_tiles
  int *status;      // device-visible error word (0 = ok)
  unsigned long long nb_magic;  // ceil(2^40 / nb): u / nb == (u * magic) >> 40
  int rows;
  int nb;      // blocks per row = units per tile
  int units;   // tiles * nb
  int ctas;    // grid size
  int ntile;   // tile counters per CTA (multiple of 4)
  uint32_t smem_bar;  // byte offset of the mbarriers
  uint32_t smem_x;    // byte offset of the x region
};


__global__ void __launch_bounds__(kGemvMaxWarps * 32, MLM_GEMV_MIN_BLOCKS)
    q4k_gemv_kernel(const __grid_constant__ CUtensorMap tmap, GemvArgs p) {
  // TMA tensor destinations need 128-byte alignment: stages sit at multiples
  // of 4608 = 36 * 128 bytes from this base
  extern __shared__ __align__(1024) uint8_t smem[];
  const int nwarps = blockDim.x >> 5;
  uint4 *xzero = reinterpret_cast<uint4 *>(smem + p.smem_x);
  uint4 *xperm = xzero + 4;  // after 64 zero bytes
  float *xsum = reinterpret_cast<float *>(xperm + p.nb * 32);  // [nb][8]
  float *xscl = xsum + p.nb * 8;                               // [nb][8]
  float *parts = xscl + p.nb * 8;                                        // [warps][2][32]
  int *tile_done = reinterpret_cast<int *>(parts + nwarps * 2 * kTileRows);  // [ntile]

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

  // this CTA's units and their order
  CtaOrder co;
  co.u0 = unit_begin(c, p);
  co.u1 = unit_begin(c + 1, p);
  co.S = co.u1 - co.u0;
  co.t_first = div_nb(co.u0, p);
  co.t_last = div_nb(co.u1 - 1, p);
  const bool first_shared = (co.u0 != co.t_first * p.nb) || (co.u1 < (co.t_first + 1) * p.nb);
  co.nf = first_shared ? min(co.u1, (co.t_first + 1) * p.nb) - co.u0 : 0;
  co.nl = (co.t_last != co.t_first && co.u1 != (co.t_last + 1) * p.nb)
              ? co.u1 - co.t_last * p.nb
              : 0;

  // this warp's contiguous run [q0, q1) of the order; no warp is left empty
  const int nwe = min(nwarps, co.S);
  const bool has_work = warp < nwe;
  auto qstart = [&](int w) { return (w * co.S) / nwe; };
  auto warp_of_q = [&](int q) { return ((q + 1) * nwe - 1) / co.S; };
  const int q0 = has_work ? qstart(warp) : 0, q1 = has_work ? qstart(warp + 1) : 0;

  const uint64_t pol = evict_first_policy();

  // ---- producer: (tile, block) of the next unit to put in flight -----------
  int qi = q0, ti = 0, bi = 0;
  if (has_work) {
    const int u = co.unit_of(q0);
    ti = div_nb(u, p);
    bi = u - ti * p.nb;
  }
  int st_in = 0;
  // step (q, t, b) to the next position of the order
  auto advance = [&](int &q, int &t, int &b) {
    ++q;
    if (q == co.nf || q == co.nf + co.nl) {  // crossing into the next group
      const int u = co.unit_of(q);
      t = div_nb(u, p);
      b = u - t * p.nb;
    } else if (++b == p.nb) {
      b = 0;
      ++t;
    }
  };
  auto issue_next = [&]() {
    if (qi >= q1) return;
    if (lane == 0) {
      const uint32_t bar = my_bar + 8 * st_in;
      mbar_expect_tx(bar, kStageBytes);
      tma_unit(my_stage_addr + st_in * kStageBytes, &tmap, bi * kBlockBytes, ti * kTileRows, bar,
               pol);
    }
    st_in = (st_in + 1 == kGemvStages) ? 0 : st_in + 1;
    advance(qi, ti, bi);
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
  // Group i = elements 8i .. 8i+7 of x as eight fp16 values v and the scale
  // sc of its sub-block (x = v * sc).  Four consecutive lanes hold the four
  // groups of a sub-block; ngroups is a multiple of 32, so whole warps take
  // part in the shuffles.
  {
    const int ngroups = p.nb * 32;
    if (threadIdx.x < 4) xzero[threadIdx.x] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < p.ntile; i += blockDim.x) tile_done[i] = 0;
    auto stage = [&](int i, const uint4 v, float sc) {
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
      if ((i & 3) == 0) {
        xsum[i >> 2] = sx * sc;
        xscl[i >> 2] = sc;
      }
    };
    auto pack = [](const float (&f)[8]) {
      uint4 v;
      __half2 h;
      h = __floats2half2_rn(f[0], f[1]); v.x = *reinterpret_cast<uint32_t *>(&h);
      h = __floats2half2_rn(f[2], f[3]); v.y = *reinterpret_cast<uint32_t *>(&h);
      h = __floats2half2_rn(f[4], f[5]); v.z = *reinterpret_cast<uint32_t *>(&h);
      h = __floats2half2_rn(f[6], f[7]); v.w = *reinterpret_cast<uint32_t *>(&h);
      return v;
    };
    auto load8 = [](const float *src, int i, float (&f)[8]) {
      const float4 a = __ldg(reinterpret_cast<const float4 *>(src) + 2 * i);
      const float4 b = __ldg(reinterpret_cast<const float4 *>(src) + 2 * i + 1);
      f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
      f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    };
    if (p.x_mode == GemvInput::kHalf) {
      const uint4 *xg = reinterpret_cast<const uint4 *>(p.x);
      constexpr int XB = 8;  // x loads in flight per thread
      for (int base = threadIdx.x; base < ngroups; base += XB * blockDim.x) {
        uint4 xv[XB];
        float xs[XB];  // sub-block scales, loaded with x (one round trip)
#pragma unroll
        for (int u = 0; u < XB; ++u) {
          const int i = base + u * blockDim.x;
          if (i < ngroups) {
            xv[u] = __ldg(xg + i);
            xs[u] = p.x_scale ? __ldg(p.x_scale + (i >> 2)) : 1.0f;
          }
        }
#pragma unroll
        for (int u = 0; u < XB; ++u) {
          const int i = base + u * blockDim.x;
          if (i < ngroups) stage(i, xv[u], xs[u]);
        }
      }
    } else if (p.x_mode == GemvInput::kRmsNorm && ngroups <= 4 * (int)blockDim.x) {
      // every CTA reduces the sum of squares of the whole hidden state
      // itself; hidden state and weights are read once, into registers, so
      // the norm costs one round trip to L2
      constexpr int XU = 4;
      float a[XU][8], w[XU][8];
      float ss = 0.f;
#pragma unroll
      for (int u = 0; u < XU; ++u) {
        const int i = threadIdx.x + u * blockDim.x;
        if (i < ngroups) {
          load8(p.xa, i, a[u]);
          load8(p.xb, i, w[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < XU; ++u) {
        const int i = threadIdx.x + u * blockDim.x;
        if (i < ngroups) {
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += a[u][e] * a[u][e];
        }
      }
      ss = warp_sum(ss);
      float *red = parts;  // free until the main loop
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int wi = 0; wi < nwarps; ++wi) tot += red[wi];
      const float scale = rms_scale(tot, ngroups * 8, p.eps);
#pragma unroll
      for (int u = 0; u < XU; ++u) {
        const int i = threadIdx.x + u * blockDim.x;
        if (i < ngroups) {  // whole warps: ngroups is a multiple of 32
#pragma unroll
          for (int e = 0; e < 8; ++e) a[u][e] = (a[u][e] * scale) * safe_weight(w[u][e]);
          stage(i, pack(a[u]), 1.0f);
        }
      }
    } else if (p.x_mode == GemvInput::kRmsNorm) {
      // the same over hidden states of more than 4 groups per thread
      float ss = 0.f;
      const float4 *a4 = reinterpret_cast<const float4 *>(p.xa);
      for (int k = threadIdx.x; k < ngroups * 2; k += blockDim.x) {
        const float4 v = __ldg(a4 + k);
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      ss = warp_sum(ss);
      float *red = parts;  // free until the main loop
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int w = 0; w < nwarps; ++w) tot += red[w];
      const float scale = rms_scale(tot, ngroups * 8, p.eps);
      // XU groups' loads in flight per thread before any is used (each
      // round trip to L2 is paid once per XU groups, not once per group)
      constexpr int XU = 4;
      for (int base = threadIdx.x; base < ngroups; base += XU * blockDim.x) {
        float a[XU][8], w[XU][8];
#pragma unroll
        for (int u = 0; u < XU; ++u) {
          const int i = base + u * blockDim.x;
          if (i < ngroups) {
            load8(p.xa, i, a[u]);
            load8(p.xb, i, w[u]);
          }
        }
#pragma unroll
        for (int u = 0; u < XU; ++u) {
          const int i = base + u * blockDim.x;
          if (i < ngroups) {
#pragma unroll
            for (int e = 0; e < 8; ++e) a[u][e] = (a[u][e] * scale) * safe_weight(w[u][e]);
            stage(i, pack(a[u]), 1.0f);
          }
        }
      }
    } else {  // kSwiGLU, with a power-of-two scale per sub-block
      constexpr int XU = 4;  // groups' loads in flight per thread, as above
      for (int base = threadIdx.x; base < ngroups; base += XU * blockDim.x) {
        float ga[XU][8], ua[XU][8];
#pragma unroll
        for (int v = 0; v < XU; ++v) {
          const int i = base + v * blockDim.x;
          if (i < ngroups) {
            load8(p.xa, i, ga[v]);
            load8(p.xb, i, ua[v]);
          }
        }
#pragma unroll
        for (int v = 0; v < XU; ++v) {
          const int i = base + v * blockDim.x;
          if (i >= ngroups) continue;  // whole warps: ngroups is a multiple of 32
          float *g = ga[v];
          float m = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            g[e] = swiglu(g[e], ua[v][e]);
            m = fmaxf(m, fabsf(g[e]));
          }
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
          const int ex = max(0, (int)((__float_as_uint(m) >> 23) & 0xFF) - 127 - 14);
          const float inv = __uint_as_float((uint32_t)(127 - ex) << 23);
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] *= inv;
          stage(i, pack(ga[v]), __uint_as_float((uint32_t)(127 + ex) << 23));
        }
      }
    }
  }
  __syncthreads();
  if (!has_work) return;

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

  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // rows g, g+8, g+16, g+24 of the current tile

  // store a finished row sum (lane = row in tile); with gate/up pairing, the
  // second of tiles t and t +- pair_tiles to be stored also forms
  // h = silu(gate) * up of their 32 rows (the scaled fp16 form)
  auto store_row = [&](int t, float s) {
    const int r = t * kTileRows + lane;
    if (r < p.rows) p.y[r] = s + (p.residual ? p.residual[r] : 0.f);
    if (p.pair_h == nullptr) return;
    const int pt = t < p.pair_tiles ? t : t - p.pair_tiles;
    __threadfence();  // this tile's rows are visible before it is counted
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(p.pair_ctr + pt, 1);
    if (__shfl_sync(0xffffffffu, old, 0) == 0) return;
    __threadfence();
    const int e = pt * kTileRows + lane;
    const float h = swiglu(__ldcg(p.y + e), __ldcg(p.y + (size_t)p.pair_tiles * kTileRows + e));
    const int ex = silu_scale_exp(warp_max(fabsf(h)));
    p.pair_h[e] = __float2half_rn(h * __uint_as_float((uint32_t)(127 - ex) << 23));
    if (lane == 0) {
      p.pair_scale[pt] = __uint_as_float((uint32_t)(127 + ex) << 23);
      p.pair_ctr[pt] = 0;
    }
  };

  // A tile shared with neighbouring CTAs: publish this CTA's part; the last
  // CTA to arrive adds the CTAs' parts in CTA order.
  auto cta_finish = [&](int t, float s) {
    const bool inside = (t * p.nb >= co.u0) && ((t + 1) * p.nb <= co.u1);
    if (inside) {
      store_row(t, s);
      return;
    }
    const int end = (t == co.t_first) ? 0 : 1;
    __stcg(p.partials + ((size_t)c * 2 + end) * kTileRows + lane, s);
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(p.counters + t, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    const int cf = cta_of_unit(t * p.nb, p), cl = cta_of_unit((t + 1) * p.nb - 1, p);
    if (old == cl - cf) {
      __threadfence();
      const int slot_cf = (unit_begin(cf, p) == t * p.nb) ? 0 : 1;
      float tot = __ldcg(p.partials + ((size_t)cf * 2 + slot_cf) * kTileRows + lane);
      for (int cc = cf + 1; cc <= cl; ++cc)
        tot += __ldcg(p.partials + ((size_t)cc * 2) * kTileRows + lane);
      store_row(t, tot);
      if (lane == 0) p.counters[t] = 0;
    }
  };

  // The warp's run of tile t ended at position q_end (exclusive) after
  // starting at q_beg: combine with the other warps' runs of the tile.
  int my_first_tile;
  {
    const int u = co.unit_of(q0);
    my_first_tile = div_nb(u, p);
  }
  auto finish_run = [&](int t, int q_beg, int q_end) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
      acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);
    }
    int qa, qb;
    co.tile_range(t, p.nb, qa, qb);
    if (q_beg == qa && q_end == qb) {  // this warp holds the CTA's whole part
      // lane r needs row r: rows g + 8i live in lane 4g (tig 0), slot i
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = __shfl_sync(0xffffffffu, acc[i], (lane & 7) << 2);
        if ((lane >> 3) == i) s = v;
      }
      cta_finish(t, s);
    } else {
      const int slot = (t == my_first_tile) ? 0 : 1;
      float *pp = parts + (warp * 2 + slot) * kTileRows;
      if (tig == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) pp[g + 8 * i] = acc[i];
      }
      __syncwarp();
      const int wa = warp_of_q(qa), wb = warp_of_q(qb - 1);
      int old = 0;
      if (lane == 0) {
        __threadfence_block();
        old = atomicAdd(tile_done + (t - co.t_first), 1);
      }
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old == wb - wa) {  // the last of the tile's warps
        __threadfence_block();
        const volatile float *vp = parts;
        const int slot_wa = (qstart(wa) == qa) ? 0 : 1;
        float s = vp[(wa * 2 + slot_wa) * kTileRows + lane];
        for (int w = wa + 1; w <= wb; ++w) s += vp[(w * 2) * kTileRows + lane];
        cta_finish(t, s);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = 0.f;
  };

  // ---- main loop: one unit per iteration ------------------------------------
  int qc = q0, tc = 0, bc = 0;  // consumer cursor
  {
    const int u = co.unit_of(q0);
    tc = div_nb(u, p);
    bc = u - tc * p.nb;
  }
  int run_beg = q0;
  int st_out = 0;
  uint32_t phases = 0;  // bit s: parity of the next completion of stage s
  bool ok = true;
  while (qc < q1) {
    issue_next();
    if (!mbar_wait_bounded(my_bar + 8 * st_out, (phases >> st_out) & 1, p.status)) {
      ok = false;
      break;
    }
    phases ^= 1u << st_out;

    const uint8_t *st = my_stages + st_out * kStageBytes;
    const uint32_t xlo = x_lo_base + bc * x_lo_step;
    const uint32_t xhi = x_hi_base + bc * x_hi_step;
    const float2 xs = *reinterpret_cast<const float2 *>(xsum + bc * 8 + 2 * tig);
    const float2 xsc = *reinterpret_cast<const float2 *>(xscl + bc * 8 + 2 * tig);

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
      // sub-block sums of the stored x, times the x scale of each sub-block
      const float cs0 = fmaf(0.0625f, cacc[mt][1][2 * hr], cacc[mt][0][2 * hr]) * xsc.x;
      const float cs1 = fmaf(0.0625f, cacc[mt][1][2 * hr + 1], cacc[mt][0][2 * hr + 1]) * xsc.y;
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

    const int t_now = tc;
    advance(qc, tc, bc);
    if (qc == q1 || tc != t_now || qc == co.nf || qc == co.nf + co.nl) {
      finish_run(t_now, run_beg, qc);
      run_beg = qc;
    }
  }
  if (!ok) {
    // a stage wait ran out of budget: let the copies still in flight land
    // (bounded again) before this warp's shared memory is released
    for (int s = 0; s < kGemvStages; ++s) {
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
  int warps, units, ctas, ntile;
  size_t smem;
  uint32_t smem_bar, smem_x;
};

// The most warps whose shared-memory footprint fits.
// The most units a warp takes when a CTA holds s units over `warps` warps.
static long long units_per_warp(long long s, int warps) {
  const long long nwe = std::min<long long>(warps, s);
  return (s + nwe - 1) / nwe;
}

// CTA count: the grid holds every SM, and each CTA a contiguous run of units
// (its first and last tiles shared with its neighbours, their partial sums
// handed over through global memory) -- unless a count between half and all
// of the SMs divides the tiles without raising the most units a warp takes:
// then every CTA owns whole tiles and no partial sum leaves a CTA.
static int pick_ctas(int tiles, int nb, int sm_count, int warps) {
  const long long units = (long long)tiles * nb;
  const int split = (int)std::min<long long>(sm_count, units);
  const long long cost = units_per_warp((units + split - 1) / split, warps);
  for (int d = std::min(sm_count, tiles); 2 * d >= sm_count; --d)
    if (tiles % d == 0 && units_per_warp((long long)(tiles / d) * nb, warps) <= cost) return d;
  return split;
}

static bool plan_gemv(int rows, int nb, int sm_count, size_t smem_max, GemvPlan &pl) {
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  const long long units = (long long)tiles * nb;
  if (units * sm_count >= (1LL << 31) || units >= (1LL << 24)) return false;
  for (int warps = kGemvMaxWarps; warps >= 2; --warps) {
    const int ctas = pick_ctas(tiles, nb, sm_count, warps);
    const int umax = (int)((units + ctas - 1) / ctas);
    const int ntile = ((umax / nb + 2) + 3) & ~3;
    const size_t smem_bar = (size_t)warps * kGemvStages * kStageBytes;
    const size_t smem_x = smem_bar + (((size_t)warps * kGemvStages * 8 + 15) & ~(size_t)15);
    const size_t smem = smem_x + 64 + (size_t)nb * 32 * 16 + (size_t)nb * 8 * 4 * 2 +
                        (size_t)warps * 2 * kTileRows * 4 + (size_t)ntile * 4;
    if (smem <= smem_max) {
      pl = {warps, (int)units, ctas, ntile, smem, (uint32_t)smem_bar, (uint32_t)smem_x};
      return true;
    }
  }
  return false;
}

// W viewed as a 2D byte tensor [rows][nb * 144]; box = one block column of
// box_rows rows (144 bytes each).  Rows past the end read as zeros.
int encode_q4k_rows_map(mlm_ctx *ctx, const void *W, int rows, int nb, int box_rows,
                        CUtensorMap *map) {
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
  const cuuint32_t box[2] = {(cuuint32_t)kBlockBytes, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(W), dims,
                            strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ctx, MLM_ERR_CUDA, "mlm_q4k_gemv: tensor map encode failed (%d)", (int)r);
  return MLM_OK;
}

int gemv_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const GemvInput &in, float *y,
                const float *residual, float *partials, int *counters, int max_ctas,
                int max_tiles, cudaStream_t stream, const GemvPair *pair) {
  const int nb = cols / kQK;
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  MLM_REQUIRE(ctx, tiles <= max_tiles, MLM_ERR_SHAPE,
              "mlm_q4k_gemv: %d rows exceed the %d-row scratch limit", rows,
              max_tiles * kTileRows);
  MLM_REQUIRE(ctx, !pair || (rows % (2 * kTileRows) == 0 && pair->h_f16 && pair->h_scale &&
                             pair->counters && !residual),
              MLM_ERR_SHAPE, "mlm_q4k_gemv: gate/up pairing needs rows=%d a multiple of %d",
              rows, 2 * kTileRows);
  GemvPlan pl;
  // 228 KB of shared memory per SM, 1 KB of it reserved per resident CTA
  const size_t smem_cap = std::min((size_t)ctx->max_smem_optin,
                                   (size_t)233472 / MLM_GEMV_MIN_BLOCKS - 1024);
  const bool ok = plan_gemv(rows, nb, std::min(ctx->sm_count, max_ctas), smem_cap, pl);
  MLM_REQUIRE(ctx, ok, MLM_ERR_UNSUPPORTED,
              "mlm_q4k_gemv: rows=%d cols=%d does not fit the shared-memory plan", rows, cols);
  CUtensorMap tmap;
  int st = encode_q4k_rows_map(ctx, W, rows, nb, kTileRows, &tmap);
  if (st != MLM_OK) return st;
  GemvArgs a;
  a.W = reinterpret_cast<const uint8_t *>(W);
  a.x = reinterpret_cast<const __half *>(in.x_f16);
  a.x_scale = in.x_scale;
  a.xa = in.a;
  a.xb = in.b;
  a.eps = in.eps;
  a.x_mode = in.mode;
  a.y = y;
  a.residual = residual;
  a.partials = partials;
  a.counters = counters;
  a.pair_h = pair ? reinterpret_cast<__half *>(pair->h_f16) : nullptr;
  a.pair_scale = pair ? pair->h_scale : nullptr;
  a.pair_ctr = pair ? pair->counters : nullptr;
  a.pair_tiles = rows / (2 * kTileRows);
  a.status = ctx->dev_status;
  a.nb_magic = ((1ull << 40) + (unsigned long long)nb - 1) / (unsigned long long)nb;
  a.rows = rows;
  a.nb = nb;
  a.units = pl.units;
  a.ctas = pl.ctas;
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

int gemv_validate(mlm_ctx *ctx, const void *W, int rows, int cols, const GemvInput &in,
                  float *y) {
  const bool half = in.mode == GemvInput::kHalf;
  const void *x = half ? in.x_f16 : in.a;
  MLM_REQUIRE(ctx, W && x && y && (half || in.b), MLM_ERR_ARG, "mlm_q4k_gemv: null buffer");
  MLM_REQUIRE(ctx, half || (aligned16(in.a) && aligned16(in.b)), MLM_ERR_ALIGN,
              "mlm_q4k_gemv: fp32 inputs must be 16-byte aligned");
  MLM_REQUIRE(ctx, rows > 0 && cols > 0, MLM_ERR_SHAPE, "mlm_q4k_gemv: rows=%d cols=%d", rows,
              cols);
  MLM_REQUIRE(ctx, cols % kQK == 0, MLM_ERR_SHAPE,
              "mlm_q4k_gemv: cols=%d is not a multiple of the 256-element super-block", cols);
  MLM_REQUIRE(ctx, aligned16(W) && (!half || aligned16(x)), MLM_ERR_ALIGN,
              "mlm_q4k_gemv: W and x must be 16-byte aligned");
  return MLM_OK;
}

}  // namespace mlm

using namespace mlm;

static int gemv_entry(mlm_ctx *ctx, const void *W, int rows, int cols, const GemvInput &in,
                      float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  int st = gemv_validate(ctx, W, rows, cols, in, y);
  if (st != MLM_OK) return st;
  return gemv_launch(ctx, W, rows, cols, in, y, residual, ctx->gemv_partials,
                     ctx->gemv_counters, ctx->gemv_max_ctas, ctx->gemv_max_tiles, ctx->stream);
}

extern "C" int mlm_q4k_gemv(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                            float *y, const float *residual) {
  return gemv_entry(ctx, W, rows, cols, gemv_half(x_f16), y, residual);
}

extern "C" int mlm_q4k_gemv_xs(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                               const float *x_scale, float *y, const float *residual) {
  if (ctx && !x_scale) return set_error(ctx, MLM_ERR_ARG, "mlm_q4k_gemv_xs: null x_scale");
  return gemv_entry(ctx, W, rows, cols, gemv_half(x_f16, x_scale), y, residual);
}

extern "C" int mlm_q4k_gemv_rmsnorm(mlm_ctx *ctx, const void *W, int rows, int cols,
                                    const float *hidden, const float *norm_w, float eps,
                                    float *y, const float *residual) {
  GemvInput in;
  in.mode = GemvInput::kRmsNorm;
  in.a = hidden;
  in.b = norm_w;
  in.eps = eps;
  return gemv_entry(ctx, W, rows, cols, in, y, residual);
}

extern "C" int mlm_q4k_gemv_swiglu(mlm_ctx *ctx, const void *W, int rows, int cols,
                                   const float *gate, const float *up, float *y,
                                   const float *residual) {
  GemvInput in;
  in.mode = GemvInput::kSwiGLU;
  in.a = gate;
  in.b = up;
  return gemv_entry(ctx, W, rows, cols, in, y, residual);
}

extern "C" int mlm_q4k_gemv_gate_up(mlm_ctx *ctx, const void *W, int rows, int cols,
                                    const float *hidden, const float *norm_w, float eps,
                                    float *y, void *h_f16, float *h_scale) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, h_f16 && h_scale, MLM_ERR_ARG, "mlm_q4k_gemv_gate_up: null h buffer");
  GemvInput in;
  in.mode = GemvInput::kRmsNorm;
  in.a = hidden;
  in.b = norm_w;
  in.eps = eps;
  int st = gemv_validate(ctx, W, rows, cols, in, y);
  if (st != MLM_OK) return st;
  GemvPair pair;
  pair.h_f16 = h_f16;
  pair.h_scale = h_scale;
  pair.counters = ctx->gemv_counters + ctx->gemv_max_tiles;
  return gemv_launch(ctx, W, rows, cols, in, y, nullptr, ctx->gemv_partials, ctx->gemv_counters,
                     ctx->gemv_max_ctas, ctx->gemv_max_tiles, ctx->stream, &pair);
}

extern "C" int mlm_q4k_gemv_plan(int rows, int cols, int sm_count, int *ctas, int *warps,
                                 int *whole_tiles) {
  if (rows <= 0 || cols <= 0 || cols % kQK != 0 || sm_count <= 0 || !ctas || !warps ||
      !whole_tiles)
    return MLM_ERR_ARG;
  GemvPlan pl;
  // the opt-in limit of a B200 (227 KB), 1 KB of an SM's 228 KB reserved per CTA
  const size_t smem_cap = std::min((size_t)232448, (size_t)233472 / MLM_GEMV_MIN_BLOCKS - 1024);
  if (!plan_gemv(rows, cols / kQK, sm_count, smem_cap, pl)) return MLM_ERR_UNSUPPORTED;
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  *ctas = pl.ctas;
  *warps = pl.warps;
  *whole_tiles = tiles % pl.ctas == 0 ? 1 : 0;
  return MLM_OK;
}

// ---------------------------------------------------------------------------
// mlm_q4k_gemv_static: the same kernel with its split-K scratch in a
// file-scope device array instead of the context's allocation.
//
// Who needs it: a host that owns every byte of device memory through its own
// pool (or runs under a hard memory budget) and may not let a library
// allocate, and code that enqueues work from a place where an allocation
// would stall or is not allowed (a latency-critical decode loop; a region
// that is being recorded into a graph).  This entry point allocates nothing:
// no cudaMalloc, no cudaFree, no allocating library routine.
//
// Limits: at most kStaticMaxRows rows and kStaticMaxCtas CTAs (the grid is
// capped there); larger shapes are rejected with MLM_ERR_SHAPE.  The array is
// 80 KB per device and lives in the library image, loaded with the module.
//
// Set-up: the first call on a device looks up the array's device address
// with cudaGetSymbolAddress (that device current) and clears it; calls after
// that only read the cached address.  Make that first call before any stream
// capture begins.
//
// Sharing: every call on a device uses the same array, which keeps the last
// call's contents.  The arrival counters are cleared on the caller's stream
// before every launch (the partials need no clearing: each is written before
// it is read).  Calls that overlap on the GPU -- two streams, two contexts on
// one device, two host threads -- race on the array and give wrong results;
// order them on one stream.
// ---------------------------------------------------------------------------

namespace mlm {

constexpr int kStaticMaxRows = 131072;                        // 4096 row tiles
constexpr int kStaticMaxTiles = kStaticMaxRows / kTileRows;
constexpr int kStaticMaxCtas = 256;
constexpr size_t kStaticPartialBytes = (size_t)kStaticMaxCtas * 2 * kTileRows * sizeof(float);
constexpr size_t kStaticScratchBytes = kStaticPartialBytes + (size_t)kStaticMaxTiles * sizeof(int);
constexpr int kStaticMaxDevices = 64;

static __device__ __align__(256) unsigned char g_gemv_static_scratch[kStaticScratchBytes];

static std::mutex g_static_mu;
static void *g_static_addr[kStaticMaxDevices];  // set once per device, under g_static_mu

static int gemv_static_scratch(mlm_ctx *ctx, void **out) {
  int cur = -1;
  MLM_CUDA_TRY(ctx, cudaGetDevice(&cur));
  MLM_REQUIRE(ctx, cur == ctx->device, MLM_ERR_STATE,
              "mlm_q4k_gemv_static: device %d is current, the context is on device %d", cur,
              ctx->device);
  MLM_REQUIRE(ctx, cur >= 0 && cur < kStaticMaxDevices, MLM_ERR_UNSUPPORTED,
              "mlm_q4k_gemv_static: device %d beyond the %d-device table", cur,
              kStaticMaxDevices);
  std::lock_guard<std::mutex> g(g_static_mu);
  if (!g_static_addr[cur]) {
    void *p = nullptr;
    MLM_CUDA_TRY(ctx, cudaGetSymbolAddress(&p, g_gemv_static_scratch));
    MLM_REQUIRE(ctx, p != nullptr, MLM_ERR_CUDA, "mlm_q4k_gemv_static: null scratch address");
    MLM_CUDA_TRY(ctx, cudaMemset(p, 0, kStaticScratchBytes));
    g_static_addr[cur] = p;
  }
  *out = g_static_addr[cur];
  return MLM_OK;
}

}  // namespace mlm

extern "C" int mlm_q4k_gemv_static(mlm_ctx *ctx, const void *W, int rows, int cols,
                                   const void *x_f16, float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  int st = mlm::gemv_validate(ctx, W, rows, cols, mlm::gemv_half(x_f16), y);
  if (st != MLM_OK) return st;
  MLM_REQUIRE(ctx, rows <= mlm::kStaticMaxRows, MLM_ERR_SHAPE,
              "mlm_q4k_gemv_static: rows=%d exceeds the static scratch limit of %d rows", rows,
              mlm::kStaticMaxRows);
  void *scratch = nullptr;
  st = mlm::gemv_static_scratch(ctx, &scratch);
  if (st != MLM_OK) return st;
  float *partials = reinterpret_cast<float *>(scratch);
  int *counters =
      reinterpret_cast<int *>(reinterpret_cast<unsigned char *>(scratch) + mlm::kStaticPartialBytes);
  const int tiles = (rows + mlm::kTileRows - 1) / mlm::kTileRows;
  MLM_CUDA_TRY(ctx, cudaMemsetAsync(counters, 0, sizeof(int) * (size_t)tiles, ctx->stream));
  return mlm::gemv_launch(ctx, W, rows, cols, mlm::gemv_half(x_f16), y, residual, partials,
                          counters, mlm::kStaticMaxCtas, mlm::kStaticMaxTiles, ctx->stream);
}
