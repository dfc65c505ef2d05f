// q4k_gemv_tiled.cu -- Q4_K x fp16 decode GEMV on weights re-laid out once at
// load time for streaming, and the re-layout itself.
//
// The same 144-byte Q4_K blocks as the GGUF file (the loader still uploads
// them unchanged, DequantKernels.metal:20-27), reordered on the device by
// mlm_q4k_tile so that the decode GEMV reads HBM as one contiguous stream.
// The reference also converts its Q4_K weights after upload (to fp16,
// ModelLoader.swift:275-299); this conversion keeps them packed.
//
// Tiled layout.  A unit is one block column of a 32-row tile: rows
// 32t .. 32t+31 of block column b, 4608 bytes, stored contiguously at
// (t * nb + b) * 4608, tiles in order.  Inside a unit:
//   bytes    0 ..  511: the 16-byte headers (d, dmin, 12 scale bytes) of
//                       rows g + 8i, as [i = 0..3][g = 0..7];
//   bytes  512 .. 4607: quants, as [i][h = 0..1][g][t = 0..3] 16-byte
//                       pieces: qs bytes 64h + 16t .. 64h + 16t + 15 of row
//                       g + 8i (sub-block t + 4h).
// Lane (g = lane/4, t = lane%4) of a warp needs exactly the headers of rows
// g + 8i and sub-blocks t and t + 4 of those rows (the MMA mapping of the
// GEMV below), so each 16-byte piece it reads is adjacent to its
// neighbours': every warp read is 512 contiguous bytes.  Rows past the end
// of the weight are zero.
//
// GEMV.  Same arithmetic and MMA mapping as the GGUF-layout GEMV
// (q4k_gemv.cu): nibbles masked into fp16 subnormals on mma.sync
// m16n8k16, per-sub-block sums scaled in the epilogue.  Work split: each
// CTA owns a contiguous range of units (its first and last tiles possibly
// shared with its neighbours), walked boundary tiles first; position q of
// that order goes to compute warp q mod 8.  A round is 8 consecutive
// positions (one unit per compute warp).  A producer warp streams rounds
// into a ring of up to 6 round buffers (up to 216 KB) with 1D bulk copies
// -- at most three per round, one per contiguous run of units -- each round
// completing on a "full" mbarrier; compute warps copy their unit to
// registers, release the round on its "empty" mbarrier and compute.  The
// first rounds are issued before the kernel waits on its predecessor
// (programmatic dependent launch): weights never depend on an earlier
// kernel, and a streaming read needs on the order of 128 KB in flight per
// SM to reach full HBM bandwidth.  Tiles are combined as in the
// GGUF-layout GEMV, except that tiles shared with a neighbouring CTA are
// finished by a reducer warp, so the global exchange (a fence and an atomic,
// microseconds under load) never stalls a compute warp.  All waits are
// bounded; a wait that runs out sets the context's error word, and the
// warps still complete every barrier they take part in.
#include <algorithm>

#include "mlm_internal.h"
#include "q4k_gemv_common.cuh"

namespace mlm {
namespace {

constexpr int kCw = 8;                                // compute warps per CTA
constexpr int kWarps = kCw + 2;                       // + producer + reducer
constexpr int kProducer = kCw, kReducer = kCw + 1;    // warp indices
constexpr int kUnitBytes = kTileRows * kBlockBytes;   // 4608
constexpr int kRoundBytes = kCw * kUnitBytes;         // 36864
constexpr int kMaxRing = 6;
constexpr int kUnitChunks = kUnitBytes / 16;          // 288 16-byte pieces

struct TiledArgs {
  const uint8_t *W;  // tiled layout
  const __half *x;
  float *y;
  const float *residual;
  float *partials;  // [ctas][2][32]
  int *counters;    // [tiles]
  int *status;      // device-visible error word (0 = ok)
  unsigned long long nb_magic;  // ceil(2^40 / nb): u / nb == (u * magic) >> 40
  int rows;
  int nb;      // blocks per row = units per tile
  int units;   // tiles * nb
  int ctas;    // grid size
  int ntile;   // tiles a CTA can touch (multiple of 4)
  int nslot;   // tiles with per-warp parts in shared memory (0 when nb == 1)
  int ring;    // round buffers
  uint32_t smem_x;  // byte offset of the x region
};

__device__ __forceinline__ void bulk_copy(uint32_t dst, const uint8_t *src, uint32_t bytes,
                                          uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t word_of(const uint4 &v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// GGUF layout -> tiled layout, one 16-byte piece per thread.
__global__ void q4k_tile_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                int rows, int nb, long long npieces) {
  for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < npieces;
       c += (long long)gridDim.x * blockDim.x) {
    const long long unit = c / kUnitChunks;
    const int k = (int)(c - unit * kUnitChunks);
    const long long t = unit / nb;
    const int b = (int)(unit - t * nb);
    int i, g, off;
    if (k < 32) {  // header of row g + 8i
      i = k >> 3;
      g = k & 7;
      off = 0;
    } else {  // quants: [i][h][g][t]
      const int k2 = k - 32;
      i = k2 >> 6;
      g = (k2 >> 2) & 7;
      off = 16 + 64 * ((k2 >> 5) & 1) + 16 * (k2 & 3);
    }
    const long long r = t * kTileRows + g + 8 * i;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < rows)
      v = *reinterpret_cast<const uint4 *>(src + ((size_t)r * nb + b) * kBlockBytes + off);
    *reinterpret_cast<uint4 *>(dst + (size_t)c * 16) = v;
  }
}

__global__ void __launch_bounds__(kWarps * 32, 1) q4k_gemv_tiled_kernel(TiledArgs p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t ring_addr = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t full_bar = ring_addr + (uint32_t)p.ring * kRoundBytes;
  const uint32_t empty_bar = full_bar + 8u * (uint32_t)p.ring;
  uint4 *xzero = reinterpret_cast<uint4 *>(smem + p.smem_x);
  uint4 *xperm = xzero + 4;                                    // after 64 zero bytes
  float *xsum = reinterpret_cast<float *>(xperm + p.nb * 32);  // [nb][8], paired
  float *parts = xsum + p.nb * 8;                              // [nslot][kCw][32]
  int *tile_done = reinterpret_cast<int *>(parts + p.nslot * kCw * kTileRows);  // [ntile]

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int c = blockIdx.x;

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
  const int K = (co.S + kCw - 1) / kCw;  // rounds
  // the compute warps that hold positions of tile t are those of positions
  // qa .. qa + npart - 1 (position q belongs to warp q mod kCw)
  const int nwe = min(kCw, co.S);
  auto npart_of = [&](int qa, int qb) { return min(nwe, qb - qa); };
  auto tile_of_q = [&](int q, int &t, int &b) {
    const int u = co.unit_of(q);
    t = div_nb(u, p);
    b = u - t * p.nb;
  };
  // boundary tiles are shared with a neighbouring CTA and finished by the
  // reducer warp: named barrier 1 (first tile), 2 (last tile)
  auto boundary_id = [&](int t) {
    if (t == co.t_first && co.nf > 0) return 1;
    if (t == co.t_last && co.nl > 0) return 2;
    return 0;
  };

  // ---- producer: round k holds positions 8k .. 8k+7 in ring slot k % ring -
  const uint64_t pol = evict_first_policy();
  auto issue_round = [&](int k) {
    const int s = k % p.ring;
    const int q0 = k * kCw, q1 = min(q0 + kCw, co.S);
    const uint32_t bar = full_bar + 8u * s;
    mbar_expect_tx(bar, (uint32_t)(q1 - q0) * kUnitBytes);
    for (int q = q0; q < q1;) {  // runs of positions contiguous in memory
      int qe = q1;
      if (q < co.nf)
        qe = min(qe, co.nf);
      else if (q < co.nf + co.nl)
        qe = min(qe, co.nf + co.nl);
      bulk_copy(ring_addr + (uint32_t)s * kRoundBytes + (uint32_t)(q - q0) * kUnitBytes,
                p.W + (size_t)co.unit_of(q) * kUnitBytes, (uint32_t)(qe - q) * kUnitBytes, bar,
                pol);
      q = qe;
    }
  };
  int issued = 0;
  if (warp == kProducer && lane == 0) {
    for (int s = 0; s < p.ring; ++s) {
      mbar_init(full_bar + 8u * s, 1);
      mbar_init(empty_bar + 8u * s, kCw);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // weights never depend on an earlier kernel: fill the ring now
    for (; issued < min(p.ring, K); ++issued) issue_round(issued);
  }

  // Programmatic dependent launch: x, y and the split-K scratch may belong to
  // the previous kernel on the stream, so wait for it here.  Dependents may
  // start as soon as SMs free up.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");

  // ---- x -> shared memory, permuted, plus per-sub-block sums ---------------
  // xsum keeps the sums of sub-blocks j and j + 4 of a block side by side
  // (position 2j and 2j + 1), the pair one lane scales.
  {
    const uint4 *xg = reinterpret_cast<const uint4 *>(p.x);
    const int ngroups = p.nb * 32;  // multiple of 32: whole warps stay converged
    constexpr int XB = 4;           // x loads in flight per thread
    if (threadIdx.x < 4) xzero[threadIdx.x] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < p.ntile; i += blockDim.x) tile_done[i] = 0;
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
          if ((i & 3) == 0) {
            const int sb = i >> 2, j = sb & 7;
            xsum[(sb & ~7) + ((j < 4) ? 2 * j : 2 * (j - 4) + 1)] = sx;
          }
        }
      }
    }
  }
  __syncthreads();

  if (warp == kProducer) {
    if (lane == 0) {
      for (; issued < K; ++issued) {  // refill a slot once its round is read
        const int k = issued, s = k % p.ring;
        if (!mbar_wait_bounded(empty_bar + 8u * s, ((k / p.ring) - 1) & 1, p.status)) break;
        issue_round(k);
      }
      // the copies in flight land before this CTA's shared memory is released
      for (int k = max(0, issued - p.ring); k < issued; ++k)
        if (!mbar_wait_bounded(full_bar + 8u * (k % p.ring), (k / p.ring) & 1, p.status)) break;
    }
    return;
  }

  // store a finished row sum (lane = row in tile)
  auto store_row = [&](int t, float s) {
    const int r = t * kTileRows + lane;
    if (r < p.rows) p.y[r] = s + (p.residual ? p.residual[r] : 0.f);
  };
  // sum of tile t's parts in the order of the positions that hold them
  auto sum_parts = [&](int t, int qa, int npart) {
    const volatile float *vp = parts + (size_t)(t - co.t_first) * kCw * kTileRows;
    float s = vp[(qa % nwe) * kTileRows + lane];
    for (int k = 1; k < npart; ++k) s += vp[((qa + k) % nwe) * kTileRows + lane];
    return s;
  };

  if (warp == kReducer) {
    // Boundary tiles: add the compute warps' parts, then publish this CTA's
    // part; the last CTA to arrive adds the CTAs' parts in CTA order.
    for (int id = 1; id <= 2; ++id) {
      if ((id == 1 && co.nf == 0) || (id == 2 && co.nl == 0)) continue;
      const int t = (id == 1) ? co.t_first : co.t_last;
      int qa, qb;
      co.tile_range(t, p.nb, qa, qb);
      const int npart = npart_of(qa, qb);
      asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(32 * (npart + 1)) : "memory");
      const float s = sum_parts(t, qa, npart);
      const int end = (id == 1) ? 0 : 1;
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
    }
    return;
  }

  // ---- compute warps ----------------------------------------------------------
  // B operands: thread (g, t) carries x of sub-block t when g == 2t and of
  // sub-block t + 4 when g == 2t + 1 (the B columns those sub-blocks sum
  // into), zeros otherwise.
  const int act = g - 2 * tig;
  const uint32_t xzero_addr = (uint32_t)__cvta_generic_to_shared(xzero);
  const uint32_t xperm_addr = (uint32_t)__cvta_generic_to_shared(xperm);
  const uint32_t x_lo_base = (act == 0) ? xperm_addr + 16 * (4 * tig) : xzero_addr;
  const uint32_t x_hi_base = (act == 1) ? xperm_addr + 16 * (16 + 4 * tig) : xzero_addr;
  const uint32_t x_lo_step = (act == 0) ? 512u : 0u;  // per block column
  const uint32_t x_hi_step = (act == 1) ? 512u : 0u;

  // scale/min unpack of sub-blocks t and t + 4 (get_scale_min_k4): one byte
  // permute gathers bytes t of the three scale words, masks finish the
  // 6-bit values (sub-block t + 4 takes its top two bits from the bytes of
  // sub-block t).
  const uint32_t psel = tig | ((4 + tig) << 4) | (tig << 8) | (tig << 12);

  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // rows g, g+8, g+16, g+24 of the current tile

  // This warp is done with tile t: leave its part, then either hand the
  // tile to the reducer warp (boundary tiles) or, for the last of the
  // tile's warps, add the parts and store y.
  auto finish_tile = [&](int t) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
      acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);
    }
    int qa, qb;
    co.tile_range(t, p.nb, qa, qb);
    const int npart = npart_of(qa, qb);
    const int id = boundary_id(t);
    if (npart == 1 && id == 0) {
      // lane r needs row r: rows g + 8i live in lane 4g (tig 0), slot i
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float v = __shfl_sync(0xffffffffu, acc[i], (lane & 7) << 2);
        if ((lane >> 3) == i) s = v;
      }
      store_row(t, s);
    } else {
      float *pp = parts + ((size_t)(t - co.t_first) * kCw + warp) * kTileRows;
      if (tig == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) pp[g + 8 * i] = acc[i];
      }
      __syncwarp();
      if (id != 0) {
        __threadfence_block();
        asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(32 * (npart + 1)) : "memory");
      } else {
        int old = 0;
        if (lane == 0) {
          __threadfence_block();
          old = atomicAdd(tile_done + (t - co.t_first), 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == npart - 1) {  // the last of the tile's warps
          __threadfence_block();
          store_row(t, sum_parts(t, qa, npart));
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = 0.f;
  };

  // one unit: sub-block sums on the tensor cores, then the scales
  auto compute_unit = [&](const uint4 (&buf)[12], int bc) {
    const uint32_t xlo = x_lo_base + bc * x_lo_step;
    const uint32_t xhi = x_hi_base + bc * x_hi_step;
    const float2 xs = *reinterpret_cast<const float2 *>(xsum + bc * 8 + 2 * tig);

    // [mt][chain]: chain 0 = mask 0x000F000F, chain 1 = mask 0x00F000F0 (x16).
    // Column 2t only collects sub-block t and column 2t+1 sub-block t + 4
    // (their B columns), so one chain holds both sub-block sums.
    float cacc[2][2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int ch = 0; ch < 2; ++ch)
        cacc[mt][ch][0] = cacc[mt][ch][1] = cacc[mt][ch][2] = cacc[mt][ch][3] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint4 xb = lds128((j < 4) ? xlo + 16 * j : xhi + 16 * (j - 4));
      const int part = 1 + (j >> 2), k = j & 3;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint32_t w0 = word_of(buf[3 * (2 * mt) + part], k);
        const uint32_t w1 = word_of(buf[3 * (2 * mt + 1) + part], k);
        const uint32_t t0 = w0 >> 8, t1 = w1 >> 8;
        const uint32_t M = 0x000F000Fu, M16 = 0x00F000F0u;
        mma_f16_16816(cacc[mt][0], w0 & M, w1 & M, t0 & M, t1 & M, xb.x, xb.y);
        mma_f16_16816(cacc[mt][1], w0 & M16, w1 & M16, t0 & M16, t1 & M16, xb.z, xb.w);
      }
    }

    // epilogue: scale the sub-block sums of columns 2t (sub-block t) and
    // 2t + 1 (sub-block t + 4)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int mt = i >> 1, hr = i & 1;
      const uint4 h = buf[3 * i];
      const float cs0 = fmaf(0.0625f, cacc[mt][1][2 * hr], cacc[mt][0][2 * hr]);
      const float cs1 = fmaf(0.0625f, cacc[mt][1][2 * hr + 1], cacc[mt][0][2 * hr + 1]);
      const uint32_t P = __byte_perm(h.y, h.w, psel);  // [s_t, s_8+t, -, s_t]
      const uint32_t Q = __byte_perm(h.z, h.w, psel);  // [s_4+t, s_8+t, -, s_4+t]
      const uint32_t scp = (P & 0x0F3Fu) | ((P >> 18) & 0x3000u);
      const uint32_t mp = (Q & 0x003Fu) | ((Q >> 4) & 0x0F00u) | ((Q >> 18) & 0x3000u);
      const float D = half_bits_to_float(h.x) * 16777216.0f;  // d * 2^24
      const float Dm = half_bits_to_float(h.x >> 16);
      const float qs = (float)(scp & 0xFF) * cs0 + (float)(scp >> 8) * cs1;
      const float ms = (float)(mp & 0xFF) * xs.x + (float)(mp >> 8) * xs.y;
      acc[i] += D * qs - Dm * ms;
    }
  };

  // this warp's unit inside a round buffer
  const uint32_t unit_off = (uint32_t)warp * kUnitBytes;
  const uint32_t hdr_off = (uint32_t)g * 16;
  const uint32_t q_off = 512u + (uint32_t)lane * 16;
  int tc = 0, bc = 0;
  if (warp < co.S) tile_of_q(warp, tc, bc);
  bool ok = true;
  for (int k = 0; k < K; ++k) {
    const int s = k % p.ring;
    const int q = k * kCw + warp;
    const bool mine = q < co.S;
    uint4 buf[12];
    // Every compute warp waits for every round, its unit or not: a round
    // exists only once the slot's previous round was released by all eight
    // warps, so this warp's release below always counts toward this round.
    if (ok) ok = mbar_wait_bounded(full_bar + 8u * s, (k / p.ring) & 1, p.status);
    if (mine && ok) {
      const uint32_t u = ring_addr + (uint32_t)s * kRoundBytes + unit_off;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        buf[3 * i] = lds128(u + hdr_off + 128u * i);
        buf[3 * i + 1] = lds128(u + q_off + 1024u * i);
        buf[3 * i + 2] = lds128(u + q_off + 1024u * i + 512u);
      }
    }
    // the round's reads are done (in registers): release its buffer
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar + 8u * s);
    if (!mine) continue;
    if (ok) compute_unit(buf, bc);
    const int qn = q + kCw;
    if (qn >= co.S) {
      finish_tile(tc);
    } else {
      const int t_now = tc;
      tile_of_q(qn, tc, bc);
      if (tc != t_now) finish_tile(t_now);
    }
  }
}

struct TiledPlan {
  int units, ctas, ntile, nslot, ring;
  size_t smem;
  uint32_t smem_x;
};

static bool plan_tiled(int rows, int nb, int sm_count, size_t smem_max, TiledPlan &pl) {
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  const long long units = (long long)tiles * nb;
  const int ctas = (int)std::min<long long>(sm_count, units);
  if (units * ctas >= (1LL << 31) || units >= (1LL << 24)) return false;
  const int umax = (int)((units + ctas - 1) / ctas);
  const int ntile = ((umax / nb + 2) + 3) & ~3;
  const int nslot = (nb == 1) ? 0 : ntile;  // one-unit tiles never share
  const size_t xbytes = 64 + (size_t)nb * 32 * 16 + (size_t)nb * 8 * 4 +
                        (size_t)nslot * kCw * kTileRows * 4 + (size_t)ntile * 4;
  for (int ring = kMaxRing; ring >= 2; --ring) {
    const size_t smem_x = (size_t)ring * kRoundBytes + 16 * (size_t)ring;
    if (smem_x + xbytes <= smem_max) {
      pl = {(int)units, ctas, ntile, nslot, ring, smem_x + xbytes, (uint32_t)smem_x};
      return true;
    }
  }
  return false;
}

}  // namespace

int gemv_tiled_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q4k_gemv_tiled_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ctx->max_smem_optin));
  return MLM_OK;
}

}  // namespace mlm

using namespace mlm;

extern "C" size_t mlm_q4k_tiled_bytes(int rows, int cols) {
  if (rows <= 0 || cols <= 0 || cols % kQK != 0) return 0;
  const size_t tiles = ((size_t)rows + kTileRows - 1) / kTileRows;
  return tiles * (size_t)(cols / kQK) * kUnitBytes;
}

extern "C" int mlm_q4k_tile(mlm_ctx *ctx, const void *W, int rows, int cols, void *W_tiled) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, W && W_tiled, MLM_ERR_ARG, "mlm_q4k_tile: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && cols > 0 && cols % kQK == 0, MLM_ERR_SHAPE,
              "mlm_q4k_tile: rows=%d cols=%d (cols must be a multiple of 256)", rows, cols);
  MLM_REQUIRE(ctx, aligned16(W) && aligned16(W_tiled), MLM_ERR_ALIGN,
              "mlm_q4k_tile: buffers must be 16-byte aligned");
  const int nb = cols / kQK;
  const long long npieces = (long long)mlm_q4k_tiled_bytes(rows, cols) / 16;
  const int grid = (int)std::min<long long>((npieces + 255) / 256, (long long)ctx->sm_count * 8);
  q4k_tile_kernel<<<grid, 256, 0, ctx->stream>>>(reinterpret_cast<const uint8_t *>(W),
                                                  reinterpret_cast<uint8_t *>(W_tiled), rows, nb,
                                                  npieces);
  return check_launch(ctx, "mlm_q4k_tile");
}

extern "C" int mlm_q4k_gemv_tiled(mlm_ctx *ctx, const void *W_tiled, int rows, int cols,
                                  const void *x_f16, float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, W_tiled && x_f16 && y, MLM_ERR_ARG, "mlm_q4k_gemv_tiled: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && cols > 0 && cols % kQK == 0, MLM_ERR_SHAPE,
              "mlm_q4k_gemv_tiled: rows=%d cols=%d (cols must be a multiple of 256)", rows, cols);
  MLM_REQUIRE(ctx, aligned16(W_tiled) && aligned16(x_f16), MLM_ERR_ALIGN,
              "mlm_q4k_gemv_tiled: W and x must be 16-byte aligned");
  const int nb = cols / kQK;
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  MLM_REQUIRE(ctx, tiles <= ctx->gemv_max_tiles, MLM_ERR_SHAPE,
              "mlm_q4k_gemv_tiled: %d rows exceed the %d-row scratch limit", rows,
              ctx->gemv_max_tiles * kTileRows);
  TiledPlan pl;
  MLM_REQUIRE(ctx,
              plan_tiled(rows, nb, std::min(ctx->sm_count, ctx->gemv_max_ctas),
                         (size_t)ctx->max_smem_optin, pl),
              MLM_ERR_UNSUPPORTED,
              "mlm_q4k_gemv_tiled: rows=%d cols=%d does not fit the shared-memory plan", rows,
              cols);
  TiledArgs a;
  a.W = reinterpret_cast<const uint8_t *>(W_tiled);
  a.x = reinterpret_cast<const __half *>(x_f16);
  a.y = y;
  a.residual = residual;
  a.partials = ctx->gemv_partials;
  a.counters = ctx->gemv_counters;
  a.status = ctx->dev_status;
  a.nb_magic = ((1ull << 40) + (unsigned long long)nb - 1) / (unsigned long long)nb;
  a.rows = rows;
  a.nb = nb;
  a.units = pl.units;
  a.ctas = pl.ctas;
  a.ntile = pl.ntile;
  a.nslot = pl.nslot;
  a.ring = pl.ring;
  a.smem_x = pl.smem_x;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.ctas);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, q4k_gemv_tiled_kernel, a);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(ctx, MLM_ERR_CUDA, "mlm_q4k_gemv_tiled: launch failed: %s",
                     cudaGetErrorString(e));
  }
  return MLM_OK;
}
