// q4k_gemv_batch.cu -- the decode linears for a batch of up to 8 tokens:
// Y[t][n] = sum_k X[t][k] * W[n][k] (+ R[t][n]), W packed Q4_K, X bf16.
//
// The reference runs one token at a time through encodeMPSMatrixMultiply on
// fp16 weights (MetalService.swift:797-925); a batch of independent
// sequences streams every weight once for all of them here.  The weights go
// to the tensor cores as in the single-token GEMV: a nibble masked into the
// low mantissa bits of a binary16 is the exact subnormal q 2^-24 (16 q 2^-24
// for the high nibble), two nibbles per 32-bit word; mma.sync m16n8k16 with
// the batch's tokens as the 8 columns forms the sub-block sums sum q x, the
// low and the high nibbles in two accumulators; per sub-block the row's
// (d sc) 2^24 and the min term (dmin m) sum x are applied in fp32.  Element i
// of a block is nibble i%2 of qs byte i/2, so the 8 elements of a qs word are
// the low/high nibbles of 4 bytes: the masks take elements {0,4}, {2,6}
// (low) and {1,5}, {3,7} (high), and x is staged in that order.
//
// Work: 16-row tiles x chunks of 8 block columns (2048 elements).  A CTA
// owns one chunk: it stages the chunk's x of every token once in shared
// memory (fp16 with a power-of-two scale per token, which keeps large
// activations in range and is undone in fp32 after the chunk; the x of the
// high-nibble positions is also divided by 16, an exact exponent shift, so
// both nibble MMAs of a sub-block add into one accumulator) and its warps
// take the chunk's tiles.  A warp walks its (tile, block column) items
// through a ring of kBgStages shared-memory stages, one TMA box per item (16
// rows x 144 bytes, an mbarrier per stage, bounded waits), the next items'
// copies overlapping the current one's MMAs across tile boundaries; with the
// 144-byte row stride every fragment load is conflict-free.  One CTA of 16
// warps per SM with a 3-deep ring measured faster than two CTAs with 2-deep
// rings (more bytes in flight per SM).  Each
// (tile, chunk) adds its partial into Y with fp32 atomics; Y starts from the
// residual (or zero).
#include <algorithm>

#include "mlm_device.cuh"
#include "mlm_internal.h"
#include "q4k_gemv_common.cuh"

namespace mlm {
namespace {

constexpr int kBgRows = 16;      // rows per tile (the MMA's M)
constexpr int kBgChunk = 8;      // Q4_K block columns per chunk, at most
constexpr int kBgSub = kBgChunk * 8;  // sub-blocks per chunk, at most
constexpr int kBgWarps = 16;
constexpr int kBgThreads = kBgWarps * 32;
constexpr int kBgMaxT = 8;
// uint4 per token: a quarter warp reads tokens g, g + 1 at lanes t = 0..3, so
// the token pitch is 64 bytes past a multiple of 128 (no bank conflicts)
constexpr int kBgXStride = kBgSub * 4 + 4;
constexpr int kBgStage = kBgRows * kBlockBytes;  // one block column of a tile: 2304 bytes
#ifndef MLM_BG_STAGES
#define MLM_BG_STAGES 3
#endif
#ifndef MLM_BG_MIN_BLOCKS
#define MLM_BG_MIN_BLOCKS 1
#endif
constexpr int kBgStages = MLM_BG_STAGES;         // ring depth per warp
constexpr int kBgBlocks = MLM_BG_MIN_BLOCKS;     // resident CTAs per SM
constexpr int kBgSmem = kBgWarps * kBgStages * kBgStage;  // dynamic: the warps' weight stages

struct BgArgs {
  const __nv_bfloat16 *x;  // [T][cols]
  float *y;                // [T][rows]
  int *status;             // device-visible error word (0 = ok)
  int rows, cols, T, nb, tiles, ctas_per_chunk;
  int chunk;  // block columns per chunk (1..kBgChunk)
};

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// The 8 (scale, min) pairs of a block (get_scale_min_k4, DequantKernels.metal:
// 43-56) as bytes of four words: scales of sub-blocks 0-3 / 4-7, mins 0-3 / 4-7
__device__ __forceinline__ void q4k_scales_packed(const uint4 &h, uint32_t &sc_lo, uint32_t &sc_hi,
                                                  uint32_t &m_lo, uint32_t &m_hi) {
  sc_lo = h.y & 0x3F3F3F3Fu;
  m_lo = h.z & 0x3F3F3F3Fu;
  sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
}

// byte b of w as the fp32 value 2^23 + byte (a byte permute)
__device__ __forceinline__ float byte_plus_2p23(uint32_t w, int b) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + b));
}

__global__ void __launch_bounds__(kBgThreads, kBgBlocks)
    q4k_gemv_batch_kernel(const __grid_constant__ CUtensorMap tmap, BgArgs p) {
  // x of the chunk: [token][sub-block][lane t] -> 8 fp16 in mask order
  __shared__ uint4 xperm[kBgMaxT * kBgXStride];
  extern __shared__ __align__(128) uint8_t wstage[];  // TMA destinations: 128-byte aligned
  __shared__ float xsum[kBgSub][kBgMaxT];    // per (sub-block, token): sum of the x
  __shared__ uint32_t tokmax[kBgMaxT];       // per token: bits of the chunk's max |x|
  __shared__ float tokscale[kBgMaxT];        // per token: the power of two x was divided by

  const int chunk = blockIdx.x / p.ctas_per_chunk, cj = blockIdx.x % p.ctas_per_chunk;
  const int kb0 = chunk * p.chunk, nkb = min(p.chunk, p.nb - kb0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  uint8_t *mystage = wstage + warp * kBgStages * kBgStage;
  const uint32_t stage_addr = (uint32_t)__cvta_generic_to_shared(mystage);
  __shared__ __align__(8) uint64_t bars[kBgWarps * kBgStages];  // one per stage of each warp
  const uint32_t my_bar = (uint32_t)__cvta_generic_to_shared(&bars[warp * kBgStages]);
  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < kBgStages; ++b) mbar_init(my_bar + 8 * b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  const uint64_t pol = evict_first_policy();
  uint32_t phases = 0, pending = 0;  // bit b: parity of stage b's next completion / a copy in flight
  // The warp's work items: block column kb of tiles first_tile + j stride,
  // item i = (j, kb) with j = i / nkb, in a ring of kBgStages stages.
  const int stride = p.ctas_per_chunk * kBgWarps;
  const int first_tile = cj + p.ctas_per_chunk * warp;
  const int nitems = first_tile < p.tiles ? ((p.tiles - 1 - first_tile) / stride + 1) * nkb : 0;
  int in_j = 0, in_kb = 0, in_buf = 0;  // the next item to put in flight
  // the next item's 16 rows of one block column -> its stage, one TMA box
  // (rows past the end read as zeros)
  auto issue_next = [&]() {
    if (lane == 0) {
      mbar_expect_tx(my_bar + 8 * in_buf, kBgStage);
      tma_unit(stage_addr + in_buf * kBgStage, &tmap, (kb0 + in_kb) * kBlockBytes,
               (first_tile + in_j * stride) * kBgRows, my_bar + 8 * in_buf, pol);
    }
    pending |= 1u << in_buf;
    if (++in_kb == nkb) {
      in_kb = 0;
      ++in_j;
    }
    in_buf = in_buf + 1 == kBgStages ? 0 : in_buf + 1;
  };
  // bounded wait for stage buf; false (and the error word set) on timeout
  auto wait_stage = [&](int buf) {
    if (!mbar_wait_bounded(my_bar + 8 * buf, (phases >> buf) & 1, p.status)) return false;
    phases ^= 1u << buf;
    pending &= ~(1u << buf);
    return true;
  };
  // the weights do not depend on the kernel before this one: the warp's
  // first items are in flight before waiting for it (x, y)
#pragma unroll
  for (int i = 0; i < kBgStages - 1; ++i)
    if (i < nitems) issue_next();
  pdl_wait_then_release();

  // ---- stage x: one thread per (token, sub-block, t): elements 8t .. 8t+7 --
  if (threadIdx.x < kBgMaxT) tokmax[threadIdx.x] = 0;
  __syncthreads();
  auto load8 = [&](int n, int s, int tq, float (&v)[8]) {
    if (n < p.T && s < nkb * 8) {
      const __nv_bfloat16 *src = p.x + (size_t)n * p.cols + (size_t)kb0 * 256 + 32 * s + 8 * tq;
      const uint4 raw = *reinterpret_cast<const uint4 *>(src);
      const __nv_bfloat162 *b2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(b2[e]);
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
  };
  // pass 1: the sub-blocks' sums and each token's largest magnitude
  for (int i = threadIdx.x; i < kBgMaxT * kBgSub * 4; i += kBgThreads) {
    const int tq = i & 3, s = (i >> 2) % kBgSub, n = i / (kBgSub * 4);
    float v[8];
    load8(n, s, tq, v);
    float mx = 0.f, sm = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      mx = fmaxf(mx, fabsf(v[e]));
      sm += v[e];
    }
    // the 4 threads of a sub-block are consecutive lanes
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    sm += __shfl_xor_sync(0xffffffffu, sm, 1);
    sm += __shfl_xor_sync(0xffffffffu, sm, 2);
    if (tq == 0) {
      xsum[s][n] = sm;
      atomicMax(tokmax + n, __float_as_uint(mx));  // non-negative: bit order = value order
    }
  }
  __syncthreads();
  if (threadIdx.x < kBgMaxT) {
    // 2^-ex keeps the token's largest magnitude below 2^15
    const int ex = max(0, (int)((tokmax[threadIdx.x] >> 23) & 0xFF) - 127 - 14);
    tokscale[threadIdx.x] = __uint_as_float((uint32_t)(127 + ex) << 23);
  }
  __syncthreads();
  // pass 2: scaled fp16 in the order of the nibble masks
  for (int i = threadIdx.x; i < kBgMaxT * kBgSub * 4; i += kBgThreads) {
    const int tq = i & 3, s = (i >> 2) % kBgSub, n = i / (kBgSub * 4);
    float v[8];
    load8(n, s, tq, v);
    const float inv = 1.0f / tokscale[n], inv16 = inv * 0.0625f;  // powers of two: exact
    xperm[n * kBgXStride + s * 4 + tq] =
        make_uint4(h2(v[0] * inv, v[4] * inv), h2(v[2] * inv, v[6] * inv),
                   h2(v[1] * inv16, v[5] * inv16), h2(v[3] * inv16, v[7] * inv16));
  }
  __syncthreads();

  // ---- tiles of this chunk, round-robin over the CTA's warps ---------------
  const uint32_t M = 0x000F000Fu, MH = 0x00F000F0u;
  bool ok = true;
  // (r0, 2t) (r0, 2t+1) (r1, 2t) (r1, 2t+1): the scaled-x products and the
  // min terms of the current tile
  float aq[4] = {0.f, 0.f, 0.f, 0.f}, am[4] = {0.f, 0.f, 0.f, 0.f};
  int buf = 0, kb = 0, tile = first_tile;
  for (int i = 0; i < nitems; ++i) {
    if (i + kBgStages - 1 < nitems) issue_next();
    if (!wait_stage(buf)) {
      ok = false;
      break;
    }
    const uint8_t *s0 = mystage + buf * kBgStage + g * kBlockBytes;
    const uint8_t *s1 = s0 + 8 * kBlockBytes;
    const uint4 h0 = *reinterpret_cast<const uint4 *>(s0);
    const uint4 h1 = *reinterpret_cast<const uint4 *>(s1);
    // d 2^24 (undoes the subnormal scale of the nibbles) and dmin; with
    // f = 2^23 + sc, fma(D, f, -D 2^23) is D sc exactly (at most 17
    // significant bits), so the 6-bit values need no conversion
    const float D0 = half_bits_to_float(h0.x) * 16777216.0f, Dm0 = half_bits_to_float(h0.x >> 16);
    const float D1 = half_bits_to_float(h1.x) * 16777216.0f, Dm1 = half_bits_to_float(h1.x >> 16);
    const float nD0 = -D0 * 8388608.0f, nDm0 = -Dm0 * 8388608.0f;
    const float nD1 = -D1 * 8388608.0f, nDm1 = -Dm1 * 8388608.0f;
    uint32_t scl0, sch0, ml0, mh0, scl1, sch1, ml1, mh1;
    q4k_scales_packed(h0, scl0, sch0, ml0, mh0);
    q4k_scales_packed(h1, scl1, sch1, ml1, mh1);
#pragma unroll
    for (int sb = 0; sb < 8; ++sb) {
      const int s = kb * 8 + sb;
      const uint4 xv = xperm[g * kBgXStride + s * 4 + t];
      const uint32_t w0 = *reinterpret_cast<const uint32_t *>(s0 + 16 + 16 * sb + 4 * t);
      const uint32_t w1 = *reinterpret_cast<const uint32_t *>(s1 + 16 + 16 * sb + 4 * t);
      const uint32_t u0 = w0 >> 8, u1 = w1 >> 8;
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816(c, w0 & M, w1 & M, u0 & M, u1 & M, xv.x, xv.y);
      mma16816(c, w0 & MH, w1 & MH, u0 & MH, u1 & MH, xv.z, xv.w);
      const int bsel = sb & 3;
      const float ds0 = fmaf(D0, byte_plus_2p23(sb < 4 ? scl0 : sch0, bsel), nD0);
      const float dm0 = fmaf(Dm0, byte_plus_2p23(sb < 4 ? ml0 : mh0, bsel), nDm0);
      const float ds1 = fmaf(D1, byte_plus_2p23(sb < 4 ? scl1 : sch1, bsel), nD1);
      const float dm1 = fmaf(Dm1, byte_plus_2p23(sb < 4 ? ml1 : mh1, bsel), nDm1);
      const float2 xm = *reinterpret_cast<const float2 *>(&xsum[s][2 * t]);
      aq[0] = fmaf(ds0, c[0], aq[0]);
      aq[1] = fmaf(ds0, c[1], aq[1]);
      aq[2] = fmaf(ds1, c[2], aq[2]);
      aq[3] = fmaf(ds1, c[3], aq[3]);
      am[0] = fmaf(dm0, xm.x, am[0]);
      am[1] = fmaf(dm0, xm.y, am[1]);
      am[2] = fmaf(dm1, xm.x, am[2]);
      am[3] = fmaf(dm1, xm.y, am[3]);
    }
    __syncwarp();  // the stage is read before the next copy overwrites it
    buf = buf + 1 == kBgStages ? 0 : buf + 1;
    if (++kb < nkb) continue;
    // the tile's last block column: add its partial into Y
    const int r0 = tile * kBgRows + g, r1 = r0 + 8;
    const bool ok0 = r0 < p.rows, ok1 = r1 < p.rows;
    const int n0 = 2 * t, n1 = 2 * t + 1;
    const float xs0 = tokscale[n0], xs1 = tokscale[n1];
    const float acc[4] = {aq[0] * xs0 - am[0], aq[1] * xs1 - am[1], aq[2] * xs0 - am[2],
                          aq[3] * xs1 - am[3]};
    if (ok0 && n0 < p.T) atomicAdd(p.y + (size_t)n0 * p.rows + r0, acc[0]);
    if (ok0 && n1 < p.T) atomicAdd(p.y + (size_t)n1 * p.rows + r0, acc[1]);
    if (ok1 && n0 < p.T) atomicAdd(p.y + (size_t)n0 * p.rows + r1, acc[2]);
    if (ok1 && n1 < p.T) atomicAdd(p.y + (size_t)n1 * p.rows + r1, acc[3]);
#pragma unroll
    for (int e = 0; e < 4; ++e) aq[e] = am[e] = 0.f;
    kb = 0;
    tile += stride;
  }
  if (!ok) {
    // a stage wait ran out of budget: let the copies still in flight land
    // (bounded again) before this warp's shared memory is released
    for (int b = 0; b < kBgStages; ++b)
      if ((pending >> b) & 1) wait_stage(b);
  }
}

}  // namespace

// Chunk width: the widest (fewest partial sums per output) whose grid fills
// the SMs -- narrow weights (a rank's share of a row-parallel projection)
// otherwise leave most SMs idle, since a warp takes whole 16-row tiles of a
// chunk; then at most kBgBlocks CTAs per SM over all chunks (one wave: a CTA
// past it would run alone after the others), never more CTAs than tiles.
static void batch_plan(int tiles, int nb, int sm_count, int &chunk, int &nchunks,
                       int &ctas_per_chunk) {
  auto per_chunk = [&](int nch) {
    return std::max(1, std::min(tiles / kBgWarps + 1, kBgBlocks * sm_count / nch));
  };
  for (int c = kBgChunk; c >= 1; c /= 2) {
    chunk = c;
    nchunks = (nb + c - 1) / c;
    if (nchunks * per_chunk(nchunks) >= kBgBlocks * sm_count * 3 / 4) break;
  }
  ctas_per_chunk = per_chunk(nchunks);
}

int gemv_batch_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q4k_gemv_batch_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kBgSmem));
  return MLM_OK;
}

int gemv_batch_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                      int tokens, float *y, const float *residual, cudaStream_t stream,
                      bool y_zeroed) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, W && x_bf16 && y, MLM_ERR_ARG, "mlm_q4k_gemv_batch: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && cols > 0 && cols % kQK == 0 && tokens >= 1 && tokens <= kBgMaxT,
              MLM_ERR_SHAPE,
              "mlm_q4k_gemv_batch: rows=%d cols=%d tokens=%d (cols a multiple of 256, 1..8 "
              "tokens)",
              rows, cols, tokens);
  MLM_REQUIRE(ctx, aligned16(W) && aligned16(x_bf16), MLM_ERR_ALIGN,
              "mlm_q4k_gemv_batch: W and X must be 16-byte aligned");
  const size_t ybytes = sizeof(float) * (size_t)rows * tokens;
  if (!residual) {
    if (!y_zeroed) MLM_CUDA_TRY(ctx, cudaMemsetAsync(y, 0, ybytes, stream));
  } else if (residual != y)
    MLM_CUDA_TRY(ctx, cudaMemcpyAsync(y, residual, ybytes, cudaMemcpyDeviceToDevice, stream));
  BgArgs a;
  a.x = reinterpret_cast<const __nv_bfloat16 *>(x_bf16);
  a.y = y;
  a.status = ctx->dev_status;
  a.rows = rows;
  a.cols = cols;
  a.T = tokens;
  a.nb = cols / kQK;
  a.tiles = (rows + kBgRows - 1) / kBgRows;
  int nchunks = 0;
  batch_plan(a.tiles, a.nb, ctx->sm_count, a.chunk, nchunks, a.ctas_per_chunk);
  CUtensorMap tmap;
  const int st = encode_q4k_rows_map(ctx, W, rows, a.nb, kBgRows, &tmap);
  if (st != MLM_OK) return st;
  return check_launch_pdl(ctx,
                          launch_pdl(q4k_gemv_batch_kernel, dim3(nchunks * a.ctas_per_chunk),
                                     dim3(kBgThreads), kBgSmem, stream, tmap, a),
                          "mlm_q4k_gemv_batch");
}

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_q4k_gemv_batch_plan(int rows, int cols, int sm_count, int *chunk,
                                       int *ctas) {
  if (rows <= 0 || cols <= 0 || cols % kQK != 0 || sm_count <= 0 || !chunk || !ctas)
    return MLM_ERR_ARG;
  int nchunks = 0, per = 0;
  batch_plan((rows + kBgRows - 1) / kBgRows, cols / kQK, sm_count, *chunk, nchunks, per);
  *ctas = nchunks * per;
  return MLM_OK;
}

extern "C" int mlm_q4k_gemv_batch(mlm_ctx *ctx, const void *W, int rows, int cols,
                                  const void *x_bf16, int tokens, float *y,
                                  const float *residual) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, !residual || aligned4(residual), MLM_ERR_ALIGN,
              "mlm_q4k_gemv_batch: residual");
  return gemv_batch_launch(ctx, W, rows, cols, x_bf16, tokens, y, residual, ctx->stream);
}
