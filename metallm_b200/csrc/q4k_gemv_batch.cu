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
// memory (fp16 with a power-of-two scale per token and sub-block, which
// keeps large activations in range; the scale is undone in fp32) and its
// warps take the chunk's tiles.  Each (tile, chunk) adds its partial into Y
// with fp32 atomics; Y starts from the residual (or zero).
#include <algorithm>

#include "mlm_device.cuh"
#include "mlm_internal.h"

namespace mlm {
namespace {

constexpr int kBgRows = 16;      // rows per tile (the MMA's M)
constexpr int kBgChunk = 8;      // Q4_K block columns per chunk
constexpr int kBgSub = kBgChunk * 8;  // sub-blocks per chunk
constexpr int kBgWarps = 16;
constexpr int kBgThreads = kBgWarps * 32;
constexpr int kBgMaxT = 8;

struct BgArgs {
  const uint8_t *W;
  const __nv_bfloat16 *x;  // [T][cols]
  float *y;                // [T][rows]
  int rows, cols, T, nb, tiles, ctas_per_chunk;
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

__global__ void __launch_bounds__(kBgThreads) q4k_gemv_batch_kernel(BgArgs p) {
  // x of the chunk: [token][sub-block][lane t] -> 8 fp16 in mask order
  __shared__ uint4 xperm[kBgMaxT * kBgSub * 4];
  __shared__ float xscale[kBgSub][kBgMaxT];  // power of two per (sub-block, token)
  __shared__ float xsum[kBgSub][kBgMaxT];    // sum of the unscaled x

  const int chunk = blockIdx.x / p.ctas_per_chunk, cj = blockIdx.x % p.ctas_per_chunk;
  const int kb0 = chunk * kBgChunk, nkb = min(kBgChunk, p.nb - kb0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  // ---- stage x: one thread per (token, sub-block, t): elements 8t .. 8t+7 --
  for (int i = threadIdx.x; i < kBgMaxT * kBgSub * 4; i += kBgThreads) {
    const int tq = i & 3, s = (i >> 2) % kBgSub, n = i / (kBgSub * 4);
    float v[8];
    const bool live = n < p.T && s < nkb * 8;
    if (live) {
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
    // scale 2^-ex keeps the sub-block's largest magnitude below 2^15
    const int ex = max(0, (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127 - 14);
    const float inv = __uint_as_float((uint32_t)(127 - ex) << 23);
    xperm[i] = make_uint4(h2(v[0] * inv, v[4] * inv), h2(v[2] * inv, v[6] * inv),
                          h2(v[1] * inv, v[5] * inv), h2(v[3] * inv, v[7] * inv));
    if (tq == 0) {
      xscale[s][n] = __uint_as_float((uint32_t)(127 + ex) << 23);
      xsum[s][n] = sm;
    }
  }
  __syncthreads();

  // ---- tiles of this chunk, round-robin over the CTA's warps ---------------
  const uint32_t M = 0x000F000Fu, MH = 0x00F000F0u;
  for (int tile = cj + p.ctas_per_chunk * warp; tile < p.tiles;
       tile += p.ctas_per_chunk * kBgWarps) {
    const int r0 = tile * kBgRows + g, r1 = r0 + 8;
    const bool ok0 = r0 < p.rows, ok1 = r1 < p.rows;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // (r0, 2t) (r0, 2t+1) (r1, 2t) (r1, 2t+1)
    for (int kb = 0; kb < nkb; ++kb) {
      const uint8_t *b0 = p.W + ((size_t)(ok0 ? r0 : 0) * p.nb + kb0 + kb) * kBlockBytes;
      const uint8_t *b1 = p.W + ((size_t)(ok1 ? r1 : 0) * p.nb + kb0 + kb) * kBlockBytes;
      uint4 h0 = make_uint4(0, 0, 0, 0), h1 = make_uint4(0, 0, 0, 0);
      uint32_t q0[8], q1[8];
      if (ok0) h0 = __ldg(reinterpret_cast<const uint4 *>(b0));
      if (ok1) h1 = __ldg(reinterpret_cast<const uint4 *>(b1));
#pragma unroll
      for (int sb = 0; sb < 8; ++sb) {
        q0[sb] = ok0 ? __ldg(reinterpret_cast<const uint32_t *>(b0 + 16 + 16 * sb + 4 * t)) : 0u;
        q1[sb] = ok1 ? __ldg(reinterpret_cast<const uint32_t *>(b1 + 16 + 16 * sb + 4 * t)) : 0u;
      }
      const float D0 = half_bits_to_float(h0.x) * 16777216.0f, Dm0 = half_bits_to_float(h0.x >> 16);
      const float D1 = half_bits_to_float(h1.x) * 16777216.0f, Dm1 = half_bits_to_float(h1.x >> 16);
#pragma unroll
      for (int sb = 0; sb < 8; ++sb) {
        const int s = kb * 8 + sb;
        const uint4 xv = xperm[(g * kBgSub + s) * 4 + t];
        const uint32_t w0 = q0[sb], w1 = q1[sb], u0 = w0 >> 8, u1 = w1 >> 8;
        float clo[4] = {0.f, 0.f, 0.f, 0.f}, chi[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(clo, w0 & M, w1 & M, u0 & M, u1 & M, xv.x, xv.y);
        mma16816(chi, w0 & MH, w1 & MH, u0 & MH, u1 & MH, xv.z, xv.w);
        int sc0, m0, sc1, m1;
        q4k_scale_min_regs(sb, h0.y, h0.z, h0.w, sc0, m0);
        q4k_scale_min_regs(sb, h1.y, h1.z, h1.w, sc1, m1);
        const float ds0 = D0 * (float)sc0, dm0 = Dm0 * (float)m0;
        const float ds1 = D1 * (float)sc1, dm1 = Dm1 * (float)m1;
        const float2 xs = *reinterpret_cast<const float2 *>(&xscale[s][2 * t]);
        const float2 xm = *reinterpret_cast<const float2 *>(&xsum[s][2 * t]);
        acc[0] += ds0 * (fmaf(0.0625f, chi[0], clo[0]) * xs.x) - dm0 * xm.x;
        acc[1] += ds0 * (fmaf(0.0625f, chi[1], clo[1]) * xs.y) - dm0 * xm.y;
        acc[2] += ds1 * (fmaf(0.0625f, chi[2], clo[2]) * xs.x) - dm1 * xm.x;
        acc[3] += ds1 * (fmaf(0.0625f, chi[3], clo[3]) * xs.y) - dm1 * xm.y;
      }
    }
    const int n0 = 2 * t, n1 = 2 * t + 1;
    if (ok0 && n0 < p.T) atomicAdd(p.y + (size_t)n0 * p.rows + r0, acc[0]);
    if (ok0 && n1 < p.T) atomicAdd(p.y + (size_t)n1 * p.rows + r0, acc[1]);
    if (ok1 && n0 < p.T) atomicAdd(p.y + (size_t)n0 * p.rows + r1, acc[2]);
    if (ok1 && n1 < p.T) atomicAdd(p.y + (size_t)n1 * p.rows + r1, acc[3]);
  }
}

}  // namespace

int gemv_batch_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                      int tokens, float *y, const float *residual, cudaStream_t stream) {
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
  if (!residual)
    MLM_CUDA_TRY(ctx, cudaMemsetAsync(y, 0, ybytes, stream));
  else if (residual != y)
    MLM_CUDA_TRY(ctx, cudaMemcpyAsync(y, residual, ybytes, cudaMemcpyDeviceToDevice, stream));
  BgArgs a;
  a.W = reinterpret_cast<const uint8_t *>(W);
  a.x = reinterpret_cast<const __nv_bfloat16 *>(x_bf16);
  a.y = y;
  a.rows = rows;
  a.cols = cols;
  a.T = tokens;
  a.nb = cols / kQK;
  a.tiles = (rows + kBgRows - 1) / kBgRows;
  const int nchunks = (a.nb + kBgChunk - 1) / kBgChunk;
  // about two CTAs per SM over all chunks; never more CTAs than tiles
  a.ctas_per_chunk =
      std::max(1, std::min(a.tiles / kBgWarps + 1, (2 * ctx->sm_count + nchunks - 1) / nchunks));
  q4k_gemv_batch_kernel<<<nchunks * a.ctas_per_chunk, kBgThreads, 0, stream>>>(a);
  return check_launch(ctx, "mlm_q4k_gemv_batch");
}

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_q4k_gemv_batch(mlm_ctx *ctx, const void *W, int rows, int cols,
                                  const void *x_bf16, int tokens, float *y,
                                  const float *residual) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, !residual || aligned4(residual), MLM_ERR_ALIGN,
              "mlm_q4k_gemv_batch: residual");
  return gemv_batch_launch(ctx, W, rows, cols, x_bf16, tokens, y, residual, ctx->stream);
}
