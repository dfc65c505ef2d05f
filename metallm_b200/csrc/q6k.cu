// q6k.cu -- Q6_K super-blocks: seeded generator, dequantization and the
// decode GEMV.
//
// Block layout (block_q6_K, MetalLM/Backend/Metal/DequantKernels.metal:29-34):
// ql[128] low 4 bits, qh[64] high 2 bits, int8 scales[16], fp16 d = 210
// bytes per 256 elements.  Element order (kernel_dequantize_q6_K_f32,
// DequantKernels.metal:131-172, the GGUF order): element e of a block lies in
// half h = e / 128 at t = e % 128, quarter k = t / 32, l = t % 32; its quant is
// the low (k < 2) or high (k >= 2) nibble of ql[64h + l + 32 (k & 1)] with
// bits 2k, 2k+1 of qh[32h + l] above it, minus 32, and its scale is
// scales[8h + 2k + l / 16]:  out = (d * scale) * q in fp32.
//
// The reference also has a Q6_K -> fp16 kernel (:176-215) that reads the
// block in a different element order than its own fp32 kernel; this library
// follows the fp32 kernel (the GGUF order) for every output type, the fp16
// and bf16 outputs being the rounding of the fp32 value.  The reference uses
// Q6_K only at load time (ModelLoader.swift:282-287, dequantized to fp16 or
// fp32 for MPS); here the GEMV reads the packed blocks directly.
#include <algorithm>

#include "mlm_device.cuh"
#include "mlm_internal.h"

namespace mlm {

constexpr int kQ6Bytes = 210;
constexpr uint64_t kTagQ6K = 0x66ULL;

// ---- generator ---------------------------------------------------------------

// block b of a generated Q6_K tensor: 208 uniform bytes (ql, qh, scales),
// then d = fp16(|N(0,1)| * 0.01) -- the arithmetic of orc_gen_q6k
__global__ void gen_q6k_kernel(uint64_t seed, uint64_t stream, uint64_t first_block,
                               uint64_t nblocks, uint8_t *out) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  const uint64_t b = first_block + i;
  const uint64_t st = stream ^ (kTagQ6K << 56);
  uint16_t *o = reinterpret_cast<uint16_t *>(out + i * kQ6Bytes);  // 2-byte aligned
#pragma unroll 2
  for (int k = 0; k < 26; ++k) {
    const uint64_t r = rng_u64(seed, st, b * 26 + (uint64_t)k);
    o[4 * k + 0] = (uint16_t)r;
    o[4 * k + 1] = (uint16_t)(r >> 16);
    o[4 * k + 2] = (uint16_t)(r >> 32);
    o[4 * k + 3] = (uint16_t)(r >> 48);
  }
  const float d = (float)fabs(rng_normal(seed, st, b));
  o[104] = __half_as_ushort(__float2half_rn(__fmul_rn(d, 0.01f)));
}

// ---- dequantization ------------------------------------------------------------

template <class OutT>
__device__ __forceinline__ OutT q6_out(float v);
template <>
__device__ __forceinline__ float q6_out<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half q6_out<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 q6_out<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// One warp per block: lane l writes elements 128h + 32k + l (k = 0..3) of
// both halves, so every store instruction covers 32 consecutive outputs.
template <class OutT>
__global__ void __launch_bounds__(256) q6k_dequant_kernel(const uint8_t *__restrict__ blocks,
                                                          OutT *__restrict__ out,
                                                          uint64_t nblocks) {
  const int lane = threadIdx.x & 31;
  const uint64_t w0 = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const uint64_t nw = (gridDim.x * (uint64_t)blockDim.x) >> 5;
  for (uint64_t b = w0; b < nblocks; b += nw) {
    const uint8_t *blk = blocks + b * kQ6Bytes;
    const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(blk + 208)));
    OutT *o = out + b * kQK;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t ql0 = blk[64 * h + lane], ql1 = blk[64 * h + 32 + lane];
      const uint32_t qh = blk[128 + 32 * h + lane];
      const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * h) + lane / 16;
      const int q0 = (int)((ql0 & 0xF) | ((qh & 3) << 4)) - 32;
      const int q1 = (int)((ql1 & 0xF) | (((qh >> 2) & 3) << 4)) - 32;
      const int q2 = (int)((ql0 >> 4) | (((qh >> 4) & 3) << 4)) - 32;
      const int q3 = (int)((ql1 >> 4) | (((qh >> 6) & 3) << 4)) - 32;
      o[128 * h + lane] = q6_out<OutT>(__fmul_rn(__fmul_rn(d, (float)sc[0]), (float)q0));
      o[128 * h + 32 + lane] = q6_out<OutT>(__fmul_rn(__fmul_rn(d, (float)sc[2]), (float)q1));
      o[128 * h + 64 + lane] = q6_out<OutT>(__fmul_rn(__fmul_rn(d, (float)sc[4]), (float)q2));
      o[128 * h + 96 + lane] = q6_out<OutT>(__fmul_rn(__fmul_rn(d, (float)sc[6]), (float)q3));
    }
  }
}

// ---- decode GEMV ------------------------------------------------------------------
//
// y[r] = sum_k deq(W[r][k]) x[k] (+ residual[r]), x fp16, fp32 accumulation.
// Each warp owns rows r = gw, gw + nw, ...; its weights stream through a
// per-warp ring of shared-memory stages, one stage per 8-block chunk of a
// row (1,680 bytes = 105 x 16, 16-byte aligned when a row holds a multiple
// of 8 blocks), copied with coalesced 16-byte cp.async and continuing across
// row boundaries.  Lane (k = lane / 8, g = lane % 8) takes the four elements
// 32k + 4g .. 32k + 4g + 3 of each half of every block: one 32-bit word of
// ql and one of qh give the four 6-bit quants, a byte permute puts each under
// the exponent of 2^23, and one subtraction of 2^23 + 32 gives q - 32
// exactly; the four products with x are exact in fp32 and the block's
// d * scale (exact, 19 bits) multiplies their sum.  x is staged once per CTA
// in shared memory as fp32.
constexpr int kQ6Warps = 8;
constexpr int kQ6Threads = kQ6Warps * 32;
constexpr int kQ6ChunkBlocks = 8;
constexpr int kQ6ChunkBytes = kQ6ChunkBlocks * kQ6Bytes;  // 1680
constexpr int kQ6Stages = 4;
constexpr int kQ6StageSmem = kQ6Warps * kQ6Stages * kQ6ChunkBytes;  // 53,760
constexpr int kQ6MaxCols = 32768;

struct Q6GemvArgs {
  const uint8_t *W;
  const __half *x;
  float *y;
  const float *residual;
  int rows, nb, nchunk;
};

__device__ __forceinline__ void q6_cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// a 32-bit word at a 2-byte-aligned shared-memory address
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t *p) {
  const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
  return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
}

__global__ void __launch_bounds__(kQ6Threads, 2) q6k_gemv_kernel(Q6GemvArgs p) {
  extern __shared__ __align__(16) uint8_t smem[];
  float *xs = reinterpret_cast<float *>(smem);  // [nb * 256]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint8_t *my = smem + (size_t)p.nb * kQK * 4 + (size_t)warp * kQ6Stages * kQ6ChunkBytes;
  const uint32_t my_s = (uint32_t)__cvta_generic_to_shared(my);

  const int gw = blockIdx.x * kQ6Warps + warp, nw = gridDim.x * kQ6Warps;
  const int my_rows = gw < p.rows ? (p.rows - 1 - gw) / nw + 1 : 0;
  const int total = my_rows * p.nchunk;  // this warp's chunks, row-major

  // chunk q of the sequence into stage q % kQ6Stages; always one commit group
  auto issue = [&](int q) {
    if (q < total) {
      const int ri = q / p.nchunk, c = q - ri * p.nchunk;
      const size_t r = (size_t)gw + (size_t)ri * nw;
      const uint8_t *src = p.W + (r * p.nb + (size_t)c * kQ6ChunkBlocks) * kQ6Bytes;
      const uint32_t dst = my_s + (uint32_t)(q % kQ6Stages) * kQ6ChunkBytes;
      for (int k = lane; k < kQ6ChunkBytes / 16; k += 32) q6_cp_async16(dst + 16 * k, src + 16 * k);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // the weights do not depend on the kernel before this one
#pragma unroll
  for (int q = 0; q < kQ6Stages - 1; ++q) issue(q);
  pdl_wait_then_release();

  {
    const uint4 *xg = reinterpret_cast<const uint4 *>(p.x);
    float4 *xo = reinterpret_cast<float4 *>(xs);
    for (int i = threadIdx.x; i < p.nb * 32; i += kQ6Threads) {
      const uint4 v = __ldg(xg + i);
      const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
      const float2 c = __half22float2(*reinterpret_cast<const __half2 *>(&v.z));
      const float2 e = __half22float2(*reinterpret_cast<const __half2 *>(&v.w));
      xo[2 * i] = make_float4(a.x, a.y, b.x, b.y);
      xo[2 * i + 1] = make_float4(c.x, c.y, e.x, e.y);
    }
  }
  __syncthreads();

  const int k = lane >> 3, g = lane & 7;
  const int ql_off = 32 * (k & 1) + 4 * g;  // + 64 h
  const int qh_off = 128 + 4 * g;           // + 32 h
  const int sc_off = 192 + 2 * k + (g >> 2);  // + 8 h
  const int sh_lo = (k >= 2) ? 4 : 0;
  const int x_off = 32 * k + 4 * g;  // + 128 h
  const float kMagic = 8388640.0f;   // 2^23 + 32
  float acc = 0.f;
  for (int q = 0; q < total; ++q) {
    issue(q + kQ6Stages - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(kQ6Stages - 1) : "memory");
    __syncwarp();
    const uint8_t *st = my + (q % kQ6Stages) * kQ6ChunkBytes;
    const int ri = q / p.nchunk, c = q - ri * p.nchunk;
    const float *xc = xs + (size_t)c * kQ6ChunkBlocks * kQK;
#pragma unroll 2
    for (int bi = 0; bi < kQ6ChunkBlocks; ++bi) {
      const uint8_t *blk = st + bi * kQ6Bytes;
      const float d =
          __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t *>(blk + 208)));
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t qlw = ld_u32_a2(blk + 64 * h + ql_off);
        const uint32_t qhw = ld_u32_a2(blk + qh_off + 32 * h);
        // bits 2k, 2k+1 of each qh byte to bits 4, 5; the nibble below
        const uint32_t q4 = ((qlw >> sh_lo) & 0x0F0F0F0Fu) | (((qhw >> (2 * k)) << 4) & 0x30303030u);
        const float4 xv = *reinterpret_cast<const float4 *>(xc + bi * kQK + 128 * h + x_off);
        const float f0 = __int_as_float(__byte_perm(q4, 0x4B000000u, 0x7440)) - kMagic;
        const float f1 = __int_as_float(__byte_perm(q4, 0x4B000000u, 0x7441)) - kMagic;
        const float f2 = __int_as_float(__byte_perm(q4, 0x4B000000u, 0x7442)) - kMagic;
        const float f3 = __int_as_float(__byte_perm(q4, 0x4B000000u, 0x7443)) - kMagic;
        float s = f0 * xv.x;
        s = fmaf(f1, xv.y, s);
        s = fmaf(f2, xv.z, s);
        s = fmaf(f3, xv.w, s);
        const float ds = d * (float)(int8_t)blk[sc_off + 8 * h];
        acc = fmaf(ds, s, acc);
      }
    }
    __syncwarp();  // the stage is read before the next issue overwrites it
    if (c == p.nchunk - 1) {
      acc = warp_sum(acc);
      if (lane == 0) {
        const size_t r = (size_t)gw + (size_t)ri * nw;
        p.y[r] = acc + (p.residual ? p.residual[r] : 0.f);
      }
      acc = 0.f;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

size_t q6k_gemv_smem(int cols) { return (size_t)cols * 4 + kQ6StageSmem; }

int q6k_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q6k_gemv_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)q6k_gemv_smem(kQ6MaxCols)));
  return MLM_OK;
}

template <class OutT>
static int q6k_dequant_entry(mlm_ctx *ctx, const void *blocks, OutT *out, uint64_t n,
                             const char *name) {
  MLM_CHECK_CTX(ctx);
  if (n == 0) return MLM_OK;
  MLM_REQUIRE(ctx, blocks && out, MLM_ERR_ARG, "%s: null buffer", name);
  MLM_REQUIRE(ctx, n % kQK == 0, MLM_ERR_SHAPE,
              "%s: n=%llu is not a multiple of the 256-element super-block", name,
              (unsigned long long)n);
  MLM_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(blocks) & 1) == 0 &&
                       (reinterpret_cast<uintptr_t>(out) & (sizeof(OutT) - 1)) == 0,
              MLM_ERR_ALIGN, "%s: blocks must be 2-byte and out element aligned", name);
  const uint64_t nblocks = n / kQK;
  const uint64_t warps = std::min<uint64_t>(nblocks, (uint64_t)ctx->sm_count * 64);
  const unsigned grid = (unsigned)((warps * 32 + 255) / 256);
  q6k_dequant_kernel<OutT><<<grid, 256, 0, ctx->stream>>>(
      reinterpret_cast<const uint8_t *>(blocks), out, nblocks);
  return check_launch(ctx, name);
}

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_gen_q6k(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t first_block,
                           uint64_t nblocks, void *out) {
  MLM_CHECK_CTX(ctx);
  if (nblocks == 0) return MLM_OK;
  MLM_REQUIRE(ctx, out, MLM_ERR_ARG, "mlm_gen_q6k: null output");
  MLM_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(out) & 1) == 0, MLM_ERR_ALIGN,
              "mlm_gen_q6k: output must be 2-byte aligned");
  const unsigned grid = (unsigned)((nblocks + 127) / 128);
  gen_q6k_kernel<<<grid, 128, 0, ctx->stream>>>(seed, stream, first_block, nblocks,
                                                reinterpret_cast<uint8_t *>(out));
  return check_launch(ctx, "mlm_gen_q6k");
}

extern "C" int mlm_q6k_dequant_f32(mlm_ctx *ctx, const void *blocks, float *out, uint64_t n) {
  return q6k_dequant_entry(ctx, blocks, out, n, "mlm_q6k_dequant_f32");
}

extern "C" int mlm_q6k_dequant_f16(mlm_ctx *ctx, const void *blocks, void *out, uint64_t n) {
  return q6k_dequant_entry(ctx, blocks, reinterpret_cast<__half *>(out), n,
                           "mlm_q6k_dequant_f16");
}

extern "C" int mlm_q6k_dequant_bf16(mlm_ctx *ctx, const void *blocks, void *out, uint64_t n) {
  return q6k_dequant_entry(ctx, blocks, reinterpret_cast<__nv_bfloat16 *>(out), n,
                           "mlm_q6k_dequant_bf16");
}

extern "C" int mlm_q6k_gemv(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                            float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, W && x_f16 && y, MLM_ERR_ARG, "mlm_q6k_gemv: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && cols > 0 && cols % (kQK * kQ6ChunkBlocks) == 0 && cols <= kQ6MaxCols,
              MLM_ERR_SHAPE,
              "mlm_q6k_gemv: rows=%d cols=%d (cols a multiple of 2048, at most %d)", rows, cols,
              kQ6MaxCols);
  MLM_REQUIRE(ctx, aligned16(W) && aligned16(x_f16) && (!residual || aligned4(residual)),
              MLM_ERR_ALIGN, "mlm_q6k_gemv: W and x must be 16-byte aligned");
  Q6GemvArgs a;
  a.W = reinterpret_cast<const uint8_t *>(W);
  a.x = reinterpret_cast<const __half *>(x_f16);
  a.y = y;
  a.residual = residual;
  a.rows = rows;
  a.nb = cols / kQK;
  a.nchunk = a.nb / kQ6ChunkBlocks;
  const int ctas = std::max(1, std::min((rows + kQ6Warps - 1) / kQ6Warps, 2 * ctx->sm_count));
  return check_launch_pdl(ctx,
                          launch_pdl(q6k_gemv_kernel, dim3(ctas), dim3(kQ6Threads),
                                     q6k_gemv_smem(cols), ctx->stream, a),
                          "mlm_q6k_gemv");
}
