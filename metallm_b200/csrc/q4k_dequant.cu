// q4k_dequant.cu -- Q4_K super-block dequantization (fp32 / fp16 / bf16)
// and the seeded synthetic-data generators.
//
// The arithmetic is that of kernel_dequantize_q4_K_f32 / _f16
// (MetalLM/Backend/Metal/DequantKernels.metal:63-125): element i of a block
// is (d*sc_j)*q_i - dmin*m_j with j = i/32 and q_i the low nibble of
// qs[i/2] for even i, the high nibble for odd i.  d*sc and dmin*m are exact
// in fp32 (11-bit * 6-bit), so is (d*sc)*q (<= 21 bits): the fp32 result has
// a single rounding and matches the reference bit for bit.
//
// Mapping: one warp per super-block per iteration; lane l owns qs word l,
// i.e. elements 8l..8l+7 of sub-block l/4, and writes them as 32 contiguous
// bytes (fp32) or 16 bytes (fp16/bf16), so a warp stores 1 KiB / 512 B
// contiguously.  The kernel is HBM-bound (read 144 B, write 1024 B / 512 B
// per block); a grid-stride loop with four blocks in flight per warp keeps
// enough loads outstanding.
#include <algorithm>

#include "mlm_device.cuh"
#include "mlm_internal.h"

namespace mlm {

enum DeqOut { kOutF32 = 0, kOutF16 = 1, kOutBF16 = 2 };

// q holds elements 8l..8l+7: byte p carries element 2p in its low nibble
// and 2p+1 in its high nibble, so element e sits at bit 4*e.
template <int OUT>
__device__ __forceinline__ void deq_store(void *out, uint64_t n, uint64_t base, uint32_t q,
                                          float d, float dmin, int sc, int m) {
  float v[8];
  if (OUT == kOutF16) {
    // half locals rounded as the reference assigns them; the expression
    // final_scale*q - final_min formed in fp32 and rounded once
    const float fs = __half2float(__float2half_rn(d * (float)sc));
    const float fm = __half2float(__float2half_rn(dmin * (float)m));
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float qq = (float)((q >> (4 * e)) & 0xF);
      v[e] = __fsub_rn(__fmul_rn(fs, qq), fm);
    }
  } else {
    const float fs = d * (float)sc;   // exact
    const float fm = dmin * (float)m; // exact
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float qq = (float)((q >> (4 * e)) & 0xF);
      v[e] = __fsub_rn(__fmul_rn(fs, qq), fm);
    }
  }
  if (base + 8 <= n) {
    if (OUT == kOutF32) {
      float *o = reinterpret_cast<float *>(out) + base;
      stg_stream(o, make_float4(v[0], v[1], v[2], v[3]));
      stg_stream(o + 4, make_float4(v[4], v[5], v[6], v[7]));
    } else {
      uint32_t w[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        if (OUT == kOutF16) {
          __half2 h = __halves2half2(__float2half_rn(v[2 * p]), __float2half_rn(v[2 * p + 1]));
          w[p] = *reinterpret_cast<uint32_t *>(&h);
        } else {
          __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * p], v[2 * p + 1]);
          w[p] = *reinterpret_cast<uint32_t *>(&h);
        }
      }
      uint4 *o = reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) + base);
      asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(o), "r"(w[0]), "r"(w[1]),
                   "r"(w[2]), "r"(w[3])
                   : "memory");
    }
  } else {
    for (int e = 0; e < 8; ++e) {
      if (base + e >= n) break;
      if (OUT == kOutF32) {
        reinterpret_cast<float *>(out)[base + e] = v[e];
      } else if (OUT == kOutF16) {
        reinterpret_cast<__half *>(out)[base + e] = __float2half_rn(v[e]);
      } else {
        reinterpret_cast<__nv_bfloat16 *>(out)[base + e] = __float2bfloat16_rn(v[e]);
      }
    }
  }
}

template <int OUT>
__global__ void __launch_bounds__(256) q4k_dequant_kernel(const uint8_t *__restrict__ blocks,
                                                          void *__restrict__ out, uint64_t n,
                                                          uint64_t nblocks) {
  const int lane = threadIdx.x & 31;
  const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const int j = lane >> 2;  // sub-block of this lane's 8 elements
  constexpr int U = 4;      // blocks in flight per warp

  for (uint64_t b0 = warp; b0 < nblocks; b0 += nwarps * U) {
    uint4 hdr[U];
    uint32_t qw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t b = b0 + (uint64_t)u * nwarps;
      if (b < nblocks) {
        const uint8_t *blk = blocks + b * kBlockBytes;
        hdr[u] = ldg_stream(blk);
        asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];"
                     : "=r"(qw[u])
                     : "l"(blk + 16 + 4 * lane));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t b = b0 + (uint64_t)u * nwarps;
      if (b < nblocks) {
        int sc, m;
        q4k_scale_min_regs(j, hdr[u].y, hdr[u].z, hdr[u].w, sc, m);
        const float d = half_bits_to_float(hdr[u].x);
        const float dmin = half_bits_to_float(hdr[u].x >> 16);
        deq_store<OUT>(out, n, b * kQK + 8ull * lane, qw[u], d, dmin, sc, m);
      }
    }
  }
}

// fp32 output: lane l owns elements 4l..4l+3 (qs half-word l, sub-block l/8)
// and 128+4l..128+4l+3 (half-word 32+l, sub-block 4+l/8), so every warp store
// covers 512 contiguous bytes.
__global__ void __launch_bounds__(256) q4k_dequant_f32_kernel(const uint8_t *__restrict__ blocks,
                                                              float *__restrict__ out, uint64_t n,
                                                              uint64_t nblocks) {
  const int lane = threadIdx.x & 31;
  const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  const int j0 = lane >> 3, j1 = 4 + (lane >> 3);
  constexpr int U = 4;

  for (uint64_t b0 = warp; b0 < nblocks; b0 += nwarps * U) {
    uint4 hdr[U];
    uint32_t q0[U], q1[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t b = b0 + (uint64_t)u * nwarps;
      if (b < nblocks) {
        const uint8_t *blk = blocks + b * kBlockBytes;
        hdr[u] = ldg_stream(blk);
        unsigned short a, c;
        asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(a) : "l"(blk + 16 + 2 * lane));
        asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(c) : "l"(blk + 80 + 2 * lane));
        q0[u] = a;
        q1[u] = c;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint64_t b = b0 + (uint64_t)u * nwarps;
      if (b >= nblocks) continue;
      const float d = half_bits_to_float(hdr[u].x);
      const float dmin = half_bits_to_float(hdr[u].x >> 16);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        int sc, m;
        q4k_scale_min_regs(half ? j1 : j0, hdr[u].y, hdr[u].z, hdr[u].w, sc, m);
        const float fs = d * (float)sc;    // exact
        const float fm = dmin * (float)m;  // exact
        const uint32_t q = half ? q1[u] : q0[u];
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = __fsub_rn(__fmul_rn(fs, (float)((q >> (4 * e)) & 0xF)), fm);
        const uint64_t base = b * kQK + 128ull * half + 4ull * lane;
        if (base + 4 <= n) {
          stg_stream(out + base, make_float4(v[0], v[1], v[2], v[3]));
        } else {
          for (int e = 0; e < 4; ++e)
            if (base + e < n) out[base + e] = v[e];
        }
      }
    }
  }
}

// ---- GGUF element order -> the order the kernels read ----------------------------
//
// GGUF (ggml) Q4_K blocks hold element 64j + l (l < 32) in the low nibble of
// qs[32j + l] and element 64j + 32 + l in its high nibble; the reference's
// kernels, and every kernel of this library, read element i from qs[i / 2],
// low nibble for even i (DequantKernels.metal:86-88).  The repack is a byte
// shuffle of the 128 quant bytes (d, dmin and the scales are the same in
// both), so dequantizing the repacked block is bit-identical to
// dequantizing the GGUF block in its own order.  A CTA stages 128 blocks
// (18,432 bytes) with coalesced 16-byte loads, one thread shuffles each
// block in shared memory, and the CTA stores them back coalesced; in place
// (src == dst) is allowed.
constexpr int kRepackBlocks = 128;

// interleaved quant word w (bytes 4w .. 4w+3 of a 64-element group) from the
// group's 8 GGUF words c: w < 4 takes the low nibbles of bytes 8w .. 8w+7,
// w >= 4 the high nibbles of bytes 8(w-4) .. 8(w-4)+7
__device__ __forceinline__ uint32_t repack_word(const uint32_t *c, int w) {
  const int sh = w < 4 ? 0 : 4;
  const int s = w & 3;
  const uint32_t a = (c[2 * s] >> sh) & 0x0F0F0F0Fu, b = (c[2 * s + 1] >> sh) & 0x0F0F0F0Fu;
  // bytes 0 and 2 of x | (x >> 4) are (n0 | n1 << 4) and (n2 | n3 << 4)
  return __byte_perm(a | (a >> 4), b | (b >> 4), 0x6420);
}

__global__ void __launch_bounds__(kRepackBlocks) q4k_repack_kernel(const uint8_t *src,
                                                                   uint8_t *dst,
                                                                   uint64_t nblocks) {
  __shared__ __align__(16) uint8_t s[kRepackBlocks * kBlockBytes];
  uint4 *sv = reinterpret_cast<uint4 *>(s);
  for (uint64_t b0 = blockIdx.x * (uint64_t)kRepackBlocks; b0 < nblocks;
       b0 += gridDim.x * (uint64_t)kRepackBlocks) {
    const int nbk = (int)min((uint64_t)kRepackBlocks, nblocks - b0);
    const uint4 *g = reinterpret_cast<const uint4 *>(src + b0 * kBlockBytes);
    for (int i = threadIdx.x; i < nbk * 9; i += kRepackBlocks) sv[i] = g[i];
    __syncthreads();
    if (threadIdx.x < nbk) {
      uint32_t *qs = reinterpret_cast<uint32_t *>(s + threadIdx.x * kBlockBytes + 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t c[8], o[8];
#pragma unroll
        for (int w = 0; w < 8; ++w) c[w] = qs[8 * j + w];
#pragma unroll
        for (int w = 0; w < 8; ++w) o[w] = repack_word(c, w);
#pragma unroll
        for (int w = 0; w < 8; ++w) qs[8 * j + w] = o[w];
      }
    }
    __syncthreads();
    uint4 *gd = reinterpret_cast<uint4 *>(dst + b0 * kBlockBytes);
    for (int i = threadIdx.x; i < nbk * 9; i += kRepackBlocks) gd[i] = sv[i];
    __syncthreads();
  }
}

// ---- generators -------------------------------------------------------------

// block b of a generated tensor, written to o (144 bytes, 16-byte aligned)
__device__ void gen_q4k_block(uint64_t seed, uint64_t stream, uint64_t b, uint8_t *out_blk) {
  const float d = (float)fabs(rng_normal(seed, stream, 2 * b));
  const float dm = (float)fabs(rng_normal(seed, stream, 2 * b + 1));
  const uint32_t hd = __half_as_ushort(__float2half_rn(__fmul_rn(d, 0.01f)));
  const uint32_t hm = __half_as_ushort(__float2half_rn(__fmul_rn(dm, 0.01f)));
  uint32_t w[36];
  w[0] = hd | (hm << 16);
#pragma unroll
  for (int k = 0; k < 18; ++k) {
    const uint64_t r = rng_u64(seed, stream ^ (kTagBytes << 56), b * 18 + (uint64_t)k);
    if (2 * k + 1 < 36) w[2 * k + 1] = (uint32_t)r;
    if (2 * k + 2 < 36) w[2 * k + 2] = (uint32_t)(r >> 32);
  }
  uint4 *o = reinterpret_cast<uint4 *>(out_blk);
#pragma unroll
  for (int c = 0; c < 9; ++c) o[c] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

__global__ void gen_q4k_kernel(uint64_t seed, uint64_t stream, uint64_t first_block,
                               uint64_t nblocks, uint8_t *__restrict__ out) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  gen_q4k_block(seed, stream, first_block + i, out + i * kBlockBytes);
}

// the sub-matrix rows row0.., block columns kb0 .. kb0+nkb of a generated
// tensor with nb_full block columns, stored densely ([rows][nkb] blocks)
__global__ void gen_q4k_sub_kernel(uint64_t seed, uint64_t stream, uint64_t nb_full,
                                   uint64_t row0, uint64_t rows, uint64_t kb0, uint64_t nkb,
                                   uint8_t *__restrict__ out) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= rows * nkb) return;
  const uint64_t r = i / nkb, c = i % nkb;
  gen_q4k_block(seed, stream, (row0 + r) * nb_full + kb0 + c, out + i * kBlockBytes);
}

__global__ void gen_f16_kernel(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n,
                               float mean, float stdv, __half *__restrict__ out) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = (float)rng_normal(seed, stream, first + i);
  out[i] = __float2half_rn(__fadd_rn(mean, __fmul_rn(stdv, v)));
}

__global__ void gen_f32_kernel(uint64_t seed, uint64_t stream, uint64_t first, uint64_t n,
                               float mean, float stdv, float *__restrict__ out) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = (float)rng_normal(seed, stream, first + i);
  out[i] = __fadd_rn(mean, __fmul_rn(stdv, v));
}

template <int OUT>
static int launch_dequant(mlm_ctx *ctx, const void *blocks, void *out, uint64_t n,
                          const char *name) {
  MLM_CHECK_CTX(ctx);
  if (n == 0) return MLM_OK;  // the reference returns an empty buffer
  MLM_REQUIRE(ctx, blocks && out, MLM_ERR_ARG, "%s: null buffer", name);
  MLM_REQUIRE(ctx, aligned16(blocks) && aligned16(out), MLM_ERR_ALIGN,
              "%s: blocks and output must be 16-byte aligned", name);
  const uint64_t nblocks = (n + kQK - 1) / kQK;
  const int threads = 256;
  const uint64_t want_warps = (nblocks + 3) / 4;
  uint64_t grid = (want_warps * 32 + threads - 1) / threads;
  const uint64_t cap = (uint64_t)ctx->sm_count * 8;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  if (OUT == kOutF32)
    q4k_dequant_f32_kernel<<<(unsigned)grid, threads, 0, ctx->stream>>>(
        reinterpret_cast<const uint8_t *>(blocks), reinterpret_cast<float *>(out), n, nblocks);
  else
    q4k_dequant_kernel<OUT><<<(unsigned)grid, threads, 0, ctx->stream>>>(
        reinterpret_cast<const uint8_t *>(blocks), out, n, nblocks);
  return check_launch(ctx, name);
}

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_q4k_dequant_f32(mlm_ctx *ctx, const void *blocks, float *out, uint64_t n) {
  return launch_dequant<kOutF32>(ctx, blocks, out, n, "mlm_q4k_dequant_f32");
}

extern "C" int mlm_q4k_dequant_f16(mlm_ctx *ctx, const void *blocks, void *out, uint64_t n) {
  return launch_dequant<kOutF16>(ctx, blocks, out, n, "mlm_q4k_dequant_f16");
}

extern "C" int mlm_q4k_dequant_bf16(mlm_ctx *ctx, const void *blocks, void *out, uint64_t n) {
  return launch_dequant<kOutBF16>(ctx, blocks, out, n, "mlm_q4k_dequant_bf16");
}

extern "C" int mlm_q4k_repack_canonical(mlm_ctx *ctx, const void *src, void *dst,
                                        uint64_t nblocks) {
  MLM_CHECK_CTX(ctx);
  if (nblocks == 0) return MLM_OK;
  MLM_REQUIRE(ctx, src && dst, MLM_ERR_ARG, "mlm_q4k_repack_canonical: null buffer");
  MLM_REQUIRE(ctx, aligned16(src) && aligned16(dst), MLM_ERR_ALIGN,
              "mlm_q4k_repack_canonical: buffers must be 16-byte aligned");
  const char *s0 = reinterpret_cast<const char *>(src), *d0 = reinterpret_cast<const char *>(dst);
  const size_t bytes = (size_t)nblocks * kBlockBytes;
  MLM_REQUIRE(ctx, s0 == d0 || s0 + bytes <= d0 || d0 + bytes <= s0, MLM_ERR_ARG,
              "mlm_q4k_repack_canonical: src and dst overlap without being equal");
  const uint64_t groups = (nblocks + kRepackBlocks - 1) / kRepackBlocks;
  const unsigned grid = (unsigned)std::min<uint64_t>(groups, (uint64_t)ctx->sm_count * 8);
  q4k_repack_kernel<<<grid, kRepackBlocks, 0, ctx->stream>>>(
      reinterpret_cast<const uint8_t *>(src), reinterpret_cast<uint8_t *>(dst), nblocks);
  return check_launch(ctx, "mlm_q4k_repack_canonical");
}

extern "C" int mlm_gen_q4k(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t first_block,
                           uint64_t nblocks, void *out) {
  MLM_CHECK_CTX(ctx);
  if (nblocks == 0) return MLM_OK;
  MLM_REQUIRE(ctx, out, MLM_ERR_ARG, "mlm_gen_q4k: null output");
  MLM_REQUIRE(ctx, aligned16(out), MLM_ERR_ALIGN, "mlm_gen_q4k: output must be 16-byte aligned");
  const unsigned grid = (unsigned)((nblocks + 127) / 128);
  gen_q4k_kernel<<<grid, 128, 0, ctx->stream>>>(seed, stream, first_block, nblocks,
                                                reinterpret_cast<uint8_t *>(out));
  return check_launch(ctx, "mlm_gen_q4k");
}

extern "C" int mlm_gen_q4k_sub(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t nb_full,
                               uint64_t row0, uint64_t rows, uint64_t kb0, uint64_t nkb,
                               void *out) {
  MLM_CHECK_CTX(ctx);
  if (rows == 0 || nkb == 0) return MLM_OK;
  MLM_REQUIRE(ctx, out, MLM_ERR_ARG, "mlm_gen_q4k_sub: null output");
  MLM_REQUIRE(ctx, kb0 + nkb <= nb_full, MLM_ERR_SHAPE,
              "mlm_gen_q4k_sub: block columns %llu..%llu of %llu", (unsigned long long)kb0,
              (unsigned long long)(kb0 + nkb), (unsigned long long)nb_full);
  MLM_REQUIRE(ctx, aligned16(out), MLM_ERR_ALIGN, "mlm_gen_q4k_sub: output must be 16-byte aligned");
  const uint64_t n = rows * nkb;
  gen_q4k_sub_kernel<<<(unsigned)((n + 127) / 128), 128, 0, ctx->stream>>>(
      seed, stream, nb_full, row0, rows, kb0, nkb, reinterpret_cast<uint8_t *>(out));
  return check_launch(ctx, "mlm_gen_q4k_sub");
}

extern "C" int mlm_gen_f16(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t first,
                           uint64_t n, float mean, float stdv, void *out) {
  MLM_CHECK_CTX(ctx);
  if (n == 0) return MLM_OK;
  MLM_REQUIRE(ctx, out, MLM_ERR_ARG, "mlm_gen_f16: null output");
  gen_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
      seed, stream, first, n, mean, stdv, reinterpret_cast<__half *>(out));
  return check_launch(ctx, "mlm_gen_f16");
}

extern "C" int mlm_gen_f32(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t first,
                           uint64_t n, float mean, float stdv, float *out) {
  MLM_CHECK_CTX(ctx);
  if (n == 0) return MLM_OK;
  MLM_REQUIRE(ctx, out, MLM_ERR_ARG, "mlm_gen_f32: null output");
  gen_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(seed, stream, first, n,
                                                                      mean, stdv, out);
  return check_launch(ctx, "mlm_gen_f32");
}
