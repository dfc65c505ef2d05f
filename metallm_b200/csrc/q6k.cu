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
#include "q4k_gemv_common.cuh"

namespace mlm {

constexpr int kQ6Bytes = 210;
constexpr uint64_t kTagQ6K = 0x66ULL;

// ---- generator ---------------------------------------------------------------

// block b of a generated Q6_K tensor: 208 uniform bytes (ql, qh, scales),
// then d = fp16(|N(0,1)| * 0.01) -- the arithmetic of orc_gen_q6k
__device__ __forceinline__ void gen_q6k_block(uint64_t seed, uint64_t stream, uint64_t b,
                                              uint8_t *out) {
  const uint64_t st = stream ^ (kTagQ6K << 56);
  uint16_t *o = reinterpret_cast<uint16_t *>(out);  // 2-byte aligned
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

__global__ void gen_q6k_kernel(uint64_t seed, uint64_t stream, uint64_t first_block,
                               uint64_t nblocks, uint8_t *out) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  gen_q6k_block(seed, stream, first_block + i, out + i * kQ6Bytes);
}

// block columns [kb0, kb0 + nkb) of rows [row0, row0 + rows) of a generated
// tensor with nb_full blocks per row (a column shard under tensor parallelism)
__global__ void gen_q6k_sub_kernel(uint64_t seed, uint64_t stream, uint64_t nb_full,
                                   uint64_t row0, uint64_t rows, uint64_t kb0, uint64_t nkb,
                                   uint8_t *__restrict__ out) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= rows * nkb) return;
  const uint64_t r = i / nkb, c = i % nkb;
  gen_q6k_block(seed, stream, (row0 + r) * nb_full + kb0 + c, out + i * kQ6Bytes);
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
// y[r] = sum_k deq(W[r][k]) x[k] (+ residual[r]), x fp16, fp32 accumulation,
// on the tensor cores the way the Q4_K GEMV uses them: a 6-bit quant placed
// under the fp16 exponent of 1024 (a byte permute) minus 1056 is q - 32
// exactly, so the quants are exact fp16 operands of mma.sync.m16n8k16 and
// their products with x are exact in the fp32 accumulators.
//
// MMA mapping: thread (g = lane / 4, t = lane % 4) holds, for rows g and g+8
// of a 16-row tile, quarter k = t of each 128-element half of a block:
// elements 32t + l (l = 0..31), i.e. the scale groups 2t (l < 16) and 2t + 1
// (l >= 16) of the half.  One 32-bit word of ql and one of qh give four
// consecutive quants; per word one MMA takes (l0, l1) and (l2, l3) as its
// k-slots 2t, 2t+1 and 2t+8, 2t+9.  B column n carries x only for the
// threads whose word belongs to scale group n (the others read zeros), so
// after the 8 words of a half C[row][2t] and C[row][2t+1] hold the sums of
// q * x of groups 2t and 2t+1 -- in the thread that holds their scales; the
// epilogue multiplies them by d * scale and accumulates per row.
//
// Work: a CTA takes 16-row tiles; per tile it stages 8-block chunks of the
// 16 rows (26,880 bytes, coalesced 16-byte cp.async, a 3-stage ring shared
// by the CTA) and warp w takes block column w of each chunk.  Blocks sit at
// 2-byte alignment (210 bytes each), so a thread loads the 9 aligned words
// around its 8 and funnel-shifts them.  At the end of a tile the warps' row
// sums are added in warp order (deterministic) and y is stored.
constexpr int kQ6TileRows = 16;
constexpr int kQ6Warps = 8;  // one block column of a chunk per warp
constexpr int kQ6Threads = kQ6Warps * 32;
constexpr int kQ6ChunkBlocks = kQ6Warps;
constexpr int kQ6RowChunk = kQ6ChunkBlocks * kQ6Bytes;       // 1680 = 105 x 16
constexpr int kQ6StageBytes = kQ6TileRows * kQ6RowChunk;     // 26,880
constexpr int kQ6Stages = 3;
constexpr int kQ6ZeroBytes = 512;  // zeros read by the inactive B columns
constexpr int kQ6FixedSmem = kQ6ZeroBytes + kQ6Stages * kQ6StageBytes + kQ6Warps * kQ6TileRows * 4;
constexpr int kQ6MaxCols = 32768;

struct Q6GemvArgs {
  const uint8_t *W;
  const __half *x;       // kHalf: fp16 x
  const float *x_scale;  // kHalf: per 32-element sub-block of x (NULL: 1)
  const float *xa, *xb;  // fp32 sources of x in the kRmsNorm / kSwiGLU modes
  float eps;
  int x_mode;            // GemvInput::Mode
  float *y;
  const float *residual;
  int rows, nb, nchunk, tiles;
};

__device__ __forceinline__ void q6_cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// the 8 words at the 2-byte-aligned shared address a: 9 aligned loads,
// funnel-shifted by 0 or 16 bits
__device__ __forceinline__ void lds8_a2(uint32_t a, uint32_t (&w)[8]) {
  const uint32_t base = a & ~3u, sh = (a & 2u) * 8u;
  uint32_t r[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) r[i] = lds32(base + 4 * i);
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}

// four 6-bit quants (bytes of q4) -> two fp16x2 of q - 32
__device__ __forceinline__ void q6_to_f16x2(uint32_t q4, uint32_t &lo, uint32_t &hi) {
  const uint32_t kBias = 0xE420E420u;  // fp16 -1056 in both halves
  uint32_t a = __byte_perm(q4, 0x64646464u, 0x4140), b = __byte_perm(q4, 0x64646464u, 0x4342);
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(kBias));
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(kBias));
}

// kScaled: x carries a scale per 32-element sub-block (fp16 x with x_scale,
// or the kSwiGLU staging); the scale multiplies the sub-block's MMA sums.
template <bool kScaled>
__global__ void __launch_bounds__(kQ6Threads, 2) q6k_gemv_kernel(Q6GemvArgs p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int cols = p.nb * kQK;
  uint8_t *xs = smem;                                   // fp16 x [cols]
  uint8_t *zero = xs + (size_t)cols * 2;                // kQ6ZeroBytes
  uint8_t *stages = zero + kQ6ZeroBytes;                // kQ6Stages x [16][1680]
  float *red = reinterpret_cast<float *>(stages + kQ6Stages * kQ6StageBytes);  // [8][16]
  float *xscl = red + kQ6Warps * kQ6TileRows;           // [cols / 32] scales of x
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t stages_s = (uint32_t)__cvta_generic_to_shared(stages);

  const int my_tiles = (int)blockIdx.x < p.tiles ? (p.tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int total = my_tiles * p.nchunk;

  // unit q (tile blockIdx.x + (q / nchunk) gridDim.x, chunk q % nchunk) into
  // stage q % kQ6Stages; always one commit group
  auto issue = [&](int q) {
    if (q < total) {
      const int ti = q / p.nchunk, c = q - ti * p.nchunk;
      const int r0 = ((int)blockIdx.x + ti * (int)gridDim.x) * kQ6TileRows;
      const uint32_t dst0 = stages_s + (uint32_t)(q % kQ6Stages) * kQ6StageBytes;
      for (int i = threadIdx.x; i < kQ6TileRows * (kQ6RowChunk / 16); i += kQ6Threads) {
        const int rr = i / (kQ6RowChunk / 16), k = i - rr * (kQ6RowChunk / 16);
        if (r0 + rr < p.rows) {
          const uint8_t *src =
              p.W + ((size_t)(r0 + rr) * p.nb + (size_t)c * kQ6ChunkBlocks) * kQ6Bytes + 16 * k;
          q6_cp_async16(dst0 + rr * kQ6RowChunk + 16 * k, src);
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // the weights do not depend on the kernel before this one
#pragma unroll
  for (int q = 0; q < kQ6Stages - 1; ++q) issue(q);
  pdl_wait_then_release();
  {
    // x -> fp16 in shared memory (the modes of the Q4_K GEMV's staging):
    // kHalf copies x (and its scales); kRmsNorm stores fp16(a * rms * w);
    // kSwiGLU stores silu(g) * u with one power-of-two scale per sub-block,
    // four consecutive lanes holding the four 8-element groups of one
    uint4 *xo = reinterpret_cast<uint4 *>(xs);
    const int ngroups = cols / 8;
    for (int i = threadIdx.x; i < kQ6ZeroBytes / 16; i += kQ6Threads)
      reinterpret_cast<uint4 *>(zero)[i] = make_uint4(0, 0, 0, 0);
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
      for (int i = threadIdx.x; i < ngroups; i += kQ6Threads) xo[i] = __ldg(xg + i);
      if (kScaled)
        for (int i = threadIdx.x; i < cols / 32; i += kQ6Threads) xscl[i] = __ldg(p.x_scale + i);
    } else if (p.x_mode == GemvInput::kRmsNorm) {
      float ss = 0.f;
      const float4 *a4 = reinterpret_cast<const float4 *>(p.xa);
      for (int k = threadIdx.x; k < cols / 4; k += kQ6Threads) {
        const float4 v = __ldg(a4 + k);
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.f;
      for (int w = 0; w < kQ6Warps; ++w) tot += red[w];
      const float scale = rms_scale(tot, cols, p.eps);
      for (int i = threadIdx.x; i < ngroups; i += kQ6Threads) {
        float a[8], w[8];
        load8(p.xa, i, a);
        load8(p.xb, i, w);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = (a[e] * scale) * safe_weight(w[e]);
        xo[i] = pack(a);
      }
      __syncthreads();  // red is reused by the tile sums
    } else {  // kSwiGLU (ngroups is a multiple of 32: whole warps in the shuffles)
      for (int i = threadIdx.x; i < ngroups; i += kQ6Threads) {
        float gv[8], uv[8];
        load8(p.xa, i, gv);
        load8(p.xb, i, uv);
        float m = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          gv[e] = swiglu(gv[e], uv[e]);
          m = fmaxf(m, fabsf(gv[e]));
        }
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        const int ex = max(0, (int)((__float_as_uint(m) >> 23) & 0xFF) - 127 - 14);
        const float inv = __uint_as_float((uint32_t)(127 - ex) << 23);
#pragma unroll
        for (int e = 0; e < 8; ++e) gv[e] *= inv;
        xo[i] = pack(gv);
        if ((i & 3) == 0) xscl[i >> 2] = __uint_as_float((uint32_t)(127 + ex) << 23);
      }
    }
  }

  // B operands: words 0..3 of a half belong to group 2t (column 2t), words
  // 4..7 to group 2t + 1; thread (g, t) supplies x of its words when g is
  // that column, zeros otherwise
  const bool lo_on = g == 2 * t, hi_on = g == 2 * t + 1;
  const uint32_t xs_s = (uint32_t)__cvta_generic_to_shared(xs) + 64 * t;  // element 32t
  const uint32_t zero_s = (uint32_t)__cvta_generic_to_shared(zero);
  const int sh_lo = t >= 2 ? 4 : 0;  // high nibbles for quarters 2, 3
  const int ql_off = 32 * (t & 1);

  float acc[2] = {0.f, 0.f};  // rows g, g + 8 of the tile
  for (int q = 0; q < total; ++q) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kQ6Stages - 2) : "memory");
    __syncthreads();  // unit q landed for every thread; stage (q - 1) is free
    issue(q + kQ6Stages - 1);
    const int ti = q / p.nchunk, c = q - ti * p.nchunk;
    const uint32_t st = stages_s + (uint32_t)(q % kQ6Stages) * kQ6StageBytes;
    const uint32_t blk_g = st + g * kQ6RowChunk + warp * kQ6Bytes;
    const uint32_t blk_g8 = blk_g + 8 * kQ6RowChunk;
    const uint32_t xblk = (uint32_t)(c * kQ6ChunkBlocks + warp) * (kQK * 2);  // byte offset of the block's x
    const uint32_t xlo = lo_on ? xs_s + xblk : zero_s;
    const uint32_t xhi = hi_on ? xs_s + xblk : zero_s;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t qlg[8], qhg[8], ql8[8], qh8[8];
      lds8_a2(blk_g + 64 * h + ql_off, qlg);
      lds8_a2(blk_g + 128 + 32 * h, qhg);
      lds8_a2(blk_g8 + 64 * h + ql_off, ql8);
      lds8_a2(blk_g8 + 128 + 32 * h, qh8);
      float cacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const uint32_t q4g = ((qlg[w] >> sh_lo) & 0x0F0F0F0Fu) | (((qhg[w] >> (2 * t)) << 4) & 0x30303030u);
        const uint32_t q48 = ((ql8[w] >> sh_lo) & 0x0F0F0F0Fu) | (((qh8[w] >> (2 * t)) << 4) & 0x30303030u);
        uint32_t a0, a2, a1, a3;
        q6_to_f16x2(q4g, a0, a2);
        q6_to_f16x2(q48, a1, a3);
        // x of elements 128h + 32t + 4w .. +3 of this block (zeros when inactive)
        const uint32_t xa = (w < 4 ? xlo : xhi) + 256 * h + 8 * w;
        uint32_t b0, b1;
        asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(xa));
        mma_f16_16816(cacc, a0, a1, a2, a3, b0, b1);
      }
      // scales of groups 8h + 2t, 8h + 2t + 1 and d of rows g and g + 8
      const uint32_t scg = lds32((blk_g + 192 + 8 * h + 2 * t) & ~3u) >> (((blk_g + 2 * t) & 2u) * 8u);
      const uint32_t sc8 = lds32((blk_g8 + 192 + 8 * h + 2 * t) & ~3u) >> (((blk_g8 + 2 * t) & 2u) * 8u);
      const uint32_t dg = lds32((blk_g + 208) & ~3u) >> (((blk_g + 208) & 2u) * 8u);
      const uint32_t d8 = lds32((blk_g8 + 208) & ~3u) >> (((blk_g8 + 208) & 2u) * 8u);
      float fdg = half_bits_to_float(dg & 0xFFFFu), fd8 = half_bits_to_float(d8 & 0xFFFFu);
      if (kScaled) {  // sub-block 4h + t of block c * 8 + warp
        const float xsc = xscl[(c * kQ6ChunkBlocks + warp) * 8 + 4 * h + t];
        fdg *= xsc;
        fd8 *= xsc;
      }
      acc[0] = fmaf(fdg * (float)(int8_t)(scg & 0xFF), cacc[0], acc[0]);
      acc[0] = fmaf(fdg * (float)(int8_t)((scg >> 8) & 0xFF), cacc[1], acc[0]);
      acc[1] = fmaf(fd8 * (float)(int8_t)(sc8 & 0xFF), cacc[2], acc[1]);
      acc[1] = fmaf(fd8 * (float)(int8_t)((sc8 >> 8) & 0xFF), cacc[3], acc[1]);
    }
    if (c == p.nchunk - 1) {  // the tile's last chunk: add the warps' rows, store y
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
        acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);
      }
      if (t == 0) {
        red[warp * kQ6TileRows + g] = acc[0];
        red[warp * kQ6TileRows + g + 8] = acc[1];
      }
      acc[0] = acc[1] = 0.f;
      __syncthreads();
      const int r0 = ((int)blockIdx.x + ti * (int)gridDim.x) * kQ6TileRows;
      if (threadIdx.x < kQ6TileRows && r0 + (int)threadIdx.x < p.rows) {
        float s = red[threadIdx.x];
#pragma unroll
        for (int w = 1; w < kQ6Warps; ++w) s += red[w * kQ6TileRows + threadIdx.x];
        const int r = r0 + threadIdx.x;
        p.y[r] = s + (p.residual ? p.residual[r] : 0.f);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

size_t q6k_gemv_smem(int cols) { return (size_t)cols * 2 + kQ6FixedSmem + (size_t)cols / 8; }

int q6k_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q6k_gemv_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)q6k_gemv_smem(kQ6MaxCols)));
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q6k_gemv_kernel<true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)q6k_gemv_smem(kQ6MaxCols)));
  return MLM_OK;
}

int q6k_gemv_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const GemvInput &in,
                    float *y, const float *residual, cudaStream_t stream) {
  const bool half = in.mode == GemvInput::kHalf;
  const void *x = half ? in.x_f16 : in.a;
  MLM_REQUIRE(ctx, W && x && y && (half || in.b), MLM_ERR_ARG, "mlm_q6k_gemv: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && cols > 0 && cols % (kQK * kQ6ChunkBlocks) == 0 && cols <= kQ6MaxCols,
              MLM_ERR_SHAPE,
              "mlm_q6k_gemv: rows=%d cols=%d (cols a multiple of 2048, at most %d)", rows, cols,
              kQ6MaxCols);
  MLM_REQUIRE(ctx, aligned16(W) && aligned16(x) && (half || aligned16(in.b)) &&
                       (!residual || aligned4(residual)),
              MLM_ERR_ALIGN, "mlm_q6k_gemv: W and x must be 16-byte aligned");
  Q6GemvArgs a;
  a.W = reinterpret_cast<const uint8_t *>(W);
  a.x = reinterpret_cast<const __half *>(in.x_f16);
  a.x_scale = in.x_scale;
  a.xa = in.a;
  a.xb = in.b;
  a.eps = in.eps;
  a.x_mode = in.mode;
  a.y = y;
  a.residual = residual;
  a.rows = rows;
  a.nb = cols / kQK;
  a.nchunk = a.nb / kQ6ChunkBlocks;
  a.tiles = (rows + kQ6TileRows - 1) / kQ6TileRows;
  const int ctas = std::max(1, std::min(a.tiles, 2 * ctx->sm_count));
  const bool scaled = in.mode == GemvInput::kSwiGLU || (half && in.x_scale != nullptr);
  auto kern = scaled ? q6k_gemv_kernel<true> : q6k_gemv_kernel<false>;
  return check_launch_pdl(ctx,
                          launch_pdl(kern, dim3(ctas), dim3(kQ6Threads), q6k_gemv_smem(cols),
                                     stream, a),
                          "mlm_q6k_gemv");
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

int q6k_dequant_bf16_launch(mlm_ctx *ctx, const void *blocks, void *out, uint64_t n,
                            cudaStream_t stream) {
  MLM_REQUIRE(ctx, n % kQK == 0 && (reinterpret_cast<uintptr_t>(blocks) & 1) == 0,
              MLM_ERR_SHAPE, "Q6_K dequant: n=%llu", (unsigned long long)n);
  const uint64_t nblocks = n / kQK;
  if (nblocks == 0) return MLM_OK;
  const uint64_t warps = std::min<uint64_t>(nblocks, (uint64_t)ctx->sm_count * 64);
  const unsigned grid = (unsigned)((warps * 32 + 255) / 256);
  q6k_dequant_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
      reinterpret_cast<const uint8_t *>(blocks), reinterpret_cast<__nv_bfloat16 *>(out), nblocks);
  return check_launch(ctx, "Q6_K dequant");
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

extern "C" int mlm_gen_q6k_sub(mlm_ctx *ctx, uint64_t seed, uint64_t stream, uint64_t nb_full,
                               uint64_t row0, uint64_t rows, uint64_t kb0, uint64_t nkb,
                               void *out) {
  MLM_CHECK_CTX(ctx);
  if (rows == 0 || nkb == 0) return MLM_OK;
  MLM_REQUIRE(ctx, out, MLM_ERR_ARG, "mlm_gen_q6k_sub: null output");
  MLM_REQUIRE(ctx, kb0 + nkb <= nb_full, MLM_ERR_SHAPE,
              "mlm_gen_q6k_sub: block columns %llu..%llu of %llu", (unsigned long long)kb0,
              (unsigned long long)(kb0 + nkb), (unsigned long long)nb_full);
  MLM_REQUIRE(ctx, (reinterpret_cast<uintptr_t>(out) & 1) == 0, MLM_ERR_ALIGN,
              "mlm_gen_q6k_sub: output must be 2-byte aligned");
  const uint64_t n = rows * nkb;
  gen_q6k_sub_kernel<<<(unsigned)((n + 127) / 128), 128, 0, ctx->stream>>>(
      seed, stream, nb_full, row0, rows, kb0, nkb, reinterpret_cast<uint8_t *>(out));
  return check_launch(ctx, "mlm_gen_q6k_sub");
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
  return q6k_gemv_launch(ctx, W, rows, cols, gemv_half(x_f16), y, residual, ctx->stream);
}

extern "C" int mlm_q6k_gemv_xs(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_f16,
                               const float *x_scale, float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  if (!x_scale) return set_error(ctx, MLM_ERR_ARG, "mlm_q6k_gemv_xs: null x_scale");
  return q6k_gemv_launch(ctx, W, rows, cols, gemv_half(x_f16, x_scale), y, residual,
                         ctx->stream);
}

extern "C" int mlm_q6k_gemv_rmsnorm(mlm_ctx *ctx, const void *W, int rows, int cols,
                                    const float *hidden, const float *norm_w, float eps,
                                    float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  GemvInput in;
  in.mode = GemvInput::kRmsNorm;
  in.a = hidden;
  in.b = norm_w;
  in.eps = eps;
  return q6k_gemv_launch(ctx, W, rows, cols, in, y, residual, ctx->stream);
}

extern "C" int mlm_q6k_gemv_swiglu(mlm_ctx *ctx, const void *W, int rows, int cols,
                                   const float *gate, const float *up, float *y,
                                   const float *residual) {
  MLM_CHECK_CTX(ctx);
  GemvInput in;
  in.mode = GemvInput::kSwiGLU;
  in.a = gate;
  in.b = up;
  return q6k_gemv_launch(ctx, W, rows, cols, in, y, residual, ctx->stream);
}

extern "C" int mlm_q6k_gemm(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                            int tokens, float *y, const float *residual, void *scratch_bf16) {
  MLM_CHECK_CTX(ctx);
  return q6k_gemm_launch(ctx, W, rows, cols, x_bf16, tokens, y, residual, scratch_bf16,
                         ctx->stream);
}
