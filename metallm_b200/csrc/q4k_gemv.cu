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
// mantissa bits of a binary16 is the subnormal q * 2^-24, so one LOP3 turns
// two nibbles into an exact f16x2 operand with no unpack arithmetic.  The
// products q*2^-24*x are exact in fp32 and accumulate in fp32; the 2^24 is
// folded into d in the epilogue.
//
// MMA mapping (mma.sync.m16n8k16, A = quants [16 rows x 16 k], B = x):
// thread (g = lane/4, t = lane%4) owns, for each of its rows, the qs words
// 8t..8t+7 of a block, i.e. sub-blocks 2t and 2t+1.  Word w yields four
// f16x2 registers (e0,e4) (e1,e5) (e2,e6) (e3,e7) via (w >> 4s) & 0x000F000F;
// two MMAs consume a word, the k order inside a chunk being that
// permutation.  B column n carries x of sub-block n only, so C[row][n] is
// the per-sub-block sum and lands in the thread that holds that sub-block's
// scale (C columns 2t, 2t+1).  x is staged once per CTA in shared memory in
// the permuted order [x0 x4 x1 x5 x2 x6 x3 x7] per 8-element group.
//
// Work split.  Units are (32-row tile, block column) pairs; each warp gets a
// contiguous range of units in tile-major order, so every SM streams the
// same number of bytes whatever the shape.  A tile covered by one warp is
// stored directly; a tile split between warps leaves one partial per warp
// in the context scratch, and the last warp to arrive (atomic counter) sums
// the partials in k order -- deterministic -- stores y and re-zeroes the
// counter.  Weights reach shared memory through a per-warp ring of
// cp.async (16 B, L1 bypass) stages, one block column of the warp's 32 rows
// per stage, so bytes in flight do not cost registers.
#include "mlm_device.cuh"
#include "mlm_internal.h"

namespace mlm {

constexpr int kGemvWarps = 8;                       // warps per CTA
constexpr int kGemvStages = 4;                      // smem stages per warp
constexpr int kTileRows = 32;                       // rows per warp tile
constexpr int kStageBytes = kTileRows * kBlockBytes;  // 4608
constexpr int kChunksPerStage = kStageBytes / 16;     // 288 = 9 per lane

struct GemvArgs {
  const uint8_t *W;
  const __half *x;
  float *y;
  const float *residual;
  float *partials;  // [nwarps][2][32]
  int *counters;    // [tiles]
  int rows;
  int nb;     // blocks per row
  int tiles;  // ceil(rows / 32)
  long long units;
  int nwarps;  // warps that own work (<= units)
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

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void *gptr, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr), "l"(gptr),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ long long unit_begin(long long w, long long units, int nwarps) {
  return (w * units) / nwarps;
}
// warp whose unit range contains unit u (ranges are never empty: nwarps <= units)
__device__ __forceinline__ int warp_of_unit(long long u, long long units, int nwarps) {
  return (int)(((u + 1) * nwarps - 1) / units);
}

// Copy unit (tile t, block column b) into a stage: 32 rows x 144 B.
__device__ __forceinline__ void issue_stage(const GemvArgs &p, uint32_t stage_addr, int t, int b,
                                            int lane) {
  const size_t row_bytes = (size_t)p.nb * kBlockBytes;
  const uint8_t *tile_base = p.W + (size_t)t * kTileRows * row_bytes + (size_t)b * kBlockBytes;
#pragma unroll
  for (int k = 0; k < kChunksPerStage / 32; ++k) {
    const int c = lane + 32 * k;
    const int row = c / 9, col = c - row * 9;
    const bool ok = t * kTileRows + row < p.rows;
    const uint8_t *src = ok ? tile_base + (size_t)row * row_bytes + col * 16 : p.W;
    cp_async16(stage_addr + row * kBlockBytes + col * 16, src, ok ? 16 : 0);
  }
}

__global__ void __launch_bounds__(kGemvWarps * 32, 1) q4k_gemv_kernel(GemvArgs p) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t *stages = smem;  // [warps][stages][4608]
  uint4 *xperm = reinterpret_cast<uint4 *>(smem + kGemvWarps * kGemvStages * kStageBytes);
  float *xsum = reinterpret_cast<float *>(xperm + p.nb * 32);

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int wg = blockIdx.x * kGemvWarps + warp;
  const bool has_work = wg < p.nwarps;

  long long u0 = 0, u1 = 0;
  uint8_t *my_stages = stages + warp * kGemvStages * kStageBytes;
  const uint32_t my_stage_addr = (uint32_t)__cvta_generic_to_shared(my_stages);
  if (has_work) {
    u0 = unit_begin(wg, p.units, p.nwarps);
    u1 = unit_begin(wg + 1, p.units, p.nwarps);
  }
  // next unit to put in flight, as (tile, block column)
  int it = 0, ib = 0;
  long long un = u0;
  if (has_work) {
    it = (int)(u0 / p.nb);
    ib = (int)(u0 - (long long)it * p.nb);
    // put the first stages in flight before staging x
#pragma unroll
    for (int s = 0; s < kGemvStages - 1; ++s) {
      if (un < u1) {
        issue_stage(p, my_stage_addr + s * kStageBytes, it, ib, lane);
        ++un;
        if (++ib == p.nb) { ib = 0; ++it; }
      }
      cp_async_commit();
    }
  }

  // ---- x -> shared memory, permuted, plus per-sub-block sums ---------------
  {
    const uint4 *xg = reinterpret_cast<const uint4 *>(p.x);
    const int ngroups = p.nb * 32;  // multiple of 32: whole warps stay converged
    for (int i = threadIdx.x; i < ngroups; i += blockDim.x) {
      const uint4 v = __ldg(xg + i);
      uint4 o;
      o.x = __byte_perm(v.x, v.z, 0x5410);  // (x0, x4)
      o.y = __byte_perm(v.x, v.z, 0x7632);  // (x1, x5)
      o.z = __byte_perm(v.y, v.w, 0x5410);  // (x2, x6)
      o.w = __byte_perm(v.y, v.w, 0x7632);  // (x3, x7)
      xperm[i] = o;
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
      const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&v.z));
      const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&v.w));
      float s = ((f0.x + f0.y) + (f1.x + f1.y)) + ((f2.x + f2.y) + (f3.x + f3.y));
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if ((i & 3) == 0) xsum[i >> 2] = s;
    }
  }
  __syncthreads();
  if (!has_work) return;

  // B operands are live only for the thread whose column matches the
  // sub-block of the word: thread (g, t) carries x for words 0..3 of its
  // slice when g == 2t, words 4..7 when g == 2t + 1.
  const int act = g - 2 * tig;  // 0 or 1 when active
  const bool active = (act == 0) || (act == 1);
  const int xoff = 8 * tig + 4 * (act & 1);

  // byte-pair selectors for the scale/min unpack of sub-blocks 2t, 2t+1
  const int sh = (tig & 1) * 16;
  const bool upper = tig >= 2;

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int cur_tile = -1;
  const int first_tile = (int)(u0 / p.nb);
  int t = first_tile, b = (int)(u0 - (long long)first_tile * p.nb);  // current unit

  auto finish_tile = [&](int t, int bstart, int bend) {
    // reduce over the four threads of a row group
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
      acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 2);
    }
    const bool full = (bstart == 0) && (bend == p.nb);
    if (full) {
      if (tig == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = t * kTileRows + g + 8 * i;
          if (r < p.rows) p.y[r] = acc[i] + (p.residual ? p.residual[r] : 0.f);
        }
      }
    } else {
      const int slot = (t == first_tile) ? 0 : 1;
      float *pp = p.partials + ((size_t)wg * 2 + slot) * kTileRows;
      if (tig == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) __stcg(pp + g + 8 * i, acc[i]);
      }
      __threadfence();
      __syncwarp();
      int old = 0;
      if (lane == 0) old = atomicAdd(p.counters + t, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      const long long tu0 = (long long)t * p.nb;
      const int wf = warp_of_unit(tu0, p.units, p.nwarps);
      const int wl = warp_of_unit(tu0 + p.nb - 1, p.units, p.nwarps);
      if (old == wl - wf) {  // last of the (wl - wf + 1) contributors
        __threadfence();
        float s = 0.f;
        for (int w = wf; w <= wl; ++w) {
          const int ft = (int)(unit_begin(w, p.units, p.nwarps) / p.nb);
          const int sl = (ft == t) ? 0 : 1;
          s += __ldcg(p.partials + ((size_t)w * 2 + sl) * kTileRows + lane);
        }
        const int r = t * kTileRows + lane;
        if (r < p.rows) p.y[r] = s + (p.residual ? p.residual[r] : 0.f);
        if (lane == 0) p.counters[t] = 0;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = 0.f;
  };

  int tile_bstart = 0;
  for (long long u = u0; u < u1; ++u) {
    if (un < u1) {
      issue_stage(p, my_stage_addr + (int)(un % kGemvStages) * kStageBytes, it, ib, lane);
      ++un;
      if (++ib == p.nb) { ib = 0; ++it; }
    }
    cp_async_commit();
    if (t != cur_tile) {
      if (cur_tile >= 0) finish_tile(cur_tile, tile_bstart, p.nb);
      cur_tile = t;
      tile_bstart = b;
    }
    cp_async_wait<kGemvStages - 1>();
    __syncwarp();

    const uint8_t *st = my_stages + (int)(u % kGemvStages) * kStageBytes;

    // x operands of this block
    uint4 xv[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      xv[jj] = active ? xperm[b * 32 + xoff + jj] : make_uint4(0, 0, 0, 0);
    }
    const float2 xs = *reinterpret_cast<const float2 *>(xsum + b * 8 + 2 * tig);

#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const uint8_t *r0 = st + (g + 16 * mt) * kBlockBytes;  // rows g, g+16
      const uint8_t *r1 = r0 + 8 * kBlockBytes;               // rows g+8, g+24
      const uint4 h0 = *reinterpret_cast<const uint4 *>(r0);
      const uint4 h1 = *reinterpret_cast<const uint4 *>(r1);
      uint32_t q0[8], q1[8];
      *reinterpret_cast<uint4 *>(&q0[0]) = *reinterpret_cast<const uint4 *>(r0 + 16 + 32 * tig);
      *reinterpret_cast<uint4 *>(&q0[4]) = *reinterpret_cast<const uint4 *>(r0 + 32 + 32 * tig);
      *reinterpret_cast<uint4 *>(&q1[0]) = *reinterpret_cast<const uint4 *>(r1 + 16 + 32 * tig);
      *reinterpret_cast<uint4 *>(&q1[4]) = *reinterpret_cast<const uint4 *>(r1 + 32 + 32 * tig);

      float c0[4] = {0.f, 0.f, 0.f, 0.f};  // words 0..3 (even chain)
      float c1[4] = {0.f, 0.f, 0.f, 0.f};  // words 4..7
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t M = 0x000F000Fu;
        const uint32_t w0 = q0[j], w1 = q1[j];
        const uint4 xb = (j < 4) ? ((act == 0) ? xv[j] : make_uint4(0, 0, 0, 0))
                                 : ((act == 1) ? xv[j - 4] : make_uint4(0, 0, 0, 0));
        float(&c)[4] = (j < 4) ? c0 : c1;
        mma_f16_16816(c, w0 & M, w1 & M, (w0 >> 4) & M, (w1 >> 4) & M, xb.x, xb.y);
        mma_f16_16816(c, (w0 >> 8) & M, (w1 >> 8) & M, (w0 >> 12) & M, (w1 >> 12) & M, xb.z,
                      xb.w);
      }
      // sub-block 2t and 2t+1 sums for row g (c[0], c[1]) and row g+8 (c[2], c[3])
      // (columns of the other sub-blocks are exact zeros)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const uint4 h = hr ? h1 : h0;
        // chain c0 only feeds column 2t, chain c1 only column 2t+1
        const float cs0 = c0[2 * hr];
        const float cs1 = c1[2 * hr + 1];
        const uint32_t s1 = h.y >> sh, s2 = h.z >> sh, s3 = h.w >> sh;
        const uint32_t scp = upper ? ((s3 & 0x0F0Fu) | ((s1 >> 2) & 0x3030u)) : (s1 & 0x3F3Fu);
        const uint32_t mp =
            upper ? (((s3 >> 4) & 0x0F0Fu) | ((s2 >> 2) & 0x3030u)) : (s2 & 0x3F3Fu);
        const float D = half_bits_to_float(h.x) * 16777216.0f;  // d * 2^24
        const float Dm = half_bits_to_float(h.x >> 16);
        const float qs = (float)(scp & 0xFF) * cs0 + (float)((scp >> 8) & 0xFF) * cs1;
        const float ms = (float)(mp & 0xFF) * xs.x + (float)((mp >> 8) & 0xFF) * xs.y;
        acc[2 * mt + hr] += D * qs - Dm * ms;
      }
    }
    __syncwarp();  // stage fully read before it is refilled
    if (++b == p.nb) { b = 0; ++t; }
  }
  cp_async_wait<0>();
  if (cur_tile >= 0) {
    const long long last_u = u1 - 1;
    const int bend = (int)(last_u - (long long)cur_tile * p.nb) + 1;
    finish_tile(cur_tile, tile_bstart, bend);
  }
}

// called once per context, with its device current
int gemv_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q4k_gemv_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ctx->max_smem_optin));
  return MLM_OK;
}

size_t gemv_smem_bytes(int nb) {
  return (size_t)kGemvWarps * kGemvStages * kStageBytes + (size_t)nb * 32 * 16 +
         (size_t)nb * 8 * sizeof(float);
}

int gemv_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x, float *y,
                const float *residual, float *partials, int *counters, int max_warps,
                int max_tiles, cudaStream_t stream) {
  const int nb = cols / kQK;
  const int tiles = (rows + kTileRows - 1) / kTileRows;
  MLM_REQUIRE(ctx, tiles <= max_tiles, MLM_ERR_SHAPE,
              "mlm_q4k_gemv: %d rows exceed the %d-row scratch limit", rows,
              max_tiles * kTileRows);
  const size_t smem = gemv_smem_bytes(nb);
  MLM_REQUIRE(ctx, smem <= (size_t)ctx->max_smem_optin, MLM_ERR_UNSUPPORTED,
              "mlm_q4k_gemv: cols=%d needs %zu B shared memory (max %d)", cols, smem,
              ctx->max_smem_optin);
  GemvArgs a;
  a.W = reinterpret_cast<const uint8_t *>(W);
  a.x = reinterpret_cast<const __half *>(x);
  a.y = y;
  a.residual = residual;
  a.partials = partials;
  a.counters = counters;
  a.rows = rows;
  a.nb = nb;
  a.tiles = tiles;
  a.units = (long long)tiles * nb;
  long long want = (long long)ctx->sm_count * kGemvWarps;
  if (want > a.units) want = a.units;
  if (want > max_warps) want = max_warps;
  a.nwarps = (int)want;
  const int grid = (a.nwarps + kGemvWarps - 1) / kGemvWarps;
  q4k_gemv_kernel<<<grid, kGemvWarps * 32, smem, stream>>>(a);
  return check_launch(ctx, "mlm_q4k_gemv");
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
                     ctx->gemv_counters, ctx->gemv_max_warps, ctx->gemv_max_tiles, ctx->stream);
}
