// q4k_gemm.cu -- prefill Q4_K GEMM on the 5th-generation tensor cores:
// Y[t][n] = sum_k X[t][k] * W[n][k] for T tokens at once.
//
// Replaces the prefill linears of the reference (encodeMPSMatrixMultiply on
// weights dequantized to fp16 at load, MetalService.swift:797-925; the
// reference has no batched prefill, it runs forward() token by token,
// LlamaRunner.swift:320).  W stays packed Q4_K in HBM (GGUF layout); each CTA
// dequantizes its weight tile to bf16 in shared memory and feeds
// tcgen05.mma with fp32 accumulators in tensor memory.
//
// CTA tile: 128 weight rows (the MMA's M) x 512 tokens (two MMAs of N = 256)
// with the fp32 accumulator filling all 512 TMEM columns, so a weight tile is
// dequantized once per 512 tokens.  K advances 64 elements (one 128-byte
// bf16 row of a 128-byte swizzle atom) per pipeline stage, two stages.
// Warp roles (192 threads):
//   warp 0     TMA: packed W block columns (128 rows x 144 bytes, 2 buffers)
//              and the bf16 X tile of each stage (512 tokens x 64, 128-byte
//              swizzle -- the canonical K-major layout tcgen05 reads);
//   warp 1     allocates TMEM; one thread issues the MMAs and commits;
//   warps 2-5  dequantize (thread = weight row; 64 values per stage:
//              (d*sc)*q - dmin*m in fp32 rounded to bf16, written in the
//              same swizzled layout), then run the epilogue: tcgen05.ld
//              of their 32-lane quarter of the accumulator, stores to Y.
// Stages are tracked by mbarriers (full: TMA bytes / dequant warps, empty:
// the MMA commit); every wait is bounded and reports a device error.  K may
// be split across CTAs (grid z) for narrow weights, the parts then added with
// fp32 atomics into a Y that starts from the residual (or zero).
#include <cuda.h>

#include <algorithm>

#include "mlm_internal.h"
#include "q4k_gemv_common.cuh"

namespace mlm {
namespace {

constexpr int kGemmRows = 128;   // weight rows per tile (MMA M)
constexpr int kGemmTok = 512;    // tokens per tile (two MMAs of N = 256)
constexpr int kGemmKStep = 64;   // K per stage
constexpr int kGemmStages = 2;
constexpr int kGemmThreads = 192;
constexpr int kAStage = kGemmRows * kGemmKStep * 2;  // 16 KB
constexpr int kBStage = kGemmTok * kGemmKStep * 2;   // 64 KB
constexpr int kBHalf = kBStage / 2;                  // 256 tokens
constexpr int kWpk = kGemmRows * kBlockBytes;        // 18 KB
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kGemmStages * kAStage;
constexpr int kOffW = kOffB + kGemmStages * kBStage;
constexpr int kOffBar = kOffW + 2 * kWpk;
// mbarriers: wfull[2] wempty[2] bfull[2] afull[2] sempty[2] done, then the
// TMEM base address
constexpr int kNumBars = 11;
constexpr int kGemmSmem = kOffBar + kNumBars * 8 + 8;
constexpr int kTmemCols = 512;

// tcgen05 instruction descriptor: fp32 accumulate, bf16 A and B, both
// K-major, N = 256, M = 128
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) |
                            ((128u >> 4) << 24);

// shared-memory matrix descriptor of a K-major bf16 tile in the 128-byte
// swizzle layout: 8-row atoms of 1024 bytes (stride 1024), descriptor
// version 1
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46) | (2ull << 61);
}

struct GemmArgs {
  float *y;      // [T][N] fp32
  const float *residual;  // [T][N] or NULL (the atomic path starts y from it)
  int *status;   // device-visible error word
  int N, K, T;
  int kb_per_split;  // Q4_K block columns per split
  int atomic;        // splits > 1: add into y
};

__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap *map, int x, int y,
                                      uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    q4k_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_x, GemmArgs p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t bar = sbase + kOffBar;
  const uint32_t wfull = bar, wempty = bar + 16, bfull = bar + 32, afull = bar + 48,
                 sempty = bar + 64, done = bar + 80;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + kNumBars * 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kGemmRows;
  const int t0 = blockIdx.y * kGemmTok;
  const int nb = p.K / kQK;
  const int kb0 = blockIdx.z * p.kb_per_split;
  const int kb1 = min(nb, kb0 + p.kb_per_split);
  const int KS = (kb1 - kb0) * (kQK / kGemmKStep);  // stages of 64

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(wfull + 8 * i, 1);
      mbar_init(wempty + 8 * i, 4);
      mbar_init(bfull + 8 * i, 1);
      mbar_init(afull + 8 * i, 4);
      mbar_init(sempty + 8 * i, 1);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // the whole warp allocates the accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- TMA producer --------------------------------------------------------
    if (lane == 0 && KS > 0) {
      int wj = 0;  // W block columns issued
      int issued_k = 0;
      bool ok = true;
      for (int kk = 0; kk < KS && ok; ++kk) {
        const int s = kk & 1;
        if ((kk & 3) == 0) {
          const int j = kk >> 2, wb = j & 1;
          if (j >= 2 && !mbar_wait_bounded(wempty + 8 * wb, ((j >> 1) - 1) & 1, p.status)) {
            ok = false;
            break;
          }
          mbar_expect_tx(wfull + 8 * wb, kWpk);
          tma2d(sbase + kOffW + wb * kWpk, &tmap_w, (kb0 + j) * kBlockBytes, n0, wfull + 8 * wb);
          wj = j + 1;
        }
        if (kk >= 2 && !mbar_wait_bounded(sempty + 8 * s, ((kk >> 1) - 1) & 1, p.status)) {
          ok = false;
          break;
        }
        mbar_expect_tx(bfull + 8 * s, kBStage);
        const int kx = kb0 * kQK + kk * kGemmKStep;
        tma2d(sbase + kOffB + s * kBStage, &tmap_x, kx, t0, bfull + 8 * s);
        tma2d(sbase + kOffB + s * kBStage + kBHalf, &tmap_x, kx, t0 + kGemmTok / 2, bfull + 8 * s);
        issued_k = kk + 1;
      }
      // copies in flight land before shared memory is released
      for (int kk = max(0, issued_k - 2); kk < issued_k; ++kk)
        if (!mbar_wait_bounded(bfull + 8 * (kk & 1), (kk >> 1) & 1, p.status)) break;
      for (int j = max(0, wj - 2); j < wj; ++j)
        if (!mbar_wait_bounded(wfull + 8 * (j & 1), (j >> 1) & 1, p.status)) break;
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------
    if (lane == 0 && KS > 0) {
      for (int kk = 0; kk < KS; ++kk) {
        const int s = kk & 1;
        const uint32_t ph = (kk >> 1) & 1;
        if (!mbar_wait_bounded(afull + 8 * s, ph, p.status)) break;
        if (!mbar_wait_bounded(bfull + 8 * s, ph, p.status)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_addr = sbase + kOffA + s * kAStage;
        const uint32_t b_addr = sbase + kOffB + s * kBStage;
#pragma unroll
        for (int k16 = 0; k16 < kGemmKStep / 16; ++k16) {
          const uint64_t adesc = sw128_desc(a_addr + 32 * k16);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint64_t bdesc = sw128_desc(b_addr + half * kBHalf + 32 * k16);
            const uint32_t acc = (kk > 0 || k16 > 0) ? 1u : 0u;
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(
                    tmem + half * 256),
                "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(acc)
                : "memory");
          }
        }
        // stage s is free once these MMAs have read it
        asm volatile(
            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                sempty + 8 * s)
            : "memory");
      }
      asm volatile(
          "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(done)
          : "memory");
    }
  } else {
    // ---- dequantize (thread = weight row), then the epilogue ------------------
    const int r = threadIdx.x - 64;  // 0..127
    bool ok = true;
    for (int kk = 0; kk < KS; ++kk) {
      const int s = kk & 1, j = kk >> 2, s4 = kk & 3, wb = j & 1;
      if (ok && s4 == 0) ok = mbar_wait_bounded(wfull + 8 * wb, (j >> 1) & 1, p.status);
      if (ok && kk >= 2) ok = mbar_wait_bounded(sempty + 8 * s, ((kk >> 1) - 1) & 1, p.status);
      if (ok) {
        const uint8_t *blk = smem + kOffW + wb * kWpk + r * kBlockBytes;
        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
        const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
        int sc0, m0, sc1, m1;
        q4k_scale_min_regs(2 * s4, h.y, h.z, h.w, sc0, m0);
        q4k_scale_min_regs(2 * s4 + 1, h.y, h.z, h.w, sc1, m1);
        const float fs0 = d * (float)sc0, fm0 = dmin * (float)m0;  // exact
        const float fs1 = d * (float)sc1, fm1 = dmin * (float)m1;
        const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * s4);
        const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * s4);
        const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        uint8_t *arow = smem + kOffA + s * kAStage + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // elements 8c .. 8c+7 = qs word c
          const uint32_t w = qw[c];
          const float fs = (c < 4) ? fs0 : fs1, fm = (c < 4) ? fm0 : fm1;
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {  // byte e: elements 2e (low), 2e+1 (high)
            const uint32_t byte = (w >> (8 * e)) & 0xFFu;
            const float lo = __fsub_rn(__fmul_rn(fs, (float)(byte & 0xF)), fm);
            const float hi = __fsub_rn(__fmul_rn(fs, (float)(byte >> 4)), fm);
            const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
            o[e] = *reinterpret_cast<const uint32_t *>(&v);
          }
          *reinterpret_cast<uint4 *>(arow + ((c ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        // generic-proxy writes become visible to the tensor cores' reads
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive1(afull + 8 * s);
        if (s4 == 3 || kk == KS - 1) mbar_arrive1(wempty + 8 * wb);
      }
    }
    // epilogue: this warp's 32-lane quarter of the accumulator
    if (KS > 0 && mbar_wait_bounded(done, 0, p.status)) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int quarter = warp & 3;
      const int n = n0 + quarter * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
      for (int col = 0; col < kGemmTok; col += 8) {
        uint32_t v[8];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
              "=r"(v[7])
            : "r"(taddr + col));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (n < p.N) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int t = t0 + col + i;
            if (t < p.T) {
              float *dst = p.y + (size_t)t * p.N + n;
              if (p.atomic)
                atomicAdd(dst, __uint_as_float(v[i]));
              else
                *dst = __uint_as_float(v[i]) + (p.residual ? p.residual[(size_t)t * p.N + n] : 0.f);
            }
          }
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                              const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                              const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn tensor_map_encoder(mlm_ctx *ctx) {
  static EncodeFn encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      set_error(ctx, MLM_ERR_CUDA, "mlm_q4k_gemm: cuTensorMapEncodeTiled unavailable");
      return nullptr;
    }
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  return encode;
}

}  // namespace

int gemm_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q4k_gemm_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
  return MLM_OK;
}

}  // namespace mlm

using namespace mlm;

namespace mlm {
int gemm_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16, int tokens,
                float *y, const float *residual, cudaStream_t stream) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, W && x_bf16 && y, MLM_ERR_ARG, "mlm_q4k_gemm: null buffer");
  MLM_REQUIRE(ctx, rows > 0 && cols > 0 && tokens > 0 && cols % kQK == 0, MLM_ERR_SHAPE,
              "mlm_q4k_gemm: rows=%d cols=%d tokens=%d (cols a multiple of 256)", rows, cols,
              tokens);
  MLM_REQUIRE(ctx, aligned16(W) && aligned16(x_bf16), MLM_ERR_ALIGN,
              "mlm_q4k_gemm: W and X must be 16-byte aligned");
  MLM_REQUIRE(ctx, kGemmSmem <= ctx->max_smem_optin, MLM_ERR_UNSUPPORTED,
              "mlm_q4k_gemm: needs %d bytes of shared memory", kGemmSmem);
  EncodeFn encode = tensor_map_encoder(ctx);
  if (!encode) return MLM_ERR_CUDA;
  const int nb = cols / kQK;
  CUtensorMap mw, mx;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)nb * kBlockBytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)nb * kBlockBytes};
    const cuuint32_t box[2] = {(cuuint32_t)kBlockBytes, (cuuint32_t)kGemmRows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(W), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MLM_REQUIRE(ctx, r == CUDA_SUCCESS, MLM_ERR_CUDA, "mlm_q4k_gemm: W tensor map (%d)", (int)r);
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)tokens};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kGemmKStep, (cuuint32_t)(kGemmTok / 2)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x_bf16),
                        dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MLM_REQUIRE(ctx, r == CUDA_SUCCESS, MLM_ERR_CUDA, "mlm_q4k_gemm: X tensor map (%d)", (int)r);
  }
  // split K so that narrow weights still fill the SMs
  const int tiles = ((rows + kGemmRows - 1) / kGemmRows) * ((tokens + kGemmTok - 1) / kGemmTok);
  int splits = 1;
  while (splits < 8 && tiles * splits * 2 <= ctx->sm_count && nb % (splits * 2) == 0) splits *= 2;
  GemmArgs a;
  a.y = y;
  a.residual = residual;
  a.status = ctx->dev_status;
  a.N = rows;
  a.K = cols;
  a.T = tokens;
  a.kb_per_split = nb / splits;
  a.atomic = splits > 1;
  if (splits > 1) {  // the parts are added into y, which starts from the residual or zero
    const size_t bytes = sizeof(float) * (size_t)rows * tokens;
    if (residual) {
      if (residual != y)
        MLM_CUDA_TRY(ctx, cudaMemcpyAsync(y, residual, bytes, cudaMemcpyDeviceToDevice, stream));
    } else {
      MLM_CUDA_TRY(ctx, cudaMemsetAsync(y, 0, bytes, stream));
    }
  }
  dim3 grid((rows + kGemmRows - 1) / kGemmRows, (tokens + kGemmTok - 1) / kGemmTok, splits);
  q4k_gemm_kernel<<<grid, kGemmThreads, kGemmSmem, stream>>>(mw, mx, a);
  return check_launch(ctx, "mlm_q4k_gemm");
}
}  // namespace mlm

extern "C" int mlm_q4k_gemm(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                            int tokens, float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, !residual || aligned4(residual), MLM_ERR_ALIGN, "mlm_q4k_gemm: residual");
  return gemm_launch(ctx, W, rows, cols, x_bf16, tokens, y, residual, ctx->stream);
}
