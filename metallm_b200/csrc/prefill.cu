// prefill.cu -- the per-token kernels of a batched prompt pass (T tokens at
// once): embedding rows, RMSNorm rows to bf16 (the tensor-core GEMM's
// input), RoPE of q and k with the KV-cache append, causal GQA attention
// over the cache, and the SiLU-gated product to bf16.
//
// The reference has no batched prefill: it runs forward() once per prompt
// token (LlamaRunner.swift:320-1210); these kernels are that per-token
// arithmetic for many positions at once, around mlm_q4k_gemm.
#include <algorithm>

#include "mlm_device.cuh"
#include "mlm_internal.h"
#include "mlm_rope.cuh"

namespace mlm {
namespace {

// hidden[t] = float(table[tokens[t]]) (tokens clamped into the vocabulary)
__global__ void embed_rows_kernel(const __half *__restrict__ table, int vocab, int dim,
                                  const int32_t *__restrict__ tokens, float *__restrict__ out) {
  pdl_wait_then_release();
  const int t = blockIdx.y;
  int tok = tokens[t];
  tok = tok < 0 ? 0 : (tok >= vocab ? vocab - 1 : tok);
  const __half *row = table + (size_t)tok * dim;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    out[(size_t)t * dim + i] = __half2float(row[i]);
}

// one row per CTA: bf16(x * rms_scale(x) * w) (NormalizationKernels.metal:31-79).
// The row is read once: each thread keeps its float4 pieces in registers
// across the reduction (rows of up to 512 x 4 x kRmsPer elements).  When
// zero is set the CTAs also clear zero[0 .. zero_n) (the output of the
// accumulating GEMV that consumes these rows).
constexpr int kRmsThreads = 512;
constexpr int kRmsPer = 8;  // float4 pieces per thread: rows up to 16384
__global__ void __launch_bounds__(kRmsThreads) rmsnorm_rows_bf16_kernel(
    const float *__restrict__ x, const float *__restrict__ w, __nv_bfloat16 *__restrict__ y, int n,
    float eps, float *__restrict__ zero, size_t zero_n, int rows) {
  __shared__ float red[kRmsThreads / 32];
  pdl_wait_then_release();
  if (zero) {
    float4 *z4 = reinterpret_cast<float4 *>(zero);
    const size_t n4 = zero_n / 4;
    for (size_t i = (size_t)blockIdx.x * kRmsThreads + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * kRmsThreads)
      z4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if ((int)blockIdx.x >= rows) return;  // CTAs beyond the rows only clear
  const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)blockIdx.x * n);
  const float4 *w4 = reinterpret_cast<const float4 *>(w);
  const int n4 = n / 4;
  float4 v[kRmsPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRmsPer; ++k) {
    const int i = threadIdx.x + k * kRmsThreads;
    v[k] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int k = 0; k < kRmsPer; ++k)
    ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kRmsThreads / 32; ++i) tot += red[i];
  const float scale = rms_scale(tot, n, eps);
  uint2 *yr = reinterpret_cast<uint2 *>(y + (size_t)blockIdx.x * n);
#pragma unroll
  for (int k = 0; k < kRmsPer; ++k) {
    const int i = threadIdx.x + k * kRmsThreads;
    if (i < n4) {
      const float4 ww = __ldg(w4 + i);
      const __nv_bfloat162 lo = __floats2bfloat162_rn((v[k].x * scale) * safe_weight(ww.x),
                                                      (v[k].y * scale) * safe_weight(ww.y));
      const __nv_bfloat162 hi = __floats2bfloat162_rn((v[k].z * scale) * safe_weight(ww.z),
                                                      (v[k].w * scale) * safe_weight(ww.w));
      yr[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&lo),
                         *reinterpret_cast<const uint32_t *>(&hi));
    }
  }
}

// RoPE of q and k of token t at position pos0 + t; q -> fp16 q_out, rotated
// k and v -> fp16 cache rows (rope_qk_kv_kernel for many tokens).
// qkv: fp32 [T][nq*d | nkv*d | nkv*d].  With pos_dev (a batch of sequences,
// one token each): token t is at position pos_dev[t] of sequence t, whose
// caches start kv_bs elements after sequence t-1's.
__global__ void rope_kv_rows_kernel(mlm_rope_args a, RopeConsts k, const float *__restrict__ freqs,
                                    const float *__restrict__ qkv, int nq, int nkv, int d,
                                    int pos0, __half *__restrict__ q_out, __half *__restrict__ kc,
                                    __half *__restrict__ vc, const int *__restrict__ pos_dev,
                                    size_t kv_bs) {
  pdl_wait_then_release();
  const int t = blockIdx.y;
  const int pos = pos_dev ? pos_dev[t] : pos0 + t;
  if (pos_dev) {
    kc += t * kv_bs;
    vc += t * kv_bs;
  }
  const int pairs = d / 2;
  const int nqp = nq * pairs, nkp = nkv * pairs;
  const float *row = qkv + (size_t)t * (nq + 2 * nkv) * d;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nqp + nkp) {
    const bool is_q = i < nqp;
    const int j = is_q ? i : i - nqp;
    const int h = j / pairs, pp = j - h * pairs;
    const float *src = row + (is_q ? 0 : nq * d) + (size_t)h * d + 2 * pp;
    float x0 = src[0], x1 = src[1];
    if (2 * pp < (int)a.n_dims) {
      float c, s;
      rope_cos_sin(a, k, freqs, pos, pp, c, s);
      const float r0 = x0 * c - x1 * s;
      const float r1 = x0 * s + x1 * c;
      x0 = r0;
      x1 = r1;
    }
    const __half2 o = __floats2half2_rn(x0, x1);
    if (is_q)
      *reinterpret_cast<__half2 *>(q_out + ((size_t)t * nq + h) * d + 2 * pp) = o;
    else
      *reinterpret_cast<__half2 *>(kc + ((size_t)pos * nkv + h) * d + 2 * pp) = o;
  } else if (i < nqp + 2 * nkp) {
    const int j = i - nqp - nkp;
    const int h = j / pairs, pp = j - h * pairs;
    const float *src = row + (size_t)(nq + nkv) * d + (size_t)h * d + 2 * pp;
    *reinterpret_cast<__half2 *>(vc + ((size_t)pos * nkv + h) * d + 2 * pp) =
        __floats2half2_rn(src[0], src[1]);
  }
}

// out[t][i] = bf16(silu(gu[t][i]) * gu[t][ffn + i])
__global__ void swiglu_rows_bf16_kernel(const float *__restrict__ gu, int ffn,
                                        __nv_bfloat16 *__restrict__ out) {
  pdl_wait_then_release();
  const int t = blockIdx.y;
  const float *row = gu + (size_t)t * 2 * ffn;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ffn; i += gridDim.x * blockDim.x)
    out[(size_t)t * ffn + i] = __float2bfloat16_rn(swiglu(row[i], row[ffn + i]));
}

// ---- causal GQA attention of T queries over the cache ----------------------
// Flash attention on the tensor cores (mma.sync m16n8k16, fp16 in, fp32
// accumulate).  CTA = one query head x 64 consecutive query tokens, warp =
// 16 of them, their Q fragments held in registers for the whole key loop.
// Keys in blocks of 64 staged in shared memory: K rows as stored (padded to
// 272 bytes, so the 8 rows a fragment load touches fall in distinct banks)
// and V transposed (dims as rows, padded to 144 bytes), so both MMA operands
// are single 32-bit loads.  Per block: S = Q K^T (64 MMAs per warp), the
// causal mask (key position > query position), the online softmax in base 2
// with the 1/sqrt(128) scale folded in, then O += P V (64 MMAs) with P taken
// straight from the S accumulators as fp16 A fragments.  The reference runs
// the same softmax(q k^T / sqrt(d)) v per token with MPS (LlamaRunner.swift:
// 669-952); GQA head h reads KV head h / (n_heads / n_kv)
// (AttentionKernels.metal:43).
constexpr int kFaQ = 64;                // queries per CTA (16 per warp)
constexpr int kFaK = 64;                // keys per block
constexpr int kFaD = 128;               // head dim
constexpr int kFaThreads = 128;
constexpr int kKs = kFaD + 8;           // K row stride in halves (272 bytes)
constexpr int kVs = kFaK + 8;           // transposed V row stride in halves (144 bytes)

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

__global__ void __launch_bounds__(kFaThreads) attn_prefill_kernel(
    const __half *__restrict__ q16, const __half *__restrict__ kc, const __half *__restrict__ vc,
    int pos0, int T, int n_heads, int n_kv, float scale_log2, __nv_bfloat16 *__restrict__ out) {
  __shared__ __align__(16) __half ks[kFaK * kKs];
  __shared__ __align__(16) __half vt[kFaD * kVs];
  const int h = blockIdx.x, kvh = h / (n_heads / n_kv);
  const int qb = blockIdx.y * kFaQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = qb + warp * 16;  // first query token of the warp
  const int r0 = q0 + g, r1 = q0 + g + 8;

  // Q fragments (rows g, g+8; dims 16 ks + 2t, +1 and + 8)
  uint32_t qa[8][4];
  {
    const __half *qr0 = q16 + ((size_t)min(r0, T - 1) * n_heads + h) * kFaD;
    const __half *qr1 = q16 + ((size_t)min(r1, T - 1) * n_heads + h) * kFaD;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      qa[k][0] = r0 < T ? *reinterpret_cast<const uint32_t *>(qr0 + 16 * k + 2 * t) : 0u;
      qa[k][1] = r1 < T ? *reinterpret_cast<const uint32_t *>(qr1 + 16 * k + 2 * t) : 0u;
      qa[k][2] = r0 < T ? *reinterpret_cast<const uint32_t *>(qr0 + 16 * k + 8 + 2 * t) : 0u;
      qa[k][3] = r1 < T ? *reinterpret_cast<const uint32_t *>(qr1 + 16 * k + 8 + 2 * t) : 0u;
    }
  }
  const int qp0 = pos0 + r0, qp1 = pos0 + r1;  // query positions
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;

  // keys 0 .. kend-1: up to the CTA's last query position
  const int kend = pos0 + min(qb + kFaQ, T);
  for (int kb = 0; kb < kend; kb += kFaK) {
    __syncthreads();  // the previous block is no longer read
    for (int i = threadIdx.x; i < kFaK * 16; i += kFaThreads) {
      const int key = i % kFaK, chunk = i / kFaK;  // consecutive keys per warp
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (kb + key < kend) {
        const size_t off = ((size_t)(kb + key) * n_kv + kvh) * kFaD + chunk * 8;
        kv = *reinterpret_cast<const uint4 *>(kc + off);
        vv = *reinterpret_cast<const uint4 *>(vc + off);
      }
      *reinterpret_cast<uint4 *>(ks + key * kKs + chunk * 8) = kv;
      const __half *ve = reinterpret_cast<const __half *>(&vv);
#pragma unroll
      for (int e = 0; e < 8; ++e) vt[(chunk * 8 + e) * kVs + key] = ve[e];
    }
    __syncthreads();

    // S = Q K^T: 16 queries x 64 keys per warp
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
      const __half *kr = ks + (8 * j + g) * kKs + 2 * t;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(kr + 16 * k);
        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(kr + 16 * k + 8);
        mma_16816(sc[j], qa[k], b0, b1);
      }
    }
    // mask, scale (base 2), row maxima
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int kp = kb + 8 * j + 2 * t + (c & 1);
        const int qp = (c < 2) ? qp0 : qp1;
        const float v = (kp <= qp && kp < kend) ? sc[j][c] * scale_log2 : -INFINITY;
        sc[j][c] = v;
        mx[c >> 1] = fmaxf(mx[c >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
      const float mn = fmaxf(m[rr], mx[rr]);
      corr[rr] = (mn == -INFINITY) ? 1.f : exp2f(m[rr] - mn);
      m[rr] = mn;
      l[rr] *= corr[rr];
    }
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      o[d][0] *= corr[0];
      o[d][1] *= corr[0];
      o[d][2] *= corr[1];
      o[d][3] *= corr[1];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float mm = m[c >> 1];
        const float p = (sc[j][c] == -INFINITY) ? 0.f : exp2f(sc[j][c] - mm);
        sc[j][c] = p;
        l[c >> 1] += p;
      }
    }
    // O += P V: P from the S accumulators (keys 16 kk .. 16 kk + 15)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa[4] = {pack_half2(sc[2 * kk][0], sc[2 * kk][1]),
                              pack_half2(sc[2 * kk][2], sc[2 * kk][3]),
                              pack_half2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]),
                              pack_half2(sc[2 * kk + 1][2], sc[2 * kk + 1][3])};
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        const __half *vr = vt + (8 * d + g) * kVs + 16 * kk + 2 * t;
        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(vr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(vr + 8);
        mma_16816(o[d], pa, b0, b1);
      }
    }
  }
  // normalise and store (bf16, the output projection's GEMM input)
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
    l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
  }
  const float inv0 = 1.f / l[0], inv1 = 1.f / l[1];
#pragma unroll
  for (int d = 0; d < 16; ++d) {
    const int col = h * kFaD + 8 * d + 2 * t;
    if (r0 < T)
      *reinterpret_cast<__nv_bfloat162 *>(out + (size_t)r0 * n_heads * kFaD + col) =
          __floats2bfloat162_rn(o[d][0] * inv0, o[d][1] * inv0);
    if (r1 < T)
      *reinterpret_cast<__nv_bfloat162 *>(out + (size_t)r1 * n_heads * kFaD + col) =
          __floats2bfloat162_rn(o[d][2] * inv1, o[d][3] * inv1);
  }
}

}  // namespace

int prefill_init(mlm_ctx *ctx) {
  return MLM_OK;
}

int embed_rows_launch(mlm_ctx *ctx, const void *table, int vocab, int dim, const int32_t *tokens,
                      int T, float *out, cudaStream_t stream) {
  return check_launch_pdl(
      ctx,
      launch_pdl(embed_rows_kernel, dim3((dim + 255) / 256, T), dim3(256), 0, stream,
                 reinterpret_cast<const __half *>(table), vocab, dim, tokens, out),
      "prefill (embedding)");
}

int rmsnorm_rows_bf16_launch(mlm_ctx *ctx, const float *x, const float *w, void *y, int rows,
                             int n, float eps, cudaStream_t stream, float *zero, size_t zero_n) {
  MLM_REQUIRE(ctx, n % 4 == 0 && n <= 4 * kRmsThreads * kRmsPer && zero_n % 4 == 0,
              MLM_ERR_SHAPE, "rmsnorm rows: n=%d", n);
  // a few rows clearing a large output get extra CTAs for the clearing
  const size_t zero_ctas = zero ? std::min<size_t>(148, (zero_n / 4 + 4095) / 4096) : 0;
  const int grid = (int)std::max<size_t>(rows, zero_ctas);
  return check_launch_pdl(
      ctx,
      launch_pdl(rmsnorm_rows_bf16_kernel, dim3(grid), dim3(kRmsThreads), 0, stream, x, w,
                 reinterpret_cast<__nv_bfloat16 *>(y), n, eps, zero, zero_n, rows),
      "prefill (rmsnorm)");
}

int rope_kv_rows_launch(mlm_ctx *ctx, const float *qkv, const float *freqs, const mlm_rope_args &a,
                        int nq, int nkv, int d, int pos0, int T, void *q_out, void *kc, void *vc,
                        cudaStream_t stream) {
  const RopeConsts k = rope_consts(a);
  const int total = nq * (d / 2) + 2 * nkv * (d / 2);
  rope_kv_rows_kernel<<<dim3((total + 255) / 256, T), 256, 0, stream>>>(
      a, k, freqs, qkv, nq, nkv, d, pos0, reinterpret_cast<__half *>(q_out),
      reinterpret_cast<__half *>(kc), reinterpret_cast<__half *>(vc), nullptr, 0);
  return check_launch(ctx, "prefill (rope)");
}

int attn_prefill_launch(mlm_ctx *ctx, const void *q16, const void *kc, const void *vc, int pos0,
                        int T, int n_heads, int n_kv, int head_dim, void *out, cudaStream_t stream) {
  MLM_REQUIRE(ctx, head_dim == kFaD && n_kv > 0 && n_heads % n_kv == 0, MLM_ERR_UNSUPPORTED,
              "prefill attention: head_dim=%d heads=%d/%d", head_dim, n_heads, n_kv);
  // log2(e) / sqrt(head_dim): the softmax runs in base 2
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  attn_prefill_kernel<<<dim3(n_heads, (T + kFaQ - 1) / kFaQ), kFaThreads, 0, stream>>>(
      reinterpret_cast<const __half *>(q16), reinterpret_cast<const __half *>(kc),
      reinterpret_cast<const __half *>(vc), pos0, T, n_heads, n_kv, scale_log2,
      reinterpret_cast<__nv_bfloat16 *>(out));
  return check_launch(ctx, "prefill (attention)");
}

int swiglu_rows_bf16_launch(mlm_ctx *ctx, const float *gu, int ffn, int T, void *out,
                            cudaStream_t stream) {
  return check_launch_pdl(ctx,
                          launch_pdl(swiglu_rows_bf16_kernel, dim3((ffn + 255) / 256, T), dim3(256),
                                     0, stream, gu, ffn, reinterpret_cast<__nv_bfloat16 *>(out)),
                          "prefill (swiglu)");
}

// out[t] = (a[t] | b[t]): two row-major blocks of T rows, ra and rb floats
// wide, side by side (the q/k rows of a Q4_K QKV matrix beside the v rows of
// a Q6_K one)
__global__ void interleave_rows_kernel(const float *__restrict__ a, int ra,
                                       const float *__restrict__ b, int rb, int T,
                                       float *__restrict__ out) {
  const size_t W = (size_t)ra + rb, n = (size_t)T * W;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / W, c = i - t * W;
    out[i] = c < (size_t)ra ? a[t * ra + c] : b[t * rb + (c - ra)];
  }
}

int interleave_rows_launch(mlm_ctx *ctx, const float *a, int ra, const float *b, int rb, int T,
                           float *out, cudaStream_t stream) {
  const size_t n = (size_t)T * (ra + rb);
  const unsigned grid = (unsigned)std::min<size_t>((n + 255) / 256, (size_t)ctx->sm_count * 8);
  interleave_rows_kernel<<<grid, 256, 0, stream>>>(a, ra, b, rb, T, out);
  return check_launch(ctx, "interleave rows");
}

}  // namespace mlm
