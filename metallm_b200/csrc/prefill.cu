// prefill.cu -- the per-token kernels of a batched prompt pass (T tokens at
// once): embedding rows, RMSNorm rows to bf16 (the tensor-core GEMM's
// input), RoPE of q and k with the KV-cache append, causal GQA attention
// over the cache, and the SiLU-gated product to bf16.
//
// The reference has no batched prefill: it runs forward() once per prompt
// token (LlamaRunner.swift:320-1210); these kernels are that per-token
// arithmetic for many positions at once, around mlm_q4k_gemm.
#include "mlm_device.cuh"
#include "mlm_internal.h"
#include "mlm_rope.cuh"

namespace mlm {
namespace {

// hidden[t] = float(table[tokens[t]]) (tokens clamped into the vocabulary)
__global__ void embed_rows_kernel(const __half *__restrict__ table, int vocab, int dim,
                                  const int32_t *__restrict__ tokens, float *__restrict__ out) {
  const int t = blockIdx.y;
  int tok = tokens[t];
  tok = tok < 0 ? 0 : (tok >= vocab ? vocab - 1 : tok);
  const __half *row = table + (size_t)tok * dim;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    out[(size_t)t * dim + i] = __half2float(row[i]);
}

// one row per CTA: bf16(x * rms_scale(x) * w) (NormalizationKernels.metal:31-79)
__global__ void __launch_bounds__(512) rmsnorm_rows_bf16_kernel(const float *__restrict__ x,
                                                               const float *__restrict__ w,
                                                               __nv_bfloat16 *__restrict__ y,
                                                               int n, float eps) {
  __shared__ float red[32];
  const float *xr = x + (size_t)blockIdx.x * n;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += xr[i] * xr[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float scale = rms_scale(tot, n, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    y[(size_t)blockIdx.x * n + i] = __float2bfloat16_rn((xr[i] * scale) * safe_weight(w[i]));
}

// RoPE of q and k of token t at position pos0 + t; q -> fp16 q_out, rotated
// k and v -> fp16 cache rows (rope_qk_kv_kernel for many tokens).
// qkv: fp32 [T][nq*d | nkv*d | nkv*d].
__global__ void rope_kv_rows_kernel(mlm_rope_args a, RopeConsts k, const float *__restrict__ freqs,
                                    const float *__restrict__ qkv, int nq, int nkv, int d,
                                    int pos0, __half *__restrict__ q_out, __half *__restrict__ kc,
                                    __half *__restrict__ vc) {
  const int t = blockIdx.y;
  const int pos = pos0 + t;
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
  const int t = blockIdx.y;
  const float *row = gu + (size_t)t * 2 * ffn;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < ffn; i += gridDim.x * blockDim.x)
    out[(size_t)t * ffn + i] = __float2bfloat16_rn(swiglu(row[i], row[ffn + i]));
}

// ---- causal GQA attention of T queries over the cache ----------------------
// CTA = one query head x kPfQ consecutive query tokens (8 per warp); keys in
// blocks of kPfK staged in shared memory (K rows with their 16-byte chunks
// rotated by the row index, so lanes reading different rows hit different
// banks); fp32 online softmax; lane l holds output dims 4l .. 4l+3.
constexpr int kPfQ = 32;
constexpr int kPfK = 64;
constexpr int kPfD = 128;
constexpr int kPfThreads = 128;
constexpr int kPfSmem = kPfQ * kPfD * 4 + 2 * kPfK * kPfD * 2;  // 48 KB

__global__ void __launch_bounds__(kPfThreads) attn_prefill_kernel(
    const __half *__restrict__ q16, const __half *__restrict__ kc, const __half *__restrict__ vc,
    int pos0, int T, int n_heads, int n_kv, float scale, __nv_bfloat16 *__restrict__ out) {
  extern __shared__ __align__(16) uint8_t pf_smem[];
  float *sq = reinterpret_cast<float *>(pf_smem);               // [kPfQ][128], scaled
  uint4 *sk = reinterpret_cast<uint4 *>(sq + kPfQ * kPfD);      // [kPfK][16], rotated
  uint4 *sv = sk + kPfK * 16;                                   // [kPfK][16]
  const int h = blockIdx.x, kvh = h / (n_heads / n_kv);
  const int qt0 = blockIdx.y * kPfQ;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kPfQ * kPfD; i += kPfThreads) {
    const int t = qt0 + i / kPfD;
    sq[i] = (t < T) ? __half2float(q16[((size_t)t * n_heads + h) * kPfD + (i % kPfD)]) * scale
                    : 0.f;
  }
  const int qi0 = warp * 8;
  float m[8], l[8], o[8][4];
#pragma unroll
  for (int qi = 0; qi < 8; ++qi) {
    m[qi] = -INFINITY;
    l[qi] = 0.f;
    o[qi][0] = o[qi][1] = o[qi][2] = o[qi][3] = 0.f;
  }
  const int kmax = pos0 + min(qt0 + kPfQ, T);  // keys [0, kmax) are needed
  const size_t row_stride = (size_t)n_kv * kPfD;
  for (int kbase = 0; kbase < kmax; kbase += kPfK) {
    const int rows = min(kPfK, kmax - kbase);
    __syncthreads();  // previous block fully used (and q staged on the first pass)
    for (int i = threadIdx.x; i < rows * 16; i += kPfThreads) {
      const int j = i >> 4, c = i & 15;
      const size_t g = (size_t)(kbase + j) * row_stride + kvh * kPfD + c * 8;
      sk[j * 16 + ((c + j) & 15)] = *reinterpret_cast<const uint4 *>(kc + g);
      sv[j * 16 + c] = *reinterpret_cast<const uint4 *>(vc + g);
    }
    __syncthreads();
    // scores of keys lane and lane + 32 for the warp's 8 queries
    float s[8][2];
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      const int j = lane + 32 * jj;
      float acc[8];
#pragma unroll
      for (int qi = 0; qi < 8; ++qi) acc[qi] = 0.f;
      if (j < rows) {
        for (int c = 0; c < 16; ++c) {
          const uint4 kv = sk[j * 16 + ((c + j) & 15)];
          const __half2 *kh = reinterpret_cast<const __half2 *>(&kv);
          float kf[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(kh[e]);
            kf[2 * e] = f.x;
            kf[2 * e + 1] = f.y;
          }
#pragma unroll
          for (int qi = 0; qi < 8; ++qi) {
            const float4 qa = *reinterpret_cast<const float4 *>(sq + (qi0 + qi) * kPfD + c * 8);
            const float4 qb = *reinterpret_cast<const float4 *>(sq + (qi0 + qi) * kPfD + c * 8 + 4);
            acc[qi] += qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] +
                       qb.y * kf[5] + qb.z * kf[6] + qb.w * kf[7];
          }
        }
      }
#pragma unroll
      for (int qi = 0; qi < 8; ++qi) {
        const int tq = qt0 + qi0 + qi;
        const bool ok = j < rows && tq < T && kbase + j <= pos0 + tq;
        s[qi][jj] = ok ? acc[qi] : -INFINITY;
      }
    }
    // online softmax update
#pragma unroll
    for (int qi = 0; qi < 8; ++qi) {
      const float mx = warp_max(fmaxf(s[qi][0], s[qi][1]));
      const float mnew = fmaxf(m[qi], mx);
      if (mnew == -INFINITY) {  // no visible key yet for this query
        s[qi][0] = s[qi][1] = 0.f;
        continue;
      }
      const float alpha = __expf(m[qi] - mnew);
      s[qi][0] = __expf(s[qi][0] - mnew);
      s[qi][1] = __expf(s[qi][1] - mnew);
      l[qi] = l[qi] * alpha + warp_sum(s[qi][0] + s[qi][1]);
#pragma unroll
      for (int d = 0; d < 4; ++d) o[qi][d] *= alpha;
      m[qi] = mnew;
    }
    // P . V: lane l accumulates dims 4l .. 4l+3
#pragma unroll
    for (int jj = 0; jj < 2; ++jj) {
      for (int jl = 0; jl < 32 && 32 * jj + jl < rows; ++jl) {
        const int j = 32 * jj + jl;
        const uint2 vv = *reinterpret_cast<const uint2 *>(reinterpret_cast<const __half *>(sv) +
                                                          j * kPfD + 4 * lane);
        const float2 va = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
        const float2 vb = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
#pragma unroll
        for (int qi = 0; qi < 8; ++qi) {
          const float p = __shfl_sync(0xffffffffu, s[qi][jj], jl);
          o[qi][0] += p * va.x;
          o[qi][1] += p * va.y;
          o[qi][2] += p * vb.x;
          o[qi][3] += p * vb.y;
        }
      }
    }
  }
#pragma unroll
  for (int qi = 0; qi < 8; ++qi) {
    const int tq = qt0 + qi0 + qi;
    if (tq < T) {
      const float inv = 1.0f / l[qi];
      __nv_bfloat16 *dst = out + ((size_t)tq * n_heads + h) * kPfD + 4 * lane;
      *reinterpret_cast<__nv_bfloat162 *>(dst) = __floats2bfloat162_rn(o[qi][0] * inv, o[qi][1] * inv);
      *reinterpret_cast<__nv_bfloat162 *>(dst + 2) =
          __floats2bfloat162_rn(o[qi][2] * inv, o[qi][3] * inv);
    }
  }
}

}  // namespace

int prefill_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_prefill_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem));
  return MLM_OK;
}

int embed_rows_launch(mlm_ctx *ctx, const void *table, int vocab, int dim, const int32_t *tokens,
                      int T, float *out, cudaStream_t stream) {
  embed_rows_kernel<<<dim3((dim + 255) / 256, T), 256, 0, stream>>>(
      reinterpret_cast<const __half *>(table), vocab, dim, tokens, out);
  return check_launch(ctx, "prefill (embedding)");
}

int rmsnorm_rows_bf16_launch(mlm_ctx *ctx, const float *x, const float *w, void *y, int rows,
                             int n, float eps, cudaStream_t stream) {
  rmsnorm_rows_bf16_kernel<<<rows, 512, 0, stream>>>(x, w, reinterpret_cast<__nv_bfloat16 *>(y), n,
                                                     eps);
  return check_launch(ctx, "prefill (rmsnorm)");
}

int rope_kv_rows_launch(mlm_ctx *ctx, const float *qkv, const float *freqs, const mlm_rope_args &a,
                        int nq, int nkv, int d, int pos0, int T, void *q_out, void *kc, void *vc,
                        cudaStream_t stream) {
  const RopeConsts k = rope_consts(a);
  const int total = nq * (d / 2) + 2 * nkv * (d / 2);
  rope_kv_rows_kernel<<<dim3((total + 255) / 256, T), 256, 0, stream>>>(
      a, k, freqs, qkv, nq, nkv, d, pos0, reinterpret_cast<__half *>(q_out),
      reinterpret_cast<__half *>(kc), reinterpret_cast<__half *>(vc));
  return check_launch(ctx, "prefill (rope)");
}

int attn_prefill_launch(mlm_ctx *ctx, const void *q16, const void *kc, const void *vc, int pos0,
                        int T, int n_heads, int n_kv, int head_dim, void *out, cudaStream_t stream) {
  MLM_REQUIRE(ctx, head_dim == kPfD && n_kv > 0 && n_heads % n_kv == 0, MLM_ERR_UNSUPPORTED,
              "prefill attention: head_dim=%d heads=%d/%d", head_dim, n_heads, n_kv);
  attn_prefill_kernel<<<dim3(n_heads, (T + kPfQ - 1) / kPfQ), kPfThreads, kPfSmem, stream>>>(
      reinterpret_cast<const __half *>(q16), reinterpret_cast<const __half *>(kc),
      reinterpret_cast<const __half *>(vc), pos0, T, n_heads, n_kv, 1.0f / sqrtf((float)head_dim),
      reinterpret_cast<__nv_bfloat16 *>(out));
  return check_launch(ctx, "prefill (attention)");
}

int swiglu_rows_bf16_launch(mlm_ctx *ctx, const float *gu, int ffn, int T, void *out,
                            cudaStream_t stream) {
  swiglu_rows_bf16_kernel<<<dim3((ffn + 255) / 256, T), 256, 0, stream>>>(
      gu, ffn, reinterpret_cast<__nv_bfloat16 *>(out));
  return check_launch(ctx, "prefill (swiglu)");
}

}  // namespace mlm
