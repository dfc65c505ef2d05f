// attention.cu -- GQA decode attention over an fp16 KV cache, split along the
// sequence ("flash-decoding"), plus embedding gather and device argmax.
//
// The reference computes one decode step's attention with a repeat-KV copy
// (AttentionKernels.metal:16-59), 32 per-head MPS GEMMs for q.K^T scaled by
// 1/sqrt(d), an MPS row softmax and 32 more GEMMs for P.V
// (LlamaRunner.swift:669-952).  Here one CTA owns one KV head and one chunk
// of positions and serves all n_heads/n_kv_heads query heads of that KV head,
// so each K and V row is read from HBM exactly once.  Softmax is fp32 with a
// running max; each CTA writes (max, sum, unnormalised output) for its chunk.
// The last CTA of a KV head to finish merges the chunks (mlm_attn_decode).
// The runner's decode steps, one sequence or a batch, use the fused kernel
// further down: RoPE and the KV append folded in, both products on the
// tensor cores, chunks merged through distributed shared memory.
#include <algorithm>

#include "mlm_device.cuh"
#include "mlm_internal.h"
#include "mlm_rope.cuh"

namespace mlm {

constexpr int kAttnD = 128;       // head_dim handled by this kernel
constexpr int kAttnChunk = 64;    // positions per CTA (upper bound)
constexpr int kAttnMaxChunks = 64;
constexpr int kAttnMaxArrivals = 8192;  // (sequence, KV head) pairs of one launch
constexpr int kAttnThreads = 128;

// partial layout per (chunk, head): [m, l, o[128]]
constexpr int kAttnPartial = 2 + kAttnD;
// K and V rows of one chunk staged in shared memory (dynamic)
constexpr int kAttnStageBytes = 2 * (2 * kAttnChunk) * kAttnD * (int)sizeof(__half);

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <int G, class OutT>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_partial_kernel(
    const __half *__restrict__ q, const __half *__restrict__ kc, const __half *__restrict__ vc,
    int n_heads, int n_kv, int seq_len, int chunk_len, float scale,
    float *__restrict__ partials, const int *__restrict__ pos_dev, size_t q_bs, size_t kv_bs,
    size_t part_bs, OutT *__restrict__ out, size_t out_bs, int *__restrict__ arrivals) {
  __shared__ float s_scores[G][kAttnChunk * 2];
  __shared__ float s_out[kAttnThreads / 32][G][kAttnD];
  pdl_wait_then_release();
  const int kvh = blockIdx.x;
  const int chunk = blockIdx.y;
  const int p0 = chunk * chunk_len;
  // sequence blockIdx.z of a batch: its query, cache and scratch
  const int bz = blockIdx.z;
  q += bz * q_bs;
  kc += bz * kv_bs;
  vc += bz * kv_bs;
  partials += bz * part_bs;
  // graph-replayed decode: the position lives in device memory and the grid
  // covers the cache's capacity; chunks past the sequence do nothing
  if (pos_dev) seq_len = pos_dev[bz] + 1;
  if (p0 >= seq_len) return;
  const int p1 = min(seq_len, p0 + chunk_len);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarp = kAttnThreads / 32;
  const size_t row_stride = (size_t)n_kv * kAttnD;

  // Stage the chunk's K rows, then its V rows, into shared memory: every
  // 16-byte piece is requested up front (~64 KB in flight per CTA), so the
  // loops below never wait on HBM one position at a time.
  extern __shared__ __align__(16) __half s_kv[];  // [2][2 * kAttnChunk][kAttnD]
  __half *s_k = s_kv, *s_v = s_kv + 2 * kAttnChunk * kAttnD;
  {
    constexpr int kPiecesPerRow = kAttnD * (int)sizeof(__half) / 16;  // 16
    const int pieces = (p1 - p0) * kPiecesPerRow;
    const uint32_t sk = (uint32_t)__cvta_generic_to_shared(s_k);
    const uint32_t sv = (uint32_t)__cvta_generic_to_shared(s_v);
    for (int j = threadIdx.x; j < pieces; j += kAttnThreads) {
      const int r = j / kPiecesPerRow, c = j - r * kPiecesPerRow;
      cp_async16(sk + (uint32_t)(r * kAttnD + c * 8) * 2,
                 kc + (size_t)(p0 + r) * row_stride + kvh * kAttnD + c * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int j = threadIdx.x; j < pieces; j += kAttnThreads) {
      const int r = j / kPiecesPerRow, c = j - r * kPiecesPerRow;
      cp_async16(sv + (uint32_t)(r * kAttnD + c * 8) * 2,
                 vc + (size_t)(p0 + r) * row_stride + kvh * kAttnD + c * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  // q of the G heads of this group, dims 4*lane .. 4*lane+3
  float qv[G][4];
#pragma unroll
  for (int gh = 0; gh < G; ++gh) {
    const __half *qh = q + (size_t)(kvh * G + gh) * kAttnD + 4 * lane;
    const uint2 raw = *reinterpret_cast<const uint2 *>(qh);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
    qv[gh][0] = a.x * scale;
    qv[gh][1] = a.y * scale;
    qv[gh][2] = b.x * scale;
    qv[gh][3] = b.y * scale;
  }

  asm volatile("cp.async.wait_group 1;" ::: "memory");  // K landed
  __syncthreads();

  // scores: warp w handles positions p0 + w, p0 + w + nwarp, ...
  for (int p = p0 + warp; p < p1; p += nwarp) {
    const uint2 raw = *reinterpret_cast<const uint2 *>(s_k + (p - p0) * kAttnD + 4 * lane);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      float s = qv[gh][0] * a.x + qv[gh][1] * a.y + qv[gh][2] * b.x + qv[gh][3] * b.y;
      s = warp_sum(s);
      if (lane == 0) s_scores[gh][p - p0] = s;
    }
  }
  __syncthreads();

  // chunk max and exp-sum per head (warp gh handles head gh, strided)
  __shared__ float s_m[G], s_l[G];
  for (int gh = warp; gh < G; gh += nwarp) {
    float m = -INFINITY;
    for (int i = lane; i < p1 - p0; i += 32) m = fmaxf(m, s_scores[gh][i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < p1 - p0; i += 32) {
      const float e = __expf(s_scores[gh][i] - m);
      s_scores[gh][i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      s_m[gh] = m;
      s_l[gh] = l;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");  // V landed
  __syncthreads();

  // P.V: warp w accumulates positions p0 + w (+ nwarp ...) for dims 4*lane..
  float o[G][4];
#pragma unroll
  for (int gh = 0; gh < G; ++gh) o[gh][0] = o[gh][1] = o[gh][2] = o[gh][3] = 0.f;
  for (int p = p0 + warp; p < p1; p += nwarp) {
    const uint2 raw = *reinterpret_cast<const uint2 *>(s_v + (p - p0) * kAttnD + 4 * lane);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      const float w = s_scores[gh][p - p0];
      o[gh][0] += w * a.x;
      o[gh][1] += w * a.y;
      o[gh][2] += w * b.x;
      o[gh][3] += w * b.y;
    }
  }
#pragma unroll
  for (int gh = 0; gh < G; ++gh)
#pragma unroll
    for (int e = 0; e < 4; ++e) s_out[warp][gh][4 * lane + e] = o[gh][e];
  __syncthreads();

  for (int i = threadIdx.x; i < G * kAttnD; i += kAttnThreads) {
    const int gh = i / kAttnD, dd = i - gh * kAttnD;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < nwarp; ++w) acc += s_out[w][gh][dd];
    float *pp = partials + ((size_t)chunk * n_heads + kvh * G + gh) * kAttnPartial;
    pp[2 + dd] = acc;
    if (dd == 0) {
      pp[0] = s_m[gh];
      pp[1] = s_l[gh];
    }
  }

  // The last chunk of this (sequence, KV head) to finish merges the chunks
  // of its G query heads, in chunk order; it re-zeroes the arrival counter
  // for the next launch.
  __threadfence();
  __syncthreads();
  __shared__ bool s_last;
  const int nlive = (seq_len + chunk_len - 1) / chunk_len;  // chunks with positions
  if (threadIdx.x == 0) {
    int *arr = arrivals + (size_t)bz * n_kv + kvh;
    s_last = atomicAdd(arr, 1) == nlive - 1;
    if (s_last) *arr = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  out += bz * out_bs;
  // (max, sum) of every (chunk, head) into shared memory (s_out is free now)
  static_assert(kAttnThreads == kAttnD, "one thread per output dimension");
  static_assert(3 * kAttnMaxChunks <= (kAttnThreads / 32) * kAttnD, "merge scratch");
  float *s_cm = &s_out[0][0][0];           // [chunk][G] chunk maxima
  float *s_cl = s_cm + kAttnMaxChunks * G;  // [chunk][G] chunk sums
  float *s_cw = s_cl + kAttnMaxChunks * G;  // [chunk][G] chunk weights exp(m - M)
  __shared__ float s_L[G];
  for (int i = threadIdx.x; i < nlive * G; i += kAttnThreads) {
    const float *pp = partials + ((size_t)(i / G) * n_heads + kvh * G) * kAttnPartial +
                      (i % G) * kAttnPartial;
    s_cm[i] = __ldcg(pp);
    s_cl[i] = __ldcg(pp + 1);
  }
  __syncthreads();
  for (int gh = warp; gh < G; gh += nwarp) {
    float m = -INFINITY;
    for (int c = lane; c < nlive; c += 32) m = fmaxf(m, s_cm[c * G + gh]);
    m = warp_max(m);
    float l = 0.f;
    for (int c = lane; c < nlive; c += 32) {
      const float w = __expf(s_cm[c * G + gh] - m);
      s_cw[c * G + gh] = w;
      l += s_cl[c * G + gh] * w;
    }
    l = warp_sum(l);
    if (lane == 0) s_L[gh] = l;
  }
  __syncthreads();
  // thread dd: dimension dd of the G heads, chunks in order
  const int dd = threadIdx.x;
  float O[G];
#pragma unroll
  for (int gh = 0; gh < G; ++gh) O[gh] = 0.f;
#pragma unroll 4
  for (int c = 0; c < nlive; ++c) {
    const float *pc = partials + ((size_t)c * n_heads + kvh * G) * kAttnPartial + 2 + dd;
#pragma unroll
    for (int gh = 0; gh < G; ++gh) O[gh] += __ldcg(pc + gh * kAttnPartial) * s_cw[c * G + gh];
  }
#pragma unroll
  for (int gh = 0; gh < G; ++gh)
    out[(size_t)(kvh * G + gh) * kAttnD + dd] = from_float<OutT>(O[gh] / s_L[gh]);
}

// ---------------------------------------------------------------------------
// One decode step's attention of one sequence with RoPE and the KV append
// folded in (the runner's path: LlamaRunner.swift:612-952 -- applyRoPE on q
// and k, the cache append, then attention).  Input: the QKV projection in
// fp32 (q [n_heads][128], k and v [n_kv][128]) and the position in device
// memory.
//
// One thread-block cluster of kClusterCtas CTAs per KV head; CTA r of the
// cluster owns positions [r * chunk_len, (r + 1) * chunk_len), staged in
// shared memory by cp.async in phases of up to kPhaseRows rows (K and V rows
// padded to 272 bytes, so every ldmatrix below is free of bank conflicts).
// The first phase's rows are put in flight before the dependent wait: they
// were written by earlier steps, not by the QKV GEMV this kernel follows.
//
// Both products run on the tensor cores (mma.sync m16n8k16, fp32
// accumulators) with fp16 operands split in two so that they carry fp32
// accuracy: q (rotated in fp32, scaled by 1/sqrt(d) and by a power of two
// 2^-e that keeps it inside the fp16 range) as q_hi + q_lo, the softmax
// weights as p_hi + p_lo; K and V are fp16 already.  Scores: A = 16 cached
// rows x 16 dimensions, B = the group's heads (padded to 8); the warp owning
// a head then takes the max, the exponentials and the running sum over the
// phase's rows (online softmax across phases).  Output: A = the weights of
// the group's heads (padded to 16) x 16 rows, B = V^T through ldmatrix.trans,
// warp w holding dimensions [32w, 32w + 32).  The CTA holding the position
// also rotates k, rounds k and v to fp16, appends them to the caches and
// uses them for that row.  The CTAs' (max, sum, output) triples are merged
// through distributed shared memory after a cluster barrier: CTA h of the
// cluster finishes head h of the group from the other CTAs' partials.
#ifndef MLM_ATTN_CLUSTER
#define MLM_ATTN_CLUSTER 8
#endif
constexpr int kClusterCtas = MLM_ATTN_CLUSTER;  // CTAs per KV head
// rows staged at once: 96 rows keep the CTA (about 65 KB of shared memory,
// at most 64 registers a thread) small enough to sit beside a decode GEMV's
// CTA on one SM, so it is resident, with its first rows in flight, before
// the QKV GEMV it depends on has finished
constexpr int kPhaseRows = 96;
constexpr int kKPitch = kAttnD + 8;            // K and V row pitch in halves (272 bytes)
constexpr int kRowBytes = 2 * kKPitch * 2;     // shared memory per staged row (K and V)
constexpr int kSPitch = kPhaseRows + 4;        // score rows (fp32) per head
constexpr int kPPitch = kPhaseRows + 8;        // weight rows (fp16) per head: 208 bytes

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the float at the same shared-memory address in CTA `rank` of the cluster
__device__ __forceinline__ float ld_cluster_f32(const float *local, uint32_t rank) {
  uint32_t a = (uint32_t)__cvta_generic_to_shared(local), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}
// two floats to the same shared-memory address in CTA `rank` of the cluster
__device__ __forceinline__ void st_cluster_f32x2(const float *local, uint32_t rank, float a,
                                                 float b) {
  uint32_t la = (uint32_t)__cvta_generic_to_shared(local), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(ra), "f"(a), "f"(b) : "memory");
}
// four 8x8 fp16 matrices; lane l gives the address of row (l & 7) of
// matrix l >> 3 (.trans: each lane receives the transposed elements)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// v as fp16 hi + lo (hi = fp16(v), lo = fp16(v - hi))
__device__ __forceinline__ void split_f16(float v, __half &hi, __half &lo) {
  hi = __float2half_rn(v);
  lo = __float2half_rn(v - __half2float(hi));
}

// Sequence b = blockIdx.y of a batch reads qkv + b qkv_bs, the caches at
// b kv_bs elements, its position pos_dev[b], and writes out + b out_bs.
template <int G, class OutT>
__global__ void __launch_bounds__(kAttnThreads, 8) attn_rope_decode_kernel(
    const float *__restrict__ qkv, mlm_rope_args ra, RopeConsts rk,
    const float *__restrict__ freqs, __half *__restrict__ kc, __half *__restrict__ vc,
    int n_heads, int n_kv, int chunk_len, int rows_cap, float scale,
    const int *__restrict__ pos_dev, OutT *__restrict__ out, size_t qkv_bs, size_t kv_bs,
    size_t out_bs) {
  static_assert(kAttnThreads == 128 && kAttnD == 128, "4 warps; warp w outputs dims 32w..32w+31");
  static_assert(G <= 8 && G <= kClusterCtas,
                "a group's heads are padded to 8 (scores) and 16 (output); CTA h finishes head h");
  constexpr int HW = (G + 3) / 4;  // heads per warp in the softmax: w, w + 4
  extern __shared__ __align__(16) uint8_t s_dyn[];
  // q as fp16 hi / lo [head][dim] (heads padded to 8)
  __shared__ __align__(16) __half s_q[2][8][kKPitch];
  __shared__ __align__(16) float s_s[G][kSPitch];       // the phase's scores
  __shared__ __align__(16) __half s_p[2][16][kPPitch];  // weights hi / lo [head][row]
  __shared__ __align__(16) float s_recv[kClusterCtas][kAttnD + 4];  // partials of head rank
  __shared__ float s_corr[G], s_qmax[2];
  const uint32_t rank = cluster_ctarank();
  const int kvh = blockIdx.x / kClusterCtas;
  qkv += blockIdx.y * qkv_bs;
  kc += blockIdx.y * kv_bs;
  vc += blockIdx.y * kv_bs;
  out += blockIdx.y * out_bs;
  // the position and the cached rows before it were written by earlier
  // steps, not by the kernel this one depends on: read them before the wait
  const int pos = pos_dev[blockIdx.y];
  const int seq_len = pos + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const size_t row_stride = (size_t)n_kv * kAttnD;
  const float *kf = qkv + (size_t)n_heads * kAttnD;
  const float *vf = kf + row_stride;
  const int p_begin = (int)rank * chunk_len;
  const int p_end = min(p_begin + chunk_len, seq_len);
  // rows staged per phase: rows_cap (a multiple of 32, at most kPhaseRows)
  const int nphase = p_end > p_begin ? (p_end - p_begin + rows_cap - 1) / rows_cap : 0;
  const bool has_new = nphase > 0 && p_end == seq_len;  // this CTA holds row `pos`
  __half *s_k = reinterpret_cast<__half *>(s_dyn);        // [rows_cap][kKPitch]
  __half *s_v = s_k + (size_t)rows_cap * kKPitch;         // [rows_cap][kKPitch]

  // Cached rows of phase ph by cp.async, K and V as separate groups, so the
  // next phase's K is in flight during this phase's softmax and P.V and its
  // V after this phase's P.V (row pos, when it falls in a phase, comes from
  // registers once q, k and v are available).
  auto phase_rows = [&](int ph, int &a, int &n, int &cached) {
    a = p_begin + ph * rows_cap;
    n = min(rows_cap, p_end - a);
    cached = (has_new && a + n == p_end) ? n - 1 : n;
  };
  auto load_rows = [&](int ph, const __half *src, __half *dst) {
    int a, n, cached;
    phase_rows(ph, a, n, cached);
    constexpr int kPieces = kAttnD * (int)sizeof(__half) / 16;  // 16 per row
    const uint32_t sd = (uint32_t)__cvta_generic_to_shared(dst);
    for (int j = threadIdx.x; j < cached * kPieces; j += kAttnThreads) {
      const int r = j / kPieces, c = j - r * kPieces;
      cp_async16(sd + (uint32_t)(r * kKPitch + c * 8) * 2,
                 src + (size_t)(a + r) * row_stride + kvh * kAttnD + c * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (nphase > 0) {
    load_rows(0, kc, s_k);
    load_rows(0, vc, s_v);
  }
  // padding: weight rows of heads G..15 and q rows of heads G..7 are zero
  for (int i = threadIdx.x; i < 2 * (16 - G) * kPPitch; i += kAttnThreads) {
    const int hl = i / ((16 - G) * kPPitch), rem = i - hl * (16 - G) * kPPitch;
    s_p[hl][G + rem / kPPitch][rem % kPPitch] = __float2half_rn(0.f);
  }
  for (int i = threadIdx.x; i < 2 * (8 - G) * kKPitch; i += kAttnThreads) {
    const int hl = i / ((8 - G) * kKPitch), rem = i - hl * (8 - G) * kKPitch;
    s_q[hl][G + rem / kKPitch][rem % kKPitch] = __float2half_rn(0.f);
  }
  // the rotation of pair t at this position (threads t < 64)
  float c = 1.f, sn = 0.f;
  if (threadIdx.x < 64 && 2 * (int)threadIdx.x < (int)ra.n_dims)
    rope_cos_sin(ra, rk, freqs, pos, threadIdx.x, c, sn);

  // q, k and v of this step come from the QKV GEMV before this kernel
  pdl_wait_then_release();

  // q of the group rotated in fp32 (pair t of every head by thread t < 64)
  // and scaled by 1/sqrt(d), the new k row rotated likewise, the new v row
  // by threads 64..127
  __half2 kv_new = __floats2half2_rn(0.f, 0.f);
  float qr[G][2];
  float qm = 0.f;
  {
    const int t = threadIdx.x & 63;
    if (threadIdx.x < 64) {
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float2 x =
            *reinterpret_cast<const float2 *>(qkv + (size_t)(kvh * G + h) * kAttnD + 2 * t);
        qr[h][0] = (x.x * c - x.y * sn) * scale;
        qr[h][1] = (x.x * sn + x.y * c) * scale;
        qm = fmaxf(qm, fmaxf(fabsf(qr[h][0]), fabsf(qr[h][1])));
      }
      if (has_new) {
        const float2 x = *reinterpret_cast<const float2 *>(kf + kvh * kAttnD + 2 * t);
        kv_new = __floats2half2_rn(x.x * c - x.y * sn, x.x * sn + x.y * c);
        *reinterpret_cast<__half2 *>(kc + ((size_t)pos * n_kv + kvh) * kAttnD + 2 * t) = kv_new;
      }
    } else if (has_new) {
      const float2 x = *reinterpret_cast<const float2 *>(vf + kvh * kAttnD + 2 * t);
      kv_new = __floats2half2_rn(x.x, x.y);
      *reinterpret_cast<__half2 *>(vc + ((size_t)pos * n_kv + kvh) * kAttnD + 2 * t) = kv_new;
    }
  }
  qm = warp_max(qm);
  if (lane == 0 && warp < 2) s_qmax[warp] = qm;
  __syncthreads();
  // q * 2^-qe stays below 2^15 (fp16); the scores are multiplied back
  const int qe = silu_scale_exp(fmaxf(s_qmax[0], s_qmax[1]));
  const float sback = __uint_as_float((uint32_t)(127 + qe) << 23);
  if (threadIdx.x < 64) {
    const float qinv = __uint_as_float((uint32_t)(127 - qe) << 23);
    const int t = threadIdx.x;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      __half h0, l0, h1, l1;
      split_f16(qr[h][0] * qinv, h0, l0);
      split_f16(qr[h][1] * qinv, h1, l1);
      *reinterpret_cast<__half2 *>(&s_q[0][h][2 * t]) = __halves2half2(h0, h1);
      *reinterpret_cast<__half2 *>(&s_q[1][h][2 * t]) = __halves2half2(l0, l1);
    }
  }

  const uint32_t sq = (uint32_t)__cvta_generic_to_shared(&s_q[0][0][0]);
  const uint32_t sp = (uint32_t)__cvta_generic_to_shared(&s_p[0][0][0]);
  const uint32_t skb = (uint32_t)__cvta_generic_to_shared(s_k);
  const uint32_t svb = (uint32_t)__cvta_generic_to_shared(s_v);
  // ldmatrix row addresses of this lane: A tiles (rows r0 + (lane & 15)),
  // B tiles of q (head lane & 7, 8-column block lane >> 3)
  const int a_row = (lane & 7) + ((lane >> 3) & 1) * 8, a_col = (lane >> 4) * 8;
  const int b_row = lane & 7, b_col = (lane >> 3) * 8;
  constexpr uint32_t kQBytes = 8 * kKPitch * 2, kPBytes = 16 * kPPitch * 2;

  float m_run[HW], l_run[HW];
#pragma unroll
  for (int i = 0; i < HW; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
  }
  float o[4][4];  // output dims 32w + 8nt + 2tq (+1) of head g (rows g + 8: padding)
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;

  // the new row of phase ph into its K (threads < 64) or V (64..127) stage,
  // and (V) zero rows n..n16-1, which meet zero weights but may hold NaN
  auto fill_k = [&](int ph) {
    int a, n, cached;
    phase_rows(ph, a, n, cached);
    if (cached < n && threadIdx.x < 64)
      *reinterpret_cast<__half2 *>(s_k + (size_t)cached * kKPitch + 2 * threadIdx.x) = kv_new;
  };
  auto fill_v = [&](int ph) {
    int a, n, cached;
    phase_rows(ph, a, n, cached);
    if (cached < n && threadIdx.x >= 64)
      *reinterpret_cast<__half2 *>(s_v + (size_t)cached * kKPitch + 2 * (threadIdx.x - 64)) =
          kv_new;
    const int n16 = (n + 15) & ~15;
    for (int i = threadIdx.x; i < (n16 - n) * (kAttnD / 2); i += kAttnThreads)
      reinterpret_cast<uint32_t *>(s_v + (size_t)(n + i / (kAttnD / 2)) * kKPitch)[i % (kAttnD / 2)] =
          0u;
  };
  if (nphase > 0) {
    fill_k(0);
    fill_v(0);
  }
  for (int ph = 0; ph < nphase; ++ph) {
    const int n = min(rows_cap, p_end - (p_begin + ph * rows_cap));
    const int n16 = (n + 15) & ~15;
    const bool more = ph + 1 < nphase;
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // this phase's K (its V may fly)
    __syncthreads();

    // scores of 16-row tiles w, w + 4, ...: S = K (q_hi + q_lo)^T
    for (int j0 = 16 * warp; j0 < n; j0 += 64) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f}, acl[4] = {0.f, 0.f, 0.f, 0.f};  // q_hi, q_lo
#pragma unroll
      for (int s = 0; s < kAttnD / 16; s += 2) {
        uint32_t qh[4], ql[4], ka[4];
        const uint32_t qo = (uint32_t)(b_row * kKPitch + 16 * s + b_col) * 2;
        ldsm_x4(sq + qo, qh);
        ldsm_x4(sq + kQBytes + qo, ql);
        ldsm_x4(skb + (uint32_t)((j0 + a_row) * kKPitch + 16 * s + a_col) * 2, ka);
        mma_16816(acc, ka, qh[0], qh[1]);
        mma_16816(acl, ka, ql[0], ql[1]);
        ldsm_x4(skb + (uint32_t)((j0 + a_row) * kKPitch + 16 * (s + 1) + a_col) * 2, ka);
        mma_16816(acc, ka, qh[2], qh[3]);
        mma_16816(acl, ka, ql[2], ql[3]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] += acl[e];
      // C: rows j0 + g (acc 0, 1) and j0 + g + 8 (acc 2, 3), heads 2tq, 2tq + 1
      if (2 * tq < G) {
        s_s[2 * tq][j0 + g] = acc[0] * sback;
        s_s[2 * tq][j0 + g + 8] = acc[2] * sback;
      }
      if (2 * tq + 1 < G) {
        s_s[2 * tq + 1][j0 + g] = acc[1] * sback;
        s_s[2 * tq + 1][j0 + g + 8] = acc[3] * sback;
      }
    }
    __syncthreads();
    if (more) {  // the K stage is free: the next phase's K
      load_rows(ph + 1, kc, s_k);
      fill_k(ph + 1);
    }

    // softmax of head h by warp h % 4 over rows lane + 32 i; weights as
    // fp16 hi / lo (zero for rows n..n16-1)
#pragma unroll
    for (int hi = 0; hi < HW; ++hi) {
      const int h = warp + 4 * hi;
      if (h >= G) break;
      float sv[kPhaseRows / 32];
      float mloc = -INFINITY;
#pragma unroll
      for (int i = 0; i < kPhaseRows / 32; ++i) {
        const int j = lane + 32 * i;
        sv[i] = j < n ? s_s[h][j] : -INFINITY;
        mloc = fmaxf(mloc, sv[i]);
      }
      const float m_new = fmaxf(m_run[hi], warp_max(mloc));
      float lsum = 0.f;
#pragma unroll
      for (int i = 0; i < kPhaseRows / 32; ++i) {
        const int j = lane + 32 * i;
        const float p = j < n ? __expf(sv[i] - m_new) : 0.f;
        lsum += p;
        if (j < n16) {
          __half ph16, pl16;
          split_f16(p, ph16, pl16);
          s_p[0][h][j] = ph16;
          s_p[1][h][j] = pl16;
        }
      }
      const float corr = __expf(m_run[hi] - m_new);
      l_run[hi] = l_run[hi] * corr + warp_sum(lsum);
      m_run[hi] = m_new;
      if (lane == 0) s_corr[h] = corr;
    }
    // this phase's V (the next phase's K, if any, may still fly)
    if (more)
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    else
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();

    // output: O[h][d] = corr O + (p_hi + p_lo) V over the phase's rows,
    // dims [32w, 32w + 32) of warp w
    {
      const float cr = g < G ? s_corr[g] : 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        o[nt][0] *= cr;
        o[nt][1] *= cr;
      }
      for (int j0 = 0; j0 < n16; j0 += 16) {
        uint32_t pa[4], pl[4];
        const uint32_t po = (uint32_t)(a_row * kPPitch + j0 + a_col) * 2;
        ldsm_x4(sp + po, pa);
        ldsm_x4(sp + kPBytes + po, pl);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t vb[4];
          ldsm_x4_t(svb + (uint32_t)((j0 + a_row) * kKPitch + 32 * warp + 16 * half + a_col) * 2, vb);
          mma_16816(o[2 * half], pa, vb[0], vb[1]);
          mma_16816(o[2 * half], pl, vb[0], vb[1]);
          mma_16816(o[2 * half + 1], pa, vb[2], vb[3]);
          mma_16816(o[2 * half + 1], pl, vb[2], vb[3]);
        }
      }
    }
    __syncthreads();  // the V stage, scores and weights are free for the next phase
    if (more) {
      load_rows(ph + 1, vc, s_v);
      fill_v(ph + 1);
    }
  }

  // this CTA's partials go straight into the shared memory of the CTA that
  // finishes each head (CTA h of the cluster for head h), in slot `rank`:
  // (max, sum, output[128]); the cluster barrier makes them visible there,
  // and after it no CTA touches another's shared memory
  if (g < G) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
      st_cluster_f32x2(&s_recv[rank][2 + 32 * warp + 8 * nt + 2 * tq], g, o[nt][0], o[nt][1]);
  }
#pragma unroll
  for (int hi = 0; hi < HW; ++hi) {
    const int h = warp + 4 * hi;
    if (h < G && lane == 0) st_cluster_f32x2(&s_recv[rank][0], h, m_run[hi], l_run[hi]);
  }
  cluster_sync_all();

  // CTA h < G finishes head h from every CTA's partials (CTA 0 always holds
  // rows, so M is finite)
  if ((int)rank < G) {
    const int h = (int)rank;
    float M = -INFINITY;
#pragma unroll
    for (int cc = 0; cc < kClusterCtas; ++cc) M = fmaxf(M, s_recv[cc][0]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int cc = 0; cc < kClusterCtas; ++cc) {
      const float w = __expf(s_recv[cc][0] - M);
      L += s_recv[cc][1] * w;
      O += s_recv[cc][2 + threadIdx.x] * w;
    }
    out[(size_t)(kvh * G + h) * kAttnD + threadIdx.x] = from_float<OutT>(O / L);
  }
}

// positions per CTA of the fused kernel: the capacity over the cluster,
// rounded up to whole 32-row groups
static int attn_rope_chunk_len(int capacity) {
  const int per = (capacity + kClusterCtas - 1) / kClusterCtas;
  return (per + 31) / 32 * 32;
}

template <class OutT>
static int attn_rope_launch(mlm_ctx *ctx, const float *qkv, const float *freqs,
                            const mlm_rope_args &ra, int n_heads, int n_kv, int head_dim,
                            int capacity, void *kc, void *vc, OutT *out, int batch,
                            size_t qkv_bs, size_t kv_bs, size_t out_bs, cudaStream_t stream,
                            const int *pos_dev) {
  MLM_REQUIRE(ctx, head_dim == kAttnD, MLM_ERR_UNSUPPORTED,
              "attention: head_dim=%d (this build handles %d)", head_dim, kAttnD);
  MLM_REQUIRE(ctx, n_kv > 0 && n_heads % n_kv == 0, MLM_ERR_SHAPE,
              "attention: %d query heads not a multiple of %d KV heads", n_heads, n_kv);
  const int G = n_heads / n_kv;
  MLM_REQUIRE(ctx, G == 1 || G == 2 || G == 4 || G == 8, MLM_ERR_UNSUPPORTED,
              "attention: GQA group %d (supported 1, 2, 4, 8)", G);
  MLM_REQUIRE(ctx, capacity > 0 && batch > 0 && batch <= 65535, MLM_ERR_SHAPE,
              "attention: cache capacity %d, batch %d", capacity, batch);
  const int chunk_len = attn_rope_chunk_len(capacity);
  // A grid past three CTAs per SM (a batch) stages 64-row phases: at
  // 53 KB four CTAs fit an SM, so the grid runs in one wave
  const int ctas = n_kv * kClusterCtas * batch;
  const int rows_cap = std::min(chunk_len, ctas > 3 * ctx->sm_count ? 64 : kPhaseRows);
  const RopeConsts rk = rope_consts(ra);
  const float scale = 1.0f / sqrtf((float)head_dim);
  auto kern = G == 1   ? attn_rope_decode_kernel<1, OutT>
              : G == 2 ? attn_rope_decode_kernel<2, OutT>
              : G == 4 ? attn_rope_decode_kernel<4, OutT>
                       : attn_rope_decode_kernel<8, OutT>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_kv * kClusterCtas, batch);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = (size_t)rows_cap * kRowBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(
      &cfg, kern, qkv, ra, rk, freqs, reinterpret_cast<__half *>(kc),
      reinterpret_cast<__half *>(vc), n_heads, n_kv, chunk_len, rows_cap, scale, pos_dev, out,
      qkv_bs, kv_bs, out_bs);
  return check_launch_pdl(ctx, e, "attention (RoPE, append, decode)");
}

int attn_rope_decode_launch(mlm_ctx *ctx, const float *qkv, const float *freqs,
                            const mlm_rope_args &ra, int n_heads, int n_kv, int head_dim,
                            int capacity, void *kc, void *vc, void *out, cudaStream_t stream,
                            const int *pos_dev) {
  return attn_rope_launch(ctx, qkv, freqs, ra, n_heads, n_kv, head_dim, capacity, kc, vc,
                          reinterpret_cast<__half *>(out), 1, 0, 0, 0, stream, pos_dev);
}

int attn_rope_decode_batch_launch(mlm_ctx *ctx, const float *qkv, size_t qkv_bs,
                                  const float *freqs, const mlm_rope_args &ra, int n_heads,
                                  int n_kv, int head_dim, int capacity, int batch, size_t kv_bs,
                                  void *kc, void *vc, void *out_bf16, cudaStream_t stream,
                                  const int *pos_dev) {
  return attn_rope_launch(ctx, qkv, freqs, ra, n_heads, n_kv, head_dim, capacity, kc, vc,
                          reinterpret_cast<__nv_bfloat16 *>(out_bf16), batch, qkv_bs, kv_bs,
                          (size_t)n_heads * head_dim, stream, pos_dev);
}

// seq_len positions, or, when pos_dev is set, pos_dev[b] + 1 positions read
// on the device out of a cache of capacity seq_len (a launch a captured graph
// can replay at every step): fixed 128-position chunks covering the capacity.
// `batch` sequences (grid z; mlm_attn_decode passes one): sequence b reads
// q + b q_bs, caches + b kv_bs, uses partials + b part_bs and writes
// out + b out_bs (as OutT).
template <class OutT>
static int attn_decode_impl(mlm_ctx *ctx, const void *q, const void *kc, const void *vc,
                            int n_heads, int n_kv, int head_dim, int seq_len, OutT *out,
                            float *partials, size_t partial_floats, cudaStream_t stream,
                            const int *pos_dev, int batch, size_t q_bs, size_t kv_bs,
                            size_t out_bs) {
  MLM_REQUIRE(ctx, head_dim == kAttnD, MLM_ERR_UNSUPPORTED,
              "mlm_attn_decode: head_dim=%d (this build handles %d)", head_dim, kAttnD);
  MLM_REQUIRE(ctx, n_kv > 0 && n_heads % n_kv == 0, MLM_ERR_SHAPE,
              "mlm_attn_decode: %d query heads not a multiple of %d KV heads", n_heads, n_kv);
  const int G = n_heads / n_kv;
  MLM_REQUIRE(ctx, G == 1 || G == 2 || G == 4 || G == 8, MLM_ERR_UNSUPPORTED,
              "mlm_attn_decode: GQA group %d (supported 1, 2, 4, 8)", G);
  MLM_REQUIRE(ctx, seq_len > 0 && batch > 0, MLM_ERR_SHAPE, "mlm_attn_decode: seq_len=%d batch=%d",
              seq_len, batch);
  int nchunks, chunk_len;
  if (pos_dev) {
    chunk_len = 2 * kAttnChunk;
    nchunks = (seq_len + chunk_len - 1) / chunk_len;
    MLM_REQUIRE(ctx, nchunks <= kAttnMaxChunks, MLM_ERR_SHAPE,
                "mlm_attn_decode: cache capacity %d exceeds %d positions", seq_len,
                2 * kAttnChunk * kAttnMaxChunks);
  } else {
    nchunks = (seq_len + kAttnChunk - 1) / kAttnChunk;
    if (nchunks > kAttnMaxChunks) nchunks = kAttnMaxChunks;
    chunk_len = (seq_len + nchunks - 1) / nchunks;
  }
  MLM_REQUIRE(ctx, chunk_len <= 2 * kAttnChunk, MLM_ERR_SHAPE,
              "mlm_attn_decode: seq_len=%d exceeds %d positions", seq_len,
              2 * kAttnChunk * kAttnMaxChunks);
  const size_t part_bs = (size_t)nchunks * n_heads * kAttnPartial;
  MLM_REQUIRE(ctx, part_bs * batch <= partial_floats, MLM_ERR_SHAPE,
              "mlm_attn_decode: %d heads x %d sequences exceed the attention scratch", n_heads,
              batch);
  const float scale = 1.0f / sqrtf((float)head_dim);
  dim3 grid(n_kv, nchunks, batch);
  const __half *qh = reinterpret_cast<const __half *>(q);
  const __half *kh = reinterpret_cast<const __half *>(kc);
  const __half *vh = reinterpret_cast<const __half *>(vc);
  auto kern = G == 1   ? attn_decode_partial_kernel<1, OutT>
              : G == 2 ? attn_decode_partial_kernel<2, OutT>
              : G == 4 ? attn_decode_partial_kernel<4, OutT>
                       : attn_decode_partial_kernel<8, OutT>;
  return check_launch_pdl(
      ctx,
      launch_pdl(kern, grid, dim3(kAttnThreads), kAttnStageBytes, stream, qh, kh, vh, n_heads,
                 n_kv, seq_len, chunk_len, scale, partials, pos_dev, q_bs, kv_bs, part_bs, out,
                 out_bs, ctx->attn_arrivals),
      "mlm_attn_decode");
}

int attn_decode_launch(mlm_ctx *ctx, const void *q, const void *kc, const void *vc, int n_heads,
                       int n_kv, int head_dim, int seq_len, void *out, float *partials,
                       size_t partial_floats, cudaStream_t stream, const int *pos_dev) {
  return attn_decode_impl(ctx, q, kc, vc, n_heads, n_kv, head_dim, seq_len,
                          reinterpret_cast<__half *>(out), partials, partial_floats, stream,
                          pos_dev, 1, 0, 0, 0);
}

// called once per context, with its device current
template <class OutT>
static int attn_init_out(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_decode_partial_kernel<1, OutT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnStageBytes));
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_decode_partial_kernel<2, OutT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnStageBytes));
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_decode_partial_kernel<4, OutT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnStageBytes));
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_decode_partial_kernel<8, OutT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnStageBytes));
  return MLM_OK;
}

template <int G, class OutT>
static int attn_rope_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_rope_decode_kernel<G, OutT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kPhaseRows * kRowBytes));
  if (kClusterCtas > 8)
    MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_rope_decode_kernel<G, OutT>,
                                           cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  return MLM_OK;
}

template <class OutT>
static int attn_rope_init_all(mlm_ctx *ctx) {
  int st = attn_rope_init<1, OutT>(ctx);
  if (st == MLM_OK) st = attn_rope_init<2, OutT>(ctx);
  if (st == MLM_OK) st = attn_rope_init<4, OutT>(ctx);
  if (st == MLM_OK) st = attn_rope_init<8, OutT>(ctx);
  return st;
}

int attn_init(mlm_ctx *ctx) {
  int st = attn_rope_init_all<__half>(ctx);
  if (st == MLM_OK) st = attn_rope_init_all<__nv_bfloat16>(ctx);
  if (st != MLM_OK) return st;
  st = attn_init_out<__half>(ctx);
  if (st != MLM_OK) return st;
  // arrival counters of the chunk merge, zero between launches
  if (cudaMalloc(&ctx->attn_arrivals, sizeof(int) * kAttnMaxArrivals) != cudaSuccess)
    return set_error(ctx, MLM_ERR_ALLOC, "attention: arrival counters");
  MLM_CUDA_TRY(ctx, cudaMemset(ctx->attn_arrivals, 0, sizeof(int) * kAttnMaxArrivals));
  return MLM_OK;
}

size_t attn_partial_floats_max(int max_heads) {
  return (size_t)kAttnMaxChunks * max_heads * kAttnPartial;
}

// ---- embedding gather and argmax ------------------------------------------------

__global__ void embed_f16_kernel(const __half *__restrict__ table, int vocab, int dim,
                                 const int32_t *__restrict__ token, float *__restrict__ out) {
  pdl_wait_then_release();
  int t = *token;
  t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
  const __half *row = table + (size_t)t * dim;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    out[i] = __half2float(row[i]);
}

// Argmax as one 64-bit maximum: the high word orders the float values, the
// low word is ~index so that equal values (-0 and +0 included) resolve to
// the first index.  NaN never wins; an all-NaN row yields 0 (key 0).
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  const uint32_t b = __float_as_uint(__fadd_rn(v, 0.0f));  // -0 -> +0: equal values tie
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (uint32_t)(~(uint32_t)i);
}

constexpr int kArgmaxThreads = 256;

// grid-stride partial maxima, combined with atomicMax in scratch[0]; the
// last CTA to finish (ticket in scratch[1]) writes the index and zeroes the
// scratch for the next call
// (with key_out set, the last CTA stores the key of the maximum, indices
// counted from `offset`, instead of the index)
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(
    const float *__restrict__ x, int n, int offset, unsigned long long *scratch,
    int32_t *__restrict__ out, unsigned long long *key_out) {
  pdl_wait_then_release();
  unsigned long long best = 0;
  const int stride = gridDim.x * blockDim.x;
#pragma unroll 8
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = x[i];
    if (v == v) best = max(best, argmax_key(v, i + offset));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  __shared__ unsigned long long sb[kArgmaxThreads / 32];
  __shared__ bool last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sb[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = sb[0];
    for (int w = 1; w < kArgmaxThreads / 32; ++w) b = max(b, sb[w]);
    if (b) atomicMax(scratch, b);
    __threadfence();
    last = atomicAdd(scratch + 1, 1ull) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    const unsigned long long k = atomicExch(scratch, 0ull);
    scratch[1] = 0;
    if (key_out)
      *key_out = k;
    else
      *out = k ? (int32_t)~(uint32_t)(k & 0xFFFFFFFFull) : 0;
  }
}

// rows of keys laid out [nkeys][rows] (an all-gather of every rank's row
// keys): out[b] = the index of the largest key of row b
__global__ void argmax_keys_rows_kernel(const unsigned long long *keys, int nkeys, int rows,
                                        int32_t *out) {
  pdl_wait_then_release();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= rows) return;
  unsigned long long k = 0;
  for (int i = 0; i < nkeys; ++i) k = max(k, keys[(size_t)i * rows + b]);
  out[b] = k ? (int32_t)~(uint32_t)(k & 0xFFFFFFFFull) : 0;
}

__global__ void argmax_keys_kernel(const unsigned long long *keys, int nkeys, int32_t *out) {
  pdl_wait_then_release();
  unsigned long long k = 0;
  for (int i = 0; i < nkeys; ++i) k = max(k, keys[i]);
  *out = k ? (int32_t)~(uint32_t)(k & 0xFFFFFFFFull) : 0;
}

int argmax_launch(mlm_ctx *ctx, const float *x, int n, int32_t *out, cudaStream_t stream) {
  const int ctas = std::max(1, std::min(ctx->sm_count, (n + 8 * kArgmaxThreads - 1) /
                                                           (8 * kArgmaxThreads)));
  return check_launch_pdl(ctx,
                          launch_pdl(argmax_kernel, dim3(ctas), dim3(kArgmaxThreads), 0, stream,
                                     x, n, 0, ctx->argmax_scratch, out, nullptr),
                          "mlm_argmax_f32");
}

int argmax_keys_rows_launch(mlm_ctx *ctx, const unsigned long long *keys, int nkeys, int rows,
                            int32_t *out, cudaStream_t stream) {
  return check_launch_pdl(ctx,
                          launch_pdl(argmax_keys_rows_kernel, dim3((rows + 127) / 128), dim3(128),
                                     0, stream, keys, nkeys, rows, out),
                          "argmax (row keys)");
}

int argmax_key_launch(mlm_ctx *ctx, const float *x, int n, int offset, unsigned long long *key,
                      cudaStream_t stream) {
  const int ctas = std::max(1, std::min(ctx->sm_count, (n + 8 * kArgmaxThreads - 1) /
                                                           (8 * kArgmaxThreads)));
  return check_launch_pdl(ctx,
                          launch_pdl(argmax_kernel, dim3(ctas), dim3(kArgmaxThreads), 0, stream,
                                     x, n, offset, ctx->argmax_scratch, nullptr, key),
                          "argmax (key)");
}

int argmax_keys_launch(mlm_ctx *ctx, const unsigned long long *keys, int nkeys, int32_t *out,
                       cudaStream_t stream) {
  return check_launch_pdl(
      ctx, launch_pdl(argmax_keys_kernel, dim3(1), dim3(1), 0, stream, keys, nkeys, out),
      "argmax (keys)");
}

int embed_launch(mlm_ctx *ctx, const void *table, int vocab, int dim, const int32_t *tok,
                 float *out, cudaStream_t stream) {
  return check_launch_pdl(
      ctx,
      launch_pdl(embed_f16_kernel, dim3((dim + 255) / 256), dim3(256), 0, stream,
                 reinterpret_cast<const __half *>(table), vocab, dim, tok, out),
      "mlm_embed_f16");
}

}  // namespace mlm

using namespace mlm;

extern "C" int mlm_attn_decode(mlm_ctx *ctx, const void *q, const void *kc, const void *vc,
                               int n_heads, int n_kv_heads, int head_dim, int seq_len,
                               void *out) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, q && kc && vc && out, MLM_ERR_ARG, "mlm_attn_decode: null buffer");
  MLM_REQUIRE(ctx, aligned16(q) && aligned16(kc) && aligned16(vc), MLM_ERR_ALIGN,
              "mlm_attn_decode: q and caches must be 16-byte aligned");
  return attn_decode_launch(ctx, q, kc, vc, n_heads, n_kv_heads, head_dim, seq_len, out,
                            ctx->attn_partials, ctx->attn_partials_floats, ctx->stream, nullptr);
}

extern "C" int mlm_embed_f16(mlm_ctx *ctx, const void *table, int vocab, int dim,
                             const int32_t *token, float *out) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, table && token && out, MLM_ERR_ARG, "mlm_embed_f16: null buffer");
  MLM_REQUIRE(ctx, vocab > 0 && dim > 0, MLM_ERR_SHAPE, "mlm_embed_f16: vocab=%d dim=%d", vocab,
              dim);
  return embed_launch(ctx, table, vocab, dim, token, out, ctx->stream);
}

extern "C" int mlm_argmax_f32(mlm_ctx *ctx, const float *logits, int n, int32_t *out) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, logits && out, MLM_ERR_ARG, "mlm_argmax_f32: null buffer");
  MLM_REQUIRE(ctx, n > 0, MLM_ERR_SHAPE, "mlm_argmax_f32: n=%d", n);
  return argmax_launch(ctx, logits, n, out, ctx->stream);
}
