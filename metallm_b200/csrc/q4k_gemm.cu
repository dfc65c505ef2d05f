// q4k_gemm.cu -- prefill Q4_K GEMM on the 5th-generation tensor cores:
// Y[t][n] = sum_k X[t][k] * W[n][k] (+ R[t][n]) for T tokens at once.
//
// Replaces the prefill linears of the reference (encodeMPSMatrixMultiply on
// weights dequantized to fp16 at load, MetalService.swift:797-925; the
// reference has no batched prefill, it runs forward() token by token,
// LlamaRunner.swift:320).  W stays packed Q4_K in HBM (GGUF layout); each CTA
// dequantizes its weight tile to bf16 in shared memory and feeds tcgen05.mma
// with fp32 accumulators in tensor memory.
//
// Output tile: 256 weight rows x 256 tokens, held as two M = 128 x N = 256
// fp32 accumulators in all 512 TMEM columns, so every X tile brought into
// shared memory serves 256 weight rows (X bytes per FLOP is what bounds a
// 128-row tile: the whole chip's L2-to-SM ingest runs out near 7.5 TB/s).
// K advances 32 elements (one Q4_K sub-block) per pipeline stage, four
// stages of A (256 x 32 bf16) and B (256 tokens x 32 bf16), both in the
// 64-byte-swizzled K-major layout tcgen05 reads.
//
// Schedule (data-parallel waves, then stream-K): one persistent CTA per SM.
// Tiles are numbered with the row tile fastest, so the CTAs of a wave share
// their X tile in L2.  All but the last one to two waves' worth of tiles go
// out whole, CTA c taking tiles c, c + grid, ...; the (tile, K-stage) work of
// the rest is cut into equal contiguous ranges, one per CTA, so no wave is
// left partly empty.  A range covers whole tiles and at most a trailing and
// a leading part of a tile shared with its neighbours.  A tile part that
// ends the tile's K range ("tail") opens its CTA's range; it stores
// Y = acc (+ R) and then raises the tile's flag to the number of other
// parts.  Every other part (the last of its CTA) waits for the flag
// (bounded), adds its accumulator into Y with fp32 atomics and counts the
// flag back down, so the flags are zero again when the launch ends.
//
// Warp roles (64 + 512 threads):
//   warp 0     TMA: packed W block columns (256 rows x 144 bytes, 2 buffers)
//              and the bf16 X tile of each stage (256 tokens x 32);
//   warp 1     allocates TMEM; one thread issues the MMAs and commits;
//   warps 2-17 16 dequantizing warps in G groups (group g takes the stages
//              with index % G == g; a thread converts one or two weight rows:
//              (d*sc)*q - dmin*m in fp32 rounded to bf16, 32 values per row
//              and stage); together they run each part's epilogue (tcgen05.ld
//              of their lane quarter and column share, stores or atomics).
// Stages are tracked by mbarriers (full: TMA bytes / dequant warps, empty:
// the MMA commit; the accumulator is handed back by the epilogue warps);
// every wait is bounded and reports a device error.
#include <cuda.h>

#include <algorithm>

#include "mlm_internal.h"
#include "q4k_gemv_common.cuh"

namespace mlm {
namespace {

constexpr int kMmaM = 128;       // rows per MMA and per accumulator
constexpr int kGemmRows = 256;   // weight rows per tile: two accumulators
constexpr int kGemmTok = 256;    // tokens per tile (MMAs of N = 256)
constexpr int kGemmKStep = 32;   // K per stage: one Q4_K sub-block
constexpr int kGemmStages = 4;
constexpr int kStagesPerBlock = kQK / kGemmKStep;  // 8 stages per W block column
#ifndef MLM_GEMM_DQ_GROUPS
#define MLM_GEMM_DQ_GROUPS 4
#endif
// 16 dequantizing warps in G groups; group g takes the stages kk with
// kk % G == g, so the per-stage latency of a dequantizing warp (barrier,
// loads, convert, store) overlaps across groups; a group's threads cover the
// tile's 256 rows (one or two rows each)
constexpr int kDqWarps = 16;
constexpr int kDqGroups = MLM_GEMM_DQ_GROUPS;
constexpr int kWarpsPerGroup = kDqWarps / kDqGroups;
constexpr int kRowsPerThread = kGemmRows / (32 * kWarpsPerGroup);
static_assert(kStagesPerBlock % kDqGroups == 0, "groups divide a block column's stages");
static_assert(kRowsPerThread == 1 || kRowsPerThread == 2, "one or two rows per thread");
constexpr int kGemmThreads = 64 + 32 * kDqWarps;
constexpr int kAHalf = kMmaM * kGemmKStep * 2;       // 8 KB: one accumulator's rows
constexpr int kAStage = 2 * kAHalf;                  // 16 KB
constexpr int kBStage = kGemmTok * kGemmKStep * 2;   // 16 KB
constexpr int kWpk = kGemmRows * kBlockBytes;        // 36 KB
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kGemmStages * kAStage;
constexpr int kOffW = kOffB + kGemmStages * kBStage;
constexpr int kOffBar = kOffW + 2 * kWpk;
// mbarriers: wfull[2] wempty[2] bfull[S] afull[S] sempty[S] done accfree,
// then the TMEM base address and the epilogue's flag verdict
constexpr int kBarWfull = 0, kBarWempty = 2, kBarBfull = 4, kBarAfull = 4 + kGemmStages,
              kBarSempty = 4 + 2 * kGemmStages, kBarDone = 4 + 3 * kGemmStages,
              kBarAccFree = kBarDone + 1;
constexpr int kNumBars = kBarAccFree + 1;
constexpr int kGemmSmem = kOffBar + kNumBars * 8 + 16;
constexpr int kMinUnitsPerCta = 16;  // K stages: keeps each CTA's share above two block columns
constexpr int kTmemCols = 512;  // two fp32 accumulators of 256 columns

// tcgen05 instruction descriptor: fp32 accumulate, bf16 A and B, both
// K-major, M = 128, N = n (16 .. 256 in steps of 16)
constexpr uint32_t idesc_for(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((128u >> 4) << 24);
}

// shared-memory matrix descriptor of a K-major bf16 tile in the 64-byte
// swizzle layout: rows of 64 bytes, 8-row atoms of 512 bytes (stride 512),
// 16-byte chunk c of row r stored at chunk c ^ ((r >> 1) & 3); descriptor
// version 1, layout type 4 (64-byte swizzle)
__device__ __forceinline__ uint64_t sw64_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(512 >> 4) << 32) |
         (1ull << 46) | (4ull << 61);
}

struct GemmArgs {
  float *y;               // [T][N] fp32
  const float *residual;  // [T][N] or NULL (may be y itself)
  int *status;            // device-visible error word
  int *flags;             // per output tile: the stream-K hand-off
  int N, K, T;
  int tiles_n;            // row tiles (the fast index of a tile number)
  int ks;                 // K stages per tile
  int dp_waves;           // whole-tile waves before the stream-K tiles
  int mma_n;              // tokens per MMA: 256, or the tokens rounded up to 16
                          // when they fit one tile (a decode batch)
  long long units;        // stream-K stages: (tiles - dp_waves * grid) * ks
};

// first stream-K unit of CTA c's contiguous share
__device__ __forceinline__ long long range_begin(const GemmArgs &p, int c) {
  return p.units * c / gridDim.x;
}

// The parts (tile, K stages k0..k1) a CTA computes, in order; every role
// walks the same sequence.
struct PartIter {
  int q = 0;           // whole tiles taken
  long long u, u_end;  // stream-K share
  __device__ explicit PartIter(const GemmArgs &p)
      : u(range_begin(p, blockIdx.x)), u_end(range_begin(p, blockIdx.x + 1)) {}
  __device__ bool next(const GemmArgs &p, int &tile, int &k0, int &k1) {
    if (q < p.dp_waves) {
      tile = blockIdx.x + q * gridDim.x;
      k0 = 0;
      k1 = p.ks;
      ++q;
      return true;
    }
    if (u >= u_end) return false;
    tile = p.dp_waves * gridDim.x + (int)(u / p.ks);
    k0 = (int)(u % p.ks);
    k1 = (int)(u_end - u < (long long)(p.ks - k0) ? k0 + (u_end - u) : p.ks);
    u += k1 - k0;
    return true;
  }
};

__device__ __forceinline__ bool flag_wait_bounded(const int *f, int *status) {
  const unsigned long long t0 = global_ns();
  for (;;) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v != 0) return true;
    if (global_ns() - t0 > kWaitBudgetNs) {
      atomicExch(status, MLM_ERR_TIMEOUT);
      return false;
    }
    __nanosleep(128);
  }
}

__device__ __forceinline__ void epilogue_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(32 * kDqWarps) : "memory");
}

__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap *map, int x, int y,
                                      uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Two consecutive Q4_K elements (the low and high nibble of one byte) to a
// bf16 pair, bit-identical to rounding __fsub_rn(__fmul_rn(fs, q), fm): each
// nibble sits in the mantissa of 2^23 (a byte permute), 2^23 is subtracted
// exactly, and one fma gives fs*q - fm with a single rounding because fs*q
// (at most 11 + 6 + 4 significant bits) is exact in fp32.  Two packed fp32x2
// operations and a pack to bf16x2: no integer-to-float conversion.
__device__ __forceinline__ uint32_t q4k_pair_bf16(uint32_t lo_bits, uint32_t hi_bits,
                                                  uint64_t fs2, uint64_t nfm2) {
  uint32_t out;
  asm("{\n .reg .b64 t;\n .reg .f32 lo, hi;\n"
      " mov.b64 t, {%1, %2};\n"
      " add.rn.f32x2 t, t, %3;\n"
      " fma.rn.f32x2 t, t, %4, %5;\n"
      " mov.b64 {lo, hi}, t;\n"
      " cvt.rn.bf16x2.f32 %0, hi, lo;\n}"
      : "=r"(out)
      : "r"(lo_bits), "r"(hi_bits), "l"(0xCB000000CB000000ull), "l"(fs2), "l"(nfm2));
  return out;
}

__device__ __forceinline__ uint64_t f32x2_splat(float v) {
  const uint64_t b = __float_as_uint(v);
  return b | (b << 32);
}

__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// kDense: W is already bf16 [N][K] (a weight dequantized ahead of the call):
// the TMA warp loads each stage's A tile (256 rows x 32, the same 64-byte
// swizzle) beside the X tile, and the dequantizing warps only run the
// epilogues.
template <bool kDense>
__global__ void __launch_bounds__(kGemmThreads, 1)
    q4k_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_x, GemmArgs p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t bar = sbase + kOffBar;
  const uint32_t wfull = bar + 8 * kBarWfull, wempty = bar + 8 * kBarWempty,
                 bfull = bar + 8 * kBarBfull, afull = bar + 8 * kBarAfull,
                 sempty = bar + 8 * kBarSempty, done = bar + 8 * kBarDone,
                 accfree = bar + 8 * kBarAccFree;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffBar + kNumBars * 8);
  volatile int *flag_verdict = reinterpret_cast<volatile int *>(smem + kOffBar + kNumBars * 8 + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(wfull + 8 * i, 1);
      mbar_init(wempty + 8 * i, kDqWarps);
    }
    for (int i = 0; i < kGemmStages; ++i) {
      mbar_init(bfull + 8 * i, 1);
      mbar_init(afull + 8 * i, kDense ? 1 : kWarpsPerGroup);
      mbar_init(sempty + 8 * i, 1);
    }
    mbar_init(done, 1);
    mbar_init(accfree, kDqWarps);
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
    if (lane == 0) {
      uint32_t it = 0, wl = 0;  // stages and W block columns issued
      bool ok = true;
      PartIter parts(p);
      int tile, k0, k1;
      while (ok && parts.next(p, tile, k0, k1)) {
        const int n0 = (tile % p.tiles_n) * kGemmRows, t0 = (tile / p.tiles_n) * kGemmTok;
        for (int k = k0; k < k1; ++k) {
          if (!kDense && (k == k0 || k % kStagesPerBlock == 0)) {
            const uint32_t wb = wl & 1;
            if (wl >= 2 && !mbar_wait_bounded(wempty + 8 * wb, ((wl >> 1) - 1) & 1, p.status)) {
              ok = false;
              break;
            }
            mbar_expect_tx(wfull + 8 * wb, kWpk);
            tma2d(sbase + kOffW + wb * kWpk, &tmap_w, (k / kStagesPerBlock) * kBlockBytes, n0,
                  wfull + 8 * wb);
            ++wl;
          }
          const uint32_t s = it % kGemmStages;
          if (it >= (uint32_t)kGemmStages &&
              !mbar_wait_bounded(sempty + 8 * s, (it / kGemmStages - 1) & 1, p.status)) {
            ok = false;
            break;
          }
          if (kDense) {  // A: rows n0 .. n0 + 255 (past the end: zeros)
            mbar_expect_tx(afull + 8 * s, kAStage);
            tma2d(sbase + kOffA + s * kAStage, &tmap_w, k * kGemmKStep, n0, afull + 8 * s);
          }
          mbar_expect_tx(bfull + 8 * s, p.mma_n * kGemmKStep * 2);
          tma2d(sbase + kOffB + s * kBStage, &tmap_x, k * kGemmKStep, t0, bfull + 8 * s);
          ++it;
        }
      }
      // copies in flight land before shared memory is released
      for (uint32_t i = it > (uint32_t)kGemmStages ? it - kGemmStages : 0; i < it; ++i)
        if (!mbar_wait_bounded(bfull + 8 * (i % kGemmStages), (i / kGemmStages) & 1, p.status))
          break;
      for (uint32_t w = wl > 2 ? wl - 2 : 0; w < wl; ++w)
        if (!mbar_wait_bounded(wfull + 8 * (w & 1), (w >> 1) & 1, p.status)) break;
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------
    if (lane == 0) {
      uint32_t it = 0, seg = 0;
      bool ok = true;
      PartIter parts(p);
      int tile, k0, k1;
      while (ok && parts.next(p, tile, k0, k1)) {
        // the accumulator is free once the previous part's epilogue read it
        if (seg > 0 && !mbar_wait_bounded(accfree, (seg - 1) & 1, p.status)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        for (int k = k0; k < k1; ++k) {
          const uint32_t s = it % kGemmStages, ph = (it / kGemmStages) & 1;
          if (!mbar_wait_bounded(afull + 8 * s, ph, p.status) ||
              !mbar_wait_bounded(bfull + 8 * s, ph, p.status)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = sbase + kOffA + s * kAStage;
          const uint32_t b_addr = sbase + kOffB + s * kBStage;
#pragma unroll
          for (int k16 = 0; k16 < kGemmKStep / 16; ++k16) {
            const uint64_t bdesc = sw64_desc(b_addr + 32 * k16);
            const uint32_t acc = (k > k0 || k16 > 0) ? 1u : 0u;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint64_t adesc = sw64_desc(a_addr + h * kAHalf + 32 * k16);
              asm volatile(
                  "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                  " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(
                      tmem + h * kGemmTok),
                  "l"(adesc), "l"(bdesc), "r"(idesc_for(p.mma_n)), "r"(acc)
                  : "memory");
            }
          }
          // stage s is free once these MMAs have read it
          asm volatile(
              "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                  sempty + 8 * s)
              : "memory");
          ++it;
        }
        if (!ok) break;
        asm volatile(
            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                done)
            : "memory");
        ++seg;
      }
    }
  } else {
    // ---- dequantize (thread = weight rows r and r + 128), then each part's
    // epilogue; a warp reaches TMEM lanes 32 (warp % 4) .. 32 (warp % 4) + 31
    const int quarter = warp & 3;
    const int group = (warp - 2) / kWarpsPerGroup;
    // with one row per thread, the warp's rows lie in accumulator h_one
    const int h_one = ((warp - 2) >> 2) & 1;
    const int r = quarter * 32 + lane;  // row within an accumulator, 0..127
    const uint32_t tq = tmem + ((uint32_t)(quarter * 32) << 16);
    bool ok = true;
    uint32_t it = 0, wl = 0, seg = 0;
    int waited_w = -1;
    PartIter parts(p);
    int tile, k0, k1;
    while (parts.next(p, tile, k0, k1)) {
      for (int k = k0; k < k1 && !kDense; ++k) {
        if (k == k0 || k % kStagesPerBlock == 0) {
          // done with the previous W block column (whether or not this warp
          // had a stage in it)
          if (wl > 0) {
            __syncwarp();
            if (lane == 0) mbar_arrive1(wempty + 8 * ((wl - 1) & 1));
          }
          ++wl;
        }
        if ((int)(it % kDqGroups) == group) {
          const uint32_t s = it % kGemmStages, wb = (wl - 1) & 1;
          const int sb = k % kStagesPerBlock;
          if (ok && waited_w != (int)(wl - 1)) {
            ok = mbar_wait_bounded(wfull + 8 * wb, ((wl - 1) >> 1) & 1, p.status);
            waited_w = (int)(wl - 1);
          }
          if (ok && it >= (uint32_t)kGemmStages)
            ok = mbar_wait_bounded(sempty + 8 * s, (it / kGemmStages - 1) & 1, p.status);
          ok = __all_sync(0xFFFFFFFFu, ok);
          if (ok) {
#pragma unroll
            for (int rp = 0; rp < kRowsPerThread; ++rp) {
              const int h = kRowsPerThread == 2 ? rp : h_one;
              const uint8_t *blk = smem + kOffW + wb * kWpk + (h * kMmaM + r) * kBlockBytes;
              const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
              const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
              int sc, m;
              q4k_scale_min_regs(sb, hd.y, hd.z, hd.w, sc, m);
              const uint64_t fs = f32x2_splat(d * (float)sc),
                             nfm = f32x2_splat(-(dmin * (float)m));
              // sub-block sb: elements 32 sb .. 32 sb + 31 are qs bytes 16 sb .. 16 sb + 15
              const uint4 q = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * sb);
              const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
              uint8_t *arow = smem + kOffA + s * kAStage + h * kAHalf + (r >> 3) * 512 + (r & 7) * 64;
#pragma unroll
              for (int c = 0; c < 4; ++c) {  // elements 8c .. 8c+7 = qs word c
                const uint32_t w = qw[c];
                const uint32_t lo4 = w & 0x0F0F0F0Fu, hi4 = (w >> 4) & 0x0F0F0F0Fu;
                uint32_t o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {  // byte e: elements 2e (low), 2e+1 (high)
                  // bytes (nibble, 0, 0, 0x4B): the fp32 value 2^23 + nibble
                  const uint32_t sel = 0x7540u + e;
                  o[e] = q4k_pair_bf16(__byte_perm(lo4, 0x4B000000u, sel),
                                       __byte_perm(hi4, 0x4B000000u, sel), fs, nfm);
                }
                *reinterpret_cast<uint4 *>(arow + ((c ^ ((r >> 1) & 3)) << 4)) =
                    make_uint4(o[0], o[1], o[2], o[3]);
              }
            }
            // generic-proxy writes become visible to the tensor cores' reads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          }
          __syncwarp();
          if (lane == 0) mbar_arrive1(afull + 8 * s);
        }
        ++it;
      }

      // ---- epilogue of this part: Y tile (n0.., t0..), K stages k0..k1 ----
      const bool tail = k1 == p.ks, whole = tail && k0 == 0;
      const int n0 = (tile % p.tiles_n) * kGemmRows, t0 = (tile / p.tiles_n) * kGemmTok;
      bool go = __all_sync(0xFFFFFFFFu, ok && mbar_wait_bounded(done, seg & 1, p.status));
      if (!tail) {  // wait until the tail part has stored its share
        if (warp == 2 && lane == 0) *flag_verdict = go && flag_wait_bounded(p.flags + tile, p.status);
        epilogue_bar();
        go = go && *flag_verdict != 0;
      }
      if (go) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        constexpr int kCols = kGemmTok / kDqGroups;
        const int col_end = min((group + 1) * kCols, p.mma_n);
#pragma unroll 1
        for (int rp = 0; rp < kRowsPerThread; ++rp) {
          const int h = kRowsPerThread == 2 ? rp : h_one;
          const int n = n0 + h * kMmaM + r;
          for (int col = group * kCols; col < col_end; col += 8) {
            uint32_t v[8];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                  "=r"(v[6]), "=r"(v[7])
                : "r"(tq + h * kGemmTok + col));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (n < p.N) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int t = t0 + col + i;
                if (t < p.T) {
                  float *dst = p.y + (size_t)t * p.N + n;
                  if (!tail)
                    atomicAdd(dst, __uint_as_float(v[i]));
                  else
                    *dst = __uint_as_float(v[i]) +
                           (p.residual ? p.residual[(size_t)t * p.N + n] : 0.f);
                }
              }
            }
          }
        }
      }
      // the accumulator may be overwritten by the next part
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive1(accfree);
      if (tail && !whole) {
        // publish: every epilogue thread's stores, then the flag
        __threadfence();
        epilogue_bar();
        if (warp == 2 && lane == 0 && go) {
          // CTAs before this one whose stream-K shares start inside the tile
          const long long first = (long long)(tile - p.dp_waves * (int)gridDim.x) * p.ks;
          int others = 0;
          for (int c = blockIdx.x; c > 0 && range_begin(p, c) > first; --c) ++others;
          asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p.flags + tile), "r"(others)
                       : "memory");
        }
      } else if (!tail && go && warp == 2 && lane == 0) {
        atomicSub(p.flags + tile, 1);  // this part has been counted
      }
      ++seg;
    }
    // the last W block column's buffer is released (balances the arrivals)
    if (!kDense && wl > 0) {
      __syncwarp();
      if (lane == 0) mbar_arrive1(wempty + 8 * ((wl - 1) & 1));
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

// output tiles a launch may have (the hand-off flags are allocated once):
// 65536 x 128 x 256, e.g. 57344 rows x 16384 tokens needs 28672
constexpr int kGemmMaxTiles = 65536;

int gemm_init(mlm_ctx *ctx) {
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q4k_gemm_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
  MLM_CUDA_TRY(ctx, cudaFuncSetAttribute(q4k_gemm_kernel<true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmem));
  if (!ctx->gemm_flags) {
    MLM_CUDA_TRY(ctx, cudaMalloc(&ctx->gemm_flags, sizeof(int) * kGemmMaxTiles));
    MLM_CUDA_TRY(ctx, cudaMemset(ctx->gemm_flags, 0, sizeof(int) * kGemmMaxTiles));
    ctx->gemm_max_tiles = kGemmMaxTiles;
  }
  return MLM_OK;
}

}  // namespace mlm

using namespace mlm;

namespace mlm {
// dense: W is bf16 [rows][cols] instead of Q4_K blocks
static int gemm_launch_impl(mlm_ctx *ctx, const void *W, bool dense, int rows, int cols,
                            const void *x_bf16, int tokens, float *y, const float *residual,
                            cudaStream_t stream) {
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
  // a single token tile (a decode batch, a short prompt) multiplies only its
  // tokens, rounded up to the MMA's N granularity of 16
  const int mma_n = tokens <= kGemmTok ? (tokens + 15) / 16 * 16 : kGemmTok;
  const int nb = cols / kQK;
  CUtensorMap mw, mx;
  if (dense) {  // 32 x 256-row bf16 tiles in the 64-byte swizzle of the X tiles
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kGemmKStep, (cuuint32_t)kGemmRows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(W), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MLM_REQUIRE(ctx, r == CUDA_SUCCESS, MLM_ERR_CUDA, "gemm: bf16 W tensor map (%d)", (int)r);
  } else {
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
    const cuuint32_t box[2] = {(cuuint32_t)kGemmKStep, (cuuint32_t)mma_n};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x_bf16),
                        dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MLM_REQUIRE(ctx, r == CUDA_SUCCESS, MLM_ERR_CUDA, "mlm_q4k_gemm: X tensor map (%d)", (int)r);
  }
  const int tiles_n = (rows + kGemmRows - 1) / kGemmRows;
  const int tiles_t = (tokens + kGemmTok - 1) / kGemmTok;
  MLM_REQUIRE(ctx, (long long)tiles_n * tiles_t <= ctx->gemm_max_tiles, MLM_ERR_SHAPE,
              "mlm_q4k_gemm: %d x %d output tiles exceed %d", tiles_n, tiles_t,
              ctx->gemm_max_tiles);
  GemmArgs a;
  a.y = y;
  a.residual = residual;
  a.status = ctx->dev_status;
  a.flags = ctx->gemm_flags;
  a.N = rows;
  a.K = cols;
  a.T = tokens;
  a.tiles_n = tiles_n;
  a.mma_n = mma_n;
  a.ks = nb * kStagesPerBlock;
  const long long tiles = (long long)tiles_n * tiles_t;
  // one persistent CTA per SM, each with at least kMinUnitsPerCta stages
  const long long ctas = std::min<long long>(
      ctx->sm_count, (tiles * a.ks + kMinUnitsPerCta - 1) / kMinUnitsPerCta);
  // whole-tile waves, leaving between one and two waves' worth to stream-K
  a.dp_waves = (int)std::max<long long>(0, tiles / ctas - 1);
  a.units = (tiles - (long long)a.dp_waves * ctas) * a.ks;
  if (dense)
    q4k_gemm_kernel<true><<<(unsigned)ctas, kGemmThreads, kGemmSmem, stream>>>(mw, mx, a);
  else
    q4k_gemm_kernel<false><<<(unsigned)ctas, kGemmThreads, kGemmSmem, stream>>>(mw, mx, a);
  return check_launch(ctx, "mlm_q4k_gemm");
}

int gemm_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16, int tokens,
                float *y, const float *residual, cudaStream_t stream) {
  return gemm_launch_impl(ctx, W, false, rows, cols, x_bf16, tokens, y, residual, stream);
}

int gemm_dense_launch(mlm_ctx *ctx, const void *W_bf16, int rows, int cols, const void *x_bf16,
                      int tokens, float *y, const float *residual, cudaStream_t stream) {
  return gemm_launch_impl(ctx, W_bf16, true, rows, cols, x_bf16, tokens, y, residual, stream);
}

// A Q6_K weight in the prompt pass: dequantized to bf16 (the fp32 value
// rounded once) into the caller's scratch, then the GEMM on it.
int q6k_gemm_launch(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                    int tokens, float *y, const float *residual, void *scratch_bf16,
                    cudaStream_t stream) {
  MLM_REQUIRE(ctx, W && scratch_bf16, MLM_ERR_ARG, "mlm_q6k_gemm: null buffer");
  MLM_REQUIRE(ctx, aligned16(scratch_bf16), MLM_ERR_ALIGN, "mlm_q6k_gemm: scratch alignment");
  int st = q6k_dequant_bf16_launch(ctx, W, scratch_bf16, (uint64_t)rows * cols, stream);
  if (st != MLM_OK) return st;
  return gemm_dense_launch(ctx, scratch_bf16, rows, cols, x_bf16, tokens, y, residual, stream);
}
}  // namespace mlm

extern "C" int mlm_q4k_gemm(mlm_ctx *ctx, const void *W, int rows, int cols, const void *x_bf16,
                            int tokens, float *y, const float *residual) {
  MLM_CHECK_CTX(ctx);
  MLM_REQUIRE(ctx, !residual || aligned4(residual), MLM_ERR_ALIGN, "mlm_q4k_gemm: residual");
  return gemm_launch(ctx, W, rows, cols, x_bf16, tokens, y, residual, ctx->stream);
}
