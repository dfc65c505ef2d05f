// q4k_gemv_common.cuh -- device pieces shared by the Q4_K GEMV kernels:
// the tensor-core MMA, cache policies, bounded mbarrier waits and the split
// of a weight's units over CTAs.
#pragma once

#include "../../include/metallm_cuda.h"
#include "mlm_device.cuh"

namespace mlm {

constexpr int kTileRows = 32;  // rows per tile (two m16 MMA tiles)
constexpr unsigned long long kWaitBudgetNs = 200ull * 1000 * 1000;  // 200 ms

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One box of W (144 bytes of each of its rows at byte column x, from row y)
// into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_unit(uint32_t dst, const CUtensorMap *tmap, int x, int y,
                                         uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(pol)
      : "memory");
}

// Weights are read exactly once: copy them with an L2 evict-first policy so
// they do not push x, y and the KV cache out of L2.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// try_wait suspends the thread until the phase completes or the hint (ns)
// elapses, so a waiting warp does not spin on the issue slots
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(bar), "r"(phase), "r"(1000000u)
      : "memory");
  return done != 0;
}
// Bounded wait for a stage: gives up after kWaitBudgetNs and reports it.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t phase, int *status) {
  if (mbar_try_wait(bar, phase)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, phase)) {
    if (global_ns() - t0 > kWaitBudgetNs) {
      atomicExch(status, MLM_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// first unit of CTA c, and the CTA whose range holds unit u
// (all products stay below 2^31: checked on the host)
template <class A>
__device__ __forceinline__ int unit_begin(int c, const A &p) {
  return (c * p.units) / p.ctas;
}
template <class A>
__device__ __forceinline__ int cta_of_unit(int u, const A &p) {
  return ((u + 1) * p.ctas - 1) / p.units;
}
template <class A>
__device__ __forceinline__ int div_nb(int u, const A &p) {
  return (int)(((unsigned long long)(unsigned)u * p.nb_magic) >> 40);
}

// The CTA's units [u0, u1) in processing order: its first tile when shared
// with the previous CTA, its last tile when shared with the next, then the
// interior.  q is the position in that order.
struct CtaOrder {
  int u0, u1, S, nf, nl, t_first, t_last;
  __device__ __forceinline__ int unit_of(int q) const {
    if (q < nf) return u0 + q;
    if (q < nf + nl) return u1 - nl + (q - nf);
    return u0 + q - nl;
  }
  // queue positions [qa, qb) of tile t's units in this CTA
  __device__ __forceinline__ void tile_range(int t, int nb, int &qa, int &qb) const {
    const int a = max(u0, t * nb), b = min(u1, (t + 1) * nb);
    if (t == t_first && nf > 0) {
      qa = a - u0;
      qb = b - u0;
    } else if (t == t_last && nl > 0) {
      qa = nf + (a - (u1 - nl));
      qb = nf + (b - (u1 - nl));
    } else {
      qa = a - u0 + nl;
      qb = b - u0 + nl;
    }
  }
};

}  // namespace mlm
