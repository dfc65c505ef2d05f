// mlm_device.cuh -- device helpers: Q4_K block layout, scale/min unpack,
// the seeded counter-based generator, and small warp utilities.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mlm {

constexpr int kQK = 256;          // elements per Q4_K super-block
constexpr int kBlockBytes = 144;  // bytes per Q4_K super-block
constexpr int kSubBlocks = 8;     // 32-element sub-blocks per super-block

// ---- counter-based generator (identical arithmetic to the CPU oracle) -----
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t rng_u64(uint64_t seed, uint64_t stream,
                                                     uint64_t idx) {
  uint64_t s = mix64(seed + 0x9E3779B97F4A7C15ULL * (stream + 1));
  return mix64(s ^ (idx * 0xD1B54A32D192ED03ULL + 0x632BE59BD9B4E019ULL));
}

// Irwin-Hall(12) - 6: an approximately standard normal value built from
// integer sums, so host and device agree bit for bit.
__host__ __device__ __forceinline__ double rng_normal(uint64_t seed, uint64_t stream,
                                                      uint64_t idx) {
  uint64_t sum = 0;
  for (int k = 0; k < 6; ++k) {
    uint64_t r = rng_u64(seed, stream, idx * 6 + (uint64_t)k);
    sum += (r & 0xffffffffULL) + (r >> 32);
  }
  return (double)sum * (1.0 / 4294967296.0) - 6.0;
}

constexpr uint64_t kTagBytes = 0x51ULL;

// ---- Q4_K scale / min unpack (get_scale_min_k4, DequantKernels.metal:43-56)
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *s, int &sc, int &m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// Same unpack from the header words of a block held in registers:
// w1 = scales[0..3], w2 = scales[4..7], w3 = scales[8..11].
__device__ __forceinline__ void q4k_scale_min_regs(int j, uint32_t w1, uint32_t w2,
                                                   uint32_t w3, int &sc, int &m) {
  const int jj = (j & 3) * 8;
  const uint32_t s1 = (w1 >> jj) & 0xFF, s2 = (w2 >> jj) & 0xFF, s3 = (w3 >> jj) & 0xFF;
  if (j < 4) {
    sc = s1 & 63;
    m = s2 & 63;
  } else {
    sc = (s3 & 0xF) | ((s1 >> 6) << 4);
    m = (s3 >> 4) | ((s2 >> 6) << 4);
  }
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

// Programmatic dependent launch (see launch_pdl): wait for the preceding
// kernel's completion and memory, then let the next kernel be scheduled.
// Both are no-ops in a grid that was not launched as a dependent.
__device__ __forceinline__ void pdl_wait_then_release() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- RMSNorm pieces (NormalizationKernels.metal:31-79) ---------------------
// scale = min(1 / sqrt(max(mean(x^2), 1e-10) + eps), 1e6)
__device__ __forceinline__ float rms_scale(float sum_sq, int n, float eps) {
  const float mean_sq = sum_sq / (float)n;
  const float safe = fmaxf(mean_sq, 1e-10f);
  const float rms = sqrtf(safe + eps);
  return fminf(1.0f / rms, 1e6f);
}
// NaN / Inf weights read as 1
__device__ __forceinline__ float safe_weight(float w) {
  return (isnan(w) || isinf(w)) ? 1.0f : w;
}
// round an fp32 value to the storage type of an output (round to nearest even)
template <class T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ __half from_float<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// SiLU-gated product of the decode FFN (kernel_silu_f16 then kernel_mul_f16,
// ActivationKernels.metal:6-27, in fp32)
__device__ __forceinline__ float swiglu(float g, float u) {
  return g * (1.0f / (1.0f + expf(-g))) * u;
}

// Exponent e of the scaled fp16 form of a 32-element sub-block whose largest
// magnitude is m: its values are stored as fp16(v * 2^-e) with scale 2^e, so
// the largest stays below 2^15 (e = 0 when it already does).
__device__ __forceinline__ int silu_scale_exp(float m) {
  return max(0, (int)((__float_as_uint(m) >> 23) & 0xFF) - 127 - 14);
}

// 128-bit streaming load that does not allocate in L1 (weights are read once)
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void stg_stream(void *p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

}  // namespace mlm
