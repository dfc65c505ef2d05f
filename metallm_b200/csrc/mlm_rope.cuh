// mlm_rope.cuh -- RoPE angle of a rotation pair (calculate_rope_yarn,
// PositionalEmbeddingsKernels.metal:106-124): theta = pos * base^(-i0/n_dims)
// / freq_factor, optional YaRN blend; cos/sin from a double-precision
// sincos so that large angles keep full fp32 accuracy.
#pragma once

#include <cmath>

#include "../../include/metallm_cuda.h"

namespace mlm {

struct RopeConsts {
  float inv_ndims;
  float corr0, corr1;
};

__host__ __device__ inline float yarn_corr_factor(int n_dims, int n_ctx_orig, float n_rot,
                                                  float base) {
  if (n_rot <= 0.0f || base <= 0.0f || n_ctx_orig <= 0) return 0.0f;
  const float lb = logf(base);
  if (fabsf(lb) < 1e-6f) return 0.0f;
  const float term = (float)n_ctx_orig / (n_rot * 2.0f * 3.14159265358979323846f);
  if (term <= 0.0f) return 0.0f;
  return (float)n_dims * logf(term) / (2.0f * lb);
}

inline RopeConsts rope_consts(const mlm_rope_args &a) {
  RopeConsts c;
  c.inv_ndims = -1.0f / (float)a.n_dims;
  const float fast = yarn_corr_factor((int)a.n_dims, a.n_ctx_orig, a.beta_fast, a.freq_base);
  const float slow = yarn_corr_factor((int)a.n_dims, a.n_ctx_orig, a.beta_slow, a.freq_base);
  float c0 = floorf(fast);
  if (c0 < 0.0f) c0 = 0.0f;
  float c1 = ceilf(slow);
  if (c1 < c0) c1 = c0;
  if (c1 > (float)a.n_dims - 2.0f) c1 = (float)a.n_dims - 2.0f;
  c.corr0 = c0;
  c.corr1 = c1;
  return c;
}

// cos/sin of pair p at position pos (calculate_rope_yarn)
__device__ __forceinline__ void rope_cos_sin(const mlm_rope_args &a, const RopeConsts &k,
                                             const float *freqs, int pos, int p, float &c,
                                             float &s) {
  const int i0 = 2 * p;
  const float theta_extrap = (float)pos * powf(a.freq_base, k.inv_ndims * (float)i0);
  const float ff = a.has_freq_factors ? freqs[p] : 1.0f;
  const float theta_scaled = theta_extrap / fmaxf(0.0001f, ff);
  const float theta_interp = a.freq_scale * theta_scaled;
  float theta = theta_interp;
  float mscale = a.attn_factor;
  if (a.ext_factor != 0.0f) {
    const float diff = fmaxf(0.001f, k.corr1 - k.corr0);
    const float y = ((float)i0 / 2.0f - k.corr0) / diff;
    const float ramp = 1.0f - fminf(1.0f, fmaxf(0.0f, y));
    const float mix = ramp * a.ext_factor;
    theta = theta_interp * (1.0f - mix) + theta_scaled * mix;
    if (a.freq_scale > 0.0f) mscale *= (1.0f + 0.1f * logf(1.0f / a.freq_scale));
  }
  double sd, cd;
  sincos((double)theta, &sd, &cd);
  c = (float)cd * mscale;
  s = (float)sd * mscale;
}

}  // namespace mlm
