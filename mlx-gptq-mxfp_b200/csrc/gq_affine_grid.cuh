// Warp-cooperative MLX affine grid: the MSE range-shrink clip search and the
// quantize step, shared by the RTN kernel and the GPTQ column loop.
//
// A warp owns one group of G = 32 * VPL consecutive values; lane l holds
// elements l, l + 32, l + 64, ... in v[0..VPL).
#pragma once

#include "gq_common.cuh"

namespace gq {

constexpr int kMaxShrinks = 21;  // grid_steps + 1 with grid_steps = 20 (grid.py:172)

// Shrink factors of choose_qparams (grid.py:192, 198-199): p_i = 1 - 0.2*i/20
// evaluated in double exactly as Python does, then cast to float32 the way torch
// casts a Python scalar multiplied into a float32 tensor: pr = f32(p/maxq), pf = f32(p).
__device__ __forceinline__ void shrink_factors(int i, int bits, float& pr, float& pf) {
  double maxq = double((1 << bits) - 1);
  double p = 1.0 - 0.2 * double(i) / 20.0;
  pr = __double2float_rn(p / maxq);
  pf = __double2float_rn(p);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, o);
  return x;
}
__device__ __forceinline__ float warp_min(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fminf(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
  return x;
}
__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
  return x;
}

// quantize_with_params for one value (grid.py:215-221): q = clamp(rne((w-b)/s_safe), 0, maxq),
// dq = q*s + b, with s_safe = 1 where |s| < 1e-12.
__device__ __forceinline__ float affine_quant(float w, float s, float b, float maxq, float& q) {
  float ss = fabsf(s) < 1e-12f ? 1.0f : s;
  q = fminf(fmaxf(rintf((w - b) / ss), 0.0f), maxq);
  return q * s + b;
}

// choose_qparams over one warp-held group (grid.py:167-212). All lanes return the
// same (s, b): the storage-rounded scale and bias as float32. Candidate errors are
// butterfly-reduced, which gives every lane bit-identical sums; the first minimum
// wins (strict <), as in the reference.
// pr/pf: shrink factors for this bit width (shared memory), nshrink = 21 for mse, 1 for minmax.
template <int VPL>
__device__ __forceinline__ void warp_choose_qparams(const float (&v)[VPL], float maxq, const float* pr,
                                                    const float* pf, int nshrink, int storage, float& s_best,
                                                    float& b_best) {
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int k = 1; k < VPL; ++k) {
    mn = fminf(mn, v[k]);
    mx = fmaxf(mx, v[k]);
  }
  mn = warp_min(mn);
  mx = warp_max(mx);
  const float rng = mx - mn;
  float best = 0.0f;
  for (int i = 0; i < nshrink; ++i) {
    const float s = round_storage(rng * pr[i], storage);
    const float b = round_storage(mn * pf[i], storage);
    float err = 0.0f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      float q;
      const float d = affine_quant(v[k], s, b, maxq, q) - v[k];
      err = fmaf(d, d, err);
    }
    err = warp_sum(err);
    if (i == 0 || err < best) {
      best = err;
      s_best = s;
      b_best = b;
    }
  }
}

__device__ __forceinline__ float load_any(const void* base, int64_t idx, int dtype) {
  if (dtype == GQ_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  if (dtype == GQ_F16) return __half2float(reinterpret_cast<const __half*>(base)[idx]);
  return reinterpret_cast<const float*>(base)[idx];
}

__device__ __forceinline__ void store_any(void* base, int64_t idx, float v, int dtype) {
  if (dtype == GQ_BF16)
    reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  else if (dtype == GQ_F16)
    reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(base)[idx] = v;
}

}  // namespace gq
