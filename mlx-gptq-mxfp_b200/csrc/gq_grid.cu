// Data-free grids and packing: RTN affine / MXFP, dequantization, code packing.
// HBM-bound elementwise work; warps own whole groups so the group reductions
// (min/max/err sums, max |w|) stay in registers and shuffles.
#include "gq_affine_grid.cuh"

namespace gq {

// --------------------------------------------------------------------------
// RTN affine: one warp per (row, group)
// --------------------------------------------------------------------------
template <int VPL>
__global__ void __launch_bounds__(256) rtn_affine_kernel(const void* __restrict__ W, int w_dtype, int64_t rows,
                                                         int64_t C, int bits, int nshrink, int storage,
                                                         uint8_t* __restrict__ q, void* __restrict__ scales,
                                                         void* __restrict__ biases, void* __restrict__ w_dq,
                                                         int wdq_dtype) {
  __shared__ float pr[kMaxShrinks], pf[kMaxShrinks];
  if (threadIdx.x < kMaxShrinks) shrink_factors(threadIdx.x, bits, pr[threadIdx.x], pf[threadIdx.x]);
  __syncthreads();
  constexpr int G = 32 * VPL;
  const int lane = threadIdx.x & 31;
  const int64_t ngroups = C / G;
  const int64_t gw = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= rows * ngroups) return;
  const int64_t r = gw / ngroups, g = gw % ngroups;
  const int64_t base = r * C + g * G;
  float v[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) v[k] = load_any(W, base + lane + 32 * k, w_dtype);
  const float maxq = float((1 << bits) - 1);
  float s, b;
  warp_choose_qparams<VPL>(v, maxq, pr, pf, nshrink, storage, s, b);
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    float qq;
    float dq = affine_quant(v[k], s, b, maxq, qq);
    q[base + lane + 32 * k] = uint8_t(qq);
    if (w_dq) store_any(w_dq, base + lane + 32 * k, dq, wdq_dtype);
  }
  if (lane == 0) {
    store_any(scales, r * ngroups + g, s, storage);
    store_any(biases, r * ngroups + g, b, storage);
  }
}

// --------------------------------------------------------------------------
// RTN MXFP: one warp per (row, 32-group), lane per element
// --------------------------------------------------------------------------
template <int MODE>
__global__ void __launch_bounds__(256) rtn_mxfp_kernel(const void* __restrict__ W, int w_dtype, int64_t ngroups_total,
                                                       uint8_t* __restrict__ q, uint8_t* __restrict__ q_packed,
                                                       uint8_t* __restrict__ scales, void* __restrict__ w_dq,
                                                       int wdq_dtype) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= ngroups_total) return;
  const int64_t idx = gw * 32 + lane;
  const float w = load_any(W, idx, w_dtype);
  const float amax = warp_max(fabsf(w));
  const int e = mx_scale_exponent(amax, MODE == GQ_MXFP4 ? 6.0f : 448.0f);
  float dq, unused;
  const uint32_t code = mx_quant2<MODE>(w, 0.0f, exp2i(-e), exp2i(e), dq, unused) & (MODE == GQ_MXFP4 ? 0xFu : 0xFFu);
  q[idx] = uint8_t(code);
  if (MODE == GQ_MXFP4 && q_packed) {
    uint32_t hi = __shfl_down_sync(0xFFFFFFFFu, code, 1);
    if ((lane & 1) == 0) q_packed[idx >> 1] = uint8_t(code | (hi << 4));
  }
  if (w_dq) store_any(w_dq, idx, dq, wdq_dtype);
  if (lane == 0) scales[gw] = uint8_t(e + 127);
}

// --------------------------------------------------------------------------
// dequantize_artifact
// --------------------------------------------------------------------------
__global__ void dequant_kernel(const uint8_t* __restrict__ q, const void* __restrict__ scales,
                               const void* __restrict__ biases, int scale_dtype, int64_t n, int64_t C, int mode,
                               int G, float* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t r = i / C, c = i % C;
  const int64_t gi = r * (C / G) + c / G;
  const uint32_t code = q[i];
  float v;
  if (mode == GQ_AFFINE) {
    v = float(code) * load_any(scales, gi, scale_dtype) + load_any(biases, gi, scale_dtype);
  } else {
    const float sc = exp2i(int(reinterpret_cast<const uint8_t*>(scales)[gi]) - 127);
    v = (mode == GQ_MXFP4 ? e2m1_value(code & 15u) : e4m3_decode(code)) * sc;
  }
  out[i] = v;
}

// --------------------------------------------------------------------------
// packing
// --------------------------------------------------------------------------
__global__ void pack_q_kernel(const uint8_t* __restrict__ q, int64_t nwords, int bits, uint32_t* __restrict__ words) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nwords) return;
  const int per = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  uint32_t w = 0;
  for (int k = 0; k < per; ++k) w |= (uint32_t(q[i * per + k]) & mask) << (bits * k);
  words[i] = w;
}

// Vectorized forms (q and the output 16-byte aligned): every thread turns 16 x BITS/2
// code bytes into four words (one 16-byte store), or 16 codes into 8 nibble bytes and
// back; the scalar kernels above finish any remainder.
template <int BITS>
__device__ __forceinline__ uint32_t pack_word(const uint8_t* b) {  // 32/BITS codes, LSB first
  constexpr int per = 32 / BITS;
  constexpr uint32_t mask = (1u << BITS) - 1u;
  uint32_t w = 0;
#pragma unroll
  for (int k = 0; k < per; ++k) w |= (uint32_t(b[k]) & mask) << (BITS * k);
  return w;
}

template <int BITS>
__global__ void pack_q_vec_kernel(const uint4* __restrict__ q, int64_t nquads, uint4* __restrict__ words) {
  constexpr int per = 32 / BITS, loads = per / 4;  // uint4 loads per 4 output words
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nquads) return;
  uint4 in[loads];
#pragma unroll
  for (int l = 0; l < loads; ++l) in[l] = q[i * loads + l];
  const uint8_t* b = reinterpret_cast<const uint8_t*>(in);
  words[i] = make_uint4(pack_word<BITS>(b), pack_word<BITS>(b + per), pack_word<BITS>(b + 2 * per),
                        pack_word<BITS>(b + 3 * per));
}

__global__ void pack_nibbles_vec_kernel(const uint4* __restrict__ q, int64_t n16, uint2* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n16) return;
  const uint4 v = q[i];
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
  uint32_t h[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {  // bytes b0..b3 -> (b0 | b1 << 4) | (b2 | b3 << 4) << 8
    const uint32_t x = u[k] & 0xFFFFFFFFu;
    const uint32_t lo = (x & 0xFFu) | ((x >> 4) & 0xFF0u);          // b0 | b1 << 4 (bits 0-11)
    const uint32_t hi = ((x >> 16) & 0xFFu) | ((x >> 20) & 0xFF0u);  // b2 | b3 << 4
    h[k] = (lo & 0xFFu) | ((hi & 0xFFu) << 8);
  }
  out[i] = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
}

__global__ void unpack_nibbles_vec_kernel(const uint2* __restrict__ p, int64_t n8, uint4* __restrict__ q) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const uint2 v = p[i];
  const uint32_t u[2] = {v.x, v.y};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 2; ++k) {  // 4 packed bytes -> 8 code bytes
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t x = (u[k] >> (16 * half)) & 0xFFFFu;  // two packed bytes
      o[2 * k + half] = (x & 0xFu) | ((x & 0xF0u) << 4) | ((x & 0xF00u) << 8) | ((x & 0xF000u) << 12);
    }
  }
  q[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void unpack_q_kernel(const uint32_t* __restrict__ words, int64_t rows, int64_t nw, int bits,
                                int64_t out_cols, uint8_t* __restrict__ q) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * out_cols) return;
  const int per = 32 / bits;
  const int64_t r = i / out_cols, c = i % out_cols;
  const uint32_t w = words[r * nw + c / per];
  q[i] = uint8_t((w >> (bits * (c % per))) & ((1u << bits) - 1u));
}

__global__ void pack_nibbles_kernel(const uint8_t* __restrict__ q, int64_t nbytes, uint8_t* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nbytes) return;
  out[i] = uint8_t(q[2 * i] | (q[2 * i + 1] << 4));
}

__global__ void unpack_nibbles_kernel(const uint8_t* __restrict__ p, int64_t nbytes, uint8_t* __restrict__ q) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nbytes) return;
  const uint8_t b = p[i];
  q[2 * i] = b & 15u;
  q[2 * i + 1] = b >> 4;
}

static inline unsigned blocks_for(int64_t n, int per_block) { return unsigned((n + per_block - 1) / per_block); }

static bool valid_dtype(int d) { return d == GQ_F32 || d == GQ_BF16 || d == GQ_F16; }

}  // namespace gq

using namespace gq;

extern "C" int gq_rtn_affine(const void* W, int w_dtype, int64_t rows, int64_t C, int bits, int group_size, int clip,
                             int storage_dtype, uint8_t* q, void* scales, void* biases, void* w_dq, int wdq_dtype,
                             void* stream) {
  GQ_REQUIRE(valid_dtype(w_dtype) && valid_dtype(storage_dtype) && valid_dtype(wdq_dtype), "gq_rtn_affine: dtype");
  GQ_REQUIRE(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8,
             "gq_rtn_affine: bits %d unsupported", bits);
  GQ_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128 || group_size == 256,
             "gq_rtn_affine: group size %d unsupported (32/64/128/256)", group_size);
  GQ_REQUIRE(rows >= 0 && C >= 0 && C % group_size == 0, "gq_rtn_affine: C=%lld not divisible by group %d",
             (long long)C, group_size);
  GQ_REQUIRE(clip == GQ_CLIP_MSE || clip == GQ_CLIP_MINMAX, "gq_rtn_affine: clip");
  const int64_t nw = rows * (C / group_size);
  if (nw == 0) return GQ_OK;
  GQ_REQUIRE(W && q && scales && biases, "gq_rtn_affine: null pointer");
  const int nshrink = clip == GQ_CLIP_MSE ? kMaxShrinks : 1;
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned grid = blocks_for(nw, 8);
#define LAUNCH(VPL)                                                                                              \
  rtn_affine_kernel<VPL><<<grid, 256, 0, s>>>(W, w_dtype, rows, C, bits, nshrink, storage_dtype, q, scales, biases, \
                                              w_dq, wdq_dtype)
  switch (group_size) {
    case 32: LAUNCH(1); break;
    case 64: LAUNCH(2); break;
    case 128: LAUNCH(4); break;
    default: LAUNCH(8); break;
  }
#undef LAUNCH
  return check_launch("rtn_affine_kernel");
}

extern "C" int gq_rtn_mxfp(const void* W, int w_dtype, int64_t rows, int64_t C, int mode, uint8_t* q,
                           uint8_t* q_packed, uint8_t* scales, void* w_dq, int wdq_dtype, void* stream) {
  GQ_REQUIRE(mode == GQ_MXFP4 || mode == GQ_MXFP8, "gq_rtn_mxfp: not a microscaling mode: %d", mode);
  GQ_REQUIRE(valid_dtype(w_dtype) && valid_dtype(wdq_dtype), "gq_rtn_mxfp: dtype");
  GQ_REQUIRE(rows >= 0 && C >= 0 && C % 32 == 0, "gq_rtn_mxfp: columns %lld not divisible by 32", (long long)C);
  const int64_t ng = rows * (C / 32);
  if (ng == 0) return GQ_OK;
  GQ_REQUIRE(W && q && scales, "gq_rtn_mxfp: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  if (mode == GQ_MXFP4)
    rtn_mxfp_kernel<GQ_MXFP4><<<blocks_for(ng, 8), 256, 0, s>>>(W, w_dtype, ng, q, q_packed, scales, w_dq, wdq_dtype);
  else
    rtn_mxfp_kernel<GQ_MXFP8><<<blocks_for(ng, 8), 256, 0, s>>>(W, w_dtype, ng, q, nullptr, scales, w_dq, wdq_dtype);
  return check_launch("rtn_mxfp_kernel");
}

extern "C" int gq_dequantize(const uint8_t* q, const void* scales, const void* biases, int scale_dtype, int64_t rows,
                             int64_t C, int mode, int group_size, float* out, void* stream) {
  GQ_REQUIRE(mode == GQ_AFFINE || mode == GQ_MXFP4 || mode == GQ_MXFP8, "gq_dequantize: mode %d", mode);
  GQ_REQUIRE(mode == GQ_AFFINE || group_size == 32, "gq_dequantize: MXFP requires group size 32");
  GQ_REQUIRE(mode != GQ_AFFINE || (biases && valid_dtype(scale_dtype)), "gq_dequantize: affine needs biases");
  GQ_REQUIRE(group_size > 0 && C % group_size == 0, "gq_dequantize: C %% group");
  const int64_t n = rows * C;
  if (n == 0) return GQ_OK;
  GQ_REQUIRE(q && scales && out, "gq_dequantize: null pointer");
  dequant_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(q, scales, biases, scale_dtype, n, C, mode,
                                                                        group_size, out);
  return check_launch("dequant_kernel");
}

extern "C" int gq_pack_q(const uint8_t* q, int64_t rows, int64_t C, int bits, uint32_t* words, void* stream) {
  GQ_REQUIRE(bits == 2 || bits == 4 || bits == 8, "cannot pack %d-bit for MLX (supported: (2, 4, 8))", bits);
  GQ_REQUIRE(C % (32 / bits) == 0, "gq_pack_q: last dim %lld not divisible by %d", (long long)C, 32 / bits);
  const int64_t nw = rows * C / (32 / bits);
  if (nw == 0) return GQ_OK;
  GQ_REQUIRE(q && words, "gq_pack_q: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  int64_t done = 0;  // words written by the vectorized kernel (whole groups of four)
  if (aligned16(q) && aligned16(words)) {
    const int64_t nquads = nw / 4;
    if (nquads > 0) {
      if (bits == 4)
        pack_q_vec_kernel<4><<<blocks_for(nquads, 256), 256, 0, s>>>(reinterpret_cast<const uint4*>(q), nquads,
                                                                    reinterpret_cast<uint4*>(words));
      else if (bits == 2)
        pack_q_vec_kernel<2><<<blocks_for(nquads, 256), 256, 0, s>>>(reinterpret_cast<const uint4*>(q), nquads,
                                                                    reinterpret_cast<uint4*>(words));
      else
        pack_q_vec_kernel<8><<<blocks_for(nquads, 256), 256, 0, s>>>(reinterpret_cast<const uint4*>(q), nquads,
                                                                    reinterpret_cast<uint4*>(words));
      int st = check_launch("pack_q_vec_kernel");
      if (st != GQ_OK) return st;
      done = nquads * 4;
    }
  }
  if (done == nw) return GQ_OK;
  const int64_t per = 32 / bits;
  pack_q_kernel<<<blocks_for(nw - done, 256), 256, 0, s>>>(q + done * per, nw - done, bits, words + done);
  return check_launch("pack_q_kernel");
}

extern "C" int gq_unpack_q(const uint32_t* words, int64_t rows, int64_t n_words, int bits, int64_t out_cols,
                           uint8_t* q, void* stream) {
  GQ_REQUIRE(bits == 2 || bits == 4 || bits == 8, "gq_unpack_q: bits %d", bits);
  GQ_REQUIRE(out_cols <= n_words * (32 / bits), "gq_unpack_q: out_cols too large");
  const int64_t n = rows * out_cols;
  if (n == 0) return GQ_OK;
  GQ_REQUIRE(words && q, "gq_unpack_q: null pointer");
  unpack_q_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(words, rows, n_words, bits, out_cols, q);
  return check_launch("unpack_q_kernel");
}

extern "C" int gq_pack_nibbles(const uint8_t* q, int64_t rows, int64_t C, uint8_t* out, void* stream) {
  GQ_REQUIRE(C % 2 == 0, "gq_pack_nibbles: odd last dim");
  const int64_t n = rows * C / 2;
  if (n == 0) return GQ_OK;
  GQ_REQUIRE(q && out, "gq_pack_nibbles: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  int64_t done = 0;  // output bytes written by the vectorized kernel (whole groups of eight)
  if (aligned16(q) && (reinterpret_cast<uintptr_t>(out) & 7u) == 0) {
    const int64_t n8 = n / 8;
    if (n8 > 0) {
      pack_nibbles_vec_kernel<<<blocks_for(n8, 256), 256, 0, s>>>(reinterpret_cast<const uint4*>(q), n8,
                                                                 reinterpret_cast<uint2*>(out));
      int st = check_launch("pack_nibbles_vec_kernel");
      if (st != GQ_OK) return st;
      done = n8 * 8;
    }
  }
  if (done == n) return GQ_OK;
  pack_nibbles_kernel<<<blocks_for(n - done, 256), 256, 0, s>>>(q + 2 * done, n - done, out + done);
  return check_launch("pack_nibbles_kernel");
}

extern "C" int gq_unpack_nibbles(const uint8_t* packed, int64_t rows, int64_t n_bytes, uint8_t* q, void* stream) {
  const int64_t n = rows * n_bytes;
  if (n == 0) return GQ_OK;
  GQ_REQUIRE(packed && q, "gq_unpack_nibbles: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  int64_t done = 0;  // packed bytes consumed by the vectorized kernel (whole groups of eight)
  if ((reinterpret_cast<uintptr_t>(packed) & 7u) == 0 && aligned16(q)) {
    const int64_t n8 = n / 8;
    if (n8 > 0) {
      unpack_nibbles_vec_kernel<<<blocks_for(n8, 256), 256, 0, s>>>(reinterpret_cast<const uint2*>(packed), n8,
                                                                   reinterpret_cast<uint4*>(q));
      int st = check_launch("unpack_nibbles_vec_kernel");
      if (st != GQ_OK) return st;
      done = n8 * 8;
    }
  }
  if (done == n) return GQ_OK;
  unpack_nibbles_kernel<<<blocks_for(n - done, 256), 256, 0, s>>>(packed + done, n - done, q + 2 * done);
  return check_launch("unpack_nibbles_kernel");
}
