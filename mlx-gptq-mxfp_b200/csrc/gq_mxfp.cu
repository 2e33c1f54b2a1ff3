// MXFP GPTQ (mlx_gptq/gptq.py:69-180) and the solver pieces it shares with the
// affine path: dead columns, weight preparation, block-diagonal 32x32 factors,
// rel_err reduction.
//
// Layout: W / W_dq / q [B, R, C] row-major, H [B, C, C], U_g [B, C/32, 32, 32].
// The column loop runs one thread per weight row and one CTA per
// (32-column group, 128-row tile, batch item); U_g sits in shared memory and is
// read by all 128 threads as broadcasts. For safe-scale-search the eight objectives
// e^T H_g e of the tile's 128 rows run on the tensor cores (tcgen05, kind::tf32,
// accumulators in TMEM, one lane per row).
#include "gq_affine_grid.cuh"

namespace gq {

// --------------------------------------------------------------------------
// dead columns / weight preparation
// --------------------------------------------------------------------------
__global__ void dead_columns_kernel(float* __restrict__ H, int64_t B, int64_t C, uint8_t* __restrict__ dead) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= B * C) return;
  const int64_t b = i / C, j = i % C;
  float* d = H + (b * C + j) * C + j;
  const bool is_dead = *d <= 0.0f;
  if (is_dead) *d = 1.0f;
  dead[i] = is_dead ? 1 : 0;
}

template <typename Tin>
__global__ void prepare_weights_kernel(const Tin* __restrict__ W, const uint8_t* __restrict__ dead, int64_t B,
                                       int64_t R, int64_t C, float* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= B * R * C) return;
  const int64_t c = i % C, b = i / (R * C);
  float v = to_f32<Tin>(W[i]);
  if (dead && dead[b * C + c]) v = 0.0f;
  out[i] = v;
}

// --------------------------------------------------------------------------
// 32x32 damped factor, one warp per diagonal block
// --------------------------------------------------------------------------

// In-place lower Cholesky of the 32x32 matrix in A (row stride 33), by one warp.
// Returns false (uniformly) if a pivot is not > 0 (covers NaN), like potrf's info.
__device__ __forceinline__ bool warp_chol32(float (*A)[33], int lane) {
  for (int k = 0; k < 32; ++k) {
    __syncwarp();
    const float piv = A[k][k];
    if (!(piv > 0.0f)) return false;
    const float d = sqrtf(piv);
    __syncwarp();
    if (lane > k) A[lane][k] = A[lane][k] / d;
    if (lane == k) A[k][k] = d;
    __syncwarp();
    if (lane > k) {
      const float lik = A[lane][k];
      for (int j = k + 1; j <= lane; ++j) A[lane][j] = A[lane][j] - lik * A[j][k];
    }
  }
  __syncwarp();
  return true;
}

// gptq.py:27-66 per 32x32 diagonal block (called per group by gptq.py:99-100).
__global__ void __launch_bounds__(128) mx_hinv_kernel(const float* __restrict__ H, int64_t B, int64_t C, float damp,
                                                      float* __restrict__ U, int32_t* __restrict__ info,
                                                      float* __restrict__ damp_used) {
  __shared__ float sA[4][32][33];
  __shared__ float sM[4][32][33];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t G = C / 32;
  const int64_t item = int64_t(blockIdx.x) * 4 + w;
  if (item >= B * G) return;  // whole warp
  const int64_t b = item / G, g = item % G;
  const float* Hg = H + (b * C + g * 32) * C + g * 32;
  float (*A)[33] = sA[w];
  float (*M)[33] = sM[w];

  // mean(diag).clamp(min=1e-8)
  float dm = Hg[int64_t(lane) * C + lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dm += __shfl_xor_sync(0xFFFFFFFFu, dm, o);
  dm = fmaxf(dm / 32.0f, 1e-8f);

  float cur = damp;
  bool ok = false;
  for (int attempt = 0; attempt < 6; ++attempt) {
    const float lam = dm * cur;
    for (int i = 0; i < 32; ++i) {
      float v = Hg[int64_t(i) * C + lane];
      if (i == lane) v = v + lam;
      A[i][lane] = v;
    }
    ok = warp_chol32(A, lane);
    if (ok) break;
    cur = cur * 10.0f;
  }
  if (lane == 0) {
    info[item] = ok ? 0 : 1;
    if (damp_used) damp_used[item] = cur;
  }
  if (!ok) return;

  // Linv = L^-1 (lower): lane j solves L x = e_j (column j).
  for (int i = 0; i < 32; ++i) {
    float x = 0.0f;
    if (i == lane) {
      x = 1.0f / A[i][i];
    } else if (i > lane) {
      float acc = 0.0f;
      for (int k = 0; k < i; ++k)
        if (k >= lane) acc = fmaf(A[i][k], M[k][lane], acc);
      x = -acc / A[i][i];
    }
    M[i][lane] = x;
    __syncwarp();
  }
  // Hinv = Linv^T Linv (cholesky_inverse), column `lane`
  __syncwarp();
  for (int i = 0; i < 32; ++i) {
    float acc = 0.0f;
    const int k0 = i > lane ? i : lane;
    for (int k = k0; k < 32; ++k) acc = fmaf(M[k][i], M[k][lane], acc);
    A[i][lane] = acc;
  }
  __syncwarp();
  const bool ok2 = warp_chol32(A, lane);
  if (!ok2) {
    if (lane == 0) info[item] = 2;
    return;
  }
  // U = Lh^T (upper)
  float* Ug = U + item * 1024;
  for (int i = 0; i < 32; ++i) Ug[i * 32 + lane] = lane >= i ? A[lane][i] : 0.0f;
}

// --------------------------------------------------------------------------
// MXFP column loop
// --------------------------------------------------------------------------

// tf32 part of x (round to nearest, ties away): the hi term of the 3xTF32 split.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// Grid value (without the scale) of w * inv for the mode.
template <int MODE>
__device__ __forceinline__ float mx_round(float w, float inv) {
  if (MODE == GQ_MXFP4) return e2m1_round(w * inv);
  float d0, d1;
  mx_quant2<MODE>(w, 0.0f, inv, 1.0f, d0, d1);
  return d0;
}

template <typename T>
__device__ __forceinline__ void load_row32(const T* __restrict__ p, float (&o)[32]);
template <>
__device__ __forceinline__ void load_row32<float>(const float* __restrict__ p, float (&o)[32]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p) + k);
    o[4 * k] = v.x, o[4 * k + 1] = v.y, o[4 * k + 2] = v.z, o[4 * k + 3] = v.w;
  }
}
template <>
__device__ __forceinline__ void load_row32<__nv_bfloat16>(const __nv_bfloat16* __restrict__ p, float (&o)[32]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + k);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      o[8 * k + 2 * t] = __uint_as_float(u[t] << 16);
      o[8 * k + 2 * t + 1] = __uint_as_float(u[t] & 0xFFFF0000u);
    }
  }
}
template <>
__device__ __forceinline__ void load_row32<__half>(const __half* __restrict__ p, float (&o)[32]) {
#pragma unroll
  for (int k = 0; k < 32; ++k) o[k] = __half2float(p[k]);
}

template <typename T>
__device__ __forceinline__ void store_row32(T* __restrict__ p, const float (&v)[32]);
template <>
__device__ __forceinline__ void store_row32<float>(float* __restrict__ p, const float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 8; ++k)
    reinterpret_cast<float4*>(p)[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}
template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16* __restrict__ p, const float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t u[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * k + 2 * t], v[8 * k + 2 * t + 1]);
      u[t] = *reinterpret_cast<const uint32_t*>(&h);
    }
    reinterpret_cast<uint4*>(p)[k] = make_uint4(u[0], u[1], u[2], u[3]);
  }
}

// Code storage of one row group: mxfp4 = 16 bytes of nibble pairs (the artifact
// layout: column c at bits 4*(c%8) of word c/8); mxfp8 = 32 E4M3 bytes.
template <int MODE> struct Codes {
  static constexpr int kWords = MODE == GQ_MXFP4 ? 4 : 8;
  uint32_t w[kWords];
  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int i = 0; i < kWords; ++i) w[i] = 0;
  }
  // pair (c, c+1), c even, as returned by mx_quant2
  __device__ __forceinline__ void put2(int c, uint32_t codes) {
    if (MODE == GQ_MXFP4) w[c >> 3] |= codes << (4 * (c & 7));
    else w[c >> 2] |= codes << (8 * (c & 3));
  }
};

// ---------------------------------------------------------------------------
// Objectives of a 128-row tile on the 5th-generation tensor cores (safe-scale-search)
// ---------------------------------------------------------------------------
// Y = E * H_g for the CTA's 128 rows at once: one tcgen05.mma (kind::tf32, M = 128,
// N = 32, K = 8) per K step and split term, issued by one thread, accumulating in 32
// TMEM columns; TMEM lane r is row r, so thread r reads its row of Y with one
// tcgen05.ld and forms e_r^T H_g e_r = sum_c Y[r][c] * e_r[c] itself. E and H_g go to
// shared memory as 3xTF32 splits (x = hi + lo, hi = tf32(x); D = Ehi*Hhi + Ehi*Hlo +
// Elo*Hhi) in the K-major 128-byte-swizzled layout: row r (128 bytes = 32 fp32) at
// r * 128, 16-byte chunk j stored at chunk j ^ (r % 8).
namespace tc {
constexpr uint32_t kRows = 128, kRowBytes = 128;
constexpr uint32_t A_BYTES = kRows * kRowBytes;  // 16 KB per split of E
constexpr uint32_t B_BYTES = 32 * kRowBytes;     // 4 KB per split of H_g
constexpr uint32_t TMEM_COLS = 32;

__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t col) {  // byte offset of (row, fp32 col)
  return row * kRowBytes + ((((col >> 2) ^ (row & 7u)) << 4) | ((col & 3u) << 2));
}
// Shared-memory descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t(1) << 16;             // leading byte offset (unused: K fits one swizzle atom)
  d |= uint64_t(1024 >> 4) << 32;     // stride byte offset: next 8-row group
  d |= uint64_t(1) << 46;             // descriptor version for sm_100
  d |= uint64_t(2) << 61;             // SWIZZLE_128B
  return d;
}
// Instruction descriptor, kind::tf32: f32 accumulate, tf32 A and B, both K-major.
constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
__device__ __forceinline__ void mma_tf32_128x32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  constexpr uint32_t idesc = idesc_tf32(128, 32);
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
}  // namespace tc

// Writes this thread's error vector (row `row` of E) as its hi/lo tf32 split.
__device__ __forceinline__ void tc_stage_row(uint8_t* ahi, uint8_t* alo, uint32_t row, const float (&e)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // one 16-byte chunk (4 columns) at a time
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[i] = to_tf32(e[4 * j + i]);
      l[i] = __float_as_uint(e[4 * j + i] - __uint_as_float(h[i]));
    }
    const uint32_t off = tc::swz(row, 4 * j);
    *reinterpret_cast<uint4*>(ahi + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(alo + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// e_r^T H_g e_r for the thread's row after every thread of the CTA staged its row:
// thread 0 issues the 12 MMAs and commits to `bar`; every thread waits for that phase,
// reads its TMEM lane and contracts it with e.
__device__ __forceinline__ float tc_objective(uint32_t ahi, uint32_t alo, uint32_t bhi, uint32_t blo,
                                              uint32_t tmem, uint64_t* bar, uint32_t& phase, const float (&e)[32],
                                              int tid, volatile int* abort_flag) {
  tc::fence_proxy_async_smem();  // this thread's rows are visible to the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // K = 8 tf32 = 32 bytes per step inside the 128-byte rows
      const uint32_t ko = uint32_t(k) * 32u;
      const uint64_t dahi = tc::desc_kmajor_sw128(ahi + ko), dalo = tc::desc_kmajor_sw128(alo + ko);
      const uint64_t dbhi = tc::desc_kmajor_sw128(bhi + ko), dblo = tc::desc_kmajor_sw128(blo + ko);
      tc::mma_tf32_128x32(tmem, dahi, dbhi, k > 0 ? 1u : 0u);
      tc::mma_tf32_128x32(tmem, dahi, dblo, 1u);
      tc::mma_tf32_128x32(tmem, dalo, dbhi, 1u);
    }
    umma_commit(bar);
  }
  mbar_wait(bar, phase, abort_flag, nullptr);
  phase ^= 1u;
  tc_fence_after();
  float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {  // 16 columns at a time keeps the row's Y out of the register peak
    uint32_t y[16];
    tmem_ld16(tmem + (uint32_t((tid >> 5) * 32) << 16) + uint32_t(16 * h), y);
    tmem_ld_wait();
#pragma unroll
    for (int c = 0; c < 16; c += 2) {
      o0 = fmaf(__uint_as_float(y[c]), e[16 * h + c], o0);
      o1 = fmaf(__uint_as_float(y[c + 1]), e[16 * h + c + 1], o1);
    }
  }
  tc_fence_before();  // the TMEM reads finish before the next MMA (after the next barrier)
  return o0 + o1;
}

// Grid values (without the scale) of a code pair as stored in Codes.
template <int MODE>
__device__ __forceinline__ float2 code_pair_values(uint32_t pair) {
  return MODE == GQ_MXFP4 ? e2m1x2_to_f32(pair) : e4m3x2_to_f32(pair);
}

// One thread per weight row, one CTA per (32-column group, 128-row tile, batch item).
// Registers hold the row's 32 original values and the 32 working values of the GPTQ
// pass; codes are packed as they are produced and every grid value is read back from
// its code (exact: the codes are the hardware casts of on-grid values), so no grid
// value or error array is kept. Error vectors for the objectives go straight to the
// warp's shared-memory staging area.
template <int MODE, bool SAFE, typename Tin, typename Tout>
__global__ void __launch_bounds__(128, SAFE ? 3 : 4) mx_gptq_kernel(const Tin* __restrict__ W, const float* __restrict__ H,
                                                      const float* __restrict__ U, const uint8_t* __restrict__ dead,
                                                      const int32_t* __restrict__ info, int64_t R, int64_t C,
                                                      uint8_t* __restrict__ q, uint8_t* __restrict__ qp,
                                                      uint8_t* __restrict__ scales, Tout* __restrict__ wdq,
                                                      float* __restrict__ partials, int64_t partials_cap) {
  // safe-scale-search: E (hi, lo) and H_g (hi, lo) operand tiles of the objectives
  constexpr uint32_t kTcBytes = SAFE ? 2 * tc::A_BYTES + 2 * tc::B_BYTES : 16;
  __shared__ __align__(1024) uint8_t Tsm[kTcBytes];
  __shared__ __align__(16) float Us[32][32];
  __shared__ float red[2][4];
  __shared__ uint32_t s_dmask;
  __shared__ uint64_t s_bar;         // MMA completion (safe-scale-search)
  __shared__ uint32_t s_tmem;        // TMEM base of the 32 accumulator columns
  __shared__ int s_abort;
  const int64_t G = C / 32;
  const int64_t g = blockIdx.x, tile = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  // (num, den) slot of this CTA; slots past partials_cap (the caller's workspace)
  // are never written, whatever the grid
  const int64_t pslot = (b * gridDim.y + tile) * G + g;
  float* p_out = partials && pslot < partials_cap ? partials + pslot * 2 : nullptr;
  if (info && info[b * G + g] != 0) {  // factorization failed: host raises
    if (p_out && tid == 0) p_out[0] = p_out[1] = 0.0f;  // rel_err then ignores this group
    return;
  }
  const float* Ug = U + (b * G + g) * 1024;
  uint8_t* const a_hi = Tsm;  // (groupwise: a 16-byte placeholder, never used)
  uint8_t* const a_lo = Tsm + (SAFE ? tc::A_BYTES : 0u);
  uint8_t* const b_hi = Tsm + (SAFE ? 2 * tc::A_BYTES : 0u);
  uint8_t* const b_lo = b_hi + (SAFE ? tc::B_BYTES : 0u);
  if (SAFE) {
    // B operand: row n of H_g (symmetric, so B[n][k] = H_g[k][n] = H_g[n][k]), hi/lo split
    const float* Hg = H + (b * C + g * 32) * C + g * 32;
    for (int i = tid; i < 1024; i += 128) {
      const uint32_t n = uint32_t(i >> 5), k = uint32_t(i & 31);
      const float h = Hg[int64_t(n) * C + k];
      const uint32_t hi = to_tf32(h);
      *reinterpret_cast<uint32_t*>(b_hi + tc::swz(n, k)) = hi;
      *reinterpret_cast<uint32_t*>(b_lo + tc::swz(n, k)) = __float_as_uint(h - __uint_as_float(hi));
    }
    if (tid == 0) {
      mbar_init(&s_bar, 1);
      s_abort = 0;
      fence_mbar_init();
    }
    if (tid < 32) tmem_alloc(&s_tmem, tc::TMEM_COLS);
  }
  for (int i = tid; i < 1024; i += 128) Us[i >> 5][i & 31] = Ug[i];
  if (tid < 32) {
    const bool d = dead ? dead[b * C + g * 32 + tid] != 0 : false;
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, d);
    if (tid == 0) s_dmask = m;
  }
  if (SAFE) tc_fence_before();
  __syncthreads();
  if (SAFE) tc_fence_after();
  const uint32_t dmask = s_dmask;
  const int64_t r = tile * 128 + tid;
  const uint32_t tmem = SAFE ? s_tmem : 0u;
  const uint32_t sa_hi = smem_u32(a_hi), sa_lo = smem_u32(a_lo), sb_hi = smem_u32(b_hi), sb_lo = smem_u32(b_lo);
  uint32_t phase = 0;
  float num = 0.0f, den = 0.0f;
  const bool active = r < R;  // rows past R run on zeros (the objectives need whole warps)
  {
    const int64_t off = (b * R + (active ? r : 0)) * C + g * 32;
    float o[32];
    if (active) {
      load_row32<Tin>(W + off, o);
    } else {
#pragma unroll
      for (int c = 0; c < 32; ++c) o[c] = 0.0f;
    }
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      den = fmaf(o[c], o[c], den);
      if (dmask & (1u << c)) o[c] = 0.0f;  // gptq.py:219-221 (rel_err keeps the raw value)
    }
    constexpr float kFmax = MODE == GQ_MXFP4 ? 6.0f : 448.0f;
    float amax = 0.0f;
#pragma unroll
    for (int c = 0; c < 32; ++c) amax = fmaxf(amax, fabsf(o[c]));
    const int e0 = mx_scale_exponent(amax, kFmax);

    // scale choice: groupwise = RTN scale; safe-scale-search = min e^T H e over offsets
    int best_e = e0;
    float best_obj = 0.0f;
    if (SAFE) {
      // offsets (0, -1, -2, -3, -4, +1, +2) for mxfp4, (0, -1, +1) for mxfp8 (gptq.py:92)
      constexpr int kNoff = MODE == GQ_MXFP4 ? 7 : 3;
#pragma unroll 1
      for (int t = 0; t < kNoff; ++t) {
        const int d = MODE == GQ_MXFP4 ? (t <= 4 ? -t : t - 4) : (t == 0 ? 0 : (t == 1 ? -1 : 1));
        int e = e0 + d;
        e = e < -127 ? -127 : (e > 127 ? 127 : e);
        const float sc = exp2i(e), inv = exp2i(-e);
        float err[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) err[c] = mx_round<MODE>(o[c], inv) * sc - o[c];
        tc_stage_row(a_hi, a_lo, uint32_t(tid), err);
        const float obj = tc_objective(sa_hi, sa_lo, sb_hi, sb_lo, tmem, &s_bar, phase, err, tid, &s_abort);
        if (t == 0 || obj < best_obj) {
          best_obj = obj;
          best_e = e;
        }
      }
    }
    const float sc = exp2i(best_e), inv = exp2i(-best_e);
    const float limit = fmaxf(amax * 32.0f, 1.1754943508222875e-38f);  // range guard bound

    // sequential GPTQ over the 32 columns with the fixed scale: codes packed as they
    // are produced (pairs), the range guard tracked on the way; after column c is
    // quantized wv[c] holds its error dq[c] - o[c] (the GPTQ objective's vector)
    Codes<MODE> code;
    code.clear();
    bool valid = true;
    float wv[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) wv[c] = o[c];
    float gprev = 0.0f;
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const float gvc = mx_round<MODE>(wv[c], inv);
      const float dq = gvc * sc;
      valid = valid && (fabsf(dq) <= limit);
      const float err = (wv[c] - dq) / Us[c][c];
#pragma unroll
      for (int k = c + 1; k < 32; ++k) wv[k] = wv[k] - err * Us[c][k];
      wv[c] = dq - o[c];
      if (c & 1) code.put2(c - 1, MODE == GQ_MXFP4 ? cvt_e2m1x2(gprev, gvc) : cvt_e4m3x2(gprev, gvc));
      gprev = gvc;
    }
    bool use_gptq = true;
    if (SAFE) {
      tc_stage_row(a_hi, a_lo, uint32_t(tid), wv);
      use_gptq = tc_objective(sa_hi, sa_lo, sb_hi, sb_lo, tmem, &s_bar, phase, wv, tid, &s_abort) <= best_obj;
    }
    use_gptq = use_gptq && valid;
    if (!use_gptq) {  // baseline: RTN with the chosen scale
      code.clear();
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const float g0 = mx_round<MODE>(o[c], inv), g1 = mx_round<MODE>(o[c + 1], inv);
        code.put2(c, MODE == GQ_MXFP4 ? cvt_e2m1x2(g0, g1) : cvt_e4m3x2(g0, g1));
      }
    }
    // outputs (active rows only)
    if (active) {
      if (q) {
        uint32_t qw[8];
        if (MODE == GQ_MXFP4) {
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            const uint32_t nb = (code.w[w >> 1] >> (16 * (w & 1))) & 0xFFFFu;
            qw[w] = (nb & 0xFu) | ((nb & 0xF0u) << 4) | ((nb & 0xF00u) << 8) | ((nb & 0xF000u) << 12);
          }
        } else {
#pragma unroll
          for (int w = 0; w < 8; ++w) qw[w] = code.w[w];
        }
        uint4* qd = reinterpret_cast<uint4*>(q + off);
        qd[0] = make_uint4(qw[0], qw[1], qw[2], qw[3]);
        qd[1] = make_uint4(qw[4], qw[5], qw[6], qw[7]);
      }
      if (MODE == GQ_MXFP4 && qp)
        *reinterpret_cast<uint4*>(qp + off / 2) = make_uint4(code.w[0], code.w[1], code.w[2], code.w[3]);
      scales[(b * R + r) * G + g] = uint8_t(best_e + 127);
      if (dmask && partials) {  // dead columns: rel_err compares against the raw weights
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (dmask & (1u << c)) o[c] = to_f32<Tin>(W[off + c]);
      }
      // dequantized values pair by pair from the codes: W_dq and the rel_err numerator
      float gdq[32];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const uint32_t pair = MODE == GQ_MXFP4 ? (code.w[c >> 3] >> (4 * (c & 7))) & 0xFFu
                                               : (code.w[c >> 2] >> (8 * (c & 3))) & 0xFFFFu;
        const float2 v = code_pair_values<MODE>(pair);
        gdq[c] = v.x * sc;
        gdq[c + 1] = v.y * sc;
      }
      if (wdq) store_row32<Tout>(wdq + off, gdq);
      if (partials) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float d = gdq[c] - o[c];
          num = fmaf(d, d, num);
        }
      }
    }  // active
  }
  if (partials) {
    num = warp_sum(num);
    den = warp_sum(den);
    if ((tid & 31) == 0) {
      red[0][tid >> 5] = num;
      red[1][tid >> 5] = den;
    }
    __syncthreads();
    if (tid == 0 && p_out) {
      p_out[0] = (red[0][0] + red[0][1]) + (red[0][2] + red[0][3]);
      p_out[1] = (red[1][0] + red[1][1]) + (red[1][2] + red[1][3]);
    }
  }
  if (SAFE) {  // every TMEM read is done: release the columns
    tc_fence_before();
    __syncthreads();
    if (tid < 32) {
      tc_fence_after();
      tmem_dealloc(tmem, tc::TMEM_COLS);
    }
  }
}

// rel_err[b] = sqrt(sum num) / max(sqrt(sum den), 1e-12), fixed-order reduction.
__global__ void rel_err_kernel(const float* __restrict__ partials, int64_t per_b, float* __restrict__ rel) {
  const int64_t b = blockIdx.x;
  double n = 0.0, d = 0.0;
  for (int64_t i = threadIdx.x; i < per_b; i += blockDim.x) {
    n += partials[(b * per_b + i) * 2];
    d += partials[(b * per_b + i) * 2 + 1];
  }
  __shared__ double sn[256], sd[256];
  sn[threadIdx.x] = n;
  sd[threadIdx.x] = d;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) {
      sn[threadIdx.x] += sn[threadIdx.x + s];
      sd[threadIdx.x] += sd[threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) rel[b] = float(sqrt(sn[0]) / fmax(sqrt(sd[0]), 1e-12));
}

static bool valid_in(int d) { return d == GQ_F32 || d == GQ_BF16 || d == GQ_F16; }

int launch_rel_err(const float* partials, int64_t B, int64_t per_b, float* rel, cudaStream_t s) {
  rel_err_kernel<<<unsigned(B), 256, 0, s>>>(partials, per_b, rel);
  return check_launch("rel_err_kernel");
}

}  // namespace gq

using namespace gq;

extern "C" int gq_dead_columns(float* H, int64_t B, int64_t C, uint8_t* dead, void* stream) {
  GQ_REQUIRE(H && dead, "gq_dead_columns: null pointer");
  GQ_REQUIRE(B >= 0 && C >= 0, "gq_dead_columns: negative size");
  if (B * C == 0) return GQ_OK;
  dead_columns_kernel<<<unsigned((B * C + 255) / 256), 256, 0, (cudaStream_t)stream>>>(H, B, C, dead);
  return check_launch("dead_columns_kernel");
}

extern "C" int gq_prepare_weights(const void* W_in, int w_dtype, const uint8_t* dead, int64_t B, int64_t R, int64_t C,
                                  float* W_out, void* stream) {
  GQ_REQUIRE(W_in && W_out && valid_in(w_dtype), "gq_prepare_weights: bad argument");
  const int64_t n = B * R * C;
  if (n == 0) return GQ_OK;
  const unsigned grid = unsigned((n + 255) / 256);
  cudaStream_t s = (cudaStream_t)stream;
  if (w_dtype == GQ_F32)
    prepare_weights_kernel<float><<<grid, 256, 0, s>>>((const float*)W_in, dead, B, R, C, W_out);
  else if (w_dtype == GQ_BF16)
    prepare_weights_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)W_in, dead, B, R, C, W_out);
  else
    prepare_weights_kernel<__half><<<grid, 256, 0, s>>>((const __half*)W_in, dead, B, R, C, W_out);
  return check_launch("prepare_weights_kernel");
}

extern "C" int gq_mx_prepare_hinv(const float* H, int64_t B, int64_t C, float damp, float* U, int32_t* info,
                                  float* damp_used, void* stream) {
  GQ_REQUIRE(H && U && info, "gq_mx_prepare_hinv: null pointer");
  GQ_REQUIRE(B >= 0 && C >= 0 && C % 32 == 0, "gq_mx_prepare_hinv: C=%lld not a multiple of 32", (long long)C);
  const int64_t items = B * (C / 32);
  if (items == 0) return GQ_OK;
  mx_hinv_kernel<<<unsigned((items + 3) / 4), 128, 0, (cudaStream_t)stream>>>(H, B, C, damp, U, info, damp_used);
  return check_launch("mx_hinv_kernel");
}

extern "C" size_t gq_gptq_mxfp_workspace_size(int64_t B, int64_t R, int64_t C) {
  if (B <= 0 || R <= 0 || C <= 0) return 0;
  return size_t(B) * size_t((R + 127) / 128) * size_t(C / 32) * 2 * sizeof(float);
}

extern "C" int gq_gptq_mxfp(const void* W, int w_dtype, const float* H, const float* U, const uint8_t* dead,
                            const int32_t* info, int64_t B, int64_t R, int64_t C, int mode, int algorithm, uint8_t* q,
                            uint8_t* q_packed, uint8_t* scales, void* w_dq, int wdq_dtype, float* rel_err,
                            void* workspace, size_t workspace_bytes, void* stream) {
  GQ_REQUIRE(mode == GQ_MXFP4 || mode == GQ_MXFP8, "gq_gptq_mxfp: not a microscaling mode: %d", mode);
  GQ_REQUIRE(algorithm == GQ_MX_GROUPWISE || algorithm == GQ_MX_SAFE_SCALE_SEARCH,
             "unsupported MXFP GPTQ algorithm: %d", algorithm);
  GQ_REQUIRE(W && H && U && scales, "gq_gptq_mxfp: null pointer");
  GQ_REQUIRE(w_dtype == GQ_F32 || w_dtype == GQ_BF16 || w_dtype == GQ_F16, "gq_gptq_mxfp: w_dtype");
  GQ_REQUIRE(!w_dq || wdq_dtype == GQ_F32 || wdq_dtype == GQ_BF16, "gq_gptq_mxfp: wdq_dtype");
  GQ_REQUIRE(B >= 0 && R >= 0 && C >= 0 && C % 32 == 0, "gq_gptq_mxfp: C=%lld not a multiple of 32", (long long)C);
  GQ_REQUIRE(aligned16(W) && (!q || aligned16(q)) && (!q_packed || aligned16(q_packed)) && (!w_dq || aligned16(w_dq)),
             "gq_gptq_mxfp: W, q, q_packed and w_dq must be 16-byte aligned");
  GQ_REQUIRE(R / 128 < 65535 && B < 65536 && C / 32 < (int64_t(1) << 31), "gq_gptq_mxfp: shape too large");
  const size_t need = gq_gptq_mxfp_workspace_size(B, R, C);
  GQ_REQUIRE(!rel_err || (workspace && workspace_bytes >= need), "gq_gptq_mxfp: workspace too small (%zu < %zu)",
             workspace_bytes, need);
  if (B * R * C == 0) return GQ_OK;
  cudaStream_t s = (cudaStream_t)stream;
  float* partials = rel_err ? reinterpret_cast<float*>(workspace) : nullptr;
  const int64_t partials_cap = rel_err ? int64_t(workspace_bytes / (2 * sizeof(float))) : 0;
  const dim3 grid(unsigned(C / 32), unsigned((R + 127) / 128), unsigned(B));
  const bool safe = algorithm == GQ_MX_SAFE_SCALE_SEARCH;
#define MXL(MODE, SAFE, TIN, TOUT)                                                                              \
  mx_gptq_kernel<MODE, SAFE, TIN, TOUT><<<grid, 128, 0, s>>>((const TIN*)W, H, U, dead, info, R, C, q, q_packed, \
                                                             scales, (TOUT*)w_dq, partials, partials_cap)
#define MXL_OUT(MODE, SAFE, TIN)                  \
  do {                                            \
    if (wdq_dtype == GQ_BF16)                     \
      MXL(MODE, SAFE, TIN, __nv_bfloat16);        \
    else                                          \
      MXL(MODE, SAFE, TIN, float);                \
  } while (0)
#define MXL_IN(MODE, SAFE)                     \
  do {                                         \
    if (w_dtype == GQ_F32)                     \
      MXL_OUT(MODE, SAFE, float);              \
    else if (w_dtype == GQ_BF16)               \
      MXL_OUT(MODE, SAFE, __nv_bfloat16);      \
    else                                       \
      MXL_OUT(MODE, SAFE, __half);             \
  } while (0)
  if (mode == GQ_MXFP4) {
    if (safe) MXL_IN(GQ_MXFP4, true); else MXL_IN(GQ_MXFP4, false);
  } else {
    if (safe) MXL_IN(GQ_MXFP8, true); else MXL_IN(GQ_MXFP8, false);
  }
#undef MXL_IN
#undef MXL_OUT
#undef MXL
  int st = check_launch("mx_gptq_kernel");
  if (st != GQ_OK || !rel_err) return st;
  return launch_rel_err(partials, B, ((R + 127) / 128) * (C / 32), rel_err, s);
}

// ---------------------------------------------------------------------------
// MXFP GPTQ without caller workspace (see gq_gptq_mxfp_noalloc in gptq_b200.h)
// ---------------------------------------------------------------------------
#include <mutex>

namespace gq {

// Scratch for the rel_err partial sums of gq_gptq_mxfp_noalloc: one (num, den)
// float pair per (batch item, 128-row tile, 32-column group). Every GPU that
// loads this library holds it (4 MiB) until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_noalloc_scratch on the current device, looked up once per
// device. In host code the symbol itself is only a host-side stand-in and must
// never be handed to a kernel.
static int noalloc_scratch(void** out) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  GQ_CUDA_TRY(cudaGetDevice(&dev));
  GQ_REQUIRE(dev >= 0 && dev < kMaxDevices, "gq_gptq_mxfp_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    GQ_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    addr[dev] = p;
  }
  *out = addr[dev];
  return GQ_OK;
}

}  // namespace gq

extern "C" int gq_gptq_mxfp_noalloc(const void* W, int w_dtype, const float* H, const float* U, const uint8_t* dead,
                                    const int32_t* info, int64_t B, int64_t R, int64_t C, int mode, int algorithm,
                                    uint8_t* q, uint8_t* q_packed, uint8_t* scales, void* w_dq, int wdq_dtype,
                                    float* rel_err, void* stream) {
  // Without rel_err the column loop needs no scratch at all: no limit, no lookup.
  if (!rel_err)
    return gq_gptq_mxfp(W, w_dtype, H, U, dead, info, B, R, C, mode, algorithm, q, q_packed, scales, w_dq,
                        wdq_dtype, nullptr, nullptr, 0, stream);
  const size_t need = gq_gptq_mxfp_workspace_size(B, R, C);
  GQ_REQUIRE(need <= kNoAllocScratchBytes,
             "gq_gptq_mxfp_noalloc: B*ceil(R/128)*(C/32) = %zu (row tile, group) pairs exceed the fixed scratch "
             "limit of %zu; split the batch or use gq_gptq_mxfp with a workspace",
             need / (2 * sizeof(float)), kNoAllocScratchBytes / (2 * sizeof(float)));
  void* scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st != GQ_OK) return st;
  return gq_gptq_mxfp(W, w_dtype, H, U, dead, info, B, R, C, mode, algorithm, q, q_packed, scales, w_dq, wdq_dtype,
                      rel_err, scratch, kNoAllocScratchBytes, stream);
}
