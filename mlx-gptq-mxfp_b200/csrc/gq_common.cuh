// Shared device helpers for the GPTQ calibration library (sm_100a).
//
// The whole library is compiled with -fmad=false: every float expression
// rounds once per operation, the way the reference's torch code does
// (one kernel per op). Where a fused multiply-add is wanted (GEMM-style
// accumulations whose order differs from the reference anyway) it is
// written explicitly with fmaf().
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gptq_b200.h"

namespace gq {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
void set_last_error(const char* fmt, ...);
int check_launch(const char* what);  // GQ_OK or GQ_ERR_CUDA (message recorded)

// cuTensorMapEncodeTiled from the driver (looked up once), or nullptr.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encoder();

#define GQ_REQUIRE(cond, ...)              \
  do {                                     \
    if (!(cond)) {                         \
      ::gq::set_last_error(__VA_ARGS__);   \
      return GQ_ERR_ARG;                   \
    }                                      \
  } while (0)

#define GQ_CUDA_TRY(expr)                                                        \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess) {                                                     \
      ::gq::set_last_error("%s: %s", #expr, cudaGetErrorString(_e));             \
      return GQ_ERR_CUDA;                                                        \
    }                                                                            \
  } while (0)

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// exact float helpers
// ---------------------------------------------------------------------------

// float32 -> bfloat16 round-to-nearest-even -> float32; NaN -> canonical quiet NaN.
__device__ __forceinline__ float round_bf16(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return __uint_as_float(0x7FC00000u);
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  return __uint_as_float(u);
}

__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

__device__ __forceinline__ float round_storage(float x, int dtype) {
  return dtype == GQ_BF16 ? round_bf16(x) : (dtype == GQ_F16 ? round_f16(x) : x);
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Exact 2^e for integer e in [-127, 127] (2^-127 is a float32 subnormal).
__device__ __forceinline__ float exp2i(int e) {
  return e >= -126 ? __uint_as_float(uint32_t(e + 127) << 23) : __uint_as_float(0x00400000u);
}

// ---------------------------------------------------------------------------
// MXFP grids
// ---------------------------------------------------------------------------

// Per-binade thresholds of round(log2(y)) measured from the reference's torch
// arithmetic: entry E+127 is the smallest float32 bit pattern in [2^E, 2^(E+1))
// that rounds up to E+1.
__constant__ const uint32_t kLog2Thresholds[255] = {
#include "gq_log2_table.inc"
};

// Shared E8M0 exponent of a group with maximum |w| == max_abs:
// clamp(round(log2(max_abs / fmax)), -127, 127), 0 when max_abs == 0.
// (mlx_gptq/grid.py:68-73)
__device__ __forceinline__ int mx_scale_exponent(float max_abs, float fmax) {
  if (max_abs == 0.0f) return 0;
  float y = max_abs / fmax;  // IEEE division, same rounding as torch
  uint32_t bits = __float_as_uint(y);
  if (bits >= 0x7F800000u) return -127;  // inf / NaN: torch's int cast + clamp gives -127
  int efield = int(bits >> 23);
  int E = efield ? efield - 127 : (bits >= 0x00400000u ? -127 : -128);
  if (E < -127) return -127;
  int ex = E + (bits >= kLog2Thresholds[E + 127] ? 1 : 0);
  return ex > 127 ? 127 : ex;
}

// E2M1 code of x: 3-bit magnitude from the reference's thresholds plus sign bit 3.
// (mlx_gptq/grid.py:82-105)
__device__ __forceinline__ uint32_t e2m1_code(float x) {
  float a = fabsf(x);
  uint32_t m = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.0f);
  return m | (x < 0.0f ? 8u : 0u);
}

// E2M1 code -> value (grid.py:23-40).
__device__ __forceinline__ float e2m1_value(uint32_t code) {
  // magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6 as (mantissa, exponent) pairs
  uint32_t m = code & 7u;
  float v = m < 4u ? 0.5f * float(m) : float(2u << ((m - 4u) >> 1)) * (1.0f + 0.5f * float(m & 1u));
  return (code & 8u) ? -v : v;
}

// float32 -> float8_e4m3fn bits with round-to-nearest-even; |x| >= 480, inf and
// NaN give the NaN code 0x7F (sign kept). The reference clamps to +-448 first.
__device__ __forceinline__ uint32_t e4m3_encode(float x) {
  uint32_t u = __float_as_uint(x);
  uint32_t sign = (u >> 24) & 0x80u;
  uint32_t a = u & 0x7FFFFFFFu;
  uint32_t code;
  if (a >= 0x43F00000u) {
    code = 0x7Fu;
  } else if (a < 0x3C800000u) {  // below 2^-6: multiples of 2^-9
    code = uint32_t(rintf(__uint_as_float(a) * 512.0f));
  } else {
    uint32_t e = (a >> 23) - 127u + 7u;
    uint32_t m = a & 0x7FFFFFu;
    uint32_t q = m >> 20, rem = m & 0xFFFFFu;
    q += (rem > 0x80000u) || (rem == 0x80000u && (q & 1u));
    e += q >> 3;
    code = (e << 3) | (q & 7u);
  }
  return code | sign;
}

__device__ __forceinline__ float e4m3_decode(uint32_t c) {
  uint32_t ef = (c >> 3) & 0xFu, mt = c & 7u;
  float v;
  if ((c & 0x7Fu) == 0x7Fu) return __uint_as_float(0x7FC00000u);
  if (ef == 0)
    v = float(mt) * 0.001953125f;  // 2^-9
  else
    v = __uint_as_float(((ef - 7u + 127u) << 23) | (mt << 20));
  return (c & 0x80u) ? -v : v;
}

// ---------------------------------------------------------------------------
// sm_100 hardware conversions, two values per instruction. E2M1 and E4M3 with
// round-to-nearest-even and saturation are exactly the reference's grids: the
// E2M1 thresholds of grid.py:82-105 are the RNE midpoints (ties at 0.25, 1.25,
// 2.5, 5 go down to the even code, ties at 0.75, 1.75, 3.5 up), everything
// above 5 maps to 6; E4M3 after the reference's +-448 clamp is the satfinite
// RNE cast. The one difference is the sign of zero: the reference sets the E2M1
// sign bit from (x < 0), so -0.0 and NaN give code 0 -- callers pass +0.0 for them.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {  // byte: lo in bits 0-3
  uint16_t r;
  asm("{ .reg .b8 t; cvt.rn.satfinite.e2m1x2.f32 t, %1, %2; mov.b16 %0, {t, 0}; }" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float2 e2m1x2_to_f32(uint32_t byte) {  // .x from bits 0-3
  uint32_t h2;
  const uint16_t t = uint16_t(byte);
  asm("{ .reg .b8 a, z; mov.b16 {a, z}, %1; cvt.rn.f16x2.e2m1x2 %0, a; }" : "=r"(h2) : "h"(t));
  return __half22float2(*reinterpret_cast<const __half2*>(&h2));
}
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {  // 16 bits: lo in bits 0-7
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float2 e4m3x2_to_f32(uint32_t two) {  // .x from bits 0-7
  uint32_t h2;
  const uint16_t t = uint16_t(two);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(t));
  return __half22float2(*reinterpret_cast<const __half2*>(&h2));
}
__device__ __forceinline__ float e2m1_sanitize(float x) { return (x == 0.0f || x != x) ? 0.0f : x; }

// E2M1 grid value (without the scale) of x, by arithmetic on the full-rate
// pipes: round-to-nearest-even at spacing 0.5 below 2, 1 in [2, 4), 2 above,
// saturating at 6 -- the reference's thresholds (grid.py:82-105) -- with the
// reference's sign convention (negative only when x < 0; NaN -> 0).
__device__ __forceinline__ float e2m1_round(float x) {
  float a = fabsf(x);
  a = a == a ? a : 0.0f;
  const float k = a < 2.0f ? 2.0f : (a < 4.0f ? 1.0f : 0.5f);
  const float ik = a < 2.0f ? 0.5f : (a < 4.0f ? 1.0f : 2.0f);
  const float v = fminf(rintf(a * k) * ik, 6.0f);
  return x < 0.0f ? -v : v;
}

// Two MXFP elements at once (scale 2^e, inv = 2^-e): codes packed as in the
// artifact (mxfp4: one byte, element 0 in the low nibble; mxfp8: two bytes,
// element 0 in the low byte) and the dequantized values.
template <int MODE>
__device__ __forceinline__ uint32_t mx_quant2(float w0, float w1, float inv, float sc, float& dq0, float& dq1) {
  float x0 = w0 * inv, x1 = w1 * inv;
  uint32_t codes;
  float2 v;
  if (MODE == GQ_MXFP4) {
    codes = cvt_e2m1x2(e2m1_sanitize(x0), e2m1_sanitize(x1));
    v = e2m1x2_to_f32(codes);
  } else {
    codes = cvt_e4m3x2(x0, x1);
    v = e4m3x2_to_f32(codes);
  }
  dq0 = v.x * sc;
  dq1 = v.y * sc;
  return codes;
}

// Grid value of an MXFP code (without the scale).
template <int MODE>
__device__ __forceinline__ float mx_value(uint32_t code) {
  return MODE == GQ_MXFP4 ? e2m1_value(code) : e4m3_decode(code);
}

// One MXFP element: code and dequantized value for value w with scale 2^e,
// inv = 2^-e (w * 2^-e == w / 2^e exactly, including under/overflow rounding).
template <int MODE>
__device__ __forceinline__ float mx_quant(float w, float inv, float sc, uint32_t& code) {
  float x = w * inv;
  if (MODE == GQ_MXFP4) {
    code = e2m1_code(x);
    return e2m1_value(code) * sc;
  } else {
    x = fminf(fmaxf(x, -448.0f), 448.0f);
    if (w != w) x = w;  // clamp keeps NaN, as torch.clamp does
    code = e4m3_encode(x);
    return e4m3_decode(code) * sc;
  }
}

// ---------------------------------------------------------------------------
// bounded waits (every spin in this library gives up after kWaitLimitNs)
// ---------------------------------------------------------------------------
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up after
// limit_ns (kWaitLimitNs by default) or as soon as another role of the CTA has
// given up, raising *abort_flag and recording GQ_ERR_TIMEOUT in *status (device,
// nullable).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* status, unsigned long long limit_ns = kWaitLimitNs) {
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u) {
      if (*abort_flag) return false;
      unsigned long long now = global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > limit_ns) {
        *abort_flag = 1;
        if (status) atomicExch(status, GQ_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA and tcgen05 wrappers (inline PTX, sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, one elected thread.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns (each thread gets its lane's 32 columns).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// UMMA shared-memory descriptor: SWIZZLE_128B canonical layout, version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;  // descriptor version for sm_100
  d |= uint64_t(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16 with bf16 inputs and f32 accumulate.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                        // D format f32
         | (1u << 7)                      // A bf16
         | (1u << 10)                     // B bf16
         | (uint32_t(a_mn_major) << 15)   // A major-ness
         | (uint32_t(b_mn_major) << 16)   // B major-ness
         | (uint32_t(N >> 3) << 17)       // N / 8
         | (uint32_t(M >> 4) << 24);      // M / 16
}

}  // namespace gq
