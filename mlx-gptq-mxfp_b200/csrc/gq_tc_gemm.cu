// float32 GEMM on the 5th-generation tensor cores for the affine solver: the lazy
// trailing update W[:, i2:] -= Err * U[i1:i2, i2:] of mlx_gptq/gptq.py:269-270 and
// the products of the factorization (gptq.py:27-66).
//
// Persistent CTAs (one per SM) walk 128 x 128 output tiles; K advances in chunks of
// 32. Warp roles:
//   warp 0     TMA: the raw float32 chunk of A and of B (4-D tensor maps: column,
//              row, inner batch, outer batch) into a 2-stage raw ring;
//   warp 1     MMA: per chunk 4 k-steps x 3 tcgen05.mma (kind::tf32, M = N = 128,
//              K = 8) into one of two 128-column TMEM accumulators;
//   warps 2-5  convert: each thread one row of A and one row of B of the chunk,
//              x = hi + lo with hi = rna_tf32(x), lo = x - hi (3xTF32: hi*hi +
//              hi*lo + lo*hi keeps float32 accuracy), written K-major with the
//              128-byte swizzle into a 2-stage ring the MMAs read;
//   warps 6-9  epilogue, overlapping the next tile's main loop: TMEM -> registers ->
//              alpha * acc into a per-warp 32 x 32 staging box -> a TMA reduce-add
//              into C in L2 (beta == 1: the trailing update W -= Err U never reads W
//              into the SM) or a TMA store (beta == 0); other beta: coalesced
//              read-modify-write C = beta * C + alpha * acc.
// A K-contiguous operand arrives already swizzled (TMA SWIZZLE_128B, box 32 x 128);
// an M/N-contiguous one arrives as a plain [32][128] box and is transposed by the
// converting thread. Every wait is bounded (gq_common.cuh: mbar_wait); a wait that
// gives up records GQ_ERR_TIMEOUT in *status (nullable), copies and MMAs already in
// flight are waited for, TMEM is freed and the kernel returns.
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "gq_common.cuh"
#include "gq_gemm.cuh"

namespace gq {
namespace tcg {

constexpr int BM = 128, BN = 128, BK = 32;
constexpr int RAW_STAGES = 2, CONV_STAGES = 2;
constexpr int THREADS = 320;
constexpr uint32_t TILE_BYTES = 128 * 32 * 4;       // one operand chunk: 128 rows x 32 fp32
constexpr uint32_t RAW_BYTES = 2 * TILE_BYTES;      // A, B as loaded
constexpr uint32_t CONV_BYTES = 4 * TILE_BYTES;     // A hi, A lo, B hi, B lo
constexpr int EPI_LD = 33;                          // read-modify-write staging row stride (floats)
constexpr uint32_t EPI_WARP_BYTES = 2 * 4096;       // per epilogue warp: two 32 x 32 fp32 staging tiles
constexpr uint32_t EPI_BYTES = 4 * EPI_WARP_BYTES;
constexpr uint32_t TMEM_COLS = 256;                 // two 128-column accumulators
constexpr uint32_t BAR_OFF = CONV_STAGES * CONV_BYTES + RAW_STAGES * RAW_BYTES + EPI_BYTES;
constexpr size_t SMEM_BYTES = size_t(BAR_OFF) + 16 * 8 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
static_assert(32 * EPI_LD * 4 <= EPI_WARP_BYTES, "read-modify-write staging fits a warp's share");

// How the epilogue writes C: read-modify-write (any beta), a TMA store (beta == 0) or a
// TMA reduce-add in L2 (beta == 1, C += alpha * acc; nothing of C is read by the SM).
enum EpiMode : int { EPI_RMW = 0, EPI_TMA_STORE = 1, EPI_TMA_ADD = 2 };

// Byte offset of (row, fp32 column) in a K-major 128-byte-swizzled 128 x 32 tile.
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t col) {
  return row * 128u + ((((col >> 2) ^ (row & 7u)) << 4) | ((col & 3u) << 2));
}

__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFFu);
  d |= uint64_t(1) << 16;          // leading byte offset (unused: a chunk row is one swizzle atom)
  d |= uint64_t(1024 >> 4) << 32;  // stride byte offset: next group of 8 rows
  d |= uint64_t(1) << 46;          // descriptor version for sm_100
  d |= uint64_t(2) << 61;          // SWIZZLE_128B
  return d;
}

// kind::tf32, f32 accumulate, A and B K-major, N = 128, M = 128
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

// 32 x 32 fp32 box from shared memory to C: plain store, or element-wise add in L2.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z, int w,
                                             bool add) {
  if (add)
    asm volatile(
        "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
  else
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void split4(float4 x, uint4& h, uint4& l) {
  h = make_uint4(tf32_rna(x.x), tf32_rna(x.y), tf32_rna(x.z), tf32_rna(x.w));
  l = make_uint4(__float_as_uint(x.x - __uint_as_float(h.x)), __float_as_uint(x.y - __uint_as_float(h.y)),
                 __float_as_uint(x.z - __uint_as_float(h.z)), __float_as_uint(x.w - __uint_as_float(h.w)));
}

// Row `row` of one operand chunk into the hi / lo tiles. KMAJOR: the raw tile is
// already K-major and swizzled (same offsets); else it is [32 k][128 rows] plain.
template <bool KMAJOR>
__device__ __forceinline__ void convert_row(const uint8_t* raw, uint8_t* hi, uint8_t* lo, uint32_t row) {
  if (KMAJOR) {
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint32_t off = swz(row, 4 * j);
      uint4 h, l;
      split4(*reinterpret_cast<const float4*>(raw + off), h, l);
      *reinterpret_cast<uint4*>(hi + off) = h;
      *reinterpret_cast<uint4*>(lo + off) = l;
    }
  } else {
    const float* r = reinterpret_cast<const float*>(raw);
    float v[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) v[t] = r[t * 128 + row];
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint32_t off = swz(row, 4 * j);
      uint4 h, l;
      split4(make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]), h, l);
      *reinterpret_cast<uint4*>(hi + off) = h;
      *reinterpret_cast<uint4*>(lo + off) = l;
    }
  }
}

// Tile t -> (outer, inner item, m0, n0). lower: only tiles on or below the diagonal
// of a square product (per item tiles_n * (tiles_n + 1) / 2, row by row).
struct TileWalk {
  int64_t tiles, per_item;
  int tiles_n, n_inner, lower;
  const int32_t* skip;
  __device__ bool at(int64_t t, int64_t& o, int64_t& in, int& m0, int& n0) const {
    const int64_t z = t / per_item, r = t % per_item;
    o = z / n_inner;
    in = z % n_inner;
    if (lower) {
      int mi = int((sqrtf(8.0f * float(r) + 1.0f) - 1.0f) * 0.5f);
      while (int64_t(mi + 1) * (mi + 2) / 2 <= r) ++mi;
      while (int64_t(mi) * (mi + 1) / 2 > r) --mi;
      m0 = mi * BM;
      n0 = int(r - int64_t(mi) * (mi + 1) / 2) * BN;
    } else {
      m0 = int(r / tiles_n) * BM;
      n0 = int(r % tiles_n) * BN;
    }
    return !(skip && skip[o]);
  }
};

template <bool A_KMAJOR, bool B_KMAJOR>
__global__ void __launch_bounds__(THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapC, GemmBatch p, TileWalk walk, int epi_mode,
                   int32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* conv = smem;
  uint8_t* raw = smem + CONV_STAGES * CONV_BYTES;
  uint8_t* epi = raw + RAW_STAGES * RAW_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* raw_full = bars;        // [2] TMA bytes landed
  uint64_t* raw_empty = bars + 2;   // [2] converters done reading (128 arrivals)
  uint64_t* conv_full = bars + 4;   // [2] hi / lo written (128 arrivals)
  uint64_t* conv_empty = bars + 6;  // [2] MMAs of the stage done (commit)
  uint64_t* acc_full = bars + 8;    // [2] accumulator complete (commit)
  uint64_t* acc_empty = bars + 10;  // [2] accumulator drained (128 arrivals)
  uint64_t* drain = bars + 12;      // MMAs in flight at an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 128);
      mbar_init(&conv_full[s], 128);
      mbar_init(&conv_empty[s], 1);
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nch = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mapA)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mapB)) : "memory");
      int it = 0, issued = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && t < walk.tiles; t += gridDim.x) {
        int64_t o, in;
        int m0, n0;
        if (!walk.at(t, o, in, m0, n0)) continue;
        for (int c = 0; c < nch; ++c, ++it) {
          const int s = it % RAW_STAGES;
          if (!mbar_wait(&raw_empty[s], ((it / RAW_STAGES) & 1) ^ 1, abort_flag, status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&raw_full[s], RAW_BYTES);
          uint8_t* dst = raw + s * RAW_BYTES;
          const int k0 = c * BK;
          if (A_KMAJOR)
            tma_load_4d(dst, &mapA, k0, m0, int(in), int(o), &raw_full[s]);
          else
            tma_load_4d(dst, &mapA, m0, k0, int(in), int(o), &raw_full[s]);
          if (B_KMAJOR)
            tma_load_4d(dst + TILE_BYTES, &mapB, k0, n0, int(in), int(o), &raw_full[s]);
          else
            tma_load_4d(dst + TILE_BYTES, &mapB, n0, k0, int(in), int(o), &raw_full[s]);
          issued = it + 1;
        }
      }
      if (*abort_flag) {  // let copies already in flight land before the CTA exits
        volatile int never = 0;
        for (int i = issued > RAW_STAGES ? issued - RAW_STAGES : 0; i < issued; ++i)
          mbar_wait(&raw_full[i % RAW_STAGES], (i / RAW_STAGES) & 1, &never, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, tc = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && t < walk.tiles; t += gridDim.x) {
        int64_t o, in;
        int m0, n0;
        if (!walk.at(t, o, in, m0, n0)) continue;
        const int b = tc & 1;
        if (!mbar_wait(&acc_empty[b], ((tc >> 1) & 1) ^ 1, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(b * BN);
        for (int c = 0; c < nch; ++c, ++it) {
          const int s = it % CONV_STAGES;
          if (!mbar_wait(&conv_full[s], (it / CONV_STAGES) & 1, abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_hi = smem_u32(conv + s * CONV_BYTES), a_lo = a_hi + TILE_BYTES,
                         b_hi = a_hi + 2 * TILE_BYTES, b_lo = a_hi + 3 * TILE_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {  // 8 tf32 = 32 bytes per MMA inside the 128-byte rows
            const uint32_t ko = uint32_t(k) * 32u;
            const uint64_t ah = desc_kmajor_sw128(a_hi + ko), al = desc_kmajor_sw128(a_lo + ko);
            const uint64_t bh = desc_kmajor_sw128(b_hi + ko), bl = desc_kmajor_sw128(b_lo + ko);
            mma(d, ah, bh, (c > 0 || k > 0) ? 1u : 0u);
            mma(d, ah, bl, 1u);
            mma(d, al, bh, 1u);
          }
          umma_commit(&conv_empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[b]);
        ++tc;
      }
      if (*abort_flag) {  // MMAs still in flight finish before TMEM is freed
        volatile int never = 0;
        umma_commit(drain);
        mbar_wait(drain, 0, &never, nullptr);
      }
    }
  } else if (warp < 6) {
    const uint32_t row = uint32_t(threadIdx.x - 64);
    int it = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; ok && t < walk.tiles; t += gridDim.x) {
      int64_t o, in;
      int m0, n0;
      if (!walk.at(t, o, in, m0, n0)) continue;
      for (int c = 0; c < nch; ++c, ++it) {
        const int rs = it % RAW_STAGES, cs = it % CONV_STAGES;
        if (!mbar_wait(&raw_full[rs], (it / RAW_STAGES) & 1, abort_flag, status) ||
            !mbar_wait(&conv_empty[cs], ((it / CONV_STAGES) & 1) ^ 1, abort_flag, status)) {
          ok = false;
          break;
        }
        const uint8_t* r = raw + rs * RAW_BYTES;
        uint8_t* cv = conv + cs * CONV_BYTES;
        convert_row<A_KMAJOR>(r, cv, cv + TILE_BYTES, row);
        convert_row<B_KMAJOR>(r + TILE_BYTES, cv + 2 * TILE_BYTES, cv + 3 * TILE_BYTES, row);
        mbar_arrive(&raw_empty[rs]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // hi / lo -> tensor-core proxy
        mbar_arrive(&conv_full[cs]);
      }
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. of this warp
    uint8_t* wbuf = epi + (warp - 6) * EPI_WARP_BYTES;
    int tc = 0, pc = 0;
    for (int64_t t = blockIdx.x; t < walk.tiles; t += gridDim.x) {
      int64_t o, in;
      int m0, n0;
      if (!walk.at(t, o, in, m0, n0)) continue;
      const int b = tc & 1;
      if (!mbar_wait(&acc_full[b], (tc >> 1) & 1, abort_flag, status)) break;
      tc_fence_after();
      const int rb = m0 + quarter * 32;
#pragma unroll 1
      for (int q = 0; q < BN / 32; ++q, ++pc) {
        uint32_t r[32];
        tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(b * BN + q * 32), r);
        tmem_ld_wait();
        if (epi_mode != EPI_RMW) {
          // row `lane` of a 32 x 32 box, 128-byte swizzled like the tensor map's box
          uint8_t* sb = wbuf + (pc & 1) * 4096;
          if (lane == 0) bulk_wait_read_le1();  // the store that used this buffer has read it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(sb + swz(uint32_t(lane), uint32_t(4 * j))) =
                make_float4(p.alpha * __uint_as_float(r[4 * j]), p.alpha * __uint_as_float(r[4 * j + 1]),
                            p.alpha * __uint_as_float(r[4 * j + 2]), p.alpha * __uint_as_float(r[4 * j + 3]));
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) tma_store_4d(&mapC, sb, n0 + q * 32, rb, int(in), int(o), epi_mode == EPI_TMA_ADD);
        } else {
          float* stg = reinterpret_cast<float*>(wbuf);
#pragma unroll
          for (int j = 0; j < 32; ++j) stg[lane * EPI_LD + j] = __uint_as_float(r[j]);
          __syncwarp();
          const int col = n0 + q * 32 + lane;
          if (col < p.N) {
            float* cp = p.Cm + o * p.sc_o + in * p.sc_i + int64_t(rb) * p.ldc + col;
            float cv[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) cv[i] = (p.beta != 0.0f && rb + i < p.M) ? cp[int64_t(i) * p.ldc] : 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (rb + i < p.M) cp[int64_t(i) * p.ldc] = p.beta * cv[i] + p.alpha * stg[i * EPI_LD + lane];
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
      ++tc;
    }
    if (epi_mode != EPI_RMW && lane == 0) bulk_wait_all();  // C written before the kernel ends
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// 4-D float32 tensor map over an operand whose element (r, t) (r: M or N index, t: K
// index) of batch item (outer, inner) sits at base + outer*s_o + inner*s_i + r*ld + t
// (K-contiguous: box 32 x 128, 128-byte swizzle) or + t*ld + r (box 128 x 32, plain).
static int operand_map(CUtensorMap* map, const float* base, bool k_contig, int64_t rows, int64_t K, int64_t ld,
                       int64_t s_i, int64_t n_inner, int64_t s_o, int64_t n_outer) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) {
    set_last_error("cuTensorMapEncodeTiled unavailable");
    return GQ_ERR_CUDA;
  }
  const int64_t d0 = k_contig ? K : rows, d1 = k_contig ? rows : K;
  // a batch dimension of extent 1 is never stepped; give it a valid stride anyway
  const int64_t si = n_inner > 1 ? s_i : ld * d1;
  const int64_t so = n_outer > 1 ? s_o : si * n_inner;
  cuuint64_t dims[4] = {cuuint64_t(d0), cuuint64_t(d1), cuuint64_t(n_inner), cuuint64_t(n_outer)};
  cuuint64_t strides[3] = {cuuint64_t(ld) * 4, cuuint64_t(si) * 4, cuuint64_t(so) * 4};
  cuuint32_t box[4] = {k_contig ? 32u : 128u, k_contig ? 128u : 32u, 1u, 1u};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, k_contig ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d) for a GEMM operand", int(r));
    return GQ_ERR_CUDA;
  }
  return GQ_OK;
}

// 4-D float32 tensor map over C (element (r, c) of item (outer, inner) at base +
// outer*s_o + inner*s_i + r*ld + c), 32 x 32 boxes, 128-byte swizzle.
static int result_map(CUtensorMap* map, float* base, int64_t M, int64_t N, int64_t ld, int64_t s_i,
                      int64_t n_inner, int64_t s_o, int64_t n_outer) {
  EncodeTiledFn enc = tensor_map_encoder();
  if (!enc) {
    set_last_error("cuTensorMapEncodeTiled unavailable");
    return GQ_ERR_CUDA;
  }
  const int64_t si = n_inner > 1 ? s_i : ld * M;
  const int64_t so = n_outer > 1 ? s_o : si * n_inner;
  cuuint64_t dims[4] = {cuuint64_t(N), cuuint64_t(M), cuuint64_t(n_inner), cuuint64_t(n_outer)};
  cuuint64_t strides[3] = {cuuint64_t(ld) * 4, cuuint64_t(si) * 4, cuuint64_t(so) * 4};
  cuuint32_t box[4] = {32u, 32u, 1u, 1u};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d) for a GEMM result", int(r));
    return GQ_ERR_CUDA;
  }
  return GQ_OK;
}

static int sm_count() {
  static std::mutex mu;
  static std::map<int, int> counts;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  auto it = counts.find(dev);
  if (it != counts.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  counts[dev] = n;
  return n;
}

template <bool AK, bool BK_>
static int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const GemmBatch& p,
                     const TileWalk& w, int epi_mode, int32_t* status, cudaStream_t s) {
  {  // the shared-memory opt-in, once per device
    static std::mutex mu;
    static std::map<int, bool> done;
    int dev = 0;
    GQ_CUDA_TRY(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
      GQ_CUDA_TRY(cudaFuncSetAttribute(tc_gemm_kernel<AK, BK_>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(SMEM_BYTES)));
      done[dev] = true;
    }
  }
  const int sms = sm_count();
  const int64_t grid = std::min<int64_t>(w.tiles, sms > 0 ? sms : 148);
  tc_gemm_kernel<AK, BK_><<<unsigned(grid), THREADS, SMEM_BYTES, s>>>(ma, mb, mc, p, w, epi_mode, status);
  return check_launch("tc_gemm_kernel");
}

}  // namespace tcg

// Tensor maps need 16-byte aligned bases and strides that are whole multiples of
// 16 bytes for every operand dimension that is stepped.
bool tc_gemm_usable(const GemmBatch& p, bool trans_a, bool trans_b) {
  (void)trans_a;
  (void)trans_b;
  auto ok = [&](const float* base, int64_t ld, int64_t s_o, int64_t s_i) {
    return (reinterpret_cast<uintptr_t>(base) & 15) == 0 && ld % 4 == 0 && ld > 0 && s_o % 4 == 0 &&
           s_i % 4 == 0 && (p.n_inner == 1 || s_i > 0);
  };
  return p.M > 0 && p.N > 0 && p.K > 0 && p.n_inner > 0 && ok(p.A, p.lda, p.sa_o, p.sa_i) &&
         ok(p.Bm, p.ldb, p.sb_o, p.sb_i);
}

int tc_gemm(const GemmBatch& p, bool trans_a, bool trans_b, int64_t batches, int32_t* status, cudaStream_t s,
            bool lower_only) {
  if (batches <= 0 || p.M <= 0 || p.N <= 0) return GQ_OK;
  GQ_REQUIRE(!lower_only || p.M == p.N, "tc_gemm: lower_only needs a square product");
  GQ_REQUIRE(tc_gemm_usable(p, trans_a, trans_b), "tc_gemm: operand layout not supported");
  GQ_REQUIRE(batches % p.n_inner == 0, "tc_gemm: batch count not a multiple of the inner batch");
  const int64_t n_outer = batches / p.n_inner;
  CUtensorMap ma, mb;
  // op(A)(r, t): K-contiguous unless transposed; op(B)(t, c) read as rows c: K-contiguous if transposed
  int r = tcg::operand_map(&ma, p.A, !trans_a, p.M, p.K, p.lda, p.sa_i, p.n_inner, p.sa_o, n_outer);
  if (r != GQ_OK) return r;
  r = tcg::operand_map(&mb, p.Bm, trans_b, p.N, p.K, p.ldb, p.sb_i, p.n_inner, p.sb_o, n_outer);
  if (r != GQ_OK) return r;
  // C through TMA when beta is 0 or 1 and a tensor map can describe it
  CUtensorMap mc;
  memset(&mc, 0, sizeof(mc));
  int epi = tcg::EPI_RMW;
  const bool c_tma = (reinterpret_cast<uintptr_t>(p.Cm) & 15) == 0 && p.ldc % 4 == 0 && p.ldc > 0 &&
                     p.sc_o % 4 == 0 && p.sc_i % 4 == 0 && (p.n_inner == 1 || p.sc_i > 0);
  if (c_tma && (p.beta == 0.0f || p.beta == 1.0f)) {
    r = tcg::result_map(&mc, p.Cm, p.M, p.N, p.ldc, p.sc_i, p.n_inner, p.sc_o, n_outer);
    if (r != GQ_OK) return r;
    epi = p.beta == 0.0f ? tcg::EPI_TMA_STORE : tcg::EPI_TMA_ADD;
  }
  tcg::TileWalk w;
  w.tiles_n = (p.N + tcg::BN - 1) / tcg::BN;
  w.lower = lower_only ? 1 : 0;
  w.per_item = lower_only ? int64_t(w.tiles_n) * (w.tiles_n + 1) / 2
                          : int64_t((p.M + tcg::BM - 1) / tcg::BM) * w.tiles_n;
  w.tiles = w.per_item * batches;
  w.n_inner = p.n_inner;
  w.skip = p.skip;
  if (!trans_a && trans_b) return tcg::launch_tc<true, true>(ma, mb, mc, p, w, epi, status, s);
  if (!trans_a) return tcg::launch_tc<true, false>(ma, mb, mc, p, w, epi, status, s);
  if (trans_b) return tcg::launch_tc<false, true>(ma, mb, mc, p, w, epi, status, s);
  return tcg::launch_tc<false, false>(ma, mb, mc, p, w, epi, status, s);
}

}  // namespace gq
