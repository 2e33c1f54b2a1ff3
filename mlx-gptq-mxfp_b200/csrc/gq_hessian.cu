// Hessian accumulation H = beta*H + alpha * X^T X on the 5th-generation tensor
// cores (replaces mlx_gptq/capture.py:68-76, Stash.hessian).
//
// X is bf16 [n tokens, c channels], row-major. Both GEMM operands are X itself:
// A[m][k] = X[k][i0 + m] and B[j][k] = X[k][j0 + j], i.e. both "MN-major" (the
// output index is the contiguous one), which tcgen05 consumes directly from
// 128-byte-swizzled shared memory -- no transpose pass.
//
// One CTA per 128 x 256 output tile on or above the diagonal (H is symmetric;
// the epilogue mirrors). Warp roles: warp 0 = TMA producer, warp 1 = TMEM owner
// and MMA issuer, warps 2-9 = accumulator warps (TMEM lanes 32*(warp%4) .. +31,
// column half (warp-2)/4).
//
// Precision: the tensor core's fp32 accumulation is biased (it loses ~1e-7
// relative per MMA step, always toward zero), so one accumulator over 131072
// tokens drifts by ~7e-4. The token range is therefore cut into chunks of
// kChunkTiles * 64 tokens; each chunk accumulates in one of two TMEM buffers
// (2 x 256 columns) while the accumulator warps add the previous chunk into
// fp32 registers with round-to-nearest adds. Error stays ~2e-6 relative, the
// tensor pipe never waits, and no extra memory traffic is generated.
// Pipeline: 4 stages x (A 128x64 + B 256x64 bf16) = 192 KB of shared memory.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "gq_common.cuh"

namespace gq {
namespace hess {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int EPI_WARPS = 8, THREADS = 64 + 32 * EPI_WARPS;
constexpr int kChunkTiles = 16;                      // 1024 tokens per TMEM chunk
constexpr uint32_t BOX_BYTES = 64 * 64 * 2;          // one 64-channel x 64-token TMA box
constexpr uint32_t A_BYTES = BM * BK * 2;            // 16 KB
constexpr uint32_t B_BYTES = BN * BK * 2;            // 32 KB
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr uint32_t TMEM_COLS = 512;                  // two 256-column accumulators
constexpr size_t SMEM_BYTES = size_t(STAGES) * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;

// Tiles (tm, tn) with tm <= 2*tn + 1 touch the upper triangle; enumerate them
// column-panel by column-panel (neighbouring CTAs share the B panel in L2).
__host__ __device__ inline int64_t tiles_in_panel(int64_t tn, int64_t mt) { return 2 * tn + 2 < mt ? 2 * tn + 2 : mt; }

__host__ inline int64_t num_tiles(int64_t c) {
  const int64_t mt = (c + BM - 1) / BM, nt = (c + BN - 1) / BN;
  int64_t t = 0;
  for (int64_t tn = 0; tn < nt; ++tn) t += tiles_in_panel(tn, mt);
  return t;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Write one accumulator row slab: row gr, columns cb .. cb+127 of the tile
// (acc scaled in place by alpha). Elements on or above the diagonal go to
// H[gr][col] (= beta*H + value), strictly-above ones also to the mirror H[col][gr];
// all_upper: every column of the tile is above every row (no masking).
__device__ __forceinline__ void store_row_slab(float* __restrict__ H, int64_t ldh, int64_t c, int64_t gr,
                                               int64_t cb, float (&acc)[128], float alpha, float beta,
                                               bool all_upper) {
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    const int64_t c0 = cb + q4 * 32;
    if (c0 >= c) break;
    float* v = acc + q4 * 32;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = alpha * v[j];
    if (gr < c) {
      float* hp = H + gr * ldh + c0;
      if (all_upper && c0 + 32 <= c) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          if (beta != 0.0f) {
            const float4 h = *reinterpret_cast<const float4*>(hp + j);
            o.x = beta * h.x + o.x, o.y = beta * h.y + o.y, o.z = beta * h.z + o.z, o.w = beta * h.w + o.w;
          }
          *reinterpret_cast<float4*>(hp + j) = o;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int64_t gc = c0 + j;
          if (gc >= gr && gc < c) hp[j] = beta != 0.0f ? beta * hp[j] + v[j] : v[j];
        }
      }
    }
    // mirror (strictly lower) part: H[gc][gr] for gc > gr; lanes hold consecutive gr
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int64_t gc = c0 + j;
      if (gc > gr && gc < c && gr < c) {
        float* hp = H + gc * ldh + gr;
        *hp = beta != 0.0f ? beta * *hp + v[j] : v[j];
      }
    }
  }
}

// Grouped form: `sched` (nullable) lists one entry per CTA, expert * tiles_per_expert +
// tile (heaviest experts first); expert e's rows are X rows seg[e] .. seg[e+1] (a
// multiple of 64, zero-padded by the gather pass) and its output is H + e*c*ldh.
// Dense form (sched == nullptr): one expert, rows 0 .. n.
__global__ void __launch_bounds__(THREADS, 1)
    hessian_kernel(const __grid_constant__ CUtensorMap tmap, int64_t n, int64_t c, float* __restrict__ H,
                   int64_t ldh, float alpha, float beta, int32_t* status, const int32_t* __restrict__ sched,
                   const int64_t* __restrict__ seg, int64_t tiles_per_expert, int64_t tile_begin) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2] chunk accumulated in TMEM buffer b
  uint64_t* tempty = tfull + 2;      // [2] TMEM buffer b drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t mt = (c + BM - 1) / BM;
  int64_t t = blockIdx.x + tile_begin, tn = 0, y0 = 0;
  if (sched) {
    const int64_t v = sched[blockIdx.x], e = v / tiles_per_expert;
    t = v % tiles_per_expert;
    y0 = seg[e];
    n = seg[e + 1] - y0;
    H += e * c * ldh;
  }
  while (t >= tiles_in_panel(tn, mt)) {
    t -= tiles_in_panel(tn, mt);
    ++tn;
  }
  const int64_t tm = t;
  const int KT = int((n + BK - 1) / BK);
  const int NCH = (KT + kChunkTiles - 1) / kChunkTiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, status)) break;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        uint8_t* st = smem + s * STAGE_BYTES;
        const int y = int(y0) + kt * BK;
        const int xa = int(tm * BM), xb = int(tn * BN);
        tma_load_2d(st, &tmap, xa, y, &full[s]);
        tma_load_2d(st + BOX_BYTES, &tmap, xa + 64, y, &full[s]);
#pragma unroll
        for (int i = 0; i < 4; ++i) tma_load_2d(st + A_BYTES + i * BOX_BYTES, &tmap, xb + 64 * i, y, &full[s]);
        issued = kt + 1;
      }
      if (*abort_flag) {  // let copies already in flight land before the CTA exits
        volatile int never = 0;
        for (int kt = issued > STAGES ? issued - STAGES : 0; kt < issued; ++kt)
          mbar_wait(&full[kt % STAGES], (kt / STAGES) & 1, &never, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, true, true);
      for (int kt = 0; kt < KT; ++kt) {
        const int ch = kt / kChunkTiles, buf = ch & 1;
        const bool chunk_start = kt % kChunkTiles == 0;
        const bool chunk_end = kt % kChunkTiles == kChunkTiles - 1 || kt == KT - 1;
        if (chunk_start && !mbar_wait(&tempty[buf], ((ch >> 1) & 1) ^ 1, abort_flag, status)) break;
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + s * STAGE_BYTES), b0 = a0 + A_BYTES;
        const uint32_t d = tmem + uint32_t(buf * BN);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // K advances 16 rows of 128 B inside the swizzled boxes; LBO = next
          // 64-channel box, SBO = next 8-row core-matrix group.
          const uint64_t ad = umma_desc_sw128(a0 + kk * 2048, BOX_BYTES, 1024);
          const uint64_t bd = umma_desc_sw128(b0 + kk * 2048, BOX_BYTES, 1024);
          umma_f16(d, ad, bd, idesc, (!chunk_start || kk != 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
        if (chunk_end) umma_commit(&tfull[buf]);
      }
    }
  } else {
    // accumulator warps: drain each chunk into fp32 registers, then write H
    const int qw = warp & 3, half = (warp - 2) >> 2;
    const uint32_t lane_base = uint32_t(qw * 32) << 16;
    float acc[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) acc[j] = 0.0f;
    bool ok = true;
    for (int ch = 0; ch < NCH; ++ch) {
      const int buf = ch & 1;
      ok = mbar_wait(&tfull[buf], (ch >> 1) & 1, abort_flag, status);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + uint32_t(buf * BN + half * 128 + q4 * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[q4 * 32 + j] = acc[q4 * 32 + j] + __uint_as_float(r[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (ok && !*abort_flag) {  // KT == 0 (an expert without tokens): writes beta * H
      const int64_t gr = tm * BM + qw * 32 + lane;
      store_row_slab(H, ldh, c, gr, tn * BN + half * 128, acc, alpha, beta, tn * BN > tm * BM + BM - 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs computes one 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256). Each CTA loads only its own 128 rows of A
// and its half (128 columns) of B -- 32 KB per 64-token step instead of 48 KB --
// so six stages fit in shared memory and hold 50% more MMA work in flight, and
// L2 reads drop by a third. The even CTA of the pair issues the MMAs; both CTAs'
// TMA bytes land on its stage barriers; its commits reach both CTAs' barriers.
// Each CTA drains its own TMEM rows as in the 1-SM kernel.
// ---------------------------------------------------------------------------
namespace two {
constexpr int STAGES = 6;
constexpr uint32_t HALF_BYTES = 128 * BK * 2;            // 16 KB: 128 channels x 64 tokens
constexpr uint32_t STAGE_BYTES = 2 * HALF_BYTES;         // A half + B half per CTA
constexpr size_t SMEM_BYTES = size_t(STAGES) * STAGE_BYTES + 1024 + 512;
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;          // shared::cluster address -> even CTA of the pair

__host__ __device__ inline int64_t tiles(int64_t c) {
  const int64_t t = (c + 255) / 256;
  return t * (t + 1) / 2;
}

// Tile order: the upper triangle of T x T tiles (tm <= tn) in super-tiles of
// kSuper x kSuper tiles, super-tiles (I <= J) row by row, tiles inside row by row.
// CTAs run in launch order in waves of ~74 clusters, so a wave covers about one
// super-tile: it reads 2 * kSuper * 256 channels of every 64-token slab of X
// instead of all of them, which cuts DRAM re-reads of X by ~3x at C = 11008.
constexpr int64_t kSuper = 8;
__device__ inline void tile_of(int64_t q, int64_t T, int64_t& tm, int64_t& tn) {
  const int64_t ST = (T + kSuper - 1) / kSuper;
  for (int64_t I = 0; I < ST; ++I) {
    const int64_t r0 = I * kSuper, r1 = r0 + kSuper < T ? r0 + kSuper : T;
    for (int64_t J = I; J < ST; ++J) {
      const int64_t c0 = J * kSuper, c1 = c0 + kSuper < T ? c0 + kSuper : T;
      int64_t cnt;
      if (I < J) {
        cnt = (r1 - r0) * (c1 - c0);
        if (q < cnt) {
          tm = r0 + q / (c1 - c0);
          tn = c0 + q % (c1 - c0);
          return;
        }
      } else {  // diagonal super-tile: tm <= tn inside it, row by row
        cnt = (r1 - r0) * (r1 - r0 + 1) / 2;
        if (q < cnt) {
          for (int64_t m = r0; m < r1; ++m) {
            const int64_t row = r1 - m;  // tiles (m, m..r1-1)
            if (q < row) {
              tm = m;
              tn = m + q;
              return;
            }
            q -= row;
          }
        }
      }
      q -= cnt;
    }
  }
  tm = tn = 0;  // unreachable for q < tiles(c)
}

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2sm(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar) & kPeerBitMask)
      : "memory");
}
__device__ __forceinline__ void umma_f16_2sm(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on the barrier at this smem offset in both CTAs once the issued MMAs complete.
__device__ __forceinline__ void umma_commit_2sm(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(uint16_t(3))
      : "memory");
}
}  // namespace two

// Span form (span != nullptr): expert e's rows are X[span[2e] .. span[2e] + span[2e+1]),
// read in place with tiled loads (tmap over X); its partial last 64-row step, if any,
// comes from a tail buffer (tail_map, rows tail_off[e] .. +63: the remaining rows, then
// zeros), so a step never reads another expert's rows and nothing is copied but tails.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    hessian2_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap tail_map,
                    int64_t n, int64_t c, float* __restrict__ H, int64_t ldh, float alpha, float beta,
                    int32_t* status, const int32_t* __restrict__ sched, const int64_t* __restrict__ seg,
                    int64_t tiles_per_expert, int64_t tile_begin, const int64_t* __restrict__ span,
                    const int64_t* __restrict__ tail_off) {
  constexpr int STAGES = two::STAGES;
  constexpr uint32_t STAGE_BYTES = two::STAGE_BYTES, HALF_BYTES = two::HALF_BYTES;
  using two::arrive_remote;
  using two::cluster_sync;
  using two::cta_rank;
  using two::mapa;
  using two::tma_load_2sm;
  using two::umma_commit_2sm;
  using two::umma_f16_2sm;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2] chunk accumulated in TMEM buffer b (both CTAs)
  uint64_t* tempty = tfull + 2;      // [2] buffer b drained by both CTAs (used in the even CTA)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank();
  int64_t q = (blockIdx.x >> 1) + tile_begin, y0 = 0, ytail = 0;
  if (sched) {
    const int64_t v = sched[q], e = v / tiles_per_expert;
    q = v % tiles_per_expert;
    if (span) {
      y0 = span[2 * e];
      n = span[2 * e + 1];
      ytail = tail_off[e];
    } else {
      y0 = seg[e];
      n = seg[e + 1] - y0;
    }
    H += e * c * ldh;
  }
  int64_t tm, tn;
  two::tile_of(q, (c + 255) / 256, tm, tn);
  const int KT = int((n + BK - 1) / BK);
  const int full_steps = span ? int(n / BK) : KT;  // steps read in place; the rest from the tail buffer
  const int NCH = (KT + kChunkTiles - 1) / kChunkTiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      if (span) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tail_map)) : "memory");
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, status)) break;
        if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);  // both CTAs' bytes
        uint8_t* st = smem + s * STAGE_BYTES;
        const bool tail = kt >= full_steps;
        const CUtensorMap* m = tail ? &tail_map : &tmap;
        const int y = tail ? int(ytail) : int(y0) + kt * BK;
        const int xa = int(tm * 256 + rank * 128), xb = int(tn * 256 + rank * 128);
        tma_load_2sm(st, m, xa, y, &full[s]);
        tma_load_2sm(st + BOX_BYTES, m, xa + 64, y, &full[s]);
        tma_load_2sm(st + HALF_BYTES, m, xb, y, &full[s]);
        tma_load_2sm(st + HALF_BYTES + BOX_BYTES, m, xb + 64, y, &full[s]);
        issued = kt + 1;
      }
      if (*abort_flag && rank == 0) {  // let copies already in flight land before the CTA exits
        volatile int never = 0;
        for (int kt = issued > STAGES ? issued - STAGES : 0; kt < issued; ++kt)
          mbar_wait(&full[kt % STAGES], (kt / STAGES) & 1, &never, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(256, BN, true, true);
      for (int kt = 0; kt < KT; ++kt) {
        const int ch = kt / kChunkTiles, buf = ch & 1;
        const bool chunk_start = kt % kChunkTiles == 0;
        const bool chunk_end = kt % kChunkTiles == kChunkTiles - 1 || kt == KT - 1;
        if (chunk_start && !mbar_wait(&tempty[buf], ((ch >> 1) & 1) ^ 1, abort_flag, status)) break;
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(smem + s * STAGE_BYTES), b0 = a0 + HALF_BYTES;
        const uint32_t d = tmem + uint32_t(buf * BN);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(a0 + kk * 2048, BOX_BYTES, 1024);
          const uint64_t bd = umma_desc_sw128(b0 + kk * 2048, BOX_BYTES, 1024);
          umma_f16_2sm(d, ad, bd, idesc, (!chunk_start || kk != 0) ? 1u : 0u);
        }
        umma_commit_2sm(&empty[s]);
        if (chunk_end) umma_commit_2sm(&tfull[buf]);
      }
    }
  } else {
    const int qw = warp & 3, half = (warp - 2) >> 2;
    const uint32_t lane_base = uint32_t(qw * 32) << 16;
    const uint32_t tempty_even0 = mapa(smem_u32(&tempty[0]), 0), tempty_even1 = mapa(smem_u32(&tempty[1]), 0);
    float acc[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) acc[j] = 0.0f;
    bool ok = true;
    for (int ch = 0; ch < NCH; ++ch) {
      const int buf = ch & 1;
      ok = mbar_wait(&tfull[buf], (ch >> 1) & 1, abort_flag, status);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + uint32_t(buf * BN + half * 128 + q4 * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[q4 * 32 + j] = acc[q4 * 32 + j] + __uint_as_float(r[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_remote(buf ? tempty_even1 : tempty_even0);
    }
    if (ok && !*abort_flag) {
      const int64_t gr = tm * 256 + rank * 128 + qw * 32 + lane;
      store_row_slab(H, ldh, c, gr, tn * 256 + half * 128, acc, alpha, beta, tn > tm);
    }
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// H = beta * H for the empty-token case
__global__ void scale_kernel(float* H, int64_t c, int64_t ldh, float beta) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= c * c) return;
  float* p = H + (i / c) * ldh + (i % c);
  *p = beta == 0.0f ? 0.0f : beta * *p;
}

static EncodeTiledFn encode_fn() { return tensor_map_encoder(); }

// 2-D bf16 tensor map over X [rows, cols] (row stride ld elements), 64 x 64 boxes, 128B swizzle.
int make_x_map(CUtensorMap* map, const void* X, int64_t rows, int64_t cols, int64_t ld) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_last_error("cuTensorMapEncodeTiled unavailable");
    return GQ_ERR_CUDA;
  }
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(X), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d)", int(r));
    return GQ_ERR_CUDA;
  }
  return GQ_OK;
}

}  // namespace hess
}  // namespace gq

using namespace gq;

namespace gq {
namespace hess {
// Copy each expert's routed rows into a contiguous, 64-row-padded segment:
// dst rows seg[e] .. seg[e+1] = X[token_idx[offsets[e] ..]] then zeros.
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ X, int64_t c, int64_t ldx,
                                   const int32_t* __restrict__ token_idx, const int64_t* __restrict__ offsets,
                                   const int64_t* __restrict__ seg, int64_t E, int64_t total,
                                   __nv_bfloat16* __restrict__ dst) {
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= total) return;
  int64_t lo = 0, hi = E;  // find e with seg[e] <= row < seg[e+1]
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (seg[mid] <= row) lo = mid; else hi = mid;
  }
  const int64_t local = row - seg[lo];
  const int64_t cnt = offsets[lo + 1] - offsets[lo];
  uint4* d = reinterpret_cast<uint4*>(dst + row * c);
  const int64_t nvec = c / 8;
  if (local < cnt) {
    const uint4* src = reinterpret_cast<const uint4*>(X + int64_t(token_idx[offsets[lo] + local]) * ldx);
    for (int64_t i = lane; i < nvec; i += 32) d[i] = src[i];
  } else {
    for (int64_t i = lane; i < nvec; i += 32) d[i] = make_uint4(0, 0, 0, 0);
  }
}

// Span form: tail slot t (expert tail_expert[t]) gets rows 64t .. 64t+63 = the rows of
// the expert's partial last step, then zeros.
__global__ void span_tails_kernel(const __nv_bfloat16* __restrict__ X, int64_t c, int64_t ldx,
                                  const int64_t* __restrict__ span, const int32_t* __restrict__ tail_expert,
                                  int64_t rows, __nv_bfloat16* __restrict__ dst) {
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t e = tail_expert[row / BK], i = row % BK;
  const int64_t cnt = span[2 * e + 1], first = cnt / BK * BK;
  uint4* d = reinterpret_cast<uint4*>(dst + row * c);
  const int64_t nvec = c / 8;
  if (first + i < cnt) {
    const uint4* src = reinterpret_cast<const uint4*>(X + (span[2 * e] + first + i) * ldx);
    for (int64_t k = lane; k < nvec; k += 32) d[k] = src[k];
  } else {
    for (int64_t k = lane; k < nvec; k += 32) d[k] = make_uint4(0, 0, 0, 0);
  }
}

// Span-form plan: tail slots, and the CTA schedule (experts by descending rows).
struct SpanPlan {
  std::vector<int64_t> tail_off;     // E: first tail-buffer row (0 when the expert has no tail)
  std::vector<int32_t> tail_expert;  // tail slot -> expert
  std::vector<int32_t> sched;
};

static SpanPlan plan_spans(const int64_t* host_spans, int64_t E, int64_t tpe) {
  SpanPlan p;
  p.tail_off.assign(E, 0);
  std::vector<int64_t> order(E);
  for (int64_t e = 0; e < E; ++e) {
    order[e] = e;
    if (host_spans[2 * e + 1] % BK) {
      p.tail_off[e] = int64_t(p.tail_expert.size()) * BK;
      p.tail_expert.push_back(int32_t(e));
    }
  }
  std::stable_sort(order.begin(), order.end(),
                   [&](int64_t a, int64_t b) { return host_spans[2 * a + 1] > host_spans[2 * b + 1]; });
  p.sched.reserve(E * tpe);
  for (int64_t e : order)
    for (int64_t t = 0; t < tpe; ++t) p.sched.push_back(int32_t(e * tpe + t));
  return p;
}

struct GroupedPlan {
  std::vector<int64_t> seg;     // E + 1 padded row starts
  std::vector<int32_t> sched;   // one entry per CTA
  int64_t total = 0;            // padded rows
};

static GroupedPlan plan_grouped(const int64_t* host_offsets, int64_t E, int64_t tpe) {
  GroupedPlan p;
  p.seg.resize(E + 1);
  p.seg[0] = 0;
  for (int64_t e = 0; e < E; ++e) {
    const int64_t cnt = host_offsets[e + 1] - host_offsets[e];
    p.seg[e + 1] = p.seg[e] + (cnt + BK - 1) / BK * BK;
  }
  p.total = p.seg[E];
  std::vector<int64_t> order(E);
  for (int64_t e = 0; e < E; ++e) order[e] = e;
  std::stable_sort(order.begin(), order.end(), [&](int64_t a, int64_t b) {
    return (p.seg[a + 1] - p.seg[a]) > (p.seg[b + 1] - p.seg[b]);
  });
  p.sched.reserve(E * tpe);
  for (int64_t e : order)
    for (int64_t t = 0; t < tpe; ++t) p.sched.push_back(int32_t(e * tpe + t));
  return p;
}
// Kernel choice: 256x256 tiles on CTA pairs (default; ~9% faster at C = 11008), or
// GQ_HESSIAN_KERNEL=1sm for 128x256 tiles on one CTA each.
static bool use_2sm() {
  const char* v = getenv("GQ_HESSIAN_KERNEL");
  return !(v && v[0] == '1');
}
static int64_t tiles_for(int64_t c, bool two_sm) { return two_sm ? two::tiles(c) : num_tiles(c); }

static int launch(const CUtensorMap& map, int64_t n, int64_t c, float* H, int64_t ldh, float alpha, float beta,
                  int32_t* status, const int32_t* sched, const int64_t* seg, int64_t tpe, int64_t units,
                  bool two_sm, cudaStream_t s, int64_t tile_begin = 0, const CUtensorMap* tail_map = nullptr,
                  const int64_t* span = nullptr, const int64_t* tail_off = nullptr) {
  if (two_sm) {
    GQ_CUDA_TRY(cudaFuncSetAttribute(hessian2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     int(two::SMEM_BYTES)));
    hessian2_kernel<<<unsigned(2 * units), THREADS, two::SMEM_BYTES, s>>>(
        map, tail_map ? *tail_map : map, n, c, H, ldh, alpha, beta, status, sched, seg, tpe, tile_begin, span,
        tail_off);
    return check_launch("hessian2_kernel");
  }
  GQ_CUDA_TRY(cudaFuncSetAttribute(hessian_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(SMEM_BYTES)));
  hessian_kernel<<<unsigned(units), THREADS, SMEM_BYTES, s>>>(map, n, c, H, ldh, alpha, beta, status, sched, seg,
                                                              tpe, tile_begin);
  return check_launch("hessian_kernel");
}
}  // namespace hess
}  // namespace gq

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

extern "C" size_t gq_hessian_grouped_workspace_size(const int64_t* host_offsets, int64_t E, int64_t c) {
  if (!host_offsets || E <= 0 || c <= 0) return 0;
  int64_t total = 0;
  for (int64_t e = 0; e < E; ++e) total += (host_offsets[e + 1] - host_offsets[e] + 63) / 64 * 64;
  return align256(size_t(total) * size_t(c) * 2) + align256(size_t(E + 1) * 8) +
         align256(size_t(E) * size_t(std::max(gq::hess::num_tiles(c), gq::hess::two::tiles(c))) * 4);
}

extern "C" int gq_hessian_grouped_bf16(const void* X, int64_t n, int64_t c, int64_t ldx, const int32_t* token_idx,
                                       const int64_t* offsets, const int64_t* host_offsets, int64_t E, float* H,
                                       float alpha, float beta, void* workspace, size_t workspace_bytes,
                                       int32_t* status, void* stream) {
  GQ_REQUIRE(H && offsets && host_offsets && E > 0, "gq_hessian_grouped_bf16: null pointer or E <= 0");
  GQ_REQUIRE(c > 0 && c % 8 == 0 && ldx >= c && ldx % 8 == 0, "gq_hessian_grouped_bf16: c, ldx must be multiples of 8");
  GQ_REQUIRE(aligned16(H), "gq_hessian_grouped_bf16: H must be 16-byte aligned");
  for (int64_t e = 0; e < E; ++e)
    GQ_REQUIRE(host_offsets[e + 1] >= host_offsets[e], "gq_hessian_grouped_bf16: offsets must be non-decreasing");
  GQ_REQUIRE(host_offsets[0] == 0, "gq_hessian_grouped_bf16: offsets[0] must be 0");
  const size_t need = gq_hessian_grouped_workspace_size(host_offsets, E, c);
  GQ_REQUIRE(workspace && workspace_bytes >= need && aligned16(workspace),
             "gq_hessian_grouped_bf16: workspace too small (%zu < %zu)", workspace_bytes, need);
  GQ_REQUIRE(host_offsets[E] == 0 || (X && token_idx && aligned16(X)), "gq_hessian_grouped_bf16: X / token_idx");
  const bool two_sm = hess::use_2sm();
  const int64_t tpe = hess::tiles_for(c, two_sm);
  hess::GroupedPlan plan = hess::plan_grouped(host_offsets, E, tpe);
  GQ_REQUIRE(plan.total < (int64_t(1) << 31) && int64_t(plan.sched.size()) < (int64_t(1) << 31),
             "gq_hessian_grouped_bf16: too many rows");
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  __nv_bfloat16* Xg = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += align256(size_t(plan.total) * size_t(c) * 2);
  int64_t* seg = reinterpret_cast<int64_t*>(ws);
  ws += align256(size_t(E + 1) * 8);
  int32_t* sched = reinterpret_cast<int32_t*>(ws);
  GQ_CUDA_TRY(cudaMemcpyAsync(seg, plan.seg.data(), size_t(E + 1) * 8, cudaMemcpyHostToDevice, s));
  GQ_CUDA_TRY(cudaMemcpyAsync(sched, plan.sched.data(), plan.sched.size() * 4, cudaMemcpyHostToDevice, s));
  if (plan.total > 0) {
    hess::gather_rows_kernel<<<unsigned((plan.total + 7) / 8), 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(X), c, ldx, token_idx, offsets, seg, E, plan.total, Xg);
    int st = check_launch("gather_rows_kernel");
    if (st != GQ_OK) return st;
  }
  CUtensorMap map;
  // a map needs at least one row; with no routed rows at all every CTA has KT == 0
  int st = hess::make_x_map(&map, plan.total > 0 ? (const void*)Xg : workspace, plan.total > 0 ? plan.total : 1, c, c);
  if (st != GQ_OK) return st;
  return hess::launch(map, 0, c, H, c, alpha, beta, status, sched, seg, tpe, int64_t(plan.sched.size()), two_sm, s);
}

extern "C" int64_t gq_hessian_tile_count(int64_t c) {
  if (c <= 0) return 0;
  return gq::hess::tiles_for(c, gq::hess::use_2sm());
}

extern "C" int64_t gq_hessian_concurrent_tiles(int64_t sm_count) {
  if (sm_count <= 0) return 0;
  return gq::hess::use_2sm() ? sm_count / 2 : sm_count;  // one tile per CTA pair, or per CTA
}

extern "C" int gq_hessian_bf16_range(const void* X, int64_t n, int64_t c, int64_t ldx, float* H, int64_t ldh,
                                     float alpha, float beta, int64_t tile_begin, int64_t tile_end, int32_t* status,
                                     void* stream) {
  GQ_REQUIRE(H && (X || n == 0), "gq_hessian_bf16: null pointer");
  GQ_REQUIRE(n >= 0 && c > 0 && n < (int64_t(1) << 31) && c < (int64_t(1) << 31), "gq_hessian_bf16: sizes");
  GQ_REQUIRE(ldh >= c && ldh % 4 == 0 && aligned16(H), "gq_hessian_bf16: H must be 16-byte aligned, ldh %% 4 == 0");
  const bool two_sm = hess::use_2sm();
  const int64_t tiles = hess::tiles_for(c, two_sm);
  GQ_REQUIRE(tile_begin >= 0 && tile_begin <= tile_end && tile_end <= tiles,
             "gq_hessian_bf16_range: tile range [%lld, %lld) outside [0, %lld)", (long long)tile_begin,
             (long long)tile_end, (long long)tiles);
  cudaStream_t s = (cudaStream_t)stream;
  if (tile_end == tile_begin) return GQ_OK;
  if (n == 0) {
    GQ_REQUIRE(tile_begin == 0 && tile_end == tiles, "gq_hessian_bf16_range: n == 0 needs the full tile range");
    if (beta == 1.0f) return GQ_OK;
    hess::scale_kernel<<<unsigned((c * c + 255) / 256), 256, 0, s>>>(H, c, ldh, beta);
    return check_launch("hessian scale_kernel");
  }
  GQ_REQUIRE(ldx >= c && ldx % 8 == 0 && aligned16(X), "gq_hessian_bf16: X must be 16-byte aligned, ldx %% 8 == 0");
  CUtensorMap map;
  int st = hess::make_x_map(&map, X, n, c, ldx);
  if (st != GQ_OK) return st;
  return hess::launch(map, n, c, H, ldh, alpha, beta, status, nullptr, nullptr, tiles, tile_end - tile_begin, two_sm,
                      s, tile_begin);
}

extern "C" int gq_hessian_bf16(const void* X, int64_t n, int64_t c, int64_t ldx, float* H, int64_t ldh, float alpha,
                               float beta, int32_t* status, void* stream) {
  GQ_REQUIRE(c > 0, "gq_hessian_bf16: sizes");
  return gq_hessian_bf16_range(X, n, c, ldx, H, ldh, alpha, beta, 0, gq_hessian_tile_count(c), status, stream);
}

static size_t spans_tail_bytes(const int64_t* host_spans, int64_t E, int64_t c) {
  int64_t tails = 0;
  for (int64_t e = 0; e < E; ++e) tails += host_spans[2 * e + 1] % 64 ? 1 : 0;
  return align256(size_t(std::max<int64_t>(tails, 1)) * 64 * size_t(c) * 2);
}

extern "C" size_t gq_hessian_spans_workspace_size(const int64_t* host_spans, int64_t E, int64_t c) {
  if (!host_spans || E <= 0 || c <= 0) return 0;
  return spans_tail_bytes(host_spans, E, c) + align256(size_t(E) * 16) + 2 * align256(size_t(E) * 8) +
         align256(size_t(E) * size_t(gq::hess::two::tiles(c)) * 4);
}

namespace gq {
namespace hess {
// H[targets[t]] += H[p] for p = pieces[piece_ptr[t]], ..., pieces[piece_ptr[t+1] - 1], added
// one after another in that order (bit-identical to adding them one by one).
template <int V>
__global__ void merge_pieces_kernel(float* __restrict__ H, int64_t cc, const int64_t* __restrict__ targets,
                                    const int64_t* __restrict__ piece_ptr, const int64_t* __restrict__ pieces) {
  const int64_t t = blockIdx.y;
  const int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * V;
  if (i >= cc) return;
  float* dst = H + targets[t] * cc + i;
  const int64_t p0 = piece_ptr[t], p1 = piece_ptr[t + 1];
  if (V == 4) {
    float4 acc = *reinterpret_cast<const float4*>(dst);
    for (int64_t p = p0; p < p1; ++p) {
      const float4 v = *reinterpret_cast<const float4*>(H + pieces[p] * cc + i);
      acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
    }
    *reinterpret_cast<float4*>(dst) = acc;
  } else {
    float acc = *dst;
    for (int64_t p = p0; p < p1; ++p) acc += H[pieces[p] * cc + i];
    *dst = acc;
  }
}
}  // namespace hess
}  // namespace gq

extern "C" int gq_hessian_merge_pieces(float* H, int64_t c, int64_t n_targets, const int64_t* targets,
                                       const int64_t* piece_ptr, const int64_t* pieces, void* stream) {
  GQ_REQUIRE(c > 0 && n_targets >= 0, "gq_hessian_merge_pieces: sizes");
  if (n_targets == 0) return GQ_OK;
  GQ_REQUIRE(H && targets && piece_ptr && pieces, "gq_hessian_merge_pieces: null pointer");
  GQ_REQUIRE(n_targets < 65536, "gq_hessian_merge_pieces: too many targets");
  const int64_t cc = c * c;
  cudaStream_t s = (cudaStream_t)stream;
  if (cc % 4 == 0 && aligned16(H)) {
    const dim3 grid(unsigned((cc / 4 + 255) / 256), unsigned(n_targets));
    gq::hess::merge_pieces_kernel<4><<<grid, 256, 0, s>>>(H, cc, targets, piece_ptr, pieces);
  } else {
    const dim3 grid(unsigned((cc + 255) / 256), unsigned(n_targets));
    gq::hess::merge_pieces_kernel<1><<<grid, 256, 0, s>>>(H, cc, targets, piece_ptr, pieces);
  }
  return check_launch("merge_pieces_kernel");
}

extern "C" int gq_hessian_spans_bf16(const void* X, int64_t n, int64_t c, int64_t ldx, const int64_t* host_spans,
                                    int64_t E, float* H, float alpha, float beta, void* workspace,
                                    size_t workspace_bytes, int32_t* status, void* stream) {
  GQ_REQUIRE(H && host_spans && E > 0, "gq_hessian_spans_bf16: null pointer or E <= 0");
  GQ_REQUIRE(c > 0 && c % 8 == 0 && ldx >= c && ldx % 8 == 0, "gq_hessian_spans_bf16: c, ldx must be multiples of 8");
  GQ_REQUIRE(aligned16(H), "gq_hessian_spans_bf16: H must be 16-byte aligned");
  GQ_REQUIRE(n >= 0 && n < (int64_t(1) << 31), "gq_hessian_spans_bf16: n");
  int64_t rows = 0;
  for (int64_t e = 0; e < E; ++e) {
    const int64_t a = host_spans[2 * e], k = host_spans[2 * e + 1];
    GQ_REQUIRE(a >= 0 && k >= 0 && a + k <= n, "gq_hessian_spans_bf16: span %lld = [%lld, +%lld) outside [0, %lld)",
               (long long)e, (long long)a, (long long)k, (long long)n);
    rows += k;
  }
  const size_t need = gq_hessian_spans_workspace_size(host_spans, E, c);
  GQ_REQUIRE(workspace && workspace_bytes >= need && aligned16(workspace),
             "gq_hessian_spans_bf16: workspace too small (%zu < %zu)", workspace_bytes, need);
  GQ_REQUIRE(rows == 0 || (X && aligned16(X)), "gq_hessian_spans_bf16: X");
  const int64_t tpe = hess::two::tiles(c);
  GQ_REQUIRE(E * tpe < (int64_t(1) << 31), "gq_hessian_spans_bf16: too many experts");
  hess::SpanPlan plan = hess::plan_spans(host_spans, E, tpe);
  const int64_t tails = int64_t(plan.tail_expert.size());
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  __nv_bfloat16* tail_buf = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += spans_tail_bytes(host_spans, E, c);
  int64_t* span = reinterpret_cast<int64_t*>(ws);
  ws += align256(size_t(E) * 16);
  int64_t* tail_off = reinterpret_cast<int64_t*>(ws);
  ws += align256(size_t(E) * 8);
  int32_t* tail_expert = reinterpret_cast<int32_t*>(ws);
  ws += align256(size_t(E) * 8);
  int32_t* sched = reinterpret_cast<int32_t*>(ws);
  GQ_CUDA_TRY(cudaMemcpyAsync(span, host_spans, size_t(E) * 16, cudaMemcpyHostToDevice, s));
  GQ_CUDA_TRY(cudaMemcpyAsync(tail_off, plan.tail_off.data(), size_t(E) * 8, cudaMemcpyHostToDevice, s));
  GQ_CUDA_TRY(cudaMemcpyAsync(sched, plan.sched.data(), plan.sched.size() * 4, cudaMemcpyHostToDevice, s));
  if (tails > 0) {
    GQ_CUDA_TRY(cudaMemcpyAsync(tail_expert, plan.tail_expert.data(), size_t(tails) * 4, cudaMemcpyHostToDevice, s));
    hess::span_tails_kernel<<<unsigned((tails * 64 + 7) / 8), 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(X), c, ldx, span, tail_expert, tails * 64, tail_buf);
    int st = check_launch("span_tails_kernel");
    if (st != GQ_OK) return st;
  }
  // a map needs at least one row: with no rows at all every CTA has KT == 0
  CUtensorMap xmap, tmap;
  int st = hess::make_x_map(&xmap, rows > 0 ? X : workspace, rows > 0 ? n : 1, c, rows > 0 ? ldx : c);
  if (st != GQ_OK) return st;
  st = hess::make_x_map(&tmap, tail_buf, std::max<int64_t>(tails, 1) * 64, c, c);
  if (st != GQ_OK) return st;
  return hess::launch(xmap, 0, c, H, c, alpha, beta, status, sched, nullptr, tpe, int64_t(plan.sched.size()), true,
                      s, 0, &tmap, span, tail_off);
}
