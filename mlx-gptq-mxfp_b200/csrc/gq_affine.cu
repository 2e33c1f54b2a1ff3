// Affine GPTQ (mlx_gptq/gptq.py:183-272) and the full-size damped factor
// U = chol((H + damp*mean(diag H)*I)^-1, upper) (gptq.py:27-66).
//
// Factor. With J the index reversal, if J Hd J = L L^T (lower Cholesky) then
// Hd = V V^T with V = J L J upper and Hd^-1 = U^T U for U = V^-1 = J L^-1 J. So
// the upper Cholesky factor of the inverse is the reversed inverse of the
// Cholesky factor of the reversed matrix: one factorization and one triangular
// inversion (C^3/3 each) instead of factor + cholesky_inverse + factor. Both run
// blocked on 64x64 tiles in float32: the factorization right-looking (diagonal
// block factor + inverse in one CTA, then the panel solve, the next block column's
// update and the rest of the trailing update as tcgen05 GEMMs, the rest on a side
// stream), the inversion by doubling (inverses of 2^k-blocks combined pairwise
// with two GEMMs).
//
// Column loop. One warp per weight row owns one block of bs columns in
// registers (lane l holds columns l, l+32, ...): the clip search at each group
// start, the per-column quantize / error / in-block rank-1 update. Err [B, R, bs]
// goes to the workspace and the trailing update W[:, :, i2:] -= Err * U[i1:i2, i2:]
// is a batched float32 GEMM on the tensor cores (gq_tc_gemm.cu).
#include <map>
#include <mutex>
#include <vector>

#include "gq_affine_grid.cuh"
#include "gq_gemm.cuh"

namespace gq {
namespace aff {

constexpr int NB = 64;  // factorization block

// One non-blocking side stream per device for the factorization's lookahead,
// created on first use and kept for the life of the process.
static cudaError_t side_stream(cudaStream_t* out) {
  static std::mutex mu;
  static std::map<int, cudaStream_t> streams;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto it = streams.find(dev);
  if (it == streams.end()) {
    cudaStream_t st = nullptr;
    e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e != cudaSuccess) return e;
    it = streams.emplace(dev, st).first;
  }
  *out = it->second;
  return cudaSuccess;
}

// ---------------------------------------------------------------------------
// 64x64 float32 tile GEMM building block on the tensor cores (256 threads)
// acc += sum_t A(r, t) * B(t, c) over K, with
//   A(r, t) = TRANS_A ? A[t * lda + r] : A[r * lda + t]
//   B(t, c) = TRANS_B ? B[c * ldb + t] : B[t * ldb + c]
// Rows >= m_lim / columns >= n_lim read as zero. 16-deep chunks of A and B are
// staged k-major in shared memory (stride 72: the fragment loads below are
// bank-conflict free); warp w computes rows 16*(w&3).. and columns 32*(w>>2).. as
// four m16n8k8 fragments, each product in 3xTF32 (x = hi + lo with hi = tf32(x);
// hi*hi + hi*lo + lo*hi), which keeps float32 accuracy.
// ---------------------------------------------------------------------------
constexpr int TS = 72;  // staging row stride (floats)

__device__ __forceinline__ uint32_t tf32_of(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_of(x);
  lo = tf32_of(x - __uint_as_float(hi));
}

__device__ __forceinline__ void mma_tf32_acc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool TRANS_A, bool TRANS_B>
__device__ __forceinline__ void tile_gemm(const float* __restrict__ A, int64_t lda, const float* __restrict__ Bm,
                                          int64_t ldb, int K, int m_lim, int n_lim, float (&acc)[4][4],
                                          float (*As)[TS], float (*Bs)[TS]) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const int mb = 16 * (warp & 3), nb = 32 * (warp >> 2);
  for (int k0 = 0; k0 < K; k0 += 16) {
    // A chunk 64 x 16 into As[t][r]
    if (TRANS_A) {
      const int t = tid >> 4, r4 = (tid & 15) * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int r = r4 + u;
        As[t][r] = (r < m_lim && k0 + t < K) ? A[int64_t(k0 + t) * lda + r] : 0.0f;
      }
    } else {
      const int r = tid >> 2, t4 = (tid & 3) * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = k0 + t4 + u;
        As[t4 + u][r] = (r < m_lim && t < K) ? A[int64_t(r) * lda + t] : 0.0f;
      }
    }
    if (TRANS_B) {
      const int cc = tid >> 2, t4 = (tid & 3) * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = k0 + t4 + u;
        Bs[t4 + u][cc] = (cc < n_lim && t < K) ? Bm[int64_t(cc) * ldb + t] : 0.0f;
      }
    } else {
      const int t = tid >> 4, c4 = (tid & 15) * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int cc = c4 + u;
        Bs[t][cc] = (cc < n_lim && k0 + t < K) ? Bm[int64_t(k0 + t) * ldb + cc] : 0.0f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < 16; ks += 8) {
      uint32_t ahi[4], alo[4];
      split_tf32(As[ks + tq][mb + g], ahi[0], alo[0]);
      split_tf32(As[ks + tq][mb + g + 8], ahi[1], alo[1]);
      split_tf32(As[ks + tq + 4][mb + g], ahi[2], alo[2]);
      split_tf32(As[ks + tq + 4][mb + g + 8], ahi[3], alo[3]);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        uint32_t bh0, bl0, bh1, bl1;
        split_tf32(Bs[ks + tq][nb + 8 * nt + g], bh0, bl0);
        split_tf32(Bs[ks + tq + 4][nb + 8 * nt + g], bh1, bl1);
        mma_tf32_acc(acc[nt], alo, bh0, bh1);
        mma_tf32_acc(acc[nt], ahi, bl0, bl1);
        mma_tf32_acc(acc[nt], ahi, bh0, bh1);
      }
    }
    __syncthreads();
  }
}

// C(r, c) = alpha * acc + beta * C(r, c) for the thread's fragment outputs:
// acc[nt][i] is row 16*(w&3) + g + 8*(i >> 1), column 32*(w>>2) + 8*nt + 2*tq + (i & 1).
__device__ __forceinline__ void tile_store(float* __restrict__ Cm, int64_t ldc, int m_lim, int n_lim,
                                           const float (&acc)[4][4], float alpha, float beta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int mb = 16 * (warp & 3), nb = 32 * (warp >> 2);
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = mb + g + 8 * (i >> 1), cc = nb + 8 * nt + 2 * tq + (i & 1);
      if (r >= m_lim || cc >= n_lim) continue;
      float* p = Cm + int64_t(r) * ldc + cc;
      const float v = alpha * acc[nt][i];
      *p = beta == 0.0f ? v : beta * *p + v;
    }
}

// Batched GEMM C = alpha*A*B + beta*C (GemmBatch, gq_gemm.cuh) on 64x64 tiles.

template <bool TRANS_A, bool TRANS_B>
__global__ void __launch_bounds__(256) gemm_kernel(GemmBatch p) {
  __shared__ __align__(16) float As[16][TS];
  __shared__ __align__(16) float Bs[16][TS];
  const int64_t z = blockIdx.z;
  const int64_t o = z / p.n_inner, in = z % p.n_inner;
  if (p.skip && p.skip[o]) return;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const float* A = p.A + o * p.sa_o + in * p.sa_i + (TRANS_A ? int64_t(m0) : int64_t(m0) * p.lda);
  const float* Bm = p.Bm + o * p.sb_o + in * p.sb_i + (TRANS_B ? int64_t(n0) * p.ldb : int64_t(n0));
  float* Cm = p.Cm + o * p.sc_o + in * p.sc_i + int64_t(m0) * p.ldc + n0;
  float acc[4][4] = {};
  tile_gemm<TRANS_A, TRANS_B>(A, p.lda, Bm, p.ldb, p.K, p.M - m0, p.N - n0, acc, As, Bs);
  tile_store(Cm, p.ldc, p.M - m0, p.N - n0, acc, p.alpha, p.beta);
}

// ---------------------------------------------------------------------------
// 128x128-tile GEMM on the tensor cores for the large products (the trailing
// update W[:, i2:] -= Err U[i1:i2, i2:] and the inverse-doubling GEMMs): 8 warps as
// 2 (M) x 4 (N), each 64 x 32 = 4 x 4 m16n8k8 fragments in 3xTF32; 32-deep K tiles
// double-buffered in shared memory with cp.async (16-byte chunks, zero-filled past
// the matrix edges). Each operand is staged in the orientation its global layout
// copies contiguously, with row strides (36 or 136 floats) that make every
// fragment load bank-conflict free. Used for deep products (K >= 256: the
// inverse doubling) whose copied chunks are all 16-byte aligned (checked on the
// host); the 64x64 tiles above, at several CTAs per SM, serve the rest, the
// K = 128 trailing update among them (measured faster there).
// ---------------------------------------------------------------------------
namespace g128 {
constexpr int BM = 128, BN = 128, BK = 32, THREADS = 256;
constexpr int LDS_ROW = BK + 4;    // [128][36]: rows are M (or N), 32 k each
constexpr int LDS_COL = BM + 8;    // [32][136]: rows are k, 128 M (or N) each
constexpr int A_FLOATS = BM * LDS_ROW > BK * LDS_COL ? BM * LDS_ROW : BK * LDS_COL;
constexpr int STAGE_FLOATS = 2 * A_FLOATS;
constexpr size_t SMEM_BYTES = size_t(2) * STAGE_FLOATS * 4;

__device__ __forceinline__ void cp_async16(float* dst, const float* src, int src_bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(src_bytes));
}

// Stage a (rows x 32) or (32 x rows) block of one operand. ROWMAJOR_K: the global
// layout has k contiguous (element (i, k) at p[i * ld + k]); else i is contiguous.
template <bool K_CONTIG>
__device__ __forceinline__ void stage(float* sm, const float* p, int64_t ld, int lim_i, int k0, int K) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int ch = tid + u * THREADS;  // 1024 chunks of 4 floats
    if (K_CONTIG) {
      const int i = ch >> 3, kc = (ch & 7) * 4, k = k0 + kc;
      int bytes = 0;
      if (i < lim_i && k < K) bytes = (K - k >= 4 ? 4 : K - k) * 4;
      cp_async16(sm + i * LDS_ROW + kc, bytes ? p + int64_t(i) * ld + k : p, bytes);
    } else {
      const int kr = ch >> 5, ic = (ch & 31) * 4, k = k0 + kr;
      int bytes = 0;
      if (k < K && ic < lim_i) bytes = (lim_i - ic >= 4 ? 4 : lim_i - ic) * 4;
      cp_async16(sm + kr * LDS_COL + ic, bytes ? p + int64_t(k) * ld + ic : p, bytes);
    }
  }
}

template <bool TRANS_A, bool TRANS_B>
__global__ void __launch_bounds__(THREADS) gemm128_kernel(GemmBatch p) {
  extern __shared__ __align__(16) float smem[];
  const int64_t z = blockIdx.z;
  const int64_t o = z / p.n_inner, in = z % p.n_inner;
  if (p.skip && p.skip[o]) return;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  // A(r, k): TRANS_A ? A[k * lda + r] : A[r * lda + k];  B(k, c): TRANS_B ? B[c * ldb + k] : B[k * ldb + c]
  const float* A = p.A + o * p.sa_o + in * p.sa_i + (TRANS_A ? int64_t(m0) : int64_t(m0) * p.lda);
  const float* Bm = p.Bm + o * p.sb_o + in * p.sb_i + (TRANS_B ? int64_t(n0) * p.ldb : int64_t(n0));
  const int lim_m = p.M - m0, lim_n = p.N - n0, K = p.K;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const int wm = 64 * (warp & 1), wn = 32 * (warp >> 1);
  float acc[4][4][4] = {};
  const int KT = (K + BK - 1) / BK;
  auto issue = [&](int kt) {
    float* st = smem + (kt & 1) * STAGE_FLOATS;
    stage<!TRANS_A>(st, A, p.lda, lim_m, kt * BK, K);
    stage<TRANS_B>(st + A_FLOATS, Bm, p.ldb, lim_n, kt * BK, K);
    asm volatile("cp.async.commit_group;\n" ::);
  };
  issue(0);
  for (int kt = 0; kt < KT; ++kt) {
    if (kt + 1 < KT) {
      issue(kt + 1);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();
    const float* As = smem + (kt & 1) * STAGE_FLOATS;
    const float* Bs = As + A_FLOATS;
#pragma unroll
    for (int kk = 0; kk < BK; kk += 8) {
      uint32_t bh[4][2], bl[4][2];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = wn + 8 * j + g;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int k = kk + tq + 4 * h;
          const float v = TRANS_B ? Bs[c * LDS_ROW + k] : Bs[k * LDS_COL + c];
          split_tf32(v, bh[j][h], bl[j][h]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t ah[4], al[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int r = wm + 16 * i + g + 8 * (q & 1), k = kk + tq + 4 * (q >> 1);
          const float v = TRANS_A ? As[k * LDS_COL + r] : As[r * LDS_ROW + k];
          split_tf32(v, ah[q], al[q]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          mma_tf32_acc(acc[i][j], al, bh[j][0], bh[j][1]);
          mma_tf32_acc(acc[i][j], ah, bl[j][0], bl[j][1]);
          mma_tf32_acc(acc[i][j], ah, bh[j][0], bh[j][1]);
        }
      }
    }
    __syncthreads();  // this stage is refilled by the next iteration's issue
  }
  float* Cm = p.Cm + o * p.sc_o + in * p.sc_i + int64_t(m0) * p.ldc + n0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = wm + 16 * i + g + 8 * (q >> 1), c = wn + 8 * j + 2 * tq + (q & 1);
        if (r >= lim_m || c >= lim_n) continue;
        float* ptr = Cm + int64_t(r) * p.ldc + c;
        const float v = p.alpha * acc[i][j][q];
        *ptr = p.beta == 0.0f ? v : p.beta * *ptr + v;
      }
}

// Every cp.async source must be 16-byte aligned: bases, leading dimensions and
// batch strides in whole 4-float units.
static bool usable(const GemmBatch& p) {
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  return al(p.A) && al(p.Bm) && p.lda % 4 == 0 && p.ldb % 4 == 0 && p.sa_o % 4 == 0 && p.sa_i % 4 == 0 &&
         p.sb_o % 4 == 0 && p.sb_i % 4 == 0 && (p.M >= BM || p.N >= BN) && p.K >= 8 * BK;
}

template <bool TA, bool TB>
static int launch(const GemmBatch& p, int64_t batches, cudaStream_t s) {
  GQ_CUDA_TRY(cudaFuncSetAttribute(gemm128_kernel<TA, TB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(SMEM_BYTES)));
  const dim3 grid(unsigned((p.N + BN - 1) / BN), unsigned((p.M + BM - 1) / BM), unsigned(batches));
  gemm128_kernel<TA, TB><<<grid, THREADS, SMEM_BYTES, s>>>(p);
  return check_launch("gemm128_kernel");
}
}  // namespace g128

static int launch_gemm(const GemmBatch& p, bool trans_a, bool trans_b, int64_t batches, cudaStream_t s) {
  if (batches <= 0 || p.M <= 0 || p.N <= 0) return GQ_OK;
  if (g128::usable(p)) {
    if (trans_a && trans_b) return g128::launch<true, true>(p, batches, s);
    if (trans_a) return g128::launch<true, false>(p, batches, s);
    if (trans_b) return g128::launch<false, true>(p, batches, s);
    return g128::launch<false, false>(p, batches, s);
  }
  const dim3 grid(unsigned((p.N + 63) / 64), unsigned((p.M + 63) / 64), unsigned(batches));
  if (trans_a && trans_b)
    gemm_kernel<true, true><<<grid, 256, 0, s>>>(p);
  else if (trans_a)
    gemm_kernel<true, false><<<grid, 256, 0, s>>>(p);
  else if (trans_b)
    gemm_kernel<false, true><<<grid, 256, 0, s>>>(p);
  else
    gemm_kernel<false, false><<<grid, 256, 0, s>>>(p);
  return check_launch("gemm_kernel");
}

// Products whose tiles fill the 128 x 128 tensor-core tile go to tc_gemm (TMA-fed
// tcgen05, gq_tc_gemm.cu); smaller ones and layouts a tensor map cannot describe to
// the mma.sync kernels above.
static int gemm(const GemmBatch& p, bool trans_a, bool trans_b, int64_t batches, int32_t* status, cudaStream_t s) {
  if (p.M >= 128 && p.N >= 128 && tc_gemm_usable(p, trans_a, trans_b))
    return tc_gemm(p, trans_a, trans_b, batches, status, s);
  return launch_gemm(p, trans_a, trans_b, batches, s);
}

// ---------------------------------------------------------------------------
// factorization kernels (blockIdx.y = batch item; items with skip[b] != 0 idle)
// ---------------------------------------------------------------------------
struct FactorState {
  float* diag_mean;  // [B]
  float* cur_damp;   // [B]
  int32_t* info;     // [B] 0 = ok, else failing column + 1
  int32_t* skip;     // [B] 1 = do not (re)factor this item
};

__global__ void diag_mean_kernel(const float* __restrict__ H, int64_t C, float damp, FactorState st) {
  const int64_t b = blockIdx.x;
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < C; i += blockDim.x) s += H[(b * C + i) * C + i];
  __shared__ float red[256];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int k = blockDim.x / 2; k > 0; k >>= 1) {
    if (threadIdx.x < k) red[threadIdx.x] += red[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    st.diag_mean[b] = fmaxf(red[0] / float(C), 1e-8f);
    st.cur_damp[b] = damp;
    st.info[b] = 0;
    st.skip[b] = 0;
  }
}

// Hr[b] = J (H[b] + lam_b I) J, lower triangle (incl. diagonal), lam_b = diag_mean * cur_damp.
__global__ void build_reversed_kernel(const float* __restrict__ H, int64_t C, float* __restrict__ Hr, FactorState st) {
  const int64_t b = blockIdx.y;
  if (st.skip[b]) return;
  const float lam = st.diag_mean[b] * st.cur_damp[b];
  const int64_t n = C * C;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < n; idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = idx / C, j = idx % C;
    if (j > i) continue;
    float v = H[(b * C + (C - 1 - i)) * C + (C - 1 - j)];
    if (i == j) v = v + lam;
    Hr[(b * C + i) * C + j] = v;
  }
}

// 1 / sqrt(piv) for a positive pivot: the hardware reciprocal square root, or the
// correctly rounded quotient for pivots below the smallest normal float.
__device__ __forceinline__ float inv_sqrt_pivot(float piv) {
  return piv >= 1.17549435e-38f ? rsqrtf(piv) : 1.0f / sqrtf(piv);
}

// One warp, 32 x 32 blocks held in registers, lane i owning row i (a[0..31]).
// Cholesky, right-looking: the pivot and column k come from lane k / lane j by
// shuffles; every update of a step is independent. Each step multiplies by
// 1/sqrt(pivot) instead of dividing. Returns 0, or the failing column + 1 (a
// non-positive pivot); a[] then holds L (lower; upper part garbage) and inv_diag
// this lane's 1 / L[lane][lane].
__device__ __forceinline__ int warp_potrf32_reg(float (&a)[32], float& inv_diag, int lane) {
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const float piv = __shfl_sync(0xFFFFFFFFu, a[k], k);
    if (!(piv > 0.0f)) return k + 1;  // uniform across the warp
    const float r = inv_sqrt_pivot(piv);
    if (lane == k) inv_diag = r;
    const float lik = lane == k ? piv * r : a[k] * r;
    a[k] = lane >= k ? lik : a[k];
#pragma unroll
    for (int j = k + 1; j < 32; ++j) {
      const float ljk = __shfl_sync(0xFFFFFFFFu, lik, j);
      a[j] = fmaf(-lik, ljk, a[j]);
    }
  }
  return 0;
}

// Column `lane` of X = L^-1 for a 32x32 lower L in shared memory: L x = e_lane,
// forward substitution with the diagonal reciprocals inv_d[t].
__device__ __forceinline__ void col_trinv32(float (&x)[32], const float* L, int ld, const float* inv_d, int lane) {
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = i == lane ? 1.0f : 0.0f;
#pragma unroll
  for (int t = 0; t < 32; ++t) {
    x[t] = x[t] * inv_d[t];
#pragma unroll
    for (int i = t + 1; i < 32; ++i) x[i] = fmaf(-L[i * ld + t], x[t], x[i]);
  }
}

// 32 x 32 x 32 shared-memory product for 128 threads, each a 4 x 2 block of outputs
// (rows i0..i0+3, columns j0, j0+1) with eight independent accumulators:
// acc[a][c] = sum_t P[(i0+a)*pld + t] * Q(t, j0+c), Q(t, j) = QT ? Q[j*qld + t] : Q[t*qld + j].
template <bool QT>
__device__ __forceinline__ void mm32_4x2(const float* P, int pld, const float* Q, int qld, int i0, int j0,
                                         float (&acc)[4][2]) {
#pragma unroll
  for (int a = 0; a < 4; ++a) acc[a][0] = acc[a][1] = 0.0f;
#pragma unroll
  for (int t = 0; t < 32; ++t) {
    const float q0 = QT ? Q[j0 * qld + t] : Q[t * qld + j0];
    const float q1 = QT ? Q[(j0 + 1) * qld + t] : Q[t * qld + j0 + 1];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float pv = P[(i0 + a) * pld + t];
      acc[a][0] = fmaf(pv, q0, acc[a][0]);
      acc[a][1] = fmaf(pv, q1, acc[a][1]);
    }
  }
}

// Factor the 64x64 diagonal block k of Hr[b] (lower) and store its inverse (lower,
// zeros above) in Dinv[b][k]; records the failing column. As a 2 x 2 block of 32 x 32
// pieces: for each half h (one copy of the code, so the unrolled register loops fit
// the instruction cache), warp 0 factors the diagonal piece in registers
// (L_hh = chol(A_hh)) and inverts it (X_hh = L_hh^-1); after the first half all four
// warps form L21 = A21 X11^T and A22 -= L21 L21^T in shared memory; at the end
// X21 = -X22 (L21 X11). The block is read with every load in flight at once; the
// chain runs on fused multiply-adds and reciprocal square roots.
__global__ void __launch_bounds__(128) potrf_diag_kernel(float* __restrict__ Hr, int64_t C, int k,
                                                         float* __restrict__ Dinv, FactorState st) {
  constexpr int LD = NB + 1;
  __shared__ float S[NB * LD];   // the block, then L (lower)
  __shared__ float X[NB * LD];   // L^-1 (lower)
  __shared__ float T[32 * 33];   // A21 / L21 X11 scratch
  __shared__ float inv_d[NB];    // 1 / L[i][i]
  __shared__ int fail_s;
  const int64_t b = blockIdx.x;
  if (st.skip[b] || st.info[b]) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i0 = (tid >> 4) * 4, j0 = (tid & 15) * 2;  // this thread's 4 x 2 block of 32 x 32 products
  float* blk = Hr + (b * C + int64_t(k) * NB) * C + int64_t(k) * NB;
  {
    float v[NB * NB / 128];
#pragma unroll
    for (int r = 0; r < NB * NB / 128; ++r) {
      const int i = tid + 128 * r;
      v[r] = blk[int64_t(i >> 6) * C + (i & 63)];
    }
#pragma unroll
    for (int r = 0; r < NB * NB / 128; ++r) {
      const int i = tid + 128 * r;
      S[(i >> 6) * LD + (i & 63)] = v[r];
    }
  }
  if (tid == 0) fail_s = 0;
  __syncthreads();
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    const int o = 32 * h;
    if (warp == 0) {
      float a[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) a[j] = S[(o + lane) * LD + o + j];
      float inv = 0.0f;
      const int f = warp_potrf32_reg(a, inv, lane);
      if (f) {
        if (lane == 0) fail_s = o + f;
      } else {
        inv_d[o + lane] = inv;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j <= lane) S[(o + lane) * LD + o + j] = a[j];
        __syncwarp();
        col_trinv32(a, S + o * LD + o, LD, inv_d + o, lane);
#pragma unroll
        for (int i = 0; i < 32; ++i) X[(o + i) * LD + o + lane] = a[i];
      }
    }
    __syncthreads();
    if (fail_s) {
      if (tid == 0) st.info[b] = k * NB + fail_s;
      return;
    }
    if (h == 0) {
      for (int e = tid; e < 32 * 32; e += 128) T[(e >> 5) * 33 + (e & 31)] = S[(32 + (e >> 5)) * LD + (e & 31)];
      __syncthreads();
      float acc[4][2];
      // L21 = A21 X11^T (X11 is lower with exact zeros above, so the full sum is exact)
      mm32_4x2<true>(T, 33, X, LD, i0, j0, acc);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        S[(32 + i0 + a) * LD + j0] = acc[a][0];
        S[(32 + i0 + a) * LD + j0 + 1] = acc[a][1];
      }
      __syncthreads();
      // A22 -= L21 L21^T (lower)
      mm32_4x2<true>(S + 32 * LD, LD, S + 32 * LD, LD, i0, j0, acc);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          if (j0 + c <= i0 + a) S[(32 + i0 + a) * LD + 32 + j0 + c] -= acc[a][c];
      __syncthreads();
    }
  }
#pragma unroll 4
  for (int i = tid; i < NB * NB; i += 128) {  // write L back (lower)
    const int r = i >> 6, c = i & 63;
    if (c <= r) blk[int64_t(r) * C + c] = S[r * LD + c];
  }
  {
    float acc[4][2];
    mm32_4x2<false>(S + 32 * LD, LD, X, LD, i0, j0, acc);  // T = L21 X11
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      T[(i0 + a) * 33 + j0] = acc[a][0];
      T[(i0 + a) * 33 + j0 + 1] = acc[a][1];
    }
    __syncthreads();
    mm32_4x2<false>(X + 32 * LD + 32, LD, T, 33, i0, j0, acc);  // X21 = -X22 T
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      X[(32 + i0 + a) * LD + j0] = -acc[a][0];
      X[(32 + i0 + a) * LD + j0 + 1] = -acc[a][1];
    }
  }
  __syncthreads();
  float* D = Dinv + (b * (C / NB) + k) * NB * NB;
#pragma unroll 4
  for (int i = tid; i < NB * NB; i += 128) {
    const int r = i >> 6, c = i & 63;
    D[i] = c <= r ? X[r * LD + c] : 0.0f;
  }
}

// Linv initialisation: diagonal blocks = Dinv, everything else zero.
__global__ void init_linv_kernel(float* __restrict__ Li, int64_t C, const float* __restrict__ Dinv, FactorState st) {
  const int64_t b = blockIdx.y;
  if (st.info[b]) return;
  const int64_t n = C * C;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < n; idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = idx / C, j = idx % C;
    float v = 0.0f;
    if (i / NB == j / NB) v = Dinv[((b * (C / NB) + i / NB) * NB + (i % NB)) * NB + (j % NB)];
    Li[b * n + idx] = v;
  }
}

// In-place 180-degree rotation: U[i][j] <- Li[C-1-i][C-1-j] (Li lower -> U upper).
__global__ void rotate_kernel(float* __restrict__ M, int64_t C, FactorState st) {
  const int64_t b = blockIdx.y;
  if (st.info[b]) return;
  const int64_t n = C * C, half = n / 2;
  float* m = M + b * n;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < half; idx += int64_t(gridDim.x) * blockDim.x) {
    const float a = m[idx], c = m[n - 1 - idx];
    m[idx] = c;
    m[n - 1 - idx] = a;
  }
}

__global__ void escalate_kernel(int64_t B, FactorState st) {
  const int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (st.info[b]) {
    st.cur_damp[b] = st.cur_damp[b] * 10.0f;
    st.info[b] = 0;
    st.skip[b] = 0;
  } else {
    st.skip[b] = 1;
  }
}

// ---------------------------------------------------------------------------
// affine column loop: a segment of LPR lanes per (row, item), 32 / LPR rows per
// warp; block columns [i1, i1 + 16*LPR), lane `sl` of a segment holding columns
// sl, sl + LPR, ... (16 slots). The per-column scalar work (quantize, error) is
// done by the LPR lanes of the row's segment, not by a whole warp.
// ---------------------------------------------------------------------------
template <int W>
__device__ __forceinline__ float seg_sum(float x) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, o);
  return x;
}
template <int W>
__device__ __forceinline__ float seg_min(float x) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) x = fminf(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
  return x;
}
template <int W>
__device__ __forceinline__ float seg_max(float x) {
#pragma unroll
  for (int o = W / 2; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
  return x;
}

// choose_qparams (grid.py:167-212) over one segment-held group of GS * LPR values:
// every lane of the segment returns the same storage-rounded (s, b); candidate
// errors are butterfly-reduced inside the segment (bit-identical on its lanes) and
// the first minimum wins (strict <), as in the reference. Candidates are evaluated
// three at a time so their reductions overlap.
template <int GS, int LPR>
__device__ __forceinline__ void seg_choose_qparams(const float (&v)[GS], float maxq, const float* pr, const float* pf,
                                                   int nshrink, int storage, float& s_best, float& b_best) {
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int k = 1; k < GS; ++k) {
    mn = fminf(mn, v[k]);
    mx = fmaxf(mx, v[k]);
  }
  mn = seg_min<LPR>(mn);
  mx = seg_max<LPR>(mx);
  const float rng = mx - mn;
  float best = 0.0f;
  constexpr int U = 3;
  for (int i0 = 0; i0 < nshrink; i0 += U) {
    float sc[U], bc[U], err[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u < nshrink ? i0 + u : i0;
      sc[u] = round_storage(rng * pr[i], storage);
      bc[u] = round_storage(mn * pf[i], storage);
      err[u] = 0.0f;
#pragma unroll
      for (int k = 0; k < GS; ++k) {
        float q;
        const float d = affine_quant(v[k], sc[u], bc[u], maxq, q) - v[k];
        err[u] = fmaf(d, d, err[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) err[u] = seg_sum<LPR>(err[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (i0 + u < nshrink && (i0 + u == 0 || err[u] < best)) {
        best = err[u];
        s_best = sc[u];
        b_best = bc[u];
      }
    }
  }
}

template <int LPR, int GS>
__global__ void __launch_bounds__(128) affine_rows_kernel(float* __restrict__ W, const float* __restrict__ U,
                                                          int64_t R, int64_t C, int64_t i1, int nslots, int bits,
                                                          int nshrink, int storage, uint8_t* __restrict__ q,
                                                          void* __restrict__ scales, void* __restrict__ biases,
                                                          float* __restrict__ Err) {
  constexpr int SL = 16, BS = SL * LPR, RPW = 32 / LPR, G = GS * LPR;
  constexpr bool kSmemU = BS <= 128;  // 128 x 128 U block (64 KB) staged in shared memory
  __shared__ float pr[kMaxShrinks], pf[kMaxShrinks];
  extern __shared__ __align__(16) float Us[];  // [BS][BS] when kSmemU
  const int lane = threadIdx.x & 31, sl = lane % LPR;
  const int64_t b = blockIdx.y;
  const float* Ug = U + b * C * C + i1 * C + i1;  // U1 = U[i1:i2, i1:i2], row stride C
  if (threadIdx.x < kMaxShrinks) shrink_factors(threadIdx.x, bits, pr[threadIdx.x], pf[threadIdx.x]);
  if (kSmemU) {  // 16-byte loads, eight in flight per thread (rows of U are 16-byte aligned: C % 32 == 0)
    const int n = nslots * LPR, nv = n / 4, total = n * nv;
    for (int i0 = threadIdx.x; i0 < total; i0 += 8 * blockDim.x) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < total) v[u] = __ldg(reinterpret_cast<const float4*>(Ug + int64_t(i / nv) * C) + (i % nv));
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < total) reinterpret_cast<float4*>(Us + (i / nv) * BS)[i % nv] = v[u];
      }
    }
  }
  __syncthreads();
  const int64_t r = (int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + lane / LPR;
  const bool row_ok = r < R;  // rows past R still take part in the segment shuffles
  const int64_t ng = C / G;
  float* wrow = W + (b * R + (row_ok ? r : 0)) * C + i1;
  // nslots = columns in this block / LPR (< SL only for the last, partial block)
  float w[SL], dqv[SL], ev[SL], qv[SL];
#pragma unroll
  for (int k = 0; k < SL; ++k) w[k] = row_ok && k < nslots ? wrow[sl + LPR * k] : 0.0f;
  const float maxq = float((1 << bits) - 1);
  float s = 0.0f, bb = 0.0f;
#pragma unroll
  for (int k = 0; k < SL; ++k) {  // slot k = columns LPR*k .. LPR*k + LPR-1 of the block
    if (k >= nslots) break;
    if (k % GS == 0) {  // group start (gptq.py:250-256)
      float v[GS];
#pragma unroll
      for (int t = 0; t < GS; ++t) v[t] = w[k + t];
      seg_choose_qparams<GS, LPR>(v, maxq, pr, pf, nshrink, storage, s, bb);
      if (sl == 0 && row_ok) {
        const int64_t g = (i1 + LPR * k) / G;
        store_any(scales, (b * R + r) * ng + g, s, storage);
        store_any(biases, (b * R + r) * ng + g, bb, storage);
      }
    }
#pragma unroll 1
    for (int l = 0; l < LPR; ++l) {
      const int j = LPR * k + l;
      const float wj = __shfl_sync(0xFFFFFFFFu, w[k], l, LPR);
      float qj;
      const float dq = affine_quant(wj, s, bb, maxq, qj);
      const float* urow = kSmemU ? Us + j * BS : Ug + int64_t(j) * C;
      const float e = (wj - dq) / urow[j];
      if (sl == l) {
        dqv[k] = dq;
        ev[k] = e;
        qv[k] = qj;
      }
#pragma unroll
      for (int kk = k; kk < SL; ++kk) {
        const int col = LPR * kk + sl;
        if (kk < nslots && col > j) w[kk] = w[kk] - e * urow[col];
      }
    }
  }
  if (!row_ok) return;
  uint8_t* qrow = q + (b * R + r) * C + i1;
  float* erow = Err + (b * R + r) * BS;
#pragma unroll
  for (int k = 0; k < SL; ++k) {
    if (k >= nslots) break;
    wrow[sl + LPR * k] = dqv[k];
    qrow[sl + LPR * k] = uint8_t(qv[k]);
    erow[sl + LPR * k] = ev[k];
  }
}

// rel_err partial sums over rows: partials[b][row-block] = (sum (dq-w)^2, sum w^2)
template <typename Tin>
__global__ void rel_partials_kernel(const float* __restrict__ Wdq, const Tin* __restrict__ W0, int64_t RC,
                                    float* __restrict__ partials) {
  const int64_t b = blockIdx.y;
  float n = 0.0f, d = 0.0f;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < RC; i += int64_t(gridDim.x) * blockDim.x) {
    const float w = to_f32<Tin>(W0[b * RC + i]);
    const float e = Wdq[b * RC + i] - w;
    n = fmaf(e, e, n);
    d = fmaf(w, w, d);
  }
  n = warp_sum(n);
  d = warp_sum(d);
  __shared__ float rn[8], rd[8];
  if ((threadIdx.x & 31) == 0) {
    rn[threadIdx.x >> 5] = n;
    rd[threadIdx.x >> 5] = d;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sn = 0.0f, sd = 0.0f;
    for (int w = 0; w < 8; ++w) sn += rn[w], sd += rd[w];
    partials[(b * gridDim.x + blockIdx.x) * 2] = sn;
    partials[(b * gridDim.x + blockIdx.x) * 2 + 1] = sd;
  }
}

}  // namespace aff

int launch_rel_err(const float* partials, int64_t B, int64_t per_b, float* rel, cudaStream_t s);

}  // namespace gq

using namespace gq;
using namespace gq::aff;

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

extern "C" size_t gq_prepare_hinv_workspace_size(int64_t B, int64_t C) {
  if (B <= 0 || C <= 0) return 0;
  return align256(size_t(B) * C * C * 4) + align256(size_t(B) * C * NB * 4) + 4 * align256(size_t(B) * 4);
}

extern "C" int gq_prepare_hinv(const float* H, int64_t B, int64_t C, float damp, float* U, int32_t* info,
                               float* damp_used, void* workspace, size_t workspace_bytes, int32_t* status,
                               void* stream) {
  GQ_REQUIRE(H && U && info, "gq_prepare_hinv: null pointer");
  GQ_REQUIRE(B > 0 && C > 0 && C % NB == 0, "gq_prepare_hinv: C=%lld must be a positive multiple of %d",
             (long long)C, NB);
  GQ_REQUIRE(B < 65536, "gq_prepare_hinv: batch too large");
  const size_t need = gq_prepare_hinv_workspace_size(B, C);
  GQ_REQUIRE(workspace && workspace_bytes >= need, "gq_prepare_hinv: workspace too small (%zu < %zu)",
             workspace_bytes, need);
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  float* Hr = reinterpret_cast<float*>(ws);
  ws += align256(size_t(B) * C * C * 4);
  float* Dinv = reinterpret_cast<float*>(ws);
  ws += align256(size_t(B) * C * NB * 4);
  FactorState st;
  st.diag_mean = reinterpret_cast<float*>(ws);
  ws += align256(size_t(B) * 4);
  st.cur_damp = reinterpret_cast<float*>(ws);
  ws += align256(size_t(B) * 4);
  st.info = reinterpret_cast<int32_t*>(ws);
  ws += align256(size_t(B) * 4);
  st.skip = reinterpret_cast<int32_t*>(ws);

  const int nb = int(C / NB);
  const unsigned ew_blocks = unsigned(std::min<int64_t>((C * C + 255) / 256, 4096));
  diag_mean_kernel<<<unsigned(B), 256, 0, s>>>(H, C, damp, st);
  std::vector<int32_t> hinfo(B);
  bool ok = false;
  // Lookahead: the trailing update of step k is split; its next block column runs on
  // the caller's stream (the next diagonal factor and panel solve need it), the rest
  // on a side stream beside them. Events order the two: the rest of step k starts
  // after the panel solve and next-column update of step k, and the next-column
  // update of step k + 1 (which writes tiles the rest of step k also writes) waits
  // for it. No tile is written by both streams at once.
  cudaStream_t side = nullptr;
  cudaEvent_t ev_main = nullptr, ev_side = nullptr;
  GQ_CUDA_TRY(side_stream(&side));
  GQ_CUDA_TRY(cudaEventCreateWithFlags(&ev_main, cudaEventDisableTiming));
  GQ_CUDA_TRY(cudaEventCreateWithFlags(&ev_side, cudaEventDisableTiming));
  struct EventGuard {
    cudaEvent_t a, b;
    ~EventGuard() {
      cudaEventDestroy(a);
      cudaEventDestroy(b);
    }
  } guard{ev_main, ev_side};
  for (int attempt = 0; attempt < 6; ++attempt) {
    build_reversed_kernel<<<dim3(ew_blocks, unsigned(B)), 256, 0, s>>>(H, C, Hr, st);
    bool side_pending = false;
    for (int k = 0; k < nb; ++k) {
      potrf_diag_kernel<<<unsigned(B), 128, 0, s>>>(Hr, C, k, Dinv, st);
      const int m = nb - k - 1;
      if (m > 0) {
        // panel: L[i][k] = A[i][k] * Dinv_k^T for block rows i > k, in place
        GemmBatch g{};
        g.A = Hr + int64_t(k + 1) * NB * C + int64_t(k) * NB;
        g.lda = C;
        g.Bm = Dinv + int64_t(k) * NB * NB;
        g.ldb = NB;
        g.Cm = Hr + int64_t(k + 1) * NB * C + int64_t(k) * NB;
        g.ldc = C;
        g.sa_o = g.sc_o = C * C;
        g.sb_o = C * NB;
        g.n_inner = 1;
        g.M = m * NB;
        g.N = NB;
        g.K = NB;
        g.alpha = 1.0f;
        g.beta = 0.0f;
        g.skip = st.skip;
        int r = tc_gemm(g, false, true, B, status, s);
        if (r != GQ_OK) return r;
        if (side_pending) GQ_CUDA_TRY(cudaStreamWaitEvent(s, ev_side, 0));
        // next block column: A[i][k+1] -= L[i][k] L[k+1][k]^T, i > k
        GemmBatch u = g;
        u.Bm = g.A;
        u.ldb = C;
        u.sb_o = C * C;
        u.Cm = Hr + int64_t(k + 1) * NB * C + int64_t(k + 1) * NB;
        u.alpha = -1.0f;
        u.beta = 1.0f;
        r = tc_gemm(u, false, true, B, status, s);
        if (r != GQ_OK) return r;
        side_pending = false;
        if (m > 1) {
          // the rest, beside the next steps: A[i][j] -= L[i][k] L[j][k]^T, k + 2 <= j <= i
          GQ_CUDA_TRY(cudaEventRecord(ev_main, s));
          GQ_CUDA_TRY(cudaStreamWaitEvent(side, ev_main, 0));
          GemmBatch w = u;
          w.A = Hr + int64_t(k + 2) * NB * C + int64_t(k) * NB;
          w.Bm = w.A;
          w.Cm = Hr + int64_t(k + 2) * NB * C + int64_t(k + 2) * NB;
          w.M = w.N = (m - 1) * NB;
          r = tc_gemm(w, false, true, B, status, side, true);
          if (r != GQ_OK) return r;
          GQ_CUDA_TRY(cudaEventRecord(ev_side, side));
          side_pending = true;
        }
      }
    }
    if (side_pending) GQ_CUDA_TRY(cudaStreamWaitEvent(s, ev_side, 0));
    int stl = check_launch("cholesky kernels");
    if (stl != GQ_OK) return stl;
    GQ_CUDA_TRY(cudaMemcpyAsync(hinfo.data(), st.info, size_t(B) * 4, cudaMemcpyDeviceToHost, s));
    GQ_CUDA_TRY(cudaStreamSynchronize(s));
    bool any_fail = false;
    for (int64_t b = 0; b < B; ++b) any_fail |= hinfo[b] != 0;
    if (!any_fail) {
      ok = true;
      break;
    }
    if (attempt < 5) escalate_kernel<<<unsigned((B + 255) / 256), 256, 0, s>>>(B, st);
  }
  if (damp_used) GQ_CUDA_TRY(cudaMemcpyAsync(damp_used, st.cur_damp, size_t(B) * 4, cudaMemcpyDeviceToDevice, s));
  GQ_CUDA_TRY(cudaMemcpyAsync(info, st.info, size_t(B) * 4, cudaMemcpyDeviceToDevice, s));
  if (!ok) {
    GQ_CUDA_TRY(cudaStreamSynchronize(s));
    set_last_error("Hessian not positive definite after damping escalation");
    return GQ_ERR_NOT_PD;
  }
  // L^-1 by doubling. At level sz every diagonal block of size sz starting at a
  // multiple of sz is already inverted (in U); a pair [A 0; Bk D] gets the
  // off-diagonal block -D^-1 * Bk * A^-1 of its inverse. X = Bk * A^-1 is kept
  // transposed (sz x dsz) in the unused strict upper triangle of Hr (rows c0..,
  // columns r0..), so a trailing partial pair (dsz < sz) stays inside the matrix.
  init_linv_kernel<<<dim3(ew_blocks, unsigned(B)), 256, 0, s>>>(U, C, Dinv, st);
  for (int64_t sz = NB; sz < C; sz *= 2) {
    const int64_t full = C / (2 * sz);
    const bool partial = (C % (2 * sz)) > sz;
    for (int part = 0; part < 2; ++part) {
      const int64_t npairs = part == 0 ? full : (partial ? 1 : 0);
      if (npairs == 0) continue;
      const int64_t c0 = part == 0 ? 0 : full * 2 * sz, r0 = c0 + sz;
      const int64_t dsz = part == 0 ? sz : C - r0;
      const int64_t pstride = 2 * sz * (C + 1);  // next pair down the diagonal
      GemmBatch g1{};  // Xt(r, c) = sum_t Ainv[t][r] * Bk[c][t]   (Xt = (Bk Ainv)^T)
      g1.A = U + c0 * C + c0;
      g1.lda = C;
      g1.Bm = Hr + r0 * C + c0;
      g1.ldb = C;
      g1.Cm = Hr + c0 * C + r0;
      g1.ldc = C;
      g1.sa_o = g1.sb_o = g1.sc_o = C * C;
      g1.sa_i = g1.sb_i = g1.sc_i = pstride;
      g1.n_inner = int(npairs);
      g1.M = int(sz);
      g1.N = int(dsz);
      g1.K = int(sz);
      g1.alpha = 1.0f;
      g1.beta = 0.0f;
      g1.skip = st.info;
      int r = gemm(g1, true, true, B * npairs, status, s);
      if (r != GQ_OK) return r;
      GemmBatch g2 = g1;  // Linv(r0.., c0..) = -Dinv * X, X(t, c) = Xt[c][t]
      g2.A = U + r0 * C + r0;
      g2.Bm = Hr + c0 * C + r0;
      g2.Cm = U + r0 * C + c0;
      g2.M = int(dsz);
      g2.N = int(sz);
      g2.K = int(dsz);
      g2.alpha = -1.0f;
      r = gemm(g2, false, true, B * npairs, status, s);
      if (r != GQ_OK) return r;
    }
  }
  rotate_kernel<<<dim3(ew_blocks, unsigned(B)), 256, 0, s>>>(U, C, st);
  return check_launch("prepare_hinv tail");
}

extern "C" size_t gq_gptq_affine_workspace_size(int64_t B, int64_t R, int64_t C, int group_size, int block_size) {
  if (B <= 0 || R <= 0 || C <= 0 || group_size <= 0) return 0;
  int64_t bs = std::max<int64_t>(block_size, group_size);
  bs -= bs % group_size;
  return align256(size_t(B) * R * bs * 4) + align256(size_t(B) * 1024 * 2 * 4);
}

extern "C" int gq_gptq_affine(float* W, const void* W_orig, int w_dtype, const float* U, int64_t B, int64_t R,
                              int64_t C, int bits, int group_size, int block_size, int clip, int storage_dtype,
                              uint8_t* q, void* scales, void* biases, float* rel_err, void* workspace,
                              size_t workspace_bytes, int32_t* status, void* stream) {
  GQ_REQUIRE(W && U && q && scales && biases, "gq_gptq_affine: null pointer");
  GQ_REQUIRE(bits >= 1 && bits <= 8, "gq_gptq_affine: bits %d", bits);
  GQ_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128 || group_size == 256,
             "gq_gptq_affine: group size %d unsupported (32/64/128/256)", group_size);
  GQ_REQUIRE(C % group_size == 0, "in_features %lld not divisible by group %d", (long long)C, group_size);
  GQ_REQUIRE(clip == GQ_CLIP_MSE || clip == GQ_CLIP_MINMAX, "gq_gptq_affine: clip");
  GQ_REQUIRE(storage_dtype == GQ_F32 || storage_dtype == GQ_BF16 || storage_dtype == GQ_F16, "storage dtype");
  GQ_REQUIRE(B > 0 && R >= 0 && B < 65536, "gq_gptq_affine: sizes");
  GQ_REQUIRE(!rel_err || (W_orig && (w_dtype == GQ_F32 || w_dtype == GQ_BF16 || w_dtype == GQ_F16)),
             "gq_gptq_affine: rel_err needs W_orig");
  int64_t bs = std::max<int64_t>(block_size, group_size);
  bs -= bs % group_size;
  GQ_REQUIRE(bs == 128 || bs == 256, "gq_gptq_affine: block of %lld columns unsupported (128/256)", (long long)bs);
  const size_t need = gq_gptq_affine_workspace_size(B, R, C, group_size, block_size);
  GQ_REQUIRE(workspace && workspace_bytes >= need, "gq_gptq_affine: workspace too small (%zu < %zu)",
             workspace_bytes, need);
  if (R == 0 || C == 0) return GQ_OK;
  cudaStream_t s = (cudaStream_t)stream;
  float* Err = reinterpret_cast<float*>(workspace);
  float* partials = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + align256(size_t(B) * R * bs * 4));
  const int nshrink = clip == GQ_CLIP_MSE ? kMaxShrinks : 1;
  for (int64_t i1 = 0; i1 < C; i1 += bs) {
    // the last block may be partial (gptq.py:242); it is still a whole number of groups
    const int64_t n = std::min<int64_t>(bs, C - i1);
#define AB(LPR, GS)                                                                                                \
  do {                                                                                                            \
    const size_t sm = 16 * LPR <= 128 ? size_t(16 * LPR) * (16 * LPR) * 4 : 0;                                    \
    if (sm) GQ_CUDA_TRY(cudaFuncSetAttribute(affine_rows_kernel<LPR, GS>,                                          \
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)));               \
    const dim3 cgrid(unsigned((R + 4 * (32 / LPR) - 1) / (4 * (32 / LPR))), unsigned(B));                        \
    affine_rows_kernel<LPR, GS><<<cgrid, 128, sm, s>>>(W, U, R, C, i1, int(n / LPR), bits, nshrink, storage_dtype, \
                                                       q, scales, biases, Err);                                   \
  } while (0)
    if (bs == 128) {  // 8 lanes per row, 4 rows per warp
      switch (group_size) {
        case 32: AB(8, 4); break;
        case 64: AB(8, 8); break;
        default: AB(8, 16); break;
      }
    } else {  // 256 columns: 16 lanes per row, 2 rows per warp
      switch (group_size) {
        case 32: AB(16, 2); break;
        case 64: AB(16, 4); break;
        case 128: AB(16, 8); break;
        default: AB(16, 16); break;
      }
    }
#undef AB
    int r = check_launch("affine_rows_kernel");
    if (r != GQ_OK) return r;
    const int64_t i2 = i1 + n;
    if (i2 < C) {
      GemmBatch g{};
      g.A = Err;
      g.lda = bs;
      g.sa_o = R * bs;
      g.Bm = U + i1 * C + i2;
      g.ldb = C;
      g.sb_o = C * C;
      g.Cm = W + i2;
      g.ldc = C;
      g.sc_o = R * C;
      g.n_inner = 1;
      g.M = int(R);
      g.N = int(C - i2);
      g.K = int(bs);
      g.alpha = -1.0f;
      g.beta = 1.0f;
      r = gemm(g, false, false, B, status, s);
      if (r != GQ_OK) return r;
    }
  }
  if (rel_err) {
    const dim3 pg(1024, unsigned(B));
    if (w_dtype == GQ_F32)
      rel_partials_kernel<float><<<pg, 256, 0, s>>>(W, (const float*)W_orig, R * C, partials);
    else if (w_dtype == GQ_BF16)
      rel_partials_kernel<__nv_bfloat16><<<pg, 256, 0, s>>>(W, (const __nv_bfloat16*)W_orig, R * C, partials);
    else
      rel_partials_kernel<__half><<<pg, 256, 0, s>>>(W, (const __half*)W_orig, R * C, partials);
    int r = check_launch("rel_partials_kernel");
    if (r != GQ_OK) return r;
    return launch_rel_err(partials, B, 1024, rel_err, s);
  }
  return GQ_OK;
}

extern "C" int gq_gemm_f32(const float* A, const float* Bm, float* Cm, int64_t M, int64_t N, int64_t K, int64_t lda,
                           int64_t ldb, int64_t ldc, int trans_a, int trans_b, int64_t batches, int64_t n_inner,
                           int64_t sa_o, int64_t sa_i, int64_t sb_o, int64_t sb_i, int64_t sc_o, int64_t sc_i,
                           float alpha, float beta, const int32_t* skip, int engine, int32_t* status, void* stream) {
  GQ_REQUIRE(A && Bm && Cm, "gq_gemm_f32: null pointer");
  GQ_REQUIRE(M > 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31),
             "gq_gemm_f32: bad sizes");
  GQ_REQUIRE(batches > 0 && n_inner > 0 && batches % n_inner == 0 && batches < 65536,
             "gq_gemm_f32: bad batch counts");
  GemmBatch g{};
  g.A = A;
  g.Bm = Bm;
  g.Cm = Cm;
  g.lda = lda;
  g.ldb = ldb;
  g.ldc = ldc;
  g.sa_o = sa_o;
  g.sa_i = sa_i;
  g.sb_o = sb_o;
  g.sb_i = sb_i;
  g.sc_o = sc_o;
  g.sc_i = sc_i;
  g.n_inner = int(n_inner);
  g.M = int(M);
  g.N = int(N);
  g.K = int(K);
  g.alpha = alpha;
  g.beta = beta;
  g.skip = skip;
  cudaStream_t s = (cudaStream_t)stream;
  if (engine == 1) {
    GQ_REQUIRE(tc_gemm_usable(g, trans_a != 0, trans_b != 0), "gq_gemm_f32: layout not supported by tcgen05 path");
    return tc_gemm(g, trans_a != 0, trans_b != 0, batches, status, s);
  }
  GQ_REQUIRE(engine == 0, "gq_gemm_f32: engine must be 0 (mma.sync) or 1 (tcgen05)");
  return launch_gemm(g, trans_a != 0, trans_b != 0, batches, s);
}
