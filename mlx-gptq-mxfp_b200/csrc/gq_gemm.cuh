// Batched float32 GEMM descriptor shared by the affine solver's kernels:
// C = alpha * op(A) * op(B) + beta * C per batch item, with
//   op(A)(r, t) = TRANS_A ? A[t * lda + r] : A[r * lda + t]   (M x K)
//   op(B)(t, c) = TRANS_B ? B[c * ldb + t] : B[t * ldb + c]   (K x N)
// and batch item z = outer * n_inner + inner.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gq {

struct GemmBatch {
  const float* A;
  const float* Bm;
  float* Cm;
  int64_t lda, ldb, ldc;
  int64_t sa_o, sb_o, sc_o;  // outer strides (elements)
  int64_t sa_i, sb_i, sc_i;  // inner strides
  int n_inner;
  int M, N, K;
  float alpha, beta;
  const int32_t* skip;  // per outer item: nonzero = skip (nullable)
};

// The same product on the 5th-generation tensor cores (TMA-fed tcgen05.mma kind::tf32
// in a 3xTF32 split, accumulators in TMEM), for operands a tensor map can describe:
// tc_gemm_usable says whether it takes this product; tc_gemm launches it. A device
// wait that gives up writes GQ_ERR_TIMEOUT to *status (device int32, nullable).
// lower_only (square products): 128 x 128 tiles strictly above the diagonal are not
// computed; tiles on it are computed whole (their upper part included).
bool tc_gemm_usable(const GemmBatch& p, bool trans_a, bool trans_b);
int tc_gemm(const GemmBatch& p, bool trans_a, bool trans_b, int64_t batches, int32_t* status, cudaStream_t s,
            bool lower_only = false);

}  // namespace gq
