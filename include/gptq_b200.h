/*
 * gptq_b200.h -- C ABI of the B200 (sm_100a) GPTQ calibration library.
 *
 * Drop-in compute boundary for Stage A of the mlx_gptq calibration engine:
 * Hessian accumulation -> damped Cholesky / H^-1 factor -> GPTQ column loop on
 * the MLX affine, MXFP4 or MXFP8 grid -> code/scale packing. Each entry point
 * names the reference interface (file:line, paths inside the mlx_gptq project)
 * whose computation it replaces.
 *
 * Conventions
 *  - Every pointer argument is DEVICE memory unless its comment says "host".
 *  - Tensors are dense row-major with the shapes given; B = batch (experts),
 *    R = out_features (rows), C = in_features (columns), G = group size.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    Calls only enqueue work unless a comment says the call synchronizes.
 *  - Return value: GQ_OK or one of the GQ_ERR_* codes; gq_last_error() gives a
 *    message for the last failing call on the calling host thread.
 *  - Re-entrant: no mutable global state; the library allocates no device memory.
 *    Scratch is caller-provided ("workspace"), sized by the *_workspace_size
 *    queries. (gq_gptq_mxfp_noalloc is the one exception: it uses a fixed array
 *    inside the library instead of a workspace; see its comment.)
 *  - Device-side waits are bounded (2 s); a kernel that gives up writes
 *    GQ_ERR_TIMEOUT to the optional device word `status` and returns.
 */
#ifndef GPTQ_B200_H_
#define GPTQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GQ_ABI_VERSION 1

/* status codes */
#define GQ_OK 0
#define GQ_ERR_ARG 1      /* bad argument (shape, dtype, alignment, mode)      */
#define GQ_ERR_NOT_PD 2   /* Hessian not positive definite after escalation    */
#define GQ_ERR_CUDA 3     /* CUDA runtime / driver error                       */
#define GQ_ERR_TIMEOUT 4  /* a bounded device-side wait gave up                */

/* element types */
#define GQ_F32 0
#define GQ_BF16 1
#define GQ_F16 2

/* quantization modes (mlx_gptq/grid.py:20) */
#define GQ_AFFINE 0
#define GQ_MXFP4 1
#define GQ_MXFP8 2

/* affine clip search (mlx_gptq/grid.py:167-212) */
#define GQ_CLIP_MINMAX 0
#define GQ_CLIP_MSE 1

/* MXFP GPTQ algorithm (mlx_gptq/gptq.py:90-92) */
#define GQ_MX_GROUPWISE 0
#define GQ_MX_SAFE_SCALE_SEARCH 1

int gq_abi_version(void);
const char* gq_status_string(int status);
const char* gq_last_error(void);

/* Self-test of the bounded device waits (no reference counterpart: the
 * reference has no device code). Launches one CTA that waits, through the same
 * wait routine as the tcgen05 pipelines, on a barrier phase that nothing
 * completes; after limit_ns (<= 2 s) the wait gives up, writes GQ_ERR_TIMEOUT to
 * *status and 1 to *gave_up (both device int32), and the kernel returns. */
int gq_selftest_wait_timeout(unsigned long long limit_ns, int32_t* status, int32_t* gave_up, void* stream);

/* ------------------------------------------------------------------------
 * Hessian accumulation
 * ------------------------------------------------------------------------ */

/* H = beta * H + alpha * X^T X.
 * X: bf16 [n, c] with row stride ldx elements (ldx % 8 == 0, X 16-byte aligned).
 * H: fp32 [c, c] with row stride ldh elements. Products of bf16 values are
 * accumulated in fp32 on the tensor cores (tcgen05, TMEM accumulators); only
 * tiles on or above the diagonal are computed and the result is mirrored, so
 * the written H is exactly symmetric.
 * Replaces Stash.hessian (mlx_gptq/capture.py:68-76), which is the case
 * alpha = 1, beta = 0 (first chunk) / 1 (later chunks). */
int gq_hessian_bf16(const void* X, int64_t n, int64_t c, int64_t ldx, float* H, int64_t ldh, float alpha,
                    float beta, int32_t* status, void* stream);

/* The same over output tiles [tile_begin, tile_end) of the kernel's schedule
 * (gq_hessian_tile_count(c) tiles in all, each a block on or above the diagonal
 * plus its mirror): only those blocks of H are written, with exactly the values
 * the full call writes there. Ranks that each hold every row of X split one H
 * this way and merge disjoint blocks; no reference counterpart (the reference
 * forms each H on one device, mlx_gptq/sequential.py:479-487). */
int64_t gq_hessian_tile_count(int64_t c);
/* Tiles the kernel runs at once on a GPU with sm_count SMs (one per CTA pair for
 * the default kernel). Each tile sweeps every row of X, so a range of at most this
 * many tiles takes about as long as one wave. */
int64_t gq_hessian_concurrent_tiles(int64_t sm_count);
int gq_hessian_bf16_range(const void* X, int64_t n, int64_t c, int64_t ldx, float* H, int64_t ldh, float alpha,
                          float beta, int64_t tile_begin, int64_t tile_end, int32_t* status, void* stream);

/* Per-expert Hessians in one launch:
 * H[e] = beta * H[e] + alpha * sum over t in token_idx[offsets[e] .. offsets[e+1]) of X[t]^T X[t],
 * for e < E. X: bf16 [n, c] (ldx % 8 == 0, c % 8 == 0); token_idx: int32 row indices into X;
 * offsets: int64 [E + 1] (device) and host_offsets (the same values in host memory, used
 * to plan the launch); H: fp32 [E, c, c]. Experts without tokens get H[e] = beta * H[e].
 * The routed rows are first copied into zero-padded per-expert segments of the
 * workspace (gq_hessian_grouped_workspace_size bytes), then one tcgen05 launch covers
 * every (expert, tile) pair, heaviest experts first.
 * Replaces the per-expert Stash.hessian calls of mlx_gptq/sequential.py:546-555
 * (stashes filled by the expert routing of mlx_gptq/capture.py:192-207). */
size_t gq_hessian_grouped_workspace_size(const int64_t* host_offsets, int64_t E, int64_t c);
int gq_hessian_grouped_bf16(const void* X, int64_t n, int64_t c, int64_t ldx, const int32_t* token_idx,
                            const int64_t* offsets, const int64_t* host_offsets, int64_t E, float* H, float alpha,
                            float beta, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Per-expert Hessians over contiguous row spans, in one launch:
 * H[e] = beta * H[e] + alpha * X[s_e .. s_e + k_e)^T X[s_e .. s_e + k_e), e < E, with
 * host_spans[2e] = s_e and host_spans[2e+1] = k_e (host memory; spans may overlap and
 * come in any order, 0 <= s_e, s_e + k_e <= n). The rows are read in place; only each
 * expert's partial last 64-row step (k_e % 64 rows, zero-padded) is copied into the
 * workspace (gq_hessian_spans_workspace_size bytes). Always the 2-SM kernel.
 * Replaces the per-expert Stash.hessian calls of mlx_gptq/sequential.py:546-555 when
 * each expert's stash is one contiguous block of rows (capture.py:33-76 stores an
 * expert's rows as its own chunks), e.g. down_proj inputs laid out expert by expert. */
size_t gq_hessian_spans_workspace_size(const int64_t* host_spans, int64_t E, int64_t c);
int gq_hessian_spans_bf16(const void* X, int64_t n, int64_t c, int64_t ldx, const int64_t* host_spans, int64_t E,
                          float* H, float alpha, float beta, void* workspace, size_t workspace_bytes, int32_t* status,
                          void* stream);

/* Partial Hessians of an expert whose rows were cut into pieces (one grouped launch
 * over all pieces), summed into the expert's first: for t < n_targets,
 * H[targets[t]] += H[p] for p = pieces[piece_ptr[t]] .. pieces[piece_ptr[t+1] - 1],
 * added in that order (the same bits as adding them one by one). H: fp32 [V, c, c];
 * targets [n_targets], piece_ptr [n_targets + 1], pieces: int64 device arrays.
 * No counterpart in the reference, which forms each expert's Hessian in one call
 * (mlx_gptq/sequential.py:546-555). */
int gq_hessian_merge_pieces(float* H, int64_t c, int64_t n_targets, const int64_t* targets,
                            const int64_t* piece_ptr, const int64_t* pieces, void* stream);

/* ------------------------------------------------------------------------
 * Solver pieces (mlx_gptq/gptq.py)
 * ------------------------------------------------------------------------ */

/* Dead columns (gptq.py:216-222): for every (b, j) with H[b, j, j] <= 0 set
 * H[b, j, j] = 1 (in place) and dead[b, j] = 1, else dead[b, j] = 0.
 * H: fp32 [B, C, C]; dead: uint8 [B, C]. */
int gq_dead_columns(float* H, int64_t B, int64_t C, uint8_t* dead, void* stream);

/* Upper Cholesky factor of the damped inverse of every 32x32 diagonal block:
 * U[b, g] = chol((H[b, g, g] + damp * mean(diag) * I)^-1, upper), with the damping
 * escalated x10 per block on failure, at most 6 attempts (gptq.py:27-66 as
 * called per group by gptq.py:99-100).
 * H: fp32 [B, C, C] (C % 32 == 0); U: fp32 [B, C/32, 32, 32];
 * info: int32 [B, C/32], 0 = factored (possibly after escalation), 1 = not
 * positive definite after 6 attempts, 2 = the inverse could not be factored;
 * damp_used: fp32 [B, C/32] damping factor that succeeded (nullable). */
int gq_mx_prepare_hinv(const float* H, int64_t B, int64_t C, float damp, float* U, int32_t* info,
                       float* damp_used, void* stream);

/* Upper Cholesky factor of the damped inverse of the full H (gptq.py:27-66):
 * U[b] = chol((H[b] + damp_b * mean(diag H[b]) * I)^-1, upper); damp_b starts at
 * `damp` and is escalated x10 for items whose factorization fails, at most 6
 * attempts. SYNCHRONIZES `stream` after each attempt to read the per-item
 * status. Returns GQ_ERR_NOT_PD if an item still fails (info[b] != 0).
 * H: fp32 [B, C, C] (C % 64 == 0); U: fp32 [B, C, C] (upper; lower part zero);
 * info: int32 [B]; damp_used: fp32 [B] (nullable). status: optional device int32;
 * a bounded wait of the tensor-core GEMMs that gives up writes GQ_ERR_TIMEOUT there. */
size_t gq_prepare_hinv_workspace_size(int64_t B, int64_t C);
int gq_prepare_hinv(const float* H, int64_t B, int64_t C, float damp, float* U, int32_t* info, float* damp_used,
                    void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* MXFP GPTQ (gptq.py:69-180): per 32-column group, sequential GPTQ with a fixed
 * E8M0 scale (groupwise: the RTN scale; safe-scale-search: the scale offset with
 * the smallest e^T H_g e, then GPTQ kept only if its objective is <= the best
 * RTN objective), range guard |dq| <= max(32 * max|w|, 2^-126).
 * W: [B, R, C] of w_dtype (GQ_F32/GQ_BF16/GQ_F16), the original weights;
 *    columns with dead[b, j] != 0 are treated as zero (dead: uint8 [B, C], nullable).
 * H: fp32 [B, C, C] (after gq_dead_columns); U: from gq_mx_prepare_hinv;
 * info: from gq_mx_prepare_hinv (groups with info != 0 are skipped; nullable).
 * Outputs (each nullable except scales): q uint8 [B, R, C] codes (E2M1 nibble
 * code or E4M3 byte); q_packed uint8 [B, R, C/2] two E2M1 codes per byte, low
 * nibble first (mxfp4 only; the MLX uint32 words are these bytes read
 * little-endian); scales uint8 [B, R, C/32] E8M0 bytes; w_dq [B, R, C] of
 * wdq_dtype (GQ_F32 / GQ_BF16); rel_err fp32 [B] = ||W_dq - W||_F / ||W||_F
 * (solve_gptq, gptq.py:300-302; needs workspace).
 * Replaces gptq_quantize / solve_gptq for mode mxfp4 / mxfp8. */
size_t gq_gptq_mxfp_workspace_size(int64_t B, int64_t R, int64_t C);
int gq_gptq_mxfp(const void* W, int w_dtype, const float* H, const float* U, const uint8_t* dead,
                 const int32_t* info, int64_t B, int64_t R, int64_t C, int mode, int algorithm, uint8_t* q,
                 uint8_t* q_packed, uint8_t* scales, void* w_dq, int wdq_dtype, float* rel_err, void* workspace,
                 size_t workspace_bytes, void* stream);

/* Same computation and arguments as gq_gptq_mxfp, but the library allocates
 * nothing and the caller passes no workspace: the rel_err partial sums live in a
 * fixed 4 MiB array inside the library (every GPU that loads the library holds
 * it until the process exits). For hosts that cannot call cudaMalloc: callers
 * that own all device memory through their own pool or arena, that must not
 * allocate while running (an embedded runtime, a real-time serving loop), or
 * whose binding layer has no CUDA allocator to reach (a JNI, cgo or ctypes shim
 * given only the tensors it must read and write). Inputs and outputs are still
 * the caller's.
 * Limit (only when rel_err is requested): B * ceil(R/128) * (C/32) <= 524288
 * (row tile, group) pairs, else GQ_ERR_ARG; e.g. [1, 11008, 4096] uses 11008 and
 * [128, 1536, 2048] uses 98304. With rel_err == NULL the column loop needs no
 * scratch at all: any size is accepted and the array is not touched.
 * The first call on a device that asks for rel_err looks up the array's device
 * address (once per device, with that device current) and caches it; make that
 * first call before any stream capture, and do not reset the device
 * (cudaDeviceReset) between calls, which would leave the cached address stale.
 * The array is shared by all calls and keeps the last call's contents; each call
 * rewrites every entry it reads (groups whose factor failed, info != 0, write
 * zeros and so drop out of rel_err), so nothing needs clearing, but calls that
 * overlap on the GPU (other streams, other host threads) race on it.
 * This entry point has no counterpart in the reference. */
int gq_gptq_mxfp_noalloc(const void* W, int w_dtype, const float* H, const float* U, const uint8_t* dead,
                         const int32_t* info, int64_t B, int64_t R, int64_t C, int mode, int algorithm, uint8_t* q,
                         uint8_t* q_packed, uint8_t* scales, void* w_dq, int wdq_dtype, float* rel_err, void* stream);

/* Affine GPTQ (gptq.py:183-272): blocked column loop (block = max(block_size, G)
 * rounded down to a multiple of G) with the MSE/minmax clip search at each group
 * start on the compensated weights, bf16/fp16/fp32-rounded scale and bias
 * before error feedback, in-block rank-1 updates and the lazy trailing update
 * W[:, :, i2:] -= Err * U[i1:i2, i2:] after every block.
 * W: fp32 [B, R, C] working weights, overwritten with W_dq (dead columns must
 *    already be zero, see gq_prepare_weights); W_orig: [B, R, C] of w_dtype, the
 *    untouched originals for rel_err (nullable).
 * U: from gq_prepare_hinv. q: uint8 [B, R, C]; scales / biases: [B, R, C/G] of
 * storage_dtype (GQ_BF16 / GQ_F16 / GQ_F32); rel_err fp32 [B] (nullable).
 * G % 32 == 0 and G <= 256. status: optional device int32 (as in gq_prepare_hinv). */
size_t gq_gptq_affine_workspace_size(int64_t B, int64_t R, int64_t C, int group_size, int block_size);
int gq_gptq_affine(float* W, const void* W_orig, int w_dtype, const float* U, int64_t B, int64_t R, int64_t C,
                   int bits, int group_size, int block_size, int clip, int storage_dtype, uint8_t* q, void* scales,
                   void* biases, float* rel_err, void* workspace, size_t workspace_bytes, int32_t* status,
                   void* stream);

/* The float32 GEMM the affine solver runs its trailing updates and factor
 * products on, exposed for testing: per batch item z = outer * n_inner + inner,
 * C = alpha * op(A) op(B) + beta * C with op(A)(r, t) = A[t*lda + r] if trans_a else
 * A[r*lda + t] (M x K), op(B)(t, c) = B[c*ldb + t] if trans_b else B[t*ldb + c]
 * (K x N), item offsets outer*s?_o + inner*s?_i (elements); items whose outer index
 * has skip[outer] != 0 are left alone (skip nullable). engine 1: TMA-fed tcgen05
 * kind::tf32 in a 3xTF32 split (16-byte aligned A and B, leading dimensions and
 * strides multiples of 4); engine 0: the mma.sync 3xTF32 kernels. No counterpart in
 * the reference (its torch.bmm / matmul calls, gptq.py:269-270). */
int gq_gemm_f32(const float* A, const float* Bm, float* Cm, int64_t M, int64_t N, int64_t K, int64_t lda,
                int64_t ldb, int64_t ldc, int trans_a, int trans_b, int64_t batches, int64_t n_inner, int64_t sa_o,
                int64_t sa_i, int64_t sb_o, int64_t sb_i, int64_t sc_o, int64_t sc_i, float alpha, float beta,
                const int32_t* skip, int engine, int32_t* status, void* stream);

/* W_out (fp32 [B, R, C]) = W_in converted to fp32, with columns where
 * dead[b, j] != 0 set to zero (the W.float().clone() + dead-column zeroing of
 * gptq.py:288 and gptq.py:219-221). dead is nullable. */
int gq_prepare_weights(const void* W_in, int w_dtype, const uint8_t* dead, int64_t B, int64_t R, int64_t C,
                       float* W_out, void* stream);

/* ------------------------------------------------------------------------
 * Grids (mlx_gptq/grid.py)
 * ------------------------------------------------------------------------ */

/* RTN on the MLX affine grid (rtn_quantize, grid.py:224-246 with choose_qparams
 * grid.py:167-212 and quantize_with_params grid.py:215-221).
 * W: [rows, C] of w_dtype; q uint8 [rows, C]; scales / biases [rows, C/G] of
 * storage_dtype; w_dq [rows, C] of wdq_dtype (nullable). */
int gq_rtn_affine(const void* W, int w_dtype, int64_t rows, int64_t C, int bits, int group_size, int clip,
                  int storage_dtype, uint8_t* q, void* scales, void* biases, void* w_dq, int wdq_dtype,
                  void* stream);

/* Native MXFP RTN (rtn_quantize_mxfp, grid.py:142-151 with choose_mxfp_scale
 * grid.py:61-79 and quantize_mxfp_with_scale grid.py:108-124).
 * W: [rows, C] (C % 32 == 0); q uint8 [rows, C]; scales uint8 [rows, C/32];
 * q_packed uint8 [rows, C/2] (mxfp4 only, nullable); w_dq nullable. */
int gq_rtn_mxfp(const void* W, int w_dtype, int64_t rows, int64_t C, int mode, uint8_t* q, uint8_t* q_packed,
                uint8_t* scales, void* w_dq, int wdq_dtype, void* stream);

/* dequantize_artifact (grid.py:154-164, dequantize_mxfp grid.py:127-139):
 * affine: out = q * scale + bias (scales/biases [rows, C/G] of scale_dtype);
 * mxfp: out = value(q) * 2^(scale_byte - 127) (scales uint8 [rows, C/32]). */
int gq_dequantize(const uint8_t* q, const void* scales, const void* biases, int scale_dtype, int64_t rows,
                  int64_t C, int mode, int group_size, float* out, void* stream);

/* ------------------------------------------------------------------------
 * Packing (mlx_gptq/packing.py, mlx_gptq/artifacts.py)
 * ------------------------------------------------------------------------ */

/* pack_q (packing.py:15-26): words[r, i] = sum_k q[r, i*per + k] << (bits*k),
 * per = 32/bits, bits in {2, 4, 8}; q uint8 [rows, C] (C % per == 0). */
int gq_pack_q(const uint8_t* q, int64_t rows, int64_t C, int bits, uint32_t* words, void* stream);
/* unpack_q (packing.py:33-39): q[r, j] for j < out_cols from words [rows, n_words]. */
int gq_unpack_q(const uint32_t* words, int64_t rows, int64_t n_words, int bits, int64_t out_cols, uint8_t* q,
                void* stream);
/* pack_nibbles (artifacts.py:30-32): out[r, i] = q[r, 2i] | q[r, 2i+1] << 4. */
int gq_pack_nibbles(const uint8_t* q, int64_t rows, int64_t C, uint8_t* out, void* stream);
/* unpack_nibbles (artifacts.py:35-39). */
int gq_unpack_nibbles(const uint8_t* packed, int64_t rows, int64_t n_bytes, uint8_t* q, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GPTQ_B200_H_ */
