/*
 * sparsecore_b200 — C-ABI of the B200 (sm_100a) padded-CSR sparse-training
 * kernels.
 *
 * Every entry point takes plain device pointers and sizes, enqueues its work
 * on the CUDA stream passed as `stream` (a cudaStream_t passed as void*;
 * NULL = legacy default stream) and returns 0 on success or a nonzero
 * SL_ERR_* code, with a human-readable message in sl_last_error() (per
 * thread).  Nothing here synchronises the device unless stated.
 *
 * Layout (identical to the reference's sparselab::PaddedCSR,
 * csrc/kernels/padded_csr.hpp:47-74):
 *   values       float[total_capacity]   live slots first in each row
 *   col_indices  int32[total_capacity]   ascending within a row; padding -1
 *   row_start    int32[nrows]            exclusive prefix sum of row_capacity
 *   row_nnz      int32[nrows]
 *   row_capacity int32[nrows]
 * Dense operands are row-major float32: X[K,N], Y[M,N], dY[M,N].
 */
#ifndef SPARSECORE_B200_H
#define SPARSECORE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SL_API __attribute__((visibility("default")))
#else
#define SL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SL_OK = 0,
    SL_ERR_INVALID = 1,     /* bad shape / argument (reference: ValueError) */
    SL_ERR_CUDA = 2,        /* a CUDA runtime call failed                   */
    SL_ERR_UNSUPPORTED = 3, /* size beyond a documented kernel limit        */
    SL_ERR_TIMEOUT = 4      /* a bounded device-side wait ran out           */
};

/* Device-resident padded CSR (all pointers are device pointers). */
typedef struct sl_csr {
    int64_t nrows;
    int64_t ncols;
    int64_t total_capacity;
    float* values;
    int32_t* col_indices;
    int32_t* row_start;
    int32_t* row_nnz;
    int32_t* row_capacity;
} sl_csr;

/* Message of the last failed call on this host thread ("" if none). */
SL_API const char* sl_last_error(void);
/* Name of the kernel that the last sl_spmm_fwd / sl_sddmm_dw call on this
 * host thread launched (a diagnostic with no reference counterpart: tests
 * use it to prove which decomposition produced the values they check). */
SL_API const char* sl_last_kernel(void);
/* Roofline probes (no reference counterpart): sl_probe_ffma runs
 * sl_probe_threads() threads, each advancing 8 independent fp32 FMA chains
 * for `iters` steps (16 * iters FLOPs per thread); sl_probe_smem has the same
 * threads each read 4 * `iters` conflict-free 8-byte shared-memory words
 * (each address depends on the previous load, so none is optimised away).
 * `out` receives one float per thread (sl_probe_threads() floats).  Timed by
 * the caller (CUDA events) to give the measured FP32 and shared-memory
 * ceilings the kernels' fractions are reported against. */
SL_API int64_t sl_probe_threads(void);
SL_API int sl_probe_ffma(int64_t iters, float* out, void* stream);
SL_API int sl_probe_smem(int64_t iters, float* out, void* stream);
/* Library version string. */
SL_API const char* sl_version(void);
/* Status word of the current device (synchronous): bit 0 set = a bounded
 * device-side wait (TMA / mbarrier) gave up instead of hanging; that call's
 * output is invalid.  reset != 0 clears the word after reading. */
SL_API int sl_device_status(int reset, unsigned* out);
/* Self-test of the bounded device waits (no reference counterpart): launches
 * one warp that waits on an mbarrier nothing completes; after `spins` polls
 * (1 .. 2^24) the wait gives up, raises bit 0 of the status word and the
 * kernel returns -- the context stays usable.  Read it with
 * sl_device_status. */
SL_API int sl_selftest_bounded_wait(int64_t spins, void* stream);

/* ── Forward SpMM ─────────────────────────────────────────────────────────
 * Y[M,N] = W[M,K] . X[K,N].  Each Y element is the fp32 FMA chain over the
 * row's live slots in slot order, starting from +0 — bit-identical to the
 * reference CPU kernel.
 * Replaces: csrc/kernels/spmm_avx2.cpp:82 spmm_simd_avx2 (and spmm_scalar,
 * csrc/kernels/spmm.cpp:122) behind csrc/bindings.cpp:253 py_spmm_simd.
 * Also computes dX = W^T . dY when given the transposed CSR
 * (sparselab/ops.py:201-203). */
SL_API int sl_spmm_fwd(const sl_csr* W, const float* X, int64_t K, int64_t N,
                float* Y, void* stream);
/* Forward with the GELU of a SparseLinear -> GELU pair fused in
 * (sparselab/nn.py:229-245 applies the activation separately): Y as
 * sl_spmm_fwd and H[M,N] = gelu(Y) with torch's exact-erf GELU rounding
 * ((y * 0.5) * (1 + erf(y * sqrt(1/2))), each step rounded to fp32), written
 * by the same kernel where the X-stationary or row-gather decomposition
 * runs, else by a second pass.  Y is kept for the GELU backward. */
SL_API int sl_spmm_fwd_gelu(const sl_csr* W, const float* X, int64_t K, int64_t N,
                     float* Y, float* H, void* stream);
/* Forward with a SparseLinear's bias and activation fused into the kernel
 * (sparselab/nn.py:239-241 adds the bias after the layer; the activation of
 * an FFN pair runs as a separate torch op):
 *   Y[M,N] = W . X + bias[M] (broadcast along N; bias may be NULL), and
 *   H[M,N] = act(Y) for act = 1 (ReLU: negative -> 0, NaN kept) or 2 (GELU,
 *   exact erf, torch's rounding); act = 0 writes no H (H may be NULL).
 * The bias add is one fp32 add per element, as torch's, so Y and H are
 * bit-identical to the unfused ops.  Fused into the X-stationary and
 * row-gather kernels' epilogue, else applied by a second pass. */
SL_API int sl_spmm_fwd_act(const sl_csr* W, const float* X, int64_t K, int64_t N,
                    const float* bias, int act, float* Y, float* H, void* stream);

/* ── SDDMM weight gradient ────────────────────────────────────────────────
 * dW[slot] = <dY[i,:], X[col[slot],:]> for live slots of row i, 0 for
 * padding; dW has total_capacity entries aligned with W.values.  The dot is
 * evaluated in the reference AVX2 kernel's lane order (bit-identical).
 * Replaces: csrc/kernels/spmm_grad_avx2.cpp:73 spmm_grad_w_simd behind
 * csrc/bindings.cpp:410 py_spmm_grad_w_simd. */
SL_API int sl_sddmm_dw(const sl_csr* W, const float* dY, const float* X,
                int64_t N, float* dW, void* stream);

/* ── Transpose with permutation ───────────────────────────────────────────
 * Two-phase GPU build of W^T (sparselab/layout.py:460 transpose_with_perm).
 * Phase 1 counts: fills out_row_nnz/out_row_capacity/out_row_start (int32
 * [ncols]) and *out_total_dev (device int64) with the transpose's total
 * capacity, using `scratch` (device, sl_transpose_scratch_bytes bytes).
 * Capacity per row = max(1, ceil(nnz * one_plus_padding_ratio)) in float64.
 * Phase 2 fills WT (whose row arrays are the phase-1 outputs and whose slot
 * arrays hold *out_total_dev entries) and perm[int64, WT total capacity]:
 * perm[slot_T] = source slot in W, -1 for padding.  Output rows list the
 * source rows in ascending order.  `scratch` must be passed unchanged from
 * phase 1. */
SL_API int64_t sl_transpose_scratch_bytes(int64_t nrows, int64_t ncols);
SL_API int sl_transpose_count(const sl_csr* W, double one_plus_padding_ratio,
                       int32_t* out_row_nnz, int32_t* out_row_capacity,
                       int32_t* out_row_start, int64_t* out_total_dev,
                       void* scratch, void* stream);
SL_API int sl_transpose_fill(const sl_csr* W, const sl_csr* WT, int64_t* perm,
                      const void* scratch, void* stream);

/* Transpose with permutation that allocates nothing.
 * No counterpart in the reference: it is an addition for callers that cannot
 * call cudaMalloc -- e.g. code running inside a memory pool or allocator
 * hook, a real-time loop that forbids allocation, or an embedding host that
 * owns all device memory -- and so cannot provide the scratch buffer that
 * sl_transpose_count / sl_transpose_fill need.  It writes the same WT and
 * perm as sl_transpose_count followed by sl_transpose_fill, in one call:
 *   * scratch is a file-scope device array of 4 MiB (2^20 int32 counters)
 *     that every GPU loading the library holds until the process exits;
 *     inputs need ceil(nrows/32) * ncols <= 2^20 (and ncols <= 57344), else
 *     SL_ERR_UNSUPPORTED with a message;
 *   * WT's row arrays (int32[W.ncols]) receive row_nnz / row_capacity /
 *     row_start; its slot arrays (values, col_indices) and `perm` must hold
 *     WT->total_capacity >= floor(one_plus_padding_ratio * W.total_capacity)
 *     + W.ncols + 2 entries (an upper bound of the true size), else
 *     SL_ERR_INVALID.  The true total capacity is written to *out_total_dev;
 *     entries past it are padding (-1, 0.0f, perm -1);
 *   * the first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current.  If no other kernel
 *     of this library has run on that device yet, that lookup is also what
 *     makes CUDA load the library's device code there (with lazy module
 *     loading, the CUDA 12 default) and place the array: memory the driver
 *     sets aside once.  Make that first call at initialisation, before any
 *     stream capture and before the point from which nothing may allocate;
 *   * every call shares the one array and leaves its contents behind (the
 *     kernels overwrite all of it they read, so nothing must be cleared);
 *     calls whose work overlaps on the GPU (different streams, or several
 *     host threads) race on it and give wrong results -- serialise them.
 * After that first call a successful call allocates no device or host
 * memory and calls no allocating routine; a failing call formats its
 * message for sl_last_error() in a host string. */
SL_API int sl_transpose_with_perm_noalloc(const sl_csr* W, double one_plus_padding_ratio,
                                   const sl_csr* WT, int64_t* perm,
                                   int64_t* out_total_dev, void* stream);

/* Cached-transpose value refresh: dst[t] = src[perm[t]] where perm[t] >= 0
 * (sparselab/ops.py:83-94, the cache-hit path of _cached_transpose). */
SL_API int sl_values_gather(const int64_t* perm, const float* src, float* dst,
                     int64_t n, void* stream);

/* ── Layout factories ─────────────────────────────────────────────────────
 * Dense [M,K] -> padded CSR (sparselab/layout.py:172 from_dense, via
 * from_torch_sparse_csr :75).  live = |w| > threshold if threshold > 0,
 * else w != 0.
 * Phase 1: row_nnz, row_capacity, row_start and *out_total_dev.
 * Phase 2: fill values/col_indices of `out` (sized from phase 1). */
SL_API int sl_dense_count(const float* dense, int64_t M, int64_t K, float threshold,
                   double one_plus_padding_ratio, int32_t* row_nnz,
                   int32_t* row_capacity, int32_t* row_start,
                   int64_t* out_total_dev, void* stream);
SL_API int sl_dense_fill(const float* dense, float threshold, const sl_csr* out,
                  void* stream);
/* Capacity + exclusive scan for given per-row counts (layout.py:46-68,
 * :131-133). */
SL_API int sl_capacity_scan(const int32_t* row_nnz, int64_t n,
                     double one_plus_padding_ratio, int32_t* row_capacity,
                     int32_t* row_start, int64_t* out_total_dev,
                     void* stream);
/* Padded CSR -> dense [M,K] (layout.py:262 to_dense); `dense` is fully
 * overwritten. */
SL_API int sl_to_dense(const sl_csr* W, float* dense, void* stream);

/* Invariant check (csrc/kernels/padded_csr.cpp:79 check_invariants_str).
 * report (device int64[4]) receives {code, row, slot, 0}; code 0 = all hold,
 * else 3 (row_start), 4 (row_nnz range), 6 (live column), 7 (padding
 * column) of the first violation in the reference's check order.
 * Array-length checks (invariants 1, 2) are the caller's. */
SL_API int sl_check_invariants(const sl_csr* W, int64_t n_slots, int64_t* report,
                        void* stream);

/* ── Dense gradient (RigL grow criterion) ─────────────────────────────────
 * G[M,K] = dY[M,N] . X[K,N]^T in fp32, each element accumulated over N in
 * the reference build's rounding sequence (bit-identical).  Replaces csrc/kernels/dense_grad.cpp:463 dense_grad behind
 * csrc/bindings.cpp:445 py_dense_grad. */
SL_API int sl_dense_grad(const float* dY, const float* X, int64_t M, int64_t K,
                  int64_t N, float* G, void* stream);

/* RigL grow selection without materialising G (sparselab/router.py:631-721:
 * G = dense_grad(dY, X), survivors masked to -inf, np.argpartition of -|G|
 * per row; the streaming top-k of docs/design/rigl.md:86-93), in three
 * calls after sl_dst_threshold / sl_dst_keep:
 *   sl_rigl_prep: survivor bitmap uint32[M][ceil(K/32)] (|v| > thr or the
 *     row's forced keep) and n_grow[M] = min(n_drop, K - n_keep) (0 for
 *     empty rows);
 *   sl_rigl_candidates: the dense-gradient GEMM (same per-element rounding
 *     as sl_dense_grad) whose epilogue keeps, per row and tile of T =
 *     tile_cols columns (64 or 128; sl_rigl_tile_cols gives the GEMM's
 *     preferred tiling), the min(n_grow + 1, lmax) largest candidate keys
 *     (|G| bits + 1) and their columns: cand_key / cand_col
 *     [M][ceil(K/T)][lmax], cand_cnt [M][ceil(K/T)]; lmax in [1, 128] must
 *     be >= n_grow + 1 for every row or >= T.  row_flag[M] must be zero on
 *     entry; bit 0 is set for rows with a NaN candidate;
 *   sl_rigl_merge: per row the n_grow largest keys become grow_cols at
 *     grow_offsets[row] (exclusive scan of n_grow); rows where the next key
 *     ties the cut, or with a NaN, get row_flag = 1 and row_mask = 0 (the
 *     caller resolves them with the reference's argpartition on G rows it
 *     recomputes); other live rows get row_mask = 1 for sl_dst_apply_cols. */
SL_API int sl_rigl_prep(const sl_csr* W, const float* thr_dev, const int32_t* force_idx,
                 uint32_t* survivor_bits, int32_t* n_grow, void* stream);
SL_API int64_t sl_rigl_tile_cols(int64_t M, int64_t K);
SL_API int sl_rigl_candidates(const float* dY, const float* X, int64_t M, int64_t K, int64_t N,
                       const uint32_t* survivor_bits, const int32_t* n_grow, int64_t lmax,
                       int64_t tile_cols, uint32_t* cand_key, int32_t* cand_col,
                       int32_t* cand_cnt, int32_t* row_flag, void* stream);
SL_API int sl_rigl_merge(int64_t M, int64_t K, int64_t lmax, int64_t tile_cols,
                  const uint32_t* cand_key,
                  const int32_t* cand_col, const int32_t* cand_cnt, const int32_t* n_grow,
                  const int32_t* grow_offsets, const int32_t* row_nnz, int32_t* row_flag,
                  int32_t* row_mask, int32_t* grow_cols, void* stream);

/* ── Dynamic-sparsity prune / regrow (sparselab/router.py) ───────────────
 * sl_dst_threshold: k-th smallest |value| (1-based k) over all live slots,
 *   exact (router.py:395-412, np.partition).  Writes the float to *thr_dev.
 *   scratch: sl_dst_scratch_bytes() bytes of device memory.
 * sl_dst_keep: per row, n_keep[i] = #{live |v| > thr} with the reference's
 *   force-keep of the first max-|v| slot when none survives
 *   (router.py:420-439); force_idx[i] = that slot offset or -1.
 * sl_dst_apply_random: SET rewrite (router.py:441-478).  grow_offsets
 *   [nrows+1] (exclusive scan) delimit, per row, the 0-based ranks drawn
 *   on the host among the row's non-surviving columns in ascending order
 *   (numpy Generator.choice(pool, n_grow, replace=False)).  Grown slots get
 *   value 0; the row is rewritten column-sorted with (-1, 0) padding.
 * sl_dst_apply_topk: RigL rewrite (router.py:641-733): grows the n_grow =
 *   min(n_live - n_keep, ncols - n_keep) non-surviving columns of largest
 *   |G[i,:]|.  Rows whose choice is not unique (ties at the cut, or NaN)
 *   are left untouched and flagged in row_flag[i] = 1 for the caller to
 *   resolve (then sl_dst_apply_cols); row_flag[i] = 0 otherwise.
 * sl_dst_apply_cols: rewrite given rows with explicit grown columns:
 *   grow_offsets[nrows+1] delimit per-row column lists; rows with
 *   row_mask[i] == 0 are not touched.
 * All apply kernels need ncols <= sl_dst_max_ncols(). */
SL_API int64_t sl_dst_scratch_bytes(void);
SL_API int64_t sl_dst_max_ncols(void);
SL_API int sl_dst_threshold(const sl_csr* W, int64_t k, float* thr_dev,
                     void* scratch, void* stream);
SL_API int sl_dst_keep(const sl_csr* W, const float* thr_dev, int32_t* n_keep,
                int32_t* force_idx, void* stream);
SL_API int sl_dst_apply_random(const sl_csr* W, const float* thr_dev,
                        const int32_t* force_idx, const int32_t* grow_offsets,
                        const int32_t* grow_ranks, void* stream);
SL_API int sl_dst_apply_topk(const sl_csr* W, const float* thr_dev,
                      const int32_t* force_idx, const float* G,
                      int32_t* row_flag, void* stream);
SL_API int sl_dst_apply_cols(const sl_csr* W, const float* thr_dev,
                      const int32_t* force_idx, const int32_t* row_mask,
                      const int32_t* grow_offsets, const int32_t* grow_cols,
                      void* stream);

/* SET regrow draws, on the host (no device work; host pointers).  For each
 * row i with n_live[i] > 0, pool = ncols - n_keep[i], n_drop = n_live[i] -
 * n_keep[i], and (when pool and n_drop are non-zero) n_grow = min(n_drop,
 * pool) ranks drawn exactly as numpy's Generator(PCG64).choice(pool,
 * size=n_grow, replace=False) called row by row (sparselab/router.py:457-470
 * SET._update_layer); counts[i] = n_grow (0 otherwise) and the ranks are
 * concatenated into ranks[0 .. *n_ranks).  Generator state in / out:
 * pcg_state = {state_hi, state_lo, inc_hi, inc_lo}, *has_uint32, *uinteger
 * (numpy's bit_generator.state fields).  SL_ERR_INVALID when ranks_cap is
 * too small. */
SL_API int sl_set_regrow_draws(uint64_t* pcg_state, int32_t* has_uint32, uint32_t* uinteger,
                        int64_t nrows, const int32_t* n_live, const int32_t* n_keep,
                        int64_t ncols, int32_t* counts, int32_t* ranks, int64_t ranks_cap,
                        int64_t* n_ranks);

/* ── Dense layout helper ──────────────────────────────────────────────────
 * dst[cols, rows] = src[rows, cols]^T (fp32, row-major, not in place).
 * Replaces the torch copies of the reference's SparseLinear
 * (sparselab/nn.py:229-237: x.reshape(-1, in).t().contiguous() and the .t()
 * of the result): activations stay token-major [tokens, features] outside
 * the layer and column-per-token [features, tokens] for the kernels. */
SL_API int sl_transpose_f32(const float* src, int64_t rows, int64_t cols, float* dst,
                     void* stream);
/* dst[cols, rows] = src[rows, cols]^T + bias[rows] broadcast along the new
 * rows: the SparseLinear output transpose with the layer's bias add fused in
 * (sparselab/nn.py:229-245 adds the bias to the strided Y.t() afterwards).
 * Each element is one fp32 add, as torch's, so the result is bit-identical. */
SL_API int sl_transpose_bias_f32(const float* src, int64_t rows, int64_t cols,
                                 const float* bias, float* dst, void* stream);

/* Fused AdamW over a SparseLinear's live slots (the "fused optimizer over
 * padded values" item of the reference's sparse-training path; the reference
 * itself runs torch's AdamW over the whole padded values tensor,
 * sparselab/nn.py:183-184).  One pass over W's slots: padding slots (col -1)
 * are skipped -- their value stays 0 and their moments untouched -- and each
 * live slot gets torch.optim.AdamW's update with decoupled weight decay:
 *   p *= 1 - lr*wd;  m = lerp(m, g, 1 - beta1);  v = beta2*v + (1-beta2)*g*g;
 *   p -= lr / (1 - beta1^step) * m / (sqrt(v) / sqrt(1 - beta2^step) + eps).
 * grad / exp_avg / exp_avg_sq are float[total_capacity] aligned with
 * W->values (updated in place); step >= 1 is the step being taken. */
SL_API int sl_adamw_live(const sl_csr* W, const float* grad, float* exp_avg, float* exp_avg_sq,
                  float lr, float beta1, float beta2, float eps, float weight_decay,
                  int64_t step, void* stream);

/* ── Data-parallel packing of live gradient slots ────────────────────────
 * packed_offsets[nrows] = exclusive scan of row_nnz.  pack copies the live
 * slots of src[total_capacity] into dst[nnz]; unpack scatters back into
 * dst[total_capacity] and, when scale != 1, multiplies by `scale`
 * (padding slots of dst are left as they are). */
SL_API int sl_pack_live(const sl_csr* W, const int32_t* packed_offsets,
                 const float* src, float* dst, void* stream);
SL_API int sl_unpack_live(const sl_csr* W, const int32_t* packed_offsets,
                   const float* src, float* dst, float scale, void* stream);
/* Batched pack / unpack of many layers' live gradient slots in one launch
 * (the per-layer calls above, fused; no reference counterpart).  `descs`
 * is a DEVICE array of n_descs descriptors; descriptor i owns launch blocks
 * [first_block_i, first_block_{i+1}) with first_block_0 = 0 and
 * ceil(nrows_i / 8) blocks each; n_blocks is the total.  pack copies
 * grad[row_start[r] + k] (k < row_nnz[r]) to
 * bucket[bucket_offset + packed_offsets[r] + k]; unpack copies back. */
typedef struct sl_live_desc {
    const int32_t* row_start;
    const int32_t* row_nnz;
    const int32_t* packed_offsets;
    float* grad;
    int64_t nrows;
    int64_t bucket_offset;
    int64_t first_block;
} sl_live_desc;
SL_API int sl_pack_live_batch(const sl_live_desc* descs, int64_t n_descs, int64_t n_blocks,
                       float* bucket, void* stream);
SL_API int sl_unpack_live_batch(const sl_live_desc* descs, int64_t n_descs, int64_t n_blocks,
                         const float* bucket, void* stream);
/* Exclusive scan of int32 counts (n <= 2^31 total) into out[n];
 * *total_dev (device int64) receives the sum. */
SL_API int sl_exclusive_scan(const int32_t* counts, int64_t n, int32_t* out,
                      int64_t* total_dev, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SPARSECORE_B200_H */
