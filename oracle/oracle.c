/*
 * CPU oracle for the padded-CSR sparse-training hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file restates, in plain C, the arithmetic
 * of the reference project's CPU kernels so that the CUDA kernels of
 * sparsecore_b200 can be checked against it.  Nothing in the product path
 * links or calls this code; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py load it (as liboracle.so, via ctypes).
 *
 * Compiled with -ffp-contract=off: every fused multiply-add below is an
 * explicit fmaf(), every plain add/multiply is a separately rounded IEEE op,
 * so the rounding sequence is exactly the one written here.
 *
 * Parity pinned against the reference's own compiled `_core` (built from the
 * reference sources by oracle/Makefile) through tests/golden/ fixtures.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Row capacity: max(1, ceil(nnz * (1 + padding_ratio))) evaluated in
 * float64, as sparselab/layout.py:46-68 (_compute_row_capacity) does with
 * numpy.  `one_plus_pr` is the already-rounded double (1.0 + padding_ratio). */
void or_capacity(const int32_t* row_nnz, int64_t n, double one_plus_pr,
                 int32_t* cap_out) {
    for (int64_t i = 0; i < n; ++i) {
        double scaled = ceil((double)row_nnz[i] * one_plus_pr);
        if (scaled < 1.0) scaled = 1.0;
        cap_out[i] = (int32_t)scaled;
    }
}

/* Forward SpMM Y[M,N] = W[M,K] . X[K,N].
 * Follows csrc/kernels/spmm_avx2.cpp:82-263 (spmm_simd_avx2): Y is zeroed,
 * then for each live slot s of row i in slot order and every column j,
 * y[i,j] = fma(v_s, X[c_s, j], y[i,j]).  The 16-wide / 8-wide / scalar
 * stages of the AVX2 code all perform that same per-element fused update,
 * so each output element is one FMA chain in slot order. */
void or_spmm(int64_t M, int64_t N,
             const int32_t* row_start, const int32_t* row_nnz,
             const int32_t* cols, const float* vals,
             const float* X, float* Y) {
    memset(Y, 0, sizeof(float) * (size_t)M * (size_t)N);
    for (int64_t i = 0; i < M; ++i) {
        float* y = Y + i * N;
        for (int32_t s = 0; s < row_nnz[i]; ++s) {
            const int32_t slot = row_start[i] + s;
            const float v = vals[slot];
            const float* x = X + (int64_t)cols[slot] * N;
            for (int64_t j = 0; j < N; ++j) y[j] = fmaf(v, x[j], y[j]);
        }
    }
}

/* Sequential accumulation r += a[j]*b[j] for j in [j0, N) as the reference's
 * x86-64-v3 build executes its plain scalar loops (GCC vectorises them as an
 * in-order reduction; there is no -ffast-math): whole groups of 4 terms are
 * multiplied (one rounding) and then added one by one in j order; the last
 * (N - j0) mod 4 terms run as the scalar epilogue, contracted to FMA.
 * (Groups of 8 behave the same as two groups of 4.)  Pinned bit-exactly
 * against the reference's spmm_grad_w_simd tail and dense_grad outputs. */
static float gcc_vec_tail(const float* a, const float* b, int64_t j0, int64_t N,
                          float r) {
    const int64_t vec_end = j0 + ((N - j0) / 4) * 4;
    int64_t j = j0;
    for (; j < vec_end; ++j) {
        const float p = a[j] * b[j];
        r = r + p;
    }
    for (; j < N; ++j) r = fmaf(a[j], b[j], r);
    return r;
}

/* One dot product in the lane order of csrc/kernels/spmm_grad_avx2.cpp:
 * 112-257: two 8-lane FMA accumulators over 16-float steps (lane l of the
 * first takes j = 16m + l, of the second j = 16m + 8 + l), their lane-wise
 * sum, one optional 8-wide FMA step, the 3-step horizontal reduction
 * (l+h per quarter, then pairs (0,2),(1,3), then the two halves), then the
 * scalar loop over the remaining N mod 8 elements in its compiled order
 * (gcc_vec_tail). */
static float avx2_order_dot(const float* a, const float* b, int64_t N) {
    float acc_a[8] = {0}, acc_b[8] = {0}, acc[8];
    int64_t j = 0;
    for (; j + 16 <= N; j += 16) {
        for (int l = 0; l < 8; ++l) {
            acc_a[l] = fmaf(a[j + l], b[j + l], acc_a[l]);
            acc_b[l] = fmaf(a[j + 8 + l], b[j + 8 + l], acc_b[l]);
        }
    }
    for (int l = 0; l < 8; ++l) acc[l] = acc_a[l] + acc_b[l];
    if (j + 8 <= N) {
        for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[j + l], b[j + l], acc[l]);
        j += 8;
    }
    float s4[4];
    for (int q = 0; q < 4; ++q) s4[q] = acc[q] + acc[q + 4];
    const float s2a = s4[0] + s4[2];
    const float s2b = s4[1] + s4[3];
    float r = s2a + s2b;
    return gcc_vec_tail(a, b, j, N, r);
}

/* SDDMM weight gradient at live slots (spmm_grad_w_simd,
 * csrc/kernels/spmm_grad_avx2.cpp:73-259): dW[slot] = <dY[i,:], X[c,:]>
 * for live slots, 0 for padding; output length = total capacity. */
void or_sddmm(int64_t M, int64_t N, int64_t cap,
              const int32_t* row_start, const int32_t* row_nnz,
              const int32_t* cols, const float* dY, const float* X,
              float* dW) {
    memset(dW, 0, sizeof(float) * (size_t)cap);
    for (int64_t i = 0; i < M; ++i) {
        for (int32_t s = 0; s < row_nnz[i]; ++s) {
            const int32_t slot = row_start[i] + s;
            dW[slot] = avx2_order_dot(dY + i * N,
                                      X + (int64_t)cols[slot] * N, N);
        }
    }
}

/* Scalar-kernel dot (csrc/kernels/spmm_grad.cpp:308-388, spmm_grad_w) in
 * its compiled order (gcc_vec_tail); kept for cross-checking. */
void or_sddmm_sequential(int64_t M, int64_t N, int64_t cap,
                         const int32_t* row_start, const int32_t* row_nnz,
                         const int32_t* cols, const float* dY,
                         const float* X, float* dW) {
    memset(dW, 0, sizeof(float) * (size_t)cap);
    for (int64_t i = 0; i < M; ++i) {
        for (int32_t s = 0; s < row_nnz[i]; ++s) {
            const int32_t slot = row_start[i] + s;
            const float* a = dY + i * N;
            const float* b = X + (int64_t)cols[slot] * N;
            dW[slot] = gcc_vec_tail(a, b, 0, N, 0.0f);
        }
    }
}

/* Dense gradient G[M,K] = dY[M,N] . X[K,N]^T for RigL
 * (csrc/kernels/dense_grad.cpp:463-523).  mode 0: the reference's compiled
 * order for its scalar loop (gcc_vec_tail over the whole row); mode 1: the
 * AVX2 lane order above. */
void or_dense_grad(int64_t M, int64_t K, int64_t N, const float* dY,
                   const float* X, float* G, int mode) {
    for (int64_t i = 0; i < M; ++i) {
        for (int64_t k = 0; k < K; ++k) {
            const float* a = dY + i * N;
            const float* b = X + k * N;
            float r;
            if (mode == 1) {
                r = avx2_order_dot(a, b, N);
            } else {
                r = gcc_vec_tail(a, b, 0, N, 0.0f);
            }
            G[i * K + k] = r;
        }
    }
}

/* Transpose with permutation (sparselab/layout.py:460-536,
 * transpose_with_perm).  Output row k lists the source rows i that hold
 * column k, ascending (the stable argsort of the row-major entry stream by
 * column).  Capacities per or_capacity; padding col -1 / value 0 / perm -1.
 * Pass 1 (count) fills out_row_nnz/out_row_capacity/out_row_start and
 * returns the total capacity; pass 2 (fill, out arrays sized by that total)
 * scatters. */
int64_t or_transpose_count(int64_t M, int64_t K, const int32_t* row_start,
                           const int32_t* row_nnz, const int32_t* cols,
                           double one_plus_pr, int32_t* out_row_nnz,
                           int32_t* out_row_capacity, int32_t* out_row_start) {
    memset(out_row_nnz, 0, sizeof(int32_t) * (size_t)K);
    for (int64_t i = 0; i < M; ++i)
        for (int32_t s = 0; s < row_nnz[i]; ++s)
            out_row_nnz[cols[row_start[i] + s]]++;
    or_capacity(out_row_nnz, K, one_plus_pr, out_row_capacity);
    int64_t total = 0;
    for (int64_t k = 0; k < K; ++k) {
        out_row_start[k] = (int32_t)total;
        total += out_row_capacity[k];
    }
    return total;
}

void or_transpose_fill(int64_t M, int64_t K, const int32_t* row_start,
                       const int32_t* row_nnz, const int32_t* cols,
                       const float* vals, const int32_t* out_row_start,
                       int64_t out_cap, float* out_vals, int32_t* out_cols,
                       int64_t* perm) {
    for (int64_t t = 0; t < out_cap; ++t) {
        out_vals[t] = 0.0f;
        out_cols[t] = -1;
        perm[t] = -1;
    }
    int32_t* cursor = (int32_t*)malloc(sizeof(int32_t) * (size_t)(K > 0 ? K : 1));
    for (int64_t k = 0; k < K; ++k) cursor[k] = out_row_start[k];
    for (int64_t i = 0; i < M; ++i) {
        for (int32_t s = 0; s < row_nnz[i]; ++s) {
            const int32_t slot = row_start[i] + s;
            const int32_t dst = cursor[cols[slot]]++;
            out_vals[dst] = vals[slot];
            out_cols[dst] = (int32_t)i;
            perm[dst] = slot;
        }
    }
    free(cursor);
}

/* Invariant check (csrc/kernels/padded_csr.cpp:79-196,
 * check_invariants_str), in the same order.  Returns 0 when all hold, else
 * the invariant code of the first violation (1 shape, 2 lengths, 3
 * row_start, 4 nnz range, 6 live columns, 7 padding column) and the row in
 * *where_row, the slot offset in *where_slot. */
int or_check_invariants(int64_t nrows, int64_t ncols, int64_t n_slots,
                        const int32_t* row_start, const int32_t* row_nnz,
                        const int32_t* row_capacity, const int32_t* cols,
                        int64_t* where_row, int64_t* where_slot) {
    *where_row = -1;
    *where_slot = -1;
    if (nrows < 0 || ncols < 0) return 1;
    int64_t total = 0;
    for (int64_t i = 0; i < nrows; ++i) total += row_capacity[i];
    if (total != n_slots) return 2;
    if (nrows > 0 && row_start[0] != 0) { *where_row = 0; return 3; }
    for (int64_t i = 1; i < nrows; ++i)
        if (row_start[i] != row_start[i - 1] + row_capacity[i - 1]) {
            *where_row = i;
            return 3;
        }
    for (int64_t i = 0; i < nrows; ++i)
        if (row_nnz[i] < 0 || row_nnz[i] > row_capacity[i]) {
            *where_row = i;
            return 4;
        }
    for (int64_t i = 0; i < nrows; ++i) {
        int32_t prev = -1;
        for (int32_t k = 0; k < row_nnz[i]; ++k) {
            const int32_t c = cols[row_start[i] + k];
            if (c < 0 || c >= ncols || c <= prev) {
                *where_row = i;
                *where_slot = k;
                return 6;
            }
            prev = c;
        }
        for (int32_t k = row_nnz[i]; k < row_capacity[i]; ++k)
            if (cols[row_start[i] + k] != -1) {
                *where_row = i;
                *where_slot = k;
                return 7;
            }
    }
    return 0;
}
