// Layout factories and checks: dense -> padded CSR, padded CSR -> dense,
// and the invariant checker.
//   sparselab/layout.py:75-208  (from_torch_sparse_csr / from_dense)
//   sparselab/layout.py:262-292 (to_dense)
//   csrc/kernels/padded_csr.cpp:79-196 (check_invariants_str)
#include "common.cuh"

namespace slb {
namespace {

__device__ __forceinline__ bool is_live(float w, float thr) {
    return thr > 0.0f ? fabsf(w) > thr : w != 0.0f;
}

// Warp per row: live count.
__global__ void __launch_bounds__(256)
dense_count_kernel(const float* __restrict__ D, int M, int64_t K, float thr,
                   int32_t* __restrict__ row_nnz) {
    const int warps = gridDim.x * 8;
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < M; row += warps) {
        const float* d = D + static_cast<int64_t>(row) * K;
        int c = 0;
        for (int64_t k = lane; k < K; k += 32) c += is_live(d[k], thr) ? 1 : 0;
        c = warp_sum(c);
        if (lane == 0) row_nnz[row] = c;
    }
}

// Warp per row: ballot compaction in column order, then padding.
__global__ void __launch_bounds__(256)
dense_fill_kernel(const float* __restrict__ D, int M, int64_t K, float thr,
                  const int32_t* __restrict__ row_start, const int32_t* __restrict__ row_capacity,
                  float* __restrict__ vals, int32_t* __restrict__ cols) {
    const int warps = gridDim.x * 8;
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < M; row += warps) {
        const float* d = D + static_cast<int64_t>(row) * K;
        const int rs = row_start[row], cap = row_capacity[row];
        int base = 0;
        for (int64_t k0 = 0; k0 < K; k0 += 32) {
            const int64_t k = k0 + lane;
            const float w = k < K ? d[k] : 0.0f;
            const bool live = k < K && is_live(w, thr);
            const unsigned m = __ballot_sync(0xffffffffu, live);
            if (live) {
                const int p = base + __popc(m & ((1u << lane) - 1u));
                vals[rs + p] = w;
                cols[rs + p] = static_cast<int32_t>(k);
            }
            base += __popc(m);
        }
        for (int p = base + lane; p < cap; p += 32) {
            vals[rs + p] = 0.0f;
            cols[rs + p] = -1;
        }
    }
}

__global__ void __launch_bounds__(256)
to_dense_kernel(int M, int64_t K, const int32_t* __restrict__ row_start,
                const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                const float* __restrict__ vals, float* __restrict__ D) {
    const int warps = gridDim.x * 8;
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < M; row += warps) {
        const int rs = row_start[row], nn = row_nnz[row];
        float* d = D + static_cast<int64_t>(row) * K;
        for (int s = lane; s < nn; s += 32) d[cols[rs + s]] = vals[rs + s];
    }
}

constexpr long long kNone = 0x7f7f7f7f7f7f7f7fLL;  // memset(0x7f) sentinel

// Warp per row.  mins[0] = first row violating invariant 3 (row_start chain),
// mins[1] = first row violating invariant 4, mins[2] = first (row << 32 |
// slot) with a bad column (live: out of range / not strictly ascending;
// padding: != -1).  Every access is bounds-checked against n_slots.
__global__ void __launch_bounds__(256)
check_kernel(int M, int K, int64_t n_slots, const int32_t* __restrict__ row_start,
             const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ row_capacity,
             const int32_t* __restrict__ cols, long long* __restrict__ mins) {
    const int warps = gridDim.x * 8;
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < M; row += warps) {
        const int rs = row_start[row], nn = row_nnz[row], cap = row_capacity[row];
        if (lane == 0) {
            const long long expect =
                row == 0 ? 0LL
                         : static_cast<long long>(row_start[row - 1]) + row_capacity[row - 1];
            if (static_cast<long long>(rs) != expect) atomicMin(&mins[0], static_cast<long long>(row));
            if (nn < 0 || nn > cap) atomicMin(&mins[1], static_cast<long long>(row));
        }
        if (rs < 0 || cap < 0 || static_cast<int64_t>(rs) + cap > n_slots || nn < 0 || nn > cap)
            continue;  // reported above (or by the length check on the host)
        long long first = kNone;
        for (int k0 = 0; k0 < cap && first == kNone; k0 += 32) {
            const int k = k0 + lane;
            bool bad = false;
            if (k < cap) {
                const int c = cols[rs + k];
                if (k < nn) {
                    const int prev = k > 0 ? cols[rs + k - 1] : -1;
                    bad = c < 0 || c >= K || c <= prev;
                } else {
                    bad = c != -1;
                }
            }
            const unsigned m = __ballot_sync(0xffffffffu, bad);
            if (m) first = (static_cast<long long>(row) << 32) | (k0 + __ffs(m) - 1);
        }
        if (lane == 0 && first != kNone) atomicMin(&mins[2], first);
    }
}

// Resolve the first violation in the reference's check order.
__global__ void check_finalize_kernel(const int32_t* __restrict__ row_nnz, long long* rep) {
    const long long r3 = rep[0], r4 = rep[1], r67 = rep[2];
    long long code = 0, row = -1, slot = -1;
    if (r3 != kNone) {
        code = 3;
        row = r3;
    } else if (r4 != kNone) {
        code = 4;
        row = r4;
    } else if (r67 != kNone) {
        row = r67 >> 32;
        slot = r67 & 0xffffffffLL;
        code = slot < row_nnz[row] ? 6 : 7;
    }
    rep[0] = code;
    rep[1] = row;
    rep[2] = slot;
    rep[3] = 0;
}

}  // namespace
}  // namespace slb

using namespace slb;

extern "C" {

int sl_dense_count(const float* dense, int64_t M, int64_t K, float threshold,
                   double one_plus_padding_ratio, int32_t* row_nnz, int32_t* row_capacity,
                   int32_t* row_start, int64_t* out_total_dev, void* stream) {
    if (M < 0 || K < 0) return fail(SL_ERR_INVALID, "sl_dense_count: negative shape");
    if (M > INT_MAX || K > INT_MAX)
        return fail(SL_ERR_UNSUPPORTED, "sl_dense_count: shape beyond int32");
    SL_REQUIRE(M == 0 || K == 0 || dense != nullptr, "sl_dense_count", "NULL dense input");
    SL_REQUIRE(M == 0 || (row_nnz != nullptr && row_capacity != nullptr && row_start != nullptr),
               "sl_dense_count", "NULL row array");
    SL_REQUIRE(out_total_dev != nullptr, "sl_dense_count", "NULL out_total_dev");
    cudaStream_t s = as_stream(stream);
    if (M > 0) {
        dense_count_kernel<<<row_grid(M), 256, 0, s>>>(dense, static_cast<int>(M), K, threshold,
                                                       row_nnz);
        SL_RETURN_IF_LAUNCH_FAILED("sl_dense_count");
    }
    return sl_capacity_scan(row_nnz, M, one_plus_padding_ratio, row_capacity, row_start,
                            out_total_dev, stream);
}

int sl_dense_fill(const float* dense, float threshold, const sl_csr* out, void* stream) {
    if (int rc = check_csr(out, "sl_dense_fill")) return rc;
    if (out->nrows == 0) return SL_OK;
    SL_REQUIRE(out->ncols == 0 || dense != nullptr, "sl_dense_fill", "NULL dense input");
    dense_fill_kernel<<<row_grid(out->nrows), 256, 0, as_stream(stream)>>>(
        dense, static_cast<int>(out->nrows), out->ncols, threshold, out->row_start,
        out->row_capacity, out->values, out->col_indices);
    SL_RETURN_IF_LAUNCH_FAILED("sl_dense_fill");
    return SL_OK;
}

int sl_to_dense(const sl_csr* W, float* dense, void* stream) {
    if (int rc = check_csr(W, "sl_to_dense")) return rc;
    cudaStream_t s = as_stream(stream);
    const size_t bytes = sizeof(float) * static_cast<size_t>(W->nrows) * W->ncols;
    if (bytes == 0) return SL_OK;
    SL_REQUIRE(dense != nullptr, "sl_to_dense", "NULL output");
    if (int rc = cuda_status(cudaMemsetAsync(dense, 0, bytes, s), "sl_to_dense memset")) return rc;
    to_dense_kernel<<<row_grid(W->nrows), 256, 0, s>>>(static_cast<int>(W->nrows), W->ncols,
                                                       W->row_start, W->row_nnz, W->col_indices,
                                                       W->values, dense);
    SL_RETURN_IF_LAUNCH_FAILED("sl_to_dense");
    return SL_OK;
}

int sl_check_invariants(const sl_csr* W, int64_t n_slots, int64_t* report, void* stream) {
    if (int rc = check_csr(W, "sl_check_invariants")) return rc;
    SL_REQUIRE(report != nullptr, "sl_check_invariants", "NULL report");
    cudaStream_t s = as_stream(stream);
    if (int rc = cuda_status(cudaMemsetAsync(report, 0x7f, 4 * sizeof(int64_t), s),
                             "sl_check_invariants memset"))
        return rc;
    long long* rep = reinterpret_cast<long long*>(report);
    if (W->nrows > 0) {
        check_kernel<<<row_grid(W->nrows), 256, 0, s>>>(static_cast<int>(W->nrows),
                                                        static_cast<int>(W->ncols), n_slots,
                                                        W->row_start, W->row_nnz,
                                                        W->row_capacity, W->col_indices, rep);
        SL_RETURN_IF_LAUNCH_FAILED("sl_check_invariants");
    }
    check_finalize_kernel<<<1, 1, 0, s>>>(W->row_nnz, rep);
    SL_RETURN_IF_LAUNCH_FAILED("sl_check_invariants");
    return SL_OK;
}

}  // extern "C"
