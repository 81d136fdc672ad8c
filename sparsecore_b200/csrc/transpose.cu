// Padded-CSR transpose with slot permutation, bit-identical to the
// reference's sparselab/layout.py:460-536 (transpose_with_perm):
//   * output row k holds the source rows i that have column k, ascending
//     (the reference's stable argsort of the row-major entry stream),
//   * capacity max(1, ceil(nnz_k * (1 + padding_ratio))) in float64,
//     row_start = exclusive scan, padding (col -1, value 0, perm -1),
//   * perm[slot_T] = source slot in W.
//
// Deterministic GPU algorithm (no atomics on the output order):
//   1. count   - source rows are cut into blocks of kRowsPerBlock; each CTA
//                builds a shared-memory histogram of its block's columns and
//                writes it to scratch[b][k].
//   2. colscan - per column k, exclusive scan of scratch[.][k] over blocks
//                (the rank of block b's first entry inside output row k) and
//                the column total nnz_k.
//   3. capscan - capacities + exclusive scan -> row_start_T, total.
//   4. fill    - padding everywhere, then each CTA replays its rows in
//                ascending order: a row's columns are distinct, so every
//                thread can bump its own column's shared cursor without
//                contention; a barrier between rows keeps source-row order.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace slb {
namespace {

constexpr int kTrThreads = 256;
constexpr int kRowsPerBlock = 32;
constexpr int64_t kMaxSharedCols = 56 * 1024;  // int32 counters in shared memory

__global__ void __launch_bounds__(kTrThreads)
tr_count_kernel(int M, int K, const int32_t* __restrict__ row_start,
                const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                int32_t* __restrict__ counts) {
    extern __shared__ int hist[];
    for (int k = threadIdx.x; k < K; k += kTrThreads) hist[k] = 0;
    __syncthreads();
    const int r0 = blockIdx.x * kRowsPerBlock;
    const int r1 = min(M, r0 + kRowsPerBlock);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = r0 + warp; r < r1; r += kTrThreads / 32) {
        const int rs = row_start[r], nn = row_nnz[r];
        for (int s = lane; s < nn; s += 32) atomicAdd(&hist[cols[rs + s]], 1);
    }
    __syncthreads();
    int32_t* out = counts + static_cast<int64_t>(blockIdx.x) * K;
    for (int k = threadIdx.x; k < K; k += kTrThreads) out[k] = hist[k];
}

__global__ void __launch_bounds__(kTrThreads)
tr_colscan_kernel(int nb, int K, int32_t* __restrict__ counts, int32_t* __restrict__ col_nnz) {
    const int k = blockIdx.x * kTrThreads + threadIdx.x;
    if (k >= K) return;
    int run = 0;
    for (int b = 0; b < nb; ++b) {
        int32_t* p = counts + static_cast<int64_t>(b) * K + k;
        const int t = *p;
        *p = run;
        run += t;
    }
    col_nnz[k] = run;
}

__global__ void __launch_bounds__(kTrThreads)
tr_pad_kernel(int64_t n, float* __restrict__ vals, int32_t* __restrict__ cols,
              int64_t* __restrict__ perm) {
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kTrThreads + threadIdx.x; t < n;
         t += static_cast<int64_t>(gridDim.x) * kTrThreads) {
        vals[t] = 0.0f;
        cols[t] = -1;
        perm[t] = -1;
    }
}

__global__ void __launch_bounds__(kTrThreads)
tr_scatter_kernel(int M, int K, const int32_t* __restrict__ row_start,
                  const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                  const float* __restrict__ vals, const int32_t* __restrict__ offsets,
                  const int32_t* __restrict__ out_row_start, float* __restrict__ out_vals,
                  int32_t* __restrict__ out_cols, int64_t* __restrict__ perm) {
    extern __shared__ int cursor[];
    const int32_t* off = offsets + static_cast<int64_t>(blockIdx.x) * K;
    for (int k = threadIdx.x; k < K; k += kTrThreads) cursor[k] = out_row_start[k] + off[k];
    __syncthreads();
    const int r0 = blockIdx.x * kRowsPerBlock;
    const int r1 = min(M, r0 + kRowsPerBlock);
    for (int r = r0; r < r1; ++r) {
        const int rs = row_start[r], nn = row_nnz[r];
        for (int s = threadIdx.x; s < nn; s += kTrThreads) {
            const int slot = rs + s;
            const int c = cols[slot];
            const int dst = cursor[c];
            cursor[c] = dst + 1;
            out_vals[dst] = vals[slot];
            out_cols[dst] = r;
            perm[dst] = slot;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kTrThreads)
gather_kernel(const int64_t* __restrict__ perm, const float* __restrict__ src,
              float* __restrict__ dst, int64_t n) {
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * kTrThreads + threadIdx.x; t < n;
         t += static_cast<int64_t>(gridDim.x) * kTrThreads) {
        const int64_t p = perm[t];
        if (p >= 0) dst[t] = src[p];
    }
}

int grid_for(int64_t n) {
    int64_t b = (n + kTrThreads - 1) / kTrThreads;
    const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
    if (b > cap) b = cap;
    return static_cast<int>(b < 1 ? 1 : b);
}

int64_t n_blocks(int64_t M) { return (M + kRowsPerBlock - 1) / kRowsPerBlock; }

}  // namespace
}  // namespace slb

using namespace slb;

extern "C" {

int64_t sl_transpose_scratch_bytes(int64_t nrows, int64_t ncols) {
    const int64_t nb = n_blocks(nrows > 0 ? nrows : 1);
    return nb * (ncols > 0 ? ncols : 1) * static_cast<int64_t>(sizeof(int32_t));
}

int sl_transpose_count(const sl_csr* W, double one_plus_padding_ratio, int32_t* out_row_nnz,
                       int32_t* out_row_capacity, int32_t* out_row_start, int64_t* out_total_dev,
                       void* scratch, void* stream) {
    if (int rc = check_csr(W, "sl_transpose_count")) return rc;
    if (W->ncols > kMaxSharedCols)
        return fail(SL_ERR_UNSUPPORTED, "sl_transpose_count: ncols=" + std::to_string(W->ncols) +
                                            " exceeds the supported maximum of " +
                                            std::to_string(kMaxSharedCols));
    if (!(one_plus_padding_ratio >= 1.0))
        return fail(SL_ERR_INVALID, "sl_transpose_count: padding_ratio must be >= 0");
    SL_REQUIRE(W->ncols == 0 || (out_row_nnz != nullptr && out_row_capacity != nullptr &&
                                 out_row_start != nullptr),
               "sl_transpose_count", "NULL output row array");
    SL_REQUIRE(out_total_dev != nullptr, "sl_transpose_count", "NULL out_total_dev");
    SL_REQUIRE(W->nrows == 0 || W->ncols == 0 || scratch != nullptr, "sl_transpose_count",
               "NULL scratch");
    cudaStream_t s = as_stream(stream);
    const int M = static_cast<int>(W->nrows), K = static_cast<int>(W->ncols);
    if (K == 0) {
        return cuda_status(cudaMemsetAsync(out_total_dev, 0, sizeof(int64_t), s),
                           "sl_transpose_count memset");
    }
    int32_t* counts = static_cast<int32_t*>(scratch);
    const int nb = static_cast<int>(n_blocks(M));
    const size_t smem = sizeof(int) * static_cast<size_t>(K);
    if (smem > 48 * 1024) {
        cudaFuncSetAttribute(tr_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
        cudaFuncSetAttribute(tr_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    }
    if (M > 0) {
        tr_count_kernel<<<nb, kTrThreads, smem, s>>>(M, K, W->row_start, W->row_nnz,
                                                     W->col_indices, counts);
        SL_RETURN_IF_LAUNCH_FAILED("sl_transpose_count");
        tr_colscan_kernel<<<(K + kTrThreads - 1) / kTrThreads, kTrThreads, 0, s>>>(
            nb, K, counts, out_row_nnz);
        SL_RETURN_IF_LAUNCH_FAILED("sl_transpose_count");
    } else {
        if (int rc = cuda_status(cudaMemsetAsync(out_row_nnz, 0, sizeof(int32_t) * K, s),
                                 "sl_transpose_count memset"))
            return rc;
    }
    return sl_capacity_scan(out_row_nnz, K, one_plus_padding_ratio, out_row_capacity,
                            out_row_start, out_total_dev, stream);
}

int sl_transpose_fill(const sl_csr* W, const sl_csr* WT, int64_t* perm, const void* scratch,
                      void* stream) {
    if (int rc = check_csr(W, "sl_transpose_fill")) return rc;
    if (int rc = check_csr(WT, "sl_transpose_fill")) return rc;
    if (WT->nrows != W->ncols || WT->ncols != W->nrows)
        return fail(SL_ERR_INVALID, "sl_transpose_fill: WT shape must be W's swapped");
    if (W->ncols > kMaxSharedCols)
        return fail(SL_ERR_UNSUPPORTED, "sl_transpose_fill: ncols too large");
    SL_REQUIRE(WT->total_capacity == 0 || perm != nullptr, "sl_transpose_fill", "NULL perm");
    SL_REQUIRE(W->nrows == 0 || W->ncols == 0 || scratch != nullptr, "sl_transpose_fill",
               "NULL scratch");
    cudaStream_t s = as_stream(stream);
    const int M = static_cast<int>(W->nrows), K = static_cast<int>(W->ncols);
    const int64_t capT = WT->total_capacity;
    if (capT > 0) {
        tr_pad_kernel<<<grid_for(capT), kTrThreads, 0, s>>>(capT, WT->values, WT->col_indices,
                                                            perm);
        SL_RETURN_IF_LAUNCH_FAILED("sl_transpose_fill");
    }
    if (M == 0 || K == 0) return SL_OK;
    const size_t smem = sizeof(int) * static_cast<size_t>(K);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(tr_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    tr_scatter_kernel<<<static_cast<int>(n_blocks(M)), kTrThreads, smem, s>>>(
        M, K, W->row_start, W->row_nnz, W->col_indices, W->values,
        static_cast<const int32_t*>(scratch), WT->row_start, WT->values, WT->col_indices, perm);
    SL_RETURN_IF_LAUNCH_FAILED("sl_transpose_fill");
    return SL_OK;
}

int sl_values_gather(const int64_t* perm, const float* src, float* dst, int64_t n, void* stream) {
    if (n < 0) return fail(SL_ERR_INVALID, "sl_values_gather: negative n");
    if (n == 0) return SL_OK;
    SL_REQUIRE(perm != nullptr && src != nullptr && dst != nullptr, "sl_values_gather", "NULL array");
    gather_kernel<<<grid_for(n), kTrThreads, 0, as_stream(stream)>>>(perm, src, dst, n);
    SL_RETURN_IF_LAUNCH_FAILED("sl_values_gather");
    return SL_OK;
}

}  // extern "C"

// ── Transpose without any allocation ─────────────────────────────────────
// For callers that cannot call cudaMalloc (see the header): the per-block
// column histograms live in this file-scope device array instead of caller
// scratch.  Every GPU that loads the library holds it until the process
// exits.  Host code must not pass `g_noalloc_scratch` itself to a kernel:
// on the host that name is only a stand-in, so its device address is looked
// up once per device with cudaGetSymbolAddress and cached.
namespace slb {
namespace {

constexpr int64_t kNoAllocScratchInts = int64_t(1) << 20;  // 4 MiB per device
__device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocScratchInts];

// Device addresses of the array, one slot per device ordinal, in a fixed
// table: the lookup itself allocates nothing on the host either.
constexpr int kNoAllocMaxDevices = 64;
int32_t* g_noalloc_addr[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;

int noalloc_scratch(int32_t** out) {
    int dev = 0;
    if (int rc = cuda_status(cudaGetDevice(&dev), "sl_transpose_with_perm_noalloc")) return rc;
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(SL_ERR_UNSUPPORTED, "sl_transpose_with_perm_noalloc: device ordinal above 63");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr) {
        void* p = nullptr;
        if (int rc = cuda_status(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                                 "sl_transpose_with_perm_noalloc: cudaGetSymbolAddress"))
            return rc;
        g_noalloc_addr[dev] = static_cast<int32_t*>(p);
    }
    *out = g_noalloc_addr[dev];
    return SL_OK;
}

}  // namespace
}  // namespace slb

extern "C" int sl_transpose_with_perm_noalloc(const sl_csr* W, double one_plus_padding_ratio,
                                              const sl_csr* WT, int64_t* perm,
                                              int64_t* out_total_dev, void* stream) {
    const char* fn = "sl_transpose_with_perm_noalloc";
    if (int rc = check_csr(W, fn)) return rc;
    if (WT == nullptr || out_total_dev == nullptr)
        return fail(SL_ERR_INVALID, std::string(fn) + ": NULL WT or out_total_dev");
    if (WT->nrows != W->ncols || WT->ncols != W->nrows)
        return fail(SL_ERR_INVALID, std::string(fn) + ": WT shape must be W's swapped");
    if (!(one_plus_padding_ratio >= 1.0))
        return fail(SL_ERR_INVALID, std::string(fn) + ": padding_ratio must be >= 0");
    const int64_t need_ints = n_blocks(W->nrows > 0 ? W->nrows : 1) * (W->ncols > 0 ? W->ncols : 1);
    if (need_ints > kNoAllocScratchInts)
        return fail(SL_ERR_UNSUPPORTED,
                    std::string(fn) + ": ceil(nrows/32) * ncols = " + std::to_string(need_ints) +
                        " exceeds the static scratch of " + std::to_string(kNoAllocScratchInts) +
                        " int32 counters; use sl_transpose_count/sl_transpose_fill with "
                        "caller-allocated scratch");
    // Upper bound of the transpose's total capacity: sum_k max(1, ceil(n_k * r))
    // < r * nnz + ncols + 1 <= r * total_capacity + ncols + 1.
    const int64_t bound = static_cast<int64_t>(
                              std::floor(one_plus_padding_ratio * static_cast<double>(W->total_capacity))) +
                          W->ncols + 2;
    if (WT->total_capacity < bound)
        return fail(SL_ERR_INVALID,
                    std::string(fn) + ": WT slot arrays hold " + std::to_string(WT->total_capacity) +
                        " entries; at least floor((1+padding_ratio)*total_capacity) + ncols + 2 = " +
                        std::to_string(bound) + " are required");
    if (WT->total_capacity > 0 && perm == nullptr)
        return fail(SL_ERR_INVALID, std::string(fn) + ": NULL perm");
    int32_t* scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    if (int rc = sl_transpose_count(W, one_plus_padding_ratio, WT->row_nnz, WT->row_capacity,
                                    WT->row_start, out_total_dev, scratch, stream))
        return rc;
    return sl_transpose_fill(W, WT, perm, scratch, stream);
}
