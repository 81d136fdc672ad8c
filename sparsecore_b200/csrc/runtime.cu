// Library plumbing: error reporting, device properties, generic scans and
// the live-slot pack/unpack used by data-parallel gradient exchange.
#include <mutex>
#include <vector>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "tma.cuh"

namespace slb {

thread_local std::string g_last_error;
thread_local const char* g_last_kernel = "";

void set_error(const std::string& msg) { g_last_error = msg; }
void note_kernel(const char* name) { g_last_kernel = name; }

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return SL_OK;
    return fail(SL_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int num_sms() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= static_cast<int>(cache.size())) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int check_csr(const sl_csr* W, const char* fn) {
    if (W == nullptr) return fail(SL_ERR_INVALID, std::string(fn) + ": W is NULL");
    if (W->nrows < 0 || W->ncols < 0)
        return fail(SL_ERR_INVALID, std::string(fn) + ": negative shape");
    if (W->nrows > INT_MAX || W->ncols > INT_MAX || W->total_capacity > INT_MAX)
        return fail(SL_ERR_UNSUPPORTED,
                    std::string(fn) + ": sizes beyond int32 indexing are not supported");
    if (W->nrows > 0 && (W->row_start == nullptr || W->row_nnz == nullptr ||
                         W->row_capacity == nullptr))
        return fail(SL_ERR_INVALID, std::string(fn) + ": NULL row array");
    if (W->total_capacity > 0 && (W->values == nullptr || W->col_indices == nullptr))
        return fail(SL_ERR_INVALID, std::string(fn) + ": NULL slot array");
    return SL_OK;
}

// ── single-CTA exclusive scan over an int32 array (n up to a few million) ──
constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kScanThreads)
exclusive_scan_kernel(const int32_t* __restrict__ in, int64_t n, int32_t* __restrict__ out,
                      int64_t* __restrict__ total) {
    __shared__ int ws[kScanThreads / 32];
    int64_t carry = 0;
    for (int64_t base = 0; base < n; base += kScanThreads) {
        const int64_t idx = base + threadIdx.x;
        const int v = idx < n ? in[idx] : 0;
        int tot;
        const int ex = block_exclusive_scan<kScanThreads>(v, ws, &tot);
        if (idx < n) out[idx] = static_cast<int32_t>(carry + ex);
        carry += tot;
    }
    if (threadIdx.x == 0 && total) *total = carry;
}

// Capacity max(1, ceil(nnz * one_plus_pr)) in float64 (IEEE multiply and
// ceil, same rounding as numpy in the reference), then exclusive scan.
__global__ void __launch_bounds__(kScanThreads)
capacity_scan_kernel(const int32_t* __restrict__ nnz, int64_t n, double one_plus_pr,
                     int32_t* __restrict__ cap, int32_t* __restrict__ start,
                     int64_t* __restrict__ total) {
    __shared__ int ws[kScanThreads / 32];
    int64_t carry = 0;
    for (int64_t base = 0; base < n; base += kScanThreads) {
        const int64_t idx = base + threadIdx.x;
        int c = 0;
        if (idx < n) {
            double s = ceil(__dmul_rn(static_cast<double>(nnz[idx]), one_plus_pr));
            if (s < 1.0) s = 1.0;
            c = static_cast<int>(s);
            cap[idx] = c;
        }
        int tot;
        const int ex = block_exclusive_scan<kScanThreads>(c, ws, &tot);
        if (idx < n) start[idx] = static_cast<int32_t>(carry + ex);
        carry += tot;
    }
    if (threadIdx.x == 0 && total) *total = carry;
}

// ── live-slot pack / unpack (warp per row) ──
__global__ void __launch_bounds__(256)
pack_live_kernel(int M, const int32_t* __restrict__ row_start, const int32_t* __restrict__ row_nnz,
                 const int32_t* __restrict__ off, const float* __restrict__ src,
                 float* __restrict__ dst) {
    const int warps = gridDim.x * 8;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < M; row += warps) {
        const int rs = row_start[row], nn = row_nnz[row], o = off[row];
        for (int k = threadIdx.x & 31; k < nn; k += 32) dst[o + k] = src[rs + k];
    }
}

__global__ void __launch_bounds__(256)
unpack_live_kernel(int M, const int32_t* __restrict__ row_start,
                   const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ off,
                   const float* __restrict__ src, float* __restrict__ dst, float scale) {
    const int warps = gridDim.x * 8;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < M; row += warps) {
        const int rs = row_start[row], nn = row_nnz[row], o = off[row];
        for (int k = threadIdx.x & 31; k < nn; k += 32) {
            const float v = src[o + k];
            dst[rs + k] = scale == 1.0f ? v : __fmul_rn(v, scale);
        }
    }
}

// Batched form: descriptor d covers blocks [d.first_block, next first
// block); each block of 8 warps takes 8 rows of its layer.
__device__ __forceinline__ int find_desc(const sl_live_desc* __restrict__ d, int64_t n, int64_t blk) {
    int lo = 0, hi = static_cast<int>(n);
    while (hi - lo > 1) {  // last descriptor whose first_block <= blk
        const int mid = (lo + hi) >> 1;
        if (d[mid].first_block <= blk) lo = mid; else hi = mid;
    }
    return lo;
}

template <bool PACK>
__global__ void __launch_bounds__(256)
live_batch_kernel(const sl_live_desc* __restrict__ descs, int64_t n, float* __restrict__ bucket) {
    const sl_live_desc& d = descs[find_desc(descs, n, blockIdx.x)];
    const int64_t row = (static_cast<int64_t>(blockIdx.x) - d.first_block) * 8 + (threadIdx.x >> 5);
    if (row >= d.nrows) return;
    const int rs = d.row_start[row], nn = d.row_nnz[row];
    float* b = bucket + d.bucket_offset + d.packed_offsets[row];
    for (int k = threadIdx.x & 31; k < nn; k += 32) {
        if (PACK) b[k] = d.grad[rs + k];
        else d.grad[rs + k] = b[k];
    }
}

bool make_tmap_2d(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int box_rows,
                  int box_cols, bool swizzle128) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (encode == nullptr || !aligned16(base) || (cols * 4) % 16 != 0) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * sizeof(float)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

unsigned* device_status_word() {
    static std::mutex mu;
    static std::vector<unsigned*> words;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= static_cast<int>(words.size())) words.resize(dev + 1, nullptr);
    if (words[dev] == nullptr) {
        void* p = nullptr;
        if (cudaMalloc(&p, sizeof(unsigned)) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, sizeof(unsigned));
        words[dev] = static_cast<unsigned*>(p);
    }
    return words[dev];
}

// Self-test of the bounded waits: one thread waits on an mbarrier that no
// arrival will ever complete; after `spins` polls the wait gives up, raises
// the status word and the kernel returns.
__global__ void bounded_wait_selftest_kernel(unsigned* status, long long spins) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        mbar_wait(&bar, 0u, status, spins);  // phase 0 never completes: times out
    }
}

int row_grid(int64_t M) {
    const int64_t want = (M + 7) / 8;
    const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
    return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace slb

using namespace slb;

extern "C" {

const char* sl_last_error(void) { return slb::g_last_error.c_str(); }

const char* sl_last_kernel(void) { return slb::g_last_kernel; }

const char* sl_version(void) { return "sparsecore_b200 0.1.0 (sm_100a)"; }

int sl_device_status(int reset, unsigned* out) {
    unsigned* w = device_status_word();
    if (w == nullptr) return fail(SL_ERR_CUDA, "sl_device_status: no device status word");
    unsigned v = 0;
    if (int rc = cuda_status(cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost),
                             "sl_device_status"))
        return rc;
    if (reset && v)
        if (int rc = cuda_status(cudaMemset(w, 0, sizeof(unsigned)), "sl_device_status")) return rc;
    if (out) *out = v;
    return SL_OK;
}

int sl_selftest_bounded_wait(int64_t spins, void* stream) {
    if (spins < 1 || spins > (int64_t(1) << 24))
        return fail(SL_ERR_INVALID, "sl_selftest_bounded_wait: spins must be in [1, 2^24]");
    unsigned* w = device_status_word();
    if (w == nullptr) return fail(SL_ERR_CUDA, "sl_selftest_bounded_wait: no device status word");
    bounded_wait_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>(w, spins);
    SL_RETURN_IF_LAUNCH_FAILED("sl_selftest_bounded_wait");
    return SL_OK;
}

int sl_exclusive_scan(const int32_t* counts, int64_t n, int32_t* out, int64_t* total_dev,
                      void* stream) {
    if (n < 0) return fail(SL_ERR_INVALID, "sl_exclusive_scan: negative n");
    SL_REQUIRE(n == 0 || (counts != nullptr && out != nullptr), "sl_exclusive_scan", "NULL array");
    exclusive_scan_kernel<<<1, kScanThreads, 0, as_stream(stream)>>>(counts, n, out, total_dev);
    SL_RETURN_IF_LAUNCH_FAILED("sl_exclusive_scan");
    return SL_OK;
}

int sl_capacity_scan(const int32_t* row_nnz, int64_t n, double one_plus_padding_ratio,
                     int32_t* row_capacity, int32_t* row_start, int64_t* out_total_dev,
                     void* stream) {
    if (n < 0) return fail(SL_ERR_INVALID, "sl_capacity_scan: negative n");
    if (!(one_plus_padding_ratio >= 1.0))
        return fail(SL_ERR_INVALID, "sl_capacity_scan: padding_ratio must be >= 0");
    SL_REQUIRE(n == 0 || (row_nnz != nullptr && row_capacity != nullptr && row_start != nullptr),
               "sl_capacity_scan", "NULL row array");
    SL_REQUIRE(out_total_dev != nullptr, "sl_capacity_scan", "NULL out_total_dev");
    capacity_scan_kernel<<<1, kScanThreads, 0, as_stream(stream)>>>(
        row_nnz, n, one_plus_padding_ratio, row_capacity, row_start, out_total_dev);
    SL_RETURN_IF_LAUNCH_FAILED("sl_capacity_scan");
    return SL_OK;
}

int sl_pack_live(const sl_csr* W, const int32_t* packed_offsets, const float* src, float* dst,
                 void* stream) {
    if (int rc = check_csr(W, "sl_pack_live")) return rc;
    if (W->nrows == 0) return SL_OK;
    SL_REQUIRE(packed_offsets != nullptr && src != nullptr && dst != nullptr, "sl_pack_live",
               "NULL array");
    pack_live_kernel<<<row_grid(W->nrows), 256, 0, as_stream(stream)>>>(
        static_cast<int>(W->nrows), W->row_start, W->row_nnz, packed_offsets, src, dst);
    SL_RETURN_IF_LAUNCH_FAILED("sl_pack_live");
    return SL_OK;
}

int sl_unpack_live(const sl_csr* W, const int32_t* packed_offsets, const float* src, float* dst,
                   float scale, void* stream) {
    if (int rc = check_csr(W, "sl_unpack_live")) return rc;
    if (W->nrows == 0) return SL_OK;
    SL_REQUIRE(packed_offsets != nullptr && src != nullptr && dst != nullptr, "sl_unpack_live",
               "NULL array");
    unpack_live_kernel<<<row_grid(W->nrows), 256, 0, as_stream(stream)>>>(
        static_cast<int>(W->nrows), W->row_start, W->row_nnz, packed_offsets, src, dst, scale);
    SL_RETURN_IF_LAUNCH_FAILED("sl_unpack_live");
    return SL_OK;
}

static int live_batch(const sl_live_desc* descs, int64_t n, int64_t n_blocks, float* bucket,
                      void* stream, bool pack, const char* fn) {
    if (n < 0 || n_blocks < 0) return fail(SL_ERR_INVALID, std::string(fn) + ": negative count");
    if (n == 0 || n_blocks == 0) return SL_OK;
    SL_REQUIRE(descs != nullptr && bucket != nullptr, fn, "NULL descriptors or bucket");
    if (n_blocks > INT_MAX) return fail(SL_ERR_UNSUPPORTED, std::string(fn) + ": too many blocks");
    if (pack)
        live_batch_kernel<true><<<static_cast<unsigned>(n_blocks), 256, 0, as_stream(stream)>>>(descs, n, bucket);
    else
        live_batch_kernel<false><<<static_cast<unsigned>(n_blocks), 256, 0, as_stream(stream)>>>(descs, n, bucket);
    SL_RETURN_IF_LAUNCH_FAILED(fn);
    return SL_OK;
}

int sl_pack_live_batch(const sl_live_desc* descs, int64_t n_descs, int64_t n_blocks, float* bucket,
                       void* stream) {
    return live_batch(descs, n_descs, n_blocks, bucket, stream, true, "sl_pack_live_batch");
}

int sl_unpack_live_batch(const sl_live_desc* descs, int64_t n_descs, int64_t n_blocks,
                         const float* bucket, void* stream) {
    return live_batch(descs, n_descs, n_blocks, const_cast<float*>(bucket), stream, false,
                      "sl_unpack_live_batch");
}

}  // extern "C"
