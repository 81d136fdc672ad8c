// Forward SpMM with one dense column (SpMV, also dX = W^T . dY at N = 1):
//   Y[i] = fma chain over row i's live slots in slot order, from +0
// (bit-identical to the reference's csrc/kernels/spmm_avx2.cpp:82-263 with
// N = 1, whose every stage performs y = fma(v_s, X[c_s], y) per element).
//
// The chain of a row is serial, so the row is the unit of parallelism and a
// lane owns one: a one-warp CTA runs 32 rows' chains side by side.  What
// bounds such a kernel is how many bytes each SM keeps in flight and how
// few instructions a lane spends per slot, so:
//  * every lane streams its own row through shared memory with 1-D bulk
//    copies (cp.async.bulk, one per array per window of WIN slots, no
//    multicast), ST windows in flight on ST mbarriers (32 arrivals each:
//    every lane posts the bytes of its own copies with arrive.expect_tx).
//    The copies cover [rs & ~3, ceil4(rs + nnz)) -- live slots plus at most
//    three on each side, never the row's padding;
//  * after a window lands, the lane overwrites the at most three foreign
//    slots at either end of its row with the neutral pair (col -1, value
//    0); X sits in shared memory with X[-1] = 0, so a neutral slot performs
//    y = fma(0, 0, y) = y exactly (y is never -0: it starts at +0 and a
//    round-to-nearest sum is -0 only when both addends are -0).  The walk
//    over a window is then predicate-free: per 4 slots two 128-bit shared
//    loads (cols, values), four X loads and four FMAs;
//  * lane slices are WIN + 4 words apart, so the 8 lanes of a quarter-warp
//    read distinct bank groups.
// K above kMaxKs keeps X in global memory (read through L1, -1 -> 0).
#include <cstdlib>

#include "common.cuh"
#include "tma.cuh"

namespace slb {
namespace {

constexpr int64_t kMaxKs = 16384;  // largest K whose X is staged in shared memory

template <int WIN, int ST>
struct BulkShape {
    static constexpr int kStride = WIN + 4;                 // words per lane slice
    static constexpr int kStageWords = 32 * kStride;        // one array, one stage
    static constexpr size_t kRing = size_t(ST) * kStageWords * 4 * 2;  // cols + values
    static constexpr size_t kXOff = kRing + 16;              // X[-1] sits at kRing + 12
};

template <int WIN, int ST, bool KS>
__global__ void __launch_bounds__(32)
spmv_bulk_kernel(int M, int64_t K, int64_t cap_total, const int32_t* __restrict__ row_start,
                 const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                 const float* __restrict__ vals, const float* __restrict__ X,
                 float* __restrict__ Y, unsigned* status) {
    using S = BulkShape<WIN, ST>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t bar[ST];
    __shared__ __align__(8) uint64_t xbar;
    int* cring = reinterpret_cast<int*>(smem_raw);
    float* vring = reinterpret_cast<float*>(smem_raw + S::kRing / 2);
    float* xs = reinterpret_cast<float*>(smem_raw + S::kXOff);

    const int lane = threadIdx.x;
    const int row = blockIdx.x * 32 + lane;
    const bool live = row < M;
    const int64_t rs = live ? __ldg(row_start + row) : 0;
    const int64_t nn = live ? __ldg(row_nnz + row) : 0;
    const int64_t a = rs & ~int64_t(3);                       // first copied slot
    const int64_t e = nn > 0 ? ((rs + nn + 3) & ~int64_t(3)) : a;  // one past the last
    // Copies stop at the last whole 16-byte group of the arrays; the at most
    // three slots after it are read with plain loads.
    const int64_t ecopy = e > (cap_total & ~int64_t(3)) ? (cap_total & ~int64_t(3)) : e;
    const int nw = static_cast<int>((e - a + WIN - 1) / WIN);
    const int NW = __reduce_max_sync(0xffffffffu, nw);

    if (lane == 0) {
        for (int b = 0; b < ST; ++b) mbar_init(&bar[b], 32);
        mbar_init(&xbar, 1);
        fence_barrier_init();
    }
    __syncwarp();

    // X -> shared memory (one bulk copy when aligned), X[-1] = 0.
    bool xbulk = false;
    if (KS) {
        xbulk = (K % 4 == 0) && ((reinterpret_cast<uintptr_t>(X) & 15u) == 0);
        if (xbulk) {
            if (lane == 0) {
                mbar_expect_tx(&xbar, static_cast<unsigned>(K * 4));
                bulk_load_1d(xs, X, static_cast<unsigned>(K * 4), &xbar);
            }
        } else {
            for (int64_t k = lane; k < K; k += 32) xs[k] = __ldg(X + k);
        }
        if (lane == 0) xs[-1] = 0.0f;
    }

    int* cslice = cring + lane * S::kStride;
    float* vslice = vring + lane * S::kStride;

    auto issue = [&](int w) {
        const int b = w % ST;
        unsigned bytes = 0;
        int64_t s0 = 0, s1 = 0;
        if (w < nw) {
            s0 = a + static_cast<int64_t>(w) * WIN;
            s1 = s0 + WIN < ecopy ? s0 + WIN : ecopy;
            if (s1 > s0) bytes = static_cast<unsigned>((s1 - s0) * 8);
        }
        if (bytes) {
            mbar_expect_tx(&bar[b], bytes);
            const unsigned half = bytes / 2;
            bulk_load_1d(cslice + b * S::kStageWords, cols + s0, half, &bar[b]);
            bulk_load_1d(vslice + b * S::kStageWords, vals + s0, half, &bar[b]);
        } else {
            mbar_arrive(&bar[b]);
        }
    };

    fence_proxy_async();
#pragma unroll
    for (int w = 0; w < ST; ++w)
        if (w < NW) issue(w);

    bool ok = true;
    if (KS) {
        if (xbulk) ok = mbar_wait(&xbar, 0u, status);
        __syncwarp();
    }

    float y = 0.0f;
    int w = 0;
    for (; w < NW && ok; ++w) {
        const int b = w % ST;
        if (!mbar_wait(&bar[b], static_cast<unsigned>((w / ST) & 1), status)) {
            ok = false;
            break;
        }
        if (w < nw) {
            int* cb = cslice + b * S::kStageWords;
            float* vb = vslice + b * S::kStageWords;
            const int64_t s0 = a + static_cast<int64_t>(w) * WIN;
            const int len = static_cast<int>((s0 + WIN < e ? s0 + WIN : e) - s0);
            // Fix-ups in the lane's own slice: the foreign slots before the
            // row (first window), the uncopied tail group (plain loads) and
            // the foreign slots after the row (last window).
            if (w == 0)
                for (int64_t q = a; q < rs; ++q) { cb[q - s0] = -1; vb[q - s0] = 0.0f; }
            if (w == nw - 1)
                for (int64_t q = ecopy > s0 ? ecopy : s0; q < e; ++q) {
                    const bool in = q < rs + nn;
                    cb[q - s0] = in ? __ldg(cols + q) : -1;
                    vb[q - s0] = in ? __ldg(vals + q) : 0.0f;
                }
            if (w == nw - 1)
                for (int64_t q = rs + nn; q < e && q < ecopy; ++q) { cb[q - s0] = -1; vb[q - s0] = 0.0f; }
            const int4* c4 = reinterpret_cast<const int4*>(cb);
            const float4* v4 = reinterpret_cast<const float4*>(vb);
#pragma unroll 4
            for (int g = 0; g < len / 4; ++g) {
                const int4 c = c4[g];
                const float4 v = v4[g];
                float x0, x1, x2, x3;
                if (KS) {
                    x0 = xs[c.x]; x1 = xs[c.y]; x2 = xs[c.z]; x3 = xs[c.w];
                } else {
                    x0 = c.x >= 0 ? __ldg(X + c.x) : 0.0f;
                    x1 = c.y >= 0 ? __ldg(X + c.y) : 0.0f;
                    x2 = c.z >= 0 ? __ldg(X + c.z) : 0.0f;
                    x3 = c.w >= 0 ? __ldg(X + c.w) : 0.0f;
                }
                y = fmaf(v.x, x0, y);
                y = fmaf(v.y, x1, y);
                y = fmaf(v.z, x2, y);
                y = fmaf(v.w, x3, y);
            }
        }
        __syncwarp();
        // The stage is free again: refill it (its generic writes above are
        // ordered before the async-proxy copies by the fence).
        if (w + ST < NW) {
            fence_proxy_async();
            issue(w + ST);
        }
    }
    if (!ok) {
        // A wait gave up: let the copies already issued land (bounded) and
        // leave Y unwritten; the status word reports it.
        for (int h = w; h < NW && h < w + ST; ++h)
            if (h >= 0) mbar_wait(&bar[h % ST], static_cast<unsigned>((h / ST) & 1), status, 1 << 16);
        return;
    }
    if (live) Y[row] = y;
}

template <int WIN, int ST, bool KS>
int launch_cfg(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    using S = BulkShape<WIN, ST>;
    unsigned* status = device_status_word();
    if (status == nullptr) return -1;
    const size_t smem = S::kXOff + (KS ? static_cast<size_t>(K) * 4 : 0);
    auto kern = spmv_bulk_kernel<WIN, ST, KS>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int M = static_cast<int>(W->nrows);
    kern<<<(M + 31) / 32, 32, smem, s>>>(M, K, W->total_capacity, W->row_start, W->row_nnz,
                                         W->col_indices, W->values, X, Y, status);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd (N = 1, bulk)");
    return SL_OK;
}

}  // namespace

// Few rows (at most one warp per SM): 128-slot windows, 4 in flight (one
// CTA per SM).  More rows: 64-slot windows, 4 in flight, two CTAs per SM.
// SPARSECORE_B200_N1_WIN=64|128 overrides (measurements).  Returns -1 when
// the kernel cannot be configured (caller falls back).
int launch_spmv_bulk(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    if (!aligned16(W->col_indices) || !aligned16(W->values) || W->nrows <= 0 || K < 1 ||
        W->nrows > INT_MAX - 32)
        return -1;
    const int64_t warps = (W->nrows + 31) / 32;
    int win = warps <= num_sms() ? 128 : 64;
    if (const char* e = std::getenv("SPARSECORE_B200_N1_WIN")) {
        const int v = std::atoi(e);
        if (v == 64 || v == 128) win = v;
    }
    const bool ks = K <= kMaxKs;
    if (win == 128) return ks ? launch_cfg<128, 4, true>(W, X, K, Y, s) : launch_cfg<128, 4, false>(W, X, K, Y, s);
    return ks ? launch_cfg<64, 4, true>(W, X, K, Y, s) : launch_cfg<64, 4, false>(W, X, K, Y, s);
}

}  // namespace slb
