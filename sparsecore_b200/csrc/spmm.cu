// Forward SpMM over padded CSR:  Y[M,N] = W[M,K] . X[K,N]   (fp32)
//
// Numerics: every Y element is the FMA chain  y = fma(v_s, X[c_s, j], y)
// over the row's live slots in slot order, starting from +0.  This is the
// rounding sequence of the reference CPU kernel (csrc/kernels/spmm_avx2.cpp:
// 82-263, whose 16/8/1-wide stages all perform that same fused update per
// element), so results are bit-identical.
//
// Work decomposition (gather-bound, no tensor cores): a warp owns a group of
// RPW = 32/LPR consecutive rows and a tile of TILE = LPR*VEC*CPL columns.
// Each row of the group is handled by LPR lanes; each lane owns CPL vectors
// of VEC consecutive columns, strided by LPR*VEC so that the lanes of a row
// read X rows as contiguous, coalesced 128-bit segments.  The warp stages
// the (col, value) pairs of its rows' contiguous slot segment through shared
// memory in chunks (coalesced 32-bit loads), then every lane walks its row's
// live slots from shared memory (broadcast reads).  Work items (row group,
// column tile) are ordered column-tile fastest so that warps resident
// together share the same W segment (L1/L2 hits) and sweep X once.
#include "common.cuh"
#include "tma.cuh"

namespace slb {
namespace {

constexpr int kFwdThreads = 256;
constexpr int kFwdWarps = kFwdThreads / 32;
constexpr int kChunk = 128;  // staged slots per warp

template <int VEC>
struct Vec;
template <>
struct Vec<4> {
    using T = float4;
    static __device__ __forceinline__ float4 load(const float* p) {
        return __ldg(reinterpret_cast<const float4*>(p));
    }
};
template <>
struct Vec<1> {
    using T = float;
    static __device__ __forceinline__ float load(const float* p) { return __ldg(p); }
};

__device__ __forceinline__ void fma_vec(float v, float4 x, float* acc) {
    acc[0] = fmaf(v, x.x, acc[0]);
    acc[1] = fmaf(v, x.y, acc[1]);
    acc[2] = fmaf(v, x.z, acc[2]);
    acc[3] = fmaf(v, x.w, acc[3]);
}
__device__ __forceinline__ void fma_vec(float v, float x, float* acc) { acc[0] = fmaf(v, x, acc[0]); }

template <int VEC, int LPR, int CPL>
__global__ void __launch_bounds__(kFwdThreads)
spmm_fwd_kernel(int M, int64_t N, const int32_t* __restrict__ row_start,
                const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                const float* __restrict__ vals, const float* __restrict__ X,
                float* __restrict__ Y, int64_t n_tiles, int64_t n_items) {
    constexpr int RPW = 32 / LPR;
    constexpr int TILE = LPR * VEC * CPL;
    __shared__ int2 stage[kFwdWarps][kChunk];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane / LPR, li = lane % LPR;
    int2* st = stage[warp];

    for (int64_t item = static_cast<int64_t>(blockIdx.x) * kFwdWarps + warp; item < n_items;
         item += static_cast<int64_t>(gridDim.x) * kFwdWarps) {
        const int64_t nt = item % n_tiles;
        const int row0 = static_cast<int>(item / n_tiles) * RPW;
        const int row = row0 + g;
        const bool valid = row < M;
        int rs = 0, nn = 0;
        if (valid) {
            rs = __ldg(row_start + row);
            nn = __ldg(row_nnz + row);
        }
        // Contiguous slot segment covering the live slots of the warp's rows.
        int lo = (nn > 0) ? rs : INT_MAX;
        int hi = (nn > 0) ? rs + nn : INT_MIN;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
            hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        }

        const int64_t jbase = nt * TILE + static_cast<int64_t>(li) * VEC;
        int64_t jl[CPL];
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc) {
            const int64_t j = jbase + static_cast<int64_t>(cc) * LPR * VEC;
            jl[cc] = j < N - VEC ? j : N - VEC;  // clamp: always a valid address
        }
        float acc[CPL][VEC];
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc)
#pragma unroll
            for (int e = 0; e < VEC; ++e) acc[cc][e] = 0.0f;

        for (int cb = lo; cb < hi; cb += kChunk) {
            const int cnt = min(kChunk, hi - cb);
            for (int t = lane; t < cnt; t += 32)
                st[t] = make_int2(__ldg(cols + cb + t), __float_as_int(__ldg(vals + cb + t)));
            __syncwarp();
            const int s0 = max(rs, cb) - cb;
            const int s1 = min(rs + nn, cb + cnt) - cb;
#pragma unroll 4
            for (int s = s0; s < s1; ++s) {
                const int2 e = st[s];
                const float v = __int_as_float(e.y);
                const float* xr = X + static_cast<int64_t>(e.x) * N;
#pragma unroll
                for (int cc = 0; cc < CPL; ++cc) fma_vec(v, Vec<VEC>::load(xr + jl[cc]), acc[cc]);
            }
            __syncwarp();
        }

        if (valid) {
            float* yr = Y + static_cast<int64_t>(row) * N;
#pragma unroll
            for (int cc = 0; cc < CPL; ++cc) {
                const int64_t j = jbase + static_cast<int64_t>(cc) * LPR * VEC;
                if (j < N) {
                    if constexpr (VEC == 4) {
                        *reinterpret_cast<float4*>(yr + j) =
                            make_float4(acc[cc][0], acc[cc][1], acc[cc][2], acc[cc][3]);
                    } else {
                        yr[j] = acc[cc][0];
                    }
                }
            }
        }
    }
}

template <int VEC, int LPR, int CPL>
int launch_fwd(const sl_csr* W, const float* X, int64_t N, float* Y, cudaStream_t s) {
    constexpr int RPW = 32 / LPR;
    constexpr int TILE = LPR * VEC * CPL;
    const int M = static_cast<int>(W->nrows);
    const int64_t n_tiles = (N + TILE - 1) / TILE;
    const int64_t n_items = ((M + RPW - 1) / RPW) * n_tiles;
    int64_t blocks = (n_items + kFwdWarps - 1) / kFwdWarps;
    const int64_t max_blocks = static_cast<int64_t>(num_sms()) * 64;
    if (blocks > max_blocks) blocks = max_blocks;
    spmm_fwd_kernel<VEC, LPR, CPL><<<static_cast<unsigned>(blocks), kFwdThreads, 0, s>>>(
        M, N, W->row_start, W->row_nnz, W->col_indices, W->values, X, Y, n_tiles, n_items);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd");
    return SL_OK;
}

// Lane layout by the number of column vectors per row.
template <int VEC>
int dispatch_fwd(const sl_csr* W, const float* X, int64_t N, float* Y, cudaStream_t s) {
    const int64_t nv = (N + VEC - 1) / VEC;
    if (nv >= 64) return launch_fwd<VEC, 32, 2>(W, X, N, Y, s);
    if (nv > 16) return launch_fwd<VEC, 32, 1>(W, X, N, Y, s);
    if (nv > 8) return launch_fwd<VEC, 16, 1>(W, X, N, Y, s);
    if (nv > 4) return launch_fwd<VEC, 8, 1>(W, X, N, Y, s);
    if (nv > 2) return launch_fwd<VEC, 4, 1>(W, X, N, Y, s);
    if (nv > 1) return launch_fwd<VEC, 2, 1>(W, X, N, Y, s);
    return launch_fwd<VEC, 1, 1>(W, X, N, Y, s);
}


// ── X-stationary variant (large N) ───────────────────────────────────────
// A CTA keeps the full column tile X[:, j0 : j0+TN] (all K rows) resident in
// shared memory -- loaded by TMA as 128-row boxes completing on one mbarrier
// -- and streams rows of W against it: every FMA's X operand then comes from
// shared memory (one conflict-free 128-bit read per lane per slot) instead
// of L2.  Work items are (column tile, block of rows), tile-major; each CTA
// takes a contiguous run of items and reloads X only when its tile changes.
// Numerics are identical to spmm_fwd_kernel (same per-element FMA chain).
constexpr int kXsThreads = 512;
constexpr int kXsWarps = kXsThreads / 32;
constexpr int kXsBoxRows = 128;
constexpr int kXsRowsPerItemMul = 4;

template <int LPR>
__global__ void __launch_bounds__(kXsThreads)
spmm_xs_kernel(const __grid_constant__ CUtensorMap xmap, int M, int64_t N,
               const int32_t* __restrict__ row_start, const int32_t* __restrict__ row_nnz,
               const int32_t* __restrict__ cols, const float* __restrict__ vals,
               float* __restrict__ Y, int nbox, int row_chunks, int64_t n_items,
               int64_t items_per_cta, unsigned* status) {
    constexpr int TN = 4 * LPR;
    constexpr int RPW = 32 / LPR;
    constexpr int ROWS_PER_ITEM = kXsWarps * RPW * kXsRowsPerItemMul;
    extern __shared__ __align__(128) unsigned char smem[];
    float* xs = reinterpret_cast<float*>(smem);
    int2* stage = reinterpret_cast<int2*>(smem + static_cast<size_t>(nbox) * kXsBoxRows * TN * 4);
    __shared__ __align__(8) uint64_t bar;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane / LPR, li = lane % LPR;
    int2* st = stage + warp * kChunk;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();

    const int64_t it0 = static_cast<int64_t>(blockIdx.x) * items_per_cta;
    const int64_t it1 = min(it0 + items_per_cta, n_items);
    int64_t cur_tile = -1;
    unsigned phase = 0;
    for (int64_t item = it0; item < it1; ++item) {
        const int64_t tile = item / row_chunks;
        const int chunk = static_cast<int>(item % row_chunks);
        if (tile != cur_tile) {
            __syncthreads();  // every reader of the previous tile is done
            if (threadIdx.x == 0) {
                fence_proxy_async();
                mbar_expect_tx(&bar, static_cast<unsigned>(nbox) * kXsBoxRows * TN * 4);
                for (int b = 0; b < nbox; ++b)
                    tma_load_2d(xs + static_cast<size_t>(b) * kXsBoxRows * TN, &xmap,
                                static_cast<int>(tile * TN), b * kXsBoxRows, &bar);
            }
            if (!mbar_wait(&bar, phase, status)) {
                mbar_wait(&bar, phase, status);  // let copies in flight land, then leave
                return;
            }
            phase ^= 1u;
            cur_tile = tile;
        }
        const int64_t j = tile * TN + li * 4;
        for (int rg = warp; rg < ROWS_PER_ITEM / RPW; rg += kXsWarps) {
            const int row = chunk * ROWS_PER_ITEM + rg * RPW + g;
            const bool valid = row < M;
            int rs = 0, nn = 0;
            if (valid) {
                rs = __ldg(row_start + row);
                nn = __ldg(row_nnz + row);
            }
            int lo = (nn > 0) ? rs : INT_MAX;
            int hi = (nn > 0) ? rs + nn : INT_MIN;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
                hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
            }
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int cb = lo; cb < hi; cb += kChunk) {
                const int cnt = min(kChunk, hi - cb);
                for (int t = lane; t < cnt; t += 32)
                    st[t] = make_int2(__ldg(cols + cb + t), __float_as_int(__ldg(vals + cb + t)));
                __syncwarp();
                const int s0 = max(rs, cb) - cb;
                const int s1 = min(rs + nn, cb + cnt) - cb;
#pragma unroll 4
                for (int s = s0; s < s1; ++s) {
                    const int2 e = st[s];
                    const float4 x = *reinterpret_cast<const float4*>(xs + e.x * TN + li * 4);
                    fma_vec(__int_as_float(e.y), x, acc);
                }
                __syncwarp();
            }
            if (valid && j < N)
                *reinterpret_cast<float4*>(Y + static_cast<int64_t>(row) * N + j) =
                    make_float4(acc[0], acc[1], acc[2], acc[3]);
        }
    }
}

// Tile width by K so that the resident tile fits in shared memory.
int xs_lanes_for(int64_t K) {
    const int64_t rows = (K + kXsBoxRows - 1) / kXsBoxRows * kXsBoxRows;
    const int64_t budget = 200 * 1024;
    if (rows * 32 * 4 <= budget) return 8;   // TN = 32
    if (rows * 16 * 4 <= budget) return 4;   // TN = 16
    if (rows * 8 * 4 <= budget) return 2;    // TN = 8
    return 0;
}

template <int LPR>
int launch_xs(const sl_csr* W, const float* X, int64_t K, int64_t N, float* Y, cudaStream_t s) {
    constexpr int TN = 4 * LPR;
    constexpr int RPW = 32 / LPR;
    constexpr int ROWS_PER_ITEM = kXsWarps * RPW * kXsRowsPerItemMul;
    CUtensorMap map;
    if (!make_tmap_2d(&map, X, K, N, kXsBoxRows, TN)) return -1;
    unsigned* status = device_status_word();
    if (status == nullptr) return -1;
    const int M = static_cast<int>(W->nrows);
    const int nbox = static_cast<int>((K + kXsBoxRows - 1) / kXsBoxRows);
    const size_t smem = static_cast<size_t>(nbox) * kXsBoxRows * TN * 4 +
                        static_cast<size_t>(kXsWarps) * kChunk * sizeof(int2);
    if (cudaFuncSetAttribute(spmm_xs_kernel<LPR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int row_chunks = (M + ROWS_PER_ITEM - 1) / ROWS_PER_ITEM;
    const int64_t n_tiles = (N + TN - 1) / TN;
    const int64_t n_items = n_tiles * row_chunks;
    const int per_sm = smem <= 110 * 1024 ? 2 : 1;
    int64_t grid = static_cast<int64_t>(num_sms()) * per_sm;
    if (grid > n_items) grid = n_items;
    const int64_t per_cta = (n_items + grid - 1) / grid;
    grid = (n_items + per_cta - 1) / per_cta;
    spmm_xs_kernel<LPR><<<static_cast<unsigned>(grid), kXsThreads, smem, s>>>(
        map, M, N, W->row_start, W->row_nnz, W->col_indices, W->values, Y, nbox, row_chunks,
        n_items, per_cta, status);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd (x-stationary)");
    return SL_OK;
}

// Returns -1 when the X-stationary path does not apply.
int try_xs(const sl_csr* W, const float* X, int64_t K, int64_t N, float* Y, cudaStream_t s) {
    if (N < 256 || N % 4 != 0 || !aligned16(X) || !aligned16(Y) || K < 1 || K > INT_MAX) return -1;
    switch (xs_lanes_for(K)) {
        case 8: return launch_xs<8>(W, X, K, N, Y, s);
        case 4: return launch_xs<4>(W, X, K, N, Y, s);
        case 2: return launch_xs<2>(W, X, K, N, Y, s);
        default: return -1;
    }
}
}  // namespace
}  // namespace slb

using namespace slb;

extern "C" int sl_spmm_fwd(const sl_csr* W, const float* X, int64_t K, int64_t N, float* Y,
                           void* stream) {
    if (int rc = check_csr(W, "sl_spmm_fwd")) return rc;
    if (W->ncols != K)
        return fail(SL_ERR_INVALID, "sl_spmm_fwd: shape mismatch. W has ncols=" +
                                        std::to_string(W->ncols) + " but X has shape[0]=" +
                                        std::to_string(K) +
                                        ". Inner dimensions must match for matmul.");
    if (N < 0) return fail(SL_ERR_INVALID, "sl_spmm_fwd: negative N");
    if (W->nrows == 0 || N == 0) return SL_OK;
    if (Y == nullptr || (K > 0 && X == nullptr))
        return fail(SL_ERR_INVALID, "sl_spmm_fwd: NULL dense operand");
    cudaStream_t s = as_stream(stream);
    if (K == 0) return cuda_status(cudaMemsetAsync(Y, 0, sizeof(float) * W->nrows * N, s),
                                   "sl_spmm_fwd memset");
    const int rc = try_xs(W, X, K, N, Y, s);
    if (rc >= 0) return rc;
    const bool vec4 = (N % 4 == 0) && aligned16(X) && aligned16(Y);
    return vec4 ? dispatch_fwd<4>(W, X, N, Y, s) : dispatch_fwd<1>(W, X, N, Y, s);
}
