// Dense gradient for the RigL grow criterion:  G[M,K] = dY[M,N] . X[K,N]^T
// (csrc/kernels/dense_grad.cpp:463-523).  Full fp32 on the FMA pipe -- no
// TF32: the |G| ranking that picks grown columns must stay fp32-accurate.
//
// Classic register-tiled SIMT GEMM: a CTA computes a 64x64 tile of G with
// 256 threads (4x4 outputs each), staging 16-wide slices of the reduction
// dimension of both operands through shared memory (transposed, padded).
// Each output element accumulates over j = 0..N-1 in ascending order with the
// rounding sequence of the reference's compiled scalar loop (an in-order
// vectorised reduction): for j < 4*floor(N/4) a rounded product added to the
// running sum, for the last N mod 4 terms an FMA -- bit-identical results.
#include <cstdlib>

#include "common.cuh"

namespace slb {
namespace {

constexpr int BM = 64, BK = 64, BJ = 16, kGThreads = 256;

// Epilogue of the fused RigL path (TOPK): instead of storing the tile, the
// CTA turns it into per-row grow candidates.  key = |G| bits + 1 for
// candidate columns (not survivors, inside K), 0 otherwise; each row keeps
// its L = min(n_grow + 1, Lmax) largest keys of the tile's 128 columns (ties
// by lowest column).  A NaN candidate flags the row (the host resolves it).
struct TopkArgs {
    const uint32_t* bits;   // survivors: [M][ceil(K/32)] bitmap
    const int32_t* n_grow;  // [M]
    int lmax;
    int tiles;              // ceil(K / tile width)
    uint32_t* cand_key;     // [M][tiles][lmax]
    int32_t* cand_col;      // [M][tiles][lmax]
    int32_t* cand_cnt;      // [M][tiles]
    int32_t* row_flag;      // [M], bit 0 = resolve on the host
};


// Per-row candidate selection of a BT x BT tile whose keys (see TopkArgs)
// are staged in shared memory as keys[BT][BT + 1]: one warp per row keeps
// the row's min(n_grow + 1, lmax) largest keys (ties -> lowest column).
template <int BT>
__device__ __forceinline__ void topk_select_tile(const uint32_t* keys, int m0, int k0, int M,
                                                 const TopkArgs& ta, int tile) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int Q = BT / 32;
    for (int lr2 = warp; lr2 < BT; lr2 += kGThreads / 32) {
        const int m = m0 + lr2;
        if (m >= M) break;
        const int L = min(__ldg(ta.n_grow + m) + 1, ta.lmax);
        uint32_t kv[Q];
#pragma unroll
        for (int q = 0; q < Q; ++q) kv[q] = keys[lr2 * (BT + 1) + lane + 32 * q];
        const int64_t base = (static_cast<int64_t>(m) * ta.tiles + tile) * ta.lmax;
        int cnt = 0;
        for (; cnt < L; ++cnt) {
            uint32_t best = kv[0];
            int bq = 0;
#pragma unroll
            for (int q = 1; q < Q; ++q)
                if (kv[q] > best) { best = kv[q]; bq = q; }
            int bcol = lane + 32 * bq;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const uint32_t ob = __shfl_xor_sync(0xffffffffu, best, o);
                const int oc = __shfl_xor_sync(0xffffffffu, bcol, o);
                if (ob > best || (ob == best && oc < bcol)) { best = ob; bcol = oc; }
            }
            if (best == 0u) break;  // no candidate left in this tile
            if (lane == 0) {
                ta.cand_key[base + cnt] = best;
                ta.cand_col[base + cnt] = k0 + bcol;
            }
            if (lane == (bcol & 31)) kv[bcol >> 5] = 0u;
        }
        if (lane == 0) ta.cand_cnt[static_cast<int64_t>(m) * ta.tiles + tile] = cnt;
    }
}

// Candidate key of G[m][k] (0 = not a candidate); a NaN sets *nan.
__device__ __forceinline__ uint32_t candidate_key(const TopkArgs& ta, int M, int K, int m, int k,
                                                  float g, bool* nan) {
    const int KW = (K + 31) >> 5;
    if (m >= M || k >= K || ((__ldg(ta.bits + static_cast<int64_t>(m) * KW + (k >> 5)) >> (k & 31)) & 1u))
        return 0u;
    const uint32_t a = __float_as_uint(g) & 0x7fffffffu;
    *nan |= a > 0x7f800000u;
    return a + 1u;
}


template <bool VEC4, bool TOPK>
__global__ void __launch_bounds__(kGThreads)
dense_grad_kernel(const float* __restrict__ A, const float* __restrict__ B, int M, int K,
                  int64_t N, float* __restrict__ G, TopkArgs ta) {
    __shared__ float As[BJ][BM + 4];
    __shared__ float Bs[BJ][BK + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * BM, k0 = blockIdx.x * BK;
    float acc[4][4] = {};

    // Loader mapping: 64 rows x 16 j per operand = 256 float4 -> 1 per thread.
    const int lr = threadIdx.x >> 2;       // 0..63
    const int lj = (threadIdx.x & 3) * 4;  // 0,4,8,12
    for (int64_t j0 = 0; j0 < N; j0 += BJ) {
        float a[4], b[4];
        const int64_t j = j0 + lj;
        const int am = m0 + lr, bk = k0 + lr;
        if (VEC4 && j + 3 < N) {
            float4 va = am < M ? __ldg(reinterpret_cast<const float4*>(A + static_cast<int64_t>(am) * N + j))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 vb = bk < K ? __ldg(reinterpret_cast<const float4*>(B + static_cast<int64_t>(bk) * N + j))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            a[0] = va.x; a[1] = va.y; a[2] = va.z; a[3] = va.w;
            b[0] = vb.x; b[1] = vb.y; b[2] = vb.z; b[3] = vb.w;
        } else {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const bool in = j + t < N;
                a[t] = (in && am < M) ? __ldg(A + static_cast<int64_t>(am) * N + j + t) : 0.f;
                b[t] = (in && bk < K) ? __ldg(B + static_cast<int64_t>(bk) * N + j + t) : 0.f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            As[lj + t][lr] = a[t];
            Bs[lj + t][lr] = b[t];
        }
        __syncthreads();
        const int jn = static_cast<int>(N - j0 < BJ ? N - j0 : BJ);
        const int64_t n4 = N & ~static_cast<int64_t>(3);
        const int jv = static_cast<int>(n4 - j0 >= jn ? jn : (n4 - j0 > 0 ? n4 - j0 : 0));
        for (int jj = 0; jj < jv; ++jj) {
            const float4 ra = *reinterpret_cast<const float4*>(&As[jj][ty * 4]);
            const float4 rb = *reinterpret_cast<const float4*>(&Bs[jj][tx * 4]);
            const float av[4] = {ra.x, ra.y, ra.z, ra.w};
            const float bv[4] = {rb.x, rb.y, rb.z, rb.w};
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(av[r], bv[c]));
        }
        for (int jj = jv; jj < jn; ++jj) {
            const float4 ra = *reinterpret_cast<const float4*>(&As[jj][ty * 4]);
            const float4 rb = *reinterpret_cast<const float4*>(&Bs[jj][tx * 4]);
            const float av[4] = {ra.x, ra.y, ra.z, ra.w};
            const float bv[4] = {rb.x, rb.y, rb.z, rb.w};
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
        }
    }
    if constexpr (!TOPK) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int m = m0 + ty * 4 + r;
            if (m >= M) continue;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int k = k0 + tx * 4 + c;
                if (k < K) G[static_cast<int64_t>(m) * K + k] = acc[r][c];
            }
        }
    } else {
        __shared__ uint32_t keys[BM * (BM + 1)];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int m = m0 + ty * 4 + r;
            bool nan_row = false;
#pragma unroll
            for (int c = 0; c < 4; ++c)
                keys[(ty * 4 + r) * (BM + 1) + tx * 4 + c] =
                    candidate_key(ta, M, K, m, k0 + tx * 4 + c, acc[r][c], &nan_row);
            if (nan_row) atomicOr(ta.row_flag + m, 1);
        }
        __syncthreads();
        topk_select_tile<BM>(keys, m0, k0, M, ta, blockIdx.x);
    }
}

// Larger tiles for larger shapes: a CTA computes a 128x128 tile of G with
// 256 threads holding 8x8 outputs each (two 4-wide row groups and two
// 4-wide column groups 64 apart, so a quarter-warp's 128-bit shared reads are
// conflict-free), reduction slices of 8 staged in shared memory and
// double-buffered: the next slice is loaded into registers while the
// current one is consumed.  Per element the same ascending-j sequence as
// above (rounded product + add for j < 4*floor(N/4), FMA after), so the
// results are bit-identical to the 64x64 kernel's.
constexpr int BB = 128, BJ2 = 8;

template <bool VEC4, bool TOPK>
__global__ void __launch_bounds__(kGThreads)
dense_grad128_kernel(const float* __restrict__ A, const float* __restrict__ B, int M, int K,
                     int64_t N, float* __restrict__ G, TopkArgs ta) {
    __shared__ __align__(16) float As[2][BJ2][BB + 4];
    __shared__ __align__(16) float Bs[2][BJ2][BB + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * BB, k0 = blockIdx.x * BB;
    float acc[8][8];
#pragma unroll
    for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[r][c] = 0.0f;

    // Loader: 128 rows x 8 j per operand = 256 float4 -> one per thread.
    const int lr = threadIdx.x >> 1;       // 0..127
    const int lj = (threadIdx.x & 1) * 4;  // 0 or 4
    const int am = m0 + lr, bk = k0 + lr;
    auto load = [&](int64_t j0, float* a, float* b) {
        const int64_t j = j0 + lj;
        if (VEC4 && j + 3 < N) {
            const float4 va = am < M ? __ldg(reinterpret_cast<const float4*>(A + static_cast<int64_t>(am) * N + j))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 vb = bk < K ? __ldg(reinterpret_cast<const float4*>(B + static_cast<int64_t>(bk) * N + j))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
            a[0] = va.x; a[1] = va.y; a[2] = va.z; a[3] = va.w;
            b[0] = vb.x; b[1] = vb.y; b[2] = vb.z; b[3] = vb.w;
        } else {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const bool in = j + t < N;
                a[t] = (in && am < M) ? __ldg(A + static_cast<int64_t>(am) * N + j + t) : 0.f;
                b[t] = (in && bk < K) ? __ldg(B + static_cast<int64_t>(bk) * N + j + t) : 0.f;
            }
        }
    };
    float a[4], b[4];
    load(0, a, b);
    const int64_t n4 = N & ~static_cast<int64_t>(3);
    int buf = 0;
    for (int64_t j0 = 0; j0 < N; j0 += BJ2) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            As[buf][lj + t][lr] = a[t];
            Bs[buf][lj + t][lr] = b[t];
        }
        __syncthreads();
        if (j0 + BJ2 < N) load(j0 + BJ2, a, b);  // next slice in flight during this one
        const int jn = static_cast<int>(N - j0 < BJ2 ? N - j0 : BJ2);
        const int jv = static_cast<int>(n4 - j0 >= jn ? jn : (n4 - j0 > 0 ? n4 - j0 : 0));
#pragma unroll
        for (int jj = 0; jj < BJ2; ++jj) {
            if (jj >= jn) break;
            float av[8], bv[8];
            const float4 ra0 = *reinterpret_cast<const float4*>(&As[buf][jj][ty * 4]);
            const float4 ra1 = *reinterpret_cast<const float4*>(&As[buf][jj][64 + ty * 4]);
            const float4 rb0 = *reinterpret_cast<const float4*>(&Bs[buf][jj][tx * 4]);
            const float4 rb1 = *reinterpret_cast<const float4*>(&Bs[buf][jj][64 + tx * 4]);
            av[0] = ra0.x; av[1] = ra0.y; av[2] = ra0.z; av[3] = ra0.w;
            av[4] = ra1.x; av[5] = ra1.y; av[6] = ra1.z; av[7] = ra1.w;
            bv[0] = rb0.x; bv[1] = rb0.y; bv[2] = rb0.z; bv[3] = rb0.w;
            bv[4] = rb1.x; bv[5] = rb1.y; bv[6] = rb1.z; bv[7] = rb1.w;
            if (jj < jv) {
#pragma unroll
                for (int r = 0; r < 8; ++r)
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(av[r], bv[c]));
            } else {
#pragma unroll
                for (int r = 0; r < 8; ++r)
#pragma unroll
                    for (int c = 0; c < 8; ++c) acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
            }
        }
        buf ^= 1;
    }
    if constexpr (!TOPK) {
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int m = m0 + (r < 4 ? ty * 4 + r : 64 + ty * 4 + r - 4);
            if (m >= M) continue;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int k = k0 + (c < 4 ? tx * 4 + c : 64 + tx * 4 + c - 4);
                if (k < K) G[static_cast<int64_t>(m) * K + k] = acc[r][c];
            }
        }
    } else {
        extern __shared__ uint32_t keys[];  // [128][129]
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            const int lr2 = r < 4 ? ty * 4 + r : 64 + ty * 4 + r - 4;
            const int m = m0 + lr2;
            bool nan_row = false;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int lc = c < 4 ? tx * 4 + c : 64 + tx * 4 + c - 4;
                keys[lr2 * 129 + lc] = candidate_key(ta, M, K, m, k0 + lc, acc[r][c], &nan_row);
            }
            if (nan_row) atomicOr(ta.row_flag + m, 1);
        }
        __syncthreads();
        topk_select_tile<BB>(keys, m0, k0, M, ta, blockIdx.x);
    }
}

// Survivor bitmap and grow count per row for the fused RigL path: a slot
// survives when |v| > thr or it is the row's forced keep (the same rule as
// the rewrite kernel); n_grow = min(n_drop, K - n_keep), 0 for empty rows.
__global__ void __launch_bounds__(256)
rigl_prep_kernel(int M, int K, const int32_t* __restrict__ row_start,
                 const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                 const float* __restrict__ vals, const float* __restrict__ thr_dev,
                 const int32_t* __restrict__ force_idx, uint32_t* __restrict__ bits,
                 int32_t* __restrict__ n_grow) {
    const int lane = threadIdx.x & 31;
    const int KW = (K + 31) >> 5;
    const float thr = *thr_dev;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M; row += warps) {
        uint32_t* br = bits + static_cast<int64_t>(row) * KW;
        for (int w = lane; w < KW; w += 32) br[w] = 0u;
        __syncwarp();
        const int rs = row_start[row], nn = row_nnz[row], fidx = force_idx[row];
        int keep = 0;
        for (int s = lane; s < nn; s += 32) {
            if (fabsf(vals[rs + s]) > thr || s == fidx) {
                const int c = cols[rs + s];
                atomicOr(br + (c >> 5), 1u << (c & 31));
                ++keep;
            }
        }
        keep = warp_sum(keep);
        if (lane == 0) n_grow[row] = nn > 0 ? min(nn - keep, K - keep) : 0;
    }
}

// Merge the tiles' candidates of each row: the n_grow largest keys are the
// grown columns, unless the (n_grow+1)-th key equals the n_grow-th (ties
// straddle the cut: numpy's argpartition decides, so the row goes to the
// host) or a NaN was seen.  row_mask = 1 for rows rewritten on the device.
__global__ void __launch_bounds__(256)
rigl_merge_kernel(int M, int tiles, int lmax, const uint32_t* __restrict__ cand_key,
                  const int32_t* __restrict__ cand_col, const int32_t* __restrict__ cand_cnt,
                  const int32_t* __restrict__ n_grow, const int32_t* __restrict__ grow_off,
                  const int32_t* __restrict__ row_nnz, int32_t* __restrict__ row_flag,
                  int32_t* __restrict__ row_mask, int32_t* __restrict__ grow_cols) {
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M; row += warps) {
        const int ng = n_grow[row];
        int flag = row_flag[row];
        if (row_nnz[row] == 0) {
            if (lane == 0) row_mask[row] = 0;
            continue;
        }
        const int64_t cbase = static_cast<int64_t>(row) * tiles * lmax;
        const int ncand = tiles * lmax;
        uint32_t prev = 0;
        int taken = 0;
        // Selection rounds over the row's candidates (ng + 1 of them at most);
        // consumed ones are skipped through their key drop below `prev`.
        for (int t = 0; t <= ng && !flag; ++t) {
            uint32_t best = 0u;
            int bcol = INT_MAX;
            for (int e = lane; e < ncand; e += 32) {
                const int tl = e / lmax, q = e % lmax;
                if (q >= cand_cnt[static_cast<int64_t>(row) * tiles + tl]) continue;
                const uint32_t k = cand_key[cbase + e];
                const int c = cand_col[cbase + e];
                // strictly after the previous pick in (key desc, col asc) order
                const bool after = t == 0 || k < prev || (k == prev && c > taken);
                if (after && (k > best || (k == best && c < bcol))) { best = k; bcol = c; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const uint32_t ob = __shfl_xor_sync(0xffffffffu, best, o);
                const int oc = __shfl_xor_sync(0xffffffffu, bcol, o);
                if (ob > best || (ob == best && oc < bcol)) { best = ob; bcol = oc; }
            }
            if (t < ng) {
                if (best == 0u) { flag = 1; break; }  // fewer candidates than n_grow
                if (lane == 0) grow_cols[grow_off[row] + t] = bcol;
            } else if (best != 0u && best == prev) {
                flag = 1;  // the (n_grow+1)-th key ties the n_grow-th
            }
            prev = best;
            taken = bcol;
        }
        if (lane == 0) {
            row_flag[row] = flag;
            row_mask[row] = flag ? 0 : 1;
        }
    }
}

}  // namespace
}  // namespace slb

using namespace slb;

extern "C" int sl_dense_grad(const float* dY, const float* X, int64_t M, int64_t K, int64_t N,
                             float* G, void* stream) {
    if (M < 0 || K < 0 || N < 0)
        return fail(SL_ERR_INVALID, "dense_grad: shape params must be non-negative");
    if (M > INT_MAX || K > INT_MAX) return fail(SL_ERR_UNSUPPORTED, "dense_grad: shape beyond int32");
    if (M == 0 || K == 0) return SL_OK;
    SL_REQUIRE(G != nullptr, "dense_grad", "NULL output G");
    SL_REQUIRE(N == 0 || (dY != nullptr && X != nullptr), "dense_grad", "NULL dense operand");
    cudaStream_t s = as_stream(stream);
    if (N == 0) return cuda_status(cudaMemsetAsync(G, 0, sizeof(float) * M * K, s), "dense_grad memset");
    const bool vec4 = (N % 4 == 0) && aligned16(dY) && aligned16(X);
    // 128x128 tiles where they fill the GPU (SPARSECORE_B200_DG=64|128
    // forces one kernel: tests and measurements).
    const char* e = std::getenv("SPARSECORE_B200_DG");
    const int64_t tiles128 = ((M + BB - 1) / BB) * ((K + BB - 1) / BB);
    const bool big = e != nullptr ? e[0] == '1' : tiles128 >= num_sms();
    if (big) {
        const dim3 g2(static_cast<unsigned>((K + BB - 1) / BB), static_cast<unsigned>((M + BB - 1) / BB));
        if (vec4)
            dense_grad128_kernel<true, false><<<g2, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                                       static_cast<int>(K), N, G, TopkArgs{});
        else
            dense_grad128_kernel<false, false><<<g2, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                                        static_cast<int>(K), N, G, TopkArgs{});
        SL_RETURN_IF_LAUNCH_FAILED("sl_dense_grad");
        return SL_OK;
    }
    const dim3 grid(static_cast<unsigned>((K + BK - 1) / BK), static_cast<unsigned>((M + BM - 1) / BM));
    if (vec4)
        dense_grad_kernel<true, false><<<grid, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                                  static_cast<int>(K), N, G, TopkArgs{});
    else
        dense_grad_kernel<false, false><<<grid, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                                   static_cast<int>(K), N, G, TopkArgs{});
    SL_RETURN_IF_LAUNCH_FAILED("sl_dense_grad");
    return SL_OK;
}

extern "C" int sl_rigl_prep(const sl_csr* W, const float* thr_dev, const int32_t* force_idx,
                            uint32_t* survivor_bits, int32_t* n_grow, void* stream) {
    if (int rc = check_csr(W, "sl_rigl_prep")) return rc;
    if (W->nrows == 0) return SL_OK;
    SL_REQUIRE(thr_dev != nullptr && force_idx != nullptr && survivor_bits != nullptr &&
                   n_grow != nullptr,
               "sl_rigl_prep", "NULL argument");
    if (W->ncols > INT_MAX - 32) return fail(SL_ERR_UNSUPPORTED, "sl_rigl_prep: ncols beyond int32");
    rigl_prep_kernel<<<row_grid(W->nrows), 256, 0, as_stream(stream)>>>(
        static_cast<int>(W->nrows), static_cast<int>(W->ncols), W->row_start, W->row_nnz,
        W->col_indices, W->values, thr_dev, force_idx, survivor_bits, n_grow);
    SL_RETURN_IF_LAUNCH_FAILED("sl_rigl_prep");
    return SL_OK;
}

extern "C" int64_t sl_rigl_tile_cols(int64_t M, int64_t K) {
    // The GEMM's tiling: 128x128 where those tiles fill the GPU, else 64x64.
    // SPARSECORE_B200_DG=64|128 forces one (tests and measurements).
    const char* e = std::getenv("SPARSECORE_B200_DG");
    if (e != nullptr) return e[0] == '1' ? 128 : 64;
    const int64_t tiles128 = ((M + BB - 1) / BB) * ((K + BB - 1) / BB);
    return tiles128 >= num_sms() ? 128 : 64;
}

extern "C" int sl_rigl_candidates(const float* dY, const float* X, int64_t M, int64_t K, int64_t N,
                                  const uint32_t* survivor_bits, const int32_t* n_grow,
                                  int64_t lmax, int64_t tile_cols, uint32_t* cand_key,
                                  int32_t* cand_col, int32_t* cand_cnt, int32_t* row_flag,
                                  void* stream) {
    const char* fn = "sl_rigl_candidates";
    if (M < 0 || K < 0 || N < 1) return fail(SL_ERR_INVALID, std::string(fn) + ": bad shape");
    if (M > INT_MAX || K > INT_MAX - 128) return fail(SL_ERR_UNSUPPORTED, std::string(fn) + ": shape beyond int32");
    if (lmax < 1 || lmax > 128) return fail(SL_ERR_INVALID, std::string(fn) + ": lmax must be in [1, 128]");
    if (tile_cols != 64 && tile_cols != 128) return fail(SL_ERR_INVALID, std::string(fn) + ": tile_cols must be 64 or 128");
    if (M == 0 || K == 0) return SL_OK;
    SL_REQUIRE(dY && X && survivor_bits && n_grow && cand_key && cand_col && cand_cnt && row_flag, fn,
               "NULL argument");
    const bool vec4 = (N % 4 == 0) && aligned16(dY) && aligned16(X);
    TopkArgs ta{survivor_bits, n_grow, static_cast<int>(lmax),
                static_cast<int>((K + tile_cols - 1) / tile_cols), cand_key, cand_col, cand_cnt, row_flag};
    cudaStream_t s = as_stream(stream);
    if (tile_cols == 128) {
        const size_t smem = static_cast<size_t>(BB) * 129 * 4;
        auto kern = vec4 ? dense_grad128_kernel<true, true> : dense_grad128_kernel<false, true>;
        if (int rc = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                      static_cast<int>(smem)), fn))
            return rc;
        const dim3 g2(static_cast<unsigned>((K + BB - 1) / BB), static_cast<unsigned>((M + BB - 1) / BB));
        kern<<<g2, kGThreads, smem, s>>>(dY, X, static_cast<int>(M), static_cast<int>(K), N, nullptr, ta);
    } else {
        auto kern = vec4 ? dense_grad_kernel<true, true> : dense_grad_kernel<false, true>;
        const dim3 g(static_cast<unsigned>((K + BK - 1) / BK), static_cast<unsigned>((M + BM - 1) / BM));
        kern<<<g, kGThreads, 0, s>>>(dY, X, static_cast<int>(M), static_cast<int>(K), N, nullptr, ta);
    }
    SL_RETURN_IF_LAUNCH_FAILED(fn);
    return SL_OK;
}

extern "C" int sl_rigl_merge(int64_t M, int64_t K, int64_t lmax, int64_t tile_cols,
                             const uint32_t* cand_key,
                             const int32_t* cand_col, const int32_t* cand_cnt,
                             const int32_t* n_grow, const int32_t* grow_offsets,
                             const int32_t* row_nnz, int32_t* row_flag, int32_t* row_mask,
                             int32_t* grow_cols, void* stream) {
    const char* fn = "sl_rigl_merge";
    if (M < 0 || K < 1 || lmax < 1 || lmax > 128 || (tile_cols != 64 && tile_cols != 128))
        return fail(SL_ERR_INVALID, std::string(fn) + ": bad arguments");
    if (M == 0) return SL_OK;
    SL_REQUIRE(cand_key && cand_col && cand_cnt && n_grow && grow_offsets && row_nnz && row_flag &&
                   row_mask && grow_cols,
               fn, "NULL argument");
    rigl_merge_kernel<<<row_grid(M), 256, 0, as_stream(stream)>>>(
        static_cast<int>(M), static_cast<int>((K + tile_cols - 1) / tile_cols), static_cast<int>(lmax), cand_key,
        cand_col, cand_cnt, n_grow, grow_offsets, row_nnz, row_flag, row_mask, grow_cols);
    SL_RETURN_IF_LAUNCH_FAILED(fn);
    return SL_OK;
}
