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

template <bool VEC4>
__global__ void __launch_bounds__(kGThreads)
dense_grad_kernel(const float* __restrict__ A, const float* __restrict__ B, int M, int K,
                  int64_t N, float* __restrict__ G) {
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

template <bool VEC4>
__global__ void __launch_bounds__(kGThreads)
dense_grad128_kernel(const float* __restrict__ A, const float* __restrict__ B, int M, int K,
                     int64_t N, float* __restrict__ G) {
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
            dense_grad128_kernel<true><<<g2, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                                static_cast<int>(K), N, G);
        else
            dense_grad128_kernel<false><<<g2, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                                 static_cast<int>(K), N, G);
        SL_RETURN_IF_LAUNCH_FAILED("sl_dense_grad");
        return SL_OK;
    }
    const dim3 grid(static_cast<unsigned>((K + BK - 1) / BK), static_cast<unsigned>((M + BM - 1) / BM));
    if (vec4)
        dense_grad_kernel<true><<<grid, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                           static_cast<int>(K), N, G);
    else
        dense_grad_kernel<false><<<grid, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                            static_cast<int>(K), N, G);
    SL_RETURN_IF_LAUNCH_FAILED("sl_dense_grad");
    return SL_OK;
}
