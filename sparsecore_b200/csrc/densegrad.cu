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
    const dim3 grid(static_cast<unsigned>((K + BK - 1) / BK), static_cast<unsigned>((M + BM - 1) / BM));
    const bool vec4 = (N % 4 == 0) && aligned16(dY) && aligned16(X);
    if (vec4)
        dense_grad_kernel<true><<<grid, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                           static_cast<int>(K), N, G);
    else
        dense_grad_kernel<false><<<grid, kGThreads, 0, s>>>(dY, X, static_cast<int>(M),
                                                            static_cast<int>(K), N, G);
    SL_RETURN_IF_LAUNCH_FAILED("sl_dense_grad");
    return SL_OK;
}
