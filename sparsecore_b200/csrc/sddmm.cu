// SDDMM weight gradient at live slots:
//   dW[slot] = <dY[i,:], X[col[slot],:]>   (fp32, padding slots -> 0)
//
// Numerics: the dot is evaluated in exactly the lane order of the reference
// AVX2 kernel (csrc/kernels/spmm_grad_avx2.cpp:112-257), so results are
// bit-identical:  16 FMA chains (lane t takes j = 16m + t, m ascending;
// chains 0-7 are the first 256-bit accumulator, 8-15 the second), the
// lane-wise sum of the two accumulators, one optional 8-wide FMA step, the
// horizontal reduction ((l0+h0)+(l2+h2)) + ((l1+h1)+(l3+h3)), then the
// scalar tail over the last N mod 8 elements as the reference's compiler
// emits it (an in-order vectorised reduction): whole groups of 4 terms as
// rounded products added one by one, the final (tail mod 4) terms as FMAs.
//
// GPU mapping: a quad of 4 lanes evaluates one slot's dot; quad lane q owns
// chains 4q..4q+3 and reads X[c, 16m+4q .. +3] (and the matching dY) as one
// 128-bit load per step, so each quad streams a contiguous 64-byte piece of
// the X row per step.  A CTA of 64 quads works on one row of W at a time
// (all its quads share the row's dY, which stays L1-resident) and each quad
// carries S slots of that row concurrently, reusing each dY vector S times.
// CTAs sweep rows grid-stride.
#include "common.cuh"

namespace slb {
namespace {

constexpr int kDwThreads = 256;
constexpr int kQuads = kDwThreads / 4;

template <bool VEC4>
__device__ __forceinline__ float4 load4(const float* p) {
    if constexpr (VEC4) {
        return __ldg(reinterpret_cast<const float4*>(p));
    } else {
        return make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
    }
}

__device__ __forceinline__ void fma4(float4 a, float4 b, float4& acc) {
    acc.x = fmaf(a.x, b.x, acc.x);
    acc.y = fmaf(a.y, b.y, acc.y);
    acc.z = fmaf(a.z, b.z, acc.z);
    acc.w = fmaf(a.w, b.w, acc.w);
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                       __fadd_rn(a.w, b.w));
}

__device__ __forceinline__ float4 shfl_xor4(float4 v, int m) {
    return make_float4(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m),
                       __shfl_xor_sync(0xffffffffu, v.z, m), __shfl_xor_sync(0xffffffffu, v.w, m));
}

template <bool VEC4, int S>
__global__ void __launch_bounds__(kDwThreads)
sddmm_kernel(int M, int64_t N, const int32_t* __restrict__ row_start,
             const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ row_capacity,
             const int32_t* __restrict__ cols, const float* __restrict__ dY,
             const float* __restrict__ X, float* __restrict__ dW) {
    const int q = threadIdx.x & 3;
    const int quad = threadIdx.x >> 2;
    const int64_t nfull = N >> 4;
    const int rem = static_cast<int>(N & 15);
    const int64_t jtail = nfull * 16 + (rem >= 8 ? 8 : 0);
    const int64_t jfma = jtail + ((N - jtail) & ~static_cast<int64_t>(3));

    for (int row = blockIdx.x; row < M; row += gridDim.x) {
        const int rs = __ldg(row_start + row);
        const int nn = __ldg(row_nnz + row);
        const int cap = __ldg(row_capacity + row);
        for (int k = nn + threadIdx.x; k < cap; k += kDwThreads) dW[rs + k] = 0.0f;
        const float* dyr = dY + static_cast<int64_t>(row) * N;

        for (int kb = 0; kb < nn; kb += kQuads * S) {
            const float* xr[S];
            bool act[S];
#pragma unroll
            for (int u = 0; u < S; ++u) {
                const int k = kb + quad + kQuads * u;
                act[u] = k < nn;
                const int c = act[u] ? __ldg(cols + rs + k) : 0;
                xr[u] = X + static_cast<int64_t>(c) * N;
            }
            float4 acc[S];
#pragma unroll
            for (int u = 0; u < S; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);

            // 16-wide steps: quad lane q advances chains 4q..4q+3.
#pragma unroll 2
            for (int64_t m = 0; m < nfull; ++m) {
                const int64_t j = m * 16 + q * 4;
                const float4 d = load4<VEC4>(dyr + j);
#pragma unroll
                for (int u = 0; u < S; ++u)
                    if (act[u]) fma4(d, load4<VEC4>(xr[u] + j), acc[u]);
            }
            // acc = acc_a + acc_b (lanes 0,1 receive lanes 2,3).
#pragma unroll
            for (int u = 0; u < S; ++u) {
                const float4 o = shfl_xor4(acc[u], 2);
                if (q < 2) acc[u] = add4(acc[u], o);
            }
            // Optional 8-wide step on lanes 0,1 (chains 0-3 and 4-7).
            if (rem >= 8 && q < 2) {
                const int64_t j = nfull * 16 + q * 4;
                const float4 d = load4<VEC4>(dyr + j);
#pragma unroll
                for (int u = 0; u < S; ++u) fma4(d, load4<VEC4>(xr[u] + j), acc[u]);
            }
            // Horizontal reduction: lane 0 holds acc[0..3], lane 1 acc[4..7].
#pragma unroll
            for (int u = 0; u < S; ++u) {
                const float4 hi = shfl_xor4(acc[u], 1);
                if (q == 0 && act[u]) {
                    const float4 s4 = add4(acc[u], hi);
                    float r = __fadd_rn(__fadd_rn(s4.x, s4.z), __fadd_rn(s4.y, s4.w));
                    for (int64_t j = jtail; j < jfma; ++j)
                        r = __fadd_rn(r, __fmul_rn(__ldg(dyr + j), __ldg(xr[u] + j)));
                    for (int64_t j = jfma; j < N; ++j) r = fmaf(__ldg(dyr + j), __ldg(xr[u] + j), r);
                    dW[rs + kb + quad + kQuads * u] = r;
                }
            }
        }
    }
}

template <bool VEC4>
int launch_dw(const sl_csr* W, const float* dY, const float* X, int64_t N, float* dW,
              cudaStream_t s) {
    const int M = static_cast<int>(W->nrows);
    int blocks = num_sms() * 6;
    if (blocks > M) blocks = M;
    sddmm_kernel<VEC4, 4><<<blocks, kDwThreads, 0, s>>>(M, N, W->row_start, W->row_nnz,
                                                        W->row_capacity, W->col_indices, dY, X, dW);
    SL_RETURN_IF_LAUNCH_FAILED("sl_sddmm_dw");
    return SL_OK;
}

}  // namespace
}  // namespace slb

using namespace slb;

extern "C" int sl_sddmm_dw(const sl_csr* W, const float* dY, const float* X, int64_t N, float* dW,
                           void* stream) {
    if (int rc = check_csr(W, "sl_sddmm_dw")) return rc;
    if (N < 0) return fail(SL_ERR_INVALID, "sl_sddmm_dw: negative N");
    if (W->total_capacity == 0 || W->nrows == 0) return SL_OK;
    if (dW == nullptr) return fail(SL_ERR_INVALID, "sl_sddmm_dw: NULL dW");
    if (N > 0 && (dY == nullptr || (W->ncols > 0 && X == nullptr)))
        return fail(SL_ERR_INVALID, "sl_sddmm_dw: NULL dense operand");
    cudaStream_t s = as_stream(stream);
    const bool vec4 = (N % 4 == 0) && aligned16(X) && aligned16(dY);
    return vec4 ? launch_dw<true>(W, dY, X, N, dW, s) : launch_dw<false>(W, dY, X, N, dW, s);
}
