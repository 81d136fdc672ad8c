// N = 32 (one warp-wide column tile): forward SpMM / dX and SDDMM dW with
// the gathered X rows staged through shared memory by cp.async.
//
// With 32 dense columns every slot needs one 128-byte X row, and each row is
// used by exactly one slot, so the kernels are bound by how many of those
// gathers are in flight.  Loading them into registers (LDG) leaves a warp
// waiting one L2 round trip per group of slots; here every warp keeps R
// chunks of 32 slots' X rows in flight in its own shared-memory ring
// (cp.async, 16 bytes per lane, four 128-byte rows per instruction), and the
// (col, value) pairs of the next chunks are already in registers four chunks
// ahead.  A warp owns one W row at a time.
//
// Numerics as the other kernels (bit-identical to the reference CPU ones):
//  * forward: lane j accumulates y[j] = fma(v_s, X[c_s, j], y[j]) over the
//    row's slots in slot order (csrc/kernels/spmm_avx2.cpp:82-263);
//  * SDDMM: lane u evaluates slot u's dot in the AVX2 order of
//    csrc/kernels/spmm_grad_avx2.cpp:112-257 with N = 32: 16 chains over two
//    16-wide steps, the lane-wise sum of the two 8-wide halves, the
//    horizontal reduction ((l0+h0)+(l2+h2)) + ((l1+h1)+(l3+h3)), no tail.
//    The dY row sits in the lane's registers (broadcast load); the X rows
//    are staged with their 16-byte pieces XOR-swizzled by the row index, so
//    the 8 lanes of a quarter-warp reading piece p of 8 different rows hit 8
//    different bank groups.
#include <cstdlib>

#include "common.cuh"

namespace slb {
namespace {

constexpr int kG32Warps = 4;              // warps per CTA
constexpr int kG32Q = 4;                  // (col, value) register ring, chunks
constexpr int kRowFloats = 32;            // X row = 128 bytes
constexpr int kChunkFloats = 32 * kRowFloats;

__device__ __forceinline__ void g32_cp16(float* dst, const float* src, bool pred) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n"
        " @p cp.async.cg.shared.global [%0], [%1], 16;\n}\n"
        ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src),
        "r"(static_cast<int>(pred))
        : "memory");
}
__device__ __forceinline__ void g32_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void g32_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Copy the X rows of one chunk (slots whose col is held by lane u in `c`,
// u < cnt) into `buf` (32 rows x 128 bytes).  Lane l copies piece l & 7 of
// rows (l >> 3) + 4p, p = 0..7; SWZ stores piece q of row u at q ^ (u & 7).
template <bool SWZ>
__device__ __forceinline__ void g32_issue(float* buf, const float* __restrict__ X, int c, int cnt,
                                          int lane) {
    const int piece = lane & 7;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const int u = (lane >> 3) + 4 * p;
        const int cu = __shfl_sync(0xffffffffu, c, u);
        const int q = SWZ ? (piece ^ (u & 7)) : piece;
        g32_cp16(buf + u * kRowFloats + 4 * q, X + cu * kRowFloats + 4 * piece, u < cnt);
    }
}

// KIND 0 = forward (Y row = W row . X), 1 = SDDMM (dW slots of the row).
template <int KIND, int R>
__global__ void __launch_bounds__(kG32Warps * 32)
gather32_kernel(int M, const int32_t* __restrict__ row_start, const int32_t* __restrict__ row_nnz,
                const int32_t* __restrict__ row_capacity, const int32_t* __restrict__ cols,
                const float* __restrict__ vals, const float* __restrict__ X,
                const float* __restrict__ dY, float* __restrict__ out) {
    extern __shared__ __align__(16) float g32_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* ring = g32_smem + static_cast<size_t>(warp) * R * kChunkFloats;
    const int warps = gridDim.x * kG32Warps;
    for (int row = blockIdx.x * kG32Warps + warp; row < M; row += warps) {
        const int rs = __ldg(row_start + row);
        const int nn = __ldg(row_nnz + row);
        const int nch = (nn + 31) >> 5;
        if (KIND == 1) {  // padding slots of the row -> 0
            const int cp = __ldg(row_capacity + row);
            for (int k = nn + lane; k < cp; k += 32) out[rs + k] = 0.0f;
        }
        int cr[kG32Q];
        float vr[kG32Q];
#pragma unroll
        for (int j = 0; j < kG32Q; ++j) {
            const int k = 32 * j + lane;
            cr[j] = k < nn ? __ldg(cols + rs + k) : 0;
            vr[j] = (KIND == 0 && k < nn) ? __ldg(vals + rs + k) : 0.0f;
        }
        float d[KIND == 1 ? 32 : 1];
        if constexpr (KIND == 1) {
            const float4* dr = reinterpret_cast<const float4*>(dY + static_cast<int64_t>(row) * 32);
#pragma unroll
            for (int p = 0; p < 8; ++p) {
                const float4 t = __ldg(dr + p);
                d[4 * p] = t.x; d[4 * p + 1] = t.y; d[4 * p + 2] = t.z; d[4 * p + 3] = t.w;
            }
        }
#pragma unroll
        for (int j = 0; j < R - 1; ++j) {
            if (j < nch) g32_issue<KIND == 1>(ring + j * kChunkFloats, X, cr[j], nn - 32 * j, lane);
            g32_commit();
        }
        float acc = 0.0f;
        for (int kb = 0; kb < nch; kb += kG32Q) {
#pragma unroll
            for (int j = 0; j < kG32Q; ++j) {
                const int k = kb + j;
                if (k >= nch) break;
                const int kn = k + R - 1;  // chunk whose copies go out now
                if (kn < nch)
                    g32_issue<KIND == 1>(ring + (kn % R) * kChunkFloats, X, cr[(j + R - 1) % kG32Q],
                                         nn - 32 * kn, lane);
                g32_commit();
                g32_wait<R - 1>();
                __syncwarp();
                const float* buf = ring + (k % R) * kChunkFloats;
                const int cnt = min(32, nn - 32 * k);
                if constexpr (KIND == 0) {
#pragma unroll 8
                    for (int u = 0; u < cnt; ++u)
                        acc = fmaf(__shfl_sync(0xffffffffu, vr[j], u), buf[u * kRowFloats + lane], acc);
                } else if (lane < cnt) {
                    const float4* xr = reinterpret_cast<const float4*>(buf + lane * kRowFloats);
                    const int sw = lane & 7;
                    float a[16];
#pragma unroll
                    for (int p = 0; p < 4; ++p) {  // j = 0..15: chains start at fma(d, x, 0)
                        const float4 x = xr[p ^ sw];
                        a[4 * p] = fmaf(d[4 * p], x.x, 0.0f);
                        a[4 * p + 1] = fmaf(d[4 * p + 1], x.y, 0.0f);
                        a[4 * p + 2] = fmaf(d[4 * p + 2], x.z, 0.0f);
                        a[4 * p + 3] = fmaf(d[4 * p + 3], x.w, 0.0f);
                    }
#pragma unroll
                    for (int p = 4; p < 8; ++p) {  // j = 16..31
                        const float4 x = xr[p ^ sw];
                        const int t = 4 * (p - 4);
                        a[t] = fmaf(d[4 * p], x.x, a[t]);
                        a[t + 1] = fmaf(d[4 * p + 1], x.y, a[t + 1]);
                        a[t + 2] = fmaf(d[4 * p + 2], x.z, a[t + 2]);
                        a[t + 3] = fmaf(d[4 * p + 3], x.w, a[t + 3]);
                    }
#pragma unroll
                    for (int t = 0; t < 8; ++t) a[t] = __fadd_rn(a[t], a[t + 8]);
                    float s4[4];
#pragma unroll
                    for (int t = 0; t < 4; ++t) s4[t] = __fadd_rn(a[t], a[t + 4]);
                    out[rs + 32 * k + lane] =
                        __fadd_rn(__fadd_rn(s4[0], s4[2]), __fadd_rn(s4[1], s4[3]));
                }
                __syncwarp();  // the buffer is refilled R - 1 chunks later
                // Refill ring entry j with chunk k + Q.
                const int kq = 32 * (k + kG32Q) + lane;
                cr[j] = kq < nn ? __ldg(cols + rs + kq) : 0;
                if (KIND == 0) vr[j] = kq < nn ? __ldg(vals + rs + kq) : 0.0f;
            }
        }
        g32_wait<0>();
        if (KIND == 0) out[static_cast<int64_t>(row) * 32 + lane] = acc;
    }
}

template <int KIND, int R>
int launch_g32(const sl_csr* W, const float* X, const float* dY, float* out, cudaStream_t s) {
    const size_t smem = static_cast<size_t>(kG32Warps) * R * kChunkFloats * 4;
    auto kern = gather32_kernel<KIND, R>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kG32Warps * 32, smem) !=
            cudaSuccess || per_sm < 1)
        return -1;
    const int M = static_cast<int>(W->nrows);
    int64_t blocks = (static_cast<int64_t>(M) + kG32Warps - 1) / kG32Warps;
    const int64_t max_blocks = static_cast<int64_t>(num_sms()) * per_sm;
    if (blocks > max_blocks) blocks = max_blocks;
    note_kernel(KIND == 0 ? "gather32_fwd_kernel" : "gather32_sddmm_kernel");
    kern<<<static_cast<unsigned>(blocks), kG32Warps * 32, smem, s>>>(
        M, W->row_start, W->row_nnz, W->row_capacity, W->col_indices, W->values, X, dY, out);
    SL_RETURN_IF_LAUNCH_FAILED(KIND == 0 ? "sl_spmm_fwd (N = 32)" : "sl_sddmm_dw (N = 32)");
    return SL_OK;
}

bool g32_applies(const sl_csr* W, const float* X, const float* other) {
    return W->nrows > 0 && W->ncols > 0 && W->ncols * 32 <= INT_MAX && aligned16(X) &&
           aligned16(other) && W->nrows <= INT_MAX;
}

}  // namespace

bool gather32_enabled() {
    const char* e = std::getenv("SPARSECORE_B200_N32");
    return e == nullptr || e[0] != 'r';
}

bool gather32_forced() {
    const char* e = std::getenv("SPARSECORE_B200_N32");
    return e != nullptr && e[0] == 'g';
}

// Three chunks in flight per warp (12 KB of X rows); -1 when not applicable.
int launch_gather32_fwd(const sl_csr* W, const float* X, float* Y, cudaStream_t s) {
    if (!g32_applies(W, X, Y)) return -1;
    return launch_g32<0, 3>(W, X, nullptr, Y, s);
}

int launch_gather32_sddmm(const sl_csr* W, const float* dY, const float* X, float* dW,
                          cudaStream_t s) {
    if (!g32_applies(W, X, dY)) return -1;
    return launch_g32<1, 3>(W, X, dY, dW, s);
}

}  // namespace slb
