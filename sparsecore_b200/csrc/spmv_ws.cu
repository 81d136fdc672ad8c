// Forward SpMM with one dense column (SpMV, also dX = W^T . dY at N = 1):
//   Y[i] = fma chain over row i's live slots in slot order, from +0
// (bit-identical to the reference's csrc/kernels/spmm_avx2.cpp:82-263 with
// N = 1, whose every stage performs y = fma(v_s, X[c_s], y) per element).
//
// The chain of a row is serial, so the row is the unit of parallelism and a
// lane owns one: each CTA serves 32 rows, and the 32 chains advance side by
// side in one consumer warp.  One warp per 32 rows leaves a single warp per
// SM when there are few rows, and one warp cannot issue the copies, the
// gathers and the chain fast enough, so the work is split over three warps
// (see spmv_ws_kernel):
//  * two producer warps stage the rows through shared memory in windows of
//    WIN = 64 slots per row, cooperatively: one 16-byte cp.async per lane,
//    16 lanes per row, so each copy instruction moves two rows' contiguous
//    256-byte runs (coalesced) instead of 32 scattered 16-byte pieces.  A
//    row's windows cover [rs & ~3, ceil4(rs + nnz)): live slots plus at
//    most three on each side, never the row's padding;
//  * after a window lands, the producer lane of each row overwrites the at
//    most three foreign slots at either end of its row with the neutral pair
//    (col -1, value 0) and replaces every col by X[col] in place.  X sits in
//    shared memory with X[-1] = 0 (or is read through L1 with -1 -> 0), so a
//    neutral slot performs y = fma(0, 0, y) = y exactly (y is never -0: it
//    starts at +0 and a round-to-nearest sum is -0 only when both addends
//    are -0);
//  * the consumer warp then walks each window predicate-free: per 4 slots
//    two 128-bit shared loads (x, value) and four FMAs, at FMA latency;
//  * row slices are WIN + 4 words apart, so the 8 lanes of a quarter-warp
//    read distinct bank groups.
#include <cstdlib>

#include "common.cuh"
#include "tma.cuh"

namespace slb {
namespace {

constexpr int64_t kMaxKs = 16384;  // largest K whose X is staged in shared memory
constexpr int kWin = 64;           // slots per row per window
__device__ __forceinline__ uint32_t cvta_shared(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp16(void* dst, const void* src, bool pred) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n"
        " @p cp.async.cg.shared.global [%0], [%1], 16;\n}\n"
        ::"r"(cvta_shared(dst)), "l"(src), "r"(static_cast<int>(pred))
        : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ── Warp-specialised kernel ──────────────────────────────────────────────
// Stage s (window w % S) is handed to the consumer on full[s] (32 producer
// arrivals) and back on empty[s] (one consumer arrival); every wait is
// bounded.  Producer p owns windows w = p, p + 2, ...; it keeps D - 1 =
// S/2 - 1 of them in flight and refills the stage of its window w - 2 once
// the consumer has released it.  (Measured on B200 and not kept: a
// single-warp version of the same windows, 1.2-1.9x slower with few rows,
// and 1-D bulk copies of each row's window instead of cp.async, up to 1.9x
// slower.)
template <int WIN, int RPC = 32>
struct WsShape {
    static constexpr int kStride = WIN + 4;                 // words per row slice
    static constexpr int kStageWords = RPC * kStride;       // one array, one stage
};

// RPC = rows per CTA: 32, or 16 (lanes 16-31 idle) so that with few rows
// twice as many CTAs -- and copies in flight -- share the SMs.
template <int WIN, int S, bool KS, int RPC = 32>
__global__ void __launch_bounds__(96, 1)
spmv_ws_kernel(int M, int64_t K, int64_t cap_total, const int32_t* __restrict__ row_start,
               const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
               const float* __restrict__ vals, const float* __restrict__ X,
               float* __restrict__ Y, unsigned* status) {
    static_assert(S % 2 == 0 && S >= 4, "two producers, at least two stages each");
    constexpr int D = S / 2;
    constexpr int kStr = WsShape<WIN>::kStride;
    constexpr int kSW = WsShape<WIN, RPC>::kStageWords;
    constexpr size_t kRing = size_t(S) * kSW * 4 * 2;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[S];
    __shared__ __align__(8) uint64_t empty[S];
    __shared__ __align__(8) uint64_t xbar;
    int* cring = reinterpret_cast<int*>(smem_raw);
    float* vring = reinterpret_cast<float*>(smem_raw + kRing / 2);
    float* xs = reinterpret_cast<float*>(smem_raw + kRing + 16);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * RPC + lane;
    const bool live = lane < RPC && row < M;
    const int rs = live ? __ldg(row_start + row) : 0;
    const int nn = live ? __ldg(row_nnz + row) : 0;
    const int a = rs & ~3;
    const int e = nn > 0 ? ((rs + nn + 3) & ~3) : a;
    const int cap4 = static_cast<int>(cap_total & ~int64_t(3));
    const int ecopy = e > cap4 ? cap4 : e;
    const int nw = (e - a + WIN - 1) / WIN;
    const int NW = __reduce_max_sync(0xffffffffu, nw);

    if (threadIdx.x == 0) {
        for (int b = 0; b < S; ++b) {
            mbar_init(&full[b], 32);
            mbar_init(&empty[b], 1);
        }
        mbar_init(&xbar, 32);
        fence_barrier_init();
    }
    __syncthreads();

    int* cslice = cring + lane * kStr;
    float* vslice = vring + lane * kStr;
    bool ok = true;

    if (warp == 0) {  // consumer: X staging, then the chains
        if (KS) {
            if ((K % 4 == 0) && ((reinterpret_cast<uintptr_t>(X) & 15u) == 0)) {
                for (int64_t k = 4 * lane; k < K; k += 128) cp16(xs + k, X + k, true);
            } else {
                for (int64_t k = lane; k < K; k += 32) xs[k] = __ldg(X + k);
            }
            if (lane == 0) xs[-1] = 0.0f;
            cp_commit();
            cp_wait<0>();
        }
        mbar_arrive(&xbar);
        float y = 0.0f;
        for (int w = 0; w < NW; ++w) {
            const int b = w % S;
            if (!mbar_wait(&full[b], static_cast<unsigned>((w / S) & 1), status)) { ok = false; break; }
            if (w < nw) {
                const int s0 = a + w * WIN;
                const int ng = ((s0 + WIN < e ? s0 + WIN : e) - s0) >> 2;
                const float4* x4 = reinterpret_cast<const float4*>(cslice + b * kSW);
                const float4* v4 = reinterpret_cast<const float4*>(vslice + b * kSW);
#pragma unroll 8
                for (int g = 0; g < ng; ++g) {
                    const float4 x = x4[g];
                    const float4 v = v4[g];
                    y = fmaf(v.x, x.x, y);
                    y = fmaf(v.y, x.y, y);
                    y = fmaf(v.z, x.z, y);
                    y = fmaf(v.w, x.w, y);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[b]);
        }
        if (ok && live) Y[row] = y;
        return;
    }

    // producers
    const int p = warp - 1;
    constexpr int LPR = WIN / 4 < 32 ? WIN / 4 : 32;  // lanes per row in a copy
    constexpr int RPI = 32 / LPR;                     // rows per copy instruction
    const int sub = lane / LPR, li = lane % LPR;
    auto issue = [&](int w) {
        const int b = w % S;
        int* cdst = cring + b * kSW + sub * kStr + 4 * li;
        float* vdst = vring + b * kSW + sub * kStr + 4 * li;
#pragma unroll 4
        for (int rr = 0; rr < RPC; rr += RPI) {
            const int r = rr + sub;
            const int ra = __shfl_sync(0xffffffffu, a, r);
            const int re = __shfl_sync(0xffffffffu, ecopy, r);
#pragma unroll
            for (int h = 0; h < WIN / (4 * LPR); ++h) {
                const int slot = ra + w * WIN + 4 * (li + LPR * h);
                const bool pr = slot < re;
                const int src = pr ? slot : 0;
                cp16(cdst + rr * kStr + 4 * LPR * h, cols + src, pr);
                cp16(vdst + rr * kStr + 4 * LPR * h, vals + src, pr);
            }
        }
        cp_commit();
    };
#pragma unroll
    for (int i = 0; i < D - 1; ++i) {
        const int w = p + 2 * i;
        if (w < NW) issue(w);
        else cp_commit();
    }
    if (KS && !mbar_wait(&xbar, 0u, status)) ok = false;
    for (int w = p; w < NW && ok; w += 2) {
        const int b = w % S;
        const int wn = w + 2 * (D - 1);  // refill: into the stage of window w - 2
        if (wn < NW) {
            if (w >= 2 && !mbar_wait(&empty[(w - 2) % S], static_cast<unsigned>(((w - 2) / S) & 1), status)) {
                ok = false;
                break;
            }
            issue(wn);
        } else {
            cp_commit();
        }
        cp_wait<D - 1>();  // this thread's copies of window w have landed
        __syncwarp();      // ... and every other lane's
        if (w < nw) {
            int* cb = cslice + b * kSW;
            float* vb = vslice + b * kSW;
            const int s0 = a + w * WIN;
            const int s1 = s0 + WIN < e ? s0 + WIN : e;
            if (w == 0)
                for (int q = a; q < rs; ++q) { cb[q - s0] = -1; vb[q - s0] = 0.0f; }
            if (w == nw - 1) {
                for (int q = ecopy > s0 ? ecopy : s0; q < e; ++q) {
                    const bool in = q < rs + nn;
                    cb[q - s0] = in ? __ldg(cols + q) : -1;
                    vb[q - s0] = in ? __ldg(vals + q) : 0.0f;
                }
                for (int q = rs + nn; q < e && q < ecopy; ++q) { cb[q - s0] = -1; vb[q - s0] = 0.0f; }
            }
            int4* c4 = reinterpret_cast<int4*>(cb);
            float4* x4 = reinterpret_cast<float4*>(cb);
            const int ng = (s1 - s0) >> 2;
#pragma unroll 8
            for (int g = 0; g < ng; ++g) {
                const int4 c = c4[g];
                float4 x;
                if (KS) {
                    x = make_float4(xs[c.x], xs[c.y], xs[c.z], xs[c.w]);
                } else {
                    x.x = c.x >= 0 ? __ldg(X + c.x) : 0.0f;
                    x.y = c.y >= 0 ? __ldg(X + c.y) : 0.0f;
                    x.z = c.z >= 0 ? __ldg(X + c.z) : 0.0f;
                    x.w = c.w >= 0 ? __ldg(X + c.w) : 0.0f;
                }
                x4[g] = x;
            }
        }
        mbar_arrive(&full[b]);
    }
    cp_wait<0>();
}

template <int WIN, int S, bool KS, int RPC>
int launch_ws(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    unsigned* status = device_status_word();
    if (status == nullptr) return -1;
    const size_t smem = size_t(S) * WsShape<WIN, RPC>::kStageWords * 4 * 2 + 16 +
                        (KS ? static_cast<size_t>(K) * 4 : 0);
    auto kern = spmv_ws_kernel<WIN, S, KS, RPC>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int M = static_cast<int>(W->nrows);
    note_kernel("spmv_ws_kernel");
    kern<<<(M + RPC - 1) / RPC, 96, smem, s>>>(M, K, W->total_capacity, W->row_start, W->row_nnz,
                                               W->col_indices, W->values, X, Y, status);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd (N = 1, warp-specialised)");
    return SL_OK;
}

template <int S, int RPC>
int launch_ws_x(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s, bool ks) {
    return ks ? launch_ws<64, S, true, RPC>(W, X, K, Y, s) : launch_ws<64, S, false, RPC>(W, X, K, Y, s);
}

}  // namespace

// At most one CTA per SM (few rows): 8 windows per CTA, 3 in flight per
// producer.  More rows: 4 windows, two CTAs per SM.  X is staged in shared
// memory when it is at most half the bytes of the CTA's rows (otherwise the
// per-CTA staging costs more than it saves, e.g. 99% sparsity) and fits.
// SPARSECORE_B200_N1_ST=4|8 and SPARSECORE_B200_N1_XS=0|1 override
// (measurements and tests).  Returns -1 when the kernel cannot be
// configured (the caller falls back).
int launch_spmv_ws(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    if (!aligned16(W->col_indices) || !aligned16(W->values) || W->nrows <= 0 || K < 1 ||
        W->nrows > INT_MAX - 32 || W->total_capacity > INT_MAX - 4 * kWin * 16)
        return -1;
    const int64_t warps = (W->nrows + 31) / 32;
    int st = warps <= num_sms() ? 8 : 4;
    if (const char* e = std::getenv("SPARSECORE_B200_N1_ST")) {
        const int v = std::atoi(e);
        if (v == 4 || v == 8) st = v;
    }
    const double row_bytes = 8.0 * static_cast<double>(W->total_capacity) / 1.2 / W->nrows;
    bool ks = K <= kMaxKs && 4.0 * K <= 0.5 * 32.0 * row_bytes;
    if (const char* e = std::getenv("SPARSECORE_B200_N1_XS")) ks = (e[0] == '1') && K <= kMaxKs;
    // Rows per CTA: 32.  16-row CTAs (two per SM when rows are few) measured
    // on B200: 4096 x 4096 at 50% sparsity 4% faster, at 90% 7% slower; the
    // dX of 16384 x 4096 (W^T: 4096 rows of 1600-8200 slots, X staged per
    // CTA) 1.6x slower.  Kept behind SPARSECORE_B200_N1_RPC=16 (tests).
    int rpc = 32;
    if (const char* e = std::getenv("SPARSECORE_B200_N1_RPC")) rpc = std::atoi(e) == 16 ? 16 : 32;
    if (rpc == 16) return st == 8 ? launch_ws_x<8, 16>(W, X, K, Y, s, ks) : launch_ws_x<4, 16>(W, X, K, Y, s, ks);
    return st == 8 ? launch_ws_x<8, 32>(W, X, K, Y, s, ks) : launch_ws_x<4, 32>(W, X, K, Y, s, ks);
}

}  // namespace slb
