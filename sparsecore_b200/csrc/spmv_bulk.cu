// Forward SpMM with one dense column (SpMV, also dX = W^T . dY at N = 1):
//   Y[i] = fma chain over row i's live slots in slot order, from +0
// (bit-identical to the reference's csrc/kernels/spmm_avx2.cpp:82-263 with
// N = 1, whose every stage performs y = fma(v_s, X[c_s], y) per element).
//
// The chain of a row is serial, so the row is the unit of parallelism and a
// lane owns one: a one-warp CTA runs 32 rows' chains side by side.  What
// bounds such a kernel is how many bytes each SM keeps in flight and how
// few instructions a lane spends per slot, so:
//  * the warp stages its 32 rows through shared memory in windows of WIN =
//    64 slots per row, ST windows in flight, and it copies them
//    cooperatively: one 16-byte cp.async per lane, 16 lanes per row, so each
//    copy instruction moves two rows' contiguous 256-byte runs (coalesced)
//    instead of 32 scattered 16-byte pieces.  A row's windows cover
//    [rs & ~3, ceil4(rs + nnz)): live slots plus at most three on each side,
//    never the row's padding;
//  * after a window lands, the lane overwrites the at most three foreign
//    slots at either end of its own row with the neutral pair (col -1,
//    value 0).  X sits in shared memory with X[-1] = 0, so a neutral slot
//    performs y = fma(0, 0, y) = y exactly (y is never -0: it starts at +0
//    and a round-to-nearest sum is -0 only when both addends are -0).  The
//    walk over a window is then predicate-free, in two passes: a gather
//    pass replaces each col by X[col] in place (independent loads, many in
//    flight), then the chain pass reads (value, x) as 128-bit pairs and
//    runs at FMA latency;
//  * row slices are WIN + 4 words apart, so the 8 lanes of a quarter-warp
//    read distinct bank groups.
// K above kMaxKs keeps X in global memory (read through L1, -1 -> 0).
#include <cstdlib>

#include "common.cuh"
#include "tma.cuh"

namespace slb {
namespace {

constexpr int64_t kMaxKs = 16384;  // largest K whose X is staged in shared memory
constexpr int kWin = 64;           // slots per row per window
constexpr int kLpr = kWin / 4;     // lanes per row in a copy instruction
constexpr int kRpi = 32 / kLpr;    // rows per copy instruction
constexpr int kStride = kWin + 4;  // words per row slice

template <int ST>
struct CoopShape {
    static constexpr int kStageWords = 32 * kStride;                   // one array, one stage
    static constexpr size_t kRing = size_t(ST) * kStageWords * 4 * 2;  // cols + values
    static constexpr size_t kXOff = kRing + 16;                         // X[-1] at kRing + 12
};

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

template <int ST, bool KS>
__global__ void __launch_bounds__(32)
spmv_coop_kernel(int M, int64_t K, int64_t cap_total, const int32_t* __restrict__ row_start,
                 const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                 const float* __restrict__ vals, const float* __restrict__ X,
                 float* __restrict__ Y) {
    using S = CoopShape<ST>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    int* cring = reinterpret_cast<int*>(smem_raw);
    float* vring = reinterpret_cast<float*>(smem_raw + S::kRing / 2);
    float* xs = reinterpret_cast<float*>(smem_raw + S::kXOff);

    const int lane = threadIdx.x;
    const int row = blockIdx.x * 32 + lane;
    const bool live = row < M;
    const int64_t rs = live ? __ldg(row_start + row) : 0;
    const int64_t nn = live ? __ldg(row_nnz + row) : 0;
    const int64_t a = rs & ~int64_t(3);                            // first staged slot
    const int64_t e = nn > 0 ? ((rs + nn + 3) & ~int64_t(3)) : a;  // one past the last
    // Copies stop at the arrays' last whole 16-byte group; the at most three
    // slots after it are read with plain loads.
    const int64_t cap4 = cap_total & ~int64_t(3);
    const int64_t ecopy = e > cap4 ? cap4 : e;
    const int nw = static_cast<int>((e - a + kWin - 1) / kWin);
    const int NW = __reduce_max_sync(0xffffffffu, nw);

    // Copy window w of all 32 rows: lanes [kLpr*j, kLpr*j + kLpr) copy row
    // rr + j, group li = lane % kLpr of the window.  Slot indices fit in 32
    // bits (row_start is int32), which keeps the address math short.
    const int sub = lane / kLpr, li = lane % kLpr;
    const int a32 = static_cast<int>(a), ec32 = static_cast<int>(ecopy);
    auto issue = [&](int w) {
        const int b = w % ST;
        const int woff = w * kWin + 4 * li;
        int* cdst = cring + b * S::kStageWords + sub * kStride + 4 * li;
        float* vdst = vring + b * S::kStageWords + sub * kStride + 4 * li;
#pragma unroll
        for (int rr = 0; rr < 32; rr += kRpi) {
            const int r = rr + sub;
            const int slot = __shfl_sync(0xffffffffu, a32, r) + woff;
            const bool p = slot < __shfl_sync(0xffffffffu, ec32, r);
            const int src = p ? slot : 0;
            cp16(cdst + rr * kStride, cols + src, p);
            cp16(vdst + rr * kStride, vals + src, p);
        }
        cp_commit();
    };

    if (KS) {
        if ((K % 4 == 0) && ((reinterpret_cast<uintptr_t>(X) & 15u) == 0)) {
            for (int64_t k = 4 * lane; k < K; k += 128) cp16(xs + k, X + k, true);
        } else {
            for (int64_t k = lane; k < K; k += 32) xs[k] = __ldg(X + k);
        }
        if (lane == 0) xs[-1] = 0.0f;
    }
    cp_commit();  // X: the oldest group
#pragma unroll
    for (int w = 0; w < ST - 1; ++w) issue(w);  // empty groups past NW are harmless

    int* cslice = cring + lane * kStride;
    float* vslice = vring + lane * kStride;
    float y = 0.0f;
    for (int w = 0; w < NW; ++w) {
        issue(w + ST - 1);  // refill the buffer freed at w - 1 (empty past NW)
        cp_wait<ST - 1>();  // this thread's copies of window w (and X) have landed
        __syncwarp();       // ... and every other lane's
        if (w < nw) {
            const int b = w % ST;
            int* cb = cslice + b * S::kStageWords;
            float* vb = vslice + b * S::kStageWords;
            const int64_t s0 = a + static_cast<int64_t>(w) * kWin;
            const int64_t s1 = s0 + kWin < e ? s0 + kWin : e;
            // Fix-ups in the lane's own row slice: the foreign slots before
            // the row (first window), the uncopied tail group (plain loads)
            // and the foreign slots after the row (last window).
            if (w == 0)
                for (int64_t q = a; q < rs; ++q) { cb[q - s0] = -1; vb[q - s0] = 0.0f; }
            if (w == nw - 1) {
                for (int64_t q = ecopy > s0 ? ecopy : s0; q < e; ++q) {
                    const bool in = q < rs + nn;
                    cb[q - s0] = in ? __ldg(cols + q) : -1;
                    vb[q - s0] = in ? __ldg(vals + q) : 0.0f;
                }
                for (int64_t q = rs + nn; q < e && q < ecopy; ++q) { cb[q - s0] = -1; vb[q - s0] = 0.0f; }
            }
            // Two passes over the window.  (1) Gather: X[c] replaces c in
            // place -- groups are independent, so the loads of many groups
            // are in flight together.  (2) The serial chain: per 4 slots two
            // 128-bit loads (value, x) that do not depend on the chain, so
            // they run ahead of it and the chain proceeds at FMA latency.
            const int ng = static_cast<int>(s1 - s0) >> 2;
            int4* c4 = reinterpret_cast<int4*>(cb);
            float4* x4 = reinterpret_cast<float4*>(cb);
            const float4* v4 = reinterpret_cast<const float4*>(vb);
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
        __syncwarp();  // every lane is done with buffer w % ST before it is refilled
    }
    cp_wait<0>();
    if (live) Y[row] = y;
}

// ── Warp-specialised variant ────────────────────────────────────────────
// With few rows an SM runs a single warp of the kernel above, and one warp
// cannot issue the copies, the gathers and the chain fast enough (about 9
// instructions per slot at one instruction every few cycles).  Here a CTA
// of three warps serves 32 rows: two producer warps (windows alternate
// between them) bring a window in, apply the edge fix-ups and replace each
// col by X[col] in place, and one consumer warp runs only the chains -- per
// 4 slots two 128-bit loads and four FMAs, at FMA latency.
// Copies: BULK = one 1-D bulk copy (cp.async.bulk, no multicast) per row and
// array per window, posted on the stage's mbarrier by the row's producer
// lane: the copy engine keeps them in flight without the L1 miss-tracking
// limit that caps cp.async and plain loads at a few tens of KB per SM.
// Otherwise the warp copies cooperatively with 16-byte cp.async as above.
// Stage s (window w % S) is handed over on full[s] (32 producer arrivals)
// and back on empty[s] (one consumer arrival); every wait is bounded.
// Producer p owns windows w = p, p + 2, ...; it keeps D - 1 = S/2 - 1 of
// them in flight and refills the stage of its window w - 2 once the
// consumer has released it.
template <int WIN>
struct WsShape {
    static constexpr int kStride = WIN + 4;                 // words per row slice
    static constexpr int kStageWords = 32 * kStride;        // one array, one stage
};

template <int WIN, int S, bool KS, bool BULK>
__global__ void __launch_bounds__(96, 1)
spmv_ws_kernel(int M, int64_t K, int64_t cap_total, const int32_t* __restrict__ row_start,
               const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
               const float* __restrict__ vals, const float* __restrict__ X,
               float* __restrict__ Y, unsigned* status) {
    static_assert(S % 2 == 0 && S >= 4, "two producers, at least two stages each");
    constexpr int D = S / 2;
    constexpr int kStr = WsShape<WIN>::kStride;
    constexpr int kSW = WsShape<WIN>::kStageWords;
    constexpr size_t kRing = size_t(S) * kSW * 4 * 2;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[S];
    __shared__ __align__(8) uint64_t empty[S];
    __shared__ __align__(8) uint64_t landed[S];
    __shared__ __align__(8) uint64_t xbar;
    int* cring = reinterpret_cast<int*>(smem_raw);
    float* vring = reinterpret_cast<float*>(smem_raw + kRing / 2);
    float* xs = reinterpret_cast<float*>(smem_raw + kRing + 16);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * 32 + lane;
    const bool live = row < M;
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
            mbar_init(&landed[b], 32);
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
    auto issue = [&](int w) {
        const int b = w % S;
        if constexpr (BULK) {
            unsigned bytes = 0;
            int s0 = 0;
            if (w < nw) {
                s0 = a + w * WIN;
                const int s1 = s0 + WIN < ecopy ? s0 + WIN : ecopy;
                if (s1 > s0) bytes = static_cast<unsigned>(s1 - s0) * 4u;
            }
            if (bytes) {
                mbar_expect_tx(&landed[b], 2 * bytes);
                bulk_load_1d(cslice + b * kSW, cols + s0, bytes, &landed[b]);
                bulk_load_1d(vslice + b * kSW, vals + s0, bytes, &landed[b]);
            } else {
                mbar_arrive(&landed[b]);
            }
        } else {
            constexpr int LPR = WIN / 4 < 32 ? WIN / 4 : 32;  // lanes per row
            constexpr int RPI = 32 / LPR;                     // rows per instruction
            const int sub = lane / LPR, li = lane % LPR;
            int* cdst = cring + b * kSW + sub * kStr + 4 * li;
            float* vdst = vring + b * kSW + sub * kStr + 4 * li;
#pragma unroll 4
            for (int rr = 0; rr < 32; rr += RPI) {
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
        }
    };
    auto landed_wait = [&](int w) -> bool {
        if constexpr (BULK) {
            return mbar_wait(&landed[w % S], static_cast<unsigned>((w / S) & 1), status);
        } else {
            cp_wait<D - 1>();
            return true;
        }
    };
#pragma unroll
    for (int i = 0; i < D - 1; ++i) {
        const int w = p + 2 * i;
        if (w < NW) issue(w);
        else if (!BULK) cp_commit();
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
            if (BULK) fence_proxy_async();  // this warp's gather writes -> the copy engine's
            issue(wn);
        } else if (!BULK) {
            cp_commit();
        }
        if (!landed_wait(w)) { ok = false; break; }
        __syncwarp();  // every lane's copies of window w are visible
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
    if (!ok && BULK) {
        // A wait gave up: let this warp's issued copies land (bounded) before exiting.
        for (int w = p; w < NW; w += 2) mbar_wait(&landed[w % S], static_cast<unsigned>((w / S) & 1), status, 1 << 12);
    }
    if (!BULK) cp_wait<0>();
}

template <int WIN, int S, bool KS, bool BULK>
int launch_ws(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    unsigned* status = device_status_word();
    if (status == nullptr) return -1;
    const size_t smem = size_t(S) * WsShape<WIN>::kStageWords * 4 * 2 + 16 +
                        (KS ? static_cast<size_t>(K) * 4 : 0);
    auto kern = spmv_ws_kernel<WIN, S, KS, BULK>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int M = static_cast<int>(W->nrows);
    note_kernel("spmv_ws_kernel");
    kern<<<(M + 31) / 32, 96, smem, s>>>(M, K, W->total_capacity, W->row_start, W->row_nnz,
                                         W->col_indices, W->values, X, Y, status);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd (N = 1, warp-specialised)");
    return SL_OK;
}

template <int ST, bool KS>
int launch_cfg(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    using S = CoopShape<ST>;
    const size_t smem = S::kXOff + (KS ? static_cast<size_t>(K) * 4 : 0);
    auto kern = spmv_coop_kernel<ST, KS>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int M = static_cast<int>(W->nrows);
    note_kernel("spmv_coop_kernel");
    kern<<<(M + 31) / 32, 32, smem, s>>>(M, K, W->total_capacity, W->row_start, W->row_nnz,
                                         W->col_indices, W->values, X, Y);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd (N = 1, cooperative windows)");
    return SL_OK;
}

}  // namespace

// At most one warp per SM: 8 windows in flight (one CTA per SM keeps about
// 120 KB in flight).  More rows: 4 windows, two or more CTAs per SM.
// SPARSECORE_B200_N1_ST=4|8 overrides the ring depth and
// SPARSECORE_B200_N1_WS=0 selects the single-warp kernel (measurements and
// tests).  Returns -1 when the kernel cannot be configured (caller falls
// back).
int launch_spmv_bulk(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    if (!aligned16(W->col_indices) || !aligned16(W->values) || W->nrows <= 0 || K < 1 ||
        W->nrows > INT_MAX - 32 || W->total_capacity > INT_MAX - 4 * kWin * 16)
        return -1;
    const int64_t warps = (W->nrows + 31) / 32;
    int st = warps <= num_sms() ? 8 : 4;
    if (const char* e = std::getenv("SPARSECORE_B200_N1_ST")) {
        const int v = std::atoi(e);
        if (v == 4 || v == 8) st = v;
    }
    // SPARSECORE_B200_N1_WS=0: single-warp kernel; =1: warp-specialised with
    // cp.async copies; default (=2): warp-specialised with bulk copies of
    // 128-slot windows, 6 stages (4 when X takes 64 KB of shared memory).
    int ws = 2;
    if (const char* e = std::getenv("SPARSECORE_B200_N1_WS")) ws = e[0] - '0';
    const bool ks = K <= kMaxKs;
    if (ws == 2) {
        const bool deep = !ks || K <= 4096;
        if (deep) return ks ? launch_ws<128, 6, true, true>(W, X, K, Y, s) : launch_ws<128, 6, false, true>(W, X, K, Y, s);
        return launch_ws<128, 4, true, true>(W, X, K, Y, s);
    }
    if (ws == 1) {
        if (st == 8) return ks ? launch_ws<64, 8, true, false>(W, X, K, Y, s) : launch_ws<64, 8, false, false>(W, X, K, Y, s);
        return ks ? launch_ws<64, 4, true, false>(W, X, K, Y, s) : launch_ws<64, 4, false, false>(W, X, K, Y, s);
    }
    if (st == 8) return ks ? launch_cfg<8, true>(W, X, K, Y, s) : launch_cfg<8, false>(W, X, K, Y, s);
    return ks ? launch_cfg<4, true>(W, X, K, Y, s) : launch_cfg<4, false>(W, X, K, Y, s);
}

}  // namespace slb
