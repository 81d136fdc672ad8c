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
// GPU mapping: work items are (row, segment) pairs; a segment is a run of
// 32 slots of one row, and a row has SPR = ceil(average capacity / 32)
// segments (segment s of a longer row also takes slots s*32 + k*SPR*32).
// One warp works on one item at a time, so short rows waste at most one
// partial segment and long rows still spread over several warps.
//  * N >= 16 (quad kernel): a quad of 4 lanes evaluates one slot's dot;
//    quad lane q owns chains 4q..4q+3 and reads X[c, 16m+4q .. +3] (and the
//    matching dY) as one 128-bit load per step, so each quad streams a
//    contiguous 64-byte piece of the X row per step; each quad carries S = 4
//    slots of the row, reusing each dY vector 4 times.
//  * N < 16 (lane kernel): each lane evaluates one slot's whole dot
//    (segments of 128 slots, 4 per lane).
#include <cmath>
#include <cstdlib>
#include <functional>
#include <map>
#include <mutex>

#include "common.cuh"
#include "tma.cuh"

namespace slb {
namespace {

constexpr int kDwThreads = 256;
constexpr int kDwWarps = kDwThreads / 32;
constexpr int kSeg = 32;  // slots per (row, segment) work item and warp pass

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

// Scalar tail after the horizontal reduction (see the file comment).
__device__ __forceinline__ float dot_tail(float r, const float* dyr, const float* xr, int64_t jtail,
                                          int64_t jfma, int64_t N) {
    for (int64_t j = jtail; j < jfma; ++j) r = __fadd_rn(r, __fmul_rn(__ldg(dyr + j), __ldg(xr + j)));
    for (int64_t j = jfma; j < N; ++j) r = fmaf(__ldg(dyr + j), __ldg(xr + j), r);
    return r;
}

struct DwShape {
    int64_t N, nfull, jtail, jfma;
    int rem;
    __device__ __forceinline__ explicit DwShape(int64_t n) : N(n) {
        nfull = n >> 4;
        rem = static_cast<int>(n & 15);
        jtail = nfull * 16 + (rem >= 8 ? 8 : 0);
        jfma = jtail + ((n - jtail) & ~static_cast<int64_t>(3));
    }
};

// Zero the padding slots of `row` (lanes of one warp).
__device__ __forceinline__ void zero_padding(float* dW, int rs, int nn, int cap, int lane) {
    for (int k = nn + lane; k < cap; k += 32) dW[rs + k] = 0.0f;
}

template <bool VEC4>
__global__ void __launch_bounds__(kDwThreads)
sddmm_quad_kernel(int M, int spr, int64_t N, const int32_t* __restrict__ row_start,
                  const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ row_capacity,
                  const int32_t* __restrict__ cols, const float* __restrict__ dY,
                  const float* __restrict__ X, float* __restrict__ dW) {
    constexpr int S = 4;
    const int lane = threadIdx.x & 31;
    const int q = lane & 3;
    const int quad = lane >> 2;  // 0..7
    const DwShape sh(N);
    const int64_t n_items = static_cast<int64_t>(M) * spr;
    for (int64_t item = static_cast<int64_t>(blockIdx.x) * kDwWarps + (threadIdx.x >> 5);
         item < n_items; item += static_cast<int64_t>(gridDim.x) * kDwWarps) {
        const int row = static_cast<int>(item / spr);
        const int seg = static_cast<int>(item % spr);
        const int rs = __ldg(row_start + row);
        const int nn = __ldg(row_nnz + row);
        if (seg == 0) zero_padding(dW, rs, nn, __ldg(row_capacity + row), lane);
        const float* dyr = dY + static_cast<int64_t>(row) * N;

        for (int kb = seg * kSeg; kb < nn; kb += spr * kSeg) {
            const float* xr[S];
            bool act[S];
#pragma unroll
            for (int u = 0; u < S; ++u) {
                const int k = kb + quad + 8 * u;
                act[u] = k < nn;
                const int c = act[u] ? __ldg(cols + rs + k) : 0;
                xr[u] = X + static_cast<int64_t>(c) * N;
            }
            float4 acc[S];
#pragma unroll
            for (int u = 0; u < S; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);

            // 16-wide steps: quad lane q advances chains 4q..4q+3.
#pragma unroll 2
            for (int64_t m = 0; m < sh.nfull; ++m) {
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
            if (sh.rem >= 8 && q < 2) {
                const int64_t j = sh.nfull * 16 + q * 4;
                const float4 d = load4<VEC4>(dyr + j);
#pragma unroll
                for (int u = 0; u < S; ++u)
                    if (act[u]) fma4(d, load4<VEC4>(xr[u] + j), acc[u]);
            }
            // Horizontal reduction: lane 0 holds acc[0..3], lane 1 acc[4..7].
#pragma unroll
            for (int u = 0; u < S; ++u) {
                const float4 hi = shfl_xor4(acc[u], 1);
                if (q == 0 && act[u]) {
                    const float4 s4 = add4(acc[u], hi);
                    float r = __fadd_rn(__fadd_rn(s4.x, s4.z), __fadd_rn(s4.y, s4.w));
                    dW[rs + kb + quad + 8 * u] = dot_tail(r, dyr, xr[u], sh.jtail, sh.jfma, N);
                }
            }
        }
    }
}

// One slot's whole dot for small N: the 16 chains in registers (16-wide
// steps as four 128-bit loads of each operand when VEC4), then the same
// combination, optional 8-wide step, horizontal reduction and tail.
template <bool VEC4>
__device__ __forceinline__ float lane_dot(const float* dyr, const float* xr, const DwShape& sh) {
    float a[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) a[t] = 0.0f;
    for (int64_t m = 0; m < sh.nfull; ++m) {
        const float* d = dyr + m * 16;
        const float* x = xr + m * 16;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const float4 dv = load4<VEC4>(d + 4 * h), xv = load4<VEC4>(x + 4 * h);
            a[4 * h + 0] = fmaf(dv.x, xv.x, a[4 * h + 0]);
            a[4 * h + 1] = fmaf(dv.y, xv.y, a[4 * h + 1]);
            a[4 * h + 2] = fmaf(dv.z, xv.z, a[4 * h + 2]);
            a[4 * h + 3] = fmaf(dv.w, xv.w, a[4 * h + 3]);
        }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) a[t] = __fadd_rn(a[t], a[t + 8]);
    if (sh.rem >= 8)
#pragma unroll
        for (int t = 0; t < 8; ++t)
            a[t] = fmaf(__ldg(dyr + sh.nfull * 16 + t), __ldg(xr + sh.nfull * 16 + t), a[t]);
    float s4[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) s4[t] = __fadd_rn(a[t], a[t + 4]);
    const float r = __fadd_rn(__fadd_rn(s4[0], s4[2]), __fadd_rn(s4[1], s4[3]));
    return dot_tail(r, dyr, xr, sh.jtail, sh.jfma, sh.N);
}

// Small N: one lane per slot (segments of 128 slots, 4 per lane), all
// chains in registers.
constexpr int kLaneSeg = 128;
template <bool VEC4>
__global__ void __launch_bounds__(kDwThreads)
sddmm_lane_kernel(int M, int spr, int64_t N, const int32_t* __restrict__ row_start,
                  const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ row_capacity,
                  const int32_t* __restrict__ cols, const float* __restrict__ dY,
                  const float* __restrict__ X, float* __restrict__ dW) {
    const int lane = threadIdx.x & 31;
    const DwShape sh(N);
    const int64_t n_items = static_cast<int64_t>(M) * spr;
    for (int64_t item = static_cast<int64_t>(blockIdx.x) * kDwWarps + (threadIdx.x >> 5);
         item < n_items; item += static_cast<int64_t>(gridDim.x) * kDwWarps) {
        const int row = static_cast<int>(item / spr);
        const int seg = static_cast<int>(item % spr);
        const int rs = __ldg(row_start + row);
        const int nn = __ldg(row_nnz + row);
        if (seg == 0) zero_padding(dW, rs, nn, __ldg(row_capacity + row), lane);
        const float* dyr = dY + static_cast<int64_t>(row) * N;
        for (int kb = seg * kLaneSeg; kb < nn; kb += spr * kLaneSeg) {
            // All four slots' loads are issued before any dot is finished.
            constexpr int U = kLaneSeg / 32;
            const float* xr[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int k = kb + u * 32 + lane;
                xr[u] = X + static_cast<int64_t>(k < nn ? __ldg(cols + rs + k) : 0) * N;
            }
            float r[U];
#pragma unroll
            for (int u = 0; u < U; ++u) r[u] = lane_dot<VEC4>(dyr, xr[u], sh);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int k = kb + u * 32 + lane;
                if (k < nn) dW[rs + k] = r[u];
            }
        }
    }
}

// ── Tiled SDDMM (large N, N % 32 == 0) ───────────────────────────────────
// The per-slot kernels above gather X[col] from L2 once per slot, so they are
// bound by L2 bandwidth.  Here a CTA owns a 2-D tile of W (TR rows x TC
// columns) and streams the two operand blocks dY[tile rows, :] and
// X[tile cols, :] through shared memory in 32-column chunks (TMA, 128-byte
// swizzle, double-buffered on two mbarriers).  The tile's live slots keep
// their 16 chains in registers for the whole sweep over N (quad layout as
// above: quad lane q owns chains 4q..4q+3), so every operand element is
// fetched from L2 once per tile instead of once per slot.  A tile holding
// more than 512 slots sweeps N once per batch of 512.  Within a batch the
// slots are ordered so that the two quads of each quarter-warp read opposite
// bank halves (see the batch-order comment in the kernel).  Same rounding
// sequence as the other SDDMM kernels (N % 16 == 0: no 8-wide step, no tail).
constexpr int kTThreads = 256;
constexpr int kTQuads = kTThreads / 4;
constexpr int kTS = 8;                    // slots per quad per batch
constexpr int kTBatch = kTQuads * kTS;    // 512
static_assert(kTBatch == 2 * kTThreads, "batch setup: two positions per consumer thread");
constexpr int kTJ = 32;                   // columns per chunk: 128-byte rows
constexpr int kTMaxRows = 128;
constexpr int kTStages = 5;

__device__ __forceinline__ int lower_bound_cols(const int32_t* __restrict__ c, int n, int key) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(c + mid) < key) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// Named barrier 1 over the kTThreads consumer threads (the producer warp
// never joins it).
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kTThreads) : "memory"); }

// Exclusive scan over the kTThreads consumer threads.
__device__ __forceinline__ int consumer_exclusive_scan(int v, int* ws, int* total) {
    constexpr int NW = kTThreads / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int inc = warp_inclusive_scan(v);
    if (lane == 31) ws[warp] = inc;
    consumer_bar();
    if (warp == 0) {
        int w = lane < NW ? ws[lane] : 0;
        w = warp_inclusive_scan(w);
        if (lane < NW) ws[lane] = w;
    }
    consumer_bar();
    const int base = warp ? ws[warp - 1] : 0;
    *total = ws[NW - 1];
    consumer_bar();
    return base + inc - v;
}

template <bool SEG>
__global__ void __launch_bounds__(kTThreads + 32, 2)
sddmm_tiled_kernel(const __grid_constant__ CUtensorMap dymap, const __grid_constant__ CUtensorMap xmap,
                   int M, int64_t N, int TR, int TC, int n_bc, int n_bi, int col_major, int shared_first,
                   const int32_t* __restrict__ row_start, const int32_t* __restrict__ row_nnz,
                   const int32_t* __restrict__ row_capacity, const int32_t* __restrict__ cols,
                   float* __restrict__ dW, unsigned* status) {
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte aligned for the 128-byte swizzle.  The offset is added to the
    // shared array itself (not through an integer round trip), so the
    // compiler keeps every access below a shared-memory access.
    float* sbase = reinterpret_cast<float*>(smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u));
    __shared__ __align__(8) uint64_t full[kTStages];
    __shared__ __align__(8) uint64_t empty[kTStages];
    __shared__ int run_lo[kTMaxRows];
    __shared__ int run_pref[kTMaxRows + 1];
    __shared__ int ws[(kTThreads + 32) / 32];
    __shared__ int ord_slot[kTBatch];  // batch position -> global slot (-1 = none)
    __shared__ int ord_rc[kTBatch];    // (tile row << 16) | tile column
    __shared__ int seg_pref[kTMaxRows + 1];  // SEG: exclusive scan of ceil(run / 8)

    const int tid = threadIdx.x, lane = tid & 31, q = lane & 3, quad = tid >> 2;
    const bool producer = tid >= kTThreads;  // warp 8 issues the copies
    // Tile order: CTAs resident together share the larger operand's tile
    // (col_major: the same X column tile, row tiles fastest), so it is read
    // from DRAM about once and the smaller operand stays in L2.
    const int bi = col_major ? static_cast<int>(blockIdx.x % n_bi) : static_cast<int>(blockIdx.x / n_bc);
    const int bc = col_major ? static_cast<int>(blockIdx.x / n_bi) : static_cast<int>(blockIdx.x % n_bc);
    const int r0 = bi * TR, c0 = bc * TC;
    const int nrows = min(TR, M - r0);

    // Each tile row's live slots in [c0, c0+TC) are one run of its sorted row.
    int cnt = 0;
    if (tid < nrows) {
        const int rs = __ldg(row_start + r0 + tid), nn = __ldg(row_nnz + r0 + tid);
        const int lo = lower_bound_cols(cols + rs, nn, c0);
        const int hi = lo + lower_bound_cols(cols + rs + lo, nn - lo, c0 + TC);
        run_lo[tid] = rs + lo;
        cnt = hi - lo;
    }
    int total;
    const int ex = block_exclusive_scan<kTThreads + 32>(cnt, ws, &total);
    if (tid < TR) run_pref[tid] = ex;
    if (tid == 0) run_pref[TR] = total;
    int nseg = 0;  // SEG: segments of up to kTS slots of one row, the batching unit
    if constexpr (SEG) {
        const int sx = block_exclusive_scan<kTThreads + 32>((cnt + kTS - 1) / kTS, ws, &nseg);
        if (tid < TR) seg_pref[tid] = sx;
        if (tid == 0) seg_pref[TR] = nseg;
    }
    if (bc == 0) {  // padding slots of the tile's rows -> 0
        for (int r = tid >> 5; r < nrows; r += (kTThreads + 32) / 32) {
            const int rs = __ldg(row_start + r0 + r);
            for (int k = __ldg(row_nnz + r0 + r) + lane; k < __ldg(row_capacity + r0 + r); k += 32)
                dW[rs + k] = 0.0f;
        }
    }
    if (tid == 0) {
        for (int b = 0; b < kTStages; ++b) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], kTThreads / 32);
        }
        fence_barrier_init();
    }
    __syncthreads();
    if (total == 0) return;

    // Stage b: dY block at sbase + b*stage, X block right after it.
    const int stage = (TR + TC) * kTJ;
    const int nchunks = static_cast<int>(N / kTJ);
    const int nbatch = SEG ? (nseg + kTQuads - 1) / kTQuads : (total + kTBatch - 1) / kTBatch;
    const int nsteps = nbatch * nchunks;  // step g = batch * nchunks + chunk

    if (producer) {
        if (lane == 0) {
            // The operand the resident CTAs share is streamed once (evict
            // first); the other one is re-read by the later bands of tiles
            // and should stay in L2 (evict last).
            const uint64_t shared = shared_first ? l2_policy_evict_first() : l2_policy_evict_normal();
            const uint64_t pol_rows = col_major ? l2_policy_evict_last() : shared;
            const uint64_t pol_cols = col_major ? shared : l2_policy_evict_last();
            const unsigned chunk_bytes = static_cast<unsigned>(stage * 4);
            unsigned eph = 0u;  // bit b = parity of stage b's next release
            int g = 0;
            for (; g < nsteps; ++g) {
                const int b = g % kTStages;
                if (g >= kTStages) {
                    if (!mbar_wait(&empty[b], (eph >> b) & 1u, status)) break;
                    eph ^= 1u << b;
                }
                const int k = g % nchunks;
                fence_proxy_async();
                mbar_expect_tx(&full[b], chunk_bytes);
                tma_load_2d_hint(sbase + b * stage, &dymap, k * kTJ, r0, &full[b], pol_rows);
                tma_load_2d_hint(sbase + b * stage + TR * kTJ, &xmap, k * kTJ, c0, &full[b], pol_cols);
            }
            // Before the CTA may exit, every issued copy must have landed:
            // wait (bounded) for the full-barrier completion of the last
            // kTStages issued steps.
            const int g0 = g > kTStages ? g - kTStages : 0;
            for (int h = g0; h < g; ++h) mbar_wait(&full[h % kTStages], (h / kTStages) & 1u, status);
        }
        return;
    }

    // A timed-out wait sets ok = false; the thread then skips further waits
    // but still reaches every named barrier, so no consumer is left waiting.
    bool ok = true;
    unsigned fph = 0u;  // bit b = parity of stage b's next fill
    if constexpr (SEG) {
        // Segmented batches: quad Q takes segment g = bt * 64 + Q, i.e. up
        // to kTS consecutive live slots of ONE tile row, so the quad loads
        // that row's dY chunk once per chunk instead of at every row change
        // inside its slots.  Within the segment the slots are ordered by the
        // bank half of their X row -- even quads take class 0 first, odd
        // quads class 1 first -- so the two quads of a quarter-warp mostly
        // read opposite bank halves.  Each slot is its own dot product, so
        // the order of a quad's slots does not touch the rounding.
        for (int bt = 0; bt < nbatch; ++bt) {
            const int g = bt * kTQuads + quad;
            int r = 0, ns = 0, base = 0;
            if (g < nseg) {
                int lo = 0, hi = TR;  // last r with seg_pref[r] <= g
                while (hi - lo > 1) {
                    const int mid = (lo + hi) >> 1;
                    if (seg_pref[mid] <= g) lo = mid; else hi = mid;
                }
                r = lo;
                const int j0 = kTS * (g - seg_pref[r]);
                ns = min(kTS, run_pref[r + 1] - run_pref[r] - j0);
                base = run_lo[r] + j0;
            }
            int cl[kTS];
            unsigned cls = 0u;
#pragma unroll
            for (int t = 0; t < kTS; ++t) {
                cl[t] = t < ns ? __ldg(cols + base + t) - c0 : 0;
                if ((cl[t] >> 2) & 1) cls |= 1u << t;
            }
            const unsigned want = (quad & 1) ? 1u : 0u;  // class taken first
            int off[kTS], sid[kTS], key[kTS];
#pragma unroll
            for (int t = 0; t < kTS; ++t) {
                off[t] = TR * kTJ + cl[t] * kTJ + ((q ^ (cl[t] & 7)) << 2);
                sid[t] = base + t;
                key[t] = t < ns ? (((cls >> t) & 1u) == want ? 0 : 1) : 2;
            }
            // Batcher's odd-even merge sort of the 8 (key, off, sid) triples
            // by key: fixed compare-exchanges keep the arrays in registers.
            constexpr int kNet[19][2] = {{0, 1}, {2, 3}, {4, 5}, {6, 7}, {0, 2}, {1, 3}, {4, 6},
                                         {5, 7}, {1, 2}, {5, 6}, {0, 4}, {1, 5}, {2, 6}, {3, 7},
                                         {2, 4}, {3, 5}, {1, 2}, {3, 4}, {5, 6}};
#pragma unroll
            for (int e = 0; e < 19; ++e) {
                const int a = kNet[e][0], b = kNet[e][1];
                const bool sw = key[b] < key[a];
                const int ka = sw ? key[b] : key[a], kb = sw ? key[a] : key[b];
                const int oa = sw ? off[b] : off[a], ob = sw ? off[a] : off[b];
                const int ia = sw ? sid[b] : sid[a], ib = sw ? sid[a] : sid[b];
                key[a] = ka; key[b] = kb; off[a] = oa; off[b] = ob; sid[a] = ia; sid[b] = ib;
            }
            const int yo = r * kTJ + ((q ^ (r & 7)) << 2);
            float4 acc[kTS];
#pragma unroll
            for (int t = 0; t < kTS; ++t) acc[t] = make_float4(0.f, 0.f, 0.f, 0.f);
            int b = (bt * nchunks) % kTStages;  // stage of the batch's first chunk
            for (int kc = 0; kc < nchunks; ++kc) {
                if (ok && !mbar_wait(&full[b], (fph >> b) & 1u, status)) ok = false;  // bounded
                fph ^= 1u << b;
                const float* sb = sbase + b * stage;
                const float4 d0 = *reinterpret_cast<const float4*>(sb + yo);
                const float4 d1 = *reinterpret_cast<const float4*>(sb + (yo ^ 16));
#pragma unroll
                for (int t = 0; t < kTS; ++t) {
                    if (t < ns) {
                        fma4(d0, *reinterpret_cast<const float4*>(sb + off[t]), acc[t]);
                        fma4(d1, *reinterpret_cast<const float4*>(sb + (off[t] ^ 16)), acc[t]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[b]);  // this warp is done with stage b
                b = b + 1 == kTStages ? 0 : b + 1;
            }
#pragma unroll
            for (int t = 0; t < kTS; ++t) {
                const float4 o = shfl_xor4(acc[t], 2);
                if (q < 2) acc[t] = add4(acc[t], o);
                const float4 hi = shfl_xor4(acc[t], 1);
                if (q == 0 && ok && t < ns) {
                    const float4 s4 = add4(acc[t], hi);
                    dW[sid[t]] = __fadd_rn(__fadd_rn(s4.x, s4.z), __fadd_rn(s4.y, s4.w));
                }
            }
        }
        return;
    }
    for (int bt = 0; bt < nbatch; ++bt) {
        // Batch order.  A warp-wide 128-bit shared load is served one
        // quarter-warp (two quads) at a time, and a quad reads one 64-byte
        // half of a swizzled 128-byte X row: banks 0-15 when (c & 4) == 0,
        // banks 16-31 otherwise (the other half the opposite way).  The
        // batch's slots (tile row-major order) are split by that bit into two
        // lists and interleaved, so the two quads of a quarter-warp take one
        // slot of each class and never share a bank; only the unmatched tail
        // of the longer list pairs equal classes.  Each list keeps row order,
        // so a quad's consecutive slots still share dY rows.
        const int b0 = bt * kTBatch;
        int sl2[2], rc2[2], cls2[2];
        int packed = 0;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int t = b0 + 2 * tid + u;
            sl2[u] = -1; rc2[u] = 0; cls2[u] = -1;
            if (t < total) {
                int lo = 0, hi = TR;  // last r with run_pref[r] <= t
                while (hi - lo > 1) {
                    const int mid = (lo + hi) >> 1;
                    if (run_pref[mid] <= t) lo = mid; else hi = mid;
                }
                sl2[u] = run_lo[lo] + (t - run_pref[lo]);
                const int c = __ldg(cols + sl2[u]) - c0;
                rc2[u] = (lo << 16) | c;
                cls2[u] = (c >> 2) & 1;
                packed += cls2[u] ? (1 << 16) : 1;
            }
        }
        int tot_packed;
        const int exs = consumer_exclusive_scan(packed, ws, &tot_packed);
        const int n0 = tot_packed & 0xffff, n1 = tot_packed >> 16, m = min(n0, n1);
        int rank0 = exs & 0xffff, rank1 = exs >> 16;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int p = 2 * tid + u;
            if (cls2[u] < 0) {
                if (p >= n0 + n1) { ord_slot[p] = -1; ord_rc[p] = 0; }
                continue;
            }
            const int i = cls2[u] ? rank1++ : rank0++;
            const int dest = i < m ? 2 * i + cls2[u] : 2 * m + (i - m);
            ord_slot[dest] = sl2[u];
            ord_rc[dest] = rc2[u];
        }
        consumer_bar();

        // Quad Q's slot s sits at position 16 * (Q >> 1) + 2 * s + (Q & 1).
        // Per slot: swizzled float offsets of its dY row and X row for the
        // chunk's first 16 columns (the second 16 are the same ^ 16), packed
        // as (dY << 16) | X; `fresh` bit s = slot s starts a new W row.
        const int qbase = 16 * (quad >> 1) + (quad & 1);
        // The float offsets of both 16-column halves, precomputed (no
        // decode in the chunk loop).
        int xa[kTS], xb[kTS], ya[kTS];
        unsigned fresh = 0u;
        int prev_r = -1;
#pragma unroll
        for (int s = 0; s < kTS; ++s) {
            const int rc = ord_rc[qbase + 2 * s];
            const int r = rc >> 16, c = rc & 0xffff;
            ya[s] = r * kTJ + ((q ^ (r & 7)) << 2);
            xa[s] = TR * kTJ + c * kTJ + ((q ^ (c & 7)) << 2);
            xb[s] = xa[s] ^ 16;
            if (s == 0 || r != prev_r) fresh |= 1u << s;
            prev_r = r;
        }
        float4 acc[kTS];
#pragma unroll
        for (int s = 0; s < kTS; ++s) acc[s] = make_float4(0.f, 0.f, 0.f, 0.f);

        int b = (bt * nchunks) % kTStages;  // stage of the batch's first chunk
        for (int k = 0; k < nchunks; ++k) {
            if (ok && !mbar_wait(&full[b], (fph >> b) & 1u, status)) ok = false;  // bounded
            fph ^= 1u << b;
            const float* sb = sbase + b * stage;
            float4 d0 = make_float4(0.f, 0.f, 0.f, 0.f), d1 = d0;
#pragma unroll
            for (int s = 0; s < kTS; ++s) {
                if (fresh & (1u << s)) {
                    d0 = *reinterpret_cast<const float4*>(sb + ya[s]);
                    d1 = *reinterpret_cast<const float4*>(sb + (ya[s] ^ 16));
                }
                fma4(d0, *reinterpret_cast<const float4*>(sb + xa[s]), acc[s]);
                fma4(d1, *reinterpret_cast<const float4*>(sb + xb[s]), acc[s]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[b]);  // this warp is done with stage b
            b = b + 1 == kTStages ? 0 : b + 1;
        }
        // acc = acc_a + acc_b, then the horizontal reduction (N % 16 == 0).
#pragma unroll
        for (int s = 0; s < kTS; ++s) {
            const float4 o = shfl_xor4(acc[s], 2);
            if (q < 2) acc[s] = add4(acc[s], o);
            const float4 hi = shfl_xor4(acc[s], 1);
            const int sl = (q == 0 && ok) ? ord_slot[qbase + 2 * s] : -1;
            if (sl >= 0) {
                const float4 s4 = add4(acc[s], hi);
                dW[sl] = __fadd_rn(__fadd_rn(s4.x, s4.z), __fadd_rn(s4.y, s4.w));
            }
        }
        consumer_bar();  // ord_* are rewritten by the next batch's setup
    }
}

// ── N = 1 ───────────────────────────────────────────────────────────────
// With one column the reference's order reduces to dW = fma(dY, X, +0)
// (all 16 chains and the 8-wide step are empty; the single term is the
// FMA of the scalar tail onto the +0 horizontal sum), so the SDDMM is a
// stream over the slot arrays: one warp per row writes the row's whole
// capacity (live slots and zeroed padding) with coalesced loads of the
// column indices and coalesced stores, X gathered through L1.  A warp keeps
// the next group's column loads in flight while it gathers and stores the
// current one (U strips of 32 slots per group), so each SM has tens of KB of
// loads outstanding.
constexpr int kN1U = 8;
__global__ void __launch_bounds__(256)
sddmm_n1_kernel(int M, const int32_t* __restrict__ row_start, const int32_t* __restrict__ row_nnz,
                const int32_t* __restrict__ row_capacity, const int32_t* __restrict__ cols,
                const float* __restrict__ dY, const float* __restrict__ X, float* __restrict__ dW) {
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M; row += warps) {
        const int rs = __ldg(row_start + row), nn = __ldg(row_nnz + row);
        const int cp = __ldg(row_capacity + row);
        const float dy = __ldg(dY + row);
        int c[kN1U];
#pragma unroll
        for (int u = 0; u < kN1U; ++u) {
            const int k = 32 * u + lane;
            c[u] = k < nn ? __ldg(cols + rs + k) : -1;
        }
        for (int k0 = 0; k0 < cp; k0 += 32 * kN1U) {
            int cn[kN1U];  // the next group of strips' columns, in flight while this group is gathered
#pragma unroll
            for (int u = 0; u < kN1U; ++u) {
                const int k = k0 + 32 * (kN1U + u) + lane;
                cn[u] = k < nn ? __ldg(cols + rs + k) : -1;
            }
            float x[kN1U];
#pragma unroll
            for (int u = 0; u < kN1U; ++u) x[u] = c[u] >= 0 ? __ldg(X + c[u]) : 0.0f;
#pragma unroll
            for (int u = 0; u < kN1U; ++u) {
                const int k = k0 + 32 * u + lane;
                if (k < cp) dW[rs + k] = c[u] >= 0 ? fmaf(dy, x[u], 0.0f) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < kN1U; ++u) c[u] = cn[u];
        }
    }
}

int launch_dw_n1(const sl_csr* W, const float* dY, const float* X, float* dW, cudaStream_t s) {
    const int M = static_cast<int>(W->nrows);
    int64_t blocks = (static_cast<int64_t>(M) + 7) / 8;
    const int64_t max_blocks = static_cast<int64_t>(num_sms()) * 8;
    if (blocks > max_blocks) blocks = max_blocks;
    note_kernel("sddmm_n1_kernel");
    sddmm_n1_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        M, W->row_start, W->row_nnz, W->row_capacity, W->col_indices, dY, X, dW);
    SL_RETURN_IF_LAUNCH_FAILED("sl_sddmm_dw (N = 1)");
    return SL_OK;
}

// One launch of the tiled kernel, slot batches (seg = false) or segmented
// batches (seg = true).  Returns -1 when it cannot be configured.
int launch_tiled(const sl_csr* W, const float* dY, const float* X, int64_t N, float* dW,
                 cudaStream_t s, double dens, bool seg) {
    const int64_t M = W->nrows, K = W->ncols;
    // Wide tiles at low density (more slots per tile row: fewer dY reloads).
    int TC = dens <= 0.15 ? 128 : 64;
    if (const char* e = std::getenv("SPARSECORE_B200_DW_TC")) {  // tuning knob: 64|128|256
        const int v = std::atoi(e);
        if (v == 64 || v == 128 || v == 256) TC = v;
    }
    // Slot batches: about 480 slots per tile (the batch holds 512).
    // Segmented batches: about 60 of the 64 quads' segments per tile.
    int TR = seg ? static_cast<int>(std::floor(60.0 / (TC * dens / kTS + 0.55) / 8.0)) * 8
                 : static_cast<int>(std::floor(480.0 / (TC * dens) / 8.0)) * 8;
    TR = TR < 8 ? 8 : (TR > kTMaxRows ? kTMaxRows : TR);
    unsigned* status = device_status_word();
    if (status == nullptr) return -1;
    CUtensorMap dymap, xmap;
    if (!make_tmap_2d(&dymap, dY, M, N, TR, kTJ, true) || !make_tmap_2d(&xmap, X, K, N, TC, kTJ, true))
        return -1;
    const size_t smem = static_cast<size_t>(kTStages * (TR + TC) * kTJ * 4) + 1024;
    auto kern = seg ? sddmm_tiled_kernel<true> : sddmm_tiled_kernel<false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int n_bi = static_cast<int>((M + TR - 1) / TR), n_bc = static_cast<int>((K + TC - 1) / TC);
    int col_major = K > M ? 1 : 0;  // X (K x N) is the larger operand
    if (const char* e = std::getenv("SPARSECORE_B200_DW_ORDER"))  // row|col (measurements)
        col_major = e[0] == 'c' ? 1 : 0;
    // L2 policy of the operand the resident CTAs share: evict-first (its
    // bytes are read once) or normal (SPARSECORE_B200_DW_L2=first|normal).
    // Measured on B200 (config-5 layers, N = 16384, ncu DRAM bytes per
    // launch): evict-first in row order cuts qkv 353 -> 233 MB, ffn_up
    // 312 -> 281 MB, o 142 -> 110 MB; in column order (ffn_down) normal
    // keeps 322 MB against 333.
    int shared_first = col_major ? 0 : 1;
    if (const char* e = std::getenv("SPARSECORE_B200_DW_L2")) shared_first = e[0] == 'f' ? 1 : 0;
    note_kernel("sddmm_tiled_kernel");
    kern<<<n_bi * n_bc, kTThreads + 32, smem, s>>>(
        dymap, xmap, static_cast<int>(M), N, TR, TC, n_bc, n_bi, col_major, shared_first, W->row_start,
        W->row_nnz, W->row_capacity, W->col_indices, dW, status);
    SL_RETURN_IF_LAUNCH_FAILED("sl_sddmm_dw (tiled)");
    return SL_OK;
}

// Batch form: slot batches by default.  SPARSECORE_B200_DW_SEG=1 forces the
// segmented form, =auto picks per problem shape by timing both on the
// shape's first call (outside stream capture; both are bit-identical, so
// the choice never changes a value) and caches it.  Measured on B200 at N =
// 16384: timed alone, segmented batches win on config-5 o (7.7 vs 6.5
// TFLOP/s) and config-4 qkv (7.0 vs 5.5) and lose on the other config-4/5
// layers (e.g. ffn_up 6.9 vs 7.6); but in the config-5 training step, where
// the SDDMM runs beside dX on a side stream, the per-shape choice made the
// step slower (110.8 vs 109.8 ms), so it is not the default.
struct DwKey {
    int64_t M, K, cap, N;
    bool operator<(const DwKey& o) const {
        if (M != o.M) return M < o.M;
        if (K != o.K) return K < o.K;
        if (cap != o.cap) return cap < o.cap;
        return N < o.N;
    }
};
std::mutex g_dw_mu;
std::map<std::pair<int, DwKey>, bool> g_dw_seg;  // (device, shape) -> segmented

float time_launch_ms(cudaStream_t s, const std::function<int()>& fn, int* rc) {
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess) return -1.0f;
    if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return -1.0f; }
    cudaEventRecord(a, s);
    *rc = fn();
    cudaEventRecord(b, s);
    float ms = -1.0f;
    if (*rc == SL_OK && cudaEventSynchronize(b) == cudaSuccess) cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return ms;
}

// Returns -1 when the tiled path does not apply.
int try_tiled(const sl_csr* W, const float* dY, const float* X, int64_t N, float* dW, cudaStream_t s) {
    const int64_t M = W->nrows, K = W->ncols;
    if (N < 1024 || N % kTJ != 0 || !aligned16(dY) || !aligned16(X) || N > INT_MAX / 2) return -1;
    // Live density estimate from the capacity (live + about 20% padding).
    // Measured on B200 (standalone sweep): the tiled kernel wins for
    // 2% <= density <= 40% once N >= 1024; at N = 256 its pipeline barely
    // fills, and at 50% density its tiles shrink to 8 rows.
    const double dens = static_cast<double>(W->total_capacity) / 1.2 / (static_cast<double>(M) * K);
    if (dens < 0.02 || dens > 0.4) return -1;
    const char* mode = std::getenv("SPARSECORE_B200_DW_SEG");
    if (mode == nullptr || mode[0] != 'a')
        return launch_tiled(W, dY, X, N, dW, s, dens, mode != nullptr && mode[0] == '1');
    int dev = 0;
    cudaGetDevice(&dev);
    const std::pair<int, DwKey> key{dev, DwKey{M, K, W->total_capacity, N}};
    {
        std::lock_guard<std::mutex> lock(g_dw_mu);
        auto it = g_dw_seg.find(key);
        if (it != g_dw_seg.end()) return launch_tiled(W, dY, X, N, dW, s, dens, it->second);
    }
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone)
        return launch_tiled(W, dY, X, N, dW, s, dens, false);  // cannot time under capture
    // Warm both (module load, attributes), then time one launch of each.
    int rc_a = launch_tiled(W, dY, X, N, dW, s, dens, false);
    if (rc_a != SL_OK) return rc_a;
    int rc_b = launch_tiled(W, dY, X, N, dW, s, dens, true);
    const bool seg_ok = rc_b == SL_OK;
    float ms_a = time_launch_ms(s, [&] { return launch_tiled(W, dY, X, N, dW, s, dens, false); }, &rc_a);
    if (rc_a != SL_OK) return rc_a;
    float ms_b = -1.0f;
    if (seg_ok) ms_b = time_launch_ms(s, [&] { return launch_tiled(W, dY, X, N, dW, s, dens, true); }, &rc_b);
    const bool seg = seg_ok && rc_b == SL_OK && ms_a > 0.0f && ms_b > 0.0f && ms_b < ms_a;
    {
        std::lock_guard<std::mutex> lock(g_dw_mu);
        g_dw_seg[key] = seg;
    }
    // The last launch left the same dW as either form would; finish with the
    // chosen one so sl_last_kernel and the output are those of the choice.
    return launch_tiled(W, dY, X, N, dW, s, dens, seg);
}

// SPARSECORE_B200_DW=quad forces the per-slot kernels (tuning and tests).
bool tiled_disabled() {
    const char* e = std::getenv("SPARSECORE_B200_DW");
    return e != nullptr && e[0] == 'q';
}

int launch_dw(const sl_csr* W, const float* dY, const float* X, int64_t N, float* dW,
              cudaStream_t s) {
    const int M = static_cast<int>(W->nrows);
    int64_t lane_max = 16;  // lane kernel below this N (tuning knob: SPARSECORE_B200_DW_LANE)
    if (const char* e = std::getenv("SPARSECORE_B200_DW_LANE")) lane_max = std::atoi(e);
    const bool lane_kernel = N < lane_max;
    const int seg = lane_kernel ? kLaneSeg : kSeg;
    const int64_t avg_cap = (W->total_capacity + M - 1) / M;
    const int spr = static_cast<int>(avg_cap > seg ? (avg_cap + seg - 1) / seg : 1);
    const int64_t n_items = static_cast<int64_t>(M) * spr;
    int64_t blocks = (n_items + kDwWarps - 1) / kDwWarps;
    const int64_t max_blocks = static_cast<int64_t>(num_sms()) * 8;
    if (blocks > max_blocks) blocks = max_blocks;
    const bool vec4 = (N % 4 == 0) && aligned16(X) && aligned16(dY);
    note_kernel(lane_kernel ? "sddmm_lane_kernel" : "sddmm_quad_kernel");
    if (lane_kernel) {
        if (vec4)
            sddmm_lane_kernel<true><<<static_cast<unsigned>(blocks), kDwThreads, 0, s>>>(
                M, spr, N, W->row_start, W->row_nnz, W->row_capacity, W->col_indices, dY, X, dW);
        else
            sddmm_lane_kernel<false><<<static_cast<unsigned>(blocks), kDwThreads, 0, s>>>(
                M, spr, N, W->row_start, W->row_nnz, W->row_capacity, W->col_indices, dY, X, dW);
    } else if (vec4) {
        sddmm_quad_kernel<true><<<static_cast<unsigned>(blocks), kDwThreads, 0, s>>>(
            M, spr, N, W->row_start, W->row_nnz, W->row_capacity, W->col_indices, dY, X, dW);
    } else {
        sddmm_quad_kernel<false><<<static_cast<unsigned>(blocks), kDwThreads, 0, s>>>(
            M, spr, N, W->row_start, W->row_nnz, W->row_capacity, W->col_indices, dY, X, dW);
    }
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
    if (N == 1 && W->ncols > 0) {  // SPARSECORE_B200_N1=warp keeps the per-slot kernel (tests)
        const char* e = std::getenv("SPARSECORE_B200_N1");
        if (e == nullptr || e[0] != 'w') return launch_dw_n1(W, dY, X, dW, s);
    }
    if (N == 32 && W->ncols > 0 && gather32_enabled()) {
        const int rc = launch_gather32_sddmm(W, dY, X, dW, s);
        if (rc >= 0) return rc;
    }
    if (!tiled_disabled() && W->ncols > 0) {
        const int rc = try_tiled(W, dY, X, N, dW, s);
        if (rc >= 0) return rc;
    }
    return launch_dw(W, dY, X, N, dW, s);
}
