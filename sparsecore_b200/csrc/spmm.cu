// Forward SpMM over padded CSR:  Y[M,N] = W[M,K] . X[K,N]   (fp32)
//
// Numerics: every Y element is the FMA chain  y = fma(v_s, X[c_s, j], y)
// over the row's live slots in slot order, starting from +0.  This is the
// rounding sequence of the reference CPU kernel (csrc/kernels/spmm_avx2.cpp:
// 82-263, whose 16/8/1-wide stages all perform that same fused update per
// element), so results are bit-identical.  The chain is sequential per
// element, so parallelism comes only from rows and columns.
//
// Work decomposition (gather-bound, no tensor cores): a warp owns a group of
// RPW = 32/LPR consecutive rows and a tile of TILE = LPR*VEC*CPL columns.
// Each row of the group is handled by its own LPR lanes; each lane owns CPL
// vectors of VEC consecutive columns, strided by LPR*VEC so that the lanes
// of a row read X rows as contiguous, coalesced 128-bit segments.  All rows
// of the group advance together: per chunk the warp stages the next CH
// (col, value) pairs of EVERY row of the group into shared memory with
// coalesced loads (one row-run of CH slots per load instruction; rows padded
// to CH+1 pairs so the groups' broadcast reads fall in different banks),
// then each lane walks its own row's staged slots.  Work items (row group,
// column tile) are ordered row-group fastest, so that the warps resident
// together work on one band of column tiles whose X slice stays in L2.
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "tma.cuh"

namespace slb {
namespace {

constexpr int kFwdWarps = 4;
constexpr int kFwdThreads = kFwdWarps * 32;

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

// Exact (erf) GELU with the rounding steps of torch's CUDA kernel for
// F.gelu(approximate="none"): (x * 0.5) * (1 + erf(x * sqrt(1/2))), each
// operation rounded to fp32 -- so a fused epilogue matches torch bit for bit.
__device__ __forceinline__ float gelu_erf(float x) {
    const float kAlpha = 0.70710678118654752440f;
    return __fmul_rn(__fmul_rn(x, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn(x, kAlpha))));
}

// Forward epilogue: Y = acc (+ bias[row]) and, with H, H = act(Y); act 0 =
// none, 1 = ReLU (torch.relu: negative -> 0, NaN stays), 2 = GELU (exact erf).
// The bias add is one fp32 add, as torch's broadcast add after the layer.
struct Epi {
    float* H = nullptr;
    const float* bias = nullptr;
    int act = 0;
};
__device__ __forceinline__ float epi_act(float v, int act) {
    if (act == 2) return gelu_erf(v);
    if (act == 1) return v < 0.0f ? 0.0f : v;
    return v;
}
__device__ __forceinline__ void epi_store4(const Epi& epi, float* y, int64_t off, int row, float a0,
                                           float a1, float a2, float a3) {
    if (epi.bias) {
        const float b = __ldg(epi.bias + row);
        a0 = __fadd_rn(a0, b); a1 = __fadd_rn(a1, b); a2 = __fadd_rn(a2, b); a3 = __fadd_rn(a3, b);
    }
    *reinterpret_cast<float4*>(y + off) = make_float4(a0, a1, a2, a3);
    if (epi.H)
        *reinterpret_cast<float4*>(epi.H + off) =
            make_float4(epi_act(a0, epi.act), epi_act(a1, epi.act), epi_act(a2, epi.act),
                        epi_act(a3, epi.act));
}
__device__ __forceinline__ void epi_store1(const Epi& epi, float* y, int64_t off, int row, float a) {
    if (epi.bias) a = __fadd_rn(a, __ldg(epi.bias + row));
    y[off] = a;
    if (epi.H) epi.H[off] = epi_act(a, epi.act);
}

// Slot staging.  Per chunk the warp moves slots [base, base+CH) of each of
// its RPW rows into shared memory (row r at st + r*(CH+1)).  The loads of a
// chunk go to registers first (ITER = RPW*CH/32 per lane, one row-run of CH
// slots per warp-wide load), so the next chunk's loads can be in flight while
// the current chunk is computed.  rs/nn are held by the lanes of each row
// group (lane r*LPR has row r's).  Slots past a row's nnz are not loaded.
// Rows are STRIDE pairs apart (CH + 1 by default; CH + 2 keeps every row
// 16-byte aligned for paired 128-bit reads).
template <int LPR, int CH, int STRIDE = CH + 1>
struct SlotStager {
    static constexpr int RPW = 32 / LPR;
    static constexpr int ITER = RPW * CH / 32;
    static_assert(ITER * 32 == RPW * CH, "CH must fill whole warp loads");
    int c[ITER];
    float v[ITER];

    __device__ __forceinline__ void load(int rs, int nn, int base, const int32_t* __restrict__ cols,
                                         const float* __restrict__ vals) {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int it = 0; it < ITER; ++it) {
            const int idx = it * 32 + lane;
            const int r = idx / CH, t = idx % CH;
            const int r_rs = __shfl_sync(0xffffffffu, rs, r * LPR);
            const int r_nn = __shfl_sync(0xffffffffu, nn, r * LPR);
            c[it] = 0;
            v[it] = 0.0f;
            if (base + t < r_nn) {
                c[it] = __ldg(cols + r_rs + base + t);
                v[it] = __ldg(vals + r_rs + base + t);
            }
        }
    }
    __device__ __forceinline__ void store(int2* st) const {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int it = 0; it < ITER; ++it) {
            const int idx = it * 32 + lane;
            st[(idx / CH) * STRIDE + idx % CH] = make_int2(c[it], __float_as_int(v[it]));
        }
    }
};

// Staged slots per row per chunk.  Small N (many rows per warp, short
// compute per chunk): ITER = 16 loads per lane in flight.  Large N (one row
// per warp, long compute per chunk): ITER = 2 keeps registers for the
// accumulators.
template <int LPR>
struct ChunkOf {
    static constexpr int value = LPR >= 16 ? 2 * LPR : 16 * LPR;
};

template <int VEC, int LPR, int CPL>
__global__ void __launch_bounds__(kFwdThreads)
spmm_fwd_kernel(int M, int64_t N, const int32_t* __restrict__ row_start,
                const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                const float* __restrict__ vals, const float* __restrict__ X,
                float* __restrict__ Y, int64_t n_tiles, int64_t n_items, Epi epi) {
    constexpr int RPW = 32 / LPR;
    constexpr int TILE = LPR * VEC * CPL;
    constexpr int CH = ChunkOf<LPR>::value;
    __shared__ int2 stage[kFwdWarps][RPW * (CH + 1)];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane / LPR, li = lane % LPR;
    const int warps_per_block = blockDim.x >> 5;
    int2* st = stage[warp];
    const int2* my = st + g * (CH + 1);

    for (int64_t item = static_cast<int64_t>(blockIdx.x) * warps_per_block + warp; item < n_items;
         item += static_cast<int64_t>(gridDim.x) * warps_per_block) {
        // Row groups fastest: the warps resident together share one band of
        // column tiles, whose X slice stays in L2 (W is small and stays in
        // L2 across bands).
        const int64_t n_groups = (M + RPW - 1) / RPW;
        const int64_t nt = item / n_groups;
        const int row = static_cast<int>(item % n_groups) * RPW + g;
        const bool valid = row < M;
        int rs = 0, nn = 0;
        if (valid) {
            rs = __ldg(row_start + row);
            nn = __ldg(row_nnz + row);
        }
        int maxnn = nn;
#pragma unroll
        for (int o = 16; o >= LPR; o >>= 1) maxnn = max(maxnn, __shfl_xor_sync(0xffffffffu, maxnn, o));

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

        SlotStager<LPR, CH> sg;
        if (maxnn > 0) sg.load(rs, nn, 0, cols, vals);
        for (int base = 0; base < maxnn; base += CH) {
            sg.store(st);
            __syncwarp();
            if (base + CH < maxnn) sg.load(rs, nn, base + CH, cols, vals);  // next chunk in flight
            const int cnt = min(CH, nn - base);
#pragma unroll 8
            for (int t = 0; t < cnt; ++t) {
                const int2 e = my[t];
                const float v = __int_as_float(e.y);
                const float* xr = X + static_cast<int64_t>(e.x) * N;
#pragma unroll
                for (int cc = 0; cc < CPL; ++cc) fma_vec(v, Vec<VEC>::load(xr + jl[cc]), acc[cc]);
            }
            __syncwarp();
        }

        if (valid) {
#pragma unroll
            for (int cc = 0; cc < CPL; ++cc) {
                const int64_t j = jbase + static_cast<int64_t>(cc) * LPR * VEC;
                if (j < N) {
                    if constexpr (VEC == 4)
                        epi_store4(epi, Y, static_cast<int64_t>(row) * N + j, row, acc[cc][0],
                                   acc[cc][1], acc[cc][2], acc[cc][3]);
                    else
                        epi_store1(epi, Y, static_cast<int64_t>(row) * N + j, row, acc[cc][0]);
                }
            }
        }
    }
}

// ── Small N: one row per warp ───────────────────────────────────────────
// For N < 128 a row's work is short, so rows (not columns) must supply the
// parallelism: each warp owns one row at a time (M warps in flight).  The
// row is consumed in chunks of 32 slots: every lane holds one (col, value)
// pair of a chunk, and the pairs of the next three chunks are already in
// flight in a four-entry register ring (a chunk's chain is short, so the
// loads need that distance to cover HBM latency).  A chunk's pairs go to the
// warp's shared-memory buffer and the warp walks them in slot order, two
// pairs per 128-bit broadcast read; lane j accumulates columns j, j+32, ...
// (CPL of them).  With N = 1 each lane gathers X[col] of its pair one chunk
// ahead and the buffer holds (value, x), so the chain costs half a shared
// load and one FMA per slot.  Same FMA chain per element as above.
// OFF32 (K * N < 2^31): the staged pair holds the X row's element offset
// c * N instead of c, so each gather's address is one 32x32+64 multiply-add
// from a per-lane base instead of 64-bit multiply, add and shift (those made
// the N = 32 walk issue-bound at 11 instructions per slot).
template <int CPL, bool N1, bool FULL, bool OFF32 = false>
__global__ void __launch_bounds__(256)
spmm_rowwarp_kernel(int M, int64_t N, const int32_t* __restrict__ row_start,
                    const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                    const float* __restrict__ vals, const float* __restrict__ X,
                    float* __restrict__ Y) {
    constexpr int R = 4;  // register ring of chunk pairs
    __shared__ __align__(16) int2 buf[8][32];
    const int lane = threadIdx.x & 31;
    int2* st = buf[threadIdx.x >> 5];
    const int4* st4 = reinterpret_cast<const int4*>(st);
    // Columns past N (FULL = false) read a valid clamped address; their
    // accumulators are never stored, so the loads need no predicate.
    int jcol[CPL];
#pragma unroll
    for (int k = 0; k < CPL; ++k) jcol[k] = FULL ? lane + 32 * k : min(lane + 32 * k, static_cast<int>(N) - 1);
    const float* xq[CPL];  // OFF32: per-lane column bases
#pragma unroll
    for (int k = 0; k < CPL; ++k) xq[k] = X + jcol[k];
    const int Ni = static_cast<int>(N);
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M; row += warps) {
        const int rs = __ldg(row_start + row);
        const int nn = __ldg(row_nnz + row);
        float acc[CPL];
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc) acc[cc] = 0.0f;
        int cr[R];
        float vr[R];
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int k = 32 * j + lane;
            cr[j] = k < nn ? __ldg(cols + rs + k) : 0;
            vr[j] = k < nn ? __ldg(vals + rs + k) : 0.0f;
        }
        float xn = 0.0f;
        if constexpr (N1) xn = lane < nn ? __ldg(X + cr[0]) : 0.0f;
        for (int base = 0; base < nn; base += 32 * R) {
#pragma unroll
            for (int j = 0; j < R; ++j) {
                const int b = base + 32 * j;
                if (b >= nn) break;
                if constexpr (N1) {
                    st[lane] = make_int2(__float_as_int(vr[j]), __float_as_int(xn));
                    xn = b + 32 + lane < nn ? __ldg(X + cr[(j + 1) % R]) : 0.0f;  // next chunk's gather
                } else {
                    st[lane] = make_int2(OFF32 ? cr[j] * Ni : cr[j], __float_as_int(vr[j]));
                }
                const int k = b + 32 * R + lane;  // refill: chunk b + 32R
                if (k < nn) {
                    cr[j] = __ldg(cols + rs + k);
                    vr[j] = __ldg(vals + rs + k);
                }
                __syncwarp();
                const int cnt = min(32, nn - b);
                int t = 0;
                if constexpr (N1) {
                    if (cnt == 32) {
                        // Full chunk: every shared read first, then the chain
                        // (one load latency per chunk on the critical path).
                        float4 q[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) q[i] = reinterpret_cast<const float4*>(st4)[i];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            acc[0] = fmaf(q[i].x, q[i].y, acc[0]);
                            acc[0] = fmaf(q[i].z, q[i].w, acc[0]);
                        }
                        t = 32;
                    }
#pragma unroll 8
                    for (; t + 1 < cnt; t += 2) {
                        const float4 q = reinterpret_cast<const float4*>(st4)[t >> 1];
                        acc[0] = fmaf(q.x, q.y, acc[0]);
                        acc[0] = fmaf(q.z, q.w, acc[0]);
                    }
                    if (t < cnt) {
                        const int2 e = st[t];
                        acc[0] = fmaf(__int_as_float(e.x), __int_as_float(e.y), acc[0]);
                    }
                } else {
                    if (cnt == 32) {
                        // Full chunk, in groups of G pairs: the group's shared
                        // reads, then its X loads, then its FMAs.
                        constexpr int G = CPL == 1 ? 8 : (CPL == 2 ? 4 : 2);  // int4 = two slots
#pragma unroll
                        for (int h = 0; h < 16; h += G) {
                            int4 e[G];
#pragma unroll
                            for (int i = 0; i < G; ++i) e[i] = st4[h + i];
                            float xa[G][CPL], xb[G][CPL];
#pragma unroll
                            for (int i = 0; i < G; ++i)
#pragma unroll
                                for (int q = 0; q < CPL; ++q) {
                                    if constexpr (OFF32) {
                                        xa[i][q] = __ldg(xq[q] + e[i].x);
                                        xb[i][q] = __ldg(xq[q] + e[i].z);
                                    } else {
                                        xa[i][q] = __ldg(X + static_cast<int64_t>(e[i].x) * N + jcol[q]);
                                        xb[i][q] = __ldg(X + static_cast<int64_t>(e[i].z) * N + jcol[q]);
                                    }
                                }
#pragma unroll
                            for (int i = 0; i < G; ++i)
#pragma unroll
                                for (int q = 0; q < CPL; ++q) {
                                    acc[q] = fmaf(__int_as_float(e[i].y), xa[i][q], acc[q]);
                                    acc[q] = fmaf(__int_as_float(e[i].w), xb[i][q], acc[q]);
                                }
                        }
                        t = 32;
                    }
                    constexpr int kUnroll = CPL >= 3 ? 4 : 8;
#pragma unroll kUnroll
                    for (; t + 1 < cnt; t += 2) {
                        const int4 e = st4[t >> 1];
#pragma unroll
                        for (int q = 0; q < CPL; ++q) {
                            float a0, a1;
                            if constexpr (OFF32) {
                                a0 = __ldg(xq[q] + e.x);
                                a1 = __ldg(xq[q] + e.z);
                            } else {
                                a0 = __ldg(X + static_cast<int64_t>(e.x) * N + jcol[q]);
                                a1 = __ldg(X + static_cast<int64_t>(e.z) * N + jcol[q]);
                            }
                            acc[q] = fmaf(__int_as_float(e.y), a0, acc[q]);
                            acc[q] = fmaf(__int_as_float(e.w), a1, acc[q]);
                        }
                    }
                    if (t < cnt) {
                        const int2 e = st[t];
#pragma unroll
                        for (int q = 0; q < CPL; ++q) {
                            const float a0 = OFF32 ? __ldg(xq[q] + e.x)
                                                   : __ldg(X + static_cast<int64_t>(e.x) * N + jcol[q]);
                            acc[q] = fmaf(__int_as_float(e.y), a0, acc[q]);
                        }
                    }
                }
                __syncwarp();
            }
        }
        float* yr = Y + static_cast<int64_t>(row) * N;
#pragma unroll
        for (int k = 0; k < CPL; ++k) {
            const int64_t j = lane + 32 * k;
            if (j < N) yr[j] = acc[k];
        }
    }
}

// ── N = 1: one lane per row ─────────────────────────────────────────────
// With one dense column the bit-exact chain of a row is a single serial
// FMA sequence, so the row is the unit of parallelism and a lane (not a
// warp) owns it: the 32 lanes of a warp run 32 rows' chains side by side,
// one SIMT FMA per slot for all of them (the warp-per-row kernel spends a
// warp instruction or two per slot instead).  Each lane streams its own
// row's (col, value) arrays into its own slice of shared memory with
// 16-byte cp.async copies, kVStages stages of SEG 4-slot groups in flight;
// a lane only reads what it copied itself, so a per-thread
// cp.async.wait_group is the only synchronisation in the loop.  Copies
// start at the row's start rounded down to 4 slots; the lane skips slots
// outside [rs, rs + nnz).  X is staged in shared memory once per CTA
// (K <= kVMaxKs) or gathered through L1.  Lane slices are SEG * 4 + 4
// words apart, so the 8 lanes of a quarter-warp read distinct bank groups.
// One warp per CTA; SEG = 16-byte groups per lane per stage (16 when there
// are too few rows to give every SM two warps, so each warp keeps more
// bytes in flight; 8 otherwise).
constexpr int64_t kVMaxKs = 16384;  // largest K staged in shared memory
template <int SEG, int kVStages>
struct SpmvShape {
    static constexpr int kStride = SEG * 4 + 4;  // words per lane slice (bank spread)
    static constexpr int kStageWords = 32 * kStride;
    static constexpr size_t kBytes = size_t(kVStages) * kStageWords * 4 * 2;  // cols + values
};

template <bool CA>
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src, bool pred) {
    if constexpr (CA)
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n"
            " @p cp.async.ca.shared.global [%0], [%1], 16;\n}\n"
            ::"r"(smem_addr(smem_dst)), "l"(src), "r"(static_cast<int>(pred))
            : "memory");
    else
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n"
            " @p cp.async.cg.shared.global [%0], [%1], 16;\n}\n"
            ::"r"(smem_addr(smem_dst)), "l"(src), "r"(static_cast<int>(pred))
            : "memory");
}
__device__ __forceinline__ bool aligned16_dev(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int NPEND>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(NPEND) : "memory"); }

template <bool KS, int SEG, bool CA, int kVStages>
__global__ void __launch_bounds__(32)
spmv_lane_kernel(int M, int64_t K, int64_t cap, const int32_t* __restrict__ row_start,
                 const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                 const float* __restrict__ vals, const float* __restrict__ X,
                 float* __restrict__ Y) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    using S = SpmvShape<SEG, kVStages>;
    const int lane = threadIdx.x;
    int* cbase = reinterpret_cast<int*>(smem_raw);
    float* vbase = reinterpret_cast<float*>(smem_raw + S::kBytes / 2);
    float* xs = reinterpret_cast<float*>(smem_raw + S::kBytes);

    const int row = blockIdx.x * 32 + lane;
    const bool live = row < M;
    const int rs = live ? __ldg(row_start + row) : 0;
    const int nn = live ? __ldg(row_nnz + row) : 0;
    const int a = rs & ~3;  // first copied slot
    const int ngroups = nn > 0 ? (rs + nn - a + 3) >> 2 : 0;
    // A last group that would read past the arrays' end is loaded directly.
    const int tailg = (nn > 0 && a + 4 * static_cast<int64_t>(ngroups) > cap) ? ngroups - 1 : -1;
    const int ncopy = tailg >= 0 ? ngroups - 1 : ngroups;
    const int nst = __reduce_max_sync(0xffffffffu, (ngroups + SEG - 1) / SEG);

    // Each lane copies its own row's groups (16 bytes per copy).
    auto issue = [&](int st) {  // one commit group per stage, empty ones included
        const int b = st % kVStages;
#pragma unroll
        for (int g = 0; g < SEG; ++g) {
            const int gi = st * SEG + g;
            const bool p = gi < ncopy;
            const int64_t off = p ? a + 4 * static_cast<int64_t>(gi) : 0;
            const int dw = b * S::kStageWords + lane * S::kStride + 4 * g;
            cp_async16<CA>(cbase + dw, cols + off, p);
            cp_async16<CA>(vbase + dw, vals + off, p);
        }
        cp_async_commit();
    };
    const bool xasync = KS && (K % 4 == 0) && aligned16_dev(X);
    if (KS) {
        if (xasync) {
            for (int64_t k = 4 * lane; k < K; k += 128) cp_async16<false>(xs + k, X + k, true);
        } else {
            for (int64_t k = lane; k < K; k += 32) xs[k] = __ldg(X + k);
        }
    }
    cp_async_commit();  // X (oldest group)
#pragma unroll
    for (int st = 0; st < kVStages - 1; ++st) issue(st);
    cp_async_wait<kVStages - 1>();  // X has landed
    __syncwarp();

    float y = 0.0f;
    const int* cb = cbase + lane * S::kStride;
    const float* vb = vbase + lane * S::kStride;
    for (int st = 0; st < nst; ++st) {
        issue(st + kVStages - 1);      // refill the slot freed at st - 1
        cp_async_wait<kVStages - 1>();  // stage st has landed (a lane reads only its own copies)
        const int b = st % kVStages;
        const int4* c4 = reinterpret_cast<const int4*>(cb + b * S::kStageWords);
        const float4* v4 = reinterpret_cast<const float4*>(vb + b * S::kStageWords);
        // Straight-line over the stage: every shared load (group and X
        // gather, clamped to a valid address) is unconditional so they can
        // all be in flight before the chain; only the FMA is predicated.
#pragma unroll
        for (int g = 0; g < SEG; ++g) {
            const int gi = st * SEG + g;
            const int64_t s0 = a + 4 * static_cast<int64_t>(gi);
            int c[4];
            float v[4];
            if (gi == tailg) {
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const bool in = s0 + t < rs + nn;
                    c[t] = in ? __ldg(cols + s0 + t) : 0;
                    v[t] = in ? __ldg(vals + s0 + t) : 0.0f;
                }
            } else {
                const int4 cc = c4[g];
                const float4 vv = v4[g];
                c[0] = cc.x; c[1] = cc.y; c[2] = cc.z; c[3] = cc.w;
                v[0] = vv.x; v[1] = vv.y; v[2] = vv.z; v[3] = vv.w;
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const bool in = static_cast<unsigned>(static_cast<int>(s0) + t - rs) < static_cast<unsigned>(nn);
                const int cc = in ? c[t] : 0;
                const float x = KS ? xs[cc] : __ldg(X + cc);
                if (in) y = fmaf(v[t], x, y);
            }
        }
    }
    cp_async_wait<0>();
    if (live) Y[row] = y;
}

template <bool KS, int SEG, bool CA, int ST>
int launch_spmv_cfg(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    const int M = static_cast<int>(W->nrows);
    const size_t smem = SpmvShape<SEG, ST>::kBytes + (KS ? static_cast<size_t>(K) * 4 : 0);
    auto kern = spmv_lane_kernel<KS, SEG, CA, ST>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int blocks = (M + 31) / 32;
    note_kernel("spmv_lane_kernel");
    kern<<<blocks, 32, smem, s>>>(M, K, W->total_capacity, W->row_start, W->row_nnz,
                                  W->col_indices, W->values, X, Y);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd (N = 1)");
    return SL_OK;
}

// Measured on B200 (4096 and 16384 rows x 4096 at 50-95%): with fewer warps
// than two per SM, 16-group stages through L1 (cp.async.ca) keep the most
// bytes in flight; with more, 8-group stages that bypass L1 (cp.async.cg),
// so the many warps' rows do not evict each other.  Four stages, X in
// shared memory, in both (deeper rings or X through L1 were slower).
int launch_spmv(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s) {
    const int64_t warps = (W->nrows + 31) / 32;
    const bool small = warps <= 2 * num_sms();
    if (K <= kVMaxKs)
        return small ? launch_spmv_cfg<true, 16, true, 4>(W, X, K, Y, s)
                     : launch_spmv_cfg<true, 8, false, 4>(W, X, K, Y, s);
    return small ? launch_spmv_cfg<false, 16, true, 4>(W, X, K, Y, s)
                 : launch_spmv_cfg<false, 8, false, 4>(W, X, K, Y, s);
}

// ── N = 4 or 8: one lane per row ─────────────────────────────────────────
// The N = 1 scheme with N / 4 float4 columns per lane: lane = row, its
// (col, value) stream staged by per-lane cp.async exactly as above, and per
// slot the lane gathers its X row (NV 16-byte loads through L1) and updates
// its 4 * NV column accumulators, each in slot order (the reference's chain
// per output element).  A warp advances 32 rows by one slot with NV loads
// and 4 * NV FMAs, where the warp-per-row kernel spends several warp
// instructions and a dependent shared round trip per slot.
template <int NV>
__global__ void __launch_bounds__(32)
spmm_lanerow_kernel(int M, int64_t cap, const int32_t* __restrict__ row_start,
                    const int32_t* __restrict__ row_nnz, const int32_t* __restrict__ cols,
                    const float* __restrict__ vals, const float* __restrict__ X,
                    float* __restrict__ Y) {
    constexpr int SEG = 8, ST = 4;
    constexpr int N = 4 * NV;
    using S = SpmvShape<SEG, ST>;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x;
    int* cbase = reinterpret_cast<int*>(smem_raw);
    float* vbase = reinterpret_cast<float*>(smem_raw + S::kBytes / 2);
    const int row = blockIdx.x * 32 + lane;
    const bool live = row < M;
    const int rs = live ? __ldg(row_start + row) : 0;
    const int nn = live ? __ldg(row_nnz + row) : 0;
    const int a = rs & ~3;
    const int ngroups = nn > 0 ? (rs + nn - a + 3) >> 2 : 0;
    const int tailg = (nn > 0 && a + 4 * static_cast<int64_t>(ngroups) > cap) ? ngroups - 1 : -1;
    const int ncopy = tailg >= 0 ? ngroups - 1 : ngroups;
    const int nst = __reduce_max_sync(0xffffffffu, (ngroups + SEG - 1) / SEG);
    auto issue = [&](int st) {
        const int b = st % ST;
#pragma unroll
        for (int g = 0; g < SEG; ++g) {
            const int gi = st * SEG + g;
            const bool p = gi < ncopy;
            const int64_t off = p ? a + 4 * static_cast<int64_t>(gi) : 0;
            const int dw = b * S::kStageWords + lane * S::kStride + 4 * g;
            cp_async16<false>(cbase + dw, cols + off, p);
            cp_async16<false>(vbase + dw, vals + off, p);
        }
        cp_async_commit();
    };
#pragma unroll
    for (int st = 0; st < ST - 1; ++st) issue(st);

    float4 acc[NV];
#pragma unroll
    for (int q = 0; q < NV; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int* cb = cbase + lane * S::kStride;
    const float* vb = vbase + lane * S::kStride;
    for (int st = 0; st < nst; ++st) {
        issue(st + ST - 1);
        cp_async_wait<ST - 1>();
        const int b = st % ST;
        const int4* c4 = reinterpret_cast<const int4*>(cb + b * S::kStageWords);
        const float4* v4 = reinterpret_cast<const float4*>(vb + b * S::kStageWords);
#pragma unroll 2
        for (int g = 0; g < SEG; ++g) {
            const int gi = st * SEG + g;
            const int64_t s0 = a + 4 * static_cast<int64_t>(gi);
            int c[4];
            float v[4];
            if (gi == tailg) {
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const bool in = s0 + t < rs + nn;
                    c[t] = in ? __ldg(cols + s0 + t) : 0;
                    v[t] = in ? __ldg(vals + s0 + t) : 0.0f;
                }
            } else {
                const int4 cc = c4[g];
                const float4 vv = v4[g];
                c[0] = cc.x; c[1] = cc.y; c[2] = cc.z; c[3] = cc.w;
                v[0] = vv.x; v[1] = vv.y; v[2] = vv.z; v[3] = vv.w;
            }
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const bool in = static_cast<unsigned>(static_cast<int>(s0) + t - rs) < static_cast<unsigned>(nn);
                const float4* xr = reinterpret_cast<const float4*>(X + static_cast<int64_t>(in ? c[t] : 0) * N);
                float4 x[NV];
#pragma unroll
                for (int q = 0; q < NV; ++q) x[q] = __ldg(xr + q);
                if (in) {
#pragma unroll
                    for (int q = 0; q < NV; ++q) {
                        acc[q].x = fmaf(v[t], x[q].x, acc[q].x);
                        acc[q].y = fmaf(v[t], x[q].y, acc[q].y);
                        acc[q].z = fmaf(v[t], x[q].z, acc[q].z);
                        acc[q].w = fmaf(v[t], x[q].w, acc[q].w);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
    if (live) {
        float4* yr = reinterpret_cast<float4*>(Y + static_cast<int64_t>(row) * N);
#pragma unroll
        for (int q = 0; q < NV; ++q) yr[q] = acc[q];
    }
}

template <int NV>
int launch_lanerow_nv(const sl_csr* W, const float* X, float* Y, cudaStream_t s) {
    const size_t smem = SpmvShape<8, 4>::kBytes;
    if (cudaFuncSetAttribute(spmm_lanerow_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int M = static_cast<int>(W->nrows);
    note_kernel("spmm_lanerow_kernel");
    spmm_lanerow_kernel<NV><<<(M + 31) / 32, 32, smem, s>>>(M, W->total_capacity, W->row_start,
                                                             W->row_nnz, W->col_indices, W->values, X, Y);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd (lane per row)");
    return SL_OK;
}

// Returns -1 when the lane-per-row path does not apply.  Measured on B200
// (4096 and 16384 rows x 4096, 50-99%): it wins only for N <= 8 with at
// least three warps of rows per SM (16384 x 4096, N = 8: 225 vs 458 us at
// 50%); with fewer rows, or N = 32 (a 128-byte X row per lane per slot
// through L1), the warp-per-row kernel is faster.
// SPARSECORE_B200_SMALLN=warp|lane forces one of the two (tests).
int try_lanerow(const sl_csr* W, const float* X, int64_t N, float* Y, cudaStream_t s) {
    if (N < 4 || N > 8 || N % 4 != 0 || !aligned16(X) || !aligned16(Y) ||
        !aligned16(W->col_indices) || !aligned16(W->values) || W->nrows == 0)
        return -1;
    bool use = W->nrows >= static_cast<int64_t>(3) * 32 * num_sms();
    if (const char* e = std::getenv("SPARSECORE_B200_SMALLN")) use = e[0] == 'l';
    if (!use) return -1;
    return N == 4 ? launch_lanerow_nv<1>(W, X, Y, s) : launch_lanerow_nv<2>(W, X, Y, s);
}

// SPARSECORE_B200_N1=warp keeps N = 1 on the warp-per-row kernel (tests).
bool spmv_lane_enabled(const sl_csr* W) {
    const char* e = std::getenv("SPARSECORE_B200_N1");
    if (e != nullptr && e[0] == 'w') return false;
    return aligned16(W->col_indices) && aligned16(W->values) && W->nrows > 0;
}

template <int CPL, bool N1, bool FULL = false, bool OFF32 = false>
int launch_rowwarp(const sl_csr* W, const float* X, int64_t N, float* Y, cudaStream_t s) {
    const int M = static_cast<int>(W->nrows);
    int64_t blocks = (static_cast<int64_t>(M) + 7) / 8;
    const int64_t max_blocks = static_cast<int64_t>(num_sms()) * 8;
    if (blocks > max_blocks) blocks = max_blocks;
    note_kernel("spmm_rowwarp_kernel");
    spmm_rowwarp_kernel<CPL, N1, FULL, OFF32><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        M, N, W->row_start, W->row_nnz, W->col_indices, W->values, X, Y);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd");
    return SL_OK;
}

int dispatch_rowwarp(const sl_csr* W, const float* X, int64_t N, float* Y, cudaStream_t s) {
    if (N == 1) return launch_rowwarp<1, true>(W, X, N, Y, s);
    if (W->ncols * N <= INT_MAX) {
        if (N == 32) return launch_rowwarp<1, false, true, true>(W, X, N, Y, s);
        if (N == 64) return launch_rowwarp<2, false, true, true>(W, X, N, Y, s);
        if (N == 96) return launch_rowwarp<3, false, true, true>(W, X, N, Y, s);
        if (N <= 32) return launch_rowwarp<1, false, false, true>(W, X, N, Y, s);
        if (N <= 64) return launch_rowwarp<2, false, false, true>(W, X, N, Y, s);
        if (N <= 96) return launch_rowwarp<3, false, false, true>(W, X, N, Y, s);
        return launch_rowwarp<4, false, false, true>(W, X, N, Y, s);
    }
    if (N == 32) return launch_rowwarp<1, false, true>(W, X, N, Y, s);
    if (N == 64) return launch_rowwarp<2, false, true>(W, X, N, Y, s);
    if (N == 96) return launch_rowwarp<3, false, true>(W, X, N, Y, s);
    if (N <= 32) return launch_rowwarp<1, false>(W, X, N, Y, s);
    if (N <= 64) return launch_rowwarp<2, false>(W, X, N, Y, s);
    if (N <= 96) return launch_rowwarp<3, false>(W, X, N, Y, s);
    return launch_rowwarp<4, false>(W, X, N, Y, s);
}

template <int VEC, int LPR, int CPL>
int launch_fwd(const sl_csr* W, const float* X, int64_t N, float* Y, cudaStream_t s,
               Epi epi = Epi{}) {
    constexpr int RPW = 32 / LPR;
    constexpr int TILE = LPR * VEC * CPL;
    const int M = static_cast<int>(W->nrows);
    const int64_t n_tiles = (N + TILE - 1) / TILE;
    const int64_t n_items = ((M + RPW - 1) / RPW) * n_tiles;
    const int sms = num_sms();
    // Few items: one warp per CTA so that they spread over all SMs.
    const int threads = n_items < static_cast<int64_t>(sms) * kFwdWarps ? 32 : kFwdThreads;
    const int wpb = threads / 32;
    int64_t blocks = (n_items + wpb - 1) / wpb;
    const int64_t max_blocks = static_cast<int64_t>(sms) * (2048 / threads);
    if (blocks > max_blocks) blocks = max_blocks;
    note_kernel("spmm_fwd_kernel");
    spmm_fwd_kernel<VEC, LPR, CPL><<<static_cast<unsigned>(blocks), threads, 0, s>>>(
        M, N, W->row_start, W->row_nnz, W->col_indices, W->values, X, Y, n_tiles, n_items, epi);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd");
    return SL_OK;
}

// Lane layout by the number of column vectors per row.
template <int VEC>
int dispatch_fwd(const sl_csr* W, const float* X, int64_t N, float* Y, cudaStream_t s,
                 Epi epi = Epi{}) {
    const int64_t nv = (N + VEC - 1) / VEC;
    // SPARSECORE_B200_FWD_TILE=32|64|128|256: column tile of the row-gather
    // kernel at large N (measurements; narrower tiles make the resident
    // warps' X slice smaller, so more of its gathers hit L1).
    if (const char* e = std::getenv("SPARSECORE_B200_FWD_TILE")) {
        const int t = std::atoi(e);
        if (VEC == 4 && nv >= 64) {
            if (t == 32) return launch_fwd<VEC, 8, 1>(W, X, N, Y, s, epi);
            if (t == 64) return launch_fwd<VEC, 16, 1>(W, X, N, Y, s, epi);
            if (t == 128) return launch_fwd<VEC, 32, 1>(W, X, N, Y, s, epi);
            if (t == 256) return launch_fwd<VEC, 32, 2>(W, X, N, Y, s, epi);
        }
    }
    // 256-column tiles, or 128 when that leaves fewer than about four
    // warps' items per SM (small layers: the work per warp is a serial walk
    // of its row's slots, so more, narrower items finish sooner; config 1,
    // 256 x 784 at N = 256, measured 18.0 -> 12.1 us).
    if (nv >= 64) {
        const int64_t items256 = W->nrows * ((N + 255) / 256);
        if (items256 < 4LL * num_sms()) return launch_fwd<VEC, 32, 1>(W, X, N, Y, s, epi);
        return launch_fwd<VEC, 32, 2>(W, X, N, Y, s, epi);
    }
    if (nv > 16) return launch_fwd<VEC, 32, 1>(W, X, N, Y, s, epi);
    if (nv > 8) return launch_fwd<VEC, 16, 1>(W, X, N, Y, s, epi);
    if (nv > 4) return launch_fwd<VEC, 8, 1>(W, X, N, Y, s, epi);
    if (nv > 2) return launch_fwd<VEC, 4, 1>(W, X, N, Y, s, epi);
    if (nv > 1) return launch_fwd<VEC, 2, 1>(W, X, N, Y, s, epi);
    return launch_fwd<VEC, 1, 1>(W, X, N, Y, s, epi);
}


// ── X-stationary variant (large N) ───────────────────────────────────────
// A CTA keeps the full column tile X[:, j0 : j0+TN] (all K rows) resident in
// shared memory -- loaded by TMA as 128-row boxes completing on one mbarrier
// -- and streams rows of W against it: every FMA's X operand then comes from
// shared memory (one conflict-free 128-bit read per lane per slot) instead
// of L1/L2.  Lanes are laid out as in spmm_fwd_kernel with VEC = 4, CPL = 1
// (LPR = TN/4 lanes per row, all rows of a warp advancing together).  Work
// items are (column tile, block of rows), tile-major; each CTA takes a
// contiguous run of items and reloads X only when its tile changes.
// Numerics are identical to spmm_fwd_kernel (same per-element FMA chain).
// Threads per CTA: 1024 for the one-CTA-per-SM wide tiles (TN >= 64), so
// that 32 warps hide the shared-memory latency; 512 otherwise (two CTAs).
template <int LPR>
__host__ __device__ constexpr int xs_threads() { return LPR >= 16 ? 1024 : 512; }
constexpr int kXsBoxRows = 128;
// Staged slots per row per chunk: 16, or 32 with one row per warp (TN = 128)
// so that a chunk still fills whole warp-wide loads.
template <int LPR>
__host__ __device__ constexpr int xs_ch() { return LPR == 32 ? 32 : 16; }
constexpr int kXsRowsPerItemMul = 4;

template <int LPR, bool PACK>
__global__ void __launch_bounds__(xs_threads<LPR>())
spmm_xs_kernel(const __grid_constant__ CUtensorMap xmap, int M, int64_t N,
               const int32_t* __restrict__ row_start, const int32_t* __restrict__ row_nnz,
               const int32_t* __restrict__ cols, const float* __restrict__ vals,
               float* __restrict__ Y, Epi epi, int nbox, int row_chunks, int64_t n_items,
               int64_t items_per_cta, unsigned* status) {
    constexpr int TN = 4 * LPR;
    constexpr int RPW = 32 / LPR;
    constexpr int kXsWarps = xs_threads<LPR>() / 32;
    constexpr int ROWS_PER_ITEM = kXsWarps * RPW * kXsRowsPerItemMul;
    extern __shared__ __align__(128) unsigned char smem[];
    float* xs = reinterpret_cast<float*>(smem);
    int2* stage = reinterpret_cast<int2*>(smem + static_cast<size_t>(nbox) * kXsBoxRows * TN * 4);
    __shared__ __align__(8) uint64_t bar;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane / LPR, li = lane % LPR;
    constexpr int kXsCh = xs_ch<LPR>();
    constexpr int XST = kXsCh + 2;  // 16-byte aligned rows: two pairs per 128-bit read
    int2* st = stage + warp * RPW * XST;
    const int2* my = st + g * XST;
    const int4* my4 = reinterpret_cast<const int4*>(my);
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
            // Bounded wait; all threads agree at the barrier whether any gave
            // up, so that they leave together.
            const bool ok = mbar_wait(&bar, phase, status);
            if (__syncthreads_or(!ok)) {
                mbar_wait(&bar, phase, status);  // let copies in flight land, then leave
                return;
            }
            phase ^= 1u;
            cur_tile = tile;
        }
        const int64_t j = tile * TN + li * 4;
        const float* xcol = xs + li * 4;
        for (int rg = warp; rg < ROWS_PER_ITEM / RPW; rg += kXsWarps) {
            const int row = chunk * ROWS_PER_ITEM + rg * RPW + g;
            const bool valid = row < M;
            int rs = 0, nn = 0;
            if (valid) {
                rs = __ldg(row_start + row);
                nn = __ldg(row_nnz + row);
            }
            int maxnn = nn;
#pragma unroll
            for (int o = 16; o >= LPR; o >>= 1)
                maxnn = max(maxnn, __shfl_xor_sync(0xffffffffu, maxnn, o));
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            SlotStager<LPR, kXsCh, XST> sg;
            if (maxnn > 0) sg.load(rs, nn, 0, cols, vals);
            for (int base = 0; base < maxnn; base += kXsCh) {
                if constexpr (PACK) {
                    // Packed staging: per row kXsCh values, then kXsCh 16-bit
                    // X-tile offsets col * TN (below 65536: the K x TN tile
                    // fits in shared memory), so 8 slots cost three 128-bit
                    // reads instead of four and no lane multiplies.
#pragma unroll
                    for (int it = 0; it < SlotStager<LPR, kXsCh, XST>::ITER; ++it) {
                        const int idx = it * 32 + lane;
                        float* rv = reinterpret_cast<float*>(st + (idx / kXsCh) * XST);
                        rv[idx % kXsCh] = sg.v[it];
                        reinterpret_cast<unsigned short*>(rv + kXsCh)[idx % kXsCh] =
                            static_cast<unsigned short>(sg.c[it] * TN);
                    }
                } else {
                    sg.store(st);
                }
                __syncwarp();
                if (base + kXsCh < maxnn) sg.load(rs, nn, base + kXsCh, cols, vals);
                const int cnt = min(kXsCh, nn - base);
                int t = 0;
                if constexpr (PACK) {
                    const float* vrow = reinterpret_cast<const float*>(my);
                    const unsigned short* crow = reinterpret_cast<const unsigned short*>(vrow + kXsCh);
                    for (; t + 8 <= cnt; t += 8) {
                        const uint4 cw = *reinterpret_cast<const uint4*>(crow + t);
                        const float4 va = *reinterpret_cast<const float4*>(vrow + t);
                        const float4 vb = *reinterpret_cast<const float4*>(vrow + t + 4);
                        const unsigned cwa[4] = {cw.x, cw.y, cw.z, cw.w};
                        const float vv[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            const int c = static_cast<int>((cwa[u >> 1] >> (16 * (u & 1))) & 0xffffu);
                            fma_vec(vv[u], *reinterpret_cast<const float4*>(xcol + c), acc);
                        }
                    }
                    for (; t < cnt; ++t)
                        fma_vec(vrow[t], *reinterpret_cast<const float4*>(xcol + crow[t]), acc);
                } else {
#pragma unroll 4
                    for (; t + 1 < cnt; t += 2) {
                        const int4 e = my4[t >> 1];
                        const float4 x0 = *reinterpret_cast<const float4*>(xcol + e.x * TN);
                        const float4 x1 = *reinterpret_cast<const float4*>(xcol + e.z * TN);
                        fma_vec(__int_as_float(e.y), x0, acc);
                        fma_vec(__int_as_float(e.w), x1, acc);
                    }
                    if (t < cnt) {
                        const int2 e = my[t];
                        const float4 x = *reinterpret_cast<const float4*>(xcol + e.x * TN);
                        fma_vec(__int_as_float(e.y), x, acc);
                    }
                }
                __syncwarp();
            }
            if (valid && j < N)
                epi_store4(epi, Y, static_cast<int64_t>(row) * N + j, row, acc[0], acc[1], acc[2],
                           acc[3]);
        }
    }
}

bool xs_lanes_for128(int64_t K) {
    const int64_t rows = (K + kXsBoxRows - 1) / kXsBoxRows * kXsBoxRows;
    return rows * 128 * 4 <= 200 * 1024;
}

// Whether a K x 64 tile (TMA boxes of 128 rows) fits next to the staging.
bool xs_lanes_for64(int64_t K) {
    const int64_t rows = (K + kXsBoxRows - 1) / kXsBoxRows * kXsBoxRows;
    return rows * 64 * 4 <= 200 * 1024;
}

// Tile width by K so that the resident tile fits in shared memory.
int xs_lanes_for(int64_t K) {
    const int64_t rows = (K + kXsBoxRows - 1) / kXsBoxRows * kXsBoxRows;
    const int64_t budget = 192 * 1024;
    // Narrower tiles put more rows on a warp and lose to the row-gather
    // kernel (measured on B200), so only TN = 32 is used.
    return rows * 32 * 4 <= budget ? 8 : 0;
}

template <int LPR>
int launch_xs(const sl_csr* W, const float* X, int64_t K, int64_t N, float* Y, cudaStream_t s,
              Epi epi = Epi{}) {
    constexpr int TN = 4 * LPR;
    constexpr int RPW = 32 / LPR;
    constexpr int kXsWarps = xs_threads<LPR>() / 32;
    constexpr int ROWS_PER_ITEM = kXsWarps * RPW * kXsRowsPerItemMul;
    CUtensorMap map;
    if (!make_tmap_2d(&map, X, K, N, kXsBoxRows, TN)) return -1;
    unsigned* status = device_status_word();
    if (status == nullptr) return -1;
    const int M = static_cast<int>(W->nrows);
    const int nbox = static_cast<int>((K + kXsBoxRows - 1) / kXsBoxRows);
    const size_t smem = static_cast<size_t>(nbox) * kXsBoxRows * TN * 4 +
                        static_cast<size_t>(kXsWarps) * RPW * (xs_ch<LPR>() + 2) * sizeof(int2);
    // Packed (16-bit column) staging by default; SPARSECORE_B200_XS_PACK=0
    // keeps (col, value) pairs (tests and measurements).
    const char* pk = std::getenv("SPARSECORE_B200_XS_PACK");
    const bool pack = !(pk != nullptr && pk[0] == '0') && K * TN < 65536;
    auto kern = pack ? spmm_xs_kernel<LPR, true> : spmm_xs_kernel<LPR, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return -1;
    const int row_chunks = (M + ROWS_PER_ITEM - 1) / ROWS_PER_ITEM;
    const int64_t n_tiles = (N + TN - 1) / TN;
    const int64_t n_items = n_tiles * row_chunks;
    // Resident CTAs per SM: one for the 1024-thread wide tiles (registers),
    // else two when the shared memory allows.
    const int per_sm = (xs_threads<LPR>() == 1024 || smem > 112 * 1024) ? 1 : 2;
    int64_t grid = static_cast<int64_t>(num_sms()) * per_sm;
    if (grid > n_items) grid = n_items;
    const int64_t per_cta = (n_items + grid - 1) / grid;
    grid = (n_items + per_cta - 1) / per_cta;
    note_kernel("spmm_xs_kernel");
    kern<<<static_cast<unsigned>(grid), xs_threads<LPR>(), smem, s>>>(
        map, M, N, W->row_start, W->row_nnz, W->col_indices, W->values, Y, epi, nbox, row_chunks,
        n_items, per_cta, status);
    SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd (x-stationary)");
    return SL_OK;
}

// SPARSECORE_B200_FWD=rows|xs forces one forward path (tuning and tests);
// by default the X-stationary path runs where it applies.
enum { kPathAuto = 0, kPathRows = 1, kPathXs = 2 };
int fwd_path() {
    const char* e = std::getenv("SPARSECORE_B200_FWD");
    if (e && std::strcmp(e, "rows") == 0) return kPathRows;
    if (e && std::strcmp(e, "xs") == 0) return kPathXs;
    return kPathAuto;
}

// Returns -1 when the X-stationary path does not apply.
int try_xs(const sl_csr* W, const float* X, int64_t K, int64_t N, float* Y, cudaStream_t s,
           bool forced, Epi epi = Epi{}) {
    if (N < 256 || N % 4 != 0 || !aligned16(X) || !aligned16(Y) || K < 1 || K > INT_MAX) return -1;
    // Measured on B200 (config-4/5 shapes, N = 16384): with 64- or 128-column
    // tiles (K <= 768) the X-stationary kernel beats the row-gather kernel on
    // every layer measured (384 to 3072 rows, 1-12%); with 32-column tiles
    // only when M >= 1536 (many rows per resident tile).  Below 256 rows a
    // resident tile serves too few rows; the row-gather kernel keeps those.
    if (!forced && W->nrows < 1536 && !(xs_lanes_for64(K) && W->nrows >= 256)) return -1;
    // Tile width: the widest of 128 / 64 / 32 columns whose K x TN tile fits
    // (each staged (col, value) pair feeds TN FMAs).  Measured on B200:
    // TN = 64 over 32 +6% on the config-5 K = 768 layers, TN = 128 over 64
    // +7-11% on the config-4 K = 384 layers.  Tuning knob
    // SPARSECORE_B200_XS_TN=32|64|128.
    int tn = xs_lanes_for128(K) ? 128 : xs_lanes_for64(K) ? 64 : (xs_lanes_for(K) == 8 ? 32 : 0);
    if (const char* e = std::getenv("SPARSECORE_B200_XS_TN")) {
        const int v = std::atoi(e);
        if (v == 32 && xs_lanes_for(K) == 8) tn = 32;
        if (v == 64 && xs_lanes_for64(K)) tn = 64;
        if (v == 128 && xs_lanes_for128(K)) tn = 128;
    }
    if (tn == 128) return launch_xs<32>(W, X, K, N, Y, s, epi);
    if (tn == 64) return launch_xs<16>(W, X, K, N, Y, s, epi);
    if (tn == 32) return launch_xs<8>(W, X, K, N, Y, s, epi);
    return -1;
}
}  // namespace
}  // namespace slb

using namespace slb;

namespace slb {
namespace {
// Epilogue as a second pass, for the decompositions without one: Y += bias
// (in place) and H = act(Y).
__global__ void __launch_bounds__(256) epi_kernel(float* __restrict__ Y, Epi epi, int64_t N,
                                                  int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v = Y[i];
        if (epi.bias) {
            v = __fadd_rn(v, __ldg(epi.bias + i / N));
            Y[i] = v;
        }
        if (epi.H) epi.H[i] = epi_act(v, epi.act);
    }
}

// The forward dispatch with its epilogue (bias, activation) fused into the
// X-stationary and row-gather kernels, else applied by a second pass.
int spmm_fwd_impl(const sl_csr* W, const float* X, int64_t K, int64_t N, float* Y, Epi epi,
                  cudaStream_t s) {
    const int path = fwd_path();
    int rc = -1;
    if (path != kPathRows) rc = try_xs(W, X, K, N, Y, s, path == kPathXs, epi);
    if (rc >= 0) return rc;
    if (N >= 128) {
        const bool vec4 = (N % 4 == 0) && aligned16(X) && aligned16(Y) && (epi.H == nullptr || aligned16(epi.H));
        return vec4 ? dispatch_fwd<4>(W, X, N, Y, s, epi) : dispatch_fwd<1>(W, X, N, Y, s, epi);
    }
    if (N == 1 && spmv_lane_enabled(W)) {
        // Measured on B200 (4096 and 16384 rows x 4096, 50-99%): the
        // warp-specialised window kernel wins with long rows (with one CTA
        // per SM from about 100 slots per row, with more rows from about
        // 600); short rows keep the per-lane kernel, whose start-up is
        // cheaper.  SPARSECORE_B200_N1=lane|ws forces one (tests).
        const char* e = std::getenv("SPARSECORE_B200_N1");
        const double avg = static_cast<double>(W->total_capacity) / 1.2 / static_cast<double>(W->nrows);
        bool ws = (W->nrows + 31) / 32 <= num_sms() ? avg >= 96.0 : avg >= 600.0;
        if (e != nullptr && e[0] == 'l') ws = false;
        if (e != nullptr && e[0] == 'w' && e[1] == 's') ws = true;
        rc = ws ? launch_spmv_ws(W, X, K, Y, s) : -1;
        if (rc < 0) rc = launch_spmv(W, X, K, Y, s);
    }
    if (rc < 0 && (N == 4 || N == 8)) rc = try_lanerow(W, X, N, Y, s);
    // N = 32: the row-warp kernel (32-bit offsets) measured faster than the
    // cp.async-staged gather (4096^2 at 90%: 27.3 vs 31.9 us; L1 hits on the
    // gathered X rows, which cp.async.cg bypasses); SPARSECORE_B200_N32=gather
    // selects the staged kernel (tests).
    if (rc < 0 && N == 32 && gather32_forced()) rc = launch_gather32_fwd(W, X, Y, s);
    if (rc < 0) rc = dispatch_rowwarp(W, X, N, Y, s);
    if (rc == SL_OK && (epi.H != nullptr || epi.bias != nullptr)) {
        const int64_t n = W->nrows * N;
        int64_t blocks = (n + 255) / 256;
        const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
        epi_kernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, s>>>(Y, epi, N, n);
        SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd_act");
    }
    return rc;
}

int check_fwd_args(const sl_csr* W, const float* X, int64_t K, int64_t N, const float* Y,
                   const char* fn) {
    if (int rc = check_csr(W, fn)) return rc;
    if (W->ncols != K)
        return fail(SL_ERR_INVALID, std::string(fn) + ": shape mismatch. W has ncols=" +
                                        std::to_string(W->ncols) + " but X has shape[0]=" +
                                        std::to_string(K) +
                                        ". Inner dimensions must match for matmul.");
    if (N < 0) return fail(SL_ERR_INVALID, std::string(fn) + ": negative N");
    if (W->nrows == 0 || N == 0) return -1;  // nothing to do
    if (Y == nullptr || (K > 0 && X == nullptr))
        return fail(SL_ERR_INVALID, std::string(fn) + ": NULL dense operand");
    return SL_OK;
}
}  // namespace
}  // namespace slb

extern "C" int sl_spmm_fwd(const sl_csr* W, const float* X, int64_t K, int64_t N, float* Y,
                           void* stream) {
    const int rc = check_fwd_args(W, X, K, N, Y, "sl_spmm_fwd");
    if (rc < 0) return SL_OK;
    if (rc != SL_OK) return rc;
    cudaStream_t s = as_stream(stream);
    if (K == 0) return cuda_status(cudaMemsetAsync(Y, 0, sizeof(float) * W->nrows * N, s),
                                   "sl_spmm_fwd memset");
    return spmm_fwd_impl(W, X, K, N, Y, Epi{}, s);
}

extern "C" int sl_spmm_fwd_gelu(const sl_csr* W, const float* X, int64_t K, int64_t N, float* Y,
                                float* H, void* stream) {
    const int rc = check_fwd_args(W, X, K, N, Y, "sl_spmm_fwd_gelu");
    if (rc < 0) return SL_OK;
    if (rc != SL_OK) return rc;
    if (H == nullptr) return fail(SL_ERR_INVALID, "sl_spmm_fwd_gelu: NULL H");
    cudaStream_t s = as_stream(stream);
    if (K == 0) {
        if (int e = cuda_status(cudaMemsetAsync(Y, 0, sizeof(float) * W->nrows * N, s), "sl_spmm_fwd_gelu memset"))
            return e;
        return cuda_status(cudaMemsetAsync(H, 0, sizeof(float) * W->nrows * N, s), "sl_spmm_fwd_gelu memset");
    }
    Epi epi;
    epi.H = H;
    epi.act = 2;
    return spmm_fwd_impl(W, X, K, N, Y, epi, s);
}

extern "C" int sl_spmm_fwd_act(const sl_csr* W, const float* X, int64_t K, int64_t N,
                               const float* bias, int act, float* Y, float* H, void* stream) {
    const int rc = check_fwd_args(W, X, K, N, Y, "sl_spmm_fwd_act");
    if (rc < 0) return SL_OK;
    if (rc != SL_OK) return rc;
    if (act < 0 || act > 2) return fail(SL_ERR_INVALID, "sl_spmm_fwd_act: act must be 0 (none), 1 (relu) or 2 (gelu)");
    if (act != 0 && H == nullptr) return fail(SL_ERR_INVALID, "sl_spmm_fwd_act: NULL H with an activation");
    cudaStream_t s = as_stream(stream);
    Epi epi;
    epi.H = act != 0 ? H : nullptr;
    epi.bias = bias;
    epi.act = act;
    if (K == 0) {  // Y = bias (or 0), H = act(Y): the second pass over a zeroed Y
        if (int e = cuda_status(cudaMemsetAsync(Y, 0, sizeof(float) * W->nrows * N, s), "sl_spmm_fwd_act memset"))
            return e;
        if (epi.H == nullptr && epi.bias == nullptr) return SL_OK;
        const int64_t n = W->nrows * N;
        int64_t blocks = (n + 255) / 256;
        const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
        epi_kernel<<<static_cast<unsigned>(blocks < cap ? blocks : cap), 256, 0, s>>>(Y, epi, N, n);
        SL_RETURN_IF_LAUNCH_FAILED("sl_spmm_fwd_act");
        return SL_OK;
    }
    return spmm_fwd_impl(W, X, K, N, Y, epi, s);
}
