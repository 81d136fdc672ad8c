// Dynamic-sparsity prune / regrow on padded CSR (SET and RigL), reproducing
// the topology the reference computes in sparselab/router.py bit-for-bit:
//
//  * threshold  - k-th smallest |v| over live slots (router.py:395-412,
//                 np.partition): exact radix select over the IEEE bit
//                 patterns of |v| (monotone for non-negative floats; NaN
//                 sorts last, as in numpy).  4 passes x 8-bit digits, the
//                 digit choice made on the device -> no host round trip.
//  * keep       - |v| > thr, or, when nothing in a live row survives, its
//                 first max-|v| slot (router.py:420-439; np.argmax).
//  * rewrite    - one CTA per row.  The row's survivors are tagged in a
//                 per-column table in shared memory; grown columns are
//                 tagged too; one block-wide scan over the columns then
//                 emits the new live set already column-sorted (the
//                 reference's stable argsort of survivors + grown), grown
//                 values 0, padding (-1, 0) (padded_csr.cpp:219-296).
//    SET  - grown columns = host-drawn ranks among the row's non-surviving
//           columns in ascending order (rng.choice(empty_cols, ...)).
//    RigL - grown columns = the n_grow non-survivors of largest |G[i,:]|
//           (router.py:699-721, np.argpartition).  When that set is not
//           unique (ties at the cut) the row is flagged for the host.
#include <cmath>

#include "common.cuh"

namespace slb {
namespace {

constexpr int kDstThreads = 256;
constexpr int kMaxDstCols = 24576;  // 9 bytes of shared memory per column

struct SelectState {
    unsigned prefix;
    unsigned pad;
    long long k_rem;  // 1-based rank still to find inside the current prefix
};

__device__ __forceinline__ unsigned abs_key(float v) { return __float_as_uint(v) & 0x7fffffffu; }

__global__ void select_init_kernel(SelectState* st, unsigned* hist, long long k) {
    if (threadIdx.x == 0) {
        st->prefix = 0;
        st->k_rem = k;
    }
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
}

// Histogram of digit `shift` over live |v| whose higher digits match prefix.
__global__ void __launch_bounds__(kDstThreads)
select_hist_kernel(int M, const int32_t* __restrict__ row_start,
                   const int32_t* __restrict__ row_nnz, const float* __restrict__ vals,
                   const SelectState* __restrict__ st, unsigned* __restrict__ hist, int shift) {
    __shared__ unsigned h[256];
    for (int b = threadIdx.x; b < 256; b += kDstThreads) h[b] = 0;
    __syncthreads();
    const unsigned hi_mask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
    const unsigned prefix = st->prefix;
    const int warps = gridDim.x * (kDstThreads / 32);
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * (kDstThreads / 32) + (threadIdx.x >> 5); row < M; row += warps) {
        const int rs = row_start[row], nn = row_nnz[row];
        for (int s = lane; s < nn; s += 32) {
            const unsigned key = abs_key(vals[rs + s]);
            if ((key & hi_mask) == prefix) atomicAdd(&h[(key >> shift) & 255u], 1u);
        }
    }
    __syncthreads();
    for (int b = threadIdx.x; b < 256; b += kDstThreads)
        if (h[b]) atomicAdd(&hist[b], h[b]);
}

// One warp: pick the digit containing rank k_rem, update prefix, clear hist.
__global__ void select_pick_kernel(SelectState* st, unsigned* hist, int shift, float* thr_out) {
    const int lane = threadIdx.x;
    unsigned c[8];
    unsigned local = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        c[t] = hist[lane * 8 + t];
        local += c[t];
    }
    // exclusive prefix over lanes
    unsigned inc = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
    }
    const long long k = st->k_rem;
    const long long before = static_cast<long long>(inc - local);
    const bool mine = before < k && k <= before + static_cast<long long>(local);
    __syncwarp();
    if (mine) {
        long long run = before;
        int digit = lane * 8;
        for (int t = 0; t < 8; ++t) {
            if (k <= run + c[t]) {
                digit = lane * 8 + t;
                break;
            }
            run += c[t];
        }
        st->prefix |= static_cast<unsigned>(digit) << shift;
        st->k_rem = k - run;
        if (shift == 0 && thr_out) *thr_out = __uint_as_float(st->prefix);
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < 8; ++t) hist[lane * 8 + t] = 0;
}

// Warp per row: survivors count and forced slot.
__global__ void __launch_bounds__(kDstThreads)
keep_kernel(int M, const int32_t* __restrict__ row_start, const int32_t* __restrict__ row_nnz,
            const float* __restrict__ vals, const float* __restrict__ thr_dev,
            int32_t* __restrict__ n_keep, int32_t* __restrict__ force_idx) {
    const float thr = *thr_dev;
    const int warps = gridDim.x * (kDstThreads / 32);
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * (kDstThreads / 32) + (threadIdx.x >> 5); row < M; row += warps) {
        const int rs = row_start[row], nn = row_nnz[row];
        int cnt = 0;
        unsigned best_key = 0;
        int best_k = INT_MAX;
        for (int s = lane; s < nn; s += 32) {
            const float v = vals[rs + s];
            if (fabsf(v) > thr) ++cnt;
            const unsigned key = abs_key(v);
            if (best_k == INT_MAX || key > best_key) {  // first max within the lane
                best_key = key;
                best_k = s;
            }
        }
        cnt = warp_sum(cnt);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned ok = __shfl_xor_sync(0xffffffffu, best_key, o);
            const int os = __shfl_xor_sync(0xffffffffu, best_k, o);
            if (os != INT_MAX && (best_k == INT_MAX || ok > best_key || (ok == best_key && os < best_k))) {
                best_key = ok;
                best_k = os;
            }
        }
        if (lane == 0) {
            if (nn > 0 && cnt == 0) {
                n_keep[row] = 1;
                force_idx[row] = best_k;
            } else {
                n_keep[row] = cnt;
                force_idx[row] = -1;
            }
        }
    }
}

enum GrowMode { kGrowRandom = 0, kGrowTopK = 1, kGrowCols = 2 };

constexpr int kTagEmpty = -1;
constexpr int kTagGrown = -2;

template <int MODE>
__global__ void __launch_bounds__(kDstThreads)
rewrite_kernel(int M, int K, const int32_t* __restrict__ row_start,
               int32_t* __restrict__ row_nnz, const int32_t* __restrict__ row_capacity,
               int32_t* __restrict__ cols, float* __restrict__ vals,
               const float* __restrict__ thr_dev, const int32_t* __restrict__ force_idx,
               const int32_t* __restrict__ grow_off, const int32_t* __restrict__ grow_list,
               const int32_t* __restrict__ row_mask, const float* __restrict__ G,
               int32_t* __restrict__ row_flag) {
    extern __shared__ unsigned char smem[];
    int* tag = reinterpret_cast<int*>(smem);                     // [K]
    float* sv = reinterpret_cast<float*>(smem + 4 * K);          // [K]  survivor values by slot
    unsigned char* drawn = smem + 8 * static_cast<size_t>(K);    // [K]  drawn ranks (SET)
    __shared__ int ws[kDstThreads / 32];
    __shared__ unsigned hist[256];
    __shared__ unsigned sel_prefix;
    __shared__ int sel_krem;
    __shared__ int sh_flag;

    const float thr = *thr_dev;
    for (int row = blockIdx.x; row < M; row += gridDim.x) {
        const int rs = row_start[row], nn = row_nnz[row], cap = row_capacity[row];
        if (nn == 0) continue;  // the reference skips empty rows (no rewrite)
        if (MODE == kGrowCols && row_mask[row] == 0) continue;
        const int fidx = force_idx[row];

        for (int c = threadIdx.x; c < K; c += kDstThreads) {
            tag[c] = kTagEmpty;
            if (MODE == kGrowRandom) drawn[c] = 0;
        }
        __syncthreads();
        int keep_local = 0;
        for (int s = threadIdx.x; s < nn; s += kDstThreads) {
            const float v = vals[rs + s];
            sv[s] = v;
            if (fabsf(v) > thr || s == fidx) {
                tag[cols[rs + s]] = s;
                ++keep_local;
            }
        }
        int n_keep;
        block_exclusive_scan<kDstThreads>(keep_local, ws, &n_keep);  // also a barrier
        const int n_drop = nn - n_keep;

        if (MODE == kGrowRandom) {
            const int g0 = grow_off[row], g1 = grow_off[row + 1];
            for (int t = g0 + threadIdx.x; t < g1; t += kDstThreads) drawn[grow_list[t]] = 1;
            __syncthreads();
            if (g1 > g0) {
                int carry = 0;
                for (int c0 = 0; c0 < K; c0 += kDstThreads) {
                    const int c = c0 + threadIdx.x;
                    const int e = (c < K && tag[c] == kTagEmpty) ? 1 : 0;
                    int tot;
                    const int er = carry + block_exclusive_scan<kDstThreads>(e, ws, &tot);
                    if (e && drawn[er]) tag[c] = kTagGrown;
                    carry += tot;
                }
            }
        } else if (MODE == kGrowCols) {
            const int g0 = grow_off[row], g1 = grow_off[row + 1];
            for (int t = g0 + threadIdx.x; t < g1; t += kDstThreads) tag[grow_list[t]] = kTagGrown;
        } else {  // kGrowTopK
            const int avail = K - n_keep;
            const int n_grow = min(n_drop, avail);
            if (threadIdx.x == 0) {
                sh_flag = 0;
                sel_prefix = 0;
                sel_krem = n_grow;  // rank from the top
            }
            __syncthreads();
            const float* grow_row = G + static_cast<int64_t>(row) * K;
            if (n_grow > 0) {
                // NaN among the candidates: numpy's ordering differs -> host.
                int nan_local = 0;
                for (int c = threadIdx.x; c < K; c += kDstThreads)
                    if (tag[c] == kTagEmpty && abs_key(grow_row[c]) > 0x7f800000u) nan_local = 1;
                if (__syncthreads_or(nan_local)) {
                    if (threadIdx.x == 0) sh_flag = 1;
                } else {
                    // Radix select of the n_grow-th largest key among candidates.
                    for (int shift = 24; shift >= 0; shift -= 8) {
                        for (int b = threadIdx.x; b < 256; b += kDstThreads) hist[b] = 0;
                        __syncthreads();
                        const unsigned hi_mask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
                        const unsigned pre = sel_prefix;
                        for (int c = threadIdx.x; c < K; c += kDstThreads) {
                            if (tag[c] != kTagEmpty) continue;
                            const unsigned key = abs_key(grow_row[c]);
                            if ((key & hi_mask) == pre) atomicAdd(&hist[(key >> shift) & 255u], 1u);
                        }
                        __syncthreads();
                        if (threadIdx.x == 0) {
                            int k = sel_krem;
                            int d = 255;
                            for (; d > 0; --d) {
                                if (k <= static_cast<int>(hist[d])) break;
                                k -= hist[d];
                            }
                            sel_prefix = pre | (static_cast<unsigned>(d) << shift);
                            sel_krem = k;
                        }
                        __syncthreads();
                    }
                    // sel_prefix = cut key.  Count candidates above / at the cut.
                    const unsigned cut = sel_prefix;
                    int gt = 0, eq = 0;
                    for (int c = threadIdx.x; c < K; c += kDstThreads) {
                        if (tag[c] != kTagEmpty) continue;
                        const unsigned key = abs_key(grow_row[c]);
                        gt += key > cut;
                        eq += key == cut;
                    }
                    int n_gt, n_eq;
                    block_exclusive_scan<kDstThreads>(gt, ws, &n_gt);
                    block_exclusive_scan<kDstThreads>(eq, ws, &n_eq);
                    if (n_gt + n_eq != n_grow) {
                        if (threadIdx.x == 0) sh_flag = 1;  // ties straddle the cut
                    } else {
                        for (int c = threadIdx.x; c < K; c += kDstThreads)
                            if (tag[c] == kTagEmpty && abs_key(grow_row[c]) >= cut) tag[c] = kTagGrown;
                    }
                }
            }
            __syncthreads();
            if (threadIdx.x == 0) row_flag[row] = sh_flag;
            if (sh_flag) {
                __syncthreads();
                continue;  // left untouched for the host
            }
        }
        __syncthreads();

        // Emit the new live set in column order, then padding.
        int carry = 0;
        for (int c0 = 0; c0 < K; c0 += kDstThreads) {
            const int c = c0 + threadIdx.x;
            const int t = c < K ? tag[c] : kTagEmpty;
            const int on = t != kTagEmpty ? 1 : 0;
            int tot;
            const int pos = carry + block_exclusive_scan<kDstThreads>(on, ws, &tot);
            if (on) {
                cols[rs + pos] = c;
                vals[rs + pos] = t >= 0 ? sv[t] : 0.0f;
            }
            carry += tot;
        }
        for (int p = carry + threadIdx.x; p < cap; p += kDstThreads) {
            cols[rs + p] = -1;
            vals[rs + p] = 0.0f;
        }
        if (threadIdx.x == 0) row_nnz[row] = carry;
        __syncthreads();
    }
}

template <int MODE>
int launch_rewrite(const sl_csr* W, const float* thr_dev, const int32_t* force_idx,
                   const int32_t* grow_off, const int32_t* grow_list, const int32_t* row_mask,
                   const float* G, int32_t* row_flag, void* stream, const char* fn) {
    if (int rc = check_csr(W, fn)) return rc;
    if (W->ncols > kMaxDstCols)
        return fail(SL_ERR_UNSUPPORTED, std::string(fn) + ": ncols=" + std::to_string(W->ncols) +
                                            " exceeds the supported maximum of " +
                                            std::to_string(kMaxDstCols));
    if (W->nrows == 0) return SL_OK;
    SL_REQUIRE(thr_dev != nullptr && force_idx != nullptr, fn, "NULL threshold or force_idx");
    SL_REQUIRE(MODE == kGrowTopK || (grow_off != nullptr && grow_list != nullptr), fn,
               "NULL grow_offsets or grow list");
    SL_REQUIRE(MODE != kGrowTopK || (G != nullptr && row_flag != nullptr), fn, "NULL G or row_flag");
    SL_REQUIRE(MODE != kGrowCols || row_mask != nullptr, fn, "NULL row_mask");
    const int K = static_cast<int>(W->ncols);
    const size_t smem = 9 * static_cast<size_t>(K > 0 ? K : 1);
    if (smem > 48 * 1024)
        cudaFuncSetAttribute(rewrite_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    int blocks = static_cast<int>(W->nrows);
    const int cap = num_sms() * 4;
    if (blocks > cap) blocks = cap;
    rewrite_kernel<MODE><<<blocks, kDstThreads, smem, as_stream(stream)>>>(
        static_cast<int>(W->nrows), K, W->row_start, W->row_nnz, W->row_capacity, W->col_indices,
        W->values, thr_dev, force_idx, grow_off, grow_list, row_mask, G, row_flag);
    SL_RETURN_IF_LAUNCH_FAILED(fn);
    return SL_OK;
}

}  // namespace
}  // namespace slb

using namespace slb;

extern "C" {

int64_t sl_dst_scratch_bytes(void) { return 256 * sizeof(unsigned) + sizeof(SelectState); }

int64_t sl_dst_max_ncols(void) { return kMaxDstCols; }

int sl_dst_threshold(const sl_csr* W, int64_t k, float* thr_dev, void* scratch, void* stream) {
    if (int rc = check_csr(W, "sl_dst_threshold")) return rc;
    if (k < 1) return fail(SL_ERR_INVALID, "sl_dst_threshold: k must be >= 1");
    SL_REQUIRE(thr_dev != nullptr && scratch != nullptr, "sl_dst_threshold", "NULL output or scratch");
    cudaStream_t s = as_stream(stream);
    unsigned* hist = static_cast<unsigned*>(scratch);
    SelectState* st = reinterpret_cast<SelectState*>(hist + 256);
    select_init_kernel<<<1, 256, 0, s>>>(st, hist, k);
    SL_RETURN_IF_LAUNCH_FAILED("sl_dst_threshold");
    const int M = static_cast<int>(W->nrows);
    for (int shift = 24; shift >= 0; shift -= 8) {
        if (M > 0) {
            select_hist_kernel<<<row_grid(M), kDstThreads, 0, s>>>(M, W->row_start, W->row_nnz,
                                                                   W->values, st, hist, shift);
            SL_RETURN_IF_LAUNCH_FAILED("sl_dst_threshold");
        }
        select_pick_kernel<<<1, 32, 0, s>>>(st, hist, shift, thr_dev);
        SL_RETURN_IF_LAUNCH_FAILED("sl_dst_threshold");
    }
    return SL_OK;
}

int sl_dst_keep(const sl_csr* W, const float* thr_dev, int32_t* n_keep, int32_t* force_idx,
                void* stream) {
    if (int rc = check_csr(W, "sl_dst_keep")) return rc;
    if (W->nrows == 0) return SL_OK;
    SL_REQUIRE(thr_dev != nullptr && n_keep != nullptr && force_idx != nullptr, "sl_dst_keep",
               "NULL threshold or output array");
    keep_kernel<<<row_grid(W->nrows), kDstThreads, 0, as_stream(stream)>>>(
        static_cast<int>(W->nrows), W->row_start, W->row_nnz, W->values, thr_dev, n_keep,
        force_idx);
    SL_RETURN_IF_LAUNCH_FAILED("sl_dst_keep");
    return SL_OK;
}

int sl_dst_apply_random(const sl_csr* W, const float* thr_dev, const int32_t* force_idx,
                        const int32_t* grow_offsets, const int32_t* grow_ranks, void* stream) {
    return launch_rewrite<kGrowRandom>(W, thr_dev, force_idx, grow_offsets, grow_ranks, nullptr,
                                       nullptr, nullptr, stream, "sl_dst_apply_random");
}

int sl_dst_apply_topk(const sl_csr* W, const float* thr_dev, const int32_t* force_idx,
                      const float* G, int32_t* row_flag, void* stream) {
    return launch_rewrite<kGrowTopK>(W, thr_dev, force_idx, nullptr, nullptr, nullptr, G,
                                     row_flag, stream, "sl_dst_apply_topk");
}

int sl_dst_apply_cols(const sl_csr* W, const float* thr_dev, const int32_t* force_idx,
                      const int32_t* row_mask, const int32_t* grow_offsets,
                      const int32_t* grow_cols, void* stream) {
    return launch_rewrite<kGrowCols>(W, thr_dev, force_idx, grow_offsets, grow_cols, row_mask,
                                     nullptr, nullptr, stream, "sl_dst_apply_cols");
}

}  // extern "C"

// ── Fused AdamW over live slots ─────────────────────────────────────────
// One pass over a SparseLinear's padded values: slots whose column is -1
// (padding) are skipped, so their value stays exactly 0 and their moments
// are not touched; live slots get torch's decoupled-weight-decay AdamW
// update (param *= 1 - lr*wd; m = lerp(m, g, 1-b1); v = b2*v + (1-b2)*g*g;
// param -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps)).  State is per slot, as
// with a torch optimizer on the aliased values tensor: a topology rewrite
// moves weights between slots and the moments stay with the slot.
namespace slb {
namespace {
__global__ void __launch_bounds__(256)
adamw_live_kernel(int64_t cap, const int32_t* __restrict__ cols, float* __restrict__ p,
                  const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                  float decay, float one_minus_b1, float b2, float one_minus_b2, float eps,
                  float step_size, float bc2_sqrt) {
    for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < cap;
         s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        if (__ldg(cols + s) < 0) continue;
        const float gs = __ldg(g + s);
        float ps = p[s] * decay;
        const float ms = m[s] + one_minus_b1 * (gs - m[s]);
        const float vs = v[s] * b2 + one_minus_b2 * gs * gs;
        const float denom = sqrtf(vs) / bc2_sqrt + eps;
        ps = ps - step_size * (ms / denom);
        p[s] = ps;
        m[s] = ms;
        v[s] = vs;
    }
}
}  // namespace
}  // namespace slb

extern "C" int sl_adamw_live(const sl_csr* W, const float* grad, float* exp_avg,
                             float* exp_avg_sq, float lr, float beta1, float beta2, float eps,
                             float weight_decay, int64_t step, void* stream) {
    if (int rc = check_csr(W, "sl_adamw_live")) return rc;
    SL_REQUIRE(step >= 1, "sl_adamw_live", "step must be >= 1");
    SL_REQUIRE(lr >= 0.0f && eps >= 0.0f && beta1 >= 0.0f && beta1 < 1.0f && beta2 >= 0.0f &&
                   beta2 < 1.0f,
               "sl_adamw_live", "invalid hyper-parameters");
    if (W->total_capacity == 0) return SL_OK;
    SL_REQUIRE(grad != nullptr && exp_avg != nullptr && exp_avg_sq != nullptr, "sl_adamw_live",
               "NULL gradient or state");
    const double bc1 = 1.0 - std::pow(static_cast<double>(beta1), static_cast<double>(step));
    const double bc2 = 1.0 - std::pow(static_cast<double>(beta2), static_cast<double>(step));
    const int64_t cap = W->total_capacity;
    int64_t blocks = (cap + 255) / 256;
    const int64_t max_blocks = static_cast<int64_t>(num_sms()) * 8;
    if (blocks > max_blocks) blocks = max_blocks;
    adamw_live_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
        cap, W->col_indices, W->values, grad, exp_avg, exp_avg_sq,
        1.0f - lr * weight_decay, 1.0f - beta1, beta2, 1.0f - beta2, eps,
        static_cast<float>(lr / bc1), static_cast<float>(std::sqrt(bc2)));
    SL_RETURN_IF_LAUNCH_FAILED("sl_adamw_live");
    return SL_OK;
}
