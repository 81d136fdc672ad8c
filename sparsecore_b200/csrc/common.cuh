// Shared helpers for the sparsecore_b200 CUDA kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <string>

#include "../../include/sparsecore_b200.h"

namespace slb {

// Per-host-thread error message behind sl_last_error().
void set_error(const std::string& msg);
// Records the kernel the last SpMM / SDDMM dispatch launched on this host
// thread (a string literal), read back with sl_last_kernel().
void note_kernel(const char* name);
int fail(int code, const std::string& msg);
// SL_OK, or SL_ERR_CUDA with the runtime's message prefixed by `what`.
int cuda_status(cudaError_t e, const char* what);
// SM count of the current device (cached per device).
int num_sms();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Checks shared by every entry point that takes an sl_csr.
int check_csr(const sl_csr* W, const char* fn);
// Grid size for warp-per-row kernels of 256 threads (8 warps per CTA).
int row_grid(int64_t M);
// N = 1 forward, warp-specialised row windows (spmv_ws.cu);
// -1 when it does not apply.
int launch_spmv_ws(const sl_csr* W, const float* X, int64_t K, float* Y, cudaStream_t s);
// N = 32 forward / SDDMM with X rows staged by cp.async (gather32.cu); -1
// when they do not apply.
int launch_gather32_fwd(const sl_csr* W, const float* X, float* Y, cudaStream_t s);
int launch_gather32_sddmm(const sl_csr* W, const float* dY, const float* X, float* dW,
                          cudaStream_t s);
// SPARSECORE_B200_N32=rows keeps the N = 32 SDDMM on the general kernels;
// =gather also sends the N = 32 forward to the staged kernel (tests).
bool gather32_enabled();
bool gather32_forced();

constexpr int kWarp = 32;

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ int warp_inclusive_scan(int v) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane_id() >= o) v += t;
    }
    return v;
}

// Block-wide exclusive scan of one int per thread; `ws` is shared scratch of
// NT/32 ints; *total receives the block sum.  Contains __syncthreads().
template <int NT>
__device__ __forceinline__ int block_exclusive_scan(int v, int* ws, int* total) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int inc = warp_inclusive_scan(v);
    if (lane == 31) ws[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = lane < NW ? ws[lane] : 0;
        w = warp_inclusive_scan(w);
        if (lane < NW) ws[lane] = w;
    }
    __syncthreads();
    const int base = warp ? ws[warp - 1] : 0;
    *total = ws[NW - 1];
    __syncthreads();
    return base + inc - v;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace slb

// Argument check: return SL_ERR_INVALID with "<fn>: <msg>" when cond fails.
#define SL_REQUIRE(cond, fn, msg)                                            \
    do {                                                                    \
        if (!(cond)) return ::slb::fail(SL_ERR_INVALID, std::string(fn) + ": " + (msg)); \
    } while (0)

#define SL_RETURN_IF_LAUNCH_FAILED(what)                                   \
    do {                                                                  \
        cudaError_t e_ = cudaGetLastError();                              \
        if (e_ != cudaSuccess) return ::slb::cuda_status(e_, what);       \
    } while (0)
