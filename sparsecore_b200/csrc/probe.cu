// Roofline probes: the FP32 FMA pipe and the shared-memory data path,
// measured on the device the library runs on, so the kernels' fractions are
// taken against measured ceilings rather than nominal ones.
//  * sl_probe_ffma: every thread advances 8 independent FMA chains for
//    `iters` steps (2 * 8 * iters FLOPs per thread); one CTA of 256 threads
//    per 64 resident warps' worth of work on every SM.
//  * sl_probe_smem: every thread reads 4 * `iters` conflict-free 64-bit
//    words from shared memory (a warp covers 256 contiguous bytes per load;
//    each address depends on the previous load, so none can be removed), so
//    the bytes moved are 32 * iters per thread.
// Both write one value per thread to `out` so nothing is optimised away.
#include "common.cuh"

namespace slb {
namespace {

__global__ void __launch_bounds__(256) probe_ffma_kernel(int64_t iters, float seed, float* out) {
    float a[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = seed + threadIdx.x * 1e-7f + k;
    const float m = 0.999999f, c = 1e-7f;
    for (int64_t i = 0; i < iters; ++i) {
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = fmaf(a[k], m, c);
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += a[k];
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

__global__ void __launch_bounds__(256) probe_smem_kernel(int64_t iters, float* out) {
    // Every value in the buffer is 0, but the compiler cannot know it: each
    // load's address adds the previous load's value, so no load can be
    // hoisted or merged, and four independent chains per thread keep loads
    // in flight.  A warp's 64-bit load covers 256 contiguous bytes
    // (conflict-free); measured on B200 this pattern saturates the
    // shared-memory pipe (ncu l1tex throughput 98%), while 128-bit loads in
    // the same loop reached half the bytes per cycle.
    __shared__ __align__(16) float2 buf[2048];  // 16 KB
    for (int k = threadIdx.x; k < 2048; k += blockDim.x) buf[k] = make_float2(0.f, 0.f);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int idx[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) idx[c] = ((warp * 4 + c) * 32) % 2048 + lane;
    float s = 0.0f;
    for (int64_t i = 0; i < iters; ++i) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const float2 v = buf[idx[c]];
            s += v.y;
            idx[c] = ((idx[c] + 256 + __float_as_int(v.x)) & 2047);
        }
    }
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace
}  // namespace slb

using namespace slb;

extern "C" {

int64_t sl_probe_threads(void) { return static_cast<int64_t>(num_sms()) * 2048; }

int sl_probe_ffma(int64_t iters, float* out, void* stream) {
    SL_REQUIRE(iters > 0 && out != nullptr, "sl_probe_ffma", "iters > 0 and an output buffer");
    const int blocks = num_sms() * 8;  // 8 x 256 threads = 64 warps per SM
    probe_ffma_kernel<<<blocks, 256, 0, as_stream(stream)>>>(iters, 1.0f, out);
    SL_RETURN_IF_LAUNCH_FAILED("sl_probe_ffma");
    return SL_OK;
}

int sl_probe_smem(int64_t iters, float* out, void* stream) {
    SL_REQUIRE(iters > 0 && out != nullptr, "sl_probe_smem", "iters > 0 and an output buffer");
    const int blocks = num_sms() * 8;
    probe_smem_kernel<<<blocks, 256, 0, as_stream(stream)>>>(iters, out);
    SL_RETURN_IF_LAUNCH_FAILED("sl_probe_smem");
    return SL_OK;
}

}  // extern "C"
