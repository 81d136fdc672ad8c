// Dense fp32 transpose for the SparseLinear layout change (token-major
// activations [N, K] <-> the kernels' column-per-token operands [K, N]).
// The reference does this with torch copies (sparselab/nn.py:229-237:
// x.reshape(-1, in).t().contiguous() and the .t() of the result).
//
// Tiles through shared memory with padded rows; 128-bit loads and stores in
// 64 x 64 tiles when the shape and pointers allow, else 32 x 32 scalar.
#include "common.cuh"

namespace slb {
namespace {

constexpr int kTile = 32;
constexpr int kRowsPerPass = 8;

// Scalar path (any shape / alignment).
__global__ void __launch_bounds__(kTile * kRowsPerPass)
transpose_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                 float* __restrict__ dst, int64_t tiles_c, int64_t n_tiles,
                 const float* __restrict__ bias) {
    __shared__ float t[kTile][kTile + 1];
    const int tx = threadIdx.x & (kTile - 1), ty = threadIdx.x / kTile;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int64_t r0 = (tile / tiles_c) * kTile, c0 = (tile % tiles_c) * kTile;
#pragma unroll
        for (int k = 0; k < kTile; k += kRowsPerPass) {
            const int64_t r = r0 + ty + k, c = c0 + tx;
            if (r < rows && c < cols) t[ty + k][tx] = __ldg(src + r * cols + c);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kTile; k += kRowsPerPass) {
            const int64_t c = c0 + ty + k, r = r0 + tx;  // dst row c, column r
            if (c < cols && r < rows)
                dst[c * rows + r] = bias ? __fadd_rn(t[tx][ty + k], __ldg(bias + r)) : t[tx][ty + k];
        }
        __syncthreads();
    }
}

// 128-bit path: rows % 4 == 0, cols % 4 == 0, 16-byte aligned pointers.
// 64 x 64 tiles, read as 64 rows x 16 float4 and written as 64 dst rows x
// 16 float4 (4 of each per thread): every row segment on both sides is 256
// contiguous bytes.  Measured on B200 with config-4/5 activation shapes:
// 5.2-5.7 TB/s, against 4.3-4.8 TB/s for 32 x 32 tiles (128-byte
// segments) even with four tiles in flight per CTA.
__global__ void __launch_bounds__(256)
transpose64_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                   float* __restrict__ dst, int64_t tiles_c, int64_t n_tiles,
                   const float* __restrict__ bias) {
    __shared__ float t[64][65];
    const int qx = threadIdx.x & 15, ry = threadIdx.x >> 4;  // float4 column, row (0..15)
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int64_t r0 = (tile / tiles_c) * 64, c0 = (tile % tiles_c) * 64;
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t r = r0 + ry + 16 * j, c = c0 + 4 * qx;
            v[j] = (r < rows && c < cols) ? __ldg(reinterpret_cast<const float4*>(src + r * cols + c))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            t[ry + 16 * j][4 * qx + 0] = v[j].x;
            t[ry + 16 * j][4 * qx + 1] = v[j].y;
            t[ry + 16 * j][4 * qx + 2] = v[j].z;
            t[ry + 16 * j][4 * qx + 3] = v[j].w;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int cc = ry + 16 * j;
            const int64_t c = c0 + cc, r = r0 + 4 * qx;
            if (c < cols && r < rows) {
                float4 o = make_float4(t[4 * qx + 0][cc], t[4 * qx + 1][cc], t[4 * qx + 2][cc],
                                       t[4 * qx + 3][cc]);
                if (bias) {
                    const float4 b = __ldg(reinterpret_cast<const float4*>(bias + r));
                    o = make_float4(__fadd_rn(o.x, b.x), __fadd_rn(o.y, b.y), __fadd_rn(o.z, b.z),
                                    __fadd_rn(o.w, b.w));
                }
                *reinterpret_cast<float4*>(dst + c * rows + r) = o;
            }
        }
        __syncthreads();
    }
}

}  // namespace
}  // namespace slb

using namespace slb;

namespace {
int transpose_impl(const float* src, int64_t rows, int64_t cols, float* dst, const float* bias,
                   void* stream) {
    if (rows < 0 || cols < 0) return fail(SL_ERR_INVALID, "sl_transpose: negative shape");
    if (rows == 0 || cols == 0) return SL_OK;
    if (src == nullptr || dst == nullptr)
        return fail(SL_ERR_INVALID, "sl_transpose: NULL operand");
    if (src == dst) return fail(SL_ERR_INVALID, "sl_transpose: in-place is not supported");
    const int64_t tiles_c = (cols + kTile - 1) / kTile;
    const int64_t n_tiles = ((rows + kTile - 1) / kTile) * tiles_c;
    int64_t grid = n_tiles;
    const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
    if (grid > cap) grid = cap;
    if (rows % 4 == 0 && cols % 4 == 0 && aligned16(src) && aligned16(dst) &&
        (bias == nullptr || aligned16(bias))) {
        const int64_t tc = (cols + 63) / 64, nt = ((rows + 63) / 64) * tc;
        const int64_t g = nt < cap ? nt : cap;
        transpose64_kernel<<<static_cast<unsigned>(g), 256, 0, as_stream(stream)>>>(
            src, rows, cols, dst, tc, nt, bias);
    } else {
        transpose_kernel<<<static_cast<unsigned>(grid), kTile * kRowsPerPass, 0, as_stream(stream)>>>(
            src, rows, cols, dst, tiles_c, n_tiles, bias);
    }
    SL_RETURN_IF_LAUNCH_FAILED("sl_transpose_f32");
    return SL_OK;
}
}  // namespace

extern "C" int sl_transpose_f32(const float* src, int64_t rows, int64_t cols, float* dst,
                                void* stream) {
    return transpose_impl(src, rows, cols, dst, nullptr, stream);
}

extern "C" int sl_transpose_bias_f32(const float* src, int64_t rows, int64_t cols,
                                     const float* bias, float* dst, void* stream) {
    if (bias == nullptr && rows > 0 && cols > 0)
        return fail(SL_ERR_INVALID, "sl_transpose_bias_f32: NULL bias");
    return transpose_impl(src, rows, cols, dst, bias, stream);
}
