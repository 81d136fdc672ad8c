// Dense fp32 transpose for the SparseLinear layout change (token-major
// activations [N, K] <-> the kernels' column-per-token operands [K, N]).
// The reference does this with torch copies (sparselab/nn.py:229-237:
// x.reshape(-1, in).t().contiguous() and the .t() of the result).
//
// 32 x 32 tiles through shared memory (row padded to 33 floats: the
// column-wise reads hit 32 different banks), 256 threads per tile; 128-bit
// loads and stores when the shape and pointers allow, both sides coalesced.
#include "common.cuh"

namespace slb {
namespace {

constexpr int kTile = 32;
constexpr int kRowsPerPass = 8;

// Scalar path (any shape / alignment).
__global__ void __launch_bounds__(kTile * kRowsPerPass)
transpose_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                 float* __restrict__ dst, int64_t tiles_c, int64_t n_tiles) {
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
            if (c < cols && r < rows) dst[c * rows + r] = t[tx][ty + k];
        }
        __syncthreads();
    }
}

// 128-bit path: rows % 4 == 0, cols % 4 == 0, 16-byte aligned pointers.
// A 32 x 32 tile is read as 32 rows x 8 float4 (one per thread) and written
// as 32 dst rows x 8 float4; the four values of a written float4 come from
// four consecutive tile rows of one column (padded rows: conflict-free).
// Each CTA carries kTU tiles per pass, so every thread has kTU independent
// 16-byte loads in flight (one tile per pass left the copy latency-bound
// at about 4.4 TB/s).
constexpr int kTU = 4;
__global__ void __launch_bounds__(256)
transpose4_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                  float* __restrict__ dst, int64_t tiles_c, int64_t n_tiles) {
    __shared__ float t[kTU][kTile][kTile + 1];
    const int qx = threadIdx.x & 7, ry = threadIdx.x >> 3;  // float4 column, row
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * kTU; base < n_tiles;
         base += static_cast<int64_t>(gridDim.x) * kTU) {
        float4 v[kTU];
#pragma unroll
        for (int u = 0; u < kTU; ++u) {
            const int64_t tile = base + u;
            const int64_t r = (tile / tiles_c) * kTile + ry, c = (tile % tiles_c) * kTile + 4 * qx;
            v[u] = (tile < n_tiles && r < rows && c < cols)
                       ? __ldg(reinterpret_cast<const float4*>(src + r * cols + c))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kTU; ++u) {
            t[u][ry][4 * qx + 0] = v[u].x;
            t[u][ry][4 * qx + 1] = v[u].y;
            t[u][ry][4 * qx + 2] = v[u].z;
            t[u][ry][4 * qx + 3] = v[u].w;
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < kTU; ++u) {
            const int64_t tile = base + u;
            const int64_t c = (tile % tiles_c) * kTile + ry, r = (tile / tiles_c) * kTile + 4 * qx;
            if (tile < n_tiles && c < cols && r < rows)  // dst row c, columns r..r+3
                *reinterpret_cast<float4*>(dst + c * rows + r) =
                    make_float4(t[u][4 * qx + 0][ry], t[u][4 * qx + 1][ry], t[u][4 * qx + 2][ry],
                                t[u][4 * qx + 3][ry]);
        }
        __syncthreads();
    }
}

}  // namespace
}  // namespace slb

using namespace slb;

extern "C" int sl_transpose_f32(const float* src, int64_t rows, int64_t cols, float* dst,
                                void* stream) {
    if (rows < 0 || cols < 0) return fail(SL_ERR_INVALID, "sl_transpose_f32: negative shape");
    if (rows == 0 || cols == 0) return SL_OK;
    if (src == nullptr || dst == nullptr)
        return fail(SL_ERR_INVALID, "sl_transpose_f32: NULL operand");
    if (src == dst) return fail(SL_ERR_INVALID, "sl_transpose_f32: in-place is not supported");
    const int64_t tiles_c = (cols + kTile - 1) / kTile;
    const int64_t n_tiles = ((rows + kTile - 1) / kTile) * tiles_c;
    int64_t grid = n_tiles;
    const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
    if (grid > cap) grid = cap;
    if (rows % 4 == 0 && cols % 4 == 0 && aligned16(src) && aligned16(dst)) {
        int64_t g4 = (n_tiles + kTU - 1) / kTU;
        if (g4 > cap) g4 = cap;
        transpose4_kernel<<<static_cast<unsigned>(g4), 256, 0, as_stream(stream)>>>(
            src, rows, cols, dst, tiles_c, n_tiles);
    } else {
        transpose_kernel<<<static_cast<unsigned>(grid), kTile * kRowsPerPass, 0, as_stream(stream)>>>(
            src, rows, cols, dst, tiles_c, n_tiles);
    }
    SL_RETURN_IF_LAUNCH_FAILED("sl_transpose_f32");
    return SL_OK;
}
