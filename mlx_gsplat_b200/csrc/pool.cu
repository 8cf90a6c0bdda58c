// Pool maintenance kernels: row pattern fill (gradient rows of Gaussians a
// view does not see) and single-column fill (the periodic opacity reset,
// mlx_gsplat/trainer.py:416-419).
#include "common.cuh"

namespace gs {

constexpr int kMaxPattern = 64;
struct RowPattern {
    float v[kMaxPattern];
};

__global__ void fill_rows_kernel(float* __restrict__ dst, int64_t n, int stride, RowPattern pat) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n * stride) return;
    dst[t] = pat.v[t % stride];
}

__global__ void fill_rows_v4_kernel(float4* __restrict__ dst, int64_t n, int chunks, RowPattern pat) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n * chunks) return;
    const int c = (int)(t % chunks) * 4;
    dst[t] = make_float4(pat.v[c], pat.v[c + 1], pat.v[c + 2], pat.v[c + 3]);
}

__global__ void fill_column_kernel(float* __restrict__ dst, int64_t n, int64_t stride, int col, float value) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n) dst[r * stride + col] = value;
}

}  // namespace gs

using namespace gs;

extern "C" int gs_fill_rows(float* dst, int64_t n_rows, int64_t stride, const float* pattern_host,
                            gs_stream_t stream) {
    GS_REQUIRE(stride > 0 && stride <= kMaxPattern, "fill_rows: stride must be in [1, %d]", kMaxPattern);
    GS_REQUIRE(n_rows >= 0, "fill_rows: negative rows");
    if (n_rows == 0) return GS_OK;
    GS_REQUIRE(dst && pattern_host, "fill_rows: null pointer");
    RowPattern pat;
    for (int i = 0; i < kMaxPattern; ++i) pat.v[i] = i < stride ? pattern_host[i] : 0.f;
    if (stride % 4 == 0 && aligned16(dst)) {
        const int chunks = (int)(stride / 4);
        fill_rows_v4_kernel<<<grid_for(n_rows * chunks, 256), 256, 0, (cudaStream_t)stream>>>(
            reinterpret_cast<float4*>(dst), n_rows, chunks, pat);
    } else {
        fill_rows_kernel<<<grid_for(n_rows * stride, 256), 256, 0, (cudaStream_t)stream>>>(dst, n_rows, (int)stride,
                                                                                           pat);
    }
    return check_launch("fill_rows");
}

extern "C" int gs_fill_column(float* dst, int64_t n_rows, int64_t stride, int col, float value, gs_stream_t stream) {
    GS_REQUIRE(stride > 0 && col >= 0 && col < stride && n_rows >= 0, "fill_column: bad arguments");
    if (n_rows == 0) return GS_OK;
    GS_REQUIRE(dst, "fill_column: null pointer");
    fill_column_kernel<<<grid_for(n_rows, 256), 256, 0, (cudaStream_t)stream>>>(dst, n_rows, stride, col, value);
    return check_launch("fill_column");
}
