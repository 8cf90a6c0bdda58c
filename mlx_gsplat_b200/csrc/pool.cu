// Pool maintenance kernels: row pattern fill (gradient rows of Gaussians a
// view does not see), single-column fill (the periodic opacity reset,
// mlx_gsplat/trainer.py:416-419) and the export gather of the active rows
// (mlx_gsplat/trainer.py:570-631).
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

// One export row per active id (trainer.py:570-600): means | 0 0 0 | colour
// columns | opacity logit clipped to [-5, 2] | log-scales clipped to
// [-10, -2] | the quaternion divided by (|q| + 1e-8).  The float32 operations
// follow NumPy's for the same expressions (the norm sums the four squares
// left to right; clipping keeps NaN), so the rows match the reference's bit
// for bit.
__device__ __forceinline__ float clip_keep_nan(float x, float lo, float hi) {
    return x != x ? x : fminf(fmaxf(x, lo), hi);
}

__global__ void export_rows_kernel(const float* __restrict__ theta, int64_t stride, const int32_t* __restrict__ table,
                                   int64_t n, int mean_col, int opac_col, int scale_col, int quat_col, int color_col,
                                   int color_cols, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* r = theta + (int64_t)table[i] * stride;
    const int oc = 3 + 3 + color_cols + 1 + 3 + 4;
    float* o = out + i * oc;
    for (int k = 0; k < 3; ++k) o[k] = r[mean_col + k];
    for (int k = 0; k < 3; ++k) o[3 + k] = 0.f;
    for (int k = 0; k < color_cols; ++k) o[6 + k] = r[color_col + k];
    o[6 + color_cols] = clip_keep_nan(r[opac_col], -5.f, 2.f);
    for (int k = 0; k < 3; ++k) o[7 + color_cols + k] = clip_keep_nan(r[scale_col + k], -10.f, -2.f);
    const float q0 = r[quat_col], q1 = r[quat_col + 1], q2 = r[quat_col + 2], q3 = r[quat_col + 3];
    float ss = __fmul_rn(q0, q0);
    ss = __fadd_rn(ss, __fmul_rn(q1, q1));
    ss = __fadd_rn(ss, __fmul_rn(q2, q2));
    ss = __fadd_rn(ss, __fmul_rn(q3, q3));
    const float nrm = __fadd_rn(__fsqrt_rn(ss), 1e-8f);
    float* oq = o + 10 + color_cols;
    oq[0] = __fdiv_rn(q0, nrm);
    oq[1] = __fdiv_rn(q1, nrm);
    oq[2] = __fdiv_rn(q2, nrm);
    oq[3] = __fdiv_rn(q3, nrm);
}

// mask[slots[j]] = value for j < n (slots at or past mask_len are skipped).
__global__ void mark_slots_kernel(int8_t* __restrict__ mask, int64_t mask_len, const int32_t* __restrict__ slots,
                                  int64_t n, int8_t value) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const int32_t s = slots[j];
    if (s >= 0 && s < mask_len) mask[s] = value;
}

// dst row (dst_idx ? dst_idx[j] : j) gets the first ``cols`` floats of src row
// (src_idx ? src_idx[j] : j), for j < n; 16 bytes at a time (the caller
// guarantees 16-byte rows and cols % 4 == 0).
__global__ void copy_rows_v4_kernel(const float4* __restrict__ src, int64_t src_q, const int32_t* __restrict__ src_idx,
                                    float4* __restrict__ dst, int64_t dst_q, const int32_t* __restrict__ dst_idx,
                                    int64_t n, int chunks) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n * chunks) return;
    const int64_t j = t / chunks;
    const int c = (int)(t - j * chunks);
    const int64_t rs = src_idx ? (int64_t)src_idx[j] : j, rd = dst_idx ? (int64_t)dst_idx[j] : j;
    dst[rd * dst_q + c] = src[rs * src_q + c];
}

}  // namespace gs

using namespace gs;

extern "C" int gs_export_rows(const float* theta, int64_t stride, const int32_t* table, int64_t num_active,
                              int mean_col, int opac_col, int scale_col, int quat_col, int color_col, int color_cols,
                              float* out, int64_t out_cols, gs_stream_t stream) {
    GS_REQUIRE(num_active >= 0 && stride > 0 && color_cols >= 0, "export_rows: bad sizes");
    GS_REQUIRE(out_cols == 14 + (int64_t)color_cols, "export_rows: out_cols must be 14 + color_cols");
    GS_REQUIRE(mean_col >= 0 && mean_col + 3 <= stride && opac_col >= 0 && opac_col < stride && scale_col >= 0 &&
                   scale_col + 3 <= stride && quat_col >= 0 && quat_col + 4 <= stride && color_col >= 0 &&
                   color_col + color_cols <= stride,
               "export_rows: column out of the row");
    if (num_active == 0) return GS_OK;
    GS_REQUIRE(theta && table && out, "export_rows: null pointer");
    export_rows_kernel<<<grid_for(num_active, 256), 256, 0, (cudaStream_t)stream>>>(
        theta, stride, table, num_active, mean_col, opac_col, scale_col, quat_col, color_col, color_cols, out);
    return check_launch("export_rows_kernel");
}

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

extern "C" int gs_mark_slots(int8_t* mask, int64_t mask_len, const int32_t* slots, int64_t n, int value,
                             gs_stream_t stream) {
    GS_REQUIRE(n >= 0 && mask_len >= 0, "mark_slots: bad sizes");
    if (n == 0) return GS_OK;
    GS_REQUIRE(mask && slots, "mark_slots: null pointer");
    mark_slots_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(mask, mask_len, slots, n, (int8_t)value);
    return check_launch("mark_slots_kernel");
}

extern "C" int gs_copy_rows(const float* src, int64_t src_stride, const int32_t* src_idx, float* dst,
                            int64_t dst_stride, const int32_t* dst_idx, int64_t n, int cols, gs_stream_t stream) {
    GS_REQUIRE(n >= 0 && cols > 0 && cols % 4 == 0 && src_stride % 4 == 0 && dst_stride % 4 == 0 &&
                   cols <= src_stride && cols <= dst_stride,
               "copy_rows: cols must be a positive multiple of 4 within both row strides (multiples of 4)");
    if (n == 0) return GS_OK;
    GS_REQUIRE(src && dst, "copy_rows: null pointer");
    GS_REQUIRE(aligned16(src) && aligned16(dst), "copy_rows: bases must be 16-byte aligned");
    const int chunks = cols / 4;
    copy_rows_v4_kernel<<<grid_for(n * chunks, 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const float4*>(src), src_stride / 4, src_idx, reinterpret_cast<float4*>(dst), dst_stride / 4,
        dst_idx, n, chunks);
    return check_launch("copy_rows_v4_kernel");
}
