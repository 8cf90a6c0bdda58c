// Target image preparation: the bilinear resize of mlx_gsplat/rendering.py:6-38
// (bilinear_resize_mlx), applied by the trainer to each step's target
// (mlx_gsplat/trainer.py:231-234), fused with the uint8 -> [0, 1] scaling of
// trainer.py:369 (``image / 255.0``).
//
// Every float32 operation is the reference's, rounded separately in the same
// order (no fused multiply-add), so the result is bit-identical:
//   xs_in = x * s_x              s_x = float32((W_in - 1) / max(1, W_out - 1))
//   x0 = floor(xs_in), x1 = min(x0 + 1, W_in - 1), wx = xs_in - x0   (same in y)
//   top = (1 - wx) c00 + wx c10,  bottom = (1 - wx) c01 + wx c11
//   out = (1 - wy) top + wy bottom
#include "common.cuh"

namespace gs {

template <bool kU8>
__device__ __forceinline__ float texel(const void* src, int64_t i) {
    if (kU8) return __fdiv_rn((float)__ldg(reinterpret_cast<const uint8_t*>(src) + i), 255.0f);
    return __ldg(reinterpret_cast<const float*>(src) + i);
}

template <bool kU8>
__global__ void __launch_bounds__(256) resize_bilinear_kernel(const void* __restrict__ src, int w_in, int h_in, int ch,
                                                             float* __restrict__ out, int w_out, int h_out, float s_x,
                                                             float s_y) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)w_out * h_out) return;
    const int ox = (int)(i % w_out), oy = (int)(i / w_out);
    const float xs = __fmul_rn((float)ox, s_x), ys = __fmul_rn((float)oy, s_y);
    const int x0 = min((int)floorf(xs), w_in - 1), y0 = min((int)floorf(ys), h_in - 1);
    const int x1 = min(x0 + 1, w_in - 1), y1 = min(y0 + 1, h_in - 1);
    const float wx = __fsub_rn(xs, (float)x0), wy = __fsub_rn(ys, (float)y0);
    const float ax = __fsub_rn(1.0f, wx), ay = __fsub_rn(1.0f, wy);
    const int64_t r0 = (int64_t)y0 * w_in, r1 = (int64_t)y1 * w_in;
    for (int c = 0; c < ch; ++c) {
        const float c00 = texel<kU8>(src, (r0 + x0) * ch + c), c10 = texel<kU8>(src, (r0 + x1) * ch + c);
        const float c01 = texel<kU8>(src, (r1 + x0) * ch + c), c11 = texel<kU8>(src, (r1 + x1) * ch + c);
        const float top = __fadd_rn(__fmul_rn(ax, c00), __fmul_rn(wx, c10));
        const float bot = __fadd_rn(__fmul_rn(ax, c01), __fmul_rn(wx, c11));
        out[i * ch + c] = __fadd_rn(__fmul_rn(ay, top), __fmul_rn(wy, bot));
    }
}

}  // namespace gs

using namespace gs;

extern "C" int gs_resize_bilinear(const void* src, int src_is_u8, int32_t width_in, int32_t height_in,
                                  int32_t channels, float* out, int32_t width_out, int32_t height_out,
                                  gs_stream_t stream) {
    GS_REQUIRE(src && out, "resize_bilinear: null pointer");
    GS_REQUIRE(width_in > 0 && height_in > 0 && width_out > 0 && height_out > 0 && channels > 0,
               "resize_bilinear: sizes must be positive");
    // the scale factors are Python floats in the reference, rounded to float32
    // when they multiply the float32 coordinate grid
    const float s_x = (float)((double)(width_in - 1) / (double)(width_out > 1 ? width_out - 1 : 1));
    const float s_y = (float)((double)(height_in - 1) / (double)(height_out > 1 ? height_out - 1 : 1));
    const int64_t n = (int64_t)width_out * height_out;
    auto kernel = src_is_u8 ? resize_bilinear_kernel<true> : resize_bilinear_kernel<false>;
    kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(src, width_in, height_in, channels, out, width_out,
                                                               height_out, s_x, s_y);
    return check_launch("resize_bilinear_kernel");
}
