// The reference trainer's image loss with a target (mlx_gsplat/trainer.py:
// 164-190, 276-279):  w_l1 * mean|C - T| + w_dssim * (1 - SSIM(C, T)) / 2,
// SSIM with an 11 x 11 window of ones / 121, zero padding 5, per channel, the
// mean over pixels and channels; and its gradient with respect to C.
//
// Per pixel p and channel, with box sums over the window around p,
//   mu1 = box(C), mu2 = box(T), s11 = box(C^2) - mu1^2, s22 = box(T^2) - mu2^2,
//   s12 = box(C T) - mu1 mu2,
//   S = (2 mu1 mu2 + C1)(2 s12 + C2) / ((mu1^2 + mu2^2 + C1)(s11 + s22 + C2)).
// S depends on C through box(C), box(C^2) and box(C T); with the partials
//   a = dS/dbox(C), b = dS/dbox(C^2), c = dS/dbox(C T)
// the gradient of sum_p S at pixel q is the same box filter applied to them:
//   dS/dC(q) = (box(a)(q) + 2 C(q) box(b)(q) + T(q) box(c)(q)) / 121.
// Two tiled kernels (16 x 16 outputs from a 26 x 26 shared-memory region,
// horizontal then vertical sums) compute the partials and the gradient; a
// one-CTA kernel sums the per-tile partial sums in double.
#include "common.cuh"
#include "scan.cuh"

namespace gs {

constexpr int kWin = 11, kRad = kWin / 2;
constexpr int kLT = 16;                 // output tile edge
constexpr int kLR = kLT + 2 * kRad;     // 26: tile + halo
constexpr float kSsimC1 = 0.01f * 0.01f, kSsimC2 = 0.03f * 0.03f;
constexpr float kInvWin2 = 1.0f / 121.0f;

__device__ __forceinline__ float load_target(const void* t, int u8, int64_t i) {
    return u8 ? __fdiv_rn((float)static_cast<const uint8_t*>(t)[i], 255.0f) : static_cast<const float*>(t)[i];
}

// Loads channel-planar [3][26][26] tiles of C and T (zero outside the image).
__device__ __forceinline__ void load_region(float (*sc)[kLR][kLR + 1], float (*st)[kLR][kLR + 1],
                                            const float* __restrict__ color, const void* __restrict__ target,
                                            int u8, int W, int H, int x0, int y0) {
    for (int i = threadIdx.x; i < kLR * kLR; i += blockDim.x) {
        const int ry = i / kLR, rx = i - ry * kLR;
        const int gx = x0 - kRad + rx, gy = y0 - kRad + ry;
        const bool in = gx >= 0 && gx < W && gy >= 0 && gy < H;
        const int64_t pix = (int64_t)gy * W + gx;
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            sc[ch][ry][rx] = in ? color[3 * pix + ch] : 0.f;
            st[ch][ry][rx] = in ? load_target(target, u8, 3 * pix + ch) : 0.f;
        }
    }
}

__global__ void __launch_bounds__(256) ssim_fwd_kernel(const float* __restrict__ color,
                                                       const void* __restrict__ target, int u8, int W, int H,
                                                       float* __restrict__ pa, float* __restrict__ pb,
                                                       float* __restrict__ pc, float2* __restrict__ tile_sums) {
    __shared__ float sc[3][kLR][kLR + 1], st[3][kLR][kLR + 1];
    __shared__ float hs[5][3][kLR][kLT];  // horizontal window sums of C, T, C^2, T^2, C T
    __shared__ float red[2][8];
    const int tiles_x = (W + kLT - 1) / kLT;
    const int x0 = (blockIdx.x % tiles_x) * kLT, y0 = (blockIdx.x / tiles_x) * kLT;
    load_region(sc, st, color, target, u8, W, H, x0, y0);
    __syncthreads();
    for (int i = threadIdx.x; i < 3 * kLR * kLT; i += blockDim.x) {
        const int ch = i / (kLR * kLT), r = (i / kLT) % kLR, ox = i % kLT;
        float s1 = 0.f, s2 = 0.f, s11 = 0.f, s22 = 0.f, s12 = 0.f;
#pragma unroll
        for (int k = 0; k < kWin; ++k) {
            const float c = sc[ch][r][ox + k], t = st[ch][r][ox + k];
            s1 += c;
            s2 += t;
            s11 = fmaf(c, c, s11);
            s22 = fmaf(t, t, s22);
            s12 = fmaf(c, t, s12);
        }
        hs[0][ch][r][ox] = s1;
        hs[1][ch][r][ox] = s2;
        hs[2][ch][r][ox] = s11;
        hs[3][ch][r][ox] = s22;
        hs[4][ch][r][ox] = s12;
    }
    __syncthreads();
    const int oy = threadIdx.x / kLT, ox = threadIdx.x % kLT;
    const int gx = x0 + ox, gy = y0 + oy;
    const bool in = gx < W && gy < H;
    float sum_s = 0.f, sum_l1 = 0.f;
    if (in) {
        const int64_t pix = (int64_t)gy * W + gx;
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            float v[5];
#pragma unroll
            for (int q = 0; q < 5; ++q) {
                float a = 0.f;
#pragma unroll
                for (int k = 0; k < kWin; ++k) a += hs[q][ch][oy + k][ox];
                v[q] = a * kInvWin2;
            }
            const float mu1 = v[0], mu2 = v[1];
            const float m11 = mu1 * mu1, m22 = mu2 * mu2, m12 = mu1 * mu2;
            const float sg1 = v[2] - m11, sg2 = v[3] - m22, sg12 = v[4] - m12;
            const float n1 = 2.f * m12 + kSsimC1, n2 = 2.f * sg12 + kSsimC2;
            const float d1 = m11 + m22 + kSsimC1, d2 = sg1 + sg2 + kSsimC2;
            const float inv = 1.f / (d1 * d2);
            const float S = n1 * n2 * inv;
            // partials of S with respect to mu1 = box(C)/121, box(C^2)/121 and
            // box(C T)/121 (sigma1 = box(C^2)/121 - mu1^2 and sigma12 =
            // box(C T)/121 - mu1 mu2 are folded into the first)
            const float dmu1 = (2.f * mu2 * n2 - 2.f * mu2 * n1) * inv - S * (2.f * mu1 / d1 - 2.f * mu1 / d2);
            const float ds11 = -S / d2;
            const float ds12 = 2.f * n1 * inv;
            pa[3 * pix + ch] = dmu1;
            pb[3 * pix + ch] = ds11;
            pc[3 * pix + ch] = ds12;
            sum_s += S;
            sum_l1 += fabsf(sc[ch][oy + kRad][ox + kRad] - st[ch][oy + kRad][ox + kRad]);
        }
    }
    sum_s = warp_sum(sum_s);
    sum_l1 = warp_sum(sum_l1);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        red[0][warp] = sum_s;
        red[1][warp] = sum_l1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f, b = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            a += red[0][w];
            b += red[1][w];
        }
        tile_sums[blockIdx.x] = make_float2(a, b);
    }
}

__global__ void __launch_bounds__(256) ssim_bwd_kernel(const float* __restrict__ color,
                                                       const void* __restrict__ target, int u8, int W, int H,
                                                       const float* __restrict__ pa, const float* __restrict__ pb,
                                                       const float* __restrict__ pc, float g_l1, float g_ssim,
                                                       float* __restrict__ dL_dC) {
    __shared__ float sp[3][3][kLR][kLR + 1];  // the three partial maps, channel planar
    __shared__ float hs[3][3][kLR][kLT];
    const int tiles_x = (W + kLT - 1) / kLT;
    const int x0 = (blockIdx.x % tiles_x) * kLT, y0 = (blockIdx.x / tiles_x) * kLT;
    for (int i = threadIdx.x; i < kLR * kLR; i += blockDim.x) {
        const int ry = i / kLR, rx = i - ry * kLR;
        const int gx = x0 - kRad + rx, gy = y0 - kRad + ry;
        const bool in = gx >= 0 && gx < W && gy >= 0 && gy < H;
        const int64_t pix = (int64_t)gy * W + gx;
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            sp[0][ch][ry][rx] = in ? pa[3 * pix + ch] : 0.f;
            sp[1][ch][ry][rx] = in ? pb[3 * pix + ch] : 0.f;
            sp[2][ch][ry][rx] = in ? pc[3 * pix + ch] : 0.f;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 3 * 3 * kLR * kLT; i += blockDim.x) {
        const int m = i / (3 * kLR * kLT), ch = (i / (kLR * kLT)) % 3, r = (i / kLT) % kLR, ox = i % kLT;
        float a = 0.f;
#pragma unroll
        for (int k = 0; k < kWin; ++k) a += sp[m][ch][r][ox + k];
        hs[m][ch][r][ox] = a;
    }
    __syncthreads();
    const int oy = threadIdx.x / kLT, ox = threadIdx.x % kLT;
    const int gx = x0 + ox, gy = y0 + oy;
    if (gx >= W || gy >= H) return;
    const int64_t pix = (int64_t)gy * W + gx;
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
        float box[3];
#pragma unroll
        for (int m = 0; m < 3; ++m) {
            float a = 0.f;
#pragma unroll
            for (int k = 0; k < kWin; ++k) a += hs[m][ch][oy + k][ox];
            box[m] = a;
        }
        const float c = color[3 * pix + ch], t = load_target(target, u8, 3 * pix + ch);
        const float e = c - t;
        const float sgn = e > 0.f ? 1.f : (e < 0.f ? -1.f : 0.f);
        const float dS = (box[0] + 2.f * c * box[1] + t * box[2]) * kInvWin2;
        dL_dC[3 * pix + ch] = fmaf(g_ssim, dS, g_l1 * sgn);
    }
}

__global__ void loss_finalize_kernel(const float2* __restrict__ tile_sums, int n, double inv_count, float w_l1,
                                     float w_dssim, float* __restrict__ loss_out, float* __restrict__ ssim_out) {
    __shared__ double rs[32], rl[32];
    double s = 0.0, l = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        s += tile_sums[i].x;
        l += tile_sums[i].y;
    }
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(kFull, s, o);
        l += __shfl_xor_sync(kFull, l, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        rs[warp] = s;
        rl[warp] = l;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double ts = 0.0, tl = 0.0;
        for (int w = 0; w < (int)(blockDim.x / 32); ++w) {
            ts += rs[w];
            tl += rl[w];
        }
        const double ssim = ts * inv_count;
        if (ssim_out) *ssim_out = (float)ssim;
        *loss_out = (float)((double)w_l1 * tl * inv_count + (double)w_dssim * 0.5 * (1.0 - ssim));
    }
}

size_t ssim_scratch_bytes(int W, int H) {
    const size_t P = (size_t)W * (size_t)H;
    const size_t tiles = (size_t)((W + kLT - 1) / kLT) * (size_t)((H + kLT - 1) / kLT);
    return 3 * align_up(P * 3 * sizeof(float), 256) + align_up(tiles * sizeof(float2), 256) + 256;
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_l1_dssim_scratch_bytes(int32_t width, int32_t height) {
    return width > 0 && height > 0 ? ssim_scratch_bytes(width, height) : 0;
}

extern "C" int gs_l1_dssim_loss(const float* color, const void* target, int target_is_u8, int32_t width,
                                int32_t height, float l1_weight, float dssim_weight, float* loss_out,
                                float* ssim_out, float* dL_dcolor, void* scratch, size_t scratch_bytes,
                                gs_stream_t stream) {
    GS_REQUIRE(color && target && loss_out && scratch, "l1_dssim_loss: null pointer");
    GS_REQUIRE(width > 0 && height > 0, "l1_dssim_loss: bad image size");
    GS_REQUIRE(scratch_bytes >= ssim_scratch_bytes(width, height), "l1_dssim_loss: scratch too small");
    const size_t P = (size_t)width * (size_t)height;
    char* q = reinterpret_cast<char*>(align_up(reinterpret_cast<uintptr_t>(scratch), 256));
    float* pa = reinterpret_cast<float*>(q);
    q += align_up(P * 3 * sizeof(float), 256);
    float* pb = reinterpret_cast<float*>(q);
    q += align_up(P * 3 * sizeof(float), 256);
    float* pc = reinterpret_cast<float*>(q);
    q += align_up(P * 3 * sizeof(float), 256);
    float2* tile_sums = reinterpret_cast<float2*>(q);
    const int tiles = ((width + kLT - 1) / kLT) * ((height + kLT - 1) / kLT);
    const cudaStream_t st = (cudaStream_t)stream;
    ssim_fwd_kernel<<<tiles, 256, 0, st>>>(color, target, target_is_u8 ? 1 : 0, width, height, pa, pb, pc,
                                          tile_sums);
    GS_TRY(check_launch("ssim_fwd_kernel"));
    const double inv_count = 1.0 / (3.0 * (double)P);
    loss_finalize_kernel<<<1, 1024, 0, st>>>(tile_sums, tiles, inv_count, l1_weight, dssim_weight, loss_out,
                                             ssim_out);
    GS_TRY(check_launch("loss_finalize_kernel"));
    if (!dL_dcolor) return GS_OK;
    const float g_l1 = (float)((double)l1_weight * inv_count);
    const float g_ssim = (float)(-(double)dssim_weight * 0.5 * inv_count);
    ssim_bwd_kernel<<<tiles, 256, 0, st>>>(color, target, target_is_u8 ? 1 : 0, width, height, pa, pb, pc, g_l1,
                                          g_ssim, dL_dcolor);
    return check_launch("ssim_bwd_kernel");
}
