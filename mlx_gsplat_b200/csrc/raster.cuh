// Shared device code of the rasterizer kernels: camera constants, the
// per-Gaussian projection of mlx_gsplat/rendering.py:153-244, and the
// splat-versus-tile bound used by binning.
#pragma once

#include "common.cuh"

namespace gs {

constexpr float kSH_C0 = 0.28209479177387814f;
constexpr float kSH_C1 = 0.4886025119029199f;

struct RasterParams {
    float vm[16];
    float fx, fy, cx, cy;
    float campos[3];   // -R^T t (rendering.py:221-223)
    float sx, sy, hsx, hsy;  // pixel scale and half scale (rendering.py:251-255)
    int rw, rh, tiles_x, tiles_y;
    float alpha_cut, t_min;
    float loss_scale;  // 1 / (3 * rw * rh) for the mean-based losses
    int masked;        // the splat records carry an alpha multiplier (gs_apply_sorted_mask)
};

inline RasterParams make_raster_params(const gs_camera& c, const gs_raster_settings* rs) {
    RasterParams p;
    for (int i = 0; i < 16; ++i) p.vm[i] = c.viewmat[i];
    p.fx = c.fx;
    p.fy = c.fy;
    p.cx = c.cx;
    p.cy = c.cy;
    for (int i = 0; i < 3; ++i)
        p.campos[i] = -(c.viewmat[0 * 4 + i] * c.viewmat[3] + c.viewmat[1 * 4 + i] * c.viewmat[7] +
                        c.viewmat[2 * 4 + i] * c.viewmat[11]);
    p.sx = (float)c.width / (float)c.render_width;
    p.sy = (float)c.height / (float)c.render_height;
    p.hsx = p.sx * 0.5f;
    p.hsy = p.sy * 0.5f;
    p.rw = c.render_width;
    p.rh = c.render_height;
    p.tiles_x = (c.render_width + kTile - 1) / kTile;
    p.tiles_y = (c.render_height + kTile - 1) / kTile;
    p.alpha_cut = rs ? rs->alpha_cutoff : 1e-7f;
    p.t_min = rs ? rs->transmittance_min : 1e-6f;
    p.loss_scale = (float)(1.0 / (3.0 * (double)c.render_width * (double)c.render_height));
    p.masked = rs ? (rs->alpha_mask != 0) : 0;
    return p;
}

// Everything the forward computes for one Gaussian (kept for the backward's recompute).
struct ProjState {
    float mx, my, mz;          // world mean
    float tx, ty, tz, z;       // camera point; z = max(tz, 1e-4)
    float u, v;
    float qw, qx, qy, qz, qn;  // raw quaternion and its norm sqrt(sum q^2 + 1e-8)
    float R[9];                // rotation of the normalised quaternion
    float S[3];                // exp(log-scale)
    float Sg[9];               // 3-D covariance R S S^T R^T
    float T[6];                // J W (2 x 3)
    float a, b, c, d;          // 2-D covariance + 0.3 I
    float det_raw, det;        // det before / after the 1e-6 floor
    float ca, cb, cc, cd;      // conic (inverse)
    float opac;                // sigmoid(logit)
    float dir[3], dnorm;       // unit view direction and |mean - campos|
    float pre[3];              // SH colour + 0.5 before the [0, 1] clip
    float rgb[3];
};

__device__ __forceinline__ int64_t param_row(const gs_gaussians& g, int32_t id) {
    return g.table ? (int64_t)__ldg(g.table + id) : (int64_t)id;
}

// Colour rows the projection kernels are compiled for: kDeg = 1 covers the
// reference rule (DC, plus degree 1 when colors_dim >= 12) and GS_SH_FULL at
// degree <= 1; kDeg = 2 and 3 are GS_SH_FULL at that degree.  kPerCh is the
// number of coefficients per channel after the DC term, kCols the colour
// floats of a row.
template <int kDeg>
struct ShRow {
    static_assert(kDeg >= 1 && kDeg <= 3, "SH degree of a kernel variant must be 1, 2 or 3");
    static constexpr int kPerCh = (kDeg + 1) * (kDeg + 1) - 1;
    static constexpr int kCols = 3 + 3 * kPerCh;
};

// Degree of the kernel variant that evaluates a descriptor's colours.
inline int sh_kernel_degree(const gs_gaussians& g) {
    if (g.sh_mode != GS_SH_FULL) return 1;
    return g.colors_dim >= 48 ? 3 : (g.colors_dim >= 27 ? 2 : 1);
}

// The parameters the projection reads for one Gaussian.
template <int kDeg>
struct GaussianIn {
    float mx, my, mz;
    float qw, qx, qy, qz;
    float ls[3];    // log-scales
    float logit;    // opacity logit
    float col[ShRow<kDeg>::kCols];  // DC (3), then kPerCh coefficients per channel
};

// The pooled row layout, one row per Gaussian: quats (0-3) | means (4-6) |
// opacity (7) | scales (8-10) | colours (11-).  When a descriptor's pointers
// describe exactly that (equal strides that are a multiple of 4 floats,
// 16-byte-aligned rows, colours addressed by row) a row is moved with 16-byte
// vector accesses instead of one scalar access per value.
constexpr int kRowMean = 4, kRowOpac = 7, kRowScale = 8, kRowColor = 11;

// Colour floats a kernel variant reads from a row (the degree-1 variant reads
// only the DC term when colors_dim < 12).
template <int kDeg>
__host__ __device__ __forceinline__ int sh_cols_read(const gs_gaussians& g) {
    return kDeg == 1 ? (g.colors_dim >= 12 ? 12 : 3) : ShRow<kDeg>::kCols;
}

template <int kDeg>
inline bool slab_rows(const gs_gaussians& g) {
    const int64_t S = g.quats_stride;
    const int need = kRowColor + sh_cols_read<kDeg>(g);
    return g.quats && g.colors_by_visible == 0 && S % 4 == 0 && S >= (need + 3) / 4 * 4 && g.means_stride == S &&
           g.scales_stride == S && g.opac_stride == S && g.colors_stride == S && g.means == g.quats + kRowMean &&
           g.opac == g.quats + kRowOpac && g.scales == g.quats + kRowScale && g.colors == g.quats + kRowColor &&
           (reinterpret_cast<uintptr_t>(g.quats) & 15u) == 0;
}

template <bool kSlab, int kDeg>
__device__ __forceinline__ void load_gaussian(const gs_gaussians& g, int64_t row, int64_t crow, GaussianIn<kDeg>& in) {
    constexpr int NC = ShRow<kDeg>::kCols;
    const bool sh1 = g.colors_dim >= 12;
    if (kSlab && kDeg == 1) {
        const float4* r = reinterpret_cast<const float4*>(g.quats + row * g.quats_stride);
        const float4 a = __ldg(r), b = __ldg(r + 1), c = __ldg(r + 2), d = __ldg(r + 3);
        in.qw = a.x, in.qx = a.y, in.qy = a.z, in.qz = a.w;
        in.mx = b.x, in.my = b.y, in.mz = b.z, in.logit = b.w;
        in.ls[0] = c.x, in.ls[1] = c.y, in.ls[2] = c.z;
        in.col[0] = c.w, in.col[1] = d.x, in.col[2] = d.y;
        if (sh1) {
            const float4 e = __ldg(r + 4), f = __ldg(r + 5);
            in.col[3] = d.z, in.col[4] = d.w;
            in.col[5] = e.x, in.col[6] = e.y, in.col[7] = e.z, in.col[8] = e.w;
            in.col[9] = f.x, in.col[10] = f.y, in.col[11] = f.z;
        } else {
#pragma unroll
            for (int k = 3; k < NC; ++k) in.col[k] = 0.f;
        }
    } else if (kSlab) {
        // the whole row up to the last colour float, 16 bytes at a time
        constexpr int kVec = (kRowColor + NC + 3) / 4;
        const float4* r = reinterpret_cast<const float4*>(g.quats + row * g.quats_stride);
        float buf[4 * kVec];
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
            const float4 t = __ldg(r + j);
            buf[4 * j] = t.x, buf[4 * j + 1] = t.y, buf[4 * j + 2] = t.z, buf[4 * j + 3] = t.w;
        }
        in.qw = buf[0], in.qx = buf[1], in.qy = buf[2], in.qz = buf[3];
        in.mx = buf[kRowMean], in.my = buf[kRowMean + 1], in.mz = buf[kRowMean + 2];
        in.logit = buf[kRowOpac];
        in.ls[0] = buf[kRowScale], in.ls[1] = buf[kRowScale + 1], in.ls[2] = buf[kRowScale + 2];
#pragma unroll
        for (int k = 0; k < NC; ++k) in.col[k] = buf[kRowColor + k];
    } else {
        const float* mp = g.means + row * g.means_stride;
        const float* qp = g.quats + row * g.quats_stride;
        const float* sp = g.scales + row * g.scales_stride;
        const float* cp = g.colors + crow * g.colors_stride;
        in.mx = __ldg(mp), in.my = __ldg(mp + 1), in.mz = __ldg(mp + 2);
        in.qw = __ldg(qp), in.qx = __ldg(qp + 1), in.qy = __ldg(qp + 2), in.qz = __ldg(qp + 3);
        in.ls[0] = __ldg(sp), in.ls[1] = __ldg(sp + 1), in.ls[2] = __ldg(sp + 2);
        in.logit = __ldg(g.opac + row * g.opac_stride);
        const int nc = sh_cols_read<kDeg>(g);
#pragma unroll
        for (int k = 0; k < NC; ++k) in.col[k] = k < nc ? __ldg(cp + k) : 0.f;
    }
}

// ------------------------------------------------------------------ spherical harmonics, degrees 2 and 3
// Real SH basis functions of a unit direction (x, y, z), as polynomials with
// their normalisation constants K_lm = sqrt((2l+1)/(4 pi) * (l-|m|)!/(l+|m|)!)
// times the Legendre factor, in the sign convention common to 3DGS renderers:
//   degree 2:  K0 xy, -K0 yz, K1 (2z^2 - x^2 - y^2), -K0 xz, K2 (x^2 - y^2)
//              K0 = sqrt(15/pi)/2, K1 = sqrt(5/pi)/4, K2 = sqrt(15/pi)/4
//   degree 3:  -K3 y(3x^2 - y^2), K4 xyz, -K5 y(4z^2 - x^2 - y^2),
//              K6 z(2z^2 - 3x^2 - 3y^2), -K5 x(4z^2 - x^2 - y^2),
//              K7 z(x^2 - y^2), -K3 x(x^2 - 3y^2)
//              K3 = sqrt(35/(2pi))/4, K4 = sqrt(105/pi)/2, K5 = sqrt(21/(2pi))/4,
//              K6 = sqrt(7/pi)/4, K7 = sqrt(105/pi)/4
constexpr float kShK0 = 1.0925484305920792f, kShK1 = 0.31539156525252005f, kShK2 = 0.5462742152960396f;
constexpr float kShK3 = 0.5900435899266435f, kShK4 = 2.890611442640554f, kShK5 = 0.4570457994644658f;
constexpr float kShK6 = 0.3731763325901154f, kShK7 = 1.445305721320277f;

// b[0..4] = degree-2 basis, b[5..11] = degree-3 basis (when kDeg == 3).
template <int kDeg>
__device__ __forceinline__ void sh_basis_hi(float x, float y, float z, float* b) {
    const float xx = x * x, yy = y * y, zz = z * z;
    b[0] = kShK0 * x * y;
    b[1] = -kShK0 * y * z;
    b[2] = kShK1 * (2.f * zz - xx - yy);
    b[3] = -kShK0 * x * z;
    b[4] = kShK2 * (xx - yy);
    if (kDeg >= 3) {
        b[5] = -kShK3 * y * (3.f * xx - yy);
        b[6] = kShK4 * x * y * z;
        b[7] = -kShK5 * y * (4.f * zz - xx - yy);
        b[8] = kShK6 * z * (2.f * zz - 3.f * xx - 3.f * yy);
        b[9] = -kShK5 * x * (4.f * zz - xx - yy);
        b[10] = kShK7 * z * (xx - yy);
        b[11] = -kShK3 * x * (xx - 3.f * yy);
    }
}

// Gradient with respect to (x, y, z) of sum_j w[j] b_j(x, y, z) for the basis
// of sh_basis_hi (the direction's components taken as independent).
template <int kDeg>
__device__ __forceinline__ void sh_basis_hi_grad(float x, float y, float z, const float* w, float& gx, float& gy,
                                                 float& gz) {
    const float xx = x * x, yy = y * y, zz = z * z;
    gx = kShK0 * w[0] * y - kShK0 * w[3] * z - 2.f * kShK1 * w[2] * x + 2.f * kShK2 * w[4] * x;
    gy = kShK0 * w[0] * x - kShK0 * w[1] * z - 2.f * kShK1 * w[2] * y - 2.f * kShK2 * w[4] * y;
    gz = -kShK0 * w[1] * y - kShK0 * w[3] * x + 4.f * kShK1 * w[2] * z;
    if (kDeg >= 3) {
        gx += -kShK3 * w[5] * 6.f * x * y + kShK4 * w[6] * y * z + kShK5 * w[7] * 2.f * x * y -
              kShK6 * w[8] * 6.f * x * z - kShK5 * w[9] * (4.f * zz - 3.f * xx - yy) + kShK7 * w[10] * 2.f * x * z -
              kShK3 * w[11] * 3.f * (xx - yy);
        gy += -kShK3 * w[5] * 3.f * (xx - yy) + kShK4 * w[6] * x * z - kShK5 * w[7] * (4.f * zz - xx - 3.f * yy) -
              kShK6 * w[8] * 6.f * y * z + kShK5 * w[9] * 2.f * x * y - kShK7 * w[10] * 2.f * y * z +
              kShK3 * w[11] * 6.f * x * y;
        gz += kShK4 * w[6] * x * y - kShK5 * w[7] * 8.f * y * z + kShK6 * w[8] * (6.f * zz - 3.f * xx - 3.f * yy) -
              kShK5 * w[9] * 8.f * x * z + kShK7 * w[10] * (xx - yy);
    }
}

// rendering.py:153-244 for one Gaussian.  ``sh1``: the degree-1 term is
// evaluated (kDeg = 1 only; the higher variants always evaluate every degree
// up to kDeg).
template <int kDeg>
__device__ __forceinline__ void project_one(const GaussianIn<kDeg>& in, bool sh1, const RasterParams& p,
                                            ProjState& s) {
    s.mx = in.mx;
    s.my = in.my;
    s.mz = in.mz;
    s.tx = cam_row(p.vm, 0, s.mx, s.my, s.mz);
    s.ty = cam_row(p.vm, 1, s.mx, s.my, s.mz);
    s.tz = cam_row(p.vm, 2, s.mx, s.my, s.mz);
    s.z = s.tz > 1e-4f ? s.tz : 1e-4f;
    s.u = __fadd_rn(__fdiv_rn(__fmul_rn(s.tx, p.fx), s.z), p.cx);
    s.v = __fadd_rn(__fdiv_rn(__fmul_rn(s.ty, p.fy), s.z), p.cy);

    s.qw = in.qw;
    s.qx = in.qx;
    s.qy = in.qy;
    s.qz = in.qz;
    s.qn = sqrtf(s.qw * s.qw + s.qx * s.qx + s.qy * s.qy + s.qz * s.qz + 1e-8f);
    const float r = s.qw / s.qn, x = s.qx / s.qn, y = s.qy / s.qn, z = s.qz / s.qn;
    s.R[0] = 1.f - 2.f * (y * y + z * z);
    s.R[1] = 2.f * (x * y - r * z);
    s.R[2] = 2.f * (x * z + r * y);
    s.R[3] = 2.f * (x * y + r * z);
    s.R[4] = 1.f - 2.f * (x * x + z * z);
    s.R[5] = 2.f * (y * z - r * x);
    s.R[6] = 2.f * (x * z - r * y);
    s.R[7] = 2.f * (y * z + r * x);
    s.R[8] = 1.f - 2.f * (x * x + y * y);

    s.S[0] = expf(in.ls[0]);
    s.S[1] = expf(in.ls[1]);
    s.S[2] = expf(in.ls[2]);
    float M[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) M[3 * i + j] = s.R[3 * i + j] * s.S[j];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            s.Sg[3 * i + j] = M[3 * i + 0] * M[3 * j + 0] + M[3 * i + 1] * M[3 * j + 1] + M[3 * i + 2] * M[3 * j + 2];

    // J (third row zero) times W = viewmat[:3,:3]  (rendering.py:189-199)
    const float tz2 = s.z * s.z;
    const float j00 = p.fx / s.z, j02 = -p.fx * s.tx / tz2;
    const float j11 = p.fy / s.z, j12 = -p.fy * s.ty / tz2;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        s.T[k] = j00 * p.vm[0 * 4 + k] + j02 * p.vm[2 * 4 + k];
        s.T[3 + k] = j11 * p.vm[1 * 4 + k] + j12 * p.vm[2 * 4 + k];
    }
    // X = Sigma3 T^T (3 x 2), Sigma2 = T X   (rendering.py:200)
    float X0[3], X1[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        X0[k] = s.Sg[3 * k + 0] * s.T[0] + s.Sg[3 * k + 1] * s.T[1] + s.Sg[3 * k + 2] * s.T[2];
        X1[k] = s.Sg[3 * k + 0] * s.T[3] + s.Sg[3 * k + 1] * s.T[4] + s.Sg[3 * k + 2] * s.T[5];
    }
    s.a = s.T[0] * X0[0] + s.T[1] * X0[1] + s.T[2] * X0[2] + 0.3f;
    s.b = s.T[0] * X1[0] + s.T[1] * X1[1] + s.T[2] * X1[2];
    s.c = s.T[3] * X0[0] + s.T[4] * X0[1] + s.T[5] * X0[2];
    s.d = s.T[3] * X1[0] + s.T[4] * X1[1] + s.T[5] * X1[2] + 0.3f;
    s.det_raw = s.a * s.d - s.b * s.c;
    s.det = s.det_raw > 1e-6f ? s.det_raw : 1e-6f;
    s.ca = s.d / s.det;
    s.cb = -s.b / s.det;
    s.cc = -s.c / s.det;
    s.cd = s.a / s.det;

    s.opac = 1.0f / (1.0f + expf(-in.logit));

    const float dx = s.mx - p.campos[0], dy = s.my - p.campos[1], dz = s.mz - p.campos[2];
    s.dnorm = sqrtf(dx * dx + dy * dy + dz * dz);
    const float inv = 1.0f / (s.dnorm + 1e-8f);
    s.dir[0] = dx * inv;
    s.dir[1] = dy * inv;
    s.dir[2] = dz * inv;
    constexpr int k = ShRow<kDeg>::kPerCh;
    float c[3] = {in.col[0] * kSH_C0, in.col[1] * kSH_C0, in.col[2] * kSH_C0};
    if (kDeg > 1 || sh1) {
        const float xd = s.dir[0], yd = s.dir[1], zd = s.dir[2];
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            const float* cc = in.col + 3 + k * ch;
            c[ch] += kSH_C1 * (cc[0] * yd + cc[1] * zd + cc[2] * xd);
        }
        if (kDeg > 1) {
            float b[12];
            sh_basis_hi<kDeg>(xd, yd, zd, b);
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                const float* cc = in.col + 3 + k * ch + 3;
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < k - 3; ++j) acc += cc[j] * b[j];
                c[ch] += acc;
            }
        }
    }
    s.pre[0] = c[0] + 0.5f;
    s.pre[1] = c[1] + 0.5f;
    s.pre[2] = c[2] + 0.5f;
#pragma unroll
    for (int k = 0; k < 3; ++k) s.rgb[k] = fminf(fmaxf(s.pre[k], 0.0f), 1.0f);
}

// ------------------------------------------------------------------ splat falloff
// g = exp(-m / 2) evaluated as 2^(m * (-log2(e) / 2)) with the hardware base-2
// exponential (ex2.approx, relative error ~2^-22).  Forward and backward call
// this one function, so both see bit-identical alphas.
constexpr float kHalfNegLog2e = -0.72134752044448170368f;  // -log2(e) / 2

__device__ __forceinline__ float splat_falloff(float m) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(m * kHalfNegLog2e));
    return y;
}

// Hardware reciprocal (rcp.approx, about 1 ulp).
__device__ __forceinline__ float fast_rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ------------------------------------------------------------------ compositing layout
// One CTA per 16x16 tile; each thread owns P pixels of one column, row_step
// rows apart, so warp w covers a cols-wide, rows-tall block of the tile
// (8 x 8 for P = 2, 8 x 16 for P = 4, the whole tile for P = 8).  A thread's
// pixels are taken two at a time (pair q: its pixels 2q and 2q + 1).
template <int P>
struct CompositeLayout {
    static_assert(P == 2 || P == 4 || P == 8, "compositing pixels per thread must be 2, 4 or 8");
    static constexpr int threads = kTileThreads / P;
    static constexpr int cols = P == 8 ? 16 : 8;
    static constexpr int row_step = 32 / cols;
    static constexpr int rows = row_step * P;
    static constexpr int blocks_x = kTile / cols;
    static constexpr int pairs = P / 2;
    __device__ static int block_x(int warp) { return (warp % blocks_x) * cols; }
    __device__ static int block_y(int warp) { return (warp / blocks_x) * rows; }
    __device__ static int col(int lane) { return lane % cols; }
    __device__ static int row(int lane, int k) { return lane / cols + row_step * k; }  // row of pixel k
};

// ------------------------------------------------------------------ pixel pairs
// The compositing kernels evaluate two pixels of one column together with the
// sm_100 paired fp32 instructions (one issue slot for two round-to-nearest
// multiplies / adds / fused multiply-adds); each lane of a pair rounds exactly
// like its scalar counterpart.
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Mahalanobis distances of a pixel pair at offsets (x, y.x) and (x, y.y) from a
// splat with conic (a, b; c, d), given ax = a x and cx = c x:
//   m = x (a x + b y) + y (c x + d y).
// The forward and the backward both call this, so they agree bit for bit.
__device__ __forceinline__ float2 pair_quad(float2 y, float x, float ax, float cx, float b, float d) {
    const float2 t1 = __ffma2_rn(f2(b), y, f2(ax));
    const float2 t2 = __ffma2_rn(f2(d), y, f2(cx));
    return __ffma2_rn(f2(x), t1, __fmul2_rn(y, t2));
}

// splat_falloff of both lanes.
__device__ __forceinline__ float2 pair_falloff(float2 m) {
    const float2 e = __fmul2_rn(m, f2(kHalfNegLog2e));
    float2 r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(e.x));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(e.y));
    return r;
}

// ------------------------------------------------------------------ per-pixel contribution rule
// A (pixel, splat) pair contributes iff its Mahalanobis distance m satisfies
// m <= 2 ln(opacity / alpha_cutoff), i.e. alpha = opacity * exp(-m/2) >=
// alpha_cutoff.  The bound is stored in the splat record; forward and backward
// apply the same test to the same floats, so they see the same pairs.  A
// splat too faint to reach alpha_cutoff anywhere gets -1 (never contributes).
__device__ __forceinline__ float pair_cut(float opac, const RasterParams& p) {
    return opac > p.alpha_cut ? 2.0f * logf(opac / p.alpha_cut) : -1.0f;
}

// ------------------------------------------------------------------ tile binning bound
// A splat is binned into a tile when some pixel centre of the tile can see
// alpha >= alpha_cut, i.e. Mahalanobis m <= m_cut = 2 ln(opac / alpha_cut).
// The bound is evaluated on the continuous rectangle spanned by the tile's
// pixel centres (a superset of the centres), with a small relative slack.
struct TileBox {
    int x0, x1, y0, y1;  // inclusive tile range
    bool exact;          // false: conic not positive definite -> every tile of the box
    float m_cut, s;      // cut and symmetric off-diagonal (cb + cc) / 2
};

__device__ __forceinline__ bool splat_tile_box(float u, float v, float ca, float cb, float cc, float cd, float opac,
                                               const RasterParams& p, TileBox& tb) {
    if (!(opac > p.alpha_cut)) return false;
    if (!(isfinite(u) && isfinite(v) && isfinite(ca) && isfinite(cb) && isfinite(cc) && isfinite(cd))) return false;
    tb.m_cut = pair_cut(opac, p);
    tb.s = 0.5f * (cb + cc);
    const float det = ca * cd - tb.s * tb.s;
    if (ca > 0.f && cd > 0.f && det > 0.f) {
        const float m = tb.m_cut * 1.0002f + 1e-3f;
        const float ex = sqrtf(m * cd / det) * 1.0002f + 1e-3f;
        const float ey = sqrtf(m * ca / det) * 1.0002f + 1e-3f;
        const float i0 = fmaxf(ceilf((u - ex - p.hsx) / p.sx), 0.f);
        const float i1 = fminf(floorf((u + ex - p.hsx) / p.sx), (float)(p.rw - 1));
        const float j0 = fmaxf(ceilf((v - ey - p.hsy) / p.sy), 0.f);
        const float j1 = fminf(floorf((v + ey - p.hsy) / p.sy), (float)(p.rh - 1));
        if (!(i0 <= i1 && j0 <= j1)) return false;
        tb.x0 = (int)i0 / kTile;
        tb.x1 = (int)i1 / kTile;
        tb.y0 = (int)j0 / kTile;
        tb.y1 = (int)j1 / kTile;
        tb.exact = true;
    } else {
        tb.x0 = 0;
        tb.x1 = p.tiles_x - 1;
        tb.y0 = 0;
        tb.y1 = p.tiles_y - 1;
        tb.exact = false;
    }
    return true;
}

__device__ __forceinline__ float quad_form(float ca, float s, float cd, float x, float y) {
    return ca * x * x + 2.0f * s * x * y + cd * y * y;
}

// Minimum of the positive-definite form ca x^2 + 2 s x y + cd y^2 over the
// rectangle [x0, x1] x [y0, y1] (offsets from the splat centre): zero when the
// centre is inside, otherwise the smallest of the four edge minima.
__device__ __forceinline__ float rect_min_quad(float ca, float s, float cd, float x0, float x1, float y0, float y1) {
    if (x0 <= 0.f && 0.f <= x1 && y0 <= 0.f && 0.f <= y1) return 0.f;
    // edge minimisers; an approximate reciprocal only moves them by ~1e-7 relative
    // and the form is stationary there, so the minimum changes at second order
    const float rcd = fast_rcp(cd), rca = fast_rcp(ca);
    float best = 3.4e38f;
    const float ya = fminf(fmaxf(-s * x0 * rcd, y0), y1);
    best = fminf(best, quad_form(ca, s, cd, x0, ya));
    const float yb = fminf(fmaxf(-s * x1 * rcd, y0), y1);
    best = fminf(best, quad_form(ca, s, cd, x1, yb));
    const float xa = fminf(fmaxf(-s * y0 * rca, x0), x1);
    best = fminf(best, quad_form(ca, s, cd, xa, y0));
    const float xb = fminf(fmaxf(-s * y1 * rca, x0), x1);
    best = fminf(best, quad_form(ca, s, cd, xb, y1));
    return best;
}

// Can a staged splat (records q0, q1 and its pair cut) reach any pixel centre
// of the rectangle of pixels [pi0, pi1] x [pj0, pj1]?  Conservative (continuous
// rectangle, relative slack); a conic that is not positive definite passes.
// The compositing kernels use it to skip splats that miss a warp's pixel block.
__device__ __forceinline__ bool splat_hits_block(float4 q0, float4 q1, float cut, int pi0, int pi1, int pj0, int pj1,
                                                 const RasterParams& p) {
    if (!(cut >= 0.f)) return false;
    const float ca = q0.z, cd = q1.y, s = 0.5f * (q0.w + q1.x);
    if (!(ca > 0.f && cd > 0.f && ca * cd - s * s > 0.f)) return true;
    const float x0 = (float)pi0 * p.sx + p.hsx - q0.x, x1 = (float)pi1 * p.sx + p.hsx - q0.x;
    const float y0 = (float)pj0 * p.sy + p.hsy - q0.y, y1 = (float)pj1 * p.sy + p.hsy - q0.y;
    return rect_min_quad(ca, s, cd, x0, x1, y0, y1) <= cut * 1.0002f + 1e-3f;
}

// Minimum of the (positive definite) quadratic form over the tile's pixel-centre rectangle.
__device__ __forceinline__ bool splat_hits_tile(float u, float v, float ca, float cd, const TileBox& tb, int tx,
                                                int ty, const RasterParams& p) {
    if (!tb.exact) return true;
    const int i0 = tx * kTile, i1 = min(i0 + kTile - 1, p.rw - 1);
    const int j0 = ty * kTile, j1 = min(j0 + kTile - 1, p.rh - 1);
    const float x0 = (float)i0 * p.sx + p.hsx - u, x1 = (float)i1 * p.sx + p.hsx - u;
    const float y0 = (float)j0 * p.sy + p.hsy - v, y1 = (float)j1 * p.sy + p.hsy - v;
    return rect_min_quad(ca, tb.s, cd, x0, x1, y0, y1) <= tb.m_cut * 1.0002f + 1e-3f;
}

}  // namespace gs
