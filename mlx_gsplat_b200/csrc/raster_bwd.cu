// Rasterizer backward: back-to-front compositing gradient with warp-reduced
// atomics, and the projection backward to the Gaussian parameters (the
// vector-Jacobian product MLX's autograd forms for mlx_gsplat/rendering.py:153-300).
#include "raster.cuh"

namespace gs {

// Compositing layouts (CompositeLayout), chosen per launch: 4 pixels per
// thread (64-thread CTAs, 16 per SM at 64 registers) when the image has at
// least one full wave of tiles; 2 pixels per thread (128-thread CTAs, 10 per
// SM at 48 registers) below that, where twice the warps per tile keep the
// SMs busy.  Measured: 2 pixels per thread took the 200k-Gaussian 648x420
// step's backward from 0.427 to 0.375 ms (1,161 tiles), and the 1 M-Gaussian
// 1297x840 one's from 1.263 to 1.491 ms (4,346 tiles).
constexpr int kBwdMinCtas4 = 16, kBwdMinCtas2 = 10;
template <int P>
struct BwdLayout {
    using L = CompositeLayout<P>;
    static constexpr int threads = L::threads, pairs = L::pairs;
    static constexpr int min_ctas = P == 4 ? kBwdMinCtas4 : kBwdMinCtas2;
};
constexpr int kBatch = 128;  // splats staged in shared memory per batch
static_assert(kBatch % BwdLayout<2>::threads == 0 && kBatch % BwdLayout<4>::threads == 0 && kBatch % 32 == 0,
              "batch must tile the CTA");

constexpr int kGradRec = 12;  // floats per splat gradient record

// For every tile: walk the tile's entries from the last one any pixel used
// back to the first.  Per pixel the transmittance before entry i is
// recovered as T_i = T_{i+1} / (1 - alpha_i), and with
//   val_i = dL/dC . rgb_i + dL/dA,   B_{i-1} = alpha_i val_i + (1 - alpha_i) B_i
// the alpha gradient is dL/dalpha_i = T_i (val_i - B_i).  The clip of
// opacity * g to [0, 0.99] passes the gradient only strictly inside
// (MLX's maximum/minimum rule).  Pixel layout as in the forward
// (CompositeLayout, one CTA per tile).  The nine per-splat sums of a
// warp's pixels are reduced with 14 shuffles, added into per-batch
// shared-memory accumulators, and flushed with one global vector reduction
// per (tile, splat).
//
// Two forms of a splat's step, chosen per (warp, splat), both bit-identical
// to the forward's alphas:
//  * fast — the splat's opacity is below 0.98 and its conic is positive
//    definite, so opacity * g < 0.99 wherever the splat reaches (g <= 1 up
//    to rounding): the clip is the identity and passes every gradient.  A
//    pixel that does not take part gets m = +inf, hence g = 0 and alpha = 0.
//  * general — the 0.99 clip and its gradient mask, for every other splat.
struct PixelBwd {
    float T, dr, dg, db, dA;
    int last;
};

__device__ __forceinline__ void pixel_bwd_init(PixelBwd& s, bool inside, int64_t pix, const RasterParams& p,
                                               const float* out_color, const float* final_T, const int32_t* n_contrib,
                                               int loss_mode, const void* target, const float* dL_dcolor,
                                               const float* dL_dalpha) {
    s.T = 1.f;
    s.dr = s.dg = s.db = s.dA = 0.f;
    s.last = 0;
    if (!inside) return;
    s.T = final_T[pix];
    s.last = n_contrib[pix];
    if (loss_mode == GS_LOSS_NONE) {
        s.dr = dL_dcolor[3 * pix + 0];
        s.dg = dL_dcolor[3 * pix + 1];
        s.db = dL_dcolor[3 * pix + 2];
        s.dA = dL_dalpha ? dL_dalpha[pix] : 0.f;
    } else if (loss_mode == GS_LOSS_MEAN) {
        s.dr = s.dg = s.db = p.loss_scale;
    } else {
        float t0, t1, t2;
        if (loss_mode == GS_LOSS_L1_U8) {
            const uint8_t* t8 = static_cast<const uint8_t*>(target) + 3 * pix;
            t0 = __fdiv_rn((float)t8[0], 255.0f);
            t1 = __fdiv_rn((float)t8[1], 255.0f);
            t2 = __fdiv_rn((float)t8[2], 255.0f);
        } else {
            const float* tf = static_cast<const float*>(target) + 3 * pix;
            t0 = tf[0];
            t1 = tf[1];
            t2 = tf[2];
        }
        const float e0 = out_color[3 * pix + 0] - t0, e1 = out_color[3 * pix + 1] - t1,
                    e2 = out_color[3 * pix + 2] - t2;
        s.dr = (e0 > 0.f ? 1.f : (e0 < 0.f ? -1.f : 0.f)) * p.loss_scale;
        s.dg = (e1 > 0.f ? 1.f : (e1 < 0.f ? -1.f : 0.f)) * p.loss_scale;
        s.db = (e2 > 0.f ? 1.f : (e2 < 0.f ? -1.f : 0.f)) * p.loss_scale;
    }
}

// Per-splat constants of the backward step: colour and opacity.
struct SplatBwd {
    float r, g, b, opac;
};

// Backward state of a pixel pair (lanes .x / .y: a thread's pixels 2q and 2q + 1).
// ``dA`` is carried only when the loss has an alpha cotangent (kDA).
template <bool kDA>
struct PairBwd {
    float2 T, dr, dg, db, Bv;
    int last0, last1;
};
template <>
struct PairBwd<true> {
    float2 T, dr, dg, db, dA, Bv;
    int last0, last1;
};

template <bool kDA>
__device__ __forceinline__ float2 pair_val(const PairBwd<kDA>& s, const SplatBwd& c) {
    if constexpr (kDA)
        return __ffma2_rn(s.dr, f2(c.r), __ffma2_rn(s.dg, f2(c.g), __ffma2_rn(s.db, f2(c.b), s.dA)));
    else
        return __ffma2_rn(s.dr, f2(c.r), __ffma2_rn(s.dg, f2(c.g), __fmul2_rn(s.db, f2(c.b))));
}

// One splat's step for a pixel pair, given the pair's alpha ``al`` (0 where a
// pixel does not take part) and the clip's gradient mask times the falloff
// ``gi``.  Adds w T dL/dC to the colour sums and dog = dL/dalpha * g (the
// geometry gradients are linear in it, see the kernel) with its y moments to
// the pair sums.  A pixel with alpha = 0 keeps T and B and adds nothing.
template <bool kDA>
__device__ __forceinline__ void pair_bwd_accum(PairBwd<kDA>& s, float2 al, float2 gi, float2 y, const SplatBwd& c,
                                               float2& sd, float2& sy, float2& syy, float2& sr, float2& sg,
                                               float2& sb) {
    const float2 oma = __ffma2_rn(al, f2(-1.f), f2(1.f));  // 1 - alpha >= 0.01
    s.T = __fmul2_rn(s.T, make_float2(fast_rcp(oma.x), fast_rcp(oma.y)));  // T_i = T_{i+1} / (1 - alpha_i)
    const float2 val = pair_val<kDA>(s, c);
    const float2 d = __ffma2_rn(s.Bv, f2(-1.f), val);  // val - B
    s.Bv = __ffma2_rn(al, d, s.Bv);                     // = al * val + (1 - al) * B
    const float2 wT = __fmul2_rn(al, s.T);
    sr = __ffma2_rn(wT, s.dr, sr);
    sg = __ffma2_rn(wT, s.dg, sg);
    sb = __ffma2_rn(wT, s.db, sb);
    const float2 dog = __fmul2_rn(__fmul2_rn(s.T, d), gi);
    sd = __fadd2_rn(sd, dog);
    const float2 t = __fmul2_rn(dog, y);
    sy = __fadd2_rn(sy, t);
    syy = __ffma2_rn(t, y, syy);
}

// General form: the 0.99 clip and its gradient mask; with kMask the clipped
// alpha, and with it the gradient through the clip, is scaled by the splat's
// mask multiplier ``mk`` (alpha = clip(opacity g, 0, 0.99) * mk).
template <bool kDA, bool kMask = false>
__device__ __forceinline__ void pair_bwd_step(PairBwd<kDA>& s, bool v0, bool v1, float2 m, float2 y,
                                              const SplatBwd& c, float2& sd, float2& sy, float2& syy, float2& sr,
                                              float2& sg, float2& sb, float mk = 1.f) {
    const float2 gv = pair_falloff(m);
    const float2 og = __fmul2_rn(f2(c.opac), gv);
    float2 al = make_float2(v0 ? fminf(og.x, 0.99f) : 0.f, v1 ? fminf(og.y, 0.99f) : 0.f);
    // the clip of opacity * g to [0, 0.99] passes the gradient strictly inside
    // (opacity * g > 0 holds for every pixel that takes part: m <= the pair cut)
    float2 gi = make_float2(v0 && og.x < 0.99f ? gv.x : 0.f, v1 && og.y < 0.99f ? gv.y : 0.f);
    if constexpr (kMask) {
        al = __fmul2_rn(al, f2(mk));
        gi = __fmul2_rn(gi, f2(mk));
    }
    pair_bwd_accum<kDA>(s, al, gi, y, c, sd, sy, syy, sr, sg, sb);
}

// Fast form: alpha = opacity * g with g = 0 where the pixel does not take part.
template <bool kDA>
__device__ __forceinline__ void pair_bwd_step_fast(PairBwd<kDA>& s, bool v0, bool v1, float2 m, float2 y,
                                                   const SplatBwd& c, float2& sd, float2& sy, float2& syy,
                                                   float2& sr, float2& sg, float2& sb) {
    const float inf = __int_as_float(0x7f800000);
    const float2 gv = pair_falloff(make_float2(v0 ? m.x : inf, v1 ? m.y : inf));  // ex2(-inf) = 0
    const float2 al = __fmul2_rn(f2(c.opac), gv);
    pair_bwd_accum<kDA>(s, al, gv, y, c, sd, sy, syy, sr, sg, sb);
}

template <int P, bool kDA, bool kMask>
__global__ void __launch_bounds__(BwdLayout<P>::threads, BwdLayout<P>::min_ctas) render_bwd_kernel(
    const gs_tile_range* __restrict__ ranges, const int32_t* __restrict__ tile_order, const uint32_t* __restrict__ vals, const float4* __restrict__ splats,
    int64_t nv, RasterParams p, const float* __restrict__ out_color, const float* __restrict__ final_T,
    const int32_t* __restrict__ n_contrib, int loss_mode, const void* __restrict__ target,
    const float* __restrict__ dL_dcolor, const float* __restrict__ dL_dalpha, float* __restrict__ splat_grads) {
    using Layout = typename BwdLayout<P>::L;
    constexpr int kRenderThreads = BwdLayout<P>::threads, kPairs = BwdLayout<P>::pairs;
    __shared__ float4 s0[kBatch], s1[kBatch], s2[kBatch];
    __shared__ uint32_t sv[kBatch];
    __shared__ float acc[kBatch][9];  // per-batch CTA sums of the splat gradients
    __shared__ int smax;
    const int tile = tile_order ? tile_order[blockIdx.x] : (int)blockIdx.x;
    if (tile < 0 || tile >= p.tiles_x * p.tiles_y) return;  // uniform over the CTA
    const int tx = tile % p.tiles_x, ty = tile / p.tiles_x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bx0 = tx * kTile + Layout::block_x(warp), by0 = ty * kTile + Layout::block_y(warp);  // warp block
    const int pi = bx0 + Layout::col(lane);
    const float px = (float)pi * p.sx + p.hsx;
    const gs_tile_range rg = ranges[tile];
    for (int j = threadIdx.x; j < kBatch; j += kRenderThreads)
#pragma unroll
        for (int c = 0; c < 9; ++c) acc[j][c] = 0.f;

    PairBwd<kDA> s[kPairs];
    float2 py[kPairs];
    int mylast = 0;
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
        const int pj = by0 + Layout::row(lane, 2 * q), pj1 = by0 + Layout::row(lane, 2 * q + 1);
        PixelBwd a, b;
        pixel_bwd_init(a, pi < p.rw && pj < p.rh, (int64_t)pj * p.rw + pi, p, out_color, final_T, n_contrib,
                       loss_mode, target, dL_dcolor, dL_dalpha);
        pixel_bwd_init(b, pi < p.rw && pj1 < p.rh, (int64_t)pj1 * p.rw + pi, p, out_color, final_T, n_contrib,
                       loss_mode, target, dL_dcolor, dL_dalpha);
        py[q] = make_float2((float)pj * p.sy + p.hsy, (float)pj1 * p.sy + p.hsy);
        s[q].T = make_float2(a.T, b.T);
        s[q].dr = make_float2(a.dr, b.dr);
        s[q].dg = make_float2(a.dg, b.dg);
        s[q].db = make_float2(a.db, b.db);
        if constexpr (kDA) s[q].dA = make_float2(a.dA, b.dA);
        s[q].Bv = f2(0.f);
        s[q].last0 = a.last;
        s[q].last1 = b.last;
        mylast = max(mylast, max(a.last, b.last));
    }
    if (threadIdx.x == 0) smax = 0;
    __syncthreads();
    if (mylast > 0) atomicMax(&smax, mylast);
    __syncthreads();
    const int max_last = smax;
    // this warp's own last used entry: staged splats past it reach none of its pixels
    int wlast = mylast;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wlast = max(wlast, __shfl_xor_sync(kFull, wlast, o));

    for (int bend = rg.start + max_last; bend > rg.start; bend -= kBatch) {
        const int bstart = max(bend - kBatch, rg.start);
        const int cnt = bend - bstart;
        __syncthreads();
        for (int j = threadIdx.x; j < cnt; j += kRenderThreads) {
            const uint32_t vr = vals[bstart + j];
            const uint32_t vi = vr < (uint64_t)nv ? vr : 0u;
            sv[j] = vi;
            const float4 a = splats[3 * vi], b = splats[3 * vi + 1];
            float4 c = splats[3 * vi + 2];
            // .w (the depth, unused here) becomes the fast-form flag of the splat;
            // with an alpha mask it keeps the mask multiplier (general form only)
            const float sym = 0.5f * (a.w + b.x);
            if constexpr (!kMask)
                c.w = (b.z < 0.98f && a.z > 0.f && b.y > 0.f && a.z * b.y - sym * sym > 0.f) ? 1.f : 0.f;
            s0[j] = a;
            s1[j] = b;
            s2[j] = c;
        }
        __syncthreads();
        // which staged splats can reach this warp's pixel block (same test as the forward),
        // among those before the warp's last used entry
        const int kend = min(cnt, wlast - (bstart - rg.start));
        unsigned hits[kBatch / 32];
#pragma unroll
        for (int i = 0; i < kBatch / 32; ++i) {
            const int k = 32 * i + lane;
            const bool h =
                k < kend && splat_hits_block(s0[k], s1[k], s2[k].z, bx0, bx0 + Layout::cols - 1, by0,
                                             by0 + Layout::rows - 1, p);
            hits[i] = __ballot_sync(kFull, h);
        }
#pragma unroll
        for (int i = kBatch / 32 - 1; i >= 0; --i) {
          unsigned bits = hits[i];
          while (bits) {
            const int hb = 31 - __clz(bits);
            bits &= ~(1u << hb);
            const int k = 32 * i + hb;
            const int idx = bstart + k - rg.start;
            const float4 q0 = s0[k], q1 = s1[k], q2 = s2[k];
            const bool fast = !kMask && q2.w != 0.f;  // uniform over the warp
            const float x = px - q0.x;
            const float ax = q0.z * x, cx = q1.x * x;
            float2 y[kPairs], m[kPairs];
            bool v0[kPairs], v1[kPairs];
            bool any = false;
#pragma unroll
            for (int q = 0; q < kPairs; ++q) {
                y[q] = __fadd2_rn(py[q], f2(-q0.y));
                m[q] = pair_quad(y[q], x, ax, cx, q0.w, q1.y);
                v0[q] = idx < s[q].last0 && m[q].x <= q2.z;
                v1[q] = idx < s[q].last1 && m[q].y <= q2.z;
                any |= v0[q] | v1[q];
            }
            if (!__any_sync(kFull, any)) continue;
            // Per thread sums over its pixels (same column offset x):
            //   g5 = sum dog, g0 = sum dog x, g1 = sum dog y, g2 = sum dog x^2,
            //   g3 = sum dog x y, g4 = sum dog y^2, g6..8 = sum w T dL/dC.
            // With dm = -opacity/2 * dog the splat gradients are linear in these
            // sums; the per-splat factors are applied once, at the flush.
            SplatBwd c;
            c.r = q1.w;
            c.g = q2.x;
            c.b = q2.y;
            c.opac = q1.z;
            float2 sd = f2(0.f), sy = f2(0.f), syy = f2(0.f), sr = f2(0.f), sg = f2(0.f), sb = f2(0.f);
            if (fast) {
#pragma unroll
                for (int q = 0; q < kPairs; ++q) {
                    // a pair row of the warp block that the splat misses entirely
                    // contributes exactly nothing (alpha = 0 leaves T and B as they are)
                    if (!__any_sync(kFull, v0[q] | v1[q])) continue;
                    pair_bwd_step_fast<kDA>(s[q], v0[q], v1[q], m[q], y[q], c, sd, sy, syy, sr, sg, sb);
                }
            } else {
#pragma unroll
                for (int q = 0; q < kPairs; ++q) {
                    if (!__any_sync(kFull, v0[q] | v1[q])) continue;
                    pair_bwd_step<kDA, kMask>(s[q], v0[q], v1[q], m[q], y[q], c, sd, sy, syy, sr, sg, sb, q2.w);
                }
            }
            float g[9];
            g[5] = sd.x + sd.y;
            g[1] = sy.x + sy.y;
            g[4] = syy.x + syy.y;
            g[6] = sr.x + sr.y;
            g[7] = sg.x + sg.y;
            g[8] = sb.x + sb.y;
            g[0] = g[5] * x;
            g[2] = g[0] * x;
            g[3] = g[1] * x;
            // warp totals: lane l ends with the total of value (l >> 2) & 7; g[8] by butterfly
            const float t8 = warp_sum8(g[0], g[1], g[2], g[3], g[4], g[5], g[6], g[7], lane);
            const float t9 = warp_sum(g[8]);
            red_add_shared_if(&acc[k][(lane >> 2) & 7], t8, (lane & 3) == 0);
            red_add_shared_if(&acc[k][8], t9, lane == 0);
          }
        }
        __syncthreads();
        // one global vector reduction per (tile, splat) with a non-zero gradient
        for (int j = threadIdx.x; j < cnt; j += kRenderThreads) {
            float* r = acc[j];
            bool any = false;
#pragma unroll
            for (int c = 0; c < 9; ++c) any |= r[c] != 0.f;
            if (any) {
                // dm = -opacity/2 * dog:  du = -sum dm (2a x + (b+c) y),  dv = -sum dm ((b+c) x + 2d y),
                // d conic a = sum dm x^2,  d conic b = d conic c = sum dm x y,  d conic d = sum dm y^2
                const float4 q0 = s0[j], q1 = s1[j];
                const float hop = -0.5f * q1.z, sbc = q0.w + q1.x;
                const float sx = hop * r[0], sy = hop * r[1];
                const float du = -(2.f * q0.z * sx + sbc * sy);
                const float dv = -(sbc * sx + 2.f * q1.y * sy);
                float* rec = splat_grads + (int64_t)sv[j] * kGradRec;
                red_add_v4(rec, du, dv, hop * r[2], hop * r[3]);
                red_add_v4(rec + 4, hop * r[4], r[5], r[6], r[7]);
                atomicAdd(rec + 8, r[8]);
            }
#pragma unroll
            for (int c = 0; c < 9; ++c) r[c] = 0.f;
        }
    }
}

__device__ __forceinline__ void put(float* base, int64_t off, float v, bool acc) {
    if (acc)
        atomicAdd(base + off, v);
    else
        base[off] = v;
}

// Chain rule from the splat gradient record back to means, quaternions,
// log-scales, opacity logits and SH colour coefficients.
// The gradient rows in the pooled row layout (see slab_rows), stored, not accumulated.
inline bool slab_grad_rows(const gs_gaussian_grads& o) {
    const int64_t S = o.quats_stride;
    return o.quats && o.means && o.scales && o.opac && o.colors && !o.accumulate && !o.colors_by_visible &&
           S % 4 == 0 && kRowColor + o.colors_write <= S && o.means_stride == S && o.scales_stride == S &&
           o.opac_stride == S && o.colors_stride == S && o.means == o.quats + kRowMean &&
           o.opac == o.quats + kRowOpac && o.scales == o.quats + kRowScale && o.colors == o.quats + kRowColor &&
           (reinterpret_cast<uintptr_t>(o.quats) & 15u) == 0;
}

// Degree <= 1 colour (the reference's SH mode): 8 resident CTAs per SM (64
// registers, a few spilled) instead of 4 at 105 registers took the 1 M-Gaussian
// step's projection backward from 0.069 to 0.057 ms; the degree 2-3 kernels
// spill hundreds of bytes at that budget and keep the default.
template <bool kSlabIn, bool kSlabOut, int kDeg>
__global__ void __launch_bounds__(128, kDeg == 1 ? 8 : 1) project_bwd_kernel(gs_gaussians g, const int32_t* __restrict__ ids, int64_t nv,
                                                          RasterParams p, const float* __restrict__ splat_grads,
                                                          gs_gaussian_grads o, float* __restrict__ grad2d,
                                                          float* __restrict__ count) {
    const int64_t vi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vi >= nv) return;
    const int32_t id = ids[vi];
    const int64_t row = param_row(g, id);
    GaussianIn<kDeg> in;
    load_gaussian<kSlabIn>(g, row, g.colors_by_visible ? vi : row, in);
    ProjState s;
    project_one(in, g.colors_dim >= 12, p, s);
    const float* G = splat_grads + vi * kGradRec;
    const float du = G[0], dv = G[1], dca = G[2], dcbc = G[3], dcd = G[4], dop = G[5];
    const float drgb[3] = {G[6], G[7], G[8]};

    // ---- conic = adj(Sigma2) / max(det, 1e-6)
    const float det2 = s.det * s.det;
    const float ddet = (-dca * s.d + dcbc * s.b + dcbc * s.c - dcd * s.a) / det2;
    const float mk = s.det_raw > 1e-6f ? 1.f : 0.f;
    const float dA_ = dcd / s.det + mk * ddet * s.d;
    const float dD_ = dca / s.det + mk * ddet * s.a;
    const float dB_ = -dcbc / s.det - mk * ddet * s.c;
    const float dC_ = -dcbc / s.det - mk * ddet * s.b;

    // ---- Sigma2 = T Sigma3 T^T: dSigma3 = T^T G2 T,  dT = (G2 + G2^T) T Sigma3
    const float G2[4] = {dA_, dB_, dC_, dD_};
    const float* Tm = s.T;
    float dS3[9];
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
        for (int l = 0; l < 3; ++l)
            dS3[3 * k + l] = Tm[k] * (G2[0] * Tm[l] + G2[1] * Tm[3 + l]) + Tm[3 + k] * (G2[2] * Tm[l] + G2[3] * Tm[3 + l]);
    const float Gs00 = 2.f * G2[0], Gs01 = G2[1] + G2[2], Gs11 = 2.f * G2[3];
    float TS[6];  // T Sigma3
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int l = 0; l < 3; ++l)
            TS[3 * i + l] = Tm[3 * i + 0] * s.Sg[0 * 3 + l] + Tm[3 * i + 1] * s.Sg[1 * 3 + l] + Tm[3 * i + 2] * s.Sg[2 * 3 + l];
    float dT[6];
#pragma unroll
    for (int l = 0; l < 3; ++l) {
        dT[l] = Gs00 * TS[l] + Gs01 * TS[3 + l];
        dT[3 + l] = Gs01 * TS[l] + Gs11 * TS[3 + l];
    }
    // ---- T = J W: dJ = dT W^T (only J00, J02, J11, J12 are non-zero)
    const float* W = p.vm;
    const float dJ00 = dT[0] * W[0] + dT[1] * W[1] + dT[2] * W[2];
    const float dJ02 = dT[0] * W[8] + dT[1] * W[9] + dT[2] * W[10];
    const float dJ11 = dT[3] * W[4] + dT[4] * W[5] + dT[5] * W[6];
    const float dJ12 = dT[3] * W[8] + dT[4] * W[9] + dT[5] * W[10];
    const float z = s.z, z2 = z * z, z3 = z2 * z;
    float dtx = dJ02 * (-p.fx / z2) + du * p.fx / z;
    float dty = dJ12 * (-p.fy / z2) + dv * p.fy / z;
    float dz = dJ00 * (-p.fx / z2) + dJ02 * (2.f * p.fx * s.tx / z3) + dJ11 * (-p.fy / z2) +
               dJ12 * (2.f * p.fy * s.ty / z3) - du * p.fx * s.tx / z2 - dv * p.fy * s.ty / z2;
    const float dtz = s.tz > 1e-4f ? dz : 0.f;
    // ---- camera point = W mean + t
    float dm[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) dm[k] = W[0 * 4 + k] * dtx + W[1 * 4 + k] * dty + W[2 * 4 + k] * dtz;

    // ---- Sigma3 = M M^T, M = R diag(S)
    float M[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) M[3 * i + j] = s.R[3 * i + j] * s.S[j];
    float dM[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 3; ++k) acc += (dS3[3 * i + k] + dS3[3 * k + i]) * M[3 * k + j];
            dM[3 * i + j] = acc;
        }
    float dscale[3];
#pragma unroll
    for (int j = 0; j < 3; ++j)
        dscale[j] = (dM[0 * 3 + j] * s.R[0 * 3 + j] + dM[1 * 3 + j] * s.R[1 * 3 + j] + dM[2 * 3 + j] * s.R[2 * 3 + j]) * s.S[j];
    float dR[9];
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) dR[3 * i + j] = dM[3 * i + j] * s.S[j];
    // ---- R(q), q = quat / |quat|
    const float r = s.qw / s.qn, x = s.qx / s.qn, y = s.qy / s.qn, zq = s.qz / s.qn;
    const float dqr = 2.f * (-zq * dR[1] + y * dR[2] + zq * dR[3] - x * dR[5] - y * dR[6] + x * dR[7]);
    const float dqx = 2.f * (y * dR[1] + zq * dR[2] + y * dR[3] - 2.f * x * dR[4] - r * dR[5] + zq * dR[6] + r * dR[7] -
                             2.f * x * dR[8]);
    const float dqy = 2.f * (-2.f * y * dR[0] + x * dR[1] + r * dR[2] + x * dR[3] + zq * dR[5] - r * dR[6] + zq * dR[7] -
                             2.f * y * dR[8]);
    const float dqz = 2.f * (-2.f * zq * dR[0] - r * dR[1] + x * dR[2] + r * dR[3] - 2.f * zq * dR[4] + y * dR[5] +
                             x * dR[6] + y * dR[7]);
    const float qdot = (dqr * s.qw + dqx * s.qx + dqy * s.qy + dqz * s.qz) / (s.qn * s.qn * s.qn);
    float dquat[4] = {dqr / s.qn - s.qw * qdot, dqx / s.qn - s.qx * qdot, dqy / s.qn - s.qy * qdot,
                      dqz / s.qn - s.qz * qdot};

    // ---- opacity
    const float dlogit = dop * s.opac * (1.f - s.opac);

    // ---- colour: clip mask, SH0, SH1 (and degrees 2-3) and the direction's dependence on the mean
    constexpr int NC = ShRow<kDeg>::kCols, KC = ShRow<kDeg>::kPerCh;
    float dpre[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) dpre[k] = (s.pre[k] > 0.f && s.pre[k] < 1.f) ? drgb[k] : 0.f;
    float dcol[NC];
#pragma unroll
    for (int k = 0; k < 3; ++k) dcol[k] = dpre[k] * kSH_C0;
    const bool sh1 = kDeg > 1 || g.colors_dim >= 12;
    if (sh1) {
        const float xd = s.dir[0], yd = s.dir[1], zd = s.dir[2];
        float ddir[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            const float e = kSH_C1 * dpre[ch];
            const int c0 = 3 + KC * ch;
            dcol[c0 + 0] = e * yd;
            dcol[c0 + 1] = e * zd;
            dcol[c0 + 2] = e * xd;
            ddir[1] += e * in.col[c0 + 0];
            ddir[2] += e * in.col[c0 + 1];
            ddir[0] += e * in.col[c0 + 2];
        }
        if (kDeg > 1) {
            float b[12], w[12];
            sh_basis_hi<kDeg>(xd, yd, zd, b);
#pragma unroll
            for (int j = 0; j < KC - 3; ++j) {
                w[j] = 0.f;
#pragma unroll
                for (int ch = 0; ch < 3; ++ch) {
                    dcol[3 + KC * ch + 3 + j] = dpre[ch] * b[j];
                    w[j] += dpre[ch] * in.col[3 + KC * ch + 3 + j];
                }
            }
            float gx, gy, gz;
            sh_basis_hi_grad<kDeg>(xd, yd, zd, w, gx, gy, gz);
            ddir[0] += gx;
            ddir[1] += gy;
            ddir[2] += gz;
        }
        const float n = s.dnorm, ne = n + 1e-8f;
        const float dx = s.mx - p.campos[0], dy = s.my - p.campos[1], dzz = s.mz - p.campos[2];
        const float proj = (ddir[0] * dx + ddir[1] * dy + ddir[2] * dzz) / (n * ne * ne);
        dm[0] += ddir[0] / ne - dx * proj;
        dm[1] += ddir[1] / ne - dy * proj;
        dm[2] += ddir[2] / ne - dzz * proj;
    } else {
#pragma unroll
        for (int k = 3; k < NC; ++k) dcol[k] = 0.f;
    }

    // ---- outputs
    const bool acc = o.accumulate != 0;
    const float reg = o.reg;
    // written geometry gradients carry ``reg`` unless the caller adds it later;
    // the densification statistic below always uses the full mean gradient
    const float reg_geo = o.reg_geometry ? reg : 0.f;
    float dmw[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        dmw[k] = dm[k] + reg_geo;
        dm[k] += reg;
    }
    if (kSlabOut) {
        // the row's first kVals columns from registers, 16 bytes at a time; the
        // colour columns past the evaluated degree hold only the regulariser
        constexpr int kVals = (kRowColor + NC + 1 + 3) / 4 * 4;
        float vals[kVals];
#pragma unroll
        for (int k = 0; k < 4; ++k) vals[k] = dquat[k] + reg_geo;
#pragma unroll
        for (int k = 0; k < 3; ++k) vals[kRowMean + k] = dmw[k];
        vals[kRowOpac] = dlogit + reg_geo;
#pragma unroll
        for (int k = 0; k < 3; ++k) vals[kRowScale + k] = dscale[k] + reg_geo;
#pragma unroll
        for (int k = 0; k < kVals - kRowColor; ++k)
            vals[kRowColor + k] = (k < NC ? dcol[k] : 0.f) + (k < o.reg_color_cols ? reg : 0.f);
        // the view count column (narrow gradient rows summed over GPUs)
        const int cc = o.count_col;
#pragma unroll
        for (int k = 0; k < kVals; ++k)
            if (cc > 0 && k == cc) vals[k] = 1.0f;
        float* rowp = o.quats + (int64_t)id * o.quats_stride;
        const int W = max(kRowColor + o.colors_write, cc + 1);
#pragma unroll
        for (int j = 0; j < kVals / 4; ++j) {
            if (4 * j + 3 < W) {
                reinterpret_cast<float4*>(rowp)[j] = make_float4(vals[4 * j], vals[4 * j + 1], vals[4 * j + 2],
                                                                 vals[4 * j + 3]);
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    if (4 * j + c < W) rowp[4 * j + c] = vals[4 * j + c];
            }
        }
        for (int c = kVals; c < W; c += 4) {
            float t[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                t[u] = cc > 0 && c + u == cc ? 1.0f : (c + u - kRowColor < o.reg_color_cols ? reg : 0.f);
            if (c + 3 < W) {
                reinterpret_cast<float4*>(rowp + c)[0] = make_float4(t[0], t[1], t[2], t[3]);
            } else {
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (c + u < W) rowp[c + u] = t[u];
            }
        }
    }
    if (!kSlabOut && o.means) {
#pragma unroll
        for (int k = 0; k < 3; ++k) put(o.means, (int64_t)id * o.means_stride + k, dmw[k], acc);
    }
    if (!kSlabOut && o.quats) {
#pragma unroll
        for (int k = 0; k < 4; ++k) put(o.quats, (int64_t)id * o.quats_stride + k, dquat[k] + reg_geo, acc);
    }
    if (!kSlabOut && o.scales) {
#pragma unroll
        for (int k = 0; k < 3; ++k) put(o.scales, (int64_t)id * o.scales_stride + k, dscale[k] + reg_geo, acc);
    }
    if (!kSlabOut && o.opac) put(o.opac, (int64_t)id * o.opac_stride, dlogit + reg_geo, acc);
    if (!kSlabOut && o.colors) {
        const int64_t orow = o.colors_by_visible ? vi : (int64_t)id;
        float* dst = o.colors + orow * o.colors_stride;
        for (int k = 0; k < o.colors_write; ++k) {
            float val = 0.f;
#pragma unroll
            for (int j = 0; j < NC; ++j)  // register-resident select instead of a dynamic index
                if (j == k) val = dcol[j];
            if (k < o.reg_color_cols) val += reg;
            put(dst, k, val, acc);
        }
    }
    if (grad2d) {
        const int64_t prow = param_row(g, id);
        const float gn = sqrtf(dm[0] * dm[0] + dm[1] * dm[1] + dm[2] * dm[2] + 1e-8f);
        atomicAdd(grad2d + prow, gn * fabsf(s.tz) / p.fx);
        atomicAdd(count + prow, 1.0f);
    }
}

}  // namespace gs

using namespace gs;

extern "C" int gs_render_backward(const gs_tile_range* ranges, const int32_t* tile_order, const uint32_t* entry_vals,
                                  const float* splats,
                                  int64_t num_visible, const gs_camera* cam, const gs_raster_settings* rs,
                                  const float* out_color,
                                  const float* final_T, const int32_t* n_contrib, int loss_mode, const void* target,
                                  const float* dL_dcolor, const float* dL_dalpha, float* splat_grads,
                                  gs_stream_t stream) {
    GS_REQUIRE(cam && ranges && final_T && n_contrib && splat_grads, "render_backward: null pointer");
    GS_REQUIRE(loss_mode >= GS_LOSS_NONE && loss_mode <= GS_LOSS_MEAN, "render_backward: bad loss mode");
    GS_REQUIRE(!rs || rs->transmittance_min <= 1.f, "render_backward: transmittance_min must be <= 1");
    GS_REQUIRE(loss_mode != GS_LOSS_NONE || dL_dcolor, "render_backward: dL_dcolor required");
    GS_REQUIRE(loss_mode == GS_LOSS_NONE || loss_mode == GS_LOSS_MEAN || (target && out_color),
               "render_backward: target and out_color required");
    GS_REQUIRE(aligned16(splat_grads) && aligned16(splats), "render_backward: records must be 16-byte aligned");
    const RasterParams p = make_raster_params(*cam, rs);
    const int tiles = p.tiles_x * p.tiles_y;
    // the alpha cotangent is carried per pixel only when the caller passes one
    const bool da = loss_mode == GS_LOSS_NONE && dL_dalpha;
    // fewer tiles than one wave of 4-pixel CTAs: the 2-pixel layout
    const bool px2 = tiles < sm_count() * kBwdMinCtas4;
#define GS_RBWD(P)                                                                                        \
    (p.masked ? (da ? render_bwd_kernel<P, true, true> : render_bwd_kernel<P, false, true>)             \
              : (da ? render_bwd_kernel<P, true, false> : render_bwd_kernel<P, false, false>))
    auto kernel = px2 ? GS_RBWD(2) : GS_RBWD(4);
#undef GS_RBWD
    const int threads = px2 ? BwdLayout<2>::threads : BwdLayout<4>::threads;
    kernel<<<tiles, threads, 0, (cudaStream_t)stream>>>(
        ranges, tile_order, entry_vals, reinterpret_cast<const float4*>(splats), num_visible, p, out_color, final_T,
        n_contrib, loss_mode, target, dL_dcolor, dL_dalpha, splat_grads);
    return check_launch("render_bwd_kernel");
}

extern "C" int gs_project_backward(const gs_gaussians* g, const int32_t* ids, int64_t num_visible,
                                   const gs_camera* cam, const float* splat_grads, const gs_gaussian_grads* out,
                                   float* grad2d, float* count, gs_stream_t stream) {
    GS_REQUIRE(g && cam && out, "project_backward: null descriptor");
    if (num_visible == 0) return GS_OK;
    GS_REQUIRE(ids && splat_grads, "project_backward: null pointer");
    GS_REQUIRE(!grad2d || count, "project_backward: grad2d needs count");
    GS_REQUIRE(out->colors == nullptr || out->colors_write >= 0, "project_backward: bad colors_write");
    GS_REQUIRE(out->count_col <= 0 || (slab_grad_rows(*out) && out->count_col < out->quats_stride &&
                                       out->count_col >= kRowColor + out->colors_write),
               "project_backward: a count column needs pooled gradient rows with room past the colours");
    const RasterParams p = make_raster_params(*cam, nullptr);
    GS_REQUIRE(g->sh_mode == GS_SH_REFERENCE || g->sh_mode == GS_SH_FULL, "project_backward: bad sh_mode");
    const int deg = sh_kernel_degree(*g);
    const bool out_rows = slab_grad_rows(*out);
    const bool in_rows = deg == 3 ? slab_rows<3>(*g) : deg == 2 ? slab_rows<2>(*g) : slab_rows<1>(*g);
#define GS_PBWD(D)                                                                                   \
    (in_rows ? (out_rows ? project_bwd_kernel<true, true, D> : project_bwd_kernel<true, false, D>) \
             : (out_rows ? project_bwd_kernel<false, true, D> : project_bwd_kernel<false, false, D>))
    auto kernel = deg == 3 ? GS_PBWD(3) : deg == 2 ? GS_PBWD(2) : GS_PBWD(1);
#undef GS_PBWD
    kernel<<<grid_for(num_visible, 128), 128, 0, (cudaStream_t)stream>>>(*g, ids, num_visible, p, splat_grads, *out,
                                                                         grad2d, count);
    return check_launch("project_bwd_kernel");
}
