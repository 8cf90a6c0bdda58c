// Fused Adam over pooled parameter/moment buffers (replaces the Metal kernel
// fused_adam_step, src/mlx_extensions.cpp:102-152, and the pure-MLX step,
// mlx_gsplat/optimizer.py:146-175).
//
// Every element update is written with round-to-nearest intrinsics and no
// fused multiply-add, in the reference kernel's operation order, so that the
// result matches the CPU restatement bit for bit.  The slab kernel moves one
// float4 of theta, m, v and g per thread (16-byte loads and stores), covering
// all parameter groups of a pooled row in a single launch.
#include <math.h>

#include "common.cuh"

namespace gs {

struct AdamScalars {
    float b1, b2, omb1, omb2;  // beta, (1 - beta) as the selected semantics round them
    float eps, wd, sqrt_bc2, grad_scale;
    float inv_sqrt_bc2;        // 1 / sqrt(1 - beta2^t) for the approximate step
    int scrub, clamp;
    int has_bias;              // slab: add the per-column gradient bias before scaling
};

constexpr int kMaxSlabCols = 64;
struct SlabCols {
    float step_size[kMaxSlabCols];
    float lo[kMaxSlabCols];
    float hi[kMaxSlabCols];
    float gdef[kMaxSlabCols];  // gradient of a row the visibility bits mark unseen
    float gbias[kMaxSlabCols]; // added to every row's gradient before the scale
    float gcoef[kMaxSlabCols]; // narrow gradient rows: column c >= g_cols is count * gcoef[c]
};

__device__ __forceinline__ void adam_elem(float& th, float& m, float& v, float g, const AdamScalars& s,
                                          float step_size, float lo, float hi) {
    g = __fmul_rn(g, s.grad_scale);
    if (s.scrub && isnan(g)) g = 0.0f;
    if (s.wd != 0.0f) g = __fadd_rn(g, __fmul_rn(s.wd, th));
    float mn = __fadd_rn(__fmul_rn(s.b1, m), __fmul_rn(s.omb1, g));
    float vn = __fadd_rn(__fmul_rn(s.b2, v), __fmul_rn(s.omb2, __fmul_rn(g, g)));
    if (s.scrub) {
        if (!isfinite(mn)) mn = 0.0f;
        if (!isfinite(vn)) vn = 0.0f;
    }
    const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vn), s.sqrt_bc2), s.eps);
    float delta = __fmul_rn(step_size, __fdiv_rn(mn, denom));
    if (s.scrub && !isfinite(delta)) delta = 0.0f;
    float t = __fsub_rn(th, delta);
    if (s.clamp) t = fminf(fmaxf(t, lo), hi);
    th = t;
    m = mn;
    v = vn;
}

// The same update with the moments rounded exactly as above and the step
// formed with the hardware square root and reciprocal (sqrt.approx,
// rcp.approx: a few ulp on the step, none on m and v) and without branches.
// kFused selects the fused kernel's scrub-and-clamp semantics.
__device__ __forceinline__ float approx_sqrt(float x) {
    float y;
    asm("sqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float approx_rcp(float x) {
    float y;
    asm("rcp.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float approx_rsqrt(float x) {
    float y;
    asm("rsqrt.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <bool kFused>
__device__ __forceinline__ void adam_elem_fast(float& th, float& m, float& v, float g, const AdamScalars& s,
                                               float step_size, float lo, float hi) {
    g = __fmul_rn(g, s.grad_scale);
    if (kFused) g = isnan(g) ? 0.0f : g;
    if (s.wd != 0.0f) g = __fadd_rn(g, __fmul_rn(s.wd, th));
    float mn = __fadd_rn(__fmul_rn(s.b1, m), __fmul_rn(s.omb1, g));
    float vn = __fadd_rn(__fmul_rn(s.b2, v), __fmul_rn(s.omb2, __fmul_rn(g, g)));
    if (kFused) {
        mn = isfinite(mn) ? mn : 0.0f;
        vn = isfinite(vn) ? vn : 0.0f;
    }
    const float denom = fmaf(approx_sqrt(vn), s.inv_sqrt_bc2, s.eps);
    float delta = step_size * (mn * approx_rcp(denom));
    if (kFused) delta = isfinite(delta) ? delta : 0.0f;
    float t = th - delta;
    if (kFused) t = fminf(fmaxf(t, lo), hi);
    th = t;
    m = mn;
    v = vn;
}

// One thread per (active row, column) element, as the reference dispatches it.
__global__ void adam_group_kernel(float* __restrict__ theta, const float* __restrict__ g, float* __restrict__ m,
                                  float* __restrict__ v, const int32_t* __restrict__ idx, int64_t n_elems, int dim,
                                  int64_t pool_stride, int64_t g_stride, AdamScalars s, float step_size, float lo,
                                  float hi) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n_elems) return;
    const int64_t r = t / dim;
    const int c = (int)(t - r * dim);
    const int64_t p = (int64_t)__ldg(idx + r) * pool_stride + c;
    float th = theta[p], mm = m[p], vv = v[p];
    adam_elem(th, mm, vv, __ldg(g + r * g_stride + c), s, step_size, lo, hi);
    theta[p] = th;
    m[p] = mm;
    v[p] = vv;
}

// One float4 chunk of a pooled row per work item; 2^lane_shift consecutive
// items own one row (the smallest power of two >= the row's chunk count).
// Each thread takes two items, ``half`` apart, and issues all eight 16-byte
// loads before any arithmetic so that more bytes are in flight per thread.
// Per-column constants live in shared memory: indexing the kernel-parameter
// copy with a lane-dependent column made every access a divergent constant
// load (serialised in the address-divergence unit).
struct __align__(16) ColsSmem {
    float step[kMaxSlabCols], lo[kMaxSlabCols], hi[kMaxSlabCols], gdef[kMaxSlabCols], gbias[kMaxSlabCols],
        gcoef[kMaxSlabCols];
};

// A seen row's gradient chunk c4 from a narrow gradient row: columns below
// g_cols as loaded, the others rebuilt as count * gcoef[c].
__device__ __forceinline__ float4 narrow_grad(float4 g, int c4, int g_cols, float count, const ColsSmem& cs) {
    const int c = 4 * c4;
    g.x = c + 0 < g_cols ? g.x : count * cs.gcoef[c + 0];
    g.y = c + 1 < g_cols ? g.y : count * cs.gcoef[c + 1];
    g.z = c + 2 < g_cols ? g.z : count * cs.gcoef[c + 2];
    g.w = c + 3 < g_cols ? g.w : count * cs.gcoef[c + 3];
    return g;
}

template <bool kExact, bool kFused>
__device__ __forceinline__ void slab_elem(float& th, float& m, float& v, float g, int c, int ncols,
                                          const AdamScalars& s, const ColsSmem& cs) {
    if (s.has_bias) g = __fadd_rn(g, cs.gbias[c]);
    if (kExact) {
        if (c < ncols) adam_elem(th, m, v, g, s, cs.step[c], cs.lo[c], cs.hi[c]);
    } else {
        // padding columns are computed and then discarded (no branch)
        float t = th, mn = m, vn = v;
        adam_elem_fast<kFused>(t, mn, vn, g, s, cs.step[c], cs.lo[c], cs.hi[c]);
        const bool on = c < ncols;
        th = on ? t : th;
        m = on ? mn : m;
        v = on ? vn : v;
    }
}

template <bool kExact, bool kFused>
__device__ __forceinline__ void slab_update(float4& th, float4& mm, float4& vv, const float4& gg, int c0, int ncols,
                                            bool renorm, const AdamScalars& s, const ColsSmem& cs) {
    slab_elem<kExact, kFused>(th.x, mm.x, vv.x, gg.x, c0 + 0, ncols, s, cs);
    slab_elem<kExact, kFused>(th.y, mm.y, vv.y, gg.y, c0 + 1, ncols, s, cs);
    slab_elem<kExact, kFused>(th.z, mm.z, vv.z, gg.z, c0 + 2, ncols, s, cs);
    slab_elem<kExact, kFused>(th.w, mm.w, vv.w, gg.w, c0 + 3, ncols, s, cs);
    if (!kExact && renorm) {
        const float r = approx_rsqrt(th.x * th.x + th.y * th.y + th.z * th.z + th.w * th.w + 1e-8f);
        th.x *= r;
        th.y *= r;
        th.z *= r;
        th.w *= r;
    } else if (renorm) {
        float ss = __fmul_rn(th.x, th.x);
        ss = __fadd_rn(ss, __fmul_rn(th.y, th.y));
        ss = __fadd_rn(ss, __fmul_rn(th.z, th.z));
        ss = __fadd_rn(ss, __fmul_rn(th.w, th.w));
        const float n = __fsqrt_rn(__fadd_rn(ss, 1e-8f));
        th.x = __fdiv_rn(th.x, n);
        th.y = __fdiv_rn(th.y, n);
        th.z = __fdiv_rn(th.z, n);
        th.w = __fdiv_rn(th.w, n);
    }
}

__device__ __forceinline__ float float4_comp(const float4& v, int k) {
    return k == 0 ? v.x : (k == 1 ? v.y : (k == 2 ? v.z : v.w));
}

// kNarrow: gradient rows hold only columns [0, g_cols) and a view count at
// count_col; the lane of a row whose chunk holds the count broadcasts it to the
// row's other lanes (one shuffle), and columns from g_cols on are rebuilt as
// count * gcoef[c].  Every lane stays in the kernel until after the shuffle.
template <bool kExact, bool kFused, bool kNarrow>
__global__ void __launch_bounds__(256, 4) adam_slab_kernel(float4* __restrict__ theta, const float4* __restrict__ g,
                                                        float4* __restrict__ m, float4* __restrict__ v,
                                                        const int32_t* __restrict__ idx, int64_t n_rows, int chunks,
                                                        int lane_shift, int g_chunks, int ncols, int quat_chunk,
                                                        int64_t half, const uint32_t* __restrict__ vis,
                                                        int g_cols, int count_col, int row_select, AdamScalars s,
                                                        SlabCols cols) {
    __shared__ ColsSmem cs;
    if (threadIdx.x < kMaxSlabCols) {
        cs.step[threadIdx.x] = cols.step_size[threadIdx.x];
        cs.lo[threadIdx.x] = cols.lo[threadIdx.x];
        cs.hi[threadIdx.x] = cols.hi[threadIdx.x];
        cs.gdef[threadIdx.x] = cols.gdef[threadIdx.x];
        cs.gbias[threadIdx.x] = cols.gbias[threadIdx.x];
        cs.gcoef[threadIdx.x] = cols.gcoef[threadIdx.x];
    }
    __syncthreads();
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int mask = (1 << lane_shift) - 1;
    const int c4 = (int)(t0 & mask);  // half is a multiple of 2^lane_shift: both items share the chunk
    const bool live = c4 < chunks && 4 * c4 < ncols;
    if (!kNarrow && !live) return;
    const int64_t ra = t0 >> lane_shift, rb = (t0 + half) >> lane_shift;
    bool va = live && ra < n_rows, vb = live && rb < n_rows;
    // Two dependency levels, each issued for both items before anything waits:
    // the indirection entries and visibility words, then every data load.
    int64_t offa = 0, offb = 0;
    uint32_t wa = ~0u, wb = ~0u;
    if (va) {
        offa = (int64_t)__ldg(idx + ra) * chunks + c4;
        if (vis) wa = __ldg(vis + (ra >> 5));
    }
    if (vb) {
        offb = (int64_t)__ldg(idx + rb) * chunks + c4;
        if (vis) wb = __ldg(vis + (rb >> 5));
    }
    bool ga_seen = va && ((wa >> (ra & 31)) & 1u), gb_seen = vb && ((wb >> (rb & 31)) & 1u);
    if (row_select != GS_ROWS_ALL) {
        // a row outside the selected set is neither read nor written
        const bool want_seen = row_select == GS_ROWS_SEEN;
        va = va && (((wa >> (ra & 31)) & 1u) != 0) == want_seen;
        vb = vb && (((wb >> (rb & 31)) & 1u) != 0) == want_seen;
        ga_seen = ga_seen && va;
        gb_seen = gb_seen && vb;
    }
    const float4 gdef = reinterpret_cast<const float4*>(cs.gdef)[min(c4, kMaxSlabCols / 4 - 1)];
    float4 tha = gdef, ma = gdef, vva = gdef, ga = gdef, thb = gdef, mb = gdef, vvb = gdef, gb = gdef;
    if (va) {
        tha = __ldcs(theta + offa);
        ma = __ldcs(m + offa);
        vva = __ldcs(v + offa);
    }
    if (vb) {
        thb = __ldcs(theta + offb);
        mb = __ldcs(m + offb);
        vvb = __ldcs(v + offb);
    }
    const bool load_g = !kNarrow || 4 * c4 < g_cols || c4 == (count_col >> 2);
    if (ga_seen && load_g) ga = __ldcs(g + ra * g_chunks + c4);
    if (gb_seen && load_g) gb = __ldcs(g + rb * g_chunks + c4);
    if (kNarrow) {
        const int src = count_col >> 2, k = count_col & 3, width = 1 << lane_shift;
        const float cnt_a = __shfl_sync(kFull, float4_comp(ga, k), src, width);
        const float cnt_b = __shfl_sync(kFull, float4_comp(gb, k), src, width);
        if (!live) return;
        if (4 * c4 + 3 >= g_cols) {
            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ga_seen) ga = narrow_grad(4 * c4 < g_cols ? ga : z, c4, g_cols, cnt_a, cs);
            if (gb_seen) gb = narrow_grad(4 * c4 < g_cols ? gb : z, c4, g_cols, cnt_b, cs);
        }
    }
    const bool renorm = c4 == quat_chunk;
    if (va) {
        slab_update<kExact, kFused>(tha, ma, vva, ga, 4 * c4, ncols, renorm, s, cs);
        __stcs(theta + offa, tha);
        __stcs(m + offa, ma);
        __stcs(v + offa, vva);
    }
    if (vb) {
        slab_update<kExact, kFused>(thb, mb, vvb, gb, 4 * c4, ncols, renorm, s, cs);
        __stcs(theta + offb, thb);
        __stcs(m + offb, mb);
        __stcs(v + offb, vvb);
    }
}

// ---------------------------------------------------------------- sharded multi-GPU Adam
// The slab Adam of one GPU of a views-data-parallel group, fused with the
// group's gradient sum and parameter broadcast over NVLink multicast: the GPU
// updates only the rows whose physical slot it owns (slot % world == rank).
// For such a row it loads the gradient row summed across every GPU's copy
// (multimem.ld_reduce: the switch adds them), updates theta, m and v in its own
// memory, and stores the first ``hot_chunks`` 16-byte chunks of the new theta
// row to every GPU's copy (multimem.st) — the columns the rasterizer reads each
// step; the other columns and the moments stay with the owner until the caller
// consolidates them.  Gradient rows are indexed by active id, theta/m/v rows by
// physical slot.  Semantics: the fused kernel's (scrub and clamp) with the
// approximate step, as adam_slab_kernel<false, true, .>.
__device__ __forceinline__ float4 mc_ld_reduce(const float4* p) {
    float4 r;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}

__device__ __forceinline__ void mc_st(float4* p, const float4& r) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(r.x), "f"(r.y),
                 "f"(r.z), "f"(r.w)
                 : "memory");
}

template <bool kNarrow>
__global__ void __launch_bounds__(256, 4) adam_sharded_kernel(
    float4* __restrict__ theta, float4* __restrict__ theta_mc, const float4* __restrict__ g_mc,
    float4* __restrict__ m, float4* __restrict__ v, const int32_t* __restrict__ idx, int64_t n_rows, int chunks,
    int lane_shift, int g_chunks, int ncols, int quat_chunk, int64_t half, int g_cols, int count_col, int rank,
    int world, int hot_chunks, const int32_t* __restrict__ error_flag, AdamScalars s, SlabCols cols) {
    // a group barrier before this launch gave up waiting for a peer: the
    // summed rows may be partial, so nothing is read or written (uniform
    // over the grid: the flag is written only by kernels ordered before this one)
    if (error_flag && *reinterpret_cast<const volatile int32_t*>(error_flag) != 0) return;
    __shared__ ColsSmem cs;
    if (threadIdx.x < kMaxSlabCols) {
        cs.step[threadIdx.x] = cols.step_size[threadIdx.x];
        cs.lo[threadIdx.x] = cols.lo[threadIdx.x];
        cs.hi[threadIdx.x] = cols.hi[threadIdx.x];
        cs.gdef[threadIdx.x] = cols.gdef[threadIdx.x];
        cs.gbias[threadIdx.x] = cols.gbias[threadIdx.x];
        cs.gcoef[threadIdx.x] = cols.gcoef[threadIdx.x];
    }
    __syncthreads();
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int c4 = (int)(t0 & ((1 << lane_shift) - 1));
    const bool live = c4 < chunks && 4 * c4 < ncols;
    const int64_t ra = t0 >> lane_shift, rb = (t0 + half) >> lane_shift;
    int64_t sa = 0, sb = 0;
    bool va = live && ra < n_rows, vb = live && rb < n_rows;
    if (va) sa = __ldg(idx + ra);
    if (vb) sb = __ldg(idx + rb);
    va = va && (sa % world) == rank;
    vb = vb && (sb % world) == rank;
    const int64_t offa = sa * chunks + c4, offb = sb * chunks + c4;
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 tha = z, ma = z, vva = z, ga = z, thb = z, mb = z, vvb = z, gb = z;
    const bool load_g = !kNarrow || 4 * c4 < g_cols || c4 == (count_col >> 2);
    if (va) {
        tha = __ldcs(theta + offa);
        ma = __ldcs(m + offa);
        vva = __ldcs(v + offa);
        if (load_g) ga = mc_ld_reduce(g_mc + ra * g_chunks + c4);
    }
    if (vb) {
        thb = __ldcs(theta + offb);
        mb = __ldcs(m + offb);
        vvb = __ldcs(v + offb);
        if (load_g) gb = mc_ld_reduce(g_mc + rb * g_chunks + c4);
    }
    if (kNarrow) {
        // the summed view count of the row, from the lane whose chunk holds it
        const int src = count_col >> 2, k = count_col & 3, width = 1 << lane_shift;
        const float cnt_a = __shfl_sync(kFull, float4_comp(ga, k), src, width);
        const float cnt_b = __shfl_sync(kFull, float4_comp(gb, k), src, width);
        if (4 * c4 + 3 >= g_cols) {
            if (va) ga = narrow_grad(4 * c4 < g_cols ? ga : z, c4, g_cols, cnt_a, cs);
            if (vb) gb = narrow_grad(4 * c4 < g_cols ? gb : z, c4, g_cols, cnt_b, cs);
        }
    }
    const bool renorm = c4 == quat_chunk, hot = c4 < hot_chunks;
    if (va) {
        slab_update<false, true>(tha, ma, vva, ga, 4 * c4, ncols, renorm, s, cs);
        __stcs(m + offa, ma);
        __stcs(v + offa, vva);
        if (hot)
            mc_st(theta_mc + offa, tha);
        else
            __stcs(theta + offa, tha);
    }
    if (vb) {
        slab_update<false, true>(thb, mb, vvb, gb, 4 * c4, ncols, renorm, s, cs);
        __stcs(m + offb, mb);
        __stcs(v + offb, vvb);
        if (hot)
            mc_st(theta_mc + offb, thb);
        else
            __stcs(theta + offb, thb);
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");  // publish before the group's barrier
}

// Host-side scalars for each semantics.  ``lr``/``beta1``/``beta2`` arrive in
// float64 (the Python values): the fused mode rounds them to float32 first, as
// the Metal kernel receives them (src/mlx_extensions.cpp:259-263); the pure
// mode forms 1 - beta and the bias corrections in float64 and rounds each
// scalar once, as MLX does with Python floats (optimizer.py:75-76, 162-167).
static AdamScalars make_scalars(int mode, double beta1, double beta2, float eps, float wd, int step,
                                float grad_scale, double* bc1_out) {
    AdamScalars s;
    s.b1 = (float)beta1;
    s.b2 = (float)beta2;
    s.eps = eps;
    s.wd = wd;
    s.grad_scale = grad_scale;
    s.has_bias = 0;
    if (mode == GS_ADAM_FUSED) {
        const float b1 = (float)beta1, b2 = (float)beta2;
        s.omb1 = 1.0f - b1;
        s.omb2 = 1.0f - b2;
        const float bc1 = 1.0f - powf(b1, (float)step);
        const float bc2 = 1.0f - powf(b2, (float)step);
        s.sqrt_bc2 = sqrtf(bc2);
        s.inv_sqrt_bc2 = 1.0f / s.sqrt_bc2;
        *bc1_out = bc1;
        s.scrub = 1;
        s.clamp = 1;
    } else {
        s.omb1 = (float)(1.0 - beta1);
        s.omb2 = (float)(1.0 - beta2);
        const double bc1 = 1.0 - pow(beta1, (double)step);
        const double bc2 = 1.0 - pow(beta2, (double)step);
        s.sqrt_bc2 = (float)sqrt(bc2);
        s.inv_sqrt_bc2 = (float)(1.0 / sqrt(bc2));
        *bc1_out = bc1;
        s.scrub = 0;
        s.clamp = 0;
    }
    return s;
}

static float step_size_for(int mode, double lr, double lr_scale, double bc1) {
    if (mode == GS_ADAM_FUSED) return (float)lr / (float)bc1;  // float32 division, no lr_scales
    return (float)((lr * lr_scale) / bc1);
}

}  // namespace gs

using namespace gs;

extern "C" int gs_fused_adam_group(float* theta, const float* g, float* m, float* v, const int32_t* indices,
                                   int64_t num_active, int dim, int64_t pool_stride, int64_t g_stride, double lr,
                                   double beta1, double beta2, float eps, float weight_decay, int step, float a_min,
                                   float a_max, float lr_scale, float grad_scale, int mode, gs_stream_t stream) {
    GS_REQUIRE(mode == GS_ADAM_FUSED || mode == GS_ADAM_PURE, "adam: unknown mode %d", mode);
    GS_REQUIRE(num_active >= 0 && dim > 0 && step >= 1, "adam: bad sizes (num_active=%lld dim=%d step=%d)",
               (long long)num_active, dim, step);
    if (num_active == 0) return GS_OK;
    GS_REQUIRE(theta && g && m && v && indices, "adam: null pointer");
    GS_REQUIRE(pool_stride >= dim && g_stride >= dim, "adam: stride smaller than dim");
    double bc1;
    AdamScalars s = make_scalars(mode, beta1, beta2, eps, weight_decay, step, grad_scale, &bc1);
    const float ss = step_size_for(mode, lr, lr_scale, bc1);
    const int64_t n = num_active * (int64_t)dim;
    adam_group_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(theta, g, m, v, indices, n, dim,
                                                                          pool_stride, g_stride, s, ss, a_min, a_max);
    return check_launch("adam_group_kernel");
}

extern "C" int gs_fused_adam_slab(float* theta, const float* g, float* m, float* v, const int32_t* indices,
                                  int64_t num_active, int ncols, int64_t stride, int64_t g_stride,
                                  const float* col_lo, const float* col_hi, const float* col_lr_scale, int quat_col,
                                  double lr, double beta1, double beta2, float eps, float weight_decay, int step,
                                  float grad_scale, int mode, const uint32_t* visible_words,
                                  const float* unseen_grad_host, const float* grad_bias_host, int g_cols,
                                  int count_col, const float* count_coef_host, int row_select,
                                  gs_stream_t stream) {
    const bool exact = (mode & GS_ADAM_EXACT) != 0;
    mode &= ~GS_ADAM_EXACT;
    GS_REQUIRE(mode == GS_ADAM_FUSED || mode == GS_ADAM_PURE, "adam_slab: unknown mode %d", mode);
    GS_REQUIRE(!visible_words || unseen_grad_host, "adam_slab: visible_words needs unseen_grad_host");
    GS_REQUIRE(ncols > 0 && ncols <= kMaxSlabCols, "adam_slab: ncols must be in [1, %d]", kMaxSlabCols);
    GS_REQUIRE(g_cols > 0 && g_cols <= ncols, "adam_slab: g_cols must be in [1, ncols]");
    GS_REQUIRE(row_select >= GS_ROWS_ALL && row_select <= GS_ROWS_UNSEEN, "adam_slab: bad row_select");
    GS_REQUIRE(row_select == GS_ROWS_ALL || visible_words, "adam_slab: row_select needs visible_words");
    GS_REQUIRE(stride % 4 == 0 && g_stride % 4 == 0 && stride >= ncols && g_stride >= g_cols,
               "adam_slab: strides must be multiples of 4, stride >= ncols and g_stride >= g_cols");
    GS_REQUIRE(g_cols == ncols || (count_coef_host && count_col >= g_cols && count_col < g_stride &&
                                   count_col < stride && (count_col & ~3) < ncols && stride <= 128),
               "adam_slab: narrow gradient rows need count_coef_host, a count column in [g_cols, g_stride) "
               "inside a parameter chunk, and stride <= 128");
    GS_REQUIRE(step >= 1 && num_active >= 0, "adam_slab: bad step/num_active");
    GS_REQUIRE(quat_col < 0 || (quat_col % 4 == 0 && quat_col + 4 <= ncols), "adam_slab: bad quat_col");
    if (num_active == 0) return GS_OK;
    GS_REQUIRE(theta && g && m && v && indices && col_lo && col_hi, "adam_slab: null pointer");
    GS_REQUIRE(aligned16(theta) && aligned16(g) && aligned16(m) && aligned16(v), "adam_slab: bases must be 16-byte aligned");
    double bc1;
    AdamScalars s = make_scalars(mode, beta1, beta2, eps, weight_decay, step, grad_scale, &bc1);
    SlabCols cols;
    for (int c = 0; c < kMaxSlabCols; ++c) {
        const bool on = c < ncols;
        cols.lo[c] = on ? col_lo[c] : 0.f;
        cols.hi[c] = on ? col_hi[c] : 0.f;
        cols.step_size[c] = on ? step_size_for(mode, lr, col_lr_scale ? col_lr_scale[c] : 1.0f, bc1) : 0.f;
        cols.gdef[c] = (on && unseen_grad_host) ? unseen_grad_host[c] : 0.f;
        cols.gbias[c] = (on && grad_bias_host) ? grad_bias_host[c] : 0.f;
        cols.gcoef[c] = (on && c >= g_cols) ? count_coef_host[c] : 0.f;
    }
    s.has_bias = grad_bias_host != nullptr;
    const int chunks = (int)(stride / 4);
    int shift = 0;
    while ((1 << shift) < chunks) ++shift;
    // two items per thread: the second half of the items starts ``half`` (a
    // multiple of 256, hence of 2^shift) after the first
    const int64_t n = num_active << shift;
    const int64_t half = (n + 511) / 512 * 256;
    const bool narrow = g_cols < ncols;
#define GS_ADAM_SLAB(N)                                                                                     \
    (exact ? (mode == GS_ADAM_FUSED ? adam_slab_kernel<true, true, N> : adam_slab_kernel<true, false, N>) \
           : (mode == GS_ADAM_FUSED ? adam_slab_kernel<false, true, N> : adam_slab_kernel<false, false, N>))
    auto kernel = narrow ? GS_ADAM_SLAB(true) : GS_ADAM_SLAB(false);
#undef GS_ADAM_SLAB
    kernel<<<grid_for(half, 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<float4*>(theta), reinterpret_cast<const float4*>(g), reinterpret_cast<float4*>(m),
        reinterpret_cast<float4*>(v), indices, num_active, chunks, shift, (int)(g_stride / 4), ncols,
        quat_col < 0 ? -1 : quat_col / 4, half, visible_words, g_cols, g_cols < ncols ? count_col : 0, row_select,
        s, cols);
    return check_launch("adam_slab_kernel");
}

extern "C" int gs_fused_adam_slab_sharded(float* theta, float* theta_multicast, const float* g_multicast,
                                          float* m, float* v, const int32_t* indices, int64_t num_active, int ncols,
                                          int64_t stride, int64_t g_stride, const float* col_lo, const float* col_hi,
                                          int quat_col, double lr, double beta1, double beta2, float eps,
                                          float weight_decay, int step, float grad_scale,
                                          const float* grad_bias_host, int g_cols, int count_col,
                                          const float* count_coef_host, int rank, int world, int hot_cols,
                                          const int32_t* error_flag, gs_stream_t stream) {
    GS_REQUIRE(world >= 1 && rank >= 0 && rank < world, "adam_sharded: bad rank/world");
    GS_REQUIRE(ncols > 0 && ncols <= kMaxSlabCols, "adam_sharded: ncols must be in [1, %d]", kMaxSlabCols);
    GS_REQUIRE(stride % 4 == 0 && g_stride % 4 == 0 && stride >= ncols && stride <= 128 && g_stride >= g_cols,
               "adam_sharded: strides must be multiples of 4, ncols <= stride <= 128, g_stride >= g_cols");
    GS_REQUIRE(g_cols > 0 && g_cols <= ncols, "adam_sharded: g_cols must be in [1, ncols]");
    GS_REQUIRE(g_cols == ncols || (count_coef_host && count_col >= g_cols && count_col < g_stride &&
                                   count_col < stride && (count_col & ~3) < ncols),
               "adam_sharded: narrow gradient rows need count_coef_host and a count column in [g_cols, g_stride)");
    GS_REQUIRE(hot_cols >= 0 && hot_cols % 4 == 0 && hot_cols <= stride, "adam_sharded: hot_cols must be a "
               "multiple of 4 within the row");
    GS_REQUIRE(quat_col < 0 || (quat_col % 4 == 0 && quat_col + 4 <= ncols), "adam_sharded: bad quat_col");
    GS_REQUIRE(step >= 1 && num_active >= 0, "adam_sharded: bad step/num_active");
    if (num_active == 0) return GS_OK;
    GS_REQUIRE(theta && theta_multicast && g_multicast && m && v && indices && col_lo && col_hi,
               "adam_sharded: null pointer");
    GS_REQUIRE(aligned16(theta) && aligned16(theta_multicast) && aligned16(g_multicast) && aligned16(m) &&
               aligned16(v), "adam_sharded: bases must be 16-byte aligned");
    double bc1;
    AdamScalars s = make_scalars(GS_ADAM_FUSED, beta1, beta2, eps, weight_decay, step, grad_scale, &bc1);
    SlabCols cols;
    for (int c = 0; c < kMaxSlabCols; ++c) {
        const bool on = c < ncols;
        cols.lo[c] = on ? col_lo[c] : 0.f;
        cols.hi[c] = on ? col_hi[c] : 0.f;
        cols.step_size[c] = on ? step_size_for(GS_ADAM_FUSED, lr, 1.0, bc1) : 0.f;
        cols.gdef[c] = 0.f;
        cols.gbias[c] = (on && grad_bias_host) ? grad_bias_host[c] : 0.f;
        cols.gcoef[c] = (on && c >= g_cols) ? count_coef_host[c] : 0.f;
    }
    s.has_bias = grad_bias_host != nullptr;
    const int chunks = (int)(stride / 4);
    int shift = 0;
    while ((1 << shift) < chunks) ++shift;
    const int64_t n = num_active << shift;
    const int64_t half = (n + 511) / 512 * 256;
    auto kernel = g_cols < ncols ? adam_sharded_kernel<true> : adam_sharded_kernel<false>;
    kernel<<<grid_for(half, 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<float4*>(theta), reinterpret_cast<float4*>(theta_multicast),
        reinterpret_cast<const float4*>(g_multicast), reinterpret_cast<float4*>(m), reinterpret_cast<float4*>(v),
        indices, num_active, chunks, shift, (int)(g_stride / 4), ncols, quat_col < 0 ? -1 : quat_col / 4, half,
        g_cols, g_cols < ncols ? count_col : 0, rank, world, hot_cols / 4, error_flag, s, cols);
    return check_launch("adam_sharded_kernel");
}

extern "C" int gs_launch_fused_adam_step(uint64_t theta_addr, uint64_t g_addr, uint64_t m_addr, uint64_t v_addr,
                                         uint64_t indices_addr, size_t max_gaussians, size_t num_active, int dim,
                                         float lr, float beta1, float beta2, float eps, float weight_decay, int step,
                                         float a_min, float a_max, gs_stream_t stream) {
    (void)max_gaussians;  // the pools are addressed through the indirection table, as in the reference
    float* theta = reinterpret_cast<float*>(theta_addr);
    const float* g = reinterpret_cast<const float*>(g_addr);
    float* m = reinterpret_cast<float*>(m_addr);
    float* v = reinterpret_cast<float*>(v_addr);
    const int32_t* idx = reinterpret_cast<const int32_t*>(indices_addr);
    if (dim % 4 == 0 && dim <= kMaxSlabCols && aligned16(theta) && aligned16(g) && aligned16(m) && aligned16(v)) {
        float lo[kMaxSlabCols], hi[kMaxSlabCols];
        for (int c = 0; c < dim; ++c) {
            lo[c] = a_min;
            hi[c] = a_max;
        }
        return gs_fused_adam_slab(theta, g, m, v, idx, (int64_t)num_active, dim, dim, dim, lo, hi, nullptr, -1, lr,
                                  beta1, beta2, eps, weight_decay, step, 1.0f, GS_ADAM_FUSED | GS_ADAM_EXACT,
                                  nullptr, nullptr, nullptr, dim, 0, nullptr, GS_ROWS_ALL, stream);
    }
    return gs_fused_adam_group(theta, g, m, v, idx, (int64_t)num_active, dim, dim, dim, lr, beta1, beta2, eps,
                               weight_decay, step, a_min, a_max, 1.0f, 1.0f, GS_ADAM_FUSED, stream);
}

extern "C" int gs_clear_buffer_cache(void) { return GS_OK; }
