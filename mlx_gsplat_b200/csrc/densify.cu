// Densify / prune over the fixed-capacity pool (mlx_gsplat/trainer.py:421-519
// and mlx_gsplat/allocator.py:185-292), as GPU kernels:
//   masks    - per active row: grow (clone or split) and prune decisions
//   children - child rows built from the parent rows and the noise draws
//   rows     - scatter of whole rows into the slab (children, prune resets),
//              zeroing the Adam moments and the densification statistics
//   free list- LIFO push of pruned slots and reversed pop of child slots
// Ordered compaction of the masks is gs_compact_flags (cull.cu).
#include <math.h>

#include "common.cuh"

namespace gs {

struct DensifyParams {
    float grad_thr, small_thr, large_thr, dim_thr, quat_tol;
    int prune_geometry;
};

// numpy's max propagates NaN; fmaxf would drop it
__device__ __forceinline__ float nanmax3(float a, float b, float c) {
    if (isnan(a) || isnan(b) || isnan(c)) return __int_as_float(0x7fc00000);
    return fmaxf(fmaxf(a, b), c);
}

__global__ void densify_masks_kernel(gs_gaussians g, const float* __restrict__ grad2d, const float* __restrict__ count,
                                     int64_t n, DensifyParams dp, uint8_t* __restrict__ flags) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    const int64_t row = g.table ? (int64_t)__ldg(g.table + r) : r;
    // average screen-space gradient (trainer.py:436-437)
    const float avg = __fdiv_rn(grad2d[row], fmaxf(count[row], 1.0f));
    const bool high = avg > dp.grad_thr;
    const float* sp = g.scales + row * g.scales_stride;
    const float s0 = sp[0], s1 = sp[1], s2 = sp[2];
    const float smax = nanmax3(expf(s0), expf(s1), expf(s2));
    const bool small = smax <= dp.small_thr;
    const float o = g.opac[row * g.opac_stride];
    const float raw = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-o)));
    const bool too_dim = raw < dp.dim_thr;
    const bool too_large = smax > dp.large_thr;
    const float* mp = g.means + row * g.means_stride;
    const bool nan_mask = !(isfinite(s0) && isfinite(s1) && isfinite(s2)) || !isfinite(o) ||
                          !(isfinite(mp[0]) && isfinite(mp[1]) && isfinite(mp[2]));
    const float* qp = g.quats + row * g.quats_stride;
    float ss = __fmul_rn(qp[0], qp[0]);
    ss = __fadd_rn(ss, __fmul_rn(qp[1], qp[1]));
    ss = __fadd_rn(ss, __fmul_rn(qp[2], qp[2]));
    ss = __fadd_rn(ss, __fmul_rn(qp[3], qp[3]));
    const bool bad_quat = fabsf(__fsub_rn(__fsqrt_rn(ss), 1.0f)) > dp.quat_tol;
    bool prune = nan_mask || bad_quat;
    if (dp.prune_geometry) prune = prune || too_dim || too_large;
    flags[r] = (uint8_t)((prune ? GS_FLAG_PRUNE : 0) | (high ? GS_FLAG_REFINE : 0) |
                         ((high && !small) ? GS_FLAG_SPLIT : 0));
}

struct ChildCols {
    int means, scales, quats, opac;
};

// Child rows of refine row j (trainer.py:479-507): means + 0.02 * noise (one
// draw per child), scales - log(1.6) when splitting, opacity logit * 0.95,
// quaternion normalised (child 2 after + 0.01 * noise), everything else copied.
__global__ void densify_children_kernel(const float* __restrict__ theta, int64_t stride, int ncols,
                                        const int32_t* __restrict__ parent_slots,
                                        const int32_t* __restrict__ refine_rows, const uint8_t* __restrict__ flags,
                                        const float* __restrict__ noise_m1, const float* __restrict__ noise_m2,
                                        const float* __restrict__ noise_q2, int64_t n_s, ChildCols cc,
                                        float log16, float* __restrict__ child1, float* __restrict__ child2) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n_s) return;
    const float* pr = theta + (int64_t)parent_slots[j] * stride;
    float* c1 = child1 + j * stride;
    float* c2 = child2 + j * stride;
    for (int c = 0; c < stride; ++c) {
        const float x = pr[c];
        c1[c] = x;
        c2[c] = x;
    }
    (void)ncols;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float x = pr[cc.means + k];
        c1[cc.means + k] = __fadd_rn(x, __fmul_rn(noise_m1[3 * j + k], 0.02f));
        c2[cc.means + k] = __fadd_rn(x, __fmul_rn(noise_m2[3 * j + k], 0.02f));
    }
    const bool split = (flags[refine_rows[j]] & GS_FLAG_SPLIT) != 0;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        const float x = __fsub_rn(pr[cc.scales + k], split ? log16 : 0.0f);
        c1[cc.scales + k] = x;
        c2[cc.scales + k] = x;
    }
    const float op = __fmul_rn(pr[cc.opac], 0.95f);
    c1[cc.opac] = op;
    c2[cc.opac] = op;
    float q1[4], q2[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        q1[k] = pr[cc.quats + k];
        q2[k] = __fadd_rn(q1[k], __fmul_rn(noise_q2[4 * j + k], 0.01f));
    }
    float s1 = __fmul_rn(q1[0], q1[0]), s2 = __fmul_rn(q2[0], q2[0]);
#pragma unroll
    for (int k = 1; k < 4; ++k) {
        s1 = __fadd_rn(s1, __fmul_rn(q1[k], q1[k]));
        s2 = __fadd_rn(s2, __fmul_rn(q2[k], q2[k]));
    }
    const float n1 = __fsqrt_rn(__fadd_rn(s1, 1e-8f)), n2 = __fsqrt_rn(__fadd_rn(s2, 1e-8f));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        c1[cc.quats + k] = __fdiv_rn(q1[k], n1);
        c2[cc.quats + k] = __fdiv_rn(q2[k], n2);
    }
}

constexpr int kMaxRow = 64;
struct RowVals {
    float v[kMaxRow];
};

// Row j: theta[slots[j]] = vals[j] (or the reset pattern), m and v rows zeroed,
// grad2d / count zeroed.  One thread per (row, column).
__global__ void pool_write_rows_kernel(float* __restrict__ theta, float* __restrict__ m, float* __restrict__ v,
                                       int64_t stride, const int32_t* __restrict__ slots, int64_t n,
                                       const float* __restrict__ vals, int64_t vals_stride, RowVals reset,
                                       float* __restrict__ grad2d, float* __restrict__ count) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n * stride) return;
    const int64_t j = t / stride;
    const int c = (int)(t - j * stride);
    const int64_t p = (int64_t)slots[j] * stride + c;
    theta[p] = vals ? vals[j * vals_stride + c] : reset.v[c];
    if (m) m[p] = 0.f;
    if (v) v[p] = 0.f;
    if (c == 0) {
        if (grad2d) grad2d[slots[j]] = 0.f;
        if (count) count[slots[j]] = 0.f;
    }
}

__global__ void free_pop_reversed_kernel(const int32_t* __restrict__ stack, int64_t top, int64_t n,
                                         int32_t* __restrict__ out) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n) out[j] = stack[top - 1 - j];
}

}  // namespace gs

using namespace gs;

extern "C" int gs_densify_masks(const gs_gaussians* g, const float* grad2d, const float* count, int64_t num_active,
                                float grad_threshold, float small_threshold, float large_threshold,
                                float dim_threshold, float quat_tolerance, int prune_geometry, uint8_t* flags,
                                gs_stream_t stream) {
    GS_REQUIRE(g && num_active >= 0, "densify_masks: bad arguments");
    if (num_active == 0) return GS_OK;
    GS_REQUIRE(g->means && g->quats && g->scales && g->opac && grad2d && count && flags,
               "densify_masks: null pointer");
    DensifyParams dp{grad_threshold, small_threshold, large_threshold, dim_threshold, quat_tolerance, prune_geometry};
    densify_masks_kernel<<<grid_for(num_active, 256), 256, 0, (cudaStream_t)stream>>>(*g, grad2d, count, num_active,
                                                                                      dp, flags);
    return check_launch("densify_masks_kernel");
}

extern "C" int gs_densify_children(const float* theta, int64_t stride, int ncols, const int32_t* parent_slots,
                                   const int32_t* refine_rows, const uint8_t* flags, const float* noise_means1,
                                   const float* noise_means2, const float* noise_quats2, int64_t num_children,
                                   int col_means, int col_scales, int col_quats, int col_opac, float* child1,
                                   float* child2, gs_stream_t stream) {
    GS_REQUIRE(num_children >= 0 && stride > 0, "densify_children: bad sizes");
    if (num_children == 0) return GS_OK;
    GS_REQUIRE(theta && parent_slots && refine_rows && flags && noise_means1 && noise_means2 && noise_quats2 && child1 &&
                   child2,
               "densify_children: null pointer");
    GS_REQUIRE(col_means + 3 <= stride && col_scales + 3 <= stride && col_quats + 4 <= stride && col_opac < stride,
               "densify_children: column out of range");
    ChildCols cc{col_means, col_scales, col_quats, col_opac};
    const float log16 = (float)log(1.6);
    densify_children_kernel<<<grid_for(num_children, 128), 128, 0, (cudaStream_t)stream>>>(
        theta, stride, ncols, parent_slots, refine_rows, flags, noise_means1, noise_means2, noise_quats2,
        num_children, cc, log16, child1, child2);
    return check_launch("densify_children_kernel");
}

extern "C" int gs_pool_write_rows(float* theta, float* m, float* v, int64_t stride, const int32_t* slots, int64_t n,
                                  const float* vals, int64_t vals_stride, const float* reset_row_host, float* grad2d,
                                  float* count, gs_stream_t stream) {
    GS_REQUIRE(stride > 0 && stride <= kMaxRow && n >= 0, "pool_write_rows: bad sizes");
    if (n == 0) return GS_OK;
    GS_REQUIRE(theta && slots && (vals || reset_row_host), "pool_write_rows: null pointer");
    RowVals rv;
    for (int c = 0; c < kMaxRow; ++c) rv.v[c] = (reset_row_host && c < stride) ? reset_row_host[c] : 0.f;
    pool_write_rows_kernel<<<grid_for(n * stride, 256), 256, 0, (cudaStream_t)stream>>>(
        theta, m, v, stride, slots, n, vals, vals ? vals_stride : 0, rv, grad2d, count);
    return check_launch("pool_write_rows_kernel");
}

extern "C" int gs_free_pop_reversed(const int32_t* stack, int64_t top, int64_t n, int32_t* out, gs_stream_t stream) {
    GS_REQUIRE(n >= 0 && top >= n, "free_pop: popping %lld of %lld slots", (long long)n, (long long)top);
    if (n == 0) return GS_OK;
    GS_REQUIRE(stack && out, "free_pop: null pointer");
    free_pop_reversed_kernel<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(stack, top, n, out);
    return check_launch("free_pop_reversed_kernel");
}
