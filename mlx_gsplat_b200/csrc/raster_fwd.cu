// Rasterizer forward: projection + tile counting, binning, tile ranges and the
// tile compositing kernel (mlx_gsplat/rendering.py:97-308, re-designed as a
// 16x16-tile rasterizer).
#include "raster.cuh"
#include "scan.cuh"

namespace gs {

// ---------------------------------------------------------------- projection + tile count
__global__ void __launch_bounds__(128) project_fwd_kernel(gs_gaussians g, const int32_t* __restrict__ ids,
                                                          int64_t nv, RasterParams p, float4* __restrict__ splats,
                                                          uint32_t* __restrict__ depth_keys,
                                                          uint32_t* __restrict__ tile_counts) {
    const int64_t vi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vi >= nv) return;
    const int32_t id = ids[vi];
    const int64_t row = param_row(g, id);
    const int64_t crow = g.colors_by_visible ? vi : row;
    ProjState s;
    project_one(g, row, g.colors + crow * g.colors_stride, p, s);
    splats[3 * vi + 0] = make_float4(s.u, s.v, s.ca, s.cb);
    splats[3 * vi + 1] = make_float4(s.cc, s.cd, s.opac, s.rgb[0]);
    splats[3 * vi + 2] = make_float4(s.rgb[1], s.rgb[2], pair_cut(s.opac, p), s.tz);
    depth_keys[vi] = float_sort_key(s.tz);
    uint32_t cnt = 0;
    TileBox tb;
    if (splat_tile_box(s.u, s.v, s.ca, s.cb, s.cc, s.cd, s.opac, p, tb)) {
        if (!tb.exact) {
            cnt = (uint32_t)((tb.x1 - tb.x0 + 1) * (tb.y1 - tb.y0 + 1));
        } else {
            for (int ty = tb.y0; ty <= tb.y1; ++ty)
                for (int tx = tb.x0; tx <= tb.x1; ++tx) cnt += splat_hits_tile(s.u, s.v, s.ca, s.cd, tb, tx, ty, p);
        }
    }
    tile_counts[vi] = cnt;
}

// counts in depth order: out[r] = tile_counts[order[r]]
__global__ void gather_counts_kernel(const uint32_t* __restrict__ order, const uint32_t* __restrict__ counts,
                                     int64_t n, uint32_t* __restrict__ out) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n) out[r] = counts[order[r]];
}

__global__ void __launch_bounds__(128) bin_emit_kernel(const float4* __restrict__ splats,
                                                       const uint32_t* __restrict__ order,
                                                       const uint32_t* __restrict__ offsets,
                                                       const uint32_t* __restrict__ tile_counts, int64_t nv,
                                                       RasterParams p, uint32_t* __restrict__ tile_keys,
                                                       uint32_t* __restrict__ vals, int64_t capacity,
                                                       int32_t* __restrict__ overflow) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= nv) return;
    const uint32_t vi = order[r];
    const uint32_t cnt = tile_counts[vi];
    if (cnt == 0) return;
    const int64_t base = offsets[r];
    if (base + cnt > capacity) {
        atomicExch(overflow, 1);
        return;
    }
    const float4 a = splats[3 * vi], b = splats[3 * vi + 1];
    TileBox tb;
    uint32_t k = 0;
    if (splat_tile_box(a.x, a.y, a.z, a.w, b.x, b.y, b.z, p, tb)) {
        for (int ty = tb.y0; ty <= tb.y1 && k < cnt; ++ty)
            for (int tx = tb.x0; tx <= tb.x1 && k < cnt; ++tx)
                if (splat_hits_tile(a.x, a.y, a.z, b.y, tb, tx, ty, p)) {
                    tile_keys[base + k] = (uint32_t)(ty * p.tiles_x + tx);
                    vals[base + k] = vi;
                    ++k;
                }
    }
    // The counting pass ran the same test on the same floats, so k == cnt; any
    // shortfall becomes sentinel entries that sort past every tile and are ignored.
    for (; k < cnt; ++k) {
        tile_keys[base + k] = 0xffffffffu;
        vals[base + k] = 0u;
    }
}

__global__ void tile_ranges_kernel(const uint32_t* __restrict__ keys, int64_t n, int32_t num_tiles,
                                   gs_tile_range* __restrict__ ranges) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t t = keys[i];
    if (t >= (uint32_t)num_tiles) return;
    if (i == 0 || keys[i - 1] != t) ranges[t].start = (int32_t)i;
    if (i == n - 1 || keys[i + 1] != t) ranges[t].end = (int32_t)(i + 1);
}

// ---------------------------------------------------------------- compositing
// One CTA per 16x16 tile, one thread per pixel.  Warp w owns the 8x4 pixel
// block ((w & 1) * 8, (w >> 1) * 4) of the tile.  Splats are staged 256 at a
// time in shared memory; a warp skips the rest of a batch once all its pixels
// are saturated (T < t_min) and the CTA stops when all 256 are.
__global__ void __launch_bounds__(kTileThreads) render_fwd_kernel(
    const gs_tile_range* __restrict__ ranges, const uint32_t* __restrict__ vals, const float4* __restrict__ splats,
    int64_t nv, RasterParams p, float* __restrict__ out_color, float* __restrict__ out_alpha, float* __restrict__ final_T,
    int32_t* __restrict__ n_contrib, int loss_mode, const void* __restrict__ target,
    float* __restrict__ loss_partials) {
    __shared__ float4 s0[kTileThreads], s1[kTileThreads], s2[kTileThreads];
    __shared__ float red[kTileThreads / 32];
    const int tile = blockIdx.x;
    const int tx = tile % p.tiles_x, ty = tile / p.tiles_x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pi = tx * kTile + (warp & 1) * 8 + (lane & 7);
    const int pj = ty * kTile + (warp >> 1) * 4 + (lane >> 3);
    const bool inside = pi < p.rw && pj < p.rh;
    const float px = (float)pi * p.sx + p.hsx;
    const float py = (float)pj * p.sy + p.hsy;
    const gs_tile_range rg = ranges[tile];

    float T = 1.f, cr = 0.f, cg = 0.f, cb = 0.f, A = 0.f;
    int last = 0;
    bool done = !inside;
    for (int b = rg.start; b < rg.end; b += kTileThreads) {
        if (__syncthreads_count(done) == kTileThreads) break;
        const int e = b + threadIdx.x;
        if (e < rg.end) {
            const uint32_t vr = vals[e];
            const uint32_t vi = vr < (uint64_t)nv ? vr : 0u;
            s0[threadIdx.x] = splats[3 * vi];
            s1[threadIdx.x] = splats[3 * vi + 1];
            s2[threadIdx.x] = splats[3 * vi + 2];
        }
        __syncthreads();
        const int cnt = min(kTileThreads, rg.end - b);
        for (int k = 0; k < cnt; ++k) {
            if (__all_sync(kFull, done)) break;
            const float4 q0 = s0[k], q1 = s1[k], q2 = s2[k];
            const float x = px - q0.x, y = py - q0.y;
            const float m = x * (q0.z * x + q0.w * y) + y * (q1.x * x + q1.y * y);
            if (!done && m <= q2.z) {
                const float gv = __expf(-0.5f * m);
                const float al = fminf(q1.z * gv, 0.99f);
                const float w = al * T;
                cr += w * q1.w;
                cg += w * q2.x;
                cb += w * q2.y;
                A += w;
                T *= (1.f - al);
                last = b - rg.start + k + 1;
                if (T < p.t_min) done = true;
            }
        }
        __syncthreads();
    }

    float lsum = 0.f;
    if (inside) {
        const int64_t pix = (int64_t)pj * p.rw + pi;
        out_color[3 * pix + 0] = cr;
        out_color[3 * pix + 1] = cg;
        out_color[3 * pix + 2] = cb;
        out_alpha[pix] = A;
        final_T[pix] = T;
        n_contrib[pix] = last;
        if (loss_mode == GS_LOSS_L1_U8) {
            const uint8_t* t8 = static_cast<const uint8_t*>(target) + 3 * pix;
            lsum = fabsf(cr - __fdiv_rn((float)t8[0], 255.0f)) + fabsf(cg - __fdiv_rn((float)t8[1], 255.0f)) +
                   fabsf(cb - __fdiv_rn((float)t8[2], 255.0f));
        } else if (loss_mode == GS_LOSS_L1_F32) {
            const float* tf = static_cast<const float*>(target) + 3 * pix;
            lsum = fabsf(cr - tf[0]) + fabsf(cg - tf[1]) + fabsf(cb - tf[2]);
        } else if (loss_mode == GS_LOSS_MEAN) {
            lsum = cr + cg + cb;
        }
    }
    if (loss_mode != GS_LOSS_NONE) {
        lsum = warp_sum(lsum);
        if (lane == 0) red[warp] = lsum;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kTileThreads / 32; ++w) t += red[w];
            loss_partials[tile] = t;
        }
    }
}

}  // namespace gs

using namespace gs;

extern "C" int gs_project_forward(const gs_gaussians* g, const int32_t* ids, int64_t num_visible,
                                  const gs_camera* cam, const gs_raster_settings* rs, float* splats,
                                  uint32_t* depth_keys, uint32_t* tile_counts, gs_stream_t stream) {
    GS_REQUIRE(g && cam, "project_forward: null descriptor");
    GS_REQUIRE(num_visible >= 0, "project_forward: negative count");
    if (num_visible == 0) return GS_OK;
    GS_REQUIRE(ids && splats && depth_keys && tile_counts && g->means && g->quats && g->scales && g->opac && g->colors,
               "project_forward: null pointer");
    GS_REQUIRE(g->colors_dim >= 3, "project_forward: colors_dim must be >= 3");
    GS_REQUIRE(aligned16(splats), "project_forward: splats must be 16-byte aligned");
    GS_REQUIRE(cam->render_width > 0 && cam->render_height > 0 && cam->width > 0 && cam->height > 0,
               "project_forward: bad image size");
    const RasterParams p = make_raster_params(*cam, rs);
    project_fwd_kernel<<<grid_for(num_visible, 128), 128, 0, (cudaStream_t)stream>>>(
        *g, ids, num_visible, p, reinterpret_cast<float4*>(splats), depth_keys, tile_counts);
    return check_launch("project_fwd_kernel");
}

extern "C" size_t gs_bin_offsets_scratch_bytes(int64_t num_visible) {
    return align_up((size_t)(num_visible + 1) * 4, 256) + scan_scratch_bytes(num_visible) + 256;
}

extern "C" int gs_bin_offsets(const uint32_t* order, const uint32_t* tile_counts, int64_t num_visible,
                              uint32_t* offsets, void* scratch, size_t scratch_bytes, gs_stream_t stream) {
    GS_REQUIRE(num_visible >= 0 && offsets, "bin_offsets: bad arguments");
    GS_REQUIRE(scratch && scratch_bytes >= gs_bin_offsets_scratch_bytes(num_visible), "bin_offsets: scratch too small");
    char* p = reinterpret_cast<char*>(align_up(reinterpret_cast<uintptr_t>(scratch), 256));
    uint32_t* gathered = reinterpret_cast<uint32_t*>(p);
    p += align_up((size_t)(num_visible + 1) * 4, 256);
    if (num_visible > 0) {
        GS_REQUIRE(order && tile_counts, "bin_offsets: null pointer");
        gather_counts_kernel<<<grid_for(num_visible, 256), 256, 0, (cudaStream_t)stream>>>(order, tile_counts,
                                                                                           num_visible, gathered);
        GS_TRY(check_launch("gather_counts_kernel"));
    }
    return scan_exclusive(gathered, offsets, num_visible, p, scan_scratch_bytes(num_visible), (cudaStream_t)stream);
}

extern "C" int gs_bin_emit(const float* splats, const uint32_t* order, const uint32_t* offsets,
                           const uint32_t* tile_counts, int64_t num_visible, const gs_camera* cam,
                           const gs_raster_settings* rs, uint32_t* tile_keys, uint32_t* entry_vals, int64_t capacity,
                           int32_t* overflow_flag, gs_stream_t stream) {
    GS_REQUIRE(cam, "bin_emit: null camera");
    if (num_visible == 0) return GS_OK;
    GS_REQUIRE(splats && order && offsets && tile_counts && overflow_flag, "bin_emit: null pointer");
    GS_REQUIRE(capacity == 0 || (tile_keys && entry_vals), "bin_emit: null output");
    const RasterParams p = make_raster_params(*cam, rs);
    bin_emit_kernel<<<grid_for(num_visible, 128), 128, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const float4*>(splats), order, offsets, tile_counts, num_visible, p, tile_keys, entry_vals,
        capacity, overflow_flag);
    return check_launch("bin_emit_kernel");
}

extern "C" int gs_tile_ranges(const uint32_t* sorted_tile_keys, int64_t num_entries, int32_t num_tiles,
                              gs_tile_range* ranges, gs_stream_t stream) {
    GS_REQUIRE(ranges && num_tiles > 0, "tile_ranges: bad arguments");
    cudaMemsetAsync(ranges, 0, sizeof(gs_tile_range) * (size_t)num_tiles, (cudaStream_t)stream);
    if (num_entries == 0) return check_launch("tile_ranges memset", 0);
    GS_REQUIRE(sorted_tile_keys, "tile_ranges: null keys");
    tile_ranges_kernel<<<grid_for(num_entries, 256), 256, 0, (cudaStream_t)stream>>>(sorted_tile_keys, num_entries,
                                                                                     num_tiles, ranges);
    return check_launch("tile_ranges_kernel");
}

extern "C" int gs_render_forward(const gs_tile_range* ranges, const uint32_t* entry_vals, const float* splats,
                                 int64_t num_visible, const gs_camera* cam, const gs_raster_settings* rs,
                                 float* out_color,
                                 float* out_alpha, float* final_T, int32_t* n_contrib, int loss_mode,
                                 const void* target, float* loss_partials, gs_stream_t stream) {
    GS_REQUIRE(cam && ranges && out_color && out_alpha && final_T && n_contrib, "render_forward: null pointer");
    GS_REQUIRE(loss_mode >= GS_LOSS_NONE && loss_mode <= GS_LOSS_MEAN, "render_forward: bad loss mode");
    GS_REQUIRE(loss_mode == GS_LOSS_NONE || loss_partials, "render_forward: loss_partials required");
    GS_REQUIRE(loss_mode == GS_LOSS_NONE || loss_mode == GS_LOSS_MEAN || target, "render_forward: target required");
    const RasterParams p = make_raster_params(*cam, rs);
    const int tiles = p.tiles_x * p.tiles_y;
    render_fwd_kernel<<<tiles, kTileThreads, 0, (cudaStream_t)stream>>>(
        ranges, entry_vals, reinterpret_cast<const float4*>(splats), num_visible, p, out_color, out_alpha, final_T, n_contrib,
        loss_mode, target, loss_partials);
    return check_launch("render_fwd_kernel");
}
