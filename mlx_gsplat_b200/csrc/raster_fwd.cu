// Rasterizer forward: projection + tile counting, binning, tile ranges and the
// tile compositing kernel (mlx_gsplat/rendering.py:97-308, re-designed as a
// 16x16-tile rasterizer).
#include "raster.cuh"
#include "scan.cuh"

namespace gs {

// ---------------------------------------------------------------- warp-cooperative binning
// Each lane holds one splat's tile box.  The warp visits the boxes of its
// lanes one after another and tests 32 tiles of the current box at a time
// (ballot + popcount give the output positions), so a splat covering
// thousands of tiles costs thousands / 32 warp steps rather than serialising
// one thread.  The counting pass also returns, for a box of at most 64
// tiles, the bitmask of the tiles it binned (bit t = tile t of the box in
// row-major order); the emitting pass, given that mask, expands it instead of
// testing the tiles again, so both passes agree tile for tile.
constexpr int kMaskTiles = 64;

template <bool kEmit>
__device__ __forceinline__ uint32_t warp_bin(bool has, const TileBox& tb, float u, float v, float ca, float cd,
                                             const RasterParams& p, uint32_t base, uint32_t expected, uint32_t vi,
                                             bool use_masks, uint64_t mask_in, uint32_t* __restrict__ keys,
                                             uint32_t* __restrict__ vals, uint64_t& mask_out) {
    const int lane = threadIdx.x & 31;
    const unsigned lt = lanemask_lt();
    uint32_t mine = 0;
    mask_out = 0;
    unsigned todo = __ballot_sync(kFull, has);
    while (todo) {
        const int j = __ffs(todo) - 1;
        todo &= todo - 1;
        const int x0 = __shfl_sync(kFull, tb.x0, j), x1 = __shfl_sync(kFull, tb.x1, j);
        const int y0 = __shfl_sync(kFull, tb.y0, j), y1 = __shfl_sync(kFull, tb.y1, j);
        const int w = x1 - x0 + 1;
        const int area = w * (y1 - y0 + 1);
        const bool from_mask = kEmit && use_masks && area <= kMaskTiles;
        TileBox b;
        float uj = 0.f, vj = 0.f, caj = 0.f, cdj = 0.f;
        uint64_t mj = 0;
        if (from_mask) {
            mj = ((uint64_t)__shfl_sync(kFull, (uint32_t)(mask_in >> 32), j) << 32) |
                 __shfl_sync(kFull, (uint32_t)mask_in, j);
        } else {
            b.exact = __shfl_sync(kFull, (int)tb.exact, j) != 0;
            b.m_cut = __shfl_sync(kFull, tb.m_cut, j);
            b.s = __shfl_sync(kFull, tb.s, j);
            uj = __shfl_sync(kFull, u, j);
            vj = __shfl_sync(kFull, v, j);
            caj = __shfl_sync(kFull, ca, j);
            cdj = __shfl_sync(kFull, cd, j);
        }
        uint32_t basej = 0, expj = 0, vij = 0;
        if (kEmit) {
            basej = __shfl_sync(kFull, base, j);
            expj = __shfl_sync(kFull, expected, j);
            vij = __shfl_sync(kFull, vi, j);
        }
        uint32_t cnt = 0;
        uint64_t bits = 0;
        for (int t0 = 0; t0 < area; t0 += 32) {
            const int t = t0 + lane;
            bool hit = false;
            int tile_id = 0;
            if (t < area) {
                const int r = t / w;
                const int tx = x0 + (t - r * w), ty = y0 + r;
                hit = from_mask ? ((mj >> t) & 1u) != 0 : splat_hits_tile(uj, vj, caj, cdj, b, tx, ty, p);
                tile_id = ty * p.tiles_x + tx;
            }
            const unsigned bal = __ballot_sync(kFull, hit);
            if (!kEmit && t0 < kMaskTiles) bits |= (uint64_t)bal << t0;
            if (kEmit && hit) {
                const uint32_t k = cnt + __popc(bal & lt);
                if (k < expj) {
                    keys[basej + k] = (uint32_t)tile_id;
                    vals[basej + k] = vij;
                }
            }
            cnt += __popc(bal);
        }
        if (kEmit) {
            // the counting pass gave expj == cnt; any shortfall becomes sentinel
            // entries that sort past every tile and are ignored
            for (uint32_t k = cnt + lane; k < expj; k += 32) {
                keys[basej + k] = 0xffffffffu;
                vals[basej + k] = 0u;
            }
        }
        if (lane == j) {
            mine = cnt;
            mask_out = area <= kMaskTiles ? bits : 0;
        }
    }
    return mine;
}

// ---------------------------------------------------------------- binning scratch
// Splats whose tile box has more than kBigTiles tiles are not binned by their
// warp: the counting pass appends them to a list, and CTA-wide kernels count
// and emit them (kBigThreads tiles tested at a time), so a few very large
// splats do not leave one warp running long after the rest of the launch.
constexpr int kBigTiles = 256;
constexpr int kBigThreads = 256;
constexpr unsigned kBigGrid = 2 * 148;

struct BinScratch {
    uint32_t* big_count;  // number of listed splats
    uint32_t* big_list;   // their visible indices
    uint32_t* big_base;   // per visible index: first output entry (UINT32_MAX: not to emit)
    uint64_t* masks;      // per visible index: binned-tile bitmask of a box of <= 64 tiles
};

inline size_t bin_scratch_bytes(int64_t nv) {
    const size_t n = (size_t)(nv > 0 ? nv : 1);
    return 256 + align_up(n * 4, 256) * 2 + align_up(n * 8, 256) + 256;
}

inline BinScratch bin_scratch_layout(void* scratch, int64_t nv) {
    const size_t n = (size_t)(nv > 0 ? nv : 1);
    char* q = reinterpret_cast<char*>(align_up(reinterpret_cast<uintptr_t>(scratch), 256));
    BinScratch b;
    b.big_count = reinterpret_cast<uint32_t*>(q);
    q += 256;
    b.big_list = reinterpret_cast<uint32_t*>(q);
    q += align_up(n * 4, 256);
    b.big_base = reinterpret_cast<uint32_t*>(q);
    q += align_up(n * 4, 256);
    b.masks = reinterpret_cast<uint64_t*>(q);
    return b;
}

// Tile t (row-major) of a box tests exactly as the warp path does.
__device__ __forceinline__ bool box_tile_hit(const TileBox& tb, int t, int w, float u, float v, float ca, float cd,
                                             const RasterParams& p, int& tile_id) {
    const int r = t / w;
    const int tx = tb.x0 + (t - r * w), ty = tb.y0 + r;
    tile_id = ty * p.tiles_x + tx;
    return splat_hits_tile(u, v, ca, cd, tb, tx, ty, p);
}

// Block-wide exclusive prefix of one flag per thread; returns the prefix and
// the block total in *total.  ``wsum`` holds kBigThreads / 32 entries.
__device__ __forceinline__ uint32_t block_flag_prefix(bool f, uint32_t* wsum, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned bal = __ballot_sync(kFull, f);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    uint32_t before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < kBigThreads / 32; ++w) {
        const uint32_t c = wsum[w];
        before += w < warp ? c : 0u;
        all += c;
    }
    __syncthreads();
    *total = all;
    return before + __popc(bal & lanemask_lt());
}

__global__ void __launch_bounds__(kBigThreads) bin_count_big_kernel(const float4* __restrict__ splats, BinScratch bs,
                                                                    RasterParams p,
                                                                    uint32_t* __restrict__ tile_counts) {
    pdl_wait();
    const uint32_t n = *bs.big_count;
    for (uint32_t i = blockIdx.x; i < n; i += gridDim.x) {
        const uint32_t vi = bs.big_list[i];
        const float4 a = splats[3 * vi], b = splats[3 * vi + 1];
        TileBox tb;
        splat_tile_box(a.x, a.y, a.z, a.w, b.x, b.y, b.z, p, tb);  // listed only when it has a box
        const int w = tb.x1 - tb.x0 + 1, area = w * (tb.y1 - tb.y0 + 1);
        uint32_t cnt = 0;
        for (int t0 = 0; t0 < area; t0 += kBigThreads) {
            const int t = t0 + threadIdx.x;
            int tile_id;
            const bool hit = t < area && box_tile_hit(tb, t, w, a.x, a.y, a.z, b.y, p, tile_id);
            cnt += __syncthreads_count(hit);
        }
        if (threadIdx.x == 0) tile_counts[vi] = cnt;
    }
}

__global__ void __launch_bounds__(kBigThreads) bin_emit_big_kernel(const float4* __restrict__ splats, BinScratch bs,
                                                                   const uint32_t* __restrict__ tile_counts,
                                                                   RasterParams p, uint32_t* __restrict__ tile_keys,
                                                                   uint32_t* __restrict__ vals) {
    pdl_wait();
    __shared__ uint32_t wsum[kBigThreads / 32];
    const uint32_t n = *bs.big_count;
    for (uint32_t i = blockIdx.x; i < n; i += gridDim.x) {
        const uint32_t vi = bs.big_list[i];
        const uint32_t base = bs.big_base[vi];
        if (base == 0xffffffffu) continue;  // over capacity (uniform over the block)
        const uint32_t cnt = tile_counts[vi];
        const float4 a = splats[3 * vi], b = splats[3 * vi + 1];
        TileBox tb;
        splat_tile_box(a.x, a.y, a.z, a.w, b.x, b.y, b.z, p, tb);
        const int w = tb.x1 - tb.x0 + 1, area = w * (tb.y1 - tb.y0 + 1);
        uint32_t done = 0;
        for (int t0 = 0; t0 < area; t0 += kBigThreads) {
            const int t = t0 + threadIdx.x;
            int tile_id = 0;
            const bool hit = t < area && box_tile_hit(tb, t, w, a.x, a.y, a.z, b.y, p, tile_id);
            uint32_t total;
            const uint32_t k = done + block_flag_prefix(hit, wsum, &total);
            if (hit && k < cnt) {
                tile_keys[base + k] = (uint32_t)tile_id;
                vals[base + k] = vi;
            }
            done += total;
        }
        // the counting pass gave cnt == done; a shortfall becomes sentinel entries
        for (uint32_t k = done + threadIdx.x; k < cnt; k += kBigThreads) {
            tile_keys[base + k] = 0xffffffffu;
            vals[base + k] = 0u;
        }
    }
}

// A lane counts the tiles of its own box when the box has at most
// kLaneTiles tiles (most splats): the same exact test per tile, in the same
// row-major order, so count and mask equal warp_bin's; larger boxes go
// through the warp-cooperative loop.  On the 1 M-Gaussian outdoor scene
// this took the projection kernel from 0.141 to 0.093 ms (limits of 4, 8,
// 16, 32 and 64 tiles measured: 16 was fastest there and on the 200k scene).
#ifndef GS_LANE_TILES
#define GS_LANE_TILES 16
#endif
constexpr int kLaneTiles = GS_LANE_TILES;
static_assert(kLaneTiles <= kMaskTiles, "a lane-counted box must fit the tile mask");

__device__ __forceinline__ uint32_t lane_bin(const TileBox& tb, float u, float v, float ca, float cd,
                                             const RasterParams& p, uint64_t& mask) {
    uint32_t cnt = 0;
    mask = 0;
    int t = 0;
    for (int ty = tb.y0; ty <= tb.y1; ++ty)
        for (int tx = tb.x0; tx <= tb.x1; ++tx, ++t)
            if (splat_hits_tile(u, v, ca, cd, tb, tx, ty, p)) {
                ++cnt;
                mask |= 1ull << t;
            }
    return cnt;
}

// ---------------------------------------------------------------- projection + tile count
template <bool kSlab, int kDeg>
__global__ void __launch_bounds__(128) project_fwd_kernel(gs_gaussians g, const int32_t* __restrict__ ids,
                                                          int64_t nv, RasterParams p, float4* __restrict__ splats,
                                                          uint32_t* __restrict__ depth_keys,
                                                          uint32_t* __restrict__ tile_counts, bool use_bs,
                                                          BinScratch bs) {
    const int64_t vi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const bool active = vi < nv;
    bool has = false;
    TileBox tb;
    tb.x0 = tb.x1 = tb.y0 = tb.y1 = 0;
    tb.exact = true;
    tb.m_cut = tb.s = 0.f;
    float u = 0.f, v = 0.f, ca = 0.f, cd = 0.f;
    if (active) {
        const int32_t id = ids[vi];
        const int64_t row = param_row(g, id);
        GaussianIn<kDeg> in;
        load_gaussian<kSlab>(g, row, g.colors_by_visible ? vi : row, in);
        ProjState s;
        project_one(in, g.colors_dim >= 12, p, s);
        splats[3 * vi + 0] = make_float4(s.u, s.v, s.ca, s.cb);
        splats[3 * vi + 1] = make_float4(s.cc, s.cd, s.opac, s.rgb[0]);
        splats[3 * vi + 2] = make_float4(s.rgb[1], s.rgb[2], pair_cut(s.opac, p), s.tz);
        depth_keys[vi] = float_sort_key(s.tz);
        has = splat_tile_box(s.u, s.v, s.ca, s.cb, s.cc, s.cd, s.opac, p, tb);
        if (has && use_bs && (tb.x1 - tb.x0 + 1) * (tb.y1 - tb.y0 + 1) > kBigTiles) {
            bs.big_list[atomicAdd(bs.big_count, 1u)] = (uint32_t)vi;  // counted by bin_count_big_kernel
            has = false;
        }
        u = s.u;
        v = s.v;
        ca = s.ca;
        cd = s.cd;
    }
    const bool small = has && (tb.x1 - tb.x0 + 1) * (tb.y1 - tb.y0 + 1) <= kLaneTiles;
    uint64_t mask, lane_mask = 0;
    const uint32_t lane_cnt = small ? lane_bin(tb, u, v, ca, cd, p, lane_mask) : 0u;
    uint32_t cnt = warp_bin<false>(has && !small, tb, u, v, ca, cd, p, 0u, 0u, 0u, false, 0u, nullptr, nullptr, mask);
    if (small) {
        cnt = lane_cnt;
        mask = lane_mask;
    }
    if (active) {
        tile_counts[vi] = cnt;
        if (use_bs) bs.masks[vi] = mask;
    }
}

// counts in depth order: out[r] = tile_counts[order[r]]
__global__ void gather_counts_kernel(const uint32_t* __restrict__ order, const uint32_t* __restrict__ counts,
                                     int64_t n, uint32_t* __restrict__ out) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n) out[r] = counts[order[r]];
}

// Emission: a warp owns 32 consecutive depth ranks, whose entries form one
// contiguous range of the output.  When every splat of the warp has a
// recorded mask (a box of at most 64 tiles), the lanes expand their masks into
// shared memory and the warp stores the range with consecutive lanes on
// consecutive entries; otherwise each lane expands its own mask in place and
// large boxes are tested cooperatively.
constexpr int kEmitThreads = 64;
constexpr int kEmitStage = 32 * kMaskTiles;  // entries a warp of masked splats can produce

__global__ void __launch_bounds__(kEmitThreads) bin_emit_kernel(const float4* __restrict__ splats,
                                                               const uint32_t* __restrict__ order,
                                                               const uint32_t* __restrict__ offsets,
                                                               const uint32_t* __restrict__ tile_counts, int64_t nv,
                                                               RasterParams p, uint32_t* __restrict__ tile_keys,
                                                               uint32_t* __restrict__ vals, int64_t capacity,
                                                               int32_t* __restrict__ overflow, bool use_bs,
                                                               BinScratch bs) {
    __shared__ uint32_t skey[kEmitThreads / 32][kEmitStage], sval[kEmitThreads / 32][kEmitStage];
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    bool has = false;
    TileBox tb;
    tb.x0 = tb.x1 = tb.y0 = tb.y1 = 0;
    tb.exact = true;
    tb.m_cut = tb.s = 0.f;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    uint32_t vi = 0, cnt = 0, base = 0;
    uint64_t mask = 0;
    bool staged = true;  // this lane's entries (if any) can go through the warp's staging
    if (r < nv) {
        vi = order[r];
        cnt = tile_counts[vi];
        base = offsets[r];
        if (cnt > 0) {
            const bool over = (int64_t)base + cnt > capacity;
            if (over) atomicExch(overflow, 1);
            a = splats[3 * vi];
            b = splats[3 * vi + 1];
            has = splat_tile_box(a.x, a.y, a.z, a.w, b.x, b.y, b.z, p, tb);
            const int area = (tb.x1 - tb.x0 + 1) * (tb.y1 - tb.y0 + 1);
            if (has && use_bs && area > kBigTiles) {
                // listed by the counting pass: bin_emit_big_kernel writes it
                bs.big_base[vi] = over ? 0xffffffffu : base;
                has = false;
                staged = false;  // its range lies inside the warp's span: no staging for this warp
                cnt = 0;
            } else if (over) {
                has = false;
                staged = false;
                cnt = 0;
            } else {
                if (use_bs) mask = bs.masks[vi];
                staged = has && use_bs && area <= kMaskTiles && cnt <= (uint32_t)kMaskTiles;
            }
        }
    }
    const int w = tb.x1 - tb.x0 + 1;
    const uint32_t inv_w = (65536u + (uint32_t)w - 1u) / (uint32_t)w;  // t / w = (t * inv_w) >> 16 for t < 64
    if (__all_sync(kFull, staged)) {
        // the warp's range starts at the first rank's offset (lanes past nv and
        // splats without tiles add nothing)
        const uint32_t base0 = __shfl_sync(kFull, base, 0);
        const uint32_t end = cnt > 0 ? base + cnt : 0u;
        uint32_t total = end > base0 ? end - base0 : 0u;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) total = max(total, __shfl_xor_sync(kFull, total, o));
        if (cnt > 0) {
            const uint32_t local = base - base0;
            uint64_t mm = mask;
            for (uint32_t k = 0; k < cnt; ++k) {
                // bit t: tile t of the box, row-major (none missing when both passes agree)
                uint32_t key = 0xffffffffu, val = 0u;
                if (mm) {
                    const int t = __ffsll((long long)mm) - 1;
                    mm &= mm - 1;
                    const int ty = (int)(((uint32_t)t * inv_w) >> 16), tx = t - ty * w;
                    key = (uint32_t)((tb.y0 + ty) * p.tiles_x + tb.x0 + tx);
                    val = vi;
                }
                skey[warp][local + k] = key;
                sval[warp][local + k] = val;
            }
        }
        __syncwarp();
        for (uint32_t o = lane; o < total; o += 32) {
            tile_keys[base0 + o] = skey[warp][o];
            vals[base0 + o] = sval[warp][o];
        }
        return;
    }
    if (has) {
        const int area = w * (tb.y1 - tb.y0 + 1);
        if (use_bs && area <= kMaskTiles) {
            // small box: this lane expands its own recorded mask in place
            uint32_t k = 0;
            uint64_t mm = mask;
            while (mm && k < cnt) {
                const int t = __ffsll((long long)mm) - 1;
                mm &= mm - 1;
                const int ty = (int)(((uint32_t)t * inv_w) >> 16), tx = t - ty * w;
                tile_keys[base + k] = (uint32_t)((tb.y0 + ty) * p.tiles_x + tb.x0 + tx);
                vals[base + k] = vi;
                ++k;
            }
            for (; k < cnt; ++k) {
                tile_keys[base + k] = 0xffffffffu;
                vals[base + k] = 0u;
            }
            has = false;
        }
    } else {
        // no box (cannot happen after the count pass found tiles): keep the list well formed
        for (uint32_t k = 0; k < cnt; ++k) {
            tile_keys[base + k] = 0xffffffffu;
            vals[base + k] = 0u;
        }
    }
    // large boxes: the warp tests their tiles cooperatively
    uint64_t unused;
    warp_bin<true>(has, tb, a.x, a.y, a.z, b.y, p, base, cnt, vi, false, 0u, tile_keys, vals, unused);
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

// Compositing layout (CompositeLayout): pixels per thread, batch and register budget.
#ifndef GS_FWD_PX
#define GS_FWD_PX 2
#endif
#ifndef GS_FWD_MIN_CTAS
#define GS_FWD_MIN_CTAS 8
#endif
#ifndef GS_FWD_BATCH
#define GS_FWD_BATCH 256
#endif
using Layout = CompositeLayout<GS_FWD_PX>;
constexpr int kPx = GS_FWD_PX;
constexpr int kRenderThreads = Layout::threads;
constexpr int kPairs = Layout::pairs;
constexpr int kBatch = GS_FWD_BATCH;  // splats staged in shared memory per batch
static_assert(kBatch % kRenderThreads == 0 && kBatch % 32 == 0, "batch must tile the CTA");

// Dispatch order of the compositing CTAs: tiles by decreasing entry count
// (longest-processing-time-first), so the heaviest tiles start in the first
// wave and the kernel does not end on a few long tiles.  One CTA: counts are
// bucketed linearly against the largest count into kOrderBuckets buckets and
// counting-sorted (order within a bucket is arbitrary; every tile's result is
// independent of when it runs).
constexpr int kOrderThreads = 1024;
constexpr int kOrderBuckets = 1024;
static_assert(kOrderThreads == kOrderBuckets && kOrderThreads == 32 * 32, "one bucket per thread, 32 warps");

__global__ void __launch_bounds__(kOrderThreads) tile_order_kernel(const gs_tile_range* __restrict__ ranges,
                                                                   int32_t num_tiles, int32_t* __restrict__ order) {
    __shared__ int32_t start[kOrderBuckets];
    __shared__ int32_t warp_tot[kOrderThreads / 32];
    __shared__ int32_t smax;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    if (t == 0) smax = 0;
    start[t] = 0;
    __syncthreads();
    int mx = 0;
    for (int i = t; i < num_tiles; i += kOrderThreads) mx = max(mx, ranges[i].end - ranges[i].start);
    atomicMax(&smax, mx);
    __syncthreads();
    const int64_t cmax = smax;
    auto bucket = [&](int i) -> int {
        const int64_t c = max(ranges[i].end - ranges[i].start, 0);
        return cmax > 0 ? (kOrderBuckets - 1) - (int)(c * (kOrderBuckets - 1) / cmax) : 0;
    };
    for (int i = t; i < num_tiles; i += kOrderThreads) atomicAdd(&start[bucket(i)], 1);
    __syncthreads();
    // exclusive scan of the bucket sizes (one bucket per thread)
    const int v = start[t];
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int w = warp_tot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(kFull, w, o);
            if (lane >= o) w += y;
        }
        warp_tot[lane] = w;  // inclusive per-warp totals
    }
    __syncthreads();
    start[t] = incl - v + (warp > 0 ? warp_tot[warp - 1] : 0);
    __syncthreads();
    for (int i = t; i < num_tiles; i += kOrderThreads) order[atomicAdd(&start[bucket(i)], 1)] = i;
}

// ---------------------------------------------------------------- compositing
// One CTA per 16x16 tile, pixels laid out by CompositeLayout.  Splats are
// staged kBatch at a time in shared memory and read back as broadcasts; each
// warp first tests which staged splats can reach its pixel block, then walks
// only those.  A warp skips the rest of a batch once all its pixels are
// saturated (T < t_min) and the CTA stops when all 256 are.
__device__ __forceinline__ float pixel_loss(int loss_mode, const void* target, int64_t pix, float cr, float cg,
                                            float cb) {
    if (loss_mode == GS_LOSS_L1_U8) {
        const uint8_t* t8 = static_cast<const uint8_t*>(target) + 3 * pix;
        return fabsf(cr - __fdiv_rn((float)t8[0], 255.0f)) + fabsf(cg - __fdiv_rn((float)t8[1], 255.0f)) +
               fabsf(cb - __fdiv_rn((float)t8[2], 255.0f));
    }
    if (loss_mode == GS_LOSS_L1_F32) {
        const float* tf = static_cast<const float*>(target) + 3 * pix;
        return fabsf(cr - tf[0]) + fabsf(cg - tf[1]) + fabsf(cb - tf[2]);
    }
    if (loss_mode == GS_LOSS_MEAN) return cr + cg + cb;
    return 0.f;
}

// GS_FWD_MIN_CTAS > 0 asks the register allocator for that many resident CTAs per SM
#if GS_FWD_MIN_CTAS > 0
#define GS_FWD_BOUNDS __launch_bounds__(kRenderThreads, GS_FWD_MIN_CTAS)
#else
#define GS_FWD_BOUNDS __launch_bounds__(kRenderThreads)
#endif
// kCount: the same compositing, but instead of writing the image it adds the
// number of (pixel, splat) pairs that took part to *pairs (a diagnostic of the
// work the compositing kernels do; not on the training path).
// kMask: each splat's clipped alpha is multiplied by the last float of its
// record (gs_apply_sorted_mask; mlx_gsplat/rendering.py:289-290).
template <bool kCount, bool kMask>
__global__ void GS_FWD_BOUNDS render_fwd_kernel(
    const gs_tile_range* __restrict__ ranges, const int32_t* __restrict__ tile_order, const uint32_t* __restrict__ vals, const float4* __restrict__ splats,
    int64_t nv, RasterParams p, float* __restrict__ out_color, float* __restrict__ out_alpha, float* __restrict__ final_T,
    int32_t* __restrict__ n_contrib, int loss_mode, const void* __restrict__ target,
    float* __restrict__ loss_partials, unsigned long long* __restrict__ pairs) {
    __shared__ float4 s0[kBatch], s1[kBatch], s2[kBatch];
    __shared__ float red[kRenderThreads / 32];
    const int tile = tile_order ? tile_order[blockIdx.x] : (int)blockIdx.x;
    if (tile < 0 || tile >= p.tiles_x * p.tiles_y) return;  // uniform over the CTA
    const int tx = tile % p.tiles_x, ty = tile / p.tiles_x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bx0 = tx * kTile + Layout::block_x(warp), by0 = ty * kTile + Layout::block_y(warp);  // warp block
    const int pi = bx0 + Layout::col(lane);
    const float px = (float)pi * p.sx + p.hsx;
    const gs_tile_range rg = ranges[tile];

    // pixel pairs: pair q holds the thread's pixels 2q and 2q + 1.  A pixel
    // takes part while T >= t_min; pixels outside the image start with T = -1
    // (never written back), so they never take part.
    float2 py[kPairs], T[kPairs], cr[kPairs], cg[kPairs], cb[kPairs], A[kPairs];
    int last[kPx];
    unsigned npairs = 0;
    const float t_min = p.t_min;
    const float t_out = fminf(-1.f, t_min - 1.f);
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
        const int pj = by0 + Layout::row(lane, 2 * q), pj1 = by0 + Layout::row(lane, 2 * q + 1);
        py[q] = make_float2((float)pj * p.sy + p.hsy, (float)pj1 * p.sy + p.hsy);
        T[q] = make_float2(pi < p.rw && pj < p.rh ? 1.f : t_out, pi < p.rw && pj1 < p.rh ? 1.f : t_out);
        cr[q] = cg[q] = cb[q] = A[q] = f2(0.f);
        last[2 * q] = last[2 * q + 1] = 0;
    }
    auto all_dead = [&]() {
        bool d = true;
#pragma unroll
        for (int q = 0; q < kPairs; ++q) d &= (T[q].x < t_min) & (T[q].y < t_min);
        return d;
    };
    for (int b = rg.start; b < rg.end; b += kBatch) {
        if (__syncthreads_count(all_dead()) == kRenderThreads) break;
#pragma unroll
        for (int h = 0; h < kBatch / kRenderThreads; ++h) {
            const int j = threadIdx.x + h * kRenderThreads;
            const int e = b + j;
            if (e < rg.end) {
                const uint32_t vr = vals[e];
                const uint32_t vi = vr < (uint64_t)nv ? vr : 0u;
                s0[j] = splats[3 * vi];
                s1[j] = splats[3 * vi + 1];
                s2[j] = splats[3 * vi + 2];
            }
        }
        __syncthreads();
        const int cnt = min(kBatch, rg.end - b);
        const int base1 = b - rg.start + 1;
        // which staged splats can reach this warp's pixel block at all
        bool warp_done = __all_sync(kFull, all_dead());
        unsigned hits[kBatch / 32];
#pragma unroll
        for (int i = 0; i < kBatch / 32; ++i) {
            const int k = 32 * i + lane;
            const bool h = !warp_done && k < cnt &&
                           splat_hits_block(s0[k], s1[k], s2[k].z, bx0, bx0 + Layout::cols - 1, by0,
                                            by0 + Layout::rows - 1, p);
            hits[i] = __ballot_sync(kFull, h);
        }
        // the saturation vote runs once per word of 32 staged splats: a pixel
        // that saturates inside a word stops taking part at once (T < t_min)
#pragma unroll
        for (int i = 0; i < kBatch / 32; ++i) {
            if (warp_done) break;
            unsigned bits = hits[i];
            while (bits) {
                const int k = 32 * i + __ffs(bits) - 1;
                bits &= bits - 1;
                const float4 q0 = s0[k], q1 = s1[k], q2 = s2[k];
                const float x = px - q0.x;
                const float ax = q0.z * x, cx = q1.x * x;
                const int idx1 = base1 + k;
#pragma unroll
                for (int q = 0; q < kPairs; ++q) {
                    // Branch-free front-to-back step: a pixel that is saturated or
                    // out of the splat's reach gets alpha = 0 (T, colour unchanged).
                    const float2 m = pair_quad(__fadd2_rn(py[q], f2(-q0.y)), x, ax, cx, q0.w, q1.y);
                    const float2 og = __fmul2_rn(f2(q1.z), pair_falloff(m));
                    const bool v0 = T[q].x >= t_min && m.x <= q2.z, v1 = T[q].y >= t_min && m.y <= q2.z;
                    float2 al = make_float2(v0 ? fminf(og.x, 0.99f) : 0.f, v1 ? fminf(og.y, 0.99f) : 0.f);
                    if constexpr (kMask) al = __fmul2_rn(al, f2(q2.w));
                    const float2 w = __fmul2_rn(al, T[q]);
                    cr[q] = __ffma2_rn(w, f2(q1.w), cr[q]);
                    cg[q] = __ffma2_rn(w, f2(q2.x), cg[q]);
                    cb[q] = __ffma2_rn(w, f2(q2.y), cb[q]);
                    A[q] = __fadd2_rn(A[q], w);
                    T[q] = __fmul2_rn(T[q], __ffma2_rn(al, f2(-1.f), f2(1.f)));  // T (1 - alpha)
                    last[2 * q] = v0 ? idx1 : last[2 * q];
                    last[2 * q + 1] = v1 ? idx1 : last[2 * q + 1];
                    if constexpr (kCount) npairs += (unsigned)v0 + (unsigned)v1;
                }
            }
            warp_done = __all_sync(kFull, all_dead());
        }
        __syncthreads();
    }

    if constexpr (kCount) {
        const unsigned long long w = (unsigned long long)__reduce_add_sync(kFull, npairs);
        if (lane == 0 && w) atomicAdd(pairs, w);
        return;
    }
    float lsum = 0.f;
#pragma unroll
    for (int k = 0; k < kPx; ++k) {
        const int pj = by0 + Layout::row(lane, k);
        const int q = k >> 1;
        const bool hi = k & 1;
        if (pi < p.rw && pj < p.rh) {
            const int64_t pix = (int64_t)pj * p.rw + pi;
            const float r = hi ? cr[q].y : cr[q].x, g = hi ? cg[q].y : cg[q].x, bl = hi ? cb[q].y : cb[q].x;
            out_color[3 * pix + 0] = r;
            out_color[3 * pix + 1] = g;
            out_color[3 * pix + 2] = bl;
            out_alpha[pix] = hi ? A[q].y : A[q].x;
            final_T[pix] = hi ? T[q].y : T[q].x;
            n_contrib[pix] = last[k];
            lsum += pixel_loss(loss_mode, target, pix, r, g, bl);
        }
    }
    if (loss_mode != GS_LOSS_NONE) {
        lsum = warp_sum(lsum);
        if (lane == 0) red[warp] = lsum;
        __syncthreads();
        if (threadIdx.x == 0) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kRenderThreads / 32; ++w) t += red[w];
            loss_partials[tile] = t;
        }
    }
}

}  // namespace gs

using namespace gs;

extern "C" size_t gs_bin_scratch_bytes(int64_t num_visible) { return bin_scratch_bytes(num_visible); }

extern "C" int gs_project_forward(const gs_gaussians* g, const int32_t* ids, int64_t num_visible,
                                  const gs_camera* cam, const gs_raster_settings* rs, float* splats,
                                  uint32_t* depth_keys, uint32_t* tile_counts, void* bin_scratch,
                                  gs_stream_t stream) {
    GS_REQUIRE(g && cam, "project_forward: null descriptor");
    GS_REQUIRE(num_visible >= 0, "project_forward: negative count");
    if (num_visible == 0) return GS_OK;
    GS_REQUIRE(ids && splats && depth_keys && tile_counts && g->means && g->quats && g->scales && g->opac && g->colors,
               "project_forward: null pointer");
    GS_REQUIRE(g->colors_dim >= 3, "project_forward: colors_dim must be >= 3");
    GS_REQUIRE(g->sh_mode == GS_SH_REFERENCE || g->sh_mode == GS_SH_FULL, "project_forward: bad sh_mode");
    GS_REQUIRE(aligned16(splats), "project_forward: splats must be 16-byte aligned");
    GS_REQUIRE(cam->render_width > 0 && cam->render_height > 0 && cam->width > 0 && cam->height > 0,
               "project_forward: bad image size");
    const RasterParams p = make_raster_params(*cam, rs);
    const bool use_bs = bin_scratch != nullptr;
    const BinScratch bs = use_bs ? bin_scratch_layout(bin_scratch, num_visible) : BinScratch{};
    if (use_bs) cudaMemsetAsync(bs.big_count, 0, sizeof(uint32_t), (cudaStream_t)stream);
    const int deg = sh_kernel_degree(*g);
    auto kernel = deg == 3   ? (slab_rows<3>(*g) ? project_fwd_kernel<true, 3> : project_fwd_kernel<false, 3>)
                  : deg == 2 ? (slab_rows<2>(*g) ? project_fwd_kernel<true, 2> : project_fwd_kernel<false, 2>)
                             : (slab_rows<1>(*g) ? project_fwd_kernel<true, 1> : project_fwd_kernel<false, 1>);
    kernel<<<grid_for(num_visible, 128), 128, 0, (cudaStream_t)stream>>>(*g, ids, num_visible, p,
                                                                        reinterpret_cast<float4*>(splats),
                                                                        depth_keys, tile_counts, use_bs, bs);
    if (use_bs) {
        GS_TRY(check_launch("project_fwd_kernel"));
        return launch_pdl("bin_count_big_kernel", bin_count_big_kernel, dim3(kBigGrid), dim3(kBigThreads),
                          (cudaStream_t)stream, reinterpret_cast<const float4*>(splats), bs, p, tile_counts);
    }
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
    return scan_exclusive(gathered, offsets, num_visible, p, scan_scratch_bytes(num_visible), (cudaStream_t)stream,
                          true);
}

extern "C" int gs_bin_emit(const float* splats, const uint32_t* order, const uint32_t* offsets,
                           const uint32_t* tile_counts, int64_t num_visible, const gs_camera* cam,
                           const gs_raster_settings* rs, uint32_t* tile_keys, uint32_t* entry_vals, int64_t capacity,
                           int32_t* overflow_flag, void* bin_scratch, gs_stream_t stream) {
    GS_REQUIRE(cam, "bin_emit: null camera");
    if (num_visible == 0) return GS_OK;
    GS_REQUIRE(splats && order && offsets && tile_counts && overflow_flag, "bin_emit: null pointer");
    GS_REQUIRE(capacity == 0 || (tile_keys && entry_vals), "bin_emit: null output");
    const RasterParams p = make_raster_params(*cam, rs);
    const bool use_bs = bin_scratch != nullptr;
    const BinScratch bs = use_bs ? bin_scratch_layout(bin_scratch, num_visible) : BinScratch{};
    bin_emit_kernel<<<grid_for(num_visible, kEmitThreads), kEmitThreads, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const float4*>(splats), order, offsets, tile_counts, num_visible, p, tile_keys, entry_vals,
        capacity, overflow_flag, use_bs, bs);
    if (use_bs) {
        GS_TRY(check_launch("bin_emit_kernel"));
        return launch_pdl("bin_emit_big_kernel", bin_emit_big_kernel, dim3(kBigGrid), dim3(kBigThreads),
                          (cudaStream_t)stream, reinterpret_cast<const float4*>(splats), bs, tile_counts, p, tile_keys,
                          entry_vals);
    }
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

extern "C" int gs_tile_order(const gs_tile_range* ranges, int32_t num_tiles, int32_t* order, gs_stream_t stream) {
    GS_REQUIRE(ranges && order && num_tiles > 0, "tile_order: bad arguments");
    tile_order_kernel<<<1, kOrderThreads, 0, (cudaStream_t)stream>>>(ranges, num_tiles, order);
    return check_launch("tile_order_kernel");
}

extern "C" int gs_render_forward(const gs_tile_range* ranges, const int32_t* tile_order, const uint32_t* entry_vals,
                                 const float* splats,
                                 int64_t num_visible, const gs_camera* cam, const gs_raster_settings* rs,
                                 float* out_color,
                                 float* out_alpha, float* final_T, int32_t* n_contrib, int loss_mode,
                                 const void* target, float* loss_partials, gs_stream_t stream) {
    GS_REQUIRE(cam && ranges && out_color && out_alpha && final_T && n_contrib, "render_forward: null pointer");
    GS_REQUIRE(loss_mode >= GS_LOSS_NONE && loss_mode <= GS_LOSS_MEAN, "render_forward: bad loss mode");
    GS_REQUIRE(!rs || rs->transmittance_min <= 1.f, "render_forward: transmittance_min must be <= 1");
    GS_REQUIRE(loss_mode == GS_LOSS_NONE || loss_partials, "render_forward: loss_partials required");
    GS_REQUIRE(loss_mode == GS_LOSS_NONE || loss_mode == GS_LOSS_MEAN || target, "render_forward: target required");
    const RasterParams p = make_raster_params(*cam, rs);
    const int tiles = p.tiles_x * p.tiles_y;
    auto kernel = p.masked ? render_fwd_kernel<false, true> : render_fwd_kernel<false, false>;
    kernel<<<tiles, kRenderThreads, 0, (cudaStream_t)stream>>>(
        ranges, tile_order, entry_vals, reinterpret_cast<const float4*>(splats), num_visible, p, out_color, out_alpha,
        final_T, n_contrib, loss_mode, target, loss_partials, nullptr);
    return check_launch("render_fwd_kernel");
}

extern "C" int gs_render_pair_count(const gs_tile_range* ranges, const int32_t* tile_order,
                                    const uint32_t* entry_vals, const float* splats, int64_t num_visible,
                                    const gs_camera* cam, const gs_raster_settings* rs,
                                    unsigned long long* pairs, gs_stream_t stream) {
    GS_REQUIRE(cam && ranges && pairs, "render_pair_count: null pointer");
    GS_REQUIRE(aligned16(splats), "render_pair_count: splats must be 16-byte aligned");
    GS_REQUIRE(!rs || rs->transmittance_min <= 1.f, "render_pair_count: transmittance_min must be <= 1");
    const RasterParams p = make_raster_params(*cam, rs);
    const int tiles = p.tiles_x * p.tiles_y;
    auto kernel = p.masked ? render_fwd_kernel<true, true> : render_fwd_kernel<true, false>;
    kernel<<<tiles, kRenderThreads, 0, (cudaStream_t)stream>>>(
        ranges, tile_order, entry_vals, reinterpret_cast<const float4*>(splats), num_visible, p, nullptr, nullptr,
        nullptr, nullptr, GS_LOSS_NONE, nullptr, nullptr, pairs);
    return check_launch("render_fwd_kernel<count>");
}

// Record r of depth rank j (r = order[j]) gets mask[j] (clamped to [0, 1]) as
// its alpha multiplier and the contribution cut of opacity * mask.
__global__ void apply_sorted_mask_kernel(float4* __restrict__ splats, const int32_t* __restrict__ order,
                                         const float* __restrict__ mask, int64_t nv, RasterParams p) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= nv) return;
    const int32_t r = order[j];
    if (r < 0 || r >= nv) return;
    const float mk = fminf(fmaxf(mask[j], 0.f), 1.f);
    const float opac = splats[3 * r + 1].z;
    float4 c = splats[3 * r + 2];
    c.z = pair_cut(opac * mk, p);
    c.w = mk;
    splats[3 * r + 2] = c;
}

extern "C" int gs_apply_sorted_mask(float* splats, const int32_t* order, const float* mask, int64_t num_visible,
                                    const gs_raster_settings* rs, gs_stream_t stream) {
    GS_REQUIRE(num_visible >= 0, "apply_sorted_mask: negative count");
    if (num_visible == 0) return GS_OK;
    GS_REQUIRE(splats && order && mask, "apply_sorted_mask: null pointer");
    GS_REQUIRE(aligned16(splats), "apply_sorted_mask: splats must be 16-byte aligned");
    gs_camera cam = {};
    cam.width = cam.height = cam.render_width = cam.render_height = 1;
    const RasterParams p = make_raster_params(cam, rs);  // only the cutoff is used
    apply_sorted_mask_kernel<<<grid_for(num_visible, 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<float4*>(splats), order, mask, num_visible, p);
    return check_launch("apply_sorted_mask_kernel");
}
