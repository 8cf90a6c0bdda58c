// Device-wide exclusive prefix sum of uint32 values (reduce, then scan):
//   0. up to GS_SCAN_SMALL_MAX values: one CTA, one launch (scan_small); else
//   1. per 2048-element tile: tile sums
//   2. one CTA: exclusive scan of the tile sums (loops when there are many)
//   3. per tile: block scan plus the tile's offset.
// No inter-CTA waiting, so nothing can spin.  The second and third kernels
// (and the first, when the caller's previous operation was one of this
// library's kernels) use programmatic dependent launches.
#include "common.cuh"
#include "scan.cuh"

namespace gs {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t x, uint32_t* smem_warp, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) smem_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < (int)(blockDim.x >> 5) ? smem_warp[lane] : 0u;
        uint32_t wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t y = __shfl_up_sync(kFull, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < (int)(blockDim.x >> 5)) smem_warp[lane] = wi - w;
        if (lane == (int)(blockDim.x >> 5) - 1) smem_warp[32] = wi;
    }
    __syncthreads();
    const uint32_t res = smem_warp[warp] + inc - x;
    if (total) *total = smem_warp[32];
    __syncthreads();
    return res;
}

__global__ void __launch_bounds__(kScanThreads) scan_tile_sums(const uint32_t* __restrict__ in, int64_t n,
                                                               uint32_t* __restrict__ tile_sums) {
    pdl_wait();
    __shared__ uint32_t sw[33];
    const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
    uint32_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
        if (base + k < n) s += in[base + k];
    uint32_t tot;
    block_exclusive_scan(s, sw, &tot);
    if (threadIdx.x == 0) tile_sums[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(kScanThreads) scan_tile_offsets(uint32_t* __restrict__ sums, int64_t n_tiles,
                                                                  uint32_t* __restrict__ total_out) {
    pdl_wait();
    __shared__ uint32_t sw[33];
    uint32_t carry = 0;
    for (int64_t base = 0; base < n_tiles; base += kScanThreads) {
        const int64_t i = base + threadIdx.x;
        const uint32_t x = i < n_tiles ? sums[i] : 0u;
        uint32_t tot;
        const uint32_t ex = block_exclusive_scan(x, sw, &tot);
        if (i < n_tiles) sums[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0 && total_out) *total_out = carry;
}

__global__ void __launch_bounds__(kScanThreads) scan_tiles(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                                           int64_t n, const uint32_t* __restrict__ tile_offsets) {
    pdl_wait();
    __shared__ uint32_t sw[33];
    const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
    uint32_t v[kScanItems];
    uint32_t s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = base + k < n ? in[base + k] : 0u;
        s += v[k];
    }
    uint32_t run = block_exclusive_scan(s, sw, nullptr) + tile_offsets[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        if (base + k < n) out[base + k] = run;
        run += v[k];
    }
}

// Small inputs: one CTA scans everything, kSmallChunk elements per round
// (a contiguous run of kScanItems per thread), carrying the running total
// between rounds; one launch instead of three.  Measured on the 1 M-Gaussian
// training step: the cull's scan of ~500 chunk counts 3.5 us faster; the
// depth sort's scans of 15k-63k counts were slower on one CTA (0.081 ->
// 0.102 ms and 0.090 -> 0.248 ms per sort), hence the small limit.
#ifndef GS_SCAN_SMALL_MAX
#define GS_SCAN_SMALL_MAX 4096
#endif
constexpr int kSmallThreads = 1024;
constexpr int kSmallChunk = kSmallThreads * kScanItems;

__global__ void __launch_bounds__(kSmallThreads) scan_small(const uint32_t* __restrict__ in, uint32_t* __restrict__ out,
                                                            int64_t n) {
    pdl_wait();
    __shared__ uint32_t sw[33];
    uint32_t carry = 0;
    for (int64_t c = 0; c < n; c += kSmallChunk) {
        const int64_t base = c + (int64_t)threadIdx.x * kScanItems;
        uint32_t v[kScanItems];
        uint32_t s = 0;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            v[k] = base + k < n ? in[base + k] : 0u;
            s += v[k];
        }
        uint32_t tot;
        uint32_t run = carry + block_exclusive_scan(s, sw, &tot);
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            if (base + k < n) out[base + k] = run;
            run += v[k];
        }
        carry += tot;
    }
    if (threadIdx.x == 0) out[n] = carry;
}

size_t scan_scratch_bytes(int64_t n) {
    const int64_t tiles = (n + kScanTile - 1) / kScanTile;
    return (size_t)((tiles + 4) * sizeof(uint32_t) + 256);
}

int scan_exclusive(const uint32_t* in, uint32_t* out, int64_t n, void* scratch, size_t scratch_bytes,
                   cudaStream_t stream, bool after_kernel) {
    GS_REQUIRE(n >= 0, "scan: negative n");
    GS_REQUIRE(scratch_bytes >= scan_scratch_bytes(n), "scan: scratch too small");
    if (n == 0) {
        cudaMemsetAsync(out, 0, sizeof(uint32_t), stream);
        return check_launch("scan(n=0)", 0);
    }
    if (n <= GS_SCAN_SMALL_MAX) {
        if (after_kernel)
            return launch_pdl("scan_small", scan_small, dim3(1), dim3(kSmallThreads), stream, in, out, n);
        scan_small<<<1, kSmallThreads, 0, stream>>>(in, out, n);
        return check_launch("scan_small");
    }
    const int64_t tiles = (n + kScanTile - 1) / kScanTile;
    uint32_t* sums = reinterpret_cast<uint32_t*>(scratch);
    if (after_kernel) {
        GS_TRY(launch_pdl("scan_tile_sums", scan_tile_sums, dim3((unsigned)tiles), dim3(kScanThreads), stream, in, n,
                          sums));
    } else {
        scan_tile_sums<<<(unsigned)tiles, kScanThreads, 0, stream>>>(in, n, sums);
        GS_TRY(check_launch("scan_tile_sums"));
    }
    GS_TRY(launch_pdl("scan_tile_offsets", scan_tile_offsets, dim3(1), dim3(kScanThreads), stream, sums, tiles,
                      out + n));
    return launch_pdl("scan_tiles", scan_tiles, dim3((unsigned)tiles), dim3(kScanThreads), stream, in, out, n,
                      (const uint32_t*)sums);
}

}  // namespace gs

extern "C" size_t gs_scan_scratch_bytes(int64_t n) { return gs::scan_scratch_bytes(n); }

extern "C" int gs_exclusive_scan_u32(const uint32_t* in, uint32_t* out, int64_t n, void* scratch,
                                     size_t scratch_bytes, gs_stream_t stream) {
    GS_REQUIRE(in && out && scratch, "scan: null pointer");
    return gs::scan_exclusive(in, out, n, scratch, scratch_bytes, (cudaStream_t)stream);
}
