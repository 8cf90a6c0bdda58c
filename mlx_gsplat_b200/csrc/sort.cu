// Stable LSD radix sort of (uint32 key, uint32 value) pairs, 8 bits per pass.
//
// Each pass: (1) per 2048-key tile, a 256-bin digit histogram written
// digit-major; (2) a device-wide exclusive scan of those counts, which gives
// every (digit, tile) its global output offset; (3) per tile, a stable local
// rank of each key within its digit — warps own contiguous runs of keys and
// rank them 32 at a time (the lanes sharing a digit found with one ballot per
// digit bit) plus per-warp digit counters in shared memory, then a cross-warp
// prefix — the tile staged in shared memory
// in sorted order, and written out in that order to offset + rank, so each
// digit's run of keys is stored by consecutive threads.
// There is no inter-CTA waiting (reduce-then-scan), so no kernel can spin.
#include "common.cuh"
#include "scan.cuh"

namespace gs {

constexpr int kSortThreads = 256;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;  // 2048 keys
constexpr int kBins = 256;

__global__ void __launch_bounds__(kSortThreads) radix_upsweep(const uint32_t* __restrict__ keys, int64_t n, int shift,
                                                              uint32_t mask, uint32_t* __restrict__ counts,
                                                              int64_t n_tiles) {
    pdl_wait();
    __shared__ uint32_t hist[kBins];
    hist[threadIdx.x] = 0;
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * kSortTile;
#pragma unroll
    for (int k = 0; k < kSortItems; ++k) {
        const int64_t i = base + (int64_t)k * kSortThreads + threadIdx.x;
        if (i < n) atomicAdd(&hist[(__ldg(keys + i) >> shift) & mask], 1u);
    }
    __syncthreads();
    counts[(int64_t)threadIdx.x * n_tiles + blockIdx.x] = hist[threadIdx.x];
}

// Lanes of the warp whose keys have the same digit (``bits`` low bits of d)
// and the same validity: one ballot per digit bit.  The warp-wide
// match.any instruction does the same on the address-divergence pipe, which
// limited this kernel (that pipe 67 % busy; with ballots and 5 resident CTAs
// per SM the 3.6 M-entry tile sort of the 1 M-Gaussian step took 12 us less).
#ifndef GS_SORT_BALLOT_MATCH
#define GS_SORT_BALLOT_MATCH 1
#endif
__device__ __forceinline__ unsigned digit_peers(int d, bool valid, int bits) {
#if GS_SORT_BALLOT_MATCH
    const unsigned vb = __ballot_sync(kFull, valid);
    unsigned peers = valid ? vb : ~vb;
    for (int b = 0; b < bits; ++b) {
        const bool on = (d >> b) & 1;
        const unsigned bal = __ballot_sync(kFull, on);
        peers &= on ? bal : ~bal;
    }
    return peers;
#else
    return __match_any_sync(kFull, valid ? d : kBins);
#endif
}

#ifndef GS_SORT_MIN_CTAS
#define GS_SORT_MIN_CTAS 5
#endif
__global__ void __launch_bounds__(kSortThreads, GS_SORT_MIN_CTAS) radix_downsweep(const uint32_t* __restrict__ keys_in,
                                                                const uint32_t* __restrict__ vals_in,
                                                                uint32_t* __restrict__ keys_out,
                                                                uint32_t* __restrict__ vals_out, int64_t n, int shift,
                                                                uint32_t mask, const uint32_t* __restrict__ offsets,
                                                                int64_t n_tiles) {
    pdl_wait();
    __shared__ uint32_t goff[kBins];
    __shared__ uint32_t lstart[kBins];  // tile-local start of each digit
    __shared__ uint32_t wtot[kSortWarps];
    __shared__ uint32_t wcnt[kSortWarps][kBins];
    __shared__ uint32_t skey[kSortTile], sval[kSortTile];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    goff[threadIdx.x] = offsets[(int64_t)threadIdx.x * n_tiles + blockIdx.x];
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) wcnt[w][threadIdx.x] = 0;
    __syncthreads();

    const int64_t tbase = (int64_t)blockIdx.x * kSortTile;
    const int64_t wbase = tbase + (int64_t)warp * (32 * kSortItems);
    const unsigned lt = lanemask_lt();
    const int bits = __popc(mask);
    uint32_t key[kSortItems], val[kSortItems], rank[kSortItems];
    int dig[kSortItems];
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
        const int64_t i = wbase + r * 32 + lane;
        const bool valid = i < n;
        key[r] = valid ? keys_in[i] : 0u;
        val[r] = valid ? (vals_in ? vals_in[i] : (uint32_t)i) : 0u;  // no values: the input positions
        const int d = valid ? (int)((key[r] >> shift) & mask) : kBins;  // invalid lanes form their own group
        dig[r] = d;
        const unsigned peers = digit_peers(d, valid, bits);
        const uint32_t before = __popc(peers & lt);
        const uint32_t prior = valid ? wcnt[warp][d] : 0u;
        __syncwarp();
        if (valid && before == 0) wcnt[warp][d] = prior + __popc(peers);
        __syncwarp();
        rank[r] = prior + before;
    }
    __syncthreads();
    // per digit (one per thread): cross-warp prefix, then the tile-local
    // digit starts by a block-wide exclusive scan of the digit totals
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
        const uint32_t c = wcnt[w][threadIdx.x];
        wcnt[w][threadIdx.x] = run;
        run += c;
    }
    uint32_t inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) wtot[warp] = inc;
    __syncthreads();
    uint32_t wpre = 0;
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) wpre += w < warp ? wtot[w] : 0u;
    lstart[threadIdx.x] = wpre + inc - run;
    __syncthreads();
    // stage the tile in sorted order, then write it out in that order: each
    // digit's keys go to consecutive global positions from consecutive threads
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
        const int d = dig[r];
        if (d < kBins) {
            const uint32_t lp = lstart[d] + wcnt[warp][d] + rank[r];
            skey[lp] = key[r];
            sval[lp] = val[r];
        }
    }
    __syncthreads();
    const int tile_n = (int)(n - tbase < kSortTile ? n - tbase : kSortTile);
#pragma unroll
    for (int r = 0; r < kSortItems; ++r) {
        const int j = r * kSortThreads + threadIdx.x;
        if (j < tile_n) {
            const uint32_t k = skey[j];
            const int d = (int)((k >> shift) & mask);
            const uint32_t pos = goff[d] + (uint32_t)j - lstart[d];
            keys_out[pos] = k;
            vals_out[pos] = sval[j];
        }
    }
}

static int64_t sort_tiles(int64_t n) { return (n + kSortTile - 1) / kSortTile; }

size_t radix_sort_scratch_bytes(int64_t n) {
    const int64_t tiles = sort_tiles(n);
    const int64_t nc = tiles * kBins;
    size_t b = 0;
    b += align_up((size_t)n * 4, 256) * 2;          // alternate keys + values
    b += align_up((size_t)(nc + 1) * 4, 256);       // counts -> offsets (+ total)
    b += align_up(scan_scratch_bytes(nc), 256);
    return b + 256;
}

int radix_sort_pairs(const uint32_t* keys_in, const uint32_t* vals_in, uint32_t* keys_out, uint32_t* vals_out,
                     int64_t n, int begin_bit, int end_bit, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
    GS_REQUIRE(n >= 0 && n < (int64_t)1 << 31, "radix_sort: n out of range");
    GS_REQUIRE(0 <= begin_bit && begin_bit <= end_bit && end_bit <= 32, "radix_sort: bad bit range");
    GS_REQUIRE(keys_out != keys_in && vals_out != vals_in, "radix_sort: output must not alias input");
    GS_REQUIRE(scratch_bytes >= radix_sort_scratch_bytes(n), "radix_sort: scratch too small");
    if (n == 0) return GS_OK;
    const int passes = (end_bit - begin_bit + 7) / 8;
    if (passes == 0) {
        GS_REQUIRE(vals_in, "radix_sort: an empty bit range needs vals_in");
        cudaMemcpyAsync(keys_out, keys_in, n * 4, cudaMemcpyDeviceToDevice, stream);
        cudaMemcpyAsync(vals_out, vals_in, n * 4, cudaMemcpyDeviceToDevice, stream);
        return check_launch("radix_sort copy", 0);
    }
    const int64_t tiles = sort_tiles(n);
    const int64_t nc = tiles * kBins;
    char* p = static_cast<char*>(scratch);
    p = reinterpret_cast<char*>(align_up(reinterpret_cast<uintptr_t>(p), 256));
    uint32_t* alt_k = reinterpret_cast<uint32_t*>(p);
    p += align_up((size_t)n * 4, 256);
    uint32_t* alt_v = reinterpret_cast<uint32_t*>(p);
    p += align_up((size_t)n * 4, 256);
    uint32_t* counts = reinterpret_cast<uint32_t*>(p);
    p += align_up((size_t)(nc + 1) * 4, 256);
    void* scan_scratch = p;
    const size_t scan_bytes = scan_scratch_bytes(nc);

    const uint32_t* src_k = keys_in;
    const uint32_t* src_v = vals_in;
    for (int pass = 0; pass < passes; ++pass) {
        const int shift = begin_bit + 8 * pass;
        const int bits = end_bit - shift < 8 ? end_bit - shift : 8;
        const uint32_t mask = (1u << bits) - 1u;
        const bool to_out = ((passes - 1 - pass) % 2) == 0;
        uint32_t* dk = to_out ? keys_out : alt_k;
        uint32_t* dv = to_out ? vals_out : alt_v;
        // every kernel after the first follows one of this sort's own kernels:
        // programmatic dependent launches (each kernel waits for its predecessor)
        if (pass == 0) {
            radix_upsweep<<<(unsigned)tiles, kSortThreads, 0, stream>>>(src_k, n, shift, mask, counts, tiles);
            GS_TRY(check_launch("radix_upsweep"));
        } else {
            GS_TRY(launch_pdl("radix_upsweep", radix_upsweep, dim3((unsigned)tiles), dim3(kSortThreads), stream, src_k,
                              n, shift, mask, counts, tiles));
        }
        GS_TRY(scan_exclusive(counts, counts, nc, scan_scratch, scan_bytes, stream, true));
        GS_TRY(launch_pdl("radix_downsweep", radix_downsweep, dim3((unsigned)tiles), dim3(kSortThreads), stream, src_k,
                          src_v, dk, dv, n, shift, mask, (const uint32_t*)counts, tiles));
        src_k = dk;
        src_v = dv;
    }
    return GS_OK;
}

}  // namespace gs

extern "C" size_t gs_radix_sort_scratch_bytes(int64_t n) { return gs::radix_sort_scratch_bytes(n); }

extern "C" int gs_radix_sort_pairs(const uint32_t* keys_in, const uint32_t* vals_in, uint32_t* keys_out,
                                   uint32_t* vals_out, int64_t n, int begin_bit, int end_bit, void* scratch,
                                   size_t scratch_bytes, gs_stream_t stream) {
    GS_REQUIRE(keys_in && keys_out && vals_out && scratch, "radix_sort: null pointer");
    return gs::radix_sort_pairs(keys_in, vals_in, keys_out, vals_out, n, begin_bit, end_bit, scratch, scratch_bytes,
                                (cudaStream_t)stream);
}
