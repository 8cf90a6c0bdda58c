// Frustum + opacity cull with order-preserving stream compaction
// (frustum_culling_mlx, mlx_gsplat/rendering.py:41-94).
//
// Pass 1: one bit per active id (warp ballot) and a count per 2048-id chunk.
// Pass 2: exclusive scan of the chunk counts.
// Pass 3: each chunk writes its surviving ids in ascending order.
// Reads 16 bytes per id (means + opacity), writes 4 bytes per survivor.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "scan.cuh"

namespace gs {

constexpr int kCullThreads = 256;
constexpr int kCullItems = 8;
constexpr int kCullChunk = kCullThreads * kCullItems;  // 2048 ids, 64 mask words

struct CullParams {
    float vm[16];
    float fx, fy, cx, cy;
    float width, height, near_p, far_p, opac_thr;
};

__device__ __forceinline__ bool cull_test(const gs_gaussians& g, const CullParams& p, int64_t i) {
    const int64_t r = g.table ? (int64_t)__ldg(g.table + i) : i;
    const float* mp = g.means + r * g.means_stride;
    const float x = __ldg(mp + 0), y = __ldg(mp + 1), z = __ldg(mp + 2);
    const float cx_ = cam_row(p.vm, 0, x, y, z);
    const float cy_ = cam_row(p.vm, 1, x, y, z);
    const float cz_ = cam_row(p.vm, 2, x, y, z);
    const float ds = cz_ > p.near_p ? cz_ : p.near_p;
    const float x2d = __fadd_rn(__fdiv_rn(__fmul_rn(cx_, p.fx), ds), p.cx);
    const float y2d = __fadd_rn(__fdiv_rn(__fmul_rn(cy_, p.fy), ds), p.cy);
    bool ok = (cz_ > p.near_p) && (cz_ < p.far_p) && (__fadd_rn(x2d, 50.0f) >= 0.0f) &&
              (__fsub_rn(x2d, 50.0f) < p.width) && (__fadd_rn(y2d, 50.0f) >= 0.0f) &&
              (__fsub_rn(y2d, 50.0f) < p.height);
    if (g.opac) ok = ok && (__ldg(g.opac + r * g.opac_stride) >= p.opac_thr);
    return ok;
}

// mask word w covers ids [32w, 32w + 32)
__global__ void __launch_bounds__(kCullThreads) cull_flags(gs_gaussians g, int64_t n, CullParams p,
                                                           uint32_t* __restrict__ words,
                                                           uint32_t* __restrict__ chunk_counts) {
    __shared__ uint32_t wsum[kCullThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t base = (int64_t)blockIdx.x * kCullChunk;
    uint32_t cnt = 0;
#pragma unroll
    for (int k = 0; k < kCullItems; ++k) {
        const int64_t i = base + (int64_t)k * kCullThreads + threadIdx.x;
        const bool ok = i < n && cull_test(g, p, i);
        const uint32_t b = __ballot_sync(kFull, ok);
        const int64_t wi = (base + (int64_t)k * kCullThreads + warp * 32) >> 5;
        if (lane == 0 && (wi << 5) < n) words[wi] = b;
        cnt += __popc(b);
    }
    if (lane == 0) wsum[warp] = cnt;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
#pragma unroll
        for (int w = 0; w < kCullThreads / 32; ++w) t += wsum[w];
        chunk_counts[blockIdx.x] = t;
    }
}

// Ordered write of the set bits: id r lands at its rank among the set bits;
// the value written is gather[r] when a gather map is given, else r.
__global__ void __launch_bounds__(kCullThreads) cull_write(const uint32_t* __restrict__ words, int64_t n,
                                                           const uint32_t* __restrict__ chunk_offsets,
                                                           const int32_t* __restrict__ gather,
                                                           int32_t* __restrict__ out_ids) {
    pdl_wait();
    __shared__ uint32_t woff[kCullChunk / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t base = (int64_t)blockIdx.x * kCullChunk;
    const int64_t wbase = base >> 5;
    const int64_t n_words = (n + 31) >> 5;
    if (warp == 0) {
        // exclusive prefix over the chunk's 64 words, two per lane
        const int64_t w0 = wbase + 2 * lane, w1 = w0 + 1;
        const uint32_t c0 = w0 < n_words ? __popc(words[w0]) : 0u;
        const uint32_t c1 = w1 < n_words ? __popc(words[w1]) : 0u;
        uint32_t inc = c0 + c1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(kFull, inc, o);
            if (lane >= o) inc += y;
        }
        const uint32_t ex = inc - c0 - c1;
        woff[2 * lane] = ex;
        woff[2 * lane + 1] = ex + c0;
    }
    __syncthreads();
    const uint32_t off0 = chunk_offsets[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kCullItems; ++k) {
        const int local_word = k * (kCullThreads / 32) + warp;
        const int64_t wi = wbase + local_word;
        if (wi >= n_words) break;
        const uint32_t b = words[wi];
        if ((b >> lane) & 1u) {
            const uint32_t pos = off0 + woff[local_word] + __popc(b & lanemask_lt());
            const int64_t r = (wi << 5) + lane;
            out_ids[pos] = gather ? __ldg(gather + r) : (int32_t)r;
        }
    }
}

static CullParams make_cull_params(const gs_camera& c, float near_p, float far_p, float thr) {
    CullParams p;
    for (int i = 0; i < 16; ++i) p.vm[i] = c.viewmat[i];
    p.fx = c.fx;
    p.fy = c.fy;
    p.cx = c.cx;
    p.cy = c.cy;
    p.width = (float)c.width;
    p.height = (float)c.height;
    p.near_p = near_p;
    p.far_p = far_p;
    p.opac_thr = thr;
    return p;
}

size_t cull_scratch_bytes(int64_t n) {
    const int64_t chunks = (n + kCullChunk - 1) / kCullChunk;
    size_t b = align_up((size_t)((n + 31) / 32 + 1) * 4, 256);
    b += align_up((size_t)(chunks + 1) * 4, 256);
    b += align_up(scan_scratch_bytes(chunks), 256);
    return b + 256;
}

int cull(const gs_gaussians& g, int64_t n, const gs_camera& cam, float near_p, float far_p, float thr,
         int32_t* out_ids, int32_t* out_count, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
    GS_REQUIRE(n >= 0 && n < ((int64_t)1 << 31), "cull: n out of range");
    GS_REQUIRE(g.means != nullptr && out_count != nullptr, "cull: null pointer");
    GS_REQUIRE(scratch_bytes >= cull_scratch_bytes(n) && scratch != nullptr, "cull: scratch too small");
    if (n == 0) {
        cudaMemsetAsync(out_count, 0, sizeof(int32_t), stream);
        return check_launch("cull(n=0)", 0);
    }
    GS_REQUIRE(out_ids != nullptr, "cull: null out_ids");
    const int64_t chunks = (n + kCullChunk - 1) / kCullChunk;
    char* p = reinterpret_cast<char*>(align_up(reinterpret_cast<uintptr_t>(scratch), 256));
    uint32_t* words = reinterpret_cast<uint32_t*>(p);
    p += align_up((size_t)((n + 31) / 32 + 1) * 4, 256);
    uint32_t* counts = reinterpret_cast<uint32_t*>(p);
    p += align_up((size_t)(chunks + 1) * 4, 256);
    const CullParams cp = make_cull_params(cam, near_p, far_p, thr);
    cull_flags<<<(unsigned)chunks, kCullThreads, 0, stream>>>(g, n, cp, words, counts);
    GS_TRY(check_launch("cull_flags"));
    // counts -> offsets in place; the total lands in counts[chunks]
    GS_TRY(scan_exclusive(counts, counts, chunks, p, scan_scratch_bytes(chunks), stream, true));
    GS_TRY(launch_pdl("cull_write", cull_write, dim3((unsigned)chunks), dim3(kCullThreads), stream,
                      (const uint32_t*)words, n, (const uint32_t*)counts, (const int32_t*)nullptr, out_ids));
    cudaMemcpyAsync(out_count, counts + chunks, sizeof(int32_t), cudaMemcpyDeviceToDevice, stream);
    return check_launch("cull count copy", 0);
}

// One bit per row: (flags[r] & mask) == value.
__global__ void __launch_bounds__(kCullThreads) flag_words(const uint8_t* __restrict__ flags, int64_t n, uint8_t mask,
                                                           uint8_t value, uint32_t* __restrict__ words,
                                                           uint32_t* __restrict__ chunk_counts) {
    __shared__ uint32_t wsum[kCullThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t base = (int64_t)blockIdx.x * kCullChunk;
    uint32_t cnt = 0;
#pragma unroll
    for (int k = 0; k < kCullItems; ++k) {
        const int64_t i = base + (int64_t)k * kCullThreads + threadIdx.x;
        const bool ok = i < n && (flags[i] & mask) == value;
        const uint32_t b = __ballot_sync(kFull, ok);
        const int64_t wi = (base + (int64_t)k * kCullThreads + warp * 32) >> 5;
        if (lane == 0 && (wi << 5) < n) words[wi] = b;
        cnt += __popc(b);
    }
    if (lane == 0) wsum[warp] = cnt;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
#pragma unroll
        for (int w = 0; w < kCullThreads / 32; ++w) t += wsum[w];
        chunk_counts[blockIdx.x] = t;
    }
}

int compact_flags(const uint8_t* flags, int64_t n, uint8_t mask, uint8_t value, const int32_t* gather, int32_t* out,
                  int32_t* out_count, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
    GS_REQUIRE(n >= 0 && n < ((int64_t)1 << 31), "compact: n out of range");
    GS_REQUIRE(out_count && scratch && scratch_bytes >= cull_scratch_bytes(n), "compact: bad scratch/count");
    if (n == 0) {
        cudaMemsetAsync(out_count, 0, sizeof(int32_t), stream);
        return check_launch("compact(n=0)", 0);
    }
    GS_REQUIRE(flags && out, "compact: null pointer");
    const int64_t chunks = (n + kCullChunk - 1) / kCullChunk;
    char* p = reinterpret_cast<char*>(align_up(reinterpret_cast<uintptr_t>(scratch), 256));
    uint32_t* words = reinterpret_cast<uint32_t*>(p);
    p += align_up((size_t)((n + 31) / 32 + 1) * 4, 256);
    uint32_t* counts = reinterpret_cast<uint32_t*>(p);
    p += align_up((size_t)(chunks + 1) * 4, 256);
    flag_words<<<(unsigned)chunks, kCullThreads, 0, stream>>>(flags, n, mask, value, words, counts);
    GS_TRY(check_launch("flag_words"));
    GS_TRY(scan_exclusive(counts, counts, chunks, p, scan_scratch_bytes(chunks), stream, true));
    GS_TRY(launch_pdl("compact write", cull_write, dim3((unsigned)chunks), dim3(kCullThreads), stream,
                      (const uint32_t*)words, n, (const uint32_t*)counts, gather, out));
    cudaMemcpyAsync(out_count, counts + chunks, sizeof(int32_t), cudaMemcpyDeviceToDevice, stream);
    return check_launch("compact count copy", 0);
}

// ---------------------------------------------------------------- cull without caller scratch
// gs_cull_noalloc keeps its scratch (mask words, chunk counts, scan partials)
// in the file-scope device array below instead of a caller buffer.  It is
// sized for kNoAllocMaxRows active ids; every device that loads the library
// holds it until the process exits.  Host code never dereferences the array's
// name: the device address is taken with cudaGetSymbolAddress, with the
// device current, the first time a device's context calls in, and kept per
// device together with that context's unique id.  A call from a different
// context on that device (after cudaDeviceReset made a new primary context,
// where the array may have moved) takes the address again.  Each call writes
// every scratch word before reading it, so nothing has to be cleared between
// calls.
constexpr int64_t kNoAllocMaxRows = int64_t(1) << 23;  // 8,388,608 active ids
constexpr size_t cx_align(size_t x, size_t a) { return (x + a - 1) / a * a; }
constexpr int64_t kNoAllocChunks = (kNoAllocMaxRows + kCullChunk - 1) / kCullChunk;
constexpr int64_t kNoAllocScanTiles = (kNoAllocChunks + 2047) / 2048;
constexpr size_t kNoAllocScratchBytes = cx_align((size_t)((kNoAllocMaxRows + 31) / 32 + 1) * 4, 256) +
                                        cx_align((size_t)(kNoAllocChunks + 1) * 4, 256) +
                                        cx_align((size_t)(kNoAllocScanTiles + 4) * 4 + 256, 256) + 256;

static __device__ __align__(256) unsigned char g_cull_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
struct NoAllocSlot {
    void* ptr;
    unsigned long long ctx_id;  // unique id of the context the address belongs to
};
static std::mutex g_noalloc_mu;
static NoAllocSlot g_noalloc[kNoAllocMaxDevices] = {};

// Unique id of the context current on this thread (cuCtxGetCurrent +
// cuCtxGetId, reached through the runtime's driver entry points so the
// library needs no link to the driver library); 0 when no context is
// current or the driver cannot say, in which case the address is looked up
// on every call.
static unsigned long long current_context_id() {
    using GetCurrentFn = CUresult (*)(CUcontext*);
    using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrentFn get_current = nullptr;
    static GetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrentFn>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetIdFn>(f);
        cudaGetLastError();  // a missing entry point is not this call's error
    });
    if (!get_current || !get_id) return 0;
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
    unsigned long long id = 0;
    return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of g_cull_scratch on the current device and context.
static int noalloc_scratch(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(GS_ERR_CUDA, "cull_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    GS_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "cull_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocSlot& slot = g_noalloc[dev];
    const unsigned long long ctx = current_context_id();
    if (slot.ptr == nullptr || ctx == 0 || slot.ctx_id != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_cull_scratch);
        if (e != cudaSuccess || p == nullptr)
            return set_error(GS_ERR_CUDA, "cull_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        slot.ptr = p;
        slot.ctx_id = current_context_id();  // the lookup made the device's context current
    }
    *out = slot.ptr;
    return GS_OK;
}

}  // namespace gs

extern "C" int gs_cull_noalloc(const gs_gaussians* g, int64_t n, const gs_camera* cam, float near_plane,
                               float far_plane, float opacity_threshold, int32_t* out_ids, int32_t* out_count,
                               gs_stream_t stream) {
    GS_REQUIRE(g && cam, "cull_noalloc: null descriptor");
    if (n > gs::kNoAllocMaxRows)
        return gs::set_error(GS_ERR_CAPACITY, "cull_noalloc: %lld active ids exceed the built-in limit of %lld",
                             (long long)n, (long long)gs::kNoAllocMaxRows);
    GS_REQUIRE(gs::cull_scratch_bytes(n) <= gs::kNoAllocScratchBytes, "cull_noalloc: scratch sizing mismatch");
    void* scratch = nullptr;
    GS_TRY(gs::noalloc_scratch(&scratch));
    return gs::cull(*g, n, *cam, near_plane, far_plane, opacity_threshold, out_ids, out_count, scratch,
                    gs::kNoAllocScratchBytes, (cudaStream_t)stream);
}

extern "C" size_t gs_cull_scratch_bytes(int64_t n) { return gs::cull_scratch_bytes(n); }

extern "C" int gs_compact_flags(const uint8_t* flags, int64_t n, uint8_t mask, uint8_t value, const int32_t* gather,
                                int32_t* out, int32_t* out_count, void* scratch, size_t scratch_bytes,
                                gs_stream_t stream) {
    return gs::compact_flags(flags, n, mask, value, gather, out, out_count, scratch, scratch_bytes,
                             (cudaStream_t)stream);
}

extern "C" int gs_cull(const gs_gaussians* g, int64_t n, const gs_camera* cam, float near_plane, float far_plane,
                       float opacity_threshold, int32_t* out_ids, int32_t* out_count, void* scratch,
                       size_t scratch_bytes, gs_stream_t stream) {
    GS_REQUIRE(g && cam, "cull: null descriptor");
    return gs::cull(*g, n, *cam, near_plane, far_plane, opacity_threshold, out_ids, out_count, scratch, scratch_bytes,
                    (cudaStream_t)stream);
}
