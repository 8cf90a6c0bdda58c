// Shared helpers of the sm_100a kernels: status reporting, launch checks,
// warp primitives and the float32 camera transform shared by cull and projection.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "gsplat_b200.h"

namespace gs {

int compact_flags(const uint8_t* flags, int64_t n, uint8_t mask, uint8_t value, const int32_t* gather, int32_t* out,
                  int32_t* out_count, void* scratch, size_t scratch_bytes, cudaStream_t stream);

constexpr int kTile = 16;               // tile edge in pixels
constexpr int kTileThreads = kTile * kTile;
constexpr unsigned kFull = 0xffffffffu;

int set_error(int code, const char* fmt, ...);
void note_launches(int n);  // running count of this library's kernel launches

// Records ``launched`` kernel launches and reports a launch failure.
inline int check_launch(const char* what, int launched = 1) {
    note_launches(launched);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(GS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return GS_OK;
}

#define GS_REQUIRE(cond, ...)                                  \
    do {                                                       \
        if (!(cond)) return ::gs::set_error(GS_ERR_INVALID, __VA_ARGS__); \
    } while (0)

#define GS_TRY(expr)                 \
    do {                             \
        int _st = (expr);            \
        if (_st != GS_OK) return _st; \
    } while (0)

inline unsigned grid_for(int64_t n, int block) { return (unsigned)((n + block - 1) / block); }

// Streaming multiprocessors of the current device (queried once per device).
inline int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = 0;
    }
    std::atomic<int>* c = dev >= 0 && dev < 64 ? &cache[dev] : nullptr;
    int n = c ? c->load(std::memory_order_relaxed) : 0;
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
        if (c) c->store(n, std::memory_order_relaxed);
    }
    return n;
}

// Programmatic dependent launch (sm_90+): a kernel launched with launch_pdl may
// be scheduled as soon as every block of the previous kernel in its stream has
// exited, before that grid's completion has been processed, which removes most
// of the gap between short dependent kernels.  Such a kernel must call
// pdl_wait() before it reads or writes any global memory that earlier work in
// the stream touches: the wait returns once the previous grid has completed
// and its memory operations are visible (in a kernel launched without the
// attribute it returns at once).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline int launch_pdl(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                      Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    note_launches(1);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(GS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    }
    return GS_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// Sums eight per-lane values over the warp with 9 shuffles (a butterfly that
// halves the number of values carried at each of the first three steps).  On
// return lane l holds the warp total of value index (l >> 2) & 7.
__device__ __forceinline__ float warp_sum8(float v0, float v1, float v2, float v3, float v4, float v5, float v6,
                                           float v7, int lane) {
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    // offset 16: keep values 0-3 (bit4 = 0) or 4-7 (bit4 = 1)
    float w0 = (b4 ? v4 : v0) + __shfl_xor_sync(kFull, b4 ? v0 : v4, 16);
    float w1 = (b4 ? v5 : v1) + __shfl_xor_sync(kFull, b4 ? v1 : v5, 16);
    float w2 = (b4 ? v6 : v2) + __shfl_xor_sync(kFull, b4 ? v2 : v6, 16);
    float w3 = (b4 ? v7 : v3) + __shfl_xor_sync(kFull, b4 ? v3 : v7, 16);
    // offset 8: keep (w0, w1) or (w2, w3)
    float x0 = (b3 ? w2 : w0) + __shfl_xor_sync(kFull, b3 ? w0 : w2, 8);
    float x1 = (b3 ? w3 : w1) + __shfl_xor_sync(kFull, b3 ? w1 : w3, 8);
    // offset 4: keep x0 or x1
    float y = (b2 ? x1 : x0) + __shfl_xor_sync(kFull, b2 ? x0 : x1, 4);
    y += __shfl_xor_sync(kFull, y, 2);
    y += __shfl_xor_sync(kFull, y, 1);
    return y;
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Vector reduction into global memory (16-byte aligned address).
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// Shared-memory float add when ``on`` (a predicated reduction: no branch
// around it and no returned value).
__device__ __forceinline__ void red_add_shared_if(float* addr, float v, bool on) {
    const unsigned a = (unsigned)__cvta_generic_to_shared(addr);
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t@p red.shared.add.f32 [%0], %1;\n\t}" ::"r"(a), "f"(v),
        "r"((unsigned)on)
        : "memory");
}

// Camera-space point of world position m: row i of  viewmat @ [m, 1],
// summed left to right with each product and sum rounded (no fused
// multiply-add), the order the CPU oracle uses, so the cull decision
// is reproducible bit for bit.
__device__ __forceinline__ float cam_row(const float* vm, int i, float x, float y, float z) {
    float s = __fmul_rn(x, vm[4 * i + 0]);
    s = __fadd_rn(s, __fmul_rn(y, vm[4 * i + 1]));
    s = __fadd_rn(s, __fmul_rn(z, vm[4 * i + 2]));
    return __fadd_rn(s, vm[4 * i + 3]);
}

// Sortable unsigned key of a float: ascending float order == ascending key.
__device__ __forceinline__ uint32_t float_sort_key(float f) {
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace gs
