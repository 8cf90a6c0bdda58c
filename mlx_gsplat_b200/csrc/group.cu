// Multi-GPU pieces of the training step: a device-side barrier across the
// GPUs of one group, over signal pads in symmetric (peer-mapped) memory, and
// the sum of the gradient rows over the group through NVLink multicast.
//
// Each call carries an epoch that increases by one per call and channel on
// every GPU.  Thread t writes the epoch into GPU t's pad slot [channel][rank]
// with a system-scope release store, then polls its own slot [channel][t]
// with acquire loads until it holds that epoch.  Every poll loop is bounded:
// after ``max_polls`` unsuccessful polls the kernel sets ``*error_flag`` and
// returns, so a missing peer never leaves the GPU spinning.
#include <algorithm>

#include "common.cuh"

namespace gs {

__global__ void group_barrier_kernel(uint32_t* const* __restrict__ peer_pads, int32_t rank, int32_t world,
                                     int32_t channel, uint32_t epoch, int32_t* __restrict__ error_flag,
                                     int64_t max_polls) {
    const int t = threadIdx.x;
    if (t < world && t != rank) {
        uint32_t* dst = peer_pads[t] + (int64_t)channel * world + rank;
        // everything this GPU wrote before (earlier kernels included) is
        // visible system-wide before the peer can see the signal
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
        const uint32_t* src = peer_pads[rank] + (int64_t)channel * world + t;
        for (int64_t polls = 0;; ++polls) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(src) : "memory");
            if ((int32_t)(v - epoch) >= 0) break;
            if (polls >= max_polls) {
                atomicExch(error_flag, 1);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Sum of a row range over the GPUs of a multicast group, written back to
// every GPU: each 16-byte chunk is loaded reduced across all copies
// (multimem.ld_reduce, the switch adds them) and stored to all copies
// (multimem.st).  Every GPU runs this on its own disjoint range, so each
// element has one writer and all copies end bit-identical.
constexpr int kSumUnroll = 4;  // loads in flight per thread before the stores

__global__ void __launch_bounds__(256) rows_sum_multicast_kernel(float4* __restrict__ mc, int64_t begin,
                                                                 int64_t end, const int32_t* __restrict__ error_flag) {
    // a group barrier before this launch gave up waiting for a peer: some
    // copies may be incomplete, so no partial sum is formed or broadcast
    if (error_flag && *reinterpret_cast<const volatile int32_t*>(error_flag) != 0) return;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < end; i0 += kSumUnroll * stride) {
        float4 v[kSumUnroll];
#pragma unroll
        for (int u = 0; u < kSumUnroll; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < end)
                asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                             : "=f"(v[u].x), "=f"(v[u].y), "=f"(v[u].z), "=f"(v[u].w)
                             : "l"(mc + i)
                             : "memory");
        }
#pragma unroll
        for (int u = 0; u < kSumUnroll; ++u) {
            const int64_t i = i0 + u * stride;
            if (i < end)
                asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc + i),
                             "f"(v[u].x), "f"(v[u].y), "f"(v[u].z), "f"(v[u].w)
                             : "memory");
        }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");  // publish before the group's barrier
}

}  // namespace gs

using namespace gs;

extern "C" int gs_rows_sum_multicast(float* multicast_rows, int64_t first_row, int64_t num_rows, int64_t stride,
                                     const int32_t* error_flag, gs_stream_t stream) {
    GS_REQUIRE(multicast_rows && aligned16(multicast_rows), "rows_sum_multicast: 16-byte aligned address needed");
    GS_REQUIRE(first_row >= 0 && num_rows >= 0 && stride > 0 && stride % 4 == 0,
               "rows_sum_multicast: bad rows or stride (a multiple of 4 floats)");
    if (num_rows == 0) return GS_OK;
    const int64_t q = stride / 4;
    const int64_t begin = first_row * q, end = (first_row + num_rows) * q;
    const int64_t n = end - begin;
    const unsigned blocks = (unsigned)std::min<int64_t>((n + 256 * kSumUnroll - 1) / (256 * kSumUnroll), 148 * 8);
    rows_sum_multicast_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(reinterpret_cast<float4*>(multicast_rows),
                                                                        begin, end, error_flag);
    return check_launch("rows_sum_multicast_kernel");
}

extern "C" int gs_group_barrier(uint32_t* const* peer_pads, int32_t rank, int32_t world, int32_t channel,
                                uint32_t epoch, int32_t* error_flag, int64_t max_polls, gs_stream_t stream) {
    GS_REQUIRE(peer_pads && error_flag, "group_barrier: null pointer");
    GS_REQUIRE(world >= 1 && world <= 32 && rank >= 0 && rank < world, "group_barrier: bad rank/world");
    GS_REQUIRE(channel >= 0 && max_polls > 0, "group_barrier: bad channel or poll limit");
    if (world == 1) return GS_OK;
    group_barrier_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(peer_pads, rank, world, channel, epoch, error_flag,
                                                             max_polls);
    return check_launch("group_barrier_kernel");
}
