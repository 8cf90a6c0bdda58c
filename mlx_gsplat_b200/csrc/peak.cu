// FP32 throughput probe: the denominator of the compositing kernels' compute
// roofline.  The compositing kernels are bound by fp32 instruction issue, not
// by HBM; their achieved fp32 rate (contributing (pixel, splat) pairs times the
// fp32 operations one pair costs, over the kernel's time) is reported against
// what this kernel measures on the same GPU: every thread runs kChains
// independent fused multiply-add chains, as paired (two-lane) instructions or
// as scalar ones, with enough resident warps to hide the pipeline latency.
#include "common.cuh"

namespace gs {

constexpr int kPeakChains = 8;
constexpr int kPeakThreads = 256;

template <bool kPaired>
__global__ void __launch_bounds__(kPeakThreads) fp32_peak_kernel(float* __restrict__ out, int iters, float a,
                                                                 float b) {
    const float seed = (float)(blockIdx.x * kPeakThreads + threadIdx.x) * 1e-9f;
    if constexpr (kPaired) {
        float2 acc[kPeakChains];
#pragma unroll
        for (int c = 0; c < kPeakChains; ++c) acc[c] = make_float2(seed + c, seed - c);
        const float2 a2 = make_float2(a, a), b2 = make_float2(b, b);
        for (int i = 0; i < iters; ++i) {
#pragma unroll
            for (int c = 0; c < kPeakChains; ++c) acc[c] = __ffma2_rn(acc[c], a2, b2);
        }
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < kPeakChains; ++c) s += acc[c].x + acc[c].y;
        out[blockIdx.x * kPeakThreads + threadIdx.x] = s;
    } else {
        float acc[2 * kPeakChains];
#pragma unroll
        for (int c = 0; c < 2 * kPeakChains; ++c) acc[c] = seed + c;
        for (int i = 0; i < iters; ++i) {
#pragma unroll
            for (int c = 0; c < 2 * kPeakChains; ++c) acc[c] = __fmaf_rn(acc[c], a, b);
        }
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < 2 * kPeakChains; ++c) s += acc[c];
        out[blockIdx.x * kPeakThreads + threadIdx.x] = s;
    }
}

}  // namespace gs

using namespace gs;

extern "C" int gs_fp32_peak_probe(float* out, int64_t out_len, int blocks, int iters, int paired,
                                  double* flops_per_launch, gs_stream_t stream) {
    GS_REQUIRE(out && flops_per_launch, "fp32_peak_probe: null pointer");
    GS_REQUIRE(blocks > 0 && iters > 0, "fp32_peak_probe: blocks and iters must be positive");
    GS_REQUIRE(out_len >= (int64_t)blocks * kPeakThreads, "fp32_peak_probe: out needs blocks * %d floats",
               kPeakThreads);
    auto kernel = paired ? fp32_peak_kernel<true> : fp32_peak_kernel<false>;
    kernel<<<blocks, kPeakThreads, 0, (cudaStream_t)stream>>>(out, iters, 0.999999f, 1e-7f);
    // 2 kPeakChains fused multiply-adds (2 flops each) per thread and iteration, either form
    *flops_per_launch = (double)blocks * kPeakThreads * (double)iters * (2.0 * kPeakChains) * 2.0;
    return check_launch(paired ? "fp32_peak_kernel<paired>" : "fp32_peak_kernel<scalar>");
}
