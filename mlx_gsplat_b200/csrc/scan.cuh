// Internal device-wide scan and radix sort entry points shared by the kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace gs {
size_t scan_scratch_bytes(int64_t n);
// out[0..n) = exclusive prefix sums of in; out[n] = total.  ``after_kernel``:
// the previous operation in the stream is a kernel of this library, so the
// first scan kernel may use a programmatic dependent launch too.
int scan_exclusive(const uint32_t* in, uint32_t* out, int64_t n, void* scratch, size_t scratch_bytes,
                   cudaStream_t stream, bool after_kernel = false);

size_t radix_sort_scratch_bytes(int64_t n);
int radix_sort_pairs(const uint32_t* keys_in, const uint32_t* vals_in, uint32_t* keys_out, uint32_t* vals_out,
                     int64_t n, int begin_bit, int end_bit, void* scratch, size_t scratch_bytes, cudaStream_t stream);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
}  // namespace gs
