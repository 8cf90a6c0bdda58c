/* Host C++ meanings for the handful of Metal Shading Language words used by
 * the reference's ``fused_adam_step`` kernel source (src/mlx_extensions.cpp:102-152),
 * so that the kernel text can be compiled unchanged by g++ and run on the CPU
 * as a checker.  TEST INFRASTRUCTURE ONLY (force-included by oracle/build_ref.py).
 *
 * - address-space and function qualifiers (kernel, device, constant) are empty;
 * - the [[buffer(n)]] / [[thread_position_in_grid]] attributes are unknown to
 *   g++ and ignored (-Wno-attributes);
 * - metal::pow/sqrt/isnan/isinf/clamp are the IEEE float functions, with
 *   clamp(x, lo, hi) = fmin(fmax(x, lo), hi) as the MSL specification defines it.
 */
#pragma once
#include <cmath>
#include <cstdint>
#define kernel
#define device
#define constant
typedef unsigned int uint;
namespace metal {
inline float pow(float a, float b) { return std::pow(a, b); }
inline float sqrt(float a) { return std::sqrt(a); }
inline bool isnan(float a) { return std::isnan(a); }
inline bool isinf(float a) { return std::isinf(a); }
inline float clamp(float x, float lo, float hi) { return std::fmin(std::fmax(x, lo), hi); }
}  // namespace metal
