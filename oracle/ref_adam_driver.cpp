/* Runs the reference's own Metal ``fused_adam_step`` kernel text on the CPU,
 * one grid position at a time.  TEST INFRASTRUCTURE ONLY.
 * ``ref_fused_adam_step.inc`` is written into oracle/_ref/ by oracle/build_ref.py,
 * which extracts the MSL string literal from src/mlx_extensions.cpp; it is never
 * committed.  Exported: ref_fused_adam_step (same argument meaning as the
 * reference's launch_fused_adam_step, src/mlx_extensions.cpp:75-91).
 */
#include "msl_prelude.h"
#include "ref_fused_adam_step.inc"

extern "C" void ref_fused_adam_step(float* theta, const float* g, float* m, float* v,
                                    const int* indices, long num_active, int dim, float lr,
                                    float beta1, float beta2, float eps, float weight_decay,
                                    int step, float a_min, float a_max) {
    const long n = num_active * (long)dim;
    for (long id = 0; id < n; ++id)
        fused_adam_step(theta, g, m, v, indices, lr, beta1, beta2, eps, weight_decay, step, dim,
                        a_min, a_max, (uint)id);
}
