/* CPU restatement of the reference's fused Metal Adam — TEST INFRASTRUCTURE ONLY.
 *
 * Follows the MSL kernel ``fused_adam_step`` (src/mlx_extensions.cpp:102-152)
 * one element at a time, in float32, with the same operation order:
 *   physical = indices[id / dim] * dim + id % dim          (:119-121)
 *   g = isnan(g) ? 0 : g; g += wd * theta                  (:123-130)
 *   m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2             (:131-132)
 *   m, v: NaN/Inf -> 0                                     (:134-135)
 *   bc1 = 1 - pow(b1, step); bc2 = 1 - pow(b2, step)       (:140-141)
 *   delta = (lr / bc1) * (m / (sqrt(v) / sqrt(bc2) + eps)) (:143-146)
 *   delta: NaN/Inf -> 0; theta = clamp(theta - delta, lo, hi) (:147-151)
 *
 * ``theta/m/v`` rows live at ``indices[row] * pool_stride`` (the reference has
 * pool_stride == dim); ``g`` rows at ``row * g_stride``.
 * Build: oracle/Makefile -> oracle/liboracle_adam.so (gcc, no -ffast-math,
 * -ffp-contract=off so that no multiply-add is fused).
 */
#include <math.h>
#include <stdint.h>

static float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

void oracle_fused_adam_a1(float* theta, const float* g, float* m, float* v, const int32_t* indices,
                          int64_t num_active, int dim, int64_t pool_stride, int64_t g_stride,
                          float lr, float beta1, float beta2, float eps, float weight_decay, int step,
                          float a_min, float a_max) {
    const float bc1 = 1.0f - powf(beta1, (float)step);
    const float bc2 = 1.0f - powf(beta2, (float)step);
    for (int64_t row = 0; row < num_active; ++row) {
        const int64_t base = (int64_t)indices[row] * pool_stride;
        for (int d = 0; d < dim; ++d) {
            const int64_t p = base + d;
            float grad = g[row * g_stride + d];
            if (isnan(grad)) grad = 0.0f;
            if (weight_decay != 0.0f) grad += weight_decay * theta[p];
            float m_new = beta1 * m[p] + (1.0f - beta1) * grad;
            float v_new = beta2 * v[p] + (1.0f - beta2) * (grad * grad);
            if (isnan(m_new) || isinf(m_new)) m_new = 0.0f;
            if (isnan(v_new) || isinf(v_new)) v_new = 0.0f;
            m[p] = m_new;
            v[p] = v_new;
            const float step_size = lr / bc1;
            const float denom = (sqrtf(v_new) / sqrtf(bc2)) + eps;
            float delta = step_size * (m_new / denom);
            if (isnan(delta) || isinf(delta)) delta = 0.0f;
            theta[p] = clampf(theta[p] - delta, a_min, a_max);
        }
    }
}
