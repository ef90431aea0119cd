// optim.cuh -- optimizer arguments shared by the Adam kernels.
#pragma once

#include <math.h>

namespace zb {

struct AdamArgs {
    float lr, b1, b2, one_minus_b1, one_minus_b2, inv_bc1, inv_bc2, eps;
    float grad_scale;  // multiplies the gradient before the update (1/world in data parallel)
};

// One Adam element update (also used by the data-parallel peer update).
__device__ __forceinline__ void adam_one(float &w, float g, float &m, float &v, const AdamArgs &a) {
    g *= a.grad_scale;
    m = a.b1 * m + a.one_minus_b1 * g;
    v = a.b2 * v + a.one_minus_b2 * g * g;
    w -= a.lr * (m * a.inv_bc1) / (sqrtf(v * a.inv_bc2) + a.eps);
}

AdamArgs make_adam_args(float lr, float b1, float b2, float eps, int t, float grad_scale);
int launch_sgd(float *w, const float *g, float lr, float grad_scale, long long n);
int launch_adam(float *w, const float *g, float *m, float *v, long long n, const AdamArgs &a);

int launch_softmax_ce(const float *z, const float *y, float *dz, double *row_loss, float *loss,
                      int B, int C, bool zero_first);
int launch_bias_grad(const float *dy, float *db, int B, int C);

}  // namespace zb
