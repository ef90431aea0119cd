// optim.cuh -- optimizer arguments shared by the Adam kernels.
#pragma once

namespace zb {

struct AdamArgs {
    float lr, b1, b2, one_minus_b1, one_minus_b2, inv_bc1, inv_bc2, eps;
    float grad_scale;  // multiplies the gradient before the update (1/world in data parallel)
};

AdamArgs make_adam_args(float lr, float b1, float b2, float eps, int t, float grad_scale);
int launch_sgd(float *w, const float *g, float lr, float grad_scale, long long n);
int launch_adam(float *w, const float *g, float *m, float *v, long long n, const AdamArgs &a);

int launch_softmax_ce(const float *z, const float *y, float *dz, double *row_loss, float *loss,
                      int B, int C, bool zero_first);
int launch_bias_grad(const float *dy, float *db, int B, int C);

}  // namespace zb
