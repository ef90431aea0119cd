// tc_net.cu -- bf16 tcgen05 engine of the fused training step (precision 1).
#include "net.cuh"

namespace zb {

struct TcEngine {};

int tc_create(Net &n) {
    (void)n;
    return fail(kBadArg, "zilla_net_create: precision 1 (tcgen05) engine not built yet");
}
void tc_destroy(Net &n) { n.tc = nullptr; }
int tc_step(Net &n, const float *, const float *, float *) { (void)n; return kBadArg; }
int tc_sync_params(Net &n) { (void)n; return kOk; }

}  // namespace zb
