// net.cu -- the fused training step: one C call per step instead of the ~30
// per-op FFI calls of the reference's step drivers
// (examples/mnist_cnn_gpu_v2.php:183-264, examples/mnist_cpu_v2.php:178-217,
// examples/audio_cnn_gpu.php:201-257), plus the data-parallel runner
// (one NCCL all-reduce of the flat gradient buffer per step).
//
// Layers follow src/NN: Conv2D (3x3, stride 1, weights [oC, C, 3, 3],
// src/NN/Layers/Conv2D.php:25-44), ReLU, MaxPool2D (2x2/2,
// src/NN/Layers/MaxPool2D.php:12-20), Linear (W [in, out],
// src/NN/Layers/Linear.php:14-35), Flatten implied by the NCHW layout
// (src/Tensor/Tensor.php:958-981); parameters in Sequential::parameters()
// order (src/NN/Sequential.php:32-39).
//
// This file holds the net object, the fp32 CUDA-core engine (precision 0)
// and the optimizer / all-reduce tail; the bf16 tcgen05 engine (precision 1)
// is in tc_net.cu.
#include <math.h>
#include <string.h>

#include <map>

#include "conv_pool_f32.cuh"
#include "net.cuh"

namespace zb {

int launch_softmax_ce(const float *z, const float *y, float *dz, double *row_loss, float *loss,
                      int B, int C, bool zero_first);
int launch_bias_grad(const float *dy, float *db, int B, int C);
namespace {

std::map<int, Net *> g_nets;
int g_next_net = 1;

// Linear forward: Z[b, o] = (sum_i X[b, i] W[i, o]) + bias[o] (+ ReLU): the
// sum in ascending i with separately rounded products, then the bias, as
// matmul_dev + add_bias_dev do on the CPU (native/cpu/training_ops.c:25-47,
// 113-120).
struct LinearFwdF32 {
    const float *X, *Wt, *bias;
    float *Z;
    int M, N, K;
    bool relu;
    static constexpr bool kAMFast = false, kBNFast = true, kExactOrder = true;
    __device__ float init(int, int) const { return 0.0f; }
    __device__ float a(int m, int k) const { return X[(size_t)m * K + k]; }
    __device__ float b(int k, int n) const { return Wt[(size_t)k * N + n]; }
    __device__ void store(int m, int n, float v) const {
        float o = v + bias[n];
        if (relu) o = o > 0.0f ? o : 0.0f;
        Z[(size_t)m * N + n] = o;
    }
};

// Linear input gradient: dX[b, i] = sum_o dZ[b, o] W[i, o], times the
// previous ReLU's mask (A > 0) when that ReLU was fused.
struct LinearDgradF32 {
    const float *dZ, *Wt, *mask;
    float *dX;
    int M, N, K;
    static constexpr bool kAMFast = false, kBNFast = false, kExactOrder = false;
    __device__ float init(int, int) const { return 0.0f; }
    __device__ float a(int m, int k) const { return dZ[(size_t)m * K + k]; }
    __device__ float b(int k, int n) const { return Wt[(size_t)n * K + k]; }
    __device__ void store(int m, int n, float v) const {
        const size_t at = (size_t)m * N + n;
        if (mask) v = mask[at] > 0.0f ? v : 0.0f;
        dX[at] = v;
    }
};

__global__ void relu_inplace_kernel(float *__restrict__ x, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        x[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

// gin = gout * (out > 0) [* (mask > 0)]
__global__ void relu_bwd_mask_kernel(const float *__restrict__ gout, const float *__restrict__ out,
                                     const float *__restrict__ mask, float *__restrict__ gin,
                                     long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v = out[i] > 0.0f ? gout[i] : 0.0f;
        if (mask && !(mask[i] > 0.0f)) v = 0.0f;
        gin[i] = v;
    }
}

// Max-pool backward as a gather over input elements (no zero pass, no
// atomics): input (b,c,ih,iw) receives dOut of its 2x2 window iff the
// window's argmax points at it, times the fused ReLU mask of the input.
__global__ void pool_bwd_gather_kernel(const float *__restrict__ gout, const int *__restrict__ arg,
                                       const float *__restrict__ mask, float *__restrict__ gin,
                                       int B, int C, int H, int W, int oH, int oW) {
    const long long total = (long long)B * C * H * W;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int iw = (int)(i % W);
        const int ih = (int)((i / W) % H);
        const long long bc = i / ((long long)W * H);
        const int oh = ih >> 1, ow = iw >> 1;
        float v = 0.0f;
        if (oh < oH && ow < oW) {
            const long long o = (bc * oH + oh) * oW + ow;
            if ((long long)arg[o] == i) v = gout[o];
        }
        if (mask && !(mask[i] > 0.0f)) v = 0.0f;
        gin[i] = v;
    }
}

int build_stages(Net &n) {
    const int nl = (int)n.spec.size() / 4;
    int C = n.inC, H = n.inH, W = n.inW;
    long long poff = 0;
    for (int i = 0; i < nl; ++i) {
        const int kind = n.spec[4 * i], a = n.spec[4 * i + 1], b = n.spec[4 * i + 2], c = n.spec[4 * i + 3];
        if (kind == kRelu && !n.st.empty() && !n.st.back().relu &&
            (n.st.back().kind == kConv || n.st.back().kind == kLinear)) {
            n.st.back().relu = true;
            continue;
        }
        Stage s;
        s.kind = kind;
        s.layer = i;
        s.C = C; s.H = H; s.W = W;
        switch (kind) {
        case kConv:
            if (a != C) return fail(kBadArg, "net: layer %d expects %d input channels, got %d", i, a, C);
            if (b <= 0 || c < 0) return fail(kBadArg, "net: layer %d bad conv", i);
            s.oC = b; s.pad = c; s.oH = H + 2 * c - 2; s.oW = W + 2 * c - 2;
            if (s.oH <= 0 || s.oW <= 0) return fail(kBadArg, "net: layer %d output empty", i);
            s.poff = poff; s.pn_w = (long long)b * a * 9; s.pn_b = b;
            poff += s.pn_w + s.pn_b;
            break;
        case kRelu:
            s.oC = C; s.oH = H; s.oW = W;
            break;
        case kPool:
            s.oC = C; s.oH = (H - 2) / 2 + 1; s.oW = (W - 2) / 2 + 1;
            if (H < 2 || W < 2) return fail(kBadArg, "net: layer %d pool on %dx%d", i, H, W);
            break;
        case kLinear:
            if ((long long)a != (long long)C * H * W)
                return fail(kBadArg, "net: layer %d Linear expects %d inputs, got %lld", i, a, (long long)C * H * W);
            if (b <= 0) return fail(kBadArg, "net: layer %d bad Linear", i);
            s.oC = b; s.oH = 1; s.oW = 1;
            s.poff = poff; s.pn_w = (long long)a * b; s.pn_b = b;
            poff += s.pn_w + s.pn_b;
            break;
        default:
            return fail(kBadArg, "net: layer %d has unknown kind %d", i, kind);
        }
        s.in_n = (long long)C * H * W;
        s.out_n = (long long)s.oC * s.oH * s.oW;
        C = s.oC; H = s.oH; W = s.oW;
        n.st.push_back(s);
    }
    if (n.st.empty()) return fail(kBadArg, "net: no layers");
    n.nparams = poff;
    n.classes = (int)n.st.back().out_n;
    return kOk;
}

int alloc_dev(void **p, size_t bytes) {
    if (cudaMalloc(p, bytes ? bytes : 16) != cudaSuccess) {
        cudaGetLastError();
        return fail(kBadHandle, "net: cudaMalloc of %zu bytes failed", bytes);
    }
    return kOk;
}

void dp_release_streams(Net &n) {
    if (n.comm_stream) { cudaStreamSynchronize(n.comm_stream); cudaStreamDestroy(n.comm_stream); }
    if (n.ev_ready) cudaEventDestroy(n.ev_ready);
    if (n.ev_done) cudaEventDestroy(n.ev_done);
    n.comm_stream = nullptr;
    n.ev_ready = n.ev_done = nullptr;
    n.ar_lo = -1;
}

void free_net(Net *n) {
    if (!n) return;
    cudaStreamSynchronize(stream());
    peer_release(*n);   // peers' stores into this rank ended with the last step's wait
    release_graphs(*n);
    for (int k = 0; k < 2; ++k) {
        if (n->sx[k]) cudaFree(n->sx[k]);
        if (n->sy[k]) cudaFree(n->sy[k]);
        if (n->ev_staged[k]) cudaEventDestroy(n->ev_staged[k]);
        if (n->ev_consumed[k]) cudaEventDestroy(n->ev_consumed[k]);
    }
    if (n->copy_stream) {
        cudaStreamSynchronize(n->copy_stream);
        cudaStreamDestroy(n->copy_stream);
    }
    for (int k = 0; k < 2; ++k)
        if (n->ev_loss[k]) cudaEventDestroy(n->ev_loss[k]);
    if (n->loss_host) cudaFreeHost(n->loss_host);
    if (n->tc) tc_destroy(*n);
    if (n->lm) lm_destroy(*n);
    for (auto &s : n->st) {
        if (s.out) cudaFree(s.out);
        if (s.gin) cudaFree(s.gin);
        if (s.arg_id) zilla_buffer_free(s.arg_id);
        else if (s.arg) cudaFree(s.arg);
    }
    if (n->params_id) zilla_buffer_free(n->params_id);
    if (n->grads_id) zilla_buffer_free(n->grads_id);
    for (void *p : {(void *)n->m, (void *)n->v, (void *)n->dlogits, (void *)n->row_loss, (void *)n->xin,
                    (void *)n->yin, (void *)n->loss_dev})
        if (p) cudaFree(p);
#ifdef ZB_HAVE_NCCL
    if (n->comm) ncclCommDestroy(n->comm);
#endif
    dp_release_streams(*n);
    for (auto e : n->ev_pool) cudaEventDestroy(e);
    delete n;
}

}  // namespace

void prof_mark(Net &n, const char *label) {
    if (!n.profile) return;
    if (n.prof_focus >= 0) {
        // Only the marks that bound segment prof_focus: the one before it is
        // recorded as a "start" (zilla_net_timings skips the gap up to it), so
        // every other kernel boundary of the step stays free of events.
        const int idx = strcmp(label, "start") ? ++n.prof_idx : (n.prof_idx = 0);
        if (idx == n.prof_focus) label = "start";
        else if (idx != n.prof_focus + 1) return;
    }
    if (n.ev_used >= (int)n.ev_pool.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) { cudaGetLastError(); return; }
        n.ev_pool.push_back(e);
        n.ev_label.push_back(label);
    }
    n.ev_label[n.ev_used] = label;
    cudaEventRecord(n.ev_pool[n.ev_used], stream());
    n.ev_used += 1;
}

int net_register(Net *n) {
    n->id = g_next_net++;
    g_nets[n->id] = n;
    return n->id;
}

void net_free(Net *n) { free_net(n); }

// Flat parameter / gradient buffers (registry handles; gradients carry the
// loss sum in one extra slot), Adam moments, dlogits [classes_rows], per-row
// loss and host-step staging for x_floats / y_floats inputs.
int net_alloc_common(Net &n, long long classes_rows, long long rows) {
    n.params_id = zilla_buffer_alloc((unsigned long)(n.nparams > 0 ? n.nparams : 1));
    n.grads_id = zilla_buffer_alloc((unsigned long)n.nparams + 1);
    if (n.params_id <= 0 || n.grads_id <= 0) return kBadHandle;
    n.params = ptr(n.params_id);
    n.grads = ptr(n.grads_id);
    const size_t pbytes = (size_t)(n.nparams + 1) * sizeof(float);
    int rc = alloc_dev((void **)&n.m, pbytes);
    if (!rc) rc = alloc_dev((void **)&n.v, pbytes);
    if (!rc) rc = alloc_dev((void **)&n.dlogits, (size_t)classes_rows * sizeof(float));
    if (!rc) rc = alloc_dev((void **)&n.row_loss, (size_t)rows * sizeof(double));
    if (!rc) rc = alloc_dev((void **)&n.xin, (size_t)n.x_floats * sizeof(float));
    if (!rc) rc = alloc_dev((void **)&n.yin, (size_t)n.y_floats * sizeof(float));
    if (!rc) rc = alloc_dev((void **)&n.loss_dev, sizeof(float));
    if (rc) return rc;
    cudaMemsetAsync(n.params, 0, pbytes - sizeof(float), stream());
    cudaMemsetAsync(n.grads, 0, pbytes, stream());
    cudaMemsetAsync(n.m, 0, pbytes, stream());
    cudaMemsetAsync(n.v, 0, pbytes, stream());
    return check_cuda("net_alloc_common");
}

Net *net_get(int id) {
    auto it = g_nets.find(id);
    return it == g_nets.end() ? nullptr : it->second;
}

// ---------------------------------------------------------------- fp32 engine
int fp32_forward(Net &n, const float *x) {
    const int B = n.B;
    const float *in = x;
    for (auto &s : n.st) {
        int rc = kOk;
        switch (s.kind) {
        case kConv: {
            ConvFwdF32 p(in, n.params + s.poff, n.params + s.poff + s.pn_w, s.out, B, s.C, s.H, s.W,
                         s.oC, s.oH, s.oW, 3, 3, 1, s.pad, s.relu);
            rc = run_simt_gemm(p, 1, "net conv forward");
            break;
        }
        case kLinear: {
            LinearFwdF32 p{in, n.params + s.poff, n.params + s.poff + s.pn_w, s.out, B, s.oC, (int)s.in_n, s.relu};
            rc = run_simt_gemm(p, 1, "net linear forward");
            break;
        }
        case kPool: {
            const long long no = (long long)B * s.out_n;
            maxpool_fwd_kernel<<<grid_for(no, 256), 256, 0, stream()>>>(in, s.out, s.arg, B, s.C, s.H, s.W,
                                                                        s.oH, s.oW, 2, 2, 2);
            ZB_LAUNCH_CHECK("net pool forward");
            break;
        }
        case kRelu: {
            const long long nn = (long long)B * s.out_n;
            cudaMemcpyAsync(s.out, in, nn * sizeof(float), cudaMemcpyDeviceToDevice, stream());
            relu_inplace_kernel<<<grid_for(nn, 256), 256, 0, stream()>>>(s.out, nn);
            ZB_LAUNCH_CHECK("net relu forward");
            break;
        }
        }
        if (rc) return rc;
        prof_mark(n, s.kind == kConv ? "conv_fwd" : s.kind == kLinear ? "linear_fwd" : s.kind == kPool ? "pool_fwd" : "relu_fwd");
        in = s.out;
    }
    return kOk;
}

int loss_and_dlogits(Net &n, const float *logits, const float *y, float *loss_out) {
    return launch_softmax_ce(logits, y, n.dlogits, n.row_loss, loss_out, n.B, n.classes, true);
}

int fp32_backward(Net &n, const float *x) {
    const int B = n.B;
    const float *g = n.dlogits;
    for (int i = (int)n.st.size() - 1; i >= 0; --i) {
        Stage &s = n.st[i];
        const float *in = i ? n.st[i - 1].out : x;
        const float *mask = (i && n.st[i - 1].relu) ? n.st[i - 1].out : nullptr;
        const bool need_gin = i > 0;
        int rc = kOk;
        switch (s.kind) {
        case kConv: {
            if (need_gin) {
                ConvDgradF32 pd(g, n.params + s.poff, s.gin, mask, B, s.C, s.H, s.W, s.oC, s.oH, s.oW, 3,
                                3, 1, s.pad);
                rc = run_simt_gemm(pd, 1, "net conv dgrad");
                if (rc) return rc;
            }
            ConvWgradF32 pw(in, g, n.grads + s.poff, n.grads + s.poff + s.pn_w, B, s.C, s.H, s.W, s.oC,
                            s.oH, s.oW, 3, 3, 1, s.pad);
            rc = run_conv_wgrad(pw, "net conv wgrad");
            break;
        }
        case kLinear: {
            GemmTN pw(in, g, n.grads + s.poff, (int)s.in_n, s.oC, B);
            rc = run_simt_gemm(pw, 0, "net linear wgrad");
            if (rc) return rc;
            rc = launch_bias_grad(g, n.grads + s.poff + s.pn_w, B, s.oC);
            if (rc) return rc;
            if (need_gin) {
                LinearDgradF32 pd{g, n.params + s.poff, mask, s.gin, B, (int)s.in_n, s.oC};
                rc = run_simt_gemm(pd, 1, "net linear dgrad");
            }
            break;
        }
        case kPool: {
            if (need_gin) {
                const long long ni = (long long)B * s.in_n;
                pool_bwd_gather_kernel<<<grid_for(ni, 256), 256, 0, stream()>>>(g, s.arg, mask, s.gin, B, s.C,
                                                                                s.H, s.W, s.oH, s.oW);
                ZB_LAUNCH_CHECK("net pool backward");
            }
            break;
        }
        case kRelu: {
            if (need_gin) {
                const long long nn = (long long)B * s.in_n;
                relu_bwd_mask_kernel<<<grid_for(nn, 256), 256, 0, stream()>>>(g, s.out, mask, s.gin, nn);
                ZB_LAUNCH_CHECK("net relu backward");
            }
            break;
        }
        }
        if (rc) return rc;
        prof_mark(n, s.kind == kConv ? "conv_bwd" : s.kind == kLinear ? "linear_bwd" : s.kind == kPool ? "pool_bwd" : "relu_bwd");
        g = s.gin;
    }
    return kOk;
}

// All-reduce (sum) of grads[lo, hi) on the comm stream, after everything
// enqueued so far on the library stream.
static int allreduce_range(Net &n, long long lo, long long hi) {
#ifdef ZB_HAVE_NCCL
    if (hi <= lo) return kOk;
    if (cudaEventRecord(n.ev_ready, stream()) != cudaSuccess ||
        cudaStreamWaitEvent(n.comm_stream, n.ev_ready, 0) != cudaSuccess)
        return check_cuda("net: all-reduce ordering");
    ncclResult_t r = ncclAllReduce(n.grads + lo, n.grads + lo, (size_t)(hi - lo), ncclFloat, ncclSum, n.comm,
                                   n.comm_stream);
    if (r != ncclSuccess) return fail(kCudaError, "net: ncclAllReduce failed: %s", ncclGetErrorString(r));
    return kOk;
#else
    (void)n; (void)lo; (void)hi;
    return fail(kBadArg, "net: built without NCCL");
#endif
}

int dp_bucket_ready(Net &n, long long off) {
    if (n.world <= 1 || n.ar_lo >= 0 || n.peer.in_step) return kOk;
    n.ar_lo = off;
    return allreduce_range(n, off, n.nparams + 1);
}

// Sum of gradients (and the loss slot) over the data-parallel ranks: the part
// not started early by dp_bucket_ready, then the library stream waits for the
// comm stream.  Every rank issues the same calls in the same order.
static int allreduce_grads(Net &n) {
    if (n.world <= 1) return kOk;
    const long long hi = n.ar_lo >= 0 ? n.ar_lo : n.nparams + 1;
    n.ar_lo = -1;
    int rc = allreduce_range(n, 0, hi);
    if (rc) return rc;
    if (cudaEventRecord(n.ev_done, n.comm_stream) != cudaSuccess ||
        cudaStreamWaitEvent(stream(), n.ev_done, 0) != cudaSuccess)
        return check_cuda("net: all-reduce completion");
    return kOk;
}

static int optimizer_step(Net &n) {
    const float scale = 1.0f / (float)n.world;
    n.t += 1;
    const int rc = n.opt == 2 ? launch_adam(n.params, n.grads, n.m, n.v, n.nparams,
                                            make_adam_args(n.lr, n.b1, n.b2, n.eps, n.t, scale))
                              : launch_sgd(n.params, n.grads, n.lr, scale, n.nparams);
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (!rc && cudaStreamIsCapturing(stream(), &cs) == cudaSuccess && cs == cudaStreamCaptureStatusActive) {
        // the node just captured: a replay gives it this step's Adam arguments
        const cudaGraphNode_t *deps = nullptr;
        size_t nd = 0;
        if (cudaStreamGetCaptureInfo(stream(), &cs, nullptr, nullptr, &deps, &nd) == cudaSuccess && nd == 1)
            n.captured_opt = deps[0];
    }
    return rc;
}

static int run_step_body(Net &n, const float *x, const float *y, int update);

void release_graphs(Net &n) {
    for (auto &g : n.graphs) {
        if (g.exec) cudaGraphExecDestroy(g.exec);
        if (g.graph) cudaGraphDestroy(g.graph);
    }
    n.graphs.clear();
}

// One step, replayed from a CUDA graph when enabled: the first call for a
// (x, y, update) runs as is (lazy set-up happens outside any capture), the
// second captures the step on the library stream and launches the graph,
// later calls only refresh the optimizer's arguments and launch it.
static int run_step(Net &n, const float *x, const float *y, int update) {
    // data parallel: only the one-phase peer-memory step is captured (its exchange and update
    // are two kernels of the step; the NCCL path and the two-phase side stream are not)
    const bool peer = n.peer.on && update;
    if (!n.graph_on || n.profile || (n.world > 1 && !(peer && !n.peer.two_phase)))
        return run_step_body(n, x, y, update);
    const int parity = peer ? (int)((n.peer.step + 1) & 1) : 0;   // the exchange buffer this step writes
    Net::StepGraph *g = nullptr;
    for (auto &e : n.graphs)
        if (e.x == x && e.y == y && e.update == update && e.parity == parity) g = &e;
    if (!g) {
        if (n.graphs.size() >= 16) return run_step_body(n, x, y, update);
        n.graphs.emplace_back();
        g = &n.graphs.back();
        g->x = x; g->y = y; g->update = update; g->parity = parity;
    }
    if (g->runs++ == 0) return run_step_body(n, x, y, update);
    if (!g->exec) {
        const int t0 = n.t;
        const unsigned long long s0 = n.peer.step;
        const unsigned long long l0 = zilla_launch_count();
        n.captured_opt = nullptr;
        n.peer.cap_update = n.peer.cap_wait = nullptr;
        if (cudaStreamBeginCapture(stream(), cudaStreamCaptureModeRelaxed) != cudaSuccess)
            return check_cuda("net: graph capture");
        int rc = run_step_body(n, x, y, update);
        cudaGraph_t graph = nullptr;
        const cudaError_t ce = cudaStreamEndCapture(stream(), &graph);
        cudaGraphExec_t exec = nullptr;
        const bool nodes = !update || (peer ? (n.peer.cap_update && n.peer.cap_wait) : n.captured_opt != nullptr);
        if (!rc && ce == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess && nodes) {
            g->graph = graph;
            g->exec = exec;
            g->opt_node = update && !peer ? n.captured_opt : nullptr;
            g->upd_node = peer ? n.peer.cap_update : nullptr;
            g->wait_node = peer ? n.peer.cap_wait : nullptr;
            g->nkern = (unsigned)(zilla_launch_count() - l0);
            if (cudaGraphLaunch(exec, stream()) != cudaSuccess) return check_cuda("net: graph launch");
            return check_cuda("net: graph");
        }
        // capture not possible: graphs off for this net, the step runs as is
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        release_graphs(n);
        n.graph_on = false;
        n.t = t0;
        n.peer.step = s0;
        if (n.peer.in_step) n.grads = n.peer.api_grads, n.peer.in_step = false;
        if (rc) return rc;
        return run_step_body(n, x, y, update);
    }
    if (peer) {   // this step's step number and Adam arguments for the exchange and update kernels
        int rc = peer_graph_args(n, g->exec, g->upd_node, g->wait_node);
        if (rc) return rc;
    } else if (update) {
        n.t += 1;
        if (n.opt == 2) {   // this step's Adam arguments (the bias corrections change with t)
            float *w = n.params, *m = n.m, *v = n.v;
            const float *gr = n.grads;
            long long cnt = n.nparams;
            AdamArgs a = make_adam_args(n.lr, n.b1, n.b2, n.eps, n.t, 1.0f);
            void *args[6] = {&w, &gr, &m, &v, &cnt, &a};
            cudaKernelNodeParams kp{};
            if (cudaGraphKernelNodeGetParams(g->opt_node, &kp) != cudaSuccess) return check_cuda("net: graph node");
            kp.kernelParams = args;
            kp.extra = nullptr;
            if (cudaGraphExecKernelNodeSetParams(g->exec, g->opt_node, &kp) != cudaSuccess)
                return check_cuda("net: graph optimizer arguments");
        }
    }
    if (cudaGraphLaunch(g->exec, stream()) != cudaSuccess) return check_cuda("net: graph launch");
    count_launch(g->nkern);
    return check_cuda("net: graph");
}

static int run_step_body(Net &n, const float *x, const float *y, int update) {
    int rc;
    // data parallel over peer memory: this step's gradients go to an exchange
    // buffer, and one kernel sums the rank's slice over NVLink and updates it
    const bool peer = n.peer.on && update;
    if (peer && (rc = peer_step_begin(n))) return rc;
    float *loss_slot = n.grads + n.nparams;
    prof_mark(n, "start");
    if (n.lm) {
        rc = lm_step(n, x, y, loss_slot);
    } else if (n.precision == 1) {
        rc = tc_step(n, x, y, loss_slot);
    } else {
        rc = fp32_forward(n, x);
        if (!rc) rc = loss_and_dlogits(n, n.st.back().out, y, loss_slot);
        if (!rc) prof_mark(n, "softmax_ce");
        if (!rc) rc = fp32_backward(n, x);
    }
    if (rc) {
        if (peer) n.grads = n.peer.api_grads, n.peer.in_step = false;
        return rc;
    }
    if (peer) {
        rc = peer_step_end(n);
        if (!rc) prof_mark(n, "allreduce");
        if (!rc) prof_mark(n, n.opt == 2 ? "adam" : "sgd");
        return rc;
    }
    rc = allreduce_grads(n);
    if (rc) return rc;
    if (n.world > 1) prof_mark(n, "allreduce");
    if (update) {
        rc = optimizer_step(n);
        if (rc) return rc;
        prof_mark(n, n.opt == 2 ? "adam" : "sgd");
    }
    return rc;
}

}  // namespace zb

using namespace zb;

extern "C" {

int zilla_net_create(const int *layers, int n_layers, int batch, int in_c, int in_h, int in_w,
                     int precision) {
    if (!layers || n_layers <= 0 || batch <= 0 || in_c <= 0 || in_h <= 0 || in_w <= 0)
        return fail(kBadArg, "zilla_net_create: bad arguments");
    if (precision != 0 && precision != 1) return fail(kBadArg, "zilla_net_create: precision must be 0 or 1");
    Net *n = new Net();
    n->B = batch; n->inC = in_c; n->inH = in_h; n->inW = in_w; n->precision = precision;
    n->spec.assign(layers, layers + 4 * n_layers);
    int rc = build_stages(*n);
    if (rc) { delete n; return rc; }
    n->x_floats = (long long)batch * in_c * in_h * in_w;
    n->y_floats = batch;
    rc = net_alloc_common(*n, (long long)batch * n->classes, batch);
    if (rc) { free_net(n); return rc; }
    if (precision == 0) {
        for (size_t i = 0; i < n->st.size(); ++i) {
            Stage &s = n->st[i];
            if (s.kind != kRelu || true) {
                rc = alloc_dev((void **)&s.out, (size_t)batch * s.out_n * sizeof(float));
                if (rc) break;
            }
            if (i > 0) {
                rc = alloc_dev((void **)&s.gin, (size_t)batch * s.in_n * sizeof(float));
                if (rc) break;
            }
            if (s.kind == kPool) {
                if ((long long)batch * s.in_n > 0x7fffffffLL) { rc = fail(kBadArg, "net: pool input too large"); break; }
                s.arg_id = zilla_buffer_alloc((unsigned long)(batch * s.out_n));
                if (s.arg_id <= 0) { rc = kBadHandle; break; }
                s.arg = (int *)ptr(s.arg_id);
            }
        }
    } else {
        rc = tc_create(*n);
    }
    if (!rc) rc = check_cuda("zilla_net_create");
    if (rc) { free_net(n); return rc; }
    return net_register(n);
}

int zilla_net_destroy(int id) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_destroy: unknown net %d", id);
    g_nets.erase(id);
    free_net(n);
    return kOk;
}

long zilla_net_param_count(int id) {
    Net *n = net_get(id);
    return n ? (long)n->nparams : (long)fail(kBadHandle, "zilla_net_param_count: unknown net %d", id);
}

int zilla_net_params_id(int id) {
    Net *n = net_get(id);
    return n ? n->params_id : fail(kBadHandle, "zilla_net_params_id: unknown net %d", id);
}

int zilla_net_grads_id(int id) {
    Net *n = net_get(id);
    return n ? n->grads_id : fail(kBadHandle, "zilla_net_grads_id: unknown net %d", id);
}

int zilla_net_argmax_id(int id, int layer) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_argmax_id: unknown net %d", id);
    for (auto &s : n->st)
        if (s.layer == layer && s.kind == kPool) return s.arg_id;
    return 0;
}

int zilla_net_set_optimizer(int id, int kind, float lr, float beta1, float beta2, float eps) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_set_optimizer: unknown net %d", id);
    if (kind != 1 && kind != 2) return fail(kBadArg, "zilla_net_set_optimizer: kind must be 1 (SGD) or 2 (Adam)");
    n->opt = kind; n->lr = lr; n->b1 = beta1; n->b2 = beta2; n->eps = eps;
    release_graphs(*n);   // captured optimizer launches carry the old settings
    return kOk;
}

int zilla_net_step(int id, int x_id, int y_id, int loss_id, int update) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_step: unknown net %d", id);
    float *x = ptr(x_id), *y = ptr(y_id), *loss = ptr(loss_id);
    if (!x || !y || !loss) return fail(kBadHandle, "zilla_net_step: invalid handle");
    if (capacity(x_id) < (size_t)n->x_floats || capacity(y_id) < (size_t)n->y_floats)
        return fail(kBadHandle, "zilla_net_step: input buffers smaller than the batch");

    int rc = run_step(*n, x, y, update);
    if (rc) return rc;
    cudaMemcpyAsync(loss, n->grads + n->nparams, sizeof(float), cudaMemcpyDeviceToDevice, stream());
    return check_cuda("zilla_net_step");
}

int zilla_net_forward(int id, int x_id, int y_id, int logits_id, int loss_id) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_forward: unknown net %d", id);
    if (n->lm) return fail(kBadArg, "zilla_net_forward: not available for the language model");
    float *x = ptr(x_id), *logits = ptr(logits_id);
    float *y = y_id > 0 ? ptr(y_id) : nullptr, *loss = loss_id > 0 ? ptr(loss_id) : nullptr;
    if (!x || !logits || (y_id > 0 && !y) || (loss_id > 0 && !loss))
        return fail(kBadHandle, "zilla_net_forward: invalid handle");
    if (capacity(x_id) < (size_t)n->x_floats || capacity(logits_id) < (size_t)n->B * n->classes ||
        (y && capacity(y_id) < (size_t)n->y_floats))
        return fail(kBadHandle, "zilla_net_forward: buffers smaller than the batch");
    if (loss && !y) return fail(kBadArg, "zilla_net_forward: a loss needs the targets");
    int rc;
    if (n->precision == 1) {
        rc = tc_forward(*n, x, y, logits, loss);
    } else {
        rc = fp32_forward(*n, x);
        if (!rc) {
            cudaMemcpyAsync(logits, n->st.back().out, (size_t)n->B * n->classes * sizeof(float),
                            cudaMemcpyDeviceToDevice, stream());
            if (loss) rc = loss_and_dlogits(*n, n->st.back().out, y, loss);
        }
    }
    if (rc) return rc;
    return check_cuda("zilla_net_forward");
}

int zilla_net_step_host(int id, const float *x, const float *y, float *loss_sum, int update) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_step_host: unknown net %d", id);
    if (!x || !y) return fail(kBadArg, "zilla_net_step_host: null input");
    cudaMemcpyAsync(n->xin, x, (size_t)n->x_floats * sizeof(float), cudaMemcpyHostToDevice, stream());
    cudaMemcpyAsync(n->yin, y, (size_t)n->y_floats * sizeof(float), cudaMemcpyHostToDevice, stream());
    int rc = run_step(*n, n->xin, n->yin, update);
    if (rc) return rc;
    if (loss_sum) {
        cudaMemcpyAsync(loss_sum, n->grads + n->nparams, sizeof(float), cudaMemcpyDeviceToHost, stream());
        if (cudaStreamSynchronize(stream()) != cudaSuccess) return check_cuda("zilla_net_step_host");
    }
    return check_cuda("zilla_net_step_host");
}

int zilla_net_stage_host(int id, const float *x, const float *y) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_stage_host: unknown net %d", id);
    if (!x || !y) return fail(kBadArg, "zilla_net_stage_host: null input");
    if (n->stage_count == 2) return fail(kBadArg, "zilla_net_stage_host: both slots hold batches not yet stepped");
    if (!n->copy_stream) {   // first use: the copy stream, the two slots and their events
        if (cudaStreamCreateWithFlags(&n->copy_stream, cudaStreamNonBlocking) != cudaSuccess)
            return check_cuda("zilla_net_stage_host: copy stream");
        for (int k = 0; k < 2; ++k) {
            if (cudaMalloc((void **)&n->sx[k], (size_t)n->x_floats * sizeof(float)) != cudaSuccess ||
                cudaMalloc((void **)&n->sy[k], (size_t)n->y_floats * sizeof(float)) != cudaSuccess ||
                cudaEventCreateWithFlags(&n->ev_staged[k], cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&n->ev_consumed[k], cudaEventDisableTiming) != cudaSuccess)
                return check_cuda("zilla_net_stage_host: staging slots");
            cudaEventRecord(n->ev_consumed[k], stream());
        }
    }
    const int k = n->stage_head;
    // the step that last read this slot has finished before the copy overwrites it
    cudaStreamWaitEvent(n->copy_stream, n->ev_consumed[k], 0);
    cudaMemcpyAsync(n->sx[k], x, (size_t)n->x_floats * sizeof(float), cudaMemcpyHostToDevice, n->copy_stream);
    cudaMemcpyAsync(n->sy[k], y, (size_t)n->y_floats * sizeof(float), cudaMemcpyHostToDevice, n->copy_stream);
    cudaEventRecord(n->ev_staged[k], n->copy_stream);
    n->stage_head ^= 1;
    n->stage_count += 1;
    return check_cuda("zilla_net_stage_host");
}

int zilla_net_step_staged(int id, float *loss_sum, int update) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_step_staged: unknown net %d", id);
    if (n->stage_count == 0) return fail(kBadArg, "zilla_net_step_staged: no batch staged");
    const int k = n->stage_tail;
    cudaStreamWaitEvent(stream(), n->ev_staged[k], 0);
    int rc = run_step(*n, n->sx[k], n->sy[k], update);
    cudaEventRecord(n->ev_consumed[k], stream());
    n->stage_tail ^= 1;
    n->stage_count -= 1;
    if (rc) return rc;
    if (loss_sum) {
        cudaMemcpyAsync(loss_sum, n->grads + n->nparams, sizeof(float), cudaMemcpyDeviceToHost, stream());
        if (cudaStreamSynchronize(stream()) != cudaSuccess) return check_cuda("zilla_net_step_staged");
    }
    return check_cuda("zilla_net_step_staged");
}

int zilla_net_step_staged_deferred(int id, float *prev_loss_sum, int *has_prev, int update) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_step_staged_deferred: unknown net %d", id);
    if (!prev_loss_sum || !has_prev) return fail(kBadArg, "zilla_net_step_staged_deferred: null output");
    *has_prev = 0;
    if (n->stage_count == 0) return fail(kBadArg, "zilla_net_step_staged_deferred: no batch staged");
    if (!n->loss_host) {   // first use: two pinned loss slots and their events
        if (cudaHostAlloc((void **)&n->loss_host, 2 * sizeof(float), cudaHostAllocDefault) != cudaSuccess)
            return check_cuda("zilla_net_step_staged_deferred: pinned loss slots");
        for (int k = 0; k < 2; ++k)
            if (cudaEventCreateWithFlags(&n->ev_loss[k], cudaEventDisableTiming) != cudaSuccess)
                return check_cuda("zilla_net_step_staged_deferred: events");
    }
    int rc = zilla_net_step_staged(id, nullptr, update);
    if (rc) return rc;
    // this step's loss sum goes to a pinned slot; the slot's previous content was handed out
    const int k = n->loss_next;
    cudaMemcpyAsync(n->loss_host + k, n->grads + n->nparams, sizeof(float), cudaMemcpyDeviceToHost, stream());
    cudaEventRecord(n->ev_loss[k], stream());
    n->loss_next ^= 1;
    // hand out the previous step's loss: wait only for that step (this one stays queued)
    if (n->loss_pending >= 0) {
        if (cudaEventSynchronize(n->ev_loss[n->loss_pending]) != cudaSuccess)
            return check_cuda("zilla_net_step_staged_deferred: previous step");
        *prev_loss_sum = n->loss_host[n->loss_pending];
        *has_prev = 1;
    }
    n->loss_pending = k;
    return check_cuda("zilla_net_step_staged_deferred");
}

int zilla_net_loss_flush(int id, float *loss_sum, int *has) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_loss_flush: unknown net %d", id);
    if (!loss_sum || !has) return fail(kBadArg, "zilla_net_loss_flush: null output");
    *has = 0;
    if (n->loss_pending < 0) return kOk;
    if (cudaEventSynchronize(n->ev_loss[n->loss_pending]) != cudaSuccess)
        return check_cuda("zilla_net_loss_flush");
    *loss_sum = n->loss_host[n->loss_pending];
    *has = 1;
    n->loss_pending = -1;
    return kOk;
}

int zilla_net_inspect(int id, int index, char *name, int name_len, float *host, unsigned long n_floats) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_inspect: unknown net %d", id);
    if (n->precision != 1) return 0;
    int rc = read_and_clear_device_error();
    if (rc) return fail(kCudaError, "zilla_net_inspect: device error word 0x%x", rc);
    return tc_inspect(*n, index, name, name_len, host, n_floats);
}

int zilla_net_device_status(int id) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_device_status: unknown net %d", id);
    cudaStreamSynchronize(stream());
    int code = read_and_clear_device_error();
    if (code) return fail(kCudaError, "device error word 0x%x (bounded wait expired or bad index)", code);
    return check_cuda("zilla_net_device_status");
}

int zilla_net_set_graph(int id, int enable) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_set_graph: unknown net %d", id);
    cudaStreamSynchronize(stream());
    release_graphs(*n);
    n->graph_on = enable != 0;
    return kOk;
}

int zilla_net_profile(int id, int enable) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_profile: unknown net %d", id);
    n->profile = enable != 0;
    n->prof_focus = -1;
    n->ev_used = 0;
    return kOk;
}

int zilla_net_profile_segment(int id, int segment) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_profile_segment: unknown net %d", id);
    if (segment < 0) return fail(kBadArg, "zilla_net_profile_segment: segment %d", segment);
    n->profile = true;
    n->prof_focus = segment;
    n->prof_idx = 0;
    n->ev_used = 0;
    return kOk;
}

int zilla_net_timings(int id, char *labels, int labels_len, float *ms, int max_segments) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_net_timings: unknown net %d", id);
    if (n->ev_used < 2) return 0;
    if (cudaEventSynchronize(n->ev_pool[n->ev_used - 1]) != cudaSuccess) return check_cuda("zilla_net_timings");
    int k = 0, pos = 0;
    for (int i = 1; i < n->ev_used && k < max_segments; ++i) {
        const char *l = n->ev_label[i];
        if (!strcmp(l, "start")) continue;   // gap between two profiled steps
        cudaEventElapsedTime(&ms[k++], n->ev_pool[i - 1], n->ev_pool[i]);
        int len = (int)strlen(l);
        if (labels && pos + len + 1 < labels_len) {
            memcpy(labels + pos, l, len);
            labels[pos + len] = '\n';
            pos += len + 1;
            labels[pos] = 0;
        }
    }
    return k;
}

int zilla_dp_unique_id(unsigned char *id128) {
#ifdef ZB_HAVE_NCCL
    ncclUniqueId u;
    ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) return fail(kCudaError, "zilla_dp_unique_id: %s", ncclGetErrorString(r));
    memcpy(id128, u.internal, sizeof(u.internal));
    return kOk;
#else
    (void)id128;
    return fail(kBadArg, "zilla_dp_unique_id: built without NCCL");
#endif
}

int zilla_dp_attach(int id, int rank, int world, const unsigned char *id128) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_dp_attach: unknown net %d", id);
    if (world < 1 || rank < 0 || rank >= world) return fail(kBadArg, "zilla_dp_attach: bad rank/world");
    if (world == 1) { n->rank = 0; n->world = 1; return kOk; }
#ifdef ZB_HAVE_NCCL
    ncclUniqueId u;
    memcpy(u.internal, id128, sizeof(u.internal));
    if (n->comm) { ncclCommDestroy(n->comm); n->comm = nullptr; }
    ncclResult_t r = ncclCommInitRank(&n->comm, world, u, rank);
    if (r != ncclSuccess) {
        n->comm = nullptr;
        return fail(kCudaError, "zilla_dp_attach: ncclCommInitRank failed: %s", ncclGetErrorString(r));
    }
    if (!n->comm_stream &&
        (cudaStreamCreateWithFlags(&n->comm_stream, cudaStreamNonBlocking) != cudaSuccess ||
         cudaEventCreateWithFlags(&n->ev_ready, cudaEventDisableTiming) != cudaSuccess ||
         cudaEventCreateWithFlags(&n->ev_done, cudaEventDisableTiming) != cudaSuccess)) {
        dp_release_streams(*n);
        ncclCommDestroy(n->comm);
        n->comm = nullptr;
        return check_cuda("zilla_dp_attach: comm stream");
    }
    n->rank = rank;
    n->world = world;
    peer_release(*n);          // a re-attach starts from the NCCL path
    return peer_attach(*n);    // collective: maps the peers' buffers when every rank can
#else
    (void)id128;
    return fail(kBadArg, "zilla_dp_attach: built without NCCL");
#endif
}

int zilla_dp_detach(int id) {
    Net *n = net_get(id);
    if (!n) return fail(kBadHandle, "zilla_dp_detach: unknown net %d", id);
#ifdef ZB_HAVE_NCCL
    if (n->comm) {
        int rc = peer_detach(*n);   // collective, before the communicator goes
        if (rc) return rc;
        cudaStreamSynchronize(stream());
        dp_release_streams(*n);
        ncclCommDestroy(n->comm);
        n->comm = nullptr;
    }
#endif
    n->world = 1;
    n->rank = 0;
    return kOk;
}

}  // extern "C"
