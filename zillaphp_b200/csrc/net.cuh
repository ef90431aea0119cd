// net.cuh -- the fused training step ("net") shared between the fp32
// CUDA-core engine and the bf16 tcgen05 engine.
#pragma once

#include <vector>

#include "common.cuh"
#include "optim.cuh"

#ifdef ZB_HAVE_NCCL
#include <nccl.h>
#endif

namespace zb {

enum LayerKind { kConv = 1, kRelu = 2, kPool = 3, kLinear = 4 };

// A stage is one launch group of the step: a conv or linear layer with the
// ReLU that follows it fused in, a max-pool, or a stand-alone ReLU.
struct Stage {
    int kind = 0;          // LayerKind of the main layer
    int layer = 0;         // index of the main layer in the user's list
    bool relu = false;     // a ReLU follows and is fused into this stage
    int C = 0, H = 0, W = 0;      // input shape per sample
    int oC = 0, oH = 0, oW = 0;   // output shape per sample
    int pad = 0;
    long long in_n = 0, out_n = 0;  // per-sample sizes
    long long poff = 0, pn_w = 0, pn_b = 0;  // offsets into the flat parameter buffer
    float *out = nullptr;  // [B, out_n] fp32 activations (engine 0) / NCHW mirror
    float *gin = nullptr;  // gradient w.r.t. the stage input [B, in_n] (masked by the
                           // previous stage's ReLU when that one is fused)
    int *arg = nullptr;    // max-pool argmax (global flat index, int32)
    int arg_id = 0;        // registry handle exported on request
};

// Data-parallel exchange over NVLink peer memory (peer.cu): the ranks map
// each other's gradient exchange buffers, parameters and flag words through
// CUDA IPC; each rank owns a contiguous slice of the parameters.
constexpr int kMaxPeers = 8;
struct PeerState {
    bool on = false;                       // attached with peer memory (else NCCL all-reduce)
    bool in_step = false;                  // a peer step is between begin and end
    float *ex[2] = {nullptr, nullptr};     // this rank's exchange gradient buffers (step parity)
    unsigned long long *flags = nullptr;   // this rank's flag block: [0] gradients final, [8] slice written
    unsigned int *done = nullptr;          // completion counter of the update kernel (local)
    float *api_grads = nullptr;            // the registry gradient buffer
    float *rex[2][kMaxPeers] = {};         // every rank's exchange buffers (own included)
    float *rparams[kMaxPeers] = {};        // every rank's parameters
    unsigned long long *rflags[kMaxPeers] = {};
    std::vector<void *> opened;            // IPC mappings to close
    unsigned long long step = 0;           // peer steps taken
    long long lo = 0, hi = 0, chunk = 0;   // owned slice [lo, hi); slices of `chunk` floats
    // two-phase steps: the late layers' part of the slice is exchanged and updated on a side
    // stream while the backward of the early layers runs (peer_step_mid)
    cudaStream_t side_stream = nullptr;
    cudaEvent_t ev_mid = nullptr, ev_side = nullptr;
    long long mid_off = -1;                // first parameter of the late layers this step (-1: one phase)
    bool two_phase = false;                // use peer_step_mid (ZB_PEER_TWO_PHASE=1 turns it on)
    // graph capture of a step: the update and wait kernels' nodes (their step number and Adam
    // arguments change every replay)
    cudaGraphNode_t cap_update = nullptr, cap_wait = nullptr;
};

struct TcEngine;  // bf16 tensor-core engine (tc_net.cu)
struct LmEngine;  // Transformer language-model engine (lm_net.cu)

struct Net {
    int id = 0;
    int B = 0, inC = 0, inH = 0, inW = 0, classes = 0;
    int precision = 0;
    std::vector<int> spec;
    std::vector<Stage> st;
    long long nparams = 0;
    int params_id = 0, grads_id = 0;  // registry handles (grads has nparams + 1 floats: loss last)
    float *params = nullptr, *grads = nullptr;
    float *m = nullptr, *v = nullptr;  // Adam state
    float *dlogits = nullptr;
    double *row_loss = nullptr;
    float *xin = nullptr, *yin = nullptr, *loss_dev = nullptr;  // staging for step_host
    int opt = 1;
    float lr = 0.01f, b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
    int t = 0;
    // data parallel
    int rank = 0, world = 1;
#ifdef ZB_HAVE_NCCL
    ncclComm_t comm = nullptr;
#endif
    cudaStream_t comm_stream = nullptr;        // all-reduce stream (data parallel)
    cudaEvent_t ev_ready = nullptr, ev_done = nullptr;
    long long ar_lo = -1;                      // grads [ar_lo, nparams] already launched this step
    PeerState peer;
    // staged host steps: two device input slots filled on a copy stream
    cudaStream_t copy_stream = nullptr;
    float *sx[2] = {nullptr, nullptr}, *sy[2] = {nullptr, nullptr};
    cudaEvent_t ev_staged[2] = {nullptr, nullptr}, ev_consumed[2] = {nullptr, nullptr};
    int stage_head = 0, stage_tail = 0, stage_count = 0;
    // deferred loss reads (zilla_net_step_staged_deferred): two pinned host slots
    float *loss_host = nullptr;
    cudaEvent_t ev_loss[2] = {nullptr, nullptr};
    int loss_next = 0;        // slot the next deferred step writes
    int loss_pending = -1;    // slot holding a loss not yet handed to the caller (-1: none)
    // per-step CUDA graphs (zilla_net_set_graph): one per (x, y, update) on one rank
    bool graph_on = false;
    struct StepGraph {
        const float *x = nullptr, *y = nullptr;
        int update = 0, runs = 0;
        cudaGraph_t graph = nullptr;          // kept: its optimizer node updates the exec
        cudaGraphExec_t exec = nullptr;
        cudaGraphNode_t opt_node = nullptr;   // the optimizer kernel (Adam's arguments change every step)
        int parity = 0;                       // peer steps: the exchange buffer (step parity) it was captured on
        cudaGraphNode_t upd_node = nullptr, wait_node = nullptr;   // peer steps: the update and wait kernels
        unsigned nkern = 0;                   // kernels per replay (launch counter)
    };
    std::vector<StepGraph> graphs;
    cudaGraphNode_t captured_opt = nullptr;   // set by the optimizer launch while capturing
    TcEngine *tc = nullptr;
    LmEngine *lm = nullptr;
    long long x_floats = 0, y_floats = 0;   // per-step input sizes (floats)
    // per-segment device timing (zilla_net_profile / zilla_net_timings)
    bool profile = false;
    int prof_focus = -1;   // >= 0: events only around this segment (zilla_net_profile_segment)
    int prof_idx = 0;      // marks since the step's "start" mark
    std::vector<cudaEvent_t> ev_pool;
    std::vector<const char *> ev_label;   // label of the segment ending at event i
    int ev_used = 0;
};

// Records the end of a timed segment named `label` (no-op unless profiling).
void prof_mark(Net &n, const char *label);

Net *net_get(int id);
// fp32 engine pieces used by both engines
int fp32_forward(Net &n, const float *x);
int fp32_backward(Net &n, const float *x);
int loss_and_dlogits(Net &n, const float *logits, const float *y, float *loss_out);
// bf16 engine (tc_net.cu)
int tc_create(Net &n);
void tc_destroy(Net &n);
int tc_step(Net &n, const float *x, const float *y, float *loss_out);
int tc_forward(Net &n, const float *x, const float *y, float *logits, float *loss_out);   // evaluation
int tc_sync_params(Net &n);   // refresh the bf16 operand copies from the fp32 master
int tc_inspect(Net &n, int index, char *name, int name_len, float *host, unsigned long n_floats);
// language-model engine (lm_net.cu)
void lm_destroy(Net &n);
int lm_step(Net &n, const float *tokens, const float *targets, float *loss_out);
// Data parallel: grads[off .. nparams] (the loss slot included) are final for
// this step; starts their all-reduce on the comm stream so that it overlaps
// the rest of the backward.  No-op on one rank.
int dp_bucket_ready(Net &n, long long off);
// registry helpers shared by the engines (net.cu)
int net_register(Net *n);             // assigns the id, returns it
void net_free(Net *n);                // releases everything a Net holds
int net_alloc_common(Net &n, long long classes_rows, long long rows);   // params, grads, Adam, staging
void release_graphs(Net &n);          // the net's per-step CUDA graphs
// peer.cu: set-up after the NCCL communicator exists (collective; stays on NCCL
// when a rank cannot map every peer), the step hooks, and the release
int peer_attach(Net &n);
int peer_detach(Net &n);                   // collective: gathers the Adam state slices first
void peer_release(Net &n);                 // local: unmaps and frees
int peer_step_begin(Net &n);               // gradients of this step go to the exchange buffer
int peer_step_end(Net &n);                 // exchange + update + wait for every rank's slice
// Gradients [off, nparams] of this step are final: their part of the slice is exchanged and
// updated on a side stream while the rest of the backward runs; no-op off the peer path.
int peer_step_mid(Net &n, long long off);
// A captured peer step replayed: advances the step count and Adam's t as the step
// would, and gives the graph's update and wait kernels this step's arguments.
int peer_graph_args(Net &n, cudaGraphExec_t exec, cudaGraphNode_t upd, cudaGraphNode_t wt);

}  // namespace zb
