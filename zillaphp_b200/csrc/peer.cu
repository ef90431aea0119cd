// peer.cu -- the data-parallel gradient exchange and parameter update of the
// bf16 engine as one kernel over NVLink peer memory.
//
// With NCCL the step is: gradients -> all-reduce (a library kernel, partly
// overlapped with the backward, and a latency-bound tail for the last
// bucket) -> Adam on every rank over the whole buffer.  Here each of the W
// ranks owns a contiguous slice of the flat parameter buffer, and after the
// backward one kernel per rank
//   1. publishes "my gradients of step s are final" (a flag word in its own
//      memory, release at system scope),
//   2. waits (bounded) until every peer's flag shows step s,
//   3. reads its slice of every rank's gradient buffer over NVLink and sums
//      them in rank order 0 .. W-1 (the same order on every rank),
//   4. applies Adam / SGD to its slice (the Adam moments of a slice live only
//      on its owner),
//   5. stores the updated parameters of its slice into every rank's
//      parameter buffer (peer stores), and
//   6. when its last block is done, publishes "slice of step s written".
// A one-thread kernel after it waits (bounded) until every peer has published
// step s, so the next step (or any read of the parameters) sees the whole
// buffer.  The ranks' parameters are bit-identical by construction: one
// owner computes each element once.  Per rank and step this moves
// (W-1)/W of the gradient buffer in and (W-1)/W of the parameter buffer out
// over NVLink, against the all-reduce's 2 (W-1)/W in and out.
//
// Gradients alternate between two exchange buffers by step parity.  A rank
// writes buffer p again two steps later, and by then every peer has finished
// reading it: a peer reads buffer p only inside its update kernel of step s,
// and this rank passes its own wait of step s+1 only after every peer has
// published step s+1, which each does after its update kernel of step s.
//
// Plain peer loads and stores only (no multicast objects).  Every wait is
// bounded: past the limit the kernel records an error and returns, so a rank
// that died makes the others fail their step instead of hanging the GPU.
#include <stdlib.h>
#include <string.h>

#include "net.cuh"

namespace zb {

namespace {

constexpr int kErrPeerWait = 0x50450001;   // a peer never published its step
constexpr unsigned long long kPeerWaitNs = 2000000000ull;

struct PeerArgs {
    const float *ex[kMaxPeers];                      // every rank's exchange buffer of this step
    float *params[kMaxPeers];                        // every rank's parameters
    const unsigned long long *flags[kMaxPeers];      // every rank's flag block
    unsigned long long *my_flags;
    unsigned int *done;
    float *m, *v, *api_grads;
    long long lo, hi, nparams;                       // [lo, hi): the part of the slice this launch updates
    int world, rank, opt;                            // opt 2 = Adam, else SGD
    int slot;                                        // flag word published / awaited: "gradients final"
    int do_loss;                                     // this launch sums the loss slot
    int written;                                     // the last block publishes "slice written" (slot 8)
    unsigned long long step;
    AdamArgs a;
    float lr, scale;
    int *err;
};

constexpr int kSlotFinalA = 0;   // gradients of the late layers (the first launch of a two-phase step)
constexpr int kSlotFinalB = 1;   // gradients of the early layers (the second launch)
constexpr int kSlotWritten = 8;  // this rank's whole slice of the step stored into every rank

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait, by one warp, until flag word `slot` of every other rank shows
// `step`: lane q polls rank q, so the remote round trips overlap.
__device__ bool wait_peers(const PeerArgs &A, int slot, unsigned long long step) {
    const int q = threadIdx.x & 31;
    bool ok = true;
    if (q < A.world && q != A.rank) {
        const unsigned long long t0 = now_ns();
        while (ld_acquire_sys(A.flags[q] + slot) < step)
            if (now_ns() - t0 > kPeerWaitNs) {
                atomicCAS(A.err, 0, kErrPeerWait);
                ok = false;
                break;
            }
    }
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void update_one(const PeerArgs &A, float &w, float g, float &m, float &v) {
    if (A.opt == 2) adam_one(w, g, m, v, A.a);
    else w = __fsub_rn(w, __fmul_rn(A.lr, __fmul_rn(g, A.scale)));   // as the SGD kernel: no FMA
}

// 128-thread blocks: with 74 registers a block (10,240 registers) fits beside one CTA of the
// fused conv backward (14 warps x 120 registers), so the first launch of a two-phase step runs
// on the SMs that kernel occupies.
__global__ void __launch_bounds__(128, 6) peer_update_kernel(const __grid_constant__ PeerArgs A) {
    __shared__ int ok;
    if (threadIdx.x < 32) {
        // this rank's gradients of the range (written by the kernels before this one) are final
        if (threadIdx.x == 0) st_release_sys(A.my_flags + A.slot, A.step);
        const bool w = wait_peers(A, A.slot, A.step);
        if (threadIdx.x == 0) ok = w;
    }
    __syncthreads();
    if (ok) {
        float *own = A.params[A.rank];
        // float4 groups inside [lo, hi); the < 4 elements before and after them are done singly
        const long long b4 = (A.lo + 3) >> 2, e4 = A.hi >> 2;
        const long long stride = (long long)gridDim.x * blockDim.x;
        for (long long i4 = b4 + blockIdx.x * blockDim.x + threadIdx.x; i4 < e4; i4 += stride) {
            // all ranks' loads in flight together, then the sum in rank order
            float4 t[kMaxPeers];
#pragma unroll
            for (int q = 0; q < kMaxPeers; ++q)
                if (q < A.world) t[q] = __ldcg(reinterpret_cast<const float4 *>(A.ex[q]) + i4);
            float4 g = t[0];
#pragma unroll
            for (int q = 1; q < kMaxPeers; ++q)
                if (q < A.world) { g.x += t[q].x; g.y += t[q].y; g.z += t[q].z; g.w += t[q].w; }
            float4 w = reinterpret_cast<float4 *>(own)[i4];
            float4 m = reinterpret_cast<float4 *>(A.m)[i4], v = reinterpret_cast<float4 *>(A.v)[i4];
            update_one(A, w.x, g.x, m.x, v.x);
            update_one(A, w.y, g.y, m.y, v.y);
            update_one(A, w.z, g.z, m.z, v.z);
            update_one(A, w.w, g.w, m.w, v.w);
            reinterpret_cast<float4 *>(A.m)[i4] = m;
            reinterpret_cast<float4 *>(A.v)[i4] = v;
            reinterpret_cast<float4 *>(A.api_grads)[i4] = g;
#pragma unroll
            for (int q = 0; q < kMaxPeers; ++q)
                if (q < A.world) reinterpret_cast<float4 *>(A.params[q])[i4] = w;
        }
        if (blockIdx.x == 0 && threadIdx.x < 8) {
            // threads 0-3: [lo, min(4 b4, hi)); threads 4-7: [max(4 e4, 4 b4), hi)
            const long long head_end = 4 * b4 < A.hi ? 4 * b4 : A.hi;
            const long long tail_beg = 4 * e4 > 4 * b4 ? 4 * e4 : 4 * b4;
            const long long e = threadIdx.x < 4 ? A.lo + threadIdx.x : tail_beg + (threadIdx.x - 4);
            if (threadIdx.x < 4 ? e < head_end : e < A.hi) {
                float g = __ldcg(A.ex[0] + e);
                for (int q = 1; q < A.world; ++q) g += __ldcg(A.ex[q] + e);
                float w = own[e], m = A.m[e], v = A.v[e];
                update_one(A, w, g, m, v);
                A.m[e] = m;
                A.v[e] = v;
                A.api_grads[e] = g;
                for (int q = 0; q < A.world; ++q) A.params[q][e] = w;
            }
        }
        if (A.do_loss && blockIdx.x == 0 && threadIdx.x == 0) {
            float l = 0.0f;   // the loss slot: sum over the ranks
            for (int q = 0; q < A.world; ++q) l += __ldcg(A.ex[q] + A.nparams);
            A.api_grads[A.nparams] = l;
        }
    }
    // the last block to finish publishes this rank's slice of step `step` as written
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(A.done, 1u) == gridDim.x - 1) {
            *A.done = 0;
            __threadfence_system();
            if (ok && A.written) st_release_sys(A.my_flags + kSlotWritten, A.step);
        }
    }
}

__global__ void peer_wait_kernel(const __grid_constant__ PeerArgs A) {
    wait_peers(A, kSlotWritten, A.step);   // one warp
}

#ifdef ZB_HAVE_NCCL
struct PeerRec {
    cudaIpcMemHandle_t h[4];   // exchange buffer 0, 1, flag block, parameters
    int dev, ok;
    char pad[56];
};

// every rank's `ok` ANDed (NCCL min over the ranks)
int all_ok(Net &n, int ok, int *out) {
    int *d = nullptr;
    if (cudaMalloc((void **)&d, sizeof(int)) != cudaSuccess) return check_cuda("peer: scratch");
    cudaMemcpy(d, &ok, sizeof(int), cudaMemcpyHostToDevice);
    ncclResult_t r = ncclAllReduce(d, d, 1, ncclInt32, ncclMin, n.comm, stream());
    cudaMemcpyAsync(out, d, sizeof(int), cudaMemcpyDeviceToHost, stream());
    cudaStreamSynchronize(stream());
    cudaFree(d);
    if (r != ncclSuccess) return fail(kCudaError, "peer: ncclAllReduce: %s", ncclGetErrorString(r));
    return check_cuda("peer: agreement");
}
#endif

PeerArgs make_args(Net &n, unsigned long long step) {
    PeerState &P = n.peer;
    PeerArgs A{};
    for (int q = 0; q < n.world; ++q) {
        A.ex[q] = P.rex[step & 1][q];
        A.params[q] = P.rparams[q];
        A.flags[q] = P.rflags[q];
    }
    A.my_flags = P.flags;
    A.done = P.done;
    A.m = n.m;
    A.v = n.v;
    A.api_grads = P.api_grads;
    A.lo = P.lo;
    A.hi = P.hi;
    A.nparams = n.nparams;
    A.world = n.world;
    A.rank = n.rank;
    A.opt = n.opt;
    A.step = step;
    A.lr = n.lr;
    A.scale = 1.0f / (float)n.world;
    A.err = device_error_word();
    return A;
}

}  // namespace

void peer_release(Net &n) {
    PeerState &P = n.peer;
    release_graphs(n);   // captured steps hold the peers' buffers
    if (P.side_stream) {
        cudaStreamSynchronize(P.side_stream);
        cudaStreamDestroy(P.side_stream);
        cudaEventDestroy(P.ev_mid);
        cudaEventDestroy(P.ev_side);
        P.side_stream = nullptr;
    }
    if (!P.flags && !P.ex[0] && P.opened.empty()) return;
    cudaStreamSynchronize(stream());
    for (void *p : P.opened) cudaIpcCloseMemHandle(p);
    for (void *p : {(void *)P.ex[0], (void *)P.ex[1], (void *)P.flags, (void *)P.done})
        if (p) cudaFree(p);
    if (P.api_grads) n.grads = P.api_grads;
    n.peer = PeerState();
}

int peer_attach(Net &n) {
#ifdef ZB_HAVE_NCCL
    const char *env = getenv("ZB_PEER_STEP");
    const bool want = !(env && env[0] == '0') && n.precision == 1 && !n.lm && n.world > 1 && n.world <= kMaxPeers;
    // every rank takes the same branch: the decision only depends on values equal on all ranks
    if (!want) return kOk;
    release_graphs(n);   // steps captured before the attach write the registry gradients
    PeerState &P = n.peer;
    P.api_grads = n.grads;
    const size_t gbytes = (size_t)(n.nparams + 1) * sizeof(float);
    int ok = 1;
    for (int k = 0; k < 2 && ok; ++k)
        if (cudaMalloc((void **)&P.ex[k], gbytes) != cudaSuccess || cudaMemset(P.ex[k], 0, gbytes) != cudaSuccess) ok = 0;
    if (ok && (cudaMalloc((void **)&P.flags, 256) != cudaSuccess || cudaMemset(P.flags, 0, 256) != cudaSuccess)) ok = 0;
    if (ok && (cudaMalloc((void **)&P.done, 64) != cudaSuccess || cudaMemset(P.done, 0, 64) != cudaSuccess)) ok = 0;
    PeerRec mine;
    memset(&mine, 0, sizeof(mine));
    cudaGetDevice(&mine.dev);
    if (ok) {
        void *bufs[4] = {P.ex[0], P.ex[1], P.flags, n.params};
        for (int k = 0; k < 4 && ok; ++k)
            if (cudaIpcGetMemHandle(&mine.h[k], bufs[k]) != cudaSuccess) ok = 0;
    }
    cudaGetLastError();
    mine.ok = ok;
    // every rank's record
    std::vector<PeerRec> recs(n.world);
    {
        PeerRec *d = nullptr;
        if (cudaMalloc((void **)&d, sizeof(PeerRec) * (n.world + 1)) != cudaSuccess) return check_cuda("peer: records");
        cudaMemcpy(d + n.world, &mine, sizeof(PeerRec), cudaMemcpyHostToDevice);
        ncclResult_t r = ncclAllGather(d + n.world, d, sizeof(PeerRec), ncclUint8, n.comm, stream());
        cudaMemcpyAsync(recs.data(), d, sizeof(PeerRec) * n.world, cudaMemcpyDeviceToHost, stream());
        cudaStreamSynchronize(stream());
        cudaFree(d);
        if (r != ncclSuccess) return fail(kCudaError, "peer: ncclAllGather: %s", ncclGetErrorString(r));
    }
    for (int q = 0; q < n.world; ++q) {
        if (!recs[q].ok) ok = 0;
        if (q == n.rank || !ok) continue;
        int can = 0;
        if (cudaDeviceCanAccessPeer(&can, mine.dev, recs[q].dev) != cudaSuccess || !can) ok = 0;
    }
    cudaGetLastError();
    int all = 0;
    int rc = all_ok(n, ok, &all);
    if (rc) return rc;
    if (all) {   // map every peer's buffers
        for (int q = 0; q < n.world && ok; ++q) {
            if (q == n.rank) {
                P.rex[0][q] = P.ex[0];
                P.rex[1][q] = P.ex[1];
                P.rflags[q] = P.flags;
                P.rparams[q] = n.params;
                continue;
            }
            void *p[4] = {};
            for (int k = 0; k < 4 && ok; ++k) {
                if (cudaIpcOpenMemHandle(&p[k], recs[q].h[k], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) ok = 0;
                else P.opened.push_back(p[k]);
            }
            if (!ok) break;
            P.rex[0][q] = (float *)p[0];
            P.rex[1][q] = (float *)p[1];
            P.rflags[q] = (unsigned long long *)p[2];
            P.rparams[q] = (float *)p[3];
        }
        cudaGetLastError();
        rc = all_ok(n, ok, &all);   // also the barrier: every rank's flags are zero before any step
        if (rc) return rc;
    }
    if (!all) {   // stay on the NCCL all-reduce
        peer_release(n);
        return kOk;
    }
    // ZB_PEER_TWO_PHASE=1: exchange the late layers on a side stream beside the fused conv
    // backward.  Off by default: measured on two B200s it cost 2.1% per step (the side kernel
    // slows the fused backward and the stream join breaks the programmatic-launch chain).
    const char *tp = getenv("ZB_PEER_TWO_PHASE");
    P.two_phase = tp && tp[0] == '1';
    P.chunk = ((n.nparams + n.world - 1) / n.world + 3) / 4 * 4;
    P.lo = P.chunk * n.rank < n.nparams ? P.chunk * n.rank : n.nparams;
    P.hi = P.lo + P.chunk < n.nparams ? P.lo + P.chunk : n.nparams;
    P.step = 0;
    P.on = true;
    return kOk;
#else
    (void)n;
    return kOk;
#endif
}

int peer_detach(Net &n) {
#ifdef ZB_HAVE_NCCL
    PeerState &P = n.peer;
    if (!P.on) return kOk;
    release_graphs(n);   // captured steps hold the peers' mappings
    // the Adam moments of each slice live on its owner: every rank gets all of them
    for (int q = 0; q < n.world; ++q) {
        const long long lo = P.chunk * q < n.nparams ? P.chunk * q : n.nparams;
        const long long hi = lo + P.chunk < n.nparams ? lo + P.chunk : n.nparams;
        if (hi <= lo) continue;
        if (ncclBroadcast(n.m + lo, n.m + lo, (size_t)(hi - lo), ncclFloat, q, n.comm, stream()) != ncclSuccess ||
            ncclBroadcast(n.v + lo, n.v + lo, (size_t)(hi - lo), ncclFloat, q, n.comm, stream()) != ncclSuccess)
            return fail(kCudaError, "peer: Adam state broadcast failed");
    }
    cudaStreamSynchronize(stream());
    for (void *p : P.opened) cudaIpcCloseMemHandle(p);
    P.opened.clear();
    int all = 0;
    int rc = all_ok(n, 1, &all);   // every rank has unmapped before any rank frees
    peer_release(n);
    return rc;
#else
    (void)n;
    return kOk;
#endif
}

int peer_step_begin(Net &n) {
    PeerState &P = n.peer;
    P.step += 1;
    P.in_step = true;
    P.mid_off = -1;
    n.grads = P.ex[P.step & 1];
    return kOk;
}

namespace {

// The node of the kernel just launched when the library stream is being captured, else null.
cudaGraphNode_t captured_node() {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream(), &cs) != cudaSuccess || cs != cudaStreamCaptureStatusActive) return nullptr;
    const cudaGraphNode_t *deps = nullptr;
    size_t nd = 0;
    if (cudaStreamGetCaptureInfo(stream(), &cs, nullptr, nullptr, &deps, &nd) != cudaSuccess || nd != 1) return nullptr;
    return deps[0];
}

int update_grid(long long count, int per_sm) {
    const long long n4 = count / 4 + 2;
    long long grid = (n4 + 127) / 128;
    if (grid > (long long)sm_count() * per_sm) grid = (long long)sm_count() * per_sm;
    return grid < 1 ? 1 : (int)grid;
}

}  // namespace

int peer_step_mid(Net &n, long long off) {
    PeerState &P = n.peer;
    if (!P.on || !P.in_step || P.mid_off >= 0 || off <= 0 || off >= n.nparams || !P.two_phase) return kOk;
    if (!P.side_stream) {   // first use: the side stream and its two events
        if (cudaStreamCreateWithFlags(&P.side_stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&P.ev_mid, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&P.ev_side, cudaEventDisableTiming) != cudaSuccess)
            return check_cuda("peer: side stream");
    }
    // gradients [off, nparams] (and the loss slot) of this step are final: exchange and update
    // the part of this rank's slice above `off` on the side stream, while the backward goes on
    if (cudaEventRecord(P.ev_mid, stream()) != cudaSuccess || cudaStreamWaitEvent(P.side_stream, P.ev_mid, 0) != cudaSuccess)
        return check_cuda("peer: mid-step ordering");
    P.mid_off = off;
    PeerArgs A = make_args(n, P.step);
    A.a = make_adam_args(n.lr, n.b1, n.b2, n.eps, n.t + 1, A.scale);
    A.lo = P.lo > off ? P.lo : off;
    A.hi = P.hi;
    if (A.hi < A.lo) A.hi = A.lo;
    A.slot = kSlotFinalA;
    A.do_loss = 1;
    A.written = 0;
    peer_update_kernel<<<update_grid(A.hi - A.lo, 1), 128, 0, P.side_stream>>>(A);
    ZB_LAUNCH_CHECK("peer update (late layers)");
    if (cudaEventRecord(P.ev_side, P.side_stream) != cudaSuccess) return check_cuda("peer: side event");
    return kOk;
}

int peer_step_end(Net &n) {
    PeerState &P = n.peer;
    n.grads = P.api_grads;
    P.in_step = false;
    n.t += 1;
    PeerArgs A = make_args(n, P.step);
    A.a = make_adam_args(n.lr, n.b1, n.b2, n.eps, n.t, A.scale);
    A.written = 1;
    if (P.mid_off >= 0) {   // second phase: the early layers [0, mid_off) after the first one
        if (cudaStreamWaitEvent(stream(), P.ev_side, 0) != cudaSuccess) return check_cuda("peer: join");
        A.hi = P.hi < P.mid_off ? P.hi : P.mid_off;
        if (A.hi < A.lo) A.hi = A.lo;
        A.slot = kSlotFinalB;
        A.do_loss = 0;
        P.mid_off = -1;
    } else {                // one phase: the whole slice
        A.slot = kSlotFinalA;
        A.do_loss = 1;
    }
    peer_update_kernel<<<update_grid(A.hi - A.lo, 2), 128, 0, stream()>>>(A);
    ZB_LAUNCH_CHECK("peer update");
    P.cap_update = captured_node();
    peer_wait_kernel<<<1, 32, 0, stream()>>>(A);
    ZB_LAUNCH_CHECK("peer wait");
    P.cap_wait = captured_node();
    return kOk;
}

int peer_graph_args(Net &n, cudaGraphExec_t exec, cudaGraphNode_t upd, cudaGraphNode_t wt) {
    PeerState &P = n.peer;
    if (!P.on || P.two_phase || !upd || !wt) return fail(kBadArg, "peer: no captured one-phase step");
    P.step += 1;   // as peer_step_begin and peer_step_end would
    n.t += 1;
    PeerArgs A = make_args(n, P.step);
    A.a = make_adam_args(n.lr, n.b1, n.b2, n.eps, n.t, A.scale);
    A.written = 1;
    A.slot = kSlotFinalA;
    A.do_loss = 1;
    void *args[1] = {&A};
    for (cudaGraphNode_t node : {upd, wt}) {
        cudaKernelNodeParams kp{};
        if (cudaGraphKernelNodeGetParams(node, &kp) != cudaSuccess) return check_cuda("peer: graph node");
        kp.kernelParams = args;
        kp.extra = nullptr;
        if (cudaGraphExecKernelNodeSetParams(exec, node, &kp) != cudaSuccess) return check_cuda("peer: graph arguments");
    }
    return kOk;
}

}  // namespace zb
