// tc_net.cu -- bf16 tcgen05 engine of the fused training step (precision 1).
//
// Network shape handled (the reference's CNN family, src/NN):
//   Conv2D(1 -> C1, 3x3) + ReLU [+ MaxPool]        CUDA cores (K = 9)
//   { Conv2D(Cin -> Cout, 3x3, pad 1) + ReLU + MaxPool }*   tcgen05 implicit GEMM
//   [ Linear(F -> Hd) + ReLU ]                       tcgen05 GEMM
//   Linear(Hd -> classes) + softmax cross-entropy    fused head (CUDA cores)
// Activations are NHWC bf16; parameters, gradients and Adam state stay fp32
// (master weights); bf16 operand copies of the weights are packed at the
// start of each step.  The flat parameter / gradient layout and all
// semantics are those of the fp32 engine (net.cu).
//
// Step (large CNN, 8192 x 1x28x28):
//   pack -> conv1 -> conv2(+pool) -> conv3(+pool) -> fc1 -> head(fc2, CE, dZ)
//   -> fc1 dX, fc1 dW -> unpool3 -> conv3 dX, conv3 dW -> unpool2
//   -> conv2 dX (x ReLU mask of conv1) , conv2 dW -> conv1 dW -> Adam/SGD
#include <math.h>
#include <algorithm>
#include <string.h>

#include <string>
#include <vector>

#include "net.cuh"
#include "tc_conv.cuh"
#include "tc_conv_halo.cuh"
#include "tc_gemm.cuh"
#include "tc_wgrad.cuh"
#include "tc_wgrad_halo.cuh"
#include "tc_conv_bwd_fused.cuh"
#include "tc_conv_first.cuh"

namespace zb {

using tc::ConvTcParams;
using tc::ConvHaloParams;
using tc::GemmTcParams;
using tc::WgradTcParams;
using tc::WgradHaloParams;
using tc::ConvBwdFusedParams;

// ====================================================================== host: TMA maps
namespace tc {
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
}

int make_tmap_f32(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                  const uint32_t *box, Swizzle sw) {
    return make_tmap_typed(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, base, rank, dims, strides, box, sw);
}

int make_tmap_bf16(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                   const uint32_t *box, Swizzle sw) {
    return make_tmap_typed(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides, box, sw);
}

int make_tmap_typed(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, int rank, const uint64_t *dims,
                    const uint64_t *strides, const uint32_t *box, Swizzle sw) {
    if (!g_encode) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn) {
            cudaGetLastError();
            return fail(kCudaError, "cuTensorMapEncodeTiled unavailable");
        }
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    cuuint64_t gd[5], gs[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) { gd[i] = dims[i]; bx[i] = box[i]; es[i] = 1; }
    for (int i = 0; i < rank - 1; ++i) gs[i] = strides[i];
    CUtensorMapSwizzle s = sw == kSw128 ? CU_TENSOR_MAP_SWIZZLE_128B
                           : sw == kSw128B32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                           : sw == kSw64 ? CU_TENSOR_MAP_SWIZZLE_64B
                           : sw == kSw32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                         : CU_TENSOR_MAP_SWIZZLE_NONE;
    CUresult r = g_encode(map, dtype, (cuuint32_t)rank, const_cast<void *>(base), gd, gs,
                          bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, s, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(kCudaError, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return kOk;
}
}  // namespace tc

namespace {

using bf16 = __nv_bfloat16;

// ====================================================================== SIMT kernels
// Packs fp32 master weights into the bf16 operand layouts of the tensor-core
// kernels.  Jobs: 0 conv fwd  dst[t][co][ci] = W[co][ci][t]
//                 1 conv dgrad dst[t][ci][co] = W[co][ci][8-t]
//                 2 linear W^T  dst[n][k]     = W[perm(k)][n]   (K-major forward B)
//                 3 linear W    dst[k][n]     = W[perm(k)][n]   (K-major dgrad B)
//                 4 classifier  dst[(k/8)*98 + (k%8)*NC + n] = W[perm(k)][n]  (direct head:
//                   eight input rows of NC <= 12 bf16 per 196-byte group)
// perm maps an NHWC flatten index of the previous activation to the NCHW
// flatten index of the reference (src/Tensor/Tensor.php:958-981).
struct PackJob {
    int kind;
    const float *src;
    bf16 *dst;
    int a, b;          // conv: COUT, CIN;  linear: IN (K), OUT (N)
    int C, H, W;       // linear: geometry of the flattened activation (NHWC order)
    long long n;       // elements
};
constexpr int kMaxPack = 8;
struct PackJobs {
    PackJob j[kMaxPack];
    int count;
    int conv_blocks;   // pack_kernel's grid: conv_blocks for the jobs above + blocks for `fc`
    PackJob fc;        // the hidden Linear weight's rows (n = 0: none)
};

__device__ __forceinline__ int nhwc_to_nchw(int k, int C, int H, int W) {
    const int c = k % C, hw = k / C;
    return c * H * W + hw;
}

// Direct classifier head (Linear(F -> NC) right after the last pool): its bf16
// weights in groups of eight input rows, 98 bf16 (196 bytes, 49 words) per
// group.  Lane l of a warp reads group l + 32 j, so the 49-word pitch (odd)
// spreads a warp's 32 reads over 32 banks.
constexpr int kHeadGroup = 98;

// bf16 conv weights in the tensor-core layouts (32-bit index math; the conv
// weights are < 2^31 elements):
//   kind 0 (forward): dst[(t*COUT + co)*CIN + ci] = W[co][ci][t]
//   kind 1 (dgrad)  : dst[(t*CIN + ci)*COUT + co] = W[co][ci][8 - t]   (flipped, transposed)
// The bf16 copy of the hidden Linear weight W [F][N] (row-major over NCHW
// features) that both of its GEMMs read (the forward as an MN-major operand,
// the input gradient as a K-major one): wP[k'][n] = W[nchw(k')][n], k' the
// NHWC feature index of the conv output.  Four consecutive n per thread: one
// 16-byte load (N % 64 == 0; four loads if W is not 16-byte aligned), one
// 8-byte store.  J: src W, dst wP, a = F, b = N, C/H/W the flatten geometry.
__device__ __forceinline__ void pack_fc_rows(const PackJob &J, long long t, long long nt) {
    const int n4 = J.b / 4;
    const bool vec = (reinterpret_cast<uintptr_t>(J.src) & 15) == 0;
    for (long long q = t; q < (long long)J.a * n4; q += nt) {
        const int k = (int)(q / n4), c4 = (int)(q % n4);
        const float *src = J.src + (size_t)nhwc_to_nchw(k, J.C, J.H, J.W) * J.b + 4 * c4;
        const float4 v = vec ? __ldg(reinterpret_cast<const float4 *>(src)) : make_float4(src[0], src[1], src[2], src[3]);
        uint2 pk;
        __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
        h2[0] = __floats2bfloat162_rn(v.x, v.y);
        h2[1] = __floats2bfloat162_rn(v.z, v.w);
        reinterpret_cast<uint2 *>(J.dst + (size_t)k * J.b)[c4] = pk;
    }
}

// Every bf16 operand copy of the step from the fp32 master weights: the conv
// weights in their forward / input-gradient layouts, the direct classifier's
// grouped layout, and the hidden Linear weight's rows.  Thread t of nt takes
// elements t, t + nt, ... of each job.
__device__ __forceinline__ void pack_span(const PackJobs &jobs, long long t, long long nt) {
    for (int ji = 0; ji < jobs.count; ++ji) {
        const PackJob &J = jobs.j[ji];
        for (long long ii = t; ii < J.n; ii += nt) {
            const int i = (int)ii;
            float v;
            if (J.kind == 4) {   // i = k * NC + n over the classifier weight [F][NC]
                const int n = i % J.b, k = i / J.b;
                v = J.src[(size_t)nhwc_to_nchw(k, J.C, J.H, J.W) * J.b + n];
                J.dst[(k >> 3) * kHeadGroup + (k & 7) * J.b + n] = __float2bfloat16_rn(v);
                continue;
            }
            if (J.kind == 0) {
                const int ci = i % J.b, r = i / J.b, co = r % J.a, tp = r / J.a;
                v = J.src[(co * J.b + ci) * 9 + tp];
            } else {
                const int co = i % J.a, r = i / J.a, ci = r % J.b, tp = r / J.b;
                v = J.src[(co * J.b + ci) * 9 + (8 - tp)];
            }
            J.dst[i] = __float2bfloat16_rn(v);
        }
    }
    if (jobs.fc.n) pack_fc_rows(jobs.fc, t, nt);
}

// The packing as a launch of its own (engines whose first conv is not the
// tensor-core kernel, which otherwise does it: PackWork).
__global__ void __launch_bounds__(256) pack_kernel(const __grid_constant__ PackJobs jobs) {
    griddep_launch();
    griddep_wait();
    pack_span(jobs, (long long)blockIdx.x * blockDim.x + threadIdx.x, (long long)gridDim.x * blockDim.x);
}

// The packing as side work of the first conv's tensor-core kernel: its CTAs
// run it once before their tiles, so it costs no launch of its own (the conv
// reads the fp32 weights; every reader of the bf16 copies runs after it).
struct PackWork {
    PackJobs jobs;
    __device__ void operator()(long long t, long long nt) const { pack_span(jobs, t, nt); }
};

// First conv (CIN = 1, 3x3, stride 1, pad P) + bias + ReLU on CUDA cores,
// NHWC bf16 output; with `pool`, 2x2 max-pool + codes instead (same rules as
// the tensor-core epilogue).  One thread per output (or pooled) pixel, all
// COUT channels.  The tap sum runs in the reference order with fused
// multiply-adds (the output is rounded to bf16 anyway) (bias first, then
// kh, kw ascending).
template <int COUT, bool POOL>
__global__ void conv_first_fwd_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                      const float *__restrict__ bias, bf16 *__restrict__ out,
                                      uint8_t *__restrict__ code, int B, int H, int W, int pad) {
    __shared__ float sw[COUT * 9], sb[COUT];
    for (int i = threadIdx.x; i < COUT * 9; i += blockDim.x) sw[i] = w[i];
    for (int i = threadIdx.x; i < COUT; i += blockDim.x) sb[i] = bias[i];
    __syncthreads();
    const int oH = H + 2 * pad - 2, oW = W + 2 * pad - 2;
    const int pH = POOL ? oH / 2 : oH, pW = POOL ? oW / 2 : oW;
    const long long total = (long long)B * pH * pW;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int pw = (int)(i % pW), ph = (int)((i / pW) % pH), b = (int)(i / ((long long)pW * pH));
        const float *xb = x + (size_t)b * H * W;
        constexpr int NP = POOL ? 4 : 1;
        float patch[NP][9];
#pragma unroll
        for (int q = 0; q < NP; ++q) {
            const int oh = POOL ? 2 * ph + (q >> 1) : ph, ow = POOL ? 2 * pw + (q & 1) : pw;
#pragma unroll
            for (int t = 0; t < 9; ++t) {
                const int ih = oh - pad + t / 3, iw = ow - pad + t % 3;
                patch[q][t] = ((unsigned)ih < (unsigned)H && (unsigned)iw < (unsigned)W) ? xb[ih * W + iw] : 0.0f;
            }
        }
        const size_t o = (size_t)i * COUT;
#pragma unroll 4
        for (int c0 = 0; c0 < COUT; c0 += 8) {
            float best[8];
            int pos[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int co = c0 + e;
#pragma unroll
                for (int q = 0; q < NP; ++q) {
                    float acc = sb[co];
#pragma unroll
                    for (int t = 0; t < 9; ++t) acc = fmaf(patch[q][t], sw[co * 9 + t], acc);
                    acc = acc > 0.0f ? acc : 0.0f;
                    if (q == 0 || acc > best[e]) { best[e] = acc; pos[e] = q; }
                }
            }
            uint4 pk;
            __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) h2[e] = __floats2bfloat162_rn(best[2 * e], best[2 * e + 1]);
            *reinterpret_cast<uint4 *>(out + o + c0) = pk;
            if (POOL) {
                uint2 cp;
                uint8_t *cb = reinterpret_cast<uint8_t *>(&cp);
#pragma unroll
                for (int e = 0; e < 8; ++e) cb[e] = (uint8_t)(pos[e] | (best[e] > 0.0f ? 4 : 0));
                *reinterpret_cast<uint2 *>(code + o + c0) = cp;
            }
        }
    }
}

// Packed two-lane fp32 FMA (sm_100): d = a * b + c per lane, each lane
// rounded exactly as fmaf.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    uint64_t ra = *reinterpret_cast<uint64_t *>(&a), rb = *reinterpret_cast<uint64_t *>(&b),
             rc = *reinterpret_cast<uint64_t *>(&c), rd;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
    return *reinterpret_cast<float2 *>(&rd);
}

// Zero-padded image staging for the first-conv kernels: each of the 256
// threads owns up to kStageRegs elements of the (H+2p) x (W+2p) padded image;
// their source offsets (-1 = padding) are fixed per thread, and the next
// image is loaded into registers while the current one is being used, so the
// global-load latency overlaps the compute.
constexpr int kStageRegs = 4;

// Asynchronous staging of one image into a zero-padded shared-memory buffer:
// element i of the [H][W] image goes to ((i / W) + pad) * (W + 2 pad) + (i % W) + pad
// by a 4-byte cp.async (the halo is never written, so it stays zero).  The
// coordinates advance by 256 elements per step (no division in the loop).
__device__ __forceinline__ void stage_image_async(float *buf, const float *__restrict__ xb, int H, int W, int pad) {
    const int PW = W + 2 * pad;
    int ih = (int)threadIdx.x / W, iw = (int)threadIdx.x - ih * W;
    const int dh = 256 / W, dw = 256 - dh * W;
    for (int i = threadIdx.x; i < H * W; i += 256) {
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(buf + (ih + pad) * PW + iw + pad);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(xb + i) : "memory");
        ih += dh;
        iw += dw;
        if (iw >= W) { iw -= W; ++ih; }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

struct ImageStager {
    int off[kStageRegs];
    float v[kStageRegs];
    __device__ void init(int H, int W, int pad) {
        const int PW = W + 2 * pad, PH = H + 2 * pad;
#pragma unroll
        for (int k = 0; k < kStageRegs; ++k) {
            const int i = threadIdx.x + k * 256;
            const int ih = i / PW - pad, iw = i % PW - pad;
            off[k] = (i < PH * PW && (unsigned)ih < (unsigned)H && (unsigned)iw < (unsigned)W) ? ih * W + iw
                     : (i < PH * PW ? -1 : -2);
        }
    }
    __device__ void load(const float *__restrict__ xb) {
#pragma unroll
        for (int k = 0; k < kStageRegs; ++k) v[k] = off[k] >= 0 ? __ldg(xb + off[k]) : 0.0f;
    }
    __device__ void store(float *xs) const {
#pragma unroll
        for (int k = 0; k < kStageRegs; ++k)
            if (off[k] != -2) xs[threadIdx.x + k * 256] = v[k];
    }
};

// First conv without a following pool.  A block walks whole images: the
// zero-padded image is staged in shared memory; thread = (column, pair of
// output rows, 8-channel octet), octets fastest, so for each of its two rows
// a warp writes 8 consecutive pixels x COUT bf16 as one contiguous run.  The
// two pixels share 6 of their 12 inputs and give two independent FMA chains;
// the octet's 72 weights and 8 biases live in registers.  Coordinates
// advance incrementally (no division in the loop).
template <int COUT>
__global__ void __launch_bounds__(256, 2) conv_first_fwd_img_kernel(const float *__restrict__ x,
                                                                 const float *__restrict__ w,
                                                                 const float *__restrict__ bias,
                                                                 bf16 *__restrict__ out, int B, int H, int W,
                                                                 int pad) {
    constexpr int NQ = COUT / 8;
    constexpr int LANES = 256 / NQ;
    extern __shared__ float xs[];
    const int q = threadIdx.x % NQ, pl = threadIdx.x / NQ;
    const int oH = H + 2 * pad - 2, oW = W + 2 * pad - 2;
    const int PW = W + 2 * pad, PH = H + 2 * pad;
    const int nrp = (oH + 1) / 2;            // row pairs
    const int NP = nrp * oW;                 // (row pair, column) items per image
    const int step_r = LANES / oW, step_c = LANES % oW;
    float2 wr2[4][9], br2[4];   // channel pairs (2k, 2k + 1) of the octet
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        br2[k] = make_float2(__ldg(bias + 8 * q + 2 * k), __ldg(bias + 8 * q + 2 * k + 1));
#pragma unroll
        for (int t = 0; t < 9; ++t)
            wr2[k][t] = make_float2(__ldg(w + (8 * q + 2 * k) * 9 + t), __ldg(w + (8 * q + 2 * k + 1) * 9 + t));
    }
    ImageStager stg;
    stg.init(H, W, pad);
    if (blockIdx.x < B) stg.load(x + (size_t)blockIdx.x * H * W);
    for (int b = blockIdx.x; b < B; b += gridDim.x) {
        __syncthreads();
        stg.store(xs);
        __syncthreads();
        if (b + (int)gridDim.x < B) stg.load(x + (size_t)(b + gridDim.x) * H * W);
        bf16 *ob = out + (size_t)b * oH * oW * COUT + 8 * q;
        int rp = pl / oW, ow = pl - (pl / oW) * oW;
        for (int it = pl; it < NP; it += LANES) {
            const int oh = 2 * rp;
            const float *xr = xs + oh * PW + ow;   // rows oh .. oh + 3 of the padded image
            float xv[4][3];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int k = 0; k < 3; ++k) xv[r][k] = (oh + r < PH) ? xr[r * PW + k] : 0.0f;
#pragma unroll
            for (int dr = 0; dr < 2; ++dr) {
                if (oh + dr >= oH) break;
                uint4 pk;
                __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                for (int e2 = 0; e2 < 4; ++e2) {
                    float2 a = br2[e2];
#pragma unroll
                    for (int t = 0; t < 9; ++t) {
                        const float xt = xv[dr + t / 3][t % 3];
                        a = ffma2(make_float2(xt, xt), wr2[e2][t], a);
                    }
                    h2[e2] = __floats2bfloat162_rn(a.x > 0.0f ? a.x : 0.0f, a.y > 0.0f ? a.y : 0.0f);
                }
                *reinterpret_cast<uint4 *>(ob + ((size_t)(oh + dr) * oW + ow) * COUT) = pk;
            }
            rp += step_r;
            ow += step_c;
            if (ow >= oW) { ow -= oW; ++rp; }
        }
    }
}

// First conv followed by a 2x2 max-pool, for images staged in shared memory: a
// block walks whole images (the zero-padded image copied by a plain loop);
// thread = (pooled window, 8-channel octet), octets fastest, so a warp writes
// consecutive windows' channels as one contiguous run.  The window's 4 x 4 input
// neighbourhood is read once for its four pixels; the octet's 72 weights and 8
// biases live in registers as channel pairs, and each pair's four pixels are
// summed with packed fp32x2 FMAs in the order of conv_first_fwd_kernel (bias,
// then the taps ascending; each lane rounds like fmaf), then ReLU and the pool
// with its rules (first maximum of the fp32 values, code = position | 4 when
// positive): the same outputs and codes bit for bit.
template <int COUT>
__global__ void __launch_bounds__(256, 2) conv_first_pool_img_kernel(const float *__restrict__ x,
                                                                  const float *__restrict__ w,
                                                                  const float *__restrict__ bias,
                                                                  bf16 *__restrict__ out, uint8_t *__restrict__ code,
                                                                  int B, int H, int W, int pad) {
    constexpr int NQ = COUT / 8;
    constexpr int LANES = 256 / NQ;
    extern __shared__ float xbuf[];   // two zero-padded images: the next one lands while this one is used
    const int q = threadIdx.x % NQ, pl = threadIdx.x / NQ;
    const int oH = H + 2 * pad - 2, oW = W + 2 * pad - 2;
    const int pH = oH >> 1, pW = oW >> 1, NW = pH * pW;
    const int PH = H + 2 * pad, PW = W + 2 * pad;
    float2 wr2[4][9], br2[4];   // channel pairs (2k, 2k + 1) of the octet
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        br2[k] = make_float2(__ldg(bias + 8 * q + 2 * k), __ldg(bias + 8 * q + 2 * k + 1));
#pragma unroll
        for (int t = 0; t < 9; ++t)
            wr2[k][t] = make_float2(__ldg(w + (8 * q + 2 * k) * 9 + t), __ldg(w + (8 * q + 2 * k + 1) * 9 + t));
    }
    const int NPX = PH * PW;
    for (int i = threadIdx.x; i < 2 * NPX; i += 256) xbuf[i] = 0.0f;
    __syncthreads();
    if ((int)blockIdx.x < B) stage_image_async(xbuf, x + (size_t)blockIdx.x * H * W, H, W, pad);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    int it = 0;
    for (int b = blockIdx.x; b < B; b += gridDim.x, ++it) {
        const int nb = b + (int)gridDim.x;
        if (nb < B) stage_image_async(xbuf + ((it + 1) & 1) * NPX, x + (size_t)nb * H * W, H, W, pad);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");   // this image's copies are done
        __syncthreads();
        const float *xs = xbuf + (it & 1) * NPX;
        for (int wi = pl; wi < NW; wi += LANES) {
            const int ph = wi / pW, pw = wi - ph * pW;
            const float *xr = xs + (2 * ph) * PW + 2 * pw;
            float xv[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) xv[r][c] = xr[r * PW + c];
            uint4 pk;
            __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
            uint2 cp;
            uint8_t *cb = reinterpret_cast<uint8_t *>(&cp);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float2 best = make_float2(0.0f, 0.0f);
                int px = 0, py = 0;
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) {   // window position (kh, kw) = (qq >> 1, qq & 1)
                    const int dy = qq >> 1, dx = qq & 1;
                    float2 a = br2[k];
#pragma unroll
                    for (int t = 0; t < 9; ++t) {
                        const float xt = xv[dy + t / 3][dx + t % 3];
                        a = ffma2(make_float2(xt, xt), wr2[k][t], a);
                    }
                    a.x = a.x > 0.0f ? a.x : 0.0f;
                    a.y = a.y > 0.0f ? a.y : 0.0f;
                    if (qq == 0 || a.x > best.x) { best.x = a.x; px = qq; }
                    if (qq == 0 || a.y > best.y) { best.y = a.y; py = qq; }
                }
                h2[k] = __floats2bfloat162_rn(best.x, best.y);
                cb[2 * k] = (uint8_t)(px | (best.x > 0.0f ? 4 : 0));
                cb[2 * k + 1] = (uint8_t)(py | (best.y > 0.0f ? 4 : 0));
            }
            const size_t o = ((size_t)b * NW + wi) * COUT + 8 * q;
            *reinterpret_cast<uint4 *>(out + o) = pk;
            *reinterpret_cast<uint2 *>(code + o) = cp;
        }
        __syncthreads();   // every thread is done with this buffer before it is refilled
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// First-conv weight and bias gradient: dW[co][t] = sum_p dC[p][co] x[p + t],
// db[co] = sum_p dC[p][co].  A block walks whole images: the image (with a
// zero halo) is staged in shared memory; thread (pixel lane, channel octet)
// loads 8 bf16 of dC per pixel as one 16-byte load (a warp reads 8 pixels x
// 32 channels = 512 contiguous bytes), four pixels' loads in flight at once,
// and keeps 8 x 10 accumulators.  Lanes of a warp that share an octet are
// combined by shuffles, warps in fixed order through shared memory: per-block
// partials [block][COUT][10], summed later in block order.  Dynamic shared
// memory: max((H+2p)(W+2p), 8*4*80) floats.  BIG: images past the 1024
// elements the register stager holds (e.g. 64 x 101 spectrograms) are copied
// into shared memory by a plain loop per image instead.
template <int COUT, bool BIG = false>
__global__ void __launch_bounds__(256, 2) conv_first_wgrad_kernel(const bf16 *__restrict__ dC,
                                                               const float *__restrict__ x,
                                                               float *__restrict__ partial, int B, int H, int W,
                                                               int pad) {
    constexpr int NQ = COUT / 8;            // channel octets per pixel
    constexpr int LANES = 256 / NQ;         // pixel lanes per block
    constexpr int U = 4;                    // pixels per thread in flight
    extern __shared__ float xs[];
    const int q = threadIdx.x % NQ, pl = threadIdx.x / NQ;
    const int oH = H + 2 * pad - 2, oW = W + 2 * pad - 2, P = oH * oW;
    const int PH = H + 2 * pad, PW = W + 2 * pad;
    const int step_h = LANES / oW, step_w = LANES % oW;
    float2 acc2[4][10];   // channel pairs (2k, 2k + 1); t = 9 is the bias sum
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int t = 0; t < 10; ++t) acc2[k][t] = make_float2(0.0f, 0.0f);
    ImageStager stg;
    if constexpr (!BIG) {
        stg.init(H, W, pad);
        if (blockIdx.x < B) stg.load(x + (size_t)blockIdx.x * H * W);
    }
    for (int b = blockIdx.x; b < B; b += gridDim.x) {
        __syncthreads();
        if constexpr (BIG) {
            const float *xb = x + (size_t)b * H * W;
            for (int i = threadIdx.x; i < PH * PW; i += 256) {
                const int ih = i / PW - pad, iw = i - (i / PW) * PW - pad;
                xs[i] = ((unsigned)ih < (unsigned)H && (unsigned)iw < (unsigned)W) ? __ldg(xb + ih * W + iw) : 0.0f;
            }
        } else {
            stg.store(xs);
        }
        __syncthreads();
        if constexpr (!BIG)
            if (b + (int)gridDim.x < B) stg.load(x + (size_t)(b + gridDim.x) * H * W);
        const bf16 *gb = dC + (size_t)b * P * COUT + 8 * q;
        int oh = pl / oW, ow = pl - (pl / oW) * oW;
        for (int p0 = pl; p0 < P; p0 += U * LANES) {
            uint4 raw[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int p = p0 + u * LANES;
                raw[u] = p < P ? __ldg(reinterpret_cast<const uint4 *>(gb + (size_t)p * COUT)) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (p0 + u * LANES >= P) break;
                const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&raw[u]);
                float2 g2[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) g2[k] = __bfloat1622float2(h2[k]);
                const float *xr = xs + oh * PW + ow;
                float xv[9];
#pragma unroll
                for (int t = 0; t < 9; ++t) xv[t] = xr[(t / 3) * PW + (t % 3)];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
#pragma unroll
                    for (int t = 0; t < 9; ++t) acc2[k][t] = ffma2(g2[k], make_float2(xv[t], xv[t]), acc2[k][t]);
                    acc2[k][9] = ffma2(g2[k], make_float2(1.0f, 1.0f), acc2[k][9]);
                }
                oh += step_h;
                ow += step_w;
                if (ow >= oW) { ow -= oW; ++oh; }
            }
        }
    }
    // lanes of a warp with the same octet: lane = pixel-slot * NQ + q
#pragma unroll
    for (int off = NQ; off < 32; off <<= 1)
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int t = 0; t < 10; ++t) {
                acc2[k][t].x += __shfl_xor_sync(0xffffffffu, acc2[k][t].x, off);
                acc2[k][t].y += __shfl_xor_sync(0xffffffffu, acc2[k][t].y, off);
            }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *red = xs;   // [8 warps][NQ][80]
    if (lane < NQ)
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
            for (int t = 0; t < 10; ++t) {
                red[(warp * NQ + lane) * 80 + (2 * k) * 10 + t] = acc2[k][t].x;
                red[(warp * NQ + lane) * 80 + (2 * k + 1) * 10 + t] = acc2[k][t].y;
            }
    __syncthreads();
    for (int i = threadIdx.x; i < COUT * 10; i += blockDim.x) {   // i = co*10 + t, co = 8q + e
        const int co = i / 10, t = i % 10, qq = co / 8, e = co % 8;
        float s = 0.0f;
        for (int wv = 0; wv < 8; ++wv) s += red[(wv * NQ + qq) * 80 + e * 10 + t];
        partial[(size_t)blockIdx.x * COUT * 10 + i] = s;
    }
}

// First-conv weight and bias gradient when the conv is followed by a 2x2 max-pool:
// dW[co][t] = sum_p dC[p][co] x[p + t] where dC = unpool(dP, codes) holds, per
// window and channel, dP at the position the code names (and only when the
// maximum was positive), zero at the other three.  So the sum runs over windows:
// thread = (window lane, 8-channel octet): one 16-byte dP load and one 8-byte
// code load per window, and for each routed channel the 3 x 3 patch of the
// zero-padded image (staged in shared memory per image) at the routed pixel, 10
// FMAs (9 taps + bias).  A quarter of the dense sum's FMAs and no full-size dC.
// Partials as conv_first_wgrad_kernel: [block][COUT][10], lanes of an octet
// combined by shuffles, warps in fixed order.
template <int COUT>
__global__ void __launch_bounds__(256, 2) conv_first_wgrad_pool_kernel(const bf16 *__restrict__ dP,
                                                                    const uint8_t *__restrict__ code,
                                                                    const float *__restrict__ x,
                                                                    float *__restrict__ partial, int B, int H, int W,
                                                                    int pad) {
    constexpr int NQ = COUT / 8;
    constexpr int LANES = 256 / NQ;
    extern __shared__ float xbuf[];   // two zero-padded images: the next one lands while this one is used
    const int q = threadIdx.x % NQ, pl = threadIdx.x / NQ;
    const int oH = H + 2 * pad - 2, oW = W + 2 * pad - 2;
    const int Ho = oH >> 1, Wo = oW >> 1, NW = Ho * Wo;
    const int PH = H + 2 * pad, PW = W + 2 * pad;
    float acc[8][10];
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
        for (int t = 0; t < 10; ++t) acc[e][t] = 0.0f;
    const int NPX = PH * PW;
    for (int i = threadIdx.x; i < 2 * NPX; i += 256) xbuf[i] = 0.0f;
    __syncthreads();
    if ((int)blockIdx.x < B) stage_image_async(xbuf, x + (size_t)blockIdx.x * H * W, H, W, pad);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    int it = 0;
    for (int b = blockIdx.x; b < B; b += gridDim.x, ++it) {
        const int nb = b + (int)gridDim.x;
        if (nb < B) stage_image_async(xbuf + ((it + 1) & 1) * NPX, x + (size_t)nb * H * W, H, W, pad);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");   // this image's copies are done
        __syncthreads();
        const float *xs = xbuf + (it & 1) * NPX;
        const size_t ob = (size_t)b * NW * COUT + 8 * q;
        for (int wi = pl; wi < NW; wi += LANES) {
            const int ph = wi / Wo, pw = wi - ph * Wo;
            const uint4 dv = __ldg(reinterpret_cast<const uint4 *>(dP + ob + (size_t)wi * COUT));
            const uint2 cv = __ldg(reinterpret_cast<const uint2 *>(code + ob + (size_t)wi * COUT));
            const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
            const uint32_t cw[2] = {cv.x, cv.y};
            // window top-left in padded-image coordinates of the conv output pixel (2ph, 2pw):
            // output pixel (oh, ow) reads padded rows oh .. oh + 2, columns ow .. ow + 2
            const int base0 = (2 * ph) * PW + 2 * pw;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t c = (cw[e >> 2] >> (8 * (e & 3))) & 0xFFu;
                if (!(c & 4u)) continue;   // the window's maximum was not positive: no gradient
                const float g = __uint_as_float(e & 1 ? dw[e >> 1] & 0xFFFF0000u : dw[e >> 1] << 16);
                const float *xr = xs + base0 + (int)((c >> 1) & 1u) * PW + (int)(c & 1u);
#pragma unroll
                for (int t = 0; t < 9; ++t) acc[e][t] = fmaf(g, xr[(t / 3) * PW + (t % 3)], acc[e][t]);
                acc[e][9] += g;
            }
        }
        __syncthreads();   // every thread is done with this buffer before it is refilled
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    // lanes of a warp with the same octet: lane = window-slot * NQ + q
#pragma unroll
    for (int off = NQ; off < 32; off <<= 1)
#pragma unroll
        for (int e = 0; e < 8; ++e)
#pragma unroll
            for (int t = 0; t < 10; ++t) acc[e][t] += __shfl_xor_sync(0xffffffffu, acc[e][t], off);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *red = xbuf;   // [8 warps][NQ][80]
    if (lane < NQ)
#pragma unroll
        for (int e = 0; e < 8; ++e)
#pragma unroll
            for (int t = 0; t < 10; ++t) red[(warp * NQ + lane) * 80 + e * 10 + t] = acc[e][t];
    __syncthreads();
    for (int i = threadIdx.x; i < COUT * 10; i += blockDim.x) {   // i = co*10 + t, co = 8q + e
        const int co = i / 10, t = i % 10, qq = co / 8, e = co % 8;
        float sum = 0.0f;
        for (int wv = 0; wv < 8; ++wv) sum += red[(wv * NQ + qq) * 80 + e * 10 + t];
        partial[(size_t)blockIdx.x * COUT * 10 + i] = sum;
    }
}

// Max-pool + ReLU backward as a gather: dC[b,h,w,c] = dP[b,h/2,w/2,c] when the
// window's code points at (h,w) and its maximum was positive, else 0.  One
// thread per (window, 8-channel octet): one 16-byte load of dP and one 8-byte
// load of the codes, four 16-byte stores (a warp writes whole contiguous
// 2-pixel row segments).  Rows / columns outside every window (floor pooling
// of an odd size) are zero-filled.  Bias-gradient partials sum_p dC[p][c] =
// sum over windows of dP * [max > 0], per block (fixed combine order).
__global__ void unpool_kernel(const bf16 *__restrict__ dP, const uint8_t *__restrict__ code, bf16 *__restrict__ dC,
                              float *__restrict__ bias_partial, int B, int H, int W, int C) {
    const int G = C / 8;                   // channel octets
    const int slots = blockDim.x / G;
    const int g = threadIdx.x % G, slot = threadIdx.x / G;
    const int Ho = H / 2, Wo = W / 2;
    const long long windows = (long long)B * Ho * Wo;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    if (slot < slots) {
        for (long long wi = (long long)blockIdx.x * slots + slot; wi < windows; wi += (long long)gridDim.x * slots) {
            const int pw = (int)(wi % Wo);
            const long long r = wi / Wo;
            const int ph = (int)(r % Ho);
            const long long b = r / Ho;
            const size_t o = (size_t)wi * C + g * 8;
            const uint2 cv = __ldg(reinterpret_cast<const uint2 *>(code + o));
            const uint4 dv = __ldg(reinterpret_cast<const uint4 *>(dP + o));
            const uint8_t *cb = reinterpret_cast<const uint8_t *>(&cv);
            const bf16 *db = reinterpret_cast<const bf16 *>(&dv);
            uint4 outv[4];
            const unsigned short *du = reinterpret_cast<const unsigned short *>(db);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                unsigned short *ou = reinterpret_cast<unsigned short *>(&outv[k]);
#pragma unroll
                for (int e = 0; e < 8; ++e) ou[e] = (cb[e] & 7) == (4 | k) ? du[e] : (unsigned short)0;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e)
                if (cb[e] & 4) acc[e] += __bfloat162float(db[e]);
            bf16 *row0 = dC + (((size_t)b * H + 2 * ph) * W + 2 * pw) * C + g * 8;
            *reinterpret_cast<uint4 *>(row0) = outv[0];
            *reinterpret_cast<uint4 *>(row0 + C) = outv[1];
            *reinterpret_cast<uint4 *>(row0 + (size_t)W * C) = outv[2];
            *reinterpret_cast<uint4 *>(row0 + (size_t)W * C + C) = outv[3];
        }
        // zero the last row / column that no window covers (odd H or W)
        if ((H & 1) || (W & 1)) {
            const int extra = ((H & 1) ? W : 0) + ((W & 1) ? H - (H & 1) : 0);
            const long long total = (long long)B * extra;
            for (long long i = (long long)blockIdx.x * slots + slot; i < total; i += (long long)gridDim.x * slots) {
                const long long b = i / extra;
                const int k = (int)(i % extra);
                int h, w;
                if ((H & 1) && k < W) { h = H - 1; w = k; }
                else { h = k - ((H & 1) ? W : 0); w = W - 1; }
                *reinterpret_cast<uint4 *>(dC + (((size_t)b * H + h) * W + w) * C + g * 8) = make_uint4(0, 0, 0, 0);
            }
        }
    }
    extern __shared__ float red[];   // [blockDim.x][8]
#pragma unroll
    for (int e = 0; e < 8; ++e) red[threadIdx.x * 8 + e] = acc[e];
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const int gg = c / 8, e = c % 8;
        float s = 0.0f;
        for (int sl = 0; sl < slots; ++sl) s += red[(sl * G + gg) * 8 + e];
        bias_partial[(size_t)blockIdx.x * C + c] = s;
    }
}

// A head block's partial: dW [Hd][NC], db [NC], dbPrev [Hd], the loss, then zeros up to a
// multiple of 4 floats (16-byte aligned rows for the split reduction's vector loads).
__host__ __device__ constexpr int head_pstride(int HD, int NC) { return (HD * NC + NC + HD + 1 + 3) / 4 * 4; }

// Head: last Linear (Hd -> NC, NC <= 32) + softmax cross-entropy + the start
// of the backward, one warp per row:
//   z = a W + b;  loss_r = -log softmax(z)[y];  dz = (p - onehot)/B
//   dA = dz W^T times (a > 0) (ReLU of the previous Linear) -> bf16
// The rows' a and dz are staged in shared memory, kHeadRpw rows per warp at a
// time; after each such chunk thread k adds, over the chunk's rows in order
// (warp 0's rows first), dW[k][n] += a[k] dz[n], dA[k] = (a[k] > 0) sum_n dz[n] W[k][n]
// (written out, and added into dbPrev[k]) and, for k < NC, db[k] += dz[k].  So no
// thread holds more than NC + 2 accumulators.  Block partial: dW [Hd][NC], db [NC],
// dbPrev [Hd] and the block's loss sum (warps in order).
// With SPLIT the previous Linear split its K: a[r][k] is taken here as
// bf16(relu(sum_s fpart[s][r][k] + fbias[k])), the splits added in order from
// split 0 (the split-K reduction's own arithmetic, so the values are the same),
// and written to `a` for later readers.
constexpr int kHeadRpw = 4;
template <int HD, int NC, bool SPLIT = false>
__global__ void __launch_bounds__(256, 2) head_kernel(bf16 *__restrict__ a, const float *__restrict__ Wt,
                                                      const float *__restrict__ bias, const float *__restrict__ y,
                                                      bf16 *__restrict__ dA, double *__restrict__ row_loss,
                                                      float *__restrict__ partial, int B, float invB,
                                                      const float *__restrict__ fpart, int ksplit,
                                                      const float *__restrict__ fbias) {
    static_assert(HD == 256, "one thread per input of the previous Linear");
    constexpr int KPL = HD / 32;   // inputs per lane
    constexpr int SLOTS = 8 * kHeadRpw;
    __shared__ float sW[HD * NC];
    __shared__ bf16 sA[SLOTS][HD];
    __shared__ float sDz[SLOTS][NC];
    __shared__ double sLoss[8];
    griddep_launch();
    griddep_wait();
    for (int i = threadIdx.x; i < HD * NC; i += blockDim.x) sW[i] = Wt[i];
    double lsum = 0.0;   // lane 0: this warp's rows' loss
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = threadIdx.x;   // the post-pass: input k = t
    float gW[NC], gP = 0.0f, gB = 0.0f;
#pragma unroll
    for (int n = 0; n < NC; ++n) gW[n] = 0.0f;
    const long long step = (long long)gridDim.x * 8;
    for (long long base = (long long)blockIdx.x * 8; base < B; base += step * kHeadRpw) {
        // row loop: this warp's rows base + warp + i * step, i < kHeadRpw
        for (int i = 0; i < kHeadRpw; ++i) {
            const long long rr = base + warp + i * step;
            const int slot = warp * kHeadRpw + i;
            if (rr >= B) {
                if (lane < NC) sDz[slot][lane] = 0.0f;
#pragma unroll
                for (int j = 0; j < KPL; ++j) sA[slot][lane + 32 * j] = __float2bfloat16_rn(0.0f);
                continue;
            }
            const int r = (int)rr;
            float av[KPL];
            if constexpr (SPLIT) {
                const float *pr = fpart + (size_t)r * HD + lane;
                const size_t sstride = (size_t)B * HD;
#pragma unroll
                for (int j = 0; j < KPL; ++j) av[j] = __ldcs(pr + 32 * j);
#pragma unroll 4
                for (int sp = 1; sp < ksplit; ++sp) {
                    float v[KPL];
#pragma unroll
                    for (int j = 0; j < KPL; ++j) v[j] = __ldcs(pr + sp * sstride + 32 * j);
#pragma unroll
                    for (int j = 0; j < KPL; ++j) av[j] += v[j];
                }
#pragma unroll
                for (int j = 0; j < KPL; ++j) {
                    const int k = lane + 32 * j;
                    const float x = av[j] + fbias[k];
                    const bf16 h = __float2bfloat16_rn(x > 0.0f ? x : 0.0f);
                    a[(size_t)r * HD + k] = h;
                    sA[slot][k] = h;
                    av[j] = __bfloat162float(h);
                }
            } else {
#pragma unroll
                for (int j = 0; j < KPL; ++j) {
                    const bf16 h = a[(size_t)r * HD + lane + 32 * j];
                    sA[slot][lane + 32 * j] = h;
                    av[j] = __bfloat162float(h);
                }
            }
            float z[NC];
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < KPL; ++j) s = fmaf(av[j], sW[(lane + 32 * j) * NC + n], s);
#pragma unroll
                for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                z[n] = s + bias[n];
            }
            float mx = z[0];
#pragma unroll
            for (int n = 1; n < NC; ++n) mx = fmaxf(mx, z[n]);
            float se = 0.0f;
#pragma unroll
            for (int n = 0; n < NC; ++n) se += expf(z[n] - mx);
            const int tg = (int)y[r];
            float dz[NC];
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                const float p = expf(z[n] - mx) / se;
                dz[n] = (p - (n == tg ? 1.0f : 0.0f)) * invB;
            }
            if (lane < NC) {
                float v = dz[0];
#pragma unroll
                for (int n = 1; n < NC; ++n) if (n == lane) v = dz[n];
                sDz[slot][lane] = v;
            }
            if (lane == 0) {
                float pt = 0.0f;
#pragma unroll
                for (int n = 0; n < NC; ++n) if (n == tg) pt = expf(z[n] - mx) / se;
                row_loss[r] = -(double)logf(pt);
                lsum += -(double)logf(pt);
            }
        }
        __syncthreads();
        // post-pass over the chunk's rows in slot order (rows past B hold zeros): thread t
        // takes input k = t of every row, and writes the row's dA[k] (coalesced rows)
        float wk[NC];
#pragma unroll
        for (int n = 0; n < NC; ++n) wk[n] = sW[t * NC + n];
        for (int sl = 0; sl < SLOTS; ++sl) {
            const float av = __bfloat162float(sA[sl][t]);
            float g = 0.0f;
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                const float d = sDz[sl][n];
                gW[n] = fmaf(av, d, gW[n]);
                g = fmaf(d, wk[n], g);
            }
            g = av > 0.0f ? g : 0.0f;
            gP += g;
            if (t < NC) gB += sDz[sl][t];
            const long long rr = base + (sl / kHeadRpw) + (long long)(sl % kHeadRpw) * step;
            if (rr < B) dA[(size_t)rr * HD + t] = __float2bfloat16_rn(g);
        }
        __syncthreads();
    }
    if (lane == 0) sLoss[warp] = lsum;
    __syncthreads();
    float *dst = partial + (size_t)blockIdx.x * head_pstride(HD, NC);
#pragma unroll
    for (int n = 0; n < NC; ++n) dst[t * NC + n] = gW[n];
    if (t < NC) dst[HD * NC + t] = gB;
    dst[HD * NC + NC + t] = gP;
    if (t == 0) {
        double ls = 0.0;
        for (int w = 0; w < 8; ++w) ls += sLoss[w];
        dst[HD * NC + NC + HD] = (float)ls;
    }
    for (int i = HD * NC + NC + HD + 1 + t; i < head_pstride(HD, NC); i += blockDim.x) dst[i] = 0.0f;
}

// Forward-only classifier (evaluation): one warp per row, fp32 logits
// z = a W + b with head_kernel's arithmetic, and (y given) the rows' loss
// -log softmax(z)[y] summed per block in a fixed warp order into partial[block].
template <int HD, int NC>
__global__ void __launch_bounds__(256) head_fwd_kernel(const bf16 *__restrict__ a, const float *__restrict__ Wt,
                                                       const float *__restrict__ bias, const float *__restrict__ y,
                                                       float *__restrict__ logits, float *__restrict__ partial, int B) {
    constexpr int KPL = HD / 32;
    __shared__ float sW[HD * NC];
    __shared__ double sLoss[8];
    griddep_launch();
    griddep_wait();
    for (int i = threadIdx.x; i < HD * NC; i += blockDim.x) sW[i] = Wt[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    double lsum = 0.0;
    for (int r = blockIdx.x * 8 + warp; r < B; r += gridDim.x * 8) {
        float av[KPL];
#pragma unroll
        for (int j = 0; j < KPL; ++j) av[j] = __bfloat162float(a[(size_t)r * HD + lane + 32 * j]);
        float z[NC];
#pragma unroll
        for (int n = 0; n < NC; ++n) {
            float s = 0.0f;
#pragma unroll
            for (int j = 0; j < KPL; ++j) s = fmaf(av[j], sW[(lane + 32 * j) * NC + n], s);
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            z[n] = s + bias[n];
        }
        if (lane < NC) {
            float zl = z[0];
#pragma unroll
            for (int n = 1; n < NC; ++n) if (lane == n) zl = z[n];
            logits[(size_t)r * NC + lane] = zl;
        }
        if (y && lane == 0) {
            float mx = z[0];
#pragma unroll
            for (int n = 1; n < NC; ++n) mx = fmaxf(mx, z[n]);
            float se = 0.0f;
#pragma unroll
            for (int n = 0; n < NC; ++n) se += expf(z[n] - mx);
            const int t = (int)y[r];
            float pt = 0.0f;
#pragma unroll
            for (int n = 0; n < NC; ++n) if (n == t) pt = expf(z[n] - mx) / se;
            lsum += -(double)logf(pt);
        }
    }
    if (lane == 0) sLoss[warp] = lsum;
    __syncthreads();
    if (threadIdx.x == 0 && partial) {
        double t = 0.0;
        for (int w = 0; w < 8; ++w) t += sLoss[w];
        partial[blockIdx.x] = (float)t;
    }
}

// Direct head: the classifier Linear (F -> NC, NC <= 12) on the flattened last
// pooled activation a [B][F] (NHWC order, bf16), softmax cross-entropy and the
// start of the backward:
//   z = a W + b;  loss_r = -log softmax(z)[y];  dz = (p - onehot) / B
//   dA = dz W^T -> bf16 [B][F]  (the pool's ReLU lives in the pool codes)
// W comes packed in bf16 groups (kHeadGroup) and stays in shared memory
// (F / 8 groups of 196 bytes: 147 KB at F = 6144), shared by the block's 16
// warps.  A warp takes two rows at a time: lane l owns the 8-input groups l,
// l + 32, ... of both, so each weight word read from shared memory serves two
// rows, and the next group's two 16-byte loads of a are issued before the
// current group's arithmetic.  dz goes to global memory for the weight-gradient
// kernel; the block's bias-gradient and loss partial is [NC + 1] (fixed warp
// order).  logits != null: the evaluation forward (logits out, the loss partial
// only when y is given).
constexpr int kHeadWarps = 16;

template <int NC>
__device__ __forceinline__ void head_rows_fwd(const uint32_t *__restrict__ sWq, const uint4 *a0, const uint4 *a1,
                                              bool two, int GPL, int lane, float (&z0)[NC], float (&z1)[NC]) {
#pragma unroll
    for (int n = 0; n < NC; ++n) { z0[n] = 0.0f; z1[n] = 0.0f; }
    uint4 c0 = __ldg(a0 + lane), c1 = two ? __ldg(a1 + lane) : make_uint4(0, 0, 0, 0);
    for (int j = 0; j < GPL; ++j) {
        const int g = lane + 32 * j;
        uint4 n0 = make_uint4(0, 0, 0, 0), n1 = make_uint4(0, 0, 0, 0);
        if (j + 1 < GPL) {   // the next group's loads go out before this group's arithmetic
            n0 = __ldg(a0 + g + 32);
            if (two) n1 = __ldg(a1 + g + 32);
        }
        const uint32_t w0[4] = {c0.x, c0.y, c0.z, c0.w}, w1[4] = {c1.x, c1.y, c1.z, c1.w};
        const uint32_t *wg = sWq + g * (kHeadGroup / 2);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float x0 = __uint_as_float(e & 1 ? w0[e >> 1] & 0xFFFF0000u : w0[e >> 1] << 16);
            const float x1 = __uint_as_float(e & 1 ? w1[e >> 1] & 0xFFFF0000u : w1[e >> 1] << 16);
#pragma unroll
            for (int n = 0; n < NC; n += 2) {
                const uint32_t w2 = wg[(e * NC + n) >> 1];   // NC even: bf16 pairs (n, n + 1)
                const float wa = __uint_as_float(w2 << 16), wb = __uint_as_float(w2 & 0xFFFF0000u);
                z0[n] = fmaf(x0, wa, z0[n]);
                z0[n + 1] = fmaf(x0, wb, z0[n + 1]);
                z1[n] = fmaf(x1, wa, z1[n]);
                z1[n + 1] = fmaf(x1, wb, z1[n + 1]);
            }
        }
        c0 = n0;
        c1 = n1;
    }
#pragma unroll
    for (int n = 0; n < NC; ++n) {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            z0[n] += __shfl_xor_sync(0xffffffffu, z0[n], o);
            z1[n] += __shfl_xor_sync(0xffffffffu, z1[n], o);
        }
    }
}

template <int NC>
__global__ void __launch_bounds__(kHeadWarps * 32) head_direct_kernel(
    const bf16 *__restrict__ a, const bf16 *__restrict__ wq, const float *__restrict__ bias,
    const float *__restrict__ y, float *__restrict__ dz_out, bf16 *__restrict__ dA, float *__restrict__ logits,
    float *__restrict__ partial, int B, int F, float invB) {
    extern __shared__ uint32_t sWq[];   // F / 8 groups of 49 words
    __shared__ float sAcc[kHeadWarps][NC + 1];
    __shared__ double sLoss[kHeadWarps];
    griddep_launch();
    griddep_wait();
    const int G = F / 8;
    for (int i = threadIdx.x; i < G * (kHeadGroup / 2); i += blockDim.x)
        sWq[i] = reinterpret_cast<const uint32_t *>(wq)[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int GPL = G / 32;   // groups per lane
    float gB[NC];
#pragma unroll
    for (int n = 0; n < NC; ++n) gB[n] = 0.0f;
    double lsum = 0.0;
    for (int r0 = 2 * (blockIdx.x * kHeadWarps + warp); r0 < B; r0 += 2 * gridDim.x * kHeadWarps) {
        const bool two = r0 + 1 < B;
        float z[2][NC];
        head_rows_fwd<NC>(sWq, reinterpret_cast<const uint4 *>(a + (size_t)r0 * F),
                          reinterpret_cast<const uint4 *>(a + (size_t)(r0 + (two ? 1 : 0)) * F), two, GPL, lane,
                          z[0], z[1]);
        float dz[2][NC];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int r = r0 + q;
#pragma unroll
            for (int n = 0; n < NC; ++n) z[q][n] += bias[n];
            if (q == 1 && !two) {
#pragma unroll
                for (int n = 0; n < NC; ++n) dz[q][n] = 0.0f;
                continue;
            }
            if (logits && lane < NC) {
                float zl = z[q][0];
#pragma unroll
                for (int n = 1; n < NC; ++n) if (lane == n) zl = z[q][n];
                logits[(size_t)r * NC + lane] = zl;
            }
#pragma unroll
            for (int n = 0; n < NC; ++n) dz[q][n] = 0.0f;
            if (!y) continue;
            float mx = z[q][0];
#pragma unroll
            for (int n = 1; n < NC; ++n) mx = fmaxf(mx, z[q][n]);
            float se = 0.0f;
#pragma unroll
            for (int n = 0; n < NC; ++n) se += expf(z[q][n] - mx);
            const int t = (int)y[r];
            float pt = 0.0f;
#pragma unroll
            for (int n = 0; n < NC; ++n) if (n == t) pt = expf(z[q][n] - mx) / se;
            if (lane == 0) lsum += -(double)logf(pt);
            if (logits) continue;
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                dz[q][n] = (expf(z[q][n] - mx) / se - (n == t ? 1.0f : 0.0f)) * invB;
                gB[n] += dz[q][n];
            }
            if (lane < NC) {
                float dl = dz[q][0];
#pragma unroll
                for (int n = 1; n < NC; ++n) if (lane == n) dl = dz[q][n];
                dz_out[(size_t)r * NC + lane] = dl;
            }
        }
        if (logits || !y) continue;
        // dA = dz W^T for both rows: each weight word serves the two rows
        uint4 *d0 = reinterpret_cast<uint4 *>(dA + (size_t)r0 * F);
        uint4 *d1 = reinterpret_cast<uint4 *>(dA + (size_t)(r0 + 1) * F);
        for (int j = 0; j < GPL; ++j) {
            const int g = lane + 32 * j;
            const uint32_t *wg = sWq + g * (kHeadGroup / 2);
            float o0[8], o1[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                for (int n = 0; n < NC; n += 2) {
                    const uint32_t w2 = wg[(e * NC + n) >> 1];
                    const float wa = __uint_as_float(w2 << 16), wb = __uint_as_float(w2 & 0xFFFF0000u);
                    s0 = fmaf(dz[0][n], wa, s0);
                    s0 = fmaf(dz[0][n + 1], wb, s0);
                    s1 = fmaf(dz[1][n], wa, s1);
                    s1 = fmaf(dz[1][n + 1], wb, s1);
                }
                o0[e] = s0;
                o1[e] = s1;
            }
            uint4 p0, p1;
            __nv_bfloat162 *h0 = reinterpret_cast<__nv_bfloat162 *>(&p0), *h1 = reinterpret_cast<__nv_bfloat162 *>(&p1);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                h0[e] = __floats2bfloat162_rn(o0[2 * e], o0[2 * e + 1]);
                h1[e] = __floats2bfloat162_rn(o1[2 * e], o1[2 * e + 1]);
            }
            d0[g] = p0;
            if (two) d1[g] = p1;
        }
    }
    if (!partial) return;
    if (lane == 0) {
#pragma unroll
        for (int n = 0; n < NC; ++n) sAcc[warp][n] = gB[n];
        sLoss[warp] = lsum;
    }
    __syncthreads();
    if (threadIdx.x <= NC) {   // fixed warp order
        float sacc = 0.0f;
        double sl = 0.0;
        for (int wv = 0; wv < kHeadWarps; ++wv) {
            if (threadIdx.x < NC) sacc += sAcc[wv][threadIdx.x];
            else sl += sLoss[wv];
        }
        partial[(size_t)blockIdx.x * (NC + 1) + threadIdx.x] = threadIdx.x < NC ? sacc : (float)sl;
    }
}

// Weight gradient of the direct head: dW[k][n] = sum_b a[b][k] dz[b][n] over a
// batch slice, k in NHWC order.  Block = 512 inputs (thread: 2 consecutive
// inputs, one 4-byte load per row, 2 x NC sums) x a batch slice whose dz rows
// are staged in shared memory.  Partials [split][F][NC], summed in split order.
constexpr int kHeadWgRows = 256;   // rows of dz staged per pass

template <int NC>
__global__ void __launch_bounds__(256) head_direct_wgrad_kernel(const bf16 *__restrict__ a,
                                                                const float *__restrict__ dz,
                                                                float *__restrict__ partial, int B, int F,
                                                                int splits) {
    __shared__ float sdz[kHeadWgRows * NC];
    griddep_launch();
    griddep_wait();
    const int kchunks = F / 512;
    const int kc = blockIdx.x % kchunks, split = blockIdx.x / kchunks;
    const int k = kc * 512 + 2 * threadIdx.x;
    const int b0 = (int)((long long)B * split / splits), b1 = (int)((long long)B * (split + 1) / splits);
    float acc[2][NC];
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int n = 0; n < NC; ++n) acc[e][n] = 0.0f;
    for (int c0 = b0; c0 < b1; c0 += kHeadWgRows) {
        const int rows = min(kHeadWgRows, b1 - c0);
        __syncthreads();
        for (int i = threadIdx.x; i < rows * NC; i += blockDim.x) sdz[i] = dz[(size_t)c0 * NC + i];
        __syncthreads();
        const uint32_t *ar = reinterpret_cast<const uint32_t *>(a + (size_t)c0 * F + k);
        uint32_t nxt = __ldg(ar);
        for (int r = 0; r < rows; ++r) {
            const uint32_t cur = nxt;
            if (r + 1 < rows) nxt = __ldg(ar + (size_t)(r + 1) * (F / 2));
            const float x0 = __uint_as_float(cur << 16), x1 = __uint_as_float(cur & 0xFFFF0000u);
            const float *dr = sdz + r * NC;
#pragma unroll
            for (int n = 0; n < NC; ++n) {
                const float d = dr[n];
                acc[0][n] = fmaf(x0, d, acc[0][n]);
                acc[1][n] = fmaf(x1, d, acc[1][n]);
            }
        }
    }
    float *dst = partial + ((size_t)split * F + k) * NC;
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int n = 0; n < NC; ++n) dst[e * NC + n] = acc[e][n];
}

// Sums partial[s][i] over s in order and scatters into the gradient layout.
// map 0: dst[i];  1 conv (M=COUT rows, N = 9*CIN, n = tap*CIN + ci) -> dst[(co*CIN+ci)*9+tap]
//        2 conv (M = 9*CIN rows (tap*CIN+ci), N = COUT)  -> same dst layout
//        3 linear (M = F rows in NHWC order, N = OUT)    -> dst[nchw(m)*OUT + n]
//        4 head partial [HD*NC | NC | HD | 1 | padding] -> dW5, db5, db4, loss (four destinations)
//        5 first conv [COUT][10] -> dW1[co*9+t], db1[co]
//        6 fc1 forward split-K: relu(s + bias) -> bf16
//        7 only the last element, into *dst4 (a loss behind zero partials)
struct ReduceArgs {
    const float *partial;
    int splits;
    long long n;       // elements per partial
    int map, M, N, CIN, C, H, W;
    float *dst, *dst2, *dst3;
    const float *bias;             // map 6
    __nv_bfloat16 *out_bf16;       // map 6
    float *dst4;                   // map 4: the loss
};

__device__ void r_store(const ReduceArgs &r, long long i, float s);

// Block = 32 consecutive elements x 8 split lanes: lane l sums the splits
// l, l+8, l+16, ... in order (coalesced 128-byte rows), then lane sums are
// combined in lane order: a fixed order, so the result is deterministic.
__global__ void __launch_bounds__(256) reduce_partials_kernel(ReduceArgs r) {
    griddep_launch();
    griddep_wait();
    __shared__ float part[8][33];
    const int el = threadIdx.x & 31, sl = threadIdx.x >> 5;
    for (long long base = (long long)blockIdx.x * 32; base < r.n; base += (long long)gridDim.x * 32) {
        const long long i = base + el;
        float s = 0.0f;
        if (i < r.n)
            for (int k = sl; k < r.splits; k += 8) s += r.partial[(size_t)k * r.n + i];
        part[sl][el] = s;
        __syncthreads();
        if (sl == 0 && i < r.n) {
            s = part[0][el];
#pragma unroll
            for (int l = 1; l < 8; ++l) s += part[l][el];
            r_store(r, i, s);
        }
        __syncthreads();
    }
}

// Several independent split sums of one phase in one launch: blocks [start[j],
// start[j+1]) take job j.
constexpr int kMaxReduceJobs = 6;
struct ReduceJobs {
    ReduceArgs job[kMaxReduceJobs];
    int start[kMaxReduceJobs + 1];
    int vec[kMaxReduceJobs];   // reduce_multi4_kernel: 1 = 128 elements per block (16-byte loads), 0 = 32
    int count;
};

// Eight split lanes per block: warp w sums splits w, w + 8,
// w + 16, ... in order, then the eight warp sums of each element are added in
// warp order (a fixed order: deterministic).  A job whose length is a multiple
// of 4 (16-byte aligned splits) takes 128 elements per block, four consecutive
// per lane (one 16-byte load: a warp reads 512 contiguous bytes of a split,
// eight splits in flight while at least 64 remain, then four); any other job
// 32, one per lane.  The adds run in split order either way.
__global__ void __launch_bounds__(256, 4) reduce_multi4_kernel(const __grid_constant__ ReduceJobs J) {
    griddep_launch();
    griddep_wait();
    int j = 0;
    while (j + 1 < J.count && (int)blockIdx.x >= J.start[j + 1]) ++j;
    const ReduceArgs &r = J.job[j];
    const bool vec = J.vec[j] != 0;
    __shared__ float4 part[8][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long long bx = (int)blockIdx.x - J.start[j];
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (vec) {
        const long long n4 = r.n >> 2, q = bx * 32 + lane;
        if (q < n4) {
            const float4 *p = reinterpret_cast<const float4 *>(r.partial) + q;
            int k = w;
            for (; k + 56 < r.splits; k += 64) {   // eight loads in flight per lane
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = __ldcg(p + (size_t)(k + 8 * u) * n4);
#pragma unroll
                for (int u = 0; u < 8; ++u) { s.x += v[u].x; s.y += v[u].y; s.z += v[u].z; s.w += v[u].w; }
            }
            for (; k + 24 < r.splits; k += 32) {
                const float4 a = __ldcg(p + (size_t)k * n4), b = __ldcg(p + (size_t)(k + 8) * n4);
                const float4 c = __ldcg(p + (size_t)(k + 16) * n4), d = __ldcg(p + (size_t)(k + 24) * n4);
                s.x += a.x; s.y += a.y; s.z += a.z; s.w += a.w;
                s.x += b.x; s.y += b.y; s.z += b.z; s.w += b.w;
                s.x += c.x; s.y += c.y; s.z += c.z; s.w += c.w;
                s.x += d.x; s.y += d.y; s.z += d.z; s.w += d.w;
            }
            for (; k < r.splits; k += 8) {
                const float4 a = __ldcg(p + (size_t)k * n4);
                s.x += a.x; s.y += a.y; s.z += a.z; s.w += a.w;
            }
        }
    } else {
        const long long i = bx * 32 + lane;
        if (i < r.n) {
            const float *p = r.partial + i;
            int k = w;
            for (; k + 56 < r.splits; k += 64) {   // eight loads in flight per lane
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = __ldcg(p + (size_t)(k + 8 * u) * r.n);
#pragma unroll
                for (int u = 0; u < 8; ++u) s.x += v[u];
            }
            for (; k + 8 < r.splits; k += 16) {
                const float a = __ldcg(p + (size_t)k * r.n), b = __ldcg(p + (size_t)(k + 8) * r.n);
                s.x += a;
                s.x += b;
            }
            if (k < r.splits) s.x += __ldcg(p + (size_t)k * r.n);
        }
    }
    part[w][lane] = s;
    __syncthreads();
    if (w == 0) {
        float4 t = part[0][lane];
#pragma unroll
        for (int l = 1; l < 8; ++l) {
            const float4 u = part[l][lane];
            t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
        }
        if (vec) {
            const long long q = bx * 32 + lane;
            if (q < (r.n >> 2)) {
                r_store(r, 4 * q, t.x);
                r_store(r, 4 * q + 1, t.y);
                r_store(r, 4 * q + 2, t.z);
                r_store(r, 4 * q + 3, t.w);
            }
        } else if (bx * 32 + lane < r.n) {
            r_store(r, bx * 32 + lane, t.x);
        }
    }
}

// Few splits of a long vector (the Linear weight gradient): each thread owns
// 4 consecutive elements and adds the splits in order with 16-byte loads.
__global__ void __launch_bounds__(256) reduce_wide_kernel(ReduceArgs r) {
    griddep_launch();
    griddep_wait();
    const long long n4 = r.n >> 2;
    for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
         q += (long long)gridDim.x * blockDim.x) {
        float4 s = reinterpret_cast<const float4 *>(r.partial)[q];
        for (int k = 1; k < r.splits; ++k) {
            const float4 v = reinterpret_cast<const float4 *>(r.partial + (size_t)k * r.n)[q];
            s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
        }
        r_store(r, 4 * q, s.x);
        r_store(r, 4 * q + 1, s.y);
        r_store(r, 4 * q + 2, s.z);
        r_store(r, 4 * q + 3, s.w);
    }
}

__device__ void r_store(const ReduceArgs &r, long long i, float s) {
    {
        const int m = (int)(i / r.N), n = (int)(i % r.N);
        switch (r.map) {
        case 0: r.dst[i] = s; break;
        case 1: { const int tap = n / r.CIN, ci = n % r.CIN; r.dst[((size_t)m * r.CIN + ci) * 9 + tap] = s; break; }
        case 2: { const int tap = m / r.CIN, ci = m % r.CIN; r.dst[((size_t)n * r.CIN + ci) * 9 + tap] = s; break; }
        case 3: { const int c = m % r.C, hw = m / r.C; r.dst[((size_t)c * r.H * r.W + hw) * r.N + n] = s; break; }
        case 4: {
            const long long hdnc = (long long)r.M * r.N;
            if (i < hdnc) r.dst[i] = s;
            else if (i < hdnc + r.N) r.dst2[i - hdnc] = s;
            else if (i < hdnc + r.N + r.M) r.dst3[i - hdnc - r.N] = s;
            else if (i == hdnc + r.N + r.M) *r.dst4 = s;   // (the elements after it are padding)
            break;
        }
        case 5: { const int co = (int)(i / 10), t = (int)(i % 10); if (t < 9) r.dst[co * 9 + t] = s; else r.dst2[co] = s; break; }
        case 6: { const float x = s + r.bias[n]; r.out_bf16[i] = __float2bfloat16_rn(x > 0.0f ? x : 0.0f); break; }
        case 7: if (i == r.n - 1) *r.dst4 = s; break;   // the last element only (a loss)
        }
    }
}


}  // namespace

// ====================================================================== engine
using bf16 = __nv_bfloat16;

struct ConvLayer {   // a tensor-core conv stage (conv + ReLU + pool)
    int si;          // stage index
    int CIN, COUT, H, W, R, tpi;
    bf16 *wf = nullptr, *wd = nullptr;   // packed fwd / dgrad weights
    bf16 *out = nullptr;                 // pooled output [B, H/2, W/2, COUT]
    uint8_t *code = nullptr;
    bf16 *dP = nullptr;                  // gradient w.r.t. the pooled output
    bf16 *dC = nullptr;                  // gradient w.r.t. the conv output [B, H, W, COUT]
    ConvTcParams fwd{}, dgrad{};
    bool halo = false;                   // halo-tile kernels (R * (W + 2) <= 128)
    ConvHaloParams hfwd{}, hdgrad{};
    bool fused_bwd = false;              // input + weight gradient in one kernel (32 -> 64)
    ConvBwdFusedParams fbwd{};
    int fbwd_grid = 0;
    float *fbwd_partial = nullptr;
    bool fbwd_c1 = false;                // the first conv's weight gradient taken in the same kernel
    bool fbwd_up = false;                // dY built in the kernel from dP and the pool codes (no unpool)
    float *fbwd_bias_partial = nullptr;  // fbwd_up: [fbwd_grid * 4][COUT]
    bool up = false;                     // conv3 path: dgrad + weight gradient build dY from dP and codes
    int up_grid = 0;                     // up: CTAs of the input-gradient kernel
    float *up_bias_partial = nullptr;    // up: [up_grid * 4][COUT]
    bool wg_halo = false;                // halo-tile weight gradient
    WgradHaloParams whalo{};
    int whalo_grid = 0;
    float *whalo_partial = nullptr;
    WgradTcParams wg{};
    int wg_mode = 0, wg_grid = 0, wg_smem = 0;
    float *wg_partial = nullptr;
    float *bias_partial = nullptr;
    int unpool_grid = 0;
};

struct TcEngine {
    int B = 0;
    // first conv
    int c1_si = 0, C1 = 0, H0 = 0, W0 = 0, pad1 = 0, H1 = 0, W1 = 0;
    bool c1_pool = false;
    bf16 *a1 = nullptr;        // first conv output (pooled if c1_pool)
    uint8_t *code1 = nullptr;
    bf16 *dC1 = nullptr;       // gradient w.r.t. the first conv output [B, oH, oW, C1]
    bf16 *dP1 = nullptr;       // gradient w.r.t. its pooled output (c1_pool)
    float *c1_partial = nullptr;
    int c1_wgrad_grid = 0;
    bool c1_fused = false;     // first conv's weight gradient from the next conv's backward kernel
    float *c1_bias_partial = nullptr;
    int c1_unpool_grid = 0;
    std::vector<ConvLayer> convs;
    // flattened activation geometry (NHWC) feeding the first Linear
    int fC = 0, fH = 0, fW = 0, F = 0;
    // hidden Linear (tensor cores) and head
    bool has_hidden = false;
    int hid_si = 0, HD = 0, head_si = 0, NC = 0;
    bf16 *wP = nullptr;   // hidden Linear packed W [F][HD] (NHWC feature rows)
    bf16 *a_hid = nullptr;               // [B][HD]
    bf16 *dZ_hid = nullptr;              // [B][HD]
    bf16 *dflat = nullptr;               // gradient w.r.t. the flattened activation [B][F]
    GemmTcParams fc_fwd{}, fc_dgrad{};
    WgradTcParams fc_wg{};
    int fc_wg_grid = 0, fc_wg_smem = 0;
    float *fc_partial = nullptr;
    float *fc_fwd_partial = nullptr;   // [ksplit][B][HD] when the forward splits K
    float *head_partial = nullptr;
    int head_grid = 0;
    // direct head: the classifier straight after the last pool (no hidden Linear)
    bool direct_head = false;
    bf16 *wq = nullptr;                  // packed classifier weights (kHeadGroup groups)
    float *dz = nullptr;                 // [B][NC] logit gradients
    int hdw_splits = 0;
    float *hdw_partial = nullptr;        // [hdw_splits][F][NC]
    double *row_loss = nullptr;
    PackJobs pack{};
    int pack_grid = 0;
    std::vector<void *> allocs;
    // named intermediate tensors (zilla_net_inspect)
    struct View { std::string name; const void *p; size_t n; int kind; };   // kind 0 bf16, 1 u8, 2 f32
    std::vector<View> views;
};

namespace {

template <class T>
int dalloc(TcEngine &e, T **p, size_t count) {
    if (cudaMalloc((void **)p, (count ? count : 1) * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return fail(kBadHandle, "tc engine: cudaMalloc of %zu bytes failed", count * sizeof(T));
    }
    e.allocs.push_back((void *)*p);
    return kOk;
}

// ---------------------------------------------------------------- conv dispatch
template <int CIN, int COUT, int EPI, int NS, bool SB = false>
int launch_conv(const ConvTcParams &p) {
    using S = tc::ConvTcShape<CIN, COUT, NS, EPI == tc::kEpiPool, SB>;
    auto kern = tc::conv_tc_kernel<CIN, COUT, EPI, NS, SB>;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM) != cudaSuccess)
            return check_cuda("conv_tc smem attribute");
        attr = true;
    }
    // resident CTAs per SM: shared memory (227 KB) and TMEM (512 columns) bound it
    int per_sm = (227 * 1024) / S::SMEM;
    if (per_sm > (int)(512 / S::TMEM_COLS)) per_sm = 512 / S::TMEM_COLS;
    if (per_sm < 1) per_sm = 1;
    if (per_sm > 2) per_sm = 2;
    const int slots = sm_count() * per_sm;
    const int grid = p.num_tiles < slots ? p.num_tiles : slots;
    kern<<<grid, 192, S::SMEM, stream()>>>(p);
    ZB_LAUNCH_CHECK("conv_tc");
    return kOk;
}

bool conv_shape_supported(int cin, int cout) {
    return (cin == 16 && cout == 32) || (cin == 32 && cout == 64) || (cin == 64 && cout == 128);
}

template <int CIN, int COUT, int EPI, int NS, int KS, int OB = 2, bool UP = false>
int launch_halo(const ConvHaloParams &p0, int up_grid = 0) {
    using S = tc::ConvHaloShape<CIN, COUT, NS, KS, EPI == tc::kEpiPool>;
    auto kern = tc::conv_halo_kernel<CIN, COUT, EPI, NS, KS, OB, UP>;
    ConvHaloParams p = p0;
    p.region = UP ? S::region_up(p.HR) : S::region(p.HR);
    p.stage_bytes = UP ? S::stage_bytes_up(p.HR) : S::stage_bytes(p.HR);
    if (UP && (!p.dp || !p.up_code || !p.up_bias_partial || up_grid < 1))
        return fail(kBadArg, "conv_halo: unpool inputs not set up");
    p.out_tile_bytes = EPI == tc::kEpiDgrad ? S::out_tile_bytes(p.R, p.W) : 0;
    const int smem = S::smem(p.stage_bytes, OB * p.out_tile_bytes);
    if (smem > 227 * 1024) return fail(kBadArg, "conv_halo: %d bytes of shared memory needed", smem);
    static int attr = 0;
    if (attr < smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_cuda("conv_halo smem attribute");
        attr = smem;
    }
    // resident CTAs per SM: shared memory (228 KB, 1 KB reserved per CTA) and TMEM (512 columns)
    int per_sm = (228 * 1024) / (smem + 1024);
    if (per_sm > (int)(512 / S::TMEM_COLS)) per_sm = 512 / S::TMEM_COLS;
    if (per_sm < 1) per_sm = 1;
    if (per_sm > 2) per_sm = 2;
    const int slots = sm_count() * per_sm;
    const int grid = UP ? up_grid : (p.num_tiles < slots ? p.num_tiles : slots);
    launch_pdl(kern, dim3(grid), dim3(UP ? 448 : 320), smem, p);
    ZB_LAUNCH_CHECK("conv_halo");
    return kOk;
}

int run_conv_fwd(const ConvLayer &L) {
    if (L.halo) {
        if (L.CIN == 16 && L.COUT == 32) return launch_halo<16, 32, tc::kEpiPool, 4, 1>(L.hfwd);
        if (L.CIN == 32 && L.COUT == 64) return launch_halo<32, 64, tc::kEpiPool, 3, 1>(L.hfwd);
        if (L.CIN == 64 && L.COUT == 128) return launch_halo<64, 128, tc::kEpiPool, 2, 1>(L.hfwd);
    }
    if (L.CIN == 16) return fail(kBadArg, "tc engine: 16 -> 32 conv needs halo tiles (R * (W + 2) <= 128)");
    if (L.CIN == 32 && L.COUT == 64) return launch_conv<32, 64, tc::kEpiPool, 6>(L.fwd);
    if (L.CIN == 64 && L.COUT == 128) return launch_conv<64, 128, tc::kEpiPool, 6, true>(L.fwd);
    return fail(kBadArg, "tc engine: no forward conv kernel for %d->%d", L.CIN, L.COUT);
}

int run_conv_dgrad(const ConvLayer &L, const bf16 *dp) {
    // dgrad convolves dY (COUT channels) into CIN outputs
    if (L.up) {   // dY built in the kernel from the pooled gradient and the codes
        ConvHaloParams p = L.hdgrad;
        p.dp = dp;
        return launch_halo<128, 64, tc::kEpiDgrad, 3, 2, 1, true>(p, L.up_grid);
    }
    if (L.halo) {
        if (L.CIN == 16 && L.COUT == 32) return launch_halo<32, 16, tc::kEpiDgrad, 3, 1, 2>(L.hdgrad);
        if (L.CIN == 32 && L.COUT == 64) return launch_halo<64, 32, tc::kEpiDgrad, 2, 1, 2>(L.hdgrad);
        if (L.CIN == 64 && L.COUT == 128) return launch_halo<128, 64, tc::kEpiDgrad, 3, 2, 1>(L.hdgrad);
    }
    if (L.CIN == 16) return fail(kBadArg, "tc engine: 16 -> 32 conv needs halo tiles (R * (W + 2) <= 128)");
    if (L.CIN == 32 && L.COUT == 64) return launch_conv<64, 32, tc::kEpiDgrad, 4>(L.dgrad);
    if (L.CIN == 64 && L.COUT == 128) return launch_conv<128, 64, tc::kEpiDgrad, 4, true>(L.dgrad);
    return fail(kBadArg, "tc engine: no dgrad conv kernel for %d->%d", L.CIN, L.COUT);
}

template <int CIN, int COUT, int NGRP, int NS>
int launch_wgrad_halo(const WgradHaloParams &p0, int grid) {
    using S = tc::WgradHaloShape<CIN, COUT, NGRP, NS>;
    auto kern = tc::wgrad_halo_kernel<CIN, COUT, NGRP, NS>;
    WgradHaloParams p = p0;
    p.dy_region = S::dy_region(p.R, p.Wp);
    p.x_region = S::x_region(p.HR);
    p.stage_bytes = S::stage_bytes(p.R, p.Wp, p.HR);
    const int smem = S::smem(p.R, p.Wp, p.HR);
    if (smem > 227 * 1024) return fail(kBadArg, "wgrad_halo: %d bytes of shared memory needed", smem);
    static int attr = 0;
    if (attr < smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_cuda("wgrad_halo smem attribute");
        attr = smem;
    }
    kern<<<grid, 192, smem, stream()>>>(p);
    ZB_LAUNCH_CHECK("wgrad_halo");
    return kOk;
}

template <bool C1, bool UP>
int launch_conv_bwd_fused(const ConvLayer &L, const float *x0, const bf16 *dp) {
    using S = tc::ConvBwdFusedShape<32, 64, 2, C1, UP>;   // two stages: each holds X three times
    auto kern = tc::conv_bwd_fused_kernel<32, 64, 2, C1, UP>;
    ConvBwdFusedParams p = L.fbwd;
    p.region = S::region(p.R, p.Wp);
    p.dy_region = S::dy_region(p.R, p.Wp);
    p.x_off = S::x_off(p.R, p.Wp);
    p.stage_bytes = S::stage_bytes(p.R, p.Wp);
    p.dp = dp;
    if (UP && (!dp || !p.code || !p.bias_partial || p.R != 4 || p.H % 2 || p.W % 2 || 4 * (p.W / 2) * 8 > 512))
        return fail(kBadArg, "conv_bwd_fused: unpool inputs not set up");
    p.out_tile_bytes = S::out_tile_bytes(p.R, p.W);
    p.x9_bytes = S::x9_bytes(p.R, p.W);
    p.x0 = x0;
    if (C1 && (!x0 || !p.c1_partial || (p.R * p.W) % 16 != 0))
        return fail(kBadArg, "conv_bwd_fused: first-conv weight gradient not set up");
    const int smem = S::smem(p.R, p.Wp, p.W);
    if (smem > 227 * 1024) return fail(kBadArg, "conv_bwd_fused: %d bytes of shared memory needed", smem);
    static int attr = 0;
    if (attr < smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_cuda("conv_bwd_fused smem attribute");
        attr = smem;
    }
    launch_pdl(kern, dim3(L.fbwd_grid), dim3(S::THREADS), smem, p);
    ZB_LAUNCH_CHECK("conv_bwd_fused");
    return kOk;
}

int run_conv_bwd_fused(const ConvLayer &L, const float *x0, const bf16 *dp) {
    if (L.fbwd_c1)
        return L.fbwd_up ? launch_conv_bwd_fused<true, true>(L, x0, dp) : launch_conv_bwd_fused<true, false>(L, x0, nullptr);
    return L.fbwd_up ? launch_conv_bwd_fused<false, true>(L, nullptr, dp) : launch_conv_bwd_fused<false, false>(L, nullptr, nullptr);
}

int run_wgrad_halo(const ConvLayer &L) {
    if (L.CIN == 16 && L.COUT == 32) return launch_wgrad_halo<16, 32, 1, 6>(L.whalo, L.whalo_grid);
    if (L.CIN == 32 && L.COUT == 64) return launch_wgrad_halo<32, 64, 1, 6>(L.whalo, L.whalo_grid);
    if (L.CIN == 64 && L.COUT == 128) return launch_wgrad_halo<64, 128, 2, 4>(L.whalo, L.whalo_grid);
    return fail(kBadArg, "tc engine: no halo weight-gradient kernel for %d->%d", L.CIN, L.COUT);
}

template <int MODE, bool UP = false>
int launch_wgrad(const WgradTcParams &p, int grid, int smem) {
    auto kern = tc::wgrad_tc_kernel<MODE, UP>;
    static int attr = 0;
    if (attr < smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_cuda("wgrad_tc smem attribute");
        attr = smem;
    }
    if (UP && (!p.dp || !p.up_code)) return fail(kBadArg, "wgrad_tc: unpool inputs not set up");
    launch_pdl(kern, dim3(grid), dim3(UP ? 320 : 192), smem, p);
    ZB_LAUNCH_CHECK("wgrad_tc");
    return kOk;
}

// dp: the pooled gradient when the conv-co kernel builds dY itself (null: dY from the a map)
int run_wgrad(const WgradTcParams &p0, int mode, int grid, int smem, const bf16 *dp = nullptr) {
    if (mode == tc::kWgLinear) return launch_wgrad<tc::kWgLinear>(p0, grid, smem);
    if (mode == tc::kWgLinearN128) return launch_wgrad<tc::kWgLinearN128>(p0, grid, smem);
    if (mode == tc::kWgConvCo) {
        if (!dp) return launch_wgrad<tc::kWgConvCo>(p0, grid, smem);
        WgradTcParams p = p0;
        p.dp = dp;
        return launch_wgrad<tc::kWgConvCo, true>(p, grid, smem);
    }
    return launch_wgrad<tc::kWgConvTap>(p0, grid, smem);
}

template <int BN, int EPI, int NS, bool BMN = false>
int launch_gemm(const GemmTcParams &p) {
    using S = tc::GemmTcShape<BN, NS>;
    auto kern = tc::gemm_tc_kernel<BN, EPI, NS, BMN>;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM) != cudaSuccess)
            return check_cuda("gemm_tc smem attribute");
        attr = true;
    }
    const int tiles = p.m_tiles * p.n_tiles * p.ksplit;
    launch_pdl(kern, dim3(tiles < sm_count() ? tiles : sm_count()), dim3(192), S::SMEM, p);
    ZB_LAUNCH_CHECK("gemm_tc");
    return kOk;
}

// Deep reductions (many splits, short vectors) of one phase in one launch.
int reduce_multi(const ReduceArgs *jobs, int count) {
    if (count < 1 || count > kMaxReduceJobs) return fail(kBadArg, "reduce_multi: %d jobs", count);
    ReduceJobs J{};
    J.count = count;
    // the deepest job first: its blocks (the longest) start in the first wave
    int order[kMaxReduceJobs];
    for (int j = 0; j < count; ++j) order[j] = j;
    std::stable_sort(order, order + count, [&](int a, int b) { return jobs[a].splits > jobs[b].splits; });
    int total = 0;
    for (int j = 0; j < count; ++j) {
        J.job[j] = jobs[order[j]];
        J.start[j] = total;
        // 16-byte loads: a partial vector a multiple of 4 long (16-byte aligned splits)
        J.vec[j] = J.job[j].n % 4 == 0 && (reinterpret_cast<uintptr_t>(J.job[j].partial) & 15) == 0;
        total += (int)(J.vec[j] ? (J.job[j].n / 4 + 31) / 32 : (J.job[j].n + 31) / 32);
    }
    J.start[count] = total;
    launch_pdl(reduce_multi4_kernel, dim3(total), dim3(256), 0, J);
    ZB_LAUNCH_CHECK("reduce_multi");
    return kOk;
}

int reduce(const ReduceArgs &r) {
    if (r.splits >= 32 && r.n <= 131072) return reduce_multi(&r, 1);   // many splits of a short vector
    if (r.n % 4 == 0 && r.n >= 65536 && r.splits <= 16) {
        launch_pdl(reduce_wide_kernel, dim3(grid_for(r.n / 4, 256, 8)), dim3(256), 0, r);
    } else {
        launch_pdl(reduce_partials_kernel, dim3(grid_for(r.n, 32, 8)), dim3(256), 0, r);   // 32 elements per block
    }
    ZB_LAUNCH_CHECK("reduce_partials");
    return kOk;
}

// ---------------------------------------------------------------- building
int nhwc_map(CUtensorMap *m, const bf16 *base, int C, int W, int H, int B, int box_c, int box_w, int box_h) {
    const uint64_t dims[4] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)B};
    const uint64_t strides[3] = {(uint64_t)C * 2, (uint64_t)C * W * 2, (uint64_t)C * W * H * 2};
    const uint32_t box[4] = {(uint32_t)box_c, (uint32_t)box_w, (uint32_t)box_h, 1};
    const int rowb = box_c * 2;
    return tc::make_tmap_bf16(m, base, 4, dims, strides, box,
                              rowb == 128 ? tc::kSw128 : rowb == 64 ? tc::kSw64 : tc::kSw32);
}

// 4D NHWC map whose box is one halo tile of 8 channels: {8, W + 2, R + 2, 1},
// no swizzle (the halo kernel's K-major interleaved operand layout).
int halo_map(CUtensorMap *m, const bf16 *base, int C, int W, int H, int B, int R) {
    const uint64_t dims[4] = {(uint64_t)C, (uint64_t)W, (uint64_t)H, (uint64_t)B};
    const uint64_t strides[3] = {(uint64_t)C * 2, (uint64_t)C * W * 2, (uint64_t)C * W * H * 2};
    const uint32_t box[4] = {8, (uint32_t)(W + 2), (uint32_t)(R + 2), 1};
    return tc::make_tmap_bf16(m, base, 4, dims, strides, box, tc::kSwNone);
}

void halo_params(ConvHaloParams &h, const ConvTcParams &t, int R, int W) {
    h.w_map = t.w_map;
    h.B = t.B; h.H = t.H; h.W = t.W; h.R = R; h.Wp = W + 2; h.HR = (R + 2) * (W + 2);
    h.tiles_per_img = t.tiles_per_img; h.num_tiles = t.num_tiles;
    h.bias = t.bias; h.out = t.out; h.code = t.code; h.mask = t.mask; h.err = t.err;
}

int tc_build(Net &n, TcEngine &e) {
    const int B = n.B;
    e.B = B;
    auto &st = n.st;
    size_t i = 0;
    // first conv: 1 input channel, CUDA cores
    if (st.empty() || st[0].kind != kConv || st[0].C != 1 || !st[0].relu)
        return fail(kBadArg, "tc engine: the first layer must be Conv2D(1 -> C) + ReLU");
    e.c1_si = 0;
    e.C1 = st[0].oC; e.H0 = st[0].H; e.W0 = st[0].W; e.pad1 = st[0].pad;
    e.H1 = st[0].oH; e.W1 = st[0].oW;
    if (e.C1 != 16 && e.C1 != 32) return fail(kBadArg, "tc engine: first conv must have 16 or 32 outputs");
    i = 1;
    e.c1_pool = i < st.size() && st[i].kind == kPool;
    {   // the unpooled forward stages the padded image in registers; the weight gradient in shared memory
        const int padded = (e.H0 + 2 * e.pad1) * (e.W0 + 2 * e.pad1);
        if ((!e.c1_pool && padded > kStageRegs * 256) || padded * (int)sizeof(float) > 48 * 1024)
            return fail(kBadArg, "tc engine: first-conv image too large (padded %d x %d)", e.H0 + 2 * e.pad1,
                        e.W0 + 2 * e.pad1);
    }
    int C = e.C1, H = e.H1, W = e.W1;
    if (e.c1_pool) { H = st[i].oH; W = st[i].oW; ++i; }
    int rc;
    if ((rc = dalloc(e, &e.a1, (size_t)B * H * W * C))) return rc;
    // the full-size first-conv gradient (a pooled first conv's weight gradient reads dP1 and the codes)
    if ((rc = dalloc(e, &e.dC1, e.c1_pool ? (size_t)1 : (size_t)B * e.H1 * e.W1 * C))) return rc;
    if (e.c1_pool) {
        if ((rc = dalloc(e, &e.code1, (size_t)B * H * W * C))) return rc;
        if ((rc = dalloc(e, &e.dP1, (size_t)B * H * W * C))) return rc;
    }
    // tensor-core conv stages
    const bf16 *prev = e.a1;
    while (i < st.size() && st[i].kind == kConv) {
        Stage &s = st[i];
        if (!s.relu || s.pad != 1 || i + 1 >= st.size() || st[i + 1].kind != kPool)
            return fail(kBadArg, "tc engine: inner convs must be Conv2D(pad 1) + ReLU + MaxPool");
        if (!conv_shape_supported(s.C, s.oC)) return fail(kBadArg, "tc engine: conv %d->%d not supported", s.C, s.oC);
        ConvLayer L;
        L.si = (int)i; L.CIN = s.C; L.COUT = s.oC; L.H = s.H; L.W = s.W;
        if (L.W > 64) return fail(kBadArg, "tc engine: image width %d > 64", L.W);
        L.R = (128 / L.W) & ~1;
        L.tpi = (L.H + L.R - 1) / L.R;
        const int Ho = L.H / 2, Wo = L.W / 2;
        if ((rc = dalloc(e, &L.wf, (size_t)9 * L.CIN * L.COUT))) return rc;
        if ((rc = dalloc(e, &L.wd, (size_t)9 * L.CIN * L.COUT))) return rc;
        if ((rc = dalloc(e, &L.out, (size_t)B * Ho * Wo * L.COUT))) return rc;
        if ((rc = dalloc(e, &L.code, (size_t)B * Ho * Wo * L.COUT))) return rc;
        if ((rc = dalloc(e, &L.dP, (size_t)B * Ho * Wo * L.COUT))) return rc;
        if ((rc = dalloc(e, &L.dC, (size_t)B * L.H * L.W * L.COUT))) return rc;
        // forward: input = prev activations (CIN channels)
        ConvTcParams &f = L.fwd;
        const int chunk_f = L.CIN > 64 ? 64 : L.CIN;
        if ((rc = nhwc_map(&f.in_map, prev, L.CIN, L.W, L.H, B, chunk_f, L.W, L.R))) return rc;
        {
            const uint64_t dims[3] = {(uint64_t)L.CIN, (uint64_t)L.COUT, 9};
            const uint64_t strides[2] = {(uint64_t)L.CIN * 2, (uint64_t)L.CIN * L.COUT * 2};
            const uint32_t box[3] = {(uint32_t)chunk_f, (uint32_t)L.COUT, 1};
            if ((rc = tc::make_tmap_bf16(&f.w_map, L.wf, 3, dims, strides, box,
                                         chunk_f * 2 == 128 ? tc::kSw128 : chunk_f * 2 == 64 ? tc::kSw64 : tc::kSw32)))
                return rc;
        }
        f.B = B; f.H = L.H; f.W = L.W; f.R = L.R; f.tiles_per_img = L.tpi; f.num_tiles = B * L.tpi;
        f.bias = n.params + s.poff + s.pn_w;
        f.out = L.out; f.code = L.code; f.mask = nullptr; f.err = device_error_word();
        // dgrad: input = dC (COUT channels), output CIN channels, masked by prev > 0
        ConvTcParams &d = L.dgrad;
        const int chunk_d = L.COUT > 64 ? 64 : L.COUT;
        if ((rc = nhwc_map(&d.in_map, L.dC, L.COUT, L.W, L.H, B, chunk_d, L.W, L.R))) return rc;
        {
            const uint64_t dims[3] = {(uint64_t)L.COUT, (uint64_t)L.CIN, 9};
            const uint64_t strides[2] = {(uint64_t)L.COUT * 2, (uint64_t)L.CIN * L.COUT * 2};
            const uint32_t box[3] = {(uint32_t)chunk_d, (uint32_t)L.CIN, 1};
            if ((rc = tc::make_tmap_bf16(&d.w_map, L.wd, 3, dims, strides, box,
                                         chunk_d * 2 == 128 ? tc::kSw128 : chunk_d * 2 == 64 ? tc::kSw64 : tc::kSw32)))
                return rc;
        }
        d.B = B; d.H = L.H; d.W = L.W; d.R = L.R; d.tiles_per_img = L.tpi; d.num_tiles = B * L.tpi;
        d.bias = nullptr; d.code = nullptr; d.err = device_error_word();
        // output of dgrad: gradient w.r.t. the previous activation
        const bool prev_is_first = L.si == (e.c1_pool ? 2 : 1);
        if (prev_is_first) {
            d.out = e.c1_pool ? e.dP1 : e.dC1;
            d.mask = e.c1_pool ? nullptr : e.a1;   // ReLU of conv1 (pooled: handled by unpool codes)
        } else {
            d.out = e.convs.back().dP;
            d.mask = nullptr;                      // handled by that layer's unpool codes
        }
        // halo-tile variants of the forward and input-gradient convolutions
        L.halo = L.R >= 2 && L.R * (L.W + 2) <= 128 && L.W + 2 <= 256 && L.R + 2 <= 256;
        if (L.halo) {
            halo_params(L.hfwd, f, L.R, L.W);
            halo_params(L.hdgrad, d, L.R, L.W);
            if ((rc = halo_map(&L.hfwd.in_map, prev, L.CIN, L.W, L.H, B, L.R))) return rc;
            if ((rc = halo_map(&L.hdgrad.in_map, L.dC, L.COUT, L.W, L.H, B, L.R))) return rc;
            // input-gradient output [B, H, W, CIN] written by TMA stores of R-row tiles
            const uint64_t od[4] = {(uint64_t)L.CIN, (uint64_t)L.W, (uint64_t)L.H, (uint64_t)B};
            const uint64_t os[3] = {(uint64_t)L.CIN * 2, (uint64_t)L.CIN * L.W * 2, (uint64_t)L.CIN * L.W * L.H * 2};
            const uint32_t ob[4] = {(uint32_t)L.CIN, (uint32_t)L.W, (uint32_t)L.R, 1};
            const int rb = L.CIN * 2;
            if (rb != 32 && rb != 64 && rb != 128) return fail(kBadArg, "tc engine: input-gradient row of %d bytes", rb);
            if ((rc = tc::make_tmap_bf16(&L.hdgrad.out_map, L.hdgrad.out, 4, od, os, ob,
                                         rb == 128 ? tc::kSw128 : rb == 64 ? tc::kSw64 : tc::kSw32)))
                return rc;

        }
        // halo-tile weight gradient: D[co][tap*CIN + ci], column groups x image slices
        // (only for 32 -> 64: at 64 -> 128 the per-tap kernel's single N = 192 MMA per K step
        // reads dY from shared memory once, where the halo kernel reads it once per tap)
        // whole backward of a 32 -> 64 conv on a ReLU output in one kernel: tiles of 4 rows
        // with a 32-pixel halo row (4 x 32 = 128 K rows), the input's ReLU mask from its tile
        L.fused_bwd = L.halo && L.CIN == 32 && L.COUT == 64 && L.W + 2 <= 32 && d.mask == prev;
        if (L.fused_bwd) {
            ConvBwdFusedParams &f = L.fbwd;
            f.B = B; f.H = L.H; f.W = L.W; f.Wp = 32; f.R = 128 / f.Wp;
            f.tiles_per_img = (L.H + f.R - 1) / f.R;
            f.num_tiles = B * f.tiles_per_img;
            f.err = device_error_word();
            const uint32_t hb[4] = {8, (uint32_t)f.Wp, (uint32_t)(f.R + 2), 1};
            const uint64_t dd[4] = {(uint64_t)L.COUT, (uint64_t)L.W, (uint64_t)L.H, (uint64_t)B};
            const uint64_t ds[3] = {(uint64_t)L.COUT * 2, (uint64_t)L.COUT * L.W * 2, (uint64_t)L.COUT * L.W * L.H * 2};
            if ((rc = tc::make_tmap_bf16(&f.dy_map, L.dC, 4, dd, ds, hb, tc::kSwNone))) return rc;
            const uint64_t xd[4] = {(uint64_t)L.CIN, (uint64_t)L.W, (uint64_t)L.H, (uint64_t)B};
            const uint64_t xs[3] = {(uint64_t)L.CIN * 2, (uint64_t)L.CIN * L.W * 2, (uint64_t)L.CIN * L.W * L.H * 2};
            if ((rc = tc::make_tmap_bf16(&f.x_map, prev, 4, xd, xs, hb, tc::kSwNone))) return rc;
            f.w_map = d.w_map;   // {COUT, CIN, 9}, box {64, CIN, 1}, 128-byte swizzle
            const uint32_t ob[4] = {(uint32_t)L.CIN, (uint32_t)L.W, (uint32_t)f.R, 1};
            if ((rc = tc::make_tmap_bf16(&f.out_map, d.out, 4, xd, xs, ob, tc::kSw64))) return rc;
            L.fbwd_grid = f.num_tiles < sm_count() ? f.num_tiles : sm_count();
            if ((rc = dalloc(e, &L.fbwd_partial, (size_t)L.fbwd_grid * L.COUT * 9 * L.CIN))) return rc;
            f.partial = L.fbwd_partial;
            // the masked input gradient is the first conv's output gradient (3x3, pad 1, one
            // input channel, same size): its weight gradient is taken from the staged tile
            L.fbwd_c1 = !e.c1_pool && e.C1 == L.CIN && e.pad1 == 1 && e.H1 == e.H0 && e.W1 == e.W0 &&
                        (f.R * f.W) % 16 == 0;
            e.c1_fused = L.fbwd_c1;
            // dY = max-unpool of the pooled gradient: built from dP and the codes inside the
            // kernel (even H and W, even tile rows; 4 pooled rows x W/2 x 8 octets <= 512 items)
            L.fbwd_up = L.H % 2 == 0 && L.W % 2 == 0 && f.R % 2 == 0 && f.R == 4 && 4 * (L.W / 2) * 8 <= 512;
            if (L.fbwd_up) {
                if ((rc = dalloc(e, &L.fbwd_bias_partial, (size_t)L.fbwd_grid * 4 * L.COUT))) return rc;
                f.code = L.code;
                f.bias_partial = L.fbwd_bias_partial;
            }
        }
        L.wg_halo = !L.fused_bwd && L.halo && ((L.CIN == 32 && L.COUT == 64) || (L.CIN == 16 && L.COUT == 32));
        if (L.wg_halo) {
            WgradHaloParams &w = L.whalo;
            const int ngrp = L.COUT == 128 ? 2 : 1;
            w.B = B; w.H = L.H; w.W = L.W; w.R = L.R; w.Wp = L.W + 2; w.HR = (L.R + 2) * (L.W + 2);
            w.tiles_per_img = L.tpi;
            w.splits = sm_count() / ngrp;
            if (w.splits > B) w.splits = B;
            if (w.splits < 1) w.splits = 1;
            w.err = device_error_word();
            L.whalo_grid = w.splits * ngrp;
            const uint64_t dd[4] = {(uint64_t)L.COUT, (uint64_t)L.W, (uint64_t)L.H, (uint64_t)B};
            const uint64_t ds[3] = {(uint64_t)L.COUT * 2, (uint64_t)L.COUT * L.W * 2, (uint64_t)L.COUT * L.W * L.H * 2};
            const uint32_t db[4] = {8, (uint32_t)(L.W + 2), (uint32_t)L.R, 1};
            if ((rc = tc::make_tmap_bf16(&w.dy_map, L.dC, 4, dd, ds, db, tc::kSwNone))) return rc;
            if ((rc = halo_map(&w.x_map, prev, L.CIN, L.W, L.H, B, L.R))) return rc;
            if ((rc = dalloc(e, &L.whalo_partial, (size_t)w.splits * L.COUT * 9 * L.CIN))) return rc;
            w.partial = L.whalo_partial;
        }
        // weight gradient
        WgradTcParams &g = L.wg;
        g.K_total = B; g.H = L.H; g.W = L.W; g.R = L.R; g.tiles_per_img = L.tpi;
        g.kstage_rows = L.R * L.W; g.err = device_error_word();
        if (L.COUT == 128 && L.CIN == 64) {
            L.wg_mode = tc::kWgConvCo;
            if ((rc = nhwc_map(&g.a_map, L.dC, L.COUT, L.W, L.H, B, 64, L.W, L.R))) return rc;
            if ((rc = nhwc_map(&g.b_map, prev, L.CIN, L.W, L.H, B, 64, L.W, L.R))) return rc;
            g.m_tiles = 3; g.M = L.COUT; g.N = 9 * L.CIN;
            g.splits = (sm_count() / 3) > 0 ? sm_count() / 3 : 1;
            L.wg_smem = tc::WgradTcShape<tc::kWgConvCo>::smem(g.kstage_rows);
        } else if (L.CIN == 16 && L.wg_halo) {
            L.wg_mode = -1;   // the halo weight gradient above; no per-tap fallback for 16 channels
            g.m_tiles = 1; g.M = L.COUT; g.N = 9 * L.CIN; g.splits = 1;
        } else if (L.CIN == 32 && L.COUT == 64) {
            L.wg_mode = tc::kWgConvTap;
            if ((rc = nhwc_map(&g.a_map, prev, L.CIN, L.W, L.H, B, 32, L.W, L.R))) return rc;
            if ((rc = nhwc_map(&g.b_map, L.dC, L.COUT, L.W, L.H, B, 64, L.W, L.R))) return rc;
            g.m_tiles = 1; g.M = 9 * L.CIN; g.N = L.COUT;
            g.splits = sm_count();
            L.wg_smem = tc::WgradTcShape<tc::kWgConvTap>::smem(g.kstage_rows);
        } else {
            return fail(kBadArg, "tc engine: no weight-gradient kernel for %d->%d", L.CIN, L.COUT);
        }
        if (g.splits > B) g.splits = B;
        g.mode = L.wg_mode;
        L.wg_grid = g.m_tiles * g.splits;
        // 64 -> 128 on halo tiles: both backward kernels build dY = unpool(dP, codes) themselves
        // (even H, W and R; the builders' items fit 4 rounds of 128 threads)
        L.up = L.halo && L.wg_mode == tc::kWgConvCo && L.H % 2 == 0 && L.W % 2 == 0 && L.R % 2 == 0 &&
               L.R * L.W <= 128 && ((L.R / 2) + 2) * (L.W / 2) * 8 <= 512 && (L.R / 2) * (L.W / 2) * 16 <= 512;
        if (L.up) {
            L.up_grid = L.hdgrad.num_tiles < sm_count() ? L.hdgrad.num_tiles : sm_count();
            if ((rc = dalloc(e, &L.up_bias_partial, (size_t)L.up_grid * 4 * L.COUT))) return rc;
            L.hdgrad.up_code = L.code;
            L.hdgrad.up_bias_partial = L.up_bias_partial;
            g.up_code = L.code;
        }
        if ((rc = dalloc(e, &L.wg_partial, (size_t)g.splits * g.M * g.N))) return rc;
        L.wg.partial = L.wg_partial;
        L.unpool_grid = sm_count() * 4;
        if ((rc = dalloc(e, &L.bias_partial, (size_t)L.unpool_grid * L.COUT))) return rc;
        e.convs.push_back(L);
        prev = L.out;
        C = L.COUT; H = Ho; W = Wo;
        i += 2;
    }
    e.fC = C; e.fH = H; e.fW = W; e.F = C * H * W;
    // Linear layers
    if (i < st.size() && st[i].kind == kLinear && st[i].relu) {
        Stage &s = st[i];
        e.has_hidden = true;
        e.hid_si = (int)i;
        e.HD = s.oC;
        if (e.F % 64 || e.HD % 64 || e.HD > 256)
            return fail(kBadArg, "tc engine: hidden Linear %d->%d not supported", e.F, e.HD);
        if ((rc = dalloc(e, &e.wP, (size_t)e.F * e.HD))) return rc;
        if ((rc = dalloc(e, &e.a_hid, (size_t)B * e.HD))) return rc;
        if ((rc = dalloc(e, &e.dZ_hid, (size_t)B * e.HD))) return rc;
        if ((rc = dalloc(e, &e.dflat, (size_t)B * e.F))) return rc;
        // forward: A = flattened activation [B][F], B = W [F][HD] (MN-major: 64 x 64 boxes)
        GemmTcParams &g = e.fc_fwd;
        {
            const uint64_t da[2] = {(uint64_t)e.F, (uint64_t)B}, sa[1] = {(uint64_t)e.F * 2};
            const uint32_t ba[2] = {64, 128};
            if ((rc = tc::make_tmap_bf16(&g.a_map, prev, 2, da, sa, ba, tc::kSw128))) return rc;
            const uint64_t db[2] = {(uint64_t)e.HD, (uint64_t)e.F}, sb[1] = {(uint64_t)e.HD * 2};
            const uint32_t bb[2] = {64, 64};
            if ((rc = tc::make_tmap_bf16(&g.b_map, e.wP, 2, db, sb, bb, tc::kSw128))) return rc;
        }
        // 128-wide N tiles; when the batch gives fewer tiles than SMs, split K
        // so that the tiles fill the SMs (fp32 partials, summed in split order)
        g.M = B; g.N = e.HD; g.K = e.F; g.m_tiles = (B + 127) / 128; g.n_tiles = e.HD / 128;
        {
            const int ksteps = e.F / 64, mn = g.m_tiles * g.n_tiles;
            int ks = sm_count() / mn;
            if (ks < 1) ks = 1;
            if (ks > ksteps) ks = ksteps;
            g.kper = (ksteps + ks - 1) / ks;
            g.ksplit = (ksteps + g.kper - 1) / g.kper;   // every split has at least one k step
        }
        g.bias = n.params + s.poff + s.pn_w; g.out = e.a_hid; g.err = device_error_word();
        if (g.ksplit > 1) {
            if ((rc = dalloc(e, &e.fc_fwd_partial, (size_t)g.ksplit * B * e.HD))) return rc;
            g.partial = e.fc_fwd_partial;
        }
        // input gradient: A = dZ [B][HD], B = W [F][HD] -> dflat [B][F], N tile 224/256/128
        GemmTcParams &dg = e.fc_dgrad;
        int bn = 0;
        for (int cand : {256, 224, 192, 160, 128, 96, 64})
            if (e.F % cand == 0) { bn = cand; break; }
        if (bn != 224 && bn != 256 && bn != 128) return fail(kBadArg, "tc engine: Linear input size %d", e.F);
        {
            const uint64_t da[2] = {(uint64_t)e.HD, (uint64_t)B}, sa[1] = {(uint64_t)e.HD * 2};
            const uint32_t ba[2] = {64, 128};
            if ((rc = tc::make_tmap_bf16(&dg.a_map, e.dZ_hid, 2, da, sa, ba, tc::kSw128))) return rc;
            const uint64_t db[2] = {(uint64_t)e.HD, (uint64_t)e.F}, sb[1] = {(uint64_t)e.HD * 2};
            const uint32_t bb[2] = {64, (uint32_t)bn};
            if ((rc = tc::make_tmap_bf16(&dg.b_map, e.wP, 2, db, sb, bb, tc::kSw128))) return rc;
        }
        dg.M = B; dg.N = e.F; dg.K = e.HD; dg.m_tiles = (B + 127) / 128; dg.n_tiles = e.F / bn;
        dg.ksplit = 1; dg.kper = e.HD / 64;
        dg.bias = nullptr; dg.out = e.dflat; dg.err = device_error_word();
        {   // the epilogue's TMA store: 128 x 32 chunks of dflat [B][F], 64-byte swizzle
            const uint64_t dd[2] = {(uint64_t)e.F, (uint64_t)B}, sd[1] = {(uint64_t)e.F * 2};
            const uint32_t bd[2] = {32, 128};
            if ((rc = tc::make_tmap_bf16(&dg.out_map, e.dflat, 2, dd, sd, bd, tc::kSw64))) return rc;
        }
        // weight gradient: A = flattened activation (MN-major), B = dZ
        WgradTcParams &w = e.fc_wg;
        {
            const uint64_t da[2] = {(uint64_t)e.F, (uint64_t)B}, sa[1] = {(uint64_t)e.F * 2};
            const uint32_t ba[2] = {64, 64};
            if ((rc = tc::make_tmap_bf16(&w.a_map, prev, 2, da, sa, ba, tc::kSw128))) return rc;
            const uint64_t db[2] = {(uint64_t)e.HD, (uint64_t)B}, sb[1] = {(uint64_t)e.HD * 2};
            const uint32_t bb[2] = {64, 64};
            if ((rc = tc::make_tmap_bf16(&w.b_map, e.dZ_hid, 2, db, sb, bb, tc::kSw128))) return rc;
        }
        if (e.HD != 256) return fail(kBadArg, "tc engine: hidden Linear width must be 256");
        w.mode = tc::kWgLinear; w.K_total = B; w.m_tiles = e.F / 128; w.M = e.F; w.N = e.HD;
        if (e.F % 128) return fail(kBadArg, "tc engine: Linear input %d not a multiple of 128", e.F);
        // one wave of one CTA per SM: two N halves per M tile when they fit, then K splits;
        // a single split writes the gradient itself (no partials, no reduction)
        w.n_tiles = w.m_tiles * 2 <= sm_count() ? 2 : 1;
        w.splits = sm_count() / (w.m_tiles * w.n_tiles);
        if (w.splits < 1) w.splits = 1;
        if (w.splits > (B + 63) / 64) w.splits = (B + 63) / 64;
        w.kstage_rows = 64; w.err = device_error_word();
        w.oC = e.fC; w.oHW = e.fH * e.fW; w.out = nullptr;
        e.fc_wg_grid = w.m_tiles * w.n_tiles * w.splits;
        if (w.n_tiles == 2) w.mode = tc::kWgLinearN128;
        e.fc_wg_smem = w.n_tiles == 2 ? tc::WgradTcShape<tc::kWgLinearN128>::smem(64)
                                      : tc::WgradTcShape<tc::kWgLinear>::smem(64);
        if (w.splits > 1) {
            if ((rc = dalloc(e, &e.fc_partial, (size_t)w.splits * e.F * e.HD))) return rc;
        }
        w.partial = e.fc_partial;
        ++i;
    }
    if (i + 1 != st.size() || st[i].kind != kLinear || st[i].relu)
        return fail(kBadArg, "tc engine: the network must end with Linear(-> classes)");
    e.head_si = (int)i;
    e.NC = st[i].oC;
    if (!e.has_hidden) {
        // classifier on the flattened last pooled activation: packed bf16 weights in shared
        // memory, logit gradients to global memory for the weight-gradient kernel
        e.direct_head = true;
        if (e.NC != 12 || e.F % 512 || (size_t)e.F / 8 * kHeadGroup * 2 > 200 * 1024)
            return fail(kBadArg, "tc engine: classifier %d->%d after the last pool not supported", e.F, e.NC);
        if ((rc = dalloc(e, &e.dflat, (size_t)B * e.F))) return rc;
        if ((rc = dalloc(e, &e.wq, (size_t)e.F / 8 * kHeadGroup))) return rc;
        if ((rc = dalloc(e, &e.dz, (size_t)B * e.NC))) return rc;
        e.head_grid = (B + 2 * kHeadWarps - 1) / (2 * kHeadWarps);   // two rows per warp
        if (e.head_grid > sm_count()) e.head_grid = sm_count();
        if ((rc = dalloc(e, &e.head_partial, (size_t)e.head_grid * (e.NC + 1)))) return rc;
        // weight gradient: 512-input chunks x batch slices, about two blocks per SM
        const int kchunks = e.F / 512;
        e.hdw_splits = (sm_count() * 2 + kchunks - 1) / kchunks;
        if (e.hdw_splits > B) e.hdw_splits = B;
        if (e.hdw_splits < 1) e.hdw_splits = 1;
        if ((rc = dalloc(e, &e.hdw_partial, (size_t)e.hdw_splits * e.F * e.NC))) return rc;
    } else if (e.HD != 256 || e.NC != 10) {
        return fail(kBadArg, "tc engine: head %d->%d not supported", e.HD, e.NC);
    }
    // a row per warp up to two blocks per SM (small batches: the kernel is
    // latency-bound, so more SMs), then more rows per warp (the block set-up,
    // W staging and partial write, is the fixed cost; fewer partials to sum)
    if (!e.direct_head) {
        e.head_grid = (B + 7) / 8;
        if (e.head_grid > sm_count() * 2) e.head_grid = sm_count() * 2;
        if ((rc = dalloc(e, &e.head_partial, (size_t)e.head_grid * head_pstride(e.HD, e.NC)))) return rc;
    }
    if ((rc = dalloc(e, &e.row_loss, (size_t)B))) return rc;
    e.c1_wgrad_grid = sm_count() * 2;   // the resident blocks (two per SM): each walks whole images
    if (e.c1_wgrad_grid > B) e.c1_wgrad_grid = B;
    if (e.c1_fused) {   // two partials (x_hi and x_lo products) per fused-kernel CTA
        e.c1_wgrad_grid = 2 * e.convs.front().fbwd_grid;
        e.convs.front().fbwd.c1_partial = nullptr;
    }
    if ((rc = dalloc(e, &e.c1_partial, (size_t)e.c1_wgrad_grid * e.C1 * 10))) return rc;
    if (e.c1_fused) e.convs.front().fbwd.c1_partial = e.c1_partial;
    // diagnostics
    e.views.push_back({"conv1.out", e.a1, (size_t)B * (e.c1_pool ? (e.H1 / 2) * (e.W1 / 2) : e.H1 * e.W1) * e.C1, 0});
    if (!e.c1_fused && !e.c1_pool) e.views.push_back({"conv1.dC", e.dC1, (size_t)B * e.H1 * e.W1 * e.C1, 0});
    if (e.c1_pool) {
        e.views.push_back({"conv1.code", e.code1, (size_t)B * (e.H1 / 2) * (e.W1 / 2) * e.C1, 1});
        e.views.push_back({"conv1.dP", e.dP1, (size_t)B * (e.H1 / 2) * (e.W1 / 2) * e.C1, 0});
    }
    for (size_t k = 0; k < e.convs.size(); ++k) {
        const ConvLayer &L = e.convs[k];
        const std::string pre = "conv" + std::to_string(k + 2);
        const size_t np = (size_t)B * (L.H / 2) * (L.W / 2) * L.COUT;
        e.views.push_back({pre + ".out", L.out, np, 0});
        e.views.push_back({pre + ".code", L.code, np, 1});
        e.views.push_back({pre + ".dP", L.dP, np, 0});
        if (!L.fbwd_up && !L.up) e.views.push_back({pre + ".dC", L.dC, (size_t)B * L.H * L.W * L.COUT, 0});
        e.views.push_back({pre + ".wf", L.wf, (size_t)9 * L.CIN * L.COUT, 0});
        e.views.push_back({pre + ".wd", L.wd, (size_t)9 * L.CIN * L.COUT, 0});
    }
    if (e.has_hidden) {
        e.views.push_back({"hidden.out", e.a_hid, (size_t)B * e.HD, 0});
        e.views.push_back({"hidden.dZ", e.dZ_hid, (size_t)B * e.HD, 0});
    }
    e.views.push_back({"flat.d", e.dflat, (size_t)B * e.F, 0});
    if (e.has_hidden) {
        e.views.push_back({"hidden.wP", e.wP, (size_t)e.F * e.HD, 0});
    } else {
        e.views.push_back({"head.dz", e.dz, (size_t)B * e.NC, 2});
    }
    // bf16 weight packing jobs (the hidden Linear weight's rows: `fc`)
    PackJobs &pj = e.pack;
    pj.count = 0;
    for (auto &L : e.convs) {
        const Stage &s = st[L.si];
        pj.j[pj.count++] = {0, n.params + s.poff, L.wf, L.COUT, L.CIN, 0, 0, 0, (long long)9 * L.CIN * L.COUT};
        pj.j[pj.count++] = {1, n.params + s.poff, L.wd, L.COUT, L.CIN, 0, 0, 0, (long long)9 * L.CIN * L.COUT};
    }
    if (e.direct_head)   // the classifier weight [F][NC] in its grouped bf16 layout
        pj.j[pj.count++] = {4, n.params + st[e.head_si].poff, e.wq, e.F, e.NC, e.fC, e.fH, e.fW, (long long)e.F * e.NC};
    pj.conv_blocks = sm_count();
    pj.fc = PackJob{};
    e.pack_grid = pj.conv_blocks;
    if (e.has_hidden) {
        pj.fc = {5, n.params + st[e.hid_si].poff, e.wP, e.F, e.HD, e.fC, e.fH, e.fW, (long long)e.F * e.HD};
        e.pack_grid += grid_for((long long)e.F * e.HD / 4, 256, 8);
    }
    return kOk;
}

// Dynamic shared memory above the default 48 KB for `kern` (set once per kernel and size;
// kernels of the same signature are told apart by their address).
template <class K>
int allow_smem(K *kern, size_t bytes) {
    static std::vector<std::pair<const void *, size_t>> allowed;
    if (bytes <= 48 * 1024) return kOk;
    for (const auto &a : allowed)
        if (a.first == (const void *)kern && bytes <= a.second) return kOk;
    if (bytes > 227 * 1024) return fail(kBadArg, "tc engine: %zu bytes of shared memory needed", bytes);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        return check_cuda("dynamic shared memory attribute");
    allowed.push_back({(const void *)kern, bytes});
    return kOk;
}

// One training step, or (logits_out != null) the forward pass only: logits
// [B][classes] fp32 and, with y, the loss sum; no gradients, no update.
int tc_run(Net &n, TcEngine &e, const float *x, const float *y, float *loss_out, float *logits_out = nullptr) {
    const int B = e.B;
    auto &st = n.st;
    int rc;
    // ---- pack bf16 operands from the fp32 master: inside the first conv's kernel when that is
    // the tensor-core one (the "pack" group is then empty), else a launch of its own
    const bool c1_tc = e.C1 == 32 && !e.c1_pool && e.pad1 == 1 && e.H1 == e.H0 && e.W1 == e.W0;
    if (!c1_tc) {
        launch_pdl(pack_kernel, dim3(e.pack_grid), dim3(256), 0, e.pack);
        ZB_LAUNCH_CHECK("pack");
    }
    prof_mark(n, "pack");
    // ---- forward
    const Stage &s1 = st[e.c1_si];
    const float *w1 = n.params + s1.poff, *b1 = w1 + s1.pn_w;
    {
        const long long pix = (long long)B * (e.c1_pool ? (e.H1 / 2) * (e.W1 / 2) : e.H1 * e.W1);
        const int grid = grid_for(pix, 128, 8);
        const size_t xsm = (size_t)(e.H0 + 2 * e.pad1) * (e.W0 + 2 * e.pad1) * sizeof(float);
        const int gimg = B < sm_count() * 4 ? B : sm_count() * 4;
        if (!e.c1_pool && (e.H0 + 2 * e.pad1) * (e.W0 + 2 * e.pad1) > kStageRegs * 256)
            return fail(kBadArg, "tc engine: first-conv image too large (padded %d x %d)", e.H0 + 2 * e.pad1,
                        e.W0 + 2 * e.pad1);
        if (c1_tc) {   // 3x3, pad 1, same size
            // tensor cores: one 128 x 32 x 32 MMA per 128 output pixels; the CTAs also pack
            const long long tiles = (pix + 127) / 128;
            const int g = tiles < (long long)sm_count() * 8 ? (int)tiles : sm_count() * 8;
            launch_pdl(tc::conv_first_tc_kernel<32, PackWork>, dim3(g), dim3(128), tc::ConvFirstTcShape<32>::SMEM, x,
                       w1, b1, e.a1, B, e.H0, e.W0, device_error_word(), PackWork{e.pack});
        } else if (e.C1 == 32 && !e.c1_pool) conv_first_fwd_img_kernel<32><<<gimg, 256, xsm, stream()>>>(x, w1, b1, e.a1, B, e.H0, e.W0, e.pad1);
        else if (e.C1 == 32 && xsm <= 48 * 1024) {   // two image buffers
            if ((rc = allow_smem(conv_first_pool_img_kernel<32>, 2 * xsm))) return rc;
            conv_first_pool_img_kernel<32><<<gimg, 256, 2 * xsm, stream()>>>(x, w1, b1, e.a1, e.code1, B, e.H0, e.W0, e.pad1);
        }
        else if (e.C1 == 32) conv_first_fwd_kernel<32, true><<<grid, 128, 0, stream()>>>(x, w1, b1, e.a1, e.code1, B, e.H0, e.W0, e.pad1);
        else if (!e.c1_pool) conv_first_fwd_img_kernel<16><<<gimg, 256, xsm, stream()>>>(x, w1, b1, e.a1, B, e.H0, e.W0, e.pad1);
        else if (xsm <= 48 * 1024) {
            if ((rc = allow_smem(conv_first_pool_img_kernel<16>, 2 * xsm))) return rc;
            conv_first_pool_img_kernel<16><<<gimg, 256, 2 * xsm, stream()>>>(x, w1, b1, e.a1, e.code1, B, e.H0, e.W0, e.pad1);
        }
        else conv_first_fwd_kernel<16, true><<<grid, 128, 0, stream()>>>(x, w1, b1, e.a1, e.code1, B, e.H0, e.W0, e.pad1);
        ZB_LAUNCH_CHECK("conv_first_fwd");
        prof_mark(n, "conv_fwd");
    }
    for (auto &L : e.convs) {
        if ((rc = run_conv_fwd(L))) return rc;
        prof_mark(n, "conv_fwd");
    }
    if (e.direct_head) {   // the classifier follows the last pool: forward, loss and dA in one kernel
        const Stage &sf = st[e.head_si];
        const int smem = e.F / 8 * kHeadGroup * 2;
        static int attr = 0;
        if (attr < smem) {
            if (cudaFuncSetAttribute(head_direct_kernel<12>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
                return check_cuda("head_direct smem attribute");
            attr = smem;
        }
        const bf16 *flat = e.convs.empty() ? e.a1 : e.convs.back().out;
        float *gW = n.grads + sf.poff, *gb = gW + sf.pn_w;
        launch_pdl(head_direct_kernel<12>, dim3(e.head_grid), dim3(kHeadWarps * 32), smem, flat, e.wq, n.params + sf.poff + sf.pn_w,
                   y, logits_out ? nullptr : e.dz, logits_out ? nullptr : e.dflat, logits_out,
                   (logits_out && !(y && loss_out)) ? nullptr : e.head_partial, B, e.F, 1.0f / (float)B);
        ZB_LAUNCH_CHECK("head direct");
        if (logits_out) {
            if (y && loss_out) {   // only the loss of the evaluation partials [NC zeros | loss] is kept
                ReduceArgs r{e.head_partial, e.head_grid, e.NC + 1, 7, 0, e.NC, 0, 0, 0, 0, nullptr, nullptr, nullptr};
                r.dst4 = loss_out;
                if ((rc = reduce(r))) return rc;
            }
            prof_mark(n, "softmax_ce");
            return kOk;
        }
        {   // classifier bias gradient and the loss sum (block partials, in block order)
            ReduceArgs r{e.head_partial, e.head_grid, e.NC + 1, 4, 0, e.NC, 0, 0, 0, 0, nullptr, gb, nullptr};
            r.dst4 = loss_out;
            if ((rc = reduce(r))) return rc;
        }
        prof_mark(n, "softmax_ce");
        launch_pdl(head_direct_wgrad_kernel<12>, dim3((e.F / 512) * e.hdw_splits), dim3(256), 0, flat, e.dz,
                   e.hdw_partial, B, e.F, e.hdw_splits);
        ZB_LAUNCH_CHECK("head direct weight gradient");
        {
            ReduceArgs r{e.hdw_partial, e.hdw_splits, (long long)e.F * e.NC, 3, e.F, e.NC, 0, e.fC, e.fH, e.fW,
                         gW, nullptr, nullptr};
            if ((rc = reduce(r))) return rc;
        }
        if ((rc = dp_bucket_ready(n, sf.poff))) return rc;
        prof_mark(n, "linear_bwd");
    } else if (e.fc_fwd.ksplit > 1) {
        if ((rc = launch_gemm<128, tc::kGemmPartial, 6, true>(e.fc_fwd))) return rc;
        if (logits_out) {   // (a training step's head kernel sums the splits itself)
            ReduceArgs r{e.fc_fwd_partial, e.fc_fwd.ksplit, (long long)B * e.HD, 6, B, e.HD, 0, 0, 0, 0,
                         nullptr, nullptr, nullptr, e.fc_fwd.bias, e.a_hid};
            if ((rc = reduce(r))) return rc;
        }
    } else if ((rc = launch_gemm<128, tc::kGemmBiasRelu, 6, true>(e.fc_fwd))) {
        return rc;
    }
    if (!e.direct_head) prof_mark(n, "linear_fwd");
    if (e.direct_head) {
        // (the classifier, loss and its backward ran above)
    } else if (logits_out) {   // evaluation: classifier and loss only
        const Stage &sf = st[e.head_si];
        launch_pdl(head_fwd_kernel<256, 10>, dim3(e.head_grid), dim3(256), 0, e.a_hid, n.params + sf.poff,
                   n.params + sf.poff + sf.pn_w, y, logits_out, (y && loss_out) ? e.head_partial : nullptr, B);
        ZB_LAUNCH_CHECK("head forward");
        if (y && loss_out) {
            ReduceArgs r{e.head_partial, e.head_grid, 1, 0, 1, 1, 0, 0, 0, 0, loss_out, nullptr, nullptr};
            if ((rc = reduce(r))) return rc;
        }
        prof_mark(n, "softmax_ce");
        return kOk;
    }
    // Deep reductions whose partial sums nothing reads before the next fused backward kernel
    // ends join that kernel's reduction launch (fewer launches).  Not while the data-parallel
    // exchange starts beside the fused kernel: it needs them final.
    ReduceArgs held[kMaxReduceJobs];
    int nheld = 0;
    const bool hold_ok = !(n.peer.on && n.peer.two_phase);
    // ---- head: classifier, loss, start of the backward (hidden Linear + classifier)
    if (!e.direct_head) {
    const Stage &sh = st[e.head_si];
    float *gW5 = n.grads + sh.poff, *gb5 = gW5 + sh.pn_w;
    const Stage &sd = st[e.hid_si];
    float *gW4 = n.grads + sd.poff, *gb4 = gW4 + sd.pn_w;
    if (e.fc_fwd.ksplit > 1)   // the hidden Linear's split-K sum, bias and ReLU in the head
        launch_pdl(head_kernel<256, 10, true>, dim3(e.head_grid), dim3(256), 0, e.a_hid, n.params + sh.poff,
                   n.params + sh.poff + sh.pn_w, y, e.dZ_hid, e.row_loss, e.head_partial, B, 1.0f / (float)B,
                   (const float *)e.fc_fwd_partial, e.fc_fwd.ksplit, (const float *)e.fc_fwd.bias);
    else
        launch_pdl(head_kernel<256, 10>, dim3(e.head_grid), dim3(256), 0, e.a_hid, n.params + sh.poff,
                   n.params + sh.poff + sh.pn_w, y, e.dZ_hid, e.row_loss, e.head_partial, B, 1.0f / (float)B,
                   (const float *)nullptr, 0, (const float *)nullptr);
    ZB_LAUNCH_CHECK("head");
    {   // fc2 dW, db, fc1 db and the loss sum (the blocks' partials, in block order): nothing reads
        // them before the optimizer unless an all-reduce bucket or the mid-step exchange takes them
        // first, so they join the fused phase's reduction launch
        ReduceArgs r{e.head_partial, e.head_grid, (long long)head_pstride(e.HD, e.NC), 4, e.HD, e.NC, 0, 0, 0, 0,
                     gW5, gb5, gb4};
        r.dst4 = loss_out;
        const bool hold_head = hold_ok && (n.world <= 1 || n.peer.in_step) && r.splits >= 32 && r.n <= 131072;
        if (hold_head) held[nheld++] = r;
        else if ((rc = reduce(r))) return rc;
    }
    prof_mark(n, "softmax_ce");
    // ---- hidden Linear backward
    {   // dflat = dZ W^T
        const int bn = e.F / e.fc_dgrad.n_tiles;
        rc = bn == 224 ? launch_gemm<224, tc::kGemmStore, 4>(e.fc_dgrad)
             : bn == 256 ? launch_gemm<256, tc::kGemmStore, 4>(e.fc_dgrad)
                         : launch_gemm<128, tc::kGemmStore, 4>(e.fc_dgrad);
        if (rc) return rc;
    }
    if (e.fc_wg.splits == 1) {   // the kernel writes the gradient itself
        WgradTcParams w = e.fc_wg;
        w.out = gW4;
        if ((rc = run_wgrad(w, w.mode, e.fc_wg_grid, e.fc_wg_smem))) return rc;
    } else {
        if ((rc = run_wgrad(e.fc_wg, e.fc_wg.mode, e.fc_wg_grid, e.fc_wg_smem))) return rc;
        ReduceArgs r{e.fc_partial, e.fc_wg.splits, (long long)e.F * e.HD, 3, e.F, e.HD, 0, e.fC, e.fH, e.fW,
                     gW4, nullptr, nullptr};
        if ((rc = reduce(r))) return rc;
    }
    // hidden + classifier Linear gradients and the loss are final: their
    // all-reduce (the bulk of the gradient bytes) overlaps the conv backward
    if ((rc = dp_bucket_ready(n, st[e.hid_si].poff))) return rc;
    prof_mark(n, "linear_bwd");
    }
    // ---- conv stages backward (last to first)
    const bf16 *dpooled = e.dflat;   // gradient w.r.t. the last pooled output
    for (int li = (int)e.convs.size() - 1; li >= 0; --li) {
        ConvLayer &L = e.convs[li];
        const Stage &s = st[L.si];
        const bf16 *dP = (li == (int)e.convs.size() - 1) ? dpooled : L.dP;
        if (!(L.fused_bwd && L.fbwd_up) && !L.up) {
            const int G = L.COUT / 8, slots = 256 / G;
            unpool_kernel<<<L.unpool_grid, slots * G, slots * G * 8 * sizeof(float), stream()>>>(
                dP, L.code, L.dC, L.bias_partial, B, L.H, L.W, L.COUT);
            ZB_LAUNCH_CHECK("unpool");
            ReduceArgs r{L.bias_partial, L.unpool_grid, (long long)L.COUT, 0, 1, L.COUT, 0, 0, 0, 0,
                         n.grads + s.poff + s.pn_w, nullptr, nullptr};
            if ((rc = reduce(r))) return rc;
            prof_mark(n, "pool_bwd");
        }
        if (L.fused_bwd) {
            // data parallel over peer memory: the gradients of every later layer are final, so
            // their exchange and update run on a side stream beside this kernel
            if ((rc = peer_step_mid(n, s.poff + s.pn_w + s.pn_b))) return rc;
            if ((rc = run_conv_bwd_fused(L, x, dP))) return rc;
            // the kernel's partials: conv2 dW, conv2 db (UP), conv1 dW + db (C1)
            ReduceArgs jobs[kMaxReduceJobs];
            int nj = 0;
            for (int j = 0; j < nheld; ++j) jobs[nj++] = held[j];
            nheld = 0;
            jobs[nj++] = ReduceArgs{L.fbwd_partial, L.fbwd_grid, (long long)L.COUT * 9 * L.CIN, 1, L.COUT, 9 * L.CIN,
                                    L.CIN, 0, 0, 0, n.grads + s.poff, nullptr, nullptr};
            if (L.fbwd_up)
                jobs[nj++] = ReduceArgs{L.fbwd_bias_partial, 4 * L.fbwd_grid, (long long)L.COUT, 0, 1, L.COUT, 0, 0, 0, 0,
                                        n.grads + s.poff + s.pn_w, nullptr, nullptr};
            if (L.fbwd_c1)
                jobs[nj++] = ReduceArgs{e.c1_partial, e.c1_wgrad_grid, (long long)e.C1 * 10, 5, e.C1, 10, 0, 0, 0, 0,
                                        n.grads + s1.poff, n.grads + s1.poff + s1.pn_w, nullptr};
            bool deep = true;   // every job has many splits of a short vector
            for (int j = 0; j < nj; ++j) deep = deep && jobs[j].splits >= 32 && jobs[j].n <= 131072;
            if (deep) {
                if ((rc = reduce_multi(jobs, nj))) return rc;
            } else {
                for (int j = 0; j < nj; ++j)
                    if ((rc = reduce(jobs[j]))) return rc;
            }
            prof_mark(n, "conv_bwd");
            continue;
        }
        if ((rc = run_conv_dgrad(L, dP))) return rc;
        // (up: the bias partials of the dgrad kernel's builders are summed with the weight gradient's)
        prof_mark(n, "conv_dgrad");
        if (L.wg_halo) {
            if ((rc = run_wgrad_halo(L))) return rc;
            ReduceArgs r{L.whalo_partial, L.whalo.splits, (long long)L.COUT * 9 * L.CIN, 1, L.COUT, 9 * L.CIN,
                         L.CIN, 0, 0, 0, n.grads + s.poff, nullptr, nullptr};
            if ((rc = reduce(r))) return rc;
        } else {
            if ((rc = run_wgrad(L.wg, L.wg_mode, L.wg_grid, L.wg_smem, L.up ? dP : nullptr))) return rc;
            ReduceArgs jobs[2];
            jobs[0] = ReduceArgs{L.wg_partial, L.wg.splits, (long long)L.wg.M * L.wg.N,
                                 L.wg_mode == tc::kWgConvCo ? 1 : 2, L.wg.M, L.wg.N, L.CIN, 0, 0, 0,
                                 n.grads + s.poff, nullptr, nullptr};
            const int nj = L.up ? 2 : 1;
            if (L.up)   // the bias gradient from the dgrad kernel's builders
                jobs[1] = ReduceArgs{L.up_bias_partial, 4 * L.up_grid, (long long)L.COUT, 0, 1, L.COUT, 0, 0, 0, 0,
                                     n.grads + s.poff + s.pn_w, nullptr, nullptr};
            bool deep = true;
            for (int j = 0; j < nj; ++j) deep = deep && jobs[j].splits >= 32 && jobs[j].n <= 131072;
            const bool next_fused = li > 0 && e.convs[li - 1].fused_bwd;
            if (deep && hold_ok && next_fused && nheld + nj + 3 <= kMaxReduceJobs) {
                for (int j = 0; j < nj; ++j) held[nheld++] = jobs[j];
            } else if (deep) {
                if ((rc = reduce_multi(jobs, nj))) return rc;
            } else {
                for (int j = 0; j < nj; ++j)
                    if ((rc = reduce(jobs[j]))) return rc;
            }
        }
        prof_mark(n, "conv_wgrad");
    }
    if (nheld && (rc = reduce_multi(held, nheld))) return rc;   // (no fused layer took them)
    nheld = 0;
    // ---- first conv backward (dC1 written by the next conv's dgrad, masked)
    if (e.c1_fused) return kOk;   // taken by the next conv's fused backward kernel
    {
        const int padded = (e.H0 + 2 * e.pad1) * (e.W0 + 2 * e.pad1);
        const size_t smem = (size_t)(padded > 8 * 4 * 80 ? padded : 8 * 4 * 80) * sizeof(float);
        if (smem > 48 * 1024) return fail(kBadArg, "tc engine: first-conv image too large for the weight-gradient kernel");
        const bool big = padded > kStageRegs * 256;   // past the register stager: a plain copy per image
        if (e.c1_pool) {   // straight from the pooled gradient and the codes: no unpooled dC1
            // two image buffers (the reduction reuses the first)
            const size_t psmem = (size_t)(2 * padded > 8 * 4 * 80 ? 2 * padded : 8 * 4 * 80) * sizeof(float);
            if (e.C1 == 32) {
                if ((rc = allow_smem(conv_first_wgrad_pool_kernel<32>, psmem))) return rc;
                conv_first_wgrad_pool_kernel<32><<<e.c1_wgrad_grid, 256, psmem, stream()>>>(e.dP1, e.code1, x, e.c1_partial, B, e.H0, e.W0, e.pad1);
            } else {
                if ((rc = allow_smem(conv_first_wgrad_pool_kernel<16>, psmem))) return rc;
                conv_first_wgrad_pool_kernel<16><<<e.c1_wgrad_grid, 256, psmem, stream()>>>(e.dP1, e.code1, x, e.c1_partial, B, e.H0, e.W0, e.pad1);
            }
        }
        else if (e.C1 == 32 && !big) conv_first_wgrad_kernel<32><<<e.c1_wgrad_grid, 256, smem, stream()>>>(e.dC1, x, e.c1_partial, B, e.H0, e.W0, e.pad1);
        else if (e.C1 == 32) conv_first_wgrad_kernel<32, true><<<e.c1_wgrad_grid, 256, smem, stream()>>>(e.dC1, x, e.c1_partial, B, e.H0, e.W0, e.pad1);
        else if (!big) conv_first_wgrad_kernel<16><<<e.c1_wgrad_grid, 256, smem, stream()>>>(e.dC1, x, e.c1_partial, B, e.H0, e.W0, e.pad1);
        else conv_first_wgrad_kernel<16, true><<<e.c1_wgrad_grid, 256, smem, stream()>>>(e.dC1, x, e.c1_partial, B, e.H0, e.W0, e.pad1);
    }
    ZB_LAUNCH_CHECK("conv_first_wgrad");
    {
        ReduceArgs r{e.c1_partial, e.c1_wgrad_grid, (long long)e.C1 * 10, 5, e.C1, 10, 0, 0, 0, 0,
                     n.grads + s1.poff, n.grads + s1.poff + s1.pn_w, nullptr};
        if ((rc = reduce(r))) return rc;
    }
    prof_mark(n, "conv_wgrad");
    return kOk;
}

}  // namespace

int tc_create(Net &n) {
    TcEngine *e = new TcEngine();
    int rc = tc_build(n, *e);
    if (rc) {
        for (void *p : e->allocs) cudaFree(p);
        delete e;
        return rc;
    }
    n.tc = e;
    return kOk;
}

void tc_destroy(Net &n) {
    if (!n.tc) return;
    cudaStreamSynchronize(stream());
    for (void *p : n.tc->allocs) cudaFree(p);
    delete n.tc;
    n.tc = nullptr;
}

int tc_step(Net &n, const float *x, const float *y, float *loss_out) {
    if (!n.tc) return fail(kBadArg, "tc engine missing");
    int rc = tc_run(n, *n.tc, x, y, loss_out);
    if (rc) return rc;
    return kOk;
}

int tc_forward(Net &n, const float *x, const float *y, float *logits, float *loss_out) {
    if (!n.tc) return fail(kBadArg, "tc engine missing");
    return tc_run(n, *n.tc, x, y, loss_out, logits);
}

int tc_sync_params(Net &n) {
    (void)n;
    return kOk;
}

__global__ void widen_kernel(const void *src, int kind, float *dst, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        if (kind == 0) dst[i] = __bfloat162float(reinterpret_cast<const bf16 *>(src)[i]);
        else if (kind == 1) dst[i] = (float)reinterpret_cast<const uint8_t *>(src)[i];
        else dst[i] = reinterpret_cast<const float *>(src)[i];
    }
}

int tc_inspect(Net &n, int index, char *name, int name_len, float *host, unsigned long n_floats) {
    if (!n.tc || index < 0 || index >= (int)n.tc->views.size()) return 0;
    const auto &v = n.tc->views[index];
    if (name && name_len > 0) {
        strncpy(name, v.name.c_str(), (size_t)name_len - 1);
        name[name_len - 1] = 0;
    }
    if (host && n_floats) {
        const size_t cnt = n_floats < v.n ? n_floats : v.n;
        float *tmp = nullptr;
        if (cudaMalloc((void **)&tmp, cnt * sizeof(float)) != cudaSuccess) { cudaGetLastError(); return kBadHandle; }
        widen_kernel<<<grid_for((long long)cnt, 256, 4), 256, 0, stream()>>>(v.p, v.kind, tmp, cnt);
        cudaMemcpyAsync(host, tmp, cnt * sizeof(float), cudaMemcpyDeviceToHost, stream());
        cudaStreamSynchronize(stream());
        cudaFree(tmp);
        int rc = check_cuda("zilla_net_inspect");
        if (rc) return rc;
    }
    return (int)v.n;
}

}  // namespace zb
