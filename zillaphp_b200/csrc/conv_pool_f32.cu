// conv_pool_f32.cu -- exact-fp32 contractions and pooling behind the
// reference's entry points:
//   matmul_dev / matmul_tn_dev / matmul_nt_dev (native/cuda/device_ops.cu:44-75,
//     native/cuda/training_ops.cu:233-276; cuBLAS SGEMM there, a tiled
//     CUDA-core GEMM here, no TF32),
//   matmul_f32 (native/cuda/matmul.cu:93-144, host pointers),
//   conv2d_batched_fwd_dev / conv2d_batched_bwd_dev
//     (native/cuda/conv2d_batched.cu:69-271) and the per-sample
//     conv2d_fwd_dev / conv2d_bwd_dev (native/cuda/conv2d.cu:71-259) as
//     implicit GEMMs on NCHW tensors (no im2col buffer),
//   maxpool2d_batched_fwd_dev / _bwd_dev (native/cuda/pooling_batched.cu:
//     61-116) and maxpool2d_fwd_dev / _bwd_dev (native/cuda/pooling.cu:67-124).
#include <stdlib.h>
#include <string.h>

#include "conv_pool_f32.cuh"

using namespace zb;

namespace zb {

namespace {
float *g_ws = nullptr;
size_t g_ws_cap = 0;
}  // namespace

float *gemm_workspace(size_t floats) {
    if (floats > g_ws_cap) {
        if (g_ws) {
            cudaStreamSynchronize(stream());
            cudaFree(g_ws);
        }
        g_ws = nullptr;
        g_ws_cap = 0;
        if (cudaMalloc((void **)&g_ws, floats * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_ws_cap = floats;
    }
    return g_ws;
}

// Direct weight gradient of a 3x3 stride-1 convolution (fp32, NCHW), for
// 16-channel x 32-filter tiles.  The reduction runs over the B*oH rows
// (b, oh): each block takes a contiguous range of rows and, per row, stages
// in shared memory the 32 filters' gradient rows gout[b][oc][oh][:] and the 16
// channels' three input rows x[b][c][oh-p+kh][:] (zero-padded), then every
// thread accumulates 2 filters x 1 channel x 9 taps along the row with a
// sliding 3-wide window, 18 FMAs per 5 shared-memory loads.  The next row's
// values are loaded into registers while the current row is computed.  Block
// partials go to the split-K workspace in the layout of ConvWgradF32 ([split]
// [oC][C*9 + 1], the last column the bias), which simt_gemm_reduce_kernel
// sums in split order and stores (deterministic).
constexpr int kDwOct = 32, kDwCt = 16, kDwMaxLoads = 16;

struct DirectWgradArgs {
    const float *x, *gout;
    float *ws;
    int B, C, H, W, oC, oH, oW, p;
    int Wp, XS, NG, NX;              // padded row, channel stride in Xs, staged counts
    int rows, splits, ctiles;
    FastDiv f_ow, f_rowX, f_Wp, f_oH;  // oW, 3*Wp, Wp, oH
};

__global__ void __launch_bounds__(256, 3) conv3x3_wgrad_direct_kernel(const __grid_constant__ DirectWgradArgs A) {
    extern __shared__ float dsm[];
    float *Gs = dsm, *Xs = dsm + kDwOct * A.oW;
    const int tid = threadIdx.x;
    const int z = blockIdx.x;
    const int ct = blockIdx.y % A.ctiles, ot = blockIdx.y / A.ctiles;
    const int c0 = ct * kDwCt, oc0 = ot * kDwOct;
    const int cl = tid % kDwCt, ol = tid / kDwCt;   // channel, first of two filters (ol, ol + 16)
    const long long r_lo = (long long)A.rows * z / A.splits, r_hi = (long long)A.rows * (z + 1) / A.splits;
    const int nload = A.NG + A.NX;

    float pre[kDwMaxLoads];
    auto load_row = [&](int rr) {
        const int b = A.f_oH.div(rr), oh = rr - b * A.oH;
#pragma unroll
        for (int i = 0; i < kDwMaxLoads; ++i) {
            const int idx = tid + i * 256;
            float v = 0.0f;
            if (idx < A.NG) {
                const int o = A.f_ow.div(idx), ow = idx - o * A.oW;
                v = A.gout[(((size_t)b * A.oC + oc0 + o) * A.oH + oh) * A.oW + ow];
            } else if (idx < nload) {
                const int i2 = idx - A.NG;
                const int c = A.f_rowX.div(i2), rem = i2 - c * 3 * A.Wp;
                const int kh = A.f_Wp.div(rem), jp = rem - kh * A.Wp;
                const int ih = oh - A.p + kh, iw = jp - A.p;
                if ((unsigned)ih < (unsigned)A.H && (unsigned)iw < (unsigned)A.W)
                    v = A.x[(((size_t)b * A.C + c0 + c) * A.H + ih) * A.W + iw];
            }
            pre[i] = v;
        }
    };
    auto store_row = [&]() {
#pragma unroll
        for (int i = 0; i < kDwMaxLoads; ++i) {
            const int idx = tid + i * 256;
            if (idx < A.NG) {
                Gs[idx] = pre[i];
            } else if (idx < nload) {
                const int i2 = idx - A.NG;
                const int c = A.f_rowX.div(i2);
                Xs[c * A.XS + (i2 - c * 3 * A.Wp)] = pre[i];
            }
        }
    };

    float acc[2][9];
#pragma unroll
    for (int o = 0; o < 2; ++o)
#pragma unroll
        for (int t = 0; t < 9; ++t) acc[o][t] = 0.0f;
    float bacc[2] = {0.0f, 0.0f};
    const bool do_bias = ct == 0 && cl == 0;

    if (r_lo < r_hi) load_row((int)r_lo);
    for (long long rr = r_lo; rr < r_hi; ++rr) {
        __syncthreads();            // the previous row's reads of Gs / Xs are done
        store_row();
        __syncthreads();
        if (rr + 1 < r_hi) load_row((int)rr + 1);
        const float *g0 = Gs + ol * A.oW, *g1 = Gs + (ol + 16) * A.oW;
        const float *xr = Xs + cl * A.XS;
        float w[3][3];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
            w[kh][1] = xr[kh * A.Wp];
            w[kh][2] = xr[kh * A.Wp + 1];
        }
        for (int ow = 0; ow < A.oW; ++ow) {
#pragma unroll
            for (int kh = 0; kh < 3; ++kh) {
                w[kh][0] = w[kh][1];
                w[kh][1] = w[kh][2];
                w[kh][2] = xr[kh * A.Wp + ow + 2];
            }
            const float ga = g0[ow], gb = g1[ow];
#pragma unroll
            for (int kh = 0; kh < 3; ++kh)
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    acc[0][kh * 3 + kw] = fmaf(ga, w[kh][kw], acc[0][kh * 3 + kw]);
                    acc[1][kh * 3 + kw] = fmaf(gb, w[kh][kw], acc[1][kh * 3 + kw]);
                }
            if (do_bias) {
                bacc[0] += ga;
                bacc[1] += gb;
            }
        }
    }
    const int N = A.C * 9 + 1;
#pragma unroll
    for (int o = 0; o < 2; ++o) {
        const int oc = oc0 + ol + 16 * o;
        float *row = A.ws + ((size_t)z * A.oC + oc) * N;
#pragma unroll
        for (int t = 0; t < 9; ++t) row[(c0 + cl) * 9 + t] = acc[o][t];
        if (do_bias) row[N - 1] = bacc[o];
    }
}

int run_conv_wgrad(const ConvWgradF32 &pw, const char *what) {
    const ConvGeom &g = pw.g;
    static const bool force_gemm = [] {
        const char *e = getenv("ZB_FP32_WGRAD");
        return e && !strcmp(e, "gemm");
    }();
    const int Wp = g.W + 2 * g.p;
    const int XS = (3 * Wp) | 1;   // odd channel stride: 16 channels on 16 banks
    const int NG = kDwOct * g.oW, NX = kDwCt * 3 * Wp;
    const size_t smem = (size_t)(NG + kDwCt * XS) * sizeof(float);
    const bool fits = g.kH == 3 && g.kW == 3 && g.s == 1 && g.p >= 0 && g.p <= 2 && g.C % kDwCt == 0 &&
                      g.oC % kDwOct == 0 && g.oW >= 1 && g.oH >= 1 && NG + NX <= kDwMaxLoads * 256 &&
                      smem <= 48 * 1024 && (long long)g.B * g.oH < (1LL << 31);
    if (force_gemm || !fits) return run_simt_gemm(pw, 0, what);
    DirectWgradArgs A;
    A.x = pw.x; A.gout = pw.gout;
    A.B = g.B; A.C = g.C; A.H = g.H; A.W = g.W; A.oC = g.oC; A.oH = g.oH; A.oW = g.oW; A.p = g.p;
    A.Wp = Wp; A.XS = XS; A.NG = NG; A.NX = NX;
    A.rows = g.B * g.oH;
    A.ctiles = g.C / kDwCt;
    const int tiles = A.ctiles * (g.oC / kDwOct);
    int splits = 4 * sm_count() / tiles;
    if (splits < 1) splits = 1;
    if (splits > A.rows) splits = A.rows > 0 ? A.rows : 1;
    A.splits = splits;
    A.f_ow = FastDiv(g.oW); A.f_rowX = FastDiv(3 * Wp); A.f_Wp = FastDiv(Wp); A.f_oH = FastDiv(g.oH);
    A.ws = gemm_workspace((size_t)splits * pw.M * pw.N);
    if (!A.ws) return fail(kBadHandle, "%s: weight-gradient workspace allocation failed", what);
    conv3x3_wgrad_direct_kernel<<<dim3(splits, tiles), 256, smem, stream()>>>(A);
    ZB_LAUNCH_CHECK(what);
    simt_gemm_reduce_kernel<ConvWgradF32><<<grid_for((long long)pw.M * pw.N, 256), 256, 0, stream()>>>(pw, A.ws,
                                                                                                      splits);
    ZB_LAUNCH_CHECK(what);
    return kOk;
}

// ---------------------------------------------------------------- pooling
// native/cuda/pooling_batched.cu:21-59: max from -1e30 with strict '>' in
// (kh, kw) order (first maximum wins); argmax = flat index into the whole
// [B, C, H, W] input, stored as int32 bits in the float buffer.
__global__ void maxpool_fwd_kernel(const float *__restrict__ in, float *__restrict__ out,
                                   int *__restrict__ arg, int B, int C, int H, int W, int oH,
                                   int oW, int kH, int kW, int s) {
    const long long total = (long long)B * C * oH * oW;
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int ow = (int)(idx % oW);
        const int oh = (int)((idx / oW) % oH);
        const long long bc = idx / ((long long)oW * oH);
        const long long base = bc * H * W;
        float best = -1e30f;
        long long at = base;
        for (int kh = 0; kh < kH; ++kh) {
            const int ih = oh * s + kh;
            for (int kw = 0; kw < kW; ++kw) {
                const int iw = ow * s + kw;
                if (ih >= H || iw >= W) continue;
                const float v = in[base + (long long)ih * W + iw];
                if (v > best) { best = v; at = base + (long long)ih * W + iw; }
            }
        }
        out[idx] = best;
        arg[idx] = (int)at;
    }
}

// dX[argmax] += dY (caller zeroes dX, native/cuda/pooling_batched.cu:87-98).
// Windows that do not overlap (stride >= kernel) give every input element at
// most one source, so the add is a plain read-modify-write; overlapping
// windows use atomics.  Indices outside dX are skipped and reported.
template <bool kAtomic>
__global__ void maxpool_bwd_kernel(const float *__restrict__ gout, const int *__restrict__ arg,
                                   float *__restrict__ gin, long long total, long long n_in,
                                   int *__restrict__ err) {
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long t = arg[idx];
        if (t < 0 || t >= n_in) {
            if (err) atomicCAS(err, 0, 0x504f4f4c);  // "POOL": index out of range
            continue;
        }
        if (kAtomic) atomicAdd(gin + t, gout[idx]);
        else gin[t] += gout[idx];
    }
}

}  // namespace zb

namespace {

int conv_fwd(int in_id, int w_id, int b_id, int out_id, int B, int C, int H, int W, int oC,
             int oH, int oW, int kH, int kW, int stride, int pad, const char *name) {
    float *x = ptr(in_id), *w = ptr(w_id), *b = ptr(b_id), *y = ptr(out_id);
    if (!x || !w || !b || !y) return fail(kBadHandle, "%s: invalid handle", name);
    if (B < 0 || C <= 0 || H <= 0 || W <= 0 || oC <= 0 || kH <= 0 || kW <= 0 || stride <= 0 ||
        pad < 0)
        return fail(kBadArg, "%s: bad sizes", name);
    if (oH != (H + 2 * pad - kH) / stride + 1 || oW != (W + 2 * pad - kW) / stride + 1)
        return fail(kBadArg, "%s: output size mismatch", name);
    if (capacity(in_id) < (size_t)B * C * H * W || capacity(out_id) < (size_t)B * oC * oH * oW ||
        capacity(w_id) < (size_t)oC * C * kH * kW || capacity(b_id) < (size_t)oC)
        return fail(kBadHandle, "%s: buffer smaller than the shape", name);
    ConvFwdF32 p(x, w, b, y, B, C, H, W, oC, oH, oW, kH, kW, stride, pad, false);
    return run_simt_gemm(p, 1, name);
}

int conv_bwd(int in_id, int w_id, int go_id, int gi_id, int gw_id, int gb_id, int B, int C, int H,
             int W, int oC, int oH, int oW, int kH, int kW, int stride, int pad, const char *name) {
    float *x = ptr(in_id), *w = ptr(w_id), *go = ptr(go_id), *gi = ptr(gi_id), *gw = ptr(gw_id),
          *gb = ptr(gb_id);
    if (!x || !w || !go || !gi || !gw || !gb) return fail(kBadHandle, "%s: invalid handle", name);
    if (B < 0 || C <= 0 || H <= 0 || W <= 0 || oC <= 0 || kH <= 0 || kW <= 0 || stride <= 0 ||
        pad < 0)
        return fail(kBadArg, "%s: bad sizes", name);
    if (oH != (H + 2 * pad - kH) / stride + 1 || oW != (W + 2 * pad - kW) / stride + 1)
        return fail(kBadArg, "%s: output size mismatch", name);
    if (capacity(in_id) < (size_t)B * C * H * W || capacity(gi_id) < (size_t)B * C * H * W ||
        capacity(go_id) < (size_t)B * oC * oH * oW || capacity(w_id) < (size_t)oC * C * kH * kW ||
        capacity(gw_id) < (size_t)oC * C * kH * kW || capacity(gb_id) < (size_t)oC)
        return fail(kBadHandle, "%s: buffer smaller than the shape", name);
    ConvDgradF32 pd(go, w, gi, nullptr, B, C, H, W, oC, oH, oW, kH, kW, stride, pad);
    int rc = run_simt_gemm(pd, 1, name);
    if (rc) return rc;
    ConvWgradF32 pw(x, go, gw, gb, B, C, H, W, oC, oH, oW, kH, kW, stride, pad);
    return run_conv_wgrad(pw, name);
}

int pool_fwd(int in_id, int out_id, int arg_id, int B, int C, int H, int W, int oH, int oW,
             int kH, int kW, int s, const char *name) {
    float *x = ptr(in_id), *y = ptr(out_id), *a = ptr(arg_id);
    if (!x || !y || !a) return fail(kBadHandle, "%s: invalid handle", name);
    if (B < 0 || C <= 0 || H <= 0 || W <= 0 || oH <= 0 || oW <= 0 || kH <= 0 || kW <= 0 || s <= 0)
        return fail(kBadArg, "%s: bad sizes", name);
    if ((oH - 1) * s + kH > H || (oW - 1) * s + kW > W)
        return fail(kBadArg, "%s: window exceeds the input", name);
    const long long no = (long long)B * C * oH * oW;
    if (capacity(in_id) < (size_t)B * C * H * W || capacity(out_id) < (size_t)no ||
        capacity(arg_id) < (size_t)no)
        return fail(kBadHandle, "%s: buffer smaller than the shape", name);
    if ((long long)B * C * H * W > 0x7fffffffLL)
        return fail(kBadArg, "%s: input too large for int32 argmax", name);
    if (!no) return kOk;
    maxpool_fwd_kernel<<<grid_for(no, 256), 256, 0, stream()>>>(x, y, (int *)a, B, C, H, W, oH, oW,
                                                                kH, kW, s);
    ZB_LAUNCH_CHECK(name);
    return kOk;
}

int pool_bwd(int go_id, int arg_id, int gi_id, long long total, bool overlap, const char *name) {
    float *go = ptr(go_id), *a = ptr(arg_id), *gi = ptr(gi_id);
    if (!go || !a || !gi) return fail(kBadHandle, "%s: invalid handle", name);
    if (total < 0) return fail(kBadArg, "%s: bad sizes", name);
    if (capacity(go_id) < (size_t)total || capacity(arg_id) < (size_t)total)
        return fail(kBadHandle, "%s: buffer smaller than the shape", name);
    if (!total) return kOk;
    const long long n_in = (long long)capacity(gi_id);
    if (overlap)
        maxpool_bwd_kernel<true><<<grid_for(total, 256), 256, 0, stream()>>>(go, (const int *)a, gi, total, n_in, device_error_word());
    else
        maxpool_bwd_kernel<false><<<grid_for(total, 256), 256, 0, stream()>>>(go, (const int *)a, gi, total, n_in, device_error_word());
    ZB_LAUNCH_CHECK(name);
    return kOk;
}

int matmul_any(int a_id, int b_id, int c_id, int M, int K, int N, int variant, const char *name) {
    float *A = ptr(a_id), *B = ptr(b_id), *Cm = ptr(c_id);
    if (!A || !B || !Cm) return fail(kBadHandle, "%s: invalid handle", name);
    if (M < 0 || K < 0 || N < 0) return fail(kBadArg, "%s: negative size", name);
    if (capacity(a_id) < (size_t)M * K || capacity(b_id) < (size_t)K * N ||
        capacity(c_id) < (size_t)M * N)
        return fail(kBadHandle, "%s: buffer smaller than the shape", name);
    if (variant == 0) return run_simt_gemm(GemmNN(A, B, Cm, M, N, K), 0, name);
    if (variant == 1) return run_simt_gemm(GemmTN(A, B, Cm, M, N, K), 0, name);
    return run_simt_gemm(GemmNT(A, B, Cm, M, N, K), 0, name);
}

// Host-pointer staging for matmul_f32.
float *g_hm = nullptr;
size_t g_hm_cap = 0;

}  // namespace

extern "C" {

int matmul_dev(int a, int b, int c, int M, int K, int N) { return matmul_any(a, b, c, M, K, N, 0, "matmul_dev"); }
int matmul_tn_dev(int a, int b, int c, int M, int K, int N) { return matmul_any(a, b, c, M, K, N, 1, "matmul_tn_dev"); }
int matmul_nt_dev(int a, int b, int c, int M, int K, int N) { return matmul_any(a, b, c, M, K, N, 2, "matmul_nt_dev"); }

void matmul_f32(const float *A, const float *B, float *Cm, int M, int K, int N) {
    if (M <= 0 || N <= 0 || K < 0) return;
    const size_t na = (size_t)M * K, nb = (size_t)K * N, nc = (size_t)M * N;
    const size_t need = na + nb + nc;
    if (need > g_hm_cap) {
        if (g_hm) cudaFree(g_hm);
        g_hm = nullptr;
        g_hm_cap = 0;
        if (cudaMalloc((void **)&g_hm, need * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            fail(kBadHandle, "matmul_f32: staging allocation failed");
            return;
        }
        g_hm_cap = need;
    }
    float *dA = g_hm, *dB = g_hm + na, *dC = g_hm + na + nb;
    if (na) cudaMemcpyAsync(dA, A, na * sizeof(float), cudaMemcpyHostToDevice, stream());
    if (nb) cudaMemcpyAsync(dB, B, nb * sizeof(float), cudaMemcpyHostToDevice, stream());
    if (run_simt_gemm(GemmNN(dA, dB, dC, M, N, K), 0, "matmul_f32")) return;
    cudaMemcpyAsync(Cm, dC, nc * sizeof(float), cudaMemcpyDeviceToHost, stream());
    if (cudaStreamSynchronize(stream()) != cudaSuccess) check_cuda("matmul_f32");
}

int conv2d_batched_fwd_dev(int in, int w, int b, int out, int B, int C, int H, int W, int oC,
                           int oH, int oW, int kH, int kW, int stride, int pad) {
    return conv_fwd(in, w, b, out, B, C, H, W, oC, oH, oW, kH, kW, stride, pad, "conv2d_batched_fwd_dev");
}

int conv2d_batched_bwd_dev(int in, int w, int go, int gi, int gw, int gb, int B, int C, int H,
                           int W, int oC, int oH, int oW, int kH, int kW, int stride, int pad) {
    return conv_bwd(in, w, go, gi, gw, gb, B, C, H, W, oC, oH, oW, kH, kW, stride, pad, "conv2d_batched_bwd_dev");
}

int conv2d_fwd_dev(int in, int w, int b, int out, int C, int H, int W, int oC, int oH, int oW,
                   int kH, int kW, int stride, int pad) {
    return conv_fwd(in, w, b, out, 1, C, H, W, oC, oH, oW, kH, kW, stride, pad, "conv2d_fwd_dev");
}

int conv2d_bwd_dev(int in, int w, int go, int gi, int gw, int gb, int C, int H, int W, int oC,
                   int oH, int oW, int kH, int kW, int stride, int pad) {
    return conv_bwd(in, w, go, gi, gw, gb, 1, C, H, W, oC, oH, oW, kH, kW, stride, pad, "conv2d_bwd_dev");
}

int maxpool2d_batched_fwd_dev(int in, int out, int arg, int B, int C, int H, int W, int oH,
                              int oW, int kH, int kW, int s) {
    return pool_fwd(in, out, arg, B, C, H, W, oH, oW, kH, kW, s, "maxpool2d_batched_fwd_dev");
}

int maxpool2d_batched_bwd_dev(int go, int arg, int gi, int B, int C, int oH, int oW) {
    // The ABI carries no kernel/stride; pooling windows written by this
    // library's forward never overlap when stride >= kernel, but the
    // signature cannot tell, so overlapping-safe atomics are used unless the
    // index set is known to be collision-free (the fused step uses its own
    // gather kernels).
    return pool_bwd(go, arg, gi, (long long)B * C * oH * oW, true, "maxpool2d_batched_bwd_dev");
}

int maxpool2d_fwd_dev(int in, int out, int arg, int C, int H, int W, int oH, int oW, int kH,
                      int kW, int s) {
    return pool_fwd(in, out, arg, 1, C, H, W, oH, oW, kH, kW, s, "maxpool2d_fwd_dev");
}

int maxpool2d_bwd_dev(int go, int arg, int gi, int C, int oH, int oW) {
    return pool_bwd(go, arg, gi, (long long)C * oH * oW, true, "maxpool2d_bwd_dev");
}

}  // extern "C"
