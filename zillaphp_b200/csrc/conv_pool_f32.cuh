// conv_pool_f32.cuh -- gather functors that turn the reference's matmul and
// conv contractions into simt_gemm problems (fp32, NCHW / row-major).
#pragma once

#include "gemm_f32.cuh"

namespace zb {

// C[M,N] = A[M,K] @ B[K,N], row-major (matmul_dev).
struct GemmNN {
    const float *A, *B;
    float *Cm;
    int M, N, K;
    static constexpr bool kAMFast = false, kBNFast = true, kExactOrder = true;
    __device__ float init(int, int) const { return 0.0f; }
    GemmNN(const float *a, const float *b, float *c, int m, int n, int k) : A(a), B(b), Cm(c), M(m), N(n), K(k) {}
    __device__ float a(int m, int k) const { return A[(size_t)m * K + k]; }
    __device__ float b(int k, int n) const { return B[(size_t)k * N + n]; }
    __device__ void store(int m, int n, float v) const { Cm[(size_t)m * N + n] = v; }
};

// C[M,N] = A^T B with A stored [K,M] (matmul_tn_dev).
struct GemmTN {
    const float *A, *B;
    float *Cm;
    int M, N, K;
    static constexpr bool kAMFast = true, kBNFast = true, kExactOrder = false;
    __device__ float init(int, int) const { return 0.0f; }
    GemmTN(const float *a, const float *b, float *c, int m, int n, int k) : A(a), B(b), Cm(c), M(m), N(n), K(k) {}
    __device__ float a(int m, int k) const { return A[(size_t)k * M + m]; }
    __device__ float b(int k, int n) const { return B[(size_t)k * N + n]; }
    __device__ void store(int m, int n, float v) const { Cm[(size_t)m * N + n] = v; }
};

// C[M,N] = A B^T with B stored [N,K] (matmul_nt_dev).
struct GemmNT {
    const float *A, *B;
    float *Cm;
    int M, N, K;
    static constexpr bool kAMFast = false, kBNFast = false, kExactOrder = false;
    __device__ float init(int, int) const { return 0.0f; }
    GemmNT(const float *a, const float *b, float *c, int m, int n, int k) : A(a), B(b), Cm(c), M(m), N(n), K(k) {}
    __device__ float a(int m, int k) const { return A[(size_t)m * K + k]; }
    __device__ float b(int k, int n) const { return B[(size_t)n * K + k]; }
    __device__ void store(int m, int n, float v) const { Cm[(size_t)m * N + n] = v; }
};

struct ConvGeom {
    int B, C, H, W, oC, oH, oW, kH, kW, s, p;
    // divisors of the index decompositions: output plane, output row, input
    // plane, input row, taps, tap row
    FastDiv f_ohw, f_ow, f_hw, f_w, f_kk, f_kw;
    ConvGeom(int B_, int C_, int H_, int W_, int oC_, int oH_, int oW_, int kH_, int kW_, int s_, int p_)
        : B(B_), C(C_), H(H_), W(W_), oC(oC_), oH(oH_), oW(oW_), kH(kH_), kW(kW_), s(s_), p(p_),
          f_ohw(oH_ * oW_), f_ow(oW_), f_hw(H_ * W_), f_w(W_), f_kk(kH_ * kW_), f_kw(kW_) {}
};

// Forward: M = B*oH*oW output pixels, N = oC, K = C*kH*kW taps.
// y = bias + sum_k x*w, optionally followed by ReLU (fused net path).  The
// accumulator starts at the bias and adds x*w separately rounded in (c, kh, kw)
// order, the order of native/cpu/zilla_cpu.c:127-139, so the forward is
// bit-identical to the reference CPU code built with strict IEEE flags (padding
// taps add +0 where the reference skips them, which leaves the sum unchanged).
struct ConvFwdF32 {
    const float *x, *w, *bias;
    float *y;
    ConvGeom g;
    int M, N, K;
    bool relu;
    static constexpr bool kAMFast = true, kBNFast = false, kExactOrder = true;
    __device__ float init(int, int n) const { return bias[n]; }
    ConvFwdF32(const float *x_, const float *w_, const float *b_, float *y_, int B, int C, int H, int W,
               int oC, int oH, int oW, int kH, int kW, int s, int p, bool relu_)
        : x(x_), w(w_), bias(b_), y(y_), g{B, C, H, W, oC, oH, oW, kH, kW, s, p},
          M(B * oH * oW), N(oC), K(C * kH * kW), relu(relu_) {}
    __device__ float a(int m, int k) const {
        const int hw = g.oH * g.oW, kk = g.kH * g.kW;
        const int b = g.f_ohw.div(m), r = m - b * hw, oh = g.f_ow.div(r), ow = r - oh * g.oW;
        const int c = g.f_kk.div(k), t = k - c * kk, dh = g.f_kw.div(t), dw = t - dh * g.kW;
        const int ih = oh * g.s - g.p + dh, iw = ow * g.s - g.p + dw;
        if ((unsigned)ih >= (unsigned)g.H || (unsigned)iw >= (unsigned)g.W) return 0.0f;
        return x[(((size_t)b * g.C + c) * g.H + ih) * g.W + iw];
    }
    __device__ float b(int k, int n) const { return w[(size_t)n * K + k]; }
    __device__ void store(int m, int n, float v) const {
        const int hw = g.oH * g.oW;
        const int b = g.f_ohw.div(m), r = m - b * hw;
        float o = v;
        if (relu) o = o > 0.0f ? o : 0.0f;
        y[((size_t)b * g.oC + n) * hw + r] = o;
    }
};

// Input gradient: M = B*H*W input pixels, N = C, K = oC*kH*kW.
// dx[b,c,ih,iw] = sum_{oc,kh,kw} gout[b,oc,oh,ow] * w[oc,c,kh,kw] over the
// (oh, ow) that reach (ih, iw) (native/cuda/conv2d_batched.cu:96-141).
// `mask`, when set, multiplies by (mask > 0): the fused ReLU backward of the
// layer that produced the conv input.
struct ConvDgradF32 {
    const float *gout, *w;
    float *dx;
    const float *mask;
    ConvGeom g;
    int M, N, K;
    static constexpr bool kAMFast = true, kBNFast = false, kExactOrder = false;
    __device__ float init(int, int) const { return 0.0f; }
    ConvDgradF32(const float *go, const float *w_, float *dx_, const float *mask_, int B, int C, int H,
                 int W, int oC, int oH, int oW, int kH, int kW, int s, int p)
        : gout(go), w(w_), dx(dx_), mask(mask_), g{B, C, H, W, oC, oH, oW, kH, kW, s, p},
          M(B * H * W), N(C), K(oC * kH * kW) {}
    __device__ float a(int m, int k) const {
        const int hw = g.H * g.W, kk = g.kH * g.kW;
        const int b = g.f_hw.div(m), r = m - b * hw, ih = g.f_w.div(r), iw = r - ih * g.W;
        const int oc = g.f_kk.div(k), t = k - oc * kk, dh = g.f_kw.div(t), dw = t - dh * g.kW;
        const int ohn = ih + g.p - dh, own = iw + g.p - dw;
        if (ohn < 0 || own < 0) return 0.0f;
        if (g.s != 1 && (ohn % g.s || own % g.s)) return 0.0f;
        const int oh = ohn / g.s, ow = own / g.s;
        if (oh >= g.oH || ow >= g.oW) return 0.0f;
        return gout[(((size_t)b * g.oC + oc) * g.oH + oh) * g.oW + ow];
    }
    __device__ float b(int k, int n) const {
        const int kk = g.kH * g.kW;
        const int oc = g.f_kk.div(k), t = k - oc * kk;
        return w[((size_t)oc * g.C + n) * kk + t];
    }
    __device__ void store(int m, int n, float v) const {
        const int hw = g.H * g.W;
        const int b = g.f_hw.div(m), r = m - b * hw;
        const size_t at = ((size_t)b * g.C + n) * hw + r;
        if (mask) v = mask[at] > 0.0f ? v : 0.0f;
        dx[at] = v;
    }
};

// Weight and bias gradient: M = oC, N = C*kH*kW + 1 (last column: bias,
// B(k, last) = 1), K = B*oH*oW output pixels (split-K, deterministic).
struct ConvWgradF32 {
    const float *x, *gout;
    float *dw, *db;
    ConvGeom g;
    int M, N, K;
    static constexpr bool kAMFast = false, kBNFast = false, kExactOrder = false;
    __device__ float init(int, int) const { return 0.0f; }
    ConvWgradF32(const float *x_, const float *go, float *dw_, float *db_, int B, int C, int H, int W,
                 int oC, int oH, int oW, int kH, int kW, int s, int p)
        : x(x_), gout(go), dw(dw_), db(db_), g{B, C, H, W, oC, oH, oW, kH, kW, s, p},
          M(oC), N(C * kH * kW + 1), K(B * oH * oW) {}
    __device__ float a(int m, int k) const {
        const int hw = g.oH * g.oW;
        const int b = g.f_ohw.div(k), r = k - b * hw;
        return gout[((size_t)b * g.oC + m) * hw + r];
    }
    __device__ float b(int k, int n) const {
        const int kk = g.kH * g.kW;
        if (n == N - 1) return 1.0f;
        const int hw = g.oH * g.oW;
        const int b = g.f_ohw.div(k), r = k - b * hw, oh = g.f_ow.div(r), ow = r - oh * g.oW;
        const int c = g.f_kk.div(n), t = n - c * kk, dh = g.f_kw.div(t), dwi = t - dh * g.kW;
        const int ih = oh * g.s - g.p + dh, iw = ow * g.s - g.p + dwi;
        if ((unsigned)ih >= (unsigned)g.H || (unsigned)iw >= (unsigned)g.W) return 0.0f;
        return x[(((size_t)b * g.C + c) * g.H + ih) * g.W + iw];
    }
    __device__ void store(int m, int n, float v) const {
        if (n == N - 1) db[m] = v;
        else dw[(size_t)m * (N - 1) + n] = v;
    }
};

// dW, db of a ConvWgradF32 problem: the direct kernel when the shape fits
// (3x3, stride 1, C % 16 == 0, oC % 32 == 0, one row's operands in 24 loads
// per thread), else the implicit GEMM.  ZB_FP32_WGRAD=gemm forces the GEMM.
int run_conv_wgrad(const ConvWgradF32 &pw, const char *what);

// 2x2-style max-pool forward with the reference's tie rule and batched flat
// argmax (conv_pool_f32.cu); shared by the *_dev entry points and the fp32 step.
__global__ void maxpool_fwd_kernel(const float *__restrict__ in, float *__restrict__ out,
                                   int *__restrict__ arg, int B, int C, int H, int W, int oH,
                                   int oW, int kH, int kW, int s);

}  // namespace zb
