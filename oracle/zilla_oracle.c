/*
 * zilla_oracle.c -- CPU restatement of ZillaPHP's training hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle that the CUDA library
 * is checked against; nothing in the product links, loads or calls it.
 *
 * It restates, in plain C with the same operation order, the reference's
 * CPU C-ABI (native/cpu/zilla_cpu.c, native/cpu/training_ops.c,
 * native/cpu/buffer_registry.c) and the pieces of the hot path that the
 * reference only has in PHP (src/Optim/Adam.php, src/Loss/CrossEntropy.php)
 * or only in CUDA (native/cuda/pooling_batched.cu argmax convention,
 * native/cuda/attention.cu row softmax).  Every function names the
 * reference lines it follows.  The exported names are the reference's own
 * so that the same step driver (cnn_step.c) can be linked against either
 * this restatement or the reference library built from its sources.
 *
 * Build strictly (no -ffast-math) so results are reproducible.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ *
 * Handle registry: native/cpu/buffer_registry.c:16-88.
 * 1024 slots, slot 0 never handed out, lowest free slot reused,
 * 64-byte aligned storage, free is idempotent.
 * ------------------------------------------------------------------ */
#define ORACLE_SLOTS 1024

static struct { float *p; size_t n; int used; } g_slot[ORACLE_SLOTS];

int zilla_cpu_buffer_alloc(size_t n_floats)
{
    if (n_floats == 0) return -1;
    for (int id = 1; id < ORACLE_SLOTS; ++id) {
        if (g_slot[id].used) continue;
        size_t bytes = (n_floats * sizeof(float) + 63) & ~(size_t)63;
        float *p = (float *)aligned_alloc(64, bytes);
        if (!p) return -1;
        g_slot[id].p = p;
        g_slot[id].n = n_floats;
        g_slot[id].used = 1;
        return id;
    }
    return -1;
}

void zilla_cpu_buffer_free(int id)
{
    if (id <= 0 || id >= ORACLE_SLOTS || !g_slot[id].used) return;
    free(g_slot[id].p);
    g_slot[id].p = NULL;
    g_slot[id].n = 0;
    g_slot[id].used = 0;
}

float *zilla_cpu_buffer_ptr(int id)
{
    if (id <= 0 || id >= ORACLE_SLOTS || !g_slot[id].used) return NULL;
    return g_slot[id].p;
}

int zilla_cpu_buffer_upload(int id, const float *host, size_t n_floats)
{
    float *p = zilla_cpu_buffer_ptr(id);
    if (!p || n_floats > g_slot[id].n) return -1;
    memcpy(p, host, n_floats * sizeof(float));
    return 0;
}

int zilla_cpu_buffer_download(int id, float *host, size_t n_floats)
{
    float *p = zilla_cpu_buffer_ptr(id);
    if (!p || n_floats > g_slot[id].n) return -1;
    memcpy(host, p, n_floats * sizeof(float));
    return 0;
}

/* ------------------------------------------------------------------ *
 * Host-pointer kernels: native/cpu/zilla_cpu.c:27-251 (naive paths).
 * ------------------------------------------------------------------ */

/* native/cpu/zilla_cpu.c:49-62: C = A[M,K] @ B[K,N], i-k-j order. */
void matmul_f32(const float *A, const float *B, float *C, int M, int K, int N)
{
    for (long i = 0; i < (long)M * N; ++i) C[i] = 0.0f;
    for (int i = 0; i < M; ++i) {
        float *crow = C + (size_t)i * N;
        for (int k = 0; k < K; ++k) {
            const float a = A[(size_t)i * K + k];
            const float *brow = B + (size_t)k * N;
            for (int j = 0; j < N; ++j) crow[j] += a * brow[j];
        }
    }
}

/* native/cpu/zilla_cpu.c:70-88 */
void relu_f32(const float *X, float *Y, int n) { for (int i = 0; i < n; ++i) Y[i] = X[i] > 0.0f ? X[i] : 0.0f; }
void add_f32(const float *A, const float *B, float *C, int n) { for (int i = 0; i < n; ++i) C[i] = A[i] + B[i]; }
void sub_f32(const float *A, const float *B, float *C, int n) { for (int i = 0; i < n; ++i) C[i] = A[i] - B[i]; }
void mul_f32(const float *A, const float *B, float *C, int n) { for (int i = 0; i < n; ++i) C[i] = A[i] * B[i]; }
void div_f32(const float *A, const float *B, float *C, int n) { for (int i = 0; i < n; ++i) C[i] = A[i] / B[i]; }

/* native/cpu/zilla_cpu.c:94-98 */
float sum_f32(const float *X, int n)
{
    float s = 0.0f;
    for (int i = 0; i < n; ++i) s += X[i];
    return s;
}

/* native/cpu/zilla_cpu.c:112-145: one sample [C,H,W] -> [outC,outH,outW].
 * Accumulator starts at the bias; taps in (c, kh, kw) order; padding taps
 * are skipped, not multiplied by zero. */
void conv2d_forward_f32(const float *in, const float *w, const float *bias, float *out,
                        int C, int H, int W, int outC, int kH, int kW, int stride, int pad)
{
    const int oH = (H + 2 * pad - kH) / stride + 1;
    const int oW = (W + 2 * pad - kW) / stride + 1;
    for (int oc = 0; oc < outC; ++oc)
        for (int oh = 0; oh < oH; ++oh)
            for (int ow = 0; ow < oW; ++ow) {
                float acc = bias[oc];
                for (int c = 0; c < C; ++c) {
                    const float *plane = in + (size_t)c * H * W;
                    const float *taps = w + ((size_t)oc * C + c) * kH * kW;
                    for (int kh = 0; kh < kH; ++kh) {
                        const int ih = oh * stride - pad + kh;
                        if (ih < 0 || ih >= H) continue;
                        for (int kw = 0; kw < kW; ++kw) {
                            const int iw = ow * stride - pad + kw;
                            if (iw < 0 || iw >= W) continue;
                            acc += plane[ih * W + iw] * taps[kh * kW + kw];
                        }
                    }
                }
                out[((size_t)oc * oH + oh) * oW + ow] = acc;
            }
}

/* native/cpu/zilla_cpu.c:147-195: per-sample backward.  All three outputs
 * are overwritten (zeroed first), then accumulated in (oc, oh, ow, c, kh, kw)
 * order; the bias gradient is summed in (oh, ow) order. */
void conv2d_backward_f32(const float *in, const float *w, const float *gout,
                         float *gin, float *gw, float *gb,
                         int C, int H, int W, int outC, int kH, int kW, int stride, int pad)
{
    const int oH = (H + 2 * pad - kH) / stride + 1;
    const int oW = (W + 2 * pad - kW) / stride + 1;
    memset(gin, 0, sizeof(float) * (size_t)C * H * W);
    memset(gw, 0, sizeof(float) * (size_t)outC * C * kH * kW);
    memset(gb, 0, sizeof(float) * (size_t)outC);
    for (int oc = 0; oc < outC; ++oc)
        for (int oh = 0; oh < oH; ++oh)
            for (int ow = 0; ow < oW; ++ow) {
                const float g = gout[((size_t)oc * oH + oh) * oW + ow];
                gb[oc] += g;
                for (int c = 0; c < C; ++c) {
                    const float *plane = in + (size_t)c * H * W;
                    float *gplane = gin + (size_t)c * H * W;
                    const size_t wbase = ((size_t)oc * C + c) * kH * kW;
                    for (int kh = 0; kh < kH; ++kh) {
                        const int ih = oh * stride - pad + kh;
                        if (ih < 0 || ih >= H) continue;
                        for (int kw = 0; kw < kW; ++kw) {
                            const int iw = ow * stride - pad + kw;
                            if (iw < 0 || iw >= W) continue;
                            const size_t at = (size_t)ih * W + iw;
                            gplane[at] += g * w[wbase + kh * kW + kw];
                            gw[wbase + kh * kW + kw] += g * plane[at];
                        }
                    }
                }
            }
}

/* native/cpu/zilla_cpu.c:201-232: floor output size, running max starts at
 * -1e30, strict '>' in (kh, kw) order so the first maximum wins; argmax is the
 * channel-local flat index ih*W + iw. */
void maxpool2d_forward_f32(const float *in, float *out, int *argmax,
                           int C, int H, int W, int kH, int kW, int stride)
{
    const int oH = (H - kH) / stride + 1;
    const int oW = (W - kW) / stride + 1;
    for (int c = 0; c < C; ++c) {
        const float *plane = in + (size_t)c * H * W;
        for (int oh = 0; oh < oH; ++oh)
            for (int ow = 0; ow < oW; ++ow) {
                float best = -1e30f;
                int at = 0;
                for (int kh = 0; kh < kH; ++kh)
                    for (int kw = 0; kw < kW; ++kw) {
                        const int idx = (oh * stride + kh) * W + (ow * stride + kw);
                        if (plane[idx] > best) { best = plane[idx]; at = idx; }
                    }
                const size_t o = ((size_t)c * oH + oh) * oW + ow;
                out[o] = best;
                argmax[o] = at;
            }
    }
}

/* native/cpu/zilla_cpu.c:234-251: zero, then scatter-add through argmax. */
void maxpool2d_backward_f32(const float *gout, const int *argmax, float *gin,
                            int C, int H, int W, int oH, int oW)
{
    memset(gin, 0, sizeof(float) * (size_t)C * H * W);
    for (int c = 0; c < C; ++c)
        for (int o = 0; o < oH * oW; ++o) {
            const size_t oi = (size_t)c * oH * oW + o;
            gin[(size_t)c * H * W + argmax[oi]] += gout[oi];
        }
}

/* ------------------------------------------------------------------ *
 * Handle-based training ops: native/cpu/training_ops.c:25-243 (naive paths).
 * ------------------------------------------------------------------ */

/* native/cpu/training_ops.c:25-47 (i, j, k order with a per-element sum). */
int matmul_dev(int a_id, int b_id, int c_id, int M, int K, int N)
{
    const float *A = zilla_cpu_buffer_ptr(a_id), *B = zilla_cpu_buffer_ptr(b_id);
    float *C = zilla_cpu_buffer_ptr(c_id);
    if (!A || !B || !C) return -1;
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float s = 0.0f;
            for (int k = 0; k < K; ++k) s += A[(size_t)i * K + k] * B[(size_t)k * N + j];
            C[(size_t)i * N + j] = s;
        }
    return 0;
}

/* native/cpu/training_ops.c:53-79: C[M,N] = A^T B, A stored [K,M]. */
int matmul_tn_dev(int a_id, int b_id, int c_id, int M, int K, int N)
{
    const float *A = zilla_cpu_buffer_ptr(a_id), *B = zilla_cpu_buffer_ptr(b_id);
    float *C = zilla_cpu_buffer_ptr(c_id);
    if (!A || !B || !C) return -1;
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float s = 0.0f;
            for (int k = 0; k < K; ++k) s += A[(size_t)k * M + i] * B[(size_t)k * N + j];
            C[(size_t)i * N + j] = s;
        }
    return 0;
}

/* native/cpu/training_ops.c:85-105: C[M,N] = A B^T, B stored [N,K]. */
int matmul_nt_dev(int a_id, int b_id, int c_id, int M, int K, int N)
{
    const float *A = zilla_cpu_buffer_ptr(a_id), *B = zilla_cpu_buffer_ptr(b_id);
    float *C = zilla_cpu_buffer_ptr(c_id);
    if (!A || !B || !C) return -1;
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float s = 0.0f;
            for (int k = 0; k < K; ++k) s += A[(size_t)i * K + k] * B[(size_t)j * K + k];
            C[(size_t)i * N + j] = s;
        }
    return 0;
}

/* native/cpu/training_ops.c:113-120 */
int add_bias_dev(int x_id, int b_id, int B, int C)
{
    float *X = zilla_cpu_buffer_ptr(x_id);
    const float *b = zilla_cpu_buffer_ptr(b_id);
    if (!X || !b) return -1;
    for (long i = 0; i < (long)B * C; ++i) X[i] += b[i % C];
    return 0;
}

/* native/cpu/training_ops.c:126-137: x == 0 gives y = 0 and mask = 0. */
int relu_fwd_dev(int x_id, int y_id, int mask_id, int n)
{
    const float *X = zilla_cpu_buffer_ptr(x_id);
    float *Y = zilla_cpu_buffer_ptr(y_id), *m = zilla_cpu_buffer_ptr(mask_id);
    if (!X || !Y || !m) return -1;
    for (int i = 0; i < n; ++i) {
        const int pos = X[i] > 0.0f;
        Y[i] = pos ? X[i] : 0.0f;
        m[i] = pos ? 1.0f : 0.0f;
    }
    return 0;
}

/* native/cpu/training_ops.c:143-150 */
int relu_bwd_dev(int dy_id, int mask_id, int dx_id, int n)
{
    const float *dY = zilla_cpu_buffer_ptr(dy_id), *m = zilla_cpu_buffer_ptr(mask_id);
    float *dX = zilla_cpu_buffer_ptr(dx_id);
    if (!dY || !m || !dX) return -1;
    for (int i = 0; i < n; ++i) dX[i] = dY[i] * m[i];
    return 0;
}

/* native/cpu/training_ops.c:162-206: per row max, expf, float sum, -logf of
 * the target probability summed in double and added to *loss as float;
 * dlogits = (p - onehot) / B; C > 128 is rejected with -2. */
int softmax_ce_dev(int logits_id, int targets_id, int dlogits_id, int loss_id, int B, int C)
{
    const float *Z = zilla_cpu_buffer_ptr(logits_id), *T = zilla_cpu_buffer_ptr(targets_id);
    float *D = zilla_cpu_buffer_ptr(dlogits_id), *L = zilla_cpu_buffer_ptr(loss_id);
    if (!Z || !T || !D || !L) return -1;
    double total = 0.0;
    float e[128];
    for (int i = 0; i < B; ++i) {
        const float *row = Z + (size_t)i * C;
        const int t = (int)T[i];
        float mx = row[0];
        for (int c = 1; c < C; ++c) if (row[c] > mx) mx = row[c];
        if (C > 128) return -2;
        float s = 0.0f;
        for (int c = 0; c < C; ++c) { e[c] = expf(row[c] - mx); s += e[c]; }
        total += -logf(e[t] / s);
        const float inv = 1.0f / (float)B;
        for (int c = 0; c < C; ++c)
            D[(size_t)i * C + c] = (e[c] / s - (c == t ? 1.0f : 0.0f)) * inv;
    }
    *L += (float)total;
    return 0;
}

/* native/cpu/training_ops.c:212-221: column sums in row order. */
int bias_grad_dev(int dy_id, int db_id, int B, int C)
{
    const float *dY = zilla_cpu_buffer_ptr(dy_id);
    float *db = zilla_cpu_buffer_ptr(db_id);
    if (!dY || !db) return -1;
    for (int c = 0; c < C; ++c) db[c] = 0.0f;
    for (int i = 0; i < B; ++i)
        for (int c = 0; c < C; ++c) db[c] += dY[(size_t)i * C + c];
    return 0;
}

/* native/cpu/training_ops.c:227-233 */
int sgd_update_dev(int w_id, int dw_id, float lr, int n)
{
    float *W = zilla_cpu_buffer_ptr(w_id);
    const float *dW = zilla_cpu_buffer_ptr(dw_id);
    if (!W || !dW) return -1;
    for (int i = 0; i < n; ++i) W[i] -= lr * dW[i];
    return 0;
}

/* native/cpu/training_ops.c:239-243 */
int zero_dev(int id, int n)
{
    float *X = zilla_cpu_buffer_ptr(id);
    if (!X) return -1;
    memset(X, 0, (size_t)n * sizeof(float));
    return 0;
}

/* ------------------------------------------------------------------ *
 * Pieces the reference CPU library does not have.
 * ------------------------------------------------------------------ */

/* native/cuda/training_ops.cu:282-288 */
int copy_dev(int src_id, int dst_id, int n)
{
    const float *s = zilla_cpu_buffer_ptr(src_id);
    float *d = zilla_cpu_buffer_ptr(dst_id);
    if (!s || !d) return -1;
    memmove(d, s, (size_t)n * sizeof(float));
    return 0;
}

/* src/Optim/Adam.php:36-62.  The PHP optimizer keeps m, v and the
 * parameters as doubles; here parameters, m and v live in float buffers
 * (the C-ABI's only element type) and each update is evaluated in double:
 *   m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2;
 *   theta -= lr * (m / (1-b1^t)) / (sqrt(v / (1-b2^t)) + eps)
 * with b^t from pow() as PHP's ** operator does.  t is the 1-based step. */
void oracle_adam_update(float *w, const float *g, float *m, float *v, long n,
                        double lr, double b1, double b2, double eps, int t)
{
    const double bc1 = 1.0 - pow(b1, (double)t);
    const double bc2 = 1.0 - pow(b2, (double)t);
    for (long i = 0; i < n; ++i) {
        const double gd = g[i];
        const double mi = b1 * (double)m[i] + (1.0 - b1) * gd;
        const double vi = b2 * (double)v[i] + (1.0 - b2) * gd * gd;
        m[i] = (float)mi;
        v[i] = (float)vi;
        w[i] = (float)((double)w[i] - lr * (mi / bc1) / (sqrt(vi / bc2) + eps));
    }
}

/* Batched max-pool with the GPU batched argmax convention
 * (native/cuda/pooling_batched.cu:39-52): the stored index is the flat
 * index into the whole [B,C,H,W] input.  Values and tie-breaking are those
 * of maxpool2d_forward_f32 applied per sample. */
void oracle_maxpool_batched_fwd(const float *in, float *out, int *argmax,
                                int B, int C, int H, int W, int kH, int kW, int stride)
{
    const int oH = (H - kH) / stride + 1, oW = (W - kW) / stride + 1;
    for (int b = 0; b < B; ++b) {
        const size_t ib = (size_t)b * C * H * W, ob = (size_t)b * C * oH * oW;
        maxpool2d_forward_f32(in + ib, out + ob, argmax + ob, C, H, W, kH, kW, stride);
        for (int c = 0; c < C; ++c)
            for (int o = 0; o < oH * oW; ++o)
                argmax[ob + (size_t)c * oH * oW + o] += (int)(ib + (size_t)c * H * W);
    }
}

/* native/cuda/attention.cu:31-81 restated on the CPU: max, expf, sum,
 * multiply by 1/sum. */
void oracle_softmax_rows(const float *x, float *y, int N, int M)
{
    for (int r = 0; r < N; ++r) {
        const float *a = x + (size_t)r * M;
        float *o = y + (size_t)r * M;
        float mx = -1e30f;
        for (int j = 0; j < M; ++j) if (a[j] > mx) mx = a[j];
        float s = 0.0f;
        for (int j = 0; j < M; ++j) { o[j] = expf(a[j] - mx); s += o[j]; }
        const float inv = 1.0f / s;
        for (int j = 0; j < M; ++j) o[j] *= inv;
    }
}

/* native/cuda/attention.cu:98-130: dS = P * (dP - sum_k dP*P). */
void oracle_softmax_rows_bwd(const float *P, const float *dP, float *dS, int N, int M)
{
    for (int r = 0; r < N; ++r) {
        const float *p = P + (size_t)r * M, *dp = dP + (size_t)r * M;
        float dot = 0.0f;
        for (int j = 0; j < M; ++j) dot += dp[j] * p[j];
        for (int j = 0; j < M; ++j) dS[(size_t)r * M + j] = p[j] * (dp[j] - dot);
    }
}

/* src/Loss/CrossEntropy.php:36-85: float64 softmax, mean over the batch of
 * -log(max(p, 1e-12)); gradient (p - onehot) * g / B with g = 1. */
double oracle_cross_entropy_mean(const float *logits, const int *targets, float *grad, int B, int C)
{
    double loss = 0.0;
    double *p = (double *)malloc(sizeof(double) * (size_t)C);
    for (int i = 0; i < B; ++i) {
        const float *row = logits + (size_t)i * C;
        double mx = row[0], s = 0.0;
        for (int c = 1; c < C; ++c) if (row[c] > mx) mx = row[c];
        for (int c = 0; c < C; ++c) { p[c] = exp((double)row[c] - mx); s += p[c]; }
        for (int c = 0; c < C; ++c) p[c] /= s;
        const double pt = p[targets[i]];
        loss += -log(pt > 1e-12 ? pt : 1e-12);
        if (grad)
            for (int c = 0; c < C; ++c)
                grad[(size_t)i * C + c] = (float)((p[c] - (c == targets[i] ? 1.0 : 0.0)) / B);
    }
    free(p);
    return loss / B;
}
