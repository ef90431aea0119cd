/*
 * cnn_step.c -- CPU training-step driver over ZillaPHP's CPU C-ABI.
 *
 * TEST INFRASTRUCTURE ONLY (oracle and timed CPU baseline).
 *
 * Replays the reference's batched step sequences:
 *   - MLP:  examples/mnist_cpu_v2.php:178-217
 *           (matmul_dev, add_bias_dev, relu_fwd_dev, softmax_ce_dev,
 *            matmul_tn_dev, bias_grad_dev, matmul_nt_dev, relu_bwd_dev,
 *            sgd_update_dev);
 *   - CNN:  examples/mnist_cnn_gpu_v2.php:183-264, whose batched conv/pool
 *           kernels have no CPU counterpart, so conv and pool run as the
 *           per-sample conv2d_forward_f32 / conv2d_backward_f32 /
 *           maxpool2d_forward_f32 / maxpool2d_backward_f32
 *           (native/cpu/zilla_cpu.c:112-251) looped over the batch, with
 *           weight and bias gradients summed over samples in sample order.
 *   - Adam: src/Optim/Adam.php:36-62 (restated, the reference has no native
 *           Adam).
 *
 * The same source is linked twice: against the oracle restatement
 * (zilla_oracle.c) and against the reference CPU library built from its
 * own sources.  It calls only the reference's exported names.
 *
 * Layer spec: int[4] per layer {kind, a, b, c}
 *   kind 1 conv3x3 (a = in channels, b = out channels, c = padding), stride 1
 *   kind 2 ReLU
 *   kind 3 MaxPool 2x2 stride 2
 *   kind 4 Linear  (a = in features, b = out features), W stored [in, out]
 * The last layer's output is the logits of softmax cross-entropy.
 * Parameters are one flat float array in Sequential::parameters() order
 * (src/NN/Sequential.php:32-39): [W, b] per conv/linear layer.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* reference CPU C-ABI (native/cpu/*.c) */
int zilla_cpu_buffer_alloc(size_t n_floats);
void zilla_cpu_buffer_free(int id);
float *zilla_cpu_buffer_ptr(int id);
void conv2d_forward_f32(const float *, const float *, const float *, float *,
                        int, int, int, int, int, int, int, int);
void conv2d_backward_f32(const float *, const float *, const float *, float *, float *, float *,
                         int, int, int, int, int, int, int, int);
void maxpool2d_forward_f32(const float *, float *, int *, int, int, int, int, int, int);
void maxpool2d_backward_f32(const float *, const int *, float *, int, int, int, int, int);
int matmul_dev(int, int, int, int, int, int);
int matmul_tn_dev(int, int, int, int, int, int);
int matmul_nt_dev(int, int, int, int, int, int);
int add_bias_dev(int, int, int, int);
int relu_fwd_dev(int, int, int, int);
int relu_bwd_dev(int, int, int, int);
int softmax_ce_dev(int, int, int, int, int, int);
int bias_grad_dev(int, int, int, int);
int sgd_update_dev(int, int, float, int);
int zero_dev(int, int);

#define ZO_MAX_LAYERS 32

typedef struct {
    int kind, a, b, c;
    int C, H, W;        /* input shape per sample */
    int oC, oH, oW;     /* output shape per sample */
    long in_n, out_n;   /* per-sample element counts */
    long poff, pn_w, pn_b;   /* parameter offsets / sizes */
    int out_id, mask_id, arg_id, gin_id;   /* registry handles */
    int w_id, b_id, gw_id, gb_id;          /* parameter views (registry copies) */
} zo_layer;

typedef struct {
    int nl, B, nthreads;
    zo_layer L[ZO_MAX_LAYERS];
    int x_id, y_id, loss_id, dlogit_id;
    long nparams;
    float *params, *grads, *m, *v;
    int t;
} zo_model;

static long conv_out(int n, int pad) { return n + 2 * pad - 3 + 1; }

void *zo_model_create(const int *spec, int nl, int B, int C, int H, int W, int nthreads)
{
    if (nl <= 0 || nl > ZO_MAX_LAYERS) return NULL;
    zo_model *M = (zo_model *)calloc(1, sizeof(zo_model));
    M->nl = nl;
    M->B = B;
    M->nthreads = nthreads < 1 ? 1 : nthreads;
    long poff = 0;
    for (int i = 0; i < nl; ++i) {
        zo_layer *l = &M->L[i];
        l->kind = spec[4 * i]; l->a = spec[4 * i + 1]; l->b = spec[4 * i + 2]; l->c = spec[4 * i + 3];
        l->C = C; l->H = H; l->W = W;
        l->in_n = (long)C * H * W;
        l->w_id = l->b_id = l->gw_id = l->gb_id = l->mask_id = l->arg_id = 0;
        switch (l->kind) {
        case 1:
            l->oC = l->b; l->oH = (int)conv_out(H, l->c); l->oW = (int)conv_out(W, l->c);
            l->poff = poff; l->pn_w = (long)l->b * l->a * 9; l->pn_b = l->b;
            poff += l->pn_w + l->pn_b;
            break;
        case 2:
            l->oC = C; l->oH = H; l->oW = W;
            break;
        case 3:
            l->oC = C; l->oH = (H - 2) / 2 + 1; l->oW = (W - 2) / 2 + 1;
            break;
        case 4:
            l->oC = l->b; l->oH = 1; l->oW = 1;
            l->poff = poff; l->pn_w = (long)l->a * l->b; l->pn_b = l->b;
            poff += l->pn_w + l->pn_b;
            break;
        default:
            free(M);
            return NULL;
        }
        l->out_n = (long)l->oC * l->oH * l->oW;
        C = l->oC; H = l->oH; W = l->oW;
        l->out_id = zilla_cpu_buffer_alloc((size_t)B * l->out_n);
        l->gin_id = zilla_cpu_buffer_alloc((size_t)B * l->in_n);
        if (l->kind == 2) l->mask_id = zilla_cpu_buffer_alloc((size_t)B * l->out_n);
        if (l->kind == 3) l->arg_id = zilla_cpu_buffer_alloc((size_t)B * l->out_n);
        if (l->kind == 1 || l->kind == 4) {
            l->w_id = zilla_cpu_buffer_alloc((size_t)l->pn_w);
            l->b_id = zilla_cpu_buffer_alloc((size_t)l->pn_b);
            l->gw_id = zilla_cpu_buffer_alloc((size_t)l->pn_w);
            l->gb_id = zilla_cpu_buffer_alloc((size_t)l->pn_b);
        }
    }
    M->nparams = poff;
    M->params = (float *)calloc((size_t)poff, sizeof(float));
    M->grads = (float *)calloc((size_t)poff, sizeof(float));
    M->m = (float *)calloc((size_t)poff, sizeof(float));
    M->v = (float *)calloc((size_t)poff, sizeof(float));
    M->x_id = zilla_cpu_buffer_alloc((size_t)B * M->L[0].in_n);
    M->y_id = zilla_cpu_buffer_alloc((size_t)B);
    M->loss_id = zilla_cpu_buffer_alloc(1);
    M->dlogit_id = zilla_cpu_buffer_alloc((size_t)B * M->L[nl - 1].out_n);
    return M;
}

void zo_model_destroy(void *h)
{
    zo_model *M = (zo_model *)h;
    if (!M) return;
    for (int i = 0; i < M->nl; ++i) {
        zo_layer *l = &M->L[i];
        int ids[] = {l->out_id, l->gin_id, l->mask_id, l->arg_id, l->w_id, l->b_id, l->gw_id, l->gb_id};
        for (unsigned k = 0; k < sizeof(ids) / sizeof(ids[0]); ++k) if (ids[k] > 0) zilla_cpu_buffer_free(ids[k]);
    }
    zilla_cpu_buffer_free(M->x_id);
    zilla_cpu_buffer_free(M->y_id);
    zilla_cpu_buffer_free(M->loss_id);
    zilla_cpu_buffer_free(M->dlogit_id);
    free(M->params); free(M->grads); free(M->m); free(M->v);
    free(M);
}

long zo_model_nparams(void *h) { return ((zo_model *)h)->nparams; }
float *zo_model_params(void *h) { return ((zo_model *)h)->params; }
float *zo_model_grads(void *h) { return ((zo_model *)h)->grads; }
float *zo_model_output(void *h, int layer) { return zilla_cpu_buffer_ptr(((zo_model *)h)->L[layer].out_id); }
int *zo_model_argmax(void *h, int layer) { return (int *)zilla_cpu_buffer_ptr(((zo_model *)h)->L[layer].arg_id); }
float *zo_model_dlogits(void *h) { return zilla_cpu_buffer_ptr(((zo_model *)h)->dlogit_id); }

/* ---- per-sample conv / pool over a sample range (one worker) ---- */
typedef struct {
    zo_model *M;
    zo_layer *l;
    const float *in;
    const float *gout;
    int s0, s1;
    int backward;
    float *gw, *gb;       /* private accumulators (backward) */
    float *tw, *tb;       /* per-sample scratch (backward) */
} zo_job;

static void *zo_conv_worker(void *arg)
{
    zo_job *j = (zo_job *)arg;
    zo_layer *l = j->l;
    const float *W = zilla_cpu_buffer_ptr(l->w_id), *Bs = zilla_cpu_buffer_ptr(l->b_id);
    float *out = zilla_cpu_buffer_ptr(l->out_id), *gin = zilla_cpu_buffer_ptr(l->gin_id);
    for (int s = j->s0; s < j->s1; ++s) {
        const float *xin = j->in + (size_t)s * l->in_n;
        if (!j->backward) {
            conv2d_forward_f32(xin, W, Bs, out + (size_t)s * l->out_n,
                               l->C, l->H, l->W, l->oC, 3, 3, 1, l->c);
        } else {
            conv2d_backward_f32(xin, W, j->gout + (size_t)s * l->out_n, gin + (size_t)s * l->in_n,
                                j->tw, j->tb, l->C, l->H, l->W, l->oC, 3, 3, 1, l->c);
            for (long i = 0; i < l->pn_w; ++i) j->gw[i] += j->tw[i];
            for (long i = 0; i < l->pn_b; ++i) j->gb[i] += j->tb[i];
        }
    }
    return NULL;
}

static void zo_conv(zo_model *M, zo_layer *l, const float *in, const float *gout, int backward)
{
    int nt = M->nthreads;
    if (nt > M->B) nt = M->B;
    zo_job jobs[256];
    pthread_t th[256];
    if (nt > 256) nt = 256;
    for (int t = 0; t < nt; ++t) {
        zo_job *j = &jobs[t];
        j->M = M; j->l = l; j->in = in; j->gout = gout; j->backward = backward;
        j->s0 = (int)((long)M->B * t / nt);
        j->s1 = (int)((long)M->B * (t + 1) / nt);
        j->gw = j->gb = j->tw = j->tb = NULL;
        if (backward) {
            j->gw = (float *)calloc((size_t)l->pn_w, sizeof(float));
            j->gb = (float *)calloc((size_t)l->pn_b, sizeof(float));
            j->tw = (float *)malloc(sizeof(float) * (size_t)l->pn_w);
            j->tb = (float *)malloc(sizeof(float) * (size_t)l->pn_b);
        }
    }
    if (nt == 1) {
        zo_conv_worker(&jobs[0]);
    } else {
        for (int t = 0; t < nt; ++t) pthread_create(&th[t], NULL, zo_conv_worker, &jobs[t]);
        for (int t = 0; t < nt; ++t) pthread_join(th[t], NULL);
    }
    if (backward) {
        float *gw = zilla_cpu_buffer_ptr(l->gw_id), *gb = zilla_cpu_buffer_ptr(l->gb_id);
        memset(gw, 0, sizeof(float) * (size_t)l->pn_w);
        memset(gb, 0, sizeof(float) * (size_t)l->pn_b);
        for (int t = 0; t < nt; ++t) {   /* fixed worker order: deterministic */
            for (long i = 0; i < l->pn_w; ++i) gw[i] += jobs[t].gw[i];
            for (long i = 0; i < l->pn_b; ++i) gb[i] += jobs[t].gb[i];
            free(jobs[t].gw); free(jobs[t].gb); free(jobs[t].tw); free(jobs[t].tb);
        }
    }
}

/* Adam restated from src/Optim/Adam.php:36-62 (same formula as the oracle). */
static void zo_adam(float *w, const float *g, float *m, float *v, long n,
                    double lr, double b1, double b2, double eps, int t)
{
    const double bc1 = 1.0 - pow(b1, (double)t), bc2 = 1.0 - pow(b2, (double)t);
    for (long i = 0; i < n; ++i) {
        const double gd = g[i];
        const double mi = b1 * (double)m[i] + (1.0 - b1) * gd;
        const double vi = b2 * (double)v[i] + (1.0 - b2) * gd * gd;
        m[i] = (float)mi;
        v[i] = (float)vi;
        w[i] = (float)((double)w[i] - lr * (mi / bc1) / (sqrt(vi / bc2) + eps));
    }
}

/*
 * One training step.  x: [B, in_n] floats, y: [B] float-coded labels.
 * opt: 0 = none (gradients only), 1 = SGD (sgd_update_dev), 2 = Adam.
 * *loss_sum receives the softmax_ce_dev loss buffer (a sum over rows).
 * Returns 0 on success.
 */
int zo_model_step(void *h, const float *x, const float *y, int opt, float lr, float *loss_sum)
{
    zo_model *M = (zo_model *)h;
    const int B = M->B, nl = M->nl;
    memcpy(zilla_cpu_buffer_ptr(M->x_id), x, sizeof(float) * (size_t)B * M->L[0].in_n);
    memcpy(zilla_cpu_buffer_ptr(M->y_id), y, sizeof(float) * (size_t)B);
    for (int i = 0; i < nl; ++i) {
        zo_layer *l = &M->L[i];
        if (l->kind == 1 || l->kind == 4) {
            memcpy(zilla_cpu_buffer_ptr(l->w_id), M->params + l->poff, sizeof(float) * (size_t)l->pn_w);
            memcpy(zilla_cpu_buffer_ptr(l->b_id), M->params + l->poff + l->pn_w, sizeof(float) * (size_t)l->pn_b);
        }
    }
    /* forward */
    int in_id = M->x_id;
    for (int i = 0; i < nl; ++i) {
        zo_layer *l = &M->L[i];
        const float *in = zilla_cpu_buffer_ptr(in_id);
        switch (l->kind) {
        case 1: zo_conv(M, l, in, NULL, 0); break;
        case 2: if (relu_fwd_dev(in_id, l->out_id, l->mask_id, (int)(B * l->out_n))) return -1; break;
        case 3:
            for (int s = 0; s < B; ++s)
                maxpool2d_forward_f32(in + (size_t)s * l->in_n, zilla_cpu_buffer_ptr(l->out_id) + (size_t)s * l->out_n,
                                      (int *)zilla_cpu_buffer_ptr(l->arg_id) + (size_t)s * l->out_n,
                                      l->C, l->H, l->W, 2, 2, 2);
            break;
        case 4:
            if (matmul_dev(in_id, l->w_id, l->out_id, B, l->a, l->b)) return -1;
            if (add_bias_dev(l->out_id, l->b_id, B, l->b)) return -1;
            break;
        }
        in_id = l->out_id;
    }
    zo_layer *last = &M->L[nl - 1];
    if (zero_dev(M->loss_id, 1)) return -1;
    int rc = softmax_ce_dev(last->out_id, M->y_id, M->dlogit_id, M->loss_id, B, (int)last->out_n);
    if (rc) return rc;
    if (loss_sum) *loss_sum = zilla_cpu_buffer_ptr(M->loss_id)[0];

    /* backward */
    int g_id = M->dlogit_id;
    for (int i = nl - 1; i >= 0; --i) {
        zo_layer *l = &M->L[i];
        const int prev_id = (i == 0) ? M->x_id : M->L[i - 1].out_id;
        switch (l->kind) {
        case 1:
            zo_conv(M, l, zilla_cpu_buffer_ptr(prev_id), zilla_cpu_buffer_ptr(g_id), 1);
            break;
        case 2:
            if (relu_bwd_dev(g_id, l->mask_id, l->gin_id, (int)(B * l->in_n))) return -1;
            break;
        case 3:
            for (int s = 0; s < B; ++s)
                maxpool2d_backward_f32(zilla_cpu_buffer_ptr(g_id) + (size_t)s * l->out_n,
                                       (const int *)zilla_cpu_buffer_ptr(l->arg_id) + (size_t)s * l->out_n,
                                       zilla_cpu_buffer_ptr(l->gin_id) + (size_t)s * l->in_n,
                                       l->C, l->H, l->W, l->oH, l->oW);
            break;
        case 4:
            if (matmul_tn_dev(prev_id, g_id, l->gw_id, l->a, B, l->b)) return -1;
            if (bias_grad_dev(g_id, l->gb_id, B, l->b)) return -1;
            if (matmul_nt_dev(g_id, l->w_id, l->gin_id, B, l->b, l->a)) return -1;
            break;
        }
        g_id = l->gin_id;
    }
    /* gather gradients, update */
    M->t += 1;
    for (int i = 0; i < nl; ++i) {
        zo_layer *l = &M->L[i];
        if (l->kind != 1 && l->kind != 4) continue;
        memcpy(M->grads + l->poff, zilla_cpu_buffer_ptr(l->gw_id), sizeof(float) * (size_t)l->pn_w);
        memcpy(M->grads + l->poff + l->pn_w, zilla_cpu_buffer_ptr(l->gb_id), sizeof(float) * (size_t)l->pn_b);
        if (opt == 1) {
            if (sgd_update_dev(l->w_id, l->gw_id, lr, (int)l->pn_w)) return -1;
            if (sgd_update_dev(l->b_id, l->gb_id, lr, (int)l->pn_b)) return -1;
            memcpy(M->params + l->poff, zilla_cpu_buffer_ptr(l->w_id), sizeof(float) * (size_t)l->pn_w);
            memcpy(M->params + l->poff + l->pn_w, zilla_cpu_buffer_ptr(l->b_id), sizeof(float) * (size_t)l->pn_b);
        }
    }
    if (opt == 2)
        zo_adam(M->params, M->grads, M->m, M->v, M->nparams, lr, 0.9, 0.999, 1e-8, M->t);
    return 0;
}
