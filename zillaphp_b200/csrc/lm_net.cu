// lm_net.cu -- the fused training step of ZillaPHP's decoder-only Transformer
// language model (fp32, CUDA cores): one C call per step for
// TransformerLM::forwardBatch + the autograd backward + the optimizer
// (src/Transformers/TransformerLM.php:77-116, TransformerBlock.php:28-33,
// src/Attention/MultiHeadAttention.php:41-80, src/NN/Layers/FeedForward.php,
// src/Tensor/Tensor.php:636-735 LayerNorm, src/NN/Layers/Embedding.php:35-56).
//
// Rows are the B*T tokens of the batch.  Per block (pre-LN):
//   h1 = LN1(x); [q|k|v] = h1 [Wq|Wk|Wv] + [bq|bk|bv]  (one GEMM, N = 3D)
//   per (sequence, head): P = softmax(maskfill(q k^T / sqrt(dh), -1e9 on future keys)); o = P v
//   xm = x + o Wo + bo                                  (residual fused in the GEMM store)
//   h2 = LN2(xm); f = relu(h2 W1 + b1); x' = xm + f W2 + b2
// then hf = LNf(x), logits = hf Wh + bh, softmax cross-entropy (softmax_ce_dev
// semantics: loss sum, dlogits / rows).  Attention runs per sequence: the
// reference's block-diagonal batch mask only adds -1e9 entries, whose softmax
// weight is exactly zero.  Every reduction has a fixed order (deterministic).
#include <math.h>
#include <string.h>

#include <vector>

#include "conv_pool_f32.cuh"
#include "net.cuh"
#include "tc_attn_tf32.cuh"
#include "tc_gemm_tf32.cuh"

namespace zb {

// One Linear GEMM of the tensor-core step (precision 1): its TF32 tcgen05
// problem, built once per net over the persistent activations and weights.
//   kind 0 forward      Y = X W (+ b) (+ R) (relu)     A K-major, B MN-major
//   kind 1 input grad   dX = dY W^T                    A K-major, B K-major
//   kind 2 input grad   dX = (dY W^T) * (mask > 0)     (ReLU backward)
//   kind 3 weight grad  dW = X^T dY, K split; the splits are summed in order
//                       into dst[n / seg_w][m * seg_w + n % seg_w]
struct LmTcGemm {
    tc::GemmTf32Params p;
    int kind = 0, grid = 0;
    float *dst[3] = {nullptr, nullptr, nullptr};
    int seg_w = 0;
};

int launch_softmax_ce(const float *z, const float *y, float *dz, double *row_loss, float *loss,
                      int B, int C, bool zero_first);

// The step's split sums, deferred: every weight-gradient K split (tensor-core path), bias
// column sum, LayerNorm parameter sum and embedding sum of the backward is queued as a job,
// and the jobs run together in one launch at the end of the step, before the optimizer reads
// the gradients.  Job: element i = m * N + n (i < M * N) is the sum over k < splits of
// partial[k * stride + i], in a fixed order, stored to o[n / sw][m * sw + n % sw]; elements
// i >= nvalid are stored as zero.
constexpr int kMaxLmRed = 40;
struct LmRedJob {
    const float *partial;
    long long stride, nvalid;
    int splits, M, N, sw;
    int vec;   // 16-byte loads: M * N, stride and nvalid multiples of 4, partial 16-byte aligned, sw % 4 == 0
    float *o[3];
};
struct LmRedJobs {
    LmRedJob j[kMaxLmRed];
    int start[kMaxLmRed + 1];
    int count;
};

struct LmEngine {
    int V = 0, D = 0, H = 0, L = 0, T = 0, F = 0, Bs = 0, Ts = 0, N = 0;
    long long o_tok = 0, o_pos = 0, o_lnf_g = 0, o_lnf_b = 0, o_head_W = 0, o_head_b = 0;
    struct Blk {
        long long qW, qb, kW, kb, vW, vb, oW, ob, f1W, f1b, f2W, f2b, ln1g, ln1b, ln2g, ln2b;
    };
    std::vector<Blk> blk;
    // saved forward tensors (per block) and the final ones
    std::vector<float *> x, h1, xh1, inv1, qkv, P, att, xm, h2, xh2, inv2, f1;
    float *hf = nullptr, *xhf = nullptr, *invf = nullptr, *logits = nullptr;
    // gradients
    float *g = nullptr, *gm = nullptr, *dh = nullptr, *df1 = nullptr, *datt = nullptr, *dqkv = nullptr;
    float *emb_partial = nullptr;  // [row chunks][V][D]
    int ln_blocks = 0;
    // generation (TransformerLM::forwardWithCache): per-layer K/V caches
    // [max_seq][D] and buffers for up to max_seq new rows, made on first use
    std::vector<float *> kc, vc;
    float *gx = nullptr, *gxm = nullptr, *gh = nullptr, *gxh = nullptr, *ginv = nullptr, *gqkv = nullptr,
          *gatt = nullptr, *gf1 = nullptr, *glog = nullptr, *gtok = nullptr;
    int cache_len = 0;
    // tensor-core GEMMs (precision 1), per block: 0 qkv, 1 out proj, 2 fc1, 3 fc2 (forward);
    // 4 fc2 dX, 5 fc1 dX, 6 out dX, 7 qkv dX; 8 fc2 dW, 9 fc1 dW, 10 out dW, 11 qkv dW
    std::vector<LmTcGemm> tcg;
    float *tc_partial = nullptr;   // weight-gradient split partials
    const float *tc_params = nullptr, *tc_grads = nullptr;   // the buffers the plan was built over
    // The flat parameter layout (TransformerLM::parameters() order) puts the blocks' tensors at
    // arbitrary float offsets; TMA and the 16-byte bias loads need 16-byte-aligned bases, so each
    // step first copies the blocks' weights and biases into a shadow with every tensor aligned.
    float *tc_shadow = nullptr;
    std::vector<long long> shadow_src, shadow_dst, shadow_len;
    // attention on TF32 tensor cores (precision 1, head dim 32, sequence <= 128): per block
    // the forward and backward problems and the score rows' max and exp-sum [B*H][T][2]
    std::vector<tc::AttnTcParams> attn_f, attn_b;
    std::vector<float *> attn_stats;
    // deferred split sums: the queue of this step and the scratch of the column-sum and
    // LayerNorm partials (a fresh region per call, reset every step)
    std::vector<LmRedJob> red;
    float *red_arena = nullptr;
    size_t red_cap = 0, red_used = 0;
    std::vector<void *> allocs;
};
constexpr int kLmTcPerBlock = 12;
constexpr int kColsumChunks = 296;   // row chunks of the two-stage column sums

namespace {

// ---------------------------------------------------------------- GEMM problems
// Segment s of a 3-way operand list, by selects (a runtime index into the
// parameter arrays would copy them to local memory).  Columns span at most
// three segments of width sw, so s = (c >= sw) + (c >= 2 sw) needs no division.
__device__ __forceinline__ const float *seg3(const float *const (&p)[3], int s) {
    return s == 0 ? p[0] : s == 1 ? p[1] : p[2];
}
__device__ __forceinline__ float *seg3(float *const (&p)[3], int s) { return s == 0 ? p[0] : s == 1 ? p[1] : p[2]; }

// Y[m, n] = sum_k X[m*ldx + k] W_s[k*sw + (n - s*sw)] + b_s[n - s*sw]  (s = n / sw)
//           [+ R[m*ldy + n]] [relu]
struct LinFwd {
    const float *X, *R;
    const float *W[3], *Bv[3];
    float *Y;
    int M, N, K, ldx, ldy, sw;
    bool relu;
    static constexpr bool kAMFast = false, kBNFast = true, kExactOrder = false;
    __device__ float init(int, int) const { return 0.0f; }
    __device__ float a(int m, int k) const { return X[(size_t)m * ldx + k]; }
    __device__ float b(int k, int n) const { const int s = (n >= sw) + (n >= 2 * sw); return seg3(W, s)[(size_t)k * sw + (n - s * sw)]; }
    __device__ void store(int m, int n, float v) const {
        const int s = (n >= sw) + (n >= 2 * sw);
        float o = v + seg3(Bv, s)[n - s * sw];
        if (R) o += R[(size_t)m * ldy + n];
        if (relu) o = o > 0.0f ? o : 0.0f;
        Y[(size_t)m * ldy + n] = o;
    }
};

// dX[m, j] = sum_n dY[m*ldy + n] W_s[j*sw + (n - s*sw)]  [* (mask[m*ldx + j] > 0)]
struct LinDgrad {
    const float *dY, *mask;
    const float *W[3];
    float *dX;
    int M, N, K, ldx, ldy, sw;   // N = in features, K = out features (all segments)
    static constexpr bool kAMFast = false, kBNFast = false, kExactOrder = false;
    __device__ float init(int, int) const { return 0.0f; }
    __device__ float a(int m, int k) const { return dY[(size_t)m * ldy + k]; }
    __device__ float b(int k, int n) const { const int s = (k >= sw) + (k >= 2 * sw); return seg3(W, s)[(size_t)n * sw + (k - s * sw)]; }
    __device__ void store(int m, int n, float v) const {
        const size_t at = (size_t)m * ldx + n;
        if (mask && !(mask[at] > 0.0f)) v = 0.0f;
        dX[at] = v;
    }
};

// dW_s[j*sw + (n - s*sw)] = sum_m X[m*ldx + j] dY[m*ldy + n]   (M = in, N = out, K = rows)
struct LinWgrad {
    const float *X, *dY;
    float *dW[3];
    int M, N, K, ldx, ldy, sw;
    static constexpr bool kAMFast = true, kBNFast = true, kExactOrder = false;
    __device__ float init(int, int) const { return 0.0f; }
    __device__ float a(int m, int k) const { return X[(size_t)k * ldx + m]; }
    __device__ float b(int k, int n) const { return dY[(size_t)k * ldy + n]; }
    __device__ void store(int m, int n, float v) const {
        const int s = (n >= sw) + (n >= 2 * sw);
        seg3(dW, s)[(size_t)m * sw + (n - s * sw)] = v;
    }
};

// ---------------------------------------------------------------- kernels
__global__ void embed_fwd_kernel(const float *__restrict__ tokens, const float *__restrict__ tok,
                                 const float *__restrict__ pos, float *__restrict__ x, int N, int Ts, int D, int V,
                                 int *__restrict__ err, int pos0 = 0) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)N * D;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / D), d = (int)(i % D);
        int id = (int)tokens[r];
        if (id < 0 || id >= V) {   // Embedding::forward throws OutOfRange; record and use row 0
            if (err) atomicCAS(err, 0, 0x454d4244);   // "EMBD"
            id = 0;
        }
        x[i] = tok[(size_t)id * D + d] + pos[(size_t)(pos0 + r % Ts) * D + d];
    }
}

// LayerNorm forward, one warp per row (D a multiple of 32, <= 1024):
// mean, biased variance, invstd = 1/sqrt(var + eps); y = xhat*g + b.
__global__ void ln_fwd_kernel(const float *__restrict__ x, const float *__restrict__ gam,
                              const float *__restrict__ bet, float *__restrict__ y, float *__restrict__ xhat,
                              float *__restrict__ inv, int N, int D, float eps) {
    const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < N; r += gridDim.x * warps) {
        const float *xr = x + (size_t)r * D;
        float s = 0.0f;
        for (int j = lane; j < D; j += 32) s += xr[j];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mean = s / D;
        float q = 0.0f;
        for (int j = lane; j < D; j += 32) { const float d0 = xr[j] - mean; q += d0 * d0; }
#pragma unroll
        for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        const float is = 1.0f / sqrtf(q / D + eps);
        for (int j = lane; j < D; j += 32) {
            const float xh = (xr[j] - mean) * is;
            xhat[(size_t)r * D + j] = xh;
            y[(size_t)r * D + j] = xh * gam[j] + bet[j];
        }
        if (lane == 0) inv[r] = is;
    }
}

// LayerNorm backward (src/Tensor/Tensor.php:691-712): gx = g*gamma,
// dx = inv/D (D gx - sum gx - xhat sum(gx xhat)); out = R + dx.  Per-block
// partial sums of g*xhat (dgamma) and g (dbeta), warps combined in order.
__global__ void ln_bwd_kernel(const float *__restrict__ gout, const float *__restrict__ xhat,
                              const float *__restrict__ inv, const float *__restrict__ gam,
                              const float *__restrict__ R, float *__restrict__ out,
                              float *__restrict__ partial, int N, int D) {
    extern __shared__ float red[];   // [warps][2D]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    float *mine = red + (size_t)warp * 2 * D;
    for (int j = lane; j < 2 * D; j += 32) mine[j] = 0.0f;
    __syncwarp();
    for (int r = blockIdx.x * warps + warp; r < N; r += gridDim.x * warps) {
        const float *g = gout + (size_t)r * D, *xh = xhat + (size_t)r * D;
        float s1 = 0.0f, s2 = 0.0f;
        for (int j = lane; j < D; j += 32) {
            const float gx = g[j] * gam[j];
            s1 += gx;
            s2 += gx * xh[j];
            mine[j] += g[j] * xh[j];
            mine[D + j] += g[j];
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
        const float is = inv[r];
        for (int j = lane; j < D; j += 32) {
            const float gx = g[j] * gam[j];
            float d = is / D * (D * gx - s1 - xh[j] * s2);
            if (R) d += R[(size_t)r * D + j];
            out[(size_t)r * D + j] = d;
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < 2 * D; j += blockDim.x) {
        float s = 0.0f;
        for (int w = 0; w < warps; ++w) s += red[(size_t)w * 2 * D + j];
        partial[(size_t)blockIdx.x * 2 * D + j] = s;
    }
}

// ln_bwd_kernel for D = 32 KD: lane l keeps columns l + 32 k (k < KD) of gamma and
// of its warp's dgamma / dbeta sums in registers, and loads the next row's g, xhat
// and R while it finishes the current one.  Same arithmetic and order as above.
template <int KD>
__global__ void __launch_bounds__(256) ln_bwd_reg_kernel(const float *__restrict__ gout, const float *__restrict__ xhat,
                                                         const float *__restrict__ inv, const float *__restrict__ gam,
                                                         const float *__restrict__ R, float *__restrict__ out,
                                                         float *__restrict__ partial, int N) {
    constexpr int D = 32 * KD;
    __shared__ float red[8][2 * D];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float gm[KD], dgam[KD], dbet[KD];
#pragma unroll
    for (int k = 0; k < KD; ++k) { gm[k] = gam[lane + 32 * k]; dgam[k] = 0.0f; dbet[k] = 0.0f; }
    const int stride = gridDim.x * 8;
    int r = blockIdx.x * 8 + warp;
    float g[KD], xh[KD], rr[KD], iv = 0.0f;
    auto load = [&](int row) {
        iv = inv[row];
#pragma unroll
        for (int k = 0; k < KD; ++k) {
            g[k] = __ldcs(gout + (size_t)row * D + lane + 32 * k);
            xh[k] = __ldcs(xhat + (size_t)row * D + lane + 32 * k);
            rr[k] = R ? __ldcs(R + (size_t)row * D + lane + 32 * k) : 0.0f;
        }
    };
    if (r < N) load(r);
    for (; r < N; r += stride) {
        float cg[KD], cx[KD], cr[KD];
#pragma unroll
        for (int k = 0; k < KD; ++k) { cg[k] = g[k]; cx[k] = xh[k]; cr[k] = rr[k]; }
        const float is = iv;
        if (r + stride < N) load(r + stride);
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int k = 0; k < KD; ++k) {
            const float gx = cg[k] * gm[k];
            s1 += gx;
            s2 += gx * cx[k];
            dgam[k] += cg[k] * cx[k];
            dbet[k] += cg[k];
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
#pragma unroll
        for (int k = 0; k < KD; ++k) {
            const float gx = cg[k] * gm[k];
            float d = is / D * (D * gx - s1 - cx[k] * s2);
            if (R) d += cr[k];
            out[(size_t)r * D + lane + 32 * k] = d;
        }
    }
#pragma unroll
    for (int k = 0; k < KD; ++k) { red[warp][lane + 32 * k] = dgam[k]; red[warp][D + lane + 32 * k] = dbet[k]; }
    __syncthreads();
    for (int j = threadIdx.x; j < 2 * D; j += blockDim.x) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) s += red[w][j];
        partial[(size_t)blockIdx.x * 2 * D + j] = s;
    }
}

// Column sums over rows with a row stride, first stage: block (column tile, row chunk)
// sums rows [r0, r1) of 128 (or 32) columns (8 row lanes, combined in order) into
// part[chunk][col]; the step's deferred sums add the chunks in order.
template <bool VEC>
__global__ void __launch_bounds__(256) colsum_part_kernel(const float *__restrict__ dY, int rows, int ld, int chunks,
                                                          float *__restrict__ part) {
    // VEC: lane x takes 4 consecutive columns (one 16-byte load per row), a block 128
    // columns; else one column per lane, 32 per block.  Row lane y adds rows r0 + y,
    // r0 + y + 8, ... in order, four loads in flight; the 8 row lanes are then added
    // in order (fixed order: deterministic).
    constexpr int PER = VEC ? 4 : 1;
    __shared__ float red[8][32 * PER + 1];
    const int col = (blockIdx.x * 32 + threadIdx.x) * PER;
    const int r0 = (int)((long long)rows * blockIdx.y / chunks), r1 = (int)((long long)rows * (blockIdx.y + 1) / chunks);
    float acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.0f;
    if (col < ld) {
        int r = r0 + threadIdx.y;
        for (; r + 24 < r1; r += 32) {
            float v[4][PER];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float *src = dY + (size_t)(r + 8 * u) * ld + col;
                if constexpr (VEC) {
                    const float4 q = __ldcs(reinterpret_cast<const float4 *>(src));
                    v[u][0] = q.x; v[u][1 % PER] = q.y; v[u][2 % PER] = q.z; v[u][3 % PER] = q.w;
                } else {
                    v[u][0] = __ldcs(src);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int e = 0; e < PER; ++e) acc[e] += v[u][e];
        }
        for (; r < r1; r += 8) {
            const float *src = dY + (size_t)r * ld + col;
            if constexpr (VEC) {
                const float4 q = __ldcs(reinterpret_cast<const float4 *>(src));
                acc[0] += q.x; acc[1 % PER] += q.y; acc[2 % PER] += q.z; acc[3 % PER] += q.w;
            } else {
                acc[0] += __ldcs(src);
            }
        }
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) red[threadIdx.y][threadIdx.x * PER + e] = acc[e];
    __syncthreads();
    const int t = threadIdx.y * 32 + threadIdx.x;   // one output column per thread
    if (t < 32 * PER) {
        const int c = blockIdx.x * 32 * PER + t;
        if (c < ld) {
            float s = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; ++k) s += red[k][t];
            part[(size_t)blockIdx.y * ld + c] = s;
        }
    }
}


// Causal attention forward for one (sequence, head, block of 32 query rows),
// head dim DH: S = q k^T * scale with -1e9 on future keys, P = row softmax
// (written out for the backward), o = P v into the head's columns.  Scores and
// o are 4 x 4 register tiles of one thread (float4 shared-memory rows: 8 loads
// per 64 FMAs for the scores); keys after the block's last query row are never
// used.  Shared memory: K, V [Tp][DH + 4], Q [32][DH + 4], S [32][Tp + 4].
template <int DH>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const float *__restrict__ qkv, float *__restrict__ P,
                                                       float *__restrict__ out, int Ts, int H, int D, float scale) {
    static_assert(DH == 32, "head dimension 32: 8 column tiles of 4");
    extern __shared__ __align__(16) float sm[];
    const int bh = blockIdx.x, b = bh / H, h = bh % H;
    const int i0 = blockIdx.y * 32;
    const int rows = min(32, Ts - i0);
    const int keys = min(Ts, i0 + 32);   // causal: keys after the last query row are never used
    const int kp = (keys + 3) & ~3;      // keys rounded up to a tile of 4 (zero rows past `keys`)
    const int Tp = (Ts + 3) & ~3, LD = DH + 4, SP = Tp + 4;
    float *Ks = sm, *Vs = Ks + (size_t)Tp * LD, *Qs = Vs + (size_t)Tp * LD, *S = Qs + 32 * LD;
    const size_t ld = 3 * (size_t)D;
    const float *base = qkv + (size_t)b * Ts * ld + h * DH;
    for (int i = threadIdx.x; i < kp * DH; i += blockDim.x) {
        const int j = i / DH, d = i % DH;
        const bool in = j < keys;
        Ks[j * LD + d] = in ? base[(size_t)j * ld + D + d] : 0.0f;
        Vs[j * LD + d] = in ? base[(size_t)j * ld + 2 * D + d] : 0.0f;
    }
    for (int i = threadIdx.x; i < 32 * DH; i += blockDim.x) {
        const int r = i / DH, d = i % DH;
        Qs[r * LD + d] = r < rows ? base[(size_t)(i0 + r) * ld + d] : 0.0f;
    }
    __syncthreads();
    // scores: tile (4 rows, 4 keys), 8 row tiles x kp / 4 key tiles
    const int kt = kp / 4;
    for (int t = threadIdx.x; t < 8 * kt; t += blockDim.x) {
        const int r0 = 4 * (t % 8), j0 = 4 * (t / 8);
        float acc[4][4] = {};
#pragma unroll
        for (int d = 0; d < DH; d += 4) {
            float4 qr[4], kr[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                qr[a] = *reinterpret_cast<const float4 *>(Qs + (r0 + a) * LD + d);
                kr[a] = *reinterpret_cast<const float4 *>(Ks + (j0 + a) * LD + d);
            }
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    acc[a][c] += qr[a].x * kr[c].x + qr[a].y * kr[c].y + qr[a].z * kr[c].z + qr[a].w * kr[c].w;
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) v[c] = (j0 + c > i0 + r0 + a) ? -1e9f : acc[a][c] * scale;   // maskedFill(-1e9)
            *reinterpret_cast<float4 *>(S + (r0 + a) * SP + j0) = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int r = warp; r < rows; r += 4) {
        float mx = -INFINITY;
        for (int j = lane; j < keys; j += 32) mx = fmaxf(mx, S[r * SP + j]);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
        for (int j = lane; j < keys; j += 32) {
            const float e = expf(S[r * SP + j] - mx);
            S[r * SP + j] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        float *prow = P + ((size_t)bh * Ts + i0 + r) * Ts;
        for (int j = lane; j < Ts; j += 32) {
            const float p = j < keys ? S[r * SP + j] / sum : 0.0f;
            if (j < kp) S[r * SP + j] = p;   // zero past `keys`: the o tiles read up to kp
            prow[j] = p;
        }
    }
    // rows of the block past Ts (the last block of a ragged length): zero, so o reads finite values
    for (int i = threadIdx.x; i < (32 - rows) * kp; i += blockDim.x) S[(rows + i / kp) * SP + i % kp] = 0.0f;
    __syncthreads();
    // o[r][d] = sum_j P[r][j] v[j][d]: tile (4 rows, 4 d), 8 x 8 tiles
    for (int t = threadIdx.x; t < 64; t += blockDim.x) {
        const int r0 = 4 * (t % 8), d0 = 4 * (t / 8);
        float acc[4][4] = {};
        const int jend = min(kp, i0 + r0 + 4);   // causal: P is zero past each row's own position
        for (int j = 0; j < jend; ++j) {
            const float4 vv = *reinterpret_cast<const float4 *>(Vs + j * LD + d0);
            const float vr[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const float pv = S[(r0 + a) * SP + j];
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[a][c] = fmaf(pv, vr[c], acc[a][c]);
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
            if (r0 + a < rows)
                *reinterpret_cast<float4 *>(out + ((size_t)b * Ts + i0 + r0 + a) * D + h * DH + d0) =
                    make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    }
}

// Generation: append the new rows' K and V (columns D..3D of qkv [rows][3D])
// to one layer's caches [max_seq][D] at row `at` (Tensor::concatAlongRows of
// MultiHeadAttention::forwardWithCache, src/Attention/MultiHeadAttention.php:105-112).
__global__ void kv_append_kernel(const float *__restrict__ qkv, float *__restrict__ kc, float *__restrict__ vc,
                                 int rows, int D, int at) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows * D; i += gridDim.x * blockDim.x) {
        const int r = i / D, d = i % D;
        kc[(size_t)(at + r) * D + d] = qkv[(size_t)r * 3 * D + D + d];
        vc[(size_t)(at + r) * D + d] = qkv[(size_t)r * 3 * D + 2 * D + d];
    }
}

// Generation attention for one (head, new row): scores against all `len`
// cached keys, scaled by 1/sqrt(dh), row softmax, times the cached values --
// attendHeadCached (src/Attention/MultiHeadAttention.php:127-137) applies NO
// causal mask, so the rows of a multi-token prompt see each other both ways.
// Shared memory: the len scores, 4 warps' partial outputs, the query row.
// Fixed reduction order (deterministic).
template <int DH>
__global__ void __launch_bounds__(128) attn_cached_kernel(const float *__restrict__ qkv, const float *__restrict__ kc,
                                                          const float *__restrict__ vc, float *__restrict__ out,
                                                          int len, int D, float scale) {
    extern __shared__ float sm[];
    float *qs = sm, *part = qs + DH, *red = part + 4 * DH, *S = red + 8;
    const int h = blockIdx.x, r = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x < DH) qs[threadIdx.x] = qkv[(size_t)r * 3 * D + h * DH + threadIdx.x];
    __syncthreads();
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < len; j += blockDim.x) {
        const float4 *k = reinterpret_cast<const float4 *>(kc + (size_t)j * D + h * DH);
        float s = 0.0f;
#pragma unroll
        for (int c = 0; c < DH / 4; ++c) {
            const float4 kv = k[c];
            s += qs[4 * c] * kv.x;
            s += qs[4 * c + 1] * kv.y;
            s += qs[4 * c + 2] * kv.z;
            s += qs[4 * c + 3] * kv.w;
        }
        s *= scale;
        S[j] = s;
        mx = fmaxf(mx, s);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    float sum = 0.0f;
    for (int j = threadIdx.x; j < len; j += blockDim.x) {
        const float e = expf(S[j] - mx);
        S[j] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[4 + warp] = sum;
    __syncthreads();
    sum = (red[4] + red[5]) + (red[6] + red[7]);
    // o[d] = sum_j p_j v[j][d]: warp w takes keys w, w+4, ..., lane = d
    for (int d0 = 0; d0 < DH; d0 += 32) {
        float acc = 0.0f;
        if (d0 + lane < DH)
            for (int j = warp; j < len; j += 4) acc += (S[j] / sum) * vc[(size_t)j * D + h * DH + d0 + lane];
        if (d0 + lane < DH) part[warp * DH + d0 + lane] = acc;
    }
    __syncthreads();
    if (threadIdx.x < DH)
        out[(size_t)r * D + h * DH + threadIdx.x] =
            (part[threadIdx.x] + part[DH + threadIdx.x]) + (part[2 * DH + threadIdx.x] + part[3 * DH + threadIdx.x]);
}

// Attention backward for one (sequence, head):
//   dV = P^T dO;  dP = dO V^T;  dS = P (dP - Dr) * scale  with Dr[r] = sum_j P[r][j] dP[r][j]
//   (softmax and maskedFill backward: masked entries have P = 0);  dQ = dS K;  dK = dS^T Q.
// Dr = dO[r] . O[r], O = P V the forward's output of this head (the same sum regrouped), so
// no row reduction across threads is needed.  Every product is a 4 x 4 register tile of one
// thread (float4 shared-memory reads along rows: 8 loads per 16 FMAs); only the causal lower
// triangle of dS is computed (P is zero above the diagonal, so is dS).  Shared memory: Q, K,
// V, dO [Tp][DH + 4] (Tp = Ts rounded up to 4, zero rows past Ts) and P / dS [Tp][Tp + 4].
template <int DH>
__global__ void __launch_bounds__(256) attn_bwd_kernel(const float *__restrict__ qkv, const float *__restrict__ P,
                                                       const float *__restrict__ dO, const float *__restrict__ O,
                                                       float *__restrict__ dqkv, int Ts, int H, int D, float scale) {
    static_assert(DH == 32, "head dimension 32: 8 column tiles of 4");
    extern __shared__ __align__(16) float sm[];
    const int bh = blockIdx.x, b = bh / H, h = bh % H;
    const int Tp = (Ts + 3) & ~3, LD = DH + 4, SP = Tp + 4;
    float *Qs = sm, *Ks = Qs + Tp * LD, *Vs = Ks + Tp * LD, *Gs = Vs + Tp * LD, *S = Gs + Tp * LD;
    float *Dr = S + Tp * SP;   // [Tp]
    const size_t ld = 3 * (size_t)D;
    const float *base = qkv + (size_t)b * Ts * ld + h * DH;
    for (int i = threadIdx.x; i < Tp * DH; i += blockDim.x) {
        const int j = i / DH, d = i % DH;
        const bool in = j < Ts;
        Qs[j * LD + d] = in ? base[(size_t)j * ld + d] : 0.0f;
        Ks[j * LD + d] = in ? base[(size_t)j * ld + D + d] : 0.0f;
        Vs[j * LD + d] = in ? base[(size_t)j * ld + 2 * D + d] : 0.0f;
        Gs[j * LD + d] = in ? dO[((size_t)b * Ts + j) * D + h * DH + d] : 0.0f;
    }
    const float *Pb = P + (size_t)bh * Ts * Ts;
    for (int i = threadIdx.x; i < Tp * Tp; i += blockDim.x) {
        const int r = i / Tp, c = i % Tp;
        S[r * SP + c] = (r < Ts && c <= r) ? Pb[(size_t)r * Ts + c] : 0.0f;
    }
    {   // Dr[r] = dO[r] . O[r], one warp per row
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        for (int r = warp; r < Tp; r += blockDim.x >> 5) {
            float t = r < Ts ? dO[((size_t)b * Ts + r) * D + h * DH + lane] * O[((size_t)b * Ts + r) * D + h * DH + lane]
                             : 0.0f;
#pragma unroll
            for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
            if (lane == 0) Dr[r] = t;
        }
    }
    __syncthreads();
    float *gb = dqkv + (size_t)b * Ts * ld + h * DH;
    const int RT = Tp / 4;   // row tiles
    // dV[j][d] = sum_{r >= j} P[r][j] dO[r][d]: tile (4 j, 4 d)
    for (int t = threadIdx.x; t < RT * 8; t += blockDim.x) {
        const int j0 = 4 * (t >> 3), d0 = 4 * (t & 7);
        float acc[4][4] = {};
        for (int r = j0; r < Tp; ++r) {
            const float4 p = *reinterpret_cast<const float4 *>(S + r * SP + j0);
            const float4 g = *reinterpret_cast<const float4 *>(Gs + r * LD + d0);
            const float pv[4] = {p.x, p.y, p.z, p.w}, gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[a][c] = fmaf(pv[a], gv[c], acc[a][c]);
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
            if (j0 + a < Ts)
                *reinterpret_cast<float4 *>(gb + (size_t)(j0 + a) * ld + 2 * D + d0) =
                    make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    }
    __syncthreads();
    // dS[r][j] = P[r][j] (dP[r][j] - Dr[r]) scale, dP = dO V^T: tile (4 r, 4 j), j tile <= r tile,
    // written over P (each thread reads and writes only its own tile)
    const int ntri = RT * (RT + 1) / 2;
    for (int t = threadIdx.x; t < ntri; t += blockDim.x) {
        // lower-triangle tile t -> (rt, jt), jt <= rt
        int rt = (int)((sqrtf(8.0f * t + 1.0f) - 1.0f) * 0.5f);
        while ((rt + 1) * (rt + 2) / 2 <= t) ++rt;
        while (rt * (rt + 1) / 2 > t) --rt;
        const int jt = t - rt * (rt + 1) / 2;
        const int r0 = 4 * rt, j0 = 4 * jt;
        float acc[4][4] = {};
#pragma unroll 4
        for (int d = 0; d < DH; d += 4) {
            float4 gr[4], vr[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                gr[a] = *reinterpret_cast<const float4 *>(Gs + (r0 + a) * LD + d);
                vr[a] = *reinterpret_cast<const float4 *>(Vs + (j0 + a) * LD + d);
            }
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    acc[a][c] += gr[a].x * vr[c].x + gr[a].y * vr[c].y + gr[a].z * vr[c].z + gr[a].w * vr[c].w;
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            float4 *sp = reinterpret_cast<float4 *>(S + (r0 + a) * SP + j0);
            const float4 p = *sp;
            const float dr = Dr[r0 + a];
            *sp = make_float4(p.x * (acc[a][0] - dr) * scale, p.y * (acc[a][1] - dr) * scale,
                              p.z * (acc[a][2] - dr) * scale, p.w * (acc[a][3] - dr) * scale);
        }
    }
    __syncthreads();
    // dQ[r][d] = sum_{j <= r} dS[r][j] K[j][d]: tile (4 r, 4 d)
    for (int t = threadIdx.x; t < RT * 8; t += blockDim.x) {
        const int r0 = 4 * (t >> 3), d0 = 4 * (t & 7);
        float acc[4][4] = {};
        const int jend = r0 + 4 < Tp ? r0 + 4 : Tp;
        for (int j = 0; j < jend; ++j) {
            const float4 k = *reinterpret_cast<const float4 *>(Ks + j * LD + d0);
            const float kv[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const float sv = S[(r0 + a) * SP + j];
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[a][c] = fmaf(sv, kv[c], acc[a][c]);
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
            if (r0 + a < Ts)
                *reinterpret_cast<float4 *>(gb + (size_t)(r0 + a) * ld + d0) =
                    make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    }
    // dK[j][d] = sum_{r >= j} dS[r][j] Q[r][d]: tile (4 j, 4 d)
    for (int t = threadIdx.x; t < RT * 8; t += blockDim.x) {
        const int j0 = 4 * (t >> 3), d0 = 4 * (t & 7);
        float acc[4][4] = {};
        for (int r = j0; r < Tp; ++r) {
            const float4 sr = *reinterpret_cast<const float4 *>(S + r * SP + j0);
            const float4 q = *reinterpret_cast<const float4 *>(Qs + r * LD + d0);
            const float sv[4] = {sr.x, sr.y, sr.z, sr.w}, qv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[a][c] = fmaf(sv[a], qv[c], acc[a][c]);
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
            if (j0 + a < Ts)
                *reinterpret_cast<float4 *>(gb + (size_t)(j0 + a) * ld + D + d0) =
                    make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    }
}

// Embedding backward (the one-hot matmul's gradient, src/NN/Layers/Embedding.php:35-56),
// in two fixed-order passes.  Pass 1: for each chunk of kEmbChunk rows,
// part[chunk][v][d] = sum over the chunk's rows with token v of g[row][d].  Pass 2 (with
// the step's deferred sums): dTok[v][d] = the chunk partials in chunk order, dPos[t][d] =
// sum over sequences of g[b*T + t][d] (positions past the sequence length: zero).
constexpr int kEmbChunk = 64;

// Pass 1 when a chunk's [V][D] sums fit in shared memory: thread d walks the chunk's
// rows in order, eight rows' loads in flight, and adds g[row][d] into sums[token][d]
// (a thread owns column d of every token, so nothing races); then the block writes its
// [V][D] partial.  Token ids outside [0, V) add nothing.
__global__ void __launch_bounds__(128) embed_tok_rows_kernel(const float *__restrict__ g,
                                                             const float *__restrict__ tokens,
                                                             float *__restrict__ part, int N, int D, int V) {
    extern __shared__ float sums[];   // [V][D]
    for (int i = threadIdx.x; i < V * D; i += blockDim.x) sums[i] = 0.0f;
    __syncthreads();
    const int r0 = blockIdx.x * kEmbChunk, r1 = min(N, r0 + kEmbChunk);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        int r = r0;
        for (; r + 8 <= r1; r += 8) {
            float v[8];
            int t[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                t[u] = (int)__ldg(tokens + r + u);
                v[u] = __ldcs(g + (size_t)(r + u) * D + d);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if ((unsigned)t[u] < (unsigned)V) sums[t[u] * D + d] += v[u];
        }
        for (; r < r1; ++r) {
            const int t = (int)__ldg(tokens + r);
            if ((unsigned)t < (unsigned)V) sums[t * D + d] += g[(size_t)r * D + d];
        }
    }
    __syncthreads();
    float *dst = part + (size_t)blockIdx.x * V * D;
    for (int i = threadIdx.x; i < V * D; i += blockDim.x) dst[i] = sums[i];
}

// Pass 1 for a vocabulary too large for that: thread (v, d) scans the chunk's ids.
__global__ void __launch_bounds__(256) embed_tok_partial_kernel(const float *__restrict__ g,
                                                                const float *__restrict__ tokens,
                                                                float *__restrict__ part, int N, int D, int V) {
    __shared__ int ids[kEmbChunk];
    const int r0 = blockIdx.y * kEmbChunk;
    const int rows = min(kEmbChunk, N - r0);
    for (int k = threadIdx.x; k < rows; k += blockDim.x) ids[k] = (int)tokens[r0 + k];
    __syncthreads();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= V * D) return;
    const int v = i / D, d = i % D;
    float s = 0.0f;
    for (int k = 0; k < rows; ++k)
        if (ids[k] == v) s += g[(size_t)(r0 + k) * D + d];
    part[((size_t)blockIdx.y * V + v) * D + d] = s;
}

// All queued split sums of a step in one launch: blocks [start[j], start[j+1]) take job j,
// 128 elements per block (vec: 32 lanes x 4 consecutive elements, one 16-byte load per split)
// or 32 (one element per lane); warp w adds splits w, w + 8, ... in order, then the eight warp
// sums of each element are added in warp order (fixed order: deterministic).
__global__ void __launch_bounds__(256, 4) lm_reduce_all_kernel(const __grid_constant__ LmRedJobs J) {
    int j = 0;
    while (j + 1 < J.count && (int)blockIdx.x >= J.start[j + 1]) ++j;
    const LmRedJob &r = J.j[j];
    const int bx = (int)blockIdx.x - J.start[j];
    __shared__ float4 part[8][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long long total = (long long)r.M * r.N;
    const int per = r.vec ? 4 : 1;
    const long long i = ((long long)bx * 32 + lane) * per;   // first element of this lane
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (i < total && i < r.nvalid) {
        if (r.vec) {
            const float4 *p = reinterpret_cast<const float4 *>(r.partial + i);
            const long long st4 = r.stride >> 2;
            int k = w;
            for (; k + 24 < r.splits; k += 32) {
                const float4 a = __ldcg(p + (size_t)k * st4), b = __ldcg(p + (size_t)(k + 8) * st4);
                const float4 c = __ldcg(p + (size_t)(k + 16) * st4), d = __ldcg(p + (size_t)(k + 24) * st4);
                s.x += a.x; s.y += a.y; s.z += a.z; s.w += a.w;
                s.x += b.x; s.y += b.y; s.z += b.z; s.w += b.w;
                s.x += c.x; s.y += c.y; s.z += c.z; s.w += c.w;
                s.x += d.x; s.y += d.y; s.z += d.z; s.w += d.w;
            }
            for (; k < r.splits; k += 8) {
                const float4 a = __ldcg(p + (size_t)k * st4);
                s.x += a.x; s.y += a.y; s.z += a.z; s.w += a.w;
            }
        } else {
            const float *p = r.partial + i;
            int k = w;
            for (; k + 8 < r.splits; k += 16) {
                const float a = __ldcg(p + (size_t)k * r.stride), b = __ldcg(p + (size_t)(k + 8) * r.stride);
                s.x += a;
                s.x += b;
            }
            if (k < r.splits) s.x += __ldcg(p + (size_t)k * r.stride);
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
        const float v[4] = {t.x, t.y, t.z, t.w};
        for (int e = 0; e < per; ++e) {
            const long long ie = i + e;
            if (ie >= total) break;
            const int m = (int)(ie / r.N), n = (int)(ie % r.N), seg = n / r.sw;
            float *o = seg == 0 ? r.o[0] : seg == 1 ? r.o[1] : r.o[2];
            o[(size_t)m * r.sw + (n - seg * r.sw)] = ie < r.nvalid ? v[e] : 0.0f;
        }
    }
}

template <class T>
int lalloc(LmEngine &e, T **p, size_t count) {
    if (cudaMalloc((void **)p, (count ? count : 1) * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return fail(kBadHandle, "lm: cudaMalloc of %zu bytes failed", count * sizeof(T));
    }
    e.allocs.push_back((void *)*p);
    return kOk;
}

int ln_fwd(const float *x, const float *g, const float *b, float *y, float *xh, float *inv, int N, int D) {
    ln_fwd_kernel<<<grid_for((long long)N * 32, 256, 8), 256, 0, stream()>>>(x, g, b, y, xh, inv, N, D, 1e-5f);
    ZB_LAUNCH_CHECK("lm layernorm");
    return kOk;
}

int red_push(LmEngine &e, const float *partial, long long stride, int splits, int M, int N, int sw, long long nvalid,
             float *o0, float *o1, float *o2);
float *red_take(LmEngine &e, size_t n);

// LayerNorm backward; its dgamma | dbeta block partials join the step's deferred sums.
int ln_bwd(LmEngine &e, const float *gout, const float *xh, const float *inv, const float *gam, const float *R,
           float *out, float *dg, float *db) {
    const int warps = 8;
    float *part = red_take(e, (size_t)e.ln_blocks * 2 * e.D);
    if (!part) return fail(kBadArg, "lm: split-sum scratch exhausted");
    if (e.D == 128)
        ln_bwd_reg_kernel<4><<<e.ln_blocks, warps * 32, 0, stream()>>>(gout, xh, inv, gam, R, out, part, e.N);
    else
        ln_bwd_kernel<<<e.ln_blocks, warps * 32, (size_t)warps * 2 * e.D * sizeof(float), stream()>>>(
            gout, xh, inv, gam, R, out, part, e.N, e.D);
    ZB_LAUNCH_CHECK("lm layernorm backward");
    return red_push(e, part, 2 * e.D, e.ln_blocks, 1, 2 * e.D, e.D, 2 * e.D, dg, db, nullptr);
}

// Bias gradients: column sums of dY [rows][ld] in two fixed-order stages (row chunks over
// about two blocks per SM now, the chunks in order with the step's deferred sums), into
// segments of sw columns.
int colsum(LmEngine &e, const float *dY, int rows, int ld, int sw, float *o0, float *o1 = nullptr, float *o2 = nullptr) {
    const bool vec = ld % 4 == 0 && (reinterpret_cast<uintptr_t>(dY) & 15) == 0;
    const int tiles = vec ? (ld + 127) / 128 : (ld + 31) / 32;
    int chunks = sm_count() * 2 / tiles;
    if (chunks > rows / 32) chunks = rows / 32;
    if (chunks > kColsumChunks) chunks = kColsumChunks;
    if (chunks < 1) chunks = 1;
    float *part = red_take(e, (size_t)chunks * ld);
    if (!part) return fail(kBadArg, "lm: split-sum scratch exhausted");
    if (vec) colsum_part_kernel<true><<<dim3(tiles, chunks), dim3(32, 8), 0, stream()>>>(dY, rows, ld, chunks, part);
    else colsum_part_kernel<false><<<dim3(tiles, chunks), dim3(32, 8), 0, stream()>>>(dY, rows, ld, chunks, part);
    ZB_LAUNCH_CHECK("lm column sums (chunks)");
    return red_push(e, part, ld, chunks, 1, ld, sw, ld, o0, o1, o2);   // the chunks in order, deferred
}

// Runs every queued split sum (one launch) and empties the queue.
int red_flush(LmEngine &e) {
    if (e.red.empty()) return kOk;
    LmRedJobs J{};
    J.count = (int)e.red.size();
    int total = 0;
    for (int j = 0; j < J.count; ++j) {
        J.j[j] = e.red[j];
        J.start[j] = total;
        const long long el = (long long)e.red[j].M * e.red[j].N;
        total += (int)((el + (e.red[j].vec ? 128 : 32) - 1) / (e.red[j].vec ? 128 : 32));
    }
    J.start[J.count] = total;
    e.red.clear();
    lm_reduce_all_kernel<<<total, 256, 0, stream()>>>(J);
    ZB_LAUNCH_CHECK("lm split sums");
    return kOk;
}

int red_push(LmEngine &e, const float *partial, long long stride, int splits, int M, int N, int sw, long long nvalid,
             float *o0, float *o1 = nullptr, float *o2 = nullptr) {
    if ((int)e.red.size() == kMaxLmRed) {
        int rc = red_flush(e);
        if (rc) return rc;
    }
    LmRedJob j{};
    j.partial = partial; j.stride = stride; j.nvalid = nvalid;
    j.splits = splits; j.M = M; j.N = N; j.sw = sw;
    j.vec = ((long long)M * N) % 4 == 0 && stride % 4 == 0 && nvalid % 4 == 0 && sw % 4 == 0 && N % 4 == 0 &&
            (reinterpret_cast<uintptr_t>(partial) & 15) == 0;
    j.o[0] = o0; j.o[1] = o1; j.o[2] = o2;
    e.red.push_back(j);
    return kOk;
}

// A fresh 16-byte-aligned scratch region of n floats for this step's partials.
float *red_take(LmEngine &e, size_t n) {
    const size_t n4 = (n + 3) / 4 * 4;
    if (e.red_used + n4 > e.red_cap) return nullptr;
    float *p = e.red_arena + e.red_used;
    e.red_used += n4;
    return p;
}

int lm_build(Net &n, LmEngine &e) {
    const int D = e.D, N = e.N, F = e.F, L = e.L, V = e.V;
    long long off = 0;
    auto take = [&](long long cnt) { const long long o = off; off += cnt; return o; };
    e.o_tok = take((long long)V * D);
    e.o_pos = take((long long)e.T * D);
    e.o_lnf_g = take(D);
    e.o_lnf_b = take(D);
    e.o_head_W = take((long long)D * V);
    e.o_head_b = take(V);
    for (int l = 0; l < L; ++l) {
        LmEngine::Blk b;
        b.qW = take((long long)D * D); b.qb = take(D);
        b.kW = take((long long)D * D); b.kb = take(D);
        b.vW = take((long long)D * D); b.vb = take(D);
        b.oW = take((long long)D * D); b.ob = take(D);
        b.f1W = take((long long)D * F); b.f1b = take(F);
        b.f2W = take((long long)F * D); b.f2b = take(D);
        b.ln1g = take(D); b.ln1b = take(D); b.ln2g = take(D); b.ln2b = take(D);
        e.blk.push_back(b);
    }
    n.nparams = off;
    int rc;
    const size_t ND = (size_t)N * D;
    e.x.resize(L + 1);
    for (auto *v : {&e.h1, &e.xh1, &e.inv1, &e.qkv, &e.P, &e.att, &e.xm, &e.h2, &e.xh2, &e.inv2, &e.f1})
        v->resize(L);
    for (int l = 0; l <= L; ++l)
        if ((rc = lalloc(e, &e.x[l], ND))) return rc;
    for (int l = 0; l < L; ++l) {
        if ((rc = lalloc(e, &e.h1[l], ND)) || (rc = lalloc(e, &e.xh1[l], ND)) || (rc = lalloc(e, &e.inv1[l], N)) ||
            (rc = lalloc(e, &e.qkv[l], 3 * ND)) || (rc = lalloc(e, &e.P[l], (size_t)e.Bs * e.H * e.Ts * e.Ts)) ||
            (rc = lalloc(e, &e.att[l], ND)) || (rc = lalloc(e, &e.xm[l], ND)) || (rc = lalloc(e, &e.h2[l], ND)) ||
            (rc = lalloc(e, &e.xh2[l], ND)) || (rc = lalloc(e, &e.inv2[l], N)) ||
            (rc = lalloc(e, &e.f1[l], (size_t)N * F)))
            return rc;
    }
    if ((rc = lalloc(e, &e.hf, ND)) || (rc = lalloc(e, &e.xhf, ND)) || (rc = lalloc(e, &e.invf, N)) ||
        (rc = lalloc(e, &e.logits, (size_t)N * V)) || (rc = lalloc(e, &e.g, ND)) || (rc = lalloc(e, &e.gm, ND)) ||
        (rc = lalloc(e, &e.dh, ND)) || (rc = lalloc(e, &e.df1, (size_t)N * F)) || (rc = lalloc(e, &e.datt, ND)) ||
        (rc = lalloc(e, &e.dqkv, 3 * ND)))
        return rc;
    e.ln_blocks = sm_count() * 2;
    if ((rc = lalloc(e, &e.emb_partial, (size_t)((N + kEmbChunk - 1) / kEmbChunk) * V * D))) return rc;
    // per step: 4 column sums per block and the head's, 2 LayerNorms per block and the final one
    const int widest = 3 * D > F ? (3 * D > V ? 3 * D : V) : (F > V ? F : V);
    e.red_cap = (size_t)(4 * L + 1) * ((size_t)kColsumChunks * widest + 4) +
                (size_t)(2 * L + 1) * ((size_t)e.ln_blocks * 2 * D + 4);
    if ((rc = lalloc(e, &e.red_arena, e.red_cap))) return rc;
    return kOk;
}

// ---------------------------------------------------------------- tensor-core GEMMs (precision 1)
template <bool AMN, bool BMN, int EPI>
int launch_tf32(const tc::GemmTf32Params &p, int grid) {
    constexpr int BN = 128, NS = 4;
    using S = tc::GemmTf32Shape<BN, NS>;
    auto kern = tc::gemm_tf32_kernel<BN, AMN, BMN, EPI, NS>;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM) != cudaSuccess)
            return check_cuda("lm tf32 gemm smem attribute");
        attr = true;
    }
    launch_pdl(kern, dim3(grid), dim3(192), S::SMEM, p);
    ZB_LAUNCH_CHECK("lm tf32 gemm");
    return kOk;
}

int lm_tc_run(LmEngine &e, const LmTcGemm &g) {
    switch (g.kind) {
    case 0: return launch_tf32<false, true, tc::kTfStore>(g.p, g.grid);
    case 1: return launch_tf32<false, false, tc::kTfStore>(g.p, g.grid);
    case 2: return launch_tf32<false, false, tc::kTfMask>(g.p, g.grid);
    default: {   // the K splits' partials (this GEMM's own region) join the step's deferred sums
        int rc = launch_tf32<true, true, tc::kTfPartial>(g.p, g.grid);
        if (rc) return rc;
        return red_push(e, g.p.partial, (long long)g.p.M * g.p.N, g.p.ksplit, g.p.M, g.p.N, g.seg_w,
                        (long long)g.p.M * g.p.N, g.dst[0], g.dst[1], g.dst[2]);
    }
    }
}

// 2D fp32 tensor maps: K-major {K (contiguous), rows}, box {32, box_rows}, 128-byte swizzle;
// MN-major {MN (contiguous), K rows}, box {32, 32}, 128-byte swizzle over 32-byte atoms
int fmap(CUtensorMap *m, const float *base, int inner, int outer, int box_outer, bool mn_major = false) {
    const uint64_t dims[2] = {(uint64_t)inner, (uint64_t)outer}, strides[1] = {(uint64_t)inner * 4};
    const uint32_t box[2] = {32, (uint32_t)box_outer};
    return tc::make_tmap_f32(m, base, 2, dims, strides, box, mn_major ? tc::kSw128B32 : tc::kSw128);
}

// Forward: Y [M][ldo] = X [M][K] W_s [K][N_s] over nseg segments (n tile s = segment s when nseg > 1).
int tc_fwd(LmTcGemm &g, const float *X, int M, int K, const float *const *W, int nseg, int Nseg, const float *const *bias,
           const float *res, int ldr, bool relu, float *Y, int ldo) {
    tc::GemmTf32Params &p = g.p;
    int rc;
    if ((rc = fmap(&p.a_map, X, K, M, 128))) return rc;
    for (int s = 0; s < nseg; ++s)
        if ((rc = fmap(&p.b_map[s], W[s], Nseg, K, 32, true))) return rc;
    p.M = M; p.N = nseg * Nseg; p.K = K;
    p.m_tiles = M / 128; p.n_tiles = p.N / 128; p.ksplit = 1; p.kper = K / 32;
    p.nseg = nseg; p.b_seg_by_n = nseg > 1; p.seg_k = 0;
    p.out = Y; p.ldo = ldo;
    for (int s = 0; s < 3; ++s) p.bias[s] = s < nseg ? bias[s] : nullptr;
    p.res = res; p.ldr = ldr; p.relu = relu;
    g.kind = 0;
    return kOk;
}

// Input gradient: dX [M][ldo] = sum_s dY[:, s*Kseg ..] W_s^T, W_s [N][Kseg] (the layer's [in][out]).
int tc_dgrad(LmTcGemm &g, const float *dY, int M, int Kseg, int nseg, const float *const *W, int N, const float *mask,
             float *dX) {
    tc::GemmTf32Params &p = g.p;
    int rc;
    if ((rc = fmap(&p.a_map, dY, Kseg * nseg, M, 128))) return rc;
    for (int s = 0; s < nseg; ++s)
        if ((rc = fmap(&p.b_map[s], W[s], Kseg, N, 128))) return rc;
    p.M = M; p.N = N; p.K = Kseg * nseg;
    p.m_tiles = M / 128; p.n_tiles = N / 128; p.ksplit = 1; p.kper = p.K / 32;
    p.nseg = nseg; p.b_seg_by_n = 0; p.seg_k = nseg > 1 ? Kseg : 0;
    p.out = dX; p.ldo = N;
    p.mask = mask; p.ldm = N;
    g.kind = mask ? 2 : 1;
    return kOk;
}

// Weight gradient: dW [M][N] = X^T dY over `rows` rows, X [rows][M], dY [rows][N]; the
// summed result goes to dst[n / seg_w].
int tc_wgrad(LmTcGemm &g, const float *X, int M, const float *dY, int N, int rows, float *const *dst, int seg_w) {
    tc::GemmTf32Params &p = g.p;
    int rc;
    if ((rc = fmap(&p.a_map, X, M, rows, 32, true))) return rc;
    if ((rc = fmap(&p.b_map[0], dY, N, rows, 32, true))) return rc;
    p.M = M; p.N = N; p.K = rows;
    p.m_tiles = M / 128; p.n_tiles = N / 128;
    const int stages = rows / 32;
    int ks = sm_count() / (p.m_tiles * p.n_tiles);
    if (ks > stages / 8) ks = stages / 8;   // at least eight K stages per split
    if (ks > 32) ks = 32;
    if (ks < 1) ks = 1;
    p.kper = (stages + ks - 1) / ks;
    p.ksplit = (stages + p.kper - 1) / p.kper;
    p.nseg = 1; p.b_seg_by_n = 0; p.seg_k = 0;
    g.kind = 3;
    for (int s = 0; s < 3; ++s) g.dst[s] = dst[s];
    g.seg_w = seg_w;
    return kOk;
}

// Copies of the blocks' weights and biases into the aligned shadow: job j copies
// len[j] floats from params + src[j] to shadow + dst[j] (blockIdx.y = job).
struct ShadowJobs {
    long long src[64], dst[64], len[64];
};

__global__ void __launch_bounds__(256) lm_shadow_kernel(const float *__restrict__ params, float *__restrict__ shadow,
                                                        const __grid_constant__ ShadowJobs J) {
    griddep_launch();
    griddep_wait();
    const int j = blockIdx.y;
    const float *s = params + J.src[j];
    float *d = shadow + J.dst[j];
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < J.len[j]; i += (long long)gridDim.x * blockDim.x)
        d[i] = __ldg(s + i);
}

int lm_tc_shadow(const Net &n, const LmEngine &e) {
    ShadowJobs J{};
    const int nj = (int)e.shadow_src.size();
    long long longest = 0;
    for (int j = 0; j < nj; ++j) {
        J.src[j] = e.shadow_src[j]; J.dst[j] = e.shadow_dst[j]; J.len[j] = e.shadow_len[j];
        if (J.len[j] > longest) longest = J.len[j];
    }
    // about two elements per thread of the longest tensor: each thread's loads are a
    // dependent chain of latencies, so the width of the grid sets the time
    long long bx = (longest + 511) / 512;
    if (bx > 128) bx = 128;
    if (bx < 1) bx = 1;
    launch_pdl(lm_shadow_kernel, dim3((unsigned)bx, nj), dim3(256), 0, (const float *)n.params, e.tc_shadow, J);
    ZB_LAUNCH_CHECK("lm weight shadow");
    return kOk;
}

// The plan over the net's buffers (after net_alloc_common: parameters and gradients exist).
int lm_tc_build(Net &n, LmEngine &e) {
    const int D = e.D, N = e.N, F = e.F, L = e.L;
    if (N % 128 || D % 128 || F % 128 || N % 256)
        return fail(kBadArg, "lm: tensor-core GEMMs need batch*seq %% 256 == 0 and dim, ffn %% 128 == 0 (%d, %d, %d)",
                    N, D, F);
    if (L * 12 > 64) return fail(kBadArg, "lm: tensor-core GEMMs support up to 5 blocks");
    e.tc_params = n.params;
    e.tc_grads = n.grads;
    float *G = n.grads;
    // the aligned shadow of every block weight and bias (each tensor at a multiple of 4 floats)
    e.shadow_src.clear(); e.shadow_dst.clear(); e.shadow_len.clear();
    long long sh = 0;
    auto place = [&](long long src, long long len) {
        e.shadow_src.push_back(src); e.shadow_dst.push_back(sh); e.shadow_len.push_back(len);
        const long long at = sh;
        sh += (len + 3) / 4 * 4;
        return at;
    };
    std::vector<LmEngine::Blk> sb(L);   // shadow offsets of each block's tensors
    for (int l = 0; l < L; ++l) {
        const auto &b = e.blk[l];
        LmEngine::Blk &o = sb[l];
        o.qW = place(b.qW, (long long)D * D); o.qb = place(b.qb, D);
        o.kW = place(b.kW, (long long)D * D); o.kb = place(b.kb, D);
        o.vW = place(b.vW, (long long)D * D); o.vb = place(b.vb, D);
        o.oW = place(b.oW, (long long)D * D); o.ob = place(b.ob, D);
        o.f1W = place(b.f1W, (long long)D * F); o.f1b = place(b.f1b, F);
        o.f2W = place(b.f2W, (long long)F * D); o.f2b = place(b.f2b, D);
    }
    int rc;
    if ((rc = lalloc(e, &e.tc_shadow, (size_t)sh))) return rc;
    const float *Pm = e.tc_shadow;
    size_t part = 0;
    e.tcg.assign((size_t)L * kLmTcPerBlock, LmTcGemm());
    std::vector<size_t> part_off(e.tcg.size(), 0);
    for (int l = 0; l < L; ++l) {
        const auto &b = sb[l];        // operands: the shadow copies
        const auto &bg = e.blk[l];    // gradient destinations: the flat layout
        LmTcGemm *g = &e.tcg[(size_t)l * kLmTcPerBlock];
        for (int j = 0; j < kLmTcPerBlock; ++j) g[j].p.err = device_error_word();
        const float *Wqkv[3] = {Pm + b.qW, Pm + b.kW, Pm + b.vW}, *bqkv[3] = {Pm + b.qb, Pm + b.kb, Pm + b.vb};
        const float *Wo[1] = {Pm + b.oW}, *bo[1] = {Pm + b.ob};
        const float *W1[1] = {Pm + b.f1W}, *b1[1] = {Pm + b.f1b};
        const float *W2[1] = {Pm + b.f2W}, *b2[1] = {Pm + b.f2b};
        if ((rc = tc_fwd(g[0], e.h1[l], N, D, Wqkv, 3, D, bqkv, nullptr, 0, false, e.qkv[l], 3 * D)) ||
            (rc = tc_fwd(g[1], e.att[l], N, D, Wo, 1, D, bo, e.x[l], D, false, e.xm[l], D)) ||
            (rc = tc_fwd(g[2], e.h2[l], N, D, W1, 1, F, b1, nullptr, 0, true, e.f1[l], F)) ||
            (rc = tc_fwd(g[3], e.f1[l], N, F, W2, 1, D, b2, e.xm[l], D, false, e.x[l + 1], D)))
            return rc;
        // input gradients: W [in][out] is B K-major over out
        if ((rc = tc_dgrad(g[4], e.g, N, D, 1, W2, F, e.f1[l], e.df1)) ||
            (rc = tc_dgrad(g[5], e.df1, N, F, 1, W1, D, nullptr, e.dh)) ||
            (rc = tc_dgrad(g[6], e.gm, N, D, 1, Wo, D, nullptr, e.datt)) ||
            (rc = tc_dgrad(g[7], e.dqkv, N, D, 3, Wqkv, D, nullptr, e.dh)))
            return rc;
        float *dW2[3] = {G + bg.f2W, nullptr, nullptr}, *dW1[3] = {G + bg.f1W, nullptr, nullptr};
        float *dWo[3] = {G + bg.oW, nullptr, nullptr}, *dWqkv[3] = {G + bg.qW, G + bg.kW, G + bg.vW};
        if ((rc = tc_wgrad(g[8], e.f1[l], F, e.g, D, N, dW2, D)) ||
            (rc = tc_wgrad(g[9], e.h2[l], D, e.df1, F, N, dW1, F)) ||
            (rc = tc_wgrad(g[10], e.att[l], D, e.gm, D, N, dWo, D)) ||
            (rc = tc_wgrad(g[11], e.h1[l], D, e.dqkv, 3 * D, N, dWqkv, D)))
            return rc;
        for (int j = 0; j < kLmTcPerBlock; ++j) {
            LmTcGemm &t = g[j];
            const int tiles = t.p.m_tiles * t.p.n_tiles * t.p.ksplit;
            t.grid = tiles < sm_count() ? tiles : sm_count();
            if (t.kind == 3) {   // its own partial region (summed at the end of the step)
                part_off[(size_t)l * kLmTcPerBlock + j] = part;
                part += ((size_t)t.p.ksplit * t.p.M * t.p.N + 3) / 4 * 4;
            }
        }
    }
    if ((rc = lalloc(e, &e.tc_partial, part))) return rc;
    for (size_t k = 0; k < e.tcg.size(); ++k)
        if (e.tcg[k].kind == 3) e.tcg[k].p.partial = e.tc_partial + part_off[k];
    // attention: one (sequence, head) per CTA when a sequence fits one 128-row tile
    e.attn_f.clear(); e.attn_b.clear(); e.attn_stats.clear();
    if (e.D / e.H == 32 && e.D % e.H == 0 && e.Ts <= 128) {
        static bool attr = false;
        if (!attr) {
            if (cudaFuncSetAttribute(tc::attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     tc::kAttnFwdSmem) != cudaSuccess ||
                cudaFuncSetAttribute(tc::attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     tc::kAttnBwdSmem) != cudaSuccess)
                return check_cuda("lm: attention smem attribute");
            attr = true;
        }
        const uint32_t box[2] = {32, 128};
        const uint64_t dq[2] = {(uint64_t)3 * D, (uint64_t)N}, sq[1] = {(uint64_t)3 * D * 4};
        const uint64_t dd[2] = {(uint64_t)D, (uint64_t)N}, sd[1] = {(uint64_t)D * 4};
        for (int l = 0; l < L; ++l) {
            float *st = nullptr;
            if ((rc = lalloc(e, &st, (size_t)e.Bs * e.H * e.Ts * 2))) return rc;
            tc::AttnTcParams a{};
            if ((rc = tc::make_tmap_f32(&a.qkv_k, e.qkv[l], 2, dq, sq, box, tc::kSw128)) ||
                (rc = tc::make_tmap_f32(&a.qkv_mn, e.qkv[l], 2, dq, sq, box, tc::kSw128B32)) ||
                (rc = tc::make_tmap_f32(&a.do_k, e.datt, 2, dd, sd, box, tc::kSw128)) ||
                (rc = tc::make_tmap_f32(&a.do_mn, e.datt, 2, dd, sd, box, tc::kSw128B32)))
                return rc;
            a.T = e.Ts; a.H = e.H; a.D = D;
            a.scale = 1.0f / sqrtf((float)(D / e.H));
            a.stats = st;
            a.err = device_error_word();
            tc::AttnTcParams f = a, bw = a;
            f.out = e.att[l];
            bw.O = e.att[l];
            bw.dO = e.datt;
            bw.out = e.dqkv;
            e.attn_f.push_back(f);
            e.attn_b.push_back(bw);
            e.attn_stats.push_back(st);
        }
    }
    return kOk;
}

int attn_smem_fwd(int Ts, int dh) {
    const size_t Tp = (size_t)((Ts + 3) & ~3);
    return (int)((2 * Tp * (dh + 4) + 32 * (size_t)(dh + 4) + 32 * (Tp + 4)) * sizeof(float));
}
int attn_smem_bwd(int Ts, int dh) {
    const size_t Tp = (size_t)((Ts + 3) & ~3);
    return (int)((4 * Tp * (dh + 4) + Tp * (Tp + 4) + Tp) * sizeof(float));
}

}  // namespace

// Shapes of the LM's parameter tensors in buffer order (the order lm_build
// lays them out in, which is TransformerLM::parameters() order).
int lm_param_shapes(Net &n, std::vector<std::vector<long long>> &shapes) {
    const LmEngine &e = *n.lm;
    const long long V = e.V, D = e.D, F = e.F, T = e.T;
    shapes = {{V, D}, {T, D}, {D}, {D}, {D, V}, {V}};
    for (int l = 0; l < e.L; ++l) {
        for (int k = 0; k < 4; ++k) {   // q, k, v, o: W [D, D], b [D]
            shapes.push_back({D, D});
            shapes.push_back({D});
        }
        shapes.push_back({D, F});
        shapes.push_back({F});
        shapes.push_back({F, D});
        shapes.push_back({D});
        for (int k = 0; k < 4; ++k) shapes.push_back({D});   // ln1 g, b; ln2 g, b
    }
    return kOk;
}

void lm_destroy(Net &n) {
    if (!n.lm) return;
    cudaStreamSynchronize(stream());
    for (void *p : n.lm->allocs) cudaFree(p);
    delete n.lm;
    n.lm = nullptr;
}

int lm_step(Net &n, const float *tokens, const float *targets, float *loss_out) {
    LmEngine &e = *n.lm;
    const int D = e.D, N = e.N, F = e.F, V = e.V, L = e.L;
    const float *Pm = n.params;
    float *G = n.grads;
    const float scale = 1.0f / sqrtf((float)(D / e.H));
    int rc;
    // precision 1: the Linear GEMMs of the blocks on TF32 tensor cores (the plan holds
    // the parameter and gradient buffers it was built over)
    const bool tcp = n.precision == 1 && !e.tcg.empty();
    if (tcp && (G != e.tc_grads || Pm != e.tc_params))
        return fail(kBadArg, "lm: tensor-core plan built over other parameter / gradient buffers");
    if (tcp && (rc = lm_tc_shadow(n, e))) return rc;   // this step's weights, aligned for TMA
    e.red.clear();       // (a step that failed part-way leaves nothing queued for the next)
    e.red_used = 0;
    // ---- forward
    embed_fwd_kernel<<<grid_for((long long)N * D, 256, 8), 256, 0, stream()>>>(
        tokens, Pm + e.o_tok, Pm + e.o_pos, e.x[0], N, e.Ts, D, V, device_error_word());
    ZB_LAUNCH_CHECK("lm embedding");
    prof_mark(n, "embed");
    for (int l = 0; l < L; ++l) {
        const auto &b = e.blk[l];
        const LmTcGemm *tg = tcp ? &e.tcg[(size_t)l * kLmTcPerBlock] : nullptr;
        if ((rc = ln_fwd(e.x[l], Pm + b.ln1g, Pm + b.ln1b, e.h1[l], e.xh1[l], e.inv1[l], N, D))) return rc;
        LinFwd qkv{e.h1[l], nullptr, {Pm + b.qW, Pm + b.kW, Pm + b.vW}, {Pm + b.qb, Pm + b.kb, Pm + b.vb},
                   e.qkv[l], N, 3 * D, D, D, 3 * D, D, false};
        if ((rc = tcp ? lm_tc_run(e, tg[0]) : run_simt_gemm(qkv, 1, "lm qkv"))) return rc;
        prof_mark(n, "ln1_qkv");
        if (tcp && !e.attn_f.empty())
            tc::attn_fwd_tc_kernel<<<e.Bs * e.H, 512, tc::kAttnFwdSmem, stream()>>>(e.attn_f[l]);
        else
            attn_fwd_kernel<32><<<dim3(e.Bs * e.H, (e.Ts + 31) / 32), 128, attn_smem_fwd(e.Ts, 32), stream()>>>(
                e.qkv[l], e.P[l], e.att[l], e.Ts, e.H, D, scale);
        ZB_LAUNCH_CHECK("lm attention");
        prof_mark(n, "attn_fwd");
        LinFwd o{e.att[l], e.x[l], {Pm + b.oW, nullptr, nullptr}, {Pm + b.ob, nullptr, nullptr}, e.xm[l],
                 N, D, D, D, D, D, false};
        if ((rc = tcp ? lm_tc_run(e, tg[1]) : run_simt_gemm(o, 1, "lm out proj"))) return rc;
        if ((rc = ln_fwd(e.xm[l], Pm + b.ln2g, Pm + b.ln2b, e.h2[l], e.xh2[l], e.inv2[l], N, D))) return rc;
        LinFwd f1{e.h2[l], nullptr, {Pm + b.f1W, nullptr, nullptr}, {Pm + b.f1b, nullptr, nullptr}, e.f1[l],
                  N, F, D, D, F, F, true};
        if ((rc = tcp ? lm_tc_run(e, tg[2]) : run_simt_gemm(f1, 1, "lm fc1"))) return rc;
        LinFwd f2{e.f1[l], e.xm[l], {Pm + b.f2W, nullptr, nullptr}, {Pm + b.f2b, nullptr, nullptr}, e.x[l + 1],
                  N, D, F, F, D, D, false};
        if ((rc = tcp ? lm_tc_run(e, tg[3]) : run_simt_gemm(f2, 1, "lm fc2"))) return rc;
        prof_mark(n, "oproj_ln2_ffn");
    }
    if ((rc = ln_fwd(e.x[L], Pm + e.o_lnf_g, Pm + e.o_lnf_b, e.hf, e.xhf, e.invf, N, D))) return rc;
    LinFwd head{e.hf, nullptr, {Pm + e.o_head_W, nullptr, nullptr}, {Pm + e.o_head_b, nullptr, nullptr}, e.logits,
                N, V, D, D, V, V, false};
    if ((rc = run_simt_gemm(head, 1, "lm head"))) return rc;
    if ((rc = launch_softmax_ce(e.logits, targets, n.dlogits, n.row_loss, loss_out, N, V, true))) return rc;
    prof_mark(n, "head_ce");
    // ---- backward
    {
        LinWgrad wg{e.hf, n.dlogits, {G + e.o_head_W, nullptr, nullptr}, D, V, N, D, V, V};
        if ((rc = run_simt_gemm(wg, 0, "lm head dW"))) return rc;
        if ((rc = colsum(e, n.dlogits, N, V, V, G + e.o_head_b))) return rc;
        LinDgrad dg{n.dlogits, nullptr, {Pm + e.o_head_W, nullptr, nullptr}, e.dh, N, D, V, D, V, V};
        if ((rc = run_simt_gemm(dg, 1, "lm head dX"))) return rc;
        if ((rc = ln_bwd(e, e.dh, e.xhf, e.invf, Pm + e.o_lnf_g, nullptr, e.g, G + e.o_lnf_g, G + e.o_lnf_b))) return rc;
    }
    prof_mark(n, "head_bwd");
    for (int l = L - 1; l >= 0; --l) {
        const auto &b = e.blk[l];
        const LmTcGemm *tg = tcp ? &e.tcg[(size_t)l * kLmTcPerBlock] : nullptr;
        // FFN
        LinWgrad w2{e.f1[l], e.g, {G + b.f2W, nullptr, nullptr}, F, D, N, F, D, D};
        if ((rc = tcp ? lm_tc_run(e, tg[8]) : run_simt_gemm(w2, 0, "lm fc2 dW"))) return rc;
        if ((rc = colsum(e, e.g, N, D, D, G + b.f2b))) return rc;
        LinDgrad d2{e.g, e.f1[l], {Pm + b.f2W, nullptr, nullptr}, e.df1, N, F, D, F, D, D};
        if ((rc = tcp ? lm_tc_run(e, tg[4]) : run_simt_gemm(d2, 1, "lm fc2 dX"))) return rc;
        LinWgrad w1{e.h2[l], e.df1, {G + b.f1W, nullptr, nullptr}, D, F, N, D, F, F};
        if ((rc = tcp ? lm_tc_run(e, tg[9]) : run_simt_gemm(w1, 0, "lm fc1 dW"))) return rc;
        if ((rc = colsum(e, e.df1, N, F, F, G + b.f1b))) return rc;
        LinDgrad d1{e.df1, nullptr, {Pm + b.f1W, nullptr, nullptr}, e.dh, N, D, F, D, F, F};
        if ((rc = tcp ? lm_tc_run(e, tg[5]) : run_simt_gemm(d1, 1, "lm fc1 dX"))) return rc;
        if ((rc = ln_bwd(e, e.dh, e.xh2[l], e.inv2[l], Pm + b.ln2g, e.g, e.gm, G + b.ln2g, G + b.ln2b))) return rc;
        prof_mark(n, "ffn_ln2_bwd");
        // attention
        LinWgrad wo{e.att[l], e.gm, {G + b.oW, nullptr, nullptr}, D, D, N, D, D, D};
        if ((rc = tcp ? lm_tc_run(e, tg[10]) : run_simt_gemm(wo, 0, "lm out dW"))) return rc;
        if ((rc = colsum(e, e.gm, N, D, D, G + b.ob))) return rc;
        LinDgrad dout{e.gm, nullptr, {Pm + b.oW, nullptr, nullptr}, e.datt, N, D, D, D, D, D};
        if ((rc = tcp ? lm_tc_run(e, tg[6]) : run_simt_gemm(dout, 1, "lm out dX"))) return rc;
        if (tcp && !e.attn_b.empty())
            tc::attn_bwd_tc_kernel<<<e.Bs * e.H, 512, tc::kAttnBwdSmem, stream()>>>(e.attn_b[l]);
        else
            attn_bwd_kernel<32><<<e.Bs * e.H, 256, attn_smem_bwd(e.Ts, 32), stream()>>>(e.qkv[l], e.P[l], e.datt,
                                                                                      e.att[l], e.dqkv, e.Ts, e.H, D, scale);
        ZB_LAUNCH_CHECK("lm attention backward");
        prof_mark(n, "oproj_attn_bwd");
        LinWgrad wq{e.h1[l], e.dqkv, {G + b.qW, G + b.kW, G + b.vW}, D, 3 * D, N, D, 3 * D, D};
        if ((rc = tcp ? lm_tc_run(e, tg[11]) : run_simt_gemm(wq, 0, "lm qkv dW"))) return rc;
        if ((rc = colsum(e, e.dqkv, N, 3 * D, D, G + b.qb, G + b.kb, G + b.vb))) return rc;
        LinDgrad dq{e.dqkv, nullptr, {Pm + b.qW, Pm + b.kW, Pm + b.vW}, e.dh, N, D, 3 * D, D, 3 * D, D};
        if ((rc = tcp ? lm_tc_run(e, tg[7]) : run_simt_gemm(dq, 1, "lm qkv dX"))) return rc;
        if ((rc = ln_bwd(e, e.dh, e.xh1[l], e.inv1[l], Pm + b.ln1g, e.gm, e.g, G + b.ln1g, G + b.ln1b))) return rc;
        prof_mark(n, "qkv_ln1_bwd");
    }
    const int chunks = (N + kEmbChunk - 1) / kEmbChunk;
    const size_t emb_smem = (size_t)V * D * sizeof(float);
    if (emb_smem <= 48 * 1024)
        embed_tok_rows_kernel<<<chunks, 128, emb_smem, stream()>>>(e.g, tokens, e.emb_partial, N, D, V);
    else
        embed_tok_partial_kernel<<<dim3((V * D + 255) / 256, chunks), 256, 0, stream()>>>(e.g, tokens, e.emb_partial,
                                                                                        N, D, V);
    ZB_LAUNCH_CHECK("lm embedding backward (partials)");
    // token rows: the chunk partials in order; positions: the sequences' rows in order (positions
    // past the sequence length get zero)
    if ((rc = red_push(e, e.emb_partial, (long long)V * D, chunks, 1, V * D, V * D, (long long)V * D, G + e.o_tok)) ||
        (rc = red_push(e, e.g, (long long)e.Ts * D, N / e.Ts, 1, e.T * D, e.T * D, (long long)e.Ts * D, G + e.o_pos)))
        return rc;
    if ((rc = red_flush(e))) return rc;   // every split sum of the step, before the optimizer
    prof_mark(n, "embed_bwd");
    return kOk;
}

namespace {

int attn_smem_cached(int len) { return (int)((5 * 32 + 8 + (size_t)len) * sizeof(float)); }

int lm_cache_alloc(LmEngine &e) {
    if (!e.kc.empty()) return kOk;
    const int T = e.T;
    if (attn_smem_cached(T) > 227 * 1024)
        return fail(kBadArg, "zilla_lm_forward_cached: max_seq %d above the supported 57900 for generation", T);
    const size_t TD = (size_t)T * e.D;
    int rc;
    if ((rc = lalloc(e, &e.gx, TD)) || (rc = lalloc(e, &e.gxm, TD)) || (rc = lalloc(e, &e.gh, TD)) ||
        (rc = lalloc(e, &e.gxh, TD)) || (rc = lalloc(e, &e.ginv, T)) || (rc = lalloc(e, &e.gqkv, 3 * TD)) ||
        (rc = lalloc(e, &e.gatt, TD)) || (rc = lalloc(e, &e.gf1, (size_t)T * e.F)) ||
        (rc = lalloc(e, &e.glog, (size_t)T * e.V)) || (rc = lalloc(e, &e.gtok, T)))
        return rc;
    std::vector<float *> kc(e.L), vc(e.L);
    for (int l = 0; l < e.L; ++l)
        if ((rc = lalloc(e, &kc[l], TD)) || (rc = lalloc(e, &vc[l], TD))) return rc;
    if (cudaFuncSetAttribute(attn_cached_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             attn_smem_cached(T)) != cudaSuccess)
        return check_cuda("zilla_lm_forward_cached: attention shared memory");
    e.kc = kc;
    e.vc = vc;
    return kOk;
}

}  // namespace

// TransformerLM::forwardWithCache (src/Transformers/TransformerLM.php:124-151):
// `count` new tokens (host floats, Embedding's (int) cast) at positions
// cache_len .. cache_len+count-1; per block TransformerBlock::forwardWithCache
// (TransformerBlock.php:40-45) with the K/V rows appended to the layer's cache
// and unmasked attention over all cached rows; logits [count, V] to the host.
// The cache is unchanged when the call fails (the reference throws before it
// advances the cache length).
int lm_forward_cached(Net &n, const float *tokens, int count, float *logits) {
    LmEngine &e = *n.lm;
    const int D = e.D, F = e.F, V = e.V, L = e.L;
    if (count <= 0 || !tokens) return fail(kBadArg, "zilla_lm_forward_cached: no tokens");
    if (e.cache_len + count > e.T)
        return fail(kBadArg, "zilla_lm_forward_cached: sequence position %d exceeds max %d", e.cache_len + count, e.T);
    for (int i = 0; i < count; ++i) {   // Embedding::forward (src/NN/Layers/Embedding.php:44-48)
        const float t = tokens[i];
        if (!(t > -1.0f && t < (float)V))   // (int)t in [0, V); NaN fails both compares
            return fail(kBadArg, "zilla_lm_forward_cached: token id %g out of range [0, %d)", (double)t, V);
    }
    int rc;
    if ((rc = lm_cache_alloc(e))) return rc;
    const float *Pm = n.params;
    const float scale = 1.0f / sqrtf((float)(D / e.H));
    const int off = e.cache_len, len = off + count;
    cudaMemcpyAsync(e.gtok, tokens, (size_t)count * sizeof(float), cudaMemcpyHostToDevice, stream());
    embed_fwd_kernel<<<grid_for((long long)count * D, 256, 8), 256, 0, stream()>>>(
        e.gtok, Pm + e.o_tok, Pm + e.o_pos, e.gx, count, count, D, V, device_error_word(), off);
    ZB_LAUNCH_CHECK("lm generation embedding");
    for (int l = 0; l < L; ++l) {
        const auto &b = e.blk[l];
        if ((rc = ln_fwd(e.gx, Pm + b.ln1g, Pm + b.ln1b, e.gh, e.gxh, e.ginv, count, D))) return rc;
        LinFwd qkv{e.gh, nullptr, {Pm + b.qW, Pm + b.kW, Pm + b.vW}, {Pm + b.qb, Pm + b.kb, Pm + b.vb},
                   e.gqkv, count, 3 * D, D, D, 3 * D, D, false};
        if ((rc = run_simt_gemm(qkv, 1, "lm generation qkv"))) return rc;
        kv_append_kernel<<<grid_for((long long)count * D, 256, 8), 256, 0, stream()>>>(e.gqkv, e.kc[l], e.vc[l],
                                                                                     count, D, off);
        ZB_LAUNCH_CHECK("lm generation kv append");
        attn_cached_kernel<32><<<dim3(e.H, count), 128, attn_smem_cached(len), stream()>>>(
            e.gqkv, e.kc[l], e.vc[l], e.gatt, len, D, scale);
        ZB_LAUNCH_CHECK("lm generation attention");
        LinFwd o{e.gatt, e.gx, {Pm + b.oW, nullptr, nullptr}, {Pm + b.ob, nullptr, nullptr}, e.gxm,
                 count, D, D, D, D, D, false};
        if ((rc = run_simt_gemm(o, 1, "lm generation out proj"))) return rc;
        if ((rc = ln_fwd(e.gxm, Pm + b.ln2g, Pm + b.ln2b, e.gh, e.gxh, e.ginv, count, D))) return rc;
        LinFwd f1{e.gh, nullptr, {Pm + b.f1W, nullptr, nullptr}, {Pm + b.f1b, nullptr, nullptr}, e.gf1,
                  count, F, D, D, F, F, true};
        if ((rc = run_simt_gemm(f1, 1, "lm generation fc1"))) return rc;
        LinFwd f2{e.gf1, e.gxm, {Pm + b.f2W, nullptr, nullptr}, {Pm + b.f2b, nullptr, nullptr}, e.gx,
                  count, D, F, F, D, D, false};
        if ((rc = run_simt_gemm(f2, 1, "lm generation fc2"))) return rc;
    }
    if ((rc = ln_fwd(e.gx, Pm + e.o_lnf_g, Pm + e.o_lnf_b, e.gh, e.gxh, e.ginv, count, D))) return rc;
    LinFwd head{e.gh, nullptr, {Pm + e.o_head_W, nullptr, nullptr}, {Pm + e.o_head_b, nullptr, nullptr}, e.glog,
                count, V, D, D, V, V, false};
    if ((rc = run_simt_gemm(head, 1, "lm generation head"))) return rc;
    if (logits)
        cudaMemcpyAsync(logits, e.glog, (size_t)count * V * sizeof(float), cudaMemcpyDeviceToHost, stream());
    if (cudaStreamSynchronize(stream()) != cudaSuccess) return check_cuda("zilla_lm_forward_cached");
    if ((rc = check_cuda("zilla_lm_forward_cached"))) return rc;
    e.cache_len = len;
    return kOk;
}

}  // namespace zb

using namespace zb;

extern "C" int zilla_lm_create(int vocab, int dim, int heads, int layers, int max_seq, int ffn, int batch,
                               int seq) {
    if (vocab <= 0 || dim <= 0 || heads <= 0 || layers <= 0 || ffn <= 0 || batch <= 0 || seq <= 0)
        return fail(kBadArg, "zilla_lm_create: bad arguments");
    if (dim % heads || dim / heads != 32)
        return fail(kBadArg, "zilla_lm_create: head dimension must be 32 (dim %d, heads %d)", dim, heads);
    if (dim % 32 || dim > 1024) return fail(kBadArg, "zilla_lm_create: dim must be a multiple of 32, <= 1024");
    if (seq > max_seq) return fail(kBadArg, "zilla_lm_create: sequence length %d exceeds max %d", seq, max_seq);
    if (attn_smem_bwd(seq, 32) > 227 * 1024)   // one (sequence, head) of the backward lives in shared memory
        return fail(kBadArg, "zilla_lm_create: sequence length %d above the supported 176", seq);
    if (layers > 64) return fail(kBadArg, "zilla_lm_create: too many layers");
    Net *n = new Net();
    LmEngine *e = new LmEngine();
    e->V = vocab; e->D = dim; e->H = heads; e->L = layers; e->T = max_seq; e->F = ffn;
    e->Bs = batch; e->Ts = seq; e->N = batch * seq;
    n->lm = e;
    n->B = e->N;
    n->classes = vocab;
    n->precision = 0;
    int rc = lm_build(*n, *e);
    n->x_floats = e->N;
    n->y_floats = e->N;
    if (!rc) rc = net_alloc_common(*n, (long long)e->N * vocab, e->N);
    if (!rc) {
        const int fs = attn_smem_fwd(seq, 32), bs = attn_smem_bwd(seq, 32);
        if (cudaFuncSetAttribute(attn_fwd_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, fs) != cudaSuccess ||
            cudaFuncSetAttribute(attn_bwd_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bs) != cudaSuccess ||
            cudaFuncSetAttribute(ln_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 8 * 2 * dim * (int)sizeof(float)) != cudaSuccess)
            rc = check_cuda("zilla_lm_create: attention shared memory");
    }
    if (!rc) rc = check_cuda("zilla_lm_create");
    if (rc) {
        net_free(n);
        return rc;
    }
    return net_register(n);
}

extern "C" int zilla_lm_set_precision(int net, int precision) {
    Net *n = net_get(net);
    if (!n || !n->lm) return fail(kBadHandle, "zilla_lm_set_precision: %d is not a language model", net);
    if (precision != 0 && precision != 1) return fail(kBadArg, "zilla_lm_set_precision: precision %d", precision);
    if (precision == 1 && n->lm->tcg.empty()) {
        cudaStreamSynchronize(stream());
        int rc = lm_tc_build(*n, *n->lm);
        if (rc) {
            n->lm->tcg.clear();
            return rc;
        }
    }
    cudaStreamSynchronize(stream());
    release_graphs(*n);   // captured steps carry the other kernels
    n->precision = precision;
    return check_cuda("zilla_lm_set_precision");
}

extern "C" int zilla_lm_cache_reset(int net) {
    Net *n = net_get(net);
    if (!n || !n->lm) return fail(kBadHandle, "zilla_lm_cache_reset: %d is not a language model", net);
    n->lm->cache_len = 0;
    return kOk;
}

extern "C" int zilla_lm_cache_length(int net) {
    Net *n = net_get(net);
    if (!n || !n->lm) return fail(kBadHandle, "zilla_lm_cache_length: %d is not a language model", net);
    return n->lm->cache_len;
}

extern "C" int zilla_lm_forward_cached(int net, const float *tokens, int count, float *logits) {
    Net *n = net_get(net);
    if (!n || !n->lm) return fail(kBadHandle, "zilla_lm_forward_cached: %d is not a language model", net);
    return lm_forward_cached(*n, tokens, count, logits);
}
