// tc_attn_tf32.cuh -- the language model's causal attention on TF32 tensor
// cores (tcgen05 kind::tf32, fp32 accumulation in TMEM): one CTA per
// (sequence, head), sequence length T <= 128 (one 128-row tile), head dim 32.
//
// Forward (MultiHeadAttention::forward, src/Attention/MultiHeadAttention.php:41-80):
//   S = Q K^T                  M = 128 queries, N = 128 keys, K = 32
//   P = softmax(maskfill(S * scale, -1e9 above the diagonal)) per query row
//   O = P V                    M = 128 queries, N = 32, K = 128 keys
// Four threads own each query row (TMEM lane = row, a quarter of the keys
// each): the row softmax runs in registers, P goes to shared memory as the A
// operand of O = P V, and the row's max and exp-sum are kept ([B*H][T][2])
// instead of P itself.
//
// Backward, with Dr[q] = dO[q] . O[q] (= sum_j P[q][j] dP[q][j]):
//   S, dP = dO V^T             recomputed / computed by two MMAs
//   P from S and the kept max and sum (the forward's exact arithmetic, so the
//   same values), dS = P (dP - Dr) scale
//   dV = P^T dO,  dQ = dS K,  dK = dS^T Q   (M = 128, N = 32, K = 128)
// P^T, dS and dS^T are written by the row threads into shared memory in the
// K-major layout; a thread's transposed writes fall in 32 different banks.
//
// Operand layouts (see tc_gemm_tf32.cuh): tiles come from the row-major fp32
// tensors through TMA, box {32 floats, 128 rows}.  K-major tiles (A or B read
// along the head dim): 128-byte swizzle, row r at r * 128 bytes with its
// 16-byte chunks XOR (r & 7); a K8 step is 32 bytes along the row.  MN-major
// tiles (B read along the rows, N = the head dim): 128-byte swizzle over
// 32-byte atoms; a K8 step is 8 rows (1024 bytes), 4-row groups 512 bytes apart.
// Thread-written K-major operands with K = 128 are four 32-float atoms of
// [128 rows][128 bytes], 16 KB apart.
//
// Rows past T (a short last tile) read zeros or the next sequence's rows;
// their keys are masked for every real query, their query rows are dropped in
// the backward (P = dS = 0) and never stored.  Every wait is bounded.
#pragma once

#include "tc_gemm_tf32.cuh"

namespace zb {
namespace tc {

struct AttnTcParams {
    CUtensorMap qkv_k;    // qkv [N][3D] fp32, box {32, 128}, 128-byte swizzle
    CUtensorMap qkv_mn;   // the same tensor, box {32, 128}, 128-byte swizzle over 32-byte atoms
    CUtensorMap do_k;     // backward: dO [N][D], box {32, 128}, 128-byte swizzle
    CUtensorMap do_mn;    // backward: dO, 128-byte swizzle over 32-byte atoms
    const float *O;       // backward: the forward's output [N][D]
    const float *dO;      // backward: dO [N][D]
    float *out;           // forward: O [N][D]; backward: dqkv [N][3D]
    float *stats;         // [B*H][T][2]: max and exp-sum of each scaled, masked score row
    int T, H, D;
    float scale;
    int *err;
};

constexpr int kAttnTile = 16384;                           // one 128 x 32 fp32 tile
constexpr int kAttnRed = 4096;                             // row reductions over the four key quarters
constexpr int kAttnFwdSmem = 5 * kAttnTile + kAttnRed + 64 + 1024;    // P (4 tiles, the first two over Q, K), V
constexpr int kAttnBwdSmem = 11 * kAttnTile + kAttnRed + 64 + 1024;   // Q K V dO | P^T, dS^T | dO K Q (MN)

// Element (r, k) of a thread-written K-major operand with K = 128.
__device__ __forceinline__ uint32_t attn_kmajor_off(int r, int k) {
    return (uint32_t)((k >> 5) * kAttnTile + r * 128 + ((((k & 31) >> 2) ^ (r & 7)) << 4) + (k & 3) * 4);
}

// One 128-row score row of the forward or its recomputation in the backward:
// scaled, masked (keys after the query), as the reference's maskedFill(-1e9).
__device__ __forceinline__ float attn_score(float s, int j, int q, float scale) {
    return j > q ? -1e9f : s * scale;
}

// 512 threads: warp w reads TMEM lanes 32 (w & 3) .. + 31 (the query rows q) and
// takes the 32 keys of column quarter c = w >> 2 of each row, so a row's
// softmax is four threads' work, combined through shared memory in quarter
// order (a fixed order: deterministic).  P = e * (1 / sum): the backward
// recomputes it from the same max and sum with the same two operations.
__global__ void __launch_bounds__(512, 2) attn_fwd_tc_kernel(const __grid_constant__ AttnTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sQ = base, *sK = base + kAttnTile, *sP = base, *sV = base + 4 * kAttnTile;
    float *red = reinterpret_cast<float *>(base + 5 * kAttnTile);   // [2][4][128]: quarter maxima, sums
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + 5 * kAttnTile + kAttnRed);
    uint64_t *tma_bar = bars, *mma1 = bars + 1, *mma2 = bars + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int bh = blockIdx.x, b = bh / p.H, h = bh - b * p.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = (warp & 3) * 32 + lane, c = warp >> 2;   // query row, key quarter
    const int row0 = b * p.T;
    if (threadIdx.x == 0) {
        mbar_init(tma_bar, 1);
        mbar_init(mma1, 1);
        mbar_init(mma2, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    int committed = 0;   // thread 0: MMA groups committed (drained before TMEM is freed)
    if (threadIdx.x == 0) {
        prefetch_tmap(&p.qkv_k);
        prefetch_tmap(&p.qkv_mn);
        mbar_arrive_expect_tx(tma_bar, 3 * kAttnTile);
        tma_load_2d(sQ, &p.qkv_k, tma_bar, h * 32, row0);
        tma_load_2d(sK, &p.qkv_k, tma_bar, p.D + h * 32, row0);
        tma_load_2d(sV, &p.qkv_mn, tma_bar, 2 * p.D + h * 32, row0);
        if (mbar_wait(tma_bar, 0, abort_flag, p.err, kErrFullWait)) {
            tc_fence_after();
            constexpr uint32_t ID_S = idesc_tf32(128, 128, false, false);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                mma_tf32(tmem, smem_desc(smem_u32(sQ) + kk * 32, 16, 1024, kSw128),
                         smem_desc(smem_u32(sK) + kk * 32, 16, 1024, kSw128), ID_S, kk != 0);
            mma_commit(mma1);
            committed = 1;
        } else if (!mbar_wait_drain(tma_bar, 0)) {
            atomicCAS(p.err, 0, kErrDrain);
        }
    }
    const bool ok1 = mbar_wait(mma1, 0, abort_flag, p.err, kErrAccWait);
    tc_fence_after();
    float s[32];
    const bool live = 32 * c <= q;   // some key of this quarter is at or before the query
    float mx = -INFINITY;
    if (ok1) {
        tmem_ld32(trow + 32 * c, s);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            s[i] = attn_score(s[i], 32 * c + i, q, p.scale);
            mx = fmaxf(mx, s[i]);
        }
    }
    red[c * 128 + q] = mx;
    __syncthreads();
    const float m = fmaxf(fmaxf(red[q], red[128 + q]), fmaxf(red[256 + q], red[384 + q]));
    float sum = 0.0f;
    if (live) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            s[i] = expf(s[i] - m);
            sum += s[i];
        }
    }
    red[512 + c * 128 + q] = sum;
    __syncthreads();
    const float tot = ((red[512 + q] + red[640 + q]) + red[768 + q]) + red[896 + q];
    const float inv = 1.0f / tot;
    // this quarter of P row q (K-major: row q, k = key) over the Q and K tiles, which the MMAs have read
#pragma unroll
    for (int i4 = 0; i4 < 8; ++i4)
        *reinterpret_cast<float4 *>(sP + attn_kmajor_off(q, 32 * c + 4 * i4)) =
            live ? make_float4(s[4 * i4] * inv, s[4 * i4 + 1] * inv, s[4 * i4 + 2] * inv, s[4 * i4 + 3] * inv)
                 : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (c == 0 && q < p.T) *reinterpret_cast<float2 *>(p.stats + ((size_t)bh * p.T + q) * 2) = make_float2(m, tot);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && committed && !*abort_flag) {
        tc_fence_after();
        constexpr uint32_t ID_O = idesc_tf32(128, 32, false, true);
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
            mma_tf32(tmem + 128, smem_desc(smem_u32(sP) + (kk >> 2) * kAttnTile + (kk & 3) * 32, 16, 1024, kSw128),
                     smem_desc(smem_u32(sV) + kk * 1024, 4096, 512, kSw128B32), ID_O, kk != 0);
        mma_commit(mma2);
        committed = 2;
    }
    if (mbar_wait(mma2, 0, abort_flag, p.err, kErrAccWait) && c == 0) {
        tc_fence_after();
        float o[32];
        tmem_ld32(trow + 128, o);
        if (q < p.T) {
            float4 *dst = reinterpret_cast<float4 *>(p.out + (size_t)(row0 + q) * p.D + h * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        }
    }
    if (threadIdx.x == 0) {   // every MMA finished before TMEM goes (on an abort too)
        if (committed >= 1 && !mbar_wait_drain(mma1, 0)) atomicCAS(p.err, 0, kErrDrain);
        if (committed >= 2 && !mbar_wait_drain(mma2, 0)) atomicCAS(p.err, 0, kErrDrain);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

// 512 threads, the forward's row / key-quarter split: thread (q, c) takes keys
// 32c .. 32c + 31 of row q in every phase; the outputs dV, dQ, dK (TMEM
// columns 0, 32, 64) are read by the quarters 0, 1, 2.
__global__ void __launch_bounds__(512, 1) attn_bwd_tc_kernel(const __grid_constant__ AttnTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sQk = base, *sKk = base + kAttnTile, *sVk = base + 2 * kAttnTile, *sGk = base + 3 * kAttnTile;
    uint8_t *sY = base;                        // dS (K-major rows) over Q, K, V, dO once S and dP are taken
    uint8_t *sX = base + 4 * kAttnTile;        // P^T, then dS^T
    uint8_t *sGmn = base + 8 * kAttnTile, *sKmn = base + 9 * kAttnTile, *sQmn = base + 10 * kAttnTile;
    float *red = reinterpret_cast<float *>(base + 11 * kAttnTile);   // [4][128]: quarter parts of Dr
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + 11 * kAttnTile + kAttnRed);
    uint64_t *tma_bar = bars, *mma1 = bars + 1, *mma2 = bars + 2, *mma3 = bars + 3;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int bh = blockIdx.x, b = bh / p.H, h = bh - b * p.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = (warp & 3) * 32 + lane, c = warp >> 2;
    const int row0 = b * p.T;
    const bool valid = q < p.T;
    if (threadIdx.x == 0) {
        mbar_init(tma_bar, 1);
        mbar_init(mma1, 1);
        mbar_init(mma2, 1);
        mbar_init(mma3, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    int committed = 0;
    if (threadIdx.x == 0) {
        prefetch_tmap(&p.qkv_k);
        prefetch_tmap(&p.qkv_mn);
        prefetch_tmap(&p.do_k);
        prefetch_tmap(&p.do_mn);
        mbar_arrive_expect_tx(tma_bar, 7 * kAttnTile);
        tma_load_2d(sQk, &p.qkv_k, tma_bar, h * 32, row0);
        tma_load_2d(sKk, &p.qkv_k, tma_bar, p.D + h * 32, row0);
        tma_load_2d(sVk, &p.qkv_k, tma_bar, 2 * p.D + h * 32, row0);
        tma_load_2d(sGk, &p.do_k, tma_bar, h * 32, row0);
        tma_load_2d(sGmn, &p.do_mn, tma_bar, h * 32, row0);
        tma_load_2d(sKmn, &p.qkv_mn, tma_bar, p.D + h * 32, row0);
        tma_load_2d(sQmn, &p.qkv_mn, tma_bar, h * 32, row0);
        if (mbar_wait(tma_bar, 0, abort_flag, p.err, kErrFullWait)) {
            tc_fence_after();
            constexpr uint32_t ID_S = idesc_tf32(128, 128, false, false);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)   // S = Q K^T
                mma_tf32(tmem, smem_desc(smem_u32(sQk) + kk * 32, 16, 1024, kSw128),
                         smem_desc(smem_u32(sKk) + kk * 32, 16, 1024, kSw128), ID_S, kk != 0);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)   // dP = dO V^T
                mma_tf32(tmem + 128, smem_desc(smem_u32(sGk) + kk * 32, 16, 1024, kSw128),
                         smem_desc(smem_u32(sVk) + kk * 32, 16, 1024, kSw128), ID_S, kk != 0);
            mma_commit(mma1);
            committed = 1;
        } else if (!mbar_wait_drain(tma_bar, 0)) {
            atomicCAS(p.err, 0, kErrDrain);
        }
    }
    // row q's softmax statistics, and Dr = dO . O (each quarter eight of the 32 products)
    float m = 0.0f, inv = 0.0f, part = 0.0f;
    if (valid) {
        const float2 st = *reinterpret_cast<const float2 *>(p.stats + ((size_t)bh * p.T + q) * 2);
        m = st.x;
        inv = 1.0f / st.y;
        const float4 *g4 = reinterpret_cast<const float4 *>(p.dO + (size_t)(row0 + q) * p.D + h * 32 + 8 * c);
        const float4 *o4 = reinterpret_cast<const float4 *>(p.O + (size_t)(row0 + q) * p.D + h * 32 + 8 * c);
        const float4 g0 = g4[0], g1 = g4[1], o0 = o4[0], o1 = o4[1];
        part = g0.x * o0.x + g0.y * o0.y + g0.z * o0.z + g0.w * o0.w + g1.x * o1.x + g1.y * o1.y + g1.z * o1.z +
               g1.w * o1.w;
    }
    red[c * 128 + q] = part;
    __syncthreads();
    const float dr = ((red[q] + red[128 + q]) + red[256 + q]) + red[384 + q];
    const bool live = valid && 32 * c <= q;   // some key of this quarter is at or before the query
    if (mbar_wait(mma1, 0, abort_flag, p.err, kErrAccWait)) {
        tc_fence_after();
        float sv[32], dp[32];
        tmem_ld32(trow + 32 * c, sv);
        tmem_ld32(trow + 128 + 32 * c, dp);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int j = 32 * c + i;
            const float pj = live ? expf(attn_score(sv[i], j, q, p.scale) - m) * inv : 0.0f;
            sv[i] = pj * (dp[i] - dr) * p.scale;                           // dS[q][j]
            *reinterpret_cast<float *>(sX + attn_kmajor_off(j, q)) = pj;   // P^T: row key j, k = query q
        }
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4)   // dS row q (K-major: k = key) over the tiles the MMAs read
            *reinterpret_cast<float4 *>(sY + attn_kmajor_off(q, 32 * c + 4 * i4)) =
                make_float4(sv[4 * i4], sv[4 * i4 + 1], sv[4 * i4 + 2], sv[4 * i4 + 3]);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    constexpr uint32_t ID_G = idesc_tf32(128, 32, false, true);
    if (threadIdx.x == 0 && committed && !*abort_flag) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)   // dV = P^T dO  (TMEM columns 0..31, over S: read)
            mma_tf32(tmem, smem_desc(smem_u32(sX) + (kk >> 2) * kAttnTile + (kk & 3) * 32, 16, 1024, kSw128),
                     smem_desc(smem_u32(sGmn) + kk * 1024, 4096, 512, kSw128B32), ID_G, kk != 0);
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)   // dQ = dS K  (columns 32..63)
            mma_tf32(tmem + 32, smem_desc(smem_u32(sY) + (kk >> 2) * kAttnTile + (kk & 3) * 32, 16, 1024, kSw128),
                     smem_desc(smem_u32(sKmn) + kk * 1024, 4096, 512, kSw128B32), ID_G, kk != 0);
        mma_commit(mma2);
        committed = 2;
    }
    if (mbar_wait(mma2, 0, abort_flag, p.err, kErrAccWait)) {
        // dS^T over P^T (the dV MMAs have read it): this quarter of row q of dS, written as column q
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
            const int j = 32 * c + 4 * i4;
            const float4 v = *reinterpret_cast<const float4 *>(sY + attn_kmajor_off(q, j));
            *reinterpret_cast<float *>(sX + attn_kmajor_off(j, q)) = v.x;
            *reinterpret_cast<float *>(sX + attn_kmajor_off(j + 1, q)) = v.y;
            *reinterpret_cast<float *>(sX + attn_kmajor_off(j + 2, q)) = v.z;
            *reinterpret_cast<float *>(sX + attn_kmajor_off(j + 3, q)) = v.w;
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && committed == 2 && !*abort_flag) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)   // dK = dS^T Q  (columns 64..95)
            mma_tf32(tmem + 64, smem_desc(smem_u32(sX) + (kk >> 2) * kAttnTile + (kk & 3) * 32, 16, 1024, kSw128),
                     smem_desc(smem_u32(sQmn) + kk * 1024, 4096, 512, kSw128B32), ID_G, kk != 0);
        mma_commit(mma3);
        committed = 3;
    }
    if (mbar_wait(mma3, 0, abort_flag, p.err, kErrAccWait) && c < 3) {
        tc_fence_after();
        float v[32];
        tmem_ld32(trow + 32 * c, v);   // quarter 0: dV (key row q), 1: dQ (query row q), 2: dK (key row q)
        if (valid) {
            float4 *g = reinterpret_cast<float4 *>(p.out + (size_t)(row0 + q) * 3 * p.D + (c == 0 ? 2 * p.D : c == 1 ? 0 : p.D) +
                                                   h * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) g[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    }
    if (threadIdx.x == 0) {
        if (committed >= 1 && !mbar_wait_drain(mma1, 0)) atomicCAS(p.err, 0, kErrDrain);
        if (committed >= 2 && !mbar_wait_drain(mma2, 0)) atomicCAS(p.err, 0, kErrDrain);
        if (committed >= 3 && !mbar_wait_drain(mma3, 0)) atomicCAS(p.err, 0, kErrDrain);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace tc
}  // namespace zb
