// tc_conv.cuh -- implicit-GEMM 3x3 (stride 1, pad 1) convolution on tcgen05.
//
// D[pixel, n] = sum_{tap, c} IN[pixel + tap offset, c] * Wt[tap][n][c]
//   forward:        IN = activations x (NHWC bf16), Wt[tap][co][ci] = W[co][ci][tap]
//   input gradient: IN = dY (NHWC bf16),            Wt[tap][ci][co] = W[co][ci][8 - tap]
// (the input gradient of a stride-1, pad-1 3x3 conv is the same convolution
// of dY with the flipped, channel-transposed kernel).
//
// Tile: R full image rows x W columns of one image (M = R*W <= 128 pixels,
// MMA M = 128; the rows past R*W are ignored).  K = 9 taps x CIN channels.
// For each tap the producer issues one TMA box per 64-channel chunk:
//   box {chunk, W, R, 1} at (c0, dw - 1, h0 + dh - 1, b)
// whose out-of-image elements are zero-filled by TMA: that is the padding.
// The packed weights of all 9 taps stay resident in shared memory.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer and TMEM
// owner, warps 2-5 epilogue (TMEM lane quarter = warp % 4).  Accumulators
// are double-buffered in TMEM so the epilogue of tile i overlaps the MMAs of
// tile i+1.
//
// Epilogues:
//   kEpiPool : relu(acc + bias), 2x2/2 max-pool with the reference tie rule
//              (first maximum in (kh, kw) order, native/cpu/zilla_cpu.c:215-224),
//              pooled bf16 NHWC out + a code byte per output
//              (window position 0..3 | (max > 0) << 2), which is all the
//              backward needs (argmax and the ReLU mask).
//   kEpiStore: relu(acc + bias) -> bf16 NHWC (conv without a following pool).
//   kEpiDgrad: acc [* (mask > 0)] -> bf16 NHWC (input gradient; the mask is
//              the previous layer's ReLU output).
#pragma once

#include "tc_common.cuh"

namespace zb {
namespace tc {

enum ConvEpi { kEpiPool = 0, kEpiStore = 1, kEpiDgrad = 2 };

struct ConvTcParams {
    CUtensorMap in_map;   // 4D {CIN, W, H, B} bf16, box {chunk, W, R, 1}
    CUtensorMap w_map;    // 3D {CIN, COUT, 9} bf16, box {chunk, COUT, 1}
    int B, H, W, R, tiles_per_img, num_tiles;
    const float *bias;          // [COUT] (forward)
    __nv_bfloat16 *out;         // pooled [B, H/2, W/2, COUT] or full [B, H, W, COUT]
    uint8_t *code;              // [B, H/2, W/2, COUT] (kEpiPool)
    const __nv_bfloat16 *mask;  // [B, H, W, COUT] or null (kEpiDgrad)
    int *err;
};

// SB ("stream B"): instead of keeping all 9 taps of packed weights resident,
// each pipeline stage carries its tap's weight slice next to the activation
// box.  For wide layers (64 -> 128) the resident weights would take 147 KB
// and leave room for only two or three stages.
template <int CIN, int COUT, int NS, bool POOL, bool SB = false>
struct ConvTcShape {
    static constexpr int CHUNK = CIN > 64 ? 64 : CIN;
    static constexpr int NCH = CIN / CHUNK;
    static constexpr int ROWB = CHUNK * 2;
    static constexpr Swizzle SW = ROWB == 128 ? kSw128 : (ROWB == 64 ? kSw64 : kSw32);
    static constexpr int ABLK = 128 * ROWB;
    static constexpr int BBLK = COUT * ROWB;
    static constexpr int AONLY = NCH * ABLK;                       // activation part of a stage
    static constexpr int ASTAGE = AONLY + (SB ? NCH * BBLK : 0);   // whole stage
    static constexpr int BTOTAL = SB ? 0 : 9 * NCH * BBLK;          // resident weights
    static constexpr int STAGE_F = 36;   // fp32 staging row pitch: 144 B, 16-byte aligned and
                                         // conflict-free for 128-bit accesses of 8 rows
    static constexpr int POOL_STAGE = POOL ? 128 * STAGE_F * 4 : 0;
    static constexpr uint32_t TMEM_COLS = (2 * COUT <= 32) ? 32 : (2 * COUT <= 64) ? 64 : (2 * COUT <= 128) ? 128 : (2 * COUT <= 256) ? 256 : 512;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = 1024 /*align slack*/ + BTOTAL + NS * ASTAGE + POOL_STAGE + BAR_BYTES;
    static_assert(CIN % 16 == 0 && COUT % 32 == 0 && COUT <= 256, "unsupported conv channels");
    static_assert(CIN <= 64 || CIN % 64 == 0, "CIN above 64 must be a multiple of 64");
};

template <int CIN, int COUT, int EPI, int NS, bool SB = false>
__global__ void __launch_bounds__(192, 1) conv_tc_kernel(const __grid_constant__ ConvTcParams p) {
    using S = ConvTcShape<CIN, COUT, NS, EPI == kEpiPool, SB>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sB = base;
    uint8_t *sA = sB + S::BTOTAL;
    float *stage = reinterpret_cast<float *>(sA + NS * S::ASTAGE);
    uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(stage) + S::POOL_STAGE);
    uint64_t *full = bars;               // [NS]
    uint64_t *empty = bars + NS;         // [NS]
    uint64_t *acc_full = bars + 2 * NS;  // [2]
    uint64_t *acc_empty = acc_full + 2;  // [2]
    uint64_t *wbar = acc_empty + 2;
    uint64_t *drain = wbar + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *armed = const_cast<int *>(abort_flag) + 1;   // [NS] parity+1 of the latest arm (0 = never)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t IDESC = idesc_bf16(128, COUT, false, false);

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); armed[i] = 0; }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
        mbar_init(wbar, 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t box_bytes = (uint32_t)(p.R * p.W * S::ROWB);

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (elect_one()) {
            prefetch_tmap(&p.in_map);
            prefetch_tmap(&p.w_map);
            if constexpr (!SB) {
                mbar_arrive_expect_tx(wbar, S::BTOTAL);
                for (int t = 0; t < 9; ++t)
                    for (int j = 0; j < S::NCH; ++j)
                        tma_load_3d(sB + (t * S::NCH + j) * S::BBLK, &p.w_map, wbar, j * S::CHUNK, 0, t);
            }
            const uint32_t stage_tx = box_bytes * S::NCH + (SB ? S::NCH * S::BBLK : 0);
            int s = 0;
            uint32_t ph = 0;
            for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
                const int b = tile / p.tiles_per_img;
                const int h0 = (tile - b * p.tiles_per_img) * p.R;
                for (int tap = 0; tap < 9; ++tap) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
                    mbar_arrive_expect_tx(&full[s], stage_tx);
                    armed[s] = (int)ph + 1;
                    const int dh = tap / 3, dw = tap - 3 * dh;
                    for (int j = 0; j < S::NCH; ++j)
                        tma_load_4d(sA + s * S::ASTAGE + j * S::ABLK, &p.in_map, &full[s], j * S::CHUNK, dw - 1,
                                    h0 + dh - 1, b);
                    if constexpr (SB)
                        for (int j = 0; j < S::NCH; ++j)
                            tma_load_3d(sA + s * S::ASTAGE + S::AONLY + j * S::BBLK, &p.w_map, &full[s],
                                        j * S::CHUNK, 0, tap);
                    if (++s == NS) { s = 0; ph ^= 1u; }
                }
            }
            if (*abort_flag) {   // let every copy this thread started land before exit
                for (int i = 0; i < NS; ++i)
                    if (armed[i] && !mbar_wait_drain(&full[i], (uint32_t)(armed[i] - 1)))
                        atomicCAS(p.err, 0, kErrDrain);
                if (!SB && !mbar_wait_drain(wbar, 0)) atomicCAS(p.err, 0, kErrDrain);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (elect_one()) {
            bool issued = false;
            if (SB || mbar_wait(wbar, 0, abort_flag, p.err, kErrFullWait)) {
                int s = 0, acc = 0;
                uint32_t ph = 0, acc_ph = 0;
                const uint32_t sA0 = smem_u32(sA), sB0 = smem_u32(sB);
                for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
                    if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag, p.err, kErrAccWait)) break;
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(acc * COUT);
                    bool ok = true;
                    for (int tap = 0; tap < 9; ++tap) {
                        if (!mbar_wait(&full[s], ph, abort_flag, p.err, kErrFullWait)) { ok = false; break; }
                        tc_fence_after();
#pragma unroll
                        for (int j = 0; j < S::NCH; ++j)
#pragma unroll
                            for (int k = 0; k < S::CHUNK / 16; ++k) {
                                const uint64_t ad = smem_desc(sA0 + s * S::ASTAGE + j * S::ABLK + k * 32, 16,
                                                              8 * S::ROWB, S::SW);
                                const uint32_t bsrc = SB ? sA0 + s * S::ASTAGE + S::AONLY + j * S::BBLK
                                                         : sB0 + (tap * S::NCH + j) * S::BBLK;
                                const uint64_t bd = smem_desc(bsrc + k * 32, 16, 8 * S::ROWB, S::SW);
                                mma_bf16(d, ad, bd, IDESC, (tap | j | k) != 0);
                            }
                        issued = true;
                        mma_commit(&empty[s]);
                        if (++s == NS) { s = 0; ph ^= 1u; }
                    }
                    if (!ok) break;
                    mma_commit(&acc_full[acc]);
                    if (++acc == 2) { acc = 0; acc_ph ^= 1u; }
                }
            }
            if (issued) {   // wait for every MMA this thread issued before TMEM is freed
                mma_commit(drain);
                if (!mbar_wait_drain(drain, 0)) atomicCAS(p.err, 0, kErrDrain);
            }
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..5)
        const int q = warp & 3;
        const int row = q * 32 + lane;          // accumulator row = pixel within the tile
        const int ep_tid = threadIdx.x - 64;    // 0..127
        int acc = 0;
        uint32_t acc_ph = 0;
        // The four epilogue warps leave the tile loop together: the abort flag is
        // only consulted right after a named barrier, so a warp can never wait
        // at a barrier that another epilogue warp has already left.
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            const int b = tile / p.tiles_per_img;
            const int h0 = (tile - b * p.tiles_per_img) * p.R;
            mbar_wait(&acc_full[acc], acc_ph, abort_flag, p.err, kErrAccWait);
            named_bar_sync(1, 128);
            if (*abort_flag) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * COUT);
            const int r = row / p.W, c = row - (row / p.W) * p.W;
            const int h = h0 + r;
            const bool pix_ok = (row < p.R * p.W) && (h < p.H);
            if constexpr (EPI == kEpiPool) {
                const int Ho = p.H >> 1, Wo = p.W >> 1;
                const int nwin = (p.R >> 1) * Wo;
#pragma unroll 1
                for (int cc = 0; cc < COUT / 32; ++cc) {
                    float v[32];
                    tmem_ld32(taddr + 32 * cc, v);
                    if (cc == COUT / 32 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[acc]);
                    }
                    // bias + ReLU, the row's 32 channels as eight 16-byte stores
                    float4 *srow = reinterpret_cast<float4 *>(stage + row * S::STAGE_F);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        float4 t;
                        t.x = fmaxf(v[4 * k + 0] + __ldg(p.bias + 32 * cc + 4 * k + 0), 0.0f);
                        t.y = fmaxf(v[4 * k + 1] + __ldg(p.bias + 32 * cc + 4 * k + 1), 0.0f);
                        t.z = fmaxf(v[4 * k + 2] + __ldg(p.bias + 32 * cc + 4 * k + 2), 0.0f);
                        t.w = fmaxf(v[4 * k + 3] + __ldg(p.bias + 32 * cc + 4 * k + 3), 0.0f);
                        srow[k] = t;
                    }
                    named_bar_sync(1, 128);
                    // thread = (window, channel octet): four pixels x 8 channels
                    for (int idx = ep_tid; idx < nwin * 4; idx += 128) {
                        const int wi = idx >> 2, o = idx & 3;
                        const int pr = wi / Wo, pc = wi - pr * Wo;
                        const int ho = (h0 >> 1) + pr;
                        if (ho >= Ho) continue;
                        const int r0 = (2 * pr) * p.W + 2 * pc;
                        const int rr[4] = {r0, r0 + 1, r0 + p.W, r0 + p.W + 1};
                        float best[8];
                        int pos[8];
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {   // (kh, kw) order: first maximum wins
                            const float4 *src = reinterpret_cast<const float4 *>(stage + rr[q4] * S::STAGE_F + 8 * o);
                            const float4 lo = src[0], hi = src[1];
                            const float vv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                if (q4 == 0 || vv[e] > best[e]) { best[e] = vv[e]; pos[e] = q4; }
                            }
                        }
                        uint4 pk;
                        __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                        for (int e = 0; e < 4; ++e) h2[e] = __floats2bfloat162_rn(best[2 * e], best[2 * e + 1]);
                        uint2 cd;
                        uint8_t *cb = reinterpret_cast<uint8_t *>(&cd);
#pragma unroll
                        for (int e = 0; e < 8; ++e) cb[e] = (uint8_t)(pos[e] | (best[e] > 0.0f ? 4 : 0));
                        const size_t o8 = (((size_t)b * Ho + ho) * Wo + pc) * COUT + 32 * cc + 8 * o;
                        *reinterpret_cast<uint4 *>(p.out + o8) = pk;
                        *reinterpret_cast<uint2 *>(p.code + o8) = cd;
                    }
                    named_bar_sync(1, 128);
                }
            } else {
#pragma unroll 1
                for (int cc = 0; cc < COUT / 32; ++cc) {
                    float v[32];
                    tmem_ld32(taddr + 32 * cc, v);
                    if (cc == COUT / 32 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[acc]);
                    }
                    if (!pix_ok) continue;
                    const size_t o = (((size_t)b * p.H + h) * p.W + c) * COUT + 32 * cc;
                    if constexpr (EPI == kEpiStore) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float x = v[j] + __ldg(p.bias + 32 * cc + j);
                            v[j] = x > 0.0f ? x : 0.0f;
                        }
                    } else if (p.mask) {
                        const uint4 *mk = reinterpret_cast<const uint4 *>(p.mask + o);
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            uint4 m = __ldg(mk + q4);
                            const __nv_bfloat16 *mb = reinterpret_cast<const __nv_bfloat16 *>(&m);
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                if (!(__bfloat162float(mb[e]) > 0.0f)) v[q4 * 8 + e] = 0.0f;
                        }
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + o);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint4 pk;
                        __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                        for (int e = 0; e < 4; ++e) h2[e] = __floats2bfloat162_rn(v[q4 * 8 + 2 * e], v[q4 * 8 + 2 * e + 1]);
                        dst[q4] = pk;
                    }
                }
            }
            if (++acc == 2) { acc = 0; acc_ph ^= 1u; }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, S::TMEM_COLS);
}

}  // namespace tc
}  // namespace zb
