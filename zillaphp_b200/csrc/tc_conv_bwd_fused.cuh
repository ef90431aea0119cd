// tc_conv_bwd_fused.cuh -- the whole backward of a 3x3 (stride 1, pad 1) conv
// whose input is a ReLU output, in one tcgen05 kernel: per tile it loads the
// dY halo tile and the X halo tile ONCE and runs both contractions on them.
//
//   input gradient  dX[pixel][ci] = (X > 0) * sum_{tap, co} dY[pixel - tap][co] Wd[tap][ci][co]
//   weight gradient dW[co][tap][ci] = sum_pixels dY[pixel][co] X[pixel + tap][ci]
//
// Tile: R image rows of one image with R * Wp = 128, Wp >= W + 2 (W = 28:
// Wp = 32, R = 4).  Both halo tiles hold rows h0-1 .. h0+R and columns
// -1 .. Wp-2 as 8-channel groups of 16-byte rows (zero outside the image), the
// canonical no-swizzle UMMA layout, which serves as
//   * K-major A of the input gradient (M = 128 output pixels i = r*Wp + c,
//     K = dY channels; tap (dh, dw) starts dh*Wp + dw rows further on), and
//   * MN-major A / B of the weight gradient (K = the 128 pixel rows
//     k = r*Wp + c; dY starts Wp + 1 rows in, X starts dh*Wp + dw rows in).
// With R * Wp = 128 every K row past the tile (c >= W) reads a zero halo column
// of dY, so the padding adds nothing, and every row read lies inside the tile.
// The ReLU mask of the input gradient comes from the X tile already in shared
// memory, so a stage is released only when both its MMAs and the epilogue's
// mask reads are done (two arrivals).
//
// The input gradient runs as Z[i][dw][ci] = sum_dh sum_co dY[i + dh*Wp][co]
// Wd[dh][dw][ci][co]: per kernel row dh and K16 step, ONE MMA with N = 3 * CX
// (the weight blocks of taps (dh, 0), (dh, 1), (dh, 2) lie back to back in
// shared memory, so one B descriptor covers the three columns dw), 12 MMAs
// per tile instead of 36 with N = CX; the epilogue adds
// dX[i] = Z[i][0] + Z[i+1][1] + Z[i+2][2] with warp shuffles (a warp is one
// tile row, and the columns c + dw of a real output stay inside it).  The
// MMAs come from one thread, whose issue rate bounds this kernel, so fewer,
// wider MMAs are what count.
//
// TMEM: the input gradient in two 128 x 3*CX accumulators (double-buffered: the
// epilogue of tile i overlaps the MMAs of tile i+1), the weight gradient in one
// 64-row x 9*CX accumulator that stays for the CTA's whole run (M = CY = 64:
// rows 16q .. 16q+15 in lanes 32q .. 32q+15), the first conv's in CX columns:
// 512 in all.  At the end each CTA writes its weight-gradient partial
// [cta][CY][9*CX]; a second kernel sums them in CTA order (deterministic).
//
// Warp roles (320 threads): warp 0 TMA producer, warp 1 MMA issuer and TMEM
// owner, warps 2-9 epilogue (input gradient: staged bf16 tile + TMA store, as
// conv_halo_kernel's kEpiDgrad; weight gradient partial at the end).  Every
// wait is bounded (tc_common.cuh).
//
// C1 (X is the ReLU output of a first conv with one input channel, 3x3, pad 1):
// that conv's weight gradient dW1[co][t] = sum_p dX[p][co] x[p + t] is taken here
// too, from the masked dX tile, so dX never goes to global memory.  The staged
// dX tile (rows = the R*W pixels, 64 bytes of 32 channels, 64-byte swizzle) is
// an MN-major UMMA operand with K = pixels; the second epilogue warp group
// builds the matching im2col tile of x (rows = pixels, 64 bf16: x_hi of the 9
// taps, 1.0 for the bias, x_lo of the 9 taps at 16.., with x = x_hi + x_lo so the
// fp32 input keeps its precision; 128-byte swizzle).  Once both are staged
// the epilogue marks the buffer ready, and the MMA thread, after the next
// tile's MMAs, issues the R*W/16 MMAs D1[64][32] += im2col^T dX (M = 64, N =
// 32); at the end D1's hi rows (+ bias) and lo rows go out as two [32][10]
// partials per CTA, which the deterministic split reduction adds.
//
// X is loaded three times per stage, the copies one and two columns further
// on (TMA boxes starting at columns -1, 0, +1; zero fill outside the image),
// at a uniform pitch after the first: so one MN-major B descriptor with N =
// 3 * CX starting at kernel row dh covers the taps (dh, 0), (dh, 1), (dh, 2),
// and the weight gradient takes 3 MMAs (M = CY, N = 96) per K16 step instead
// of 9 (N = CX), into accumulator columns (dh * 3 + dw) * CX + ci.
// The three weight-gradient MMAs of a K16 step share A (the dY rows): the first
// fills the tensor core's collector buffer with it and the other two read it
// from there, so shared memory serves A once per step instead of three times.
// Every MMA of the CTA comes from the one MMA thread, so nothing else is issued
// between them.
//
// UP (dY is the max-unpool of the pooled gradient dP [B, H/2, W/2, CY] by the
// pool codes [B, H/2, W/2, CY], byte = window position | 4 when routed): four
// more warps (10-13) build each stage's dY halo tile in shared memory from dP
// and the codes instead of a TMA load of dY, so dY never exists in global
// memory.  Work item = (pooled row of the halo, pooled column, 8-channel
// octet): one 16-byte dP load and one 8-byte code load give the 2 or 4
// 16-byte chunks of its 2x2 window that lie in the halo rows; a channel keeps
// its value at the position its code names and is zero at the other three.
// The halo columns outside the image are never written (zero since the
// start).  The dY octet pitch is the row block plus 16 bytes so that the
// octets of one pixel fall in different shared-memory banks.  The builders
// also sum the routed values of the tile's own pooled rows per channel: the
// bias gradient of this conv, one [CY] partial per CTA.
#pragma once

#include "tc_common.cuh"

namespace zb {
namespace tc {

struct ConvBwdFusedParams {
    CUtensorMap dy_map;   // 4D {CY, W, H, B} bf16, box {8, Wp, R + 2, 1}, no swizzle
    CUtensorMap x_map;    // 4D {CX, W, H, B} bf16, box {8, Wp, R + 2, 1}, no swizzle
    CUtensorMap w_map;    // 3D {CY, CX, 9} bf16 (flipped, transposed kernel), box {CY, CX, 1}, 128B swizzle
    CUtensorMap out_map;  // 4D {CX, W, H, B} bf16, box {CX, W, R, 1}, swizzle = CX * 2 bytes
    int B, H, W, R, Wp, tiles_per_img, num_tiles;
    int region, stage_bytes, out_tile_bytes;   // set by the launcher
    float *partial;       // [gridDim.x][CY][9 * CX]
    const float *x0;      // C1: the first conv's input [B, H, W] fp32
    float *c1_partial;    // C1: [gridDim.x * 2][CX][10] (9 taps, bias; x_hi and x_lo halves)
    int x9_bytes;         // C1: one im2col tile (R * W rows of 128 B, 1024-aligned)
    const __nv_bfloat16 *dp;   // UP: pooled gradient [B, H/2, W/2, CY]
    const uint8_t *code;       // UP: pool codes [B, H/2, W/2, CY]
    float *bias_partial;       // UP: [gridDim.x * 4][CY] (one slice per builder warp)
    int dy_region, x_off;      // dY octet pitch, offset of the X octets in a stage (set by the launcher)
    int *err;
};

template <int CX, int CY, int NS, bool C1 = false, bool UP = false>
struct ConvBwdFusedShape {
    static constexpr int THREADS = UP ? 448 : 320;
    static constexpr int NTOT = 9 * CX;
    static constexpr int DYG = CY / 8, XG = CX / 8;
    static constexpr int XCOPY = 3;                      // X at column offsets 0, +1, +2
    static constexpr int WROWB = CY * 2;                 // dgrad weight row: 128 B (CY = 64)
    static constexpr int WBLK = CX * WROWB;              // one tap
    static constexpr int WTOTAL = 9 * WBLK;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int ZCOLS = 3 * CX;                  // one input-gradient accumulator: Z[i][dw][ci]
    static constexpr int WG_COL0 = 2 * ZCOLS;             // weight-gradient columns start
    static constexpr int C1_COL0 = WG_COL0 + 9 * CX;      // first-conv weight-gradient columns (C1)
    static constexpr int SLACK = 1024;
    static constexpr int BAR_BYTES = 256;
    static __host__ __device__ int region(int R, int Wp) { return ((R + 2) * Wp * 16 + 127) / 128 * 128; }
    static __host__ __device__ int dy_region(int R, int Wp) { return region(R, Wp) + (UP ? 16 : 0); }
    static __host__ __device__ int x_off(int R, int Wp) { return (DYG * dy_region(R, Wp) + 127) / 128 * 128; }
    static __host__ __device__ int stage_bytes(int R, int Wp) { return (x_off(R, Wp) + XCOPY * XG * region(R, Wp) + 1023) / 1024 * 1024; }
    static __host__ __device__ int out_tile_bytes(int R, int W) { return (R * W * CX * 2 + 1023) / 1024 * 1024; }
    static __host__ __device__ int x9_bytes(int R, int W) { return C1 ? (R * W * 128 + 1023) / 1024 * 1024 : 0; }
    static __host__ __device__ int smem(int R, int Wp, int W) {
        return 1024 + WTOTAL + NS * stage_bytes(R, Wp) + SLACK + 2 * (out_tile_bytes(R, W) + x9_bytes(R, W)) + BAR_BYTES;
    }
    static_assert(CY == 64 && CX == 32, "built for the 32 -> 64 conv: M = 64 weight gradient, N = 32 input gradient");
    static_assert(2 * ZCOLS + NTOT + (C1 ? CX : 0) <= 512, "TMEM columns");
};

template <int CX, int CY, int NS, bool C1 = false, bool UP = false>
__global__ void __launch_bounds__(UP ? 448 : 320, 1) conv_bwd_fused_kernel(const __grid_constant__ ConvBwdFusedParams p) {
    griddep_launch();
    using S = ConvBwdFusedShape<CX, CY, NS, C1, UP>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sW = base;
    uint8_t *sA = sW + S::WTOTAL;
    const int STAGE = p.stage_bytes;
    uint8_t *outbuf = sA + NS * STAGE + S::SLACK;   // [2] staged input-gradient tiles (+ im2col tiles, C1)
    const int OBUF = p.out_tile_bytes + (C1 ? p.x9_bytes : 0);   // one buffer: [dX tile][im2col tile]
    uint64_t *bars = reinterpret_cast<uint64_t *>(outbuf + 2 * OBUF);
    uint64_t *full = bars;               // [NS]
    uint64_t *empty = bars + NS;         // [NS]: MMA commit + epilogue mask release
    uint64_t *acc_full = bars + 2 * NS;  // [2]
    uint64_t *acc_empty = acc_full + 2;  // [2]
    uint64_t *wbar = acc_empty + 2;
    uint64_t *wg_full = wbar + 1;
    uint64_t *drain = wg_full + 1;
    uint64_t *c1_done = drain + 1;       // [2] (C1): the first-conv MMAs reading buffer i finished
    uint64_t *c1_ready = c1_done + 2;    // [2] (C1): buffer i's dX and im2col tiles are staged
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(c1_ready + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *armed = const_cast<int *>(abort_flag) + 1;   // [NS]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t IDESC_DX = idesc_bf16(128, 3 * CX, false, false);   // N = the three columns dw
    constexpr uint32_t IDESC_DW = idesc_bf16(CY, 3 * CX, true, true);   // N = the taps (dh, 0..2)
    const int my_tiles = p.num_tiles > (int)blockIdx.x ? (p.num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    for (int i = threadIdx.x; i < (NS * STAGE + S::SLACK) / 16; i += blockDim.x)
        *reinterpret_cast<uint4 *>(sA + 16 * i) = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

    if (threadIdx.x == 0) {
        // full: the TMA transaction arrival (+ one per builder warp, UP)
        for (int i = 0; i < NS; ++i) { mbar_init(&full[i], UP ? 5 : 1); mbar_init(&empty[i], 2); armed[i] = 0; }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 8); }
        mbar_init(wbar, 1);
        mbar_init(wg_full, 1);
        mbar_init(drain, 1);
        mbar_init(&c1_done[0], 1);
        mbar_init(&c1_done[1], 1);
        mbar_init(&c1_ready[0], 1);
        mbar_init(&c1_ready[1], 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, S::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_wait();   // everything below may touch global memory

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (elect_one()) {
            if (!UP) prefetch_tmap(&p.dy_map);
            prefetch_tmap(&p.x_map);
            prefetch_tmap(&p.w_map);
            prefetch_tmap(&p.out_map);
            mbar_arrive_expect_tx(wbar, S::WTOTAL);
            for (int t = 0; t < 9; ++t) tma_load_3d(sW + t * S::WBLK, &p.w_map, wbar, 0, 0, t);
            const uint32_t tx = (uint32_t)(((UP ? 0 : S::DYG) + S::XCOPY * S::XG) * (p.R + 2) * p.Wp * 16);
            int s = 0;
            uint32_t ph = 0;
            for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
                const int b = tile / p.tiles_per_img;
                const int h0 = (tile - b * p.tiles_per_img) * p.R;
                if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
                mbar_arrive_expect_tx(&full[s], tx);
                armed[s] = (int)ph + 1;
                uint8_t *st = sA + s * STAGE;
                if (!UP)
                    for (int g = 0; g < S::DYG; ++g)
                        tma_load_4d(st + g * p.dy_region, &p.dy_map, &full[s], 8 * g, -1, h0 - 1, b);
                for (int c = 0; c < S::XCOPY; ++c)   // X, then the copies one and two columns on
                    for (int g = 0; g < S::XG; ++g)
                        tma_load_4d(st + p.x_off + (c * S::XG + g) * p.region, &p.x_map, &full[s], 8 * g, c - 1,
                                    h0 - 1, b);
                if (++s == NS) { s = 0; ph ^= 1u; }
            }
            if (*abort_flag) {
                for (int i = 0; i < NS; ++i)
                    if (armed[i] && !mbar_wait_drain(&full[i], (uint32_t)(armed[i] - 1))) atomicCAS(p.err, 0, kErrDrain);
                if (!mbar_wait_drain(wbar, 0)) atomicCAS(p.err, 0, kErrDrain);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (elect_one()) {
            bool issued = false;
            if (mbar_wait(wbar, 0, abort_flag, p.err, kErrFullWait)) {
                int s = 0, acc = 0;
                uint32_t ph = 0, acc_ph = 0;
                const uint32_t lbo = (uint32_t)p.dy_region, reg16 = lbo >> 4;
                // descriptors differ only in the start address (16-byte units)
                const uint64_t dx_a0 = smem_desc(smem_u32(sA), lbo, 128, kSwNone);          // K-major dY
                const uint64_t dx_b0 = smem_desc(smem_u32(sW), 16, 8 * S::WROWB, kSw128);   // weights
                const uint64_t dw_a0 = smem_desc(smem_u32(sA), 128, lbo, kSwNone);          // MN-major dY
                const uint64_t dw_b0 = smem_desc(smem_u32(sA) + (uint32_t)p.x_off, 128, (uint32_t)p.region, kSwNone);
                const uint32_t wp = (uint32_t)p.Wp;
                // C1: the first conv's weight-gradient MMAs of the CTA's m-th tile, once the
                // epilogue has staged buffer m & 1 (this thread issues every MMA of the CTA, so
                // no other MMA lands inside a run that keeps A in the collector buffer)
                auto issue_c1 = [&](int m) -> bool {
                    const int b1 = m & 1;
                    if (!mbar_wait(&c1_ready[b1], (uint32_t)((m >> 1) & 1), abort_flag, p.err, kErrAccWait)) return false;
                    tc_fence_after();
                    constexpr uint32_t IDESC_C1 = idesc_bf16(64, CX, true, true);
                    const uint32_t xa = smem_u32(outbuf + b1 * OBUF + p.out_tile_bytes);
                    const uint32_t db = smem_u32(outbuf + b1 * OBUF);
                    const int ksteps = (p.R * p.W) / 16;
                    for (int k = 0; k < ksteps; ++k)
                        mma_bf16(tmem_base + (uint32_t)S::C1_COL0, smem_desc(xa + k * 2048, 16, 1024, kSw128),
                                 smem_desc(db + k * 1024, 16, 512, kSw64), IDESC_C1, (m | k) != 0);
                    mma_commit(&c1_done[b1]);
                    return true;
                };
                int n = 0;
                bool c1_ok = true;
                for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x, ++n) {
                    if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag, p.err, kErrAccWait)) break;
                    if (!mbar_wait(&full[s], ph, abort_flag, p.err, kErrFullWait)) break;
                    tc_fence_after();
                    const uint64_t st16 = (uint64_t)((uint32_t)(s * STAGE) >> 4);
                    // input gradient: Z[i][dw][ci] = sum_dh dY[i + dh*Wp] Wd[dh][dw] (3 kernel rows x
                    // CY/16 K16 steps).  The weight blocks of taps (dh, 0..2) lie back to back in
                    // shared memory, so one MMA with N = 3 * CX takes all three columns dw into
                    // accumulator columns dw * CX + ci.  The epilogue forms
                    // dX[i] = sum_dw Z[i + dw][dw] (a shift along the tile row).
                    const uint32_t d = tmem_base + (uint32_t)(acc * S::ZCOLS);
#pragma unroll
                    for (int dh = 0; dh < 3; ++dh) {
                        const uint64_t a_dh = dx_a0 + st16 + (uint64_t)(dh * wp);
#pragma unroll
                        for (int k = 0; k < CY / 16; ++k) {
                            const uint64_t ad = a_dh + (uint64_t)(2 * k * reg16);
                            const uint64_t bd = dx_b0 + (uint64_t)((uint32_t)(dh * 3 * S::WBLK + k * 32) >> 4);
                            mma_bf16(d, ad, bd, IDESC_DX, (dh | k) != 0);
                        }
                    }
                    mma_commit(&acc_full[acc]);
                    if (++acc == 2) { acc = 0; acc_ph ^= 1u; }
                    // weight gradient: 8 K16 steps (128 pixel rows) x 3 kernel rows (N = the three
                    // taps of the row, from the X copies); the 3 MMAs of a K16 step share A (dY),
                    // which stays in the collector buffer after the first, so shared memory
                    // serves it once instead of three times
                    const uint64_t a_dy = dw_a0 + st16 + (uint64_t)(wp + 1);
#pragma unroll 1
                    for (int k = 0; k < 8; ++k) {
                        const uint64_t ad = a_dy + (uint64_t)(16 * k);
#pragma unroll
                        for (int dh = 0; dh < 3; ++dh) {
                            const uint32_t dt = tmem_base + (uint32_t)(S::WG_COL0 + dh * 3 * CX);
                            const uint64_t bd = dw_b0 + st16 + (uint64_t)(dh * wp + 16 * k);
                            if (dh == 0) mma_bf16_ca<0>(dt, ad, bd, IDESC_DW, (n | k) != 0);
                            else if (dh == 1) mma_bf16_ca<1>(dt, ad, bd, IDESC_DW, (n | k) != 0);
                            else mma_bf16_ca<2>(dt, ad, bd, IDESC_DW, (n | k) != 0);
                        }
                    }
                    issued = true;
                    mma_commit(&empty[s]);
                    if (++s == NS) { s = 0; ph ^= 1u; }
                    if constexpr (C1) {   // the previous tile's first-conv MMAs
                        if (n > 0 && !(c1_ok = issue_c1(n - 1))) break;
                    }
                }
                if constexpr (C1) {
                    if (c1_ok && n > 0 && !*abort_flag) issue_c1(n - 1);   // the last tile's
                }
            }
            if (issued) mma_commit(wg_full);
            else mbar_arrive(wg_full);   // nothing accumulated: release the partial writer
            if (issued) {
                mma_commit(drain);
                if (!mbar_wait_drain(drain, 0)) atomicCAS(p.err, 0, kErrDrain);
            }
        }
    } else if (UP && warp >= 10) {
        // ------------------------------------------------ dY builders (warps 10..13, UP)
        const int bt = threadIdx.x - 320;   // 0..127
        const int g = bt & 7;               // channel octet of every item of this thread
        const int Ho = p.H >> 1, Wo = p.W >> 1;
        const int nitems = 4 * Wo * 8;      // 4 pooled rows cover the R + 2 = 6 halo rows
        float bsum[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) bsum[e] = 0.0f;
        // an item's window (pooled row prow of the tile's four, column pw) and its halo offset do
        // not depend on the tile: worked out once (wi = prow * Wo + pw)
        int wi_[4], prow_[4], soff_[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int i = bt + 128 * m;
            wi_[m] = i >> 3;
            prow_[m] = i < nitems ? wi_[m] / Wo : -2;   // -2: no item
            const int pw = wi_[m] - (i < nitems ? prow_[m] : 0) * Wo;
            soff_[m] = ((2 * prow_[m] - 1) * p.Wp + 2 * pw + 1) * 16;   // halo row 2 prow - 1, column 2 pw + 1
        }
        int s = 0;
        uint32_t ph = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
            const int b = tile / p.tiles_per_img;
            const int h0 = (tile - b * p.tiles_per_img) * p.R;
            // this tile's dP and code loads go out before the stage wait
            const long long wbase = ((long long)b * Ho + (h0 >> 1) - 1) * Wo;   // window (phr = h0/2 - 1, 0)
            uint4 pv[4];
            uint2 cd[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int phr = (h0 >> 1) - 1 + prow_[m];   // pooled row
                pv[m] = make_uint4(0, 0, 0, 0);
                cd[m] = make_uint2(0, 0);
                if (prow_[m] >= 0 && (unsigned)phr < (unsigned)Ho) {
                    const size_t o = (size_t)(wbase + wi_[m]) * CY + 8 * g;
                    pv[m] = __ldg(reinterpret_cast<const uint4 *>(p.dp + o));
                    cd[m] = __ldg(reinterpret_cast<const uint2 *>(p.code + o));
                }
            }
            if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
            uint8_t *st = sA + s * STAGE + g * p.dy_region;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int prow = prow_[m];
                if (prow < 0) continue;
                // selector nibbles = the 8 codes (values 0..7)
                const uint32_t t0 = cd[m].x | (cd[m].x >> 4), t1 = cd[m].y | (cd[m].y >> 4);
                const uint32_t sel0 = (t0 & 0xFFu) | ((t0 >> 8) & 0xFF00u);
                const uint32_t sel1 = (t1 & 0xFFu) | ((t1 >> 8) & 0xFF00u);
                // halo row of the window's top image row: 2 * pooled row - (h0 - 1)
                const int hr0 = 2 * prow - 1;
#pragma unroll
                for (int kh = 0; kh < 2; ++kh) {
                    const int hr = hr0 + kh;
                    if (hr < 0 || hr > p.R + 1) continue;
                    uint8_t *rowp = st + soff_[m] + kh * p.Wp * 16;
#pragma unroll
                    for (int kw = 0; kw < 2; ++kw)
                        *reinterpret_cast<uint4 *>(rowp + kw * 16) =
                            unpool_select(pv[m], sel0, sel1, 0xFFu << (8 * (2 * kh + kw)));
                }
                if (prow == 1 || prow == 2) {   // the tile's own pooled rows: bias-gradient sums
                    const uint4 r4 = unpool_select(pv[m], sel0, sel1, 0xFFFFFFFFu);   // any code >= 4
                    const uint32_t w[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        bsum[2 * e] += __uint_as_float(w[e] << 16);
                        bsum[2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
                    }
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
            if (++s == NS) { s = 0; ph ^= 1u; }
        }
        // bias-gradient partial of this CTA: the 16 threads of each octet, in a fixed order
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            bsum[e] += __shfl_xor_sync(0xffffffffu, bsum[e], 8);
            bsum[e] += __shfl_xor_sync(0xffffffffu, bsum[e], 16);
        }
        if (lane < 8) {   // lane = octet: one [CY] slice per builder warp, summed by the split reduction
            float *bp = p.bias_partial + ((size_t)blockIdx.x * 4 + (warp - 10)) * CY + 8 * lane;
            reinterpret_cast<float4 *>(bp)[0] = make_float4(bsum[0], bsum[1], bsum[2], bsum[3]);
            reinterpret_cast<float4 *>(bp)[1] = make_float4(bsum[4], bsum[5], bsum[6], bsum[7]);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..9)
        const int q = warp & 3;
        const int grp = (warp - 2) >> 2;
        const int row = q * 32 + lane;          // input-gradient row: pixel (row / Wp, row % Wp)
        const int etid = threadIdx.x - 64;      // 0..255
        const int r = row / p.Wp, c = row - r * p.Wp;
        const bool in_tile = (r < p.R) && (c < p.W);
        constexpr int RB = CX * 2;              // output row bytes
        constexpr uint32_t SWM = RB == 128 ? 7u : RB == 64 ? 3u : 1u;
        int acc = 0, sb = 0, s = 0, n = 0;
        uint32_t acc_ph = 0;
        // (elected thread, C1) bit i: a commit on c1_done[i] not yet waited for; bit 2 + i: its parity
        uint32_t c1_state = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++n) {
            const int b = tile / p.tiles_per_img;
            const int h0 = (tile - b * p.tiles_per_img) * p.R;
            // C1: the second group loads the 9 taps of the first conv's input at pixel
            // (h0 + r, c) before the accumulator wait (zero outside the image)
            float xt[9];
            if (C1 && grp == 1) {
                const int h = h0 + r;
#pragma unroll
                for (int t = 0; t < 9; ++t) {
                    const int ih = h + t / 3 - 1, iw = c + t % 3 - 1;
                    xt[t] = (in_tile && h < p.H && (unsigned)ih < (unsigned)p.H && (unsigned)iw < (unsigned)p.W)
                                ? __ldg(p.x0 + ((size_t)b * p.H + ih) * p.W + iw)
                                : 0.0f;
                }
            }
            mbar_wait(&acc_full[acc], acc_ph, abort_flag, p.err, kErrAccWait);
            if (etid == 0) {
                if (C1) {   // the first-conv MMAs that last read buffer sb are done
                    if ((c1_state >> sb) & 1u) {
                        mbar_wait(&c1_done[sb], (c1_state >> (2 + sb)) & 1u, abort_flag, p.err, kErrAccWait);
                        c1_state ^= (4u << sb) | (1u << sb);
                    }
                } else {
                    bulk_wait_read<1>();   // the store that last read staging buffer sb
                }
            }
            named_bar_sync(1, 256);
            if (*abort_flag) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * S::ZCOLS);
            if (grp == 0) {   // CX = 32: dX = Z[.][0] + Z[. + 1][1] + Z[. + 2][2], taken by the first group
                // lane = tile column (Wp = 32: a warp is one tile row); columns c + dw of a real
                // output (c < W <= 30) stay inside the row
                float v[32], z[32];
                tmem_ld32(taddr, v);
                tmem_ld32(taddr + CX, z);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += __shfl_down_sync(0xffffffffu, z[j], 1);
                tmem_ld32(taddr + 2 * CX, z);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += __shfl_down_sync(0xffffffffu, z[j], 2);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
                if (in_tile) {
                    // ReLU mask: X > 0 at the same pixel, from the X halo tile of this stage
                    const uint8_t *xs = sA + s * STAGE + p.x_off + ((r + 1) * p.Wp + c + 1) * 16;
#pragma unroll
                    for (int g = 0; g < S::XG; ++g) {
                        const uint4 m = *reinterpret_cast<const uint4 *>(xs + g * p.region);
                        const __nv_bfloat16 *mb = reinterpret_cast<const __nv_bfloat16 *>(&m);
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            if (!(__bfloat162float(mb[e]) > 0.0f)) v[g * 8 + e] = 0.0f;
                    }
                    uint8_t *tile_buf = outbuf + sb * OBUF;
                    const uint32_t base_off = (uint32_t)((r * p.W + c) * RB);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint4 pk;
                        __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            h2[e] = __floats2bfloat162_rn(v[q4 * 8 + 2 * e], v[q4 * 8 + 2 * e + 1]);
                        const uint32_t o = base_off + 16 * q4;
                        *reinterpret_cast<uint4 *>(tile_buf + (o ^ (((o >> 7) & SWM) << 4))) = pk;
                    }
                }
            } else {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
                if (C1 && in_tile) {
                    // im2col row of the first conv's input for pixel (h0 + r, c): x_hi of the
                    // 9 taps, 1.0 (bias), x_lo at 16..24; zero rows past the image
                    const int h = h0 + r;
                    __nv_bfloat16 vals[32];
#pragma unroll
                    for (int t = 0; t < 9; ++t) {
                        const __nv_bfloat16 hi = __float2bfloat16_rn(xt[t]);
                        vals[t] = hi;
                        vals[16 + t] = __float2bfloat16_rn(xt[t] - __bfloat162float(hi));
                    }
                    vals[9] = __float2bfloat16_rn(h < p.H ? 1.0f : 0.0f);
#pragma unroll
                    for (int t = 10; t < 16; ++t) vals[t] = __float2bfloat16_rn(0.0f);
#pragma unroll
                    for (int t = 25; t < 32; ++t) vals[t] = __float2bfloat16_rn(0.0f);
                    uint8_t *x9 = outbuf + sb * OBUF + p.out_tile_bytes;
                    const uint32_t k = (uint32_t)(r * p.W + c);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {   // 128-byte row, 16-byte chunk j XOR (k & 7)
                        uint4 pk = make_uint4(0, 0, 0, 0);
                        if (j < 4) pk = *reinterpret_cast<const uint4 *>(&vals[8 * j]);
                        *reinterpret_cast<uint4 *>(x9 + k * 128 + ((j ^ (k & 7)) << 4)) = pk;
                    }
                }
            }
            fence_proxy_async_smem();
            named_bar_sync(2, 256);
            if (etid == 0) {
                mbar_arrive(&empty[s]);   // this stage's mask reads are done
                if (C1) {
                    // D1[64][CX] += im2col^T (MN-major, 128-byte swizzle) x dX (MN-major, 64-byte
                    // swizzle): issued by the MMA thread once this buffer is marked staged
                    mbar_arrive(&c1_ready[sb]);
                    c1_state |= 1u << sb;
                } else {
                    tma_store_4d(&p.out_map, outbuf + sb * p.out_tile_bytes, 0, 0, h0, b);
                    bulk_commit();
                }
            }
            sb ^= 1;
            if (++s == NS) s = 0;
            if (++acc == 2) { acc = 0; acc_ph ^= 1u; }
        }
        if (etid == 0) {
            bulk_wait_all();   // stores complete before exit
            if (C1)            // and every first-conv MMA finished before D1 is read or TMEM freed
                for (int i = 0; i < 2; ++i)
                    if (((c1_state >> i) & 1u) && !mbar_wait_drain(&c1_done[i], (c1_state >> (2 + i)) & 1u))
                        atomicCAS(p.err, 0, kErrDrain);
        }
        // weight-gradient partial of this CTA: rows co, columns (tap, ci)
        mbar_wait(wg_full, 0, abort_flag, p.err, kErrAccWait);
        named_bar_sync(1, 256);
        if (!*abort_flag) {
            tc_fence_after();
            const int m = q * 16 + lane;   // M = 64: lanes 32q .. 32q + 15
            const bool row_ok = lane < 16;
            float *part = p.partial + ((size_t)blockIdx.x * CY + (row_ok ? m : 0)) * S::NTOT;
            const uint32_t waddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)S::WG_COL0;
            const bool empty_cta = my_tiles == 0;
#pragma unroll 1
            for (int cc = grp; cc < S::NTOT / 32; cc += 2) {
                float v[32];
                tmem_ld32(waddr + 32 * cc, v);
                if (!row_ok) continue;
                float4 *d4 = reinterpret_cast<float4 *>(part + 32 * cc);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    d4[j] = empty_cta ? make_float4(0.0f, 0.0f, 0.0f, 0.0f)
                                      : make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
            if (C1 && grp == 0 && (q == 0 || q == 1)) {
                // D1 rows 16q + lane sit in lanes 32q + lane: quarter 0 holds the x_hi taps and
                // the bias (rows 0..9), quarter 1 the x_lo taps (rows 16..24; row 25 is zero).
                // Each writes its own [CX][10] slice; the reduction adds the two.
                float v[32];
                tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)S::C1_COL0, v);
                if (lane < 10) {
                    float *c1p = p.c1_partial + ((size_t)blockIdx.x * 2 + q) * CX * 10;
#pragma unroll
                    for (int co = 0; co < CX; ++co) c1p[co * 10 + lane] = empty_cta ? 0.0f : v[co];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, S::TMEM_COLS);
}

}  // namespace tc
}  // namespace zb
