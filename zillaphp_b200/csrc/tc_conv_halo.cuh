// tc_conv_halo.cuh -- implicit-GEMM 3x3 (stride 1, pad 1) convolution on
// tcgen05 with one halo tile per output tile.
//
// D[pixel, n] = sum_{tap, c} IN[pixel + tap offset, c] * Wt[tap][n][c]
//   forward:        IN = activations x (NHWC bf16), Wt[tap][co][ci] = W[co][ci][tap]
//   input gradient: IN = dY (NHWC bf16),            Wt[tap][ci][co] = W[co][ci][8 - tap]
// (the input gradient of a stride-1, pad-1 3x3 conv is the same convolution
// of dY with the flipped, channel-transposed kernel).
//
// Output tile: R image rows of one image.  Its input, rows h0-1 .. h0+R and
// columns -1 .. W (Wp = W + 2 wide, zero outside the image: TMA's
// out-of-bounds fill is the padding), is loaded ONCE per tile, in 8-channel
// groups: group g holds the HR = (R+2)*Wp halo pixels as 16-byte rows,
//     smem[g][rr * Wp + cc][8 channels]        (rr, cc halo coordinates).
// That is the canonical K-major no-swizzle UMMA layout (8-row core matrices of
// 16-byte rows, SBO = 128 B between 8-row groups, LBO = the group pitch
// between the two 8-channel halves of a K16 step), so MMA row i can be the
// output pixel (i / Wp, i % Wp) for every tap at once: tap (dh, dw) is the
// same descriptor started dh*Wp + dw rows further on.  Rows with
// i % Wp >= W or i / Wp >= R are padding of the M = 128 tile; they read
// halo rows that feed only those discarded outputs.
// Compared with one shifted TMA box per tap, the L2 -> SM traffic per tile
// falls from 9 boxes to (R+2)/R of one, which is what let the pipeline keep
// the tensor pipe fed.
//
// The packed weights of all 9 taps stay resident in shared memory
// (K-major, 128/64-byte swizzle).  KS > 1 splits a tile's channels over KS
// pipeline stages (wide inputs: 128 channels of dY).
//
// Warp roles (320 threads): warp 0 TMA producer, warp 1 MMA issuer and TMEM
// owner, warps 2-9 epilogue in two groups of four: group g = (warp - 2) / 4
// takes the 32-channel accumulator chunks g, g + 2, ... of TMEM lane quarter
// warp % 4.  The epilogue is latency-bound (TMEM loads, staging, barriers,
// stores), so eight warps per CTA keep the tensor pipe fed.  The pool
// epilogue stages bias + ReLU rows (bf16, all channels) in shared memory and
// then pools with consecutive threads on consecutive channel octets of
// adjacent windows, so each warp's stores are contiguous.  Accumulators are
// double-buffered in TMEM so the epilogue of tile i overlaps the MMAs of tile
// i+1.  Epilogues:
//   kEpiPool : relu(acc + bias), 2x2/2 max-pool with the reference tie rule
//              (first maximum in (kh, kw) order, native/cpu/zilla_cpu.c:215-224)
//              on the bf16-rounded values (rounding is monotonic, so the
//              pooled value equals the rounded fp32 maximum), pooled bf16
//              NHWC out + a code byte per output
//              (window position 0..3 | (max > 0) << 2).
//   kEpiStore: relu(acc + bias) -> bf16 NHWC.
//   kEpiDgrad: acc [* (mask > 0)] -> bf16 NHWC.
//
// UP (input gradient whose dY is the max-unpool of a pooled gradient dP
// [B, H/2, W/2, CIN] by the pool codes): four more warps (10-13) build each
// stage's halo octets from dP and the codes instead of a TMA load of dY (the
// same construction as the fused conv2 backward: one 16-byte dP load and one
// 8-byte code load per (pooled row, pooled column, octet) item, the channel's
// value at the window position its code names, zero at the other three; the
// halo columns outside the image stay zero from the start).  The octet pitch
// is the row block plus 16 bytes so a pixel's octets fall in different banks.
// The builders also sum the routed values of the tile's own pooled rows: the
// bias gradient of the conv whose dY this is, one [CIN] slice per builder
// warp and CTA.
#pragma once

#include "tc_common.cuh"
#include "tc_conv.cuh"

namespace zb {
namespace tc {

struct ConvHaloParams {
    CUtensorMap in_map;   // 4D {CIN, W, H, B} bf16, box {8, W + 2, R + 2, 1}, no swizzle
    CUtensorMap w_map;    // 3D {CIN, COUT, 9} bf16, box {chunk, COUT, 1}
    CUtensorMap out_map;  // kEpiDgrad: 4D {COUT, W, H, B} bf16, box {COUT, W, R, 1}, swizzle = row bytes
    int B, H, W, R, Wp, HR, region, stage_bytes, tiles_per_img, num_tiles;
    int out_tile_bytes;   // kEpiDgrad: one staged output tile (R * W * COUT * 2, 1024-aligned)
    const float *bias;          // [COUT] (forward)
    __nv_bfloat16 *out;         // pooled [B, H/2, W/2, COUT] or full [B, H, W, COUT]
    uint8_t *code;              // [B, H/2, W/2, COUT] (kEpiPool)
    const __nv_bfloat16 *mask;  // [B, H, W, COUT] or null (kEpiDgrad)
    const __nv_bfloat16 *dp;    // UP: pooled gradient [B, H/2, W/2, CIN]
    const uint8_t *up_code;     // UP: its pool codes
    float *up_bias_partial;     // UP: [gridDim.x * 4][CIN]
    int *err;
};

template <int CIN, int COUT, int NS, int KS, bool POOL>
struct ConvHaloShape {
    static constexpr int CHUNK = CIN > 64 ? 64 : CIN;   // weight K chunk
    static constexpr int NCH = CIN / CHUNK;
    static constexpr int ROWB = CHUNK * 2;
    static constexpr Swizzle SW = ROWB == 128 ? kSw128 : (ROWB == 64 ? kSw64 : kSw32);
    static constexpr int BBLK = COUT * ROWB;
    static constexpr int BTOTAL = 9 * NCH * BBLK;
    static constexpr int SC = CIN / KS;   // channels per stage
    static constexpr int NC8 = SC / 8;    // 8-channel groups per stage
    // pool staging: bf16 rows of all COUT channels, pitch COUT + 8 (an odd
    // number of 16-byte units: conflict-free 16-byte accesses), double-buffered
    // when it fits next to the resident weights
    static constexpr int SP = COUT + 8;
    static constexpr int SBUF_BYTES = 128 * SP * 2;
    static constexpr int NSBUF = (BTOTAL + 2 * SBUF_BYTES <= 150 * 1024) ? 2 : 1;
    static constexpr int POOL_STAGE = POOL ? NSBUF * SBUF_BYTES : 0;
    static constexpr int BIAS_BYTES = POOL ? COUT * 4 : 0;
    static constexpr uint32_t TMEM_COLS = (2 * COUT <= 32) ? 32 : (2 * COUT <= 64) ? 64 : (2 * COUT <= 128) ? 128 : (2 * COUT <= 256) ? 256 : 512;
    static constexpr int SLACK = 1024;    // the last stage's padding rows may be read past its end
    static constexpr int BAR_BYTES = 256;
    // group pitch: HR rows of 16 B rounded to 128 B (TMA destination alignment)
    static __host__ __device__ int region(int HR) { return (HR * 16 + 127) / 128 * 128; }
    static __host__ __device__ int stage_bytes(int HR) { return (NC8 * region(HR) + 1023) / 1024 * 1024; }
    // UP: octets written by threads, pitch + 16 bytes (no TMA alignment needed)
    static __host__ __device__ int region_up(int HR) { return region(HR) + 16; }
    static __host__ __device__ int stage_bytes_up(int HR) { return (NC8 * region_up(HR) + 1023) / 1024 * 1024; }
    // kEpiDgrad: staged output tiles for the TMA store (one or two buffers)
    static __host__ __device__ int out_tile_bytes(int R, int W) { return (R * W * COUT * 2 + 1023) / 1024 * 1024; }
    // dynamic shared memory for stages of `stage` bytes (stage_bytes or stage_bytes_up)
    static __host__ __device__ int smem(int stage, int out_total) {
        const int epi = POOL_STAGE > out_total ? POOL_STAGE : out_total;
        return 1024 + BTOTAL + NS * stage + SLACK + epi + BIAS_BYTES + BAR_BYTES;
    }
    static_assert(CIN % 16 == 0 && SC % 16 == 0 && COUT % 16 == 0 && COUT <= 256, "unsupported conv channels");
    static_assert(!POOL || COUT % 32 == 0, "the pool epilogue works on 32-channel chunks");
    static_assert(CIN <= 64 || CIN % 64 == 0, "CIN above 64 must be a multiple of 64");
    static_assert(SC % CHUNK == 0 || CHUNK % SC == 0, "stage channels and weight chunks must nest");
};

template <int CIN, int COUT, int EPI, int NS, int KS, int OB = 2, bool UP = false>
__global__ void __launch_bounds__(UP ? 448 : 320, UP ? 1 : 2) conv_halo_kernel(const __grid_constant__ ConvHaloParams p) {
    griddep_launch();
    using S = ConvHaloShape<CIN, COUT, NS, KS, EPI == kEpiPool>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sB = base;
    uint8_t *sA = sB + S::BTOTAL;
    const int STAGE = p.stage_bytes;
    float *stage = reinterpret_cast<float *>(sA + NS * STAGE + S::SLACK);   // epilogue staging
    const int EPI_BYTES = EPI == kEpiPool ? S::POOL_STAGE : (EPI == kEpiDgrad ? OB * p.out_tile_bytes : 0);
    float *sbias = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(stage) + EPI_BYTES);
    uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(sbias) + S::BIAS_BYTES);
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

    // Rows of the stages that TMA never writes (group padding, the slack) are
    // zeroed once so that the discarded accumulator rows stay finite.
    for (int i = threadIdx.x; i < (NS * STAGE + S::SLACK) / 16; i += blockDim.x)
        *reinterpret_cast<uint4 *>(sA + 16 * i) = make_uint4(0, 0, 0, 0);
    griddep_wait();   // everything below may touch global memory
    if constexpr (EPI == kEpiPool)
        for (int i = threadIdx.x; i < COUT; i += blockDim.x) sbias[i] = p.bias[i];
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

    if (threadIdx.x == 0) {
        // full: the TMA transaction arrival, or one arrival per builder warp (UP)
        for (int i = 0; i < NS; ++i) { mbar_init(&full[i], UP ? 4 : 1); mbar_init(&empty[i], 1); armed[i] = 0; }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 8); }
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

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (elect_one()) {
            if (!UP) prefetch_tmap(&p.in_map);
            prefetch_tmap(&p.w_map);
            if (EPI == kEpiDgrad) prefetch_tmap(&p.out_map);
            mbar_arrive_expect_tx(wbar, S::BTOTAL);
            for (int t = 0; t < 9; ++t)
                for (int j = 0; j < S::NCH; ++j)
                    tma_load_3d(sB + (t * S::NCH + j) * S::BBLK, &p.w_map, wbar, j * S::CHUNK, 0, t);
            const uint32_t stage_tx = (uint32_t)(S::NC8 * p.HR * 16);
            int s = 0;
            uint32_t ph = 0;
            for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag && !UP; tile += gridDim.x) {
                const int b = tile / p.tiles_per_img;
                const int h0 = (tile - b * p.tiles_per_img) * p.R;
                for (int kb = 0; kb < KS; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
                    mbar_arrive_expect_tx(&full[s], stage_tx);
                    armed[s] = (int)ph + 1;
                    uint8_t *dst = sA + s * STAGE;
                    for (int g = 0; g < S::NC8; ++g)
                        tma_load_4d(dst + g * p.region, &p.in_map, &full[s], kb * S::SC + 8 * g, -1, h0 - 1, b);
                    if (++s == NS) { s = 0; ph ^= 1u; }
                }
            }
            if (*abort_flag) {   // let every copy this thread started land before exit
                for (int i = 0; i < NS; ++i)
                    if (armed[i] && !mbar_wait_drain(&full[i], (uint32_t)(armed[i] - 1)))
                        atomicCAS(p.err, 0, kErrDrain);
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
                const uint32_t lbo = (uint32_t)p.region;
                // Descriptors are built once; an MMA's operands differ only in the
                // start-address field (bits 0-13, 16-byte units), so each one is a
                // single add.  Offsets stay below 256 KB: no carry out of the field.
                const uint64_t adesc0 = smem_desc(smem_u32(sA), lbo, 128, kSwNone);
                const uint64_t bdesc0 = smem_desc(smem_u32(sB), 16, 8 * S::ROWB, S::SW);
                const uint32_t row16 = (uint32_t)p.Wp;          // one halo row, in 16-byte units
                const uint32_t half16 = lbo >> 4;               // next 8 channels, in 16-byte units
                for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
                    if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag, p.err, kErrAccWait)) break;
                    tc_fence_after();
                    const uint32_t d = tmem_base + (uint32_t)(acc * COUT);
                    bool ok = true;
                    for (int kb = 0; kb < KS; ++kb) {
                        if (!mbar_wait(&full[s], ph, abort_flag, p.err, kErrFullWait)) { ok = false; break; }
                        tc_fence_after();
                        const uint64_t a_stage = adesc0 + (uint64_t)((uint32_t)(s * STAGE) >> 4);
                        const uint64_t b_kb = bdesc0 + (uint64_t)((uint32_t)(kb * S::SC / S::CHUNK * S::BBLK) >> 4);
#pragma unroll
                        for (int tap = 0; tap < 9; ++tap) {
                            const int dh = tap / 3, dw = tap - 3 * dh;
                            const uint64_t a_tap = a_stage + (uint64_t)(dh * row16 + dw);
#pragma unroll
                            for (int k = 0; k < S::SC / 16; ++k) {
                                // K16 step k: channels kb*SC + 16k.. (groups 2k, 2k+1 of the stage)
                                constexpr int KPC = S::CHUNK / 16;   // K16 steps per weight chunk
                                const uint32_t boff = (uint32_t)((tap * S::NCH + (k / KPC)) * S::BBLK + (k % KPC) * 32);
                                mma_bf16(d, a_tap + (uint64_t)(2 * k * half16), b_kb + (uint64_t)(boff >> 4), IDESC,
                                         (kb | tap | k) != 0);
                            }
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
    } else if (UP && warp >= 10) {
        // ------------------------------------------------ dY builders (warps 10..13, UP)
        const int bt = threadIdx.x - 320;   // 0..127
        const int g = bt & (S::NC8 - 1);    // octet (within a stage) of every item of this thread
        const int Ho = p.H >> 1, Wo = p.W >> 1;
        const int PR = (p.R >> 1) + 2;      // pooled rows covering the R + 2 halo rows
        const int nitems = PR * Wo * S::NC8;
        float bsum[KS][8];
#pragma unroll
        for (int kb = 0; kb < KS; ++kb)
#pragma unroll
            for (int e = 0; e < 8; ++e) bsum[kb][e] = 0.0f;
        // an item's window (pooled row prow of the tile's, column pw) does not depend on the
        // tile or the stage: worked out once (window index (bt + 128 m) / NC8 = prow * Wo + pw;
        // prow -2: no item)
        int prow_[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int i = bt + 128 * m;
            prow_[m] = i < nitems ? (i / S::NC8) / Wo : -2;
        }
        // this thread's dP and code loads of stage kb of `tile` (zero past the image / the tiles)
        auto load_stage = [&](int tile, int kb, uint4 (&pv)[4], uint2 (&cd)[4]) {
            const int b = tile / p.tiles_per_img;
            const int h0 = (tile - b * p.tiles_per_img) * p.R;
            const int ch = (kb * S::NC8 + g) * 8;
            const long long wbase = ((long long)b * Ho + (h0 >> 1) - 1) * Wo;   // window (h0/2 - 1, 0)
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int phr = (h0 >> 1) - 1 + prow_[m];
                pv[m] = make_uint4(0, 0, 0, 0);
                cd[m] = make_uint2(0, 0);
                if (tile < p.num_tiles && prow_[m] >= 0 && (unsigned)phr < (unsigned)Ho) {
                    const size_t o = (size_t)(wbase + (bt + 128 * m) / S::NC8) * CIN + ch;
                    pv[m] = __ldg(reinterpret_cast<const uint4 *>(p.dp + o));
                    cd[m] = __ldg(reinterpret_cast<const uint2 *>(p.up_code + o));
                }
            }
        };
        int s = 0;
        uint32_t ph = 0;
        uint4 pv[4], pvn[4];
        uint2 cd[4], cdn[4];
        load_stage(blockIdx.x, 0, pv, cd);
        for (int tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
#pragma unroll
            for (int kb = 0; kb < KS; ++kb) {
                // the next stage's loads go out first: their latency overlaps this stage
                if (kb + 1 < KS) load_stage(tile, kb + 1, pvn, cdn);
                else load_stage(tile + gridDim.x, 0, pvn, cdn);
                if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
                uint8_t *st = sA + s * STAGE + g * p.region;
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const int prow = prow_[m], pw = (bt + 128 * m) / S::NC8 - prow * Wo;
                    if (prow < 0) continue;
                    const uint32_t t0 = cd[m].x | (cd[m].x >> 4), t1 = cd[m].y | (cd[m].y >> 4);
                    const uint32_t sel0 = (t0 & 0xFFu) | ((t0 >> 8) & 0xFF00u);
                    const uint32_t sel1 = (t1 & 0xFFu) | ((t1 >> 8) & 0xFF00u);
                    const int hr0 = 2 * prow - 1;   // halo row of the window's top image row
#pragma unroll
                    for (int kh = 0; kh < 2; ++kh) {
                        const int hr = hr0 + kh;
                        if (hr < 0 || hr > p.R + 1) continue;
                        uint8_t *rowp = st + (hr * p.Wp + 2 * pw + 1) * 16;
#pragma unroll
                        for (int kw = 0; kw < 2; ++kw)
                            *reinterpret_cast<uint4 *>(rowp + kw * 16) =
                                unpool_select(pv[m], sel0, sel1, 0xFFu << (8 * (2 * kh + kw)));
                    }
                    if (prow >= 1 && prow <= (p.R >> 1)) {   // the tile's own pooled rows
                        const uint4 r4 = unpool_select(pv[m], sel0, sel1, 0xFFFFFFFFu);
                        const uint32_t w[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            bsum[kb][2 * e] += __uint_as_float(w[e] << 16);
                            bsum[kb][2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
                        }
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
                if (++s == NS) { s = 0; ph ^= 1u; }
#pragma unroll
                for (int m = 0; m < 4; ++m) { pv[m] = pvn[m]; cd[m] = cdn[m]; }
            }
        }
        // bias-gradient partial: the lanes of each octet in a fixed order, one slice per warp
#pragma unroll
        for (int kb = 0; kb < KS; ++kb)
#pragma unroll
            for (int e = 0; e < 8; ++e)
                for (int off = S::NC8; off < 32; off <<= 1)
                    bsum[kb][e] += __shfl_xor_sync(0xffffffffu, bsum[kb][e], off);
        if (lane < S::NC8) {
            float *bp = p.up_bias_partial + ((size_t)blockIdx.x * 4 + (warp - 10)) * CIN;
#pragma unroll
            for (int kb = 0; kb < KS; ++kb) {
                float4 *d4 = reinterpret_cast<float4 *>(bp + (kb * S::NC8 + lane) * 8);
                d4[0] = make_float4(bsum[kb][0], bsum[kb][1], bsum[kb][2], bsum[kb][3]);
                d4[1] = make_float4(bsum[kb][4], bsum[kb][5], bsum[kb][6], bsum[kb][7]);
            }
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..9)
        const int q = warp & 3;                 // TMEM lane quarter
        const int grp = (warp - 2) >> 2;        // warp group: chunks grp, grp + 2, ...
        const int row = q * 32 + lane;          // accumulator row: pixel (row / Wp, row % Wp) of the tile
        const int etid = threadIdx.x - 64;      // 0..255
        const int r = row / p.Wp, c = row - r * p.Wp;
        const bool in_tile = (r < p.R) && (c < p.W);
        constexpr int NCC = COUT / 32;          // 32-column accumulator chunks (pool epilogue)
        constexpr int CW = COUT % 32 == 0 ? 32 : 16;   // chunk width of the other epilogues
        constexpr int NCW = COUT / CW;
        constexpr int OCT = COUT / 8;           // channel octets per pixel
        const int Wo = p.W >> 1, Ho = p.H >> 1;
        const int nitems = (p.R >> 1) * Wo * OCT;
        // pool items etid and etid + 256 (thread = (window, channel octet)): their window's
        // pooled row and column within the tile, worked out once (later items, if any, per tile)
        int ipr[2], ipc[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int wi = (etid + 256 * j) / OCT;
            ipr[j] = wi / Wo;
            ipc[j] = wi - ipr[j] * Wo;
        }
        __nv_bfloat16 *sbuf = reinterpret_cast<__nv_bfloat16 *>(stage);
        int acc = 0, sb = 0;
        uint32_t acc_ph = 0;
        // All eight epilogue warps leave the tile loop together: the abort flag
        // is only consulted right after their common named barrier, so a warp
        // can never wait at a barrier that another epilogue warp has left.
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            const int b = tile / p.tiles_per_img;
            const int h0 = (tile - b * p.tiles_per_img) * p.R;
            mbar_wait(&acc_full[acc], acc_ph, abort_flag, p.err, kErrAccWait);
            // the TMA store that last read this tile's staging buffer (two tiles
            // ago) has finished reading before anyone writes it again
            if (EPI == kEpiDgrad && etid == 0) bulk_wait_read<OB - 1>();
            named_bar_sync(1, 256);
            if (*abort_flag) break;

            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * COUT);
            const int h = h0 + r;
            const bool pix_ok = in_tile && (h < p.H);
            if (grp >= (EPI == kEpiPool ? NCC : NCW)) {   // no chunk for this group (COUT = 32, or 16)
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[acc]);
            }
            if constexpr (EPI == kEpiPool) {
                __nv_bfloat16 *buf = sbuf + sb * 128 * S::SP;
#pragma unroll 1
                for (int cc = grp; cc < NCC; cc += 2) {
                    float v[32];
                    tmem_ld32(taddr + 32 * cc, v);
                    if (cc + 2 >= NCC) {   // this group's last chunk: the accumulator is free
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[acc]);
                    }
                    // bias + ReLU -> bf16 (packed add, converting clamp), the row's 32
                    // channels as four 16-byte stores
                    uint4 *srow = reinterpret_cast<uint4 *>(buf + row * S::SP + 32 * cc);
                    const float4 *bias4 = reinterpret_cast<const float4 *>(sbias + 32 * cc);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float4 b0 = bias4[2 * k], b1 = bias4[2 * k + 1];
                        srow[k] = make_uint4(bias_relu_bf16x2(v[8 * k + 0], v[8 * k + 1], b0.x, b0.y),
                                             bias_relu_bf16x2(v[8 * k + 2], v[8 * k + 3], b0.z, b0.w),
                                             bias_relu_bf16x2(v[8 * k + 4], v[8 * k + 5], b1.x, b1.y),
                                             bias_relu_bf16x2(v[8 * k + 6], v[8 * k + 7], b1.z, b1.w));
                    }
                }
                named_bar_sync(2, 256);
                // thread = (window, channel octet), octets fastest: four pixels x 8 channels
                for (int idx = etid, j = 0; idx < nitems; idx += 256, ++j) {
                    const int o = idx % OCT;
                    int pr, pc;
                    if (j < 2) {
                        pr = j == 0 ? ipr[0] : ipr[1];
                        pc = j == 0 ? ipc[0] : ipc[1];
                    } else {
                        const int wi = idx / OCT;
                        pr = wi / Wo;
                        pc = wi - pr * Wo;
                    }
                    const int ho = (h0 >> 1) + pr;
                    if (ho >= Ho) continue;
                    const int r0 = (2 * pr) * p.Wp + 2 * pc;
                    const int rr[4] = {r0, r0 + 1, r0 + p.Wp, r0 + p.Wp + 1};
                    uint4 px[4];
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) px[q4] = *reinterpret_cast<const uint4 *>(buf + rr[q4] * S::SP + 8 * o);
                    // (kh, kw) order, bf16x2 lanes: first maximum wins
                    uint32_t best[4] = {px[0].x, px[0].y, px[0].z, px[0].w}, pos[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                    for (int q4 = 1; q4 < 4; ++q4) {
                        pool_step_bf16x2(best[0], pos[0], px[q4].x, (uint32_t)q4);
                        pool_step_bf16x2(best[1], pos[1], px[q4].y, (uint32_t)q4);
                        pool_step_bf16x2(best[2], pos[2], px[q4].z, (uint32_t)q4);
                        pool_step_bf16x2(best[3], pos[3], px[q4].w, (uint32_t)q4);
                    }
                    const uint2 cd = make_uint2(pool_codes(best[0], pos[0], best[1], pos[1]),
                                                pool_codes(best[2], pos[2], best[3], pos[3]));
                    const size_t o8 = (((size_t)b * Ho + ho) * Wo + pc) * COUT + 8 * o;
                    *reinterpret_cast<uint4 *>(p.out + o8) = make_uint4(best[0], best[1], best[2], best[3]);
                    *reinterpret_cast<uint2 *>(p.code + o8) = cd;
                }
                // A staging buffer is rewritten only after the next tile's
                // opening barrier, which every thread reaches after its pooling.
                if constexpr (S::NSBUF == 2) sb ^= 1;
            } else {
#pragma unroll 1
                for (int cc = grp; cc < NCW; cc += 2) {
                    float v[CW];
                    if constexpr (CW == 32) tmem_ld32(taddr + 32 * cc, v);
                    else tmem_ld16(taddr + 16 * cc, v);
                    if (cc + 2 >= NCW) {   // this group's last chunk: the accumulator is free
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty[acc]);
                    }
                    if constexpr (EPI == kEpiDgrad) {
                        if (!in_tile) continue;   // rows past H are clipped by the TMA store
                        if (p.mask && pix_ok) {
                            const uint4 *mk = reinterpret_cast<const uint4 *>(
                                p.mask + (((size_t)b * p.H + h) * p.W + c) * COUT + CW * cc);
#pragma unroll
                            for (int q4 = 0; q4 < CW / 8; ++q4) {
                                uint4 m = __ldg(mk + q4);
                                const __nv_bfloat16 *mb = reinterpret_cast<const __nv_bfloat16 *>(&m);
#pragma unroll
                                for (int e = 0; e < 8; ++e)
                                    if (!(__bfloat162float(mb[e]) > 0.0f)) v[q4 * 8 + e] = 0.0f;
                            }
                        }
                        // staging tile [R][W][COUT] bf16 with the TMA store's swizzle
                        // (16-byte chunk index XOR (offset >> 7) within the row span)
                        constexpr int RB = COUT * 2;
                        constexpr uint32_t SWM = RB == 128 ? 7u : RB == 64 ? 3u : 1u;
                        uint8_t *tile_buf = reinterpret_cast<uint8_t *>(stage) + sb * p.out_tile_bytes;
                        const uint32_t base_off = (uint32_t)((r * p.W + c) * RB + 2 * CW * cc);
#pragma unroll
                        for (int q4 = 0; q4 < CW / 8; ++q4) {
                            uint4 pk;
                            __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                h2[e] = __floats2bfloat162_rn(v[q4 * 8 + 2 * e], v[q4 * 8 + 2 * e + 1]);
                            const uint32_t o = base_off + 16 * q4;
                            *reinterpret_cast<uint4 *>(tile_buf + (o ^ (((o >> 7) & SWM) << 4))) = pk;
                        }
                        continue;
                    }
                    if (!pix_ok) continue;
                    const size_t o = (((size_t)b * p.H + h) * p.W + c) * COUT + CW * cc;
                    if constexpr (EPI == kEpiStore) {
#pragma unroll
                        for (int j = 0; j < CW; ++j) {
                            const float x = v[j] + __ldg(p.bias + CW * cc + j);
                            v[j] = x > 0.0f ? x : 0.0f;
                        }
                    } else if (p.mask) {
                        const uint4 *mk = reinterpret_cast<const uint4 *>(p.mask + o);
#pragma unroll
                        for (int q4 = 0; q4 < CW / 8; ++q4) {
                            uint4 m = __ldg(mk + q4);
                            const __nv_bfloat16 *mb = reinterpret_cast<const __nv_bfloat16 *>(&m);
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                if (!(__bfloat162float(mb[e]) > 0.0f)) v[q4 * 8 + e] = 0.0f;
                        }
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + o);
#pragma unroll
                    for (int q4 = 0; q4 < CW / 8; ++q4) {
                        uint4 pk;
                        __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                        for (int e = 0; e < 4; ++e) h2[e] = __floats2bfloat162_rn(v[q4 * 8 + 2 * e], v[q4 * 8 + 2 * e + 1]);
                        dst[q4] = pk;
                    }
                }
                if constexpr (EPI == kEpiDgrad) {
                    fence_proxy_async_smem();
                    named_bar_sync(2, 256);
                    if (etid == 0) {
                        tma_store_4d(&p.out_map, reinterpret_cast<uint8_t *>(stage) + sb * p.out_tile_bytes, 0, 0, h0, b);
                        bulk_commit();
                    }
                    if (OB == 2) sb ^= 1;
                }
            }
            if (++acc == 2) { acc = 0; acc_ph ^= 1u; }
        }
        if (EPI == kEpiDgrad && etid == 0) bulk_wait_all();   // stores complete before exit
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, S::TMEM_COLS);
}

}  // namespace tc
}  // namespace zb
