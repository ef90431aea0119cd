// tc_wgrad.cuh -- weight gradients on tcgen05 with MN-major operands:
// D[m, n] = sum_k A[k][m] * B[k][n], both operands stored with the M / N
// index contiguous (NHWC activations and gradients, row-major Linear
// activations), so no transposed copies are made.  Each CTA reduces a slice
// of K (images or batch rows) into one TMEM accumulator and writes an fp32
// partial; a second kernel sums the partials in CTA order (deterministic)
// and scatters them into the parameter-gradient layout.
//
// Modes (K-stage = one TMA box height of pixels / rows):
//   kWgLinear : Linear dW = X^T dZ.  A = X [rows][M] box {64, 64},
//               B = dZ [rows][N] box {64, 64}; M tile 128 (2 A boxes),
//               N = NB*64 (NB B boxes).  Partial [split][M][N].
//   kWgConvCo : conv dW with M = out channels (128): A = dY NHWC box
//               {64, W, R, 1} x 2, B = X NHWC shifted by 3 taps of group g,
//               box {64 (=CIN), W, R, 1} x 3 -> N = 192.  Partial
//               [split][M=COUT][N = 9*CIN] (n = tap*CIN + ci).
//   kWgConvTap: conv dW with M = (tap, ci) for CIN = 32: A = X NHWC shifted by
//               all 9 taps, box {32, W, R, 1} (64-byte swizzle), M tiles of
//               4 taps; B = dY NHWC box {64 (=COUT), W, R, 1}; three
//               accumulators of 128 x 64.  Partial [split][M = 9*CIN][N = COUT].
//
// UP (kWgConvCo whose dY is the max-unpool of a pooled gradient dP
// [B, H/2, W/2, COUT] by the pool codes): four more warps (6-9) write the two
// A boxes of each stage from dP and the codes (one 16-byte dP load and one
// 8-byte code load per (pooled pixel, octet) item, the channel's value at the
// window position its code names, zero elsewhere; rows = the stage's R x W
// pixels, 128 B each with the 128-byte swizzle the TMA box would have), so dY
// never exists in global memory; TMA loads only the three X boxes.  R is even
// and tiles start on even rows, so every window lies inside one stage.
#pragma once

#include "tc_common.cuh"

namespace zb {
namespace tc {

enum WgMode { kWgLinear = 0, kWgConvCo = 1, kWgConvTap = 2, kWgLinearN128 = 3 };
// kWgLinearN128: kWgLinear for CTAs that take half of N = 256 (n_tiles = 2): two
// B boxes per stage, so six stages fit in shared memory instead of three
constexpr bool wg_linear(int mode) { return mode == kWgLinear || mode == kWgLinearN128; }

struct WgradTcParams {
    CUtensorMap a_map, b_map;
    int mode;
    int K_total;          // linear: rows; conv: images
    int splits;           // CTAs along K
    int m_tiles;          // linear: M/128; conv-co: tap groups (3)
    int n_tiles;          // linear: 1 (N = 256 per CTA) or 2 (two CTAs of N = 128); else 1
    int M, N;             // logical D (partial row / col extents)
    int H, W, R, tiles_per_img;   // conv geometry (K-stage = R rows of one image)
    int kstage_rows;      // rows (pixels) per K-stage, multiple of 16 after zero padding
    float *partial;       // [splits][M][N]
    const __nv_bfloat16 *dp;   // UP: pooled gradient [B, H/2, W/2, COUT]
    const uint8_t *up_code;    // UP: its pool codes
    float *out;           // linear, one K split: the final gradient, rows in the layout below
    int oC, oHW;          // linear: row m = hw * oC + c of the NHWC flatten goes to c * oHW + hw
    int *err;
};

template <int MODE>
struct WgradTcShape {
    // stage = A box slots + B box slots; a slot holds kpad = round16(kstage_rows)
    // k rows (the rows past kstage_rows stay zero)
    static constexpr int A_BOXES = wg_linear(MODE) ? 2 : MODE == kWgConvCo ? 2 : 12;
    static constexpr int A_ROWB = MODE == kWgConvTap ? 64 : 128;
    static constexpr int B_BOXES = MODE == kWgLinear ? 4 : MODE == kWgLinearN128 ? 2 : MODE == kWgConvCo ? 3 : 1;
    static constexpr int NS = MODE == kWgLinear ? 3 : MODE == kWgLinearN128 ? 6 : 2;
    static constexpr uint32_t TMEM_COLS = 256;
    static __host__ __device__ int kpad(int kr) { return (kr + 15) / 16 * 16; }
    static __host__ __device__ int abox(int kr) { return kpad(kr) * A_ROWB; }
    static __host__ __device__ int bbox(int kr) { return kpad(kr) * 128; }
    static __host__ __device__ int stage(int kr) { return A_BOXES * abox(kr) + B_BOXES * bbox(kr); }
    static __host__ __device__ int smem(int kr) { return 1024 + NS * stage(kr) + 256; }
};

// 32 consecutive fp32 partial values of one row (16-byte aligned) as eight
// 16-byte stores; zeros for a CTA whose K slice was empty.
__device__ __forceinline__ void store_row32(float *dst, const float (&v)[32], bool zero) {
    float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll
    for (int q = 0; q < 8; ++q)
        d4[q] = zero ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

template <int MODE, bool UP = false>
__global__ void __launch_bounds__(UP ? 320 : 192, 1) wgrad_tc_kernel(const __grid_constant__ WgradTcParams p) {
    griddep_launch();
    static_assert(!UP || MODE == kWgConvCo, "UP builds the dY boxes of kWgConvCo");
    using S = WgradTcShape<MODE>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *sbase = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const int kr = p.kstage_rows;             // valid k rows per stage
    const int kr16 = (kr + 15) / 16;          // K16 steps per stage (tail rows are zero)
    const int ABOX = S::abox(kr), BBOX = S::bbox(kr), STAGE = S::stage(kr);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sbase + S::NS * STAGE);
    uint64_t *full = bars, *empty = bars + S::NS, *acc_full = bars + 2 * S::NS, *drain = acc_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *armed = const_cast<int *>(abort_flag) + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // CTA -> (m tile / tap group, K split)
    const int mt = blockIdx.x % p.m_tiles;
    const int nt = wg_linear(MODE) ? (blockIdx.x / p.m_tiles) % p.n_tiles : 0;
    const int split = wg_linear(MODE) ? blockIdx.x / (p.m_tiles * p.n_tiles) : blockIdx.x / p.m_tiles;
    const int nb = wg_linear(MODE) ? 4 / p.n_tiles : 0;   // linear: 64-column B boxes per stage (<= B_BOXES)
    // K slices: linear splits whole 64-row stages, conv splits whole images
    const int kunits = wg_linear(MODE) ? (p.K_total + 63) / 64 : p.K_total;
    const int k0 = (int)((long long)kunits * split / p.splits);
    const int k1 = (int)((long long)kunits * (split + 1) / p.splits);
    const int nstages = wg_linear(MODE) ? (k1 - k0) : (k1 - k0) * p.tiles_per_img;

    // zero the never-written tails of every box slot once (k rows kr..127)
    for (int i = threadIdx.x; i < S::NS * STAGE / 16; i += blockDim.x) {
        const int off = i * 16;
        const int in_stage = off % STAGE;
        int row;
        if (in_stage < S::A_BOXES * ABOX) row = (in_stage % ABOX) / S::A_ROWB;
        else row = ((in_stage - S::A_BOXES * ABOX) % BBOX) / 128;
        if (row >= kr) *reinterpret_cast<uint4 *>(sbase + off) = make_uint4(0, 0, 0, 0);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

    if (threadIdx.x == 0) {
        // full: the TMA transaction arrival (+ one per builder warp, UP)
        for (int i = 0; i < S::NS; ++i) { mbar_init(&full[i], UP ? 5 : 1); mbar_init(&empty[i], 1); armed[i] = 0; }
        mbar_init(acc_full, 1);
        mbar_init(drain, 1);
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
        if (elect_one()) {
            prefetch_tmap(&p.a_map);
            prefetch_tmap(&p.b_map);
            int s = 0;
            uint32_t ph = 0;
            const uint32_t abox_bytes = (uint32_t)(kr * S::A_ROWB), bbox_bytes = (uint32_t)(kr * 128);
            for (int st = 0; st < nstages && !*abort_flag; ++st) {
                if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
                uint8_t *sa = sbase + s * STAGE;
                uint8_t *sb = sa + S::A_BOXES * ABOX;
                armed[s] = (int)ph + 1;
                if constexpr (wg_linear(MODE)) {
                    const int r0 = (k0 + st) * 64;
                    mbar_arrive_expect_tx(&full[s], 2 * abox_bytes + nb * bbox_bytes);
                    for (int j = 0; j < 2; ++j) tma_load_2d(sa + j * ABOX, &p.a_map, &full[s], mt * 128 + j * 64, r0);
                    for (int j = 0; j < nb; ++j) tma_load_2d(sb + j * BBOX, &p.b_map, &full[s], (nt * nb + j) * 64, r0);
                } else {
                    const int img = k0 + st / p.tiles_per_img;
                    const int h0 = (st % p.tiles_per_img) * p.R;
                    if constexpr (MODE == kWgConvCo) {
                        mbar_arrive_expect_tx(&full[s], (UP ? 0 : 2 * abox_bytes) + 3 * bbox_bytes);
                        if (!UP)
                            for (int j = 0; j < 2; ++j) tma_load_4d(sa + j * ABOX, &p.a_map, &full[s], j * 64, 0, h0, img);
                        for (int j = 0; j < 3; ++j) {
                            const int tap = mt * 3 + j, dh = tap / 3, dw = tap % 3;
                            tma_load_4d(sb + j * BBOX, &p.b_map, &full[s], 0, dw - 1, h0 + dh - 1, img);
                        }
                    } else {
                        mbar_arrive_expect_tx(&full[s], 9 * abox_bytes + bbox_bytes);
                        for (int tap = 0; tap < 9; ++tap) {
                            const int dh = tap / 3, dw = tap % 3;
                            tma_load_4d(sa + tap * ABOX, &p.a_map, &full[s], 0, dw - 1, h0 + dh - 1, img);
                        }
                        tma_load_4d(sb, &p.b_map, &full[s], 0, 0, h0, img);
                    }
                }
                if (++s == S::NS) { s = 0; ph ^= 1u; }
            }
            if (*abort_flag)
                for (int i = 0; i < S::NS; ++i)
                    if (armed[i] && !mbar_wait_drain(&full[i], (uint32_t)(armed[i] - 1))) atomicCAS(p.err, 0, kErrDrain);
        }
    } else if (warp == 1) {
        if (elect_one()) {
            bool issued = false;
            int s = 0;
            uint32_t ph = 0;
            const uint32_t s0 = smem_u32(sbase);
            for (int st = 0; st < nstages; ++st) {
                if (!mbar_wait(&full[s], ph, abort_flag, p.err, kErrFullWait)) break;
                tc_fence_after();
                const uint32_t a0 = s0 + s * STAGE, b0 = a0 + S::A_BOXES * ABOX;
                for (int kk = 0; kk < kr16; ++kk) {
                    const bool accum = (st | kk) != 0;
                    if constexpr (wg_linear(MODE)) {
                        // A: 2 MN blocks of 64 at ABOX; B: nb MN blocks of 64 at BBOX
                        const uint64_t ad = smem_desc(a0 + kk * 2048, ABOX, 1024, kSw128);
                        const uint64_t bd = smem_desc(b0 + kk * 2048, BBOX, 1024, kSw128);
                        mma_bf16(tmem_base, ad, bd, idesc_bf16(128, 64 * nb, true, true), accum);
                    } else if constexpr (MODE == kWgConvCo) {
                        const uint64_t ad = smem_desc(a0 + kk * 2048, ABOX, 1024, kSw128);
                        const uint64_t bd = smem_desc(b0 + kk * 2048, BBOX, 1024, kSw128);
                        mma_bf16(tmem_base, ad, bd, idesc_bf16(128, 192, true, true), accum);
                    } else {
                        // A: 64-byte swizzle, 8-row atoms of 512 B, 32-element MN blocks at ABOX
                        const uint64_t bd = smem_desc(b0 + kk * 2048, BBOX, 1024, kSw128);
#pragma unroll
                        for (int t = 0; t < 3; ++t) {
                            const uint64_t ad = smem_desc(a0 + t * 4 * ABOX + kk * 1024, ABOX, 512, kSw64);
                            mma_bf16(tmem_base + (uint32_t)(t * 64), ad, bd, idesc_bf16(128, 64, true, true), accum);
                        }
                    }
                }
                issued = true;
                mma_commit(&empty[s]);
                if (++s == S::NS) { s = 0; ph ^= 1u; }
            }
            if (issued) mma_commit(acc_full);
            else mbar_arrive(acc_full);   // nothing to accumulate: release the epilogue
            if (issued) {
                mma_commit(drain);
                if (!mbar_wait_drain(drain, 0)) atomicCAS(p.err, 0, kErrDrain);
            }
        }
    } else if (UP && warp >= 6) {
        // ------------------------------------------------ dY builders (warps 6..9, UP)
        const int bt = threadIdx.x - 192;   // 0..127
        const int o = bt & 15;              // channel octet (of 16) of every item of this thread
        const int Ho = p.H >> 1, Wo = p.W >> 1;
        const int nitems = (p.R >> 1) * Wo * 16;
        // an item's window (pooled row prow of the stage's, column pw) does not depend on the
        // stage: worked out once (wi = prow * Wo + pw; prow -1: no item)
        int wi_[4], prow_[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int i = bt + 128 * m;
            wi_[m] = i >> 4;
            prow_[m] = i < nitems ? wi_[m] / Wo : -1;
        }
        // this thread's dP and code loads of stage st (zero past the image)
        auto load_stage = [&](int st, uint4 (&pv)[4], uint2 (&cd)[4]) {
            const int img = k0 + st / p.tiles_per_img;
            const int h0 = (st % p.tiles_per_img) * p.R;
            const long long wbase = ((long long)img * Ho + (h0 >> 1)) * Wo;   // window (h0/2, 0)
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int phr = (h0 >> 1) + prow_[m];
                pv[m] = make_uint4(0, 0, 0, 0);
                cd[m] = make_uint2(0, 0);
                if (st < nstages && prow_[m] >= 0 && phr < Ho) {
                    const size_t off = (size_t)(wbase + wi_[m]) * 128 + 8 * o;
                    pv[m] = __ldg(reinterpret_cast<const uint4 *>(p.dp + off));
                    cd[m] = __ldg(reinterpret_cast<const uint2 *>(p.up_code + off));
                }
            }
        };
        int s = 0;
        uint32_t ph = 0;
        uint4 pv[4], pvn[4];
        uint2 cd[4], cdn[4];
        load_stage(0, pv, cd);
        for (int st = 0; st < nstages && !*abort_flag; ++st) {
            load_stage(st + 1, pvn, cdn);   // one stage ahead: its latency overlaps this stage
            if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
            uint8_t *sa = sbase + s * STAGE + (o >> 3) * ABOX;   // box of channels 64 (o / 8) ..
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int prow = prow_[m], pw = wi_[m] - prow * Wo;
                if (prow < 0) continue;
                const uint32_t t0 = cd[m].x | (cd[m].x >> 4), t1 = cd[m].y | (cd[m].y >> 4);
                const uint32_t sel0 = (t0 & 0xFFu) | ((t0 >> 8) & 0xFF00u);
                const uint32_t sel1 = (t1 & 0xFFu) | ((t1 >> 8) & 0xFF00u);
#pragma unroll
                for (int kh = 0; kh < 2; ++kh)
#pragma unroll
                    for (int kw = 0; kw < 2; ++kw) {
                        const int k = (2 * prow + kh) * p.W + 2 * pw + kw;   // stage pixel row
                        *reinterpret_cast<uint4 *>(sa + k * 128 + (((o & 7) ^ (k & 7)) << 4)) =
                            unpool_select(pv[m], sel0, sel1, 0xFFu << (8 * (2 * kh + kw)));
                    }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
            if (++s == S::NS) { s = 0; ph ^= 1u; }
#pragma unroll
            for (int m = 0; m < 4; ++m) { pv[m] = pvn[m]; cd[m] = cdn[m]; }
        }
    } else {
        const int q = warp & 3;
        const int row = q * 32 + lane;
        mbar_wait(acc_full, 0, abort_flag, p.err, kErrAccWait);
        named_bar_sync(1, 128);
        if (!*abort_flag) {
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16);
            float *part = p.partial + (size_t)split * p.M * p.N;
            const bool empty_slice = nstages == 0;
            if constexpr (wg_linear(MODE)) {
                const int m = mt * 128 + row;
                // one K split: straight into the gradient (the NHWC flatten's row m is
                // the NCHW row c * oHW + hw); else this split's partial
                float *dst = p.out ? p.out + ((size_t)(m % p.oC) * p.oHW + m / p.oC) * p.N
                                   : part + (size_t)m * p.N;
                dst += nt * 64 * nb;
#pragma unroll 1
                for (int cc = 0; cc < 2 * nb; ++cc) {
                    float v[32];
                    tmem_ld32(taddr + 32 * cc, v);
                    if (m < p.M) store_row32(dst + 32 * cc, v, empty_slice);
                }
            } else if constexpr (MODE == kWgConvCo) {
#pragma unroll 1
                for (int cc = 0; cc < 6; ++cc) {
                    float v[32];
                    tmem_ld32(taddr + 32 * cc, v);
                    store_row32(part + (size_t)row * p.N + mt * 192 + 32 * cc, v, empty_slice);
                }
            } else {
#pragma unroll 1
                for (int t = 0; t < 3; ++t) {
                    const int m = t * 128 + row;   // = tap * 32 + ci
#pragma unroll 1
                    for (int cc = 0; cc < 2; ++cc) {
                        float v[32];
                        tmem_ld32(taddr + t * 64 + 32 * cc, v);
                        if (m < p.M) store_row32(part + (size_t)m * p.N + 32 * cc, v, empty_slice);
                    }
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
