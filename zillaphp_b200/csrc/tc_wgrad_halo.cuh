// tc_wgrad_halo.cuh -- 3x3 (stride 1, pad 1) conv weight gradient on tcgen05
// with one halo tile per output tile:
//
//   dW[co][tap][ci] = sum_{b, pixel} dY[b, pixel][co] * X[b, pixel + tap offset][ci]
//
// as D[m = co][n = tap * CIN + ci] += A[k][m] * B[k][n] with K = pixels.
// Per tile (R image rows of one image) two TMA loads, both as 8-channel
// groups of 16-byte rows (the MN-major no-swizzle UMMA layout: 8 K-rows of
// 16 B per core matrix, LBO = 128 B between 8-row K groups, SBO = the group
// pitch between 8-channel MN groups):
//   dY : rows k = r * Wp + c (Wp = W + 2; the columns c >= W are out of the
//        image, so TMA fills them with zeros and they add nothing),
//   X  : the halo rows (R + 2) x Wp around the tile, zero outside the image.
// Tap (dh, dw) is then the X descriptor started dh * Wp + dw rows further on,
// so one X tile serves all nine taps; the per-tap weight-gradient kernel loads
// a shifted box per tap instead.  Rows of X read for k in the zero columns
// are finite (TMA data or zeroed padding) and are multiplied by zero.
//
// A CTA owns the column range [g * NG, (g + 1) * NG) of D (NG = 9 * CIN / NGRP)
// and a slice of the images; it accumulates over all its tiles in TMEM and
// writes one fp32 partial [split][COUT][9 * CIN] (its columns), which a
// second kernel sums in split order (deterministic).  M = COUT: 128 uses all
// TMEM lanes; 64 uses lanes 32q .. 32q + 15 of each quarter q.  COUT = 32 runs
// as M = 64: the A (dY) part of each stage has 64 channel groups' room, the
// upper four groups stay zero (never loaded), and their D rows are dropped.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer and TMEM
// owner, warps 2-5 write the partial.  Every wait is bounded (tc_common.cuh).
#pragma once

#include "tc_common.cuh"

namespace zb {
namespace tc {

struct WgradHaloParams {
    CUtensorMap dy_map;   // 4D {COUT, W, H, B} bf16, box {8, W + 2, R, 1}, no swizzle
    CUtensorMap x_map;    // 4D {CIN, W, H, B} bf16, box {8, W + 2, R + 2, 1}, no swizzle
    int B, H, W, R, Wp, HR, tiles_per_img, splits;
    int dy_region, x_region, stage_bytes;   // set by the launcher from the shape
    float *partial;       // [splits][COUT][9 * CIN]
    int *err;
};

template <int CIN, int COUT, int NGRP, int NS>
struct WgradHaloShape {
    static constexpr int MP = COUT < 64 ? 64 : COUT;   // MMA M (COUT = 32: padded with zero rows)
    static constexpr int NTOT = 9 * CIN;
    static constexpr int NG = NTOT / NGRP;          // D columns per CTA
    static constexpr uint32_t TMEM_COLS = NG <= 32 ? 32 : NG <= 64 ? 64 : NG <= 128 ? 128 : NG <= 256 ? 256 : 512;
    static constexpr int SLACK = 1024;              // X rows read past the last stage's end
    static constexpr int BAR_BYTES = 256;
    static __host__ __device__ int ksteps(int R, int Wp) { return (R * Wp + 15) / 16; }
    static __host__ __device__ int dy_region(int R, int Wp) { return ksteps(R, Wp) * 16 * 16; }
    static __host__ __device__ int x_region(int HR) { return (HR * 16 + 127) / 128 * 128; }
    static __host__ __device__ int stage_bytes(int R, int Wp, int HR) {
        return ((MP / 8) * dy_region(R, Wp) + (CIN / 8) * x_region(HR) + 1023) / 1024 * 1024;
    }
    static __host__ __device__ int smem(int R, int Wp, int HR) { return 1024 + NS * stage_bytes(R, Wp, HR) + SLACK + BAR_BYTES; }
    static_assert(COUT == 32 || COUT == 64 || COUT == 128, "MMA M must be 64 or 128");
    static_assert(CIN % 16 == 0 && NTOT % NGRP == 0 && NG % 16 == 0 && NG <= 512, "column split");
};

template <int CIN, int COUT, int NGRP, int NS>
__global__ void __launch_bounds__(192, 1) wgrad_halo_kernel(const __grid_constant__ WgradHaloParams p) {
    using S = WgradHaloShape<CIN, COUT, NGRP, NS>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    const int STAGE = p.stage_bytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + NS * STAGE + S::SLACK);
    uint64_t *full = bars, *empty = bars + NS, *acc_full = bars + 2 * NS, *drain = acc_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *armed = const_cast<int *>(abort_flag) + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // CTA -> (column group, slice of the images)
    const int grp = blockIdx.x % NGRP;
    const int split = blockIdx.x / NGRP;
    const int k0 = (int)((long long)p.B * split / p.splits);
    const int k1 = (int)((long long)p.B * (split + 1) / p.splits);
    const int ntiles = (k1 - k0) * p.tiles_per_img;
    const int n0 = grp * S::NG;
    const int KST = S::ksteps(p.R, p.Wp);
    const int DYB = (S::MP / 8) * p.dy_region;   // dY part of a stage (groups past COUT stay zero)

    // rows that TMA never writes (dY rows past R*Wp, X group padding, the
    // slack) are zeroed once
    for (int i = threadIdx.x; i < (NS * STAGE + S::SLACK) / 16; i += blockDim.x)
        *reinterpret_cast<uint4 *>(base + 16 * i) = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); armed[i] = 0; }
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

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (elect_one()) {
            prefetch_tmap(&p.dy_map);
            prefetch_tmap(&p.x_map);
            const uint32_t tx = (uint32_t)((COUT / 8) * p.R * p.Wp * 16 + (CIN / 8) * p.HR * 16);
            int s = 0;
            uint32_t ph = 0;
            for (int t = 0; t < ntiles && !*abort_flag; ++t) {
                const int b = k0 + t / p.tiles_per_img;
                const int h0 = (t % p.tiles_per_img) * p.R;
                if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
                mbar_arrive_expect_tx(&full[s], tx);
                armed[s] = (int)ph + 1;
                uint8_t *st = base + s * STAGE;
                for (int g = 0; g < COUT / 8; ++g)
                    tma_load_4d(st + g * p.dy_region, &p.dy_map, &full[s], 8 * g, 0, h0, b);
                for (int g = 0; g < CIN / 8; ++g)
                    tma_load_4d(st + DYB + g * p.x_region, &p.x_map, &full[s], 8 * g, -1, h0 - 1, b);
                if (++s == NS) { s = 0; ph ^= 1u; }
            }
            if (*abort_flag)
                for (int i = 0; i < NS; ++i)
                    if (armed[i] && !mbar_wait_drain(&full[i], (uint32_t)(armed[i] - 1))) atomicCAS(p.err, 0, kErrDrain);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (elect_one()) {
            bool issued = false;
            int s = 0;
            uint32_t ph = 0;
            // descriptors differ only in the start address (bits 0-13, 16-byte units)
            const uint64_t adesc0 = smem_desc(smem_u32(base), 128, (uint32_t)p.dy_region, kSwNone);
            const uint64_t bdesc0 = smem_desc(smem_u32(base) + (uint32_t)DYB, 128, (uint32_t)p.x_region, kSwNone);
            const uint32_t xr16 = (uint32_t)p.x_region >> 4;
            const int t_first = n0 / CIN, t_last = min(8, (n0 + S::NG - 1) / CIN);   // taps with columns here
            for (int t = 0; t < ntiles; ++t) {
                if (!mbar_wait(&full[s], ph, abort_flag, p.err, kErrFullWait)) break;
                tc_fence_after();
                const uint64_t a_st = adesc0 + (uint64_t)((uint32_t)(s * STAGE) >> 4);
                const uint64_t b_st = bdesc0 + (uint64_t)((uint32_t)(s * STAGE) >> 4);
#pragma unroll 1
                for (int k = 0; k < KST; ++k) {
                    const uint64_t ad = a_st + (uint64_t)(16 * k);   // 16 pixel rows of 16 B
#pragma unroll
                    for (int tap = 0; tap < 9; ++tap) {
                        // the part of tap's columns [tap*CIN, (tap+1)*CIN) inside [n0, n0 + NG)
                        const int lo = max(tap * CIN, n0), hi = min((tap + 1) * CIN, n0 + S::NG);
                        if (lo >= hi) continue;
                        const int dh = tap / 3, dw = tap - 3 * dh;
                        const uint64_t bd = b_st + (uint64_t)(((lo - tap * CIN) / 8) * xr16) +
                                            (uint64_t)(dh * p.Wp + dw + 16 * k);
                        const uint32_t idesc = idesc_bf16(S::MP, hi - lo, true, true);
                        const uint32_t dt = tmem_base + (uint32_t)(lo - n0);
                        // the taps of this CTA's columns share A (dY): it stays in the
                        // collector buffer from the first MMA to the last
                        if (t_first == t_last) mma_bf16(dt, ad, bd, idesc, (t | k) != 0);
                        else if (tap == t_first) mma_bf16_ca<0>(dt, ad, bd, idesc, (t | k) != 0);
                        else if (tap == t_last) mma_bf16_ca<2>(dt, ad, bd, idesc, (t | k) != 0);
                        else mma_bf16_ca<1>(dt, ad, bd, idesc, (t | k) != 0);
                    }
                }
                issued = true;
                mma_commit(&empty[s]);
                if (++s == NS) { s = 0; ph ^= 1u; }
            }
            if (issued) mma_commit(acc_full);
            else mbar_arrive(acc_full);   // nothing to accumulate: release the epilogue
            if (issued) {
                mma_commit(drain);
                if (!mbar_wait_drain(drain, 0)) atomicCAS(p.err, 0, kErrDrain);
            }
        }
    } else {
        // ------------------------------------------------ partial writer (warps 2..5)
        const int q = warp & 3;
        mbar_wait(acc_full, 0, abort_flag, p.err, kErrAccWait);
        named_bar_sync(1, 128);
        if (!*abort_flag) {
            tc_fence_after();
            // row of D held by this thread's TMEM lane (M = 64: lanes 32q .. 32q + 15)
            const int m = S::MP == 128 ? q * 32 + lane : q * 16 + lane;
            const bool row_ok = (S::MP == 128 || lane < 16) && m < COUT;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16);
            float *part = p.partial + ((size_t)split * COUT + (row_ok ? m : 0)) * S::NTOT + n0;
            const bool empty_slice = ntiles == 0;
#pragma unroll 1
            for (int cc = 0; cc < S::NG / 32; ++cc) {
                float v[32];
                tmem_ld32(taddr + 32 * cc, v);
                if (!row_ok) continue;
                float4 *d4 = reinterpret_cast<float4 *>(part + 32 * cc);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    d4[j] = empty_slice ? make_float4(0.0f, 0.0f, 0.0f, 0.0f)
                                        : make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
            if constexpr (S::NG % 32 != 0) {   // the last 16 columns
                constexpr int c16 = S::NG / 32 * 32;
                float v[16];
                tmem_ld16(taddr + c16, v);
                if (row_ok) {
                    float4 *d4 = reinterpret_cast<float4 *>(part + c16);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        d4[j] = empty_slice ? make_float4(0.0f, 0.0f, 0.0f, 0.0f)
                                            : make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
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
