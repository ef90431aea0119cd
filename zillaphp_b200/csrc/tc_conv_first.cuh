// tc_conv_first.cuh -- the first conv (one input channel, 3x3, pad 1, same
// size) + bias + ReLU on tcgen05, NHWC bf16 output:
//
//   out[p][co] = relu(b[co] + sum_t x[p + t] w[co][t])
//
// as one M = 128, N = CO, K = 32 MMA per tile of 128 consecutive output
// pixels (the tile's outputs are one contiguous run of 128 * CO bf16).  The
// fp32 operands keep their precision through a two-term bf16 split,
// x = xh + xl and w = wh + wl:
//
//   k   0..8   9    10..18  19..27  28    29..31
//   A   xh_t   1    xl_t    xh_t    1     0          (im2col row of pixel p)
//   B   wh_t   bh   wh_t    wl_t    bl    0          (row of channel co)
//
// so D = sum_t (xh wh + xl wh + xh wl) + bh + bl; the dropped xl wl term is
// below 2^-16 of each product.  Both operands are K-major without swizzle:
// 16-byte rows of 8 K values, [K chunk][row][16 B] (LBO = the chunk pitch,
// SBO = 128 B between 8-row groups).
//
// One CTA = 4 warps; thread m owns tile row m: it builds that im2col row (the
// 9 taps of the NEXT tile are loaded while the current MMA runs), and after
// the MMA reads its TMEM lane (row m) into the tile's staged output, which one
// bulk copy writes to global memory (the tile is one contiguous run).  Thread
// 0 issues the two K16 MMAs and the copy.  Several CTAs share an SM (32 TMEM
// columns each).  Every wait is bounded (tc_common.cuh).  (Writing the rows
// straight from registers, 64 bytes per thread, with a second accumulator so
// that a tile's MMA overlapped the previous tile's epilogue, measured slower:
// 0.156 against 0.132 ms for this kernel plus the packing at batch 8192.)
//
// EXTRA: independent side work (a functor called once per thread with its
// grid-wide index and the grid's thread count) that the CTAs run after
// issuing their first tile's loads; the engine passes its bf16 weight
// packing, so that costs no launch of its own.
#pragma once

#include "tc_common.cuh"

namespace zb {
namespace tc {

template <int CO>
struct ConvFirstTcShape {
    static constexpr int ABYTES = 4 * 128 * 16;   // 4 K chunks x 128 rows x 16 B
    static constexpr int BBYTES = 4 * CO * 16;
    static constexpr int OBYTES = 128 * CO * 2;   // one staged output tile
    static constexpr int SMEM = 1024 + ABYTES + BBYTES + 2 * OBYTES + 64;   // two output buffers
    static constexpr uint32_t TMEM_COLS = 32;
    static_assert(CO == 32, "one 32-column TMEM accumulator");
};

// bf16 bits of the two-term split of an fp32 value: hi = rn(v), lo = rn(v - hi)
__device__ __forceinline__ void split_bf16(float v, uint16_t &hi, uint16_t &lo) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    const __nv_bfloat16 l = __float2bfloat16_rn(v - __bfloat162float(h));
    hi = *reinterpret_cast<const uint16_t *>(&h);
    lo = *reinterpret_cast<const uint16_t *>(&l);
}

struct ConvFirstNoExtra {
    __device__ void operator()(long long, long long) const {}
};

template <int CO, class EXTRA = ConvFirstNoExtra>
__global__ void __launch_bounds__(128, 8) conv_first_tc_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                             const float *__restrict__ bias,
                                                             __nv_bfloat16 *__restrict__ out, int B, int H, int W,
                                                             int *err, const __grid_constant__ EXTRA extra) {
    using S = ConvFirstTcShape<CO>;
    griddep_launch();
    griddep_wait();
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sA = base;
    uint8_t *sB = sA + S::ABYTES;
    uint8_t *sO = sB + S::BBYTES;
    uint64_t *mma_done = reinterpret_cast<uint64_t *>(sO + 2 * S::OBYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    const int m = threadIdx.x, warp = m >> 5;
    const long long npix = (long long)B * H * W;
    const long long ntiles = (npix + 127) / 128;

    // weight rows: thread co (< CO) writes its 32 K values as 4 chunks
    if (m < CO) {
        uint16_t v[32];
#pragma unroll
        for (int t = 0; t < 9; ++t) {
            uint16_t hi, lo;
            split_bf16(__ldg(w + m * 9 + t), hi, lo);
            v[t] = hi;
            v[10 + t] = hi;
            v[19 + t] = lo;
        }
        uint16_t bh, bl;
        split_bf16(__ldg(bias + m), bh, bl);
        v[9] = bh;
        v[28] = bl;
        v[29] = v[30] = v[31] = 0;
#pragma unroll
        for (int kc = 0; kc < 4; ++kc)
            *reinterpret_cast<uint4 *>(sB + kc * (CO * 16) + m * 16) = *reinterpret_cast<const uint4 *>(&v[8 * kc]);
    }
    if (m == 0) {
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, S::TMEM_COLS);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    constexpr uint32_t IDESC = idesc_bf16(128, CO, false, false);
    const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);

    // the 9 taps of pixel p (zero outside the image or past the batch)
    auto load_taps = [&](long long tile, float (&xt)[9]) {
        const long long p = tile * 128 + m;
        const bool ok = p < npix;
        const long long img = ok ? p / (H * W) : 0;
        const int hw = ok ? (int)(p - img * H * W) : 0;
        const int h = hw / W, c = hw - h * W;
        const float *xb = x + img * H * W;
#pragma unroll
        for (int t = 0; t < 9; ++t) {
            const int ih = h + t / 3 - 1, iw = c + t % 3 - 1;
            xt[t] = (ok && (unsigned)ih < (unsigned)H && (unsigned)iw < (unsigned)W) ? __ldg(xb + ih * W + iw) : 0.0f;
        }
    };

    float xt[9];
    long long tile = blockIdx.x;
    if (tile < ntiles) load_taps(tile, xt);
    extra((long long)blockIdx.x * blockDim.x + threadIdx.x, (long long)gridDim.x * blockDim.x);
    uint32_t ph = 0;
    int ob = 0;   // output buffer of this tile (two, so one tile's copy overlaps the next tile)
    for (; tile < ntiles; tile += gridDim.x, ob ^= 1) {
        // im2col row m of this tile
        {
            const bool ok = tile * 128 + m < npix;
            uint16_t v[32];
#pragma unroll
            for (int t = 0; t < 9; ++t) {
                uint16_t hi, lo;
                split_bf16(xt[t], hi, lo);
                v[t] = hi;
                v[10 + t] = lo;
                v[19 + t] = hi;
            }
            const __nv_bfloat16 one = __float2bfloat16_rn(ok ? 1.0f : 0.0f);
            v[9] = v[28] = *reinterpret_cast<const uint16_t *>(&one);
            v[29] = v[30] = v[31] = 0;
#pragma unroll
            for (int kc = 0; kc < 4; ++kc)
                *reinterpret_cast<uint4 *>(sA + kc * 2048 + m * 16) = *reinterpret_cast<const uint4 *>(&v[8 * kc]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        if (m == 0) bulk_wait_read<1>();   // the copy of two tiles ago has read this tile's output buffer
        __syncthreads();   // row writes visible; the previous tile's TMEM reads are done
        if (m == 0) {
            tc_fence_after();
#pragma unroll
            for (int s = 0; s < 2; ++s)
                mma_bf16(tmem_base, smem_desc(a0 + s * 4096, 2048, 128, kSwNone),
                         smem_desc(b0 + s * (2 * CO * 16), CO * 16, 128, kSwNone), IDESC, s != 0);
            mma_commit(mma_done);
        }
        // the next tile's taps load while the MMA runs
        const long long next = tile + gridDim.x;
        if (next < ntiles) load_taps(next, xt);
        if (!mbar_wait(mma_done, ph, abort_flag, err, kErrAccWait)) break;
        ph ^= 1u;
        tc_fence_after();
        float v[32];
        tmem_ld32(tmem_base + ((uint32_t)(warp * 32) << 16), v);
        // row m of the staged tile (64 B): at step j thread m stores chunk (j + m/2) & 3,
        // so the 8 threads of a quarter-warp hit 8 different 16-byte bank slots
        uint4 pk[4];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
            pk[q4] = make_uint4(relu_bf16x2(v[8 * q4 + 0], v[8 * q4 + 1]), relu_bf16x2(v[8 * q4 + 2], v[8 * q4 + 3]),
                                relu_bf16x2(v[8 * q4 + 4], v[8 * q4 + 5]), relu_bf16x2(v[8 * q4 + 6], v[8 * q4 + 7]));
        const int rot = (m >> 1) & 3;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int q4 = (j + rot) & 3;
            uint4 val = pk[0];
            if (q4 == 1) val = pk[1];
            if (q4 == 2) val = pk[2];
            if (q4 == 3) val = pk[3];
            *reinterpret_cast<uint4 *>(sO + ob * S::OBYTES + m * (CO * 2) + q4 * 16) = val;
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (m == 0) {
            const long long p0 = tile * 128;
            const long long np = npix - p0 < 128 ? npix - p0 : 128;
            bulk_store(out + p0 * CO, sO + ob * S::OBYTES, (uint32_t)(np * CO * 2));
            bulk_commit();
        }
    }
    if (m == 0) bulk_wait_all();
    // after an abort, the MMA in flight finishes before its TMEM is freed
    if (m == 0 && *abort_flag && !mbar_wait_drain(mma_done, ph)) atomicCAS(err, 0, kErrDrain);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_base, S::TMEM_COLS);
}

}  // namespace tc
}  // namespace zb
