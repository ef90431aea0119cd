// tc_gemm.cuh -- tcgen05 GEMM: D[m, n] = sum_k A[m][k] * B(k, n) (bf16
// operands, fp32 accumulation in TMEM), used for the Linear layers:
//   forward          A = X [rows][in],     B = W [in][out] (MN-major)  -> Z [rows][out]
//   input gradient   A = dZ [rows][out],   B = W [in][out] (K-major)   -> dX [rows][in]
// Both read the same packed bf16 copy of W: K-major B tiles are BN rows of 64
// k (one box); MN-major B tiles are 64 k rows of BN, as BN / 64 boxes of
// 64 x 64 (128-byte swizzle; 8-row groups 1024 B apart, 64-wide n blocks one
// box apart).
// Tiles of 128 x BN, K staged 64 elements (128 B, 128-byte swizzle) per TMA
// box; persistent CTAs, warp-specialised (producer / MMA / 4 epilogue warps),
// double-buffered TMEM accumulators.
//
// Epilogues:
//   kGemmBiasRelu: bf16 relu(acc + bias[n])        (Linear forward + ReLU)
//   kGemmStore   : bf16 acc                       (Linear input gradient): each
//                  128 x 32 chunk is staged in shared memory with the 64-byte
//                  swizzle and written by one TMA store (double-buffered), so
//                  the output goes out as whole lines, not 16-byte pieces of
//                  32 different rows per warp store
//   kGemmPartial : fp32 acc of one K split into partial[split][M][N]; the
//                  splits are summed in split order by a separate pass
//                  (small batches: few M tiles, so K is split to fill the SMs)
#pragma once

#include "tc_common.cuh"

namespace zb {
namespace tc {

enum GemmEpi { kGemmBiasRelu = 0, kGemmStore = 1, kGemmPartial = 2 };

struct GemmTcParams {
    CUtensorMap a_map;   // 2D {K, M} bf16, box {64, 128}
    CUtensorMap b_map;   // 2D {K, N} bf16, box {64, BN}; MN-major: 2D {N, K}, box {64, 64}
    CUtensorMap out_map; // kGemmStore: 2D {N, M} bf16, box {32, 128}, 64-byte swizzle
    int M, N, K;         // N % BN == 0, K % 64 == 0
    int m_tiles, n_tiles;
    int ksplit, kper;    // K splits (1 unless kGemmPartial) and 64-wide k steps per split
    const float *bias;   // [N]
    __nv_bfloat16 *out;  // [M][N]
    float *partial;      // kGemmPartial: [ksplit][M][N]
    int *err;
};

template <int BN, int NS>
struct GemmTcShape {
    static constexpr int ABYTES = 128 * 128;
    static constexpr int BBYTES = BN * 128;
    static constexpr int STAGE = ABYTES + BBYTES;
    static constexpr uint32_t TMEM_COLS = (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
    static constexpr int OUT_STAGE = 128 * 32 * 2;   // kGemmStore: one staged 128 x 32 chunk
    static constexpr int SMEM = 1024 + NS * STAGE + 2 * OUT_STAGE + 256;
    static_assert(BN % 32 == 0 && BN <= 256, "BN");
};

template <int BN, int EPI, int NS, bool BMN = false>
__global__ void __launch_bounds__(192, 1) gemm_tc_kernel(const __grid_constant__ GemmTcParams p) {
    static_assert(!BMN || BN % 64 == 0, "MN-major B tiles are whole 64-wide boxes");
    griddep_launch();
    using S = GemmTcShape<BN, NS>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *sbase = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t *sout = sbase + NS * S::STAGE;   // [2] staged output chunks (kGemmStore)
    uint64_t *bars = reinterpret_cast<uint64_t *>(sout + 2 * S::OUT_STAGE);
    uint64_t *full = bars, *empty = bars + NS, *acc_full = bars + 2 * NS, *acc_empty = acc_full + 2;
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *armed = const_cast<int *>(abort_flag) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t IDESC = idesc_bf16(128, BN, false, BMN);
    const int mn_tiles = p.m_tiles * p.n_tiles;
    const int num_tiles = mn_tiles * p.ksplit;
    const int ksteps = p.K / 64;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NS; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); armed[i] = 0; }
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
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
            if (EPI == kGemmStore) prefetch_tmap(&p.out_map);
            int s = 0;
            uint32_t ph = 0;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                const int mn = tile % mn_tiles, ks = tile / mn_tiles;
                const int mt = mn % p.m_tiles, nt = mn / p.m_tiles;
                const int kb = ks * p.kper, ke = min(ksteps, kb + p.kper);
                for (int k = kb; k < ke; ++k) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, kErrEmptyWait)) break;
                    mbar_arrive_expect_tx(&full[s], S::STAGE);
                    armed[s] = (int)ph + 1;
                    uint8_t *st = sbase + s * S::STAGE;
                    tma_load_2d(st, &p.a_map, &full[s], k * 64, mt * 128);
                    if constexpr (BMN) {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_2d(st + S::ABYTES + j * 8192, &p.b_map, &full[s], nt * BN + j * 64, k * 64);
                    } else {
                        tma_load_2d(st + S::ABYTES, &p.b_map, &full[s], k * 64, nt * BN);
                    }
                    if (++s == NS) { s = 0; ph ^= 1u; }
                }
            }
            if (*abort_flag)
                for (int i = 0; i < NS; ++i)
                    if (armed[i] && !mbar_wait_drain(&full[i], (uint32_t)(armed[i] - 1))) atomicCAS(p.err, 0, kErrDrain);
        }
    } else if (warp == 1) {
        if (elect_one()) {
            bool issued = false;
            int s = 0, acc = 0;
            uint32_t ph = 0, acc_ph = 0;
            const uint32_t s0 = smem_u32(sbase);
            for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1u, abort_flag, p.err, kErrAccWait)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                bool ok = true;
                const int ks = tile / mn_tiles;
                const int kb = ks * p.kper, ke = min(ksteps, kb + p.kper);
                for (int k = kb; k < ke; ++k) {
                    if (!mbar_wait(&full[s], ph, abort_flag, p.err, kErrFullWait)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = s0 + s * S::STAGE, b0 = a0 + S::ABYTES;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_bf16(d, smem_desc(a0 + kk * 32, 16, 1024, kSw128),
                                 BMN ? smem_desc(b0 + kk * 2048, 8192, 1024, kSw128) : smem_desc(b0 + kk * 32, 16, 1024, kSw128),
                                 IDESC, (k > kb) || kk != 0);
                    issued = true;
                    mma_commit(&empty[s]);
                    if (++s == NS) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                mma_commit(&acc_full[acc]);
                if (++acc == 2) { acc = 0; acc_ph ^= 1u; }
            }
            if (issued) {
                mma_commit(drain);
                if (!mbar_wait_drain(drain, 0)) atomicCAS(p.err, 0, kErrDrain);
            }
        }
    } else {
        const int q = warp & 3;
        const int row = q * 32 + lane;
        int acc = 0, sb = 0;
        uint32_t acc_ph = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int mn = tile % mn_tiles, ks = tile / mn_tiles;
            const int mt = mn % p.m_tiles, nt = mn / p.m_tiles;
            mbar_wait(&acc_full[acc], acc_ph, abort_flag, p.err, kErrAccWait);
            named_bar_sync(1, 128);
            if (*abort_flag) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
            const int m = mt * 128 + row;
#pragma unroll 1
            for (int cc = 0; cc < BN / 32; ++cc) {
                float v[32];
                tmem_ld32(taddr + 32 * cc, v);
                if (cc == BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[acc]);
                }
                const int n0 = nt * BN + 32 * cc;
                if constexpr (EPI == kGemmStore) {
                    // every epilogue thread takes part (the barriers); the TMA store drops rows >= M
                    if (threadIdx.x == 64) bulk_wait_read<1>();   // the store that last read this buffer
                    named_bar_sync(1, 128);
                    uint8_t *buf = sout + sb * S::OUT_STAGE;
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint4 pk;
                        __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                        for (int e = 0; e < 4; ++e) h2[e] = __floats2bfloat162_rn(v[q4 * 8 + 2 * e], v[q4 * 8 + 2 * e + 1]);
                        const uint32_t o = (uint32_t)(row * 64 + 16 * q4);   // 64-byte swizzle: 16-byte unit ^ (row / 2) % 4
                        *reinterpret_cast<uint4 *>(buf + (o ^ (((o >> 7) & 3u) << 4))) = pk;
                    }
                    fence_proxy_async_smem();
                    named_bar_sync(1, 128);
                    if (threadIdx.x == 64) {
                        tma_store_2d(&p.out_map, buf, n0, mt * 128);
                        bulk_commit();
                    }
                    sb ^= 1;
                    continue;
                }
                if (m >= p.M) continue;
                if constexpr (EPI == kGemmPartial) {
                    float4 *dstf = reinterpret_cast<float4 *>(p.partial + ((size_t)ks * p.M + m) * p.N + n0);
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) dstf[q4] = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
                    continue;
                }
                if constexpr (EPI == kGemmBiasRelu) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float x = v[j] + __ldg(p.bias + n0 + j);
                        v[j] = x > 0.0f ? x : 0.0f;
                    }
                }
                uint4 *dst = reinterpret_cast<uint4 *>(p.out + (size_t)m * p.N + n0);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    uint4 pk;
                    __nv_bfloat162 *h2 = reinterpret_cast<__nv_bfloat162 *>(&pk);
#pragma unroll
                    for (int e = 0; e < 4; ++e) h2[e] = __floats2bfloat162_rn(v[q4 * 8 + 2 * e], v[q4 * 8 + 2 * e + 1]);
                    dst[q4] = pk;
                }
            }
            if (++acc == 2) { acc = 0; acc_ph ^= 1u; }
        }
        if (EPI == kGemmStore && threadIdx.x == 64) bulk_wait_all();   // stores complete before exit
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, S::TMEM_COLS);
}

}  // namespace tc
}  // namespace zb
