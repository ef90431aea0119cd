// tc_gemm_tf32.cuh -- tcgen05 GEMM on fp32 operands (kind::tf32: the tensor
// core reads each fp32 operand with a 10-bit mantissa and accumulates in fp32
// in TMEM), for the language model's Linear layers:
//
//   D[m, n] = sum_k A(m, k) B(k, n)
//
// The operands come straight from the row-major fp32 tensors through TMA with
// the 128-byte swizzle, in whichever major order the tensor has, so no
// transposed or converted copies are made:
//   A K-major  : A(m, k) = X[m][k]   forward, input gradient   box {32 k, 128 m}
//   A MN-major : A(m, k) = X[k][m]   weight gradient           4 boxes {32 m, 32 k}
//   B MN-major : B(k, n) = W[k][n]   forward (W [in][out])     BN/32 boxes {32 n, 32 k}
//   B K-major  : B(k, n) = W[n][k]   input gradient (W^T)      box {32 k, BN n}
//   B MN-major : B(k, n) = dY[k][n]  weight gradient
// A K stage is 32 fp32 (one 128-byte swizzle row for K-major, 32 rows for
// MN-major): four K8 MMAs of M = 128, N = BN.  K-major operands use the
// 128-byte swizzle like the bf16 kernels (tc_gemm.cuh): a K8 step is 32 bytes
// along a row.  MN-major operands of 32-bit elements have one valid layout,
// the 128-byte swizzle over 32-byte atoms (TMA's 128B_ATOM_32B, descriptor
// layout type 1): 128-byte rows of 32 MN elements, swizzled in groups of 4 K
// rows (512 bytes, the SBO); a K8 step is 8 rows (1024 bytes), and the
// 32-element MN atoms (one TMA box each) sit 4 KB apart (the LBO).
//
// Up to three B segments (the Q/K/V weights of one attention layer): with
// b_seg_by_n the n tile t reads segment t (its N coordinates restart at 0);
// otherwise the K range is split into segments of seg_k (the input gradient of
// the fused Q/K/V projection: dX = dQ Wq^T + dK Wk^T + dV Wv^T).
//
// Epilogues (fp32 out[m * ldo + n], 4 warps, one accumulator row per thread):
//   kTfStore  : acc (+ bias[seg][n]) (+ res[m * ldr + n]) (relu)
//   kTfMask   : acc * (mask[m * ldm + n] > 0)         (ReLU backward)
//   kTfPartial: partial[split][M][N] of a K split     (weight gradients; summed
//               in split order by a separate pass: deterministic)
// Persistent CTAs, warp-specialised (TMA producer / MMA issuer / 4 epilogue
// warps), double-buffered TMEM accumulators; every wait is bounded.
#pragma once

#include "tc_common.cuh"

namespace zb {
namespace tc {

enum Tf32Epi { kTfStore = 0, kTfMask = 1, kTfPartial = 2 };

struct GemmTf32Params {
    CUtensorMap a_map;
    CUtensorMap b_map[3];
    int M, N, K;            // M % 128 == 0, N % BN == 0, K % 32 == 0
    int m_tiles, n_tiles;
    int ksplit, kper;       // K splits and 32-wide K stages per split
    int nseg;               // B segments in use (1..3)
    int b_seg_by_n;         // 1: B segment = n tile; 0: B segment = k / seg_k
    int seg_k;
    float *out;             // [M][ldo]
    int ldo;
    const float *bias[3];   // kTfStore, optional, per segment (column n - seg * BN when b_seg_by_n)
    const float *res;       // kTfStore, optional residual [M][ldr]
    int ldr;
    int relu;
    const float *mask;      // kTfMask: [M][ldm]
    int ldm;
    float *partial;         // kTfPartial: [ksplit][M][N]
    int *err;
};

__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4)                      // D format: f32
           | (2u << 7)                    // A format: tf32
           | (2u << 10)                   // B format: tf32
           | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

template <int BN, int NS>
struct GemmTf32Shape {
    static constexpr int ABYTES = 128 * 128;   // 128 rows x 32 fp32
    static constexpr int BBYTES = BN * 128;
    static constexpr int STAGE = ABYTES + BBYTES;
    static constexpr uint32_t TMEM_COLS = (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
    static constexpr int SMEM = 1024 + NS * STAGE + 256;
    static_assert(BN % 32 == 0 && BN <= 256, "BN");
};

template <int BN, bool AMN, bool BMN, int EPI, int NS>
__global__ void __launch_bounds__(192, 1) gemm_tf32_kernel(const __grid_constant__ GemmTf32Params p) {
    griddep_launch();
    using S = GemmTf32Shape<BN, NS>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t *sbase = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sbase + NS * S::STAGE);
    uint64_t *full = bars, *empty = bars + NS, *acc_full = bars + 2 * NS, *acc_empty = acc_full + 2;
    uint64_t *drain = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *armed = const_cast<int *>(abort_flag) + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t IDESC = idesc_tf32(128, BN, AMN, BMN);
    const int mn_tiles = p.m_tiles * p.n_tiles;
    const int num_tiles = mn_tiles * p.ksplit;
    const int ksteps = p.K / 32;

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
        // ------------------------------------------------ TMA producer
        if (elect_one()) {
            prefetch_tmap(&p.a_map);
            for (int j = 0; j < p.nseg; ++j) prefetch_tmap(&p.b_map[j]);
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
                    if (AMN) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) tma_load_2d(st + j * 4096, &p.a_map, &full[s], mt * 128 + 32 * j, k * 32);
                    } else {
                        tma_load_2d(st, &p.a_map, &full[s], k * 32, mt * 128);
                    }
                    // B segment and its coordinates
                    int seg = 0, kk0 = k * 32, n0 = nt * BN;
                    if (p.b_seg_by_n) { seg = nt; n0 = 0; }
                    else if (p.seg_k) { seg = kk0 / p.seg_k; kk0 -= seg * p.seg_k; }
                    const CUtensorMap *bm = &p.b_map[seg];
                    if (BMN) {
#pragma unroll
                        for (int j = 0; j < BN / 32; ++j) tma_load_2d(st + S::ABYTES + j * 4096, bm, &full[s], n0 + 32 * j, kk0);
                    } else {
                        tma_load_2d(st + S::ABYTES, bm, &full[s], kk0, n0);
                    }
                    if (++s == NS) { s = 0; ph ^= 1u; }
                }
            }
            if (*abort_flag)
                for (int i = 0; i < NS; ++i)
                    if (armed[i] && !mbar_wait_drain(&full[i], (uint32_t)(armed[i] - 1))) atomicCAS(p.err, 0, kErrDrain);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
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
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = AMN ? smem_desc(a0 + kk * 1024, 4096, 512, kSw128B32)
                                                : smem_desc(a0 + kk * 32, 16, 1024, kSw128);
                        const uint64_t bd = BMN ? smem_desc(b0 + kk * 1024, 4096, 512, kSw128B32)
                                                : smem_desc(b0 + kk * 32, 16, 1024, kSw128);
                        mma_tf32(d, ad, bd, IDESC, (k > kb) || kk != 0);
                    }
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
        // ------------------------------------------------ epilogue (warps 2..5)
        const int q = warp & 3;
        const int row = q * 32 + lane;
        int acc = 0;
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
            const int seg = p.b_seg_by_n ? nt : 0;
#pragma unroll 1
            for (int cc = 0; cc < BN / 32; ++cc) {
                float v[32];
                tmem_ld32(taddr + 32 * cc, v);
                if (cc == BN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[acc]);
                }
                if (m >= p.M) continue;
                const int n0 = nt * BN + 32 * cc;
                if constexpr (EPI == kTfPartial) {
                    float4 *dstf = reinterpret_cast<float4 *>(p.partial + ((size_t)ks * p.M + m) * p.N + n0);
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) dstf[q4] = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
                    continue;
                }
                if constexpr (EPI == kTfStore) {
                    const float *bs = p.bias[seg];
                    const int bcol = p.b_seg_by_n ? 32 * cc : n0;
                    if (bs) {
                        const float4 *b4 = reinterpret_cast<const float4 *>(bs + bcol);
#pragma unroll
                        for (int q4 = 0; q4 < 8; ++q4) {
                            const float4 bb = __ldg(b4 + q4);
                            v[4 * q4] += bb.x; v[4 * q4 + 1] += bb.y; v[4 * q4 + 2] += bb.z; v[4 * q4 + 3] += bb.w;
                        }
                    }
                    if (p.res) {
                        const float4 *r4 = reinterpret_cast<const float4 *>(p.res + (size_t)m * p.ldr + n0);
#pragma unroll
                        for (int q4 = 0; q4 < 8; ++q4) {
                            const float4 rr = __ldg(r4 + q4);
                            v[4 * q4] += rr.x; v[4 * q4 + 1] += rr.y; v[4 * q4 + 2] += rr.z; v[4 * q4 + 3] += rr.w;
                        }
                    }
                    if (p.relu) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = v[j] > 0.0f ? v[j] : 0.0f;
                    }
                } else {   // kTfMask
                    const float4 *m4 = reinterpret_cast<const float4 *>(p.mask + (size_t)m * p.ldm + n0);
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) {
                        const float4 mm = __ldg(m4 + q4);
                        if (!(mm.x > 0.0f)) v[4 * q4] = 0.0f;
                        if (!(mm.y > 0.0f)) v[4 * q4 + 1] = 0.0f;
                        if (!(mm.z > 0.0f)) v[4 * q4 + 2] = 0.0f;
                        if (!(mm.w > 0.0f)) v[4 * q4 + 3] = 0.0f;
                    }
                }
                float4 *dst = reinterpret_cast<float4 *>(p.out + (size_t)m * p.ldo + n0);
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4) dst[q4] = make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
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
