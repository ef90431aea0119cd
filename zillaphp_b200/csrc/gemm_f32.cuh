// gemm_f32.cuh -- fp32 CUDA-core implicit GEMM used by the exact-fp32 path
// (the reference's matmul_dev / conv2d_*_dev semantics within 1e-4).
//
// C[m, n] = sum_k A(m, k) * B(k, n), where A and B are gather functors, so
// the same tiled kernel serves plain row-major GEMMs and the three
// convolution contractions (forward, input gradient, weight gradient) on
// NCHW tensors without materialising im2col.  256 threads per block, a tile
// shape picked per problem (run_simt_gemm), register-prefetched next k tile,
// optional split-K whose partials are combined in split order (deterministic).
#pragma once

#include "common.cuh"

namespace zb {

constexpr int kGBK = 16, kGThreads = 256;

// Problem concept:
//   int M, N, K;
//   static constexpr bool kAMFast, kBNFast;   // coalescing direction of loads
//   __device__ float a(int m, int k) const;   // callers guarantee m<M, k<K
//   __device__ float b(int k, int n) const;
//   __device__ void store(int m, int n, float v) const;
//   __device__ float init(int m, int n) const;    // initial accumulator
//   static constexpr bool kExactOrder;            // acc = acc + a*b, separately rounded,
//                                                 // k ascending (the reference CPU order)
//
// Tile BM x BN x 16 per 256-thread block; thread (ty, tx) of the
// (BM/TM) x (BN/TN) thread grid owns rows ty + (BM/TM)*i, columns tx + (BN/TN)*j.
template <class P, int BM, int BN, int TM, int TN>
__global__ void __launch_bounds__(kGThreads) simt_gemm_kernel(P p, float *__restrict__ ws,
                                                              int k_per_split) {
    constexpr int TX = BN / TN, TY = BM / TM;
    static_assert(TX * TY == kGThreads, "thread grid");
    constexpr int RA = BM * kGBK / kGThreads, RB = BN * kGBK / kGThreads;
    static_assert(RA >= 1 && RB >= 1 && BM * kGBK % kGThreads == 0 && BN * kGBK % kGThreads == 0, "loads");
    __shared__ float As[kGBK][BM + 4];
    __shared__ float Bs[kGBK][BN + 4];
    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;   // M tiles on x (up to 2^31-1)
    const int kb = blockIdx.z * k_per_split;
    const int ke = min(p.K, kb + k_per_split);

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int m = m0 + ty + TY * i, n = n0 + tx + TX * j;
            acc[i][j] = (!ws && m < p.M && n < p.N) ? p.init(m, n) : 0.0f;
        }

    float ra[RA], rb[RB];
    auto load = [&](int k0) {
#pragma unroll
        for (int r = 0; r < RA; ++r) {
            const int e = tid + r * kGThreads;
            int mm, kk;
            if (P::kAMFast) { mm = e % BM; kk = e / BM; } else { mm = e / kGBK; kk = e % kGBK; }
            const int m = m0 + mm, k = k0 + kk;
            ra[r] = (m < p.M && k < ke) ? p.a(m, k) : 0.0f;
        }
#pragma unroll
        for (int r = 0; r < RB; ++r) {
            const int e = tid + r * kGThreads;
            int nn, kk;
            if (P::kBNFast) { nn = e % BN; kk = e / BN; } else { nn = e / kGBK; kk = e % kGBK; }
            const int n = n0 + nn, k = k0 + kk;
            rb[r] = (n < p.N && k < ke) ? p.b(k, n) : 0.0f;
        }
    };
    auto stash = [&]() {
#pragma unroll
        for (int r = 0; r < RA; ++r) {
            const int e = tid + r * kGThreads;
            if (P::kAMFast) As[e / BM][e % BM] = ra[r]; else As[e % kGBK][e / kGBK] = ra[r];
        }
#pragma unroll
        for (int r = 0; r < RB; ++r) {
            const int e = tid + r * kGThreads;
            if (P::kBNFast) Bs[e / BN][e % BN] = rb[r]; else Bs[e % kGBK][e / kGBK] = rb[r];
        }
    };

    if (kb < ke) load(kb);
    for (int k0 = kb; k0 < ke; k0 += kGBK) {
        __syncthreads();
        stash();
        __syncthreads();
        if (k0 + kGBK < ke) load(k0 + kGBK);
#pragma unroll
        for (int kk = 0; kk < kGBK; ++kk) {
            float av[TM], bv[TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) av[i] = As[kk][ty + TY * i];
#pragma unroll
            for (int j = 0; j < TN; ++j) bv[j] = Bs[kk][tx + TX * j];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) {
                    if constexpr (P::kExactOrder) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
                    else acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                }
        }
    }

#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int m = m0 + ty + TY * i;
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int n = n0 + tx + TX * j;
            if (n >= p.N) continue;
            if (ws) ws[((size_t)blockIdx.z * p.M + m) * p.N + n] = acc[i][j];
            else p.store(m, n, acc[i][j]);
        }
    }
}

template <class P>
__global__ void simt_gemm_reduce_kernel(P p, const float *__restrict__ ws, int splits) {
    const long long MN = (long long)p.M * p.N;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < MN;
         i += (long long)gridDim.x * blockDim.x) {
        float s = 0.0f;
        for (int z = 0; z < splits; ++z) s += ws[(size_t)z * MN + i];
        p.store((int)(i / p.N), (int)(i % p.N), s);
    }
}

// Workspace for split-K partials (library-owned, grown on demand).
float *gemm_workspace(size_t floats);

// One tile shape: the split count, the split-K workspace and the launches.
template <class P, int BM, int BN, int TM, int TN>
int launch_simt_gemm(const P &p, int splits, const char *what) {
    const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
    if (P::kExactOrder) splits = 1;  // the reference order is one ascending pass over k
    if (splits <= 0) {
        splits = 1;
        const int want = 2 * sm_count();
        while (tiles * splits < want && p.K / (splits * 2) >= 256) splits *= 2;
    }
    int kps = kGBK;
    if (p.K > 0) {
        kps = (p.K + splits - 1) / splits;
        kps = (kps + kGBK - 1) / kGBK * kGBK;
        splits = (p.K + kps - 1) / kps;
    } else {
        splits = 1;
    }
    if (splits < 1) splits = 1;
    float *ws = nullptr;
    if (splits > 1) {
        ws = gemm_workspace((size_t)splits * p.M * p.N);
        if (!ws) return fail(kBadHandle, "%s: split-K workspace allocation failed", what);
    }
    if ((p.N + BN - 1) / BN > 65535 || splits > 65535) return fail(kBadArg, "%s: N too large", what);
    dim3 grid((p.M + BM - 1) / BM, (p.N + BN - 1) / BN, splits);
    simt_gemm_kernel<P, BM, BN, TM, TN><<<grid, kGThreads, 0, stream()>>>(p, ws, kps);
    ZB_LAUNCH_CHECK(what);
    if (splits > 1) {
        simt_gemm_reduce_kernel<P><<<grid_for((long long)p.M * p.N, 256), 256, 0, stream()>>>(p, ws, splits);
        ZB_LAUNCH_CHECK(what);
    }
    return kOk;
}

// Launches C = A*B for problem p on the library stream.  splits = 0 picks a
// split count from the K length and the tile count.  The tile follows the
// problem's shape: narrow N (conv input gradients over 16 or 32 channels,
// convs with 16 or 32 filters) gets tall, narrow tiles; short M (weight
// gradients of 16 or 32 filters) short, wide ones; large problems 128 x 128.
template <class P>
int run_simt_gemm(const P &p, int splits, const char *what) {
    if (p.M <= 0 || p.N <= 0) return kOk;
    if (p.M <= 16 && p.N <= 16) return launch_simt_gemm<P, 16, 16, 1, 1>(p, splits, what);
    if (p.M <= 32 && p.N <= 32) return launch_simt_gemm<P, 32, 32, 2, 2>(p, splits, what);
    if (p.N <= 16) return launch_simt_gemm<P, 256, 16, 4, 4>(p, splits, what);
    if (p.N <= 32) return launch_simt_gemm<P, 256, 32, 8, 4>(p, splits, what);
    if (p.M <= 32) return launch_simt_gemm<P, 32, 64, 2, 4>(p, splits, what);
    if (p.N >= 128 && (long long)((p.M + 127) / 128) * ((p.N + 127) / 128) >= 2LL * sm_count())
        return launch_simt_gemm<P, 128, 128, 8, 8>(p, splits, what);
    return launch_simt_gemm<P, 64, 64, 4, 4>(p, splits, what);
}

}  // namespace zb
