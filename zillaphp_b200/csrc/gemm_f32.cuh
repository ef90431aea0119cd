// gemm_f32.cuh -- fp32 CUDA-core implicit GEMM used by the exact-fp32 path
// (the reference's matmul_dev / conv2d_*_dev semantics within 1e-4).
//
// C[m, n] = sum_k A(m, k) * B(k, n), where A and B are gather functors, so
// the same tiled kernel serves plain row-major GEMMs and the three
// convolution contractions (forward, input gradient, weight gradient) on
// NCHW tensors without materialising im2col.  64x64x16 tiles, 256 threads,
// 4x4 outputs per thread, register-prefetched next tile, optional split-K
// whose partials are combined in split order (deterministic).
#pragma once

#include "common.cuh"

namespace zb {

constexpr int kGBM = 64, kGBN = 64, kGBK = 16, kGThreads = 256;

// Problem concept:
//   int M, N, K;
//   static constexpr bool kAMFast, kBNFast;   // coalescing direction of loads
//   __device__ float a(int m, int k) const;   // callers guarantee m<M, k<K
//   __device__ float b(int k, int n) const;
//   __device__ void store(int m, int n, float v) const;
//   __device__ float init(int m, int n) const;    // initial accumulator
//   static constexpr bool kExactOrder;            // acc = acc + a*b, separately rounded,
//                                                 // k ascending (the reference CPU order)
template <class P>
__global__ void __launch_bounds__(kGThreads) simt_gemm_kernel(P p, float *__restrict__ ws,
                                                              int k_per_split) {
    __shared__ float As[kGBK][kGBM + 4];
    __shared__ float Bs[kGBK][kGBN + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.x * kGBM, n0 = blockIdx.y * kGBN;   // M tiles on x (up to 2^31-1)
    const int kb = blockIdx.z * k_per_split;
    const int ke = min(p.K, kb + k_per_split);

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
            acc[i][j] = (!ws && m < p.M && n < p.N) ? p.init(m, n) : 0.0f;
        }

    float ra[4], rb[4];
    auto load = [&](int k0) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int e = tid + r * kGThreads;
            int mm, kk;
            if (P::kAMFast) { mm = e & 63; kk = e >> 6; } else { mm = e >> 4; kk = e & 15; }
            const int m = m0 + mm, k = k0 + kk;
            ra[r] = (m < p.M && k < ke) ? p.a(m, k) : 0.0f;
            int nn, kk2;
            if (P::kBNFast) { nn = e & 63; kk2 = e >> 6; } else { nn = e >> 4; kk2 = e & 15; }
            const int n = n0 + nn, k2 = k0 + kk2;
            rb[r] = (n < p.N && k2 < ke) ? p.b(k2, n) : 0.0f;
        }
    };
    auto stash = [&]() {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int e = tid + r * kGThreads;
            if (P::kAMFast) As[e >> 6][e & 63] = ra[r]; else As[e & 15][e >> 4] = ra[r];
            if (P::kBNFast) Bs[e >> 6][e & 63] = rb[r]; else Bs[e & 15][e >> 4] = rb[r];
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
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if constexpr (P::kExactOrder) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
                    else acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                }
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty + 16 * i;
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx + 16 * j;
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

// Launches C = A*B for problem p on the library stream.  splits = 0 picks a
// split count from the K length and the tile count.
template <class P>
int run_simt_gemm(const P &p, int splits, const char *what) {
    if (p.M <= 0 || p.N <= 0) return kOk;
    const int tiles = ((p.M + kGBM - 1) / kGBM) * ((p.N + kGBN - 1) / kGBN);
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
    if ((p.N + kGBN - 1) / kGBN > 65535 || splits > 65535) return fail(kBadArg, "%s: N too large", what);
    dim3 grid((p.M + kGBM - 1) / kGBM, (p.N + kGBN - 1) / kGBN, splits);
    simt_gemm_kernel<P><<<grid, kGThreads, 0, stream()>>>(p, ws, kps);
    ZB_LAUNCH_CHECK(what);
    if (splits > 1) {
        simt_gemm_reduce_kernel<P><<<grid_for((long long)p.M * p.N, 256), 256, 0, stream()>>>(p, ws, splits);
        ZB_LAUNCH_CHECK(what);
    }
    return kOk;
}

}  // namespace zb
