// legacy_ops.cu -- the reference's elementwise, loss, bias-grad, optimizer,
// attention and host-pointer entry points (native/cuda/device_ops.cu,
// native/cuda/training_ops.cu, native/cuda/attention.cu,
// native/cuda/elementwise.cu, native/cuda/audio.cu), re-designed for sm_100a:
// vectorised grid-stride elementwise kernels sized to the SM count,
// warp-per-row softmax/cross-entropy, deterministic (atomic-free) reductions
// and launch-error reporting.
#include <math.h>
#include <string.h>

#include "common.cuh"

using namespace zb;

namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- elementwise
enum class Bin { Add, Sub, Mul, Div };

template <Bin op>
__device__ __forceinline__ float bin(float a, float b) {
    if constexpr (op == Bin::Add) return a + b;
    if constexpr (op == Bin::Sub) return a - b;
    if constexpr (op == Bin::Mul) return a * b;
    return a / b;
}

template <Bin op>
__global__ void binary_kernel(const float *__restrict__ a, const float *__restrict__ b,
                              float *__restrict__ c, long long n) {
    const long long n4 = n >> 2;
    const long long stride = (long long)gridDim.x * blockDim.x;
    const bool vec = ((((uintptr_t)a) | ((uintptr_t)b) | ((uintptr_t)c)) & 15) == 0;
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        for (long long j = i; j < n4; j += stride) {
            float4 x = reinterpret_cast<const float4 *>(a)[j];
            float4 y = reinterpret_cast<const float4 *>(b)[j];
            reinterpret_cast<float4 *>(c)[j] =
                make_float4(bin<op>(x.x, y.x), bin<op>(x.y, y.y), bin<op>(x.z, y.z), bin<op>(x.w, y.w));
        }
        for (long long j = (n4 << 2) + i; j < n; j += stride) c[j] = bin<op>(a[j], b[j]);
    } else {
        for (long long j = i; j < n; j += stride) c[j] = bin<op>(a[j], b[j]);
    }
}

__global__ void relu_kernel(const float *__restrict__ x, float *__restrict__ y, long long n) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

// native/cuda/training_ops.cu:62-68: y = x > 0 ? x : 0, mask 1.0 / 0.0.
__global__ void relu_fwd_kernel(const float *__restrict__ x, float *__restrict__ y,
                                float *__restrict__ m, long long n) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = x[i];
        const bool pos = v > 0.0f;
        y[i] = pos ? v : 0.0f;
        m[i] = pos ? 1.0f : 0.0f;
    }
}

__global__ void add_bias_kernel(float *__restrict__ x, const float *__restrict__ b, long long n,
                                int C) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        x[i] += b[i % C];
}

__global__ void sgd_kernel(float *__restrict__ w, const float *__restrict__ g, float lr,
                           long long n) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        w[i] = __fsub_rn(w[i], __fmul_rn(lr, g[i]));   // no FMA: the CPU rounds the product
}

__global__ void scale_kernel(float *__restrict__ x, float s, long long n) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        x[i] *= s;
}

// ---------------------------------------------------------------- softmax-CE
// One warp per row: max, exp, sum by shuffles, then (p - onehot)/B.  The row's
// -log p_t goes to a per-row slot in double; a second kernel sums the slots in
// row order (deterministic, unlike the reference's float atomicAdd at
// native/cuda/training_ops.cu:141) and adds the total to *loss as the CPU
// reference does (native/cpu/training_ops.c:171,204).
// floor > 0: each row's loss is -log(max(p_target, floor)) (CrossEntropy.php's clamp);
// floor = 0 is softmax_ce_dev's plain -log(p_target).
__global__ void softmax_ce_rows_kernel(const float *__restrict__ z, const float *__restrict__ tgt,
                                       float *__restrict__ dz, double *__restrict__ row_loss,
                                       int B, int C, float floor = 0.0f) {
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    const float inv = 1.0f / (float)B;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < B; r += gridDim.x * warps) {
        const float *row = z + (size_t)r * C;
        float mx = -INFINITY;
        for (int c = lane; c < C; c += 32) mx = fmaxf(mx, row[c]);
#pragma unroll
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float s = 0.0f;
        for (int c = lane; c < C; c += 32) s += expf(row[c] - mx);
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const int t = (int)tgt[r];
        for (int c = lane; c < C; c += 32) {
            const float p = expf(row[c] - mx) / s;
            dz[(size_t)r * C + c] = (p - (c == t ? 1.0f : 0.0f)) * inv;
        }
        if (lane == 0) {
            const float pt = (t >= 0 && t < C) ? expf(row[t] - mx) / s : 0.0f;
            row_loss[r] = -(double)logf(floor > 0.0f ? fmaxf(pt, floor) : pt);
        }
    }
}

__global__ void sum_rows_into_loss_kernel(const double *__restrict__ row_loss, int B,
                                          float *__restrict__ loss) {
    __shared__ double part[kThreads];
    double acc = 0.0;
    // contiguous chunk per thread, chunks combined in thread order
    const int per = (B + blockDim.x - 1) / blockDim.x;
    const int b0 = threadIdx.x * per, b1 = min(B, b0 + per);
    int r = b0;
    for (; r + 8 <= b1; r += 8) {   // eight loads in flight, added in row order
        double v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = row_loss[r + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) acc += v[u];
    }
    for (; r < b1; ++r) acc += row_loss[r];
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int i = 0; i < (int)blockDim.x; ++i) tot += part[i];
        *loss += (float)tot;
    }
}

// ---------------------------------------------------------------- bias grad
// db[c] = sum_i dY[i, c]: 32 columns x 8 row-lanes per block, fixed-order
// combine across row lanes.
__global__ void bias_grad_kernel(const float *__restrict__ dy, float *__restrict__ db, int B,
                                 int C) {
    __shared__ float part[8][33];
    const int c = blockIdx.x * 32 + threadIdx.x;
    float acc = 0.0f;
    if (c < C)
        for (int i = threadIdx.y; i < B; i += 8) acc += dy[(size_t)i * C + c];
    part[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && c < C) {
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) s += part[k][threadIdx.x];
        db[c] = s;
    }
}

// ---------------------------------------------------------------- row softmax
// native/cuda/attention.cu:31-81 / 191-244 semantics: max from -1e30, expf,
// sum, multiply by 1/sum; `causal` first sets x[row, j > row] = maskValue.
template <bool causal>
__global__ void softmax_rows_kernel(const float *__restrict__ x, float *__restrict__ y, int N,
                                    int M, float mask_value) {
    __shared__ float red[32];
    const int row = blockIdx.x;
    if (row >= N) return;
    const float *a = x + (size_t)row * M;
    float *o = y + (size_t)row * M;
    auto val = [&](int j) { return (causal && j > row) ? mask_value : a[j]; };
    float mx = -1e30f;
    for (int j = threadIdx.x; j < M; j += blockDim.x) mx = fmaxf(mx, val(j));
#pragma unroll
    for (int k = 16; k; k >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, k));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -1e30f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float s = 0.0f;
    for (int j = threadIdx.x; j < M; j += blockDim.x) {
        const float e = expf(val(j) - mx);
        o[j] = e;
        s += e;
    }
#pragma unroll
    for (int k = 16; k; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    s = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
    const float inv = 1.0f / s;
    for (int j = threadIdx.x; j < M; j += blockDim.x) o[j] *= inv;
}

// native/cuda/attention.cu:98-130: dS = P * (dP - sum_k dP*P).
__global__ void softmax_rows_bwd_kernel(const float *__restrict__ P, const float *__restrict__ dP,
                                        float *__restrict__ dS, int N, int M) {
    __shared__ float red[32];
    const int row = blockIdx.x;
    if (row >= N) return;
    const float *p = P + (size_t)row * M, *dp = dP + (size_t)row * M;
    float d = 0.0f;
    for (int j = threadIdx.x; j < M; j += blockDim.x) d += dp[j] * p[j];
#pragma unroll
    for (int k = 16; k; k >>= 1) d += __shfl_xor_sync(0xffffffffu, d, k);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = d;
    __syncthreads();
    d = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) d += red[w];
    for (int j = threadIdx.x; j < M; j += blockDim.x) dS[(size_t)row * M + j] = p[j] * (dp[j] - d);
}

// native/cuda/attention.cu:146-157: additive mask on col > row.
__global__ void causal_mask_kernel(float *__restrict__ x, int N, int M, float mask_value) {
    const int row = blockIdx.y;
    for (int col = blockIdx.x * blockDim.x + threadIdx.x; col < M; col += gridDim.x * blockDim.x)
        if (col > row) x[(size_t)row * M + col] += mask_value;
}

// ---------------------------------------------------------------- audio (off path)
__global__ void hann_kernel(float *w, int N) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N) return;
    if (N <= 1) { w[i] = 1.0f; return; }
    w[i] = 0.5f - 0.5f * cospif(2.0f * (float)i / (float)(N - 1));
}

// Direct DFT magnitude of Hann-windowed frames; one block per frame, bins
// strided over threads; phase from exact integer (k*n mod N) arithmetic.
__global__ void stft_dft_kernel(const float *__restrict__ in, int len, int nfft, int hop,
                                int nbins, int nframes, float *__restrict__ mag) {
    extern __shared__ float frame[];
    const int f = blockIdx.x;
    for (int i = threadIdx.x; i < nfft; i += blockDim.x) {
        const int idx = f * hop + i;
        const float w = 0.5f - 0.5f * cospif(2.0f * (float)i / (float)(nfft - 1));
        frame[i] = (idx < len ? in[idx] : 0.0f) * w;
    }
    __syncthreads();
    for (int k = threadIdx.x; k < nbins; k += blockDim.x) {
        float re = 0.0f, im = 0.0f;
        for (int n = 0; n < nfft; ++n) {
            const int ph = (int)(((long long)k * n) % nfft);
            float s, c;
            sincospif(2.0f * (float)ph / (float)nfft, &s, &c);
            re += frame[n] * c;
            im -= frame[n] * s;
        }
        mag[(size_t)k * nframes + f] = sqrtf(re * re + im * im);
    }
}

// ---------------------------------------------------------------- helpers
double *g_row_loss = nullptr;
size_t g_row_loss_cap = 0;

double *row_loss_scratch(size_t n) {
    if (n > g_row_loss_cap) {
        if (g_row_loss) {
            cudaStreamSynchronize(stream());
            cudaFree(g_row_loss);
        }
        g_row_loss = nullptr;
        g_row_loss_cap = 0;
        if (cudaMalloc((void **)&g_row_loss, n * sizeof(double)) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_row_loss_cap = n;
    }
    return g_row_loss;
}

template <Bin op>
int binary_dev(int a_id, int b_id, int c_id, int n, const char *name) {
    float *a = ptr(a_id), *b = ptr(b_id), *c = ptr(c_id);
    if (!a || !b || !c) return fail(kBadHandle, "%s: invalid handle", name);
    if (n < 0) return fail(kBadArg, "%s: negative size", name);
    if (n == 0) return kOk;
    binary_kernel<op><<<grid_for(n / 4 + 1, kThreads), kThreads, 0, stream()>>>(a, b, c, n);
    ZB_LAUNCH_CHECK(name);
    return kOk;
}

// Host-pointer helpers: staging buffers grown on demand, one synchronous round trip.
float *g_stage[3] = {nullptr, nullptr, nullptr};
size_t g_stage_cap = 0;

bool stage(size_t bytes) {
    if (bytes <= g_stage_cap) return true;
    for (auto &p : g_stage) {
        if (p) cudaFree(p);
        p = nullptr;
    }
    g_stage_cap = 0;
    for (auto &p : g_stage)
        if (cudaMalloc((void **)&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
    g_stage_cap = bytes;
    return true;
}

template <Bin op>
void binary_host(const float *A, const float *B, float *Cc, int N, const char *name) {
    if (N <= 0) return;
    const size_t bytes = (size_t)N * sizeof(float);
    if (!stage(bytes)) { fail(kBadHandle, "%s: staging allocation failed", name); return; }
    cudaMemcpyAsync(g_stage[0], A, bytes, cudaMemcpyHostToDevice, stream());
    cudaMemcpyAsync(g_stage[1], B, bytes, cudaMemcpyHostToDevice, stream());
    binary_kernel<op><<<grid_for(N / 4 + 1, kThreads), kThreads, 0, stream()>>>(g_stage[0], g_stage[1], g_stage[2], N);
    count_launch();
    cudaMemcpyAsync(Cc, g_stage[2], bytes, cudaMemcpyDeviceToHost, stream());
    if (cudaStreamSynchronize(stream()) != cudaSuccess) check_cuda(name);
}

}  // namespace

namespace zb {

// Softmax cross-entropy on [B, C] logits: dz = (p - onehot)/B; the loss sum
// (double per row, summed in row order) is added to *loss (zeroed first when
// zero_first).  row_loss must hold B doubles.
int launch_softmax_ce(const float *z, const float *y, float *dz, double *row_loss, float *loss,
                      int B, int C, bool zero_first) {
    if (B <= 0) return kOk;
    if (zero_first) cudaMemsetAsync(loss, 0, sizeof(float), stream());
    softmax_ce_rows_kernel<<<grid_for((long long)B * 32, kThreads), kThreads, 0, stream()>>>(
        z, y, dz, row_loss, B, C);
    ZB_LAUNCH_CHECK("softmax_ce");
    sum_rows_into_loss_kernel<<<1, kThreads, 0, stream()>>>(row_loss, B, loss);
    ZB_LAUNCH_CHECK("softmax_ce(sum)");
    return kOk;
}

int launch_bias_grad(const float *dy, float *db, int B, int C) {
    bias_grad_kernel<<<(C + 31) / 32, dim3(32, 8), 0, stream()>>>(dy, db, B, C);
    ZB_LAUNCH_CHECK("bias_grad");
    return kOk;
}

}  // namespace zb

// ---------------------------------------------------------------- allocation-free softmax-CE
// softmax_ce_dev needs B doubles of scratch for its per-row losses and takes them from a
// buffer the library allocates with cudaMalloc on first use.  Some callers cannot let a
// library allocate device memory: code running under a caller-owned memory pool or budget,
// or a caller that only hands over device pointers it already owns.  softmax_ce_noalloc
// serves them: the per-row scratch is this fixed file-scope device array instead, reserved
// when the library is loaded, so a call allocates nothing.  Every GPU that loads the
// library holds the array (512 KB) until the process exits.  The first call on a device
// does the set-up (cudaGetSymbolAddress with that device current); callers make that
// first call before any stream capture.
namespace {

constexpr int kNoAllocMaxRows = 65536;                                 // rows per call
static __device__ __align__(256) double g_noalloc_row_loss[kNoAllocMaxRows];

constexpr int kMaxDevices = 64;
double *g_noalloc_ptr[kMaxDevices] = {};   // device address of the array, per device

}  // namespace

extern "C" int softmax_ce_noalloc(const float *logits, const float *targets, float *dlogits,
                                  float *loss, int B, int C, void *stream_handle) {
    if (!logits || !targets || !dlogits || !loss)
        return fail(kBadHandle, "softmax_ce_noalloc: null device pointer");
    if (B < 0 || C <= 0) return fail(kBadArg, "softmax_ce_noalloc: bad sizes B=%d C=%d", B, C);
    if (B > kNoAllocMaxRows)
        return fail(kBadArg, "softmax_ce_noalloc: B=%d exceeds the %d rows of its static scratch",
                    B, kNoAllocMaxRows);
    if (B == 0) return kOk;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_cuda("softmax_ce_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        return fail(kBadArg, "softmax_ce_noalloc: device %d beyond the %d devices it keeps set-up for", dev,
                    kMaxDevices);
    if (!g_noalloc_ptr[dev]) {   // set-up, once per device, with that device current
        double *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress((void **)&p, g_noalloc_row_loss);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return fail(kCudaError, "softmax_ce_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        }
        g_noalloc_ptr[dev] = p;
    }
    // NULL: the library's own stream, so the call is ordered after the *_dev ops that produced
    // the logits and before the ones that consume dlogits
    cudaStream_t s = stream_handle ? (cudaStream_t)stream_handle : stream();
    // every row slot read by the sum is written first by the row kernel: nothing to clear
    softmax_ce_rows_kernel<<<grid_for((long long)B * 32, kThreads), kThreads, 0, s>>>(
        logits, targets, dlogits, g_noalloc_ptr[dev], B, C);
    ZB_LAUNCH_CHECK("softmax_ce_noalloc");
    sum_rows_into_loss_kernel<<<1, kThreads, 0, s>>>(g_noalloc_ptr[dev], B, loss);
    ZB_LAUNCH_CHECK("softmax_ce_noalloc(sum)");
    return kOk;
}

extern "C" {

// ---- device_ops.cu:81-149 ----
int add_dev(int a, int b, int c, int n) { return binary_dev<Bin::Add>(a, b, c, n, "add_dev"); }
int sub_dev(int a, int b, int c, int n) { return binary_dev<Bin::Sub>(a, b, c, n, "sub_dev"); }
int mul_dev(int a, int b, int c, int n) { return binary_dev<Bin::Mul>(a, b, c, n, "mul_dev"); }
int div_dev(int a, int b, int c, int n) { return binary_dev<Bin::Div>(a, b, c, n, "div_dev"); }

int relu_dev(int x_id, int y_id, int n) {
    float *x = ptr(x_id), *y = ptr(y_id);
    if (!x || !y) return fail(kBadHandle, "relu_dev: invalid handle");
    if (n <= 0) return n < 0 ? fail(kBadArg, "relu_dev: negative size") : kOk;
    relu_kernel<<<grid_for(n, kThreads), kThreads, 0, stream()>>>(x, y, n);
    ZB_LAUNCH_CHECK("relu_dev");
    return kOk;
}

// ---- training_ops.cu ----
int add_bias_dev(int x_id, int b_id, int B, int C) {
    float *x = ptr(x_id), *b = ptr(b_id);
    if (!x || !b) return fail(kBadHandle, "add_bias_dev: invalid handle");
    if (B < 0 || C <= 0) return fail(kBadArg, "add_bias_dev: bad sizes");
    const long long n = (long long)B * C;
    if (!n) return kOk;
    add_bias_kernel<<<grid_for(n, kThreads), kThreads, 0, stream()>>>(x, b, n, C);
    ZB_LAUNCH_CHECK("add_bias_dev");
    return kOk;
}

int relu_fwd_dev(int x_id, int y_id, int mask_id, int n) {
    float *x = ptr(x_id), *y = ptr(y_id), *m = ptr(mask_id);
    if (!x || !y || !m) return fail(kBadHandle, "relu_fwd_dev: invalid handle");
    if (n <= 0) return n < 0 ? fail(kBadArg, "relu_fwd_dev: negative size") : kOk;
    relu_fwd_kernel<<<grid_for(n, kThreads), kThreads, 0, stream()>>>(x, y, m, n);
    ZB_LAUNCH_CHECK("relu_fwd_dev");
    return kOk;
}

int relu_bwd_dev(int dy_id, int mask_id, int dx_id, int n) {
    return binary_dev<Bin::Mul>(dy_id, mask_id, dx_id, n, "relu_bwd_dev");
}

static int softmax_ce_rows(int logits_id, int targets_id, int dlogits_id, int loss_id, int B, int C, float floor,
                           const char *name) {
    float *z = ptr(logits_id), *t = ptr(targets_id), *dz = ptr(dlogits_id), *loss = ptr(loss_id);
    if (!z || !t || !dz || !loss) return fail(kBadHandle, "%s: invalid handle", name);
    if (B < 0 || C <= 0) return fail(kBadArg, "%s: bad sizes", name);
    if (B == 0) return kOk;
    double *rl = row_loss_scratch((size_t)B);
    if (!rl) return fail(kBadHandle, "%s: scratch allocation failed", name);
    softmax_ce_rows_kernel<<<grid_for((long long)B * 32, kThreads), kThreads, 0, stream()>>>(
        z, t, dz, rl, B, C, floor);
    ZB_LAUNCH_CHECK(name);
    sum_rows_into_loss_kernel<<<1, kThreads, 0, stream()>>>(rl, B, loss);
    ZB_LAUNCH_CHECK(name);
    return kOk;
}

int softmax_ce_dev(int logits_id, int targets_id, int dlogits_id, int loss_id, int B, int C) {
    return softmax_ce_rows(logits_id, targets_id, dlogits_id, loss_id, B, C, 0.0f, "softmax_ce_dev");
}

// The loss of CrossEntropy::forward (src/Loss/CrossEntropy.php:56-59): -log(max(p, 1e-12)) per
// row; the gradient is softmax_ce_dev's.
int softmax_ce_clamped_dev(int logits_id, int targets_id, int dlogits_id, int loss_id, int B, int C) {
    return softmax_ce_rows(logits_id, targets_id, dlogits_id, loss_id, B, C, 1e-12f, "softmax_ce_clamped_dev");
}

int bias_grad_dev(int dy_id, int db_id, int B, int C) {
    float *dy = ptr(dy_id), *db = ptr(db_id);
    if (!dy || !db) return fail(kBadHandle, "bias_grad_dev: invalid handle");
    if (B < 0 || C <= 0) return fail(kBadArg, "bias_grad_dev: bad sizes");
    bias_grad_kernel<<<(C + 31) / 32, dim3(32, 8), 0, stream()>>>(dy, db, B, C);
    ZB_LAUNCH_CHECK("bias_grad_dev");
    return kOk;
}

int sgd_update_dev(int w_id, int dw_id, float lr, int n) {
    float *w = ptr(w_id), *g = ptr(dw_id);
    if (!w || !g) return fail(kBadHandle, "sgd_update_dev: invalid handle");
    if (n <= 0) return n < 0 ? fail(kBadArg, "sgd_update_dev: negative size") : kOk;
    sgd_kernel<<<grid_for(n, kThreads), kThreads, 0, stream()>>>(w, g, lr, n);
    ZB_LAUNCH_CHECK("sgd_update_dev");
    return kOk;
}

int zero_dev(int id, int n) {
    float *x = ptr(id);
    if (!x) return fail(kBadHandle, "zero_dev: invalid handle");
    if (n < 0 || (size_t)n > capacity(id)) return fail(kBadArg, "zero_dev: bad size");
    if (!n) return kOk;
    cudaMemsetAsync(x, 0, (size_t)n * sizeof(float), stream());
    return check_cuda("zero_dev");
}

int copy_dev(int src_id, int dst_id, int n) {
    float *s = ptr(src_id), *d = ptr(dst_id);
    if (!s || !d) return fail(kBadHandle, "copy_dev: invalid handle");
    if (n < 0 || (size_t)n > capacity(src_id) || (size_t)n > capacity(dst_id))
        return fail(kBadHandle, "copy_dev: size beyond capacity");
    if (!n) return kOk;
    cudaMemcpyAsync(d, s, (size_t)n * sizeof(float), cudaMemcpyDeviceToDevice, stream());
    return check_cuda("copy_dev");
}

// ---- attention.cu ----
int softmax_rows_fwd_dev(int x_id, int y_id, int N, int M) {
    float *x = ptr(x_id), *y = ptr(y_id);
    if (!x || !y) return fail(kBadHandle, "softmax_rows_fwd_dev: invalid handle");
    if (N < 0 || M <= 0) return fail(kBadArg, "softmax_rows_fwd_dev: bad sizes");
    if (!N) return kOk;
    softmax_rows_kernel<false><<<N, M >= 256 ? 256 : 128, 0, stream()>>>(x, y, N, M, 0.0f);
    ZB_LAUNCH_CHECK("softmax_rows_fwd_dev");
    return kOk;
}

int softmax_rows_bwd_dev(int P_id, int dP_id, int dS_id, int N, int M) {
    float *P = ptr(P_id), *dP = ptr(dP_id), *dS = ptr(dS_id);
    if (!P || !dP || !dS) return fail(kBadHandle, "softmax_rows_bwd_dev: invalid handle");
    if (N < 0 || M <= 0) return fail(kBadArg, "softmax_rows_bwd_dev: bad sizes");
    if (!N) return kOk;
    softmax_rows_bwd_kernel<<<N, M >= 256 ? 256 : 128, 0, stream()>>>(P, dP, dS, N, M);
    ZB_LAUNCH_CHECK("softmax_rows_bwd_dev");
    return kOk;
}

int causal_mask_dev(int x_id, int N, int M, float mask_value) {
    float *x = ptr(x_id);
    if (!x) return fail(kBadHandle, "causal_mask_dev: invalid handle");
    if (N < 0 || M <= 0) return fail(kBadArg, "causal_mask_dev: bad sizes");
    if (!N) return kOk;
    causal_mask_kernel<<<dim3((M + kThreads - 1) / kThreads, N), kThreads, 0, stream()>>>(x, N, M, mask_value);
    ZB_LAUNCH_CHECK("causal_mask_dev");
    return kOk;
}

int scale_dev(int x_id, float s, int n) {
    float *x = ptr(x_id);
    if (!x) return fail(kBadHandle, "scale_dev: invalid handle");
    if (n <= 0) return n < 0 ? fail(kBadArg, "scale_dev: negative size") : kOk;
    scale_kernel<<<grid_for(n, kThreads), kThreads, 0, stream()>>>(x, s, n);
    ZB_LAUNCH_CHECK("scale_dev");
    return kOk;
}

int causal_softmax_dev(int x_id, int N, int M, float mask_value) {
    float *x = ptr(x_id);
    if (!x) return fail(kBadHandle, "causal_softmax_dev: invalid handle");
    if (N < 0 || M <= 0) return fail(kBadArg, "causal_softmax_dev: bad sizes");
    if (!N) return kOk;
    softmax_rows_kernel<true><<<N, M >= 256 ? 256 : 128, 0, stream()>>>(x, x, N, M, mask_value);
    ZB_LAUNCH_CHECK("causal_softmax_dev");
    return kOk;
}

// ---- host-pointer elementwise (elementwise.cu:71-148) ----
void relu_f32_cuda(const float *X, float *Y, int N) {
    if (N <= 0) return;
    const size_t bytes = (size_t)N * sizeof(float);
    if (!stage(bytes)) { fail(kBadHandle, "relu_f32_cuda: staging allocation failed"); return; }
    cudaMemcpyAsync(g_stage[0], X, bytes, cudaMemcpyHostToDevice, stream());
    relu_kernel<<<grid_for(N, kThreads), kThreads, 0, stream()>>>(g_stage[0], g_stage[1], N);
    count_launch();
    cudaMemcpyAsync(Y, g_stage[1], bytes, cudaMemcpyDeviceToHost, stream());
    if (cudaStreamSynchronize(stream()) != cudaSuccess) check_cuda("relu_f32_cuda");
}
void add_f32_cuda(const float *A, const float *B, float *Cc, int N) { binary_host<Bin::Add>(A, B, Cc, N, "add_f32_cuda"); }
void sub_f32_cuda(const float *A, const float *B, float *Cc, int N) { binary_host<Bin::Sub>(A, B, Cc, N, "sub_f32_cuda"); }
void mul_f32_cuda(const float *A, const float *B, float *Cc, int N) { binary_host<Bin::Mul>(A, B, Cc, N, "mul_f32_cuda"); }
void div_f32_cuda(const float *A, const float *B, float *Cc, int N) { binary_host<Bin::Div>(A, B, Cc, N, "div_f32_cuda"); }

// ---- audio.cu (preprocessing; kept so the reference's cdef block resolves) ----
void hann_window_cuda(float *w_host, int N) {
    if (N <= 0) return;
    if (!stage((size_t)N * sizeof(float))) return;
    hann_kernel<<<(N + kThreads - 1) / kThreads, kThreads, 0, stream()>>>(g_stage[0], N);
    count_launch();
    cudaMemcpyAsync(w_host, g_stage[0], (size_t)N * sizeof(float), cudaMemcpyDeviceToHost, stream());
    cudaStreamSynchronize(stream());
}

void stft_magnitude_cuda(const float *input, int inputLen, const float *window, int fftSize,
                         int hopSize, float *output, int *outNBins, int *outNFrames) {
    (void)window;  // the reference also ignores the host window (audio.cu:127)
    *outNBins = 0;
    *outNFrames = 0;
    if (fftSize < 2 || (fftSize & (fftSize - 1)) != 0 || fftSize > 16384 || inputLen <= 0 ||
        hopSize <= 0)
        return;
    const int nbins = fftSize / 2 + 1;
    int nframes = inputLen < fftSize ? 1 : 1 + (inputLen - fftSize) / hopSize;
    if (nframes <= 0) nframes = 1;
    const size_t in_bytes = (size_t)inputLen * sizeof(float);
    const size_t out_bytes = (size_t)nbins * nframes * sizeof(float);
    if (!stage(in_bytes > out_bytes ? in_bytes : out_bytes)) return;
    cudaMemcpyAsync(g_stage[0], input, in_bytes, cudaMemcpyHostToDevice, stream());
    stft_dft_kernel<<<nframes, 256, fftSize * sizeof(float), stream()>>>(
        g_stage[0], inputLen, fftSize, hopSize, nbins, nframes, g_stage[1]);
    count_launch();
    cudaMemcpyAsync(output, g_stage[1], out_bytes, cudaMemcpyDeviceToHost, stream());
    if (cudaStreamSynchronize(stream()) != cudaSuccess) { check_cuda("stft_magnitude_cuda"); return; }
    *outNBins = nbins;
    *outNFrames = nframes;
}

}  // extern "C"
