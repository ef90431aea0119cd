// registry.cu -- persistent device buffers addressed by int handles, the
// memory model of ZillaPHP's CUDA backend (native/cuda/buffer_registry.cu:
// 20-128): slots 1..8191, lowest free slot reused, 4-byte elements, free
// idempotent, upload/download bounded by capacity.  Differences: all device
// work runs on one library stream (upload/download synchronise with it), and
// allocations are rounded up to 256 bytes so every buffer is TMA/vector
// aligned.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace zb {

namespace {
constexpr int kSlots = 8192;
struct Slot {
    float *p;
    size_t n;
    int used;
};
Slot g_slots[kSlots];
cudaStream_t g_own_stream = nullptr;
cudaStream_t g_user_stream = nullptr;
bool g_user_stream_set = false;
unsigned long long g_launches = 0;
int g_last_status = 0;
char g_last_error[512] = "";
int g_sms = 0;
}  // namespace

namespace {
int *g_err_word = nullptr;
}

int *device_error_word() {
    if (!g_err_word) {
        if (cudaMalloc((void **)&g_err_word, sizeof(int)) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        cudaMemsetAsync(g_err_word, 0, sizeof(int), stream());
    }
    return g_err_word;
}

int fail(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    g_last_status = status;
    return status;
}

int check_cuda(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(kCudaError, "%s: %s", what, cudaGetErrorString(e));
    return kOk;
}

cudaStream_t stream() {
    if (g_user_stream_set) return g_user_stream;
    if (!g_own_stream) cudaStreamCreateWithFlags(&g_own_stream, cudaStreamNonBlocking);
    return g_own_stream;
}

void count_launch(unsigned n) { g_launches += n; }

float *ptr(int id) {
    if (id <= 0 || id >= kSlots || !g_slots[id].used) return nullptr;
    return g_slots[id].p;
}

size_t capacity(int id) {
    if (id <= 0 || id >= kSlots || !g_slots[id].used) return 0;
    return g_slots[id].n;
}

int sm_count() {
    if (!g_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_sms <= 0) g_sms = 148;
    }
    return g_sms;
}

int grid_for(long long n, int threads, int per_sm) {
    long long blocks = (n + threads - 1) / threads;
    long long cap = (long long)sm_count() * per_sm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

int read_and_clear_device_error() {
    int *w = device_error_word();
    if (!w) return 0;
    int v = 0;
    cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, stream());
    cudaMemsetAsync(w, 0, sizeof(int), stream());
    cudaStreamSynchronize(stream());
    return v;
}

}  // namespace zb

using namespace zb;

extern "C" {

int zilla_buffer_alloc(unsigned long n_floats) {
    if (n_floats == 0) return fail(kBadHandle, "zilla_buffer_alloc: zero size");
    for (int i = 1; i < kSlots; ++i) {
        if (g_slots[i].used) continue;
        size_t bytes = ((size_t)n_floats * sizeof(float) + 255) & ~(size_t)255;
        float *p = nullptr;
        if (cudaMalloc((void **)&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return fail(kBadHandle, "zilla_buffer_alloc: cudaMalloc of %zu bytes failed", bytes);
        }
        g_slots[i] = {p, (size_t)n_floats, 1};
        return i;
    }
    return fail(kBadHandle, "zilla_buffer_alloc: no free slots");
}

void zilla_buffer_free(int id) {
    if (id <= 0 || id >= kSlots || !g_slots[id].used) return;
    cudaStreamSynchronize(stream());
    cudaFree(g_slots[id].p);
    g_slots[id] = {nullptr, 0, 0};
}

int zilla_buffer_upload(int id, const float *host, unsigned long n_floats) {
    float *p = ptr(id);
    if (!p) return fail(kBadHandle, "zilla_buffer_upload: invalid handle %d", id);
    if (n_floats > g_slots[id].n)
        return fail(kBadHandle, "zilla_buffer_upload: %lu floats exceed capacity %zu", n_floats,
                    g_slots[id].n);
    if (n_floats == 0) return kOk;
    cudaMemcpyAsync(p, host, n_floats * sizeof(float), cudaMemcpyHostToDevice, stream());
    cudaError_t e = cudaStreamSynchronize(stream());
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(kBadHandle, "zilla_buffer_upload: %s", cudaGetErrorString(e));
    }
    return kOk;
}

int zilla_buffer_download(int id, float *host, unsigned long n_floats) {
    float *p = ptr(id);
    if (!p) return fail(kBadHandle, "zilla_buffer_download: invalid handle %d", id);
    if (n_floats > g_slots[id].n)
        return fail(kBadHandle, "zilla_buffer_download: %lu floats exceed capacity %zu", n_floats,
                    g_slots[id].n);
    if (n_floats == 0) return kOk;
    cudaMemcpyAsync(host, p, n_floats * sizeof(float), cudaMemcpyDeviceToHost, stream());
    cudaError_t e = cudaStreamSynchronize(stream());
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(kBadHandle, "zilla_buffer_download: %s", cudaGetErrorString(e));
    }
    return kOk;
}

void zilla_sync(void) {
    cudaStreamSynchronize(stream());
    cudaDeviceSynchronize();
}

float *zilla_buffer_ptr(int id) { return ptr(id); }

const char *zilla_last_error(void) { return g_last_error; }
int zilla_last_status(void) { return g_last_status; }

int zilla_set_stream(void *s) {
    if (s) {
        g_user_stream = (cudaStream_t)s;
        g_user_stream_set = true;
    } else {
        g_user_stream_set = false;
    }
    return kOk;
}

unsigned long long zilla_launch_count(void) { return g_launches; }

int zilla_check_device(void) {
    cudaStreamSynchronize(stream());
    const int code = read_and_clear_device_error();
    if (code) return fail(kCudaError, "device error word 0x%x (bounded wait expired or index out of range)", code);
    return check_cuda("zilla_check_device");
}

}  // extern "C"
