// common.cuh -- shared helpers of libzilla_b200.so (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/zilla_b200.h"

namespace zb {

enum Status : int {
    kOk = 0,
    kBadHandle = -1,   // also: allocation failure, upload/download beyond capacity
    kBadArg = -2,
    kCudaError = -3,
};

// Records the status and message of the failing call (zilla_last_error).
int fail(int status, const char *fmt, ...);
// Checks cudaGetLastError() after a launch or a runtime call.
int check_cuda(const char *what);

// Stream all device work of the library goes to (per process).
cudaStream_t stream();
// Counts launches issued by the library (zilla_launch_count).
void count_launch(unsigned n = 1);

// Raw pointer of a registry handle, nullptr if invalid.  Records nothing.
float *ptr(int id);
// Capacity in floats of a registry handle (0 if invalid).
size_t capacity(int id);

// Programmatic dependent launch.  A kernel started by launch_pdl may begin
// while the previous kernel on the stream is still running: it calls
// griddep_wait() before its first global-memory access (read or write; only
// shared memory, mbarrier and TMEM set-up come before), and griddep_launch()
// at its start so that the next kernel's blocks can be scheduled, and run
// their own set-up, as soon as SM resources free up.  Both are no-ops in a
// kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Division by a divisor fixed at launch, as a multiply and a shift
// (Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, Theorem 4.2 with N = 31): for 1 <= d < 2^31,
// l = ceil(log2 d) and m = ceil(2^(31+l) / d), floor(n / d) equals
// (n * m) >> (31 + l) for every 0 <= n < 2^31, and m < 2^32.  The index
// arithmetic of the gather functors below stays in [0, 2^31).
struct FastDiv {
    unsigned d = 1, m = 0x80000000u;
    int sh = 31;
    FastDiv() = default;
    explicit FastDiv(int div) {
        d = div > 0 ? (unsigned)div : 1u;
        int l = 0;
        while ((1ull << l) < d) ++l;
        sh = 31 + l;
        m = (unsigned)(((1ull << sh) + d - 1) / d);
    }
    __host__ __device__ __forceinline__ int div(int n) const {
        return (int)(((unsigned long long)(unsigned)n * m) >> sh);
    }
};

// Grid size helper: enough blocks to cover n with `threads` each, capped to
// a multiple of the SM count x `per_sm` (grid-stride loops cover the rest).
int grid_for(long long n, int threads, int per_sm = 8);
int sm_count();

// Device-side error word (a cudaMalloc'd int): kernels that detect an
// impossible state (a bounded wait that ran out, an index out of range)
// record a code there instead of trapping; the host reads it after
// synchronising.  Kernels receive the pointer as an argument.
int *device_error_word();
int read_and_clear_device_error();

}  // namespace zb

#define ZB_LAUNCH_CHECK(what)                                   \
    do {                                                        \
        ::zb::count_launch();                                   \
        int _rc = ::zb::check_cuda(what);                       \
        if (_rc) return _rc;                                    \
    } while (0)
