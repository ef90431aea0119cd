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
