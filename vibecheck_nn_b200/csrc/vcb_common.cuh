// Shared helpers for libvcb: error reporting, launch bookkeeping.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "vcb.h"

namespace vcb {

// Thread-local last-error string; every entry point returns a VCB_* code.
void set_error(const std::string& msg);
int fail(int code, const char* fmt, ...);

// Maps a CUDA runtime error to VCB_ERR_CUDA / VCB_ERR_OOM with context.
int cuda_fail(cudaError_t e, const char* what);

// Launch check: returns VCB_OK or the mapped error of cudaGetLastError().
int check_launch(const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

// Raises a kernel's dynamic shared-memory limit once per (kernel, size).
int ensure_smem(const void* kernel, int bytes);

__host__ __device__ inline int pad4(int n) { return (n + 3) & ~3; }

// Smallest multiple of 4 that is >= n and whose quotient by 4 is odd: a row
// stride with this property makes 16-byte loads of consecutive rows land in
// distinct shared-memory bank groups.
inline int pad4odd(int n) {
  int p = pad4(n);
  if (((p >> 2) & 1) == 0) p += 4;
  return p;
}

}  // namespace vcb
