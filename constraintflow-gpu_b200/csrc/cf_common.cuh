// Shared helpers of libcfgpu: status plumbing, launch checks, host-side fault injection.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "cfgpu.h"

namespace cf {

// Device error word value recorded when a CROWN ReLU layer takes the all-crossing branch
// (bounded-wait timeouts record their small site numbers instead).
constexpr int kCrownCrossingSite = 900;

// Per-host-thread message of the last failing call (read through cf_last_error()).
void set_error(const char* fmt, ...);
void clear_error();

// Host-side fault injection: CF_FAULT=<site>[,<site>...] makes the host wrapper of that
// site return CF_ERR_INJECTED before any launch.  Used by the failure-path tests; no
// device code is involved.
bool fault_injected(const char* site);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Profiling hooks (cf_io.cu): a per-thread kernel-launch counter and CUDA-event pairs
// around backsubstitution steps, active only between cf_profile_enable(1) and (0).
void prof_count_launch();
bool prof_enabled();
void prof_step_begin(cudaStream_t st);
void prof_step_end(cudaStream_t st, double flops, double bytes);
// the same around a launch of a memory-bound kernel (relaxation, concretisation, conversions)
void prof_mem_begin(cudaStream_t st);
void prof_mem_end(cudaStream_t st, double bytes);
// One record spanning work that runs on several streams at once (per-launch records there
// would count overlapping time twice): between span_begin and span_end on the joining
// stream, step and memory records only add their flops and bytes to the span.
void prof_span_begin(cudaStream_t st);
void prof_span_end(cudaStream_t st);

inline cf_status check_launch(const char* what) {
  prof_count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  return CF_OK;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace cf

#define CF_REQUIRE(cond, code, ...)   \
  do {                                \
    if (!(cond)) {                    \
      cf::set_error(__VA_ARGS__);     \
      return (code);                  \
    }                                 \
  } while (0)

#define CF_TRY(expr)                   \
  do {                                 \
    cf_status _st = (expr);            \
    if (_st != CF_OK) return _st;      \
  } while (0)

#define CF_INJECT(site)                                                        \
  do {                                                                         \
    if (cf::fault_injected(site)) {                                            \
      cf::set_error("injected fault at %s", site);                             \
      return CF_ERR_INJECTED;                                                  \
    }                                                                          \
  } while (0)
