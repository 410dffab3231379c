// cf_deeppoly_run_static: the DeepPoly driver with its scratch in a fixed device array.
//
// Some callers cannot allocate device memory at the point where they certify: code that
// runs inside another framework's memory pool or allocator lock, plugins loaded into a
// host that forbids cudaMalloc after start-up, or latency-critical services that must not
// hit the allocator on the request path.  For them this entry point uses a file-scope
// device array as the workspace instead of caller-provided memory.  The caller still
// passes inputs and outputs.
//
// Costs and rules:
//  * every GPU that loads libcfgpu holds CF_STATIC_SCRATCH_BYTES for the whole process;
//  * the first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that first call
//    before any CUDA stream capture;
//  * every call shares the array, which keeps the previous call's contents: the driver
//    zeroes what must start at zero (the device error word) and overwrites everything
//    else before reading it, but calls that overlap on the GPU (different streams,
//    different host threads) race on the array and must be serialised by the caller;
//  * a network whose per-region scratch does not fit is rejected with CF_ERR_WORKSPACE;
//  * no cudaMalloc / cudaFree or allocating library routine is called.
#include <mutex>

#include "cf_common.cuh"

namespace cf {

static __device__ __align__(256) unsigned char g_static_scratch[CF_STATIC_SCRATCH_BYTES];

static std::mutex g_static_mu;
static void* g_static_ptr[128] = {nullptr};

}  // namespace cf

using namespace cf;

extern "C" cf_status cf_deeppoly_run_static(const cf_network* net, int64_t B, const float* l0, const float* u0,
                                            const float* specW, float* state_l, float* state_u, double* lb,
                                            double* ub, void* stream) {
  clear_error();
  CF_INJECT("deeppoly_run_static");
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 128) {
    set_error("deeppoly_run_static: cudaGetDevice: %s", cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (g_static_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_static_scratch);
      if (e != cudaSuccess || p == nullptr) {
        set_error("deeppoly_run_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        return CF_ERR_CUDA;
      }
      g_static_ptr[dev] = p;
    }
    ptr = g_static_ptr[dev];
  }
  const size_t need = cf_deeppoly_workspace_bytes(net, 1);
  CF_REQUIRE(need > 0, CF_ERR_SHAPE, "deeppoly_run_static: invalid network");
  CF_REQUIRE(need <= (size_t)CF_STATIC_SCRATCH_BYTES, CF_ERR_WORKSPACE,
             "deeppoly_run_static: one region needs %zu bytes of scratch, more than the fixed %zu-byte "
             "array; use cf_deeppoly_run with a workspace",
             need, (size_t)CF_STATIC_SCRATCH_BYTES);
  return cf_deeppoly_run(net, B, l0, u0, specW, state_l, state_u, lb, ub, ptr, (size_t)CF_STATIC_SCRATCH_BYTES,
                         stream);
}

extern "C" cf_status cf_deeppoly_check_static(void* stream) {
  clear_error();
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 128) {
    set_error("deeppoly_check_static: cudaGetDevice: %s", cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    ptr = g_static_ptr[dev];
  }
  CF_REQUIRE(ptr != nullptr, CF_ERR_NULL, "deeppoly_check_static: no cf_deeppoly_run_static call on device %d", dev);
  return cf_deeppoly_check(ptr, stream);
}
