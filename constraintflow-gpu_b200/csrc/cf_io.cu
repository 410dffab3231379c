// Input boundary kernels (input box, property matrix) and the profiling hooks.
#include <vector>

#include "cf_common.cuh"

namespace cf {

// ------------------------------------------------------------------ input box
// constraintflow/lib/spec.py:21-47: l = (clip(X - eps, 0, 1) - mean) / std, same for u
// with +eps; float32 IEEE operations in the same order as the torch expression.
struct Norm {
  float mean[4], std[4];
};

__global__ void k_input_box(int64_t B, int32_t C, int64_t HW, const float* __restrict__ X, float eps, Norm nm,
                            float* __restrict__ l0, float* __restrict__ u0) {
  int64_t total = B * C * HW;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int c = (int)((t / HW) % C);
    float x = X[t];
    float lo = __fsub_rn(x, eps), hi = __fadd_rn(x, eps);
    lo = fminf(fmaxf(lo, 0.0f), 1.0f);
    hi = fminf(fmaxf(hi, 0.0f), 1.0f);
    l0[t] = __fdiv_rn(__fsub_rn(lo, nm.mean[c]), nm.std[c]);
    u0[t] = __fdiv_rn(__fsub_rn(hi, nm.mean[c]), nm.std[c]);
  }
}

// constraintflow/lib/spec.py:61-72: row j of region b is e_label - e_k, k the j-th class != label.
__global__ void k_spec_matrix(int64_t B, int32_t nc, const int64_t* __restrict__ labels, float* __restrict__ W) {
  int64_t rows = nc - 1;
  int64_t total = B * rows * nc;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = t / (rows * nc), rem = t - b * rows * nc, j = rem / nc, col = rem - j * nc;
    int64_t y = labels[b];
    int64_t k = j < y ? j : j + 1;
    W[t] = (float)(col == y) - (float)(col == k);
  }
}

// ------------------------------------------------------------------ profiling
struct ProfRec {
  cudaEvent_t a, b;
  double flops, bytes;
  bool mem;
};
struct ProfState {
  bool on = false;
  int64_t launches = 0;
  std::vector<ProfRec> open;
  std::vector<cudaEvent_t> pool;
};
static thread_local ProfState g_prof;
struct ProfSpan {
  bool on = false;
  double flops = 0, bytes = 0;
};
static thread_local ProfSpan g_span;

static cudaEvent_t take_event() {
  if (!g_prof.pool.empty()) {
    cudaEvent_t e = g_prof.pool.back();
    g_prof.pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

void prof_count_launch() {
  if (g_prof.on) ++g_prof.launches;
}
bool prof_enabled() { return g_prof.on; }
static void prof_begin(cudaStream_t st, bool mem) {
  if (!g_prof.on || g_span.on) return;
  ProfRec r;
  r.a = take_event();
  r.b = take_event();
  r.flops = r.bytes = 0;
  r.mem = mem;
  cudaEventRecord(r.a, st);
  g_prof.open.push_back(r);
}
void prof_step_begin(cudaStream_t st) { prof_begin(st, false); }
void prof_mem_begin(cudaStream_t st) { prof_begin(st, true); }
void prof_mem_end(cudaStream_t st, double bytes) { prof_step_end(st, 0.0, bytes); }
void prof_step_end(cudaStream_t st, double flops, double bytes) {
  if (!g_prof.on || g_prof.open.empty()) return;
  if (g_span.on) {
    g_span.flops += flops;
    g_span.bytes += bytes;
    return;
  }
  ProfRec& r = g_prof.open.back();
  r.flops = flops;
  r.bytes = bytes;
  cudaEventRecord(r.b, st);
}

void prof_span_begin(cudaStream_t st) {
  if (!g_prof.on || g_span.on) return;
  prof_begin(st, false);
  g_span.on = true;
  g_span.flops = g_span.bytes = 0;
}
void prof_span_end(cudaStream_t st) {
  if (!g_span.on) return;
  g_span.on = false;
  prof_step_end(st, g_span.flops, g_span.bytes);
}

}  // namespace cf

using namespace cf;

extern "C" cf_status cf_input_box(int64_t B, int32_t C, int64_t HW, const float* X, float eps, const float* mean,
                                  const float* stdv, float* l0, float* u0, void* stream) {
  clear_error();
  CF_INJECT("input_box");
  CF_REQUIRE(B >= 0 && C >= 1 && C <= 4 && HW >= 0, CF_ERR_SHAPE, "input_box: bad sizes");
  CF_REQUIRE(mean && stdv, CF_ERR_NULL, "input_box: mean/std missing");
  if (B * C * HW == 0) return CF_OK;
  CF_REQUIRE(X && l0 && u0, CF_ERR_NULL, "input_box: NULL argument");
  Norm nm;
  for (int c = 0; c < 4; ++c) {
    nm.mean[c] = c < C ? mean[c] : 0.0f;
    nm.std[c] = c < C ? stdv[c] : 1.0f;
  }
  int64_t total = B * C * HW;
  int64_t blocks = ceil_div(total, 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  k_input_box<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(B, C, HW, X, eps, nm, l0, u0);
  return check_launch("k_input_box");
}

extern "C" cf_status cf_spec_matrix(int64_t B, int32_t nc, const int64_t* labels, float* W, void* stream) {
  clear_error();
  CF_INJECT("spec_matrix");
  CF_REQUIRE(B >= 0 && nc >= 2, CF_ERR_SHAPE, "spec_matrix: bad sizes");
  if (B == 0) return CF_OK;
  CF_REQUIRE(labels && W, CF_ERR_NULL, "spec_matrix: NULL argument");
  int64_t total = B * (nc - 1) * nc;
  int64_t blocks = ceil_div(total, 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  k_spec_matrix<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(B, nc, labels, W);
  return check_launch("k_spec_matrix");
}

extern "C" cf_status cf_profile_enable(int32_t on) {
  g_prof.on = on != 0;
  return CF_OK;
}

extern "C" cf_status cf_profile_collect(cf_profile_stats* out) {
  clear_error();
  CF_REQUIRE(out, CF_ERR_NULL, "profile_collect: NULL output");
  memset(out, 0, sizeof(*out));
  out->kernel_launches = g_prof.launches;
  cf_status status = CF_OK;
  for (ProfRec& r : g_prof.open) {
    float ms = 0.0f;
    cudaError_t e = cudaEventSynchronize(r.b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, r.a, r.b);
    if (e != cudaSuccess) {
      set_error("profile_collect: %s", cudaGetErrorString(e));
      status = CF_ERR_CUDA;
    }
    if (r.mem) {
      out->mem_launches += 1;
      out->mem_ms += ms;
      out->mem_bytes += r.bytes;
    } else {
      out->step_launches += 1;
      out->step_ms += ms;
      out->step_flops += r.flops;
      out->step_bytes += r.bytes;
    }
    g_prof.pool.push_back(r.a);
    g_prof.pool.push_back(r.b);
  }
  g_prof.open.clear();
  g_prof.launches = 0;
  return status;
}
