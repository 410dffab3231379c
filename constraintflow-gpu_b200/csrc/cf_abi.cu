// C ABI entry points for the individual DeepPoly building blocks (the network driver
// cf_deeppoly_run lives in cf_engine.cu).  Each validates its arguments, honours the
// host-side fault-injection switch and launches on the caller's stream.
#include "cf_common.cuh"
#include "cf_kernels.cuh"
#include "cf_step.cuh"

using namespace cf;

extern "C" cf_status cf_relu_relax(int64_t B, int64_t n, const float* l, const float* u, int64_t ld_in,
                                   float* lo, float* uo, int64_t ld_out, float* alpha, float* lam, float* mu,
                                   int32_t relaxation, void* stream) {
  clear_error();
  CF_INJECT("relu_relax");
  CF_REQUIRE(B >= 0 && n >= 0 && ld_in >= n && (lo == nullptr || ld_out >= n), CF_ERR_SHAPE,
             "relu_relax: bad sizes B=%lld n=%lld", (long long)B, (long long)n);
  CF_REQUIRE(relaxation == CF_RELAX_DEEPPOLY, CF_ERR_UNSUPPORTED, "relu_relax: relaxation %d", relaxation);
  if (B * n == 0) return CF_OK;
  CF_REQUIRE(l && u && alpha && lam && mu, CF_ERR_NULL, "relu_relax: NULL argument");
  return launch_relu_relax(B, n, l, u, ld_in, lo, uo, ld_out, alpha, lam, mu, as_stream(stream));
}

extern "C" cf_status cf_backsub_step(int64_t B, int64_t R, int64_t K, int64_t N, const float* A, int64_t a_ss,
                                     int64_t a_bs, int64_t a_rs, const float* c_in, int64_t c_ss, int64_t c_bs,
                                     const float* alpha, const float* lam, const float* mu, const float* W,
                                     const float* bias, float* A_out, float* c_out, void* stream) {
  clear_error();
  CF_INJECT("backsub_step");
  CF_REQUIRE(B >= 0 && R >= 0 && K > 0 && N > 0 && a_rs >= K, CF_ERR_SHAPE,
             "backsub_step: bad sizes B=%lld R=%lld K=%lld N=%lld a_rs=%lld", (long long)B, (long long)R,
             (long long)K, (long long)N, (long long)a_rs);
  if (B * R == 0) return CF_OK;
  CF_REQUIRE(A && W && A_out && c_out, CF_ERR_NULL, "backsub_step: NULL argument");
  CF_REQUIRE((alpha == nullptr) == (lam == nullptr) && (alpha == nullptr) == (mu == nullptr), CF_ERR_NULL,
             "backsub_step: alpha/lam/mu must be all given or all NULL");
  if (step_scratch_bytes(B, R) != 0) {
    set_error("backsub_step: this build needs scratch; use cf_deeppoly_run");
    return CF_ERR_UNSUPPORTED;
  }
  return run_step(B, R, K, N, A, a_ss, a_bs, a_rs, c_in, c_ss, c_bs, alpha, lam, mu, W, bias, A_out, c_out, nullptr,
                  as_stream(stream));
}

extern "C" cf_status cf_concretize(int64_t B, int64_t R, int64_t n0, const float* A, int64_t a_ss, int64_t a_bs,
                                   int64_t a_rs, const float* c, int64_t c_ss, int64_t c_bs, const float* l0,
                                   const float* u0, float* out_l, float* out_u, int64_t ld_out, void* stream) {
  clear_error();
  CF_INJECT("concretize");
  CF_REQUIRE(B >= 0 && R >= 0 && n0 > 0 && a_rs >= n0 && ld_out >= R, CF_ERR_SHAPE, "concretize: bad sizes");
  if (B * R == 0) return CF_OK;
  CF_REQUIRE(A && l0 && u0 && out_l && out_u, CF_ERR_NULL, "concretize: NULL argument");
  return launch_concretize(B, R, n0, A, a_ss, a_bs, a_rs, c, c_ss, c_bs, l0, u0, out_l, out_u, ld_out,
                           as_stream(stream));
}
