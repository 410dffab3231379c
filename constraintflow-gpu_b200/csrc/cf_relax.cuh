// The DeepPoly ReLU relaxation of one neuron, shared by the stand-alone relaxation kernel
// and the kernels that fuse it into the drain of the layer's own bounds (k_chain,
// k_concretize_bcast), so that every path stores bit-identical values.
#pragma once
#include "cf_common.cuh"

namespace cf {

// Where the relaxation of a ReLU layer goes, for neuron (b, i) of its input layer:
//   lo / uo      the ReLU layer's own bounds, at b*ld_out + i (optional: nullptr skips them)
//   alpha/lam/mu [B, n] contiguous: L' = alpha x, U' = lam x + mu
//   dl / du      decision replay (optional, at b*ld_dec + i): the bounds the three branch
//                decisions are taken from; the values still come from the neuron's l / u
//   strict       the lower slope is 1 where l + u > 0 (zid.cf, the custom-stop programs)
//                instead of l + u >= 0
struct ReluOut {
  float* lo;
  float* uo;
  int64_t ld_out;
  float* alpha;
  float* lam;
  float* mu;
  int64_t n;
  const float* dl;
  const float* du;
  int64_t ld_dec;
  int32_t strict;
};

// Generated deeppoly.Relu (deeppoly.cf:20-24,41):
//   l' = relu(l), u' = relu(u)
//   L' = 1[l+u>=0] * x
//   U' = x if l>=0; 0 if u<=0; else lam*x + mu, lam = u/(u-l), mu = -(u*l)/(u-l)
// float32 IEEE division, same operation order as the generated code.
__device__ __forceinline__ void relu_relax_store(const ReluOut& o, int64_t b, int64_t i, float lv, float uv) {
  const float ld = o.dl ? o.dl[b * o.ld_dec + i] : lv, ud = o.du ? o.du[b * o.ld_dec + i] : uv;
  const bool pos = ld >= 0.0f;
  const bool dead = (!pos) && (ud <= 0.0f);
  const float den = uv - lv;
  const float lam_u = __fdiv_rn(uv, den);
  const float mu_u = 0.0f - __fdiv_rn(__fmul_rn(uv, lv), den);
  if (o.lo) o.lo[b * o.ld_out + i] = pos ? lv : 0.0f;
  if (o.uo) o.uo[b * o.ld_out + i] = (ud >= 0.0f) ? uv : 0.0f;
  const float s = __fadd_rn(ld, ud);
  const int64_t t = b * o.n + i;
  o.alpha[t] = (o.strict ? s > 0.0f : s >= 0.0f) ? 1.0f : 0.0f;
  o.lam[t] = pos ? 1.0f : (dead ? 0.0f : lam_u);
  o.mu[t] = (pos || dead) ? 0.0f : mu_u;
}

}  // namespace cf
