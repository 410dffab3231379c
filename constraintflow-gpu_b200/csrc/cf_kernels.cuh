// Internal launcher declarations shared between the kernel files and the C ABI.
#pragma once
#include "cf_common.cuh"
#include "cf_relax.cuh"

namespace cf {

// dl / du (optional, rows at b*ld_in like l / u): the bounds the three branch decisions are
// taken from (decision replay); the relaxation's values still come from l / u.
cf_status launch_relu_relax(int64_t B, int64_t n, const float* l, const float* u, int64_t ld_in, float* lo,
                            float* uo, int64_t ld_out, float* alpha, float* lam, float* mu, cudaStream_t st,
                            bool strict = false, const float* dl = nullptr, const float* du = nullptr);
// the ReluOut of a layer of n neurons (decision bounds, when given, at b*ld_dec + i)
ReluOut relu_out(int64_t n, float* lo, float* uo, int64_t ld_out, float* alpha, float* lam, float* mu, bool strict,
                 const float* dl, const float* du, int64_t ld_dec);

// CROWN ReLU (whole-layer branch): flags = 2 device ints of scratch, err = device error word.
cf_status launch_crown_relax(int64_t B, int64_t n, const float* l, const float* u, int64_t ld_in, float* lo,
                             float* uo, int64_t ld_out, float* alpha, float* lam, float* mu, int* flags, int* err,
                             cudaStream_t st);

// relu (optional): the ReLU above the bounded layer is relaxed from its new bounds, fused
// into the concretisation where one thread holds both bounds of a neuron, else in a launch
// of its own right after it
cf_status launch_concretize(int64_t B, int64_t R, int64_t n0, const float* A, int64_t a_ss, int64_t a_bs,
                            int64_t a_rs, const float* c, int64_t c_ss, int64_t c_bs, const float* l0,
                            const float* u0, float* out_l, float* out_u, int64_t ld_out, cudaStream_t st,
                            const ReluOut* relu = nullptr);
// box (alpha l, lambda u + mu) [B, n] of a ReLU substituted last by a custom-stop traversal
cf_status launch_relu_box(int64_t B, int64_t n, const float* l, const float* u, int64_t ld_in, const float* alpha,
                          const float* lam, const float* mu, float* lo, float* hi, cudaStream_t st);
// the same with the box rows of region b at l0 + b*ld_box (e.g. a layer's state columns)
cf_status launch_concretize_box(int64_t B, int64_t R, int64_t n0, const float* A, int64_t a_ss, int64_t a_bs,
                                int64_t a_rs, const float* c, int64_t c_ss, int64_t c_bs, const float* l0,
                                const float* u0, int64_t ld_box, float* out_l, float* out_u, int64_t ld_out,
                                cudaStream_t st, const ReluOut* relu = nullptr);
// interval bound of a conv layer (ibp.Affine) from the previous layer's bounds (rows at
// l + b*ld_in) into the state columns (rows at sl + b*ld_state)
cf_status launch_ibp_conv_state(int64_t B, const cf_layer& L, const float* l, const float* u, int64_t ld_in,
                                float* sl, float* su, int64_t ld_state, cudaStream_t st);

cf_status launch_step_const(int64_t B, int64_t R, int64_t K, const float* A, int64_t a_ss, int64_t a_bs,
                            int64_t a_rs, const float* c_in, int64_t c_ss, int64_t c_bs, const float* alpha,
                            const float* lam, const float* mu, const float* bias, float* c_out, cudaStream_t st);

cf_status launch_step_gemm_simt(int64_t B, int64_t R, int64_t K, int64_t N, const float* A, int64_t a_ss,
                                int64_t a_bs, int64_t a_rs, const float* alpha, const float* lam, const float* W,
                                float* out, cudaStream_t st);

// both bounds of the property rows to float64 in one launch
cf_status launch_to_f64(int64_t B, int64_t n, const float* src_l, const float* src_u, int64_t ld_src, double* dst_l,
                        double* dst_u, cudaStream_t st);
cf_status launch_copy_rows(int64_t B, int64_t n, const float* src, int64_t ld_src, float* dst, int64_t ld_dst,
                           cudaStream_t st);

}  // namespace cf
