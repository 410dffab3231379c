// One backsubstitution step (ReLU sign split + affine substitution), dispatched to the
// tensor-core kernel when the shape allows it and to the CUDA-core kernel otherwise.
#pragma once
#include "cf_common.cuh"

namespace cf {

// Scratch (bytes) a step over 2*Bc*R rows may need beyond its inputs and outputs.
size_t step_scratch_bytes(int64_t Bc, int64_t R);

cf_status run_step(int64_t B, int64_t R, int64_t K, int64_t N, const float* A, int64_t a_ss, int64_t a_bs,
                   int64_t a_rs, const float* c_in, int64_t c_ss, int64_t c_bs, const float* alpha, const float* lam,
                   const float* mu, const float* W, const float* bias, float* A_out, float* c_out, char* scratch,
                   cudaStream_t st);

}  // namespace cf
