// DeepPoly building blocks on CUDA cores: ReLU relaxation, input-box concretisation,
// the constant update of a backsubstitution step, and a SIMT float32 step GEMM.
//
// Row convention of every coefficient kernel: 2*B*R rows, row r = (s, b, i) with
// s = r / (B*R) the bound (0 lower, 1 upper), b the region and i the row inside the
// region.  Strides (a_ss, a_bs, a_rs) locate row (s,b,i) of a possibly broadcast input
// (zero strides), so the first step of every layer reads the shared weight matrix
// without materialising it per region.
#include <algorithm>

#include "cf_common.cuh"
#include "cf_kernels.cuh"

namespace cf {

// ------------------------------------------------------------------ ReLU relaxation
// The relaxation of a whole layer (relu_relax_store, cf_relax.cuh).  Decision replay
// (parity tests): with dl / du given, the three branch decisions (l >= 0, u <= 0,
// l + u >= 0) and the ReLU outputs' cases are taken from (dl, du) instead of (l, u).
__global__ void k_relu_relax(int64_t B, int64_t n, const float* __restrict__ l, const float* __restrict__ u,
                             int64_t ld_in, const ReluOut o) {
  int64_t total = B * n;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = t / n, k = t - b * n;
    relu_relax_store(o, b, k, l[b * ld_in + k], u[b * ld_in + k]);
  }
}

ReluOut relu_out(int64_t n, float* lo, float* uo, int64_t ld_out, float* alpha, float* lam, float* mu, bool strict,
                 const float* dl, const float* du, int64_t ld_dec) {
  ReluOut o;
  o.lo = lo;
  o.uo = uo;
  o.ld_out = ld_out;
  o.alpha = alpha;
  o.lam = lam;
  o.mu = mu;
  o.n = n;
  o.dl = dl;
  o.du = du;
  o.ld_dec = ld_dec;
  o.strict = strict ? 1 : 0;
  return o;
}

cf_status launch_relu_relax(int64_t B, int64_t n, const float* l, const float* u, int64_t ld_in, float* lo,
                            float* uo, int64_t ld_out, float* alpha, float* lam, float* mu, cudaStream_t st,
                            bool strict, const float* dl, const float* du) {
  int64_t total = B * n;
  if (total == 0) return CF_OK;
  int threads = 256;
  int64_t blocks = ceil_div(total, threads);
  if (blocks > 148 * 16) blocks = 148 * 16;
  prof_mem_begin(st);
  k_relu_relax<<<(unsigned)blocks, threads, 0, st>>>(B, n, l, u, ld_in,
                                                     relu_out(n, lo, uo, ld_out, alpha, lam, mu, strict, dl, du, ld_in));
  prof_mem_end(st, 28.0 * total);   // l, u in; l', u', alpha, lambda, mu out
  return check_launch("k_relu_relax");
}

// The box of a ReLU layer seen through its DeepPoly relaxation, for a traversal that
// substitutes the ReLU and then stops (custom-stop programs): a coefficient a on the ReLU
// output concretises to a * lo for the lower bound when a >= 0 (a * alpha * l of the input)
// and to a * hi when a < 0 (a * (lambda * u + mu)); the upper bound the other way round.
__global__ void k_relu_box(int64_t B, int64_t n, const float* __restrict__ l, const float* __restrict__ u,
                           int64_t ld_in, const float* __restrict__ alpha, const float* __restrict__ lam,
                           const float* __restrict__ mu, float* __restrict__ lo, float* __restrict__ hi) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * n) return;
  const int64_t b = t / n, k = t - b * n;
  lo[t] = alpha[t] * l[b * ld_in + k];
  hi[t] = fmaf(lam[t], u[b * ld_in + k], mu[t]);
}

cf_status launch_relu_box(int64_t B, int64_t n, const float* l, const float* u, int64_t ld_in, const float* alpha,
                          const float* lam, const float* mu, float* lo, float* hi, cudaStream_t st) {
  if (B * n == 0) return CF_OK;
  prof_mem_begin(st);
  k_relu_box<<<(unsigned)ceil_div(B * n, 256), 256, 0, st>>>(B, n, l, u, ld_in, alpha, lam, mu, lo, hi);
  prof_mem_end(st, 28.0 * B * n);
  return check_launch("k_relu_box");
}

// ------------------------------------------------------------------ CROWN ReLU
// The reference compiles crown.cf:25, a ternary of (l, u, L, U) tuples, into whole-layer
// branches on any() over the layer's [B, n] bounds (generated crown Relu):
//   any(l >= 0)            -> pass-through: l' = l, u' = u, L' = prev[L], U' = prev[U]
//   else any(u <= 0)       -> zero:         l' = u' = 0, L' = U' = 0
//   else (all cross zero)  -> crossing:     U' substituted one layer deeper (mixed-layer
//                                           polyexps; not expressible as per-neuron slopes)
// flags[0] = any(l >= 0), flags[1] = any(u <= 0); the caller zeroes them first.
__global__ void k_crown_flags(int64_t B, int64_t n, const float* __restrict__ l, const float* __restrict__ u,
                              int64_t ld, int* __restrict__ flags) {
  int64_t total = B * n;
  bool any_l = false, any_u = false;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = t / n, k = t - b * n;
    any_l |= l[b * ld + k] >= 0.0f;
    any_u |= u[b * ld + k] <= 0.0f;
  }
  any_l = __any_sync(0xffffffffu, any_l);
  any_u = __any_sync(0xffffffffu, any_u);
  if ((threadIdx.x & 31) == 0) {
    if (any_l) atomicOr(&flags[0], 1);
    if (any_u) atomicOr(&flags[1], 1);
  }
}

// Pass-through and zero branches as per-neuron slopes for the backsubstitution kernels
// (alpha = lam = 1, mu = 0 leaves a coefficient unchanged; all 0 removes it).  The
// crossing branch records kCrownCrossingSite in the device error word.
__global__ void k_crown_relax(int64_t B, int64_t n, const float* __restrict__ l, const float* __restrict__ u,
                              int64_t ld_in, float* __restrict__ lo, float* __restrict__ uo, int64_t ld_out,
                              float* __restrict__ alpha, float* __restrict__ lam, float* __restrict__ mu,
                              const int* __restrict__ flags, int* __restrict__ err) {
  const bool pass = flags[0] != 0, zero = !pass && flags[1] != 0;
  if (!pass && !zero && blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(err, 0, kCrownCrossingSite);
  const float s = pass ? 1.0f : 0.0f;
  int64_t total = B * n;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = t / n, k = t - b * n;
    lo[b * ld_out + k] = pass ? l[b * ld_in + k] : 0.0f;
    uo[b * ld_out + k] = pass ? u[b * ld_in + k] : 0.0f;
    alpha[t] = s;
    lam[t] = s;
    mu[t] = 0.0f;
  }
}

cf_status launch_crown_relax(int64_t B, int64_t n, const float* l, const float* u, int64_t ld_in, float* lo,
                             float* uo, int64_t ld_out, float* alpha, float* lam, float* mu, int* flags, int* err,
                             cudaStream_t st) {
  int64_t total = B * n;
  if (total == 0) return CF_OK;
  int threads = 256;
  int64_t blocks = ceil_div(total, threads);
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (cudaMemsetAsync(flags, 0, 2 * sizeof(int), st) != cudaSuccess) {
    set_error("crown_relax: cudaMemsetAsync failed");
    return CF_ERR_CUDA;
  }
  k_crown_flags<<<(unsigned)blocks, threads, 0, st>>>(B, n, l, u, ld_in, flags);
  CF_TRY(check_launch("k_crown_flags"));
  k_crown_relax<<<(unsigned)blocks, threads, 0, st>>>(B, n, l, u, ld_in, lo, uo, ld_out, alpha, lam, mu, flags,
                                                      err);
  return check_launch("k_crown_relax");
}

// ------------------------------------------------------------------ concretisation
// bound(s,b,i) = c + sum_n (a>=0 ? a*box_s[n] : a*box_{1-s}[n]), box_0 = l0, box_1 = u0.
// One warp per row; lanes stride the n0 columns (coalesced), shuffle reduction.
__global__ void k_concretize(int64_t B, int64_t R, int64_t n0, const float* __restrict__ A, int64_t a_ss,
                             int64_t a_bs, int64_t a_rs, const float* __restrict__ c, int64_t c_ss, int64_t c_bs,
                             const float* __restrict__ l0, const float* __restrict__ u0, int64_t ld_box,
                             float* __restrict__ out_l, float* __restrict__ out_u, int64_t ld_out) {
  int lane = threadIdx.x & 31;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int64_t rows = 2 * B * R;
  for (int64_t r = warp; r < rows; r += nwarps) {
    int64_t s = r / (B * R), rem = r - s * B * R, b = rem / R, i = rem - b * R;
    const float* a = A + s * a_ss + b * a_bs + i * a_rs;
    const float* pos_box = (s == 0 ? l0 : u0) + b * ld_box;
    const float* neg_box = (s == 0 ? u0 : l0) + b * ld_box;
    float acc = 0.0f;
    for (int64_t k = lane; k < n0; k += 32) {
      float v = a[k];
      acc += v >= 0.0f ? v * pos_box[k] : v * neg_box[k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      float cv = c ? c[s * c_ss + b * c_bs + i] : 0.0f;
      float res = acc + cv;
      if (s == 0) out_l[b * ld_out + i] = res;
      else out_u[b * ld_out + i] = res;
    }
  }
}

// Rows shared by every region and both bounds (the first affine layer: its W rows against
// each region's box) are two sign-split GEMMs [B, n0] x [n0, R]:
//   out_l[b,i] = c[i] + sum_n W+[i,n] l0[b,n] + W-[i,n] u0[b,n]
//   out_u[b,i] = c[i] + sum_n W+[i,n] u0[b,n] + W-[i,n] l0[b,n]
// CTA tile: 16 rows x 16 regions (a 200-row layer and 256 regions give 208 CTAs), 32-wide
// k slices of W (split into W+ / W-) and of both boxes in shared memory; 16x16 threads,
// one row x one region x 2 bounds each.  With `relu` (alpha != nullptr) the thread also
// relaxes the ReLU above the layer from the two bounds it has just stored.
constexpr int kCbT = 16, kCbK = 32, kCbM = kCbT / 16;
static_assert(kCbT * kCbK % 256 == 0, "a 256-thread block loads the tiles in whole rounds");
__global__ void __launch_bounds__(256) k_concretize_bcast(int64_t B, int64_t R, int64_t n0, const float* __restrict__ A,
                                                          int64_t a_rs, const float* __restrict__ c,
                                                          const float* __restrict__ l0, const float* __restrict__ u0,
                                                          int64_t ld_box, float* __restrict__ out_l,
                                                          float* __restrict__ out_u, int64_t ld_out,
                                                          const ReluOut relu) {
  __shared__ __align__(16) float Wp[kCbK][kCbT + 4];
  __shared__ __align__(16) float Wn[kCbK][kCbT + 4];
  __shared__ __align__(16) float Ls[kCbK][kCbT + 4];
  __shared__ __align__(16) float Us[kCbK][kCbT + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t i0 = (int64_t)blockIdx.x * kCbT, b0 = (int64_t)blockIdx.y * kCbT;
  float lo[kCbM][kCbM], up[kCbM][kCbM];
#pragma unroll
  for (int a = 0; a < kCbM; ++a)
#pragma unroll
    for (int q = 0; q < kCbM; ++q) lo[a][q] = up[a][q] = 0.0f;
  // the tiles' elements of the next K chunk are loaded into registers while the current
  // chunk's FMAs run (each thread holds kCbE of them per operand)
  constexpr int kCbE = kCbT * kCbK / 256;
  float nw[kCbE], nl[kCbE], nu[kCbE];
  auto fetch = [&](int64_t k0) {
#pragma unroll
    for (int j = 0; j < kCbE; ++j) {
      const int e = tid + 256 * j, r = e / kCbK, kk = e - r * kCbK;
      const int64_t k = k0 + kk, i = i0 + r, b = b0 + r;
      nw[j] = (i < R && k < n0) ? A[i * a_rs + k] : 0.0f;
      nl[j] = (b < B && k < n0) ? l0[b * ld_box + k] : 0.0f;
      nu[j] = (b < B && k < n0) ? u0[b * ld_box + k] : 0.0f;
    }
  };
  fetch(0);
  for (int64_t k0 = 0; k0 < n0; k0 += kCbK) {
#pragma unroll
    for (int j = 0; j < kCbE; ++j) {
      const int e = tid + 256 * j, r = e / kCbK, kk = e - r * kCbK;
      Wp[kk][r] = fmaxf(nw[j], 0.0f);
      Wn[kk][r] = fminf(nw[j], 0.0f);
      Ls[kk][r] = nl[j];
      Us[kk][r] = nu[j];
    }
    __syncthreads();
    if (k0 + kCbK < n0) fetch(k0 + kCbK);
#pragma unroll 8
    for (int kk = 0; kk < kCbK; ++kk) {
      float wpa[kCbM], wna[kCbM], la[kCbM], ua[kCbM];
#pragma unroll
      for (int a = 0; a < kCbM; ++a) {
        wpa[a] = Wp[kk][ty * kCbM + a];
        wna[a] = Wn[kk][ty * kCbM + a];
        la[a] = Ls[kk][tx * kCbM + a];
        ua[a] = Us[kk][tx * kCbM + a];
      }
#pragma unroll
      for (int a = 0; a < kCbM; ++a)
#pragma unroll
        for (int q = 0; q < kCbM; ++q) {
          lo[a][q] = fmaf(wpa[a], la[q], fmaf(wna[a], ua[q], lo[a][q]));
          up[a][q] = fmaf(wpa[a], ua[q], fmaf(wna[a], la[q], up[a][q]));
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < kCbM; ++a) {
    const int64_t i = i0 + ty * kCbM + a;
    if (i >= R) continue;
    const float cv = c ? c[i] : 0.0f;
#pragma unroll
    for (int q = 0; q < kCbM; ++q) {
      const int64_t b = b0 + tx * kCbM + q;
      if (b >= B) continue;
      const float lv = lo[a][q] + cv, uv = up[a][q] + cv;
      out_l[b * ld_out + i] = lv;
      out_u[b * ld_out + i] = uv;
      if (relu.alpha) relu_relax_store(relu, b, i, lv, uv);
    }
  }
}

cf_status launch_concretize(int64_t B, int64_t R, int64_t n0, const float* A, int64_t a_ss, int64_t a_bs,
                            int64_t a_rs, const float* c, int64_t c_ss, int64_t c_bs, const float* l0,
                            const float* u0, float* out_l, float* out_u, int64_t ld_out, cudaStream_t st,
                            const ReluOut* relu) {
  return launch_concretize_box(B, R, n0, A, a_ss, a_bs, a_rs, c, c_ss, c_bs, l0, u0, n0, out_l, out_u, ld_out, st,
                               relu);
}

cf_status launch_concretize_box(int64_t B, int64_t R, int64_t n0, const float* A, int64_t a_ss, int64_t a_bs,
                                int64_t a_rs, const float* c, int64_t c_ss, int64_t c_bs, const float* l0,
                                const float* u0, int64_t ld_box, float* out_l, float* out_u, int64_t ld_out,
                                cudaStream_t st, const ReluOut* relu) {
  int64_t rows = 2 * B * R;
  if (rows == 0) return CF_OK;
  const int64_t gx = ceil_div(R, kCbT), gy = ceil_div(B, kCbT);
  // coefficient rows (once if shared by every region), the input box, the constants, the bounds
  const bool bcast = a_ss == 0 && a_bs == 0 && c_ss == 0 && c_bs == 0;
  const double bytes = 4.0 * ((bcast ? (double)R : (double)rows) * n0 + 2.0 * B * n0 + (c ? (bcast ? R : rows) : 0) +
                              2.0 * B * R);
  if (bcast && gx <= 0x7fffffff && gy <= 65535) {
    ReluOut none;
    memset(&none, 0, sizeof(none));
    prof_mem_begin(st);
    k_concretize_bcast<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, st>>>(B, R, n0, A, a_rs, c, l0, u0, ld_box, out_l,
                                                                         out_u, ld_out, relu ? *relu : none);
    prof_mem_end(st, bytes + (relu ? 20.0 * B * R : 0.0));
    return check_launch("k_concretize_bcast");
  }
  int threads = 256;
  int64_t blocks = ceil_div(rows * 32, threads);
  if (blocks > 148 * 32) blocks = 148 * 32;
  prof_mem_begin(st);
  k_concretize<<<(unsigned)blocks, threads, 0, st>>>(B, R, n0, A, a_ss, a_bs, a_rs, c, c_ss, c_bs, l0, u0, ld_box,
                                                      out_l, out_u, ld_out);
  prof_mem_end(st, bytes);
  CF_TRY(check_launch("k_concretize"));
  if (!relu) return CF_OK;
  // the rows of one neuron's two bounds lie in different warps here: relax in a launch of its own
  prof_mem_begin(st);
  k_relu_relax<<<(unsigned)std::min<int64_t>(ceil_div(B * R, 256), 148 * 16), 256, 0, st>>>(B, R, out_l, out_u,
                                                                                            ld_out, *relu);
  prof_mem_end(st, 28.0 * B * R);
  return check_launch("k_relu_relax");
}

// ------------------------------------------------------------------ step constant
// c_out = c_in + sum_k mu-term_s(a_k) + sum_k T_s(a_k) * bias[k]
//   lower (s=0): T(a) = a>=0 ? a*alpha : a*lam,   mu-term = a<0 ? a*mu : 0
//   upper (s=1): T(a) = a>=0 ? a*lam   : a*alpha, mu-term = a>0 ? a*mu : 0
__global__ void k_step_const(int64_t B, int64_t R, int64_t K, const float* __restrict__ A, int64_t a_ss,
                             int64_t a_bs, int64_t a_rs, const float* __restrict__ c_in, int64_t c_ss, int64_t c_bs,
                             const float* __restrict__ alpha, const float* __restrict__ lam,
                             const float* __restrict__ mu, const float* __restrict__ bias,
                             float* __restrict__ c_out) {
  int lane = threadIdx.x & 31;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int64_t rows = 2 * B * R;
  for (int64_t r = warp; r < rows; r += nwarps) {
    int64_t s = r / (B * R), rem = r - s * B * R, b = rem / R, i = rem - b * R;
    const float* a = A + s * a_ss + b * a_bs + i * a_rs;
    float acc_mu = 0.0f, acc_b = 0.0f;
    for (int64_t k = lane; k < K; k += 32) {
      float v = a[k];
      float t = v;
      if (alpha) {
        float al = alpha[b * K + k], la = lam[b * K + k], m = mu[b * K + k];
        if (s == 0) {
          t = v >= 0.0f ? v * al : v * la;
          if (v < 0.0f) acc_mu += v * m;
        } else {
          t = v >= 0.0f ? v * la : v * al;
          if (v > 0.0f) acc_mu += v * m;
        }
      }
      if (bias) acc_b += t * bias[k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc_mu += __shfl_xor_sync(0xffffffffu, acc_mu, o);
      acc_b += __shfl_xor_sync(0xffffffffu, acc_b, o);
    }
    if (lane == 0) {
      float cv = c_in ? c_in[s * c_ss + b * c_bs + i] : 0.0f;
      c_out[r] = (acc_mu + cv) + acc_b;
    }
  }
}

cf_status launch_step_const(int64_t B, int64_t R, int64_t K, const float* A, int64_t a_ss, int64_t a_bs,
                            int64_t a_rs, const float* c_in, int64_t c_ss, int64_t c_bs, const float* alpha,
                            const float* lam, const float* mu, const float* bias, float* c_out, cudaStream_t st) {
  int64_t rows = 2 * B * R;
  if (rows == 0) return CF_OK;
  int threads = 256;
  int64_t blocks = ceil_div(rows * 32, threads);
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_step_const<<<(unsigned)blocks, threads, 0, st>>>(B, R, K, A, a_ss, a_bs, a_rs, c_in, c_ss, c_bs, alpha, lam, mu,
                                                      bias, c_out);
  return check_launch("k_step_const");
}

// ------------------------------------------------------------------ SIMT step GEMM
// A_out[r, :] = T_s(A_in[r, :]) @ W,  W [K, N] row-major.  64x64 output tile per CTA,
// K staged 16 at a time in shared memory, 4x4 register tile per thread.  This is the
// CUDA-core path (exact float32 FMA); the tensor-core path replaces it on B200.
constexpr int SB_M = 64, SB_N = 64, SB_K = 16;

__global__ void __launch_bounds__(256) k_step_gemm_simt(int64_t B, int64_t R, int64_t K, int64_t N,
                                                         const float* __restrict__ A, int64_t a_ss, int64_t a_bs,
                                                         int64_t a_rs, const float* __restrict__ alpha,
                                                         const float* __restrict__ lam,
                                                         const float* __restrict__ W, float* __restrict__ out) {
  __shared__ float As[SB_K][SB_M + 4];
  __shared__ float Ws[SB_K][SB_N + 4];
  const int64_t rows = 2 * B * R;
  const int64_t m0 = (int64_t)blockIdx.y * SB_M;
  const int64_t n0 = (int64_t)blockIdx.x * SB_N;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  float acc[4][4] = {};
  // per-thread A-load coordinates: 4 elements (rows lr + 16*q, column lk)
  const int lk = tid & 15, lr = tid >> 4;
  int64_t rbase[4];
  int64_t rb[4];
  int rs[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    int64_t r = m0 + lr + 16 * q;
    if (r < rows) {
      int64_t s = r / (B * R), rem = r - s * B * R, b = rem / R, i = rem - b * R;
      rbase[q] = s * a_ss + b * a_bs + i * a_rs;
      rb[q] = b;
      rs[q] = (int)s;
    } else {
      rbase[q] = -1;
      rb[q] = 0;
      rs[q] = 0;
    }
  }
  for (int64_t k0 = 0; k0 < K; k0 += SB_K) {
    int64_t k = k0 + lk;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float v = 0.0f;
      if (rbase[q] >= 0 && k < K) {
        v = A[rbase[q] + k];
        if (alpha) {
          float al = alpha[rb[q] * K + k], la = lam[rb[q] * K + k];
          float pf = rs[q] == 0 ? al : la, nf = rs[q] == 0 ? la : al;
          v = v >= 0.0f ? v * pf : v * nf;
        }
      }
      As[lk][lr + 16 * q] = v;
    }
    // W tile: 16 x 64, 4 elements per thread
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int e = tid + 256 * q;
      int kk = e >> 6, nn = e & 63;
      int64_t kg = k0 + kk, ng = n0 + nn;
      Ws[kk][nn] = (kg < K && ng < N) ? W[kg * N + ng] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SB_K; ++kk) {
      float a4[4], w4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) a4[q] = As[kk][ty * 4 + q];
#pragma unroll
      for (int q = 0; q < 4; ++q) w4[q] = Ws[kk][tx * 4 + q];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a4[i], w4[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t r = m0 + ty * 4 + i;
    if (r >= rows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t n = n0 + tx * 4 + j;
      if (n < N) out[r * N + n] = acc[i][j];
    }
  }
}

// The same product for steps whose rows are already transformed (no relaxation on load, as
// the window traversal calls it): a 128 x 128 tile, 8 x 8 outputs per thread, so each pair of
// shared-memory loads feeds twice the FMAs.  Every output sums over k in the same order as
// k_step_gemm_simt.
constexpr int SL_M = 128, SL_N = 128, SL_K = 16;
__global__ void __launch_bounds__(256) k_step_gemm_simt_large(int64_t B, int64_t R, int64_t K, int64_t N,
                                                               const float* __restrict__ A, int64_t a_ss,
                                                               int64_t a_bs, int64_t a_rs,
                                                               const float* __restrict__ W, float* __restrict__ out) {
  __shared__ __align__(16) float As[SL_K][SL_M + 4];
  __shared__ __align__(16) float Ws[SL_K][SL_N + 4];
  const int64_t rows = 2 * B * R;
  const int64_t m0 = (int64_t)blockIdx.y * SL_M;
  const int64_t n0 = (int64_t)blockIdx.x * SL_N;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  // A loads: rows lr + 16*q (q < 8) at column lk of each k slice
  const int lk = tid & 15, lr = tid >> 4;
  int64_t rbase[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int64_t r = m0 + lr + 16 * q;
    if (r < rows) {
      const int64_t sb = r / (B * R), rem = r - sb * B * R, b = rem / R, i = rem - b * R;
      rbase[q] = sb * a_ss + b * a_bs + i * a_rs;
    } else {
      rbase[q] = -1;
    }
  }
  for (int64_t k0 = 0; k0 < K; k0 += SL_K) {
    const int64_t k = k0 + lk;
#pragma unroll
    for (int q = 0; q < 8; ++q) As[lk][lr + 16 * q] = (rbase[q] >= 0 && k < K) ? A[rbase[q] + k] : 0.0f;
    // W slice: 16 x 128, 8 elements per thread
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = tid + 256 * q;
      const int kk = e >> 7, nn = e & 127;
      const int64_t kg = k0 + kk, ng = n0 + nn;
      Ws[kk][nn] = (kg < K && ng < N) ? W[kg * N + ng] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SL_K; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * 8 + 4]);
      const float4 w0 = *reinterpret_cast<const float4*>(&Ws[kk][tx * 8]);
      const float4 w1 = *reinterpret_cast<const float4*>(&Ws[kk][tx * 8 + 4]);
      const float a8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float w8[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a8[i], w8[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t r = m0 + ty * 8 + i;
    if (r >= rows) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t n = n0 + tx * 8 + j;
      if (n < N) out[r * N + n] = acc[i][j];
    }
  }
}

cf_status launch_step_gemm_simt(int64_t B, int64_t R, int64_t K, int64_t N, const float* A, int64_t a_ss,
                                int64_t a_bs, int64_t a_rs, const float* alpha, const float* lam, const float* W,
                                float* out, cudaStream_t st) {
  int64_t rows = 2 * B * R;
  if (rows == 0 || N == 0) return CF_OK;
  if (!alpha && rows >= 4 * SL_M && N >= SL_N) {
    dim3 grid((unsigned)ceil_div(N, SL_N), (unsigned)ceil_div(rows, SL_M));
    CF_REQUIRE(grid.y <= 65535u, CF_ERR_SHAPE, "step gemm: %lld rows exceed the grid limit", (long long)rows);
    k_step_gemm_simt_large<<<grid, 256, 0, st>>>(B, R, K, N, A, a_ss, a_bs, a_rs, W, out);
    return check_launch("k_step_gemm_simt_large");
  }
  dim3 grid((unsigned)ceil_div(N, SB_N), (unsigned)ceil_div(rows, SB_M));
  CF_REQUIRE(grid.y <= 65535u, CF_ERR_SHAPE, "step gemm: %lld rows exceed the grid limit", (long long)rows);
  k_step_gemm_simt<<<grid, 256, 0, st>>>(B, R, K, N, A, a_ss, a_bs, a_rs, alpha, lam, W, out);
  return check_launch("k_step_gemm_simt");
}

}  // namespace cf
