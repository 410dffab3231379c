// Forward certifier programs over chain networks: the zonotope domain of zono.cf (DeepZ)
// and the interval domain of ibp.cf, run by cf_deeppoly_run when net->relaxation is
// CF_RELAX_ZONO / CF_RELAX_IBP.  Follows the generated zono / ibp transformers that
// Flow.flow (constraintflow/lib/flow_sparse.py:27-228) calls layer by layer.
//
// Zonotope layout.  A neuron is c + sum_e M[e] eps_e.  Per region the symbol coefficients
// of one layer are kept TRANSPOSED, one row per noise symbol: A [E, n] (row e = symbol
// e's coefficient on every neuron of the layer), rows of region b contiguous.  Then
//   * an affine layer is one GEMM over all rows of all regions, A' = A diag(lam) W^T,
//     where lam is the column scaling of the ReLU in between (1 / 0 / u/(u-l));
//   * the symbols a ReLU opens (one per neuron: get_new_eps, constraintflow/lib/symexp.py:14)
//     form a diagonal block, never stored: after the next affine their rows are
//     nu_k * W^T[k, :] (k_zono_diag).  The input box is such a diagonal too
//     (create_Z, spec.py:106-132: c0 = (l0+u0)/2, symbols (u0-l0)/2);
//   * the concretisation l = c - sum_e |A'[e, n]|, u = c + sum_e |A'[e, n]| needs column
//     sums over the rows: every GEMM tile writes its positive and negative column sums
//     (the reference sums M+ * (-1) and M- * 1 separately), and k_zono_bounds adds the
//     tiles of a region in a fixed order.
// The ReLU's column scaling multiplies by lam = u/(u-l) where the reference divides
// (u*M)/(u-l): the two differ by at most an ulp per coefficient.
#include <stdlib.h>
#include <string.h>

#include "cf_chain.cuh"
#include "cf_common.cuh"
#include "cf_kernels.cuh"
#include "cf_plan.cuh"

namespace cf {

constexpr int kZT = 64;   // GEMM tile: 64 rows x 64 columns
constexpr int kZK = 16;   // K step

// ------------------------------------------------------------------ zonotope kernels

// A' rows [0, E) of every region: out[b, e, n] = sum_k A[b, e, k] lam[b, k] W(b, k, n);
// tile partial column sums ppos/pneg[b, tile_row, n].  Grid (ceil(N/64), ceil(E/64), B).
__global__ void __launch_bounds__(256) k_zono_gemm(int64_t E, int64_t K, int64_t N, const float* __restrict__ A,
                                                   int64_t a_bs, const float* __restrict__ lam,
                                                   const float* __restrict__ W, int64_t w_bs, int64_t w_ks,
                                                   int64_t w_ns, float* __restrict__ out, int64_t o_bs,
                                                   float* __restrict__ ppos, float* __restrict__ pneg, int64_t p_bs) {
  __shared__ float As[kZK][kZT + 4];
  __shared__ float Bs[kZK][kZT + 4];
  __shared__ float red[2][16][kZT];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t b = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.y * kZT, n0 = (int64_t)blockIdx.x * kZT;
  const float* Ab = A + b * a_bs;
  const float* Wb = W + b * w_bs;
  const float* lb = lam ? lam + b * K : nullptr;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += kZK) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = tid + 256 * q;
      const int kk = e & 15, mm = e >> 4;
      const int64_t mg = m0 + mm, kg = k0 + kk;
      float v = 0.0f;
      if (mg < E && kg < K) {
        v = Ab[mg * K + kg];
        if (lb) v *= lb[kg];
      }
      As[kk][mm] = v;
      const int kk2 = e >> 6, nn = e & 63;
      const int64_t kg2 = k0 + kk2, ng = n0 + nn;
      Bs[kk2][nn] = (kg2 < K && ng < N) ? Wb[kg2 * w_ks + ng * w_ns] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kZK; ++kk) {
      float a4[4], b4[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) a4[q] = As[kk][ty * 4 + q];
#pragma unroll
      for (int q = 0; q < 4; ++q) b4[q] = Bs[kk][tx * 4 + q];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a4[i], b4[j], acc[i][j]);
    }
    __syncthreads();
  }
  float cp[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cn[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= E) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      const float v = acc[i][j];
      if (out && n < N) out[b * o_bs + m * N + n] = v;
      cp[j] += fmaxf(v, 0.0f);
      cn[j] += fminf(v, 0.0f);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    red[0][ty][tx * 4 + j] = cp[j];
    red[1][ty][tx * 4 + j] = cn[j];
  }
  __syncthreads();
  if (tid < 2 * kZT) {
    const int which = tid / kZT, col = tid % kZT;
    float s = 0.0f;
#pragma unroll
    for (int t = 0; t < 16; ++t) s += red[which][t][col];
    const int64_t n = n0 + col;
    if (n < N) (which ? pneg : ppos)[b * p_bs + (int64_t)blockIdx.y * N + n] = s;
  }
}

// Rows of the symbols of a diagonal block d [B, K] (the input box, or the symbols the
// previous ReLU opened): out[b, row0 + k, n] = d[b, k] W(b, k, n), with their column sums
// in dpos/dneg[b, n].  Block (32, 8): 32 columns x 8 interleaved row groups, the groups'
// sums added in a fixed order; grid (ceil(N/32), B).
__global__ void __launch_bounds__(256) k_zono_diag(int64_t K, int64_t N, const float* __restrict__ d,
                                                   const float* __restrict__ W, int64_t w_bs, int64_t w_ks,
                                                   int64_t w_ns, float* __restrict__ out, int64_t o_bs, int64_t row0,
                                                   float* __restrict__ dpos, float* __restrict__ dneg) {
  __shared__ float red[2][8][32];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t n = (int64_t)blockIdx.x * 32 + tx;
  const int64_t b = blockIdx.y;
  float sp = 0.0f, sn = 0.0f;
  if (n < N) {
    const float* db = d + b * K;
    const float* Wb = W + b * w_bs + n * w_ns;
    float* ob = out ? out + b * o_bs + row0 * N + n : nullptr;
    for (int64_t k = ty; k < K; k += 8) {
      const float v = db[k] * Wb[k * w_ks];
      if (ob) ob[k * N] = v;
      sp += fmaxf(v, 0.0f);
      sn += fminf(v, 0.0f);
    }
  }
  red[0][ty][tx] = sp;
  red[1][ty][tx] = sn;
  __syncthreads();
  if (ty < 2 && n < N) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += red[ty][j][tx];
    (ty == 0 ? dpos : dneg)[b * N + n] = s;
  }
}

// Affine constant: c'[b, n] = (sum_k W(b, k, n) c[b, k]) + bias[n].  Block (32, 8) as in
// k_zono_diag; grid (ceil(N/32), B).
__global__ void __launch_bounds__(256) k_zono_const(int64_t K, int64_t N, const float* __restrict__ c,
                                                    const float* __restrict__ W, int64_t w_bs, int64_t w_ks,
                                                    int64_t w_ns, const float* __restrict__ bias,
                                                    float* __restrict__ c_out) {
  __shared__ float red[8][32];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t n = (int64_t)blockIdx.x * 32 + tx;
  const int64_t b = blockIdx.y;
  float s = 0.0f;
  if (n < N) {
    const float* cb = c + b * K;
    const float* Wb = W + b * w_bs + n * w_ns;
    for (int64_t k = ty; k < K; k += 8) s = fmaf(Wb[k * w_ks], cb[k], s);
  }
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && n < N) {
    float t = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][tx];
    c_out[b * N + n] = t + (bias ? bias[n] : 0.0f);
  }
}

struct ConvGeo {
  int32_t cin, ih, iw, cout, oh, ow, kh, kw, stride, pad;
};

// ---- conv layers of the zonotope pass (CUDA cores): the convolution applied to every
// symbol row as an image (C, H, W); neuron n = (co, oy, ox), input k = (ci, iy, ix).

// A' rows [0, E): out[b, e, n] = sum_{ci,ky,kx} A[b, e, k] lam[b, k] W[co, ci, ky, kx] with
// (iy, ix) = (oy*s - pad + ky, ox*s - pad + kx) inside the input; tile column sums as
// k_zono_gemm ([b][row tile of 64][n]).  Block (64, 4): 64 neurons x 4 row groups of 16
// rows; grid (ceil(N/64), ceil(E/64), B).
__global__ void __launch_bounds__(256) k_zono_conv_rows(int64_t E, ConvGeo g, const float* __restrict__ A,
                                                        int64_t a_bs, const float* __restrict__ lam,
                                                        const float* __restrict__ W, float* __restrict__ out,
                                                        int64_t o_bs, float* __restrict__ ppos,
                                                        float* __restrict__ pneg, int64_t p_bs) {
  __shared__ float red[2][4][64];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t N = (int64_t)g.cout * g.oh * g.ow, K = (int64_t)g.cin * g.ih * g.iw;
  const int64_t n = (int64_t)blockIdx.x * 64 + tx, b = blockIdx.z, e0 = (int64_t)blockIdx.y * 64;
  float sp = 0.0f, sn = 0.0f;
  if (n < N) {
    const int co = (int)(n / ((int64_t)g.oh * g.ow)), rem = (int)(n % ((int64_t)g.oh * g.ow));
    const int oy = rem / g.ow, ox = rem % g.ow;
    const float* lb = lam ? lam + b * K : nullptr;
    for (int j = 0; j < 16; ++j) {
      const int64_t e = e0 + ty + 4 * j;
      if (e >= E) break;
      const float* ar = A + b * a_bs + e * K;
      float acc = 0.0f;
      for (int ci = 0; ci < g.cin; ++ci)
        for (int ky = 0; ky < g.kh; ++ky) {
          const int iy = oy * g.stride - g.pad + ky;
          if (iy < 0 || iy >= g.ih) continue;
          for (int kx = 0; kx < g.kw; ++kx) {
            const int ix = ox * g.stride - g.pad + kx;
            if (ix < 0 || ix >= g.iw) continue;
            const int64_t k = ((int64_t)ci * g.ih + iy) * g.iw + ix;
            const float v = lb ? ar[k] * lb[k] : ar[k];
            acc = fmaf(v, W[(((int64_t)co * g.cin + ci) * g.kh + ky) * g.kw + kx], acc);
          }
        }
      out[b * o_bs + e * N + n] = acc;
      sp += fmaxf(acc, 0.0f);
      sn += fminf(acc, 0.0f);
    }
  }
  red[0][ty][tx] = sp;
  red[1][ty][tx] = sn;
  __syncthreads();
  if (ty < 2 && n < N) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) s += red[ty][j][tx];
    (ty == 0 ? ppos : pneg)[b * p_bs + (int64_t)blockIdx.y * N + n] = s;
  }
}

// Rows of a diagonal block d [B, K] over the conv input neurons: out[b, row0 + k, n] =
// d[b, k] W[co, ci, iy - oy*s + pad, ix - ox*s + pad] (0 where the kernel does not cover
// input k), with their column sums in dpos/dneg[b, n].  Block (32, 8), grid (ceil(N/32), B).
__global__ void __launch_bounds__(256) k_zono_diag_conv(ConvGeo g, const float* __restrict__ d,
                                                        const float* __restrict__ W, float* __restrict__ out,
                                                        int64_t o_bs, int64_t row0, float* __restrict__ dpos,
                                                        float* __restrict__ dneg) {
  __shared__ float red[2][8][32];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t N = (int64_t)g.cout * g.oh * g.ow, K = (int64_t)g.cin * g.ih * g.iw;
  const int64_t n = (int64_t)blockIdx.x * 32 + tx, b = blockIdx.y;
  float sp = 0.0f, sn = 0.0f;
  if (n < N) {
    const int co = (int)(n / ((int64_t)g.oh * g.ow)), rem = (int)(n % ((int64_t)g.oh * g.ow));
    const int y0 = (rem / g.ow) * g.stride - g.pad, x0 = (rem % g.ow) * g.stride - g.pad;
    const float* db = d + b * K;
    float* ob = out + b * o_bs + row0 * N + n;
    for (int64_t k = ty; k < K; k += 8) {
      const int ci = (int)(k / ((int64_t)g.ih * g.iw)), r2 = (int)(k % ((int64_t)g.ih * g.iw));
      const int ky = r2 / g.iw - y0, kx = r2 % g.iw - x0;
      float v = 0.0f;
      if (ky >= 0 && ky < g.kh && kx >= 0 && kx < g.kw)
        v = db[k] * W[(((int64_t)co * g.cin + ci) * g.kh + ky) * g.kw + kx];
      ob[k * N] = v;
      sp += fmaxf(v, 0.0f);
      sn += fminf(v, 0.0f);
    }
  }
  red[0][ty][tx] = sp;
  red[1][ty][tx] = sn;
  __syncthreads();
  if (ty < 2 && n < N) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += red[ty][j][tx];
    (ty == 0 ? dpos : dneg)[b * N + n] = s;
  }
}

// Conv constant: c'[b, n] = sum W[co, ci, ky, kx] c[b, (ci, iy, ix)] + bias[co].
__global__ void k_zono_const_conv(int64_t B, ConvGeo g, const float* __restrict__ c, const float* __restrict__ W,
                                  const float* __restrict__ bias, float* __restrict__ c_out) {
  const int64_t N = (int64_t)g.cout * g.oh * g.ow, K = (int64_t)g.cin * g.ih * g.iw;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * N) return;
  const int64_t b = t / N, n = t - b * N;
  const int co = (int)(n / ((int64_t)g.oh * g.ow)), rem = (int)(n % ((int64_t)g.oh * g.ow));
  const int oy = rem / g.ow, ox = rem % g.ow;
  const float* cb = c + b * K;
  float acc = 0.0f;
  for (int ci = 0; ci < g.cin; ++ci)
    for (int ky = 0; ky < g.kh; ++ky) {
      const int iy = oy * g.stride - g.pad + ky;
      if (iy < 0 || iy >= g.ih) continue;
      for (int kx = 0; kx < g.kw; ++kx) {
        const int ix = ox * g.stride - g.pad + kx;
        if (ix < 0 || ix >= g.iw) continue;
        acc = fmaf(W[(((int64_t)co * g.cin + ci) * g.kh + ky) * g.kw + kx], cb[((int64_t)ci * g.ih + iy) * g.iw + ix],
                   acc);
      }
    }
  c_out[t] = acc + bias[co];
}

// Where the column sums of one affine layer's symbol rows are: the GEMM tiles of
// k_zono_gemm ([b][tile][n], `tiles` per region), or the per-warp sums of the tensor-core
// chain (E rows per region in 128-row CTAs: [((cta*4 + w)*2 + slot)*N + n]); then the
// diagonal block's sums ([b][n]) if one entered the layer.
struct ZonoSums {
  const float* gpos;
  const float* gneg;
  int64_t tiles;
  const float* cpos;
  const float* cneg;
  int64_t E;
  const float* dpos;
  const float* dneg;
};

// Concretisation: l = ((-P) + Nn) + c, u = (P + (-Nn)) + c with P / Nn the positive /
// negative coefficient sums, added in a fixed order.  Writes the state columns (ld_state)
// and, for the property layer, the float64 bounds.
__global__ void k_zono_bounds(int64_t B, int64_t N, ZonoSums S, const float* __restrict__ c,
                              float* __restrict__ sl, float* __restrict__ su, int64_t ld_state,
                              double* __restrict__ lb,
                              double* __restrict__ ub) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * N) return;
  const int64_t b = t / N, n = t - b * N;
  float P = 0.0f, Q = 0.0f;
  if (S.gpos) {
    for (int64_t s = 0; s < S.tiles; ++s) {
      P += S.gpos[(b * S.tiles + s) * N + n];
      Q += S.gneg[(b * S.tiles + s) * N + n];
    }
  } else if (S.cpos && S.E > 0) {
    const int64_t c_lo = b * S.E / 128, c_hi = ((b + 1) * S.E - 1) / 128;
    for (int64_t cta = c_lo; cta <= c_hi; ++cta) {
      const int64_t slot = b - cta * 128 / S.E;
      for (int w = 0; w < 4; ++w) {
        const int64_t idx = ((cta * 4 + w) * 2 + slot) * N + n;
        P += S.cpos[idx];
        Q += S.cneg[idx];
      }
    }
  }
  if (S.dpos) {
    P += S.dpos[b * N + n];
    Q += S.dneg[b * N + n];
  }
  const float cc = c[t];
  const float l = (-P + Q) + cc;
  const float u = (P + (-Q)) + cc;
  sl[b * ld_state + n] = l;
  su[b * ld_state + n] = u;
  if (lb) {
    lb[t] = (double)l;
    ub[t] = (double)u;
  }
}

// Generated zono.Relu on the affine's l, u (its state columns, row stride ld_in) and c
// [B, n]: column scaling lam, fresh-symbol coefficients nu, new constant; the ReLU layer's
// own l, u are 0.  Reading the bounds from the state lets a caller that tightened them
// there (polyzono.cf: the max / min with the DeepPoly bounds) relax with the tighter ones.
__global__ void k_zono_relu(int64_t B, int64_t n, const float* __restrict__ l, const float* __restrict__ u,
                            int64_t ld_in, const float* __restrict__ c, float* __restrict__ lam,
                            float* __restrict__ nu, float* __restrict__ c_out, float* __restrict__ sl,
                            float* __restrict__ su, int64_t ld_state) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * n) return;
  const int64_t b = t / n, k = t - b * n;
  const float lv = l[b * ld_in + k], uv = u[b * ld_in + k], cv = c[t];
  const bool pos = lv >= 0.0f;
  const bool dead = !pos && uv <= 0.0f;
  float lm, nv, co;
  if (pos) {
    lm = 1.0f; nv = 0.0f; co = cv;
  } else if (dead) {
    lm = 0.0f; nv = 0.0f; co = 0.0f;
  } else {
    const float den = __fsub_rn(uv, lv);
    const float den2 = __fmul_rn(2.0f, den);
    const float ul = __fmul_rn(uv, lv);
    lm = __fdiv_rn(uv, den);
    nv = __fdiv_rn(ul, den2);
    co = __fadd_rn(__fdiv_rn(__fmul_rn(uv, cv), den), __fdiv_rn(__fmul_rn(ul, -1.0f), den2));
  }
  lam[t] = lm;
  nu[t] = nv;
  c_out[t] = co;
  sl[b * ld_state + k] = 0.0f;
  su[b * ld_state + k] = 0.0f;
}

// create_Z: c0 = (l0 + u0) / 2, symbol coefficients (u0 - l0) / 2.
__global__ void k_zono_init(int64_t total, const float* __restrict__ l0, const float* __restrict__ u0,
                            float* __restrict__ c0, float* __restrict__ dist) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total) return;
  const float l = l0[t], u = u0[t];
  c0[t] = __fdiv_rn(__fadd_rn(l, u), 2.0f);
  dist[t] = __fdiv_rn(__fsub_rn(u, l), 2.0f);
}

// W [N, K] row-major -> Wt [K, N] (32 x 32 shared-memory tiles).
__global__ void k_transpose(int64_t N, int64_t K, const float* __restrict__ W, float* __restrict__ Wt) {
  __shared__ float t[32][33];
  const int64_t k0 = (int64_t)blockIdx.x * 32, n0 = (int64_t)blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t n = n0 + r, k = k0 + threadIdx.x;
    t[r][threadIdx.x] = (n < N && k < K) ? W[n * K + k] : 0.0f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t k = k0 + r, n = n0 + threadIdx.x;
    if (k < K && n < N) Wt[k * N + n] = t[threadIdx.x][r];
  }
}

// ------------------------------------------------------------------ interval kernels

// ibp.Affine for a linear layer (or the property layer, per-region W):
// l' = (W+ l + W- u) + b, u' = (W+ u + W- l) + b.  Grid (ceil(N/128), B).
__global__ void k_ibp_linear(int64_t K, int64_t N, const float* __restrict__ l, const float* __restrict__ u,
                             const float* __restrict__ W, int64_t w_bs, int64_t w_ks, int64_t w_ns,
                             const float* __restrict__ bias, float* __restrict__ lo, float* __restrict__ uo,
                             float* __restrict__ sl, float* __restrict__ su, int64_t ld_state,
                             double* __restrict__ lb, double* __restrict__ ub) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t b = blockIdx.y;
  if (n >= N) return;
  const float* lb_ = l + b * K;
  const float* ub_ = u + b * K;
  const float* Wb = W + b * w_bs + n * w_ns;
  float pl = 0.0f, nu = 0.0f, pu = 0.0f, nl = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    const float w = Wb[k * w_ks];
    const float wp = fmaxf(w, 0.0f), wn = fminf(w, 0.0f);
    pl = fmaf(wp, lb_[k], pl);
    nu = fmaf(wn, ub_[k], nu);
    pu = fmaf(wp, ub_[k], pu);
    nl = fmaf(wn, lb_[k], nl);
  }
  const float bv = bias ? bias[n] : 0.0f;
  const float lv = (pl + nu) + bv, uv = (pu + nl) + bv;
  lo[b * N + n] = lv;
  uo[b * N + n] = uv;
  sl[b * ld_state + n] = lv;
  su[b * ld_state + n] = uv;
  if (lb) {
    lb[b * N + n] = (double)lv;
    ub[b * N + n] = (double)uv;
  }
}

// ibp.Affine for a conv layer: one thread per output neuron (co, oy, ox) of region b; the
// input bounds of region b at l + b*ld_in; lo / uo (compact [B, n_out]) may be NULL.
__global__ void k_ibp_conv(int64_t B, ConvGeo g, const float* __restrict__ l, const float* __restrict__ u,
                           int64_t ld_in, const float* __restrict__ W, const float* __restrict__ bias,
                           float* __restrict__ lo, float* __restrict__ uo, float* __restrict__ sl,
                           float* __restrict__ su, int64_t ld_state) {
  const int64_t nout = (int64_t)g.cout * g.oh * g.ow, nin = (int64_t)g.cin * g.ih * g.iw;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * nout) return;
  const int64_t b = t / nout, o = t - b * nout;
  const int co = (int)(o / (g.oh * g.ow)), rem = (int)(o % (g.oh * g.ow));
  const int oy = rem / g.ow, ox = rem % g.ow;
  const float* lb_ = l + b * ld_in;
  const float* ub_ = u + b * ld_in;
  float pl = 0.0f, nu = 0.0f, pu = 0.0f, nl = 0.0f;
  for (int ci = 0; ci < g.cin; ++ci)
    for (int ky = 0; ky < g.kh; ++ky) {
      const int iy = oy * g.stride - g.pad + ky;
      if (iy < 0 || iy >= g.ih) continue;
      for (int kx = 0; kx < g.kw; ++kx) {
        const int ix = ox * g.stride - g.pad + kx;
        if (ix < 0 || ix >= g.iw) continue;
        const float w = W[(((int64_t)co * g.cin + ci) * g.kh + ky) * g.kw + kx];
        const int64_t i = ((int64_t)ci * g.ih + iy) * g.iw + ix;
        const float wp = fmaxf(w, 0.0f), wn = fminf(w, 0.0f);
        pl = fmaf(wp, lb_[i], pl);
        nu = fmaf(wn, ub_[i], nu);
        pu = fmaf(wp, ub_[i], pu);
        nl = fmaf(wn, lb_[i], nl);
      }
    }
  const float bv = bias[co];
  const float lv = (pl + nu) + bv, uv = (pu + nl) + bv;
  if (lo) {
    lo[t] = lv;
    uo[t] = uv;
  }
  sl[b * ld_state + o] = lv;
  su[b * ld_state + o] = uv;
}

// ibp.Relu: l' = 1[l>=0] l + (1 - 1[l>=0]) 0, likewise u.
__global__ void k_ibp_relu(int64_t B, int64_t n, const float* __restrict__ l, const float* __restrict__ u,
                           float* __restrict__ lo, float* __restrict__ uo, float* __restrict__ sl,
                           float* __restrict__ su, int64_t ld_state) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * n) return;
  const int64_t b = t / n, k = t - b * n;
  const float fl = l[t] >= 0.0f ? 1.0f : 0.0f, fu = u[t] >= 0.0f ? 1.0f : 0.0f;
  const float lv = __fadd_rn(__fmul_rn(fl, l[t]), __fmul_rn(1.0f - fl, 0.0f));
  const float uv = __fadd_rn(__fmul_rn(fu, u[t]), __fmul_rn(1.0f - fu, 0.0f));
  lo[t] = lv;
  uo[t] = uv;
  sl[b * ld_state + k] = lv;
  su[b * ld_state + k] = uv;
}

// ------------------------------------------------------------------ drivers

static inline size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// Tensor-core chain (k_chain in zonotope mode) for the symbol-row GEMMs unless
// CF_STEP_IMPL=simt selects the CUDA-core kernel; the chain needs >= 128 rows per region.
static bool zono_use_chain(int64_t E) {
  const char* e = getenv("CF_STEP_IMPL");
  return E >= 128 && !(e && strcmp(e, "simt") == 0);
}

// Symbol bookkeeping of the zonotope pass, per affine index a (a == affine.size(): the
// property layer): rows stored before the layer (E_in) and the width of the diagonal
// block entering it (D_in, 0 if none).
struct ZonoShape {
  std::vector<int64_t> K, N, E_in, D_in;
  int64_t max_rows_n = 0, max_tiles_n = 0, max_cta_rows_n = 0, n_max = 0;
};

static ZonoShape zono_shape(const cf_network* net, const Plan& p) {
  ZonoShape z;
  int64_t E = 0, D = net->n_input;
  z.n_max = net->n_input;
  const size_t na = p.affine.size();
  for (size_t a = 0; a <= na; ++a) {
    const int64_t K = a < na ? net->layers[p.affine[a]].n_in : p.n_out_last;
    const int64_t N = a < na ? net->layers[p.affine[a]].n_out : net->n_spec;
    z.K.push_back(K);
    z.N.push_back(N);
    z.E_in.push_back(E);
    z.D_in.push_back(D);
    if (a < na && (E + D) * N > z.max_rows_n) z.max_rows_n = (E + D) * N;
    if (ceil_div(E, kZT) * N > z.max_tiles_n) z.max_tiles_n = ceil_div(E, kZT) * N;
    if (a < na && E * N > z.max_cta_rows_n) z.max_cta_rows_n = E * N;
    if (N > z.n_max) z.n_max = N;
    if (K > z.n_max) z.n_max = K;
    E += D;
    D = (a < na && p.relu_after[a] >= 0) ? net->layers[p.relu_after[a]].n_out : 0;
  }
  return z;
}

struct FwdLayout {
  size_t err, wt, A[2], G[2], Z[2], Dg[2], C[2], lam, nu, zeros, lu[2], state, total;
  std::vector<size_t> wt_off, wimg_off;
};

static FwdLayout fwd_layout(const cf_network* net, const Plan& p, int64_t Bc) {
  FwdLayout w;
  size_t off = 0;
  const bool zono = net->relaxation == CF_RELAX_ZONO;
  w.err = off; off += 256;
  w.wt = off;
  w.wt_off.assign(p.affine.size(), 0);
  w.wimg_off.assign(p.affine.size(), 0);
  for (size_t a = 0; a < p.affine.size(); ++a) {
    const cf_layer& L = net->layers[p.affine[a]];
    if (L.kind != CF_LAYER_LINEAR) continue;
    w.wt_off[a] = off;
    off += al256((size_t)L.n_in * L.n_out * sizeof(float));
    if (zono) {  // tensor-core image of W^T [n_in, n_out]
      w.wimg_off[a] = off;
      off += al256(chain_wimg_bytes(L.n_in, L.n_out));
    }
  }
  const ZonoShape z = zono ? zono_shape(net, p) : ZonoShape{};
  int64_t n_max = z.n_max;
  if (!zono) {
    n_max = net->n_input > net->n_spec ? net->n_input : net->n_spec;
    for (int li = 0; li < net->n_layers; ++li)
      if (net->layers[li].n_out > n_max) n_max = net->layers[li].n_out;
  }
  const size_t a_bytes = zono ? al256((size_t)Bc * z.max_rows_n * sizeof(float)) : 0;
  const size_t g_bytes = zono ? al256((size_t)Bc * z.max_tiles_n * sizeof(float)) : 0;
  // chain column sums: 8 (warp, slot) rows of N per 128-row CTA, ceil(Bc*E/128) CTAs
  const size_t z_bytes = zono ? al256((size_t)8 * (Bc * z.max_cta_rows_n / 128 + (z.n_max + 1)) * sizeof(float)) : 0;
  const size_t v_bytes = al256((size_t)Bc * n_max * sizeof(float));
  w.A[0] = off; off += a_bytes;
  w.A[1] = off; off += a_bytes;
  w.G[0] = off; off += g_bytes;
  w.G[1] = off; off += g_bytes;
  w.Z[0] = off; off += z_bytes;
  w.Z[1] = off; off += z_bytes;
  w.Dg[0] = off; off += zono ? v_bytes : 0;
  w.Dg[1] = off; off += zono ? v_bytes : 0;
  w.C[0] = off; off += zono ? v_bytes : 0;
  w.C[1] = off; off += zono ? v_bytes : 0;
  w.lam = off; off += zono ? v_bytes : 0;
  w.nu = off; off += zono ? v_bytes : 0;
  w.zeros = off; off += zono ? v_bytes : 0;
  w.lu[0] = off; off += 2 * v_bytes;
  w.lu[1] = off; off += 2 * v_bytes;
  w.state = off; off += al256((size_t)2 * Bc * p.N * sizeof(float));
  w.total = off;
  return w;
}

size_t forward_workspace_bytes(const cf_network* net, const Plan& p, int64_t chunk) {
  return fwd_layout(net, p, chunk).total;
}

// Network layers li_begin .. li_end-1 (li == n_layers: the property layer) of the zonotope
// pass over one chunk.  Which buffers hold a layer's inputs follows from its position, so a
// range can start at any layer of a pass that ran the layers before it on this workspace.
static cf_status zono_layers(const cf_network* net, const Plan& p, int64_t Bc, const float* l0, const float* u0,
                             const float* specW, float* sl, float* su, double* lb, double* ub, char* ws,
                             const FwdLayout& w, cudaStream_t st, int li_begin, int li_end) {
  const ZonoShape z = zono_shape(net, p);
  const int64_t n0 = net->n_input, Ntot = p.N;
  float* A[2] = {reinterpret_cast<float*>(ws + w.A[0]), reinterpret_cast<float*>(ws + w.A[1])};
  float* Gp = reinterpret_cast<float*>(ws + w.G[0]);
  float* Gn = reinterpret_cast<float*>(ws + w.G[1]);
  float* Zp = reinterpret_cast<float*>(ws + w.Z[0]);
  float* Zn = reinterpret_cast<float*>(ws + w.Z[1]);
  float* Dp = reinterpret_cast<float*>(ws + w.Dg[0]);
  float* Dn = reinterpret_cast<float*>(ws + w.Dg[1]);
  float* C[2] = {reinterpret_cast<float*>(ws + w.C[0]), reinterpret_cast<float*>(ws + w.C[1])};
  float* lam = reinterpret_cast<float*>(ws + w.lam);
  float* nu = reinterpret_cast<float*>(ws + w.nu);
  float* zeros = reinterpret_cast<float*>(ws + w.zeros);
  if (li_begin == 0) {
    CF_TRY(launch_copy_rows(Bc, n0, l0, n0, sl, Ntot, st));
    CF_TRY(launch_copy_rows(Bc, n0, u0, n0, su, Ntot, st));
    k_zono_init<<<(unsigned)ceil_div(Bc * n0, 256), 256, 0, st>>>(Bc * n0, l0, u0, C[0], nu);
    CF_TRY(check_launch("k_zono_init"));
  }
  int cur = 0, cc = 0;
  const float* lam_in = nullptr;        // column scaling of the ReLU before the next affine
  bool diag = true;                     // a diagonal block (nu) enters the next affine
  const size_t na = p.affine.size();
  for (size_t a = 0; a <= na; ++a) {
    const bool spec = a == na;
    const int li_aff = spec ? net->n_layers : p.affine[a];
    const int li_relu = spec ? -1 : p.relu_after[a];
    if (li_aff >= li_end) break;
    if (li_aff < li_begin) {
      // layers already run: advance the buffer positions as they did
      cur ^= 1;
      cc ^= 1;
      lam_in = nullptr;
      diag = false;
      if (li_relu >= 0) {
        if (li_relu >= li_begin && li_relu < li_end) {
          const int64_t N = z.N[a];
          const int64_t rcol = p.col[li_relu];
          const int64_t acol = p.col[p.affine[a]];
          k_zono_relu<<<(unsigned)ceil_div(Bc * N, 256), 256, 0, st>>>(Bc, N, sl + acol, su + acol, Ntot, C[cc], lam,
                                                                       nu, C[cc ^ 1],
                                                                       sl + rcol, su + rcol, Ntot);
          CF_TRY(check_launch("k_zono_relu"));
        }
        cc ^= 1;
        lam_in = lam;
        diag = true;
      }
      continue;
    }
    const int64_t K = z.K[a], N = z.N[a], E = z.E_in[a];
    const float* W;
    int64_t w_bs, w_ks, w_ns;
    const float* bias = nullptr;
    int64_t col;
    if (spec) {
      W = specW; w_bs = N * K; w_ks = 1; w_ns = K;
      col = p.spec_col;
    } else {
      const cf_layer& L = net->layers[p.affine[a]];
      W = reinterpret_cast<const float*>(ws + w.wt_off[a]); w_bs = 0; w_ks = N; w_ns = 1;
      bias = L.b_dev;
      col = p.col[p.affine[a]];
    }
    float* out = spec ? nullptr : A[cur ^ 1];
    const int64_t o_bs = (E + (diag ? K : 0)) * N;
    ZonoSums S{nullptr, nullptr, 0, nullptr, nullptr, 0, diag ? Dp : nullptr, diag ? Dn : nullptr};
    const bool conv = !spec && net->layers[p.affine[a]].kind == CF_LAYER_CONV;
    if (conv) {
      // the convolution of every symbol row, of the diagonal block and of the constant
      const cf_layer& L = net->layers[p.affine[a]];
      const ConvGeo g{L.cin, L.ih, L.iw, L.cout, L.oh, L.ow, L.kh, L.kw, L.stride, L.pad};
      const int64_t T = ceil_div(E, kZT);
      if (E > 0) {
        dim3 grid((unsigned)ceil_div(N, 64), (unsigned)T, (unsigned)Bc);
        prof_step_begin(st);
        k_zono_conv_rows<<<grid, dim3(64, 4), 0, st>>>(E, g, A[cur], E * K, lam_in, L.W_dev, out, o_bs, Gp, Gn, T * N);
        prof_step_end(st, 2.0 * Bc * E * N * L.cin * L.kh * L.kw, 4.0 * Bc * (E * K + E * N));
        CF_TRY(check_launch("k_zono_conv_rows"));
        S.gpos = Gp; S.gneg = Gn; S.tiles = T;
      }
      if (diag) {
        dim3 grid((unsigned)ceil_div(N, 32), (unsigned)Bc);
        k_zono_diag_conv<<<grid, dim3(32, 8), 0, st>>>(g, nu, L.W_dev, out, o_bs, E, Dp, Dn);
        CF_TRY(check_launch("k_zono_diag_conv"));
      }
      k_zono_const_conv<<<(unsigned)ceil_div(Bc * N, 128), 128, 0, st>>>(Bc, g, C[cc], L.W_dev, L.b_dev, C[cc ^ 1]);
      CF_TRY(check_launch("k_zono_const_conv"));
      cc ^= 1;
    } else if (E > 0) {
      if (!spec && zono_use_chain(E) && N <= 256 && K % 4 == 0) {
        // symbol rows on the tensor cores: persistent 3xTF32 GEMM (ReLU column scaling, W^T)
        ZonoTcParams Zt{};
        Zt.wimg = reinterpret_cast<const uint8_t*>(ws + w.wimg_off[a]);
        Zt.lam = lam_in;
        Zt.A = A[cur];
        Zt.a_bs = E * K;
        Zt.K = (int32_t)K;
        Zt.N = (int32_t)N;
        Zt.B = Bc;
        Zt.E = E;
        Zt.rows = Bc * E;
        Zt.out = out;
        Zt.o_bs = o_bs;
        Zt.zpos = Zp;
        Zt.zneg = Zn;
        Zt.err = reinterpret_cast<int*>(ws + w.err);
        prof_step_begin(st);
        cf_status cs = zono_tc_launch(Zt, st);
        prof_step_end(st, 2.0 * Bc * E * K * N, 4.0 * Bc * (E * K + E * N));
        CF_TRY(cs);
        S.cpos = Zp; S.cneg = Zn; S.E = E;
      } else if (!spec && zono_use_chain(E)) {
        // N > 256 or K % 4 != 0: one k_chain step per 128-row tile (ReLU column scaling, W^T)
        ChainParams P{};
        P.S = 1;
        ChainStep& CS = P.st[0];
        CS.wimg = reinterpret_cast<const uint8_t*>(ws + w.wimg_off[a]);
        CS.alpha = lam_in;
        CS.lam = lam_in;
        CS.mu = zeros;       // constant terms of the chain are not used in this mode
        CS.bias = zeros;
        CS.K = (int32_t)K;
        CS.N = (int32_t)N;
        chain_tile((int)N, CS.tile_n, CS.n_tiles);
        CS.kchunks = (int32_t)ceil_div(K, 32);
        P.B = Bc; P.R = E; P.rows = Bc * E;
        P.A0 = A[cur]; P.a_ss = 0; P.a_bs = E * K; P.a_rs = K;
        P.n0 = N;
        P.err = reinterpret_cast<int*>(ws + w.err);
        P.a0_vec = (K % 4 == 0) ? 1 : 0;
        P.zono = 1;
        P.zout = out; P.zo_bs = o_bs;
        P.zpos = Zp; P.zneg = Zn;
        prof_step_begin(st);
        cf_status cs = chain_launch(P, st);
        prof_step_end(st, 2.0 * Bc * E * K * N, 4.0 * Bc * (E * K + E * N));
        CF_TRY(cs);
        S.cpos = Zp; S.cneg = Zn; S.E = E;
      } else {
        const int64_t T = ceil_div(E, kZT);
        dim3 grid((unsigned)ceil_div(N, kZT), (unsigned)T, (unsigned)Bc);
        prof_step_begin(st);
        k_zono_gemm<<<grid, 256, 0, st>>>(E, K, N, A[cur], E * K, lam_in, W, w_bs, w_ks, w_ns, out, o_bs, Gp,
                                           Gn, T * N);
        prof_step_end(st, 2.0 * Bc * E * K * N, 4.0 * Bc * (E * K + E * N));
        CF_TRY(check_launch("k_zono_gemm"));
        S.gpos = Gp; S.gneg = Gn; S.tiles = T;
      }
    }
    if (diag && !conv) {
      dim3 grid((unsigned)ceil_div(N, 32), (unsigned)Bc);
      k_zono_diag<<<grid, dim3(32, 8), 0, st>>>(K, N, nu, W, w_bs, w_ks, w_ns, out, o_bs, E, Dp, Dn);
      CF_TRY(check_launch("k_zono_diag"));
    }
    if (!conv) {
      dim3 grid((unsigned)ceil_div(N, 32), (unsigned)Bc);
      k_zono_const<<<grid, dim3(32, 8), 0, st>>>(K, N, C[cc], W, w_bs, w_ks, w_ns, bias, C[cc ^ 1]);
      CF_TRY(check_launch("k_zono_const"));
      cc ^= 1;
    }
    // tile column sums in, the constant in, l / u out (and the float64 property bounds)
    const double zb_in = S.gpos ? 8.0 * Bc * S.tiles * N : S.cpos ? 8.0 * 8.0 * ceil_div(Bc * S.E, 128) * N : 0.0;
    prof_mem_begin(st);
    k_zono_bounds<<<(unsigned)ceil_div(Bc * N, 256), 256, 0, st>>>(Bc, N, S, C[cc], sl + col, su + col, Ntot,
                                                                   spec ? lb : nullptr, spec ? ub : nullptr);
    prof_mem_end(st, zb_in + (S.dpos ? 8.0 * Bc * N : 0.0) + 4.0 * Bc * N + (spec ? 24.0 : 8.0) * Bc * N);
    CF_TRY(check_launch("k_zono_bounds"));
    if (spec) break;
    cur ^= 1;
    lam_in = nullptr;
    diag = false;
    if (li_relu >= 0 && li_relu < li_end) {
      const int64_t rcol = p.col[li_relu];
      prof_mem_begin(st);
      k_zono_relu<<<(unsigned)ceil_div(Bc * N, 256), 256, 0, st>>>(Bc, N, sl + col, su + col, Ntot, C[cc], lam, nu,
                                                                   C[cc ^ 1],
                                                                   sl + rcol, su + rcol, Ntot);
      prof_mem_end(st, 32.0 * Bc * N);   // l, u, c in; lambda, nu, c', l', u' out
      CF_TRY(check_launch("k_zono_relu"));
      cc ^= 1;
      lam_in = lam;
      diag = true;
    }
  }
  return CF_OK;
}

// Network layers li_begin .. li_end-1 of the interval pass over one chunk (layer li writes
// compact buffer li % 2 and reads li-1's).
static cf_status ibp_layers(const cf_network* net, const Plan& p, int64_t Bc, const float* l0, const float* u0,
                            const float* specW, float* sl, float* su, double* lb, double* ub, char* ws,
                            const FwdLayout& w, cudaStream_t st, int li_begin, int li_end) {
  const int64_t n0 = net->n_input, Ntot = p.N;
  const int64_t vstride = (int64_t)((w.lu[1] - w.lu[0]) / 2 / sizeof(float));
  float* Lb[2] = {reinterpret_cast<float*>(ws + w.lu[0]), reinterpret_cast<float*>(ws + w.lu[1])};
  float* Ub[2] = {Lb[0] + vstride, Lb[1] + vstride};
  if (li_begin == 0) {
    CF_TRY(launch_copy_rows(Bc, n0, l0, n0, sl, Ntot, st));
    CF_TRY(launch_copy_rows(Bc, n0, u0, n0, su, Ntot, st));
  }
  size_t a = 0;  // affine index of layer li
  for (int li = 0; li <= net->n_layers && li < li_end; ++li) {
    const bool spec = li == net->n_layers;
    const bool affine = spec || net->layers[li].kind != CF_LAYER_RELU;
    if (li >= li_begin) {
      const float* lc = li == 0 ? l0 : Lb[(li - 1) & 1];
      const float* uc = li == 0 ? u0 : Ub[(li - 1) & 1];
      float *lo = Lb[li & 1], *uo = Ub[li & 1];
      if (spec) {
        const int64_t K = p.n_out_last, N = net->n_spec;
        dim3 grid((unsigned)ceil_div(N, 128), (unsigned)Bc);
        k_ibp_linear<<<grid, 128, 0, st>>>(K, N, lc, uc, specW, N * K, 1, K, nullptr, lo, uo, sl + p.spec_col,
                                            su + p.spec_col, Ntot, lb, ub);
        CF_TRY(check_launch("k_ibp_linear"));
        break;
      }
      const cf_layer& L = net->layers[li];
      const int64_t col = p.col[li];
      if (L.kind == CF_LAYER_RELU) {
        k_ibp_relu<<<(unsigned)ceil_div(Bc * L.n_out, 256), 256, 0, st>>>(Bc, L.n_out, lc, uc, lo, uo, sl + col,
                                                                          su + col, Ntot);
        CF_TRY(check_launch("k_ibp_relu"));
      } else if (L.kind == CF_LAYER_LINEAR) {
        const float* Wt = reinterpret_cast<const float*>(ws + w.wt_off[a]);
        dim3 grid((unsigned)ceil_div(L.n_out, 128), (unsigned)Bc);
        k_ibp_linear<<<grid, 128, 0, st>>>(L.n_in, L.n_out, lc, uc, Wt, 0, L.n_out, 1, L.b_dev, lo, uo, sl + col,
                                            su + col, Ntot, nullptr, nullptr);
        CF_TRY(check_launch("k_ibp_linear"));
      } else {
        ConvGeo g{L.cin, L.ih, L.iw, L.cout, L.oh, L.ow, L.kh, L.kw, L.stride, L.pad};
        k_ibp_conv<<<(unsigned)ceil_div(Bc * L.n_out, 128), 128, 0, st>>>(Bc, g, lc, uc, L.n_in, L.W_dev, L.b_dev,
                                                                          lo, uo, sl + col, su + col, Ntot);
        CF_TRY(check_launch("k_ibp_conv"));
      }
    }
    if (affine) ++a;
  }
  return CF_OK;
}

// Per-call preparation of the weights of affine index a (transposed copy; tensor-core image
// for the zonotope chain).
static cf_status fwd_prep_weights(const cf_network* net, const Plan& p, size_t a, char* ws, const FwdLayout& w,
                                  cudaStream_t st) {
  const cf_layer& L = net->layers[p.affine[a]];
  if (L.kind != CF_LAYER_LINEAR) return CF_OK;
  float* Wt = reinterpret_cast<float*>(ws + w.wt_off[a]);
  dim3 grid((unsigned)ceil_div(L.n_in, 32), (unsigned)ceil_div(L.n_out, 32));
  k_transpose<<<grid, dim3(32, 8), 0, st>>>(L.n_out, L.n_in, L.W_dev, Wt);
  CF_TRY(check_launch("k_transpose"));
  if (net->relaxation == CF_RELAX_ZONO)
    CF_TRY(chain_prep_weights(Wt, L.n_in, L.n_out, reinterpret_cast<uint8_t*>(ws + w.wimg_off[a]), st));
  return CF_OK;
}

static cf_status fwd_check(const cf_network* net, const Plan& p) {
  if (net->relaxation == CF_RELAX_ZONO) {
    const ZonoShape z = zono_shape(net, p);
    for (size_t a = 0; a < z.E_in.size(); ++a)
      CF_REQUIRE(ceil_div(z.E_in[a], kZT) <= 65535, CF_ERR_SHAPE, "zono: %lld noise symbols",
                 (long long)z.E_in[a]);
  }
  return CF_OK;
}

static cf_status fwd_begin(char* ws, const FwdLayout& w, bool zono, cudaStream_t st) {
  if (cudaMemsetAsync(ws + w.err, 0, 256, st) != cudaSuccess ||
      (zono && cudaMemsetAsync(ws + w.zeros, 0, w.lu[0] - w.zeros, st) != cudaSuccess)) {
    set_error("forward run: cudaMemsetAsync failed");
    return CF_ERR_CUDA;
  }
  return CF_OK;
}

cf_status forward_layer(const cf_network* net, const Plan& p, int layer, int64_t B, const float* l0,
                        const float* u0, const float* specW, float* state_l, float* state_u, double* lb, double* ub,
                        void* workspace, size_t ws_bytes, cudaStream_t st) {
  CF_TRY(fwd_check(net, p));
  CF_REQUIRE(B <= 65535, CF_ERR_SHAPE, "per-layer runs: at most 65535 regions per call");
  const FwdLayout w = fwd_layout(net, p, B);
  CF_REQUIRE(ws_bytes >= w.total, CF_ERR_WORKSPACE,
             "per-layer runs keep the whole batch: workspace %zu < %zu bytes", ws_bytes, w.total);
  char* ws = static_cast<char*>(workspace);
  if (layer == 0) CF_TRY(fwd_begin(ws, w, net->relaxation == CF_RELAX_ZONO, st));
  for (size_t a = 0; a < p.affine.size(); ++a)
    if (p.affine[a] == layer) CF_TRY(fwd_prep_weights(net, p, a, ws, w, st));
  if (net->relaxation == CF_RELAX_ZONO)
    return zono_layers(net, p, B, l0, u0, specW, state_l, state_u, lb, ub, ws, w, st, layer, layer + 1);
  return ibp_layers(net, p, B, l0, u0, specW, state_l, state_u, lb, ub, ws, w, st, layer, layer + 1);
}

cf_status forward_run(const cf_network* net, const Plan& p, int64_t B, const float* l0, const float* u0,
                      const float* specW, float* state_l, float* state_u, double* lb, double* ub, void* workspace,
                      size_t ws_bytes, cudaStream_t st) {
  const bool zono = net->relaxation == CF_RELAX_ZONO;
  CF_TRY(fwd_check(net, p));
  const size_t base = fwd_layout(net, p, 1).total;
  CF_REQUIRE(ws_bytes >= base, CF_ERR_WORKSPACE, "workspace %zu < %zu bytes needed for one region", ws_bytes, base);
  int64_t lo = 1, hi = B < 65535 ? B : 65535;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) / 2;
    if (fwd_layout(net, p, mid).total <= ws_bytes) lo = mid;
    else hi = mid - 1;
  }
  const int64_t Bc = lo;
  const FwdLayout w = fwd_layout(net, p, Bc);
  char* ws = static_cast<char*>(workspace);
  CF_TRY(fwd_begin(ws, w, zono, st));
  for (size_t a = 0; a < p.affine.size(); ++a) CF_TRY(fwd_prep_weights(net, p, a, ws, w, st));
  const int64_t N = p.N, n0 = net->n_input, ns = net->n_spec;
  for (int64_t b0 = 0; b0 < B; b0 += Bc) {
    const int64_t nb = (B - b0 < Bc) ? (B - b0) : Bc;
    float* sl = state_l ? state_l + b0 * N : reinterpret_cast<float*>(ws + w.state);
    float* su = state_u ? state_u + b0 * N : reinterpret_cast<float*>(ws + w.state) + Bc * N;
    const float* sw = specW + b0 * ns * p.n_out_last;
    if (zono)
      CF_TRY(zono_layers(net, p, nb, l0 + b0 * n0, u0 + b0 * n0, sw, sl, su, lb + b0 * ns, ub + b0 * ns, ws, w, st, 0,
                         net->n_layers + 1));
    else
      CF_TRY(ibp_layers(net, p, nb, l0 + b0 * n0, u0 + b0 * n0, sw, sl, su, lb + b0 * ns, ub + b0 * ns, ws, w, st, 0,
                        net->n_layers + 1));
  }
  return CF_OK;
}

// l = max(l_a, l_b), u = min(u_a, u_b) over [B, n], written back to both states (rows at
// ld_a / ld_b) and, if lb is not NULL, to the float64 bounds [B, n].  NaN in either operand
// gives NaN, as torch.maximum / torch.minimum do.
__global__ void k_bounds_meet(int64_t B, int64_t n, float* __restrict__ la, float* __restrict__ ua, int64_t ld_a,
                              float* __restrict__ lb_, float* __restrict__ ub_, int64_t ld_b,
                              double* __restrict__ lo, double* __restrict__ hi) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * n) return;
  const int64_t b = t / n, k = t - b * n;
  const int64_t ia = b * ld_a + k, ib = b * ld_b + k;
  const float l1 = la[ia], l2 = lb_[ib], u1 = ua[ia], u2 = ub_[ib];
  const float l = (l1 != l1 || l2 != l2) ? __int_as_float(0x7fc00000) : fmaxf(l1, l2);
  const float u = (u1 != u1 || u2 != u2) ? __int_as_float(0x7fc00000) : fminf(u1, u2);
  la[ia] = l;
  lb_[ib] = l;
  ua[ia] = u;
  ub_[ib] = u;
  if (lo) {
    lo[t] = (double)l;
    hi[t] = (double)u;
  }
}

cf_status launch_ibp_conv_state(int64_t B, const cf_layer& L, const float* l, const float* u, int64_t ld_in,
                                float* sl, float* su, int64_t ld_state, cudaStream_t st) {
  if (B * L.n_out == 0) return CF_OK;
  const ConvGeo g{L.cin, L.ih, L.iw, L.cout, L.oh, L.ow, L.kh, L.kw, L.stride, L.pad};
  prof_mem_begin(st);
  k_ibp_conv<<<(unsigned)ceil_div(B * L.n_out, 128), 128, 0, st>>>(B, g, l, u, ld_in, L.W_dev, L.b_dev, nullptr,
                                                                    nullptr, sl, su, ld_state);
  prof_mem_end(st, 4.0 * (2.0 * B * L.n_in + (double)L.cout * L.cin * L.kh * L.kw + L.cout + 2.0 * B * L.n_out));
  return check_launch("k_ibp_conv");
}

}  // namespace cf

using namespace cf;

extern "C" cf_status cf_bounds_meet(int64_t B, int64_t n, float* l_a, float* u_a, int64_t ld_a, float* l_b,
                                    float* u_b, int64_t ld_b, double* lb, double* ub, void* stream) {
  clear_error();
  CF_INJECT("bounds_meet");
  CF_REQUIRE(B >= 0 && n >= 0 && ld_a >= n && ld_b >= n, CF_ERR_SHAPE, "bounds_meet: bad sizes");
  if (B * n == 0) return CF_OK;
  CF_REQUIRE(l_a && u_a && l_b && u_b, CF_ERR_NULL, "bounds_meet: NULL argument");
  CF_REQUIRE((lb == nullptr) == (ub == nullptr), CF_ERR_NULL, "bounds_meet: lb and ub both or neither");
  k_bounds_meet<<<(unsigned)ceil_div(B * n, 256), 256, 0, as_stream(stream)>>>(B, n, l_a, u_a, ld_a, l_b, u_b, ld_b,
                                                                              lb, ub);
  return check_launch("k_bounds_meet");
}
