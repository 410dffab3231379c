// Backsubstitution through convolution layers on per-row receptive-field windows.
//
// A coefficient row of a conv layer's neuron (co, oy, ox) is nonzero, at every level j
// below it, only inside its receptive field: a window of C_j x Ph x Pw positions whose
// origin is (oy*sig_h - pi_h, ox*sig_w - pi_w) in level j's image (the reference keeps the
// same information as PatchesBlock, constraintflow/gbcsr/sparse_block.py:2576-3100).
// Rows of a linear layer over an image use the whole image as their window.
//
// One substitution through ReLU_j + conv_j is two kernels:
//   k_win_relu_bias  per row (one block): in-place sign split with the region's relaxation
//                    at the window's absolute positions (zero outside the image), and the
//                    constant += mu-terms + sum T(a) * bias_j[c] (deterministic tree sum);
//   k_win_convT      the transposed convolution of every window (the adjoint of conv_j,
//                    constraintflow/gbcsr/sparse_block.py:839-928 conv_transpose2d),
//                    producing the window one level down; positions that fall in conv_j's
//                    zero padding are dropped (set to 0).
// Linear layers use the dense step GEMM on the (already transformed) rows.
// k_win_init places a conv kernel (or a linear row) as the first window, and
// k_win_concretize folds the input box in at level 0.  All CUDA-core float32.
#include "cf_common.cuh"
#include "cf_window.cuh"

namespace cf {

// window element e of row (s,b,i) -> (c, u, v) and absolute (Y, X) in the level image
struct WinPos {
  int c, Y, X;
  bool in;
};

__device__ __forceinline__ WinPos win_pos(const WinGeom& g, int64_t e, int oy, int ox) {
  WinPos p;
  const int64_t pp = (int64_t)g.Ph * g.Pw;
  p.c = (int)(e / pp);
  const int rem = (int)(e - (int64_t)p.c * pp);
  const int u = rem / g.Pw, v = rem - (rem / g.Pw) * g.Pw;
  p.Y = oy * g.sig_h - g.pi_h + u;
  p.X = ox * g.sig_w - g.pi_w + v;
  p.in = p.Y >= 0 && p.Y < g.H && p.X >= 0 && p.X < g.W;
  return p;
}

__device__ __forceinline__ void row_coords(const RowGeom& rg, int64_t r, int64_t& s, int64_t& b, int64_t& i, int& oy,
                                           int& ox) {
  const int64_t BR = rg.B * rg.R;
  s = r / BR;
  const int64_t rem = r - s * BR;
  b = rem / rg.R;
  i = rem - b * rg.R;
  const int64_t hw = (int64_t)rg.Hm * rg.Wm;
  const int64_t pos = i - (i / hw) * hw;
  oy = (int)(pos / rg.Wm);
  ox = (int)(pos - (int64_t)oy * rg.Wm);
}

// ------------------------------------------------------------------ init
// Row (s,b,i) of layer m, i = (co, oy, ox): its weights as a window at level m-1.
// Conv: W[co] [Cin, kh, kw] at origin (oy*s - p, ox*s - p).  Linear: W[i] over the whole
// level image (origin 0).  Positions outside the image are zero.
__global__ void k_win_init(RowGeom rg, WinGeom g, const float* __restrict__ W, int64_t w_bs, int conv,
                           float* __restrict__ out) {
  const int64_t per = (int64_t)g.C * g.Ph * g.Pw;
  const int64_t total = 2 * rg.B * rg.R * per;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / per, e = t - r * per;
    int64_t s, b, i;
    int oy, ox;
    row_coords(rg, r, s, b, i, oy, ox);
    const WinPos p = win_pos(g, e, oy, ox);
    float v = 0.0f;
    if (p.in) {
      if (conv) {
        const int64_t co = i / ((int64_t)rg.Hm * rg.Wm);
        v = W[co * per + e];  // kernel [Cin, kh, kw] matches the window layout
      } else {
        v = W[b * w_bs + i * per + e];  // linear row over the whole image (C, H, W) order
      }
    }
    out[t] = v;
  }
}

// ------------------------------------------------------------------ relu + bias
// One block per row.  T(a) = a>=0 ? a*pf : a*nf at in-image positions (0 elsewhere),
// c_out = c_in + sum mu-terms + sum T(a)*bias[c].  Block tree reduction (deterministic).
__global__ void __launch_bounds__(256) k_win_relu_bias(RowGeom rg, WinGeom g, float* __restrict__ A,
                                                       const float* __restrict__ c_in, int64_t c_ss, int64_t c_bs,
                                                       const float* __restrict__ alpha, const float* __restrict__ lam,
                                                       const float* __restrict__ mu, const float* __restrict__ bias,
                                                       float* __restrict__ c_out) {
  __shared__ float red[256];
  const int64_t per = (int64_t)g.C * g.Ph * g.Pw;
  const int64_t HW = (int64_t)g.H * g.W;
  const int64_t n_level = (int64_t)g.C * HW;
  const int64_t rows = 2 * rg.B * rg.R;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    int64_t s, b, i;
    int oy, ox;
    row_coords(rg, r, s, b, i, oy, ox);
    float* a = A + r * per;
    float acc = 0.0f;
    for (int64_t e = threadIdx.x; e < per; e += blockDim.x) {
      const WinPos p = win_pos(g, e, oy, ox);
      float v = a[e];
      float tr = 0.0f;
      if (p.in) {
        tr = v;
        if (alpha) {
          const int64_t k = b * n_level + (int64_t)p.c * HW + (int64_t)p.Y * g.W + p.X;
          const float al = alpha[k], la = lam[k], m = mu[k];
          const float pf = s == 0 ? al : la, nf = s == 0 ? la : al;
          tr = v >= 0.0f ? v * pf : v * nf;
          if (s == 0 ? (v < 0.0f) : (v > 0.0f)) acc = fmaf(v, m, acc);
        }
        if (bias) acc = fmaf(tr, bias[p.c], acc);
      }
      a[e] = tr;
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
      if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      const float cv = c_in ? c_in[s * c_ss + b * c_bs + i] : 0.0f;
      c_out[r] = cv + red[0];
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ transposed conv
// out[r, ci, Y', X'] = sum_{co,ky,kx} in[r, co, Y, X] * W[co, ci, ky, kx] with
// Y' = Y*s - p + ky (absolute image coordinates; input positions outside the input window
// hold zero), and 0 where (Y', X') lies outside the level image (the conv's zero padding).
// One thread per output element; W read through the L1 cache.
__global__ void k_win_convT(RowGeom rg, WinGeom gi, WinGeom go, ConvGeom cv, const float* __restrict__ in,
                            const float* __restrict__ W, float* __restrict__ out) {
  const int64_t per_in = (int64_t)gi.C * gi.Ph * gi.Pw;
  const int64_t per_out = (int64_t)go.C * go.Ph * go.Pw;
  const int64_t total = 2 * rg.B * rg.R * per_out;
  const int khw = cv.kh * cv.kw;
  const int64_t a_step = (int64_t)gi.Ph * gi.Pw, w_step = (int64_t)cv.cin * khw;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / per_out, e = t - r * per_out;
    int64_t s, b, i;
    int oy, ox;
    row_coords(rg, r, s, b, i, oy, ox);
    const WinPos p = win_pos(go, e, oy, ox);
    float acc = 0.0f;
    if (p.in) {
      const int y0 = oy * gi.sig_h - gi.pi_h, x0 = ox * gi.sig_w - gi.pi_w;
      const float* a = in + r * per_in;
      const float* wc = W + (int64_t)p.c * khw;
      for (int ky = 0; ky < cv.kh; ++ky) {
        const int ty = p.Y + cv.pad - ky;
        if (ty < 0 || ty % cv.s) continue;
        const int u = ty / cv.s - y0;
        if (u < 0 || u >= gi.Ph) continue;
        for (int kx = 0; kx < cv.kw; ++kx) {
          const int tx = p.X + cv.pad - kx;
          if (tx < 0 || tx % cv.s) continue;
          const int v = tx / cv.s - x0;
          if (v < 0 || v >= gi.Pw) continue;
          const float* ain = a + (int64_t)u * gi.Pw + v;
          const float* w = wc + ky * cv.kw + kx;
#pragma unroll 4
          for (int co = 0; co < gi.C; ++co) acc = fmaf(ain[co * a_step], __ldg(w + co * w_step), acc);
        }
      }
    }
    out[t] = acc;
  }
}

// ------------------------------------------------------------------ concretisation
// bound = c + sum_{in-image window positions} (a>=0 ? a*box_s : a*box_{1-s}); block per row.
__global__ void __launch_bounds__(256) k_win_concretize(RowGeom rg, WinGeom g, const float* __restrict__ A,
                                                        const float* __restrict__ c, const float* __restrict__ l0,
                                                        const float* __restrict__ u0, float* __restrict__ out_l,
                                                        float* __restrict__ out_u, int64_t ld_out) {
  __shared__ float red[256];
  const int64_t per = (int64_t)g.C * g.Ph * g.Pw;
  const int64_t HW = (int64_t)g.H * g.W;
  const int64_t n0 = (int64_t)g.C * HW;
  const int64_t rows = 2 * rg.B * rg.R;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    int64_t s, b, i;
    int oy, ox;
    row_coords(rg, r, s, b, i, oy, ox);
    const float* a = A + r * per;
    const float* pb = (s == 0 ? l0 : u0) + b * n0;
    const float* nb = (s == 0 ? u0 : l0) + b * n0;
    float acc = 0.0f;
    for (int64_t e = threadIdx.x; e < per; e += blockDim.x) {
      const WinPos p = win_pos(g, e, oy, ox);
      if (!p.in) continue;
      const int64_t k = (int64_t)p.c * HW + (int64_t)p.Y * g.W + p.X;
      const float v = a[e];
      acc += v >= 0.0f ? v * pb[k] : v * nb[k];
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) {
      if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      const float res = red[0] + c[r];
      if (s == 0) out_l[b * ld_out + i] = res;
      else out_u[b * ld_out + i] = res;
    }
    __syncthreads();
  }
}

static unsigned grid_for(int64_t work, int64_t per_block, int64_t cap) {
  int64_t g = ceil_div(work, per_block);
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

cf_status win_init(const RowGeom& rg, const WinGeom& g, const float* W, int64_t w_bs, bool conv, float* out,
                   cudaStream_t st) {
  const int64_t total = 2 * rg.B * rg.R * (int64_t)g.C * g.Ph * g.Pw;
  if (total == 0) return CF_OK;
  k_win_init<<<grid_for(total, 256, 148 * 32), 256, 0, st>>>(rg, g, W, w_bs, conv ? 1 : 0, out);
  return check_launch("k_win_init");
}

// c[(s,b,i)] = bias of neuron i: bias[co] for a conv layer (one value per channel,
// repeated over positions as constraintflow/lib/parse.py:126 does), bias[i] otherwise.
__global__ void k_win_row_bias(RowGeom rg, const float* __restrict__ bias, int conv, float* __restrict__ c) {
  const int64_t rows = 2 * rg.B * rg.R;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = r % rg.R;
    c[r] = bias ? (conv ? bias[i / ((int64_t)rg.Hm * rg.Wm)] : bias[i]) : 0.0f;
  }
}

cf_status win_row_bias(const RowGeom& rg, const float* bias, bool conv, float* c_out, cudaStream_t st) {
  const int64_t rows = 2 * rg.B * rg.R;
  if (rows == 0) return CF_OK;
  k_win_row_bias<<<grid_for(rows, 256, 148 * 8), 256, 0, st>>>(rg, bias, conv ? 1 : 0, c_out);
  return check_launch("k_win_row_bias");
}

cf_status win_relu_bias(const RowGeom& rg, const WinGeom& g, float* A, const float* c_in, int64_t c_ss, int64_t c_bs,
                        const float* alpha, const float* lam, const float* mu, const float* bias, float* c_out,
                        cudaStream_t st) {
  const int64_t rows = 2 * rg.B * rg.R;
  if (rows == 0) return CF_OK;
  k_win_relu_bias<<<grid_for(rows, 1, 148 * 64), 256, 0, st>>>(rg, g, A, c_in, c_ss, c_bs, alpha, lam, mu, bias,
                                                                c_out);
  return check_launch("k_win_relu_bias");
}

cf_status win_convT(const RowGeom& rg, const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, const float* in,
                    const float* W, float* out, cudaStream_t st) {
  const int64_t total = 2 * rg.B * rg.R * (int64_t)go.C * go.Ph * go.Pw;
  if (total == 0) return CF_OK;
  k_win_convT<<<grid_for(total, 256, 148 * 64), 256, 0, st>>>(rg, gi, go, cv, in, W, out);
  return check_launch("k_win_convT");
}

cf_status win_concretize(const RowGeom& rg, const WinGeom& g, const float* A, const float* c, const float* l0,
                         const float* u0, float* out_l, float* out_u, int64_t ld_out, cudaStream_t st) {
  const int64_t rows = 2 * rg.B * rg.R;
  if (rows == 0) return CF_OK;
  k_win_concretize<<<grid_for(rows, 1, 148 * 64), 256, 0, st>>>(rg, g, A, c, l0, u0, out_l, out_u, ld_out);
  return check_launch("k_win_concretize");
}

}  // namespace cf
