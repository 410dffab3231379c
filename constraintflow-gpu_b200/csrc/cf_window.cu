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
//   k_win_convT_gemm the transposed convolution of every window (the adjoint of conv_j,
//                    constraintflow/gbcsr/sparse_block.py:839-928 conv_transpose2d) as one
//                    implicit GEMM per stride phase, producing the window one level down;
//                    positions that fall in conv_j's zero padding are dropped (set to 0).
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

// (a window holds one level image at most: e < C*H*W fits 32 bits)
__device__ __forceinline__ WinPos win_pos(const WinGeom& g, int e, int oy, int ox) {
  WinPos p;
  const int pp = g.Ph * g.Pw;
  p.c = e / pp;
  const int rem = e - p.c * pp;
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
// A warp per row: the row's coordinates once, then its elements in 32-bit arithmetic.
__global__ void k_win_init(RowGeom rg, WinGeom g, const float* __restrict__ W, int64_t w_bs, int conv,
                           float* __restrict__ out) {
  const int per = g.C * g.Ph * g.Pw;
  const int64_t rows = 2 * rg.B * rg.R;
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < rows; r += nwarps) {
    int64_t s, b, i;
    int oy, ox;
    row_coords(rg, r, s, b, i, oy, ox);
    // conv: the kernel [Cin, kh, kw] of the row's channel matches the window layout;
    // linear: the row over the whole image in (C, H, W) order
    const float* src = conv ? W + (i / ((int64_t)rg.Hm * rg.Wm)) * per : W + b * w_bs + i * per;
    float* dst = out + r * per;
    for (int e = lane; e < per; e += 32) {
      const WinPos p = win_pos(g, e, oy, ox);
      dst[e] = p.in ? src[e] : 0.0f;
    }
  }
}

// ------------------------------------------------------------------ relu + bias
// kT threads per row (a warp for small windows, the whole block for large ones), 256 / kT
// rows per block.  T(a) = a>=0 ? a*pf : a*nf at in-image positions (0 elsewhere),
// c_out = c_in + sum mu-terms + sum T(a)*bias[c].  A thread owns one window position p of
// the Ph x Pw plane (several when the plane is larger than kT) and a fixed subset of the
// channels, so the plane coordinates and the relaxation offsets are computed once per
// position; the row sum is a fixed-order shuffle (and, for kT = 256, shared-memory) tree.
template <int kT>
__global__ void __launch_bounds__(256, 4) k_win_relu_bias(RowGeom rg, WinGeom g, float* __restrict__ A,
                                                       const float* __restrict__ c_in, int64_t c_ss, int64_t c_bs,
                                                       const float* __restrict__ alpha, const float* __restrict__ lam,
                                                       const float* __restrict__ mu, const float* __restrict__ bias,
                                                       float* __restrict__ c_out) {
  __shared__ float red[8];
  constexpr int kRowsPerBlock = 256 / kT;
  const int pp = g.Ph * g.Pw;
  const int HW = g.H * g.W;
  const int64_t per = (int64_t)g.C * pp;
  const int64_t n_level = (int64_t)g.C * HW;
  const int64_t rows = 2 * rg.B * rg.R;
  const int t = threadIdx.x % kT, slot = threadIdx.x / kT;
  // channel lanes: threads t = cl*pp + p when the plane is smaller than kT
  const int cstep = pp >= kT ? 1 : kT / pp;
  const int c0 = pp >= kT ? 0 : t / pp;
  const int p_first = pp >= kT ? t : t - (t / pp) * pp;
  const int p_step = pp >= kT ? kT : pp;
  const bool active = c0 < cstep;
  for (int64_t r0 = (int64_t)blockIdx.x * kRowsPerBlock; r0 < rows; r0 += (int64_t)gridDim.x * kRowsPerBlock) {
    const int64_t r = r0 + slot;
    float acc = 0.0f;
    int64_t s = 0, b = 0, i = 0;
    if (r < rows && active) {
      int oy, ox;
      row_coords(rg, r, s, b, i, oy, ox);
      float* a = A + r * per;
      const float* pf = nullptr;
      const float* nf = nullptr;
      if (alpha) {
        pf = s == 0 ? alpha : lam;
        nf = s == 0 ? lam : alpha;
      }
      for (int p = p_first; p < pp; p += p_step) {
        const int u = p / g.Pw, v = p - (p / g.Pw) * g.Pw;
        const int Y = oy * g.sig_h - g.pi_h + u, X = ox * g.sig_w - g.pi_w + v;
        const bool in = Y >= 0 && Y < g.H && X >= 0 && X < g.W;
        if (!in) {
          for (int c = c0; c < g.C; c += cstep) a[(int64_t)c * pp + p] = 0.0f;
          continue;
        }
        const int64_t k0 = b * n_level + (int64_t)Y * g.W + X;
        int c = c0;
        // four channels at a time: their loads are issued before any of their arithmetic
        // (the pass is latency-bound otherwise); same summation order as one at a time
        for (; c + 3 * cstep < g.C; c += 4 * cstep) {
          float x[4], pv[4], nv[4], mv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int cc = c + q * cstep;
            x[q] = a[(int64_t)cc * pp + p];
            if (alpha) {
              const int64_t k = k0 + (int64_t)cc * HW;
              pv[q] = __ldg(pf + k);
              nv[q] = __ldg(nf + k);
              mv[q] = __ldg(mu + k);
            }
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int cc = c + q * cstep;
            float tr = x[q];
            if (alpha) {
              tr = x[q] >= 0.0f ? x[q] * pv[q] : x[q] * nv[q];
              if (s == 0 ? (x[q] < 0.0f) : (x[q] > 0.0f)) acc = fmaf(x[q], mv[q], acc);
            }
            if (bias) acc = fmaf(tr, __ldg(bias + cc), acc);
            a[(int64_t)cc * pp + p] = tr;
          }
        }
        for (; c < g.C; c += cstep) {
          const int64_t e = (int64_t)c * pp + p;
          const float x = a[e];
          float tr = x;
          if (alpha) {
            const int64_t k = k0 + (int64_t)c * HW;
            tr = x >= 0.0f ? x * pf[k] : x * nf[k];
            if (s == 0 ? (x < 0.0f) : (x > 0.0f)) acc = fmaf(x, mu[k], acc);
          }
          if (bias) acc = fmaf(tr, bias[c], acc);
          a[e] = tr;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (kT == 256) {
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
      __syncthreads();
      if (threadIdx.x == 0) {
        float tot = 0.0f;
        for (int w = 0; w < 8; ++w) tot += red[w];
        acc = tot;
      }
      __syncthreads();
    }
    if (t == 0 && r < rows) {
      int64_t ss, bb, ii;
      int oy, ox;
      row_coords(rg, r, ss, bb, ii, oy, ox);
      const float cv = c_in ? c_in[ss * c_ss + bb * c_bs + ii] : 0.0f;
      c_out[r] = cv + acc;
    }
  }
}

// Whole-image windows (origin 0, the window is the level image: rows of linear layers and
// of the property): window element e of region b is relaxation index b*n_level + e, so the
// row is processed in 16-byte pieces.  Same arithmetic as k_win_relu_bias; block per row.
__global__ void __launch_bounds__(256) k_win_relu_bias_whole(RowGeom rg, WinGeom g, float* __restrict__ A,
                                                             const float* __restrict__ c_in, int64_t c_ss,
                                                             int64_t c_bs, const float* __restrict__ alpha,
                                                             const float* __restrict__ lam,
                                                             const float* __restrict__ mu,
                                                             const float* __restrict__ bias,
                                                             float* __restrict__ c_out) {
  __shared__ float red[8];
  const int pp = g.Ph * g.Pw;
  const int64_t per = (int64_t)g.C * pp;   // == n_level, a multiple of 4
  const int64_t rows = 2 * rg.B * rg.R;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    int64_t s, b, i;
    int oy, ox;
    row_coords(rg, r, s, b, i, oy, ox);
    float4* a = reinterpret_cast<float4*>(A + r * per);
    const float4* pf = nullptr;
    const float4* nf = nullptr;
    const float4* m4 = nullptr;
    if (alpha) {
      pf = reinterpret_cast<const float4*>((s == 0 ? alpha : lam) + b * per);
      nf = reinterpret_cast<const float4*>((s == 0 ? lam : alpha) + b * per);
      m4 = reinterpret_cast<const float4*>(mu + b * per);
    }
    float acc = 0.0f;
    const int64_t n4 = per / 4;
    const bool c_per4 = (pp & 3) == 0;   // the 4 elements of a piece share one channel
    // one 16-byte piece: transform in place, accumulate in element order
    auto piece = [&](int64_t q, float4 x, float4 p4, float4 n4v, float4 u4) {
      const float xs[4] = {x.x, x.y, x.z, x.w};
      float tr[4] = {x.x, x.y, x.z, x.w};
      if (alpha) {
        const float ps[4] = {p4.x, p4.y, p4.z, p4.w}, ns[4] = {n4v.x, n4v.y, n4v.z, n4v.w};
        const float ms[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          tr[e] = xs[e] >= 0.0f ? xs[e] * ps[e] : xs[e] * ns[e];
          if (s == 0 ? (xs[e] < 0.0f) : (xs[e] > 0.0f)) acc = fmaf(xs[e], ms[e], acc);
        }
      }
      if (bias) {
        if (c_per4) {
          const float bv = __ldg(bias + (4 * q) / pp);
#pragma unroll
          for (int e = 0; e < 4; ++e) acc = fmaf(tr[e], bv, acc);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) acc = fmaf(tr[e], __ldg(bias + (4 * q + e) / pp), acc);
        }
      }
      a[q] = make_float4(tr[0], tr[1], tr[2], tr[3]);
    };
    const float4 z4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    // two pieces per iteration, both loaded before either is transformed
    int64_t q = threadIdx.x;
    for (; q + blockDim.x < n4; q += 2 * (int64_t)blockDim.x) {
      const int64_t q2 = q + blockDim.x;
      const float4 x1 = a[q], x2 = a[q2];
      float4 p1 = z4, n1 = z4, u1 = z4, p2 = z4, n2 = z4, u2 = z4;
      if (alpha) {
        p1 = __ldg(pf + q);
        n1 = __ldg(nf + q);
        u1 = __ldg(m4 + q);
        p2 = __ldg(pf + q2);
        n2 = __ldg(nf + q2);
        u2 = __ldg(m4 + q2);
      }
      piece(q, x1, p1, n1, u1);
      piece(q2, x2, p2, n2, u2);
    }
    for (; q < n4; q += blockDim.x) {
      float4 p1 = z4, n1 = z4, u1 = z4;
      if (alpha) {
        p1 = __ldg(pf + q);
        n1 = __ldg(nf + q);
        u1 = __ldg(m4 + q);
      }
      piece(q, a[q], p1, n1, u1);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = 0.0f;
      for (int w = 0; w < 8; ++w) tot += red[w];
      const float cv = c_in ? c_in[s * c_ss + b * c_bs + i] : 0.0f;
      c_out[r] = cv + tot;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ transposed conv
// out[r, ci, u', v'] = sum_{co,ky,kx} in[r, co, u, v] * W[co, ci, ky, kx] over window
// coordinates, where the conv maps input-window position (u, v) of row r and tap (ky, kx)
// to output-window position u' = u*s + ky - D (D = pi_in*s + pad - pi_out: 0 for
// receptive-field windows, pad for whole-image windows), and 0 where (u', v') lies outside
// the level image (the conv's zero padding).  Since u' + D = u*s + ky, the output positions
// split into s*s stride phases (py, px) = ((u'+D) mod s, (v'+D) mod s), and within a phase
// only taps ky = py + ty*s, kx = px + tx*s contribute, at u = qy - ty, v = qx - tx with
// qy = (u' + D - py)/s.  Each phase is an implicit GEMM
//   M = rows x (phase positions), K = Cout x (phase taps), N = cin,
// A gathered from the input windows (zero outside them), B = the phase's weight taps.
// CTA tile BM x BN, k slices of BK in shared memory; 256 threads, TM x TN outputs each.
template <int BM, int BN, int TM, int TN, int BK>
__global__ void __launch_bounds__(256) k_win_convT_gemm(RowGeom rg, WinGeom gi, WinGeom go, ConvGeom cv,
                                                        ConvPhase ph, const float* __restrict__ in,
                                                        const float* __restrict__ W, float* __restrict__ out) {
  static_assert((BM / TM) * (BN / TN) == 256, "256 threads");
  static_assert(BM % 256 == 0 || 256 % BM == 0, "A tile mapping");
  constexpr int MPT = BM >= 256 ? BM / 256 : 1;   // A rows gathered by each thread
  constexpr int KSTEP = BM >= 256 ? 1 : 256 / BM;  // k stride of a thread's A loads
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  const int tid = threadIdx.x, tn = tid % (BN / TN), tm = tid / (BN / TN);
  const int pos = ph.ny * ph.nx, taps = ph.tyn * ph.txn;
  const int64_t M = 2 * rg.B * rg.R * pos;
  const int K = gi.C * taps;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int64_t plane_in = (int64_t)gi.Ph * gi.Pw, per_in = gi.C * plane_in;
  // the A rows this thread gathers in every k slice: m = m0 + (tid % BM) + 256*x
  const float* a_row[MPT];
  int a_qy[MPT], a_qx[MPT];
#pragma unroll
  for (int x = 0; x < MPT; ++x) {
    const int64_t m = m0 + (tid % BM) + 256 * x;
    a_row[x] = nullptr;
    a_qy[x] = a_qx[x] = 0;
    if (m < M) {
      const int64_t r = m / pos;
      const int rem = (int)(m - r * pos);
      const int iy = rem / ph.nx;
      a_qy[x] = ph.q0y + iy;
      a_qx[x] = ph.q0x + (rem - iy * ph.nx);
      a_row[x] = in + r * per_in;
    }
  }
  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll 4
    for (int kk = BM >= 256 ? 0 : tid / BM; kk < BK; kk += KSTEP) {
      const int k = k0 + kk;
      int co = 0, u_off = 0, v_off = 0;
      if (k < K) {
        co = k / taps;
        const int t = k - co * taps, ty = t / ph.txn;
        u_off = ty;
        v_off = t - ty * ph.txn;
      }
#pragma unroll
      for (int x = 0; x < MPT; ++x) {
        float val = 0.0f;
        if (a_row[x] && k < K) {
          const int u = a_qy[x] - u_off, v = a_qx[x] - v_off;
          if (u >= 0 && u < gi.Ph && v >= 0 && v < gi.Pw) val = a_row[x][co * plane_in + u * gi.Pw + v];
        }
        As[kk][(tid % BM) + 256 * x] = val;
      }
    }
    for (int e = tid; e < BK * BN; e += 256) {
      const int nn = e % BN, kk = e / BN;
      const int k = k0 + kk, ci = n0 + nn;
      float val = 0.0f;
      if (k < K && ci < cv.cin) {
        const int co = k / taps, t = k - co * taps, ty = t / ph.txn, tx = t - ty * ph.txn;
        const int ky = ph.py + ty * cv.s, kx = ph.px + tx * cv.s;
        val = __ldg(W + (((int64_t)co * cv.cin + ci) * cv.kh + ky) * cv.kw + kx);
      }
      Bs[kk][nn] = val;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; i += 4) {
        const float4 q = *reinterpret_cast<const float4*>(&As[kk][tm * TM + i]);
        a[i] = q.x;
        a[i + 1] = q.y;
        a[i + 2] = q.z;
        a[i + 3] = q.w;
      }
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tn * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  const int64_t plane_out = (int64_t)go.Ph * go.Pw, per_out = go.C * plane_out;
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t m = m0 + tm * TM + i;
    if (m >= M) continue;
    const int64_t r = m / pos;
    const int rem = (int)(m - r * pos);
    const int iy = rem / ph.nx, ix = rem - iy * ph.nx;
    const int uo = ph.u0 + iy * cv.s, vo = ph.v0 + ix * cv.s;
    int64_t sb, b, ri;
    int oy, ox;
    row_coords(rg, r, sb, b, ri, oy, ox);
    const int Y = oy * go.sig_h - go.pi_h + uo, X = ox * go.sig_w - go.pi_w + vo;
    const bool inside = Y >= 0 && Y < go.H && X >= 0 && X < go.W;
    float* o = out + r * per_out + (int64_t)uo * go.Pw + vo;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int ci = n0 + tn * TN + j;
      if (ci < cv.cin) o[ci * plane_out] = inside ? acc[i][j] : 0.0f;
    }
  }
}

// ------------------------------------------------------------------ concretisation
// bound = c + sum_{in-image window positions} (a>=0 ? a*box_s : a*box_{1-s}); block per row.
// kT threads per row (a warp for windows of at most 2048 elements, the block otherwise),
// 256 / kT rows per block; the row's sum is a fixed-order shuffle (and, for kT = 256,
// shared-memory) tree.
template <int kT>
__global__ void __launch_bounds__(256) k_win_concretize(RowGeom rg, WinGeom g, const float* __restrict__ A,
                                                        const float* __restrict__ c, const float* __restrict__ l0,
                                                        const float* __restrict__ u0, float* __restrict__ out_l,
                                                        float* __restrict__ out_u, int64_t ld_out) {
  __shared__ float red[8];
  constexpr int kRowsPerBlock = 256 / kT;
  const int per = g.C * g.Ph * g.Pw;
  const int64_t HW = (int64_t)g.H * g.W;
  const int64_t n0 = (int64_t)g.C * HW;
  const int64_t rows = 2 * rg.B * rg.R;
  const int t = threadIdx.x % kT, slot = threadIdx.x / kT;
  for (int64_t r0 = (int64_t)blockIdx.x * kRowsPerBlock; r0 < rows; r0 += (int64_t)gridDim.x * kRowsPerBlock) {
    const int64_t r = r0 + slot;
    float acc = 0.0f;
    int64_t s = 0, b = 0, i = 0;
    if (r < rows) {
      int oy, ox;
      row_coords(rg, r, s, b, i, oy, ox);
      const float* a = A + r * per;
      const float* pb = (s == 0 ? l0 : u0) + b * n0;
      const float* nb = (s == 0 ? u0 : l0) + b * n0;
      for (int e = t; e < per; e += kT) {
        const WinPos p = win_pos(g, e, oy, ox);
        if (!p.in) continue;
        const int64_t k = (int64_t)p.c * HW + (int64_t)p.Y * g.W + p.X;
        const float v = a[e];
        acc += v >= 0.0f ? v * pb[k] : v * nb[k];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (kT == 256) {
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
      __syncthreads();
      if (threadIdx.x == 0) {
        float tot = 0.0f;
        for (int w = 0; w < 8; ++w) tot += red[w];
        acc = tot;
      }
      __syncthreads();
    }
    if (t == 0 && r < rows) {
      const float res = acc + c[r];
      if (s == 0) out_l[b * ld_out + i] = res;
      else out_u[b * ld_out + i] = res;
    }
  }
}

static unsigned grid_for(int64_t work, int64_t per_block, int64_t cap) {
  int64_t g = ceil_div(work, per_block);
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

// ------------------------------------------------------------------ first layer, fused
// The last substitution of a traversal through a stride-1 conv layer with at most 4 input
// channels (the first layer of an image network), fused with the concretisation against the
// input box, so that the input-level window of a row is never stored.  A block takes rb
// rows at a time; their windows are staged in shared memory cc channels at a time (each
// row's channels are contiguous, so the copy is coalesced); a thread computes 4 consecutive
// output columns of one output row for every input channel, accumulating over channels and
// taps in registers (the row segment it reads is shared by the kw taps), folds its outputs
// into the box bound (a >= 0 ? a * box_s : a * box_{1-s} at in-image positions) and the
// block adds each row's partial bounds in a fixed order.
__device__ __forceinline__ void cp_async4(float* dst_smem, const float* src, bool valid) {
  // 4-byte asynchronous copy global -> shared; zero-filled (nothing read) when !valid
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst_smem)),
               "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int NCI, int KW>
__global__ void __launch_bounds__(256) k_win_first(RowGeom rg, WinGeom gi, WinGeom go, int kh, int cout, int Dy,
                                                   int Dx, int rb, int cc, const float* __restrict__ in,
                                                   const float* __restrict__ W, const float* __restrict__ c,
                                                   const float* __restrict__ l0, const float* __restrict__ u0,
                                                   float* __restrict__ out_l, float* __restrict__ out_u,
                                                   int64_t ld_out) {
  extern __shared__ float sm[];
  // weights regrouped as [cout][kh][kWG]: the NCI x KW taps of one (channel, kernel row)
  // are contiguous and padded to whole 16-byte pieces (vector loads, zero padding)
  constexpr int kWG = (NCI * KW + 3) / 4 * 4;
  const int wn = cout * kh * kWG;
  float* wsm = sm;
  const int plane = gi.Ph * gi.Pw;
  const int stage = rb * cc * plane;
  float* xs = sm + wn;                              // two stages of [rb][cc][Ph][Pw]
  float* part = xs + 2 * (size_t)stage;             // [256] partial bounds
  for (int e = threadIdx.x; e < wn; e += blockDim.x) {
    const int g = e / kWG, j = e - (e / kWG) * kWG;   // g = co * kh + ky
    const int co = g / kh, ky = g - (g / kh) * kh;
    const int ci = j / KW, kx = j - (j / KW) * KW;
    wsm[e] = j < NCI * KW ? W[((co * NCI + ci) * kh + ky) * KW + kx] : 0.0f;
  }
  const int XG = (go.Pw + 3) / 4, TPR = go.Ph * XG;
  const int64_t per_in = (int64_t)gi.C * plane;
  const int64_t rows = 2 * rg.B * rg.R;
  const int64_t HW0 = (int64_t)go.H * go.W, n0 = (int64_t)NCI * HW0;
  const int slot = threadIdx.x / TPR, task = threadIdx.x - (threadIdx.x / TPR) * TPR;
  const int up = task / XG, xg = task - (task / XG) * XG;
  const int64_t r_step = (int64_t)gridDim.x * rb;
  // the (row group, channel chunk) sequence of this block, staged two ahead by cp.async:
  // chunk (r0, co0) into stage buffer `buf`
  auto issue = [&](int64_t r0, int co0, int buf) {
    const int nc = cout - co0 < cc ? cout - co0 : cc;
    const int per_chunk = nc * plane;
    float* dst = xs + (size_t)buf * stage;
    for (int e = threadIdx.x; e < rb * per_chunk; e += blockDim.x) {
      const int rs = e / per_chunk, rem = e - rs * per_chunk;
      const int64_t row = r0 + rs;
      const bool ok = row < rows;
      cp_async4(dst + (size_t)rs * cc * plane + rem, ok ? in + row * per_in + (int64_t)co0 * plane + rem : in, ok);
    }
  };
  int64_t r0 = (int64_t)blockIdx.x * rb;
  int co0 = 0, buf = 0;
  if (r0 < rows) issue(r0, 0, 0);
  cp_async_commit();
  float acc[4][NCI];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int ci = 0; ci < NCI; ++ci) acc[j][ci] = 0.0f;
  while (r0 < rows) {
    // the next chunk of the sequence into the other buffer (its previous contents were
    // consumed before the barrier that ended the last iteration)
    int64_t r1 = r0;
    int co1 = co0 + cc;
    if (co1 >= cout) {
      co1 = 0;
      r1 = r0 + r_step;
    }
    if (r1 < rows) issue(r1, co1, buf ^ 1);
    cp_async_commit();
    cp_async_wait1();   // this chunk's copies (all but the group just issued) have landed
    __syncthreads();
    const int64_t r = r0 + slot;
    const bool active = slot < rb && r < rows;
    const int nc = cout - co0 < cc ? cout - co0 : cc;
    if (active) {
      const float* xb = xs + (size_t)buf * stage;
      for (int cix = 0; cix < nc; ++cix) {
        const float* xp = xb + ((size_t)slot * cc + cix) * plane;
        for (int ky = 0; ky < kh; ++ky) {
          const int u = up + Dy - ky;
          if (u < 0 || u >= gi.Ph) continue;
          float wk[kWG];
          const float4* wv = reinterpret_cast<const float4*>(wsm + ((size_t)(co0 + cix) * kh + ky) * kWG);
#pragma unroll
          for (int q = 0; q < kWG / 4; ++q) {
            const float4 t = wv[q];
            wk[4 * q] = t.x;
            wk[4 * q + 1] = t.y;
            wk[4 * q + 2] = t.z;
            wk[4 * q + 3] = t.w;
          }
          const float* xr = xp + u * gi.Pw;
          float xv[4 + KW - 1];
#pragma unroll
          for (int q = 0; q < 4 + KW - 1; ++q) {
            const int v = xg * 4 + Dx - (KW - 1) + q;
            xv[q] = (v >= 0 && v < gi.Pw) ? xr[v] : 0.0f;
          }
#pragma unroll
          for (int kx = 0; kx < KW; ++kx) {
#pragma unroll
            for (int ci = 0; ci < NCI; ++ci) {
              const float w = wk[ci * KW + kx];
#pragma unroll
              for (int j = 0; j < 4; ++j) acc[j][ci] = fmaf(xv[j + (KW - 1) - kx], w, acc[j][ci]);
            }
          }
        }
      }
    }
    if (co0 + cc >= cout) {
      // the row group is complete: fold its outputs into the box bound, add them per row
      float partial = 0.0f;
      if (active) {
        int64_t s, b, i;
        int oy, ox;
        row_coords(rg, r, s, b, i, oy, ox);
        const float* pb = (s == 0 ? l0 : u0) + b * n0;
        const float* nb = (s == 0 ? u0 : l0) + b * n0;
        const int Y = oy * go.sig_h - go.pi_h + up;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int vo = xg * 4 + j;
          const int X = ox * go.sig_w - go.pi_w + vo;
          if (vo >= go.Pw || Y < 0 || Y >= go.H || X < 0 || X >= go.W) continue;
#pragma unroll
          for (int ci = 0; ci < NCI; ++ci) {
            const int64_t k = (int64_t)ci * HW0 + (int64_t)Y * go.W + X;
            const float a = acc[j][ci];
            partial = fmaf(a, a >= 0.0f ? pb[k] : nb[k], partial);
          }
        }
      }
      part[threadIdx.x] = partial;
      __syncthreads();
      if (threadIdx.x < rb && r0 + threadIdx.x < rows) {
        const int64_t rr = r0 + threadIdx.x;
        float tot = 0.0f;
        for (int t = 0; t < TPR; ++t) tot += part[threadIdx.x * TPR + t];
        int64_t s, b, i;
        int oy, ox;
        row_coords(rg, rr, s, b, i, oy, ox);
        const float res = tot + c[rr];
        if (s == 0) out_l[b * ld_out + i] = res;
        else out_u[b * ld_out + i] = res;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int ci = 0; ci < NCI; ++ci) acc[j][ci] = 0.0f;
    }
    __syncthreads();   // this buffer (and the partials) are consumed
    r0 = r1;
    co0 = co1;
    buf ^= 1;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// shared-memory floats of one stage of staged windows per block (two stages)
constexpr int kFirstStageFloats = 4096;

static bool first_geometry(const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, int cout, int& rb, int& cc) {
  if (cv.s != 1 || cv.cin < 1 || cv.cin > 4 || !(cv.kw == 3 || cv.kw == 5) || cv.kh > 7 || go.C != cv.cin)
    return false;
  const int TPR = go.Ph * ((go.Pw + 3) / 4);
  const int plane = gi.Ph * gi.Pw;
  if (TPR > 256 || plane > kFirstStageFloats || cout * cv.cin * cv.kh * cv.kw > 4096) return false;
  rb = 256 / TPR;
  while (rb > 1 && rb * plane > kFirstStageFloats) --rb;
  cc = kFirstStageFloats / (rb * plane);
  if (cc > cout) cc = cout;
  return cc >= 1;
}

bool win_convT_first_applicable(const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, int cout) {
  int rb, cc;
  return first_geometry(gi, go, cv, cout, rb, cc);
}

cf_status win_convT_first(const RowGeom& rg, const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, int cout,
                          const float* in, const float* W, const float* c, const float* l0, const float* u0,
                          float* out_l, float* out_u, int64_t ld_out, cudaStream_t st) {
  int rb, cc;
  CF_REQUIRE(first_geometry(gi, go, cv, cout, rb, cc), CF_ERR_UNSUPPORTED, "win_convT_first: geometry");
  const int64_t rows = 2 * rg.B * rg.R;
  if (rows == 0) return CF_OK;
  const int Dy = gi.pi_h + cv.pad - go.pi_h, Dx = gi.pi_w + cv.pad - go.pi_w;
  const int wn = cout * cv.kh * ((cv.cin * cv.kw + 3) / 4 * 4);   // the regrouped weights (see k_win_first)
  const size_t smem = (size_t)(wn + 2 * rb * cc * gi.Ph * gi.Pw + 256) * sizeof(float);
  const unsigned grid = grid_for(rows, rb, 148 * 16);
#define CF_FIRST(NCI, KW)                                                                                          \
  do {                                                                                                             \
    cudaFuncSetAttribute(k_win_first<NCI, KW>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);            \
    k_win_first<NCI, KW><<<grid, 256, smem, st>>>(rg, gi, go, cv.kh, cout, Dy, Dx, rb, cc, in, W, c, l0, u0, out_l, \
                                                  out_u, ld_out);                                                  \
  } while (0)
  if (cv.kw == 3) {
    switch (cv.cin) {
      case 1: CF_FIRST(1, 3); break;
      case 2: CF_FIRST(2, 3); break;
      case 3: CF_FIRST(3, 3); break;
      default: CF_FIRST(4, 3); break;
    }
  } else {
    switch (cv.cin) {
      case 1: CF_FIRST(1, 5); break;
      case 2: CF_FIRST(2, 5); break;
      case 3: CF_FIRST(3, 5); break;
      default: CF_FIRST(4, 5); break;
    }
  }
#undef CF_FIRST
  return check_launch("k_win_first");
}

cf_status win_init(const RowGeom& rg, const WinGeom& g, const float* W, int64_t w_bs, bool conv, float* out,
                   cudaStream_t st) {
  const int64_t total = 2 * rg.B * rg.R * (int64_t)g.C * g.Ph * g.Pw;
  if (total == 0) return CF_OK;
  CF_REQUIRE((int64_t)g.C * g.Ph * g.Pw < 0x7fffffff, CF_ERR_SHAPE, "win_init: window too large");
  k_win_init<<<grid_for(2 * rg.B * rg.R, 8, 148 * 32), 256, 0, st>>>(rg, g, W, w_bs, conv ? 1 : 0, out);
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
  const int64_t per = (int64_t)g.C * g.Ph * g.Pw;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  const bool whole = g.sig_h == 0 && g.sig_w == 0 && g.pi_h == 0 && g.pi_w == 0 && g.Ph == g.H && g.Pw == g.W;
  if (whole && per % 4 == 0 && a16(A) && (!alpha || (a16(alpha) && a16(lam) && a16(mu)))) {
    k_win_relu_bias_whole<<<grid_for(rows, 1, 148 * 64), 256, 0, st>>>(rg, g, A, c_in, c_ss, c_bs, alpha, lam, mu,
                                                                       bias, c_out);
  } else if (per <= 2048) {   // a warp per row, 8 rows per block
    k_win_relu_bias<32><<<grid_for(rows, 8, 148 * 64), 256, 0, st>>>(rg, g, A, c_in, c_ss, c_bs, alpha, lam, mu,
                                                                     bias, c_out);
  } else {
    k_win_relu_bias<256><<<grid_for(rows, 1, 148 * 64), 256, 0, st>>>(rg, g, A, c_in, c_ss, c_bs, alpha, lam, mu,
                                                                      bias, c_out);
  }
  return check_launch("k_win_relu_bias");
}

cf_status win_convT(const RowGeom& rg, const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, const float* in,
                    const float* W, float* out, cudaStream_t st) {
  const int64_t rows = 2 * rg.B * rg.R;
  if (rows * go.C * go.Ph * go.Pw == 0) return CF_OK;
  const int s = cv.s;
  // window-relative input index u = (u' + D - ky) / s (see k_win_convT_gemm)
  const int Dy = gi.pi_h * s + cv.pad - go.pi_h, Dx = gi.pi_w * s + cv.pad - go.pi_w;
  for (int py = 0; py < s; ++py) {
    const int u0 = ((py - Dy) % s + s) % s;
    const int ny = u0 < go.Ph ? (go.Ph - u0 + s - 1) / s : 0;
    const int tyn = cv.kh > py ? (cv.kh - py + s - 1) / s : 0;
    for (int px = 0; px < s; ++px) {
      const int v0 = ((px - Dx) % s + s) % s;
      const int nx = v0 < go.Pw ? (go.Pw - v0 + s - 1) / s : 0;
      const int txn = cv.kw > px ? (cv.kw - px + s - 1) / s : 0;
      if (ny == 0 || nx == 0) continue;
      ConvPhase ph{py, px, ny, nx, tyn, txn, u0, v0, (u0 + Dy - py) / s, (v0 + Dx - px) / s};
      const int64_t M = rows * ny * nx;
      const int bm = cv.cin > 4 ? 128 : 1024;
      const int64_t gx = (M + bm - 1) / bm;
      CF_REQUIRE(gx <= 0x7fffffff, CF_ERR_SHAPE, "convT: %lld output positions", (long long)M);
      // tile by input-channel count: 128 positions x 64/32/16 channels, or 1024 x 4 for the
      // first layer of an image network (cin <= 4)
      if (cv.cin > 32) {
        k_win_convT_gemm<128, 64, 8, 4, 32><<<dim3((unsigned)gx, (unsigned)((cv.cin + 63) / 64)), 256, 0, st>>>(
            rg, gi, go, cv, ph, in, W, out);
      } else if (cv.cin > 16) {
        k_win_convT_gemm<128, 32, 8, 2, 32><<<dim3((unsigned)gx, 1), 256, 0, st>>>(rg, gi, go, cv, ph, in, W, out);
      } else if (cv.cin > 4) {
        k_win_convT_gemm<128, 16, 8, 1, 32><<<dim3((unsigned)gx, 1), 256, 0, st>>>(rg, gi, go, cv, ph, in, W, out);
      } else {
        k_win_convT_gemm<1024, 4, 4, 4, 8><<<dim3((unsigned)gx, 1), 256, 0, st>>>(rg, gi, go, cv, ph, in, W, out);
      }
      CF_TRY(check_launch("k_win_convT_gemm"));
    }
  }
  return CF_OK;
}

cf_status win_concretize(const RowGeom& rg, const WinGeom& g, const float* A, const float* c, const float* l0,
                         const float* u0, float* out_l, float* out_u, int64_t ld_out, cudaStream_t st) {
  const int64_t rows = 2 * rg.B * rg.R;
  if (rows == 0) return CF_OK;
  CF_REQUIRE((int64_t)g.C * g.Ph * g.Pw < 0x7fffffff, CF_ERR_SHAPE, "win_concretize: window too large");
  if ((int64_t)g.C * g.Ph * g.Pw <= 2048)
    k_win_concretize<32><<<grid_for(rows, 8, 148 * 64), 256, 0, st>>>(rg, g, A, c, l0, u0, out_l, out_u, ld_out);
  else
    k_win_concretize<256><<<grid_for(rows, 1, 148 * 64), 256, 0, st>>>(rg, g, A, c, l0, u0, out_l, out_u, ld_out);
  return check_launch("k_win_concretize");
}

}  // namespace cf
