// gbcsr conv blocks on the GPU: the convolution operator held as its weights (KernelBlock,
// constraintflow/gbcsr/sparse_block.py:1158) or as per-row patches (PatchesBlock, :2576).
//
// A conv block stands for the matrix M [K*ox*oy, C*ix*iy] whose row r = (k, oxi, oyi) holds
// a kx x ky x C patch placed at input rows oxi*sx - px .. + kx - 1 and columns
// oyi*sy - py .. + ky - 1 (positions outside the image are dropped).  The patch values
// are read through strides, so one set of kernels serves both kinds:
//   value of (region b, kernel k, position pos = oxi*oy + oyi, channel c, dx, dy) =
//   P[b*p_bs + k*p_ks + pos*p_ps + (c*kx + dx)*ky + dy]
// KernelBlock: P = W [K, C, kx, ky], p_bs = p_ps = 0, p_ks = C*kx*ky.
// PatchesBlock: P [B, K*ox*oy, C*kx*ky] (rows in (k, pos) order), p_ks = ox*oy*C*kx*ky,
// p_ps = C*kx*ky, p_bs = K*ox*oy*C*kx*ky (0 for a payload shared by every region).
//
//   k_conv_densify    M itself (KernelBlock.get_dense :1195, PatchesBlock.get_dense :3089)
//   k_conv_apply      M x for a batch of images x (F.conv2d in KernelBlock.matmul_*_dims
//                     :1364, :1631; the unfold-and-sum of PatchesBlock.matmul_unequal_dims :2942)
//   k_conv_scale      M diag(d): every patch value times the input value under it (the
//                     unfold products of KernelBlock / PatchesBlock.matmul_equal_dims with a
//                     DiagonalBlock)
//   k_conv_transpose  rows y times M: the transposed convolution of each row
//                     (F.conv_transpose2d in DenseBlock.matmul_equal_dims :839-911 and in
//                     PatchesBlock.matmul_equal_dims with a KernelBlock :2740-2818)
// Sums run in float32 in a fixed order (channel, kernel row, kernel column).
#include "cf_common.cuh"

namespace cf {

struct Patches {
  const float* P;
  int64_t bs, ks, ps;
};

__device__ __forceinline__ float patch_at(const Patches& p, const cf_conv_geom& g, int64_t b, int k, int64_t pos,
                                          int c, int dx, int dy) {
  return p.P[b * p.bs + k * p.ks + pos * p.ps + ((int64_t)c * g.kx + dx) * g.ky + dy];
}

__global__ void k_conv_densify(const cf_conv_geom g, int64_t nb, const Patches p, float* __restrict__ out) {
  const int64_t rows = (int64_t)g.K * g.ox * g.oy, cols = (int64_t)g.C * g.ix * g.iy;
  const int64_t total = nb * rows * cols;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / (rows * cols);
    const int64_t rc = t - b * rows * cols;
    const int64_t r = rc / cols, col = rc - r * cols;
    const int k = (int)(r / ((int64_t)g.ox * g.oy));
    const int64_t pos = r - (int64_t)k * g.ox * g.oy;
    const int oxi = (int)(pos / g.oy), oyi = (int)(pos - (int64_t)oxi * g.oy);
    const int c = (int)(col / ((int64_t)g.ix * g.iy));
    const int64_t e = col - (int64_t)c * g.ix * g.iy;
    const int x = (int)(e / g.iy), y = (int)(e - (int64_t)x * g.iy);
    const int dx = x + g.px - oxi * g.sx, dy = y + g.py - oyi * g.sy;
    out[t] = (dx >= 0 && dx < g.kx && dy >= 0 && dy < g.ky) ? patch_at(p, g, b, k, pos, c, dx, dy) : 0.0f;
  }
}

// image n = (bb, s), bb = n / per_b: element e of its input at X[bb*x_bs + s*x_ss + e*x_es],
// output row r at out[bb*o_bs + s*o_ss + r*o_rs]
__global__ void k_conv_apply(const cf_conv_geom g, int64_t n_img, int64_t per_b, const Patches p,
                             const float* __restrict__ X, int64_t x_bs, int64_t x_ss, int64_t x_es,
                             float* __restrict__ out, int64_t o_bs, int64_t o_ss, int64_t o_rs) {
  const int64_t rows = (int64_t)g.K * g.ox * g.oy;
  const int64_t total = n_img * rows;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = t / rows, r = t - n * rows;
    const int64_t bb = n / per_b, s = n - bb * per_b;
    const int k = (int)(r / ((int64_t)g.ox * g.oy));
    const int64_t pos = r - (int64_t)k * g.ox * g.oy;
    const int oxi = (int)(pos / g.oy), oyi = (int)(pos - (int64_t)oxi * g.oy);
    const float* xb = X + bb * x_bs + s * x_ss;
    float acc = 0.0f;
    for (int c = 0; c < g.C; ++c)
      for (int dx = 0; dx < g.kx; ++dx) {
        const int x = oxi * g.sx - g.px + dx;
        if (x < 0 || x >= g.ix) continue;
        for (int dy = 0; dy < g.ky; ++dy) {
          const int y = oyi * g.sy - g.py + dy;
          if (y < 0 || y >= g.iy) continue;
          const int64_t e = ((int64_t)c * g.ix + x) * g.iy + y;
          acc = fmaf(patch_at(p, g, bb, k, pos, c, dx, dy), xb[e * x_es], acc);
        }
      }
    out[bb * o_bs + s * o_ss + r * o_rs] = acc;
  }
}

// out [nb, K*ox*oy, C*kx*ky]: patch value times the input value of region b under it (0 in
// the padding); input element e of region b at X[b*x_bs + e*x_es]
__global__ void k_conv_scale(const cf_conv_geom g, int64_t nb, const Patches p, const float* __restrict__ X,
                             int64_t x_bs, int64_t x_es, float* __restrict__ out) {
  const int64_t rows = (int64_t)g.K * g.ox * g.oy, ckk = (int64_t)g.C * g.kx * g.ky;
  const int64_t total = nb * rows * ckk;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / (rows * ckk);
    const int64_t rj = t - b * rows * ckk;
    const int64_t r = rj / ckk, j = rj - r * ckk;
    const int k = (int)(r / ((int64_t)g.ox * g.oy));
    const int64_t pos = r - (int64_t)k * g.ox * g.oy;
    const int oxi = (int)(pos / g.oy), oyi = (int)(pos - (int64_t)oxi * g.oy);
    const int c = (int)(j / ((int64_t)g.kx * g.ky));
    const int q = (int)(j - (int64_t)c * g.kx * g.ky);
    const int dx = q / g.ky, dy = q - dx * g.ky;
    const int x = oxi * g.sx - g.px + dx, y = oyi * g.sy - g.py + dy;
    const float v = (x >= 0 && x < g.ix && y >= 0 && y < g.iy)
                        ? X[b * x_bs + (((int64_t)c * g.ix + x) * g.iy + y) * x_es]
                        : 0.0f;
    out[t] = patch_at(p, g, b, k, pos, c, dx, dy) * v;
  }
}

// out[n, c, X, Y] = sum over (k, dx, dy) with X = oxi*sx - px + dx, Y = oyi*sy - py + dy of
// y[n, k, oxi, oyi] * W[k, c, dx, dy]; output size OH x OW; element e of image n's input at
// Y[bb*x_bs + s*x_ss + e*x_es], output element at out[bb*o_bs + s*o_ss + e*o_es]
__global__ void k_conv_transpose(const cf_conv_geom g, int64_t n_img, int64_t per_b, const float* __restrict__ Y,
                                 int64_t x_bs, int64_t x_ss, int64_t x_es, const float* __restrict__ W, int OH, int OW,
                                 float* __restrict__ out, int64_t o_bs, int64_t o_ss, int64_t o_es) {
  const int64_t cols = (int64_t)g.C * OH * OW;
  const int64_t total = n_img * cols;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = t / cols, e = t - n * cols;
    const int64_t bb = n / per_b, s = n - bb * per_b;
    const int c = (int)(e / ((int64_t)OH * OW));
    const int64_t xy = e - (int64_t)c * OH * OW;
    const int X = (int)(xy / OW), Yc = (int)(xy - (int64_t)X * OW);
    const float* yb = Y + bb * x_bs + s * x_ss;
    float acc = 0.0f;
    for (int k = 0; k < g.K; ++k)
      for (int dx = 0; dx < g.kx; ++dx) {
        const int ax = X + g.px - dx;
        if (ax < 0 || ax % g.sx != 0 || ax / g.sx >= g.ox) continue;
        const int oxi = ax / g.sx;
        for (int dy = 0; dy < g.ky; ++dy) {
          const int ay = Yc + g.py - dy;
          if (ay < 0 || ay % g.sy != 0 || ay / g.sy >= g.oy) continue;
          const int oyi = ay / g.sy;
          const int64_t ie = ((int64_t)k * g.ox + oxi) * g.oy + oyi;
          acc = fmaf(yb[ie * x_es], W[(((int64_t)k * g.C + c) * g.kx + dx) * g.ky + dy], acc);
        }
      }
    out[bb * o_bs + s * o_ss + e * o_es] = acc;
  }
}

static cf_status check_geom(const cf_conv_geom* g) {
  CF_REQUIRE(g, CF_ERR_NULL, "conv block: NULL geometry");
  CF_REQUIRE(g->K > 0 && g->C > 0 && g->ox > 0 && g->oy > 0 && g->ix > 0 && g->iy > 0 && g->kx > 0 && g->ky > 0 &&
                 g->sx > 0 && g->sy > 0 && g->px >= 0 && g->py >= 0,
             CF_ERR_SHAPE, "conv block: bad geometry");
  return CF_OK;
}

static unsigned grid_for(int64_t total) {
  int64_t blocks = ceil_div(total, 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  return (unsigned)(blocks < 1 ? 1 : blocks);
}

}  // namespace cf

using namespace cf;

extern "C" cf_status cf_conv_densify(const cf_conv_geom* g, int64_t nb, const float* P, int64_t p_bs, int64_t p_ks,
                                     int64_t p_ps, float* out, void* stream) {
  clear_error();
  CF_INJECT("conv_densify");
  CF_TRY(check_geom(g));
  CF_REQUIRE(nb >= 0, CF_ERR_SHAPE, "conv_densify: nb < 0");
  const int64_t total = nb * g->K * g->ox * g->oy * g->C * g->ix * g->iy;
  if (total == 0) return CF_OK;
  CF_REQUIRE(P && out, CF_ERR_NULL, "conv_densify: NULL argument");
  k_conv_densify<<<grid_for(total), 256, 0, as_stream(stream)>>>(*g, nb, Patches{P, p_bs, p_ks, p_ps}, out);
  return check_launch("k_conv_densify");
}

extern "C" cf_status cf_conv_apply(const cf_conv_geom* g, int64_t nb, int64_t per_b, const float* P, int64_t p_bs,
                                   int64_t p_ks, int64_t p_ps, const float* X, int64_t x_bs, int64_t x_ss,
                                   int64_t x_es, float* out, int64_t o_bs, int64_t o_ss, int64_t o_rs, void* stream) {
  clear_error();
  CF_INJECT("conv_apply");
  CF_TRY(check_geom(g));
  CF_REQUIRE(nb >= 0 && per_b >= 1, CF_ERR_SHAPE, "conv_apply: nb %lld, per_b %lld", (long long)nb,
             (long long)per_b);
  const int64_t total = nb * per_b * g->K * g->ox * g->oy;
  if (total == 0) return CF_OK;
  CF_REQUIRE(P && X && out, CF_ERR_NULL, "conv_apply: NULL argument");
  k_conv_apply<<<grid_for(total), 256, 0, as_stream(stream)>>>(*g, nb * per_b, per_b, Patches{P, p_bs, p_ks, p_ps}, X,
                                                                x_bs, x_ss, x_es, out, o_bs, o_ss, o_rs);
  return check_launch("k_conv_apply");
}

extern "C" cf_status cf_conv_scale(const cf_conv_geom* g, int64_t nb, const float* P, int64_t p_bs, int64_t p_ks,
                                   int64_t p_ps, const float* X, int64_t x_bs, int64_t x_es, float* out,
                                   void* stream) {
  clear_error();
  CF_INJECT("conv_scale");
  CF_TRY(check_geom(g));
  CF_REQUIRE(nb >= 0, CF_ERR_SHAPE, "conv_scale: nb < 0");
  const int64_t total = nb * g->K * g->ox * g->oy * g->C * g->kx * g->ky;
  if (total == 0) return CF_OK;
  CF_REQUIRE(P && X && out, CF_ERR_NULL, "conv_scale: NULL argument");
  k_conv_scale<<<grid_for(total), 256, 0, as_stream(stream)>>>(*g, nb, Patches{P, p_bs, p_ks, p_ps}, X, x_bs, x_es,
                                                                out);
  return check_launch("k_conv_scale");
}

extern "C" cf_status cf_conv_transpose(const cf_conv_geom* g, int64_t nb, int64_t per_b, const float* Y, int64_t x_bs,
                                       int64_t x_ss, int64_t x_es, const float* W, int32_t OH, int32_t OW, float* out,
                                       int64_t o_bs, int64_t o_ss, int64_t o_es, void* stream) {
  clear_error();
  CF_INJECT("conv_transpose");
  CF_TRY(check_geom(g));
  CF_REQUIRE(nb >= 0 && per_b >= 1 && OH > 0 && OW > 0, CF_ERR_SHAPE, "conv_transpose: bad sizes");
  const int64_t total = nb * per_b * g->C * (int64_t)OH * OW;
  if (total == 0) return CF_OK;
  CF_REQUIRE(Y && W && out, CF_ERR_NULL, "conv_transpose: NULL argument");
  k_conv_transpose<<<grid_for(total), 256, 0, as_stream(stream)>>>(*g, nb * per_b, per_b, Y, x_bs, x_ss, x_es, W, OH,
                                                                    OW, out, o_bs, o_ss, o_es);
  return check_launch("k_conv_transpose");
}
