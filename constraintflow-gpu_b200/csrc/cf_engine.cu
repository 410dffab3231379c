// Network driver of libcfgpu: runs DeepPoly over a chain network for a batch of input
// regions, region chunk by region chunk, entirely stream-ordered on the caller's stream.
//
// Per chunk the abstract state is a pair of [Bc, N] float32 arrays (every neuron's lower
// and upper bound, the dense view of the reference's abs_elem.d['l'|'u']), plus the ReLU
// relaxations (alpha, lam, mu) of every ReLU layer.  An affine layer m is bounded by
// backsubstitution: its coefficient rows start as W_m (shared by every region: zero
// region stride) and are pushed through ReLU_j + affine_j for j = m-1 .. 0 by one step
// kernel each, then folded into the input box.  Follows the generated deeppoly.Affine
// while-loop and Flow.flow (constraintflow/lib/flow_sparse.py:27-228).
#include <stdarg.h>

#include <mutex>
#include <vector>

#include "cf_chain.cuh"
#include "cf_common.cuh"
#include "cf_kernels.cuh"
#include "cf_plan.cuh"
#include "cf_step.cuh"
#include "cf_window.cuh"

namespace cf {

static thread_local char g_err[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
void clear_error() { g_err[0] = 0; }

bool fault_injected(const char* site) {
  const char* env = getenv("CF_FAULT");
  if (!env || !*env) return false;
  size_t n = strlen(site);
  const char* p = env;
  while (*p) {
    const char* q = strchr(p, ',');
    size_t len = q ? (size_t)(q - p) : strlen(p);
    if (len == n && strncmp(p, site, n) == 0) return true;
    if (!q) break;
    p = q + 1;
  }
  return false;
}

// ------------------------------------------------------------------ small kernels
__global__ void k_to_f64(int64_t B, int64_t n, const float* __restrict__ src_l, const float* __restrict__ src_u,
                         int64_t ld, double* __restrict__ dst_l, double* __restrict__ dst_u) {
  int64_t total = B * n;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = t / n, k = t - b * n;
    dst_l[t] = (double)src_l[b * ld + k];
    dst_u[t] = (double)src_u[b * ld + k];
  }
}

cf_status launch_to_f64(int64_t B, int64_t n, const float* src_l, const float* src_u, int64_t ld_src, double* dst_l,
                        double* dst_u, cudaStream_t st) {
  if (B * n == 0) return CF_OK;
  int64_t blocks = ceil_div(B * n, 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  prof_mem_begin(st);
  k_to_f64<<<(unsigned)blocks, 256, 0, st>>>(B, n, src_l, src_u, ld_src, dst_l, dst_u);
  prof_mem_end(st, 24.0 * B * n);
  return check_launch("k_to_f64");
}

cf_status launch_copy_rows(int64_t B, int64_t n, const float* src, int64_t ld_src, float* dst, int64_t ld_dst,
                           cudaStream_t st) {
  if (B * n == 0) return CF_OK;
  cudaError_t e = cudaMemcpy2DAsync(dst, ld_dst * sizeof(float), src, ld_src * sizeof(float), n * sizeof(float), B,
                                    cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) {
    set_error("copy_rows: %s", cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  return CF_OK;
}

// ------------------------------------------------------------------ network plan
static void window_sizing(const cf_network* net, Plan& p);

cf_status make_plan(const cf_network* net, Plan& p) {
  CF_REQUIRE(net && net->layers && net->n_layers > 0, CF_ERR_NULL, "network: empty");
  CF_REQUIRE(net->n_input > 0 && net->n_spec > 0, CF_ERR_SHAPE, "network: bad input/spec size");
  CF_REQUIRE(net->relaxation >= CF_RELAX_DEEPPOLY && net->relaxation <= CF_RELAX_CROWNIBP_STRICT, CF_ERR_UNSUPPORTED,
             "network: relaxation %d", net->relaxation);
  CF_REQUIRE(net->stop_depth >= 0, CF_ERR_SHAPE, "network: stop_depth %d", net->stop_depth);
  CF_REQUIRE(net->stop_depth == 0 || net->relaxation == CF_RELAX_DEEPPOLY ||
                 net->relaxation == CF_RELAX_DEEPPOLY_STRICT, CF_ERR_UNSUPPORTED,
             "network: a custom stop depth applies to the DeepPoly traversal only");
  int64_t pos = net->n_input, prev_width = net->n_input;
  p.col.assign(net->n_layers, 0);
  p.relu_after.clear();
  p.affine.clear();
  p.in_img.clear();
  p.out_img.clear();
  p.has_conv = false;
  // image carried between layers: the input is (n_input,1,1) unless the first layer is a conv
  Img img{net->n_input, 1, 1};
  if (net->layers[0].kind == CF_LAYER_CONV) img = Img{net->layers[0].cin, net->layers[0].ih, net->layers[0].iw};
  for (int li = 0; li < net->n_layers; ++li) {
    const cf_layer& L = net->layers[li];
    CF_REQUIRE(L.n_in == prev_width, CF_ERR_SHAPE, "layer %d: n_in %d != previous width %lld", li, L.n_in,
               (long long)prev_width);
    if (L.kind == CF_LAYER_RELU) {
      CF_REQUIRE(!p.affine.empty() && p.relu_after.back() == -1 && net->layers[li - 1].kind != CF_LAYER_RELU,
                 CF_ERR_UNSUPPORTED, "layer %d: ReLU must follow an affine layer", li);
      CF_REQUIRE(L.n_out == L.n_in, CF_ERR_SHAPE, "layer %d: ReLU width mismatch", li);
      p.relu_after.back() = li;
      p.relu_total += L.n_out;
    } else if (L.kind == CF_LAYER_LINEAR) {
      CF_REQUIRE(L.W_dev && L.b_dev, CF_ERR_NULL, "layer %d: weights missing", li);
      CF_REQUIRE((int64_t)img.C * img.H * img.W == L.n_in, CF_ERR_SHAPE, "layer %d: input image mismatch", li);
      p.affine.push_back(li);
      p.relu_after.push_back(-1);
      p.in_img.push_back(img);
      img = Img{L.n_out, 1, 1};
      p.out_img.push_back(img);
    } else if (L.kind == CF_LAYER_CONV) {
      CF_REQUIRE(L.W_dev && L.b_dev, CF_ERR_NULL, "layer %d: weights missing", li);
      CF_REQUIRE(L.cin == img.C && L.ih == img.H && L.iw == img.W, CF_ERR_SHAPE,
                 "layer %d: conv input (%d,%d,%d) != previous image (%d,%d,%d)", li, L.cin, L.ih, L.iw, img.C,
                 img.H, img.W);
      CF_REQUIRE(L.stride >= 1 && L.kh >= 1 && L.kw >= 1 && L.pad >= 0 && L.cout >= 1, CF_ERR_SHAPE,
                 "layer %d: bad conv geometry", li);
      CF_REQUIRE(L.oh == (L.ih + 2 * L.pad - L.kh) / L.stride + 1 && L.ow == (L.iw + 2 * L.pad - L.kw) / L.stride + 1,
                 CF_ERR_SHAPE, "layer %d: conv output size", li);
      CF_REQUIRE(L.n_in == L.cin * L.ih * L.iw && L.n_out == L.cout * L.oh * L.ow, CF_ERR_SHAPE,
                 "layer %d: conv neuron counts", li);
      p.affine.push_back(li);
      p.relu_after.push_back(-1);
      p.in_img.push_back(img);
      img = Img{L.cout, L.oh, L.ow};
      p.out_img.push_back(img);
      p.has_conv = true;
    } else {
      set_error("layer %d: unknown kind %d", li, L.kind);
      return CF_ERR_UNSUPPORTED;
    }
    p.col[li] = pos;
    pos += L.n_out;
    prev_width = L.n_out;
  }
  CF_REQUIRE(net->layers[net->n_layers - 1].kind != CF_LAYER_RELU, CF_ERR_UNSUPPORTED,
             "network must end with an affine layer");
  CF_REQUIRE(net->stop_depth == 0 || !p.has_conv, CF_ERR_UNSUPPORTED,
             "network: a custom stop depth on conv layers is not supported");
  p.n_out_last = prev_width;
  p.spec_col = pos;
  p.N = pos + net->n_spec;
  p.r_max = net->n_spec;
  p.r_max_all = net->n_spec;
  for (size_t a = 0; a < p.affine.size(); ++a) {
    const cf_layer& L = net->layers[p.affine[a]];
    if (L.n_out > p.r_max_all) p.r_max_all = L.n_out;
    if (a > 0 && L.n_out > p.r_max) p.r_max = L.n_out;
    if (L.n_in > p.n_max) p.n_max = L.n_in;
    if (L.n_out > p.k_max) p.k_max = L.n_out;
  }
  window_sizing(net, p);
  return CF_OK;
}

// Windows of the bounded layer with affine index a (a == affine.size(): the property
// layer) at levels a-1, a-2, ..., 0 and finally the input image: geoms[0] is the window
// over layer a's input, geoms.back() the window over the network input.
static void window_chain(const cf_network* net, const Plan& p, size_t a, std::vector<WinGeom>& geoms) {
  geoms.clear();
  const bool spec = a == p.affine.size();
  const Img lvl = a == 0 ? p.in_img[0] : p.out_img[a - 1];
  WinGeom g;
  g.C = lvl.C;
  g.H = lvl.H;
  g.W = lvl.W;
  if (!spec && net->layers[p.affine[a]].kind == CF_LAYER_CONV) {
    const cf_layer& L = net->layers[p.affine[a]];
    g.Ph = L.kh;
    g.Pw = L.kw;
    g.sig_h = g.sig_w = L.stride;
    g.pi_h = g.pi_w = L.pad;
  } else {
    g.Ph = lvl.H;
    g.Pw = lvl.W;
    g.sig_h = g.sig_w = 0;
    g.pi_h = g.pi_w = 0;
  }
  geoms.push_back(g);
  for (int64_t j = (int64_t)a - 1; j >= 0; --j) {
    const cf_layer& Lj = net->layers[p.affine[j]];
    const Img in = p.in_img[j];
    WinGeom h;
    h.C = in.C;
    h.H = in.H;
    h.W = in.W;
    if (Lj.kind == CF_LAYER_CONV && g.sig_h > 0) {
      h.Ph = (g.Ph - 1) * Lj.stride + Lj.kh;
      h.Pw = (g.Pw - 1) * Lj.stride + Lj.kw;
      h.sig_h = g.sig_h * Lj.stride;
      h.sig_w = g.sig_w * Lj.stride;
      h.pi_h = g.pi_h * Lj.stride + Lj.pad;
      h.pi_w = g.pi_w * Lj.stride + Lj.pad;
    } else {  // a single position: the whole image below (exact, outside is zero)
      h.Ph = in.H;
      h.Pw = in.W;
      h.sig_h = h.sig_w = 0;
      h.pi_h = h.pi_w = 0;
    }
    geoms.push_back(h);
    g = h;
  }
}

static int64_t window_rows(const cf_network* net, const Plan& p, size_t a) {
  return a == p.affine.size() ? net->n_spec : net->layers[p.affine[a]].n_out;
}

static void window_sizing(const cf_network* net, Plan& p) {
  p.win_floats = 0;
  if (!p.has_conv) return;
  std::vector<WinGeom> gs;
  for (size_t a = 0; a <= p.affine.size(); ++a) {
    window_chain(net, p, a, gs);
    const int64_t R = window_rows(net, p, a);
    for (const WinGeom& g : gs) {
      const int64_t f = 2 * R * (int64_t)g.C * g.Ph * g.Pw;
      if (f > p.win_floats) p.win_floats = f;
    }
  }
}

static inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct WsLayout {
  size_t err, wimg, A[2], C[2], X[2], relu, box, state, total;
  size_t conv_wimg;  // weight image of one conv phase for the tensor-core transposed convolution
  std::vector<size_t> wimg_off;  // per affine index
};

// Tensor-core chain (cf_chain.cu) unless CF_STEP_IMPL=simt selects the CUDA-core steps.
static bool use_chain() {
  const char* e = getenv("CF_STEP_IMPL");
  return !(e && strcmp(e, "simt") == 0);
}

// The fused first-layer kernel (win_convT_first) for the last substitution of a traversal,
// unless CF_CONV_IMPL=simt or =tc selects the unfused transposed convolution.
static bool use_conv_first(const WinGeom& g, const WinGeom& h, const cf_layer& L) {
  const char* e = getenv("CF_CONV_IMPL");
  if (e && (strcmp(e, "simt") == 0 || strcmp(e, "tc") == 0)) return false;
  return win_convT_first_applicable(g, h, ConvGeom{L.cin, L.kh, L.kw, L.stride, L.pad}, L.cout);
}

// Tensor-core transposed convolution of the conv windows (cf_window_tc.cu) for a conv layer
// where it applies, unless CF_CONV_IMPL=simt selects the CUDA-core implicit GEMM.
static bool use_conv_tc(const cf_layer& L) {
  const char* e = getenv("CF_CONV_IMPL");
  if (e && strcmp(e, "simt") == 0) return false;
  return win_convT_tc_applicable(ConvGeom{L.cin, L.kh, L.kw, L.stride, L.pad}, L.cout);
}

// The chain keeps the coefficient rows in TMEM: every substitution except the last must
// be at most 256 wide, and every layer below the bounded one must be linear.
static bool chain_applicable(const cf_network* net, const Plan& p, size_t n_below, size_t j_first = 0) {
  if (!use_chain() || p.has_conv || n_below < j_first + 1 || n_below - j_first > (size_t)kChainMaxSteps) return false;
  for (size_t j = j_first; j < n_below; ++j) {
    const cf_layer& L = net->layers[p.affine[j]];
    if (L.kind != CF_LAYER_LINEAR) return false;
    if (j + 2 <= n_below && L.n_out > 256) return false;
  }
  return true;
}

// True when some layer is bounded with the unchained steps, which materialise the
// coefficient matrices in the workspace (ping-pong A and constant buffers).
static bool needs_step_buffers(const cf_network* net, const Plan& p) {
  if (p.has_conv) return false;
  for (size_t a = 1; a <= p.affine.size(); ++a)
    if (!chain_applicable(net, p, a)) return true;
  return false;
}

// Conv networks: the substitution of whole-image coefficient windows through linear layer a
// runs on the tensor cores (the chain kernel's plain-product mode, 128 rows per tile of one
// bounded layer's rows) when some layer above it, or the property, has >= 128 rows per region.
static bool linear_window_tc(const cf_network* net, const Plan& p, size_t a) {
  if (!use_chain() || net->layers[p.affine[a]].kind != CF_LAYER_LINEAR) return false;
  for (size_t m = a + 1; m <= p.affine.size(); ++m) {
    const int64_t R = m < p.affine.size() ? net->layers[p.affine[m]].n_out : net->n_spec;
    if (R >= 128) return true;
  }
  return false;
}

static WsLayout ws_layout(const cf_network* net, const Plan& p, int64_t Bc) {
  WsLayout w;
  size_t off = 0;
  // device error word, then two CROWN branch flags per affine layer
  w.err = off; off += align256(64 + 8 * p.affine.size());
  w.wimg = off;
  w.wimg_off.assign(p.affine.size(), 0);   // 0: no image (the error word sits at offset 0)
  if (use_chain()) {  // weight images for the tensor-core chain
    for (size_t a = 0; a < p.affine.size(); ++a) {
      const cf_layer& L = net->layers[p.affine[a]];
      if (p.has_conv && !linear_window_tc(net, p, a)) continue;
      w.wimg_off[a] = off;
      off += align256(chain_wimg_bytes(L.n_out, L.n_in));
    }
  }
  const bool steps = needs_step_buffers(net, p);
  size_t a_bytes = steps ? align256((size_t)2 * Bc * p.r_max * p.n_max * sizeof(float)) : 0;
  size_t c_bytes = steps ? align256((size_t)2 * Bc * p.r_max * sizeof(float)) : 0;
  w.A[0] = off; off += a_bytes;
  w.A[1] = off; off += a_bytes;
  w.C[0] = off; off += c_bytes;
  w.C[1] = off; off += c_bytes;
  const size_t x_bytes = p.has_conv ? align256((size_t)Bc * p.win_floats * sizeof(float)) : 0;
  const size_t cw_bytes = p.has_conv ? align256((size_t)2 * Bc * p.r_max_all * sizeof(float)) : 0;
  w.X[0] = off; off += x_bytes;
  w.X[1] = off; off += x_bytes;
  if (p.has_conv) {
    w.C[0] = off; off += cw_bytes;
    w.C[1] = off; off += cw_bytes;
  }
  w.conv_wimg = off;
  for (size_t a = 0; a < p.affine.size(); ++a) {
    const cf_layer& L = net->layers[p.affine[a]];
    if (L.kind == CF_LAYER_CONV && use_conv_tc(L)) {
      const size_t b = align256(win_convT_tc_scratch_bytes(ConvGeom{L.cin, L.kh, L.kw, L.stride, L.pad}, L.cout));
      if (off < w.conv_wimg + b) off = w.conv_wimg + b;
    }
  }
  w.relu = off; off += align256((size_t)3 * Bc * p.relu_total * sizeof(float));
  // custom stop: the relaxed box of a ReLU substituted last (lower and upper rows)
  w.box = off; off += net->stop_depth > 0 ? align256((size_t)2 * Bc * p.n_max * sizeof(float)) : 0;
  w.state = off; off += align256((size_t)2 * Bc * p.N * sizeof(float));
  off += step_scratch_bytes(Bc, p.r_max);
  w.total = off;
  return w;
}

// A step with optional profiling events around it.  Algorithmic work of one step:
// 2*rows*K*N FLOPs (one useful GEMM; the sign split adds none) and bytes = A in (unless
// broadcast) + A out + W + the relaxation vectors.
static cf_status timed_step(int64_t B, int64_t R, int64_t K, int64_t N, const float* A, int64_t a_ss, int64_t a_bs,
                            int64_t a_rs, const float* c_in, int64_t c_ss, int64_t c_bs, const float* alpha,
                            const float* lam, const float* mu, const float* W, const float* bias, float* A_out,
                            float* c_out, char* scratch, cudaStream_t st) {
  const double rows = 2.0 * B * R;
  prof_step_begin(st);
  cf_status s = run_step(B, R, K, N, A, a_ss, a_bs, a_rs, c_in, c_ss, c_bs, alpha, lam, mu, W, bias, A_out, c_out,
                         scratch, st);
  double a_in = (a_ss == 0 && a_bs == 0) ? (double)R * K : (a_ss == 0 ? (double)B * R * K : rows * K);
  double bytes = 4.0 * (a_in + rows * N + (double)K * N + (alpha ? 3.0 * B * K : 0.0) + rows);
  prof_step_end(st, 2.0 * rows * K * N, bytes);
  return s;
}

static cf_status launch_chain_layer(const cf_network* net, const Plan& p, const WsLayout& w, char* ws, int64_t Bc,
                                    size_t n_below, int64_t R, const float* A0, int64_t a_bs, int64_t a_rs,
                                    const float* c0, const float* l0, const float* u0, float* out_l, float* out_u,
                                    const std::vector<float*>& ra, const std::vector<float*>& rl,
                                    const std::vector<float*>& rm, cudaStream_t st, size_t j_first = 0,
                                    int64_t ld_box = 0, const ReluOut* relu = nullptr, double* lb64 = nullptr,
                                    double* ub64 = nullptr, ChainParams* defer_to = nullptr,
                                    const ChainParams* pair_with = nullptr) {
  // defer_to: fill the parameters only, to be launched later beside an independent layer
  // (pair_with: launch this layer and that one as one grid)
  ChainParams P;
  memset(&P, 0, sizeof(P));
  if (relu) P.relu = *relu;
  P.out_l64 = lb64;
  P.out_u64 = ub64;
  P.ld_out64 = R;
  P.S = (int32_t)(n_below - j_first);
  for (int s = 0; s < P.S; ++s) {
    const size_t j = n_below - 1 - s;
    const cf_layer& L = net->layers[p.affine[j]];
    ChainStep& S = P.st[s];
    S.wimg = reinterpret_cast<const uint8_t*>(ws + w.wimg_off[j]);
    S.alpha = ra[j];
    S.lam = rl[j];
    S.mu = rm[j];
    S.bias = L.b_dev;
    S.K = L.n_out;
    S.N = L.n_in;
    chain_tile(S.N, S.tile_n, S.n_tiles);
    S.kchunks = (S.K + 31) / 32;
  }
  P.B = Bc;
  P.R = R;
  P.rows = 2 * Bc * R;
  P.A0 = A0;
  P.a_ss = 0;
  P.a_bs = a_bs;
  P.a_rs = a_rs;
  P.c0 = c0;
  P.l0 = l0;
  P.u0 = u0;
  P.n0 = net->layers[p.affine[j_first]].n_in;  // width of the box: the last step's input
  P.ld_box = ld_box ? ld_box : P.n0;
  P.out_l = out_l;
  P.out_u = out_u;
  P.ld_out = p.N;
  P.err = reinterpret_cast<int*>(ws + w.err);
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  P.a0_vec = (a_bs % 4 == 0) && (a_rs % 4 == 0) && al16(A0);
  P.box_vec = (P.n0 % 4 == 0) && (P.ld_box % 4 == 0) && al16(l0) && al16(u0);
  if (defer_to) {
    *defer_to = P;
    return CF_OK;
  }
  // algorithmic flops and bytes of a launch
  auto cost = [](const ChainParams& Q, double& flops, double& bytes) {
    const double rows = 2.0 * Q.B * Q.R;
    bytes += 4.0 * rows + 8.0 * Q.B * Q.n0;
    for (int s = 0; s < Q.S; ++s) {
      flops += 2.0 * rows * Q.st[s].K * Q.st[s].N;
      bytes += (double)Q.st[s].n_tiles * chain_wimg_bytes(Q.st[s].K, Q.st[s].N) +
               (Q.st[s].alpha ? 12.0 * Q.B * Q.st[s].K : 0);
    }
  };
  double flops = 0.0, bytes = 0.0;
  cost(P, flops, bytes);
  if (pair_with) cost(*pair_with, flops, bytes);
  prof_step_begin(st);
  cf_status s = pair_with ? chain_launch_pair(*pair_with, P, st) : chain_launch(P, st);
  prof_step_end(st, flops, bytes);
  return s;
}

// Network layers li_begin .. li_end-1 (li == n_layers: the property layer) of one chunk of
// Bc regions.  All pointers already offset to the chunk.  Layer 0 also writes the input
// columns of the state.
// dec_l / dec_u (optional, [Bc, N] in the state's layout): decision replay -- every ReLU's
// branch decisions are taken from these bounds of its input layer (cf_deeppoly_run_replay).
static cf_status run_layers(const cf_network* net, const Plan& p, int64_t Bc, const float* l0, const float* u0,
                            const float* specW, float* st_l, float* st_u, double* lb, double* ub, char* ws,
                            const WsLayout& w, cudaStream_t st, int li_begin, int li_end,
                            const float* dec_l = nullptr, const float* dec_u = nullptr, int64_t relu_stride = 0,
                            int64_t relu_off = 0) {
  (void)w.wimg;
  const int64_t N = p.N, n0 = net->n_input;
  float* Abuf[2] = {reinterpret_cast<float*>(ws + w.A[0]), reinterpret_cast<float*>(ws + w.A[1])};
  float* Cbuf[2] = {reinterpret_cast<float*>(ws + w.C[0]), reinterpret_cast<float*>(ws + w.C[1])};
  float* relu_base = reinterpret_cast<float*>(ws + w.relu);
  char* scratch = ws + w.state + align256((size_t)2 * Bc * N * sizeof(float));
  // relaxation arrays per affine index: [relu_stride, n] each (relu_stride regions, default
  // Bc), this call's regions from row relu_off
  std::vector<float*> ra(p.affine.size(), nullptr), rl(p.affine.size(), nullptr), rm(p.affine.size(), nullptr);
  {
    const int64_t rs = relu_stride > 0 ? relu_stride : Bc;
    float* q = relu_base;
    for (size_t a = 0; a < p.affine.size(); ++a) {
      if (p.relu_after[a] < 0) continue;
      int64_t n = net->layers[p.relu_after[a]].n_out;
      ra[a] = q + relu_off * n; q += rs * n;
      rl[a] = q + relu_off * n; q += rs * n;
      rm[a] = q + relu_off * n; q += rs * n;
    }
  }
  if (li_begin == 0) {
    CF_TRY(launch_copy_rows(Bc, n0, l0, n0, st_l, N, st));
    CF_TRY(launch_copy_rows(Bc, n0, u0, n0, st_u, N, st));
  }

  // bound one affine-type layer: rows R, coefficient source (A0 strides), bias c0
  auto bound_layer = [&](size_t ma, int64_t R, const float* A0, int64_t a_bs, int64_t a_rs, const float* c0,
                         int64_t col, const ReluOut* relu) -> cf_status {
    const float* cur = A0;
    int64_t ss = 0, bs = a_bs, rs = a_rs;
    const float* c = c0;
    int64_t c_ss = 0, c_bs = 0;
    int t = 0;
    for (int64_t j = (int64_t)ma - 1; j >= 0; --j, ++t) {
      const cf_layer& Lj = net->layers[p.affine[j]];
      int64_t K = Lj.n_out, Nn = Lj.n_in;
      float* Aout = Abuf[t & 1];
      float* cout_ = Cbuf[t & 1];
      CF_TRY(timed_step(Bc, R, K, Nn, cur, ss, bs, rs, c, c_ss, c_bs, ra[j], rl[j], rm[j], Lj.W_dev, Lj.b_dev, Aout,
                        cout_, scratch, st));
      cur = Aout;
      ss = Bc * R * Nn;
      bs = R * Nn;
      rs = Nn;
      c = cout_;
      c_ss = Bc * R;
      c_bs = R;
    }
    return launch_concretize(Bc, R, n0, cur, ss, bs, rs, c, c_ss, c_bs, l0, u0, st_l + col, st_u + col, N, st,
                             relu);
  };

  // custom-stop traversal (stop_depth = get_start + 1 > 0, linear chains): bounding list
  // layer li_m (affine index ma; ma == affine.size(): the property layer) substitutes list
  // layers li_m-1 .. li_stop = li_m-get_start.  Full steps (ReLU_j, affine j) for affine
  // j >= j_first; the expression is then over list layer `below`, concretised with its state
  // bounds, or, when `below` is a ReLU that is itself substituted, with the box of its
  // relaxation over the bounds of its input.
  auto bound_stopped = [&](size_t ma, int64_t R, const float* A0, int64_t a_bs, int64_t a_rs, const float* c0,
                           int64_t col, const ReluOut* relu) -> cf_status {
    const int li_m = ma == p.affine.size() ? net->n_layers : p.affine[ma];
    const int li_stop = li_m - (net->stop_depth - 1);
    size_t j_first = ma;
    while (j_first > 0 && p.affine[j_first - 1] >= li_stop) --j_first;
    const float *bl = l0, *bu = u0;
    int64_t ld = n0, nb = n0;
    if (j_first > 0) {
      const int below = (j_first < ma ? p.affine[j_first] : li_m) - 1;
      nb = net->layers[below].n_out;
      if (below >= li_stop) {
        CF_REQUIRE(p.relu_after[j_first - 1] == below, CF_ERR_UNSUPPORTED, "custom stop: layer %d", below);
        float* lo = reinterpret_cast<float*>(ws + w.box);
        float* hi = lo + Bc * nb;
        const int64_t acol = p.col[p.affine[j_first - 1]];
        CF_TRY(launch_relu_box(Bc, nb, st_l + acol, st_u + acol, N, ra[j_first - 1], rl[j_first - 1],
                               rm[j_first - 1], lo, hi, st));
        bl = lo;
        bu = hi;
        ld = nb;
      } else {
        bl = st_l + p.col[below];
        bu = st_u + p.col[below];
        ld = N;
      }
    }
    if (j_first == ma)
      return launch_concretize_box(Bc, R, nb, A0, 0, a_bs, a_rs, c0, 0, 0, bl, bu, ld, st_l + col, st_u + col, N,
                                   st, relu);
    if (chain_applicable(net, p, ma, j_first))
      return launch_chain_layer(net, p, w, ws, Bc, ma, R, A0, a_bs, a_rs, c0, bl, bu, st_l + col, st_u + col, ra,
                                rl, rm, st, j_first, ld, relu);
    const float* cur = A0;
    int64_t ss = 0, bs = a_bs, rs = a_rs;
    const float* c = c0;
    int64_t c_ss = 0, c_bs = 0;
    int t = 0;
    for (int64_t j = (int64_t)ma - 1; j >= (int64_t)j_first; --j, ++t) {
      const cf_layer& Lj = net->layers[p.affine[j]];
      const int64_t K = Lj.n_out, Nn = Lj.n_in;
      float* Aout = Abuf[t & 1];
      float* cout_ = Cbuf[t & 1];
      CF_TRY(timed_step(Bc, R, K, Nn, cur, ss, bs, rs, c, c_ss, c_bs, ra[j], rl[j], rm[j], Lj.W_dev, Lj.b_dev, Aout,
                        cout_, scratch, st));
      cur = Aout;
      ss = Bc * R * Nn;
      bs = R * Nn;
      rs = Nn;
      c = cout_;
      c_ss = Bc * R;
      c_bs = R;
    }
    return launch_concretize_box(Bc, R, nb, cur, ss, bs, rs, c, c_ss, c_bs, bl, bu, ld, st_l + col, st_u + col, N,
                                 st, relu);
  };

  // receptive-field windows (conv networks): bound layer a (a == affine.size(): property)
  float* Xbuf[2] = {reinterpret_cast<float*>(ws + w.X[0]), reinterpret_cast<float*>(ws + w.X[1])};
  auto bound_window = [&](size_t a, int64_t col) -> cf_status {
    const bool spec = a == p.affine.size();
    if (!spec && a == 0 && net->layers[p.affine[0]].kind == CF_LAYER_CONV)
      // the first layer's rows concretise against the input box with no substitution: the
      // interval convolution of the box (the input columns of the state), no window built
      return launch_ibp_conv_state(Bc, net->layers[p.affine[0]], st_l, st_u, N, st_l + col, st_u + col, N, st);
    std::vector<WinGeom> gs;
    window_chain(net, p, a, gs);
    RowGeom rg;
    rg.B = Bc;
    rg.R = window_rows(net, p, a);
    const Img oimg = spec ? Img{net->n_spec, 1, 1} : p.out_img[a];
    rg.Hm = oimg.H;
    rg.Wm = oimg.W;
    const bool conv_m = !spec && net->layers[p.affine[a]].kind == CF_LAYER_CONV;
    const float* Wm = spec ? specW : net->layers[p.affine[a]].W_dev;
    const int64_t w_bs = spec ? rg.R * p.n_out_last : 0;
    float* X = Xbuf[0];
    float* Y = Xbuf[1];
    float* c = Cbuf[0];
    float* c2 = Cbuf[1];
    CF_TRY(win_init(rg, gs[0], Wm, w_bs, conv_m, X, st));
    CF_TRY(win_row_bias(rg, spec ? nullptr : net->layers[p.affine[a]].b_dev, conv_m, c, st));
    for (int64_t j = (int64_t)a - 1, k = 0; j >= 0; --j, ++k) {
      const cf_layer& Lj = net->layers[p.affine[j]];
      const WinGeom& g = gs[k];
      const WinGeom& h = gs[k + 1];
      // the ReLU window pass is memory-bound: the window read and written, the relaxation of the
      // level read once per region
      prof_mem_begin(st);
      CF_TRY(win_relu_bias(rg, g, X, c, Bc * rg.R, rg.R, ra[j], rl[j], rm[j], Lj.b_dev, c2, st));
      prof_mem_end(st, 8.0 * 2 * Bc * rg.R * g.C * g.Ph * g.Pw + 12.0 * Bc * g.C * g.H * g.W);
      prof_step_begin(st);
      const double rows = 2.0 * Bc * rg.R;
      const double macs = Lj.kind == CF_LAYER_CONV ? (double)h.C * h.Ph * h.Pw * g.C * Lj.kh * Lj.kw /
                                                         ((double)Lj.stride * Lj.stride)
                                                   : (double)Lj.n_out * Lj.n_in;
      if (j == 0 && Lj.kind == CF_LAYER_CONV && use_conv_first(g, h, Lj)) {
        // the last substitution, fused with the concretisation (the input-level window is not stored)
        ConvGeom cv{Lj.cin, Lj.kh, Lj.kw, Lj.stride, Lj.pad};
        CF_TRY(win_convT_first(rg, g, h, cv, Lj.cout, X, Lj.W_dev, c2, l0, u0, st_l + col, st_u + col, N, st));
        prof_step_end(st, 2.0 * rows * macs, 4.0 * rows * ((double)g.C * g.Ph * g.Pw * 2));
        return CF_OK;
      }
      if (Lj.kind == CF_LAYER_CONV) {
        ConvGeom cv{Lj.cin, Lj.kh, Lj.kw, Lj.stride, Lj.pad};
        if (use_conv_tc(Lj))
          CF_TRY(win_convT_tc(rg, g, h, cv, Lj.cout, X, Lj.W_dev, Y, reinterpret_cast<uint8_t*>(ws + w.conv_wimg),
                              reinterpret_cast<int*>(ws + w.err), st));
        else
          CF_TRY(win_convT(rg, g, h, cv, X, Lj.W_dev, Y, st));
      } else if (w.wimg_off[j] != 0 && rg.R >= 128) {
        // the rows times the layer's weights on the tensor cores: the chain kernel's plain
        // product (one step, no relaxation, no column sums), bound x region as its regions
        const int64_t K = Lj.n_out, Nn = Lj.n_in;
        ChainParams P;
        memset(&P, 0, sizeof(P));
        P.S = 1;
        ChainStep& S = P.st[0];
        S.wimg = reinterpret_cast<const uint8_t*>(ws + w.wimg_off[j]);
        S.bias = Lj.b_dev;
        S.K = (int32_t)K;
        S.N = (int32_t)Nn;
        chain_tile(S.N, S.tile_n, S.n_tiles);
        S.kchunks = (S.K + 31) / 32;
        P.B = 2 * Bc;
        P.R = rg.R;
        P.rows = 2 * Bc * rg.R;
        P.A0 = X;
        P.a_bs = rg.R * K;
        P.a_rs = K;
        P.n0 = Nn;
        P.ld_box = Nn;
        P.err = reinterpret_cast<int*>(ws + w.err);
        P.a0_vec = K % 4 == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0;
        P.zono = 1;
        P.zout = Y;
        P.zo_bs = rg.R * Nn;
        CF_TRY(chain_launch(P, st));
      } else {
        const int64_t K = Lj.n_out, Nn = Lj.n_in;
        CF_TRY(launch_step_gemm_simt(Bc, rg.R, K, Nn, X, Bc * rg.R * K, rg.R * K, K, nullptr, nullptr, Lj.W_dev, Y,
                                     st));
      }
      prof_step_end(st, 2.0 * rows * macs, 4.0 * rows * ((double)g.C * g.Ph * g.Pw * 2 + (double)h.C * h.Ph * h.Pw));
      float* tX = X;
      X = Y;
      Y = tX;
      float* tc = c;
      c = c2;
      c2 = tc;
    }
    return win_concretize(rg, gs.back(), X, c, l0, u0, st_l + col, st_u + col, N, st);
  };

  // The last affine layer (no ReLU above it) and the property rows need nothing from each
  // other -- the property substitutes through that layer's weights, not its bounds -- so
  // when both go through the chain they are launched as one grid: each alone fills only
  // 2*B*R/128 CTAs (40 and 36 for 256 regions of a 10-output net), a quarter of the SMs.
  const size_t last = p.affine.size() - 1;
  const auto in_call = [&](int li) { return li >= li_begin && li < li_end; };
  const bool pair_last = p.affine.size() >= 2 && !p.has_conv && net->stop_depth == 0 && !is_interval_layers(net) &&
                         net->relaxation != CF_RELAX_CROWN && in_call(p.affine[last]) &&
                         p.relu_after[last] < 0 && in_call(net->n_layers) &&
                         chain_applicable(net, p, last) && chain_applicable(net, p, p.affine.size());
  ChainParams last_params;

  for (size_t a = 0; a < p.affine.size(); ++a) {
    const cf_layer& L = net->layers[p.affine[a]];
    int64_t col = p.col[p.affine[a]];
    const bool affine_here = p.affine[a] >= li_begin && p.affine[a] < li_end;
    const bool relu_here = p.relu_after[a] >= li_begin && p.relu_after[a] < li_end;
    // DeepPoly's relaxation of the ReLU above layer a, handed to the launch that bounds layer
    // a where that launch can apply it (it holds both bounds of a neuron, or relaxes the
    // layer right after it)
    ReluOut ro;
    const ReluOut* fuse = nullptr;
    if (affine_here && relu_here && net->relaxation != CF_RELAX_CROWN) {
      const int64_t rcol = p.col[p.relu_after[a]];
      ro = relu_out(net->layers[p.relu_after[a]].n_out, st_l + rcol, st_u + rcol, N, ra[a], rl[a], rm[a],
                    is_strict_relu(net), dec_l ? dec_l + col : nullptr, dec_u ? dec_u + col : nullptr, N);
      fuse = &ro;
    }
    bool relaxed = false;
    if (affine_here) {
      if (is_interval_layers(net)) {
        // crownibp.cf: the interval bound over the previous layer's state columns (the
        // input's columns start at 0)
        const int64_t in_col = p.affine[a] == 0 ? 0 : p.col[p.affine[a] - 1];
        if (L.kind == CF_LAYER_CONV)
          CF_TRY(launch_ibp_conv_state(Bc, L, st_l + in_col, st_u + in_col, N, st_l + col, st_u + col, N, st));
        else {
          CF_TRY(launch_concretize_box(Bc, L.n_out, L.n_in, L.W_dev, 0, 0, L.n_in, L.b_dev, 0, 0, st_l + in_col,
                                       st_u + in_col, N, st_l + col, st_u + col, N, st, fuse));
          relaxed = fuse != nullptr;
        }
      } else if (net->stop_depth > 0) {
        CF_TRY(bound_stopped(a, L.n_out, L.W_dev, 0, L.n_in, L.b_dev, col, fuse));
        relaxed = fuse != nullptr;
      } else if (p.has_conv) {
        CF_TRY(bound_window(a, col));
      } else if (chain_applicable(net, p, a)) {
        CF_TRY(launch_chain_layer(net, p, w, ws, Bc, a, L.n_out, L.W_dev, 0, L.n_in, L.b_dev, l0, u0, st_l + col,
                                  st_u + col, ra, rl, rm, st, 0, 0, fuse, nullptr, nullptr,
                                  pair_last && a == last ? &last_params : nullptr));
        relaxed = fuse != nullptr;
      } else {
        CF_TRY(bound_layer(a, L.n_out, L.W_dev, 0, L.n_in, L.b_dev, col, fuse));
        relaxed = fuse != nullptr;
      }
    }
    if (relu_here && !relaxed) {
      const cf_layer& Rl = net->layers[p.relu_after[a]];
      int64_t rcol = p.col[p.relu_after[a]];
      if (net->relaxation == CF_RELAX_CROWN) {
        int* err = reinterpret_cast<int*>(ws + w.err);
        CF_TRY(launch_crown_relax(Bc, Rl.n_out, st_l + col, st_u + col, N, st_l + rcol, st_u + rcol, N, ra[a],
                                  rl[a], rm[a], err + 16 + 2 * a, err, st));
      } else {
        CF_TRY(launch_relu_relax(Bc, Rl.n_out, st_l + col, st_u + col, N, st_l + rcol, st_u + rcol, N, ra[a],
                                 rl[a], rm[a], st, is_strict_relu(net),
                                 dec_l ? dec_l + col : nullptr, dec_u ? dec_u + col : nullptr));
      }
    }
  }
  if (net->n_layers < li_begin || net->n_layers >= li_end) return CF_OK;
  // property layer: per-region matrix [Bc, n_spec, n_out_last], zero bias
  if (net->stop_depth > 0) {
    const int64_t R = net->n_spec, K = p.n_out_last;
    CF_TRY(bound_stopped(p.affine.size(), R, specW, R * K, K, nullptr, p.spec_col, nullptr));
    CF_TRY(launch_to_f64(Bc, R, st_l + p.spec_col, st_u + p.spec_col, N, lb, ub, st));
  } else if (p.has_conv) {
    const int64_t R = net->n_spec;
    CF_TRY(bound_window(p.affine.size(), p.spec_col));
    CF_TRY(launch_to_f64(Bc, R, st_l + p.spec_col, st_u + p.spec_col, N, lb, ub, st));
  } else if (chain_applicable(net, p, p.affine.size())) {
    // the drain also writes the float64 bounds
    const int64_t R = net->n_spec, K = p.n_out_last;
    CF_TRY(launch_chain_layer(net, p, w, ws, Bc, p.affine.size(), R, specW, R * K, K, nullptr, l0, u0,
                              st_l + p.spec_col, st_u + p.spec_col, ra, rl, rm, st, 0, 0, nullptr, lb, ub, nullptr,
                              pair_last ? &last_params : nullptr));
  } else {
    const int64_t R = net->n_spec, K = p.n_out_last;
    // treat it as affine index affine.size(): substitutes every affine layer below it
    const float* cur = specW;
    int64_t ss = 0, bs = R * K, rs = K;
    const float* c = nullptr;
    int64_t c_ss = 0, c_bs = 0;
    int t = 0;
    for (int64_t j = (int64_t)p.affine.size() - 1; j >= 0; --j, ++t) {
      const cf_layer& Lj = net->layers[p.affine[j]];
      int64_t Kj = Lj.n_out, Nn = Lj.n_in;
      float* Aout = Abuf[t & 1];
      float* cout_ = Cbuf[t & 1];
      CF_TRY(timed_step(Bc, R, Kj, Nn, cur, ss, bs, rs, c, c_ss, c_bs, ra[j], rl[j], rm[j], Lj.W_dev, Lj.b_dev,
                        Aout, cout_, scratch, st));
      cur = Aout;
      ss = Bc * R * Nn;
      bs = R * Nn;
      rs = Nn;
      c = cout_;
      c_ss = Bc * R;
      c_bs = R;
    }
    CF_TRY(launch_concretize(Bc, R, n0, cur, ss, bs, rs, c, c_ss, c_bs, l0, u0, st_l + p.spec_col,
                             st_u + p.spec_col, N, st));
    CF_TRY(launch_to_f64(Bc, R, st_l + p.spec_col, st_u + p.spec_col, N, lb, ub, st));
  }
  return CF_OK;
}

}  // namespace cf

using namespace cf;

extern "C" int64_t cf_network_neurons(const cf_network* net) {
  Plan p;
  if (make_plan(net, p) != CF_OK) return -1;
  return p.N;
}

extern "C" size_t cf_deeppoly_workspace_bytes(const cf_network* net, int64_t chunk) {
  Plan p;
  if (make_plan(net, p) != CF_OK || chunk < 1) return 0;
  if (is_forward(net)) return forward_workspace_bytes(net, p, chunk);
  return ws_layout(net, p, chunk).total;
}

constexpr int kMaxLanes = 4;
// Side stream i (< kMaxLanes - 1) per device for the region lanes of a chained pass (created
// once, never destroyed: they live as long as the library).
static cudaStream_t lane_stream(int i) {
  static std::mutex mu;
  static cudaStream_t streams[64][kMaxLanes - 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!streams[dev][i] && cudaStreamCreateWithFlags(&streams[dev][i], cudaStreamNonBlocking) != cudaSuccess)
    streams[dev][i] = nullptr;
  return streams[dev][i];
}

// Region lanes: when every layer of a whole DeepPoly pass after the first is bounded by the
// chain kernel and one hidden layer's launch over the nb regions of a chunk spans at least
// two waves of CTAs, the chunk's regions are split into lanes (consecutive region ranges)
// that run the pass on separate streams.  Their launches need nothing from each other, so
// the CTAs of one lane fill the SMs while the last, partial wave of another lane's launch
// drains (a launch of 800 tiles on 148 SMs leaves 60% of them idle for its last wave).
// Returns the number of lanes: 1 (no split), else CF_CHAIN_LANES (1..kMaxLanes) or 2.
static int use_lanes(const cf_network* net, const Plan& p, int64_t nb) {
  int want = 2;
  if (const char* e = getenv("CF_CHAIN_LANES")) {
    want = atoi(e);
    if (want < 1) want = 1;
    if (want > kMaxLanes) want = kMaxLanes;
  }
  if (want == 1) return 1;
  if (!use_chain() || p.has_conv || net->stop_depth != 0 || is_interval_layers(net) || p.affine.size() < 2)
    return 1;
  if (net->relaxation != CF_RELAX_DEEPPOLY && net->relaxation != CF_RELAX_DEEPPOLY_STRICT) return 1;
  for (size_t a = 1; a <= p.affine.size(); ++a)
    if (!chain_applicable(net, p, a)) return 1;
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  }
  int64_t widest = 0;
  for (size_t a = 0; a + 1 < p.affine.size(); ++a)
    widest = net->layers[p.affine[a]].n_out > widest ? net->layers[p.affine[a]].n_out : widest;
  if (ceil_div(nb * widest, 64) < 2 * (int64_t)sms || nb < want) return 1;
  return want;
}

static cf_status deeppoly_run(const cf_network* net, int64_t B, const float* l0, const float* u0,
                              const float* specW, float* state_l, float* state_u, double* lb, double* ub,
                              void* workspace, size_t ws_bytes, void* stream, const float* dec_l,
                              const float* dec_u) {
  Plan p;
  CF_TRY(make_plan(net, p));
  CF_REQUIRE(B >= 0, CF_ERR_SHAPE, "B < 0");
  if (B == 0) return CF_OK;
  CF_REQUIRE(l0 && u0 && specW && lb && ub && workspace, CF_ERR_NULL, "deeppoly_run: NULL argument");
  if (is_forward(net))
    return forward_run(net, p, B, l0, u0, specW, state_l, state_u, lb, ub, workspace, ws_bytes, as_stream(stream));
  // largest chunk that fits the workspace
  size_t base = ws_layout(net, p, 1).total;
  CF_REQUIRE(ws_bytes >= base, CF_ERR_WORKSPACE, "workspace %zu < %zu bytes needed for one region", ws_bytes, base);
  int64_t lo = 1, hi = B;
  while (lo < hi) {
    int64_t mid = (lo + hi + 1) / 2;
    if (ws_layout(net, p, mid).total <= ws_bytes) lo = mid;
    else hi = mid - 1;
  }
  const int64_t Bc = lo;
  // CROWN's ReLU branch is decided over the whole batch: one chunk only
  CF_REQUIRE(net->relaxation != CF_RELAX_CROWN || Bc == B, CF_ERR_WORKSPACE,
             "CROWN decides each ReLU branch over the whole batch: workspace %zu holds %lld of %lld regions "
             "(cf_deeppoly_workspace_bytes(net, B) = %zu)", ws_bytes, (long long)Bc, (long long)B,
             ws_layout(net, p, B).total);
  const WsLayout w = ws_layout(net, p, Bc);
  char* ws = static_cast<char*>(workspace);
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(ws + w.err, 0, w.wimg - w.err, st) != cudaSuccess) {
    set_error("deeppoly_run: cudaMemsetAsync failed");
    return CF_ERR_CUDA;
  }
  if (use_chain()) {
    std::vector<const float*> Wl;
    std::vector<int> Kl, Nl;
    std::vector<uint8_t*> img;
    for (size_t a = 0; a < p.affine.size(); ++a) {
      const cf_layer& L = net->layers[p.affine[a]];
      if (w.wimg_off[a] == 0) continue;
      Wl.push_back(L.W_dev);
      Kl.push_back(L.n_out);
      Nl.push_back(L.n_in);
      img.push_back(reinterpret_cast<uint8_t*>(ws + w.wimg_off[a]));
    }
    if (!Wl.empty())
      CF_TRY(chain_prep_weights_batch(Wl.data(), Kl.data(), Nl.data(), img.data(), (int)Wl.size(), st));
  }
  const int64_t N = p.N, n0 = net->n_input, ns = net->n_spec;
  for (int64_t b0 = 0; b0 < B; b0 += Bc) {
    int64_t nb = (B - b0 < Bc) ? (B - b0) : Bc;
    float* sl = state_l ? state_l + b0 * N : reinterpret_cast<float*>(ws + w.state);
    float* su = state_u ? state_u + b0 * N : reinterpret_cast<float*>(ws + w.state) + Bc * N;
    // lane x: regions [b0 + off, b0 + off + n) of the chunk, rows off.. of the workspace arrays
    auto lane = [&](int64_t off, int64_t n, cudaStream_t s) {
      const int64_t b = b0 + off;
      return run_layers(net, p, n, l0 + b * n0, u0 + b * n0, specW + b * ns * p.n_out_last, sl + off * N,
                        su + off * N, lb + b * ns, ub + b * ns, ws, w, s, 0, net->n_layers + 1,
                        dec_l ? dec_l + b * N : nullptr, dec_u ? dec_u + b * N : nullptr, Bc, off);
    };
    int nl = use_lanes(net, p, nb);
    cudaStream_t side[kMaxLanes - 1] = {};
    cudaEvent_t fork = nullptr, join[kMaxLanes - 1] = {};
    bool ok = nl > 1 && cudaEventCreateWithFlags(&fork, cudaEventDisableTiming) == cudaSuccess;
    for (int i = 0; ok && i + 1 < nl; ++i)
      ok = (side[i] = lane_stream(i)) != nullptr &&
           cudaEventCreateWithFlags(&join[i], cudaEventDisableTiming) == cudaSuccess;
    if (!ok) {
      if (fork) cudaEventDestroy(fork);
      for (cudaEvent_t e : join)
        if (e) cudaEventDestroy(e);
      cudaGetLastError();
      CF_TRY(lane(0, nb, st));
      continue;
    }
    // fork: the side lanes start after everything queued on st so far; join: st continues
    // after every lane, also when a lane failed to queue
    prof_span_begin(st);
    cudaEventRecord(fork, st);
    for (int i = 0; i + 1 < nl; ++i) cudaStreamWaitEvent(side[i], fork, 0);
    cf_status s = CF_OK;
    for (int i = 0; i < nl && s == CF_OK; ++i) {
      const int64_t from = nb * i / nl, to = nb * (i + 1) / nl;
      s = lane(from, to - from, i == 0 ? st : side[i - 1]);
    }
    for (int i = 0; i + 1 < nl; ++i) {
      cudaEventRecord(join[i], side[i]);
      cudaStreamWaitEvent(st, join[i], 0);
    }
    prof_span_end(st);
    cudaEventDestroy(fork);
    for (int i = 0; i + 1 < nl; ++i) cudaEventDestroy(join[i]);
    CF_TRY(s);
  }
  return CF_OK;
}

extern "C" cf_status cf_deeppoly_run(const cf_network* net, int64_t B, const float* l0, const float* u0,
                                     const float* specW, float* state_l, float* state_u, double* lb, double* ub,
                                     void* workspace, size_t ws_bytes, void* stream) {
  clear_error();
  CF_INJECT("deeppoly_run");
  return deeppoly_run(net, B, l0, u0, specW, state_l, state_u, lb, ub, workspace, ws_bytes, stream, nullptr,
                      nullptr);
}

extern "C" cf_status cf_deeppoly_run_replay(const cf_network* net, int64_t B, const float* l0, const float* u0,
                                            const float* specW, const float* dec_l, const float* dec_u,
                                            float* state_l, float* state_u, double* lb, double* ub,
                                            void* workspace, size_t ws_bytes, void* stream) {
  clear_error();
  CF_INJECT("deeppoly_run_replay");
  CF_REQUIRE(net && (net->relaxation == CF_RELAX_DEEPPOLY || net->relaxation == CF_RELAX_DEEPPOLY_STRICT),
             CF_ERR_UNSUPPORTED, "deeppoly_run_replay: DeepPoly relaxations only");
  CF_REQUIRE(dec_l && dec_u, CF_ERR_NULL, "deeppoly_run_replay: NULL decision bounds");
  return deeppoly_run(net, B, l0, u0, specW, state_l, state_u, lb, ub, workspace, ws_bytes, stream, dec_l, dec_u);
}

extern "C" cf_status cf_deeppoly_layer(const cf_network* net, int32_t layer, int64_t B, const float* l0,
                                       const float* u0, const float* specW, float* state_l, float* state_u,
                                       double* lb, double* ub, void* workspace, size_t ws_bytes, void* stream) {
  clear_error();
  CF_INJECT("deeppoly_layer");
  Plan p;
  CF_TRY(make_plan(net, p));
  CF_REQUIRE(layer >= 0 && layer <= net->n_layers, CF_ERR_SHAPE, "layer %d of a %d-layer network", layer,
             net->n_layers);
  CF_REQUIRE(B >= 0, CF_ERR_SHAPE, "B < 0");
  if (B == 0) return CF_OK;
  CF_REQUIRE(l0 && u0 && specW && state_l && state_u && lb && ub && workspace, CF_ERR_NULL,
             "deeppoly_layer: NULL argument");
  cudaStream_t st = as_stream(stream);
  if (is_forward(net))
    return forward_layer(net, p, layer, B, l0, u0, specW, state_l, state_u, lb, ub, workspace, ws_bytes, st);
  const WsLayout w = ws_layout(net, p, B);
  CF_REQUIRE(ws_bytes >= w.total, CF_ERR_WORKSPACE,
             "per-layer runs keep the whole batch: workspace %zu < %zu bytes (cf_deeppoly_workspace_bytes(net, B))",
             ws_bytes, w.total);
  char* ws = static_cast<char*>(workspace);
  if (layer == 0 && cudaMemsetAsync(ws + w.err, 0, w.wimg - w.err, st) != cudaSuccess) {
    set_error("deeppoly_layer: cudaMemsetAsync failed");
    return CF_ERR_CUDA;
  }
  if (use_chain()) {
    // the weight image of this layer (every layer of a chained net; in a conv net the linear
    // layers whose window substitutions run on the tensor cores), used by the layers above
    for (size_t a = 0; a < p.affine.size(); ++a) {
      const cf_layer& L = net->layers[p.affine[a]];
      if (p.affine[a] == layer && w.wimg_off[a] != 0)
        CF_TRY(chain_prep_weights(L.W_dev, L.n_out, L.n_in, reinterpret_cast<uint8_t*>(ws + w.wimg_off[a]), st));
    }
  }
  return run_layers(net, p, B, l0, u0, specW, state_l, state_u, lb, ub, ws, w, st, layer, layer + 1);
}

extern "C" cf_status cf_deeppoly_check(const void* workspace, void* stream) {
  clear_error();
  CF_REQUIRE(workspace, CF_ERR_NULL, "deeppoly_check: NULL workspace");
  int h = 0;
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_error("deeppoly_check: %s", cudaGetErrorString(e));
    return CF_ERR_CUDA;
  }
  if (h == kCrownCrossingSite) {
    set_error("CROWN: every neuron of a ReLU layer crosses zero in every region (the all-crossing branch of "
              "crown.cf's ReLU, whose U polyexps mix layers); this branch is not run on the GPU");
    return CF_ERR_UNSUPPORTED;
  }
  if (h != 0) {
    set_error("a bounded device wait gave up (site %d)", h);
    return CF_ERR_TIMEOUT;
  }
  return CF_OK;
}

extern "C" const char* cf_last_error(void) { return g_err; }
extern "C" const char* cf_version(void) { return "cfgpu 0.1 (sm_100a)"; }
