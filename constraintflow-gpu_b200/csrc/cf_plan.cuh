// Network plan shared by the backsubstitution driver (cf_engine.cu) and the forward
// drivers of the zonotope and interval programs (cf_zono.cu).
#pragma once
#include <vector>

#include "cf_common.cuh"

namespace cf {

struct Img {
  int32_t C, H, W;
};

struct Plan {
  std::vector<int> affine;      // layer indices of affine layers, in order
  std::vector<Img> in_img, out_img;  // per affine index: input / output image (linear: (n,1,1) out)
  bool has_conv = false;
  int64_t win_floats = 0;       // window path: per region, max rows*window floats of one buffer
  std::vector<int> relu_after;  // per affine index: layer index of the ReLU that follows, or -1
  std::vector<int64_t> col;     // per layer: first state column (input = 0)
  int64_t n_out_last = 0;       // width of the last affine layer (property matrix columns)
  int64_t N = 0;                // total neurons incl. input and property rows
  int64_t spec_col = 0;
  int64_t r_max = 0, k_max = 0, n_max = 0, relu_total = 0;
  int64_t r_max_all = 0;        // rows of the widest bounded layer, first layer and property included
};

// Validates a chain network (Input -> [Linear|Conv, ReLU]* ... -> affine) and lays out its
// neuron columns.
cf_status make_plan(const cf_network* net, Plan& p);

inline bool is_forward(const cf_network* net) {
  return net->relaxation == CF_RELAX_ZONO || net->relaxation == CF_RELAX_IBP;
}

// crownibp.cf's interval layers (CF_RELAX_CROWNIBP, and its strict variant for zid.cf)
inline bool is_interval_layers(const cf_network* net) {
  return net->relaxation == CF_RELAX_CROWNIBP || net->relaxation == CF_RELAX_CROWNIBP_STRICT;
}

// DeepPoly's lower ReLU slope is 1 where l + u > 0 (instead of >= 0)
inline bool is_strict_relu(const cf_network* net) {
  return net->relaxation == CF_RELAX_DEEPPOLY_STRICT || net->relaxation == CF_RELAX_CROWNIBP_STRICT;
}

// Forward programs (zono.cf, ibp.cf): workspace for `chunk` regions, and the whole pass.
size_t forward_workspace_bytes(const cf_network* net, const Plan& p, int64_t chunk);
cf_status forward_run(const cf_network* net, const Plan& p, int64_t B, const float* l0, const float* u0,
                      const float* specW, float* state_l, float* state_u, double* lb, double* ub, void* ws,
                      size_t ws_bytes, cudaStream_t st);
// One layer of a forward pass (layer == n_layers: the property layer); the workspace holds
// the whole batch and the layers before it ran on it.
cf_status forward_layer(const cf_network* net, const Plan& p, int layer, int64_t B, const float* l0,
                        const float* u0, const float* specW, float* state_l, float* state_u, double* lb, double* ub,
                        void* ws, size_t ws_bytes, cudaStream_t st);

}  // namespace cf
