// Receptive-field window backsubstitution (cf_window.cu): geometry and launchers.
#pragma once
#include "cf_common.cuh"

namespace cf {

// Rows 2*B*R of a bounded layer whose output image is (., Hm, Wm): row (s, b, i) with
// i = co*Hm*Wm + oy*Wm + ox.
struct RowGeom {
  int64_t B, R;
  int32_t Hm, Wm;
};

// A window at one level: image (C, H, W) of that level, window Ph x Pw over all C
// channels, origin (oy*sig_h - pi_h, ox*sig_w - pi_w).  Element order (c, u, v).
struct WinGeom {
  int32_t C, H, W, Ph, Pw, sig_h, sig_w, pi_h, pi_w;
};

// The convolution substituted by k_win_convT_gemm: weights [Cout, cin, kh, kw], stride s, pad.
struct ConvGeom {
  int32_t cin, kh, kw, s, pad;
};

cf_status win_init(const RowGeom& rg, const WinGeom& g, const float* W, int64_t w_bs, bool conv, float* out,
                   cudaStream_t st);
cf_status win_row_bias(const RowGeom& rg, const float* bias, bool conv, float* c_out, cudaStream_t st);
cf_status win_relu_bias(const RowGeom& rg, const WinGeom& g, float* A, const float* c_in, int64_t c_ss, int64_t c_bs,
                        const float* alpha, const float* lam, const float* mu, const float* bias, float* c_out,
                        cudaStream_t st);
// One stride phase of the transposed convolution (k_win_convT_gemm): output-window rows
// u' = u0 + iy*s (iy < ny), columns v' = v0 + ix*s (ix < nx), taps ky = py + ty*s (ty < tyn),
// kx = px + tx*s (tx < txn), input-window index u = q0y + iy - ty, v = q0x + ix - tx.
struct ConvPhase {
  int32_t py, px, ny, nx, tyn, txn, u0, v0, q0y, q0x;
};

cf_status win_convT(const RowGeom& rg, const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, const float* in,
                    const float* W, float* out, cudaStream_t st);
// The same transposed convolution as tcgen05 implicit GEMMs (cf_window_tc.cu), all stride
// phases in one launch: applicable when a phase's weight image (Cin padded to 16 columns)
// fits in shared memory and the stride is at most 3; `scratch` holds every phase's weight
// image (win_convT_tc_scratch_bytes), `err` is the device error word.
bool win_convT_tc_applicable(const ConvGeom& cv, int cout);
size_t win_convT_tc_scratch_bytes(const ConvGeom& cv, int cout);
cf_status win_convT_tc(const RowGeom& rg, const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, int cout,
                       const float* in, const float* W, float* out, uint8_t* scratch, int* err, cudaStream_t st);
// The last substitution of a traversal (into the network input) through a stride-1 conv
// layer with at most 4 input channels, fused with the concretisation: writes the bounds of
// rows (s, b, i) to out_l / out_u[b*ld_out + i] = c + box sum of the input-level window.
bool win_convT_first_applicable(const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, int cout);
cf_status win_convT_first(const RowGeom& rg, const WinGeom& gi, const WinGeom& go, const ConvGeom& cv, int cout,
                          const float* in, const float* W, const float* c, const float* l0, const float* u0,
                          float* out_l, float* out_u, int64_t ld_out, cudaStream_t st);
cf_status win_concretize(const RowGeom& rg, const WinGeom& g, const float* A, const float* c, const float* l0,
                         const float* u0, float* out_l, float* out_u, int64_t ld_out, cudaStream_t st);

}  // namespace cf
