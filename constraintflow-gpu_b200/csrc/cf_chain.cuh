// Chained tensor-core backsubstitution (cf_chain.cu): parameters and host entry points.
#pragma once
#include "cf_common.cuh"
#include "cf_relax.cuh"

namespace cf {

constexpr int kAStages = 2;  // shared-memory stages of the transformed A operand (32 KB each)
constexpr int kWStages = 2;  // shared-memory stages of weight chunks (2 x tile_n x 128 bytes each)
constexpr int kChainMaxSteps = 24;  // substitutions per launch (affine layers below the bounded one)
// Relaxation vectors staged in shared memory per step: alpha, lambda, mu rows (kCoefRow floats
// each) of up to kCoefSlots (bound, region) pairs, then the layer bias; two step buffers.
constexpr int kCoefSlots = 2;
constexpr int kCoefRow = 256;
constexpr int kCoefBufFloats = (kCoefSlots * 3 + 1) * kCoefRow;

// One substitution: ReLU_j (if alpha != nullptr) then affine layer j, W_j [K, N].
struct ChainStep {
  const uint8_t* wimg;  // chain_prep_weights image of W_j
  const float* alpha;   // [B, K] relaxation of the ReLU after layer j, or nullptr
  const float* lam;
  const float* mu;
  const float* bias;    // [K] bias of layer j
  int32_t K, N, tile_n, n_tiles, kchunks;
};

struct ChainParams {
  ChainStep st[kChainMaxSteps];
  int32_t S;
  // rows = 2*B*R, one per (bound, region b, row i).  Bounding mode: tile t holds the 64
  // (b, i) pairs q = 64t .. 64t+63 (q = b*R + i), TMEM lanes 0-63 their lower bounds and
  // 64-127 their upper bounds, so that both bounds of a neuron end in one CTA.  Zonotope
  // mode: row = b*R + i, 128 per tile.
  int64_t B, R, rows;
  const float* A0;                      // first coefficient rows (row (s,b,i) at s*a_ss + b*a_bs + i*a_rs)
  int64_t a_ss, a_bs, a_rs;
  const float* c0;                      // [R] constant of the bounded layer (its bias) or nullptr
  const float* l0;                      // [B, n0] box of the last step's input (rows at b*ld_box; ld_box 0: n0)
  const float* u0;
  int64_t n0;
  int64_t ld_box;
  float* out_l;                         // bound of row (0,b,i) -> out_l[b*ld_out + i]
  float* out_u;
  int64_t ld_out;
  double* out_l64;                      // optional float64 copies (the property rows):
  double* out_u64;                      //   out_l64[b*ld_out64 + i]
  int64_t ld_out64;
  ReluOut relu;                         // relu.alpha != nullptr: the ReLU above the bounded layer
                                        // is relaxed in the drain from the two new bounds
  int* err;                             // device error word (bounded-wait timeouts)
  uint32_t max_polls;                   // poll limit of every bounded wait (filled by chain_launch)
  int32_t withhold_acc;                 // failure-path test: the MMA issuer withholds the first
                                        // step's accumulator-ready arrival (filled by chain_launch)
  int32_t a0_vec, box_vec;              // 16-byte loads allowed for A0 rows / the input box
  uint32_t stage_bytes, w_lo_off;       // filled by chain_launch
  uint32_t box_smem_bytes;              // input-box staging bytes (0: read from global memory)
  int32_t coef_ok;                      // relaxation vectors may be staged in shared memory
  // Forward zonotope mode (zono != 0, one step, R >= 128, rows = B*R symbol rows of the
  // lower half only): the step's ReLU relaxation is the column scaling alpha = lam, and the
  // drain writes every row of the result to zout[b*zo_bs + i*N + n] and, per warp w = warp%4
  // and region slot (region - first region of the CTA), the column sums of the positive /
  // negative coefficients to zpos / zneg[((cta*4 + w)*2 + slot)*N + n].  No input box.
  // With zpos = zneg = null and no relaxation (alpha null) it is a plain product
  // zout = A0 rows x W, e.g. a linear substitution of whole-image coefficient windows.
  int32_t zono;
  int32_t zo_vec;                       // 16-byte stores allowed for zout rows
  float* zout;
  int64_t zo_bs;
  float* zpos;
  float* zneg;
};

// Persistent zonotope symbol-row GEMM (k_zono_persist): rows = B*E rows (b, e) of A (row
// at A + b*a_bs + e*K, K contiguous floats) times diag(lam[b]) times W^T (image of
// chain_prep_weights(W^T [K, N])), N <= 256, E >= 128.  Every 128-row tile writes its rows
// to out[b*o_bs + e*N + n] and, per TMEM lane quarter w and region slot, the column sums of
// the positive / negative coefficients to zpos / zneg[((tile*4 + w)*2 + slot)*N + n] (the
// layout of the zonotope mode of k_chain).
struct ZonoTcParams {
  const uint8_t* wimg;
  const float* lam;
  const float* A;
  int64_t a_bs;
  int32_t K, N, tile_n, kchunks;
  int64_t B, E, rows;
  float* out;
  int64_t o_bs;
  float* zpos;
  float* zneg;
  int* err;
  int32_t a_vec, lam_vec, o_vec;
  uint32_t stage_bytes, w_lo_off;  // filled by zono_tc_launch
};

cf_status zono_tc_launch(const ZonoTcParams& P, cudaStream_t st);

void chain_tile(int N, int& tile_n, int& n_tiles);
size_t chain_wimg_bytes(int K, int N);
cf_status chain_prep_weights(const float* W, int K, int N, uint8_t* img, cudaStream_t st);
// the images of n weight matrices in one launch (per group of 32)
cf_status chain_prep_weights_batch(const float* const* W, const int* K, const int* N, uint8_t* const* img, int n,
                                   cudaStream_t st);
cf_status chain_launch(const ChainParams& P, cudaStream_t st);
// Two independent bounding-mode launches as one: CTAs [0, split) run p[0], the rest p[1]
// (e.g. the output layer and the property rows, neither of which needs the other).
struct ChainPair {
  ChainParams p[2];
  int64_t split;
};
cf_status chain_launch_pair(const ChainParams& P0, const ChainParams& P1, cudaStream_t st);

}  // namespace cf
