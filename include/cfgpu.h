/*
 * cfgpu.h -- C ABI of libcfgpu.so, the B200 (sm_100a) runtime for the tensor code that
 * ConstraintFlow emits for DeepPoly-style certifiers.
 *
 * Conventions
 *   - Every pointer argument named *_dev is device memory; sizes are element counts.
 *   - All calls are stream-ordered on `stream` (a cudaStream_t passed as void*), never
 *     synchronise, never allocate or free memory, and never free caller memory.
 *     Scratch space is a caller-provided `workspace` of the size the *_workspace_bytes
 *     query returns.
 *   - Return value: cf_status (0 = CF_OK).  cf_last_error() gives a message for the
 *     last failing call on the calling host thread.
 *   - float32 everywhere (the reference forces every block to float32,
 *     constraintflow/gbcsr/sparse_block.py:141-147); final property bounds are also
 *     produced as float64 as Flow.flow returns them (constraintflow/gbcsr/
 *     sparse_tensor.py:627-654).
 *
 * The functions and the reference interface each one replaces:
 *   cf_relu_relax        generated deeppoly.Relu body (examples/compiler_examples/deeppoly.cf:20-24,41;
 *                        constraintflow/lib/llist.py:764 convert_to_poly)
 *   cf_backsub_step      one substitution iteration of the generated deeppoly.Affine while-loop:
 *                        clamp sign split (constraintflow/gbcsr/tensor_ops.py:765) + inner_prod
 *                        (tensor_ops.py:370 -> SparseTensor.matmul sparse_tensor.py:1671 ->
 *                        DenseBlock.matmul_equal_dims sparse_block.py:748) + binary add
 *                        (tensor_ops.py:163), for a ReLU layer followed by an affine layer
 *   cf_concretize        the input-layer substitution + final bound (generated Affine tail;
 *                        DenseBlock.matmul_unequal_dims sparse_block.py:964)
 *   cf_deeppoly_run      Flow.flow over a chain network (constraintflow/lib/flow_sparse.py:27-228)
 *                        with the generated deeppoly / crown transformer, or the forward flow
 *                        of zono.cf (SymExpSparse, constraintflow/lib/symexp.py:14-273;
 *                        create_Z, spec.py:106-132) and ibp.cf
 *   cf_ew_binary / cf_ew_unary / cf_ew_where / cf_ew_clamp / cf_ew_any
 *                        block kernels of the gbcsr elementwise ops: SparseBlock.binary
 *                        (sparse_block.py:181), unary_operation (:60), where_block (:104),
 *                        SparseBlock.clamp (:542), SparseTensor.any (sparse_tensor.py:1597)
 */
#ifndef CFGPU_H
#define CFGPU_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t cf_status;
enum {
  CF_OK = 0,
  CF_ERR_SHAPE = 1,        /* inconsistent sizes ("SHAPE MISMATCH", tensor_ops.py:53-77) */
  CF_ERR_UNSUPPORTED = 2,  /* layer / op combination not implemented (NotImplementedError) */
  CF_ERR_CUDA = 3,         /* a CUDA launch or runtime call failed */
  CF_ERR_TIMEOUT = 4,      /* a bounded device-side wait gave up */
  CF_ERR_NULL = 5,         /* required pointer was NULL */
  CF_ERR_WORKSPACE = 6,    /* workspace smaller than cf_deeppoly_workspace_bytes reports */
  CF_ERR_INJECTED = 7      /* host-side fault injection (env CF_FAULT=<site>) fired */
};

/* Layer kinds of a chain network (constraintflow/lib/network.py:75-87). */
enum { CF_LAYER_LINEAR = 1, CF_LAYER_CONV = 2, CF_LAYER_RELU = 3 };

/* Certifier programs the network driver runs (the ReLU transformer and traversal of
 * examples/compiler_examples/<name>.cf as the reference compiler emits them).
 *   CF_RELAX_DEEPPOLY  deeppoly.cf (and deeppoly_efficient.cf, which composes to the same
 *                      bounds): per-neuron triangle relaxation.
 *   CF_RELAX_CROWN     crown.cf: the reference lowers its tuple-valued ReLU ternary to
 *                      whole-layer branches on any() over the layer's [B, n] bounds:
 *                      any(l >= 0) -> pass-through (l' = l, u' = u, L'/U' of the affine);
 *                      else any(u <= 0) -> zero; else every neuron crosses 0 and U' is
 *                      substituted one layer deeper.  The branch couples the regions of
 *                      a batch, so cf_deeppoly_run requires the whole batch in one
 *                      workspace chunk (CF_ERR_WORKSPACE otherwise); the all-crossing
 *                      branch is not run on the GPU and cf_deeppoly_check reports it as
 *                      CF_ERR_UNSUPPORTED.
 *   CF_RELAX_ZONO      zono.cf (DeepZ): forward zonotope propagation.  The input box is one
 *                      noise symbol per input neuron (constraintflow/lib/spec.py:106-132);
 *                      an affine layer maps the symbol coefficients and concretises
 *                      l/u = c -/+ sum |coefficient|; a ReLU opens one fresh symbol per
 *                      neuron (constraintflow/lib/symexp.py:14) and its own l, u are 0.
 *                      Linear and conv layers.
 *   CF_RELAX_IBP       ibp.cf: interval bounds layer by layer (W+ l + W- u + b; ReLU
 *                      clamps), linear and conv layers.
 *   CF_RELAX_CROWNIBP  crownibp.cf: every affine layer below the property gets the
 *                      interval bound of its expression over the previous layer's l / u
 *                      (no traversal); the ReLU relaxation is DeepPoly's, from those
 *                      bounds; only the property rows are backsubstituted to the input.
 *   CF_RELAX_DEEPPOLY_STRICT  deeppoly.cf with the strict lower-slope test of the custom-stop
 *                      programs (relu_n: l + u > 0, deeppoly_custom_stop.cf:24); the
 *                      other strict comparisons there give DeepPoly's values.
 *   CF_RELAX_CROWNIBP_STRICT  CF_RELAX_CROWNIBP with that strict lower-slope test: the
 *                      interval and ReLU layers of zid.cf (relu_n: l + u > 0, zid.cf:22).
 * CF_RELAX_ZONO and CF_RELAX_IBP run forward through cf_deeppoly_run as well; their
 * regions are independent (any chunk size). */
enum {
  CF_RELAX_DEEPPOLY = 0,
  CF_RELAX_CROWN = 1,
  CF_RELAX_ZONO = 2,
  CF_RELAX_IBP = 3,
  CF_RELAX_CROWNIBP = 4,
  CF_RELAX_DEEPPOLY_STRICT = 5,
  CF_RELAX_CROWNIBP_STRICT = 6
};

/* One layer.  Linear: W_dev [n_out, n_in] row-major, b_dev [n_out].
 * Conv: W_dev [cout, cin, kh, kw], b_dev [cout]; neurons in (c, y, x) order,
 * n_in = cin*ih*iw, n_out = cout*oh*ow (constraintflow/lib/parse.py:89-126).
 * ReLU: no weights, n_in == n_out. */
typedef struct cf_layer {
  int32_t kind;
  int32_t n_in, n_out;
  int32_t cin, ih, iw, cout, oh, ow, kh, kw, stride, pad;
  const float* W_dev;
  const float* b_dev;
} cf_layer;

/* A chain network Input -> layers[0] -> ... -> layers[n_layers-1] -> property layer.
 * The property layer (y[label] - y[j], constraintflow/lib/spec.py:61-72) is given per
 * region at run time. */
typedef struct cf_network {
  int32_t n_layers;
  const cf_layer* layers;  /* host array */
  int32_t n_input;
  int32_t n_spec;          /* rows of the property layer (9 for 10 classes) */
  int32_t relaxation;      /* one of the CF_RELAX_* codes */
  int32_t stop_depth;      /* 0: every traversal reaches the input.  d > 0 (CF_RELAX_DEEPPOLY
                              or _DEEPPOLY_STRICT, linear layers): the custom-stop programs with get_start = d - 1
                              (examples/compiler_examples/deeppoly_custom_stop.cf:12-17,
                              custom_stops/): bounding list layer m substitutes list layers
                              m-1 .. m-(d-1) only and concretises the rest with the bounds
                              of the layer the expression is then over */
} cf_network;

/* Total neuron count N of the abstract state: input + every layer + property rows
 * (constraintflow/lib/parse.py:243-248). */
int64_t cf_network_neurons(const cf_network* net);

/* Workspace needed to run `chunk` regions at a time (regions beyond it are processed
 * in further chunks inside one cf_deeppoly_run call). */
size_t cf_deeppoly_workspace_bytes(const cf_network* net, int64_t chunk);

/* Whole certifier pass over B regions (the program net->relaxation names: DeepPoly /
 * CROWN backsubstitution, or the zono / ibp forward passes).
 *   l0_dev, u0_dev   [B, n_input]   normalised input box
 *   spec_W_dev       [B, n_spec, n_out(last layer)]  per-region property matrix (bias 0)
 *   state_l_dev, state_u_dev  [B, N] or NULL: every neuron's bounds in the reference's
 *                    neuron order, input columns included (abs_elem.d['l'|'u'] dense view)
 *   lb_dev, ub_dev   [B, n_spec] float64: the property bounds Flow.flow returns
 *   workspace_dev / workspace_bytes: scratch, >= cf_deeppoly_workspace_bytes(net, chunk)
 *                    for some chunk >= 1
 * A DeepPoly pass whose layers all go through the chain kernel may run half of a chunk's
 * regions on a second stream that the library owns (created once per device): it waits
 * for the work queued on `stream` before the call and `stream` waits for it before any
 * later work, so the call stays stream-ordered (and can be captured in a CUDA graph once
 * the first such call on the device, which creates that stream, has run uncaptured).
 * CF_CHAIN_LANES=1 keeps everything on `stream`. */
cf_status cf_deeppoly_run(const cf_network* net, int64_t B,
                          const float* l0_dev, const float* u0_dev, const float* spec_W_dev,
                          float* state_l_dev, float* state_u_dev,
                          double* lb_dev, double* ub_dev,
                          void* workspace_dev, size_t workspace_bytes, void* stream);

/* Decision replay, for parity testing against another implementation of the same program.
 * cf_deeppoly_run, except that every ReLU branch decision of the generated deeppoly.Relu
 * (l >= 0, u <= 0, l + u >= 0; examples/compiler_examples/deeppoly.cf:20-24) is taken from
 * the given bounds dec_l_dev / dec_u_dev [B, N] (state layout, e.g. another run's every-neuron
 * l / u) of the ReLU's input layer instead of this run's own; the relaxation's values
 * (lambda = u/(u-l), mu, l', u') still come from this run's bounds.  Two float32
 * implementations that sum in different orders can take different branches on a bound a few
 * ulps from 0, after which every later layer differs by far more than rounding; replaying
 * one side's decisions makes their bounds comparable on every layer.  CF_RELAX_DEEPPOLY and
 * CF_RELAX_DEEPPOLY_STRICT only. */
cf_status cf_deeppoly_run_replay(const cf_network* net, int64_t B,
                                 const float* l0_dev, const float* u0_dev, const float* spec_W_dev,
                                 const float* dec_l_dev, const float* dec_u_dev,
                                 float* state_l_dev, float* state_u_dev,
                                 double* lb_dev, double* ub_dev,
                                 void* workspace_dev, size_t workspace_bytes, void* stream);

/* One layer of the pass, for callers that drive the layer loop themselves as Flow.flow does
 * (constraintflow/lib/flow_sparse.py:27-228 calls the transformer once per layer; code
 * emitted by cfgpu.codegen calls this once per layer).  layer = 0 .. n_layers-1 runs that
 * network layer (an affine layer: its bounds by backsubstitution, or its zonotope / interval
 * step; a ReLU: its relaxation), layer = n_layers the property layer (lb/ub).  Layers run in
 * order 0, 1, .. on one workspace that holds the whole batch
 * (>= cf_deeppoly_workspace_bytes(net, B)); state_l / state_u are required.  The bounds
 * equal those of cf_deeppoly_run. */
cf_status cf_deeppoly_layer(const cf_network* net, int32_t layer, int64_t B,
                            const float* l0_dev, const float* u0_dev, const float* spec_W_dev,
                            float* state_l_dev, float* state_u_dev, double* lb_dev, double* ub_dev,
                            void* workspace_dev, size_t workspace_bytes, void* stream);

/* Input boundary (constraintflow/lib/spec.py:21-47, 61-72).
 * cf_input_box: l0 = (clip(X - eps, 0, 1) - mean[c]) / std[c], u0 likewise with +eps, for
 * X [B, C, HW] float32 (C mean/std values given on the host, C <= 4).
 * cf_spec_matrix: per-region property matrix W [B, n_classes-1, n_classes] with row j
 * = e_label - e_k for the k-th class k != label, from labels [B] int64. */
cf_status cf_input_box(int64_t B, int32_t C, int64_t HW, const float* X_dev, float eps,
                       const float* mean_host, const float* std_host,
                       float* l0_dev, float* u0_dev, void* stream);
cf_status cf_spec_matrix(int64_t B, int32_t n_classes, const int64_t* labels_dev, float* W_dev,
                         void* stream);

/* Profiling: while enabled (per host thread), cf_deeppoly_run records CUDA events around
 * every backsubstitution-step launch and every launch of a memory-bound kernel (ReLU
 * relaxation, concretisation, float64 conversion, weight-image preparation, zonotope
 * concretisation and ReLU) on the caller's stream and counts every kernel it launches;
 * cf_profile_collect waits for those events and returns the totals since the last
 * collect. */
typedef struct cf_profile_stats {
  int64_t kernel_launches;   /* all kernels launched by cf_deeppoly_run */
  int64_t step_launches;     /* backsubstitution steps (the dominant kernel) */
  double step_ms;            /* summed device time of the steps */
  double step_flops;         /* algorithmic FLOPs of those steps: 2*rows*K*N each */
  double step_bytes;         /* algorithmic bytes: A in + A out + W + relaxation vectors */
  int64_t mem_launches;      /* memory-bound kernel launches */
  double mem_ms;             /* their summed device time */
  double mem_bytes;          /* their algorithmic bytes (each input and output once) */
} cf_profile_stats;
cf_status cf_profile_enable(int32_t on);
cf_status cf_profile_collect(cf_profile_stats* out);

/* No counterpart in the reference.  cf_deeppoly_run for callers that cannot allocate
 * device memory (a plugin inside another framework's allocator, a service that must not
 * touch the allocator on its request path): the workspace is a fixed device array of
 * CF_STATIC_SCRATCH_BYTES inside libcfgpu, held on every GPU that loads the library
 * until exit.  The caller passes inputs and outputs as for cf_deeppoly_run.  The first
 * call on a device looks the array up (cudaGetSymbolAddress with that device current):
 * make it before any stream capture.  All calls share the array, so calls that overlap
 * on the GPU race and must be serialised by the caller.  A network whose scratch for one
 * region exceeds the array is rejected with CF_ERR_WORKSPACE; larger DeepPoly, zono and ibp
 * batches are run in region chunks that fit.  CROWN (CF_RELAX_CROWN) decides each ReLU branch
 * over the whole batch, so its whole batch must fit the array in one chunk
 * (cf_deeppoly_workspace_bytes(net, B) <= CF_STATIC_SCRATCH_BYTES); otherwise the call
 * returns CF_ERR_WORKSPACE.  cf_deeppoly_check_static reports the device status of the
 * last call on the current device. */
#define CF_STATIC_SCRATCH_BYTES (32u << 20)
cf_status cf_deeppoly_run_static(const cf_network* net, int64_t B,
                                 const float* l0_dev, const float* u0_dev, const float* spec_W_dev,
                                 float* state_l_dev, float* state_u_dev,
                                 double* lb_dev, double* ub_dev, void* stream);
/* cf_deeppoly_check on the fixed array of the current device: synchronises `stream` and
 * reports whether a bounded device wait of the last cf_deeppoly_run_static call gave up
 * (CF_ERR_TIMEOUT) or a CROWN ReLU layer took the all-crossing branch (CF_ERR_UNSUPPORTED).
 * CF_ERR_NULL if no static call was made on this device yet. */
cf_status cf_deeppoly_check_static(void* stream);

/* Synchronise `stream` and report whether a bounded device-side wait of the last
 * cf_deeppoly_run that used `workspace_dev` gave up (CF_ERR_TIMEOUT) instead of hanging,
 * or (CF_RELAX_CROWN) a ReLU layer took the all-crossing branch (CF_ERR_UNSUPPORTED; the
 * bounds of that run are not valid). */
cf_status cf_deeppoly_check(const void* workspace_dev, void* stream);

/* ReLU transformer on pre-activation bounds l, u [B, n] (row stride ld_in):
 * l' = relu(l), u' = relu(u) (row stride ld_out), and the relaxation
 * L' = alpha*x, U' = lam*x + mu as compact [B, n] arrays.  relaxation must be
 * CF_RELAX_DEEPPOLY (CROWN's batch-wide branches run inside cf_deeppoly_run only). */
cf_status cf_relu_relax(int64_t B, int64_t n, const float* l_dev, const float* u_dev, int64_t ld_in,
                        float* l_out_dev, float* u_out_dev, int64_t ld_out,
                        float* alpha_dev, float* lam_dev, float* mu_dev, int32_t relaxation,
                        void* stream);

/* One backsubstitution step for 2*B*R coefficient rows (bound s in {0 lower, 1 upper},
 * region b, row i).  Row (s,b,i) of A_in is at A_in_dev + s*a_ss + b*a_bs + i*a_rs,
 * K contiguous columns over the output of affine layer j (after its ReLU if
 * alpha/lam/mu are given).  The step substitutes that ReLU (sign split with the
 * per-region relaxation) and then the affine layer:
 *   A_out[s,b,i,:] = T_s(A_in[s,b,i,:]) @ W     (W_dev [K, N] row-major = layer weight)
 *   c_out[s,b,i]   = c_in + sum_k mu-terms + T_s(A_in) . bias
 * A_out_dev is [2, B, R, N] compact, c_out_dev [2, B, R].  c_in may be NULL (zero). */
cf_status cf_backsub_step(int64_t B, int64_t R, int64_t K, int64_t N,
                          const float* A_in_dev, int64_t a_ss, int64_t a_bs, int64_t a_rs,
                          const float* c_in_dev, int64_t c_ss, int64_t c_bs,
                          const float* alpha_dev, const float* lam_dev, const float* mu_dev,
                          const float* W_dev, const float* bias_dev,
                          float* A_out_dev, float* c_out_dev, void* stream);

/* Fold the input box into the constant: for row (s,b,i) with coefficients over the
 * input, bound = c + sum_n (a>=0 ? a*box_s : a*box_{1-s}) where box_0 = l0, box_1 = u0.
 * Lower rows go to out_l_dev[b*ld_out + i], upper rows to out_u_dev[b*ld_out + i]. */
cf_status cf_concretize(int64_t B, int64_t R, int64_t n0,
                        const float* A_dev, int64_t a_ss, int64_t a_bs, int64_t a_rs,
                        const float* c_dev, int64_t c_ss, int64_t c_bs,
                        const float* l0_dev, const float* u0_dev,
                        float* out_l_dev, float* out_u_dev, int64_t ld_out, void* stream);

/* ---- gbcsr block kernels ----------------------------------------------------------
 * Elementwise kernels over one output block of `ndim` (<= CF_MAX_DIMS) dims with sizes
 * shape[], written contiguously (row-major).  Each input has its own element strides
 * (0 = broadcast along that dim), so the broadcast views the reference builds with
 * RepeatBlock / unsqueeze (sparse_block.py:3797) are read in place. */
#define CF_MAX_DIMS 6
enum {
  CF_OP_ADD = 0, CF_OP_SUB = 1, CF_OP_MUL = 2, CF_OP_DIV = 3,
  CF_OP_GE = 4, CF_OP_GT = 5, CF_OP_LE = 6, CF_OP_LT = 7, CF_OP_EQ = 8, CF_OP_NE = 9,
  CF_OP_AND = 10, CF_OP_OR = 11, CF_OP_MAX = 12, CF_OP_MIN = 13
};
enum { CF_UOP_NEG = 0, CF_UOP_NOT = 1, CF_UOP_SIGMOID = 2, CF_UOP_RELU = 3, CF_UOP_TO_F32 = 4 };
/* dtype codes of a block: 0 float32, 1 bool (one byte, 0/1) */
enum { CF_F32 = 0, CF_BOOL = 1 };

/* out = x op y.  Arithmetic in float32 (bool reads as 0/1); comparisons, and, or give
 * bool; the result is converted to out_dtype (bool: value != 0). */
cf_status cf_ew_binary(int32_t op, int32_t ndim, const int64_t* shape,
                       const void* x_dev, int32_t x_dtype, const int64_t* x_strides,
                       const void* y_dev, int32_t y_dtype, const int64_t* y_strides,
                       void* out_dev, int32_t out_dtype, void* stream);
/* out = op(x) (neg, logical not, sigmoid, relu, or plain conversion to out_dtype). */
cf_status cf_ew_unary(int32_t op, int32_t ndim, const int64_t* shape,
                      const void* x_dev, int32_t x_dtype, const int64_t* x_strides,
                      void* out_dev, int32_t out_dtype, void* stream);
/* out = cond ? y : z  (cond bool, y and z of out_dtype). */
cf_status cf_ew_where(int32_t ndim, const int64_t* shape,
                      const uint8_t* cond_dev, const int64_t* c_strides,
                      const void* y_dev, const int64_t* y_strides,
                      const void* z_dev, const int64_t* z_strides,
                      void* out_dev, int32_t out_dtype, void* stream);
/* min_true != 0: out = max(x, c) (clamp(min=c)); else out = min(x, c) (clamp(max=c)). */
cf_status cf_ew_clamp(int32_t ndim, const int64_t* shape, const float* x_dev, const int64_t* x_strides,
                      float c, int32_t min_true, float* out_dev, void* stream);
/* C[b] (+)= A[b] @ B[b], b < nb: A [M, K] with element strides (a_bs, a_ms, a_ks), B [K, N]
 * with (b_bs, b_ks, b_ns) (zero strides broadcast), C contiguous [nb, M, N]; float32.
 * The block-pair product of SparseTensor.matmul (constraintflow/gbcsr/sparse_tensor.py:1671-2060,
 * DenseBlock.matmul_equal_dims sparse_block.py:748, matmul_unequal_dims :964). */
/* Substitution of a per-neuron (diagonal) relaxation into coefficient rows, sign-selected:
 * out[b,m,n] = A[b,m,n] * (A >= 0 ? p[b,n] : q[b,n]) (out compact [nb, M, N]) and, if dc is
 * not NULL, dc[b,m] = sum_n A[b,m,n] * (A >= 0 ? pc[b,n] : qc[b,n]) (pc or qc NULL: 0).
 * A row (b,m) at A + b*a_bs + m*a_ms, n contiguous; p, q, pc, qc rows at b*v_bs.  The fused
 * form of clamp (tensor_ops.py:765) + inner_prod with a DiagonalBlock
 * (sparse_block.py:790) + binary add for the two signs. */
cf_status cf_signscale(int64_t nb, int64_t M, int64_t N, const float* A, int64_t a_bs, int64_t a_ms,
                       const float* p, const float* q, const float* pc, const float* qc, int64_t v_bs,
                       float* out, float* dc, void* stream);

cf_status cf_bmm(int64_t nb, int64_t M, int64_t N, int64_t K,
                 const float* A_dev, int64_t a_bs, int64_t a_ms, int64_t a_ks,
                 const float* B_dev, int64_t b_bs, int64_t b_ks, int64_t b_ns,
                 float* C_dev, int32_t accumulate, void* stream);
/* Bound combination of a certifier that carries two abstract states (polyzono.cf: the
 * DeepPoly polyexps and the zonotope): l = max(l_a, l_b), u = min(u_a, u_b) over [B, n],
 * written back into both states (rows at ld_a / ld_b floats) and, when lb / ub are not
 * NULL, to float64 [B, n].  Replaces the cf_max / cf_min calls of the generated
 * polyzono.Affine (constraintflow/gbcsr/tensor_ops.py:226, :245) on dense bound blocks. */
cf_status cf_bounds_meet(int64_t B, int64_t n, float* l_a, float* u_a, int64_t ld_a,
                         float* l_b, float* u_b, int64_t ld_b, double* lb, double* ub, void* stream);
/* *flag_dev |= 1 if any element of x is nonzero (flag is a device uint32). */
cf_status cf_ew_any(int32_t ndim, const int64_t* shape, const void* x_dev, int32_t x_dtype,
                    const int64_t* x_strides, uint32_t* flag_dev, void* stream);

/* gbcsr conv blocks (constraintflow/gbcsr/sparse_block.py: KernelBlock :1158, PatchesBlock
 * :2576).  A conv block stands for the matrix M [K*ox*oy, C*ix*iy] of a convolution with K
 * kernels over C input channels (input ix x iy, output ox x oy, kernel kx x ky, stride
 * sx / sy, padding px / py; x the first spatial dim, as in the reference): row
 * r = (k, oxi, oyi) holds a patch placed at input rows oxi*sx - px + dx and columns
 * oyi*sy - py + dy, positions outside the image dropped.  Patch values are read through
 * strides: (region b, kernel k, position pos = oxi*oy + oyi, channel c, dx, dy) at
 * P[b*p_bs + k*p_ks + pos*p_ps + (c*kx + dx)*ky + dy]; a KernelBlock's weights
 * W [K, C, kx, ky] have p_bs = p_ps = 0, p_ks = C*kx*ky; a PatchesBlock payload
 * [B, K*ox*oy, C*kx*ky] has p_ks = ox*oy*C*kx*ky, p_ps = C*kx*ky and p_bs = K*ox*oy*C*kx*ky
 * (0 when shared by every region).  Sums are float32. */
typedef struct cf_conv_geom {
  int32_t K, C;            /* kernels (output channels), input channels */
  int32_t ox, oy, ix, iy;  /* output and input spatial sizes */
  int32_t kx, ky, sx, sy, px, py;
} cf_conv_geom;
/* out [nb, K*ox*oy, C*ix*iy] = M of region b (KernelBlock.get_dense :1195 as
 * conv_transpose2d of the identity; PatchesBlock.get_dense :3089). */
cf_status cf_conv_densify(const cf_conv_geom* g, int64_t nb, const float* P, int64_t p_bs, int64_t p_ks,
                          int64_t p_ps, float* out, void* stream);
/* For image n = (bb, s), bb = n / per_b < nb: out[bb*o_bs + s*o_ss + r*o_rs] =
 * sum_j M[bb][r, j] x[j], x element j at X[bb*x_bs + s*x_ss + j*x_es] (F.conv2d of the
 * columns in KernelBlock.matmul_equal_dims :1364 / matmul_unequal_dims :1631; the unfold
 * product and sum of PatchesBlock.matmul_unequal_dims :2942). */
cf_status cf_conv_apply(const cf_conv_geom* g, int64_t nb, int64_t per_b, const float* P, int64_t p_bs,
                        int64_t p_ks, int64_t p_ps, const float* X, int64_t x_bs, int64_t x_ss, int64_t x_es,
                        float* out, int64_t o_bs, int64_t o_ss, int64_t o_rs, void* stream);
/* out [nb, K*ox*oy, C*kx*ky] = every patch value times the input value under it, 0 in the
 * padding; input element j of region b at X[b*x_bs + j*x_es] (the unfold products of
 * KernelBlock / PatchesBlock.matmul_equal_dims with a DiagonalBlock, :1364, :2820). */
cf_status cf_conv_scale(const cf_conv_geom* g, int64_t nb, const float* P, int64_t p_bs, int64_t p_ks,
                        int64_t p_ps, const float* X, int64_t x_bs, int64_t x_es, float* out, void* stream);
/* Transposed convolution of rows: for image n = (bb, s), out[bb*o_bs + s*o_ss + e*o_es]
 * (e = (c, X, Y) of an OH x OW output) = sum over (k, dx, dy) with X = oxi*sx - px + dx,
 * Y = oyi*sy - py + dy of y[(k, oxi, oyi)] * W[k, c, dx, dy], y element at
 * Y[bb*x_bs + s*x_ss + i*x_es] (F.conv_transpose2d in DenseBlock.matmul_equal_dims
 * :839-911 and in PatchesBlock.matmul_equal_dims with a KernelBlock :2740-2818). */
cf_status cf_conv_transpose(const cf_conv_geom* g, int64_t nb, int64_t per_b, const float* Y, int64_t x_bs,
                            int64_t x_ss, int64_t x_es, const float* W, int32_t OH, int32_t OW, float* out,
                            int64_t o_bs, int64_t o_ss, int64_t o_es, void* stream);

/* Message for the last non-OK status on this host thread ("" if none). */
const char* cf_last_error(void);
/* Library version string. */
const char* cf_version(void);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif /* CFGPU_H */
