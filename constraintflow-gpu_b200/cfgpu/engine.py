"""Host side of the DeepPoly network driver: network upload + one call into libcfgpu.

``DeepPolyEngine`` mirrors what ``Flow(abs_elem, deeppoly(), network).flow()``
(constraintflow/lib/flow_sparse.py:27-228) computes.  For a chain network it runs the
whole layer loop inside ``cf_deeppoly_run``: one C-ABI call per batch of regions, all
work stream-ordered on the current torch stream.  Networks with Add / Concat layers (and
CROWN's all-crossing branch) run the general traversal of cfgpu.general over libcfgpu's
block kernels.  Torch only provides device memory and the stream handle.
"""
import ctypes

import torch

from . import _lib
from ._lib import lib, check, CfLayer, CfNetwork

N_CLASSES = 10


class DeepPolyEngine:
    """A network resident on one GPU, ready to certify batches of input regions.

    layers: sequence of objects with ``kind`` in {'linear','conv','relu','add','concat'}
    and, for affine layers, ``W`` / ``b`` arrays (Linear W [out, in]; Conv W [Cout, Cin,
    k, k]) plus ``in_shape`` / ``out_shape`` / ``stride`` / ``pad`` for conv layers;
    optional ``parents`` (layer-list indices, -1 = the network input; default the previous
    layer), listed in the reference reader's order (every parent before its children).
    certifier: 'deeppoly' (deeppoly.cf, deeppoly_efficient.cf), 'crown' (crown.cf, whose
    ReLU branch is decided over the whole batch: a CROWN run always takes the batch in
    one workspace chunk and checks the device status; when a layer takes the all-crossing
    branch the bounds are recomputed by the general traversal of cfgpu.general), 'zono'
    (zono.cf, DeepZ: forward zonotope pass, linear chains), 'ibp' (ibp.cf: interval
    bounds) or 'crownibp' (crownibp.cf: interval bounds below the property, DeepPoly's
    ReLU relaxation from them, one backsubstitution of the property rows; chains).
    stop_depth: the custom-stop DeepPoly programs (deeppoly_custom_stop.cf, custom_stops/)
    with get_start = stop_depth: the traversal bounding a neuron of list layer m stops below
    layer m - stop_depth and concretises there with those neurons' own bounds (linear chains;
    None: every traversal reaches the input).  relu_strict: the lower ReLU slope is 1 where
    l + u > 0 (the relu_n of those programs and of zid.cf) instead of l + u >= 0; deeppoly
    and crownibp.
    """

    def __init__(self, layers, input_size, device="cuda", n_spec=N_CLASSES - 1, certifier="deeppoly",
                 stop_depth=None, relu_strict=False):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("DeepPolyEngine runs on a CUDA device only (no CPU fallback)")
        self.input_size = int(input_size)
        self.n_spec = int(n_spec)
        relax = {"deeppoly": _lib.CF_RELAX_DEEPPOLY, "crown": _lib.CF_RELAX_CROWN, "zono": _lib.CF_RELAX_ZONO,
                 "ibp": _lib.CF_RELAX_IBP, "crownibp": _lib.CF_RELAX_CROWNIBP}
        if certifier not in relax:
            raise NotImplementedError(f"certifier {certifier!r} (the driver runs deeppoly, crown, zono, ibp and "
                                      "crownibp)")
        self.certifier = certifier
        self.stop_depth = None
        self._keep = []
        self._general = []        # (kind, W, b, parents) device tensors for cfgpu.general
        widths = []
        descs = []
        self.chain = True
        for i, L in enumerate(layers):
            parents = tuple(int(p) for p in getattr(L, "parents", None) or (i - 1,))
            if any(not -1 <= p < i for p in parents):
                raise ValueError(f"layer {i}: parents {parents} must precede it in the list")
            pw = [self.input_size if p < 0 else widths[p] for p in parents]
            self.chain &= parents == (i - 1,)
            d = CfLayer()
            if L.kind in ("relu", "add", "concat"):
                if L.kind != "relu":
                    self.chain = False
                    if len(parents) != 2:
                        raise ValueError(f"layer {i}: {L.kind} takes two parents, got {parents}")
                    if L.kind == "add" and pw[0] != pw[1]:
                        raise ValueError(f"layer {i}: add of widths {pw}")
                d.kind = _lib.CF_LAYER_RELU
                d.n_in = d.n_out = sum(pw) if L.kind == "concat" else pw[0]
                self._general.append((L.kind, None, None, parents))
            else:
                W = torch.as_tensor(L.W, dtype=torch.float32).to(self.device).contiguous()
                b = torch.as_tensor(L.b, dtype=torch.float32).to(self.device).contiguous()
                self._keep += [W, b]
                d.W_dev, d.b_dev = W.data_ptr(), b.data_ptr()
                if L.kind == "linear":
                    d.kind = _lib.CF_LAYER_LINEAR
                    d.n_out, d.n_in = int(W.shape[0]), int(W.shape[1])
                elif L.kind == "conv":
                    d.kind = _lib.CF_LAYER_CONV
                    d.cout, d.cin, d.kh, d.kw = (int(x) for x in W.shape)
                    _, d.ih, d.iw = (int(x) for x in L.in_shape)
                    _, d.oh, d.ow = (int(x) for x in L.out_shape)
                    d.stride, d.pad = int(L.stride), int(L.pad)
                    d.n_in = d.cin * d.ih * d.iw
                    d.n_out = d.cout * d.oh * d.ow
                else:
                    raise NotImplementedError(f"layer kind {L.kind}")
                geom = ((d.cin, d.ih, d.iw, d.cout, d.oh, d.ow, d.stride, d.pad) if L.kind == "conv" else None)
                self._general.append((L.kind, W, b, parents, geom))
                if d.n_in != pw[0]:
                    raise ValueError(f"layer {i}: {L.kind} reads {d.n_in} neurons, its parent has {pw[0]}")
            widths.append(int(d.n_out))
            descs.append(d)
        self.n_last = widths[-1] if widths else self.input_size
        self.kinds = [g[0] for g in self._general]
        if self.chain:
            self._layers = (CfLayer * len(descs))(*descs)
            if stop_depth is not None and (certifier != "deeppoly" or int(stop_depth) < 0 or
                                           any(g[0] == "conv" for g in self._general)):
                raise NotImplementedError("a custom stop depth applies to the DeepPoly traversal of linear chains")
            self.stop_depth = None if stop_depth is None else int(stop_depth)
            code = relax[certifier]
            if relu_strict:
                strict = {"deeppoly": _lib.CF_RELAX_DEEPPOLY_STRICT, "crownibp": _lib.CF_RELAX_CROWNIBP_STRICT}
                if certifier not in strict:
                    raise NotImplementedError("the strict lower-slope test applies to DeepPoly's relaxation "
                                              "(deeppoly, crownibp)")
                code = strict[certifier]
            self.net = CfNetwork(len(descs), self._layers, self.input_size, self.n_spec, code,
                                 0 if stop_depth is None else int(stop_depth) + 1)
            self.N = int(lib.cf_network_neurons(ctypes.byref(self.net)))
            if self.N < 0:
                check(_lib.CF_ERR_SHAPE, "network description")
        else:
            # Add / Concat: polyexps mix layers; the general traversal runs the whole network
            if certifier not in ("deeppoly", "crown"):
                raise NotImplementedError(f"{certifier} on a network with Add / Concat layers (the forward "
                                          "drivers run chain networks)")
            if stop_depth is not None or relu_strict:
                raise NotImplementedError("a custom stop depth or strict ReLU test on a network with Add / Concat "
                                          "layers")
            self.net = None
            self.N = self.input_size + sum(widths) + self.n_spec
        self._ws = None
        self.graphs = True           # CUDA-graph replay of the general traversal (DeepPoly)
        self._graph_cache = {}
        self.replayed_launches = 0   # libcfgpu kernels replayed by those graphs

    def workspace_bytes(self, chunk):
        if self.net is None:
            raise ValueError("the fused driver's workspace applies to chain networks only")
        return int(lib.cf_deeppoly_workspace_bytes(ctypes.byref(self.net), int(chunk)))

    def _workspace(self, B, budget_bytes):
        need_full = self.workspace_bytes(max(1, B))
        # CROWN needs the whole batch in one chunk; DeepPoly regions are independent
        need = need_full if self.certifier == "crown" else min(need_full, max(self.workspace_bytes(1), budget_bytes))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    # device bytes the fused driver's workspace may take; DeepPoly regions beyond what fits
    # run in further chunks of the same call
    workspace_budget = 8 << 30

    def run(self, l0, u0, spec_W, want_state=False, workspace_budget=None, out=None, check_device=False,
            replay=None):
        """Bounds for B regions.

        l0, u0: [B, n_input] float32 device tensors (normalised input box);
        spec_W: [B, n_spec, n_last] float32 device tensor (property matrix).
        Returns (lb, ub) float64 [B, n_spec] and, if want_state, (state_l, state_u)
        float32 [B, N] with every neuron's bounds in the reference's neuron order.
        check_device=True synchronises and raises if a bounded device wait gave up.
        replay=(dec_l, dec_u): [B, N] float32 device tensors (state layout) from which every
        ReLU branch decision is taken (cf_deeppoly_run_replay; DeepPoly chains only).
        """
        B = int(l0.shape[0])
        for t, shp in ((l0, (B, self.input_size)), (u0, (B, self.input_size)),
                       (spec_W, (B, self.n_spec, self.n_last))):
            if tuple(t.shape) != shp or t.dtype != torch.float32 or not t.is_contiguous() or t.device != self.device:
                raise Exception(f"SHAPE MISMATCH: expected contiguous float32 {shp} on {self.device}, "
                                f"got {tuple(t.shape)} {t.dtype} on {t.device}")
        if out is None:
            lb = torch.empty(B, self.n_spec, dtype=torch.float64, device=self.device)
            ub = torch.empty_like(lb)
        else:
            lb, ub = out
        sl = su = None
        if want_state:
            sl = torch.empty(B, self.N, dtype=torch.float32, device=self.device)
            su = torch.empty_like(sl)
        if self.net is None:
            lb, ub, sl_g, su_g = self._general_run(l0, u0, spec_W, lb, ub)
            if want_state:
                sl.copy_(sl_g)
                su.copy_(su_g)
                return lb, ub, sl, su
            return lb, ub
        ws = self._workspace(B, self.workspace_budget if workspace_budget is None else workspace_budget)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if replay is not None:
            dl, du = replay
            for t in (dl, du):
                if tuple(t.shape) != (B, self.N) or t.dtype != torch.float32 or not t.is_contiguous() or \
                        t.device != self.device:
                    raise Exception(f"SHAPE MISMATCH: replay bounds must be contiguous float32 {(B, self.N)}")
            st = lib.cf_deeppoly_run_replay(ctypes.byref(self.net), B, l0.data_ptr(), u0.data_ptr(),
                                            spec_W.data_ptr(), dl.data_ptr(), du.data_ptr(),
                                            sl.data_ptr() if sl is not None else None,
                                            su.data_ptr() if su is not None else None,
                                            lb.data_ptr(), ub.data_ptr(), ws.data_ptr(), ws.numel(), stream)
            check(st, "cf_deeppoly_run_replay")
        else:
            st = lib.cf_deeppoly_run(ctypes.byref(self.net), B, l0.data_ptr(), u0.data_ptr(), spec_W.data_ptr(),
                                     sl.data_ptr() if sl is not None else None,
                                     su.data_ptr() if su is not None else None,
                                     lb.data_ptr(), ub.data_ptr(), ws.data_ptr(), ws.numel(), stream)
            check(st, "cf_deeppoly_run")
        if self.certifier == "crown":
            st = lib.cf_deeppoly_check(ws.data_ptr(), stream)
            if st == _lib.CF_ERR_UNSUPPORTED:
                # a ReLU layer took the all-crossing branch: its polyexps mix layers
                lb, ub, sl_g, su_g = self._general_run(l0, u0, spec_W, lb, ub)
                if want_state:
                    sl.copy_(sl_g)
                    su.copy_(su_g)
            else:
                check(st, "device status")
        elif check_device:
            check(lib.cf_deeppoly_check(ws.data_ptr(), stream), "device status")
        if want_state:
            return lb, ub, sl, su
        return lb, ub

    def _general_run(self, l0, u0, spec_W, lb, ub):
        """Bounds through the general lowest-layer-first traversal (cfgpu.general).

        DeepPoly's traversal takes no data-dependent decision on the host, so for a given
        batch size its launches are captured once in a CUDA graph and replayed (the inputs
        are copied into the graph's buffers); CROWN decides its ReLU branches on the host and
        runs eagerly."""
        from . import general
        if self.certifier == "deeppoly" and self.graphs:
            g = self._graph_cache.get(int(l0.shape[0]))
            if g is None:
                g = self._capture(l0, u0, spec_W)
            if g is not None:
                g["l0"].copy_(l0)
                g["u0"].copy_(u0)
                g["W"].copy_(spec_W)
                g["graph"].replay()
                self.replayed_launches += g["launches"]
                lb.copy_(g["sl"][:, -self.n_spec:])
                ub.copy_(g["su"][:, -self.n_spec:])
                return lb, ub, g["sl"], g["su"]
        bounds, _ = general.run(self._general, l0, u0, spec_W, self.certifier)
        sl, su = general.state(l0, u0, bounds)
        lb.copy_(bounds[-1][0])
        ub.copy_(bounds[-1][1])
        return lb, ub, sl, su

    def _capture(self, l0, u0, spec_W):
        from . import general
        static = {"l0": l0.clone(), "u0": u0.clone(), "W": spec_W.clone()}
        try:
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):      # warm-up outside the capture
                general.run(self._general, static["l0"], static["u0"], static["W"], "deeppoly")
            torch.cuda.current_stream(self.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            from . import ops
            n0 = ops.LAUNCHES[0]
            with torch.cuda.graph(graph):
                bounds, _ = general.run(self._general, static["l0"], static["u0"], static["W"], "deeppoly")
                static["sl"], static["su"] = general.state(static["l0"], static["u0"], bounds)
        except RuntimeError:
            self.graphs = False                  # capture refused: run eagerly from now on
            return None
        static["graph"] = graph
        static["launches"] = ops.LAUNCHES[0] - n0
        self._graph_cache[int(l0.shape[0])] = static
        return static

    def input_spec(self, X, y, eps, dataset):
        """Device input box and property matrix from device centres X [B,C,H,W] and labels y [B].

        Same arithmetic as constraintflow/lib/spec.py:21-72 (clip, normalise, e_label - e_k).
        """
        from .nets import MNIST_MEAN, MNIST_STD, CIFAR_MEAN, CIFAR_STD
        B = int(X.shape[0])
        C = int(X.shape[1])
        HW = int(X[0, 0].numel())
        mean, std = (MNIST_MEAN, MNIST_STD) if dataset == "mnist" else (CIFAR_MEAN, CIFAR_STD)
        if len(mean) == 1:
            mean, std = mean * C, std * C
        l0 = torch.empty(B, C * HW, dtype=torch.float32, device=self.device)
        u0 = torch.empty_like(l0)
        W = torch.empty(B, self.n_spec, self.n_spec + 1, dtype=torch.float32, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(lib.cf_input_box(B, C, HW, X.data_ptr(), float(eps), _lib.f32_array(mean), _lib.f32_array(std),
                               l0.data_ptr(), u0.data_ptr(), stream), "cf_input_box")
        check(lib.cf_spec_matrix(B, self.n_spec + 1, y.data_ptr(), W.data_ptr(), stream), "cf_spec_matrix")
        return l0, u0, W

    def certify(self, X, y, eps, dataset, out=None):
        """Whole pipeline on device tensors: input box, property, certifier -> (lb, ub) float64."""
        l0, u0, W = self.input_spec(X, y, eps, dataset)
        lb, ub = self.run(l0, u0, W, out=out)
        return lb, ub


def profile_enable(on=True):
    check(lib.cf_profile_enable(1 if on else 0))


def profile_collect():
    st = _lib.CfProfileStats()
    check(lib.cf_profile_collect(ctypes.byref(st)), "cf_profile_collect")
    return dict(kernel_launches=st.kernel_launches, step_launches=st.step_launches, step_ms=st.step_ms,
                step_flops=st.step_flops, step_bytes=st.step_bytes, mem_launches=st.mem_launches,
                mem_ms=st.mem_ms, mem_bytes=st.mem_bytes)
