#!/usr/bin/env python
"""Benchmark: certified input regions/sec (DeepPoly, whole input box) on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cfgpu|reference] [--workload 2]
                    [--certifier deeppoly|crown|zono|ibp|polyzono|crownibp|custom_stop]
                    [--stop-depth D] [--batch B]

One step = one whole DeepPoly pass (input box, property matrix, every layer's
backsubstitution down to the input, final bounds) over one batch of regions of the
workload (default: ReLU MLP 784-(200x9)-10, 256 regions per GPU, eps 0.002; seeded
synthetic network and centres, since no dataset or trained model is available offline).
--certifier runs another of the reference's programs on the same workload (a zono / ibp
step is one forward pass; polyzono.cf runs a DeepPoly and a zonotope pass layer by layer).
`roofline` covers the dominant (tensor-core) kernels; `memory_bound` the HBM-bound kernels
of the pass (relaxations, concretisation, conversions): their algorithmic bytes, device
time and GB/s against the measured HBM copy bandwidth.
Multi-GPU: one process per GPU (torchrun), each certifying its own 256 regions (weak
scaling; regions are independent, no collective on the data path).  Rank 0 prints one
JSON line.

--impl reference times the CPU restatement of the reference's algorithm (oracle/, numpy
float32 with all host threads) on a bounded sample of the same workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "constraintflow-gpu_b200"))
sys.path.insert(0, HERE)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from cfgpu import nets  # noqa: E402

L2_BYTES = 126 * 2 ** 20
# DRAM bytes (read + write) of one launch of the dominant kernel, from an ncu capture of
# the default command (profiles/k_chain_mlp784-200x9_b256.txt); per workload id.
NCU_TRAFFIC = {(2, "deeppoly"): 7.52e6}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="cfgpu", choices=["cfgpu", "reference"])
    ap.add_argument("--workload", type=int, default=2)
    ap.add_argument("--batch", type=int, default=0, help="regions per GPU (default: the workload's batch)")
    ap.add_argument("--certifier", default="deeppoly", choices=["deeppoly", "crown", "zono", "ibp", "polyzono",
                                                                  "crownibp", "custom_stop", "zid"],
                    help="certifier program (deeppoly.cf, crown.cf, zono.cf, ibp.cf, polyzono.cf, crownibp.cf, "
                         "deeppoly_custom_stop.cf, zid.cf)")
    ap.add_argument("--stop-depth", type=int, default=3,
                    help="get_start of --certifier custom_stop (3: deeppoly_custom_stop.cf)")
    ap.add_argument("--cifar", default="auto", choices=["auto", "skip"],
                    help="auto: add the 'cifar' sub-record (DeepPoly, 3x32x32 conv net, 1024 regions split "
                         "over the GPUs) to the default DeepPoly line")
    return ap.parse_args()


def peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


class Clocks:
    """SM clock and clock-event-reason sampler for the timed region (one GPU).

    NVML queries every 10 ms from a thread (read-only), so that a timed region of tens of
    milliseconds still gets samples; nvidia-smi -lms 200 when NVML is not importable.
    Every sample is also written to `path` (CSV) as the record of the run.
    """

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index, path, device=None):
        import threading
        self.path = path
        self.samples = []
        self.p = None
        self.thread = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = None
            if device is not None:
                try:
                    uuid = str(torch.cuda.get_device_properties(device).uuid)
                    h = nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
                except Exception:
                    h = None
            if h is None:
                h = nv.nvmlDeviceGetHandleByIndex(index)
            self.nv, self.h = nv, h
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.stop_ev = threading.Event()

            def loop():
                while not self.stop_ev.is_set():
                    try:
                        self.samples.append((time.time(), float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                             int(get_reasons(h))))
                    except Exception:
                        pass
                    self.stop_ev.wait(0.01)
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            try:
                self.fh = open(path, "w")
                self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}",
                                           "--format=csv,noheader", "-lms", "200"],
                                          stdout=self.fh, stderr=subprocess.DEVNULL)
            except Exception:
                self.p = None

    def stop(self):
        if self.thread is not None:
            self.stop_ev.set()
            self.thread.join(timeout=5)
            sm, reasons = [], set()
            with open(self.path, "w") as fh:
                fh.write("unix_time,sm_mhz,sm_max_mhz,clocks_event_reasons\n")
                for t, mhz, r in self.samples:
                    fh.write(f"{t:.3f},{mhz:.0f},{self.max_mhz:.0f},{r:#x}\n")
                    sm.append(mhz)
                    for name, bit in self.REASONS:
                        if r & bit:
                            reasons.add(name)
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml 10 ms"}
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.fh.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1].split()[0]))
                mx = float(f[2].split()[0])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi 200 ms"}


# regions per CPU sample of the oracle port, per workload id (about 0.5-1 s each; the
# CIFAR-shaped conv net: one region, 10-30 s)
CPU_SAMPLE = {0: 1, 1: 16, 2: 8, 3: 4, 4: 1, 5: 16, 6: 256}
CPU_REPS = {4: 1}
# the CIFAR sub-record: regions in all (split over the GPUs), timed steps, warm-up steps
CIFAR_REGIONS, CIFAR_STEPS, CIFAR_WARMUP = 1024, 2, 1
CIFAR_WORKSPACE = 32 << 30   # bytes of engine workspace: regions run in chunks that fit


METRIC = {"deeppoly": "DeepPoly", "crown": "CROWN", "zono": "zonotope (DeepZ)", "ibp": "interval (IBP)",
          "polyzono": "polyzono (DeepPoly met with the zonotope)", "crownibp": "CROWN-IBP (crownibp.cf)",
          "custom_stop": "DeepPoly with a custom traversal stop", "zid": "zid (zonotope, interval, DeepPoly)"}


def _metric(certifier):
    return f"certified input regions/sec ({METRIC[certifier]}, whole box)"


def _oracle_fn(wl, certifier="deeppoly", stop_depth=3):
    """The oracle for the workload and program: the chain DeepPoly oracle, the general one
    (CROWN, or a network with Add / Concat layers), or the zonotope / interval one."""
    if certifier in ("zono", "ibp", "polyzono", "zid"):
        from oracle import zono_oracle as Z
        if certifier == "polyzono":
            return lambda l0, u0, W: Z.polyzono(wl.layers, l0, u0, W)
        if certifier == "zid":
            return lambda l0, u0, W: Z.zid(wl.layers, l0, u0, W)
        if certifier == "zono":
            return lambda l0, u0, W: Z.zono(wl.layers, l0, u0, W)
        return lambda l0, u0, W: Z.ibp(wl.layers, l0, u0, W)
    if certifier == "crown":
        from oracle import crown_oracle as C
        return lambda l0, u0, W: C.certify(wl.layers, l0, u0, W, "crown")
    if certifier == "crownibp":
        from oracle import crown_oracle as C
        return lambda l0, u0, W: C.crownibp(wl.layers, l0, u0, W)
    if certifier == "custom_stop":
        from oracle import crown_oracle as C
        return lambda l0, u0, W: C.custom_stop(wl.layers, l0, u0, W, stop_depth)
    if nets.is_chain(wl.layers):
        from oracle import deeppoly_oracle as O
        if any(L.kind == "conv" for L in wl.layers):
            # conv networks: the receptive-field-window restatement (dense rows take minutes)
            return lambda l0, u0, W: O.deeppoly_windows(wl.layers, l0, u0, W)
        return lambda l0, u0, W: O.deeppoly(wl.layers, l0, u0, W)
    from oracle import crown_oracle as C
    return lambda l0, u0, W: C.certify(wl.layers, l0, u0, W, "deeppoly")


def cpu_baseline(wl, sample, reps=3, certifier="deeppoly", stop_depth=3):
    """Oracle (numpy float32, all host threads) on `sample` regions of the workload: regions/s."""
    fn = _oracle_fn(wl, certifier, stop_depth)
    X = nets.centres(wl, sample)
    y = nets.labels(wl, X)
    l0, u0 = nets.input_box(X, wl.eps, wl.dataset)
    W = nets.spec_weight(y).numpy()
    l0, u0 = l0.numpy(), u0.numpy()
    if reps > 1:
        fn(l0[:1], u0[:1], W[:1])  # warm
    ts = []
    for _ in range(reps):
        t = time.perf_counter()
        fn(l0, u0, W)
        ts.append(time.perf_counter() - t)
    return sample / statistics.median(ts), statistics.median(ts)


def run_reference(args, rank, world):
    if rank != 0:
        return
    wl = nets.workload(args.workload)
    sample = CPU_SAMPLE[args.workload]
    if args.workload in CPU_REPS:
        # a step of this workload is 10-30 s of CPU work: at most two, no warm-up
        args.steps, args.warmup = min(args.steps, 2), 0
    fn = _oracle_fn(wl, args.certifier, args.stop_depth)
    X = nets.centres(wl, sample)
    y = nets.labels(wl, X)
    l0, u0 = nets.input_box(X, wl.eps, wl.dataset)
    W = nets.spec_weight(y).numpy()
    l0, u0 = l0.numpy(), u0.numpy()
    for _ in range(args.warmup):
        fn(l0, u0, W)
    ts = []
    for _ in range(args.steps):
        t = time.perf_counter()
        fn(l0, u0, W)
        ts.append(time.perf_counter() - t)
    ms = 1000 * statistics.mean(ts)
    val = sample / (ms / 1000)
    cores = os.cpu_count()
    desc = f"oracle port (numpy float32 BLAS, {cores} threads), {sample} regions of {wl.name} per step"
    print(json.dumps({
        "impl": "reference", "metric": _metric(args.certifier), "value": val,
        "unit": "regions/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name, "certifier": args.certifier, "regions_per_step": sample, "eps": wl.eps,
                   **({"stop_depth": args.stop_depth} if args.certifier == "custom_stop" else {})},
        "cpu_baseline": {"value": val, "unit": "regions/s", "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": val, "unit": "regions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def _make_engine(wl, certifier, stop_depth, dev):
    from cfgpu.engine import DeepPolyEngine
    if certifier == "polyzono":
        from cfgpu.polyzono import PolyZonoEngine
        return PolyZonoEngine(wl.layers, wl.input_size, dev)
    if certifier == "zid":
        from cfgpu.zid import ZidEngine
        return ZidEngine(wl.layers, wl.input_size, dev)
    if certifier == "custom_stop":
        return DeepPolyEngine(wl.layers, wl.input_size, dev, stop_depth=stop_depth, relu_strict=True)
    return DeepPolyEngine(wl.layers, wl.input_size, dev, certifier=certifier)


def measure(wl, B_total, per_rank, steps, warmup, certifier, stop_depth, rank, world, dev, workspace_budget):
    """Time `steps` certifier passes of this rank's regions (after `warmup`), device-timed with
    CUDA events; every step also all-gathers every rank's bounds (NCCL) and counts the
    certified regions on the device, inside the timed region.  Then the same end to end
    through the public API with host buffers.  Returns a dict of the figures (max over ranks)."""
    import torch.distributed as dist
    from cfgpu import dist as cdist
    from cfgpu.engine import profile_enable, profile_collect
    Xall = nets.centres(wl, B_total)
    lo, hi = cdist.shard_range(B_total, rank, world) if not per_rank else (rank * per_rank, (rank + 1) * per_rank)
    if per_rank:
        Xall = nets.centres(wl, per_rank * world)
    X = Xall[lo:hi].contiguous()
    y = nets.labels(wl, X)
    B = int(X.shape[0])
    n_regions = int(Xall.shape[0])
    eng = _make_engine(wl, certifier, stop_depth, dev)
    if workspace_budget:
        eng.workspace_budget = workspace_budget
    Xd, yd = X.to(dev), y.to(dev)
    lb = torch.empty(B, 9, dtype=torch.float64, device=dev)
    ub = torch.empty_like(lb)
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    n_cert = torch.zeros((), dtype=torch.int64, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def gather_and_count():
        # the one collective of the path: every rank's bounds to every rank, then the
        # reference's verdict rule (all property lower bounds >= 0, constraintflow/cli.py:118-121)
        if world > 1:
            lb_all, _ = cdist.gather_bounds(lb, ub, n_regions, rank, world)
        else:
            lb_all = lb
        n_cert.copy_((lb_all >= 0).all(dim=1).sum())

    def step():
        eng.certify(Xd, yd, wl.eps, wl.dataset, out=(lb, ub))
        gather_and_count()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    clk_dir = os.environ.get("CF_CLOCKS_DIR", "/tmp")   # where the per-rank clock samples are written
    clk = Clocks(int(dev.index or 0), os.path.join(clk_dir, f"cf_clocks_{wl.wid}_r{rank}.csv"), device=dev)
    barrier()
    torch.cuda.synchronize()
    profile_enable(True)
    replay0 = getattr(eng, "replayed_launches", 0)
    wall = time.perf_counter()
    for k in range(steps):
        flush.zero_()
        starts[k].record()
        step()
        ends[k].record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall
    prof = profile_collect()
    profile_enable(False)
    # kernels replayed from the CUDA graph of a general traversal are not counted by the
    # library's launch counter
    prof["kernel_launches"] += getattr(eng, "replayed_launches", 0) - replay0
    barrier()
    clocks = clk.stop()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    certified = int(n_cert.item())
    # ---- end-to-end through the public API with host buffers
    Xh = X.pin_memory()
    yh = y.pin_memory()
    lbh = torch.empty(B, 9, dtype=torch.float64).pin_memory()
    ubh = torch.empty_like(lbh).pin_memory()
    Xe = torch.empty_like(Xd)
    ye = torch.empty_like(yd)

    def e2e_step():
        Xe.copy_(Xh, non_blocking=True)
        ye.copy_(yh, non_blocking=True)
        eng.certify(Xe, ye, wl.eps, wl.dataset, out=(lb, ub))
        gather_and_count()
        lbh.copy_(lb, non_blocking=True)
        ubh.copy_(ub, non_blocking=True)

    for _ in range(warmup):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    return {"eng": eng, "B": B, "n_regions": n_regions, "ms_max": ms_max, "ms_local": ms, "prof": prof,
            "clocks": clocks, "wall": wall, "certified": certified,
            "value": n_regions * steps / (ms_max / 1000.0),
            "e2e": {"value": n_regions * steps / (float(te.item()) / 1000.0), "unit": "regions/s",
                    "h2d_bytes_per_step": int(X.numel() * 4 + y.numel() * 8),
                    "d2h_bytes_per_step": int(2 * B * 9 * 8)}}


def _roofline(m, wl, certifier, steps, dev):
    bf16, hbm, src = peaks()
    prof, ms, eng = m["prof"], m["ms_local"], m["eng"]
    achieved = prof["step_flops"] / (prof["step_ms"] / 1000.0) / 1e12 if prof["step_ms"] > 0 else None
    conv = any(L.kind == "conv" for L in wl.layers)
    chain = getattr(eng, "chain", True)
    zono_tc = certifier in ("zono", "polyzono") and os.environ.get("CF_STEP_IMPL") != "simt"
    conv_tc = conv and certifier == "deeppoly" and os.environ.get("CF_CONV_IMPL") != "simt"
    if conv_tc:
        # receptive-field windows: the transposed convolutions of the windows run as tcgen05 3xTF32
        # GEMMs (k_win_convT_tc); the first layer's (3 input channels) is fused with the
        # concretisation on the CUDA cores (k_win_first); both count as backsubstitution steps
        peak, bound, peak_src = bf16 / 2.0 / 3.0, "tensor", f"3xTF32 = bf16/2/3 of {src} MEASURED_PEAKS"
    elif conv or not chain or (certifier in ("zono", "ibp") and not zono_tc):
        # transposed-conv GEMMs on the CUDA cores (CF_CONV_IMPL=simt) or the zonotope conv kernels; a
        # network with Add / Concat layers: the general traversal's k_bmm GEMMs; the zonotope pass:
        # k_zono_gemm over the noise-symbol rows -- all on the FP32 pipe.
        # MEASURED_PEAKS holds no FP32-pipe figure, so the nominal one: SMs x 128 lanes x 2 x max clock
        props = torch.cuda.get_device_properties(dev)
        mhz = m["clocks"].get("sm_max_mhz") or 1965.0
        peak, bound, peak_src = props.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12, "fp32", \
            "nominal FP32 FMA pipe (SMs x 128 x 2 x max SM clock); no measured figure"
    else:
        peak, bound, peak_src = bf16 / 2.0 / 3.0, "tensor", f"3xTF32 = bf16/2/3 of {src} MEASURED_PEAKS"
    key = (wl.wid, certifier)
    roof = {"bound": bound, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": (achieved / peak) if achieved else None,
            "traffic": NCU_TRAFFIC.get(key),
            "traffic_source": ("dram read+write of one k_chain launch (a 200-wide hidden layer bounded "
                               "through 8 substitutions for one lane of 128 regions, 400 CTAs) from one ncu "
                               "--set full capture of this command") if key in NCU_TRAFFIC else None,
            "kernel": {"zono": "k_zono_persist" if zono_tc else "k_zono_gemm", "ibp": None,
                       "polyzono": "k_chain (backsubstitution) + k_zono_persist"}.get(
                           certifier, ("k_win_convT_tc (tcgen05 3xTF32) + k_win_first (CUDA cores, first layer), "
                                       "the transposed convolutions of the receptive-field windows" if conv_tc
                                       else "transposed convolution of the receptive-field windows" if conv else
                                       "k_chain (tcgen05 3xTF32 backsubstitution); when a pass runs its regions as "
                                       "two lanes on two streams, the step time is the device-time span of the "
                                       "lanes (first to last launch), not a sum of overlapping launches")
                                      if chain else "k_bmm (general traversal)"),
            "peak_source": peak_src,
            "step_share_of_pass": prof["step_ms"] / ms if ms > 0 else None,
            "step_launches": prof["step_launches"]}
    mem = {"kernels": {"zono": "k_zono_bounds, k_zono_relu", "polyzono": "k_relu_relax, k_zono_bounds, "
                       "k_zono_relu, k_to_f64, k_prep_wimg", "ibp": None}.get(
                           certifier, "k_win_relu_bias (ReLU window pass), k_relu_relax, k_to_f64" if conv else
                           "k_relu_relax / k_crown_relax, k_concretize, k_to_f64, k_prep_wimg"),
           "launches": int(prof["mem_launches"]),
           "bytes_per_pass": prof["mem_bytes"] / steps,
           "ms_per_pass": prof["mem_ms"] / steps,
           "achieved": prof["mem_bytes"] / (prof["mem_ms"] / 1000.0) / 1e9 if prof["mem_ms"] > 0 else None,
           "peak": hbm, "unit": "GB/s",
           "frac": prof["mem_bytes"] / (prof["mem_ms"] / 1000.0) / 1e9 / hbm if prof["mem_ms"] > 0 else None,
           "peak_source": f"{src} MEASURED_PEAKS hbm_gbs",
           "share_of_pass": prof["mem_ms"] / ms if ms > 0 else None}
    return roof, mem


def _cpu_baseline_record(wl, certifier, stop_depth):
    sample = CPU_SAMPLE[wl.wid]
    reps = CPU_REPS.get(wl.wid, 3)
    v, t1 = cpu_baseline(wl, sample, reps=reps, certifier=certifier, stop_depth=stop_depth)
    how = "receptive-field windows" if any(L.kind == "conv" for L in wl.layers) else "dense rows"
    return {"value": v, "unit": "regions/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"oracle numpy float32 ({how}, {os.cpu_count()} host threads), {sample} region(s) of "
                      f"{wl.name}, median of {reps} ({t1:.2f} s each)"}


def run_cfgpu(args, rank, world, local):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    wl = nets.workload(args.workload)
    B = args.batch or wl.B
    warm = max(3, args.warmup)
    m = measure(wl, 0, B, args.steps, warm, args.certifier, args.stop_depth, rank, world, dev, None)
    cifar = None
    if args.cifar == "auto" and args.workload == 2 and args.certifier == "deeppoly" and not args.batch:
        # the CIFAR-shaped conv net (3x32x32, 4 conv + 3 FC layers): 1024 regions in all, split
        # over the GPUs (strong scaling), chunked inside the engine to fit its workspace
        wl4 = nets.workload(4)
        cifar = measure(wl4, CIFAR_REGIONS, 0, CIFAR_STEPS, CIFAR_WARMUP, "deeppoly", 0, rank, world, dev,
                        CIFAR_WORKSPACE)
    if rank != 0:
        return
    roof, mem = _roofline(m, wl, args.certifier, args.steps, dev)
    out = {
        "metric": _metric(args.certifier), "value": m["value"], "unit": "regions/s",
        "n_gpus": world, "steps": args.steps, "warmup": warm, "ms_per_step": m["ms_max"] / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name, "certifier": args.certifier, "regions_per_gpu": B,
                   **({"stop_depth": args.stop_depth} if args.certifier == "custom_stop" else {}),
                   "global_regions": m["n_regions"], "eps": wl.eps,
                   "parallelism": f"regions sharded over {world} GPU(s); bounds all-gathered and verdicts counted "
                                  "every step inside the timed region",
                   "l2": "flushed between timed steps", "certified": m["certified"]},
        "e2e": m["e2e"],
        "gpu_launches": int(m["prof"]["kernel_launches"]),
        "roofline": roof,
        "memory_bound": mem,
        "clocks": m["clocks"],
        "wall_s_timed": m["wall"],
    }
    if world == 1:
        out["cpu_baseline"] = _cpu_baseline_record(wl, args.certifier, args.stop_depth)
    if cifar is not None:
        croof, cmem = _roofline(cifar, wl4, "deeppoly", CIFAR_STEPS, dev)
        rec = {"metric": _metric("deeppoly"), "value": cifar["value"], "unit": "regions/s", "n_gpus": world,
               "steps": CIFAR_STEPS, "warmup": CIFAR_WARMUP, "ms_per_step": cifar["ms_max"] / CIFAR_STEPS,
               "scaling": "strong",
               "config": {"workload": wl4.name, "certifier": "deeppoly", "global_regions": cifar["n_regions"],
                          "regions_per_gpu": cifar["B"], "eps": wl4.eps,
                          "parallelism": f"{CIFAR_REGIONS} regions split over {world} GPU(s)",
                          "workspace_bytes": CIFAR_WORKSPACE, "certified": cifar["certified"],
                          "l2": "flushed between timed steps (the windows far exceed L2)"},
               "e2e": cifar["e2e"], "gpu_launches": int(cifar["prof"]["kernel_launches"]),
               "roofline": croof, "memory_bound": cmem, "clocks": cifar["clocks"], "wall_s_timed": cifar["wall"]}
        if world == 1:
            rec["cpu_baseline"] = _cpu_baseline_record(wl4, "deeppoly", 0)
        out["cifar"] = rec
    print(json.dumps(out))


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        run_cfgpu(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
