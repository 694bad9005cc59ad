#!/usr/bin/env python
"""LIF-FDE layer throughput on B200: neuron-timesteps/s, forward + backward.

Workload (one "step"): for T in (8, 16) and each scheme of the hot path -- distributed-order
GL "glmulti" (full-history gradient, learnable Softplus masses), single-order GL,
L1-2 trapezoid and the fractional predictor -- one LIFNeuronFDE layer forward and backward
on an input current [T, 16, 128, 64, 64] (8,388,608 neurons) drawn i.i.d. N(0.3, 0.5^2),
with upstream gradients N(0, 1) on the spikes (and on the membrane for the single-order
schemes, which expose it).  Inputs are larger than L2 (537 MB per [16, N] tensor), so no
L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

N > 1 runs one process per GPU under torchrun: every rank processes its own 8.4M neurons
(weak scaling) and the gradients of the shared Softplus masses are summed with one NCCL
all-reduce per step.  Rank 0 prints one JSON line.
"""
import argparse
import contextlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "df-snn-official_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "LIF-FDE neuron-timesteps/s fwd+bwd"
UNIT = "neuron-timesteps/s"
SHAPE = (16, 128, 64, 64)
TS = (8, 16)
SCHEMES = ("glmulti", "gl", "trap", "predictor")
TAU, TH, SG, H = 2.0, 1.0, 5.0, 0.1
MULTI_BETA = [0.3, 0.4, 0.5]
MASSES = [0.5, 0.5, 0.7]
BETA = 0.5
FALLBACK_HBM_GBS = 6650.0
WORKLOAD = ("LIFNeuronFDE layer fwd+bwd, schemes glmulti(full history, softplus masses)/gl/trap/"
            "predictor at T=8 and T=16, input [T,16,128,64,64] = 8,388,608 neurons per GPU, "
            "x~N(0.3,0.5^2), upstream grads N(0,1)")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--e2e-steps", type=int, default=4)
    ap.add_argument("--cpu-sample", type=int, default=1 << 22,
                    help="neurons of the bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--torch-sample", type=int, default=1 << 19,
                    help="neurons of the reference PyTorch-path CPU sample")
    ap.add_argument("--network-source", choices=("example", "restatement"), default="example",
                    help="network workloads: the reference example's own module (staged) or "
                         "this repository's restatement of it")
    ap.add_argument("--network-steps", type=int, default=10,
                    help="timed CNN128 training steps of the default line's network record")
    ap.add_argument("--no-sub-workloads", action="store_true",
                    help="skip the default line's long-history and aligned-layer records")
    ap.add_argument("--sub-steps", type=int, default=10,
                    help="timed steps of the long-history record (about 52 ms each)")
    ap.add_argument("--no-network", action="store_true",
                    help="skip the default line's CNN128 network record")
    ap.add_argument("--no-gpu-reference", action="store_true",
                    help="skip the reference's own GPU path timed on the same GPU")
    ap.add_argument("--only", default="",
                    help="profiling: comma list of scheme:T (e.g. glmulti:16) instead of all")
    ap.add_argument("--neurons", type=int, default=0,
                    help="profiling: neurons per GPU instead of 16*128*64*64")
    ap.add_argument("--workload", choices=("layers", "long", "aligned", "cnn128",
                                           "spikformer256", "history", "integrator"),
                    default="layers",
                    help="layers: the LIFNeuronFDE layer step (default); long: the "
                         "long-history layer step (T = 64, 256); aligned: the layer step with "
                         "the examples' aligned glmulti kernels; cnn128 / "
                         "spikformer256: synthetic network training step, data-parallel, "
                         "samples/s; integrator: the SNN wrapper's multi-term GL "
                         "integrator and adjoint; history: the "
                         "VO-GL1 / FAGL1 / VO-PREDICTOR Functions with per-sample tables")
    args = ap.parse_args()
    global SHAPE, COMBOS, WORKLOAD, X_MEAN, X_STD, TS
    if args.workload == "aligned":
        COMBOS = [(T, "aligned") for T in TS]
        WORKLOAD = ("LIFNeuronFDE layer fwd+bwd with the examples' aligned glmulti kernels "
                    "(AlignedGLMulti, full history, softplus masses) at T=8 and T=16, input "
                    "[T,16,128,64,64] = 8,388,608 neurons per GPU, x~N(0.3,0.5^2), upstream "
                    "grads N(0,1)")
    if args.workload == "long":
        # the long-history configuration: GL and predictor at T = 64 and 256, 4,194,304
        # neurons, input current N(0.2, 0.4^2)
        SHAPE = (16, 4194304 // 16)
        TS = (64, 256)
        COMBOS = [(T, sch) for T in TS for sch in ("gl", "predictor")]
        X_MEAN, X_STD = 0.2, 0.4
        WORKLOAD = ("LIFNeuronFDE layer fwd+bwd, schemes gl/predictor (single order, beta 0.5) at "
                    "T=64 and T=256, 4,194,304 neurons per GPU, x~N(0.2,0.4^2), upstream grads "
                    "N(0,1) on spikes and membrane")
    if args.only:
        COMBOS = [(int(c.split(":")[1]), c.split(":")[0]) for c in args.only.split(",")]
    if args.neurons:
        SHAPE = (16, args.neurons // 16)
    return args


COMBOS = [(T, sch) for T in TS for sch in SCHEMES]
X_MEAN, X_STD = 0.3, 0.5


def units_per_step(neurons):
    return sum(T * neurons for T, _ in COMBOS)


# -----------------------------------------------------------------------------------------
# CPU side: the reference's own kernel sources compiled for the host (oracle/_ref) when
# built, else the oracle port; bounded sample of the same workload, all host threads.
# -----------------------------------------------------------------------------------------
def cpu_workload_time(n_sample, seed=0):
    import numpy as np

    from oracle import oracle as O
    import torch
    from dfsnn_b200 import schedule

    kind = "reference" if O.ref_available() else "port"
    impl = "ref" if kind == "reference" else "oracle"
    O.set_num_threads(len(os.sched_getaffinity(0)))   # all host threads (torchrun exports 1)
    g = np.random.default_rng(seed)
    x16 = g.normal(0.3, 0.5, size=(16, n_sample)).astype(np.float32)
    gS16 = g.standard_normal((16, n_sample)).astype(np.float32)
    gV16 = g.standard_normal((16, n_sample)).astype(np.float32)
    v0 = np.zeros(n_sample, np.float32)
    tables = {}
    for T in TS:
        basis = schedule.glmulti_basis(MULTI_BETA, T)
        terms = schedule.build_glmulti_schedule(torch.tensor(MASSES), torch.tensor(MULTI_BETA),
                                                basis, H, T)
        tables[("glmulti", T)] = (terms["scale"].contiguous().numpy(), terms["weights"].numpy())
        tables[("gl", T)] = schedule.gl_weights(BETA, T).numpy()
        tables[("trap", T)] = schedule.trap_weights(BETA, T).numpy()
        tables[("predictor", T)] = schedule.predictor_weights(BETA, T).numpy()
    hb, g1 = schedule.predictor_constants(BETA, H)
    t0 = time.perf_counter()
    for T in TS:
        x, gS, gV = x16[:T], gS16[:T], gV16[:T]
        for sch in SCHEMES:
            if sch == "glmulti":
                scale, W = tables[(sch, T)]
                fw = O.glmulti_forward(x, v0, scale, W, TAU, TH, impl=impl)
                _, _, gpre = O.glmulti_backward(True, gS, scale, W, fw["vpre"], TAU, TH, SG, impl=impl)
                O.glmulti_param_grads(gpre, fw["drift"], fw["vhist"])
            else:
                w = tables[(sch, T)]
                s, v = O.single_forward(sch, x, v0, w, TAU, BETA, TH, hb, g1, impl=impl)
                O.single_backward(sch, gS, gV, x, v0, w, TAU, BETA, TH, SG, hb, g1, impl=impl,
                                  spike=s, vseq=v)
    dt = time.perf_counter() - t0
    return dt, kind, O.num_threads()


def cpu_torch_path_time(n_sample, seed=0):
    """The reference's own PyTorch solver path on the host cores: the unmodified reference
    LIFNeuronFDE(backend='torch') (staged in baseline/_ref; spikeDE_dis/neuron.py:1765-1788
    and the single-step schemes :2292-2637) for the same layers -- glmulti, gl, trap,
    predictor at T = 8 and 16 -- forward and backward on a sample of n_sample neurons, all
    host threads.  Returns (seconds, threads) or None when the reference is not staged."""
    import torch
    from oracle import reference_gpu
    if not reference_gpu.staged():
        return None
    threads = len(os.sched_getaffinity(0))
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    ref = reference_gpu.Reference(standin=False)
    try:
        g = torch.Generator().manual_seed(seed)
        B = 16
        shape = (16, B, n_sample // B)
        x16 = torch.randn(shape, generator=g).mul_(0.5).add_(0.3)
        gS16 = torch.randn(shape, generator=g)
        gV16 = torch.randn(shape, generator=g)
        def make():
            out = []
            for T in TS:
                for sch in SCHEMES:
                    kw = dict(tau=TAU, threshold=TH, surrogate_grad_scale=SG,
                              surrogate_function="arctan", T=T, method=sch, step_size=H,
                              batchsize=B, step_mode="m", backend="torch")
                    if sch == "glmulti":
                        kw.update(beta=MULTI_BETA[0], multi_beta=MULTI_BETA,
                                  multi_coefficient=MASSES, learn_coefficient=True,
                                  coefficient_constraint="softplus", glmulti_history_grad="full")
                    else:
                        kw.update(beta=BETA, store_v_seq=True)
                    out.append((T, sch, ref.neuron.LIFNeuronFDE(**kw)))
            return out

        def run(layers, xs, gs, gv):
            for T, sch, layer in layers:
                layer_step(layer, xs[:T], gs[:T], gv[:T], sch != "glmulti")

        # first-call overhead on separate layers (the history buffers keep their first shape)
        small = slice(0, 1)
        run(make(), x16[:, :, small], gS16[:, :, small], gV16[:, :, small])
        layers = make()
        t0 = time.perf_counter()
        run(layers, x16, gS16, gV16)
        return time.perf_counter() - t0, threads
    finally:
        ref.close()
        torch.set_num_threads(prev)


def cpu_sample_desc(n, kind):
    src = ("the reference's CUDA kernel sources compiled for the host with OpenMP "
           "(oracle/_ref); shared-parameter reductions by the oracle in double"
           if kind == "reference" else "the oracle port (oracle/lif_fde_oracle.c, OpenMP)")
    return (f"{n} neurons (of 8,388,608) of the same workload: 4 schemes x T in (8,16), "
            f"forward+backward, via {src}")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    K, W = args.steps, max(args.warmup, 3)
    # size each step so that the whole run stays within ~2 minutes
    probe_n = 1 << 14
    dt, kind, cores = cpu_workload_time(probe_n)
    per_neuron = dt / probe_n
    n = int(min(1 << 20, max(1 << 12, 90.0 / max(K + W, 1) / per_neuron)))
    n = max(256, (n // 256) * 256)
    for _ in range(W):
        cpu_workload_time(n, seed=1)
    t = 0.0
    for i in range(K):
        dt, kind, cores = cpu_workload_time(n, seed=2 + i % 3)
        t += dt
    units = units_per_step(n) * K
    value = units / t
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": K, "warmup": W, "ms_per_step": 1e3 * t / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "neurons_per_step_sample": n},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": cpu_sample_desc(n, kind)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# -----------------------------------------------------------------------------------------
# GPU side
# -----------------------------------------------------------------------------------------
def measured_hbm_peak():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(kernel, Ts):
    """DRAM bytes per launch from the committed ncu summary (profiles/ncu_traffic.json),
    averaged over the step counts the bench runs (each T runs equally often), or None."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        vals = [d[f"{kernel}_T{T}"] for T in Ts]
        return sum(vals) / len(vals)
    except Exception:
        return None


class ClockSampler:
    """SM clock, its maximum and the active clock-event reasons, sampled during the timed
    region: NVML read from a thread every 10 ms (read-only queries), else nvidia-smi.
    stop() returns {"sm_mhz": median, "sm_max_mhz", "reasons": [...], "samples", "source"}
    or None."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))

    def __init__(self, device_index, period_s=0.01):
        import threading
        import torch
        self.samples, self.proc, self.thread = [], None, None
        self.source = None
        self.halt = threading.Event()
        uuid = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self._read_nvml(pynvml, h, smax)          # fails here, not in the thread
            self.source = "nvml"

            def loop():
                while not self.halt.is_set():
                    try:
                        self._read_nvml(pynvml, h, smax)
                    except Exception:
                        return
                    self.halt.wait(period_s)
            self.samples.clear()
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.samples.clear()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", uuid], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            self.source = "nvidia-smi"
            self.first = threading.Event()
            self.reader = threading.Thread(target=self._read_smi, daemon=True)
            self.reader.start()
            self.first.wait(10.0)
        except Exception:
            self.proc = None

    def _read_nvml(self, pynvml, h, smax):
        sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
        bits = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
        self.samples.append((sm, smax, {n for n, b in self.REASONS if bits & b}))

    def _read_smi(self):
        # the first line is printed before __init__ returns, i.e. before the timed region
        for i, line in enumerate(self.proc.stdout):
            parts = [p.strip() for p in line.split(",")]
            self.first.set()
            if i == 0 or len(parts) < 9:
                continue
            try:
                sm, smax = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            names = [n for n, _ in self.REASONS]
            self.samples.append((sm, smax, {n for n, v in zip(names, parts[5:9])
                                            if v.lower().startswith("active")}))
        self.first.set()

    def stop(self):
        if self.thread is not None:
            self.halt.set()
            self.thread.join(timeout=5)
        elif self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=10)
                self.reader.join(timeout=10)
            except Exception:
                self.proc.kill()
        else:
            return None
        samples = list(self.samples)
        if not samples:
            return None
        return {"sm_mhz": statistics.median(s[0] for s in samples),
                "sm_max_mhz": max(s[1] for s in samples),
                "reasons": sorted(set().union(*(s[2] for s in samples))),
                "samples": len(samples), "source": self.source}


class StepCosts:
    """What a step spends besides its kernels, reported beside the device time per step:

    * host_ms_per_step: the host's own time to launch one step, the median over a few
      isolated steps, each started on an idle device and synchronized after it, so that the
      launch queue never fills and blocks the host (in the timed loop it does, and then the
      host's time equals the device's whatever the limit is).  A step whose host time comes
      close to its device time runs at the host's pace;
    * exchange_ms_per_step: the device time of the gradient all-reduce inside the timed steps
      (CUDA events around it on the launching stream), which includes any wait for a rank
      whose launches arrive later; exchange_ms_longest: the longest single one.

    Both are the maximum over ranks.  Every rank makes the same calls in the same order."""

    def __init__(self):
        self.spans = []
        self.on = False

    @contextlib.contextmanager
    def exchange(self):
        if not self.on:
            yield
            return
        import torch
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        yield
        e.record()
        self.spans.append((s, e))

    @staticmethod
    def host_step_ms(step, reps=5):
        import torch
        times = []
        for _ in range(reps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            step()
            times.append((time.perf_counter() - t0) * 1e3)
            torch.cuda.synchronize()
        return statistics.median(times)

    def summary(self, K, host_ms, dev, world, exchange=True):
        """Call after the timed region has been synchronized (exchange=False: the step's
        collective is not bracketed, e.g. DDP's, which runs inside backward)."""
        import torch
        import torch.distributed as dist
        spans = [s.elapsed_time(e) for s, e in self.spans]
        exch = sum(spans) / K if spans else 0.0
        t = torch.tensor([host_ms, exch, max(spans, default=0.0)], device=dev,
                         dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out = {"host_ms_per_step": round(float(t[0]), 4)}
        if world > 1 and exchange:
            out["exchange_ms_per_step"] = round(float(t[1]), 4)
            out["exchange_ms_longest"] = round(float(t[2]), 4)
        return out


def make_layers(device, combos=None, batch=None):
    from dfsnn_b200.neuron import LIFNeuronFDE
    combos = COMBOS if combos is None else combos
    batch = SHAPE[0] if batch is None else batch
    if any(sch == "aligned" for _, sch in combos):
        # the examples' aligned semantics replace the library glmulti Function for the whole
        # process, as their install() does (so "aligned" and "glmulti" never share a run)
        from dfsnn_b200 import aligned_glmulti
        aligned_glmulti.install("native")
    layers = {}
    for T, sch in combos:
        method = "glmulti" if sch == "aligned" else sch
        kw = dict(tau=TAU, threshold=TH, surrogate_grad_scale=SG, surrogate_function="arctan",
                  T=T, method=method, step_size=H, batchsize=batch, step_mode="m",
                  backend="cupy")
        if method == "glmulti":
            kw.update(beta=MULTI_BETA[0], multi_beta=MULTI_BETA, multi_coefficient=MASSES,
                      learn_coefficient=True, coefficient_constraint="softplus",
                      glmulti_history_grad="full")
        else:
            kw.update(beta=BETA, store_v_seq=True)
        layers[(T, sch)] = LIFNeuronFDE(**kw).to(device)
    return layers


def run_gpu_reference(args, x16, gS16, gV16, dev, combos=None, batch=None, max_steps=50,
                      warmup=None):
    """The reference's own GPU path on this GPU, same workload: the unmodified reference
    LIFNeuronFDE(backend='cupy') (the staged package in baseline/_ref) whose CuPy launches
    run the reference's own kernel source texts, compiled for sm_100 with its options
    (oracle/build_ref.py, launched by oracle/cupy_standin), and its own PyTorch glue
    (torch.sum / torch.matmul for the glmulti parameter gradients).  For the aligned layers
    the examples' own install('cupy') binds their AlignedGLMulti first, as make_model does.
    Same layers, inputs and step as the native arm; CUDA events on the same stream."""
    import torch
    from oracle import reference_gpu
    combos = COMBOS if combos is None else combos
    batch = SHAPE[0] if batch is None else batch
    why = reference_gpu.missing()
    if why:
        return {"unavailable": why}
    aligned = any(sch == "aligned" for _, sch in combos)
    ref = reference_gpu.Reference("cnn128" if aligned else None)
    try:
        ref.use_reference()
        if aligned:
            import aligned_glmulti as example_alg
            example_alg.install("cupy")
        layers = {}
        for T, sch in combos:
            method = "glmulti" if sch == "aligned" else sch
            kw = dict(tau=TAU, threshold=TH, surrogate_grad_scale=SG, surrogate_function="arctan",
                      T=T, method=method, step_size=H, batchsize=batch, step_mode="m",
                      backend="cupy")
            if method == "glmulti":
                kw.update(beta=MULTI_BETA[0], multi_beta=MULTI_BETA, multi_coefficient=MASSES,
                          learn_coefficient=True, coefficient_constraint="softplus",
                          glmulti_history_grad="full")
            else:
                kw.update(beta=BETA, store_v_seq=True)
            layers[(T, sch)] = ref.neuron.LIFNeuronFDE(**kw).to(dev)

        def step():
            for T, sch in combos:
                layer_step(layers[(T, sch)], x16[:T], gS16[:T], gV16[:T],
                           sch not in ("glmulti", "aligned"))

        K = min(args.steps, max_steps)
        W = max(args.warmup, 3) if warmup is None else warmup
        for _ in range(W):
            step()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(K):
            step()
        end.record()
        torch.cuda.synchronize()
        ms = start.elapsed_time(end) / K
        neurons = x16[0].numel()
        return {"value": sum(T * neurons for T, _ in combos) / (ms / 1e3), "unit": UNIT,
                "ms_per_step": ms, "steps": K, "warmup": W,
                "impl": "unmodified reference LIFNeuronFDE(backend='cupy') and autograd "
                        "Functions" + (" with the examples' AlignedGLMulti" if aligned else "") +
                        "; their kernel source texts compiled for sm_100 with the reference's "
                        "options, launched through a CuPy stand-in (driver API)"}
    finally:
        ref.close()


def layer_step(layer, x, gS, gV, single):
    """One layer forward + backward; returns the gradients of the learnable masses."""
    import torch
    layer.reset()
    x = x.detach().requires_grad_(True)
    s = layer(x)
    outs, grads = [s], [gS]
    if single:
        outs.append(layer.v_seq)
        grads.append(gV)
    params = [p for p in layer.parameters()]
    res = torch.autograd.grad(outs, [x] + params, grads)
    return res[0], s, list(res[1:])


SUB_WORKLOADS = {
    "long": dict(shape=(16, 4194304 // 16), mean=0.2, std=0.4,
                 combos=[(T, sch) for T in (64, 256) for sch in ("gl", "predictor")],
                 desc="LIFNeuronFDE gl/predictor (beta 0.5) fwd+bwd at T=64 and T=256, 4,194,304 "
                      "neurons per GPU, x~N(0.2,0.4^2), upstream grads N(0,1) on spikes and "
                      "membrane"),
    "aligned": dict(shape=(16, 128, 64, 64), mean=0.3, std=0.5,
                    combos=[(8, "aligned"), (16, "aligned")],
                    desc="LIFNeuronFDE glmulti with the examples' aligned kernels (AlignedGLMulti, "
                         "full history, learnable Softplus masses) fwd+bwd at T=8 and T=16, "
                         "8,388,608 neurons per GPU, x~N(0.3,0.5^2), upstream grads N(0,1)"),
}


def by_steps_table(timer, K, peak):
    """Per-kernel, per-T breakdown of the timed region (ms per call, fraction of HBM)."""
    return {k: {"calls_per_step": v["calls"] / K, "ms_per_call": round(v["ms_per_call"], 4),
                "frac_of_hbm": round(v["gbs"] / peak, 4) if v["gbs"] else None}
            for k, v in timer.summary_by_steps().items()}


def fp32_roofline(d, combos, neurons, K, mhz, sms):
    """Roofline of the single-order forward at T >= 64: its Kahan history chains (a fused
    multiply-add and three adds per term, in a fixed order) bound it on the FP32 lanes at
    the clock seen during the run."""
    instr = 4 * sum(neurons * T * (T - 1) // 2 for T, _ in combos)
    sec = d["ms_total"] / K / 1e3
    peak_ops = sms * 128 * mhz * 1e6
    return {"bound": "fp32", "kernel": "single_forward", "achieved": instr / sec / 1e12,
            "peak": peak_ops / 1e12, "unit": "T FP32 instructions/s (per lane)",
            "frac": instr / sec / peak_ops,
            "peak_source": f"{sms} SMs x 128 FP32 lanes x {mhz:.0f} MHz (median under load)",
            "work": "4 FP32 instructions per history term (fma + 3 add/sub, Kahan), "
                    "N*T(T-1)/2 terms per call", "traffic": None}


def measure_sub_workload(args, kind, K, W, dev, world, rank, gpu_reference=False):
    """Device-timed record of one more layer configuration at this N (same step, timing
    and max-over-ranks rule as the headline): the long-history configuration or the
    examples' aligned glmulti layer."""
    import torch
    from dfsnn_b200 import fde_kernels
    from dfsnn_b200.distributed import allreduce_flat
    cfg = SUB_WORKLOADS[kind]
    combos, shape = cfg["combos"], cfg["shape"]
    neurons = math.prod(shape)
    tmax = max(T for T, _ in combos)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x = torch.randn((tmax,) + shape, device=dev, generator=g).mul_(cfg["std"]).add_(cfg["mean"])
    gS = torch.randn((tmax,) + shape, device=dev, generator=g)
    gV = torch.randn((tmax,) + shape, device=dev, generator=g)
    library = fde_kernels.LIFFDEGLMultiFunction
    try:
        layers = make_layers(dev, combos, shape[0])

        def compute():
            grads = []
            for T, sch in combos:
                _, _, pg = layer_step(layers[(T, sch)], x[:T], gS[:T], gV[:T],
                                      sch not in ("glmulti", "aligned"))
                grads += pg
            return grads

        def exchanger(costs):
            def exchange(grads):
                if world > 1 and grads:
                    with costs.exchange():
                        allreduce_flat(grads)
            return exchange

        ecosts = StepCosts()
        eexchange = exchanger(ecosts)

        def estep():
            grads = compute()
            eexchange(grads)

        ms_eager, timer, clk_eager = timed_region(estep, K, W, dev, world, ecosts)
        eager_costs = ecosts.summary(K, ecosts.host_step_ms(estep), dev, world)
        gcosts = StepCosts()
        graph, gstep, per_replay = graph_step(compute, exchanger(gcosts), dev)
        ms, _, clk = timed_region(gstep, K, W, dev, world, gcosts, timer=False)
        step_costs = gcosts.summary(K, gcosts.host_step_ms(gstep), dev, world)
        del graph, gstep
    finally:
        fde_kernels.LIFFDEGLMultiFunction = library
    summary = timer.summary()
    peak, peak_src = measured_hbm_peak()
    kernels = {k: {"calls_per_step": v["calls"] / K, "ms_per_call": round(v["ms_per_call"], 4),
                   "gbs": round(v["gbs"], 1) if v["gbs"] else None,
                   "frac_of_hbm": round(v["gbs"] / peak, 4) if v["gbs"] else None}
               for k, v in summary.items()}
    if kind == "long" and "single_forward" in summary:
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        roofline = fp32_roofline(summary["single_forward"], combos, neurons, K,
                                 (clk_eager or {}).get("sm_mhz") or 1965.0, sms)
        roofline["hbm_frac_of_measured"] = kernels["single_forward"]["frac_of_hbm"]
    else:
        name, d = max(summary.items(), key=lambda kv: kv[1]["ms_total"])
        roofline = {"bound": "hbm", "kernel": name, "achieved": d["gbs"], "peak": peak,
                    "unit": "GB/s", "frac": d["gbs"] / peak if d["gbs"] else None,
                    "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_src})",
                    "algorithmic_bytes_per_launch": d["bytes_per_call"],
                    "traffic": ncu_traffic(name, sorted({T for T, _ in combos}))}
    units = sum(T * neurons for T, _ in combos)
    rec = {"workload": cfg["desc"], "value": world * K * units / (ms / 1e3), "unit": UNIT,
           "ms_per_step": ms / K, "steps": K, "warmup": W, "n_gpus": world,
           "launch": LAUNCH_DESC, "gpu_launches": per_replay * K, "roofline": roofline,
           "kernels": kernels, "kernels_by_T": by_steps_table(timer, K, peak),
           "step_costs": step_costs, "clocks": clk,
           "eager": {"value": world * K * units / (ms_eager / 1e3), "ms_per_step": ms_eager / K,
                     "gpu_launches": timer.total_launches(), "step_costs": eager_costs,
                     "clocks": clk_eager}}
    if world == 1 and gpu_reference:
        # the reference's own GPU path on the same layers and inputs (bounded steps)
        long_t = kind == "long"      # about a second per reference step: bounded sample
        gref = run_gpu_reference(args, x, gS, gV, dev, combos, shape[0],
                                 max_steps=3 if long_t else K, warmup=1 if long_t else None)
        if gref.get("value"):
            # like for like: this library's eager steps against the reference's eager steps;
            # the CUDA-graph replay of the same steps beside it
            gref["native_over_reference"] = rec["eager"]["value"] / gref["value"]
            gref["graph_over_reference"] = rec["value"] / gref["value"]
        rec["gpu_reference"] = gref
    return rec


LAUNCH_DESC = ("each step's compute (the layers' forward and backward) replayed from a CUDA graph "
               "captured once; the gradient all-reduce (world > 1) issued after each replay; "
               "per-kernel durations and the roofline from an eager region of the same steps")


def timed_region(step, K, W, dev, world, costs, timer=True):
    """W untimed steps, then K steps between two CUDA events on the launching stream, with a
    synchronize and (world > 1) a barrier on both sides and the SM clocks sampled meanwhile.
    Returns (ms for the K steps, max over ranks; the NativeCallTimer of the region or None;
    the clock record).  `costs` brackets the region's exchanges (StepCosts)."""
    import torch
    import torch.distributed as dist
    from dfsnn_b200 import profiling
    for _ in range(W):
        step()
    clocks = ClockSampler(dev.index)     # NVML set-up (milliseconds) before the start line
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    tm = profiling.NativeCallTimer() if timer else contextlib.nullcontext()
    torch.cuda.synchronize()
    start_line(dev, world)
    with tm:
        costs.on = True
        start.record()
        for _ in range(K):
            step()
        end.record()
        costs.on = False
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    t = torch.tensor([start.elapsed_time(end)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), (tm if timer else None), clk


def graph_step(compute, exchange, dev):
    """A step whose compute -- the layers' forward and backward, every native kernel and the
    PyTorch glue between them -- is captured once into a CUDA graph (after three eager runs
    on a side stream, as capture requires) and replayed; the exchange (the NCCL all-reduce
    of the parameter gradients when world > 1) stays outside the graph and runs after each
    replay on the captured outputs, which every replay rewrites.  The host then launches one
    graph per step instead of about twenty native kernels and their glue, so its launch cost
    (0.25-0.36 ms per layer forward + backward) no longer paces the device when several
    ranks share the host's cores.  Returns (graph, step, native kernels per replay)."""
    import torch
    from dfsnn_b200 import profiling
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(3):
            compute()
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with profiling.NativeCallTimer() as timer:
        with torch.cuda.graph(graph):
            out = compute()

    def step():
        graph.replay()
        exchange(out)
        return out
    return graph, step, timer.captured_launches()


def start_line(dev, world):
    """Line the ranks up for a timed region: a host barrier, then a one-element all-reduce on
    the launching stream right before the region's start event, so that on every rank the
    event fires when the last rank has arrived (host skew after the barrier -- a rank's
    thread descheduled for a few milliseconds -- stays out of the max over ranks)."""
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
        dist.all_reduce(torch.zeros(1, device=dev))


def start_ranks(dev, world):
    """The NCCL process group for world > 1, with NCCL's INFO log on for its INIT subsystem
    (one "Init COMPLETE" line per rank, with its transport choices), also where the
    environment sets another level or subsystem list."""
    from dfsnn_b200.distributed import init_process_group
    if world > 1:
        os.environ["NCCL_DEBUG"] = "INFO"
        os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
        init_process_group("nccl", timeout_s=300, device=dev)


def finish_ranks(line, rank, world):
    """Tear the process group down, then rank 0 prints the one JSON line.  NCCL writes its
    teardown lines to stdout as well, at the destroy and again at process exit, so with
    world > 1 the line comes a second after the destroy (which every rank has reached
    through the same barrier) and every rank then leaves with os._exit(0) once its streams
    are flushed: no exit-time output can follow the line."""
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:
            time.sleep(1.0)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


def run_native(args):
    import torch
    from dfsnn_b200.distributed import allreduce_flat

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    start_ranks(dev, world)
    K, W = args.steps, max(args.warmup, 3)
    neurons = math.prod(SHAPE)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    TMAX = max(T for T, _ in COMBOS)
    x16 = torch.randn((TMAX,) + SHAPE, device=dev, generator=g).mul_(X_STD).add_(X_MEAN)
    gS16 = torch.randn((TMAX,) + SHAPE, device=dev, generator=g)
    gV16 = torch.randn((TMAX,) + SHAPE, device=dev, generator=g)
    layers = make_layers(dev)

    def compute():
        mass_grads = []
        for T, sch in COMBOS:
            _, _, pg = layer_step(layers[(T, sch)], x16[:T], gS16[:T], gV16[:T],
                                  sch not in ("glmulti", "aligned"))
            mass_grads += pg
        return mass_grads

    def exchanger(costs):
        def exchange(grads):
            if world > 1:
                with costs.exchange():
                    allreduce_flat(grads)    # the one gradient exchange per step
        return exchange

    # eager region: every native call bracketed by CUDA events (per-kernel durations)
    ecosts = StepCosts()
    eexchange = exchanger(ecosts)

    def estep():
        grads = compute()
        eexchange(grads)
        return grads

    ms_eager, timer, clk_eager = timed_region(estep, K, W, dev, world, ecosts)
    eager_costs = ecosts.summary(K, ecosts.host_step_ms(estep), dev, world)
    # the headline region: the same steps with their compute replayed from a CUDA graph
    gcosts = StepCosts()
    graph, gstep, per_replay = graph_step(compute, exchanger(gcosts), dev)
    ms_max, _, clk = timed_region(gstep, K, W, dev, world, gcosts, timer=False)
    step_costs = gcosts.summary(K, gcosts.host_step_ms(gstep), dev, world)
    del graph, gstep
    value = world * K * units_per_step(neurons) / (ms_max / 1e3)
    summary = timer.summary()
    launches = per_replay * K
    eager = {"value": world * K * units_per_step(neurons) / (ms_eager / 1e3),
             "ms_per_step": ms_eager / K, "gpu_launches": timer.total_launches(),
             "step_costs": eager_costs, "clocks": clk_eager,
             "launch": "eager: every layer's native calls and PyTorch glue launched from the "
                       "host each step; the per-kernel durations below are this region's"}

    # dominant kernel (largest device time in the timed region) and its roofline
    dom = max(summary.items(), key=lambda kv: kv[1]["ms_total"]) if summary else None
    peak, peak_src = measured_hbm_peak()
    roofline = None
    if dom is not None:
        name, d = dom
        achieved = d["gbs"]
        roofline = {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": peak,
                    "unit": "GB/s", "frac": achieved / peak if achieved else None,
                    "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_src})",
                    "algorithmic_bytes_per_launch": d["bytes_per_call"],
                    "traffic": ncu_traffic(name, sorted({T for T, _ in COMBOS}))}
    if args.workload == "long" and "single_forward" in summary:
        # T >= 64: the forward's Kahan history chains are FP32-bound (no tensor cores apply)
        d = summary["single_forward"]
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        roofline = fp32_roofline(d, COMBOS, neurons, K,
                                 (clk_eager or {}).get("sm_mhz") or 1965.0, sms)
        roofline["hbm_frac_of_measured"] = d["gbs"] / peak if d["gbs"] else None
    kernels = {k: {"calls_per_step": v["calls"] / K, "ms_per_call": round(v["ms_per_call"], 4),
                   "gbs": round(v["gbs"], 1) if v["gbs"] else None,
                   "frac_of_hbm": round(v["gbs"] / peak, 4) if v["gbs"] else None}
               for k, v in summary.items()}

    # end to end through the public API with host buffers (pinned), copies timed (the
    # headline layer workload; the long-history workload is measured on the device only)
    e2e = run_e2e(args, layers, x16, gS16, gV16, dev, world) if args.workload == "layers" else None

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "neurons_per_gpu": neurons, "T": list(TS),
                   "schemes": list(SCHEMES), "l2": "inputs larger than L2 (no flush)",
                   "parallelism": f"dp{world}" + (" (one NCCL all-reduce of the mass grads per step)"
                                                  if world > 1 else ""),
                   "launch": LAUNCH_DESC},
        "gpu_launches": launches,
        "roofline": roofline,
        "kernels": kernels,
        "kernels_by_T": by_steps_table(timer, K, peak),
        "step_costs": step_costs,
        "eager": eager,
        "clocks": clk,
        "e2e": e2e,
    }
    if rank == 0 and world == 1 and args.workload == "layers" and not args.no_gpu_reference:
        gref = run_gpu_reference(args, x16, gS16, gV16, dev)
        if gref.get("value"):
            gref["native_over_reference"] = eager["value"] / gref["value"]    # eager vs eager
            gref["graph_over_reference"] = value / gref["value"]
        line["gpu_reference"] = gref
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "layers":
        n = args.cpu_sample
        dt, kind, cores = cpu_workload_time(n)
        line["cpu_baseline"] = {"value": units_per_step(n) / dt, "unit": UNIT, "cores": cores,
                                "kind": kind, "sample": cpu_sample_desc(n, kind)}
        nt = max(16, args.torch_sample // 16 * 16)
        tp = cpu_torch_path_time(nt)
        if tp is not None:
            line["cpu_baseline"]["torch_path"] = {
                "value": units_per_step(nt) / tp[0], "unit": UNIT, "cores": tp[1],
                "kind": "reference",
                "sample": f"{nt} neurons (of 8,388,608) of the same workload through the "
                          "unmodified reference LIFNeuronFDE(backend='torch') (its PyTorch "
                          "solver path, truncated-history autograd), forward+backward, "
                          "torch.set_num_threads(all host threads)"}
    if args.workload == "layers" and not args.no_sub_workloads:
        # the long-history configuration and the examples' aligned layer, at this N too
        del x16, gS16, gV16
        layers.clear()
        torch.cuda.empty_cache()
        for kind, Ks in (("long", max(1, min(K, args.sub_steps))), ("aligned", K)):
            line[kind] = measure_sub_workload(args, kind, Ks, W, dev, world, rank,
                                              gpu_reference=not args.no_gpu_reference)
        # the history-table Functions (every N) and the SNN wrapper's GL integrator (one GPU)
        line["history"] = measure_history(args, dev, world, rank, K, W)
        if world == 1:
            line["integrator"] = measure_integrator(args, dev, max(1, min(K, args.sub_steps)), W)
    if args.workload == "layers" and not args.no_network:
        # the network configuration at every N: CNN128 synthetic training, data-parallel
        Kn = max(1, args.network_steps)
        net = measure_network(args, "cnn128", dev, world, local, False, Kn, 3, args.network_source)
        net["amp"] = measure_network(args, "cnn128", dev, world, local, True, Kn, 3,
                                     args.network_source)
        if args.network_source == "example" and not args.no_gpu_reference:
            # the same example network with the reference's own GPU kernels, same N
            refnet = measure_network(args, "cnn128", dev, world, local, False, Kn, 3,
                                     "example-reference")
            if "value" in refnet:
                refnet["amp"] = measure_network(args, "cnn128", dev, world, local, True, Kn, 3,
                                                "example-reference")
            net["reference_kernels"] = refnet
        line["network"] = net
        # the second network configuration: Spikformer256 (T = 8), same measurements
        spk = measure_network(args, "spikformer256", dev, world, local, False, Kn, 3,
                              args.network_source)
        spk["amp"] = measure_network(args, "spikformer256", dev, world, local, True, Kn, 3,
                                     args.network_source)
        if args.network_source == "example" and not args.no_gpu_reference:
            refspk = measure_network(args, "spikformer256", dev, world, local, False, Kn, 3,
                                     "example-reference")
            spk["reference_kernels"] = refspk
        line["network_spikformer256"] = spk
    finish_ranks(line, rank, world)
    return 0


def run_e2e(args, layers, x16, gS16, gV16, dev, world):
    """Same step through LIFNeuronFDE with host inputs.  Every step copies the step's inputs
    from pinned host memory -- the input current and the upstream gradients, one [16, N]
    array each, whose first T rows feed the T-step layers exactly as in the device-timed
    run -- and reads the step's results back: the gradients of the learnable Softplus masses
    and the spike count of every layer (the layers' spike and input-gradient tensors stay on
    the device, as they do between the layers of a network).  The next step's inputs stream
    in on a copy stream into a second buffer set while this step computes; events order
    every buffer reuse."""
    import torch
    import torch.distributed as dist
    from dfsnn_b200.distributed import allreduce_flat
    steps = max(1, args.e2e_steps)
    hx = x16.cpu().pin_memory()
    hgS = gS16.cpu().pin_memory()
    hgV = gV16.cpu().pin_memory()
    need_gv = any(sch not in ("glmulti", "aligned") for _, sch in COMBOS)
    bufs = [(torch.empty_like(x16), torch.empty_like(gS16), torch.empty_like(gV16))
            for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    h2d_s = torch.cuda.Stream(dev)
    done = [None, None]          # compute-done event of the last step that used each buffer
    counts = {"h2d": 0, "d2h": 0}
    host_res = None

    def issue_h2d(i):
        dx, dgS, dgV = bufs[i % 2]
        with torch.cuda.stream(h2d_s):
            if done[i % 2] is not None:
                h2d_s.wait_event(done[i % 2])
            dx.copy_(hx, non_blocking=True)
            dgS.copy_(hgS, non_blocking=True)
            n = 2 * hx.numel() * 4
            if need_gv:
                dgV.copy_(hgV, non_blocking=True)
                n += hgV.numel() * 4
            ev = torch.cuda.Event()
            ev.record(h2d_s)
        counts["h2d"] = n
        return ev

    def one(i, ev_in):
        nonlocal host_res
        comp.wait_event(ev_in)
        dx, dgS, dgV = bufs[i % 2]
        mass_grads, spike_counts = [], []
        for T, sch in COMBOS:
            _, s, pg = layer_step(layers[(T, sch)], dx[:T], dgS[:T], dgV[:T],
                                  sch not in ("glmulti", "aligned"))
            mass_grads += pg
            spike_counts.append(s.sum().reshape(1))
        if world > 1:
            allreduce_flat(mass_grads)       # the step's one gradient exchange, as in `value`
        cev = torch.cuda.Event()
        cev.record(comp)
        done[i % 2] = cev
        res = torch.cat([g.reshape(-1) for g in mass_grads] + spike_counts)
        if host_res is None:
            host_res = torch.empty(res.shape, dtype=res.dtype).pin_memory()
        host_res.copy_(res, non_blocking=True)   # the step's result, read back every step
        counts["d2h"] = res.numel() * res.element_size()

    ev = issue_h2d(0)
    one(0, ev)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start_line(dev, world)             # on `comp`, the current stream
    start.record(comp)
    h2d_s.wait_stream(comp)
    ev = issue_h2d(1)
    for i in range(1, steps + 1):
        ev_next = issue_h2d(i + 1) if i < steps else None
        one(i, ev)
        ev = ev_next
    end.record(comp)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    value = world * steps * units_per_step(math.prod(SHAPE)) / (float(t.item()) / 1e3)
    return {"value": value, "unit": UNIT, "h2d_bytes_per_step": counts["h2d"],
            "d2h_bytes_per_step": counts["d2h"], "steps": steps,
            "copies": "each step's inputs (x, grad_spike, grad_v: [16, N] fp32 each) host to "
                      "device, the next step's overlapping this step's compute; the step's "
                      "result (mass gradients, per-layer spike counts) device to host"}


# -----------------------------------------------------------------------------------------
# CNN128 synthetic training (the network configuration of the examples, data-parallel)
# -----------------------------------------------------------------------------------------
CNN_T, CNN_B, CNN_CLASSES = 16, 16, 11


def glmulti_neuron_factory(T, B):
    """LIFNeuronFDE layers as the examples configure them: glmulti with aligned semantics
    (installed as the examples do), full-history gradient, one Softplus mass parameter
    shared by every layer (examples/cnn128/cnn128_aligned.py:14-19)."""
    import torch
    import torch.nn as nn
    from dfsnn_b200 import aligned_glmulti
    from dfsnn_b200.neuron import LIFNeuronFDE
    aligned_glmulti.install("native")
    raw = nn.Parameter(torch.log(torch.expm1(torch.tensor(MASSES))))

    def neuron(name):
        return LIFNeuronFDE(tau=2.0, threshold=1.0, surrogate_grad_scale=5.0,
                            surrogate_function="arctan", beta=MULTI_BETA[0], T=T,
                            method="glmulti", step_size=0.1, batchsize=B, name=name,
                            backend="cupy", step_mode="m", multi_beta=MULTI_BETA,
                            multi_coefficient=MASSES, learn_coefficient=True,
                            coefficient_constraint="softplus", shared_multi_coefficient=raw,
                            coefficient_update_interval=1, glmulti_history_grad="full")

    return neuron


SPK_T, SPK_B, SPK_CLASSES, SPK_DIM, SPK_DEPTH, SPK_HEADS = 8, 16, 300, 256, 2, 16


def make_spikformer256(dev):
    """The direct-FDE Spikformer of the reference examples (examples/spikformer_har_lip/
    model.py:726-960, spikformer_e256_lif_fde: embed 256, depth 2, 16 heads, MLP ratio 4):
    SPS patch embedding (four Conv3x3-BN-LIF-MaxPool(3,2,1) stages 2->32->64->128->256, then a
    Conv3x3-BN-LIF relative position embedding added to its input: 8x8 = 64 tokens), two
    blocks of spiking self-attention (1x1 Conv1d-BN-LIF for q, k, v; (q k^T) v * 0.25; LIF;
    Conv1d-BN-LIF projection) and MLP (Conv1d 256->1024-BN-LIF, 1024->256-BN-LIF) with
    residuals and drop path 0.1*i/(depth-1), and the head: mean over tokens, Linear per
    time step, mean over time.  Every LIF is the glmulti neuron of the CNN128 configuration
    at T=8.  Layers applied per frame run on all T*B frames at once (the reference's
    _time_distributed, :421-427)."""
    import torch
    import torch.nn as nn
    from dfsnn_b200.neuron import LIFNeuronFDE
    neuron = glmulti_neuron_factory(SPK_T, SPK_B)

    def td(module, x):
        T, B = x.shape[:2]
        y = module(x.flatten(0, 1))
        return y.reshape((T, B) + tuple(y.shape[1:]))

    class DropPath(nn.Module):
        def __init__(self, p):
            super().__init__()
            self.p = p

        def forward(self, x):
            if self.p == 0.0 or not self.training:
                return x
            keep = 1.0 - self.p
            mask = x.new_empty((x.shape[0],) + (1,) * (x.dim() - 1)).bernoulli_(keep)
            return x * mask / keep

    class SPS(nn.Module):
        def __init__(self, dim):
            super().__init__()
            chans = [2, dim // 8, dim // 4, dim // 2, dim]
            self.convs = nn.ModuleList(nn.Conv2d(chans[i], chans[i + 1], 3, padding=1, bias=False)
                                       for i in range(4))
            self.bns = nn.ModuleList(nn.BatchNorm2d(chans[i + 1]) for i in range(4))
            self.lifs = nn.ModuleList(neuron(f"patch_lif{i + 1}") for i in range(4))
            self.pool = nn.MaxPool2d(3, stride=2, padding=1)
            self.rpe_conv = nn.Conv2d(dim, dim, 3, padding=1, bias=False)
            self.rpe_bn = nn.BatchNorm2d(dim)
            self.rpe_lif = neuron("rpe_lif")

        def forward(self, x):
            for conv, bn, lif in zip(self.convs, self.bns, self.lifs):
                x = td(self.pool, lif(td(bn, td(conv, x))))
            x = x + self.rpe_lif(td(self.rpe_bn, td(self.rpe_conv, x)))
            T, B, C, H, W = x.shape
            return x.reshape(T, B, C, H * W)

    class SSA(nn.Module):
        def __init__(self, dim, heads):
            super().__init__()
            self.dim, self.heads = dim, heads
            self.qkv = nn.ModuleList(nn.Conv1d(dim, dim, 1, bias=False) for _ in range(3))
            self.qkv_bn = nn.ModuleList(nn.BatchNorm1d(dim) for _ in range(3))
            self.qkv_lif = nn.ModuleList(neuron(n) for n in ("q_lif", "k_lif", "v_lif"))
            self.attn_lif = neuron("attn_lif")
            self.proj = nn.Conv1d(dim, dim, 1)
            self.proj_bn = nn.BatchNorm1d(dim)
            self.proj_lif = neuron("proj_lif")

        def forward(self, x):
            heads = []
            for conv, bn, lif in zip(self.qkv, self.qkv_bn, self.qkv_lif):
                y = lif(td(bn, td(conv, x)))
                T, B, C, N = y.shape
                heads.append(y.transpose(-1, -2).reshape(T, B, N, self.heads, C // self.heads)
                             .permute(0, 1, 3, 2, 4))
            q, k, v = heads
            x = ((q @ k.transpose(-2, -1)) @ v) * 0.25
            T, B, _, N, _ = x.shape
            x = self.attn_lif(x.permute(0, 1, 2, 4, 3).reshape(T, B, self.dim, N))
            return self.proj_lif(td(self.proj_bn, td(self.proj, x)))

    class MLP(nn.Module):
        def __init__(self, dim, hidden):
            super().__init__()
            self.fc1, self.bn1, self.lif1 = nn.Conv1d(dim, hidden, 1), nn.BatchNorm1d(hidden), neuron("mlp_lif1")
            self.fc2, self.bn2, self.lif2 = nn.Conv1d(hidden, dim, 1), nn.BatchNorm1d(dim), neuron("mlp_lif2")

        def forward(self, x):
            x = self.lif1(td(self.bn1, td(self.fc1, x)))
            return self.lif2(td(self.bn2, td(self.fc2, x)))

    class Block(nn.Module):
        def __init__(self, dim, heads, drop):
            super().__init__()
            self.attn, self.mlp, self.drop = SSA(dim, heads), MLP(dim, 4 * dim), DropPath(drop)

        def forward(self, x):
            x = x + td(self.drop, self.attn(x))
            return x + td(self.drop, self.mlp(x))

    class Spikformer(nn.Module):
        def __init__(self):
            super().__init__()
            self.patch_embed = SPS(SPK_DIM)
            self.blocks = nn.ModuleList(Block(SPK_DIM, SPK_HEADS, 0.1 * i / max(1, SPK_DEPTH - 1))
                                        for i in range(SPK_DEPTH))
            self.head = nn.Linear(SPK_DIM, SPK_CLASSES)
            self.apply(self._init_weights)

        @staticmethod
        def _init_weights(m):                  # as the reference model (model.py:899-910)
            if isinstance(m, nn.Conv2d):
                nn.init.kaiming_normal_(m.weight, mode="fan_out", nonlinearity="relu")
            elif isinstance(m, (nn.BatchNorm1d, nn.BatchNorm2d)):
                nn.init.constant_(m.weight, 1)
                nn.init.constant_(m.bias, 0)
            elif isinstance(m, nn.Linear):
                nn.init.trunc_normal_(m.weight, std=0.02)
                if m.bias is not None:
                    nn.init.constant_(m.bias, 0)

        def forward(self, x):
            x = self.patch_embed(x)
            for blk in self.blocks:
                x = blk(x)
            return self.head(x.mean(-1)).mean(0)

        def reset(self):
            for m in self.modules():
                if isinstance(m, LIFNeuronFDE):
                    m.reset()

    return Spikformer().to(dev)


def make_cnn128(dev):
    """The CNN128 topology of the reference examples (examples/cnn128/cnn128_aligned.py:8-40):
    five blocks Conv2d(3x3, 128, no bias) -> BatchNorm2d -> LIFNeuronFDE -> MaxPool2d(2), then
    Flatten, Dropout(0.5), Linear(2048, 512), LIF, Dropout(0.5), Linear(512, 256), LIF,
    Linear(256, classes); every LIF layer is glmulti with aligned semantics (installed as
    the examples do), full-history gradient and one shared Softplus mass parameter.  Frame
    layers run on all T frames at once (the reference loops over frames: same math), batch
    norm per frame as in the reference; output = mean over time."""
    import torch
    import torch.nn as nn
    from dfsnn_b200.neuron import LIFNeuronFDE
    neuron = glmulti_neuron_factory(CNN_T, CNN_B)

    class CNN128(nn.Module):
        def __init__(self):
            super().__init__()
            blocks = []
            for i in range(5):
                blocks += [("frames", nn.Conv2d(2 if i == 0 else 128, 128, 3, padding=1, bias=False)),
                           ("per_frame", nn.BatchNorm2d(128)), ("lif", neuron(f"conv{i}")),
                           ("frames", nn.MaxPool2d(2))]
            blocks += [("frames", nn.Flatten()), ("frames", nn.Dropout(0.5)),
                       ("frames", nn.Linear(128 * 4 * 4, 512)), ("lif", neuron("fc0")),
                       ("frames", nn.Dropout(0.5)), ("frames", nn.Linear(512, 256)),
                       ("lif", neuron("fc1")), ("frames", nn.Linear(256, CNN_CLASSES))]
            self.kinds = [k for k, _ in blocks]
            self.layers = nn.ModuleList([m for _, m in blocks])

        def forward(self, x):
            T, B = x.shape[:2]
            for kind, layer in zip(self.kinds, self.layers):
                if kind == "lif":
                    x = layer(x)
                elif kind == "per_frame":
                    x = torch.stack([layer(f) for f in x])
                else:
                    y = layer(x.flatten(0, 1))
                    x = y.reshape((T, B) + tuple(y.shape[1:]))
            return x.mean(0)

        def reset(self):
            for m in self.modules():
                if isinstance(m, LIFNeuronFDE):
                    m.reset()

    return CNN128().to(dev)


NETWORKS = {
    # name: (builder, T, B, classes, frame kind, description)
    "cnn128": ("make_cnn128", CNN_T, CNN_B, CNN_CLASSES, "poisson",
               "CNN128 (5x conv128-BN-LIF-pool, fc512-LIF, fc256-LIF, fc11) training step, AdamW, "
               "LIFNeuronFDE glmulti aligned full history, shared Softplus masses, T=16, B=16 per "
               "GPU, frames [16,16,2,128,128] Bernoulli(0.05)*Poisson(1), 11 classes"),
    "spikformer256": ("make_spikformer256", SPK_T, SPK_B, SPK_CLASSES, "bernoulli",
                      "Spikformer256 (SPS 2->256, 64 tokens, depth 2, 16 heads, MLP 1024) "
                      "training step, AdamW, LIFNeuronFDE glmulti aligned full history, shared "
                      "Softplus masses, T=8, B=16 per GPU, frames [8,16,2,128,128] "
                      "Bernoulli(0.05), 300 classes"),
}


def run_cnn128(args):
    return run_network(args, "cnn128")


EXAMPLE_DIRS = {"cnn128": "cnn128", "spikformer256": "spikformer_har_lip"}


def example_network(name, dev, reference_kernels=False):
    """The reference example itself, unmodified (staged in baseline/_ref), with this library
    installed the documented way: integrate.install() before the model is built, the
    example's own make_model() (which calls its install('cupy')), then
    integrate.rebind_aligned().  The reference is imported without any CuPy, so none of its
    own kernels can run.  With reference_kernels the same example runs its own aligned
    kernels instead (the reference's GPU path, through the CuPy stand-in of oracle/, the
    reference arm's infrastructure).  Returns (model, reset, close) or None when the example
    (or, for reference_kernels, the prebuilt reference kernels) is missing."""
    from oracle import reference_gpu
    if not reference_gpu.staged() or (reference_kernels and reference_gpu.missing()):
        return None
    from dfsnn_b200 import fde_kernels, integrate
    library = fde_kernels.LIFFDEGLMultiFunction      # before the example's install() patches it
    ref = reference_gpu.Reference(EXAMPLE_DIRS[name], standin=reference_kernels)
    if reference_kernels:
        ref.use_reference()
    else:
        ref.use_native()
    if name == "cnn128":
        import aligned_glmulti as alg
        import cnn128_aligned
        model = cnn128_aligned.make_model("cupy", MULTI_BETA, True, MASSES, batch=CNN_B, T=CNN_T,
                                          num_classes=CNN_CLASSES)
    else:
        import aligned_glmulti as alg
        model = alg.make_model("cupy", MULTI_BETA, True, MASSES, batch=SPK_B, T=SPK_T,
                               num_classes=SPK_CLASSES)
    if not reference_kernels:
        integrate.rebind_aligned(alg)
    model = model.to(dev)
    lifs = [m for m in model.modules() if isinstance(m, ref.neuron.LIFNeuronFDE)]

    def reset():
        for m in lifs:
            m.reset()

    def close():
        fde_kernels.LIFFDEGLMultiFunction = library
        ref.close()
    return model, reset, close


def measure_network(args, name, dev, world, local, amp, K, W, source="example"):
    """Synthetic training steps of CNN128 / Spikformer256, data-parallel (DDP over NCCL for
    world > 1, B per GPU), AdamW as the reference trainer (train_transformer.py:131), fp32
    or under autocast fp16 with a gradient scaler as the reference trainer runs by default
    (train_transformer.py:111, 469-488).  Returns the record (every rank takes the same
    collective steps)."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F
    from dfsnn_b200 import profiling
    torch.manual_seed(1234)                    # the same initial weights on every rank
    _, NT, NB, NCLS, frame_kind, desc = NETWORKS[name]
    if source == "example-reference":
        built = example_network(name, dev, reference_kernels=True)
        if built is None:
            return {"unavailable": "the staged reference example or its prebuilt kernels are missing"}
    else:
        built = example_network(name, dev) if source == "example" else None
    if built is None:
        source = "restatement"
        model = globals()[NETWORKS[name][0]](dev)
        reset, close = model.reset, (lambda: None)
    else:
        model, reset, close = built
    try:
        scaler = torch.amp.GradScaler("cuda", enabled=amp)
        g = torch.Generator(device=dev).manual_seed(99 + int(os.environ.get("RANK", "0")))
        shape = (NT, NB, 2, 128, 128)
        frames = (torch.rand(shape, device=dev, generator=g) < 0.05).float()
        if frame_kind == "poisson":
            frames = frames * torch.poisson(torch.ones(shape, device=dev), generator=g)
        labels = torch.randint(0, NCLS, (NB,), device=dev, generator=g)

        def make_step(net, opt):
            def step():
                reset()
                with torch.autocast("cuda", dtype=torch.float16, enabled=amp):
                    loss = F.cross_entropy(net(frames), labels)
                opt.zero_grad(set_to_none=True)
                scaler.scale(loss).backward()
                scaler.step(opt)
                scaler.update()
                return loss
            return step

        replica = None
        if world > 1 and not amp:
            # the bare module trained on every rank at once with no collective (before the
            # DDP wrap, whose construction then broadcasts rank 0's parameters): the step
            # time each GPU reaches while the ranks share the node but wait for no one
            rstep = make_step(model, torch.optim.AdamW(model.parameters(), lr=1e-4))
            for _ in range(W):
                rstep()
            torch.cuda.synchronize()
            dist.barrier()
            r0 = torch.cuda.Event(enable_timing=True)
            r1 = torch.cuda.Event(enable_timing=True)
            r0.record()
            for _ in range(K):
                rstep()
            r1.record()
            torch.cuda.synchronize()
            tr = torch.tensor([r0.elapsed_time(r1) / K], device=dev, dtype=torch.float64)
            gathered = [torch.zeros_like(tr) for _ in range(world)]
            dist.all_gather(gathered, tr)
            replica = [round(float(x.item()), 3) for x in gathered]
            del rstep
            model.zero_grad(set_to_none=True)
        net = model
        if world > 1:
            net = torch.nn.parallel.DistributedDataParallel(
                model, device_ids=[local], broadcast_buffers=False,
                gradient_as_bucket_view=True, static_graph=True)
        opt = torch.optim.AdamW(model.parameters(), lr=1e-4)
        step = make_step(net, opt)

        for _ in range(W):
            step()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start_line(dev, world)
        with profiling.NativeCallTimer() as timer:
            start.record()
            for _ in range(K):
                loss = step()
            end.record()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms_rank = start.elapsed_time(end)
        t = torch.tensor([ms_rank], device=dev, dtype=torch.float64)
        per_rank = [ms_rank]
        allreduce = None
        nparams = sum(p.numel() for p in model.parameters())
        if world > 1:
            gathered = [torch.zeros_like(t) for _ in range(world)]
            dist.all_gather(gathered, t)
            per_rank = [float(x.item()) for x in gathered]
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            # the gradient exchange alone: one all-reduce of all parameters (fp32)
            buf = torch.zeros(nparams, device=dev)
            for _ in range(3):
                dist.all_reduce(buf)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                dist.all_reduce(buf)
            e1.record()
            torch.cuda.synchronize()
            allreduce = e0.elapsed_time(e1) / 10
        ms = float(t.item())
        summary = timer.summary()
        # the host's own time per step; with AMP the GradScaler reads its overflow flag on
        # the host every step, so the host waits for the device and the figure says nothing
        step_costs = (StepCosts().summary(K, StepCosts.host_step_ms(step), dev, world,
                                          exchange=False) if not amp else None)
        rec = {
            "metric": f"{'CNN128' if name == 'cnn128' else 'Spikformer256'} synthetic training "
                      "samples/s", "value": world * NB * K / (ms / 1e3), "unit": "samples/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms / K,
            "precision": "amp fp16 (autocast + GradScaler)" if amp else "fp32",
            "model_source": {"example": "the reference example's own module, unmodified, with "
                                        "this library installed (integrate.install, "
                                        "rebind_aligned)",
                             "example-reference": "the reference example's own module, unmodified, "
                                                  "with the reference's own aligned kernels (its "
                                                  "CuPy path through the stand-in)",
                             }.get(source, "this repository's restatement"),
            "workload": desc, "parallelism": f"dp{world}" + (" (DDP, NCCL)" if world > 1 else ""),
            "params": nparams,
            "lif_ms_per_step": round(sum(v["ms_total"] for v in summary.values()) / K, 3),
            "lif_launches_per_step": timer.total_launches() / K,
            "allreduce_ms": allreduce,
            "per_rank_ms_per_step": [round(x / K, 3) for x in per_rank],
            "replica_ms_per_step": replica,
            "step_costs": step_costs,
            "loss": float(loss.item()),
        }
        if world > 1:
            net = None
        return rec
    finally:
        close()


def run_network(args, name):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    start_ranks(dev, world)
    K, W = args.steps, max(args.warmup, 3)
    clocks = ClockSampler(local)
    recs = [measure_network(args, name, dev, world, local, amp, K, W, args.network_source)
            for amp in (False, True)]
    clk = clocks.stop()
    line = dict(recs[0])
    line.update({"higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                 "dtype": "f32", "data": "synthetic",
                 "config": {"workload": recs[0]["workload"],
                            "parallelism": recs[0]["parallelism"]},
                 "amp": recs[1], "clocks": clk})
    finish_ranks(line, rank, world)
    return 0


HIST_KINDS = ("vogl1", "fagl1", "vopred")


def history_tables(T, B, dev, g):
    """Per-sample tables as LIFNeuronFDE builds them: VO-GL1 / VO-PREDICTOR from a beta[T, B]
    schedule in (0.2, 0.8); FAGL1 rows = GL coefficients (beta 0.5) x a positive attention."""
    from dfsnn_b200 import schedule
    beta = 0.2 + 0.6 * torch_rand((T, B), dev, g)
    vo = schedule.build_vogl1_schedule(beta, H)
    vp = schedule.build_vopredictor_schedule(beta, H)
    att = 0.5 + torch_rand((T, B, T), dev, g)
    gl = schedule.build_vogl1_schedule(beta.new_full((T,), 0.5), H)["weights"]
    return {"vogl1": (vo["scale"], vo["weights"]), "vopred": (vp["scale"], vp["weights"]),
            "fagl1": (None, (gl[:, None, :] * att).contiguous())}


def torch_rand(shape, dev, g):
    import torch
    return torch.rand(shape, device=dev, generator=g)


def measure_history(args, dev, world, rank, K, W, shape=(16, 128, 64, 64), ts=(8, 16)):
    """One step: VO-GL1 (full history), FAGL1 (full history) and VO-PREDICTOR, each forward +
    backward with gradients for x, scale and weights, at T = 8 and 16 on [T, N] inputs with
    per-sample tables (B = 16 samples of N/16 neurons).  Returns the record."""
    import torch
    from dfsnn_b200 import fde_kernels as fk
    from dfsnn_b200.distributed import allreduce_flat

    B = shape[0]
    neurons = math.prod(shape)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x16 = torch.randn((16, neurons), device=dev, generator=g).mul_(0.5).add_(0.3)
    gS16 = torch.randn((16, neurons), device=dev, generator=g)
    tabs = {T: history_tables(T, B, dev, g) for T in ts}
    for T in ts:
        for kind in HIST_KINDS:
            sc, Wt = tabs[T][kind]
            tabs[T][kind] = (None if sc is None else sc.detach().requires_grad_(True),
                             Wt.detach().requires_grad_(True))
    v0 = torch.zeros(neurons, device=dev)
    hb = H ** 0.5

    def compute():
        pgrads = []
        for T in ts:
            for kind in HIST_KINDS:
                sc, Wt = tabs[T][kind]
                x = x16[:T].detach().requires_grad_(True)
                if kind == "vogl1":
                    s = fk.LIFFDEVOGL1Function.apply(x, v0, sc, Wt, TAU, TH, SG, B, True)
                    ins = [x, sc, Wt]
                elif kind == "fagl1":
                    s = fk.LIFFDEFAGL1Function.apply(x, v0, Wt, TAU, hb, TH, SG, B, True)
                    ins = [x, Wt]
                else:
                    s = fk.LIFFDEVOPREDICTORFunction.apply(x, v0, sc, Wt, TAU, TH, SG, 0.25, B)
                    ins = [x, sc, Wt]
                res = torch.autograd.grad([s], ins, [gS16[:T]])
                pgrads += list(res[1:])
        return pgrads

    def exchanger(costs):
        def exchange(grads):
            if world > 1:
                with costs.exchange():
                    allreduce_flat(grads)
        return exchange

    ecosts = StepCosts()
    eexchange = exchanger(ecosts)

    def estep():
        grads = compute()
        eexchange(grads)

    ms_eager, timer, clk_eager = timed_region(estep, K, W, dev, world, ecosts)
    eager_costs = ecosts.summary(K, ecosts.host_step_ms(estep), dev, world)
    gcosts = StepCosts()
    graph, gstep, per_replay = graph_step(compute, exchanger(gcosts), dev)
    ms, _, clk = timed_region(gstep, K, W, dev, world, gcosts, timer=False)
    step_costs = gcosts.summary(K, gcosts.host_step_ms(gstep), dev, world)
    del graph, gstep
    units = sum(ts) * neurons * len(HIST_KINDS)
    summary = timer.summary()
    peak, peak_src = measured_hbm_peak()
    dom = max(summary.items(), key=lambda kv: kv[1]["ms_total"]) if summary else None
    roofline = None
    if dom is not None:
        name, d = dom
        roofline = {"bound": "hbm", "kernel": name, "achieved": d["gbs"], "peak": peak,
                    "unit": "GB/s", "frac": d["gbs"] / peak if d["gbs"] else None,
                    "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_src})",
                    "algorithmic_bytes_per_launch": d["bytes_per_call"], "traffic": None}
    return {
        "metric": "LIF-FDE history-table Functions neuron-timesteps/s fwd+bwd",
        "value": world * K * units / (ms / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": ms / K,
        "workload": "LIFFDEVOGL1Function (full history), LIFFDEFAGL1Function (full history), "
                    "LIFFDEVOPREDICTORFunction fwd+bwd with grads of x, scale and weights; "
                    "per-sample tables, B=16, x [T, 8,388,608] ~N(0.3,0.5^2), T=8 and 16",
        "neurons_per_gpu": neurons,
        "parallelism": f"dp{world}" + (" (one NCCL all-reduce of the table grads per step)"
                                       if world > 1 else ""),
        "launch": LAUNCH_DESC,
        "gpu_launches": per_replay * K,
        "roofline": roofline,
        "kernels": {k: {"calls_per_step": v["calls"] / K,
                        "ms_per_call": round(v["ms_per_call"], 4),
                        "gbs": round(v["gbs"], 1) if v["gbs"] else None,
                        "frac_of_hbm": round(v["gbs"] / peak, 4) if v["gbs"] else None}
                    for k, v in summary.items()},
        "step_costs": step_costs,
        "clocks": clk,
        "eager": {"value": world * K * units / (ms_eager / 1e3), "ms_per_step": ms_eager / K,
                  "gpu_launches": timer.total_launches(), "step_costs": eager_costs,
                  "clocks": clk_eager},
    }


def run_history(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    start_ranks(dev, world)
    rec = measure_history(args, dev, world, rank, args.steps, max(args.warmup, 3), SHAPE, TS)
    line = dict(rec)
    line.update({"higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                 "dtype": "f32", "data": "synthetic",
                 "config": {"workload": rec["workload"], "neurons_per_gpu": rec["neurons_per_gpu"],
                            "T": list(TS), "l2": "inputs larger than L2 (no flush)",
                            "parallelism": rec["parallelism"]}})
    finish_ranks(line, rank, world)
    return 0


def run_integrator(args):
    import torch
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    line = measure_integrator(args, dev, args.steps, max(args.warmup, 3))
    print(json.dumps(line), flush=True)
    return 0


def measure_integrator(args, dev, K, W):
    """One step: the SNN wrapper's multi-term GL integration (forward_glmulti_cupy, as
    FDEAdjointMethod runs it, without autograd) over T = 64 steps of a [16, 64, 64, 64] =
    4,194,304-element state and its adjoint (backward_glmulti_cupy) over the same grid.  The
    right-hand side is elementwise (-v + I_k for the state, a pass-through spike sum), so the
    time is the history steps': each step reads its f and every earlier state row (O(T^2)
    rows in total) and writes the new row."""
    import torch
    from dfsnn_b200 import fde_solver, profiling

    T = 64
    shape = (16, 64, 64, 64)
    g = torch.Generator(device=dev).manual_seed(7)
    current = torch.randn((T,) + shape, device=dev, generator=g).mul_(0.4).add_(0.2)
    adj_src = torch.randn(shape, device=dev, generator=g)
    t_grid = torch.linspace(0.0, 0.1 * T, T + 1, device=dev)
    beta = torch.tensor(MULTI_BETA)
    coef = torch.tensor(MASSES)

    calls = {"k": 0}

    def rhs(t, y):                       # step index from a call counter: no host sync on t
        k = calls["k"]
        calls["k"] += 1
        return (current[min(k, T - 1)] - y[0], y[1] + y[0])

    def adjoint_rhs(t, aug):
        _, adj, params = aug
        return None, [adj[0] * -0.5 + adj_src], []

    def step():
        calls["k"] = 0
        with torch.no_grad():
            hist = fde_solver.forward_glmulti_cupy(rhs, (torch.zeros(shape, device=dev),
                                                         torch.zeros(shape, device=dev)),
                                                   beta, t_grid, multi_coefficient=coef)
            adj, _ = fde_solver.backward_glmulti_cupy(
                adjoint_rhs, (None, [torch.ones(shape, device=dev)], []), beta, t_grid,
                hist, multi_coefficient=coef)
        return adj

    for _ in range(W):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with profiling.NativeCallTimer() as timer:
        start.record()
        for _ in range(K):
            step()
        end.record()
        torch.cuda.synchronize()
    clk = clocks.stop()
    ms = start.elapsed_time(end)
    summary = timer.summary()
    peak, peak_src = measured_hbm_peak()
    d = summary.get("gl_history_step")
    roofline = None
    if d:
        roofline = {"bound": "hbm", "kernel": "gl_history_step", "achieved": d["gbs"],
                    "peak": peak, "unit": "GB/s", "frac": d["gbs"] / peak if d["gbs"] else None,
                    "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_src})",
                    "algorithmic_bytes_per_launch": d["bytes_per_call"], "traffic": None}
    S = math.prod(shape)
    line = {
        "metric": "multi-term GL integrator state-element-steps/s (forward + adjoint)",
        "value": K * 2 * T * S / (ms / 1e3), "unit": "element-steps/s", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "forward_glmulti_cupy (no autograd) + backward_glmulti_cupy, T=64 "
                   "steps, state [16,64,64,64] = 4,194,304 elements, glmulti orders "
                   "[0.3,0.4,0.5] masses [0.5,0.5,0.7], elementwise right-hand side",
                   "T": T, "state_elements": S, "l2": "history rows larger than L2"},
        "gpu_launches": timer.total_launches(),
        "roofline": roofline,
        "kernels": {k: {"calls_per_step": v["calls"] / K, "ms_per_call": round(v["ms_per_call"], 4),
                        "gbs": round(v["gbs"], 1) if v["gbs"] else None}
                    for k, v in summary.items()},
        "clocks": clk,
    }
    return line


def main():
    args = parse()
    if args.workload == "integrator":
        return run_integrator(args) if args.impl == "native" else 0
    if args.workload in NETWORKS:
        return run_network(args, args.workload) if args.impl == "native" else 0
    if args.workload == "history":
        return run_history(args) if args.impl == "native" else 0
    if args.impl == "reference":
        return run_reference(args)
    return run_native(args)


if __name__ == "__main__":
    sys.exit(main())
