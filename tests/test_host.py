"""Host-side logic on CPU: weight tables and glmulti schedule bit-identical to the
reference's, gradient chain to the Softplus masses, LIFNeuronFDE mirror contract, no
CPU fallback, and registration under the reference's module names."""
import math
import os
import sys

import numpy as np
import pytest
import torch

from dfsnn_b200 import fde_kernels, integrate, neuron, schedule
from dfsnn_b200 import aligned_glmulti as alg
from oracle import oracle as O
from parity import assert_bitwise, assert_close

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TAU, TH, SG, H = 2.0, 1.0, 5.0, 0.1
MULTI_BETA = [0.3, 0.4, 0.5]
MASSES = [0.5, 0.5, 0.7]


def tables():
    return dict(np.load(os.path.join(GOLDEN, "torch_tables.npz")))


def make_glmulti(T=16, **kw):
    return neuron.LIFNeuronFDE(tau=TAU, threshold=TH, surrogate_grad_scale=SG,
                               surrogate_function="arctan", beta=MULTI_BETA[0], T=T,
                               method="glmulti", step_size=H, batchsize=4, step_mode="m",
                               backend="cupy", multi_beta=MULTI_BETA, multi_coefficient=MASSES,
                               learn_coefficient=True, coefficient_constraint="softplus",
                               glmulti_history_grad="full", **kw)


@pytest.mark.parametrize("method", ["gl", "trap", "predictor"])
@pytest.mark.parametrize("beta", [0.3, 0.5, 0.7])
@pytest.mark.parametrize("T", [8, 16, 20, 64, 256])
def test_weight_tables_bitwise(method, beta, T):
    ref = tables()[f"{method}_b{beta}_T{T}"]
    got = getattr(schedule, f"{method}_weights")(beta, T).numpy()
    assert_bitwise(got, ref, what=f"{method} beta={beta} T={T}")


@pytest.mark.parametrize("T", [1, 8, 16, 32])
def test_glmulti_schedule_bitwise(T):
    d = tables()
    n = make_glmulti(T)
    with torch.no_grad():
        terms = n._build_glmulti_schedule(T, torch.device("cpu"))
    assert_bitwise(terms["scale"].contiguous().numpy(), d[f"glmulti_scale_T{T}"], what="scale")
    assert_bitwise(terms["weights"].numpy(), d[f"glmulti_W_T{T}"], what="W")


@pytest.mark.parametrize("case", ["spiking_T16", "config1_T16"])
def test_glmulti_mass_gradient_chain(case):
    """Reference LIFNeuronFDE (torch path, truncated history) gradient of the shared raw
    masses == oracle (grad_scale, grad_W) pushed through this package's schedule."""
    d = dict(np.load(os.path.join(GOLDEN, f"torch_glmulti_neuron_{case}.npz")))
    T = d["x"].shape[0]
    x = d["x"].reshape(T, -1)
    N = x.shape[1]
    n = make_glmulti(T)
    terms = n._build_glmulti_schedule(T, torch.device("cpu"))
    r = O.glmulti_step(x, np.zeros(N, np.float32), terms["scale"].detach().numpy(),
                       terms["weights"].detach().numpy(), d["gS"].reshape(T, N), TAU, TH, SG, False)
    assert (r["spike"] == d["spike"].reshape(T, N)).all()
    torch.autograd.backward([terms["scale"], terms["weights"]],
                            [torch.tensor(r["gscale"], dtype=torch.float32),
                             torch.tensor(r["gW"], dtype=torch.float32)])
    assert_close(n.multi_coefficient_raw.grad.numpy(), d["graw"], rtol=1e-4, what="grad raw")
    assert_close(r["gx"], d["gx"].reshape(T, N), rtol=1e-4, what="gx")


def test_state_dict_keys_match_reference():
    d = tables()
    assert sorted(make_glmulti().state_dict().keys()) == list(d["state_dict_keys_glmulti"])
    gl = neuron.LIFNeuronFDE(method="gl", T=16, step_mode="m", backend="cupy")
    assert sorted(gl.state_dict().keys()) == list(d["state_dict_keys_gl"])


def test_shared_coefficient_and_validation():
    raw = torch.nn.Parameter(torch.log(torch.expm1(torch.tensor(MASSES))))
    a, b = make_glmulti(shared_multi_coefficient=raw), make_glmulti(shared_multi_coefficient=raw)
    assert a.multi_coefficient_raw is b.multi_coefficient_raw
    with pytest.raises(ValueError):
        neuron.LIFNeuronFDE(method="glmulti", multi_beta=[0.3], multi_coefficient=[0.5, 0.5])
    with pytest.raises(ValueError):
        neuron.LIFNeuronFDE(method="nope")


def test_no_cpu_fallback():
    x = torch.zeros(8, 4)
    with pytest.raises(RuntimeError):
        fde_kernels.LIFFDEGLMultiFunction.apply(x, torch.zeros(4), torch.ones(8), torch.zeros(8, 8),
                                                2.0, 1.0, 5.0, 1, True)
    with pytest.raises(RuntimeError):
        fde_kernels.LIFFDEGLFunction.apply(x, torch.zeros(4), torch.ones(9), 2.0, 0.5, 1.0, 0.0, 5.0)
    with pytest.raises(RuntimeError):
        make_glmulti(8)(torch.zeros(8, 2, 3))
    with pytest.raises(NotImplementedError):
        neuron.LIFNeuronFDE(method="gl", step_mode="s")(torch.zeros(2, 3))
    with pytest.raises(RuntimeError):
        fde_kernels.LIFFDEVOGL1Function.apply(x, torch.zeros(4), torch.ones(8), torch.zeros(8, 8),
                                              2.0, 1.0, 5.0, 1)
    with pytest.raises(RuntimeError):
        fde_kernels.LIFFDEFAGL1Function.apply(x, torch.zeros(4), torch.zeros(8, 8), 2.0, 0.25,
                                              1.0, 5.0, 1)
    with pytest.raises(RuntimeError):
        fde_kernels.LIFFDEFAGL1TorchFunction.apply(x, torch.zeros(4), torch.zeros(8, 8), 2.0,
                                                   0.25, 1.0, 5.0, 1)
    with pytest.raises(RuntimeError):
        fde_kernels.LIFFDEVOPREDICTORFunction.apply(x, torch.zeros(4), torch.ones(8),
                                                    torch.zeros(8, 8), 2.0, 1.0, 5.0, 0.2, 1)


def test_reference_limits_raise_value_error():
    x = torch.zeros(65, 4)
    with pytest.raises(ValueError):
        alg.AlignedGLMulti.apply(x, torch.zeros(4), torch.ones(65), torch.zeros(65, 65), 2.0, 1.0,
                                 5.0, 1, True)
    with pytest.raises(ValueError):
        alg.AlignedGLMulti.apply(torch.zeros(4, 4), torch.zeros(4), torch.ones(4),
                                 torch.zeros(4, 4), 2.0, 1.0, 5.0, 1, False)


def test_integrate_registers_reference_module_names():
    saved = {k: sys.modules.get(k) for k in (integrate.FDE_MODULE, integrate.EULER_MODULE)}
    try:
        integrate.install()
        import importlib
        m = importlib.import_module("spikeDE_dis.fde_cupy_kernels_all")
        assert m is fde_kernels and m.CUPY_AVAILABLE
        assert importlib.import_module("spikeDE_dis.direct_euler_cupy").lif_like_euler_cupy
        original = fde_kernels.LIFFDEGLMultiFunction
        integrate.rebind_aligned()
        assert fde_kernels.LIFFDEGLMultiFunction is alg.AlignedGLMulti
        fde_kernels.LIFFDEGLMultiFunction = original
    finally:
        integrate.uninstall_schedule()
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


@pytest.mark.parametrize("init", ["zero_q", "orthogonal_zero_score"])
@pytest.mark.parametrize("mode", ["per_sample", "batch_shared"])
def test_fagl1_neuron_attention_rows_vs_reference(init, mode):
    """method='fagl1': the seeded projection init and _build_fagl1_weights against the
    reference's LIFNeuronFDE (neuron.py:1205-1221, :1790-1866), bit for bit on the host."""
    d = np.load(os.path.join(GOLDEN, "torch_fagl1_neuron.npz"))
    n = neuron.LIFNeuronFDE(tau=2.0, threshold=1.0, surrogate_grad_scale=5.0, method="fagl1",
                            beta=0.6, T=8, step_size=0.1, name="lif3", step_mode="m",
                            backend="torch", attn_init=init, attn_mode=mode)
    tag = f"{init}_{mode}"
    assert np.array_equal(n.fagl_q_proj.weight.detach().numpy(), d[f"{tag}_q"])
    assert np.array_equal(n.fagl_k_proj.weight.detach().numpy(), d[f"{tag}_k"])
    W = n._build_fagl1_weights(torch.from_numpy(d["x"]))
    assert np.array_equal(W.detach().numpy(), d[f"{tag}_W"])
    assert np.float32(n.get_attention_stats()["entropy"]) == d[f"{tag}_entropy"]


def test_gl1_full_history_rows_vs_reference():
    d = np.load(os.path.join(GOLDEN, "torch_fagl1_neuron.npz"))
    n = neuron.LIFNeuronFDE(method="gl1", beta=0.6, T=8, step_size=0.1, step_mode="m")
    assert np.array_equal(n._build_gl1_causal_weights(8, torch.device("cpu")).numpy(),
                          d["gl1_rows"])


def test_history_method_validation():
    with pytest.raises(ValueError):
        neuron.LIFNeuronFDE(method="fagl1", beta_learnable=True, step_mode="m")
    with pytest.raises(ValueError):
        neuron.LIFNeuronFDE(method="vogl1", vo_solver="rk4", step_mode="m")
    with pytest.raises(ValueError):
        neuron.LIFNeuronFDE(method="gl1", history_grad_mode="exact", step_mode="m")
    with pytest.raises(ValueError):
        neuron.LIFNeuronFDE(method="fagl1", attn_dim=2, step_mode="m")


def test_fde_solver_install_rebinds_reference_names():
    """fde_solver.install() points spikeDE_dis.solver's glmulti entries (module names and the
    CuPy / torch dispatch tables, solver.py:4752-4806) and snn.py's imported name at the
    B200 integrator."""
    import types
    from dfsnn_b200 import fde_solver
    solver = types.ModuleType("spikeDE_dis.solver")
    solver.CUPY_SOLVERS_FORWARD = {"glmulti": None, "gl-f": "keep"}
    solver.CUPY_SOLVERS_BACKWARD = {"glmulti": None}
    solver.TORCH_SOLVERS_BACKWARD = {"glmulti": None}
    solver.forward_glmulti_cupy = solver.backward_glmulti_cupy = None
    snn = types.ModuleType("spikeDE_dis.snn")
    snn.forward_glmulti_cupy = None
    saved = {k: sys.modules.get(k) for k in ("spikeDE_dis.solver", "spikeDE_dis.snn")}
    try:
        sys.modules["spikeDE_dis.solver"], sys.modules["spikeDE_dis.snn"] = solver, snn
        fde_solver.install()
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    assert solver.CUPY_SOLVERS_FORWARD["glmulti"] is fde_solver.forward_glmulti_cupy
    assert solver.CUPY_SOLVERS_FORWARD["gl-f"] == "keep"
    assert solver.CUPY_SOLVERS_BACKWARD["glmulti"] is fde_solver.backward_glmulti_cupy
    assert solver.TORCH_SOLVERS_BACKWARD["glmulti"] is fde_solver.backward_glmulti_cupy
    assert solver.forward_glmulti_cupy is fde_solver.forward_glmulti_cupy
    assert snn.forward_glmulti_cupy is fde_solver.forward_glmulti_cupy


def test_fde_solver_rejects_cpu_and_half():
    from dfsnn_b200 import fde_solver
    y = torch.zeros(3)
    with pytest.raises(RuntimeError):
        fde_solver.forward_glmulti_cupy(lambda t, s: s, (y, y), [0.5], torch.tensor([0.0, 0.1]),
                                        multi_coefficient=[1.0])
    with pytest.raises(ValueError):
        fde_solver.forward_glmulti_cupy(lambda t, s: s, (y, y), [0.5], torch.tensor([0.0]),
                                        multi_coefficient=[1.0])


@pytest.mark.parametrize("workload,combos", [
    ("layers", {(8, "glmulti"), (8, "gl"), (8, "trap"), (8, "predictor"), (16, "glmulti"),
                (16, "gl"), (16, "trap"), (16, "predictor")}),
    ("long", {(64, "gl"), (64, "predictor"), (256, "gl"), (256, "predictor")}),
    ("aligned", {(8, "aligned"), (16, "aligned")}),
])
def test_bench_workload_configuration(workload, combos, monkeypatch):
    """bench.py's workloads: the schemes and step counts each one runs (no GPU needed)."""
    import importlib
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    monkeypatch.syspath_prepend(repo)
    bench = importlib.import_module("bench")
    bench = importlib.reload(bench)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--workload", workload])
    args = bench.parse()
    assert args.workload == workload
    assert set(bench.COMBOS) == combos
    neurons = 4194304 if workload == "long" else 16 * 128 * 64 * 64
    assert bench.SHAPE[0] * bench.SHAPE[1] == neurons or \
        bench.SHAPE[0] * bench.SHAPE[1] * bench.SHAPE[2] * bench.SHAPE[3] == neurons
    importlib.reload(bench)          # leave module globals at their defaults for other tests


def test_bench_clock_sampler_parses_nvidia_smi(tmp_path, monkeypatch):
    """bench.py's clock record: median SM clock, max clock and the throttle reasons reported
    Active, from a stand-in nvidia-smi on PATH; the sampler waits for its first sample and
    reports only the samples after it (no GPU needed)."""
    import importlib
    import types
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    monkeypatch.syspath_prepend(repo)
    bench = importlib.import_module("bench")
    fake = tmp_path / "nvidia-smi"
    fake.write_text(
        "#!/bin/bash\n"
        "echo '0, 1000, 1965, 300, 0x0, Not Active, Not Active, Not Active, Not Active'\n"
        "for c in 1900 1800 1700; do\n"
        "  echo \"0, $c, 1965, 700, 0x4, Not Active, Not Active, Not Active, Active\"\n"
        "  sleep 0.05\n"
        "done\n"
        "exec sleep 10\n")                     # the sampler's terminate() ends it, as nvidia-smi
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", str(tmp_path) + os.pathsep + os.environ.get("PATH", ""))
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda i: types.SimpleNamespace(uuid="00000000-0000-0000-0000-000000000000"))
    broken = types.ModuleType("pynvml")          # NVML unusable: the sampler falls back

    def fail(*a):
        raise RuntimeError("no NVML here")
    broken.nvmlInit = fail
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    sampler = bench.ClockSampler(0)
    import time
    time.sleep(0.5)
    rec = sampler.stop()
    assert rec == {"sm_mhz": 1800.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                   "samples": 3, "source": "nvidia-smi"}


def test_bench_clock_sampler_nvml(monkeypatch):
    """The NVML path: SM clock, maximum and clock-event reason bits read from a thread
    (a stand-in pynvml; no GPU needed)."""
    import importlib
    import time
    import types
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    monkeypatch.syspath_prepend(repo)
    bench = importlib.import_module("bench")
    clocks = iter([1500.0] + [1900.0, 1800.0, 1700.0] * 1000)
    fake = types.ModuleType("pynvml")
    fake.NVML_CLOCK_SM = 1
    fake.nvmlInit = lambda: None
    fake.nvmlDeviceGetHandleByUUID = lambda u: ("h", u)
    fake.nvmlDeviceGetMaxClockInfo = lambda h, c: 1965
    fake.nvmlDeviceGetClockInfo = lambda h, c: next(clocks)
    fake.nvmlDeviceGetCurrentClocksEventReasons = lambda h: 0x4 | 0x1
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    monkeypatch.setattr(torch.cuda, "get_device_properties",
                        lambda i: types.SimpleNamespace(uuid="00000000-0000-0000-0000-000000000000"))
    sampler = bench.ClockSampler(0, period_s=0.005)
    time.sleep(0.2)
    rec = sampler.stop()
    assert rec["source"] == "nvml" and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"] and rec["samples"] >= 3
    assert 1700.0 <= rec["sm_mhz"] <= 1900.0


def test_bench_example_networks_bind_the_native_function(monkeypatch):
    """bench.py builds the reference examples' own CNN128 / Spikformer256 modules with this
    library installed (install, the example's install('cupy'), rebind_aligned), imported with
    no CuPy at all, and puts everything back afterwards (no GPU needed to build them)."""
    import importlib
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    monkeypatch.syspath_prepend(repo)
    from oracle import reference_gpu
    if not reference_gpu.staged():
        pytest.skip("reference not staged (oracle/stage_ref.py)")
    bench = importlib.import_module("bench")
    original = fde_kernels.LIFFDEGLMultiFunction
    for name, n_lif in (("cnn128", 7), ("spikformer256", 19)):
        model, reset, close = bench.example_network(name, torch.device("cpu"))
        try:
            assert "cupy" not in sys.modules
            assert fde_kernels.LIFFDEGLMultiFunction is alg.AlignedGLMulti
            example = sys.modules["aligned_glmulti"]
            assert example.AlignedGLMulti is alg.AlignedGLMulti
            lifs = [m for m in model.modules() if type(m).__name__ in ("LIFNeuronFDE", "Neuron")]
            assert len(lifs) == n_lif
            reset()
        finally:
            close()
        assert fde_kernels.LIFFDEGLMultiFunction is original
        assert not any(k.startswith("spikeDE_dis") for k in sys.modules)


class _FakeEvent:
    """A CUDA event stand-in whose 'device' time is the host clock."""

    def __init__(self, enable_timing=False):
        self.t = None

    def record(self, stream=None):
        import time
        self.t = time.perf_counter()

    def elapsed_time(self, other):
        return (other.t - self.t) * 1e3


def test_bench_step_costs(monkeypatch):
    """StepCosts: the host time of isolated steps (median) and the exchange spans recorded
    only while the timed loop is on; no exchange figure on one rank."""
    import importlib
    import time
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    monkeypatch.syspath_prepend(repo)
    bench = importlib.import_module("bench")
    syncs = []
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a: syncs.append(1))
    monkeypatch.setattr(torch.cuda, "Event", _FakeEvent)
    costs = bench.StepCosts()
    with costs.exchange():
        pass
    assert costs.spans == []
    costs.on = True
    for _ in range(4):
        with costs.exchange():
            time.sleep(0.002)
    costs.on = False
    assert len(costs.spans) == 4
    host = bench.StepCosts.host_step_ms(lambda: time.sleep(0.003), reps=5)
    assert len(syncs) == 10 and 2.5 <= host < 50
    one = costs.summary(4, host, torch.device("cpu"), 1)
    assert set(one) == {"host_ms_per_step"} and one["host_ms_per_step"] == round(host, 4)


def test_integrate_rebinds_reference_glmulti_schedule():
    """install() rebinds the reference neuron's _build_glmulti_schedule to this library's
    (on CPU tensors it keeps the PyTorch chain, bitwise equal to the reference's own), and
    the reference harness gives the class its own method back."""
    from oracle import reference_gpu
    if not reference_gpu.staged():
        pytest.skip("reference not staged (oracle/stage_ref.py)")
    ref = reference_gpu.Reference(standin=False)
    try:
        cls = ref.neuron.LIFNeuronFDE
        own = cls._build_glmulti_schedule
        layer = cls(tau=TAU, threshold=TH, surrogate_grad_scale=SG, surrogate_function="arctan",
                    beta=MULTI_BETA[0], T=8, method="glmulti", step_size=H, batchsize=4,
                    step_mode="m", backend="cupy", multi_beta=MULTI_BETA,
                    multi_coefficient=MASSES, learn_coefficient=True,
                    coefficient_constraint="softplus", glmulti_history_grad="full")
        want = layer._build_glmulti_schedule(8, torch.device("cpu"))
        ref.use_native()
        assert cls._build_glmulti_schedule is neuron.LIFNeuronFDE._build_glmulti_schedule
        got = layer._build_glmulti_schedule(8, torch.device("cpu"))
        for k in ("scale", "weights"):
            assert_bitwise(got[k].detach().numpy(), want[k].detach().numpy(), what=k)
        ref.use_reference()
        assert cls._build_glmulti_schedule is own
    finally:
        ref.close()
    assert not integrate._SAVED_SCHEDULE
