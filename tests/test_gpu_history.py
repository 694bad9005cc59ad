"""GPU parity of the history-table Functions with shared or per-sample parameters:
LIFFDEVOGL1Function, LIFFDEFAGL1Function, LIFFDEFAGL1TorchFunction and
LIFFDEVOPREDICTORFunction (fde_cupy_kernels_all.py:1098-1198, :1379-1587, :1751-1843).

Per-neuron outputs (spikes, the saved v_pre / history / drift sequences, grad_x, grad_v0)
follow the reference kernels' fp32 operation order and must be bit-identical to the oracle;
grad_scale and grad_weights are reductions over neurons, compared with the double-precision
oracle at RTOL = 1e-5 of each tensor's scale.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from dfsnn_b200 import _capi, fde_kernels
from oracle import oracle as O
from parity import RTOL, assert_bitwise, assert_close, assert_spikes

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TH, SG, RM = 1.0, 5.0, 0.25
HB = np.float32(0.1 ** 0.6)
DEV = "cuda:0"
FN = {"vogl1": fde_kernels.LIFFDEVOGL1Function, "fagl1": fde_kernels.LIFFDEFAGL1Function,
      "vopred": fde_kernels.LIFFDEVOPREDICTORFunction}


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def cpu(t):
    return t.detach().float().cpu().numpy()


def tables(kind, T, B, per_batch, seed):
    """Causal tables of the shape the reference's builders produce (entries above the
    diagonal zero), with random magnitudes so every history term matters."""
    g = np.random.default_rng(seed)
    shape = (T, B, T) if per_batch else (T, T)
    mask = np.tril(np.ones((T, T), np.float32), -1)
    W = g.uniform(-0.3, 0.3, size=shape).astype(np.float32)
    W *= mask[:, None, :] if per_batch else mask
    if kind == "fagl1":
        return None, W
    scale = g.uniform(0.1, 0.4, size=(T, B) if per_batch else T).astype(np.float32)
    return scale, W


def inputs(seed, T, N):
    g = np.random.default_rng(seed)
    x = (g.standard_normal((T, N)) * 5.0).astype(np.float32)
    v0 = (g.standard_normal(N) * 0.1).astype(np.float32)
    gS = g.standard_normal((T, N)).astype(np.float32)
    return x, v0, gS


def run(kind, x, v0, scale, W, B, tau, gS, full=False, fn=None):
    fn = fn or FN[kind]
    xt, vt = cuda(x).requires_grad_(True), cuda(v0).requires_grad_(True)
    Wt = cuda(W).requires_grad_(True)
    if kind == "fagl1":
        s = fn.apply(xt, vt, Wt, tau, float(HB), TH, SG, B, full)
        st = None
    else:
        st = cuda(scale).requires_grad_(True)
        if kind == "vogl1":
            s = fn.apply(xt, vt, st, Wt, tau, TH, SG, B, full)
        else:
            s = fn.apply(xt, vt, st, Wt, tau, TH, SG, RM, B)
    s.backward(cuda(gS))
    torch.cuda.synchronize()
    return {"spike": cpu(s), "gx": cpu(xt.grad), "gv0": cpu(vt.grad), "gW": cpu(Wt.grad),
            "gs": None if st is None else cpu(st.grad)}


def check_vs_oracle(kind, x, v0, scale, W, B, tau, gS, full, got, lower_only_batch=True):
    fw = O.hfam_forward(kind, x, v0, scale, W, B, tau, TH, HB, RM)
    assert_bitwise(got["spike"], fw["spike"], what="spike")
    gx, gv0, gpre = O.hfam_backward(kind, int(full), gS, fw["vpre"], scale, W, B, tau, TH, SG, HB,
                                    RM)
    assert_bitwise(got["gx"], gx, what="gx")
    assert_bitwise(got["gv0"], gv0, what="gv0")
    gs, gW = O.hfam_params(kind, gpre, fw["hsrc"], fw["aux"], scale, W, B, lower_only_batch)
    assert_close(got["gW"], gW, what="grad_weights")
    if kind != "fagl1":
        assert_close(got["gs"], gs, what="grad_scale")


# T = 8 / 16 take the register kernels, the rest the shared-memory kernels; (B, F) covers one
# sample, samples of one neuron, samples that split warps, and a sample boundary per block.
CASES = [(T, B, F) for T in (1, 5, 8, 16, 33) for (B, F) in ((1, 1000), (4, 257), (3, 1))] + \
        [(8, 16, 4099), (16, 16, 4099), (16, 2, 70001), (64, 4, 300), (17, 5, 64)]


# VO-PREDICTOR has one backward (the truncated one), so it takes full=False only
KIND_FULL = [("vogl1", False), ("vogl1", True), ("fagl1", False), ("fagl1", True),
             ("vopred", False)]


@pytest.mark.parametrize("kind,full", KIND_FULL)
@pytest.mark.parametrize("per_batch", [False, True])
@pytest.mark.parametrize("T,B,F", CASES)
@pytest.mark.parametrize("tau", [2.0, 0.7])
def test_history_vs_oracle(kind, per_batch, T, B, F, tau, full):
    N = B * F
    x, v0, gS = inputs(T * 31 + N, T, N)
    scale, W = tables(kind, T, B, per_batch, T + B)
    got = run(kind, x, v0, scale, W, B, tau, gS, full)
    check_vs_oracle(kind, x, v0, scale, W, B, tau, gS, full, got)


@pytest.mark.parametrize("kind", ["vogl1", "vopred"])
@pytest.mark.parametrize("T,B,F", [(100, 3, 50), (256, 2, 33)])
def test_history_long_T_vs_oracle(kind, T, B, F):
    N = B * F
    x, v0, gS = inputs(T + N, T, N)
    for per_batch in (False, True):
        scale, W = tables(kind, T, B, per_batch, T)
        got = run(kind, x, v0, scale, W, B, 2.0, gS)
        check_vs_oracle(kind, x, v0, scale, W, B, 2.0, gS, False, got)


@pytest.mark.parametrize("kind", ["vogl1", "fagl1", "vopred"])
def test_history_full_size_sample(kind):
    """A CNN-layer-sized call (B=16 samples of 32x64x64 neurons, T=16): every output against
    the oracle (which runs the same size on the host cores)."""
    T, B, F = 16, 16, 32 * 64 * 64
    N = B * F
    x, v0, gS = inputs(99, T, N)
    scale, W = tables(kind, T, B, True, 3)
    got = run(kind, x, v0, scale, W, B, 2.0, gS, kind != "vopred")
    check_vs_oracle(kind, x, v0, scale, W, B, 2.0, gS, kind != "vopred", got)


@pytest.mark.parametrize("kind", ["vogl1", "fagl1", "vopred"])
@pytest.mark.parametrize("per_batch", [0, 1])
def test_saved_sequences_bitwise(kind, per_batch):
    """The forward's saved sequences (v_pre, v_hist or drift, VO-GL1's drift) through the C ABI."""
    T, B, F = 16, 4, 999
    N = B * F
    x, v0, _ = inputs(7, T, N)
    scale, W = tables(kind, T, B, per_batch, 1)
    L = _capi.lib()
    xt, vt, Wt = cuda(x), cuda(v0), cuda(W)
    out = [torch.empty((T, N), device=DEV) for _ in range(4)]
    p = [_capi.ptr(o) for o in out]
    st = 0
    if kind == "vogl1":
        code = L.dfsnn_vo_gl1_forward(_capi.ptr(xt), _capi.ptr(vt), _capi.ptr(cuda(scale)),
                                      _capi.ptr(Wt), B, per_batch, p[0], p[1], p[2], p[3], T, N,
                                      2.0, TH, st)
    elif kind == "fagl1":
        code = L.dfsnn_fa_gl1_forward(_capi.ptr(xt), _capi.ptr(vt), _capi.ptr(Wt), B, per_batch,
                                      p[0], p[1], p[2], T, N, 2.0, float(HB), TH, st)
    else:
        code = L.dfsnn_vo_predictor_forward(_capi.ptr(xt), _capi.ptr(vt), _capi.ptr(cuda(scale)),
                                            _capi.ptr(Wt), B, per_batch, p[0], p[1], p[2], T, N,
                                            2.0, TH, RM, st)
    assert code == 0, _capi.status_string(code)
    torch.cuda.synchronize()
    fw = O.hfam_forward(kind, x, v0, scale, W, B, 2.0, TH, HB, RM)
    assert_bitwise(cpu(out[0]), fw["spike"], what="spike")
    assert_bitwise(cpu(out[1]), fw["vpre"], what="v_pre")
    assert_bitwise(cpu(out[2]), fw["hsrc"], what="history")
    if kind == "vogl1":
        assert_bitwise(cpu(out[3]), fw["aux"], what="drift")


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


@pytest.mark.parametrize("kind", ["vogl1", "fagl1", "vopred"])
@pytest.mark.parametrize("tag", ["shared", "batch"])
def test_history_vs_reference_kernel_golden(kind, tag):
    d = golden(f"kern_hist_{kind}_T16.npz")
    B = int(d["B"])
    assert float(d["h_beta"]) == float(HB) and float(d["residual_mix"]) == RM
    scale = d.get(f"{tag}_scale")
    for full in ((False, True) if kind != "vopred" else (False,)):
        got = run(kind, d["x"], d["v0"], scale, d[f"{tag}_W"], B, 2.0, d["gS"], full)
        assert_bitwise(got["spike"], d[f"{tag}_spike"], what="spike")
        assert_bitwise(got["gx"], d[f"{tag}_f{int(full)}_gx"], what="gx")
        assert_bitwise(got["gv0"], d[f"{tag}_f{int(full)}_gv0"], what="gv0")


@pytest.mark.parametrize("tag", ["shared", "batch"])
@pytest.mark.parametrize("full", ["trunc", "full"])
def test_fagl1_torch_function_vs_reference_torch_golden(tag, full):
    """LIFFDEFAGL1TorchFunction against the reference's own PyTorch Function (fp32 rounding
    differs: spikes equal off the threshold band, gradients within 1e-4)."""
    d = golden(f"torch_fagl1_{tag}_{full}_T16.npz")
    B = int(d["B"])
    got = run("fagl1", d["x"], d["v0"], None, d["W"], B, 2.0, d["gS"], full == "full",
              fn=fde_kernels.LIFFDEFAGL1TorchFunction)
    fw = O.hfam_forward("fagl1", d["x"], d["v0"], None, d["W"], B, 2.0, TH, HB)
    mask = assert_spikes(got["spike"], d["spike"], fw["vpre"], TH)
    assert_close(got["gx"], d["gx"], rtol=1e-4, mask=mask, what="gx")
    assert_close(got["gv0"], d["gv0"], rtol=1e-4, mask=mask, what="gv0")
    assert_close(got["gW"], d["gW"], rtol=1e-4, what="gW")


@pytest.mark.parametrize("per_batch", [False, True])
@pytest.mark.parametrize("full", [False, True])
def test_fagl1_torch_function_vs_oracle(per_batch, full):
    T, B, F = 16, 4, 333
    x, v0, gS = inputs(3, T, B * F)
    _, W = tables("fagl1", T, B, per_batch, 2)
    got = run("fagl1", x, v0, None, W, B, 2.0, gS, full, fn=fde_kernels.LIFFDEFAGL1TorchFunction)
    check_vs_oracle("fagl1", x, v0, None, W, B, 2.0, gS, full, got, lower_only_batch=False)


def test_history_deterministic_and_dtype():
    T, B, F = 16, 8, 5000
    x, v0, gS = inputs(4, T, B * F)
    scale, W = tables("vogl1", T, B, True, 4)
    a = run("vogl1", x, v0, scale, W, B, 2.0, gS, True)
    b = run("vogl1", x, v0, scale, W, B, 2.0, gS, True)
    for k in ("gW", "gs", "gx"):
        assert np.array_equal(a[k], b[k]), k
    xt = cuda(x).half().requires_grad_(True)
    s = fde_kernels.LIFFDEVOGL1Function.apply(xt, cuda(v0), cuda(scale), cuda(W), 2.0, TH, SG, B)
    assert s.dtype == torch.float16
    s.backward(torch.ones_like(s))
    assert xt.grad.dtype == torch.float16


def test_history_param_grads_optional():
    T, B, F = 8, 2, 100
    x, v0, gS = inputs(5, T, B * F)
    scale, W = tables("vopred", T, B, False, 5)
    xt = cuda(x).requires_grad_(True)
    s = fde_kernels.LIFFDEVOPREDICTORFunction.apply(xt, cuda(v0), cuda(scale), cuda(W), 2.0, TH,
                                                    SG, RM, B)
    s.backward(cuda(gS))
    fw = O.hfam_forward("vopred", x, v0, scale, W, B, 2.0, TH, HB, RM)
    gx, _, _ = O.hfam_backward("vopred", 0, gS, fw["vpre"], scale, W, B, 2.0, TH, SG, HB, RM)
    assert_bitwise(cpu(xt.grad), gx, what="gx")


def test_history_limits_and_shapes():
    x = cuda(np.zeros((65, 8), np.float32))
    v0 = cuda(np.zeros(8, np.float32))
    with pytest.raises(ValueError):                       # FAGL1: T <= 64 (:1420-1421)
        fde_kernels.LIFFDEFAGL1Function.apply(x, v0, cuda(np.zeros((65, 65), np.float32)), 2.0,
                                              1.0, TH, SG, 1)
    s = cuda(np.zeros(65, np.float32))
    W = cuda(np.zeros((65, 65), np.float32))
    xg = x.clone().requires_grad_(True)
    out = fde_kernels.LIFFDEVOGL1Function.apply(xg, v0, s, W, 2.0, TH, SG, 1, True)
    with pytest.raises(ValueError):                       # full history: T <= 64
        out.sum().backward()
    with pytest.raises(ValueError):                       # T <= 256
        fde_kernels.LIFFDEVOGL1Function.apply(cuda(np.zeros((257, 8), np.float32)), v0,
                                              cuda(np.zeros(257, np.float32)),
                                              cuda(np.zeros((257, 257), np.float32)), 2.0, TH, SG, 1)
    x8 = cuda(np.zeros((8, 10), np.float32))
    v10 = cuda(np.zeros(10, np.float32))
    with pytest.raises(ValueError):                       # N % B != 0
        fde_kernels.LIFFDEVOGL1Function.apply(x8, v10, cuda(np.zeros(8, np.float32)),
                                              cuda(np.zeros((8, 8), np.float32)), 2.0, TH, SG, 3)
    with pytest.raises(ValueError):                       # per-sample scale, shared weights
        fde_kernels.LIFFDEVOGL1Function.apply(x8, v10, cuda(np.zeros((8, 2), np.float32)),
                                              cuda(np.zeros((8, 8), np.float32)), 2.0, TH, SG, 2)


def test_history_empty():
    T, B = 8, 1
    x = torch.zeros((T, 0), device=DEV, requires_grad=True)
    v0 = torch.zeros(0, device=DEV)
    s = cuda(np.full(T, 0.2, np.float32)).requires_grad_(True)
    W = cuda(np.zeros((T, T), np.float32)).requires_grad_(True)
    out = fde_kernels.LIFFDEVOGL1Function.apply(x, v0, s, W, 2.0, TH, SG, B)
    out.sum().backward()
    assert out.shape == (T, 0)
    assert float(s.grad.abs().sum()) == 0.0 and float(W.grad.abs().sum()) == 0.0


# -------------------------------------------------------------------------------------
# LIFNeuronFDE methods on top of these Functions (neuron.py:1718-2061)
# -------------------------------------------------------------------------------------
def _neuron(method, **kw):
    from dfsnn_b200 import neuron
    return neuron.LIFNeuronFDE(tau=2.0, threshold=TH, surrogate_grad_scale=SG, method=method,
                               beta=0.6, T=kw.pop("T", 8), step_size=0.1, name="lif1",
                               step_mode="m", backend=kw.pop("backend", "cupy"), **kw).to(DEV)


@pytest.mark.parametrize("method", ["vogl1", "vopredictor"])
@pytest.mark.parametrize("per_sample", [False, True])
def test_neuron_variable_order_vs_oracle(method, per_sample):
    from dfsnn_b200 import schedule
    T, B = 8, 4
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn((T, B, 3, 17), device=DEV, generator=g) * 5.0
    beta = 0.2 + 0.6 * torch.rand((T, B) if per_sample else (T,), device=DEV, generator=g)
    n = _neuron(method, T=T, vo_residual_mix=RM, history_grad_mode="full")
    s = n(x, beta_schedule=beta)
    build = schedule.build_vogl1_schedule if method == "vogl1" else schedule.build_vopredictor_schedule
    terms = build(beta, 0.1)
    kind = "vogl1" if method == "vogl1" else "vopred"
    N = x[0].numel()
    fw = O.hfam_forward(kind, cpu(x).reshape(T, N), np.zeros(N, np.float32), cpu(terms["scale"]),
                        cpu(terms["weights"]), B, 2.0, TH, HB, RM)
    assert_bitwise(cpu(s).reshape(T, N), fw["spike"], what="spike")
    assert float(n.v.abs().sum()) == 0.0 and n.k == T


@pytest.mark.parametrize("mode", ["per_sample", "batch_shared"])
@pytest.mark.parametrize("backend", ["cupy", "torch"])
def test_neuron_fagl1_vs_oracle(mode, backend):
    T, B = 8, 4
    g = torch.Generator(device=DEV).manual_seed(4)
    x = (torch.randn((T, B, 5, 13), device=DEV, generator=g) * 5.0).requires_grad_(True)
    n = _neuron("fagl1", T=T, attn_mode=mode, backend=backend, history_grad_mode="full")
    with torch.no_grad():
        W = n._build_fagl1_weights(x)
    n._fagl_stats_counter = 0
    s = n(x)
    N = x[0].numel()
    fw = O.hfam_forward("fagl1", cpu(x).reshape(T, N), np.zeros(N, np.float32), None, cpu(W), B,
                        2.0, TH, np.float32(0.1 ** 0.6))
    assert_bitwise(cpu(s).reshape(T, N), fw["spike"], what="spike")
    s.sum().backward()
    assert n.fagl_q_proj.weight.grad is not None and n.fagl_k_proj.weight.grad is not None
    assert torch.isfinite(x.grad).all()
    assert n.get_attention_stats() is not None


def test_neuron_gl1_full_history_vs_oracle():
    T, B = 16, 2
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn((T, B, 300), device=DEV, generator=g) * 5.0
    n = _neuron("gl1", T=T, history_grad_mode="full")
    s = n(x)
    W = n._build_gl1_causal_weights(T, x.device)
    N = x[0].numel()
    fw = O.hfam_forward("fagl1", cpu(x).reshape(T, N), np.zeros(N, np.float32), None, cpu(W), B,
                        2.0, TH, np.float32(0.1 ** 0.6))
    assert_bitwise(cpu(s).reshape(T, N), fw["spike"], what="spike")


def test_neuron_variable_order_requires_schedule():
    n = _neuron("vogl1")
    with pytest.raises(ValueError):
        n(torch.zeros((8, 2, 3), device=DEV))
    with pytest.raises(ValueError):
        n(torch.zeros((8, 2, 3), device=DEV), beta_schedule=torch.full((7,), 0.5, device=DEV))
    m = _neuron("vogl1", vo_solver="l1")
    with pytest.raises(NotImplementedError):
        m(torch.zeros((8, 2, 3), device=DEV), beta_schedule=torch.full((8,), 0.5, device=DEV))
