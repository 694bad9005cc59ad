"""GPU parity: the sm_100a kernels (through the C ABI) against the oracle and the goldens.

Per-neuron outputs (spikes, membranes, grad_x, grad_v0) follow the reference's fp32
operation order and must be bit-identical to the oracle.  Reductions over neurons
(grad_scale, grad_weights, the Euler scalars) are compared with the double-precision
oracle at RTOL = 1e-5 (parity.assert_close, scaled by each tensor's rms).
"""
import ctypes
import math
import os

import numpy as np
import pytest
import torch

from dfsnn_b200 import _capi, fde_kernels, neuron
from dfsnn_b200 import aligned_glmulti as alg
from dfsnn_b200 import direct_euler as deu
from oracle import oracle as O
from parity import RTOL, assert_bitwise, assert_close, assert_spikes

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TH, SG = 1.0, 5.0
DEV = "cuda:0"


def rng_inputs(seed, T, N, kind="spiking"):
    g = np.random.default_rng(seed)
    if kind == "spiking":
        x = g.standard_normal((T, N)) * 5.0
    elif kind == "config":
        x = g.normal(0.3, 0.5, size=(T, N))
    else:
        x = g.normal(1.5, 1.0, size=(T, N))
    gS = g.standard_normal((T, N))
    gV = g.standard_normal((T, N))
    v0 = g.standard_normal(N) * 0.1
    return (x.astype(np.float32), gS.astype(np.float32), gV.astype(np.float32),
            v0.astype(np.float32))


def glmulti_tables(T, seed=0, kind="toeplitz"):
    """The schedule as the reference builds it (Toeplitz, strictly lower, constant scale)
    or, with kind="general", arbitrary entries (the Function accepts any [T,T])."""
    if kind == "toeplitz":
        d = np.load(os.path.join(GOLDEN, "torch_tables.npz"))
        key = f"glmulti_W_T{T}"
        if key in d:
            return d[f"glmulti_scale_T{T}"], d[key]
        from dfsnn_b200 import schedule
        basis = schedule.glmulti_basis([0.3, 0.4, 0.5], T)
        terms = schedule.build_glmulti_schedule(torch.tensor([0.5, 0.5, 0.7]),
                                                torch.tensor([0.3, 0.4, 0.5]), basis, 0.1, T)
        return terms["scale"].contiguous().numpy().copy(), terms["weights"].numpy().copy()
    g = np.random.default_rng(seed)
    scale = (0.22385544 + 0.01 * g.standard_normal(T)).astype(np.float32)
    W = np.tril(g.standard_normal((T, T)).astype(np.float32) * 0.05, -1)
    return scale, W


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def cpu(t):
    return t.detach().float().cpu().numpy()


# -------------------------------------------------------------------------------------
# library glmulti
# -------------------------------------------------------------------------------------
GLM_CASES = [(T, N) for T in (1, 2, 3, 7, 8, 13, 16, 17, 31, 32) for N in (1, 255, 1000)] + \
            [(16, 4099), (8, 70001), (32, 5000)] + \
            [(T, N) for T in (8, 16) for N in (4, 32, 36, 4100, 70000, 100000)]


@pytest.mark.parametrize("T,N", GLM_CASES)
@pytest.mark.parametrize("full", [False, True])
@pytest.mark.parametrize("tau", [2.0, 1.7])
@pytest.mark.parametrize("kind", ["toeplitz", "general"])
def test_glmulti_vs_oracle(T, N, full, tau, kind):
    x, gS, _, v0 = rng_inputs(T * 1000 + N, T, N)
    scale, W = glmulti_tables(T, seed=T, kind=kind)
    r = O.glmulti_step(x, v0, scale, W, gS, tau, TH, SG, full)
    xt, v0t, st, Wt = cuda(x), cuda(v0), cuda(scale), cuda(W)
    xt.requires_grad_(True)
    v0t.requires_grad_(True)
    st.requires_grad_(True)
    Wt.requires_grad_(True)
    s = fde_kernels.LIFFDEGLMultiFunction.apply(xt, v0t, st, Wt, tau, TH, SG, 1, full)
    s.backward(cuda(gS))
    torch.cuda.synchronize()
    assert_bitwise(cpu(s), r["spike"], what="spike")
    assert_bitwise(cpu(xt.grad), r["gx"], what="gx")
    assert_bitwise(cpu(v0t.grad), r["gv0"], what="gv0")
    assert_close(cpu(st.grad), r["gscale"], what="grad_scale")
    assert_close(cpu(Wt.grad), r["gW"], what="grad_W")


def test_glmulti_forward_long_T_vs_oracle():
    for T in (33, 64, 100, 256):
        x, _, _, v0 = rng_inputs(T, T, 777)
        scale, W = glmulti_tables(T, seed=T, kind="general")
        r = O.glmulti_forward(x, v0, scale, W, 2.0, TH)
        with torch.no_grad():
            s = fde_kernels.LIFFDEGLMultiFunction.apply(cuda(x), cuda(v0), cuda(scale), cuda(W),
                                                        2.0, TH, SG, 1, False)
        assert_bitwise(cpu(s), r["spike"], what=f"spike T={T}")


def test_glmulti_dtype_and_determinism():
    T, N = 16, 30000
    x, gS, _, v0 = rng_inputs(5, T, N)
    scale, W = glmulti_tables(T)
    outs = []
    for _ in range(2):
        xt = cuda(x).half().requires_grad_(True)
        st, Wt = cuda(scale).requires_grad_(True), cuda(W).requires_grad_(True)
        s = fde_kernels.LIFFDEGLMultiFunction.apply(xt, cuda(v0), st, Wt, 2.0, TH, SG, 4, True)
        assert s.dtype == torch.float16
        s.backward(cuda(gS).half())
        assert xt.grad.dtype == torch.float16
        outs.append((cpu(st.grad), cpu(Wt.grad)))
    assert_bitwise(outs[0][0], outs[1][0], what="grad_scale rerun")
    assert_bitwise(outs[0][1], outs[1][1], what="grad_W rerun")


def test_glmulti_on_side_stream():
    T, N = 16, 5000
    x, gS, _, v0 = rng_inputs(9, T, N)
    scale, W = glmulti_tables(T)
    r = O.glmulti_step(x, v0, scale, W, gS, 2.0, TH, SG, True)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        xt = cuda(x).requires_grad_(True)
        s = fde_kernels.LIFFDEGLMultiFunction.apply(xt, cuda(v0), cuda(scale), cuda(W), 2.0, TH,
                                                    SG, 1, True)
        s.backward(cuda(gS))
    side.synchronize()
    assert_bitwise(cpu(s), r["spike"], what="spike")
    assert_bitwise(cpu(xt.grad), r["gx"], what="gx")


@pytest.mark.parametrize("T,full", [(65, True), (257, False)])
def test_glmulti_T_limit_raises(T, full):
    """Full history is limited to T <= 64 (as the reference); any history to T <= 256."""
    x = torch.zeros(T, 10, device=DEV, requires_grad=True)
    with pytest.raises(ValueError):
        fde_kernels.LIFFDEGLMultiFunction.apply(x, torch.zeros(10, device=DEV),
                                                torch.ones(T, device=DEV),
                                                torch.zeros(T, T, device=DEV), 2.0, TH, SG, 1,
                                                full)


@pytest.mark.parametrize("T,N,full", [(33, 1000, True), (48, 4099, True), (64, 2000, True),
                                      (33, 1000, False), (64, 2000, False), (100, 777, False),
                                      (256, 500, False)])
@pytest.mark.parametrize("tau", [2.0, 1.7])
@pytest.mark.parametrize("kind", ["toeplitz", "general"])
def test_glmulti_long_history_vs_oracle(T, N, full, tau, kind):
    """32 < T: shared-memory history kernels and the tiled parameter reduction."""
    x, gS, _, v0 = rng_inputs(T * 1000 + N + 7, T, N)
    scale, W = glmulti_tables(T, seed=T + 1, kind=kind)
    r = O.glmulti_step(x, v0, scale, W, gS, tau, TH, SG, full)
    xt, v0t, st, Wt = (cuda(z).requires_grad_(True) for z in (x, v0, scale, W))
    s = fde_kernels.LIFFDEGLMultiFunction.apply(xt, v0t, st, Wt, tau, TH, SG, 1, full)
    s.backward(cuda(gS))
    torch.cuda.synchronize()
    assert_bitwise(cpu(s), r["spike"], what="spike")
    assert_bitwise(cpu(xt.grad), r["gx"], what="gx")
    assert_bitwise(cpu(v0t.grad), r["gv0"], what="gv0")
    assert_close(cpu(st.grad), r["gscale"], what="grad_scale")
    assert_close(cpu(Wt.grad), r["gW"], what="grad_W")


def test_glmulti_empty_and_direct_capi():
    L = _capi.lib()
    T = 8
    scale, W = glmulti_tables(T)
    x = torch.zeros(T, 0, device=DEV)
    s = fde_kernels.LIFFDEGLMultiFunction.apply(x, torch.zeros(0, device=DEV), cuda(scale),
                                                cuda(W), 2.0, TH, SG, 1, True)
    assert s.shape == (T, 0)
    # direct C-ABI call on torch-owned buffers
    xx, _, _, v0 = rng_inputs(3, T, 513)
    out = torch.empty(T, 513, device=DEV)
    # keep every buffer referenced until the asynchronous launch has completed
    bufs = [cuda(xx), cuda(v0), cuda(scale), cuda(W)]
    code = L.dfsnn_glmulti_forward(*[_capi.ptr(b) for b in bufs], _capi.ptr(out), T, 513, 2.0,
                                   TH, None)
    torch.cuda.synchronize()
    assert code == 0
    assert_bitwise(cpu(out), O.glmulti_forward(xx, v0, scale, W, 2.0, TH)["spike"], what="spike")


# -------------------------------------------------------------------------------------
# aligned glmulti
# -------------------------------------------------------------------------------------
@pytest.mark.parametrize("T,N", [(T, N) for T in (1, 2, 5, 8, 11, 16, 24, 32) for N in (1, 300, 2049)]
                         + [(33, 300), (40, 2049), (64, 1000)]
                         + [(T, N) for T in (8, 16) for N in (4, 64, 4096, 70000)])
@pytest.mark.parametrize("tau", [2.0, 1.3])
@pytest.mark.parametrize("kind", ["toeplitz", "general"])
def test_aligned_vs_oracle(T, N, tau, kind):
    x, gS, _, v0 = rng_inputs(T * 31 + N, T, N)
    scale, W = glmulti_tables(T, seed=T, kind=kind)
    a = (scale * 4.0).astype(np.float32)
    r = O.aligned_step(x, v0, a, W, gS, tau, TH, SG, 1.0)
    xt, v0t, at, Wt = (cuda(z).requires_grad_(True) for z in (x, v0, a, W))
    s = alg.AlignedGLMulti.apply(xt, v0t, at, Wt, tau, TH, SG, 1, True)
    s.backward(cuda(gS))
    torch.cuda.synchronize()
    assert_bitwise(cpu(s), r["spike"], what="spike")
    assert_bitwise(cpu(xt.grad), r["gx"], what="gx")
    assert_bitwise(cpu(v0t.grad), r["gv0"], what="gv0")
    assert_close(cpu(at.grad), r["gscale"], what="grad_a")
    assert_close(cpu(Wt.grad), r["gW"], what="grad_w")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("T,N", [(8, 70001), (16, 4099), (16, 262144), (40, 1000)])
def test_aligned_half_precision_io(dtype, T, N):
    """Half-precision activations (autocast) are read and written in their own type by the
    forward kernel; spikes and gradients equal the fp32 path on x.float() bit for bit, which is
    what the reference's .float() / .to(dtype) casts compute (aligned_glmulti.py:112-145)."""
    x, gS, _, v0 = rng_inputs(41 + T, T, N, "steady")
    a, W = glmulti_tables(T)
    xh = cuda(x).to(dtype)
    gh = cuda(gS).to(dtype)
    outs = []
    for inp in (xh, xh.float()):
        xr = inp.clone().requires_grad_(True)
        vr = cuda(v0).requires_grad_(True)
        ar, Wr = cuda(a).requires_grad_(True), cuda(W).requires_grad_(True)
        s = alg.AlignedGLMulti.apply(xr, vr, ar, Wr, 2.0, TH, SG, 1, True)
        assert s.dtype == inp.dtype
        s.backward(gh.to(inp.dtype))
        outs.append((s.detach().float(), xr.grad.float(), vr.grad, ar.grad, Wr.grad))
    torch.cuda.synchronize()
    (s1, gx1, gv1, ga1, gw1), (s2, gx2, gv2, ga2, gw2) = outs
    assert_bitwise(cpu(s1), cpu(s2), what="spikes")
    assert_bitwise(cpu(gx1.to(dtype).float()), cpu(gx2.to(dtype).float()), what="grad_x (as dtype)")
    assert_bitwise(cpu(gv1), cpu(gv2), what="grad_v0")
    assert_bitwise(cpu(ga1), cpu(ga2), what="grad_a")
    assert_bitwise(cpu(gw1), cpu(gw2), what="grad_w")


def test_aligned_history_rho():
    T, N = 16, 1000
    x, gS, _, v0 = rng_inputs(77, T, N)
    scale, W = glmulti_tables(T)
    old = alg.HISTORY_RHO
    try:
        alg.HISTORY_RHO = 0.5
        r = O.aligned_step(x, v0, scale * 4, W, gS, 2.0, TH, SG, 0.5)
        xt = cuda(x).requires_grad_(True)
        s = alg.AlignedGLMulti.apply(xt, cuda(v0), cuda(scale * 4), cuda(W), 2.0, TH, SG, 1, True)
        s.backward(cuda(gS))
        assert_bitwise(cpu(xt.grad), r["gx"], what="gx rho=0.5")
    finally:
        alg.HISTORY_RHO = old


# -------------------------------------------------------------------------------------
# single-order schemes
# -------------------------------------------------------------------------------------
SCHEME_FN = {"gl": fde_kernels.LIFFDEGLFunction, "trap": fde_kernels.LIFFDETRAPFunction,
             "predictor": fde_kernels.LIFFDEPREDICTORFunction, "gl1": fde_kernels.LIFFDEGL1Function,
             "trap1": fde_kernels.LIFFDETRAP1Function,
             "predictor1": fde_kernels.LIFFDEPREDICTOR1Function,
             "euler": fde_kernels.LIFEulerFunction}
BASE_TABLE = {"gl1": "gl", "trap1": "trap", "predictor1": "predictor"}


def single_weights(method, beta, T):
    if method == "euler":
        return np.zeros(T + 1, np.float32)       # no history term (the Function takes no table)
    d = np.load(os.path.join(GOLDEN, "torch_tables.npz"))
    base = BASE_TABLE.get(method, method)
    key = f"{base}_b{beta}_T{T}"
    if key in d:
        return d[key]
    from dfsnn_b200 import schedule
    fn = {"gl": schedule.gl_weights, "trap": schedule.trap_weights,
          "predictor": schedule.predictor_weights}[base]
    return fn(beta, T).numpy()


def run_single(method, x, v0, w, tau, beta, gS, gV, h=0.1):
    hb, g1 = h ** beta, math.exp(math.lgamma(beta + 1.0))
    xt, v0t = cuda(x).requires_grad_(True), cuda(v0).requires_grad_(True)
    wt = cuda(w)
    fn = SCHEME_FN[method]
    if method == "euler":
        s, v = fn.apply(xt, v0t, tau, TH, 0.0, SG)
    elif method in ("gl", "trap", "trap1"):
        if method == "trap1":
            hb = 1.0                                   # the Function passes 1**beta
        s, v = fn.apply(xt, v0t, wt, tau, beta, TH, 0.0, SG)
    elif method == "gl1":
        s, v = fn.apply(xt, v0t, wt, tau, beta, h, TH, 0.0, SG)
    else:
        s, v = fn.apply(xt, v0t, wt, tau, beta, TH, 0.0, SG, hb, g1)
    torch.autograd.backward([s, v], [cuda(gS), cuda(gV)])
    torch.cuda.synchronize()
    return cpu(s), cpu(v), cpu(xt.grad), cpu(v0t.grad), hb, g1


@pytest.mark.parametrize("method", ["gl", "trap", "predictor", "gl1", "trap1", "predictor1",
                                    "euler"])
@pytest.mark.parametrize("T,N", [(1, 50), (5, 999), (8, 1000), (16, 4099), (20, 512), (32, 300),
                                 (33, 300), (64, 1000), (100, 257), (256, 130), (8, 2), (16, 2),
                                 (16, 4100), (8, 70002), (16, 70000),
                                 # around the switch to the L2-history kernel (T >= 128), with
                                 # T % 4 != 0 (weight-table alignment) and ragged 16-step blocks
                                 (127, 40), (128, 40), (131, 77), (150, 300), (203, 65),
                                 (256, 1)])
@pytest.mark.parametrize("tau", [2.0, 0.7])
def test_single_vs_oracle(method, T, N, tau):
    beta = 0.7 if T != 64 else 0.5
    x, gS, gV, v0 = rng_inputs(T * 7 + N, T, N)
    w = single_weights(method, beta, T)
    s, v, gx, gv0, hb, g1 = run_single(method, x, v0, w, tau, beta, gS, gV)
    so, vo = O.single_forward(method, x, v0, w, tau, beta, TH, hb, g1)
    assert_bitwise(s, so, what="spike")
    assert_bitwise(v, vo, what="v")
    gxo, gv0o = O.single_backward(method, gS, gV, x, v0, w, tau, beta, TH, SG, hb, g1,
                                  spike=so, vseq=vo)
    assert_bitwise(gx, gxo, what="gx")
    assert_bitwise(gv0, gv0o, what="gv0")


# -------------------------------------------------------------------------------------
# direct Euler
# -------------------------------------------------------------------------------------
@pytest.mark.parametrize("T,N", [(1, 10), (8, 1000), (16, 4099), (40, 333)])
def test_direct_euler_vs_oracle(T, N):
    x, gS, _, v0 = rng_inputs(T + N, T, N)
    sc, gain, bias = 1.2, 0.9, 0.1
    tau, th, step, rs, sdt = 2.0, 1.0, 1.0, 1.0, 0.5
    fw = O.euler_forward(x, v0, sc, gain, bias, tau, th, step, rs, sdt)
    gzf = np.random.default_rng(1).standard_normal(N).astype(np.float32)
    gxo, gz0o, g3o = O.euler_backward(gS, gzf, x, fw["zpre"], fw["sin"], sc, gain, tau, step, SG, sdt)
    xt, zt = cuda(x).requires_grad_(True), cuda(v0).requires_grad_(True)
    pt = [torch.tensor(v, device=DEV, requires_grad=True) for v in (sc, gain, bias)]
    s, zf = deu.lif_like_euler_cupy(xt, zt, pt[0], pt[1], pt[2], tau, th, step, rs, SG, sdt)
    torch.autograd.backward([s, zf], [cuda(gS), cuda(gzf)])
    torch.cuda.synchronize()
    assert_bitwise(cpu(s), fw["spike"], what="spike")
    assert_bitwise(cpu(zf), fw["zfinal"], what="z_final")
    assert_bitwise(cpu(xt.grad), gxo, what="gx")
    assert_bitwise(cpu(zt.grad), gz0o, what="gz0")
    got3 = np.array([float(p.grad) for p in pt])
    assert_close(got3, g3o, rtol=RTOL, atol_scale=float(np.abs(g3o).max()), what="scalar grads")


# -------------------------------------------------------------------------------------
# golden fixtures from the reference
# -------------------------------------------------------------------------------------
def load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


@pytest.mark.parametrize("method", ["gl", "trap", "predictor"])
def test_single_vs_reference_kernel_golden(method):
    d = load(f"kern_{method}_T16.npz")
    beta = float(d["beta"])
    hb, g1 = float(d["h_beta"]), float(d["gamma1"])
    xt, v0t = cuda(d["x"]).requires_grad_(True), cuda(d["v0"]).requires_grad_(True)
    args = (xt, v0t, cuda(d["w"]), 2.0, beta, TH, 0.0, SG)
    if method == "predictor":
        args = args + (hb, g1)
    s, v = SCHEME_FN[method].apply(*args)
    torch.autograd.backward([s, v], [cuda(d["gS"]), cuda(d["gV"])])
    assert_bitwise(cpu(s), d["spike"], what="spike")
    assert_bitwise(cpu(v), d["v"], what="v")
    assert_bitwise(cpu(xt.grad), d["gx"], what="gx")
    assert_bitwise(cpu(v0t.grad), d["gv0"], what="gv0")


def test_aligned_vs_reference_kernel_golden():
    d = load("kern_aligned_T16.npz")
    xt, v0t = cuda(d["x"]).requires_grad_(True), cuda(d["v0"]).requires_grad_(True)
    s = alg.AlignedGLMulti.apply(xt, v0t, cuda(d["a"]), cuda(d["W"]), 2.0, TH, SG, 1, True)
    s.backward(cuda(d["gS"]))
    assert_bitwise(cpu(s), d["spike"], what="spike")
    assert_bitwise(cpu(xt.grad), d["gx"], what="gx")
    assert_bitwise(cpu(v0t.grad), d["gv0"], what="gv0")


@pytest.mark.parametrize("kind", ["trunc", "full"])
def test_glmulti_vs_reference_kernel_golden(kind):
    d = load(f"kern_glmulti_{kind}_T16.npz")
    xt, v0t = cuda(d["x"]).requires_grad_(True), cuda(d["v0"]).requires_grad_(True)
    s = fde_kernels.LIFFDEGLMultiFunction.apply(xt, v0t, cuda(d["scale"]), cuda(d["W"]), 2.0, TH,
                                                SG, 1, kind == "full")
    s.backward(cuda(d["gS"]))
    mask = assert_spikes(cpu(s), d["spike"], d["vpre"], TH)
    assert_close(cpu(xt.grad), d["gx"], rtol=RTOL, mask=mask, what="gx")
    assert_close(cpu(v0t.grad), d["gv0"], rtol=RTOL, mask=mask, what="gv0")


@pytest.mark.parametrize("case", ["spiking_T16", "steady_T8"])
def test_glmulti_vs_reference_torch_golden(case):
    d = load(f"torch_glmulti_full_{case}.npz")
    T, N = d["x"].shape
    xt = cuda(d["x"]).requires_grad_(True)
    v0t = torch.zeros(N, device=DEV, requires_grad=True)
    Wt = cuda(d["W"]).requires_grad_(True)
    s = fde_kernels.LIFFDEGLMultiFunction.apply(xt, v0t, cuda(d["scale"]), Wt, 2.0, TH, SG, 4, True)
    s.backward(cuda(d["gS"]))
    r = O.glmulti_forward(d["x"], np.zeros(N, np.float32), d["scale"], d["W"], 2.0, TH)
    mask = assert_spikes(cpu(s), d["spike"], r["vpre"], TH)
    assert_close(cpu(xt.grad), d["gx"], rtol=1e-4, mask=mask, what="gx")
    assert_close(cpu(v0t.grad), d["gv0"], rtol=1e-4, mask=mask, what="gv0")
    assert_close(cpu(Wt.grad), d["gW"], rtol=1e-4, what="gW")


@pytest.mark.parametrize("case", ["spiking_T16", "config1_T16"])
def test_neuron_mirror_vs_reference_torch_neuron(case):
    """LIFNeuronFDE mirror (glmulti, truncated) vs the reference LIFNeuronFDE torch path."""
    d = load(f"torch_glmulti_neuron_{case}.npz")
    n = neuron.LIFNeuronFDE(tau=2.0, threshold=TH, surrogate_grad_scale=SG,
                            surrogate_function="arctan", beta=0.3, T=16, method="glmulti",
                            step_size=0.1, batchsize=4, step_mode="m", backend="cupy",
                            multi_beta=[0.3, 0.4, 0.5], multi_coefficient=[0.5, 0.5, 0.7],
                            learn_coefficient=True, coefficient_constraint="softplus",
                            glmulti_history_grad="truncated").to(DEV)
    xt = cuda(d["x"]).requires_grad_(True)
    s = n(xt)
    (s * cuda(d["gS"])).sum().backward()
    T = d["x"].shape[0]
    assert (cpu(s) == d["spike"]).all()
    assert_close(cpu(xt.grad).reshape(T, -1), d["gx"].reshape(T, -1), rtol=1e-4, what="gx")
    assert_close(cpu(n.multi_coefficient_raw.grad), d["graw"], rtol=1e-4, what="grad raw")


# -------------------------------------------------------------------------------------
# full-size properties (configuration sizes too large for a full oracle run)
# -------------------------------------------------------------------------------------
def test_glmulti_full_size_sampled_columns_and_reductions():
    """[T=16, N=8,388,608]: every neuron is independent, so a random sample of columns is
    checked bit-for-bit against the oracle; the reductions over all N are checked against
    the double-precision oracle on a 2**21-neuron slice computed both ways."""
    T, N = 16, 16 * 128 * 64 * 64
    g = torch.Generator(device=DEV).manual_seed(0)
    x = (torch.randn(T, N, device=DEV, generator=g) * 0.5 + 0.3)
    gS = torch.randn(T, N, device=DEV, generator=g)
    scale, W = glmulti_tables(T)
    xt = x.clone().requires_grad_(True)
    s = fde_kernels.LIFFDEGLMultiFunction.apply(xt, torch.zeros(N, device=DEV), cuda(scale),
                                                cuda(W), 2.0, TH, SG, 16, True)
    s.backward(gS)
    cols = torch.randint(0, N, (4096,), device=DEV, generator=g)
    xs, gss = cpu(x[:, cols]), cpu(gS[:, cols])
    r = O.glmulti_step(xs, np.zeros(4096, np.float32), scale, W, gss, 2.0, TH, SG, True)
    assert_bitwise(cpu(s[:, cols]), r["spike"], what="spike sample")
    assert_bitwise(cpu(xt.grad[:, cols]), r["gx"], what="gx sample")
    n2 = 1 << 21
    st, Wt = cuda(scale).requires_grad_(True), cuda(W).requires_grad_(True)
    s2 = fde_kernels.LIFFDEGLMultiFunction.apply(x[:, :n2].contiguous(), torch.zeros(n2, device=DEV),
                                                 st, Wt, 2.0, TH, SG, 1, True)
    s2.backward(gS[:, :n2].contiguous())
    r2 = O.glmulti_step(cpu(x[:, :n2]), np.zeros(n2, np.float32), scale, W, cpu(gS[:, :n2]), 2.0,
                        TH, SG, True)
    assert_close(cpu(st.grad), r2["gscale"], what="grad_scale 2M")
    assert_close(cpu(Wt.grad), r2["gW"], what="grad_W 2M")
