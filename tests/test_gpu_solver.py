"""GPU parity of the multi-term GL integrator drop-ins (dfsnn_b200.fde_solver) for the SNN
wrapper path: forward_glmulti_cupy and backward_glmulti_cupy (spikeDE_dis/solver.py
:3270-3369, :2905-3002).

The step kernel and the integrators are compared bit for bit with the oracle (whose step is
pinned against the reference's weighted_sum kernel source compiled for the host); the
ODE right-hand sides used here are exact in IEEE arithmetic (a power-of-two scale plus an
addend), so host and device evaluate them identically.  Gradients are compared with a
PyTorch autograd restatement of the reference function (stack, weighted sum, subtract,
scale) at 1e-12 (float64) / 1e-5 (float32).
"""
import numpy as np
import pytest
import torch

from dfsnn_b200 import fde_solver as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BETA = [0.3, 0.4, 0.5]
COEF = [0.5, 0.5, 0.7]


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("L,Sz", [(0, 5), (1, 1000), (5, 999), (97, 300), (200, 70001)])
@pytest.mark.parametrize("chunk", [96, 3, 0, -1])
def test_step_kernel_vs_oracle(dtype, L, Sz, chunk):
    g = torch.Generator(device=DEV).manual_seed(L * 7 + Sz)
    rows = [torch.randn(Sz, device=DEV, dtype=dtype, generator=g) for _ in range(L)]
    f = torch.randn(Sz, device=DEV, dtype=dtype, generator=g)
    c_tilde = torch.randn(L + 2, device=DEV, dtype=dtype, generator=g)
    c0_inv = torch.tensor(0.37, device=DEV, dtype=dtype)
    table = torch.tensor([r.data_ptr() for r in rows] + [0], device=DEV, dtype=torch.int64)
    out = torch.empty_like(f)
    S._launch_step(f, table, 0, L, c_tilde, L + 1, c0_inv, chunk, out, None, L)
    torch.cuda.synchronize()
    assert int(table[L].item()) == out.data_ptr()               # the kernel registered its row
    coef = _np(c_tilde)[[L + 1 - j for j in range(L)]]
    hist = np.stack([_np(r) for r in rows]) if L else np.zeros((0, Sz), _np(f).dtype)
    want = O.gl_step(_np(f), hist, coef, float(c0_inv), chunk)
    assert np.array_equal(_np(out), want)


def rhs_factory(u, dtype):
    """f(t_k, y) = (-0.5*y0 + u_k, 2*y0): exact in IEEE on host and device."""
    state = {"k": 0}

    def ode_func(t, y):
        k = state["k"]
        state["k"] += 1
        return (-0.5 * y[0] + u[k], 2.0 * y[0])

    return ode_func


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("memory", [None, 3])
@pytest.mark.parametrize("chunk", [None, 2, 0])
@pytest.mark.parametrize("T", [1, 2, 7, 20])
def test_forward_integrator_vs_oracle(dtype, memory, chunk, T):
    g = torch.Generator(device=DEV).manual_seed(T)
    shape = (3, 5, 7)
    u = torch.randn((T,) + shape, device=DEV, dtype=dtype, generator=g)
    y0 = torch.randn(shape, device=DEV, dtype=dtype, generator=g)
    t_grid = torch.linspace(0, 0.1 * T, T + 1, device=DEV, dtype=dtype)
    hist = S.forward_glmulti_cupy(rhs_factory(u, dtype), (y0, torch.zeros_like(y0)),
                                  torch.tensor(BETA), t_grid, memory=memory,
                                  multi_coefficient=torch.tensor(COEF), history_chunk_size=chunk)
    assert len(hist) == 2 and len(hist[0]) == T and len(hist[1]) == T
    c_tilde, c0_inv = S.glmulti_c_tilde(torch.tensor(BETA).to(DEV, dtype),
                                        torch.tensor(COEF).to(DEV, dtype),
                                        t_grid[-1] - t_grid[-2], T + 1, dtype, DEV)
    un = _np(u)
    want = O.glmulti_integrate(lambda k, y: (y * -0.5 + un[k]).astype(un.dtype), _np(y0),
                               _np(c_tilde), float(c0_inv), T, memory,
                               96 if chunk is None else chunk)
    for k in range(T):
        assert np.array_equal(_np(hist[0][k]), want[k]), f"step {k}"
        prev = _np(y0) if k == 0 else want[k - 1]
        assert np.array_equal(_np(hist[1][k]), 2.0 * prev)


def torch_restatement(ode_func, y0, beta, t_grid, coefficient, memory, chunk, detach):
    """The reference forward_glmulti_cupy's operations in PyTorch (stack + weighted sum over
    chunks, subtract, scale) for the autograd comparison."""
    N = len(t_grid)
    dtype, device = y0[0].dtype, y0[0].device
    h = t_grid[-1] - t_grid[-2]
    c_tilde, c0_inv = S.glmulti_c_tilde(beta, coefficient, h, N, dtype, device)
    hist = [[] for _ in y0]
    cur = list(y0)
    for k in range(N - 1):
        f = ode_func(t_grid[k], tuple(cur))
        mem = k + 1 if memory is None else min(memory, k + 1)
        start = max(0, k + 1 - mem)
        for i in range(len(y0) - 1):
            conv = torch.zeros_like(f[i])
            if k > start:
                idx = k + 1 - torch.arange(start, k, device=device)
                coeff = c_tilde.index_select(0, idx)
                H = torch.stack(hist[i][start:k])
                if detach:
                    coeff, H = coeff.detach(), H.detach()
                conv = (coeff.view(-1, *[1] * f[i].dim()) * H).sum(0)
            y = c0_inv * (f[i] - conv)
            cur[i] = y
            hist[i].append(y)
        cur[-1] = f[-1]
        hist[-1].append(f[-1])
    return hist


@pytest.mark.parametrize("detach", [True, False])
@pytest.mark.parametrize("memory", [None, 4])
def test_forward_integrator_autograd(detach, memory):
    dtype = torch.float64
    torch.manual_seed(0)
    lin = torch.nn.Linear(6, 6, dtype=dtype).to(DEV)
    T = 9
    u = torch.randn(T, 4, 6, device=DEV, dtype=dtype)
    t_grid = torch.linspace(0, 0.9, T + 1, device=DEV, dtype=dtype)
    grads = []
    for impl in ("native", "torch"):
        coefficient = torch.tensor(COEF, device=DEV, dtype=dtype, requires_grad=True)
        x0 = torch.randn(4, 6, device=DEV, dtype=dtype, generator=torch.Generator(
            device=DEV).manual_seed(1)).requires_grad_(True)
        ks = {"k": 0}

        def ode(t, y):
            k = ks["k"]
            ks["k"] += 1
            return (torch.tanh(lin(y[0])) + u[k], y[0] * 0.5)

        beta = torch.tensor(BETA, device=DEV, dtype=dtype)
        if impl == "native":
            hist = S.forward_glmulti_cupy(ode, (x0, torch.zeros_like(x0)), beta, t_grid,
                                          memory=memory, multi_coefficient=coefficient,
                                          history_chunk_size=3, detach_conv=detach)
        else:
            hist = torch_restatement(ode, (x0, torch.zeros_like(x0)), beta, t_grid, coefficient,
                                     memory, 3, detach)
        loss = sum((h * (i + 1)).sum() for i, h in enumerate(hist[0])) + hist[1][-1].sum()
        lin.zero_grad()
        loss.backward()
        grads.append([x0.grad.clone(), coefficient.grad.clone(), lin.weight.grad.clone(),
                      loss.detach()])
    for a, b in zip(*grads):
        assert torch.allclose(a, b, rtol=1e-10, atol=1e-12), (a, b)


def test_adjoint_vs_oracle():
    for dtype in (torch.float32, torch.float64):
        g = torch.Generator(device=DEV).manual_seed(2)
        N = 12
        t_grid = torch.linspace(0, 1.1, N, device=DEV, dtype=dtype)
        adj0 = [torch.randn(5, 9, device=DEV, dtype=dtype, generator=g)]
        c = torch.randn(5, 9, device=DEV, dtype=dtype, generator=g)
        yhist = [[torch.zeros(5, 9, device=DEV, dtype=dtype) for _ in range(N - 1)]]
        p = [torch.zeros(3, device=DEV, dtype=dtype)]

        def ode(tk, aug):
            _, adj, params = aug
            return None, [adj[0] * -0.5 + c], [torch.ones(3, device=DEV, dtype=dtype)]

        for memory in (None, 4):
            adj, params = S.backward_glmulti_cupy(ode, (None, adj0, [q.clone() for q in p]),
                                                  torch.tensor(BETA), t_grid, yhist, memory,
                                                  torch.tensor(COEF))
            c_tilde, c0_inv = S.glmulti_c_tilde(torch.tensor(BETA).to(DEV, dtype),
                                                torch.tensor(COEF).to(DEV, dtype),
                                                torch.abs(t_grid[-1] - t_grid[-2]), N, dtype, DEV)
            cn = _np(c)
            want = O.glmulti_adjoint(lambda k, a: (a * -0.5 + cn).astype(cn.dtype), _np(adj0[0]),
                                     _np(c_tilde), float(c0_inv), N - 1, memory)
            assert np.array_equal(_np(adj[0]), want)
            h = float(torch.abs(t_grid[-1] - t_grid[-2]))
            assert torch.allclose(params[0], torch.full((3,), (N - 2) * h, device=DEV,
                                                        dtype=dtype), rtol=1e-6)


def test_errors_and_install():
    y = torch.zeros(3, device=DEV)
    with pytest.raises(ValueError):
        S.forward_glmulti_cupy(lambda t, s: s, (y, y), [0.5], torch.tensor([0.0]),
                               multi_coefficient=[1.0])
    with pytest.raises(TypeError):
        S.forward_glmulti_cupy(lambda t, s: s, (y.half(), y.half()), [0.5],
                               torch.tensor([0.0, 0.1]), multi_coefficient=[1.0])
    with pytest.raises(RuntimeError):
        S.forward_glmulti_cupy(lambda t, s: s, (y.cpu(), y.cpu()), [0.5],
                               torch.tensor([0.0, 0.1]), multi_coefficient=[1.0])
    import types
    fake = types.ModuleType("fake_solver")
    fake.CUPY_SOLVERS_FORWARD = {"glmulti": None}
    fake.CUPY_SOLVERS_BACKWARD = {"glmulti": None}
    fake.TORCH_SOLVERS_BACKWARD = {"glmulti": None}
    S.install(fake)
    assert fake.CUPY_SOLVERS_FORWARD["glmulti"] is S.forward_glmulti_cupy
    assert fake.TORCH_SOLVERS_BACKWARD["glmulti"] is S.backward_glmulti_cupy
