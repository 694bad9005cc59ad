"""Multi-term Grünwald–Letnikov integrator of the SNN wrapper path on B200.

Drop-ins for spikeDE_dis/solver.py's forward_glmulti_cupy (:3270-3369; called by
spikeDE_dis/snn.py:906 and, through CUPY_SOLVERS_FORWARD, by FDEAdjointMethod) and
backward_glmulti_cupy (:2905-3002; CUPY_SOLVERS_BACKWARD and TORCH_SOLVERS_BACKWARD),
with the same signatures, return values, error types and autograd behaviour.

Each integrator step and state component is one native launch (dfsnn_gl_history_step):
    y_{k+1} = c~_0^{-1} * (f_k - sum_j c~[k+1-j] * y_j)
reading the history rows in place through a device table of row pointers -- the reference
stacks the rows into a new tensor every step and runs 3+ kernels.  The coefficient table
c~ is built with the reference's own PyTorch operations on the state's device, so the
values are identical.  Note: forward_glmulti_cupy weights history row j (= y_{j+1}) with
c~[k+1-j] (:3314-3316), one lag further than the PyTorch integrator
glmethod_multiterm_integrate_tuple (c~[k-j], :3879); the drop-in keeps the CuPy function's
indexing, and the adjoint's c~[k+1-j] over rows 0..k (:2968-2970).

float32 and float64 states are native; float16 (accepted by the reference through CuPy's
dot) raises TypeError.
"""
import torch

from . import _capi
from . import profiling as _prof

_DTYPE = {torch.float32: 0, torch.float64: 1}


def _check_backend(device, dtype, what):
    if device.type != "cuda":
        raise RuntimeError(f"{what} requires CUDA tensors.")
    if dtype not in _DTYPE:
        raise TypeError(f"{what} supports float32/float64 states, got {dtype}.")


def glmulti_c_tilde(beta, coefficient, h, N, dtype, device):
    """c~[0..N] and 1/c~[0] with the reference's PyTorch operations (solver.py:3302-3312):
    c[:, m] = (1 - (1+beta)/m) c[:, m-1], c~ = sum_j coefficient_j h^-beta_j c[j]."""
    n_terms = len(beta)
    c = torch.zeros(n_terms, N + 1, dtype=dtype, device=device)
    c[:, 0] = 1.0
    for m in range(1, N + 1):
        c[:, m] = (1 - (1 + beta) / m) * c[:, m - 1]
    weighted_h = coefficient * torch.pow(h, -beta)
    c_tilde = torch.sum(weighted_h.unsqueeze(1) * c, dim=0)
    return c_tilde, 1.0 / c_tilde[0]


def _as_tensor(v, dtype, device):
    if isinstance(v, torch.Tensor):
        return v.to(device=device, dtype=dtype)
    return torch.tensor(v, dtype=dtype, device=device)


def _launch_step(f, table, row_begin, row_end, c_tilde, coeff_base, c0_inv, chunk, out, diff,
                 slot):
    L = _capi.lib()
    # algorithmic bytes: f and the history rows in, y (and f - conv) out
    nbytes = f.numel() * f.element_size() * (row_end - row_begin + 2 + (diff is not None))
    with _prof.native_call("gl_history_step", 1, nbytes, f.device):
        code = L.dfsnn_gl_history_step(
            _DTYPE[f.dtype], _capi.ptr(f), _capi.ptr(table), row_begin, row_end,
            _capi.ptr(c_tilde), coeff_base, _capi.ptr(c0_inv), chunk, _capi.ptr(out),
            _capi.ptr(diff), f.numel(), _capi.ptr(table) if slot is not None else None,
            -1 if slot is None else slot, _capi.stream_of(f))
    _capi.check(code, "dfsnn_gl_history_step")


class _GLHistoryStep(torch.autograd.Function):
    """y = c0_inv * (f - conv) with the history sum attached to autograd or not (the
    reference's detach_conv); rows are the history tensors the sum reads (only passed, and
    only differentiated, when attached)."""

    @staticmethod
    def forward(ctx, f, c0_inv, c_tilde, table, row_begin, row_end, coeff_base, slot, chunk,
                attached, *rows):
        out = torch.empty_like(f)
        diff = torch.empty_like(f) if ctx.needs_input_grad[1] else None
        with torch.cuda.device(f.device):
            _launch_step(f, table, row_begin, row_end, c_tilde, coeff_base, c0_inv, chunk, out,
                         diff, slot)
        ctx.save_for_backward(c0_inv, c_tilde, diff, table)
        ctx.meta = (row_begin, row_end, coeff_base, bool(attached), len(rows), f.shape)
        ctx.keep_rows = rows      # alive while this step can be differentiated
        return out

    @staticmethod
    def backward(ctx, g):
        c0_inv, c_tilde, diff, table = ctx.saved_tensors
        row_begin, row_end, coeff_base, attached, nrows, shape = ctx.meta
        g = g.contiguous()
        L = row_end - row_begin
        grad_f = torch.empty_like(g)
        want_rows = attached and any(ctx.needs_input_grad[10:])
        want_coeff = attached and ctx.needs_input_grad[2] and L > 0
        want_c0 = ctx.needs_input_grad[1]
        grad_rows = torch.empty((L,) + tuple(shape), dtype=g.dtype, device=g.device) \
            if want_rows and L > 0 else None
        grad_coeff = torch.empty(L, dtype=g.dtype, device=g.device) if want_coeff else None
        grad_c0 = torch.empty((), dtype=g.dtype, device=g.device) if want_c0 else None
        lib = _capi.lib()
        with torch.cuda.device(g.device):
            nbytes = int(lib.dfsnn_gl_history_step_workspace_size(L, g.numel()))
            ws = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=g.device)
            code = lib.dfsnn_gl_history_step_backward(
                _DTYPE[g.dtype], _capi.ptr(g), _capi.ptr(c0_inv), _capi.ptr(table), row_begin,
                row_end, _capi.ptr(c_tilde), coeff_base, _capi.ptr(diff), _capi.ptr(grad_f),
                _capi.ptr(grad_rows), _capi.ptr(grad_coeff), _capi.ptr(grad_c0), g.numel(),
                _capi.ptr(ws), ws.numel(), _capi.stream_of(g))
        _capi.check(code, "dfsnn_gl_history_step_backward")
        gct = None
        if grad_coeff is not None:
            gct = torch.zeros_like(c_tilde)
            idx = coeff_base - torch.arange(row_begin, row_end, device=g.device)
            gct.index_add_(0, idx, grad_coeff)
        row_grads = [None] * nrows
        if grad_rows is not None:
            row_grads = list(grad_rows.unbind(0))
        return (grad_f, grad_c0, gct, None, None, None, None, None, None, None, *row_grads)


def forward_glmulti_cupy(ode_func, y0_tuple, alpha, t_grid: torch.Tensor, memory=None,
                         multi_coefficient=None, history_chunk_size=None, detach_conv=True):
    if not isinstance(y0_tuple, tuple) or len(y0_tuple) == 0:
        raise TypeError("y0_tuple must be a non-empty tuple for CuPy multi-term GL solver.")
    if multi_coefficient is None:
        raise ValueError("multi_coefficient must be provided for CuPy multi-term GL solver.")
    N = len(t_grid)
    if N < 2:
        raise ValueError("t_grid must contain at least two elements for multi-term GL integration.")
    T = N - 1
    device = y0_tuple[0].device
    dtype = y0_tuple[0].dtype
    _check_backend(device, dtype, "forward_glmulti_cupy")
    t_grid = t_grid.to(device=device, dtype=dtype)
    h = t_grid[-1] - t_grid[-2]
    beta = _as_tensor(alpha, dtype, device)
    coefficient = _as_tensor(multi_coefficient, dtype, device)
    if len(coefficient) != len(beta):
        raise ValueError("beta and multi_coefficient must have the same length.")
    c_tilde, c0_inv = glmulti_c_tilde(beta, coefficient, h, N, dtype, device)
    chunk = 96 if history_chunk_size is None else int(history_chunk_size)
    kchunk = chunk if chunk > 0 else -1
    attached = not detach_conv

    n_integrate = max(0, len(y0_tuple) - 1)
    y_history = [[] for _ in y0_tuple]
    y_current = list(y0_tuple)
    tables = [torch.zeros(max(T, 1), dtype=torch.int64, device=device) for _ in range(n_integrate)]
    for k in range(T):
        f_k = ode_func(t_grid[k], tuple(y_current))
        if not isinstance(f_k, tuple) or len(f_k) != len(y0_tuple):
            raise TypeError("ODE function must return a tuple matching y0_tuple length.")
        if memory is None or memory == -1:
            memory_length = k + 1
        else:
            memory_length = min(memory, k + 1)
            if memory_length <= 0:
                raise ValueError("memory must be greater than 0 when provided.")
        start_idx = max(0, k + 1 - memory_length)
        row_end = k if k > start_idx else start_idx
        for i in range(n_integrate):
            f = f_k[i].to(dtype=dtype).contiguous()
            rows = y_history[i][start_idx:row_end]
            grad = torch.is_grad_enabled() and (
                f.requires_grad or c0_inv.requires_grad or
                (attached and (c_tilde.requires_grad or any(r.requires_grad for r in rows))))
            if grad:
                y_val = _GLHistoryStep.apply(f, c0_inv, c_tilde, tables[i], start_idx, row_end,
                                             k + 1, k, kchunk, attached,
                                             *(rows if attached else ()))
            else:
                y_val = torch.empty_like(f)
                with torch.cuda.device(device):
                    _launch_step(f, tables[i], start_idx, row_end, c_tilde.detach(), k + 1,
                                 c0_inv.detach(), kchunk, y_val, None, k)
            y_current[i] = y_val
            y_history[i].append(y_val)
        y_current[-1] = f_k[-1]
        y_history[-1].append(y_current[-1])
    return y_history


def backward_glmulti_cupy(ode_func, y_aug, alpha, t_grid, yhistory, memory=None,
                          multi_coefficient=None):
    with torch.no_grad():
        if not yhistory:
            raise ValueError("yhistory must not be empty for GL multi-term adjoint.")
        if multi_coefficient is None:
            raise ValueError("multi_coefficient must be provided for GL multi-term adjoint.")
        N = t_grid.numel()
        if N < 2:
            raise ValueError("t_grid must contain at least two points for GL multi-term adjoint.")
        steps = N - 1
        h = torch.abs(t_grid[-1] - t_grid[-2])
        _, adj_y0, adj_params0 = y_aug
        device = adj_y0[0].device
        dtype = adj_y0[0].dtype
        _check_backend(device, dtype, "backward_glmulti_cupy")
        beta = _as_tensor(alpha, dtype, device)
        coefficient = _as_tensor(multi_coefficient, dtype, device)
        if len(coefficient) != len(beta):
            raise ValueError("beta and multi_coefficient must have the same length.")
        c_tilde, c0_inv = glmulti_c_tilde(beta, coefficient, h, N, dtype, device)

        adj_y = list(adj_y0)
        adj_params = list(adj_params0)
        shapes = [a.shape for a in adj_y0]
        esize = torch.empty((), dtype=dtype).element_size()
        buffers, tables = [], []
        for a in adj_y0:
            buf = torch.empty((steps, a.numel()), device=device, dtype=dtype)
            buf[0].copy_(a.detach().reshape(-1))
            buffers.append(buf)
            stride = a.numel() * esize
            tables.append(buf.data_ptr() + torch.arange(steps, device=device,
                                                        dtype=torch.int64) * stride)
        for k in range(N - 2):
            tk = t_grid[k]
            y_state = list(y[-k - 2] for y in yhistory)
            _, vjp_y, vjp_params = ode_func(tk, (y_state, adj_y, adj_params))
            if memory is None or memory == -1:
                memory_length = k + 1
            else:
                memory_length = min(memory, k + 1)
            start_idx = max(0, k + 1 - memory_length)
            for i in range(len(adj_y)):
                f = vjp_y[i].to(dtype=dtype).contiguous()
                out = buffers[i][k + 1]
                with torch.cuda.device(device):
                    _launch_step(f, tables[i], start_idx, k + 1, c_tilde, k + 1, c0_inv, 0, out,
                                 None, None)
                adj_y[i] = out.view(shapes[i])
            if adj_params and vjp_params:
                for ap, vp in zip(adj_params, vjp_params):
                    ap.add_(vp, alpha=h)
        if N > 2:       # the returned adjoints must not keep the history buffers alive
            adj_y = [a.clone() for a in adj_y]
        del buffers, tables
        return adj_y, adj_params


def install(solver_module=None):
    """Point spikeDE_dis.solver's glmulti entries (module attributes and the CuPy / torch
    dispatch tables, solver.py:4752-4806) at these drop-ins; spikeDE_dis.snn imports
    forward_glmulti_cupy by name at import time, so it is rebound there as well."""
    import sys
    mods = [solver_module] if solver_module is not None else \
        [sys.modules.get("spikeDE_dis.solver")]
    for m in mods:
        if m is None:
            continue
        m.forward_glmulti_cupy = forward_glmulti_cupy
        m.backward_glmulti_cupy = backward_glmulti_cupy
        for table, fn in (("CUPY_SOLVERS_FORWARD", forward_glmulti_cupy),
                          ("CUPY_SOLVERS_BACKWARD", backward_glmulti_cupy),
                          ("TORCH_SOLVERS_BACKWARD", backward_glmulti_cupy)):
            d = getattr(m, table, None)
            if isinstance(d, dict) and "glmulti" in d:
                d["glmulti"] = fn
    snn = sys.modules.get("spikeDE_dis.snn")
    if snn is not None and hasattr(snn, "forward_glmulti_cupy"):
        snn.forward_glmulti_cupy = forward_glmulti_cupy
