"""Weight tables of the LIF-FDE schemes (host side, torch ops).

Restates the reference builders in spikeDE_dis/neuron.py with the same fp32 operations, so
the tables are bit-identical to the ones LIFNeuronFDE hands to its kernels:
  * glmulti basis c_m^(beta_j) (:1314-1317), masses softplus(raw) (:1488-1489),
    c~ = sum_j m_j h^-beta_j c^(beta_j) (:1461-1479) and the [T,T] schedule (:1494-1514).
    The reference fills W row by row in a Python loop (2T small launches per call); here
    W[t,i] = c~[t-i] / c~[0] is one gather, bit-identical, differentiable in the masses.
  * GL c_rev (:1446-1459), L1-2 trapezoid (:1516-1546), fractional predictor (:1548-1570).
"""
import math

import torch
import torch.nn.functional as F


def glmulti_basis(multi_beta, T):
    """[J, T+1] basis c_lag^(beta_j): c_0 = 1, c_m = (1 - (1+beta)/m) c_{m-1}."""
    beta = torch.as_tensor(multi_beta, dtype=torch.float32)
    basis = torch.zeros(beta.numel(), T + 1, dtype=torch.float32)
    basis[:, 0] = 1.0
    for lag in range(1, T + 1):
        basis[:, lag] = (1.0 - (1.0 + beta) / lag) * basis[:, lag - 1]
    return basis


def softplus_masses(raw):
    return F.softplus(raw)


def h_pow_neg_beta(h, multi_beta, device):
    """h^-beta exactly as _get_glmulti_weights evaluates it (torch.pow of a 0-dim h tensor on
    the given device).  Constant for a neuron: callers cache it instead of paying the
    host-to-device copy of h on every forward."""
    beta = multi_beta.to(device=device, dtype=torch.float32)
    return torch.pow(torch.tensor(h, device=device, dtype=torch.float32), -beta)


def glmulti_c_tilde(coefficient, multi_beta, basis, h, h_pow=None):
    """c~ (length T+1) and 1/c~_0 exactly as _get_glmulti_weights computes them."""
    device = basis.device
    coefficient = coefficient.to(device=device, dtype=torch.float32)
    if h_pow is None:
        h_pow = h_pow_neg_beta(h, multi_beta, device)
    weighted_h = coefficient * h_pow
    c_tilde = torch.sum(weighted_h.unsqueeze(1) * basis, dim=0)
    return c_tilde, 1.0 / c_tilde[0]


_LAG_CACHE = {}


def _lag_index(T, device):
    key = (T, device.type, device.index)
    got = _LAG_CACHE.get(key)
    if got is None:
        t = torch.arange(T, device=device)
        lag = t[:, None] - t[None, :]
        mask = lag > 0
        got = (lag.clamp_min(0), mask)
        _LAG_CACHE[key] = got
    return got


def build_glmulti_schedule(coefficient, multi_beta, basis, h, T, h_pow=None):
    """{'scale': [T], 'weights': [T,T]} of LIFNeuronFDE._build_glmulti_schedule."""
    c_tilde, c0_inv = glmulti_c_tilde(coefficient, multi_beta, basis, h, h_pow)
    lag, mask = _lag_index(T, c_tilde.device)
    weights = torch.where(mask, c_tilde[lag] * c0_inv, torch.zeros((), device=c_tilde.device))
    return {"scale": c0_inv.expand(T), "weights": weights}


class GLMultiScheduleFunction(torch.autograd.Function):
    """(scale[T], W[T,T]) of build_glmulti_schedule in one native launch per direction.

    src is the raw Softplus parameter (constraint 1) or the masses themselves (constraint 0);
    basis [J, T+1] and h_pow [J] as above.  The forward is bit-identical to the PyTorch chain
    above (same fp32 operations); the backward returns grad_src accumulated in double."""

    @staticmethod
    def forward(ctx, src, basis, h_pow, constraint):
        from . import _capi
        from . import profiling as _prof
        src_f = src.detach().float().contiguous()
        basis_f = basis.float().contiguous()
        hp = h_pow.float().contiguous()
        J, T1 = basis_f.shape
        T = T1 - 1
        dev = src_f.device
        scale = torch.empty(T, device=dev, dtype=torch.float32)
        W = torch.empty((T, T), device=dev, dtype=torch.float32)
        ct = torch.empty(T + 1, device=dev, dtype=torch.float32)
        with torch.cuda.device(dev), _prof.native_call(
                "glmulti_schedule_forward", 1, _prof.schedule_forward_bytes(J, T), dev):
            code = _capi.lib().dfsnn_glmulti_schedule_forward(
                _capi.ptr(src_f), _capi.ptr(basis_f), _capi.ptr(hp), J, T, int(constraint),
                _capi.ptr(scale), _capi.ptr(W), _capi.ptr(ct), _capi.stream_of(src_f))
        _capi.check(code, "glmulti schedule forward")
        ctx.save_for_backward(src_f, basis_f, hp, ct)
        ctx.constraint = int(constraint)
        ctx.src_dtype = src.dtype
        return scale, W

    @staticmethod
    def backward(ctx, grad_scale, grad_W):
        from . import _capi
        from . import profiling as _prof
        src_f, basis_f, hp, ct = ctx.saved_tensors
        J, T1 = basis_f.shape
        gs = None if grad_scale is None else grad_scale.float().contiguous()
        gw = None if grad_W is None else grad_W.float().contiguous()
        grad = torch.empty(J, device=src_f.device, dtype=torch.float32)
        with torch.cuda.device(src_f.device), _prof.native_call(
                "glmulti_schedule_backward", 1, _prof.schedule_backward_bytes(J, T1 - 1),
                src_f.device):
            code = _capi.lib().dfsnn_glmulti_schedule_backward(
                _capi.ptr(src_f), _capi.ptr(basis_f), _capi.ptr(hp), _capi.ptr(ct),
                _capi.ptr(gs), _capi.ptr(gw), J, T1 - 1, ctx.constraint, _capi.ptr(grad),
                _capi.stream_of(src_f))
        _capi.check(code, "glmulti schedule backward")
        return grad.to(ctx.src_dtype), None, None, None


def gl_weights(beta_val, T, device=None, dtype=torch.float32):
    c = torch.zeros(T + 1, device=device, dtype=dtype)
    c[0] = 1
    for j in range(1, T + 1):
        c[j] = (1 - (1 + beta_val) / j) * c[j - 1]
    return torch.flip(c, dims=[0])


def trap_weights(beta_val, T, device=None, dtype=torch.float32):
    w = torch.zeros(T + 1, device=device, dtype=dtype)
    w[0] = 1.0
    alpha = 1.0 - beta_val
    for j in range(1, T + 1):
        if j == 1:
            w[j] = torch.pow(torch.tensor(2.0, device=device, dtype=dtype), alpha) - 2.0
        else:
            term1 = torch.pow(torch.tensor(j + 1.0, device=device, dtype=dtype), alpha)
            term2 = 2.0 * torch.pow(torch.tensor(j, device=device, dtype=dtype), alpha)
            term3 = torch.pow(torch.tensor(j - 1.0, device=device, dtype=dtype), alpha)
            w[j] = term1 - term2 + term3
    return torch.flip(w, dims=[0])


def predictor_weights(beta_val, T, device=None, dtype=torch.float32):
    w = torch.zeros(T + 1, device=device, dtype=dtype)
    w[0] = 1.0
    for j in range(1, T + 1):
        if j == 1:
            w[j] = 1.0
        else:
            w[j] = (torch.pow(torch.tensor(j, dtype=dtype, device=device), beta_val - 1)
                    - torch.pow(torch.tensor(j - 1, dtype=dtype, device=device), beta_val - 1))
    return torch.flip(w, dims=[0])


def predictor_constants(beta, h):
    """(h^beta, Gamma(beta+1)) as _multi_step_forward_cupy passes them (:2211-2215)."""
    return h ** beta, math.exp(math.lgamma(beta + 1.0))


def build_vogl1_schedule(beta_schedule, step_size):
    """VO-GL1 terms for a shared beta[T] or per-sample beta[T, B] schedule
    (LIFNeuronFDE.build_vogl1_schedule, neuron.py:2010-2031): beta clamped to
    [1e-6, 1-1e-6], scale = h**beta, weights[t, i] = c_{t-i}^(beta_t) for i < t with
    c_0 = 1, c_m = (1 - (1+beta_t)/m) c_{m-1}.  The reference builds each row in a Python loop
    over lags; here the recurrence runs once for all t at a time (the same elementwise fp32
    operations, so the same values), and the rows are one gather.  Differentiable in beta."""
    beta = beta_schedule.to(dtype=torch.float32).clamp(1e-6, 1.0 - 1e-6)
    T = beta.shape[0]
    h = torch.as_tensor(step_size, device=beta.device, dtype=torch.float32)
    scale = torch.pow(h, beta)
    cols = [torch.ones_like(beta)]
    for lag in range(1, T):
        cols.append((1.0 - (1.0 + beta) / float(lag)) * cols[-1])
    C = torch.stack(cols, dim=-1)                          # [T, (B,) lag]
    t_idx = torch.arange(T, device=beta.device)
    lag = (t_idx[:, None] - t_idx[None, :]).clamp_min(0)   # [t, i]
    causal = t_idx[None, :] < t_idx[:, None]
    if beta.dim() == 1:
        W = torch.gather(C, 1, lag) * causal
    else:
        B = beta.shape[1]
        W = torch.gather(C, 2, lag[:, None, :].expand(T, B, T)) * causal[:, None, :]
    return {"beta": beta, "scale": scale, "weights": W}


def build_vopredictor_schedule(beta_schedule, step_size):
    """VO-PREDICTOR terms (LIFNeuronFDE.build_vopredictor_schedule, neuron.py:2063-2089):
    scale = h**beta / Gamma(beta+1); row t has weights (t-i)^(beta_t-1) - (t-i-1)^(beta_t-1)
    for i <= t-2 and 1 at i = t-1.  Built row by row with the reference's tensor shapes, so
    pow sees the same operands (its vectorised CPU path rounds by shape)."""
    beta = beta_schedule.to(dtype=torch.float32).clamp(1e-6, 1.0 - 1e-6)
    T = beta.shape[0]
    dev = beta.device
    h = torch.as_tensor(step_size, device=dev, dtype=torch.float32)
    scale = torch.pow(h, beta) / torch.exp(torch.lgamma(beta + 1.0))
    per_sample = beta.dim() == 2
    tail = (beta.shape[1],) if per_sample else ()
    rows = []
    for t in range(T):
        if t == 0:
            active = torch.zeros((0,) + tail, device=dev, dtype=torch.float32)
        elif t == 1:
            active = torch.ones_like(beta[t]).unsqueeze(0)
        else:
            lags = torch.arange(t, 1, -1, device=dev, dtype=torch.float32)
            e = beta[t] - 1.0
            if per_sample:
                lags, e = lags[:, None], e[None]
            diff = torch.pow(lags, e) - torch.pow(lags - 1.0, e)
            active = torch.cat((diff, torch.ones((1,) + tail, device=dev)), dim=0)
        row = torch.cat((active, torch.zeros((T - t,) + tail, device=dev)), dim=0)
        rows.append(row.transpose(0, 1) if per_sample else row)
    return {"beta": beta_schedule, "scale": scale, "weights": torch.stack(rows)}
