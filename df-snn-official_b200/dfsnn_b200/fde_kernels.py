"""Drop-in replacement of spikeDE_dis/fde_cupy_kernels_all.py on B200.

Exports the autograd Functions LIFNeuronFDE imports lazily by name
(spikeDE_dis/neuron.py:1994, :2105-2123), with the reference's `.apply` signatures,
gradient arities, dtype behaviour and exceptions, backed by the sm_100a C ABI
(include/dfsnn_b200.h) instead of CuPy RawKernels.  `CUPY_AVAILABLE` is kept because
neuron.py gates on it (:1995); it is True because the native path never needs CuPy, and a
missing native library raises on first use rather than falling back to the CPU.

Every Function of the module is native: LIFFDEGLFunction, LIFFDEGL1Function,
LIFFDETRAPFunction, LIFFDEPREDICTORFunction, LIFFDETRAP1Function, LIFFDEPREDICTOR1Function,
LIFEulerFunction, LIFFDEGLMultiFunction, LIFFDEVOGL1Function, LIFFDEFAGL1Function,
LIFFDEFAGL1TorchFunction and LIFFDEVOPREDICTORFunction.
"""
import math

import torch

from . import _capi
from . import profiling as _prof

CUPY_AVAILABLE = True


def _require_cuda(x, name):
    if not x.is_cuda:
        raise RuntimeError(f"{name} requires CUDA tensors")


# ---------------------------------------------------------------------------------------
# single-order schemes (fde_cupy_kernels_all.py:644-1010)
# ---------------------------------------------------------------------------------------
def _single_forward(ctx, scheme, name, x_seq, v_init, weights, tau, beta, v_threshold,
                    surrogate_grad_scale, h_beta=1.0, gamma1=1.0):
    _require_cuda(x_seq, name)
    T, N = x_seq.shape
    x = x_seq.float().contiguous()
    v0 = v_init.float().contiguous()
    w = (torch.zeros(1, dtype=torch.float32, device=x.device) if weights is None
         else weights.float().contiguous())
    if weights is not None and w.numel() < T + 1:
        # The reference kernels read entries [0, T] of the table (a longer table built for a
        # larger neuron T is read the same way).
        raise ValueError(f"{name}: weight table needs at least T+1 = {T + 1} entries, got {w.numel()}")
    spike = torch.empty((T, N), dtype=torch.float32, device=x.device)
    v_seq = torch.empty((T, N), dtype=torch.float32, device=x.device)
    bits = torch.empty(((T + 31) // 32, N), dtype=torch.int32, device=x.device)
    beta_f = float(beta.item() if isinstance(beta, torch.Tensor) else beta)
    tau_f = float(tau.item() if isinstance(tau, torch.Tensor) else tau)
    with torch.cuda.device(x.device), _prof.native_call(
            "single_forward", 1, _prof.single_forward_bytes(T, N), x.device, steps=T):
        code = _capi.lib().dfsnn_single_forward(
            scheme, _capi.ptr(x), _capi.ptr(v0), _capi.ptr(w), _capi.ptr(spike),
            _capi.ptr(v_seq), _capi.ptr(bits), T, N, tau_f, beta_f, float(v_threshold),
            float(h_beta), float(gamma1), _capi.stream_of(x))
    _capi.check(code, name + ".forward")
    if scheme in (_capi.TRAP1, _capi.PREDICTOR1):
        ctx.save_for_backward(x, v0, w)       # their backward recomputes, as the reference's
    else:
        ctx.save_for_backward(v_seq, bits, w)
    ctx.scheme = scheme
    ctx.name = name
    ctx.consts = (tau_f, beta_f, float(v_threshold), float(surrogate_grad_scale), float(h_beta),
                  float(gamma1))
    ctx.T, ctx.N = T, N
    return spike, v_seq


def _single_recompute_backward(ctx, grad_spike_seq, grad_v_seq):
    x, v0, w = ctx.saved_tensors
    T, N = ctx.T, ctx.N
    gS = torch.zeros_like(x) if grad_spike_seq is None else grad_spike_seq.float().contiguous()
    gV = torch.zeros_like(x) if grad_v_seq is None else grad_v_seq.float().contiguous()
    grad_x = torch.empty((T, N), dtype=torch.float32, device=x.device)
    grad_v0 = torch.empty(N, dtype=torch.float32, device=x.device)
    tau, beta, th, sg, h_beta, gamma1 = ctx.consts
    with torch.cuda.device(x.device), _prof.native_call(
            "single_backward", 1, _prof.single1_backward_bytes(T, N), x.device, steps=T):
        code = _capi.lib().dfsnn_single_recompute_backward(
            ctx.scheme, _capi.ptr(gS), _capi.ptr(gV), _capi.ptr(x), _capi.ptr(v0), _capi.ptr(w),
            _capi.ptr(grad_x), _capi.ptr(grad_v0), T, N, tau, th, sg, h_beta, _capi.stream_of(x))
    _capi.check(code, ctx.name + ".backward")
    return grad_x, grad_v0


def _single_backward(ctx, grad_spike_seq, grad_v_seq):
    if ctx.scheme in (_capi.TRAP1, _capi.PREDICTOR1):
        return _single_recompute_backward(ctx, grad_spike_seq, grad_v_seq)
    v_seq, bits, w = ctx.saved_tensors
    T, N = ctx.T, ctx.N
    gS = (torch.zeros_like(v_seq) if grad_spike_seq is None
          else grad_spike_seq.float().contiguous())
    gV = (torch.zeros_like(v_seq) if grad_v_seq is None else grad_v_seq.float().contiguous())
    grad_x = torch.empty((T, N), dtype=torch.float32, device=v_seq.device)
    grad_v0 = torch.empty(N, dtype=torch.float32, device=v_seq.device)
    tau, beta, th, sg, h_beta, gamma1 = ctx.consts
    with torch.cuda.device(v_seq.device), _prof.native_call(
            "single_backward", 1, _prof.single_backward_bytes(T, N), v_seq.device, steps=T):
        code = _capi.lib().dfsnn_single_backward(
            ctx.scheme, _capi.ptr(gS), _capi.ptr(gV), _capi.ptr(v_seq), _capi.ptr(bits),
            _capi.ptr(w), _capi.ptr(grad_x), _capi.ptr(grad_v0), T, N, tau, beta, th, sg, h_beta,
            gamma1, _capi.stream_of(v_seq))
    _capi.check(code, ctx.name + ".backward")
    return grad_x, grad_v0


class LIFFDEGLFunction(torch.autograd.Function):
    """GL (fde_cupy_kernels_all.py:644-732)."""

    @staticmethod
    def forward(ctx, x_seq, v_init, c_rev, tau, beta, v_threshold, v_reset, surrogate_grad_scale):
        return _single_forward(ctx, _capi.GL, "LIFFDEGLFunction", x_seq, v_init, c_rev, tau, beta,
                               v_threshold, surrogate_grad_scale)

    @staticmethod
    def backward(ctx, grad_spike_seq, grad_v_seq):
        gx, gv = _single_backward(ctx, grad_spike_seq, grad_v_seq)
        return gx, gv, None, None, None, None, None, None


class LIFFDEGL1Function(torch.autograd.Function):
    """GL1, GL with the h^beta drift factor (fde_cupy_kernels_all.py:735-827)."""

    @staticmethod
    def forward(ctx, x_seq, v_init, c_rev, tau, beta, step_size, v_threshold, v_reset,
                surrogate_grad_scale):
        beta_value = beta if isinstance(beta, float) else beta.item()
        h_beta = math.pow(float(step_size), beta_value)
        return _single_forward(ctx, _capi.GL1, "LIFFDEGL1Function", x_seq, v_init, c_rev, tau,
                               beta, v_threshold, surrogate_grad_scale, h_beta=h_beta)

    @staticmethod
    def backward(ctx, grad_spike_seq, grad_v_seq):
        gx, gv = _single_backward(ctx, grad_spike_seq, grad_v_seq)
        return gx, gv, None, None, None, None, None, None, None


class LIFFDETRAPFunction(torch.autograd.Function):
    """L1-2 trapezoid (fde_cupy_kernels_all.py:829-916)."""

    @staticmethod
    def forward(ctx, x_seq, v_init, trap_weights, tau, beta, v_threshold, v_reset,
                surrogate_grad_scale):
        return _single_forward(ctx, _capi.TRAP, "LIFFDETRAPFunction", x_seq, v_init, trap_weights,
                               tau, beta, v_threshold, surrogate_grad_scale)

    @staticmethod
    def backward(ctx, grad_spike_seq, grad_v_seq):
        gx, gv = _single_backward(ctx, grad_spike_seq, grad_v_seq)
        return gx, gv, None, None, None, None, None, None


class LIFFDEPREDICTORFunction(torch.autograd.Function):
    """Fractional Adams predictor (fde_cupy_kernels_all.py:919-1010)."""

    @staticmethod
    def forward(ctx, x_seq, v_init, predictor_weights, tau, beta, v_threshold, v_reset,
                surrogate_grad_scale, h_beta, gamma_beta_plus_1):
        return _single_forward(ctx, _capi.PREDICTOR, "LIFFDEPREDICTORFunction", x_seq, v_init,
                               predictor_weights, tau, beta, v_threshold, surrogate_grad_scale,
                               h_beta=h_beta, gamma1=gamma_beta_plus_1)

    @staticmethod
    def backward(ctx, grad_spike_seq, grad_v_seq):
        gx, gv = _single_backward(ctx, grad_spike_seq, grad_v_seq)
        return gx, gv, None, None, None, None, None, None, None, None


# ---------------------------------------------------------------------------------------
# library glmulti (fde_cupy_kernels_all.py:1916-2011)
# ---------------------------------------------------------------------------------------
class LIFFDEGLMultiFunction(torch.autograd.Function):
    """Fused multi-term GL with gradients for the aggregated kernel.

    apply(x_seq[T,N], v_init[N], scale[T], weights[T,T], tau, threshold,
          surrogate_grad_scale, batch_size, full_history_grad=False) -> spikes[T,N]
    Backward returns (grad_x, grad_v_init, grad_scale[T], grad_weights[T,T], None x 5).
    """

    @staticmethod
    def forward(ctx, x_seq, v_init, scale, weights, tau, threshold, surrogate_grad_scale,
                batch_size, full_history_grad=False):
        if not x_seq.is_cuda:
            raise RuntimeError("LIFFDEGLMultiFunction requires CUDA tensors")
        original_dtype = x_seq.dtype
        x_f32, v_f32 = x_seq.float().contiguous(), v_init.float().contiguous()
        scale_f32, weights_f32 = scale.float().contiguous(), weights.float().contiguous()
        T, N = x_f32.shape
        if full_history_grad and T > 64:
            raise ValueError("Full glmulti history gradients currently support T <= 64")
        if scale_f32.shape != (T,) or weights_f32.shape != (T, T):
            raise ValueError("glmulti scale/weights must have shapes [T] and [T,T]")
        spike = torch.empty_like(x_f32)
        with torch.cuda.device(x_f32.device), _prof.native_call(
                "glmulti_forward", 1, _prof.glmulti_forward_bytes(T, N), x_f32.device, steps=T):
            code = _capi.lib().dfsnn_glmulti_forward(
                _capi.ptr(x_f32), _capi.ptr(v_f32), _capi.ptr(scale_f32), _capi.ptr(weights_f32),
                _capi.ptr(spike), T, N, float(tau), float(threshold), _capi.stream_of(x_f32))
        _capi.check(code, "LIFFDEGLMultiFunction.forward")
        ctx.save_for_backward(x_f32, v_f32, scale_f32, weights_f32)
        ctx.tau = float(tau)
        ctx.threshold = float(threshold)
        ctx.surrogate_grad_scale = float(surrogate_grad_scale)
        ctx.original_dtype = original_dtype
        ctx.full_history_grad = bool(full_history_grad)
        return spike.to(dtype=original_dtype)

    @staticmethod
    def backward(ctx, grad_spike_seq):
        x, v0, scale, weights = ctx.saved_tensors
        T, N = x.shape
        g = grad_spike_seq.float().contiguous()
        grad_x = torch.empty((T, N), device=x.device, dtype=torch.float32)
        grad_v = torch.empty(N, device=x.device, dtype=torch.float32)
        grad_scale = torch.empty(T, device=x.device, dtype=torch.float32) if ctx.needs_input_grad[2] else None
        grad_weights = torch.empty((T, T), device=x.device, dtype=torch.float32) if ctx.needs_input_grad[3] else None
        full = int(ctx.full_history_grad)
        launches = 2 if (grad_scale is not None or grad_weights is not None) else 1
        with torch.cuda.device(x.device):
            L = _capi.lib()
            ws_bytes = _capi.workspace_bytes("glmulti", x.device, T, N, full)
            ws = torch.empty(max(int(ws_bytes), 8), dtype=torch.uint8, device=x.device)
        with torch.cuda.device(x.device), _prof.native_call(
                "glmulti_backward", launches, _prof.glmulti_backward_bytes(T, N), x.device, steps=T):
            code = L.dfsnn_glmulti_backward(
                _capi.ptr(g), _capi.ptr(x), _capi.ptr(v0), _capi.ptr(scale), _capi.ptr(weights),
                _capi.ptr(grad_x), _capi.ptr(grad_v), _capi.ptr(grad_scale),
                _capi.ptr(grad_weights), T, N, ctx.tau, ctx.threshold, ctx.surrogate_grad_scale,
                full, _capi.ptr(ws), ws.numel(), _capi.stream_of(x))
        _capi.check(code, "LIFFDEGLMultiFunction.backward")
        return (grad_x.to(dtype=ctx.original_dtype), grad_v, grad_scale, grad_weights,
                None, None, None, None, None)


class LIFFDETRAP1Function(torch.autograd.Function):
    """TRAP1 (fde_cupy_kernels_all.py:2163-2276): v + h_beta*dv - hist with h_beta = 1**beta."""

    @staticmethod
    def forward(ctx, x_seq, v_init, trap_weights, tau, beta, v_threshold, v_reset,
                surrogate_grad_scale):
        beta_value = beta if isinstance(beta, float) else float(beta.item() if isinstance(
            beta, torch.Tensor) else beta)
        h_beta = math.pow(1.0, beta_value)                     # as the reference (:2190)
        return _single_forward(ctx, _capi.TRAP1, "LIFFDETRAP1Function", x_seq, v_init,
                               trap_weights, tau, beta, v_threshold, surrogate_grad_scale,
                               h_beta=h_beta)

    @staticmethod
    def backward(ctx, grad_spike_seq, grad_v_seq):
        gx, gv = _single_backward(ctx, grad_spike_seq, grad_v_seq)
        return gx, gv, None, None, None, None, None, None


class LIFFDEPREDICTOR1Function(torch.autograd.Function):
    """PREDICTOR1 (fde_cupy_kernels_all.py:2434-2545): v + h_beta*(w_T*dv + hist)."""

    @staticmethod
    def forward(ctx, x_seq, v_init, predictor_weights, tau, beta, v_threshold, v_reset,
                surrogate_grad_scale, h_beta, gamma_beta_plus_1):
        return _single_forward(ctx, _capi.PREDICTOR1, "LIFFDEPREDICTOR1Function", x_seq, v_init,
                               predictor_weights, tau, beta, v_threshold, surrogate_grad_scale,
                               h_beta=h_beta, gamma1=gamma_beta_plus_1)

    @staticmethod
    def backward(ctx, grad_spike_seq, grad_v_seq):
        gx, gv = _single_backward(ctx, grad_spike_seq, grad_v_seq)
        return gx, gv, None, None, None, None, None, None, None, None


class LIFEulerFunction(torch.autograd.Function):
    """Plain LIF, explicit Euler, no history (fde_cupy_kernels_all.py:2657-2756)."""

    @staticmethod
    def forward(ctx, x_seq, v_init, tau, v_threshold, v_reset, surrogate_grad_scale):
        return _single_forward(ctx, _capi.EULER_LIF, "LIFEulerFunction", x_seq, v_init, None, tau,
                               0.0, v_threshold, surrogate_grad_scale)

    @staticmethod
    def backward(ctx, grad_spike_seq, grad_v_seq):
        gx, gv = _single_backward(ctx, grad_spike_seq, grad_v_seq)
        return gx, gv, None, None, None, None


# ---------------------------------------------------------------------------------------
# history-table Functions with shared or per-sample parameters
# (fde_cupy_kernels_all.py:1098-1198, :1379-1587, :1751-1843)
# ---------------------------------------------------------------------------------------
def _hist_inputs(name, x_seq, v_init, scale, weights, batch_size, per_batch):
    """The reference's .float().contiguous() casts plus the shape checks the native kernels
    need (the reference reads out of bounds on a mismatch; here it is a ValueError)."""
    if not x_seq.is_cuda:
        raise RuntimeError(f"{name} requires CUDA tensors")
    x = x_seq.float().contiguous()
    v = v_init.float().contiguous()
    s = None if scale is None else scale.float().contiguous()
    w = weights.float().contiguous()
    T, N = x.shape
    B = int(batch_size)
    if B < 1 or N % B:
        raise ValueError(f"Flattened neuron count {N} is not divisible by batch size {B}")
    if v.shape != (N,):
        raise ValueError(f"{name}: v_init must have shape ({N},), got {tuple(v.shape)}")
    expected_w = (T, B, T) if per_batch else (T, T)
    if tuple(w.shape) != expected_w:
        raise ValueError(f"{name}: weights must have shape {expected_w}, got {tuple(w.shape)}")
    if s is not None and tuple(s.shape) != ((T, B) if per_batch else (T,)):
        raise ValueError(f"{name}: scale must have shape {(T, B) if per_batch else (T,)}, "
                         f"got {tuple(s.shape)}")
    return x, v, s, w, T, N, B


def _hist_save(ctx, x, tau, threshold, surrogate_grad_scale, original_dtype, B, per_batch,
               full=False, h_beta=1.0, residual_mix=0.0):
    ctx.input_shape = x.shape
    ctx.tau = float(tau)
    ctx.threshold = float(threshold)
    ctx.surrogate_grad_scale = float(surrogate_grad_scale)
    ctx.original_dtype = original_dtype
    ctx.batch_size = B
    ctx.per_batch = int(per_batch)
    ctx.full_history_grad = bool(full)
    ctx.h_beta = float(h_beta)
    ctx.residual_mix = float(residual_mix)


def _hist_launches(T, params):
    """Kernels one history-table backward launches: the sweep, and with parameter gradients
    the row reduction (fused into the sweep for T = 8 and 16), the row sums and the epilogue."""
    if not params:
        return 1
    return 3 if T in (8, 16) else 4


def _hist_workspace(ctx, device):
    T, N = ctx.input_shape
    nbytes = _capi.history_workspace_bytes(device, T, N, ctx.batch_size, ctx.per_batch)
    return torch.empty(max(nbytes, 8), dtype=torch.uint8, device=device)


class LIFFDEVOGL1Function(torch.autograd.Function):
    """Variable-order GL1 with a shared or per-sample schedule (fde_cupy_kernels_all.py:
    1751-1840).

    apply(x_seq[T,N], v_init[N], scale[T] or [T,B], weights[T,T] or [T,B,T], tau, threshold,
          surrogate_grad_scale, batch_size, full_history_grad=False) -> spikes[T,N]
    p_t = s_t*(x_t - v)/tau - sum_{i<t} W[t,i] v_i.  Backward returns (grad_x, grad_v_init,
    grad_scale, grad_weights, None x 5); grad_weights is the full matrix -grad_pre @ v_hist^T
    per sample (per-sample tables) or over all neurons.
    """

    @staticmethod
    def forward(ctx, x_seq, v_init, scale, weights, tau, threshold, surrogate_grad_scale,
                batch_size, full_history_grad=False):
        name = "LIFFDEVOGL1Function"
        original_dtype = x_seq.dtype
        per_batch = int(scale.dim() == 2)
        x, v, s, w, T, N, B = _hist_inputs(name, x_seq, v_init, scale, weights, batch_size,
                                           per_batch)
        spike, v_pre, v_hist, drift = (torch.empty_like(x) for _ in range(4))
        with torch.cuda.device(x.device), _prof.native_call(
                "vo_gl1_forward", 1, _prof.history_forward_bytes(T, N, 4), x.device):
            code = _capi.lib().dfsnn_vo_gl1_forward(
                _capi.ptr(x), _capi.ptr(v), _capi.ptr(s), _capi.ptr(w), B, per_batch,
                _capi.ptr(spike), _capi.ptr(v_pre), _capi.ptr(v_hist), _capi.ptr(drift), T, N,
                float(tau), float(threshold), _capi.stream_of(x))
        _capi.check(code, f"{name}.forward")
        ctx.save_for_backward(s, w, v_pre, v_hist, drift)
        _hist_save(ctx, x, tau, threshold, surrogate_grad_scale, original_dtype, B, per_batch,
                   full_history_grad)
        return spike.to(dtype=original_dtype)

    @staticmethod
    def backward(ctx, grad_spike_seq):
        s, w, v_pre, v_hist, drift = ctx.saved_tensors
        T, N = ctx.input_shape
        dev = v_pre.device
        g = grad_spike_seq.float().contiguous()
        grad_x = torch.empty((T, N), device=dev, dtype=torch.float32)
        grad_v = torch.empty(N, device=dev, dtype=torch.float32)
        grad_scale = torch.empty_like(s) if ctx.needs_input_grad[2] else None
        grad_weights = torch.empty_like(w) if ctx.needs_input_grad[3] else None
        nparam = (2 if grad_weights is not None else 0) + (1 if grad_scale is not None else 0)
        with torch.cuda.device(dev):
            ws = _hist_workspace(ctx, dev)
            with _prof.native_call("vo_gl1_backward", _hist_launches(T, nparam),
                                   _prof.history_backward_bytes(T, N, min(nparam, 2)), dev):
                code = _capi.lib().dfsnn_vo_gl1_backward(
                    _capi.ptr(g), _capi.ptr(s), _capi.ptr(w), _capi.ptr(v_pre), _capi.ptr(v_hist),
                    _capi.ptr(drift), ctx.batch_size, ctx.per_batch, _capi.ptr(grad_x),
                    _capi.ptr(grad_v), _capi.ptr(grad_scale), _capi.ptr(grad_weights), T, N,
                    ctx.tau, ctx.threshold, ctx.surrogate_grad_scale, int(ctx.full_history_grad),
                    _capi.ptr(ws), ws.numel(), _capi.stream_of(v_pre))
        _capi.check(code, "LIFFDEVOGL1Function.backward")
        return (grad_x.to(dtype=ctx.original_dtype), grad_v, grad_scale, grad_weights,
                None, None, None, None, None)


def _fagl1_forward(ctx, name, x_seq, v_init, weights, tau, h_beta, threshold,
                   surrogate_grad_scale, batch_size, full_history_grad, torch_variant=False):
    original_dtype = x_seq.dtype
    if not x_seq.is_cuda:
        raise RuntimeError(f"{name} requires CUDA tensors")
    T = x_seq.shape[0]
    if T > 64 and not torch_variant:
        raise ValueError("FAGL1 CuPy kernel currently supports at most 64 time steps")
    per_batch = int(weights.dim() == 3)
    x, v, _, w, T, N, B = _hist_inputs(name, x_seq, v_init, None, weights, batch_size, per_batch)
    spike, v_pre, v_hist = (torch.empty_like(x) for _ in range(3))
    L = _capi.lib()
    with torch.cuda.device(x.device), _prof.native_call(
            "fa_gl1_forward", 1, _prof.history_forward_bytes(T, N, 4 if torch_variant else 3),
            x.device):
        if torch_variant:
            # same recurrence through the VO-GL1 entry point with s_t = h_beta (no T <= 64 cap)
            s = torch.full((T, B) if per_batch else (T,), float(h_beta), device=x.device,
                           dtype=torch.float32)
            drift = torch.empty_like(x)
            code = L.dfsnn_vo_gl1_forward(
                _capi.ptr(x), _capi.ptr(v), _capi.ptr(s), _capi.ptr(w), B, per_batch,
                _capi.ptr(spike), _capi.ptr(v_pre), _capi.ptr(v_hist), _capi.ptr(drift), T, N,
                float(tau), float(threshold), _capi.stream_of(x))
        else:
            code = L.dfsnn_fa_gl1_forward(
                _capi.ptr(x), _capi.ptr(v), _capi.ptr(w), B, per_batch, _capi.ptr(spike),
                _capi.ptr(v_pre), _capi.ptr(v_hist), T, N, float(tau), float(h_beta),
                float(threshold), _capi.stream_of(x))
    _capi.check(code, f"{name}.forward")
    ctx.save_for_backward(w, v_pre, v_hist)
    _hist_save(ctx, x, tau, threshold, surrogate_grad_scale, original_dtype, B, per_batch,
               full_history_grad, h_beta=h_beta)
    return spike.to(dtype=original_dtype)


class LIFFDEFAGL1Function(torch.autograd.Function):
    """Fixed-order GL1 with per-sample causal attention rows (fde_cupy_kernels_all.py:
    1379-1498).

    apply(x_seq[T,N], v_init[N], weights[T,T] or [T,B,T], tau, h_beta, threshold,
          surrogate_grad_scale, batch_size, full_history_grad=False) -> spikes[T,N]
    T <= 64.  Backward returns (grad_x, grad_v_init, grad_weights, None x 6): per sample,
    -grad_pre @ v_hist^T on the strict lower triangle (zeros elsewhere); shared, the full matrix
    (the reference's TF32 matmul; here fp32 products summed in double).
    """

    @staticmethod
    def forward(ctx, x_seq, v_init, weights, tau, h_beta, threshold, surrogate_grad_scale,
                batch_size, full_history_grad=False):
        return _fagl1_forward(ctx, "LIFFDEFAGL1Function", x_seq, v_init, weights, tau, h_beta,
                              threshold, surrogate_grad_scale, batch_size, full_history_grad)

    @staticmethod
    def backward(ctx, grad_spike_seq):
        w, v_pre, v_hist = ctx.saved_tensors
        T, N = ctx.input_shape
        dev = v_pre.device
        g = grad_spike_seq.float().contiguous()
        grad_x = torch.empty((T, N), device=dev, dtype=torch.float32)
        grad_v = torch.empty(N, device=dev, dtype=torch.float32)
        grad_weights = torch.empty_like(w) if ctx.needs_input_grad[2] else None
        with torch.cuda.device(dev):
            ws = _hist_workspace(ctx, dev)
            with _prof.native_call("fa_gl1_backward", _hist_launches(T, grad_weights is not None),
                                   _prof.history_backward_bytes(
                                       T, N, 1 if grad_weights is not None else 0), dev):
                code = _capi.lib().dfsnn_fa_gl1_backward(
                    _capi.ptr(g), _capi.ptr(w), _capi.ptr(v_pre), _capi.ptr(v_hist),
                    ctx.batch_size, ctx.per_batch, _capi.ptr(grad_x), _capi.ptr(grad_v),
                    _capi.ptr(grad_weights), T, N, ctx.tau, ctx.h_beta, ctx.threshold,
                    ctx.surrogate_grad_scale, int(ctx.full_history_grad), _capi.ptr(ws),
                    ws.numel(), _capi.stream_of(v_pre))
        _capi.check(code, "LIFFDEFAGL1Function.backward")
        return (grad_x.to(dtype=ctx.original_dtype), grad_v, grad_weights,
                None, None, None, None, None, None)


class LIFFDEFAGL1TorchFunction(torch.autograd.Function):
    """The reference's PyTorch formulation of FAGL1 (fde_cupy_kernels_all.py:1501-1587) with
    its own gradient contract: the weight gradient is -grad_pre @ v_hist^T over every entry,
    per sample or shared.  Computed by the native VO-GL1 kernels with s_t = h_beta (the same
    recurrence), so it agrees with the PyTorch op sequence within fp32 rounding rather than bit
    for bit; it needs CUDA tensors, T <= 256, and T <= 64 with full_history_grad.
    """

    @staticmethod
    def forward(ctx, x_seq, v_init, weights, tau, h_beta, threshold, surrogate_grad_scale,
                batch_size, full_history_grad=False):
        return _fagl1_forward(ctx, "LIFFDEFAGL1TorchFunction", x_seq, v_init, weights, tau,
                              h_beta, threshold, surrogate_grad_scale, batch_size,
                              full_history_grad, torch_variant=True)

    @staticmethod
    def backward(ctx, grad_spike_seq):
        w, v_pre, v_hist = ctx.saved_tensors
        T, N = ctx.input_shape
        dev = v_pre.device
        g = grad_spike_seq.float().contiguous()
        grad_x = torch.empty((T, N), device=dev, dtype=torch.float32)
        grad_v = torch.empty(N, device=dev, dtype=torch.float32)
        grad_weights = torch.empty_like(w) if ctx.needs_input_grad[2] else None
        s = torch.full((T, ctx.batch_size) if ctx.per_batch else (T,), ctx.h_beta,
                       device=dev, dtype=torch.float32)
        with torch.cuda.device(dev):
            ws = _hist_workspace(ctx, dev)
            with _prof.native_call("fa_gl1_backward", _hist_launches(T, grad_weights is not None),
                                   _prof.history_backward_bytes(
                                       T, N, 1 if grad_weights is not None else 0), dev):
                code = _capi.lib().dfsnn_vo_gl1_backward(
                    _capi.ptr(g), _capi.ptr(s), _capi.ptr(w), _capi.ptr(v_pre), _capi.ptr(v_hist),
                    None, ctx.batch_size, ctx.per_batch, _capi.ptr(grad_x), _capi.ptr(grad_v),
                    None, _capi.ptr(grad_weights), T, N, ctx.tau, ctx.threshold,
                    ctx.surrogate_grad_scale, int(ctx.full_history_grad), _capi.ptr(ws),
                    ws.numel(), _capi.stream_of(v_pre))
        _capi.check(code, "LIFFDEFAGL1TorchFunction.backward")
        return (grad_x.to(dtype=ctx.original_dtype), grad_v, grad_weights,
                None, None, None, None, None, None)


class LIFFDEVOPREDICTORFunction(torch.autograd.Function):
    """Variable-order predictor with a shared or per-sample schedule (fde_cupy_kernels_all.py:
    1098-1191).

    apply(x_seq[T,N], v_init[N], scale[T] or [T,B], weights[T,T] or [T,B,T], tau, threshold,
          surrogate_grad_scale, residual_mix, batch_size) -> spikes[T,N]
    p_t = v0 + s_t*(d_t + sum_{i<t} W[t,i] d_i) + residual_mix*(v - v0).  Backward returns
    (grad_x, grad_v_init, grad_scale, grad_weights, None x 5) with grad_scale = sum
    grad_pre*(drift + W @ drift) and grad_weights = (grad_pre*scale) @ drift^T.
    """

    @staticmethod
    def forward(ctx, x_seq, v_init, scale, weights, tau, threshold, surrogate_grad_scale,
                residual_mix, batch_size):
        name = "LIFFDEVOPREDICTORFunction"
        original_dtype = x_seq.dtype
        per_batch = int(scale.dim() == 2)
        x, v, s, w, T, N, B = _hist_inputs(name, x_seq, v_init, scale, weights, batch_size,
                                           per_batch)
        spike, v_pre, drift = (torch.empty_like(x) for _ in range(3))
        with torch.cuda.device(x.device), _prof.native_call(
                "vo_predictor_forward", 1, _prof.history_forward_bytes(T, N, 3), x.device):
            code = _capi.lib().dfsnn_vo_predictor_forward(
                _capi.ptr(x), _capi.ptr(v), _capi.ptr(s), _capi.ptr(w), B, per_batch,
                _capi.ptr(spike), _capi.ptr(v_pre), _capi.ptr(drift), T, N, float(tau),
                float(threshold), float(residual_mix), _capi.stream_of(x))
        _capi.check(code, f"{name}.forward")
        ctx.save_for_backward(s, w, v_pre, drift)
        _hist_save(ctx, x, tau, threshold, surrogate_grad_scale, original_dtype, B, per_batch,
                   residual_mix=residual_mix)
        return spike.to(dtype=original_dtype)

    @staticmethod
    def backward(ctx, grad_spike_seq):
        s, w, v_pre, drift = ctx.saved_tensors
        T, N = ctx.input_shape
        dev = v_pre.device
        g = grad_spike_seq.float().contiguous()
        grad_x = torch.empty((T, N), device=dev, dtype=torch.float32)
        grad_v = torch.empty(N, device=dev, dtype=torch.float32)
        grad_scale = torch.empty_like(s) if ctx.needs_input_grad[2] else None
        grad_weights = torch.empty_like(w) if ctx.needs_input_grad[3] else None
        params = grad_scale is not None or grad_weights is not None
        with torch.cuda.device(dev):
            ws = _hist_workspace(ctx, dev)
            with _prof.native_call("vo_predictor_backward", _hist_launches(T, params),
                                   _prof.history_backward_bytes(T, N, 1 if params else 0), dev):
                code = _capi.lib().dfsnn_vo_predictor_backward(
                    _capi.ptr(g), _capi.ptr(s), _capi.ptr(w), _capi.ptr(v_pre), _capi.ptr(drift),
                    ctx.batch_size, ctx.per_batch, _capi.ptr(grad_x), _capi.ptr(grad_v),
                    _capi.ptr(grad_scale), _capi.ptr(grad_weights), T, N, ctx.tau,
                    ctx.threshold, ctx.surrogate_grad_scale, ctx.residual_mix, _capi.ptr(ws),
                    ws.numel(), _capi.stream_of(v_pre))
        _capi.check(code, "LIFFDEVOPREDICTORFunction.backward")
        return (grad_x.to(dtype=ctx.original_dtype), grad_v, grad_scale, grad_weights,
                None, None, None, None, None)
