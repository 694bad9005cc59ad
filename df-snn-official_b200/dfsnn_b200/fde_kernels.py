"""Drop-in replacement of spikeDE_dis/fde_cupy_kernels_all.py on B200.

Exports the autograd Functions LIFNeuronFDE imports lazily by name
(spikeDE_dis/neuron.py:1994, :2105-2123), with the reference's `.apply` signatures,
gradient arities, dtype behaviour and exceptions, backed by the sm_100a C ABI
(include/dfsnn_b200.h) instead of CuPy RawKernels.  `CUPY_AVAILABLE` is kept because
neuron.py gates on it (:1995); it is True because the native path never needs CuPy, and a
missing native library raises on first use rather than falling back to the CPU.

Native here: LIFFDEGLFunction, LIFFDEGL1Function, LIFFDETRAPFunction,
LIFFDEPREDICTORFunction, LIFFDETRAP1Function, LIFFDEPREDICTOR1Function, LIFEulerFunction,
LIFFDEGLMultiFunction.  The remaining reference Functions of the
module are outside this hot path and raise NotImplementedError.
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
            "single_forward", 1, _prof.single_forward_bytes(T, N), x.device):
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
            "single_backward", 1, _prof.single1_backward_bytes(T, N), x.device):
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
            "single_backward", 1, _prof.single_backward_bytes(T, N), v_seq.device):
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
                "glmulti_forward", 1, _prof.glmulti_forward_bytes(T, N), x_f32.device):
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
                "glmulti_backward", launches, _prof.glmulti_backward_bytes(T, N), x.device):
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
# reference Functions outside this hot path
# ---------------------------------------------------------------------------------------
def _not_native(name):
    def apply(*args, **kwargs):
        raise NotImplementedError(
            f"{name} is not part of the B200 LIF-FDE hot path (native: GL, GL1, TRAP, "
            "PREDICTOR, TRAP1, PREDICTOR1, LIF Euler, GLMULTI, aligned GLMULTI, direct Euler)")

    return type(name, (), {"apply": staticmethod(apply)})


LIFFDEVOPREDICTORFunction = _not_native("LIFFDEVOPREDICTORFunction")
LIFFDEFAGL1Function = _not_native("LIFFDEFAGL1Function")
LIFFDEFAGL1TorchFunction = _not_native("LIFFDEFAGL1TorchFunction")
LIFFDEVOGL1Function = _not_native("LIFFDEVOGL1Function")
