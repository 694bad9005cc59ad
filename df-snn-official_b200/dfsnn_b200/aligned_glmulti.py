"""Drop-in replacement of examples/*/aligned_glmulti.py's AlignedGLMulti on B200.

Same module surface the example networks use: AlignedGLMulti (the autograd Function),
install(backend) (rebinds the library glmulti Function the way the reference does,
examples/cnn128/aligned_glmulti.py:157-162), HISTORY_RHO and the CALLS counters.  The
CUDA work is the sm_100a C ABI (dfsnn_aligned_forward / dfsnn_aligned_backward).
"""
import torch

from . import _capi
from . import profiling as _prof

BACKEND = "native"
_HALF = {torch.float16: _capi.DTYPE_F16, torch.bfloat16: _capi.DTYPE_BF16}
CALLS = {"forward": 0, "backward": 0}
HISTORY_RHO = 1.0


def _rho_f32():
    # The reference substitutes f"{HISTORY_RHO:.8f}f" into the kernel source (:90).
    return float(f"{HISTORY_RHO:.8f}")


class AlignedGLMulti(torch.autograd.Function):
    """apply(x[T,N], v[N], a[T], w[T,T], tau, th, sg, batch, full=False) -> spikes[T,N].

    Backward returns (grad_x, grad_v, grad_a[T], grad_w[T,T] (strictly lower), None x 5).
    """

    @staticmethod
    def forward(ctx, x, v, a, w, tau, th, sg, batch, full=False):
        if not full or not 0 < x.shape[0] <= 64:
            raise ValueError("Requires full history and 1<=T<=64")
        if not x.is_cuda:
            raise RuntimeError("AlignedGLMulti requires CUDA tensors")
        CALLS["forward"] += 1
        ctx.dtype = x.dtype
        ctx.constants = (float(tau), float(th), float(sg))
        v, a, w = [z.float().contiguous() for z in (v, a, w)]
        io = _HALF.get(x.dtype)
        if io is not None:
            # half-precision activations (autocast): read and written in their own type by
            # the kernel -- the reference's .float() / .to(dtype) casts give the same values
            x = x.contiguous()
            elem = 2
        else:
            x = x.float().contiguous()
            io, elem = _capi.DTYPE_F32, 4
        T, N = x.shape
        s = torch.empty_like(x)
        with torch.cuda.device(x.device), _prof.native_call(
                "aligned_forward", 1, _prof.glmulti_forward_bytes(T, N, elem), x.device, steps=T):
            code = _capi.lib().dfsnn_aligned_forward_typed(
                _capi.ptr(x), _capi.ptr(v), _capi.ptr(a), _capi.ptr(w), _capi.ptr(s), io, T, N,
                float(tau), float(th), _capi.stream_of(x))
        _capi.check(code, "AlignedGLMulti.forward")
        ctx.save_for_backward(x, v, a, w)
        return s

    @staticmethod
    def backward(ctx, g):
        CALLS["backward"] += 1
        x, v, a, w = ctx.saved_tensors
        x = x.float().contiguous()
        g = g.float().contiguous()
        T, N = g.shape
        tau, th, sg = ctx.constants
        gx = torch.empty_like(g)
        gv = torch.empty(N, device=g.device, dtype=torch.float32)
        gs = torch.empty(T, device=g.device, dtype=torch.float32) if ctx.needs_input_grad[2] else None
        gw = torch.empty((T, T), device=g.device, dtype=torch.float32) if ctx.needs_input_grad[3] else None
        launches = 2 if (gs is not None or gw is not None) else 1
        with torch.cuda.device(g.device):
            L = _capi.lib()
            ws_bytes = _capi.workspace_bytes("aligned", g.device, T, N)
            ws = torch.empty(max(int(ws_bytes), 8), dtype=torch.uint8, device=g.device)
        with torch.cuda.device(g.device), _prof.native_call(
                "aligned_backward", launches, _prof.glmulti_backward_bytes(T, N), g.device, steps=T):
            code = L.dfsnn_aligned_backward(
                _capi.ptr(g), _capi.ptr(x), _capi.ptr(v), _capi.ptr(a), _capi.ptr(w),
                _capi.ptr(gx), _capi.ptr(gv), _capi.ptr(gs), _capi.ptr(gw), T, N, tau, th, sg,
                _rho_f32(), _capi.ptr(ws), ws.numel(), _capi.stream_of(g))
        _capi.check(code, "AlignedGLMulti.backward")
        return gx.to(ctx.dtype), gv, gs, gw, None, None, None, None, None


def install(backend="native", kernels_module=None):
    """Make the library glmulti Function resolve to AlignedGLMulti (as the reference's
    install() does for spikeDE_dis.fde_cupy_kernels_all).  `backend` is accepted for
    signature compatibility ('cupy' and 'native' both mean the B200 kernels here)."""
    global BACKEND
    BACKEND = backend
    if kernels_module is None:
        from . import fde_kernels as kernels_module
    kernels_module.LIFFDEGLMultiFunction = AlignedGLMulti
