"""Drop-in replacement of spikeDE_dis/direct_euler_cupy.py on B200.

DirectLIFLikeEulerCuPyFunction / lif_like_euler_cupy keep the reference signature
(direct_euler_cupy.py:139-253).  The learnable scalars stay on the device (no .cpu()
synchronisation) and their gradients are reduced without atomics.
"""
import torch

from . import _capi
from . import profiling as _prof

CUPY_AVAILABLE = True


class DirectLIFLikeEulerCuPyFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_seq_flat, z_init_flat, input_scale, spike_gain, spike_bias, tau,
                threshold, step_size, reset_strength, surrogate_scale, spike_update_dt):
        if not x_seq_flat.is_cuda or x_seq_flat.dtype != torch.float32:
            raise ValueError("CuPy direct Euler expects CUDA float32 tensors")
        x = x_seq_flat.contiguous()
        z0 = z_init_flat.contiguous()
        T, N = x.shape
        dev = x.device
        sc = input_scale.detach().reshape(1).to(device=dev, dtype=torch.float32).contiguous()
        gain = spike_gain.detach().reshape(1).to(device=dev, dtype=torch.float32).contiguous()
        bias = spike_bias.detach().reshape(1).to(device=dev, dtype=torch.float32).contiguous()
        spike = torch.empty_like(x)
        z_final = torch.empty_like(z0)
        with torch.cuda.device(dev), _prof.native_call(
                "euler_forward", 1, _prof.euler_forward_bytes(T, N), dev):
            code = _capi.lib().dfsnn_direct_euler_forward(
                _capi.ptr(x), _capi.ptr(z0), _capi.ptr(sc), _capi.ptr(gain), _capi.ptr(bias),
                _capi.ptr(spike), _capi.ptr(z_final), T, N, float(tau), float(threshold),
                float(step_size), float(reset_strength), float(spike_update_dt),
                _capi.stream_of(x))
        _capi.check(code, "DirectLIFLikeEulerCuPyFunction.forward")
        ctx.save_for_backward(x, z0, sc, gain, bias)
        ctx.params = (T, N, float(tau), float(threshold), float(step_size), float(reset_strength),
                      float(surrogate_scale), float(spike_update_dt))
        ctx.scalar_shapes = (input_scale.shape, spike_gain.shape, spike_bias.shape)
        return spike, z_final

    @staticmethod
    def backward(ctx, grad_spike, grad_z_final):
        x, z0, sc, gain, bias = ctx.saved_tensors
        T, N, tau, th, step, rs, sg, sdt = ctx.params
        gS = grad_spike.contiguous()
        gzf = None if grad_z_final is None else grad_z_final.contiguous()
        grad_x = torch.empty_like(x)
        grad_z0 = torch.empty((N,), device=x.device, dtype=x.dtype)
        g3 = torch.empty(3, device=x.device, dtype=torch.float32)
        with torch.cuda.device(x.device):
            L = _capi.lib()
            ws_bytes = _capi.workspace_bytes("euler", x.device, 0, N)
            ws = torch.empty(max(int(ws_bytes), 8), dtype=torch.uint8, device=x.device)
        with torch.cuda.device(x.device), _prof.native_call(
                "euler_backward", 2, _prof.euler_backward_bytes(T, N), x.device):
            code = L.dfsnn_direct_euler_backward(
                _capi.ptr(gS), _capi.ptr(gzf), _capi.ptr(x), _capi.ptr(z0), _capi.ptr(sc),
                _capi.ptr(gain), _capi.ptr(bias), _capi.ptr(grad_x), _capi.ptr(grad_z0),
                _capi.ptr(g3), T, N, tau, th, step, rs, sg, sdt, _capi.ptr(ws), ws.numel(),
                _capi.stream_of(x))
        _capi.check(code, "DirectLIFLikeEulerCuPyFunction.backward")
        s_scale, s_gain, s_bias = ctx.scalar_shapes
        return (grad_x, grad_z0, g3[0].reshape(s_scale), g3[1].reshape(s_gain),
                g3[2].reshape(s_bias), None, None, None, None, None, None)


def lif_like_euler_cupy(x_seq_flat, z_init_flat, input_scale, spike_gain, spike_bias, tau,
                        threshold, step_size, reset_strength, surrogate_scale, spike_update_dt):
    return DirectLIFLikeEulerCuPyFunction.apply(
        x_seq_flat, z_init_flat, input_scale, spike_gain, spike_bias, tau, threshold, step_size,
        reset_strength, surrogate_scale, spike_update_dt)
