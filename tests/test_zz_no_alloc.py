"""dfsnn_glmulti_backward_noalloc: the glmulti backward for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc (or any allocating routine) when the
backward runs -- e.g. code in a host callback or a runtime that owns all device memory.
The no-alloc entry point keeps its scratch in a fixed device array instead of a workspace.
This test calls it through the C ABI and checks its outputs against the regular entry point
(dfsnn_glmulti_backward) on two calls in a row: per-neuron gradients bit for bit, the
reduced grad_scale / grad_W within the suite's tolerance.  It is collected last on purpose.
"""
import numpy as np
import pytest
import torch

from dfsnn_b200 import _capi
from parity import assert_bitwise, assert_close

pytestmark = pytest.mark.gpu


def _call_regular(L, args, T, N, ws):
    code = L.dfsnn_glmulti_backward(*args[:9], T, N, 2.0, 1.0, 5.0, 1, _capi.ptr(ws), ws.numel(),
                                    None)
    assert code == 0, _capi.status_string(code)


def test_noalloc_matches_regular_twice():
    L = _capi.lib()
    dev = "cuda:0"
    torch.cuda.set_device(0)
    T, N = 16, 300_000
    g = torch.Generator(device=dev).manual_seed(123)
    W = torch.tril(torch.randn(T, T, device=dev, generator=g) * 0.05, -1)
    scale = torch.full((T,), 0.22385544, device=dev)
    outs = {}
    for name in ("regular", "noalloc"):
        outs[name] = []
        for call in range(2):
            gg = torch.Generator(device=dev).manual_seed(7 + call)
            x = torch.randn(T, N, device=dev, generator=gg) * 5
            gS = torch.randn(T, N, device=dev, generator=gg)
            v0 = torch.randn(N, device=dev, generator=gg) * 0.1
            gx = torch.empty(T, N, device=dev)
            gv0 = torch.empty(N, device=dev)
            gsc = torch.empty(T, device=dev)
            gW = torch.empty(T, T, device=dev)
            args = [_capi.ptr(t) for t in (gS, x, v0, scale, W, gx, gv0, gsc, gW)]
            if name == "regular":
                ws = torch.empty(int(L.dfsnn_glmulti_backward_workspace_size(T, N, 1)),
                                 dtype=torch.uint8, device=dev)
                _call_regular(L, args, T, N, ws)
            else:
                code = L.dfsnn_glmulti_backward_noalloc(*args, T, N, 2.0, 1.0, 5.0, 1, None)
                assert code == 0, _capi.status_string(code)
            torch.cuda.synchronize()
            outs[name].append([t.cpu().numpy() for t in (gx, gv0, gsc, gW)])
    for call in range(2):
        r, n = outs["regular"][call], outs["noalloc"][call]
        assert_bitwise(n[0], r[0], what=f"grad_x call {call}")
        assert_bitwise(n[1], r[1], what=f"grad_v0 call {call}")
        assert_close(n[2], r[2], what=f"grad_scale call {call}")
        assert_close(n[3], r[3], what=f"grad_W call {call}")
        assert np.isfinite(n[3]).all()


def test_noalloc_rejects_T_above_its_limit():
    L = _capi.lib()
    fake = _capi.ptr(torch.empty(1, device="cuda:0"))
    code = L.dfsnn_glmulti_backward_noalloc(*([fake] * 9), 17, 10, 2.0, 1.0, 5.0, 1, None)
    assert code == _capi.DFSNN_ERR_T_LIMIT
