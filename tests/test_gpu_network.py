"""The CNN128 network of the examples (bench.py --workload cnn128) trains through the native
aligned kernels: a small batch runs forward and backward, every LIF layer dispatches to the
B200 AlignedGLMulti, and the gradients (convolutions, linear layers, shared masses) are
finite."""
import importlib.util
import os
import sys

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("dfsnn_bench", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    try:
        sys.argv = ["bench.py"]
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def test_cnn128_trains_through_native_aligned_kernels():
    from dfsnn_b200 import aligned_glmulti, fde_kernels
    original = fde_kernels.LIFFDEGLMultiFunction
    b = _bench()
    b.CNN_B = 2
    dev = torch.device("cuda", 0)
    try:
        torch.manual_seed(0)
        model = b.make_cnn128(dev)
        assert fde_kernels.LIFFDEGLMultiFunction is aligned_glmulti.AlignedGLMulti
        before = dict(aligned_glmulti.CALLS)
        x = (torch.rand(b.CNN_T, 2, 2, 128, 128, device=dev) < 0.05).float() * 3.0
        y = torch.tensor([1, 7], device=dev)
        model.reset()
        loss = F.cross_entropy(model(x), y)
        loss.backward()
        torch.cuda.synchronize()
        assert aligned_glmulti.CALLS["forward"] - before["forward"] == 7
        assert aligned_glmulti.CALLS["backward"] - before["backward"] == 7
        grads = [p.grad for p in model.parameters() if p.requires_grad]
        assert all(g is not None and torch.isfinite(g).all() for g in grads)
        raw = model.layers[2].multi_coefficient_raw
        assert raw.grad is not None and torch.isfinite(raw.grad).all()
    finally:
        fde_kernels.LIFFDEGLMultiFunction = original
