"""The surrogate quotient of the backward kernels (Markstein's FMA-corrected division)
against CUDA's IEEE division, over every denominator the kernels divide by without the
IEEE fallback (all mantissas of the binades [2, 2^64])."""
import ctypes

import numpy as np
import pytest
import torch

from dfsnn_b200 import _capi

pytestmark = pytest.mark.gpu


def _run(a, lo, hi):
    L = _capi.lib()
    dev = torch.device("cuda", 0)
    at = torch.from_numpy(np.array(a, np.float32)).to(dev)
    out = torch.zeros(2, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        rc = L.dfsnn_check_surrogate_quotient(ctypes.c_void_p(at.data_ptr()), len(a), lo, hi,
                                              ctypes.c_void_p(out.data_ptr()),
                                              _capi.stream_of(at))
    _capi.check(rc, "dfsnn_check_surrogate_quotient")
    torch.cuda.synchronize()
    return [int(v) for v in out.cpu()]


def test_quotient_all_binades_typical_scales():
    rng = np.random.default_rng(7)
    fixed = [1.0, 2.0, 2.5, 3.0, 4.0, 5.0, 10.0, 0.5, 0.3, np.pi, 1.2345678, 7.0, 100.0, 1e-3,
             2.0 ** -60, 2.0 ** 60]
    rand = (1.0 + rng.random(112)).astype(np.float32)      # every mantissa pattern region
    q, r = _run(np.concatenate([fixed, rand]), 128, 191)
    assert r == 0, f"refined reciprocal not correctly rounded for {r} mantissas"
    assert q == 0, f"{q} quotients differ from __fdiv_rn"


def test_quotient_one_binade_many_numerators():
    rng = np.random.default_rng(11)
    a = np.frombuffer((0x3F800000 | rng.integers(0, 1 << 23, 4096, dtype=np.uint32))
                      .astype(np.uint32).tobytes(), np.float32)
    q, r = _run(a, 128, 128)
    assert (q, r) == (0, 0)
