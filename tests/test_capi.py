"""The C-ABI library loads, exports every entry point of include/dfsnn_b200.h, and rejects
bad arguments with status codes before touching the GPU (CPU-only checks)."""
import ctypes
import os
import re

import pytest

from dfsnn_b200 import _capi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "dfsnn_b200.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(dfsnn_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    return _capi.lib()


def test_every_declared_symbol_is_exported(L):
    names = header_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(L, name), name
        assert name in _capi.SIGNATURES, f"{name} has no ctypes signature"


def test_status_strings(L):
    assert _capi.status_string(_capi.DFSNN_OK) == "ok"
    for code in range(1, 8):
        assert _capi.status_string(code) != "unknown status"
    assert b"sm_100a" in L.dfsnn_version()


def test_bits_words(L):
    assert L.dfsnn_spike_bits_words(16, 1000) == 1000
    assert L.dfsnn_spike_bits_words(33, 10) == 20
    assert L.dfsnn_spike_bits_words(0, 10) == 0


FAKE = ctypes.c_void_p(0x1000)   # never dereferenced: validation fails first


def test_glmulti_validation(L):
    f = L.dfsnn_glmulti_forward
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, 0, 10, 2.0, 1.0, None) == _capi.DFSNN_ERR_SHAPE
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, 4, -1, 2.0, 1.0, None) == _capi.DFSNN_ERR_SHAPE
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, 257, 10, 2.0, 1.0, None) == _capi.DFSNN_ERR_T_LIMIT
    assert f(None, FAKE, FAKE, FAKE, FAKE, 4, 10, 2.0, 1.0, None) == _capi.DFSNN_ERR_NULL
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, 4, 10, 0.0, 1.0, None) == _capi.DFSNN_ERR_PARAM
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, 4, 10, float("nan"), 1.0, None) == _capi.DFSNN_ERR_PARAM
    # N == 0 is a valid empty call: nothing to launch
    assert f(None, None, FAKE, FAKE, None, 4, 0, 2.0, 1.0, None) == _capi.DFSNN_OK
    b = L.dfsnn_glmulti_backward
    args = [FAKE] * 9 + [16, 100, 2.0, 1.0, 5.0, 1]
    assert b(*args, None, 1 << 20, None) == _capi.DFSNN_ERR_WORKSPACE
    assert b(*args, ctypes.c_void_p(0x1004), 1 << 20, None) == _capi.DFSNN_ERR_WORKSPACE
    bad_t = [FAKE] * 9 + [65, 100, 2.0, 1.0, 5.0, 1]        # full history: T <= 64
    assert b(*bad_t, FAKE, 1 << 20, None) == _capi.DFSNN_ERR_T_LIMIT
    bad_t = [FAKE] * 9 + [257, 100, 2.0, 1.0, 5.0, 0]       # truncated: T <= 256
    assert b(*bad_t, FAKE, 1 << 20, None) == _capi.DFSNN_ERR_T_LIMIT
    assert L.dfsnn_glmulti_backward_workspace_size(65, 100, 1) == 0
    assert L.dfsnn_glmulti_backward_workspace_size(65, 100, 0) > 3 * 65 * 100 * 4
    long_ws = L.dfsnn_glmulti_backward_workspace_size(64, 100, 1)
    ok_t = [FAKE] * 9 + [64, 100, 2.0, 1.0, 5.0, 1]         # too small a workspace: rejected
    assert b(*ok_t, FAKE, long_ws - 1, None) == _capi.DFSNN_ERR_WORKSPACE
    no_w = [FAKE] * 4 + [None] + [FAKE] * 4 + [16, 100, 2.0, 1.0, 5.0, 1]
    assert b(*no_w, FAKE, 1 << 20, None) == _capi.DFSNN_ERR_NULL


def test_single_validation(L):
    f = L.dfsnn_single_forward
    ok_args = [FAKE] * 6 + [16, 100, 2.0, 0.5, 1.0, 1.0, 1.0, None]
    assert f(7, *ok_args) == _capi.DFSNN_ERR_SCHEME
    assert f(-1, *ok_args) == _capi.DFSNN_ERR_SCHEME
    assert f(0, *([FAKE] * 6 + [0, 100, 2.0, 0.5, 1.0, 1.0, 1.0, None])) == _capi.DFSNN_ERR_SHAPE
    assert f(0, *([FAKE] * 5 + [None] + [16, 100, 2.0, 0.5, 1.0, 1.0, 1.0, None])) == _capi.DFSNN_ERR_NULL
    g = L.dfsnn_single_backward
    assert g(2, *([FAKE] * 7 + [16, 100, 0.0, 0.5, 1.0, 5.0, 1.0, 1.0, None])) == _capi.DFSNN_ERR_PARAM


def test_aligned_and_euler_validation(L):
    f = L.dfsnn_aligned_forward
    assert f(FAKE, FAKE, FAKE, FAKE, FAKE, 65, 10, 2.0, 1.0, None) == _capi.DFSNN_ERR_T_LIMIT
    assert L.dfsnn_aligned_backward_workspace_size(65, 10) == 0
    t = L.dfsnn_aligned_forward_typed
    assert t(FAKE, FAKE, FAKE, FAKE, FAKE, 3, 16, 10, 2.0, 1.0, None) == _capi.DFSNN_ERR_PARAM
    assert t(FAKE, FAKE, FAKE, FAKE, FAKE, _capi.DTYPE_F16, 65, 10, 2.0, 1.0, None) \
        == _capi.DFSNN_ERR_T_LIMIT
    assert t(None, FAKE, FAKE, FAKE, FAKE, _capi.DTYPE_BF16, 16, 10, 2.0, 1.0, None) \
        == _capi.DFSNN_ERR_NULL
    e = L.dfsnn_direct_euler_backward
    args = [FAKE] * 10 + [16, 100, 2.0, 1.0, 1.0, 1.0, 5.0, 1.0]
    assert e(*args, FAKE, 8, None) == _capi.DFSNN_ERR_WORKSPACE
    assert e(*([FAKE] * 9 + [None] + [16, 100, 2.0, 1.0, 1.0, 1.0, 5.0, 1.0]), FAKE, 1 << 20, None) \
        == _capi.DFSNN_ERR_NULL


def test_check_maps_to_reference_exception_types():
    with pytest.raises(ValueError):
        _capi.check(_capi.DFSNN_ERR_T_LIMIT, "x")
    with pytest.raises(ValueError):
        _capi.check(_capi.DFSNN_ERR_SHAPE, "x")
    with pytest.raises(RuntimeError):
        _capi.check(_capi.DFSNN_ERR_CUDA, "x")
    _capi.check(_capi.DFSNN_OK, "x")


def test_quotient_check_validates_before_launch():
    L = _capi.lib()
    fake = ctypes.c_void_p(16)
    assert L.dfsnn_check_surrogate_quotient(None, 1, 128, 128, fake, None) == _capi.DFSNN_ERR_NULL
    assert L.dfsnn_check_surrogate_quotient(fake, 1, 127, 128, fake, None) == _capi.DFSNN_ERR_PARAM
    assert L.dfsnn_check_surrogate_quotient(fake, 1, 128, 192, fake, None) == _capi.DFSNN_ERR_PARAM
    assert L.dfsnn_check_surrogate_quotient(fake, 0, 128, 128, fake, None) == _capi.DFSNN_ERR_PARAM


def test_schedule_validation_before_launch():
    L = _capi.lib()
    F = ctypes.c_void_p(16)
    f, b = L.dfsnn_glmulti_schedule_forward, L.dfsnn_glmulti_schedule_backward
    assert f(None, F, F, 3, 16, 1, F, F, F, None) == _capi.DFSNN_ERR_NULL
    assert f(F, F, F, 0, 16, 1, F, F, F, None) == _capi.DFSNN_ERR_SHAPE
    assert f(F, F, F, 17, 16, 1, F, F, F, None) == _capi.DFSNN_ERR_SHAPE
    assert f(F, F, F, 3, 257, 1, F, F, F, None) == _capi.DFSNN_ERR_T_LIMIT
    assert f(F, F, F, 3, 16, 2, F, F, F, None) == _capi.DFSNN_ERR_PARAM
    assert b(F, F, F, F, None, None, 3, 16, 1, None, None) == _capi.DFSNN_ERR_NULL
    assert b(F, F, F, F, None, None, 3, 0, 1, F, None) == _capi.DFSNN_ERR_SHAPE


def test_history_validation(L):
    """VO-GL1 / FAGL1 / VO-PREDICTOR entry points reject bad arguments before any launch."""
    ws = L.dfsnn_history_backward_workspace_size
    assert ws(16, 1000, 4, 0) > 0 and ws(16, 1000, 4, 1) > 0
    assert ws(0, 1000, 4, 0) == 0 and ws(257, 1000, 4, 0) == 0
    assert ws(16, 1000, 3, 0) == 0 and ws(16, 1000, 0, 0) == 0 and ws(16, 1000, 4, 2) == 0
    F = FAKE
    vf = L.dfsnn_vo_gl1_forward
    assert vf(F, F, F, F, 3, 0, F, F, F, F, 16, 1000, 2.0, 1.0, None) == _capi.DFSNN_ERR_SHAPE
    assert vf(F, F, F, F, 0, 0, F, F, F, F, 16, 1000, 2.0, 1.0, None) == _capi.DFSNN_ERR_SHAPE
    assert vf(F, F, F, F, 4, 0, F, F, F, F, 257, 1000, 2.0, 1.0, None) == _capi.DFSNN_ERR_T_LIMIT
    assert vf(F, F, None, F, 4, 0, F, F, F, F, 16, 1000, 2.0, 1.0, None) == _capi.DFSNN_ERR_NULL
    assert vf(F, F, F, F, 4, 0, F, F, F, None, 16, 1000, 2.0, 1.0, None) == _capi.DFSNN_ERR_NULL
    assert vf(F, F, F, F, 4, 2, F, F, F, F, 16, 1000, 2.0, 1.0, None) == _capi.DFSNN_ERR_PARAM
    assert vf(F, F, F, F, 4, 0, F, F, F, F, 16, 1000, 0.0, 1.0, None) == _capi.DFSNN_ERR_PARAM
    ff = L.dfsnn_fa_gl1_forward
    assert ff(F, F, F, 1, 0, F, F, F, 65, 100, 2.0, 0.25, 1.0, None) == _capi.DFSNN_ERR_T_LIMIT
    assert ff(F, F, None, 1, 0, F, F, F, 16, 100, 2.0, 0.25, 1.0, None) == _capi.DFSNN_ERR_NULL
    assert ff(F, F, F, 1, 0, F, F, F, 16, 100, 2.0, float("nan"), 1.0, None) == _capi.DFSNN_ERR_PARAM
    pf = L.dfsnn_vo_predictor_forward
    assert pf(F, F, F, F, 1, 0, F, F, F, 16, 100, 2.0, 1.0, float("inf"), None) == _capi.DFSNN_ERR_PARAM
    assert pf(F, F, F, F, 1, 0, F, F, None, 16, 100, 2.0, 1.0, 0.2, None) == _capi.DFSNN_ERR_NULL
    vb = L.dfsnn_vo_gl1_backward
    big = ws(16, 100, 1, 0)
    assert vb(F, F, F, F, F, F, 1, 0, F, F, F, F, 65, 100, 2.0, 1.0, 5.0, 1, F, big, None) == \
        _capi.DFSNN_ERR_T_LIMIT
    assert vb(F, F, F, F, F, F, 1, 0, F, F, F, F, 16, 100, 2.0, 1.0, 5.0, 2, F, big, None) == \
        _capi.DFSNN_ERR_PARAM
    assert vb(F, F, F, F, F, F, 1, 0, F, F, F, F, 16, 100, 2.0, 1.0, 5.0, 0, F, big - 8, None) == \
        _capi.DFSNN_ERR_WORKSPACE
    assert vb(F, F, F, F, None, F, 1, 0, F, F, F, F, 16, 100, 2.0, 1.0, 5.0, 0, F, big, None) == \
        _capi.DFSNN_ERR_NULL                                       # grad_weights needs v_hist
    assert vb(F, F, F, F, F, None, 1, 0, F, F, F, None, 16, 100, 2.0, 1.0, 5.0, 0, F, big, None) == \
        _capi.DFSNN_ERR_NULL                                       # grad_scale needs drift
    fb = L.dfsnn_fa_gl1_backward
    assert fb(F, F, F, F, 1, 0, F, F, F, 65, 100, 2.0, 0.25, 1.0, 5.0, 0, F, big, None) == \
        _capi.DFSNN_ERR_T_LIMIT
    pb = L.dfsnn_vo_predictor_backward
    assert pb(F, F, F, F, F, 3, 0, F, F, F, F, 16, 100, 2.0, 1.0, 5.0, 0.2, F, big, None) == \
        _capi.DFSNN_ERR_SHAPE
