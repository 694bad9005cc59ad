"""ctypes binding of the C ABI in include/dfsnn_b200.h (libdfsnn_b200.so).

The library is built in-tree by df-snn-official_b200/build.py into _lib/.  There is no
fallback: when it is missing or a call fails, the caller gets an exception.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libdfsnn_b200.so")

DFSNN_OK = 0
DFSNN_ERR_NULL = 1
DFSNN_ERR_SHAPE = 2
DFSNN_ERR_T_LIMIT = 3
DFSNN_ERR_WORKSPACE = 4
DFSNN_ERR_CUDA = 5
DFSNN_ERR_SCHEME = 6
DFSNN_ERR_PARAM = 7

MAX_T = 256
MAX_T_FULL = 64

GL, TRAP, PREDICTOR, GL1, TRAP1, PREDICTOR1, EULER_LIF = 0, 1, 2, 3, 4, 5, 6

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2

_p = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "dfsnn_status_string": (ctypes.c_char_p, [_i]),
    "dfsnn_last_cuda_error": (_i, []),
    "dfsnn_version": (ctypes.c_char_p, []),
    "dfsnn_glmulti_forward": (_i, [_p, _p, _p, _p, _p, _i, _ll, _f, _f, _p]),
    "dfsnn_glmulti_backward_workspace_size": (_sz, [_i, _ll, _i]),
    "dfsnn_glmulti_backward": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _ll, _f, _f, _f, _i,
                                    _p, _sz, _p]),
    "dfsnn_glmulti_backward_noalloc": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _ll, _f, _f,
                                            _f, _i, _p]),
    "dfsnn_aligned_forward": (_i, [_p, _p, _p, _p, _p, _i, _ll, _f, _f, _p]),
    "dfsnn_aligned_forward_typed": (_i, [_p, _p, _p, _p, _p, _i, _i, _ll, _f, _f, _p]),
    "dfsnn_aligned_backward_workspace_size": (_sz, [_i, _ll]),
    "dfsnn_aligned_backward": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _ll, _f, _f, _f, _f,
                                    _p, _sz, _p]),
    "dfsnn_spike_bits_words": (_sz, [_i, _ll]),
    "dfsnn_single_forward": (_i, [_i, _p, _p, _p, _p, _p, _p, _i, _ll, _f, _f, _f, _f, _f, _p]),
    "dfsnn_single_backward": (_i, [_i, _p, _p, _p, _p, _p, _p, _p, _i, _ll, _f, _f, _f, _f, _f,
                                   _f, _p]),
    "dfsnn_single_recompute_backward": (_i, [_i, _p, _p, _p, _p, _p, _p, _p, _i, _ll, _f, _f, _f,
                                             _f, _p]),
    "dfsnn_direct_euler_forward": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _ll, _f, _f, _f, _f, _f,
                                        _p]),
    "dfsnn_direct_euler_backward_workspace_size": (_sz, [_ll]),
    "dfsnn_direct_euler_backward": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _ll, _f, _f,
                                         _f, _f, _f, _f, _p, _sz, _p]),
    "dfsnn_check_surrogate_quotient": (_i, [_p, _i, _i, _i, _p, _p]),
    "dfsnn_glmulti_schedule_forward": (_i, [_p, _p, _p, _i, _i, _i, _p, _p, _p, _p]),
    "dfsnn_glmulti_schedule_backward": (_i, [_p, _p, _p, _p, _p, _p, _i, _i, _i, _p, _p]),
    "dfsnn_vo_gl1_forward": (_i, [_p, _p, _p, _p, _i, _i, _p, _p, _p, _p, _i, _ll, _f, _f, _p]),
    "dfsnn_fa_gl1_forward": (_i, [_p, _p, _p, _i, _i, _p, _p, _p, _i, _ll, _f, _f, _f, _p]),
    "dfsnn_vo_predictor_forward": (_i, [_p, _p, _p, _p, _i, _i, _p, _p, _p, _i, _ll, _f, _f, _f,
                                        _p]),
    "dfsnn_history_backward_workspace_size": (_sz, [_i, _ll, _i, _i]),
    "dfsnn_gl_history_step": (_i, [_i, _p, _p, _i, _i, _p, _i, _p, _i, _p, _p, _ll, _p, _i, _p]),
    "dfsnn_gl_history_step_workspace_size": (_sz, [_i, _ll]),
    "dfsnn_gl_history_step_backward": (_i, [_i, _p, _p, _p, _i, _i, _p, _i, _p, _p, _p, _p, _p,
                                            _ll, _p, _sz, _p]),
    "dfsnn_vo_gl1_backward": (_i, [_p, _p, _p, _p, _p, _p, _i, _i, _p, _p, _p, _p, _i, _ll, _f,
                                   _f, _f, _i, _p, _sz, _p]),
    "dfsnn_fa_gl1_backward": (_i, [_p, _p, _p, _p, _i, _i, _p, _p, _p, _i, _ll, _f, _f, _f, _f,
                                   _i, _p, _sz, _p]),
    "dfsnn_vo_predictor_backward": (_i, [_p, _p, _p, _p, _p, _i, _i, _p, _p, _p, _p, _i, _ll, _f,
                                         _f, _f, _f, _p, _sz, _p]),
}

_lib = None


class NativeLibraryMissing(RuntimeError):
    pass


def lib():
    """Load libdfsnn_b200.so (once); raise NativeLibraryMissing if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"{LIB_PATH} not found: build the sm_100a library with "
                "`python df-snn-official_b200/build.py` (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


_WS_CACHE = {}


def workspace_bytes(kind, device, T, N, full=0):
    """Workspace size of a backward entry point (cached: the query consults the occupancy
    API, which costs host time on every call)."""
    key = (kind, device.index, T, N, full)
    got = _WS_CACHE.get(key)
    if got is None:
        L = lib()
        if kind == "glmulti":
            got = int(L.dfsnn_glmulti_backward_workspace_size(T, N, full))
        elif kind == "aligned":
            got = int(L.dfsnn_aligned_backward_workspace_size(T, N))
        else:
            got = int(L.dfsnn_direct_euler_backward_workspace_size(N))
        _WS_CACHE[key] = got
    return got


def history_workspace_bytes(device, T, N, B, per_batch):
    """Workspace of the VO-GL1 / FAGL1 / VO-PREDICTOR backward entry points (cached)."""
    key = ("history", device.index, T, N, B, per_batch)
    got = _WS_CACHE.get(key)
    if got is None:
        got = int(lib().dfsnn_history_backward_workspace_size(T, N, B, per_batch))
        _WS_CACHE[key] = got
    return got


def status_string(code):
    return lib().dfsnn_status_string(code).decode()


def check(code, what):
    """Map a DFSNN status to the exception types the reference Functions raise."""
    if code == DFSNN_OK:
        return
    msg = f"{what}: {status_string(code)}"
    if code == DFSNN_ERR_CUDA:
        msg += f" (cudaError {lib().dfsnn_last_cuda_error()})"
        raise RuntimeError(msg)
    if code == DFSNN_ERR_WORKSPACE:
        raise RuntimeError(msg)
    raise ValueError(msg)


def ptr(t):
    """Device address of a tensor (or None for a missing optional argument)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t):
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
