"""A stand-in for the few CuPy calls that the reference's LIF kernels make, so that the
reference's own Python code runs its own CUDA kernels on a GPU without CuPy
(TEST AND BASELINE INFRASTRUCTURE ONLY: the GPU reference arm and the GPU-to-GPU parity
tests put oracle/cupy_standin on sys.path; nothing of the library imports it).

Covered: RawKernel(code, name, options) and its launch (grid, block, args, shared_mem,
stream), from_dlpack of torch tensors, the scalar types (int32, float32, ...), and
cuda.Device / cuda.ExternalStream / cuda.get_current_stream.  Everything else the real
CuPy offers (asarray, empty, array arithmetic) raises NotImplementedError.  Unlike CuPy, a
launch whose arguments do not match the kernel's declared parameters (count and byte sizes,
recorded in the manifest) is refused with TypeError before it reaches the GPU.

CuPy compiles a RawKernel's source with NVRTC when it is first launched.  Here the same
source texts, with the same options, are compiled ahead of time by oracle/build_ref.py
with nvcc into cubins for sm_100 (oracle/_ref/cuda/, keyed by a hash of source and
options); RawKernel looks its source up by that key and refuses any source that was not
prebuilt, so a launch always runs exactly the text the reference handed over.  Modules
are loaded and launched through the CUDA driver API (cuModuleLoadData,
cuModuleGetFunction, cuLaunchKernel), as CuPy does.
"""
import ctypes
import json
import os
import threading

import numpy as np

from . import cuda
from ._source_key import source_key

int8, int16, int32, int64 = np.int8, np.int16, np.int32, np.int64
uint8, uint16, uint32, uint64 = np.uint8, np.uint16, np.uint32, np.uint64
float16, float32, float64 = np.float16, np.float32, np.float64
bool_ = np.bool_

_HERE = os.path.dirname(os.path.abspath(__file__))
KERNEL_DIR = os.environ.get(
    "DFSNN_REF_CUDA_DIR", os.path.join(os.path.dirname(os.path.dirname(_HERE)), "_ref", "cuda"))

_lock = threading.Lock()
_manifest = None
_modules = {}        # (key, device ordinal) -> CUmodule
_contexts = {}       # device ordinal -> primary CUcontext


def _load_manifest():
    global _manifest
    if _manifest is None:
        path = os.path.join(KERNEL_DIR, "manifest.json")
        if not os.path.exists(path):
            raise RuntimeError(f"no prebuilt reference kernels at {KERNEL_DIR} "
                               "(run oracle/build_ref.py where the reference checkout exists)")
        with open(path) as f:
            _manifest = json.load(f)
    return _manifest


def available():
    return os.path.exists(os.path.join(KERNEL_DIR, "manifest.json"))


def _context(device):
    ctx = _contexts.get(device)
    if ctx is None:
        d = cuda._driver()
        dev = ctypes.c_int()
        cuda._check(d.cuDeviceGet(ctypes.byref(dev), device), "cuDeviceGet")
        c = ctypes.c_void_p()
        cuda._check(d.cuDevicePrimaryCtxRetain(ctypes.byref(c), dev), "cuDevicePrimaryCtxRetain")
        ctx = _contexts[device] = c
    cuda._check(cuda._driver().cuCtxSetCurrent(ctx), "cuCtxSetCurrent")
    return ctx


class _Memory:
    def __init__(self, ptr):
        self.ptr = ptr


class ndarray:
    """A view of a torch CUDA tensor (what from_dlpack returns); kernels take its address."""

    def __init__(self, tensor):
        self._tensor = tensor
        self.data = _Memory(int(tensor.data_ptr()))
        self.shape = tuple(tensor.shape)
        self.size = tensor.numel()
        self.device = cuda.Device(tensor.device.index)

    def __getattr__(self, name):
        raise NotImplementedError(f"cupy.ndarray.{name} is not covered by the CuPy stand-in")


def from_dlpack(obj):
    import torch
    if not isinstance(obj, torch.Tensor):
        obj = torch.utils.dlpack.from_dlpack(obj)
    if not obj.is_cuda:
        raise ValueError("from_dlpack: the CuPy stand-in takes CUDA tensors only")
    return ndarray(obj)


def _not_covered(name):
    def f(*a, **k):
        raise NotImplementedError(f"cupy.{name} is not covered by the CuPy stand-in")
    return f


asarray = _not_covered("asarray")
empty = _not_covered("empty")
zeros = _not_covered("zeros")

_SCALARS = {
    np.int8: ctypes.c_int8, np.int16: ctypes.c_int16, np.int32: ctypes.c_int32,
    np.int64: ctypes.c_int64, np.uint8: ctypes.c_uint8, np.uint16: ctypes.c_uint16,
    np.uint32: ctypes.c_uint32, np.uint64: ctypes.c_uint64, np.float32: ctypes.c_float,
    np.float64: ctypes.c_double, np.bool_: ctypes.c_bool,
}


def _pack(arg):
    if isinstance(arg, ndarray):
        return ctypes.c_void_p(arg.data.ptr), arg.device.id
    t = type(arg)
    if t in _SCALARS:
        return _SCALARS[t](arg.item()), None
    # CuPy passes Python scalars as 64-bit values
    if isinstance(arg, bool):
        return ctypes.c_bool(arg), None
    if isinstance(arg, int):
        return ctypes.c_int64(arg), None
    if isinstance(arg, float):
        return ctypes.c_double(arg), None
    raise TypeError(f"unsupported kernel argument type {t.__name__}")


def _dims(v):
    v = (v,) if isinstance(v, int) else tuple(int(x) for x in v)
    if not 1 <= len(v) <= 3 or min(v) < 1:
        raise ValueError(f"bad launch dimensions {v}")
    return v + (1,) * (3 - len(v))


class RawKernel:
    def __init__(self, code, name, options=(), backend="nvrtc", translate_cucomplex=False,
                 enable_cooperative_groups=False, jitify=False):
        self.code, self.name, self.options = code, name, tuple(options)
        self.key = source_key(code, self.options)
        entry = _load_manifest().get(self.key)
        if entry is None:
            raise RuntimeError(f"RawKernel {name}: this source/options pair was not prebuilt "
                               f"(key {self.key}); rebuild oracle/_ref with oracle/build_ref.py")
        if name not in entry["names"]:
            raise RuntimeError(f"RawKernel {name}: not a kernel of this source")
        self._cubin = os.path.join(KERNEL_DIR, entry["cubin"])
        self._params = entry["params"][name]     # byte size of every declared parameter

    def _function(self, device):
        with _lock:
            _context(device)
            mod = _modules.get((self.key, device))
            if mod is None:
                with open(self._cubin, "rb") as f:
                    image = f.read()
                mod = ctypes.c_void_p()
                cuda._check(cuda._driver().cuModuleLoadData(ctypes.byref(mod), image),
                            "cuModuleLoadData")
                _modules[(self.key, device)] = mod
            fn = ctypes.c_void_p()
            cuda._check(cuda._driver().cuModuleGetFunction(ctypes.byref(fn), mod,
                                                           self.name.encode()),
                        "cuModuleGetFunction")
            return fn

    def __call__(self, grid, block, args, shared_mem=0, stream=None):
        import torch
        held, device = [], None
        for a in args:
            c, dev = _pack(a)
            held.append(c)
            if device is None and dev is not None:
                device = dev
        # the driver reads every declared parameter from the argument list: a launch with a
        # different count or size would read past it, so it is refused here instead
        sizes = [ctypes.sizeof(c) for c in held]
        if sizes != self._params:
            raise TypeError(f"RawKernel {self.name}: arguments of {sizes} bytes for parameters "
                            f"of {self._params} bytes; not launched")
        if device is None:
            device = torch.cuda.current_device()
        fn = self._function(device)
        params = (ctypes.c_void_p * max(1, len(held)))(
            *[ctypes.cast(ctypes.pointer(c), ctypes.c_void_p) for c in held])
        g, b = _dims(grid), _dims(block)
        h = (stream if stream is not None else cuda.get_current_stream()).ptr
        cuda._check(cuda._driver().cuLaunchKernel(fn, g[0], g[1], g[2], b[0], b[1], b[2],
                                                  int(shared_mem), ctypes.c_void_p(h), params,
                                                  None), f"cuLaunchKernel({self.name})")
