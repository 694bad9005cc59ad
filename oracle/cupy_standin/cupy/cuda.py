"""cupy.cuda subset of the CuPy stand-in: Device, ExternalStream, get_current_stream
(TEST AND BASELINE INFRASTRUCTURE ONLY).  Streams follow CuPy: the current stream is the
legacy default stream unless an ExternalStream context is active on this thread."""
import ctypes
import threading

_drv = None
_tls = threading.local()


def _driver():
    global _drv
    if _drv is None:
        d = ctypes.CDLL("libcuda.so.1")
        p, i, u = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint
        d.cuInit.argtypes = [u]
        d.cuDeviceGet.argtypes = [ctypes.POINTER(i), i]
        d.cuDevicePrimaryCtxRetain.argtypes = [ctypes.POINTER(p), i]
        d.cuCtxSetCurrent.argtypes = [p]
        d.cuModuleLoadData.argtypes = [ctypes.POINTER(p), ctypes.c_char_p]
        d.cuModuleGetFunction.argtypes = [ctypes.POINTER(p), p, ctypes.c_char_p]
        d.cuLaunchKernel.argtypes = [p, u, u, u, u, u, u, u, p, ctypes.POINTER(p), p]
        d.cuStreamSynchronize.argtypes = [p]
        d.cuGetErrorName.argtypes = [i, ctypes.POINTER(ctypes.c_char_p)]
        _check(d.cuInit(0), "cuInit", d)
        _drv = d
    return _drv


def _check(res, what, d=None):
    if res != 0:
        name = ctypes.c_char_p()
        try:
            (d or _driver()).cuGetErrorName(res, ctypes.byref(name))
        except Exception:
            pass
        raise RuntimeError(f"{what} failed: CUDA driver error {res} "
                           f"({(name.value or b'?').decode()})")


class Device:
    def __init__(self, device=None):
        import torch
        self.id = torch.cuda.current_device() if device is None else int(device)
        self._prev = []

    def use(self):
        import torch
        torch.cuda.set_device(self.id)

    def __enter__(self):
        import torch
        self._prev.append(torch.cuda.current_device())
        torch.cuda.set_device(self.id)
        return self

    def __exit__(self, *exc):
        import torch
        torch.cuda.set_device(self._prev.pop())
        return False


class _Stream:
    def __init__(self, ptr):
        self.ptr = int(ptr)

    def synchronize(self):
        _check(_driver().cuStreamSynchronize(ctypes.c_void_p(self.ptr)), "cuStreamSynchronize")


class ExternalStream(_Stream):
    def __init__(self, ptr, device_id=-1):
        super().__init__(ptr)

    def __enter__(self):
        stack = getattr(_tls, "stack", None)
        if stack is None:
            stack = _tls.stack = []
        stack.append(self)
        return self

    def __exit__(self, *exc):
        _tls.stack.pop()
        return False


def get_current_stream():
    stack = getattr(_tls, "stack", None)
    return stack[-1] if stack else _Stream(0)
