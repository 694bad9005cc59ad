"""Import the unmodified reference next to this library, in one process (TEST AND
BASELINE INFRASTRUCTURE ONLY: the GPU-to-GPU parity tests and bench.py's GPU reference
leg use it; the library never does).

The reference package is the staged copy in baseline/_ref (oracle/stage_ref.py) and its
CuPy calls go to oracle/cupy_standin, which launches the reference's own kernel source
texts compiled for the GPU (oracle/build_ref.py).  `use_reference()` points the
reference's lazy `from .fde_cupy_kernels_all import ...` (spikeDE_dis/neuron.py:1994,
2105-2123) at its own module; `use_native()` at this library, exactly as
dfsnn_b200.integrate.install() does for a user.  `close()` removes every module the
reference brought in, so later tests see a clean interpreter.
"""
import os
import sys
import types

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STANDIN = os.path.join(REPO, "oracle", "cupy_standin")
STAGED = os.path.join(REPO, "baseline", "_ref")
EXAMPLES = os.path.join(STAGED, "examples")
CUDA_MANIFEST = os.path.join(REPO, "oracle", "_ref", "cuda", "manifest.json")
FDE = "spikeDE_dis.fde_cupy_kernels_all"
EULER = "spikeDE_dis.direct_euler_cupy"
_OWNED = ("spikeDE_dis", "cupy", "h5py", "aligned_glmulti", "cnn128_aligned", "model", "timm",
          "einops")


def staged():
    """True when the reference package and the example modules are staged."""
    return os.path.isdir(os.path.join(STAGED, "spikeDE_dis")) and os.path.isdir(EXAMPLES)


def missing():
    """Why the reference arm cannot run here, or None."""
    if not os.path.isdir(os.path.join(STAGED, "spikeDE_dis")):
        return "reference not staged (oracle/stage_ref.py)"
    if not os.path.exists(CUDA_MANIFEST):
        return "reference kernels not built for the GPU (oracle/build_ref.py)"
    return None


def _stub_h5py():
    # spikeDE_dis/solver.py:4 imports h5py.h5z.FLAG_SKIP_EDC; h5py is not installed
    h5 = types.ModuleType("h5py")
    h5z = types.ModuleType("h5py.h5z")
    h5z.FLAG_SKIP_EDC = 0
    h5.h5z = h5z
    sys.modules["h5py"] = h5
    sys.modules["h5py.h5z"] = h5z


def _stub_timm():
    """The four timm names examples/*/model.py imports (timm is not installed): the same
    definitions timm gives them, written here."""
    import torch
    import torch.nn as nn

    class DropPath(nn.Module):
        def __init__(self, drop_prob=0.0):
            super().__init__()
            self.drop_prob = drop_prob

        def forward(self, x):
            if self.drop_prob == 0.0 or not self.training:
                return x
            keep = 1.0 - self.drop_prob
            mask = x.new_empty((x.shape[0],) + (1,) * (x.ndim - 1)).bernoulli_(keep)
            return x * mask / keep

    layers = types.ModuleType("timm.models.layers")
    layers.to_2tuple = lambda v: tuple(v) if isinstance(v, (tuple, list)) else (v, v)
    layers.trunc_normal_ = lambda t, mean=0.0, std=1.0, a=-2.0, b=2.0: \
        torch.nn.init.trunc_normal_(t, mean, std, a, b)
    layers.DropPath = DropPath
    registry = types.ModuleType("timm.models.registry")
    registry.register_model = lambda fn: fn
    vit = types.ModuleType("timm.models.vision_transformer")
    vit._cfg = lambda url="", **kw: dict(url=url, **kw)
    models = types.ModuleType("timm.models")
    timm = types.ModuleType("timm")
    timm.models, models.layers, models.registry, models.vision_transformer = \
        models, layers, registry, vit
    for name, mod in (("timm", timm), ("timm.models", models), ("timm.models.layers", layers),
                      ("timm.models.registry", registry),
                      ("timm.models.vision_transformer", vit)):
        sys.modules[name] = mod


class Reference:
    """standin=False imports the reference without the CuPy stand-in: its own kernels then
    cannot run at all (CUPY_AVAILABLE is false and every CuPy launch fails), which is how
    the native benchmark uses the reference's network code."""

    def __init__(self, example=None, standin=True):
        self._path = list(sys.path)
        self._before = set(sys.modules)
        paths = ([STANDIN] if standin else []) + [STAGED] + \
            ([os.path.join(EXAMPLES, example)] if example else [])
        for p in reversed(paths):
            sys.path.insert(0, p)
        _stub_h5py()
        if example and example.startswith("spikformer"):
            _stub_timm()
        import spikeDE_dis.direct_euler_cupy as euler
        import spikeDE_dis.fde_cupy_kernels_all as kernels
        import spikeDE_dis.neuron as neuron
        if standin and not kernels.CUPY_AVAILABLE:
            raise RuntimeError("the CuPy stand-in was not picked up")
        if not standin and "cupy" in sys.modules:
            raise RuntimeError("a cupy module is importable; the native benchmark expects none")
        self.kernels, self.euler, self.neuron = kernels, euler, neuron
        self.pkg = sys.modules["spikeDE_dis"]

    def use_reference(self):
        from dfsnn_b200 import integrate
        integrate.uninstall_schedule()
        sys.modules[FDE] = self.kernels
        sys.modules[EULER] = self.euler
        self.pkg.fde_cupy_kernels_all = self.kernels
        self.pkg.direct_euler_cupy = self.euler

    def use_native(self):
        from dfsnn_b200 import integrate
        integrate.install()

    def close(self):
        from dfsnn_b200 import integrate
        integrate.uninstall_schedule()
        for name in list(sys.modules):
            if name not in self._before and name.split(".")[0] in _OWNED:
                del sys.modules[name]
        for name in ("h5py", "h5py.h5z"):
            if name not in self._before:
                sys.modules.pop(name, None)
        sys.path[:] = self._path
