"""Register the B200 drop-ins under the reference's module names.

    import dfsnn_b200.integrate as I
    I.install()                      # before `from spikeDE_dis.neuron import LIFNeuronFDE`
    ...build the reference model...
    I.rebind_aligned(aligned_glmulti_module)   # after an example's make_model()

install() places dfsnn_b200.fde_kernels at sys.modules['spikeDE_dis.fde_cupy_kernels_all']
and dfsnn_b200.direct_euler at sys.modules['spikeDE_dis.direct_euler_cupy'], so the lazy
`from .fde_cupy_kernels_all import ...` statements of spikeDE_dis/neuron.py (:1994,
:2105-2123, :958) resolve to the native Functions without editing the reference.  It also
rebinds the neuron's glmulti schedule builder (install_schedule).
"""
import importlib
import sys

from . import aligned_glmulti, direct_euler, fde_kernels
from . import neuron as _mirror

FDE_MODULE = "spikeDE_dis.fde_cupy_kernels_all"
EULER_MODULE = "spikeDE_dis.direct_euler_cupy"
NEURON_MODULE = "spikeDE_dis.neuron"
_SAVED_SCHEDULE = {}          # reference LIFNeuronFDE class -> its own _build_glmulti_schedule


def install(schedule=True):
    sys.modules[FDE_MODULE] = fde_kernels
    sys.modules[EULER_MODULE] = direct_euler
    pkg = sys.modules.get("spikeDE_dis")
    if pkg is not None:
        setattr(pkg, "fde_cupy_kernels_all", fde_kernels)
        setattr(pkg, "direct_euler_cupy", direct_euler)
    if schedule:
        install_schedule()
    return fde_kernels


def install_schedule():
    """Rebind spikeDE_dis.neuron.LIFNeuronFDE._build_glmulti_schedule (neuron.py:1494-1514) to
    this library's: for learnable Softplus masses (or fixed masses) on CUDA, scale and W come
    from one native launch and their gradient to the raw masses from one more
    (GLMultiScheduleFunction), instead of the reference's chain of about 2T + 10 small PyTorch
    kernels per direction, which every glmulti layer runs on every step.  scale and W are
    bit-identical; the mass gradient is accumulated in double (the reference's autograd sums
    in fp32).  Softmax masses and CPU tensors keep the PyTorch chain.  Imports
    spikeDE_dis.neuron when the package is importable; returns whether the method was rebound."""
    mod = sys.modules.get(NEURON_MODULE)
    if mod is None:
        try:
            mod = importlib.import_module(NEURON_MODULE)
        except Exception:
            return False
    cls = getattr(mod, "LIFNeuronFDE", None)
    if cls is None or not hasattr(cls, "_build_glmulti_schedule"):
        return False
    if cls not in _SAVED_SCHEDULE:
        _SAVED_SCHEDULE[cls] = cls.__dict__.get("_build_glmulti_schedule")
    cls._build_glmulti_schedule = _mirror.LIFNeuronFDE._build_glmulti_schedule
    return True


def uninstall_schedule():
    """Give the reference neuron class(es) their own schedule builder back."""
    for cls, fn in _SAVED_SCHEDULE.items():
        if fn is None:
            if "_build_glmulti_schedule" in cls.__dict__:
                delattr(cls, "_build_glmulti_schedule")
        else:
            cls._build_glmulti_schedule = fn
    _SAVED_SCHEDULE.clear()


def rebind_aligned(example_module=None):
    """After an example's make_model(): point every glmulti lookup at the native
    AlignedGLMulti, replacing what the example's install('cupy') bound
    (examples/cnn128/aligned_glmulti.py:157-162)."""
    fde_kernels.LIFFDEGLMultiFunction = aligned_glmulti.AlignedGLMulti
    if example_module is not None:
        example_module.AlignedGLMulti = aligned_glmulti.AlignedGLMulti
        example_module.install = lambda backend="native": aligned_glmulti.install(backend, fde_kernels)
    return aligned_glmulti.AlignedGLMulti
