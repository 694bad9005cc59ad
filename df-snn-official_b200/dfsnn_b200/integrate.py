"""Register the B200 drop-ins under the reference's module names.

    import dfsnn_b200.integrate as I
    I.install()                      # before `from spikeDE_dis.neuron import LIFNeuronFDE`
    ...build the reference model...
    I.rebind_aligned(aligned_glmulti_module)   # after an example's make_model()

install() places dfsnn_b200.fde_kernels at sys.modules['spikeDE_dis.fde_cupy_kernels_all']
and dfsnn_b200.direct_euler at sys.modules['spikeDE_dis.direct_euler_cupy'], so the lazy
`from .fde_cupy_kernels_all import ...` statements of spikeDE_dis/neuron.py (:1994,
:2105-2123, :958) resolve to the native Functions without editing the reference.
"""
import sys

from . import aligned_glmulti, direct_euler, fde_kernels

FDE_MODULE = "spikeDE_dis.fde_cupy_kernels_all"
EULER_MODULE = "spikeDE_dis.direct_euler_cupy"


def install():
    sys.modules[FDE_MODULE] = fde_kernels
    sys.modules[EULER_MODULE] = direct_euler
    pkg = sys.modules.get("spikeDE_dis")
    if pkg is not None:
        setattr(pkg, "fde_cupy_kernels_all", fde_kernels)
        setattr(pkg, "direct_euler_cupy", direct_euler)
    return fde_kernels


def rebind_aligned(example_module=None):
    """After an example's make_model(): point every glmulti lookup at the native
    AlignedGLMulti, replacing what the example's install('cupy') bound
    (examples/cnn128/aligned_glmulti.py:157-162)."""
    fde_kernels.LIFFDEGLMultiFunction = aligned_glmulti.AlignedGLMulti
    if example_module is not None:
        example_module.AlignedGLMulti = aligned_glmulti.AlignedGLMulti
        example_module.install = lambda backend="native": aligned_glmulti.install(backend, fde_kernels)
    return aligned_glmulti.AlignedGLMulti
