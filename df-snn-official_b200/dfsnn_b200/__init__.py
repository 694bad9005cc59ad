"""dfsnn_b200 -- B200 (sm_100a) implementation of DF-SNN's LIFNeuronFDE hot path.

Modules
  fde_kernels      drop-in for spikeDE_dis.fde_cupy_kernels_all (autograd Functions)
  aligned_glmulti  drop-in for examples/*/aligned_glmulti.py (AlignedGLMulti, install)
  direct_euler     drop-in for spikeDE_dis.direct_euler_cupy
  neuron           LIFNeuronFDE mirror for the multi-step B200 path
  schedule         weight tables (glmulti schedule, GL / trapezoid / predictor)
  integrate        registers the drop-ins under the reference's module names
The kernels live in libdfsnn_b200.so (C ABI: include/dfsnn_b200.h), built by
df-snn-official_b200/build.py.
"""
from . import _capi  # noqa: F401

__all__ = ["fde_kernels", "aligned_glmulti", "direct_euler", "neuron", "schedule", "integrate"]
