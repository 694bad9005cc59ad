"""CPU checks of the GPU reference arm's plumbing: every kernel source text the reference
hands to cupy.RawKernel -- each autograd Function's get_kernels(), the direct-Euler
kernels and the examples' aligned kernels for the prebuilt HISTORY_RHO values -- is found
among the prebuilt cubins, and the stand-in rejects a text that was not prebuilt."""
import pytest

import refenv

pytestmark = pytest.mark.skipif(refenv.missing() is not None, reason=str(refenv.missing()))


@pytest.fixture(scope="module")
def ref():
    r = refenv.Reference("cnn128")
    yield r
    r.close()


def test_every_reference_function_finds_its_kernels(ref):
    names = [n for n in dir(ref.kernels)
             if n.endswith("Function") and hasattr(getattr(ref.kernels, n), "get_kernels")]
    assert len(names) >= 11
    for n in names:
        kernels = getattr(ref.kernels, n).get_kernels()
        assert all(k is not None for k in kernels), n


def test_direct_euler_and_aligned_kernels(ref):
    import aligned_glmulti as alg
    import cupy
    assert ref.euler._get_forward_kernel() is not None
    assert ref.euler._get_backward_kernel() is not None
    for rho in (1.0, 0.5):
        code = alg.BACKWARD.replace("adj[j]-=w[t*T+j]*r;", f"adj[j]-={rho:.8f}f*w[t*T+j]*r;")
        for name in ("aligned_forward", "aligned_backward", "aligned_scale",
                     "aligned_weight_partial"):
            cupy.RawKernel(alg.FORWARD + code, name, options=("--fmad=false",))


def test_standin_rejects_unbuilt_source(ref):
    import cupy
    with pytest.raises(RuntimeError, match="not prebuilt"):
        cupy.RawKernel("extern \"C\" __global__ void k(){}", "k")
    import aligned_glmulti as alg
    with pytest.raises(RuntimeError, match="not prebuilt"):       # options are part of the key
        cupy.RawKernel(alg.FORWARD, "aligned_forward")
    with pytest.raises(NotImplementedError):
        cupy.asarray([1.0])


def test_standin_refuses_mismatched_arguments(ref):
    """A launch whose arguments do not match the kernel's declared parameters is refused on
    the host (the driver would read past the argument list).  The reference's own
    LIFFDEVOPREDICTORFunction.backward is such a launch: six arrays for the seven pointers of
    lif_fde_vo_predictor_backward_kernel (fde_cupy_kernels_all.py:1160-1170, :1047-1062)."""
    import cupy
    import numpy as np
    k = cupy.RawKernel(ref.kernels.vo_predictor_backward_kernel_code,
                       "lif_fde_vo_predictor_backward_kernel")
    assert len(k._params) == 15 and k._params[:7] == [8] * 7
    with pytest.raises(TypeError, match="not launched"):
        k((1,), (256,), (np.int32(1), np.float32(2.0)))
    with pytest.raises(TypeError, match="not launched"):       # sizes, not just the count
        k((1,), (256,), tuple([1] * 7 + [1] * 4 + [np.float32(1.0)] * 4))   # int64, not int32
