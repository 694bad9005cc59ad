"""Comparison helpers shared by the tests (spike-flip-aware, tolerance-stated)."""
import numpy as np

# Tolerances of the hot path (fp32): membranes and gradients within 1e-5 relative,
# spikes identical except for neurons that come within 1e-6 of the threshold.
RTOL = 1e-5
BAND = 1e-6


def near_threshold_neurons(p, th, band=BAND):
    """Neurons [N] whose pre-reset potential p[T,N] ever comes within `band` of th."""
    return np.any(np.abs(np.asarray(p, dtype=np.float64) - th) < band, axis=0)


def assert_spikes(got, ref, p_ref, th, band=BAND):
    """Spikes equal everywhere except on near-threshold neurons; returns the mask."""
    mask = near_threshold_neurons(p_ref, th, band)
    bad = (np.asarray(got) != np.asarray(ref))[:, ~mask]
    assert not bad.any(), f"{int(bad.sum())} spike mismatches outside the near-threshold band"
    return mask


def assert_close(got, ref, rtol=RTOL, atol_scale=None, mask=None, what=""):
    """|got-ref| <= rtol*(|ref| + s), s = atol_scale or the rms of ref (so values that are
    small only through cancellation are measured at the scale of their inputs)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if mask is not None and got.ndim == 2:
        got, ref = got[:, ~mask], ref[:, ~mask]
    elif mask is not None and got.ndim == 1:
        got, ref = got[~mask], ref[~mask]
    if ref.size == 0:
        return
    s = atol_scale if atol_scale is not None else float(np.sqrt(np.mean(ref ** 2)) + 1e-30)
    err = np.abs(got - ref)
    lim = rtol * (np.abs(ref) + s)
    worst = float(np.max(err / lim))
    assert worst <= 1.0, f"{what}: max err/limit = {worst:.3g} (max abs err {err.max():.3g})"


def assert_bitwise(got, ref, mask=None, what=""):
    got = np.asarray(got)
    ref = np.asarray(ref)
    if mask is not None:
        got, ref = (got[:, ~mask], ref[:, ~mask]) if got.ndim == 2 else (got[~mask], ref[~mask])
    bad = got.view(np.uint32) != ref.view(np.uint32)
    # +0.0 and -0.0 compare equal numerically; both are accepted
    bad &= ~((got == 0) & (ref == 0))
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} values differ bitwise " \
                          f"(max abs diff {np.abs(got.astype(np.float64) - ref).max():.3g})"


def differing_gpu(a, b):
    """Number of elements of two same-shape tensors whose float32 bits differ (+0 and -0
    count as equal), computed where the tensors live."""
    import torch
    a = a.detach().float().contiguous()
    b = b.detach().float().contiguous()
    eq = (a.view(torch.int32) == b.view(torch.int32)) | ((a == 0) & (b == 0))
    return int((~eq).sum())


def assert_bitwise_gpu(got, want, what=""):
    n = differing_gpu(got, want)
    assert n == 0, f"{what}: {n} of {got.numel()} values differ"
