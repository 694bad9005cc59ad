"""The fused glmulti schedule (one native launch per direction) against the PyTorch chain it
replaces, on the GPU: scale and W bit for bit, the raw-mass gradient within 1e-5."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from dfsnn_b200 import schedule

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("T", [1, 2, 8, 16, 33, 64, 256])
@pytest.mark.parametrize("betas,masses", [([0.3, 0.4, 0.5], [0.5, 0.5, 0.7]),
                                          ([0.1, 0.3, 0.5], [0.5, 0.5, 0.7]),
                                          ([0.2, 0.9], [1.3, 0.05]),
                                          ([0.35], [21.5])])
@pytest.mark.parametrize("constraint", [1, 0])
def test_fused_schedule_matches_torch_chain(T, betas, masses, constraint):
    h = 0.1
    beta = torch.tensor(betas, dtype=torch.float32)
    basis = schedule.glmulti_basis(betas, T).to(DEV)
    hpow = schedule.h_pow_neg_beta(h, beta, DEV)
    coef = torch.tensor(masses, dtype=torch.float32)
    raw0 = torch.log(torch.expm1(coef)) if constraint == 1 else coef.clone()
    raw_a = raw0.to(DEV).requires_grad_(True)
    raw_b = raw0.to(DEV).requires_grad_(True)
    # reference chain
    m = F.softplus(raw_a) if constraint == 1 else raw_a
    ref = schedule.build_glmulti_schedule(m, beta, basis, h, T, h_pow=hpow)
    # fused
    scale, W = schedule.GLMultiScheduleFunction.apply(raw_b, basis, hpow, constraint)
    torch.cuda.synchronize()
    assert torch.equal(scale, ref["scale"].contiguous()), "scale differs"
    assert torch.equal(W, ref["weights"]), "W differs"
    g = torch.Generator(device=DEV).manual_seed(T)
    gs = torch.randn(T, device=DEV, generator=g)
    gW = torch.randn(T, T, device=DEV, generator=g)
    torch.autograd.backward([ref["scale"], ref["weights"]], [gs, gW])
    torch.autograd.backward([scale, W], [gs, gW])
    a, b = raw_a.grad.double().cpu().numpy(), raw_b.grad.double().cpu().numpy()
    # reference: fp32 autograd; fused: double accumulation
    assert np.allclose(b, a, rtol=1e-5, atol=1e-5 * np.abs(a).max()), (a, b)
