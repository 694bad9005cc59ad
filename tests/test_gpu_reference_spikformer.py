"""The Spikformer256 example of the reference (examples/spikformer_har_lip: aligned_glmulti
.make_model building model.DirectFDESpikformer, embed 256, depth 2, 19 LIF layers), run
unmodified on the GPU: one training step with the reference's own aligned kernels (through
the CuPy stand-in), then the same step with this library installed the documented way
(integrate.install(), the example's install('cupy'), integrate.rebind_aligned()).  Spikes
are bit-identical, so the logits and every non-LIF gradient are too; the shared mass
gradient is a reduction (1e-5 of its scale, with margin for the reference's own float32
sums)."""
import pytest
import torch

import refenv
from parity import assert_bitwise_gpu
from dfsnn_b200 import aligned_glmulti as native_aligned
from dfsnn_b200 import fde_kernels, integrate

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(refenv.missing() is not None, reason=str(refenv.missing()))]
DEV = "cuda:0"


def test_spikformer256_example_drop_in():
    ref = refenv.Reference("spikformer_har_lip")
    library_ref, library_native = ref.kernels.LIFFDEGLMultiFunction, fde_kernels.LIFFDEGLMultiFunction
    det, bench = torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark
    torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark = True, False
    try:
        import aligned_glmulti as alg
        example_install, example_function = alg.install, alg.AlignedGLMulti
        ref.use_reference()
        torch.manual_seed(0)
        model = alg.make_model("cupy", [0.3, 0.4, 0.5], True, [0.5, 0.5, 0.7], batch=16, T=8,
                               num_classes=300).to(DEV)
        g = torch.Generator(device=DEV).manual_seed(9)
        frames = (torch.rand((8, 16, 2, 128, 128), device=DEV, generator=g) < 0.05).float()
        labels = torch.randint(0, 300, (16,), device=DEV, generator=g)

        def train_step():
            for m in model.modules():
                if isinstance(m, ref.neuron.LIFNeuronFDE):
                    m.reset()
            model.zero_grad(set_to_none=True)
            torch.manual_seed(1)
            out = model(frames)
            torch.nn.functional.cross_entropy(out, labels).backward()
            torch.cuda.synchronize()
            return out.detach(), {n: p.grad.detach().clone()
                                  for n, p in model.named_parameters() if p.grad is not None}

        calls = dict(alg.CALLS)
        want_out, want_grads = train_step()
        n_lif = alg.CALLS["forward"] - calls["forward"]
        assert n_lif == 19
        ref.use_native()
        alg.install("cupy")
        integrate.rebind_aligned(alg)
        calls, native_calls = dict(alg.CALLS), dict(native_aligned.CALLS)
        got_out, got_grads = train_step()
        assert alg.CALLS == calls, "a reference kernel ran after the rebind"
        assert native_aligned.CALLS["forward"] - native_calls["forward"] == n_lif
        assert native_aligned.CALLS["backward"] - native_calls["backward"] == n_lif
    finally:
        torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark = det, bench
        ref.kernels.LIFFDEGLMultiFunction = library_ref
        fde_kernels.LIFFDEGLMultiFunction = library_native
        try:
            alg.install, alg.AlignedGLMulti = example_install, example_function
        except NameError:
            pass
        ref.close()
    assert_bitwise_gpu(got_out, want_out, "Spikformer256 logits")
    assert set(got_grads) == set(want_grads)
    shared = [n for n in want_grads if "multi_coefficient" in n]
    assert shared, "no shared mass parameter found"
    for n in want_grads:
        if n in shared:
            w, gg = want_grads[n], got_grads[n]
            assert float((gg - w).abs().max()) <= 1e-4 * (float(w.abs().max()) + 1e-30), n
        else:
            assert_bitwise_gpu(got_grads[n], want_grads[n], f"Spikformer256 grad {n}")
