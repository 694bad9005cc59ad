"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that holds the reference checkout ($DFSNN_REFERENCE, else the default
of oracle/build_ref.py):
    python tests/golden/make_golden.py [--reference PATH]

Two kinds of fixture are written, each an .npz holding its inputs and outputs:
  * torch_*.npz  -- the reference's own PyTorch code:
        LIFNeuronFDE(backend='torch') for gl / trap / predictor / glmulti
        (spikeDE_dis/neuron.py:1642-1788, 2292-2637), the reference autograd Function
        LIFFDEFAGL1TorchFunction with the glmulti schedule (the library glmulti recurrence
        and full-history VJP, spikeDE_dis/fde_cupy_kernels_all.py:1501-1587), and the
        authors' definition of the aligned semantics, aligned_glmulti.reference()
        (examples/cnn128/aligned_glmulti.py:147-155), differentiated by autograd.
  * kern_*.npz   -- the reference's CUDA kernel sources compiled for the host
        (oracle/build_ref.py), i.e. the arithmetic of the CuPy kernels themselves.
Fixtures stay small (N <= 512) so the whole set is a few hundred KB.
"""
import argparse
import math
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

TAU, TH, SG, H = 2.0, 1.0, 5.0, 0.1
MULTI_BETA = [0.3, 0.4, 0.5]
MASSES = [0.5, 0.5, 0.7]


def _stub_h5py():
    if "h5py" not in sys.modules:
        h5 = types.ModuleType("h5py")
        h5z = types.ModuleType("h5py.h5z")
        h5z.FLAG_SKIP_EDC = 0
        h5.h5z = h5z
        sys.modules["h5py"] = h5
        sys.modules["h5py.h5z"] = h5z


def _save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    print("wrote", path)


def _inputs(seed, T, B, F, kind):
    g = np.random.default_rng(seed)
    if kind == "config1":      # N(0.3, 0.5^2): the BASELINE CPU configuration's distribution
        x = g.normal(0.3, 0.5, size=(T, B, F))
    elif kind == "spiking":    # randn*5, as the reference's test_method (:2788)
        x = g.standard_normal((T, B, F)) * 5.0
    else:                      # N(1.5, 1): steady spiking
        x = g.normal(1.5, 1.0, size=(T, B, F))
    gS = g.standard_normal((T, B, F))
    gV = g.standard_normal((T, B, F))
    return x.astype(np.float32), gS.astype(np.float32), gV.astype(np.float32)


def torch_single(ref, method, beta, T, B, F, kind, seed):
    import torch
    from spikeDE_dis.neuron import LIFNeuronFDE
    x, gS, gV = _inputs(seed, T, B, F, kind)
    neuron = LIFNeuronFDE(tau=TAU, threshold=TH, surrogate_grad_scale=SG, surrogate_function="arctan",
                          beta=beta, T=T, method=method, step_size=H, batchsize=B, step_mode="m",
                          backend="torch", store_v_seq=True)
    xt = torch.tensor(x, requires_grad=True)
    s = neuron(xt)
    v = neuron.v_seq
    loss = (s * torch.tensor(gS)).sum() + (v * torch.tensor(gV)).sum()
    loss.backward()
    _save(f"torch_{method}_{kind}_T{T}.npz", x=x, gS=gS, gV=gV, beta=np.float32(beta),
          spike=s.detach().numpy(), v=v.detach().numpy(), gx=xt.grad.numpy())


def torch_glmulti_neuron(ref, T, B, F, kind, seed):
    """LIFNeuronFDE torch path for glmulti: truncated history, grads reach the raw masses."""
    import torch
    from spikeDE_dis.neuron import LIFNeuronFDE
    x, gS, _ = _inputs(seed, T, B, F, kind)
    neuron = LIFNeuronFDE(tau=TAU, threshold=TH, surrogate_grad_scale=SG, surrogate_function="arctan",
                          beta=MULTI_BETA[0], T=T, method="glmulti", step_size=H, batchsize=B,
                          step_mode="m", backend="torch", store_v_seq=True, multi_beta=MULTI_BETA,
                          multi_coefficient=MASSES, learn_coefficient=True,
                          coefficient_constraint="softplus", glmulti_history_grad="full")
    xt = torch.tensor(x, requires_grad=True)
    s = neuron(xt)
    loss = (s * torch.tensor(gS)).sum()
    loss.backward()
    _save(f"torch_glmulti_neuron_{kind}_T{T}.npz", x=x, gS=gS, spike=s.detach().numpy(),
          v=neuron.v_seq.detach().numpy(), gx=xt.grad.numpy(),
          graw=neuron.multi_coefficient_raw.grad.numpy(),
          raw=neuron.multi_coefficient_raw.detach().numpy())


def glmulti_schedule(T):
    """scale[T] and W[T,T] exactly as LIFNeuronFDE._build_glmulti_schedule builds them."""
    import torch
    from spikeDE_dis.neuron import LIFNeuronFDE
    neuron = LIFNeuronFDE(tau=TAU, threshold=TH, surrogate_grad_scale=SG, surrogate_function="arctan",
                          beta=MULTI_BETA[0], T=T, method="glmulti", step_size=H, batchsize=1,
                          step_mode="m", backend="torch", multi_beta=MULTI_BETA,
                          multi_coefficient=MASSES, learn_coefficient=True,
                          coefficient_constraint="softplus", glmulti_history_grad="full")
    with torch.no_grad():
        terms = neuron._build_glmulti_schedule(T, torch.device("cpu"))
    return terms["scale"].contiguous().numpy().copy(), terms["weights"].numpy().copy()


def torch_glmulti_function(ref, T, B, F, kind, seed):
    """Library glmulti recurrence + full-history VJP via LIFFDEFAGL1TorchFunction."""
    import torch
    from spikeDE_dis.fde_cupy_kernels_all import LIFFDEFAGL1TorchFunction
    x, gS, _ = _inputs(seed, T, B, F, kind)
    scale, W = glmulti_schedule(T)
    N = B * F
    xt = torch.tensor(x.reshape(T, N), requires_grad=True)
    v0 = torch.zeros(N, requires_grad=True)
    Wt = torch.tensor(W, requires_grad=True)
    s = LIFFDEFAGL1TorchFunction.apply(xt, v0, Wt, TAU, float(scale[0]), TH, SG, B, True)
    (s * torch.tensor(gS.reshape(T, N))).sum().backward()
    _save(f"torch_glmulti_full_{kind}_T{T}.npz", x=x.reshape(T, N), gS=gS.reshape(T, N),
          scale=scale, W=W, spike=s.detach().numpy(), gx=xt.grad.numpy(), gv0=v0.grad.numpy(),
          gW=Wt.grad.numpy())


def torch_aligned(ref, T, B, F, kind, seed):
    import torch
    import aligned_glmulti as alg
    x, gS, _ = _inputs(seed, T, B, F, kind)
    scale, W = glmulti_schedule(T)
    N = B * F
    xt = torch.tensor(x.reshape(T, N), requires_grad=True)
    v0 = torch.zeros(N, requires_grad=True)
    a = torch.tensor(scale, requires_grad=True)
    w = torch.tensor(W, requires_grad=True)
    s = alg.reference(xt, v0, a, w, TAU, TH, SG)
    (s * torch.tensor(gS.reshape(T, N))).sum().backward()
    _save(f"torch_aligned_{kind}_T{T}.npz", x=x.reshape(T, N), gS=gS.reshape(T, N), a=scale, W=W,
          spike=s.detach().numpy(), gx=xt.grad.numpy(), gv0=v0.grad.numpy(),
          ga=a.grad.numpy(), gw=w.grad.numpy())


def kernel_fixtures(T, N, seed):
    """Outputs of the reference kernel sources compiled for the host (oracle/_ref)."""
    sys.path.insert(0, REPO)
    from oracle import build_ref, oracle
    if not oracle.ref_available():
        build_ref.build(build_ref_reference)
    g = np.random.default_rng(seed)
    x = (g.standard_normal((T, N)) * 5.0).astype(np.float32)
    v0 = (g.standard_normal(N) * 0.1).astype(np.float32)
    gS = g.standard_normal((T, N)).astype(np.float32)
    gV = g.standard_normal((T, N)).astype(np.float32)
    beta = 0.7
    c = np.zeros(T + 1, dtype=np.float32)
    c[0] = 1.0
    for j in range(1, T + 1):
        c[j] = np.float32(1.0 - (1.0 + beta) / j) * c[j - 1]
    crev = c[::-1].copy()
    hb = np.float32(H ** beta)
    g1 = np.float32(math.exp(math.lgamma(beta + 1.0)))
    for scheme in ("gl", "trap", "predictor", "gl1", "trap1", "predictor1", "euler"):
        # TRAP1 receives h_beta = 1**beta = 1 from its Function (fde_cupy_kernels_all.py:2190)
        hbs = np.float32(1.0) if scheme == "trap1" else hb
        s, v = oracle.single_forward(scheme, x, v0, crev, TAU, beta, TH, hbs, g1, impl="ref")
        gx, gv0 = oracle.single_backward(scheme, gS, gV, x, v0, crev, TAU, beta, TH, SG, hbs, g1,
                                         impl="ref")
        _save(f"kern_{scheme}_T{T}.npz", x=x, v0=v0, w=crev, gS=gS, gV=gV, beta=np.float32(beta),
              h_beta=hbs, gamma1=g1, spike=s, v=v, gx=gx, gv0=gv0)
    scale, W = glmulti_schedule(T)
    for full in (0, 1):
        fw = oracle.glmulti_forward(x, v0, scale, W, TAU, TH, impl="ref")
        gx, gv0, gpre = oracle.glmulti_backward(full, gS, scale, W, fw["vpre"], TAU, TH, SG, impl="ref")
        _save(f"kern_glmulti_{'full' if full else 'trunc'}_T{T}.npz", x=x, v0=v0, scale=scale, W=W,
              gS=gS, spike=fw["spike"], vpre=fw["vpre"], vhist=fw["vhist"], drift=fw["drift"],
              gx=gx, gv0=gv0, gpre=gpre)
    a = (scale * 4.0).astype(np.float32)
    fw = oracle.aligned_forward(x, v0, a, W, TAU, TH, impl="ref")
    gx, gv, ga = oracle.aligned_backward(gS, a, W, fw["pred"], TAU, TH, SG, 1.0, impl="ref")
    _save(f"kern_aligned_T{T}.npz", x=x, v0=v0, a=a, W=W, gS=gS, spike=fw["spike"],
          pred=fw["pred"], hist=fw["hist"], gx=gx, gv0=gv, ga=ga)


def history_tables(T, B, seed):
    """VO-GL1 / VO-PREDICTOR schedules from the reference's builders
    (LIFNeuronFDE.build_vogl1_schedule / build_vopredictor_schedule, neuron.py:2010-2090) for
    a shared beta[T] and a per-sample beta[T, B]; FAGL1 rows = GL coefficients x a random
    positive causal attention, shared [T, T] and per-sample [T, B, T] (the shape of
    _build_fagl1_weights, neuron.py:1790-1888)."""
    import torch
    from spikeDE_dis.neuron import LIFNeuronFDE
    g = torch.Generator().manual_seed(seed)
    out = {}
    for tag, beta in (("shared", 0.2 + 0.6 * torch.rand(T, generator=g)),
                      ("batch", 0.2 + 0.6 * torch.rand(T, B, generator=g))):
        vo = LIFNeuronFDE.build_vogl1_schedule(beta, H)
        vp = LIFNeuronFDE.build_vopredictor_schedule(beta, H)
        out[f"vogl1_{tag}"] = (vo["scale"].numpy().copy(), vo["weights"].numpy().copy())
        out[f"vopred_{tag}"] = (vp["scale"].numpy().copy(), vp["weights"].numpy().copy())
        out[f"beta_{tag}"] = beta.numpy().copy()
    beta = 0.6
    c = [1.0]
    for k in range(1, T + 1):
        c.append(c[-1] * (1.0 - (1.0 + beta) / k))
    lag = np.subtract.outer(np.arange(T), np.arange(T))
    gl = np.where(lag > 0, np.asarray(c, np.float64)[np.clip(lag, 0, T)], 0.0)
    rnd = np.random.default_rng(seed)
    att_s = rnd.uniform(0.5, 1.5, size=(T, T))
    att_b = rnd.uniform(0.5, 1.5, size=(T, B, T))
    out["fagl1_shared"] = (None, (gl * att_s).astype(np.float32))
    out["fagl1_batch"] = (None, (gl[:, None, :] * att_b).astype(np.float32))
    return out


def history_fixtures(T, B, F, seed):
    """kern_hist_<kind>_T<T>.npz: the reference's VO-GL1 / FAGL1 / VO-PREDICTOR kernel
    sources compiled for the host (fde_cupy_kernels_all.py:1017-1096, :1200-1312,
    :1594-1709), shared and per-sample tables, truncated and full history; and
    torch_fagl1_<tables>_T<T>.npz from the reference's LIFFDEFAGL1TorchFunction
    (:1501-1587) with autograd."""
    import torch
    sys.path.insert(0, REPO)
    from oracle import build_ref, oracle
    if not oracle.ref_available():
        build_ref.build(build_ref_reference)
    from spikeDE_dis.fde_cupy_kernels_all import LIFFDEFAGL1TorchFunction
    N = B * F
    g = np.random.default_rng(seed)
    x = (g.standard_normal((T, N)) * 5.0).astype(np.float32)
    v0 = (g.standard_normal(N) * 0.1).astype(np.float32)
    gS = g.standard_normal((T, N)).astype(np.float32)
    tables = history_tables(T, B, seed)
    hb = np.float32(H ** 0.6)
    rm = 0.25
    for kind in ("vogl1", "fagl1", "vopred"):
        arrays = dict(x=x, v0=v0, gS=gS, B=np.int32(B), h_beta=hb, residual_mix=np.float32(rm))
        for tag in ("shared", "batch"):
            scale, W = tables[f"{kind}_{tag}"]
            if scale is not None:
                arrays[f"{tag}_scale"] = scale
                arrays[f"{tag}_beta"] = tables[f"beta_{tag}"]
            arrays[f"{tag}_W"] = W
            fw = oracle.hfam_forward(kind, x, v0, scale, W, B, TAU, TH, hb, rm, impl="ref")
            for k in ("spike", "vpre", "hsrc"):
                arrays[f"{tag}_{k}"] = fw[k]
            for full in ((0, 1) if kind != "vopred" else (0,)):
                gx, gv0, gpre = oracle.hfam_backward(kind, full, gS, fw["vpre"], scale, W, B, TAU,
                                                     TH, SG, hb, rm, impl="ref")
                arrays[f"{tag}_f{full}_gx"] = gx
                arrays[f"{tag}_f{full}_gv0"] = gv0
                arrays[f"{tag}_f{full}_gpre"] = gpre
        _save(f"kern_hist_{kind}_T{T}.npz", **arrays)
    for tag in ("shared", "batch"):
        _, W = tables[f"fagl1_{tag}"]
        for full in (False, True):
            xt = torch.from_numpy(x).requires_grad_(True)
            vt = torch.from_numpy(v0).requires_grad_(True)
            Wt = torch.from_numpy(W).requires_grad_(True)
            s = LIFFDEFAGL1TorchFunction.apply(xt, vt, Wt, TAU, float(hb), TH, SG, B, full)
            s.backward(torch.from_numpy(gS))
            _save(f"torch_fagl1_{tag}_{'full' if full else 'trunc'}_T{T}.npz", x=x, v0=v0, W=W,
                  gS=gS, B=np.int32(B), h_beta=hb, spike=s.detach().numpy(),
                  gx=xt.grad.numpy(), gv0=vt.grad.numpy(), gW=Wt.grad.numpy())


def fagl1_neuron_fixture():
    """torch_fagl1_neuron.npz: LIFNeuronFDE(method='fagl1') attention projections after
    __init__ (seeded per layer name) and _build_fagl1_weights on a fixed input
    (neuron.py:1205-1221, :1790-1866) for both attn_init and attn_mode values; plus the
    GL1 full-history rows _build_gl1_causal_weights (:1880-1896)."""
    import torch
    from spikeDE_dis.neuron import LIFNeuronFDE
    g = torch.Generator().manual_seed(21)
    x = torch.randn((8, 4, 3, 5), generator=g) * 2.0 + 0.5
    out = {"x": x.numpy()}
    for init in ("zero_q", "orthogonal_zero_score"):
        for mode in ("per_sample", "batch_shared"):
            n = LIFNeuronFDE(tau=TAU, threshold=TH, surrogate_grad_scale=SG, method="fagl1",
                             beta=0.6, T=8, step_size=H, name="lif3", step_mode="m",
                             backend="torch", attn_init=init, attn_mode=mode)
            tag = f"{init}_{mode}"
            out[f"{tag}_q"] = n.fagl_q_proj.weight.detach().numpy().copy()
            out[f"{tag}_k"] = n.fagl_k_proj.weight.detach().numpy().copy()
            out[f"{tag}_W"] = n._build_fagl1_weights(x).detach().numpy().copy()
            out[f"{tag}_entropy"] = np.float32(n.get_attention_stats()["entropy"])
    n = LIFNeuronFDE(method="gl1", beta=0.6, T=8, step_size=H, step_mode="m", backend="torch")
    out["gl1_rows"] = n._build_gl1_causal_weights(8, torch.device("cpu")).numpy()
    _save("torch_fagl1_neuron.npz", **out)


def weight_tables():
    """GL / trapezoid / predictor tables and the glmulti schedule, as the reference builds
    them (neuron.py:1446-1459, :1516-1570, :1494-1514), plus LIFNeuronFDE state_dict keys."""
    import torch
    from spikeDE_dis.neuron import LIFNeuronFDE
    out = {}
    for beta in (0.3, 0.5, 0.7):
        for T in (8, 16, 20, 64, 256):
            n = LIFNeuronFDE(beta=beta, T=T, step_size=H, step_mode="m", backend="torch", method="gl")
            dev, dt = torch.device("cpu"), torch.float32
            out[f"gl_b{beta}_T{T}"] = n._get_gl_weights(T, dev, dt).numpy()
            out[f"trap_b{beta}_T{T}"] = n._get_trap_weights(T, dev, dt).numpy()
            out[f"predictor_b{beta}_T{T}"] = n._get_predictor_weights(T, dev, dt).numpy()
    for T in (1, 8, 16, 32):
        scale, W = glmulti_schedule(T)
        out[f"glmulti_scale_T{T}"] = scale
        out[f"glmulti_W_T{T}"] = W
    keys = {}
    for method in ("glmulti", "gl"):
        kw = dict(tau=TAU, threshold=TH, surrogate_grad_scale=SG, surrogate_function="arctan",
                  beta=MULTI_BETA[0], T=16, method=method, step_size=H, batchsize=4,
                  step_mode="m", backend="cupy")
        if method == "glmulti":
            kw.update(multi_beta=MULTI_BETA, multi_coefficient=MASSES, learn_coefficient=True,
                      coefficient_constraint="softplus", glmulti_history_grad="full")
        keys[method] = sorted(LIFNeuronFDE(**kw).state_dict().keys())
    out["state_dict_keys_glmulti"] = np.array(keys["glmulti"])
    out["state_dict_keys_gl"] = np.array(keys["gl"], dtype="U64")
    _save("torch_tables.npz", **out)


build_ref_reference = None


def main():
    global build_ref_reference
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    from build_ref import reference_path
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--only", choices=["history"], default=None,
                    help="write only this group of fixtures")
    args = ap.parse_args()
    args.reference = reference_path(args.reference)
    build_ref_reference = args.reference
    _stub_h5py()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, os.path.join(args.reference, "examples", "cnn128"))
    import torch
    torch.set_num_threads(4)
    if args.only == "history":
        history_fixtures(16, 4, 32, 11)
        fagl1_neuron_fixture()
        return
    for method in ("gl", "trap", "predictor"):
        torch_single(None, method, 0.7, 20, 4, 128, "spiking", 42)
        torch_single(None, method, 0.5, 16, 4, 128, "config1", 0)
    torch_glmulti_neuron(None, 16, 4, 128, "spiking", 1)
    torch_glmulti_neuron(None, 16, 4, 128, "config1", 0)
    torch_glmulti_function(None, 16, 4, 128, "spiking", 2)
    torch_glmulti_function(None, 8, 4, 64, "steady", 3)
    torch_aligned(None, 16, 4, 128, "spiking", 4)
    torch_aligned(None, 8, 4, 64, "steady", 5)
    kernel_fixtures(16, 256, 7)
    history_fixtures(16, 4, 32, 11)
    fagl1_neuron_fixture()
    weight_tables()


if __name__ == "__main__":
    main()
