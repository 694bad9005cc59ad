"""CUDA-graph capture of the native path.

One layer's forward + backward -- every scheme of the layer benchmark, the examples' aligned
layer and the history-table Functions -- is captured once into a CUDA graph (after eager
warm-up runs on a side stream) and replayed on new input values copied into the captured
inputs.  Each replay must equal an eager run on the same values bit for bit: every native
entry point takes its workspace from the caller, synchronizes nothing on the host and reads
no device value back, so the captured launches are the eager ones.  The profiling timer
counts the kernels the graph holds.
"""
import os
import sys

import pytest
import torch

from dfsnn_b200 import fde_kernels, profiling
from parity import assert_bitwise_gpu

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402  (the layer and table builders the benchmark captures)

pytestmark = pytest.mark.gpu

B, M = 4, 4096                    # 16,384 neurons


def capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with profiling.NativeCallTimer() as timer:
        with torch.cuda.graph(graph):
            out = fn()
    return graph, out, timer.captured_launches()


def replay_matches_eager(fn, inputs, g, what):
    graph, out, launches = capture(fn)
    assert launches >= 2, f"{what}: {launches} native kernels captured"
    for trial in range(2):
        for t in inputs:
            t.copy_(torch.randn(t.shape, device=t.device, generator=g) * (1 + trial))
        graph.replay()
        got = [o.clone() for o in out]
        want = fn()
        assert len(got) == len(want)
        for i, (a, b) in enumerate(zip(got, want)):
            assert_bitwise_gpu(a, b, what=f"{what} output {i} replay {trial}")
    del graph


@pytest.mark.parametrize("T", [8, 16])
@pytest.mark.parametrize("sch", ["glmulti", "gl", "trap", "predictor", "aligned"])
def test_layer_step_graph_replay_bitwise(T, sch):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    library = fde_kernels.LIFFDEGLMultiFunction
    try:
        layer = bench.make_layers(dev, [(T, sch)], B)[(T, sch)]
        single = sch not in ("glmulti", "aligned")
        g = torch.Generator(device=dev).manual_seed(5)
        x, gS, gV = (torch.randn((T, B, M), device=dev, generator=g) for _ in range(3))

        def fn():
            gx, s, pg = bench.layer_step(layer, x, gS, gV, single)
            return [gx, s] + list(pg) + ([layer.v_seq] if single else [])

        replay_matches_eager(fn, (x, gS, gV), g, f"{sch} T={T}")
    finally:
        fde_kernels.LIFFDEGLMultiFunction = library


@pytest.mark.parametrize("T", [8, 16])
@pytest.mark.parametrize("kind", ["vogl1", "fagl1", "vopred"])
def test_history_function_graph_replay_bitwise(T, kind):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    N = B * M
    g = torch.Generator(device=dev).manual_seed(6)
    x, gS = (torch.randn((T, N), device=dev, generator=g) for _ in range(2))
    v0 = torch.zeros(N, device=dev)
    sc, Wt = bench.history_tables(T, B, dev, g)[kind]
    sc = None if sc is None else sc.detach().requires_grad_(True)
    Wt = Wt.detach().requires_grad_(True)
    fk = fde_kernels

    def fn():
        xx = x.detach().requires_grad_(True)
        if kind == "vogl1":
            s = fk.LIFFDEVOGL1Function.apply(xx, v0, sc, Wt, bench.TAU, bench.TH, bench.SG, B, True)
            ins = [xx, sc, Wt]
        elif kind == "fagl1":
            s = fk.LIFFDEFAGL1Function.apply(xx, v0, Wt, bench.TAU, bench.H ** 0.5, bench.TH,
                                             bench.SG, B, True)
            ins = [xx, Wt]
        else:
            s = fk.LIFFDEVOPREDICTORFunction.apply(xx, v0, sc, Wt, bench.TAU, bench.TH, bench.SG,
                                                   0.25, B)
            ins = [xx, sc, Wt]
        return [s] + list(torch.autograd.grad([s], ins, [gS]))

    replay_matches_eager(fn, (x, gS), g, f"{kind} T={T}")
