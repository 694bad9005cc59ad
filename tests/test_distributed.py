"""Data-parallel host logic on CPU (gloo, world size 2): sharded neuron ranges cover the axis,
per-shard parameter gradients summed by one all-reduce equal the single-process result, and a
rank that fails before the collective makes its peer fail within the process-group timeout."""
import json
import os
import socket
import sys
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dfsnn_b200.distributed import allreduce_flat, init_process_group, neuron_shard

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_neuron_shard_covers_axis():
    for n in (0, 1, 7, 8388608, 1000003):
        for world in (1, 2, 3, 8):
            spans = [neuron_shard(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _worker_reduce(rank, world, port, out_path):
    sys.path[:0] = [REPO, os.path.join(REPO, "df-snn-official_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    from oracle import oracle as O
    init_process_group("gloo", timeout_s=30)
    T, N = 8, 5000
    g = np.random.default_rng(0)
    x = (g.standard_normal((T, N)) * 5).astype(np.float32)
    gS = g.standard_normal((T, N)).astype(np.float32)
    scale = np.full(T, 0.22385544, np.float32)
    W = np.tril(g.standard_normal((T, T)).astype(np.float32) * 0.05, -1)
    a, b = neuron_shard(N, rank, world)
    r = O.glmulti_step(x[:, a:b], np.zeros(b - a, np.float32), scale, W, gS[:, a:b], 2.0, 1.0,
                       5.0, True)
    gs = torch.tensor(r["gscale"], dtype=torch.float64)
    gw = torch.tensor(r["gW"], dtype=torch.float64)
    allreduce_flat([gs, gw])
    if rank == 0:
        full = O.glmulti_step(x, np.zeros(N, np.float32), scale, W, gS, 2.0, 1.0, 5.0, True)
        np.savez(out_path, gs=gs.numpy(), gw=gw.numpy(), gs_full=full["gscale"], gw_full=full["gW"])
    dist.destroy_process_group()


def test_sharded_reduction_equals_full(tmp_path):
    out = str(tmp_path / "r.npz")
    mp.start_processes(_worker_reduce, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    d = np.load(out)
    np.testing.assert_allclose(d["gs"], d["gs_full"], rtol=1e-12, atol=1e-9)
    np.testing.assert_allclose(d["gw"], d["gw_full"], rtol=1e-12, atol=1e-9)


def _worker_fail(rank, world, port, out_path):
    sys.path[:0] = [REPO, os.path.join(REPO, "df-snn-official_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    init_process_group("gloo", timeout_s=5)
    if rank == 1:
        raise SystemExit(3)              # leaves between steps, before the collective
    t0 = time.time()
    status = "completed"
    try:
        allreduce_flat([torch.ones(4)])
    except Exception as exc:             # the survivor learns of it through the collective
        status = type(exc).__name__
    with open(out_path, "w") as f:
        f.write(f"{status} {time.time() - t0:.1f}")


def test_failed_rank_is_detected_by_timeout(tmp_path):
    out = str(tmp_path / "status.txt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker_fail, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    deadline = time.time() + 90
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "survivor did not return within the bound"
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    status, secs = open(out).read().split()
    assert status != "completed"
    assert float(secs) < 60


def _worker_step_costs(rank, world, port, out_path):
    sys.path[:0] = [REPO, os.path.join(REPO, "df-snn-official_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    import bench
    init_process_group("gloo", timeout_s=30)
    bench.start_line(torch.device("cpu"), world)    # both ranks meet at the start line
    costs = bench.StepCosts()
    out = costs.summary(4, 1.0 + rank, torch.device("cpu"), world)
    no_exch = costs.summary(4, 5.0 - rank, torch.device("cpu"), world, exchange=False)
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump([out, no_exch], f)
    dist.destroy_process_group()


def test_bench_step_costs_max_over_ranks(tmp_path):
    """The bench's start line and per-step host and exchange costs: every rank takes part in
    the same collectives, and the costs are the maximum over ranks (gloo, world size 2)."""
    out = str(tmp_path / "c.txt")
    mp.start_processes(_worker_step_costs, args=(2, _free_port(), out), nprocs=2,
                       start_method="spawn")
    with open(out) as f:
        a, b = json.load(f)
    assert a == {"host_ms_per_step": 2.0, "exchange_ms_per_step": 0.0, "exchange_ms_longest": 0.0}
    assert b == {"host_ms_per_step": 5.0}


_FINISH_SCRIPT = """
import os, sys
sys.path[:0] = [{repo!r}, os.path.join({repo!r}, "df-snn-official_b200")]
import bench
from dfsnn_b200.distributed import init_process_group
init_process_group("gloo", timeout_s=30)
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
print(f"rank {{rank}} before", flush=True)
bench.finish_ranks({{"metric": "m", "value": 1.0, "n_gpus": world}}, rank, world)
print("never printed", flush=True)
"""


def test_bench_finish_ranks_prints_the_line_last(tmp_path):
    """Under torchrun (gloo, world size 2) every rank exits 0 and rank 0's JSON line is the
    last line of the run's stdout: nothing a rank prints at exit can follow it."""
    import json
    import subprocess
    script = tmp_path / "finish.py"
    script.write_text(_FINISH_SCRIPT.format(repo=REPO))
    proc = subprocess.run(
        [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
         "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script)],
        capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.strip()]
    assert json.loads(lines[-1]) == {"metric": "m", "value": 1.0, "n_gpus": 2}
    assert sum(l.startswith("{") for l in lines) == 1
    assert "never printed" not in proc.stdout
