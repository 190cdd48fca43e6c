"""The multi-GPU path on CPU: two gloo ranks, as bench.py --gpus 2 runs them.

Requests are sharded round-robin with no data-path collective; the only
cross-rank operations are the barrier and the max / sum over ranks of the
timed region. These tests run bench.py's own helpers in two processes and
check that the shards partition the batch exactly and that per-rank
attention (the CPU oracle standing in for each GPU's kernel) reassembles to
the single-process result.
"""

from __future__ import annotations

import importlib
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank: int, world: int, port: int, result_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, REPO)
    import torch.distributed as dist
    bench = importlib.import_module("bench")
    wl = importlib.import_module("llm-inference-runtime_b200.workloads")
    from oracle import attention
    r, w, _ = bench._dist()
    assert (r, w) == (rank, world)
    per_gpu = 6
    lengths_all = bench._global_lengths(per_gpu * w, 16, 300)
    mine = wl.round_robin(per_gpu * w, w, r)
    prob = wl.make_decode_problem(wl.TINYLLAMA, len(mine), 0, 0, seed=77, num_layers=1,
                                  lengths=lengths_all[mine], dtype=torch.float32)
    # every rank builds q for the whole batch from one seed and keeps its rows,
    # so the reassembled batch equals a single-process run
    q_all = torch.randn((per_gpu * w, 32, 64), generator=torch.Generator().manual_seed(5))
    q = q_all[torch.from_numpy(mine)]
    out, _ = attention.decode(q, prob.pool[0], prob.kv_indptr, prob.kv_indices,
                              prob.kv_last_page_len)
    # timed-region reductions as bench.py does them
    t_max = bench._max_over_ranks(float(rank + 1), w)
    t_sum = bench._sum_over_ranks(float(len(mine)), w)
    per_rank = bench._gather({"rank": r, "requests": len(mine)}, w)
    bench._barrier(w)
    gathered = [None] * w
    dist.all_gather_object(gathered, (mine.tolist(), out.numpy(), prob.pool[0].numpy(),
                                      prob.kv_indptr.tolist(), prob.kv_indices.tolist(),
                                      prob.kv_last_page_len.tolist()))
    if rank == 0:
        np.save(os.path.join(result_dir, "meta.npy"),
                np.array([t_max, t_sum, per_gpu * w], dtype=np.float64))
        assert per_rank == [{"rank": i, "requests": per_gpu} for i in range(w)]
        torch.save({"gathered": gathered, "q_all": q_all, "lengths": lengths_all},
                   os.path.join(result_dir, "gathered.pt"))
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_gloo_ranks_shard_requests_without_collective(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    t_max, t_sum, batch = np.load(tmp_path / "meta.npy")
    assert t_max == 2.0 and t_sum == batch
    data = torch.load(tmp_path / "gathered.pt", weights_only=False)
    owned = sorted(i for ids, *_ in data["gathered"] for i in ids)
    assert owned == list(range(int(batch)))          # every request exactly once
    from oracle import attention
    for ids, out, pool, indptr, indices, last in data["gathered"]:
        # each rank's result equals the oracle on that rank's own pool and tables
        q = data["q_all"][torch.tensor(ids)]
        want, _ = attention.decode(q, torch.from_numpy(pool), np.array(indptr),
                                   np.array(indices), np.array(last))
        assert torch.allclose(torch.from_numpy(out), want, atol=1e-6)
        # and its context lengths are the global draw's, for its own requests
        lens = [(indptr[b + 1] - indptr[b] - 1) * 16 + last[b] for b in range(len(ids))]
        assert lens == data["lengths"][ids].tolist()


@pytest.mark.timeout(300)
def test_reference_arm_runs_on_rank_zero_only(tmp_path):
    """bench.py --impl reference under two ranks: rank 0 prints the line,
    rank 1 exits without work (checked through the launcher's output)."""
    import subprocess
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(REPO, "bench.py"),
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=280, cwd=REPO, env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    import json
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["cpu_baseline"]["kind"] == "port"


def test_reference_arm_reports_the_same_config_as_this_package():
    """The reference arm's config object is built by the same function as
    this package's line for the workload, so the keys and the values that
    describe the workload agree."""
    bench = importlib.import_module("bench")
    wl, geom, per_gpu, lo, hi, layers, _ = bench._workload("cfg2")
    cfg = bench._config("cfg2", geom, layers, per_gpu, 1, lo, hi, "x")
    assert cfg["global_batch"] == 256 and cfg["requests_per_gpu"] == 256
    assert cfg["parallelism"] == "request-sharded x1, no collective"
    strong = bench._config("cfg5", wl.LLAMA3_8B, 1, 512, 8, 8192, 32768, "x", strong=True)
    assert strong["global_batch"] == 512 and strong["requests_per_gpu"] == 64
