"""Multi-rank plumbing of the sequence-sharded path, on CPU with gloo
(world size 2): shards cover the batch exactly once, each rank's work is
independent (its own pool and tables), the max/sum reductions the bench uses
are correct, and a rank that leaves early makes the other rank's next
collective fail within the group timeout instead of hanging."""
from __future__ import annotations

import datetime
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _worker_shards(rank, world, port, out_dir):
    sys.path.insert(0, str(REPO))
    import importlib
    dist = _init(rank, world, port)
    W = importlib.import_module("distributed-llm-inference_b200.workloads")
    S = importlib.import_module("distributed-llm-inference_b200.sharding")
    from oracle import paged_attention as opa
    full = W.llama3_8b(batch=12, layers=1)
    shard = full.shard(rank, world, "contiguous")
    lo, hi = S.shard_bounds(full.batch, world, rank)
    assert shard.meta["shard"][3] == list(range(lo, hi))
    assert torch.equal(shard.lengths, full.lengths[lo:hi])
    t = W.materialize(shard, "cpu")
    out = opa.paged_attention(t.q[0], t.k_pools[0], t.v_pools[0], shard.tables, shard.lengths,
                              shard.max_length)
    local_sum = float(out.double().abs().sum())
    total = S.sum_over_ranks(local_sum)
    slowest = S.max_over_ranks(float(rank + 1))
    counts = S.sum_over_ranks(float(hi - lo))
    S.barrier()
    torch.save(dict(rank=rank, lo=lo, hi=hi, local=local_sum, total=total, slowest=slowest,
                    counts=counts), os.path.join(out_dir, f"rank{rank}.pt"))
    dist.destroy_process_group()


def _worker_leaves(rank, world, port, out_dir):
    sys.path.insert(0, str(REPO))
    import importlib
    dist = _init(rank, world, port, timeout_s=5)
    S = importlib.import_module("distributed-llm-inference_b200.sharding")
    S.barrier()
    if rank == 1:
        return  # leaves between steps, with no collective in flight
    err = ""
    try:
        S.max_over_ranks(1.0)
    except Exception as e:  # noqa: BLE001
        err = type(e).__name__ + ": " + str(e)[:200]
    torch.save(dict(err=err), os.path.join(out_dir, "rank0.pt"))


def _spawn(fn, tmp_path, world=2):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=fn, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    return procs


def test_sharded_ranks_cover_batch_and_reduce(tmp_path):
    procs = _spawn(_worker_shards, tmp_path)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [torch.load(tmp_path / f"rank{r}.pt") for r in range(2)]
    assert res[0]["lo"] == 0 and res[0]["hi"] == res[1]["lo"] and res[1]["hi"] == 12
    assert res[0]["counts"] == 12.0
    assert res[0]["slowest"] == res[1]["slowest"] == 2.0
    expect = res[0]["local"] + res[1]["local"]
    assert abs(res[0]["total"] - expect) < 1e-9 * max(1.0, expect)


def test_rank_leaving_fails_peer_collective(tmp_path):
    procs = _spawn(_worker_leaves, tmp_path)
    assert procs[1].exitcode == 0
    res = torch.load(tmp_path / "rank0.pt")
    assert res["err"], "the surviving rank's collective should fail, not hang"


def test_shard_bounds_even():
    sys.path.insert(0, str(REPO))
    import importlib
    S = importlib.import_module("distributed-llm-inference_b200.sharding")
    for B in (1, 7, 256):
        for P in (1, 2, 4, 8):
            spans = [S.shard_bounds(B, P, r) for r in range(P)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [h - l for l, h in spans]
            assert max(sizes) - min(sizes) <= 1


def test_balanced_assignment_equal_counts_and_tokens():
    sys.path.insert(0, str(REPO))
    import importlib
    S = importlib.import_module("distributed-llm-inference_b200.sharding")
    W = importlib.import_module("distributed-llm-inference_b200.workloads")
    lengths = W.llama3_8b().lengths
    for P in (1, 2, 4, 8):
        owned = S.balanced_assignment(lengths, P)
        flat = sorted(i for o in owned for i in o)
        assert flat == list(range(len(lengths)))             # every sequence exactly once
        assert {len(o) for o in owned} == set(S.shard_counts(len(lengths), P))
        loads = [int(lengths[o].sum()) for o in owned]
        assert max(loads) / (sum(loads) / P) < 1.01           # token-balanced
        contiguous = [int(lengths[S.shard_indices(lengths, P, r, "contiguous")].sum())
                      for r in range(P)]
        assert max(loads) <= max(contiguous)
    w = W.llama3_8b(batch=16, layers=1)
    shards = [w.shard(r, 4) for r in range(4)]
    assert sorted(i for sh in shards for i in sh.meta["shard"][3]) == list(range(16))
    for sh in shards:
        assert torch.equal(sh.lengths, w.lengths[torch.tensor(sh.meta["shard"][3])])
