"""Multi-rank host logic of the (batch, kv-head) sharding, on CPU gloo ranks.

Two processes each regenerate only their own slabs from per-slab seeds,
compute their shard (here with the CPU oracle; on GPUs bench.py calls the
CUDA op), and the all-gathered result must equal a single-process run over
the whole batch. Failure cases: a rank that dies before the gather, and ranks
with mismatched shard shapes, must surface as errors, not hangs.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import kv_oracle as O

shard = pytest.importorskip("llmik_cuda.shard")

HQ, HKV, D, S = 8, 4, 128, 96
SCALE = 1.0 / np.sqrt(D)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _slab(b, h, base=100):
    g = torch.Generator().manual_seed(shard.slab_seed(base, b, h, HKV))
    k = torch.randn(S, D, generator=g).half()
    v = torch.randn(S, D, generator=g).half()
    return k, v


def _q(b, base=7):
    g = torch.Generator().manual_seed(base + b)
    return torch.randn(HQ, D, generator=g).half()


def _shard_out(b0, b1):
    outs = []
    for b in range(b0, b1):
        kv = [_slab(b, h) for h in range(HKV)]
        k = torch.stack([x[0] for x in kv])[None]
        v = torch.stack([x[1] for x in kv])[None]
        outs.append(torch.from_numpy(O.decode_attention(_q(b)[None].numpy(), k.numpy(), v.numpy(), SCALE)))
    return torch.cat(outs)


def _worker(rank, world, port, batch, mode, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=6))
    status = "ok"
    try:
        if mode == "normal":
            b0, b1 = shard.batch_range(batch, world, rank)
            full = shard.gather_shards(_shard_out(b0, b1))
            t = shard.max_over_ranks(float(rank + 1))
            if rank == 0:
                torch.save({"full": full, "t": t}, os.path.join(result_dir, "r0.pt"))
        elif mode == "dead_rank":
            if rank == 1:
                os._exit(3)  # leaves between steps without joining the collective
            shard.gather_shards(torch.zeros(2, HQ, D))
            status = "no-error"
        elif mode == "mismatch":
            shard.gather_shards(torch.zeros(1 + rank, HQ, D))
            status = "no-error"
    except Exception as e:  # noqa: BLE001 - the test inspects the outcome
        status = "error: " + type(e).__name__
    with open(os.path.join(result_dir, f"status{rank}.txt"), "w") as f:
        f.write(status)
    try:
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        pass


def _run(world, batch, mode):
    d = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, PORTS[mode], batch, mode, d))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    return d


PORTS = {"normal": _free_port(), "dead_rank": _free_port(), "mismatch": _free_port()}


def test_unit_and_batch_ranges_partition():
    for n, w in ((512, 8), (64, 3), (7, 2), (1, 1)):
        spans = [shard.unit_range(n, w, r) for r in range(w)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert shard.batch_range(64, 8, 7) == (56, 64)
    with pytest.raises(ValueError):
        shard.batch_range(10, 4, 0)


def test_two_gloo_ranks_match_single_process():
    d = _run(2, 4, "normal")
    res = torch.load(os.path.join(d, "r0.pt"))
    ref = _shard_out(0, 4)
    assert torch.equal(res["full"], ref)
    assert res["t"] == 2.0   # max over ranks of (rank + 1)


def test_dead_rank_surfaces_as_error_not_hang():
    d = _run(2, 4, "dead_rank")
    with open(os.path.join(d, "status0.txt")) as f:
        assert f.read().startswith("error")


def test_mismatched_shards_are_rejected():
    d = _run(2, 4, "mismatch")
    for r in range(2):
        with open(os.path.join(d, f"status{r}.txt")) as f:
            assert f.read().startswith("error")
