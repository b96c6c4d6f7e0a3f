"""Host-side logic of the split-KV path on CPU ranks (gloo, world size 2).

The partial attention of each rank is computed by the fp64 oracle here (there is
no GPU); the product code under test is the partitioning (``shard_range``) and
the partial exchange (``gather_partials``), which the GPU path uses unchanged
with NCCL.  A second test injects a host-side failure: one rank raises before
the collective and the surviving rank's all-gather ends with an error after the
process group's short timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import nsn_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _partial(q, k, v):
    """fp64 oracle partial of one shard: (o [hq,128], lse [hq])."""
    out, lse = O.bridge_attention(q, k, v)
    return out[0], lse[0]


def _worker(rank, world, port, result_q, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        from nsn_b200.splitkv import gather_partials, shard_range
        rng = np.random.default_rng(3)
        h, hq, nb = 2, 8, 7
        k = rng.standard_normal((1, h, nb * 64, 128)).astype(np.float32)
        v = rng.standard_normal((1, h, nb * 64, 128)).astype(np.float32)
        q = (rng.standard_normal((1, hq, 1, 128)) / np.sqrt(128)).astype(np.float32)
        s, e = shard_range(nb, world, rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the exchange")
        o, lse = _partial(q, k[:, :, s * 64:e * 64], v[:, :, s * 64:e * 64])
        Og, Sg = gather_partials(torch.from_numpy(o.astype(np.float32)), torch.from_numpy(lse.astype(np.float32)))
        Sn = Sg.double().numpy()
        M = Sn.max(0)
        wts = np.exp(Sn - M)
        merged = (wts[..., None] * Og.double().numpy()).sum(0) / wts.sum(0)[..., None]
        full, _ = O.bridge_attention(q, k, v)
        result_q.put((rank, "ok", float(np.abs(merged - full[0]).max())))
    except Exception as ex:  # reported to the parent
        result_q.put((rank, "error", type(ex).__name__ + ": " + str(ex)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, fail_rank)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r, kind, val = q.get(timeout=120)
        out[r] = (kind, val)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_shard_range_partitions_blocks():
    from nsn_b200.splitkv import shard_range
    for n in (1, 2, 7, 2047):
        for world in (1, 2, 4, 8):
            ranges = [shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [e - s for s, e in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_gather_and_merge_world2():
    out = _run(fail_rank=-1)
    for r in (0, 1):
        kind, val = out[r]
        assert kind == "ok", val
        assert val < 1e-5  # partials travel as fp32


def test_injected_rank_failure_ends_with_error():
    out = _run(fail_rank=1)
    assert out[1][0] == "error" and "injected" in out[1][1]
    assert out[0][0] == "error", out[0]
