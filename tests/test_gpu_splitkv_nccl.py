"""Split-KV decode over NCCL on 2 GPUs (skipped when fewer are visible).

Each rank holds a contiguous block range of one INT5 GQA 64:8 sequence (the last
rank also holds the tail), runs the fused attention locally, all-gathers the
(o, lse) partials and merges them; rank 0 compares with one-pass attention over
the whole sequence on its GPU.  The exchange over peer memory
(nsnkv_peer_merge_records) must give the same bits, eagerly and from CUDA-graph
replays.  NVLink multicast stays off (NCCL_NVLS_ENABLE=0; the peer kernel uses
plain stores).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q_out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from nsn_b200 import codec, kernel, workloads
        from nsn_b200.splitkv import ShardedSequence, shard_range
        from oracle import nsn_oracle as O
        gen = torch.Generator(device="cuda").manual_seed(44)
        h, hq, nb, t = 8, 64, 23, 64
        T = nb * 64 + t
        k = workloads.torch_kv(gen, (1, h, T, 128), workloads.K_OUTLIERS_8, 0.5)
        v = workloads.torch_kv(gen, (1, h, T, 128), (), 1.0)
        q = (torch.randn((1, hq, 1, 128), generator=gen, device="cuda") / np.sqrt(128)).half()
        g = codec.encode_group(k[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0, bits=5)
        vg = codec.encode_group(v[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0, bits=5)
        s, e = shard_range(nb, world, rank)
        last = rank == world - 1
        sub = lambda gr: dict(codes=gr["codes"][:, :, s:e].contiguous(),
                              metas=tuple(m[:, :, s:e].contiguous() for m in gr["metas"]))
        kt, vt = k[:, :, nb * 64:].contiguous(), v[:, :, nb * 64:].contiguous()
        sh = ShardedSequence(sub(g), sub(vg), kt if last else None, vt if last else None, h, hq, 5)
        out = sh.decode(q)
        torch.cuda.synchronize()
        sh.check()
        # the exchange over peer memory merges to the same bits, eagerly and in graph replays
        from nsn_b200.splitkv import PeerRecords
        peer = PeerRecords(hq)
        same = True
        for _ in range(3):
            same &= torch.equal(sh.decode(q, peer=peer).view(torch.int16), out.view(torch.int16))
        static = torch.empty_like(out)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            sh.decode(q, out=static, peer=peer)
        for _ in range(3):
            static.zero_()
            graph.replay()
            torch.cuda.synchronize()
            same &= torch.equal(static.view(torch.int16), out.view(torch.int16))
        del graph
        sh.check()
        if rank == 0:
            one = kernel.pipeline("GQA_FUSED", (g, kt, q, vg, vt)).float().reshape(hq, 128)
            ok, err = O.within_tolerance(out.float().cpu().numpy(), one.cpu().numpy(), *O.TOLERANCE["float16"])
            q_out.put(("ok" if ok and same else "mismatch", (err, same)))
        else:
            q_out.put(("ok" if same else "mismatch", same))
    except Exception as ex:
        q_out.put(("error", repr(ex)[:300]))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_split_kv_over_nccl_two_gpus():
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
    for kind, val in res:
        assert kind == "ok", val


def _single_rank(q_out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_port())
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", 0))
    try:
        from nsn_b200 import _lib as L
        from nsn_b200.splitkv import PeerRecords, merge_records
        hq = 64
        gen = torch.Generator(device="cuda").manual_seed(9)
        peer = PeerRecords(hq)
        status = L.status_tensor(torch.device("cuda", 0))
        same = True
        for _ in range(4):  # the epochs advance: every call waits on its own fresh flags
            rec = torch.randn(hq * 129, generator=gen, device="cuda")
            got = peer.merge(rec, torch.empty((hq, 128), dtype=torch.float16, device="cuda"), status)
            want, _ = merge_records(rec, 1, hq, dtype=torch.float16)
            same &= torch.equal(got.view(torch.int16), want.view(torch.int16))
        torch.cuda.synchronize()
        q_out.put(("ok" if same and int(status.item()) == 0 else "mismatch", int(status.item())))
    except Exception as ex:
        q_out.put(("error", repr(ex)[:300]))
    finally:
        dist.destroy_process_group()


def test_peer_merge_single_rank():
    """One rank: the kernel pushes into its own area, finds its own flag and merges as
    nsnkv_merge_shard_records does."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_single_rank, args=(q,))
    p.start()
    kind, val = q.get(timeout=300)
    p.join(timeout=120)
    assert kind == "ok", val
