"""Sequence-split (split-KV) decode across GPUs with a log-sum-exp merge.

For one long sequence (cfg4: 2047 INT5 blocks + 64-token tail, GQA 64:8), rank r
of N holds a contiguous range of sealed blocks (the last rank also holds the
native tail).  Each rank runs the fused attention over its range, writing the
fp32 context and the log-sum-exp of its scores per query head straight into one
send record [o (hq x 128) | lse (hq)]; one all-gather (NCCL over NVLink /
NVSwitch, about 33 KB per rank at cfg4) collects the records and
``nsnkv_merge_shard_records`` combines them in place:

    L = log sum_r exp(lse_r),  out = sum_r exp(lse_r - L) * o_r.

This is the reference's intra-GPU tile merge (experiments/ac08/source/
loop_kv_af01_kernel.py:70-84) lifted across GPUs.  The data path has no other
exchange; no TMA load ever reads another GPU's memory.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import primitives as w
from .kernel import decode_attention, group_pool


def shard_range(n_blocks: int, world: int, rank: int):
    """Contiguous, balanced block range [start, end) of `rank` (every rank gets >= 1 block if n_blocks >= world)."""
    base, extra = divmod(n_blocks, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_partials(o: torch.Tensor, lse: torch.Tensor, group=None):
    """All-gather per-rank (o [rows,128] fp32, lse [rows] fp32) -> ([N,rows,128], [N,rows])."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    o = o.contiguous()
    lse = lse.contiguous()
    # concatenated along dim 0 (the layout every backend accepts), viewed as [N, rows, ...]
    O = torch.empty((world * o.shape[0],) + tuple(o.shape[1:]), dtype=o.dtype, device=o.device)
    S = torch.empty((world * lse.shape[0],), dtype=lse.dtype, device=lse.device)
    dist.all_gather_into_tensor(O, o, group=group)
    dist.all_gather_into_tensor(S, lse, group=group)
    return O.view((world,) + tuple(o.shape)), S.view(world, lse.shape[0])


def merge_shards(O: torch.Tensor, S: torch.Tensor, dtype=torch.float16, out=None, out_f32=None, lse_out=None,
                 status=None):
    """Combine gathered partials on the GPU with nsnkv_merge_shards."""
    L.require_cuda()
    n, rows = S.shape[0], S.shape[1]
    dev = O.device
    if out is None:
        out = torch.empty((rows, 128), dtype=dtype, device=dev)
    if status is None:
        status = L.status_tensor(dev)
    L.check(L.load().nsnkv_merge_shards(n, rows, L.ptr(O), L.ptr(S), L.DTYPE_CODE[dtype], L.ptr(out),
                                        L.ptr(out_f32), L.ptr(lse_out), L.ptr(status), L.stream_handle(dev)),
            "nsnkv_merge_shards")
    return out, status


def gather_records(rec: torch.Tensor, group=None, out=None):
    """All-gather one flat fp32 record per rank -> [N * len(rec)] (one collective)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world * rec.numel(),), dtype=rec.dtype, device=rec.device)
    dist.all_gather_into_tensor(out, rec, group=group)
    return out


def merge_records(records: torch.Tensor, n_shards: int, rows: int, dtype=torch.float16, out=None, status=None):
    """Combine gathered records (each [o rows x 128 | lse rows]) with nsnkv_merge_shard_records."""
    L.require_cuda()
    dev = records.device
    if out is None:
        out = torch.empty((rows, 128), dtype=dtype, device=dev)
    if status is None:
        status = L.status_tensor(dev)
    L.check(L.load().nsnkv_merge_shard_records(n_shards, rows, L.ptr(records), records.numel() // n_shards,
                                               L.DTYPE_CODE[dtype], L.ptr(out), None, None, L.ptr(status),
                                               L.stream_handle(dev)),
            "nsnkv_merge_shard_records")
    return out, status


class PeerRecords:
    """The (o, lse) record exchange over peer memory, fused with the merge
    (nsnkv_peer_merge_records): every rank maps every other rank's area (torch's
    symmetric memory), writes its record into all of them with NVLink stores and merges
    once the peers' records have landed in its own.  One kernel per step instead of an
    NCCL all-gather and a merge kernel; capturable in a CUDA graph (the epochs live on the
    device).  Every rank of ``group`` constructs it with the same hq, and then calls
    ``merge`` once per step."""

    def __init__(self, hq: int, group=None, device=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        self.group = group if group is not None else dist.group.WORLD
        self.world, self.rank, self.hq = dist.get_world_size(self.group), dist.get_rank(self.group), hq
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        words = L.load().nsnkv_peer_area_words(self.world, hq)
        if hasattr(symm, "enable_symm_mem_for_group"):
            symm.enable_symm_mem_for_group(self.group.group_name)
        self.area = symm.empty(words, dtype=torch.float32, device=dev)
        self.area.zero_()
        self.handle = symm.rendezvous(self.area, self.group)
        self.epochs = torch.zeros(hq, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(self.group)  # every area is zero before any rank pushes into it
        self.peers = self.handle.buffer_ptrs_dev

    def merge(self, record: torch.Tensor, out: torch.Tensor, status: torch.Tensor):
        """record [hq * 129] fp32 ([o | lse]) -> out [hq, 128] merged over the ranks."""
        rc = L.load().nsnkv_peer_merge_records(
            self.world, self.rank, self.hq, L.DTYPE_CODE[out.dtype], L.ptr(record), self.peers, L.ptr(self.area),
            L.ptr(self.epochs), L.ptr(out), None, None, L.ptr(status), L.stream_handle(out.device))
        L.check(rc, "nsnkv_peer_merge_records")
        return out


class ShardedSequence:
    """One rank's share of a long sequence: its block range of K/V (reference group
    layout [1, h, n_r, ...]) plus, on the last rank, the native tail."""

    def __init__(self, k_group, v_group, k_tail, v_tail, h, hq, bits, records=None):
        """records: attend over block records with per-token renorm factors on the
        tensor-core kernel (K rounded like the bridge, V exact; INT3 or INT5 with
        hq / h <= 8), which is the default where it applies; False keeps the groups and
        the restore kernel (K and V rounded like the bridge)."""
        self.kg, self.vg = k_group, v_group
        self.kt, self.vt = k_tail, v_tail
        self.h, self.hq, self.bits = h, hq, bits
        self.n = 0 if k_group is None else k_group["codes"].shape[2]
        self.t = 0 if k_tail is None else k_tail.shape[2]
        dev = (k_group["codes"] if k_group is not None else k_tail).device
        if records is None:
            records = bits in (3, 5) and hq // h <= 8
        self.kp = self.vp = None
        if self.n:
            if records:
                from .paged import group_record_pools
                self.records, self.kp, self.vp = group_record_pools(k_group, v_group, bits)
            else:
                self.kp, self.vp = group_pool(k_group, h), group_pool(v_group, h)
        # send record: o [hq, 128] then lse [hq], written in place by the attention kernel
        self.rec = torch.empty((hq * 129,), dtype=torch.float32, device=dev)
        self.o = self.rec[:hq * 128].view(hq, 128)
        self.lse = self.rec[hq * 128:]
        self.recv = None
        self.lout = torch.empty((1, hq, 128), dtype=(k_tail.dtype if k_tail is not None else torch.float16),
                                device=dev)
        self.status = L.status_tensor(dev)

    def local(self, q, out=None):
        """Fused attention over this rank's share -> fp32 (o, lse) per query head."""
        if out is None:
            out = self.lout if self.lout.dtype == q.dtype else torch.empty((1, self.hq, 128), dtype=q.dtype,
                                                                           device=q.device)
        decode_attention(q.reshape(1, self.hq, 128), self.kp, self.vp, h=self.h, bits=self.bits,
                         blk_stride_head=self.n, blk_stride_page=1, n_blocks=self.n, max_blocks=self.n,
                         k_tail=self.kt if self.t else None, v_tail=self.vt if self.t else None,
                         tail_stride_seq=self.h * self.t, tail_stride_head=self.t, tail_len=self.t, max_tail=self.t,
                         out=out, out_f32=self.o.reshape(1, self.hq, 128), lse=self.lse.reshape(1, self.hq),
                         status=self.status)
        return self.o, self.lse

    def decode(self, q, group=None, out=None, peer=None):
        """Split-KV decode of q [1, hq, 1, 128]: local partials, then the exchange and merge:
        over peer memory when ``peer`` (a PeerRecords of the group) is given, else one NCCL
        all-gather and nsnkv_merge_shard_records.

        Without an initialised process group (or with one rank) the local pass
        already covers the whole sequence and its output is returned as is."""
        import torch.distributed as dist
        if not dist.is_initialized() or dist.get_world_size(group) == 1:
            res = torch.empty((self.hq, 128), dtype=q.dtype, device=q.device) if out is None else out
            self.local(q, out=res.view(1, self.hq, 128))
            return res
        self.local(q)
        if peer is not None:
            res = torch.empty((self.hq, 128), dtype=q.dtype, device=q.device) if out is None else out
            return peer.merge(self.rec, res, self.status)
        world = dist.get_world_size(group)
        if self.recv is None or self.recv.numel() != world * self.rec.numel():
            self.recv = torch.empty((world * self.rec.numel(),), dtype=torch.float32, device=self.rec.device)
        gather_records(self.rec, group, out=self.recv)
        res, _ = merge_records(self.recv, world, self.hq, dtype=q.dtype, out=out, status=self.status)
        return res

    def check(self):
        st = int(self.status.item())
        if st:
            w._status_to_error(st, "Nonfinite decode input", output_msg="Nonfinite decode output")
