"""Benchmark: batched packed-KV decode on B200 (cfg2 of the NSN packed-KV path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nsn|reference] [--batch B]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one rank per GPU)

Workload (cfg2, seed 2): batch 64 sequences, 32 query heads / 8 kv heads, head
dim 128; per-sequence context = U{32..256} sealed INT3 64-token blocks + a tail
of U[0,63] fp16 tokens.  One step = for every sequence append one new K/V token,
attend with one query over sealed blocks + tail (fused packed-KV decode
attention), and seal+encode every tail that reached 64 tokens.  Sequences are
sharded across ranks (greedy by packed bytes), no collective on the data path.
Synthetic data (seeded torch generator per sequence, the specification's
distributions); the reference measures on captured model K/V that is not
available here.

Prints one JSON line on rank 0.  `value` = decoded tokens/s of the whole job
(batch / max-over-ranks device time per step), K steps back to back between one
pair of CUDA events.  Inputs larger than L2 instead of a flush: the timed steps
rotate over as many caches of the rank's sequences as make two L2 sizes of
blocks (one at 64 sequences, five at 8), so every step reads its blocks from HBM.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HBM_FALLBACK = 6650.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return HBM_FALLBACK, "fallback"


# Algorithmic bytes of the hot path (per decode call): per (sequence, kv head) each sealed
# INT3 K or V block is 3072 code bytes + 128 norm + 512 min / scale = 3712 B (headers are
# never read), each native tail token 256 B for K and for V, q and out 256 B per query
# head.  The tensor-core kernels read fp32 renorm factors (256 B per block) in place of
# the fp16 norms (128 B): 128 B per K or V block of the kernel's own overhead.
BLOCK_BYTES = 3712
FACTOR_OVERHEAD = 128


# ------------------------------------------------------------------ clocks sampling
class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region (every 200 ms)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ workload
def shard_sequences(blocks, tails, world, rank):
    """Greedy balance of sequences across ranks by packed bytes (largest first)."""
    order = sorted(range(len(blocks)), key=lambda i: -(int(blocks[i]) * 3712 + int(tails[i]) * 256))
    load = [0] * world
    owner = [0] * len(blocks)
    for i in order:
        r = min(range(world), key=lambda x: load[x])
        owner[i] = r
        load[r] += int(blocks[i]) * 3712 + int(tails[i]) * 256
    return sorted(i for i in range(len(blocks)) if owner[i] == rank)


def build_cache(seqs, blocks, tails, steps, device, hq=32, h=8, rounding="exact"):
    from nsn_b200 import workloads
    from nsn_b200.paged import PagedKVCache
    c = workloads.CONFIGS[2]
    max_blocks = int(max(blocks[i] for i in seqs)) + (steps + 64) // 64 + 2
    cache = PagedKVCache(len(seqs), h, max_blocks, bits=3, dtype=torch.float16, device=device, hq=hq,
                         restore_rounding=rounding)
    for j, i in enumerate(seqs):
        T = int(blocks[i]) * 64 + int(tails[i])
        gen = torch.Generator(device=device).manual_seed(c["seed"] * 100003 + i)
        k = workloads.torch_kv(gen, (h, T, 128), c["k_outliers"], 0.5, device=device)
        v = workloads.torch_kv(gen, (h, T, 128), (), c["v_sigma"], device=device)
        cache.prefill(j, k, v)
        del k, v
    torch.cuda.synchronize(device)
    cache.check()
    return cache


def step_inputs(n_seq, steps, device, hq=32, h=8, seed=2):
    gen = torch.Generator(device=device).manual_seed(seed * 7919 + 17)
    q = (torch.randn((steps, n_seq, hq, 128), generator=gen, device=device) / math.sqrt(128)).half()
    kn = (torch.randn((steps, n_seq, h, 128), generator=gen, device=device)).half()
    vn = (torch.randn((steps, n_seq, h, 128), generator=gen, device=device)).half()
    return q, kn, vn


# ------------------------------------------------------------------ CPU baseline (reference bridge port)
def bridge_sample(n_seq=4, device="cpu"):
    """Four cfg2 sequences for the CPU bridge (the 1/8, 3/8, 5/8 and 7/8 quantiles of the
    batch's lengths, mean close to the batch mean), encoded with the port's own encoder.
    Returns (sequences, description)."""
    from oracle import bridge_torch as B
    from nsn_b200 import workloads
    c = workloads.CONFIGS[2]
    blocks, tails = workloads.np_cfg2_lengths()
    order = sorted(range(len(blocks)), key=lambda i: (int(blocks[i]), i))
    picks = [order[int(len(order) * (2 * j + 1) / (2 * n_seq))] for j in range(n_seq)]
    seqs = []
    for i in picks:
        nb, t = int(blocks[i]), int(tails[i])
        gen = torch.Generator(device=device).manual_seed(c["seed"] * 100003 + i)
        k = workloads.torch_kv(gen, (1, 8, nb * 64 + t, 128), c["k_outliers"], 0.5, device=device)
        v = workloads.torch_kv(gen, (1, 8, nb * 64 + t, 128), (), c["v_sigma"], device=device)
        kc, km = B.encode_group(k[:, :, :nb * 64].reshape(1, 8, nb, 64, 128))
        vc, vm = B.encode_group(v[:, :, :nb * 64].reshape(1, 8, nb, 64, 128))
        seqs.append(B.BridgeSequence(kc, km, k[:, :, nb * 64:].contiguous(), vc, vm, v[:, :, nb * 64:].contiguous()))
    desc = (f"cfg2 sequences {picks} ({', '.join(str(int(blocks[i])) for i in picks)} sealed blocks; batch mean "
            f"{float(blocks.mean()):.1f}), one sequence per step in turn")
    return seqs, desc


def bridge_steps(seqs, n_steps, seed=11):
    """Run n_steps single-sequence decode steps (round robin over seqs); returns seconds per step."""
    gen = torch.Generator().manual_seed(seed)
    times = []
    for i in range(n_steps):
        q = (torch.randn((1, 32, 1, 128), generator=gen) / math.sqrt(128)).half()
        kn = torch.randn((1, 8, 1, 128), generator=gen).half()
        vn = torch.randn((1, 8, 1, 128), generator=gen).half()
        t0 = time.perf_counter()
        seqs[i % len(seqs)].step(q, kn, vn)
        times.append(time.perf_counter() - t0)
    return times


def cpu_bridge_rate(budget_s=12.0):
    """The cpu_baseline record: the reference's CPU bridge (torch port, all host threads)
    on a bounded sample of cfg2 decode steps."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    seqs, desc = bridge_sample()
    bridge_steps(seqs, len(seqs))  # warm-up
    n, t0, times = 0, time.perf_counter(), []
    while (time.perf_counter() - t0 < budget_s or n < 8) and n < 400:
        times += bridge_steps(seqs, len(seqs), seed=100 + n)
        n += len(seqs)
    ms = 1000.0 * sum(times) / len(times)
    return {"value": 1000.0 / ms, "unit": "tokens/s", "cores": threads, "kind": "port",
            "ms_per_sample_step": ms, "timed_s": sum(times),
            "sample": f"reference CPU bridge (oracle/bridge_torch port: append by torch.cat, restore_group fp16 + "
                      f"cat + repeat_kv + SDPA, seal-at-64 by encode_group + torch.cat) over {len(times)} "
                      f"single-sequence decode steps of {desc}; torch threads={threads}"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU bridge on the host cores, rank 0 only.

    A step is one decode step of one sequence from a fixed sample of four cfg2 sequences
    (append, bridge attention, seal at 64), taken in turn; W untimed steps, then K timed
    steps.  value = decoded tokens/s = 1 / mean step time, the rate the CPU path would
    sustain over the whole batch (it decodes one sequence at a time);
    ms_per_step * steps is the timed region."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    seqs, desc = bridge_sample()
    bridge_steps(seqs, max(args.warmup, 1), seed=1)
    times = bridge_steps(seqs, args.steps, seed=2)
    ms = 1000.0 * sum(times) / len(times)
    v = 1000.0 / ms
    line = {"metric": "decode tokens/s (batched packed-KV decode, cfg2)", "value": v, "unit": "tokens/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "cfg2-batched-64 decode step (append + bridge attention + seal at 64) on the CPU: "
                                   "restore_group + cat + repeat_kv + SDPA per sequence",
                       "batch": 64, "hq": 32, "h": 8, "bits": 3,
                       "step": "one sequence's decode step (a bounded sample of the batched step)",
                       "timed_region_s": sum(times), "sample": desc},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} single-sequence decode steps of {desc}"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ cfg4: sequence-split decode + full-context encode
def run_cfg1(args, rank, world, local, dist):
    """cfg1: one sequence of 511 INT3 blocks + a 64-token fp16 tail, GQA 32:8 (rank 0 only).

    Times one decode-attention call two ways: replays of a CUDA graph of 100 calls (the
    reference's method; the 30.6 MB working set then stays in the 126 MB L2), and single
    calls with L2 flushed before each, on the same blocks: the paged cache's default
    (nsnkv_decode_attn_alpha over block records, K rounded like the bridge), its exact mode,
    and the restore path (nsnkv_decode_attn, the drop-in VF01 entry point with bridge
    rounding).  value: the default's latency with L2 flushed."""
    if rank != 0:
        return
    from nsn_b200 import primitives as P
    from nsn_b200 import workloads
    from nsn_b200.kernel import decode_attention
    from nsn_b200.paged import block_record_pools
    device = torch.device("cuda", local)
    c = workloads.CONFIGS[1]
    h, hq, nb, t = c["h"], c["hq"], c["blocks"], c["tail"]
    gen = torch.Generator(device=device).manual_seed(c["seed"] * 1000003)
    k = workloads.torch_kv(gen, (h, nb * 64 + t, 128), c["k_outliers"], 0.5, device=device)
    v = workloads.torch_kv(gen, (h, nb * 64 + t, 128), (), c["v_sigma"], device=device)
    q = (torch.randn((1, hq, 128), generator=gen, device=device) * c["q_scale"]).half()

    def pools_of(alpha):
        # the renorm-factor path in the paged cache's block-record layout, the restore path in dense arrays
        if alpha:
            _, kp_, vp_ = block_record_pools(h, nb, 3, device)
        else:
            kp_, vp_ = [dict(codes=torch.empty((h, nb, 3072), dtype=torch.uint8, device=device),
                             norm=torch.empty((h, nb, 64), dtype=torch.float16, device=device),
                             min=torch.empty((h, nb, 128), dtype=torch.float16, device=device),
                             scale=torch.empty((h, nb, 128), dtype=torch.float16, device=device)) for _ in range(2)]
        for x, pool in ((k, kp_), (v, vp_)):
            P.encode_blocks(x[:, :nb * 64].reshape(h, nb, 64, 128), 3, out=pool, out_row_stride=nb)
        return kp_, vp_

    kt = k[None, :, nb * 64:].contiguous()
    vt = v[None, :, nb * 64:].contiguous()
    out = torch.empty((1, hq, 128), dtype=torch.float16, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    lib = __import__("nsn_b200._lib", fromlist=["load"]).load()
    ws = torch.empty(lib.nsnkv_decode_attn_workspace_bytes(1, hq, h, nb, t), dtype=torch.uint8, device=device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    res = {}
    for name, alpha, exact in (("default_k_rounded", True, False), ("exact", True, True),
                               ("restore_path", False, False)):
        kp, vp = pools_of(alpha)

        def call():
            decode_attention(q, kp, vp, h=h, bits=3, blk_stride_head=nb, blk_stride_page=1, n_blocks=nb,
                             max_blocks=nb, k_tail=kt, v_tail=vt, tail_stride_seq=h * t, tail_stride_head=t,
                             tail_len=t, max_tail=t, out=out, status=status, ws=ws, exact=exact)

        for _ in range(5):
            call()
        torch.cuda.synchronize(device)
        P._status_to_error(int(status.item()), "Nonfinite cfg1 input", output_msg="Nonfinite cfg1 output")
        cold = []
        for _ in range(30):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            call()
            e1.record(stream)
            torch.cuda.synchronize(device)
            cold.append(e0.elapsed_time(e1) * 1000.0)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(100):
                call()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(device)
        warm = []
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(device)
            warm.append(e0.elapsed_time(e1) * 1000.0 / 100)
        del graph
        nbytes = h * nb * 2 * BLOCK_BYTES + h * t * 2 * 256 + 2 * hq * 256  # algorithmic bytes, every path
        cold.sort()
        warm.sort()
        res[name] = {"us_per_call_graph_replay": warm[len(warm) // 2], "us_per_call_l2_flushed": cold[len(cold) // 2],
                     "bytes_per_call": nbytes,
                     "gbs_l2_flushed": nbytes / (cold[len(cold) // 2] * 1e-6) / 1e9}
    hbm, peak_kind = peaks()
    for r in res.values():
        r["frac_l2_flushed"] = r["gbs_l2_flushed"] / hbm
    line = {"metric": "cfg1 single-sequence decode attention (511 INT3 blocks + 64 tail, GQA 32:8)",
            "unit": "us/call", "value": res["default_k_rounded"]["us_per_call_l2_flushed"],
            "higher_is_better": False, "n_gpus": 1, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "cfg1", "seed": c["seed"], "paths": res, "peak_gbs": hbm, "peak_kind": peak_kind,
                       "note": "graph replay keeps the 30.6 MB working set in L2; the flushed figure is the HBM one"}}
    print(json.dumps(line), flush=True)


def cfg4_measure(args, rank, world, local, dist, with_encode=True, steps=None, warmup=None):
    """cfg4 on `world` ranks: one 131072-token INT5 sequence (2047 blocks + 64 tail, GQA
    64:8), split by block ranges; optionally the timed full-context encode of each rank's
    blocks.  Every rank returns the same dict (times are maxima over ranks)."""
    from nsn_b200 import workloads
    from nsn_b200.splitkv import ShardedSequence, shard_range
    from nsn_b200 import primitives as P
    steps = args.steps if steps is None else steps
    warmup = args.warmup if warmup is None else warmup
    device = torch.device("cuda", local)
    c = workloads.CONFIGS[4]
    nb_total, h, hq, bits = c["blocks"], c["h"], c["hq"], c["bits"]
    s, e = shard_range(nb_total, world, rank)
    last = rank == world - 1
    n = e - s
    # 2048 blocks (2047 sealed + the tail) drawn in 32 chunks of 64 blocks, each from its
    # own seeded generator; shard boundaries at 1..8 ranks are chunk multiples, so every
    # world size sees the same data.
    CH = 64
    hi_blk = e + (1 if last else 0)
    ks, vs = [], []
    for ch in range(s // CH, (hi_blk + CH - 1) // CH):
        gen = torch.Generator(device=device).manual_seed(c["seed"] * 1000003 + ch)
        kc = workloads.torch_kv(gen, (h, CH * 64, 128), c["k_outliers"], 0.5, device=device)
        vc = workloads.torch_kv(gen, (h, CH * 64, 128), (), c["v_sigma"], device=device)
        a, b = max(s, ch * CH) - ch * CH, min(hi_blk, ch * CH + CH) - ch * CH
        ks.append(kc[:, a * 64:b * 64])
        vs.append(vc[:, a * 64:b * 64])
    kall, vall = torch.cat(ks, 1), torch.cat(vs, 1)
    del ks, vs
    k = kall[:, :n * 64].reshape(1, h, n, 64, 128).contiguous()
    v = vall[:, :n * 64].reshape(1, h, n, 64, 128).contiguous()
    kt = kall[None, :, n * 64:].contiguous() if last else None
    vt = vall[None, :, n * 64:].contiguous() if last else None
    del kall, vall
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def encode_kv():
        # the public encoder with its status check deferred, so no host sync splits K from V
        rk = P.encode_blocks(k, bits, packed=True, headers_start=s * 64, check=False)
        rv = P.encode_blocks(v, bits, packed=True, headers_start=s * 64, check=False)
        return rk, rv

    enc_ms = 0.0
    if with_encode:
        for _ in range(3):
            encode_kv()
        flush.zero_()
        torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
            torch.cuda.synchronize(device)  # the barrier's own device work stays outside the events
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        rk, rv = encode_kv()
        e1.record(stream)
        torch.cuda.synchronize(device)
        enc_ms = e0.elapsed_time(e1)
    else:
        rk, rv = encode_kv()
    for r_ in (rk, rv):
        P._status_to_error(int(r_["status"].item()), "Nonfinite input to NSN")
    g = dict(codes=rk["codes"], metas=tuple(rk["metas"]), headers=rk["headers"])
    vg = dict(codes=rv["codes"], metas=tuple(rv["metas"]), headers=rv["headers"])
    del k, v
    sh = ShardedSequence(g, vg, kt, vt, h, hq, bits)
    gen = torch.Generator(device=device).manual_seed(4 * 7919)
    qs = (torch.randn((warmup + steps, 1, hq, 1, 128), generator=gen, device=device) / math.sqrt(128)).half()
    # one decode step (local attention, one all-gather of the (o, lse) records, merge) is
    # captured once as a CUDA graph and replayed, so the step carries no host launch gaps
    static_q = qs[0].clone()
    static_out = torch.empty((hq, 128), dtype=torch.float16, device=device)
    for i in range(warmup):
        static_q.copy_(qs[i])
        sh.decode(static_q, out=static_out)
    torch.cuda.synchronize(device)
    sh.check()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        sh.decode(static_q, out=static_out)
    local_graph = torch.cuda.CUDAGraph()  # the same step's local attention alone
    with torch.cuda.graph(local_graph):
        sh.local(static_q)
    # the exchange over peer memory fused with the merge (more than one rank)
    peer, peer_graph, peer_note = None, None, None
    if dist is not None and world > 1:
        from nsn_b200.splitkv import PeerRecords
        try:
            peer = PeerRecords(hq)
        except Exception as ex:  # symmetric memory unavailable: the NCCL path only
            peer_note = f"peer exchange unavailable: {type(ex).__name__}"
        flag = torch.tensor([0 if peer is None else 1], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)  # every rank takes the same path
        if int(flag.item()) == 0:
            peer = None
        if peer is not None:
            # used only once it reproduces the NCCL path's bits with a clean status on every rank
            static_q.copy_(qs[0])
            want = sh.decode(static_q).clone()
            for i in range(warmup):
                static_q.copy_(qs[i])
                got = sh.decode(static_q, out=static_out, peer=peer)
            static_q.copy_(qs[0])
            got = sh.decode(static_q, out=static_out, peer=peer)
            torch.cuda.synchronize(device)
            good = torch.equal(got.view(torch.int16), want.view(torch.int16)) and int(sh.status.item()) == 0
            flag = torch.tensor([1 if good else 0], device=device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if int(flag.item()) == 0:
                peer, peer_note = None, "peer exchange disagreed with the NCCL path or timed out: not used"
                sh.status.zero_()
        if peer is not None:
            peer_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(peer_graph):
                sh.decode(static_q, out=static_out, peer=peer)
    torch.cuda.synchronize(device)

    def timed(gr, n_steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_steps)]
        for i in range(n_steps):
            flush.zero_()
            static_q.copy_(qs[warmup + i])
            if dist:
                dist.barrier()
                torch.cuda.synchronize(device)
            ev[i][0].record(stream)
            gr.replay()
            ev[i][1].record(stream)
        torch.cuda.synchronize(device)
        return sum(a.elapsed_time(b) for a, b in ev) / n_steps

    if dist:
        dist.barrier()
    with ClockSampler(local) as clk:
        nccl_ms = timed(graph, steps)
        local_ms = timed(local_graph, steps)
        peer_ms = timed(peer_graph, steps) if peer_graph is not None else 0.0
    sh.check()
    del graph, local_graph, peer_graph  # graphs holding NCCL work are released before the process group
    torch.cuda.synchronize(device)
    t = torch.tensor([nccl_ms, enc_ms, local_ms, peer_ms], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    nccl_ms, enc_ms_max, local_ms, peer_ms = t.tolist()
    # both exchanges give the same bits (the peer path is used only once it reproduced the
    # NCCL path's); the step is the faster of the two at this world size
    use_peer = 0 < peer_ms < nccl_ms
    step_ms = peer_ms if use_peer else nccl_ms
    exchange = ("peer memory (nsnkv_peer_merge_records: NVLink stores into every rank's symmetric area, fused "
                "with the merge)" if use_peer else "NCCL all-gather + nsnkv_merge_shard_records")
    total_bytes = 2 * 8 * (nb_total * 5760 + 64 * 256) + 2 * hq * 256
    total_enc_bytes = 2 * (nb_total * 8 * 64 * 128 * 2 + nb_total * 8 * 5760)
    hbm, peak_kind = peaks()
    return {"n_gpus": world, "step_ms": step_ms, "tokens_per_s": 1000.0 / step_ms,
            "exchange": exchange if world > 1 else "none (one rank)",
            "nccl_step_ms": nccl_ms if world > 1 else None, "peer_step_ms": peer_ms if peer_ms > 0 else None,
            "peer_note": peer_note,
            "local_attention_ms": local_ms, "gather_merge_ms": max(step_ms - local_ms, 0.0),
            "decode_gbs_whole_job": total_bytes / (step_ms / 1000.0) / 1e9,
            "frac_per_gpu": total_bytes / (step_ms / 1000.0) / 1e9 / world / hbm, "peak": hbm, "peak_kind": peak_kind,
            "bytes_per_step": total_bytes, "blocks_per_rank": n,
            "encode_ms": enc_ms_max if with_encode else None, "encode_bytes": total_enc_bytes,
            "clocks": clk.summary()}


def run_cfg4(args, rank, world, local, dist):
    """One 131072-token INT5 sequence (2047 blocks + 64 tail, GQA 64:8) split across ranks."""
    r = cfg4_measure(args, rank, world, local, dist, with_encode=True)
    if rank == 0:
        hbm = r["peak"]
        line = {"metric": "decode tokens/s (split-KV long-context decode, cfg4)", "value": r["tokens_per_s"],
                "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": r["step_ms"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "fp16", "data": "synthetic",
                "config": {"workload": "cfg4-long-131k-int5: 2047 INT5 blocks + 64 tail, GQA 64:8, split-KV "
                                       "(local fused attention + the (o, lse) record exchange and merge, "
                                       "replayed as a CUDA graph)",
                           "exchange": r["exchange"], "nccl_step_ms": r["nccl_step_ms"],
                           "global_batch": 1, "context": 131072, "parallelism": f"seq-split{world}",
                           "l2": "flushed before every timed step"},
                "decode_gbs_whole_job": r["decode_gbs_whole_job"],
                "local_attention_ms": r["local_attention_ms"], "gather_merge_ms": r["gather_merge_ms"],
                "encode": {"ms_max_over_ranks": r["encode_ms"], "bytes_total": r["encode_bytes"],
                           "gbs_whole_job": r["encode_bytes"] / (r["encode_ms"] / 1000.0) / 1e9,
                           "what": "nsnkv_encode_blocks of the 131008 sealed tokens (2047 blocks) x 8 kv heads, K "
                                   "and V (read fp16, write INT5 codes + fp16 metadata + headers), L2 flushed before"},
                "roofline": {"bound": "hbm", "peak": hbm, "peak_kind": r["peak_kind"], "unit": "GB/s",
                             "achieved": r["decode_gbs_whole_job"] / world, "frac": r["frac_per_gpu"],
                             "note": "per GPU: whole-job packed bytes / step time / GPUs"},
                "clocks": r["clocks"]}
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ cfg3: looped model, teacher-forced decode
def run_cfg3(args, rank, world, local, dist):
    """cfg3: a 24-layer looped decoder (hidden 2048, 16 MHA heads x 128, SwiGLU 5632, RoPE
    theta 1e4, vocab 32000, 4 loops sharing weights: 96 (loop, layer) INT3 KV slots),
    random-init fp16 weights.  4 sequences of 2048 random prompt ids, then teacher-forced
    decode steps; sequences are sharded over ranks (at most 4).

    Headline: nsn_b200.looped.PagedLoopedDecoder, the rank's sequences as one batch, one
    PagedKVCache per slot, the decode step replayed as a CUDA graph.  Timed: the decode
    steps back to back (prefill and capture outside the events; the 2.47 GB of weights each
    step streams four times exceed L2, so no flush).  Beside it: the same driver launching
    eagerly, and the reference's own per-sequence driver shape (connection cache per slot,
    one sequence at a time) with this library's fused kernels and with the bridge."""
    from transformers import LlamaConfig
    from nsn_b200 import adapter
    from nsn_b200.looped import PagedLoopedDecoder
    device = torch.device("cuda", local)
    cfg = LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632, num_hidden_layers=24,
                      num_attention_heads=16, num_key_value_heads=16, head_dim=128, max_position_embeddings=4096,
                      rope_theta=10000.0, attn_implementation="sdpa")
    torch.manual_seed(3)
    model = adapter.LoopedDecoder(cfg, loops=4).to(device).half().eval()
    n_seq, prompt_len, steps = 4, 2048, args.cfg3_steps
    mine = [i for i in range(n_seq) if i % world == rank]
    gen = torch.Generator(device="cpu").manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (n_seq, prompt_len + steps + 8), generator=gen)
    x = ids[mine].to(device)
    E = lambda: torch.cuda.Event(enable_timing=True)
    warm = 3

    def driver_run(graph):
        drv = PagedLoopedDecoder(model, len(mine), prompt_len + warm + steps)
        drv.prefill(x[:, :prompt_len])
        for t in range(warm):
            drv.step(x[:, prompt_len + t])
        if graph:
            drv.capture()
        torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        e0, e1 = E(), E()
        e0.record()
        for t in range(warm, warm + steps):
            (drv.replay if graph else drv.step)(x[:, prompt_len + t])
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / steps
        if graph:
            drv.sync_counters()
            drv.release()
        drv.check()
        kv = drv.kv_bytes()
        del drv
        torch.cuda.empty_cache()
        return ms, kv

    with ClockSampler(local) as clk:
        graph_ms, kv_bytes = driver_run(True)
    eager_ms, _ = driver_run(False)

    # the reference's per-sequence driver shape, a bounded number of steps per arm
    restore = adapter.install(model)
    Cache = adapter.make_cache()
    ref_steps = min(steps, 16)
    per_seq = {}
    for arm, checks in (("GQA_FUSED", "step"), ("TORCH_SDPA", "call")):
        total = 0.0
        for i in mine:
            cache = Cache(arm, 4, checks)
            xi = ids[i:i + 1].to(device)
            model(xi[:, :prompt_len], cache, 0)
            cache.post_prefill()
            torch.cuda.synchronize(device)
            e0, e1 = E(), E()
            e0.record()
            for t in range(ref_steps):
                model(xi[:, prompt_len + t:prompt_len + t + 1], cache, prompt_len + t)
                cache.post_decode()
            e1.record()
            torch.cuda.synchronize(device)
            total += e0.elapsed_time(e1) / ref_steps
            del cache
        per_seq[arm] = total  # ms per decode step of every rank sequence, one after another
    restore()
    t = torch.tensor([graph_ms, eager_ms, per_seq["GQA_FUSED"], per_seq["TORCH_SDPA"]], dtype=torch.float64,
                     device=device)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    graph_ms, eager_ms, ref_fused_ms, ref_bridge_ms = t.tolist()
    clocks = clk.summary()
    if rank == 0:
        tok_step = n_seq  # one token per sequence per step, all ranks together
        weights = sum(p.numel() * p.element_size() for p in model.parameters())
        line = {"metric": "decode tokens/s (looped model, cfg3)", "value": tok_step / (graph_ms / 1000.0),
                "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": graph_ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
                "data": "synthetic (random-init weights, random token ids)",
                "config": {"workload": "cfg3-looped-24x4: hidden 2048, 16 MHA heads x 128, SwiGLU 5632, vocab 32000, "
                                       "4 loops (96 INT3 KV slots), 4 seqs x 2048 prompt + teacher-forced decode",
                           "global_batch": n_seq, "seqs_per_rank": len(mine), "parallelism": f"seq-shard{world}",
                           "driver": "nsn_b200.looped.PagedLoopedDecoder, decode step replayed as a CUDA graph",
                           "l2": "not flushed: each step streams the 2.47 GB of weights four times"},
                "weight_stream_floor_ms": 4 * weights / (peaks()[0] * 1e9) * 1000.0,
                "kv_bytes_per_rank": kv_bytes, "kv_fp16_bytes_per_rank": 96 * 2 * 16 * (prompt_len + warm + steps)
                * 128 * 2 * len(mine),
                "eager_driver": {"value": tok_step / (eager_ms / 1000.0), "unit": "tokens/s", "ms_per_step": eager_ms},
                "per_sequence_driver": {
                    "what": "the reference's driver shape: one sequence at a time through a connection cache per "
                            f"slot (adapter.install + make_cache), {ref_steps} steps per sequence",
                    "fused_kernels": {"value": tok_step / (ref_fused_ms / 1000.0), "unit": "tokens/s"},
                    "bridge": {"value": tok_step / (ref_bridge_ms / 1000.0), "unit": "tokens/s"}},
                "clocks": clocks}
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ main GPU arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="nsn", choices=["nsn", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--as-rank", default=None, metavar="R/N",
                    help="one GPU, one process: time rank R's share of an N-way run of the cfg2 batch (the "
                         "sequences shard_sequences gives that rank), to study a rank of a multi-GPU run alone")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cfg4", action="store_true", help="skip the cfg4 split-KV sub-record of the cfg2 line")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4],
                    help="2: batched decode (the default bench line); 3: looped model; 4: split-KV long context + encode")
    ap.add_argument("--cfg3-steps", type=int, default=256, help="teacher-forced decode steps per sequence (cfg3)")
    ap.add_argument("--restore-rounding", default="exact", choices=["exact", "k", "kv"],
                    help="PagedKVCache restore_rounding of the timed cache (cfg2): exact (the headline: exact fp32 "
                         "restore, the fastest kernel), k (the library default: K rounded like the bridge), kv "
                         "(restore kernel, K and V rounded)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # CPU only: rank 0 runs, the other ranks exit at once (no process group, no GPU work)
        run_reference(args, rank, world)
        return
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if args.config in (1, 3, 4):
        torch.cuda.set_device(local)
        {1: run_cfg1, 3: run_cfg3, 4: run_cfg4}[args.config](args, rank, world, local, dist)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from nsn_b200 import workloads
    from nsn_b200 import _lib as L
    blocks, tails = workloads.np_cfg2_lengths(args.batch)
    if args.as_rank:
        if world > 1:
            raise SystemExit("--as-rank runs one process")
        r_, n_ = (int(x) for x in args.as_rank.split("/"))
        seqs = shard_sequences(blocks, tails, n_, r_)
    else:
        seqs = shard_sequences(blocks, tails, world, rank)
    total_steps = args.warmup + args.steps + 16
    # (+ the end-to-end and latency steps below)
    cache = build_cache(seqs, blocks, tails, total_steps + 1 + 48, device, rounding=args.restore_rounding)
    lib = L.load()
    n_seq = len(seqs)
    tok_step = n_seq if args.as_rank else args.batch  # tokens one timed step decodes, whole job
    q, kn, vn = step_inputs(n_seq, total_steps + 1, device)
    stream = torch.cuda.current_stream(device)
    # The timed steps rotate over R caches holding the same sequences (built from the same
    # seeds), R the smallest count whose bytes reach two L2 sizes: between two steps on one
    # cache at least two L2 sizes of other blocks stream in, so every step reads its blocks
    # from HBM without an L2 flush between steps (at 64 sequences R = 1).
    rot_bytes = int((2 * 8 * (cache.host_blocks.astype(np.int64) * BLOCK_BYTES
                              + (cache.host_tail.astype(np.int64) + 1) * 256)).sum())
    l2 = getattr(torch.cuda.get_device_properties(device), "L2_cache_size", 0) or (126 << 20)
    n_rot = max(1, -(-2 * l2 // max(rot_bytes, 1)))
    rot = [cache] + [build_cache(seqs, blocks, tails, total_steps + 1 + 48, device, rounding=args.restore_rounding)
                     for _ in range(n_rot - 1)]

    for i in range(max(args.warmup, n_rot)):
        rot[i % n_rot].step(q[i % args.warmup], kn[i % args.warmup], vn[i % args.warmup])
    torch.cuda.synchronize(device)
    for c in rot:
        c.check()

    E = lambda: torch.cuda.Event(enable_timing=True)
    launches = 0
    if dist:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clk:
        # the timed steps: back to back, rotating over the caches, one event pair around all
        t0, t1 = E(), E()
        t0.record(stream)
        for i in range(args.steps):
            s = args.warmup + i
            c = rot[i % n_rot]
            c.step(q[s], kn[s], vn[s])
            launches += lib.nsnkv_paged_plan_last_launches(c._plan)
        t1.record(stream)
        torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    for c in rot:
        c.check()
    mean_step = t0.elapsed_time(t1) / args.steps
    # ---- attention alone, the roofline's kernel time: one decode call's chain of launches
    # (chunk grid, tail grid, merge unless fused) with the appended token, as inside a step but
    # without the seal, back to back in a CUDA graph that rotates over the caches as the timed
    # steps do (every call reads its blocks from HBM), replayed between one event pair.  The
    # calls advance no counter: each writes its cache's next tail row, which the next step
    # overwrites.  Algorithmic bytes per call from each cache's host counters.
    from nsn_b200.kernel import decode_attention
    from nsn_b200 import primitives as P
    n_calls = n_rot * max(1, -(-16 // n_rot))
    s_attn = args.warmup + args.steps

    def graph_ms(call):
        for i in range(3):
            call(rot[i % n_rot], s_attn + i)
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n_calls):
                call(rot[i % n_rot], s_attn + i % 16)
        g.replay()
        torch.cuda.synchronize(device)
        a0, a1 = E(), E()
        a0.record(stream)
        g.replay()
        a1.record(stream)
        torch.cuda.synchronize(device)
        del g
        for c in rot:
            c.check()
        return a0.elapsed_time(a1) / n_calls

    def call_bytes(c):
        nb = c.host_blocks.astype(np.int64)
        tl = c.host_tail.astype(np.int64) + 1
        algo = int((2 * 8 * (nb * BLOCK_BYTES + tl * 256)).sum() + 2 * n_seq * 32 * 256)
        over = int((2 * 8 * nb).sum()) * FACTOR_OVERHEAD if c.uses_alpha_path() else 0
        return algo, over

    mean_attn = graph_ms(lambda c, s: c.attend(q[s], kn[s], vn[s]))
    bytes_attn = sum(call_bytes(rot[i % n_rot])[0] for i in range(n_calls)) / n_calls
    bytes_over = sum(call_bytes(rot[i % n_rot])[1] for i in range(n_calls)) / n_calls
    t = torch.tensor([mean_step, mean_attn], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    mean_step, mean_attn_max = t.tolist()

    # ---- both tensor-core kernels on the same blocks, timed as above: the library default
    # (K rounded like the bridge) and the exact restore
    kernels = None
    if cache.uses_alpha_path() and cache.hq // cache.h <= 4:
        def via(ex):
            def call(c, s):
                decode_attention(q[s], c.k_pool, c.v_pool, h=c.h, bits=3, blk_stride_head=c.pages, blk_stride_page=1,
                                 n_blocks=c.n_blocks, max_blocks=c.max_blocks, k_tail=c.k_tail, v_tail=c.v_tail,
                                 tail_stride_seq=c.h * P.BLOCK, tail_stride_head=P.BLOCK, tail_len=c.tail_len,
                                 max_tail=P.BLOCK - 1, block_table=c.block_table, k_new=kn[s], v_new=vn[s],
                                 out=c.out, status=c.status, ws=c.ws, blk_bytes=c.blk_bytes, exact=ex,
                                 blocks_total=int(c.host_blocks.sum()))
            return call

        res = {name: graph_ms(via(ex)) for name, ex in (("default", False), ("exact", True))}
        kernels = {"what": "attention (with the append, no seal), back to back in a CUDA graph rotating over the "
                           "timed caches, rank 0",
                   "default_k_rounded": {"attn_ms": res["default"],
                                         "frac": bytes_attn / (res["default"] / 1000.0) / 1e9 / peaks()[0],
                                         "contract": "K rounded to fp16 as restore_group rounds it, V exact: "
                                                     "within the parity bar of the reference bridge on every "
                                                     "input (golden cases incl. unscaled cfg0 queries)"},
                   "exact": {"attn_ms": res["exact"],
                             "frac": bytes_attn / (res["exact"] / 1000.0) / 1e9 / peaks()[0],
                             "contract": "exact fp32 restore of K and V: within the parity bar of the bridge "
                                         "on this workload's 1/sqrt(128)-scaled queries (full-size cfg2 test)"}}

    # ---- end to end through the public API with host buffers (pinned), rank-local
    e2e = None
    if True:
        # a step's q, k_new and v_new sit back to back in one pinned host buffer, and the output
        # returns to pinned host memory: PagedKVCache.step_host (nsnkv_paged_step_host), whose
        # plan stages them through two device slots on copy streams of its own, so the copies
        # of neighbouring steps overlap each step's kernels
        inh = torch.cat([q[:4].reshape(4, -1), kn[:4].reshape(4, -1), vn[:4].reshape(4, -1)], 1).cpu().pin_memory()
        outh = [torch.empty((n_seq, 32, 128), dtype=torch.float16).pin_memory() for _ in range(2)]
        fin = [E() for _ in rot]  # per cache: its last output copy
        e_steps = max(8, min(args.steps, 32))
        for i, c in enumerate(rot):  # untimed: each plan makes its staging at its first host step
            c.step_host(inh[i % 4], outh[0], done_event=fin[i])
        torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        e0, e1 = E(), E()
        e0.record(stream)
        for i in range(e_steps):
            rot[i % n_rot].step_host(inh[i % 4], outh[i % 2], done_event=fin[i % n_rot])
        for ev_ in fin:
            stream.wait_event(ev_)
        e1.record(stream)
        torch.cuda.synchronize(device)
        te = torch.tensor([e0.elapsed_time(e1) / e_steps], dtype=torch.float64, device=device)
        if dist:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = te.item()
        e2e = {"value": tok_step / (e2e_ms / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": int(inh[0].numel() * 2), "d2h_bytes_per_step": int(outh[0].numel() * 2),
               "ms_per_step": e2e_ms,
               "path": "PagedKVCache.step_host (nsnkv_paged_step_host, the C-ABI step with host buffers): pinned "
                       "host q|k_new|v_new in, output to pinned host memory, per rank; steps enqueued back to back "
                       "(throughput), the plan's copy streams overlapping neighbouring steps; rotating over the "
                       "same caches as the timed steps"}
        # latency: the same call with the host waiting for each step's output
        lat = []
        for i in range(min(args.steps, 16)):
            l0, l1 = E(), E()
            l0.record(stream)
            rot[i % n_rot].step_host(inh[i % 4], outh[0], done_event=l1)
            l1.synchronize()
            lat.append(l0.elapsed_time(l1))
        lat.sort()
        e2e["latency_ms_per_step"] = lat[len(lat) // 2]
        e2e["latency_what"] = ("median of device time from the call's entry on the stream to its output copy's end, "
                               "the host waiting for each step")
        for c in rot:
            c.check()

    hbm, peak_kind = peaks()
    achieved = bytes_attn / (mean_attn / 1000.0) / 1e9  # this rank
    clocks = clk.summary()

    # ---- cfg4 split-KV on the same ranks (every rank takes part in its all-gathers)
    cfg4 = None
    if not args.no_cfg4:
        del cache, rot, c, q, kn, vn
        torch.cuda.empty_cache()
        cfg4 = cfg4_measure(args, rank, world, local, dist, with_encode=False, steps=min(args.steps, 20), warmup=3)
        cfg4["what"] = ("cfg4 split-KV decode step: one 131072-token INT5 sequence (2047 blocks + 64 tail, GQA "
                        "64:8) split by block ranges over the ranks; local fused attention (attn_sealed_kernel "
                        "over INT5 block records, K rounded like the bridge) + the (o, lse) record exchange and "
                        "merge named by `exchange`, the faster of the two verified exchanges (nccl_step_ms: the NCCL "
                        "all-gather + merge kernel; peer_step_ms: the peer-memory exchange fused with the merge), "
                        "replayed as a CUDA graph, L2 flushed; gather_merge_ms = step - local attention alone "
                        "(max over ranks)")
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_bridge_rate()
        line = {
            "metric": "decode tokens/s (batched packed-KV decode, cfg2)",
            "value": tok_step / (mean_step / 1000.0),
            "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": mean_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "cfg2-batched-64: append 1 token + fused INT3 decode attention + seal, "
                                   "GQA 32:8, head_dim 128, ctx U{32..256} blocks + tail U[0,63], "
                                   f"q N(0,1)/sqrt(128); PagedKVCache restore_rounding={args.restore_rounding!r}",
                       "global_batch": args.batch, "hq": 32, "h": 8, "bits": 3, "parallelism": f"batch-shard{world}",
                       "l2": f"not flushed: inputs larger than L2; the timed steps rotate over {n_rot} cache(s) of "
                             f"the rank's sequences ({rot_bytes / 1e6:.1f} MB of blocks each), so at least two L2 "
                             "sizes of other blocks stream in between two steps on one cache",
                       "rotation_caches_rank0": n_rot,
                       "as_rank": args.as_rank,
                       "attn_bytes_per_step_rank0": bytes_attn, "attn_ms_rank0": mean_attn,
                       "attn_ms_max_over_ranks": mean_attn_max, "seqs_rank0": n_seq},
            "roofline": {"bound": "hbm",
                         "kernel": {"exact": "nsnkv_decode_attn_alpha with NSNKV_ATTN_EXACT (PagedKVCache "
                                             "restore_rounding='exact'): attn_sealed3_kernel + "
                                             "attn_native_rows_kernel on the tails + attn_merge_kernel",
                                    "k": "nsnkv_decode_attn_alpha, library default (PagedKVCache "
                                         "restore_rounding='k'): attn_sealed_kernel (K rounded like the bridge) "
                                         "+ attn_native_rows_kernel + attn_merge_kernel",
                                    "kv": "nsnkv_decode_attn (attn_partial_kernel + attn_merge_kernel)"}[
                                        args.restore_rounding],
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_kind": peak_kind, "traffic": None,
                         "time_what": f"mean device time of one attention call (with the append, no seal) over "
                                      f"{n_calls} calls back to back in a CUDA graph rotating over the timed caches, "
                                      "rank 0",
                         "traffic_note": "not captured in this run (ncu figures are in the committed profile summaries)",
                         "bytes_per_launch": bytes_attn,
                         "bytes_what": "algorithmic: 3712 B per sealed K or V block (codes + fp16 norm + min/scale), "
                                       "256 B per tail token of K and V (with the appended one), q and out",
                         "overhead_bytes": bytes_over,
                         "overhead_what": "the kernel's own extra reads: fp32 renorm factors (256 B) in place of the "
                                          "fp16 norms (128 B) per K or V block"},
            "restore_rounding": args.restore_rounding,
            "kernels": kernels,
            "e2e": e2e,
            # this library's kernels in the timed steps, as nsnkv_paged_plan_last_launches counted
            # them: attention (chunk grid, tail grid, merge unless fused) and the seal
            "gpu_launches": launches,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "cfg4_splitkv": cfg4,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
