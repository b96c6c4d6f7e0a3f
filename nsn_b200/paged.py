"""PagedKVCache: batched packed-KV cache for decode serving (append + attend + seal).

The reference grows each slot's packed groups with ``torch.cat`` on every seal
(experiments/nb06/source/loop_kv_nb06_packed.py:36-50, ``append_group``
loop_kv_nb06_codec.py:40-45), which re-copies the whole packed history and syncs
the host.  Here the packed blocks live in a fixed page pool addressed through a
block table, and one decode step (``step``) is one native call, nsnkv_paged_step,
over a plan made once per cache, with no host sync:

  1. nsnkv_decode_attn_alpha  appends the new K/V token to each sequence's fp16 tail
                         and attends over sealed blocks + tail (split-KV partials
                         + log-sum-exp merge);
  2. nsnkv_seal_full_tails_alpha  encodes every tail that reached 64 tokens into the
                         sequence's next page and advances n_blocks / tail_len;
  3. on the host, the plan advances this object's copies of those counters.

Policy: seal whenever a tail reaches 64 tokens, so tails hold 0..63 tokens
between steps (the benchmark specification's batched policy; the reference's
per-slot PackedCache keeps 64..127, see nsn_b200.packed).

Layout (head-major pools so one sequence's blocks of one head are contiguous):
  codes [h, pages, code_bytes] uint8, norm [h, pages, 64], min/scale [h, pages, 128] fp16,
  alpha [h, pages, 64] fp32: per-token renorm factors n / max(||d||, eps), written
  whenever a block is (sealed, prefilled or imported) so attention does not recompute
  ||d|| per step; derived data, not part of the reference's format or of the exports
  block (sequence b, head j, block i) = pool row j, page block_table[b, i]
  For caches on the tensor-core path (INT3, hq / h <= 8) codes / min / scale /
  alpha of K and then of V are fields of one block record per (head, page),
  records [h, pages, 7680] uint8, so the attention kernel moves a block with one copy;
  the pool dicts hold views of those fields (norms stay dense).
  block_table [batch, max_blocks] int32 (sequence b owns pages b*max_blocks ..)
  n_blocks, tail_len [batch] int32 (device), k_tail/v_tail [batch, h, 64, 128].
"""
from __future__ import annotations

import ctypes
import struct

import numpy as np
import torch

from . import _lib as L
from . import checks
from . import primitives as w
from .kernel import decode_attention

# ------------------------------------------------------------ sequence container format
# A sealed sequence as bytes, for moving it between caches or processes:
#   preamble  '<8sHHBBHII': magic, format version 1, kv heads h, bits, tail dtype
#             (0 fp16, 1 bf16), reserved 0, sealed blocks n, tail tokens t      (24 bytes)
#   K blocks  for head j, block i: the block's 12-byte '<QHBB' header (64*i, 64, bits, 0;
#             loop_kv_nb06_codec.py:32), codes (64*128*bits/8 bytes), norm (64 fp16),
#             min (128 fp16), scale (128 fp16)
#   V blocks  the same
#   tails     K [h, t, 128] then V [h, t, 128] in the tail dtype
# Everything after the preamble is what planned_bytes (loop_kv_nb06_primitives.py:72-81)
# counts for K and V.
SEQ_MAGIC = b"NSNKVSEQ"
_PREAMBLE = struct.Struct("<8sHHBBHII")
_TAIL_CODE = {torch.float16: 0, torch.bfloat16: 1}


def sequence_to_bytes(kg, kt, vg, vt) -> bytes:
    """Serialise a sequence given in the reference's layout (groups + tails [1, h, t, 128])."""
    h, t = kt.shape[1], kt.shape[2]
    n = 0 if kg is None else kg["codes"].shape[2]
    bits = 3 if kg is None else kg["codes"].shape[-1] * 8 // (w.BLOCK * w.DIM)
    w.require(kt.dtype in _TAIL_CODE and vt.shape == kt.shape and vt.dtype == kt.dtype, "Tail layout")
    parts = [_PREAMBLE.pack(SEQ_MAGIC, 1, h, bits, _TAIL_CODE[kt.dtype], 0, n, t)]
    for g in (kg, vg):
        if n == 0:
            continue
        w.require(g["codes"].shape[2] == n and checks.headers_ok(g), "Block headers")
        hdr = g["headers"].cpu().numpy().reshape(h, n, 12)
        codes = g["codes"].cpu().numpy().reshape(h, n, -1)
        metas = [m.cpu().contiguous().view(torch.int16).numpy().reshape(h, n, -1) for m in g["metas"]]
        for j in range(h):
            for i in range(n):
                parts += [hdr[j, i].tobytes(), codes[j, i].tobytes()] + [m[j, i].tobytes() for m in metas]
    for tail in (kt, vt):
        parts.append(tail.cpu().contiguous().view(torch.int16).numpy().tobytes())
    return b"".join(parts)


def sequence_from_bytes(blob: bytes, device="cpu"):
    """Parse sequence_to_bytes output back into (kg, kt, vg, vt) on `device`; headers are verified."""
    import numpy as np
    w.require(len(blob) >= _PREAMBLE.size, "Sequence container")
    magic, version, h, bits, tcode, reserved, n, t = _PREAMBLE.unpack_from(blob, 0)
    w.require(magic == SEQ_MAGIC and version == 1 and bits in (3, 4, 5) and tcode in (0, 1) and reserved == 0,
              "Sequence container")
    cb = w.code_bytes(bits)
    per_block = 12 + cb + 2 * (w.BLOCK + 2 * w.DIM)
    want = _PREAMBLE.size + 2 * h * n * per_block + 2 * h * t * w.DIM * 2
    w.require(len(blob) == want, "Sequence container length")
    buf = np.frombuffer(blob, np.uint8, offset=_PREAMBLE.size)
    dtype = torch.float16 if tcode == 0 else torch.bfloat16
    groups, off = [], 0
    for _ in range(2):
        if n == 0:
            groups.append(None)
            continue
        blk = buf[off:off + h * n * per_block].reshape(h, n, per_block)
        off += h * n * per_block
        f16 = lambda a, b_, shape: torch.from_numpy(blk[:, :, a:b_].copy().view(np.int16)).view(torch.float16) \
            .reshape(shape).to(device)
        g = dict(headers=torch.from_numpy(blk[:, :, :12].copy()).reshape(1, h, n, 12).to(device),
                 codes=torch.from_numpy(blk[:, :, 12:12 + cb].copy()).reshape(1, h, n, cb).to(device),
                 metas=(f16(12 + cb, 12 + cb + 2 * w.BLOCK, (1, h, n, w.BLOCK, 1)),
                        f16(12 + cb + 2 * w.BLOCK, 12 + cb + 2 * w.BLOCK + 2 * w.DIM, (1, h, n, 1, w.DIM)),
                        f16(12 + cb + 2 * w.BLOCK + 2 * w.DIM, per_block, (1, h, n, 1, w.DIM))))
        w.require(checks.headers_ok(g), "Block headers")
        groups.append(g)
    tails = []
    for _ in range(2):
        nbytes = h * t * w.DIM * 2
        tails.append(torch.from_numpy(buf[off:off + nbytes].copy().view(np.int16)).view(dtype)
                     .reshape(1, h, t, w.DIM).to(device))
        off += nbytes
    return groups[0], tails[0], groups[1], tails[1]


def block_record_pools(h: int, pages: int, bits: int, device):
    """Zeroed block records [h, pages, 2 * (code_bytes + 768)] uint8 and the K / V pool dicts.

    Record (head j, page p): K codes | K min (128 fp16) | K scale (128 fp16) | K alpha
    (64 fp32), then the same four fields for V (7680 bytes for INT3).  The pool dicts
    hold views of those fields, so every operator that takes a pool writes or reads the
    records; norms [h, pages, 64] fp16 stay dense.  nsnkv_decode_attn_alpha moves each
    block with one copy when given these pools (blk_bytes = the record size).  The K
    codes are paired halves and the V codes paired rows (``pool["code_order"]`` 2 and 1,
    see primitives.pair_halves / pair_rows): the orders the tensor-core kernel reads
    cheapest; exports and imports convert.
    """
    cb = w.code_bytes(bits)
    half = cb + 2 * w.DIM * 2 + w.BLOCK * 4
    rec = torch.zeros((h, pages, 2 * half), dtype=torch.uint8, device=device)

    def fields(off):
        return dict(codes=rec[..., off:off + cb],
                    norm=torch.zeros((h, pages, w.BLOCK), dtype=torch.float16, device=device),
                    min=rec[..., off + cb:off + cb + 2 * w.DIM].view(torch.float16),
                    scale=rec[..., off + cb + 2 * w.DIM:off + cb + 4 * w.DIM].view(torch.float16),
                    alpha=rec[..., off + cb + 4 * w.DIM:off + half].view(torch.float32))

    kp, vp = fields(0), fields(half)
    kp["code_order"] = 2  # K codes as paired halves (primitives.pair_halves)
    vp["code_order"] = 1  # V codes as paired rows (primitives.pair_rows)
    return rec, kp, vp


def group_record_pools(k_group, v_group, bits: int):
    """Block records (see block_record_pools) holding the blocks of reference-layout groups
    ([1, h, n, ...], as encode_group returns them): codes in the records' orders, fp16
    metadata, and the renorm factors computed from them.  Returns (records, k_pool, v_pool)
    with block (j, i) at row j, page i, for nsnkv_decode_attn_alpha's tensor-core kernels."""
    _, h, n, cb = k_group["codes"].shape
    w.require(cb == w.code_bytes(bits) and tuple(v_group["codes"].shape) == (1, h, n, cb), "group record shapes")
    records, kp, vp = block_record_pools(h, n, bits, k_group["codes"].device)
    for g, pool in ((k_group, kp), (v_group, vp)):
        pool["codes"].copy_(w.to_code_order(g["codes"][0], bits, pool["code_order"]))
        pool["norm"].copy_(g["metas"][0].reshape(h, n, w.BLOCK))
        pool["min"].copy_(g["metas"][1].reshape(h, n, w.DIM))
        pool["scale"].copy_(g["metas"][2].reshape(h, n, w.DIM))
        w.block_renorm(pool, bits, h, n, n)
    return records, kp, vp


ROUNDING_MODES = ("k", "kv", "exact")


class PagedKVCache:
    def __init__(self, batch: int, h: int, max_blocks: int, bits: int = 3, dtype=torch.float16, device="cuda",
                 hq: int | None = None, bridge_rounding: bool = False, restore_rounding: str | None = None):
        """How attention treats the restored rows (``restore_rounding``):

        ``"k"`` (default): K rows rounded to the cache dtype exactly as the reference
            bridge (restore_group(g, dtype) + SDPA) rounds them, V applied as the exact fp32
            restore.  INT3 and INT5 caches with hq / h <= 8 keep per-token renorm factors in
            block records and attend over them on the tensor cores; other shapes (INT4,
            hq / h > 8) use the restore kernel, which rounds K and V.
        ``"kv"`` (or ``bridge_rounding=True``): the restore kernel, K and V rounded as the
            bridge rounds them.
        ``"exact"``: K and V both the exact fp32 restore, nothing rounded (INT3 fp16
            caches with hq / h <= 4): the fastest kernel, a stricter contract than the
            bridge's, whose fp16 rounding of K moves outputs by up to a few 1e-3 when the
            queries are not scaled down.
        """
        w.require(batch > 0 and h > 0 and max_blocks > 0 and bits in (3, 4, 5), "paged cache shape")
        w.require(dtype in (torch.float16, torch.bfloat16), "paged cache dtype")
        mode = restore_rounding if restore_rounding is not None else ("kv" if bridge_rounding else "k")
        w.require(mode in ROUNDING_MODES, "paged cache restore_rounding")
        L.require_cuda()
        self.batch, self.h, self.max_blocks, self.bits, self.dtype = batch, h, max_blocks, bits, dtype
        self.hq = hq or h
        w.require(self.hq % h == 0 and self.hq // h <= 8, "paged cache head grouping")
        self.restore_rounding = mode
        self.bridge_rounding = mode == "kv"
        w.require(mode != "exact" or (bits == 3 and dtype == torch.float16 and self.hq // h <= 4),
                  "exact attention needs an INT3 fp16 cache with hq / h <= 4")
        self.device = torch.device(device)
        w.require(self.device.type == "cuda", "paged cache device (CUDA only)")
        if self.device.index is None:  # "cuda": the current device, named, so tensors compare equal
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.pages = batch * max_blocks
        cb = w.code_bytes(bits)
        dev = self.device

        def pool():
            return dict(codes=torch.zeros((h, self.pages, cb), dtype=torch.uint8, device=dev),
                        norm=torch.zeros((h, self.pages, w.BLOCK), dtype=torch.float16, device=dev),
                        min=torch.zeros((h, self.pages, w.DIM), dtype=torch.float16, device=dev),
                        scale=torch.zeros((h, self.pages, w.DIM), dtype=torch.float16, device=dev))

        self.records = None
        self.blk_bytes = 0
        if self.uses_alpha_path():
            self.records, self.k_pool, self.v_pool = block_record_pools(h, self.pages, bits, dev)
            self.blk_bytes = self.records.shape[-1]
        else:
            self.k_pool, self.v_pool = pool(), pool()
        self.block_table = torch.arange(self.pages, dtype=torch.int32, device=dev).reshape(batch, max_blocks)
        self.n_blocks = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.tail_len = torch.zeros(batch, dtype=torch.int32, device=dev)
        # host copies of n_blocks / tail_len, kept without reading the device: every change
        # to the counters comes from this object's prefill, import and seal (seal-at-64 is
        # deterministic); they size the attention kernels' work (never their correctness)
        # (int32, changed in place only: the step plan advances them through their memory)
        self.host_blocks = np.zeros(batch, np.int32)
        self.host_tail = np.zeros(batch, np.int32)
        self.k_tail = torch.zeros((batch, h, w.BLOCK, w.DIM), dtype=dtype, device=dev)
        self.v_tail = torch.zeros_like(self.k_tail)
        self.status = L.status_tensor(dev)
        self.seal_counters = torch.zeros(batch, dtype=torch.int32, device=dev)  # left at zero by every seal
        self.out = torch.empty((batch, self.hq, w.DIM), dtype=dtype, device=dev)
        lib = L.load()
        self.ws = torch.empty(lib.nsnkv_decode_attn_workspace_bytes(batch, self.hq, h, max_blocks, w.BLOCK - 1),
                              dtype=torch.uint8, device=dev)
        self._plan = None
        self._plan = self._make_plan(lib)
        self._step_fn = lib.nsnkv_paged_step
        self._step_host_fn = lib.nsnkv_paged_step_host
        self._q_shape = (batch, self.hq, w.DIM)
        self._kv_shape = (batch, h, w.DIM)

    def _make_plan(self, lib):
        """The native decode-step plan (nsnkv_paged_plan_create) over this cache's buffers."""
        kp, vp = self.k_pool, self.v_pool
        alpha = "alpha" in kp
        flags = 0
        if alpha:
            flags = L.ATTN_RECORD_ORDER | (L.ATTN_EXACT if self.restore_rounding == "exact" else 0)
        p = lambda t: t.data_ptr() if t is not None else None
        d = L.PagedDesc(
            struct_bytes=ctypes.sizeof(L.PagedDesc), batch=self.batch, hq=self.hq, h=self.h, bits=self.bits,
            dtype=L.DTYPE_CODE[self.dtype], flags=flags, max_blocks=self.max_blocks,
            k_codes=p(kp["codes"]), k_norm=p(kp["norm"]), k_min=p(kp["min"]), k_scale=p(kp["scale"]),
            k_alpha=p(kp.get("alpha")), v_codes=p(vp["codes"]), v_norm=p(vp["norm"]), v_min=p(vp["min"]),
            v_scale=p(vp["scale"]), v_alpha=p(vp.get("alpha")), blk_bytes=self.blk_bytes,
            blk_stride_head=self.pages, blk_stride_page=1, block_table=p(self.block_table),
            table_stride=self.max_blocks, n_blocks=p(self.n_blocks), tail_len=p(self.tail_len),
            k_tail=p(self.k_tail), v_tail=p(self.v_tail), tail_stride_seq=self.h * w.BLOCK,
            tail_stride_head=w.BLOCK, seq_counters=p(self.seal_counters) if alpha else None,
            workspace=p(self.ws), workspace_bytes=self.ws.numel(), status=p(self.status),
            host_n_blocks=self.host_blocks.ctypes.data, host_tail_len=self.host_tail.ctypes.data)
        handle = ctypes.c_void_p()
        L.check(lib.nsnkv_paged_plan_create(ctypes.byref(d), ctypes.byref(handle)), "nsnkv_paged_plan_create")
        return handle

    def __del__(self):
        plan, self._plan = getattr(self, "_plan", None), None
        if plan is not None and L._lib is not None:
            L._lib.nsnkv_paged_plan_destroy(plan)

    # ------------------------------------------------------------ prefill
    def prefill(self, b: int, k: torch.Tensor, v: torch.Tensor):
        """Load sequence b from native K/V [h, T, 128]: seal T//64 blocks, keep T%64 as the tail."""
        w.require(k.shape == v.shape and k.ndim == 3 and k.shape[0] == self.h and k.shape[2] == w.DIM, "prefill shape")
        T = k.shape[1]
        nb, t = T // w.BLOCK, T % w.BLOCK
        w.require(nb <= self.max_blocks, "prefill exceeds max_blocks")
        for src, pool, tail in ((k, self.k_pool, self.k_tail), (v, self.v_pool, self.v_tail)):
            if nb:
                x = src[:, :nb * w.BLOCK].reshape(self.h, nb, w.BLOCK, w.DIM).to(self.dtype)
                w.encode_blocks(x, self.bits, out=pool, out_row_stride=self.pages, out_offset=b * self.max_blocks,
                                check=False)
            if t:
                tail[b, :, :t].copy_(src[:, nb * w.BLOCK:])
        self.n_blocks[b] = nb
        self.tail_len[b] = t
        self.host_blocks[b], self.host_tail[b] = nb, t

    # ------------------------------------------------------------ exchange with the reference layout
    def export_groups(self, b: int):
        """Sequence b as the reference's data: (k_group, k_tail, v_group, v_tail).

        Groups are what encode_group(x, 0) returns for the same tokens
        (loop_kv_nb06_codec.py:28-34): codes [1, h, n, CB], metas (norm [1, h, n, 64, 1],
        min / scale [1, h, n, 1, 128]) and '<QHBB' headers [1, h, n, 12]; None when nothing
        is sealed.  Tails are [1, h, t, 128] in the cache dtype.
        """
        nb, t = int(self.n_blocks[b]), int(self.tail_len[b])
        pages = self.block_table[b, :nb].long()
        h = self.h

        def group(pool):
            if nb == 0:
                return None
            codes = w.from_code_order(pool["codes"][:, pages], self.bits, pool.get("code_order", 0))
            return dict(codes=codes.unsqueeze(0).contiguous(),
                        metas=(pool["norm"][:, pages].reshape(1, h, nb, w.BLOCK, 1).contiguous(),
                               pool["min"][:, pages].reshape(1, h, nb, 1, w.DIM).contiguous(),
                               pool["scale"][:, pages].reshape(1, h, nb, 1, w.DIM).contiguous()),
                        headers=checks.expected_headers(nb, h, self.bits, 0, self.device).contiguous())

        return (group(self.k_pool), self.k_tail[b, :, :t].unsqueeze(0).contiguous(), group(self.v_pool),
                self.v_tail[b, :, :t].unsqueeze(0).contiguous())

    def import_groups(self, b: int, kg, kt, vg, vt):
        """Load sequence b from the reference's layout; headers are verified.

        A tail of 64 tokens or more (the reference's PackedCache keeps 64..127) is sealed
        into further blocks, so the cache's seal-at-64 invariant holds afterwards.
        """
        h = self.h
        n = 0 if kg is None else kg["codes"].shape[2]
        w.require((kg is None) == (vg is None) and kt.shape == vt.shape and tuple(kt.shape[:2]) == (1, h)
                  and kt.shape[-1] == w.DIM, "import layout")
        for g in (kg, vg):
            if g is not None:
                w.require(tuple(g["codes"].shape) == (1, h, n, w.code_bytes(self.bits)) and checks.headers_ok(g),
                          "import blocks")
        t = kt.shape[2]
        extra, rest = t // w.BLOCK, t % w.BLOCK
        w.require(n + extra <= self.max_blocks, "import exceeds max_blocks")
        pages = self.block_table[b, :n].long()
        for g, pool in ((kg, self.k_pool), (vg, self.v_pool)):
            if g is None:
                continue
            codes = g["codes"][0].to(self.device)
            pool["codes"][:, pages] = w.to_code_order(codes, self.bits, pool.get("code_order", 0))
            pool["norm"][:, pages] = g["metas"][0].reshape(h, n, w.BLOCK).to(self.device)
            pool["min"][:, pages] = g["metas"][1].reshape(h, n, w.DIM).to(self.device)
            pool["scale"][:, pages] = g["metas"][2].reshape(h, n, w.DIM).to(self.device)
            if "alpha" in pool:
                w.block_renorm(pool, self.bits, h, n, self.pages, b * self.max_blocks)
        for src, pool, tail in ((kt, self.k_pool, self.k_tail), (vt, self.v_pool, self.v_tail)):
            src = src[0].to(self.device, self.dtype)
            if extra:
                x = src[:, :extra * w.BLOCK].reshape(h, extra, w.BLOCK, w.DIM)
                w.encode_blocks(x, self.bits, out=pool, out_row_stride=self.pages,
                                out_offset=b * self.max_blocks + n, check=False)
            tail[b, :, :rest].copy_(src[:, extra * w.BLOCK:])
        self.n_blocks[b] = n + extra
        self.tail_len[b] = rest
        self.host_blocks[b], self.host_tail[b] = n + extra, rest

    def to_bytes(self, b: int) -> bytes:
        """Sequence b in the sequence container format (see sequence_to_bytes)."""
        return sequence_to_bytes(*self.export_groups(b))

    def load_bytes(self, b: int, blob: bytes):
        """Load sequence b from sequence container bytes."""
        kg, kt, vg, vt = sequence_from_bytes(blob, self.device)
        self.import_groups(b, kg, kt, vg, vt)

    def lengths(self):
        return (self.n_blocks.long() * w.BLOCK + self.tail_len.long()).cpu()

    # ------------------------------------------------------------ decode
    def attend(self, q: torch.Tensor, k_new=None, v_new=None, out=None, out_f32=None, lse=None):
        """Attention of q [batch, hq, 128] over the cache (+ the appended token when given)."""
        return decode_attention(
            q, self.k_pool, self.v_pool, h=self.h, bits=self.bits, blk_stride_head=self.pages, blk_stride_page=1,
            n_blocks=self.n_blocks, max_blocks=self.max_blocks, k_tail=self.k_tail, v_tail=self.v_tail,
            tail_stride_seq=self.h * w.BLOCK, tail_stride_head=w.BLOCK, tail_len=self.tail_len,
            max_tail=w.BLOCK - 1, block_table=self.block_table, k_new=k_new, v_new=v_new,
            out=self.out if out is None else out, out_f32=out_f32, lse=lse, status=self.status, ws=self.ws,
            blk_bytes=self.blk_bytes, exact=self.restore_rounding == "exact",
            blocks_total=int(self.host_blocks.sum()))[0]

    def seal(self, pending_append: int = 1):
        t = self.host_tail + pending_append
        full = t >= w.BLOCK
        self.host_blocks += full
        self.host_tail[:] = t - w.BLOCK * full
        lib = L.load()
        if self.records is None:
            rc = lib.nsnkv_seal_full_tails(
                self.batch, self.h, self.bits, L.DTYPE_CODE[self.dtype], L.ptr(self.k_tail), L.ptr(self.v_tail),
                self.h * w.BLOCK, w.BLOCK, L.ptr(self.tail_len), L.ptr(self.n_blocks), pending_append,
                L.ptr(self.block_table), self.max_blocks,
                L.ptr(self.k_pool["codes"]), L.ptr(self.k_pool["norm"]), L.ptr(self.k_pool["min"]),
                L.ptr(self.k_pool["scale"]), L.ptr(self.v_pool["codes"]), L.ptr(self.v_pool["norm"]),
                L.ptr(self.v_pool["min"]), L.ptr(self.v_pool["scale"]), self.pages, 1, L.ptr(self.status),
                L.stream_handle(self.device))
            L.check(rc, "nsnkv_seal_full_tails")
            return
        rc = lib.nsnkv_seal_full_tails_alpha(
            self.batch, self.h, self.bits, L.DTYPE_CODE[self.dtype], L.ptr(self.k_tail), L.ptr(self.v_tail),
            self.h * w.BLOCK, w.BLOCK, L.ptr(self.tail_len), L.ptr(self.n_blocks), pending_append,
            L.ptr(self.block_table), self.max_blocks,
            L.ptr(self.k_pool["codes"]), L.ptr(self.k_pool["norm"]), L.ptr(self.k_pool["min"]),
            L.ptr(self.k_pool["scale"]), L.ptr(self.v_pool["codes"]), L.ptr(self.v_pool["norm"]),
            L.ptr(self.v_pool["min"]), L.ptr(self.v_pool["scale"]), L.ptr(self.k_pool["alpha"]),
            L.ptr(self.v_pool["alpha"]), self.blk_bytes, 1, L.ptr(self.seal_counters), self.pages, 1,
            L.ptr(self.status), L.stream_handle(self.device))
        L.check(rc, "nsnkv_seal_full_tails_alpha")

    def step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, out=None, attn_event=None):
        """One decode step: append (k_new, v_new) [batch, h, 128], attend with q [batch, hq, 128],
        seal full tails.  One native call (nsnkv_paged_step): the attention launches of
        ``attend`` and the seal of ``seal(1)``, with the host counters advanced in place.
        ``attn_event`` (a torch.cuda.Event) is recorded between the attention and the seal."""
        o = self.out if out is None else out
        dt, dev = self.dtype, self.device
        ok = (q.shape == self._q_shape and o.shape == self._q_shape and k_new.shape == self._kv_shape
              and v_new.shape == self._kv_shape and q.dtype == dt and k_new.dtype == dt and v_new.dtype == dt
              and o.dtype == dt and q.device == dev and k_new.device == dev and v_new.device == dev
              and o.device == dev and q.is_contiguous() and k_new.is_contiguous() and v_new.is_contiguous()
              and o.is_contiguous())
        w.require(ok, "paged step operands: contiguous q / out [batch, hq, 128] and k_new / v_new "
                      "[batch, h, 128] in the cache dtype, on the cache device")
        stream = torch.cuda.current_stream(dev)
        ev = None
        if attn_event is not None:
            if not attn_event.cuda_event:  # torch creates the event at its first record
                attn_event.record(stream)
            ev = attn_event.cuda_event
        rc = self._step_fn(self._plan, q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), o.data_ptr(), ev,
                           stream.cuda_stream)
        if rc:
            L.check(rc, "nsnkv_paged_step")
        return o

    def step_host(self, host_in: torch.Tensor, host_out: torch.Tensor, done_event=None):
        """One decode step from host memory (nsnkv_paged_step_host): ``host_in`` holds the
        step's q [batch, hq, 128], k_new and v_new [batch, h, 128] back to back, ``host_out``
        receives the output [batch, hq, 128]; both CPU tensors of the cache dtype, pinned for
        the copies to overlap the neighbouring steps.  The copies run on the plan's own
        streams: ``host_out`` is written (and ``host_in`` free again) once ``done_event`` (a
        torch.cuda.Event, recorded by the call) completed."""
        dt = self.dtype
        n_in = self.batch * (self.hq + 2 * self.h) * 128
        ok = (host_in.device.type == "cpu" and host_out.device.type == "cpu" and host_in.dtype == dt
              and host_out.dtype == dt and host_in.is_contiguous() and host_out.is_contiguous()
              and host_in.numel() == n_in and host_out.numel() == self.batch * self.hq * 128)
        w.require(ok, "paged host step operands: contiguous CPU tensors of the cache dtype, q|k_new|v_new "
                      "(batch * (hq + 2 h) * 128 elements) in and batch * hq * 128 out")
        stream = torch.cuda.current_stream(self.device)
        ev = None
        if done_event is not None:
            if not done_event.cuda_event:  # torch creates the event at its first record
                done_event.record(stream)
            ev = done_event.cuda_event
        with torch.cuda.device(self.device):
            rc = self._step_host_fn(self._plan, host_in.data_ptr(), host_out.data_ptr(), ev, stream.cuda_stream)
        if rc:
            L.check(rc, "nsnkv_paged_step_host")
        return host_out

    def check(self):
        st = int(self.status.item())
        if st:
            w._status_to_error(st, "Nonfinite decode input", output_msg="Nonfinite decode output")

    # ------------------------------------------------------------ accounting
    def kv_bytes(self):
        """Bytes held for K and V: what the reference's planned_bytes counts (codes, fp16
        metadata, 12-byte headers, native tail tokens; loop_kv_nb06_primitives.py:72-81)
        plus this cache's own derived data, the fp32 renorm factors (64 per K or V block)."""
        return self.reference_kv_bytes() + self.factor_bytes()

    def reference_kv_bytes(self):
        """planned_bytes of the cached tokens: codes + fp16 metadata + headers + tails."""
        nb = int(self.n_blocks.sum())
        t = int(self.tail_len.sum())
        per_block = w.code_bytes(self.bits) + w.BLOCK * 2 + w.DIM * 4 + 12
        return 2 * self.h * (nb * per_block + t * w.DIM * 2)

    def factor_bytes(self):
        """Bytes of the per-token renorm factors kept beside the sealed blocks (0 without)."""
        return 2 * self.h * int(self.n_blocks.sum()) * w.BLOCK * 4 if self.records is not None else 0

    def uses_alpha_path(self):
        """True when attend() runs the sealed blocks on the tensor-core kernels (block
        records with per-token renorm factors)."""
        return self.restore_rounding != "kv" and self.bits in (3, 5) and self.hq // self.h <= 8

    def read_bytes_per_step(self):
        """Algorithmic bytes one attend() reads: sealed blocks (codes + metadata) and tails, q and out.

        The renorm-factor kernel reads codes, min, scale and the fp32 factors of each
        block; the restore kernel reads codes, min, scale and the fp16 norms."""
        nb = int(self.n_blocks.sum())
        t = int(self.tail_len.sum())
        per_tok = 4 if self.uses_alpha_path() else 2
        per_block = w.code_bytes(self.bits) + w.BLOCK * per_tok + w.DIM * 4
        return 2 * self.h * (nb * per_block + t * w.DIM * 2) + 2 * self.batch * self.hq * w.DIM * 2
