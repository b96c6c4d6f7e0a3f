"""PagedKVCache: batched packed-KV cache for decode serving (append + attend + seal).

The reference grows each slot's packed groups with ``torch.cat`` on every seal
(experiments/nb06/source/loop_kv_nb06_packed.py:36-50, ``append_group``
loop_kv_nb06_codec.py:40-45), which re-copies the whole packed history and syncs
the host.  Here the packed blocks live in a fixed page pool addressed through a
block table, and one decode step is three launches with no host sync:

  1. nsnkv_decode_attn   appends the new K/V token to each sequence's fp16 tail
                         and attends over sealed blocks + tail (split-KV partials
                         + log-sum-exp merge);
  2. nsnkv_seal_full_tails  encodes every tail that reached 64 tokens into the
                         sequence's next page and advances n_blocks / tail_len.

Policy: seal whenever a tail reaches 64 tokens, so tails hold 0..63 tokens
between steps (the benchmark specification's batched policy; the reference's
per-slot PackedCache keeps 64..127, see nsn_b200.packed).

Layout (head-major pools so one sequence's blocks of one head are contiguous):
  codes [h, pages, code_bytes] uint8, norm [h, pages, 64], min/scale [h, pages, 128] fp16
  block (sequence b, head j, block i) = pool row j, page block_table[b, i]
  block_table [batch, max_blocks] int32 (sequence b owns pages b*max_blocks ..)
  n_blocks, tail_len [batch] int32 (device), k_tail/v_tail [batch, h, 64, 128].
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import primitives as w
from .kernel import decode_attention


class PagedKVCache:
    def __init__(self, batch: int, h: int, max_blocks: int, bits: int = 3, dtype=torch.float16, device="cuda",
                 hq: int | None = None):
        w.require(batch > 0 and h > 0 and max_blocks > 0 and bits in (3, 4, 5), "paged cache shape")
        w.require(dtype in (torch.float16, torch.bfloat16), "paged cache dtype")
        L.require_cuda()
        self.batch, self.h, self.max_blocks, self.bits, self.dtype = batch, h, max_blocks, bits, dtype
        self.hq = hq or h
        self.device = torch.device(device)
        self.pages = batch * max_blocks
        cb = w.code_bytes(bits)
        dev = self.device

        def pool():
            return dict(codes=torch.zeros((h, self.pages, cb), dtype=torch.uint8, device=dev),
                        norm=torch.zeros((h, self.pages, w.BLOCK), dtype=torch.float16, device=dev),
                        min=torch.zeros((h, self.pages, w.DIM), dtype=torch.float16, device=dev),
                        scale=torch.zeros((h, self.pages, w.DIM), dtype=torch.float16, device=dev))

        self.k_pool, self.v_pool = pool(), pool()
        self.block_table = torch.arange(self.pages, dtype=torch.int32, device=dev).reshape(batch, max_blocks)
        self.n_blocks = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.tail_len = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.k_tail = torch.zeros((batch, h, w.BLOCK, w.DIM), dtype=dtype, device=dev)
        self.v_tail = torch.zeros_like(self.k_tail)
        self.status = L.status_tensor(dev)
        self.out = torch.empty((batch, self.hq, w.DIM), dtype=dtype, device=dev)
        lib = L.load()
        self.ws = torch.empty(lib.nsnkv_decode_attn_workspace_bytes(batch, self.hq, h, max_blocks, w.BLOCK - 1),
                              dtype=torch.uint8, device=dev)

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
            out=self.out if out is None else out, out_f32=out_f32, lse=lse, status=self.status, ws=self.ws)[0]

    def seal(self, pending_append: int = 1):
        lib = L.load()
        rc = lib.nsnkv_seal_full_tails(
            self.batch, self.h, self.bits, L.DTYPE_CODE[self.dtype], L.ptr(self.k_tail), L.ptr(self.v_tail),
            self.h * w.BLOCK, w.BLOCK, L.ptr(self.tail_len), L.ptr(self.n_blocks), pending_append,
            L.ptr(self.block_table), self.max_blocks,
            L.ptr(self.k_pool["codes"]), L.ptr(self.k_pool["norm"]), L.ptr(self.k_pool["min"]),
            L.ptr(self.k_pool["scale"]), L.ptr(self.v_pool["codes"]), L.ptr(self.v_pool["norm"]),
            L.ptr(self.v_pool["min"]), L.ptr(self.v_pool["scale"]), self.pages, 1, L.ptr(self.status),
            L.stream_handle(self.device))
        L.check(rc, "nsnkv_seal_full_tails")

    def step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, out=None):
        """One decode step: append (k_new, v_new) [batch, h, 128], attend with q, seal full tails."""
        o = self.attend(q, k_new, v_new, out=out)
        self.seal(1)
        return o

    def check(self):
        st = int(self.status.item())
        if st:
            w._status_to_error(st, "Nonfinite decode input", output_msg="Nonfinite decode output")

    # ------------------------------------------------------------ accounting
    def kv_bytes(self):
        """Bytes held for K and V: codes + fp16 metadata + 12-byte headers + fp16 tail tokens."""
        nb = int(self.n_blocks.sum())
        t = int(self.tail_len.sum())
        per_block = w.code_bytes(self.bits) + w.BLOCK * 2 + w.DIM * 4 + 12
        return 2 * self.h * (nb * per_block + t * w.DIM * 2)

    def read_bytes_per_step(self):
        """Algorithmic bytes one attend() reads: sealed blocks (codes + metadata) and tails, q and out."""
        nb = int(self.n_blocks.sum())
        t = int(self.tail_len.sum())
        per_block = w.code_bytes(self.bits) + w.BLOCK * 2 + w.DIM * 4
        return 2 * self.h * (nb * per_block + t * w.DIM * 2) + 2 * self.batch * self.hq * w.DIM * 2
