"""Batched decode of a looped decoder over paged packed-KV caches (the cfg3 shape).

The reference drives its looped model one sequence at a time through a connection cache
per (loop, layer) slot (experiments/ac08/source/loop_kv_ac08_attention.py:46-96,
experiments/nb06/source/loop_kv_nb06_attention.py:33-88): per token, loops x layers
attention calls, each with host-side cache updates and a ``torch.cat`` of the slot's
tails.  Here a batch of sequences steps together:

* one ``PagedKVCache`` per (loop, layer) slot holds every sequence of the batch
  (seal-at-64, block records on the tensor-core kernel);
* a decode step is, per layer evaluation, four projections on [batch, hidden] rows
  (nsnkv_gemv_rows, fused q|k|v and gate|up weights), this library's fused per-token
  kernels (nsnkv_add_rmsnorm twice, nsnkv_rope_split, nsnkv_swiglu) and one
  ``nsnkv_paged_step`` (append + attention + seal);
* nothing in a step reads the device or allocates, so the whole step is captured once
  as a CUDA graph (``capture``) and replayed per token (``replay``);
* prefill runs causal SDPA (its FlashAttention kernels) over the fp16 prompt and encodes
  each slot's keys and values into its cache.

Keys are cached after RoPE, as the model's own cache update receives them.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib as L
from .paged import PagedKVCache


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def add_rmsnorm(x, residual, weight, eps):
    """(x + residual, RMSNorm(x + residual) * weight) over rows [rows, dim] (nsnkv_add_rmsnorm);
    residual may be None, then x itself is normalised and returned as the residual."""
    rows, dim = x.shape
    out = torch.empty_like(x)
    res = torch.empty_like(x) if residual is not None else x
    rc = L.load().nsnkv_add_rmsnorm(rows, dim, L.DTYPE_CODE[x.dtype], x.data_ptr(),
                                    residual.data_ptr() if residual is not None else None, weight.data_ptr(),
                                    eps, res.data_ptr() if residual is not None else None, out.data_ptr(), _stream(x))
    L.check(rc, "nsnkv_add_rmsnorm")
    return res, out


def rope_split(qkv, cos, sin, hq, h):
    """Fused projection rows [rows, (hq + 2h) * 128] -> RoPE'd q [rows, hq, 128], k and v
    [rows, h, 128] (nsnkv_rope_split); cos / sin [128] shared by every row."""
    rows = qkv.shape[0]
    q = torch.empty((rows, hq, 128), dtype=qkv.dtype, device=qkv.device)
    k = torch.empty((rows, h, 128), dtype=qkv.dtype, device=qkv.device)
    v = torch.empty_like(k)
    rc = L.load().nsnkv_rope_split(rows, hq, h, L.DTYPE_CODE[qkv.dtype], qkv.data_ptr(), cos.data_ptr(),
                                   sin.data_ptr(), 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), _stream(qkv))
    L.check(rc, "nsnkv_rope_split")
    return q, k, v


def linear_rows(x, weight, fixed_weight=False):
    """x [m, k] @ weight[n, k]^T for decode rows (nsnkv_gemv_rows when m <= 8, n % 8 == 0 and
    k % 256 == 0; torch's linear otherwise).  ``fixed_weight``: no work enqueued before this
    call writes ``weight`` (model weights while decoding), so the kernel may start streaming
    it before the preceding kernel on the stream has finished."""
    m, k = x.shape
    n = weight.shape[0]
    if not (m <= 8 and n % 8 == 0 and k % 256 == 0 and x.is_contiguous() and weight.is_contiguous()
            and x.data_ptr() % 16 == 0 and weight.data_ptr() % 16 == 0):
        return F.linear(x, weight)
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    rc = L.load().nsnkv_gemv_rows(m, n, k, L.DTYPE_CODE[x.dtype], x.data_ptr(), weight.data_ptr(), y.data_ptr(),
                                  L.GEMV_FIXED_WEIGHTS if fixed_weight else 0, _stream(x))
    L.check(rc, "nsnkv_gemv_rows")
    return y


def swiglu(gate_up):
    """Rows [rows, 2 * inter] = [gate | up] -> silu(gate) * up [rows, inter] (nsnkv_swiglu)."""
    rows, two = gate_up.shape
    out = torch.empty((rows, two // 2), dtype=gate_up.dtype, device=gate_up.device)
    rc = L.load().nsnkv_swiglu(rows, two // 2, L.DTYPE_CODE[gate_up.dtype], gate_up.data_ptr(), out.data_ptr(),
                               _stream(gate_up))
    L.check(rc, "nsnkv_swiglu")
    return out


class PagedLoopedDecoder:
    """Decode driver for an ``adapter.LoopedDecoder`` (its weights and layer modules).

    ``batch`` sequences, up to ``max_tokens`` tokens each (prompt + decoded), one paged
    cache per (loop, layer) slot with ``restore_rounding`` as in ``PagedKVCache``.
    """

    def __init__(self, model, batch: int, max_tokens: int, restore_rounding: str = "k"):
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
        self.model, self.batch = model, batch
        cfg = model.config
        self.h, self.hq = cfg.num_key_value_heads, cfg.num_attention_heads
        self.head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        if self.head_dim != 128:
            raise ValueError("PagedLoopedDecoder: the packed cache stores head_dim 128")
        self.rope = apply_rotary_pos_emb
        self.device = model.embed.weight.device
        self.dtype = model.embed.weight.dtype
        self.max_blocks = -(-max_tokens // 64) + 1  # a spare page: a full tail always finds one
        n_slots = model.loops * len(model.layers)
        self.caches = [PagedKVCache(batch, self.h, self.max_blocks, bits=3, dtype=self.dtype, device=self.device,
                                    hq=self.hq, restore_rounding=restore_rounding) for _ in range(n_slots)]
        # the decode step's fused weights: q|k|v and gate|up concatenated (copies; the model's
        # own modules keep theirs for the prefill)
        self.fused = []
        for layer in model.layers:
            a, mlp = layer.self_attn, layer.mlp
            if any(getattr(m, "bias", None) is not None for m in (a.q_proj, a.k_proj, a.v_proj, a.o_proj,
                                                                  mlp.gate_proj, mlp.up_proj, mlp.down_proj)):
                raise ValueError("PagedLoopedDecoder: projections without biases (Llama) only")
            self.fused.append((torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight]).contiguous(),
                               torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight]).contiguous()))
        self.length = 0  # tokens per sequence held by the caches
        self.graph = None
        self._ids = torch.zeros(batch, dtype=torch.long, device=self.device)
        self._pos = torch.zeros((1, 1), dtype=torch.long, device=self.device)
        self._logits = None

    # ------------------------------------------------------------ prefill: the model's own modules
    def _prefill_layer(self, layer, h, cos, sin, cache):
        attn = layer.self_attn
        B, T, _ = h.shape
        x = layer.input_layernorm(h)
        q = attn.q_proj(x).view(B, T, self.hq, self.head_dim).transpose(1, 2)
        k = attn.k_proj(x).view(B, T, self.h, self.head_dim).transpose(1, 2)
        v = attn.v_proj(x).view(B, T, self.h, self.head_dim).transpose(1, 2)
        q, k = self.rope(q, k, cos, sin)
        rep = self.hq // self.h
        kr = k.repeat_interleave(rep, dim=1) if rep > 1 else k
        vr = v.repeat_interleave(rep, dim=1) if rep > 1 else v
        o = F.scaled_dot_product_attention(q, kr, vr, is_causal=True)
        o = o.transpose(1, 2).reshape(B, T, self.hq * self.head_dim)
        for b in range(B):
            cache.prefill(b, k[b], v[b])
        h = h + attn.o_proj(o)
        return h + layer.mlp(layer.post_attention_layernorm(h))

    def _prefill_forward(self, ids, pos):
        m = self.model
        h = m.embed(ids)
        cos, sin = m.rotary(h, pos)
        slot = 0
        for _ in range(m.loops):
            for layer in m.layers:
                h = self._prefill_layer(layer, h, cos, sin, self.caches[slot])
                slot += 1
        return m.lm_head(m.norm(h[:, -1]))

    # ------------------------------------------------------------ decode: fused per-token ops
    def _attend(self, cache, q, k, v):
        """Decode attention of q [B, hq, 128] with (k, v) [B, h, 128] appended: the paged step."""
        return cache.step(q, k, v)

    def _decode_forward(self, ids, pos):
        """ids [B], pos [1, 1] -> logits [B, vocab].  The residual stream h and the pending
        block output are added by the next norm (nsnkv_add_rmsnorm)."""
        m = self.model
        h = m.embed(ids)  # [B, hidden]
        cos, sin = m.rotary(h[:, None], pos)
        cos, sin = cos.reshape(-1), sin.reshape(-1)
        pending, slot = None, 0
        for _ in range(m.loops):
            for layer, (wqkv, wgu) in zip(m.layers, self.fused):
                a, mlp = layer.self_attn, layer.mlp
                ln1, ln2 = layer.input_layernorm, layer.post_attention_layernorm
                if pending is None:
                    h, x = add_rmsnorm(h, None, ln1.weight, ln1.variance_epsilon)
                else:
                    h, x = add_rmsnorm(pending, h, ln1.weight, ln1.variance_epsilon)
                q, k, v = rope_split(linear_rows(x, wqkv, True), cos, sin, self.hq, self.h)
                o = self._attend(self.caches[slot], q, k, v)
                h, x = add_rmsnorm(linear_rows(o.reshape(h.shape[0], -1), a.o_proj.weight, True), h, ln2.weight,
                                   ln2.variance_epsilon)
                pending = linear_rows(swiglu(linear_rows(x, wgu, True)), mlp.down_proj.weight, True)
                slot += 1
        _, x = add_rmsnorm(pending, h, m.norm.weight, m.norm.variance_epsilon)
        return linear_rows(x, m.lm_head.weight, True)

    # ------------------------------------------------------------ public API
    @torch.no_grad()
    def prefill(self, ids: torch.Tensor) -> torch.Tensor:
        """Prompt ids [batch, P] (every sequence the same length) -> last-token logits [batch, vocab]."""
        if ids.shape[0] != self.batch or self.length:
            raise ValueError("PagedLoopedDecoder.prefill: one prompt per sequence, into empty caches")
        P = ids.shape[1]
        if P + 1 > 64 * (self.max_blocks - 1):
            raise ValueError("PagedLoopedDecoder.prefill: the prompt exceeds max_tokens")
        pos = torch.arange(P, device=self.device)[None]
        logits = self._prefill_forward(ids.to(self.device), pos)
        self.length = P
        return logits

    @torch.no_grad()
    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """One token per sequence, ids [batch] -> logits [batch, vocab] (eager launches)."""
        if self.length + 1 > 64 * (self.max_blocks - 1):
            raise ValueError("PagedLoopedDecoder.step: max_tokens reached")
        self._pos.fill_(self.length)
        logits = self._decode_forward(ids.to(self.device).reshape(self.batch), self._pos)
        self.length += 1
        return logits

    @torch.no_grad()
    def capture(self):
        """Record the next decode step as a CUDA graph over static id / position buffers.

        Capturing launches nothing; the caches' host counters (which size the attention
        grid) advance once during the capture and are re-read from the device by
        ``sync_counters``, which ``replay`` callers run when they stop replaying."""
        if self.length + 1 > 64 * (self.max_blocks - 1):
            raise ValueError("PagedLoopedDecoder.capture: max_tokens reached")
        self._pos.fill_(self.length)
        torch.cuda.synchronize(self.device)
        snap = [(c.host_blocks.copy(), c.host_tail.copy()) for c in self.caches]
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._logits = self._decode_forward(self._ids, self._pos)
        for c, (nb, tl) in zip(self.caches, snap):  # nothing ran: the counters are where they were
            c.host_blocks[:] = nb
            c.host_tail[:] = tl

    @torch.no_grad()
    def replay(self, ids: torch.Tensor) -> torch.Tensor:
        """One decode step through the captured graph: ids [batch] -> logits [batch, vocab]
        (a view of the graph's output buffer, overwritten by the next replay)."""
        if self.graph is None:
            raise RuntimeError("PagedLoopedDecoder.replay: capture() first")
        if self.length + 1 > 64 * (self.max_blocks - 1):
            raise ValueError("PagedLoopedDecoder.replay: max_tokens reached")
        self._ids.copy_(ids.reshape(self.batch), non_blocking=True)
        self._pos.fill_(self.length)
        self.graph.replay()
        self.length += 1
        return self._logits

    def sync_counters(self):
        """Re-read every cache's n_blocks / tail_len from the device into its host copies."""
        for c in self.caches:
            c.host_blocks[:] = c.n_blocks.cpu().numpy()
            c.host_tail[:] = c.tail_len.cpu().numpy()

    def check(self):
        for c in self.caches:
            c.check()

    def kv_bytes(self):
        """Bytes the caches hold for the sequences' tokens (reference format + renorm factors)."""
        return sum(c.kv_bytes() for c in self.caches)

    def release(self):
        """Drop the captured graph (before the caches it references)."""
        self.graph = None
        self._logits = None
