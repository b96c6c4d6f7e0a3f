"""Model adapter: single-query decode of an HF attention module over the packed cache.

Serves the role of experiments/nb06/source/loop_kv_nb06_attention.py:13-88. ``make_cache``
is a PackedCache whose ``append_for_attention`` appends a decode token without
restoring the slot's K/V. ``decode`` runs the projections, RoPE and the fused packed
attention of one query. ``install`` patches every layer's ``self_attn.forward`` and
returns a ``restore`` callable.

The module targets the current transformers attention signature
``forward(hidden_states, position_embeddings, attention_mask, past_key_values, **kw)``,
the one experiments/ac08/source/loop_kv_ac08_attention.py:46-96 patches. Looped
models get their KV slot as ``loop_idx * layers + layer_idx``, with ``loop_idx``
passed through the layer's keyword arguments.

Arms: 'OFFICIAL' leaves every call to the original forward. 'NATIVE' keeps a native
(unpacked) cache behind the same connection. 'GQA_FUSED' runs nsnkv_decode_attn on
the packed blocks plus tail. 'TORCH_SDPA' runs the reference's bridge (restore +
repeat_kv + SDPA). Prefill (more than one query token) through a connection cache
appends to the slot and runs causal SDPA over the materialised K/V. That matches the
bridge; the reference leaves prefill to the model's own forward, whose layer index
does not carry the loop.

``LoopedDecoder`` drives a shared-weight stack of decoder layers for ``loops``
passes, one KV slot per (loop, layer): the cfg3 looped-transformer shape.
"""
from __future__ import annotations

import inspect
from collections import Counter
from types import MethodType

import torch

from . import kernel as K
from . import primitives as w
from .packed import make_packed_cache

ARMS = ("OFFICIAL", "NATIVE", "GQA_FUSED", "TORCH_SDPA")


class ListCacheBase:
    """Per-slot key/value lists: the HF DynamicCache surface the packed cache builds on."""

    def __init__(self):
        self.key_cache = []
        self.value_cache = []
        self._seen_tokens = 0

    def get_seq_length(self, layer_idx=0):
        if layer_idx >= len(self.key_cache) or self.key_cache[layer_idx] is None:
            return 0
        return self.key_cache[layer_idx].shape[-2]

    def update(self, key, value, layer_idx, cache_kwargs=None):
        while len(self.key_cache) <= layer_idx:
            self.key_cache.append(None)
            self.value_cache.append(None)
        for data, x in ((self.key_cache, key), (self.value_cache, value)):
            data[layer_idx] = x if data[layer_idx] is None else torch.cat((data[layer_idx], x), -2)
        self._seen_tokens = self.get_seq_length(layer_idx)
        return self.key_cache[layer_idx], self.value_cache[layer_idx]


def make_cache(base=ListCacheBase):
    """The connection cache class: a PackedCache over `base` as the patched layers use it.

    Besides the packed cache it carries the arm, the check granularity and per-slot
    counters, and ``append_for_attention``, which appends a decode token to a slot
    without restoring it: the fused arm reads the sealed blocks and the tail directly,
    and the bridge arm restores them itself (experiments/nb06/source/loop_kv_nb06_attention.py:13-31
    defers the restoration the same way; skipped_k / skipped_v count the restorations
    saved, as there)."""
    parent = make_packed_cache(base)

    class ConnectionCache(parent):
        def __init__(self, arm, loops=1, checks="call"):
            w.require(arm in ARMS, "Unknown model arm")
            w.require(checks in ("call", "step"), "Check granularity")
            super().__init__(loops, None if arm in ("OFFICIAL", "NATIVE") else 3)
            self.arm = arm
            # "call": every attention call runs the reference pipeline's checks (host syncs);
            # "step": fused calls OR their device status into one word that post_decode reads
            self.checks = checks
            self.status = None
            self.connections = Counter()  # attention calls per slot
            self.skipped_k = Counter()    # restorations saved per slot
            self.skipped_v = Counter()
            self.capture = None           # optional callable(slot, data, out) after each decode call

        def append_for_attention(self, key, value, slot, kwargs):
            w.require(self.restore_observer is None, "Recursive/decorated restore")
            if self._append(key, value, slot, kwargs) is None:
                self.skipped_k[slot] += 1
                self.skipped_v[slot] += 1

        def post_decode(self):
            if self.checks == "step" and self.status is not None:
                st = int(self.status.item())
                if st:
                    self.status.zero_()
                    K._raise_status(st)
            super().post_decode()

    return ConnectionCache


def _slot(attn, loop_idx):
    layers = attn.config.num_hidden_layers
    w.require(type(loop_idx) is int and loop_idx >= 0, "Loop/cache slot identity")
    return attn.layer_idx + loop_idx * layers


def _project(attn, module, hidden_states, position_embeddings):
    bsz, q_len, _ = hidden_states.shape
    shape = (bsz, q_len, -1, attn.head_dim)
    q = attn.q_proj(hidden_states).view(shape).transpose(1, 2)
    k = attn.k_proj(hidden_states).view(shape).transpose(1, 2)
    v = attn.v_proj(hidden_states).view(shape).transpose(1, 2)
    cos, sin = position_embeddings
    q, k = module.apply_rotary_pos_emb(q, k, cos, sin)
    return q, k, v, cos, sin


def decode(attn, module, hidden_states, position_embeddings, cache, loop_idx=0, cache_position=None):
    """One query token of one sequence through the packed cache and the arm's attention."""
    bsz, q_len, _ = hidden_states.shape
    w.require((bsz, q_len) == (1, 1) and not attn.training, "Single-query eval/cache only")
    w.require(attn.head_dim == w.DIM and attn.scaling == w.DIM ** -0.5, "GQA dimensions")
    slot = _slot(attn, loop_idx)
    q, k, v, cos, sin = _project(attn, module, hidden_states, position_embeddings)
    cache.append_for_attention(k, v, slot, {"sin": sin, "cos": cos, "cache_position": cache_position})
    data = (cache.packed.get((slot, "K")), cache.key_cache[slot], q.contiguous(), cache.packed.get((slot, "V")),
            cache.value_cache[slot])
    if cache.checks == "step" and cache.arm == "GQA_FUSED":
        from . import checks
        checks.structural(*data)
        if cache.status is None:
            cache.status = torch.zeros(1, dtype=torch.int32, device=q.device)
        out = K.launch(*data, check=False, status=cache.status)[0]
    else:
        out = K.pipeline("GQA_FUSED" if cache.arm == "GQA_FUSED" else "TORCH_SDPA", data)
    cache.connections[slot] += 1
    if cache.capture is not None:
        cache.capture(slot, data, out)
    out = out.reshape(bsz, q_len, -1)
    return attn.o_proj(out), None


def prefill(attn, module, hidden_states, position_embeddings, cache, loop_idx=0, cache_position=None):
    """Prompt tokens of one sequence: append to the slot, causal SDPA over the materialised K/V."""
    bsz, q_len, _ = hidden_states.shape
    slot = _slot(attn, loop_idx)
    w.require(bsz == 1 and cache.get_seq_length(slot) == 0, "Prefill starts an empty slot")
    q, k, v, cos, sin = _project(attn, module, hidden_states, position_embeddings)
    kk, vv = cache.update(k, v, slot, {"sin": sin, "cos": cos, "cache_position": cache_position})
    rep = q.shape[1] // kk.shape[1]
    out = torch.nn.functional.scaled_dot_product_attention(q, K.repeat_kv(kk, rep), K.repeat_kv(vv, rep),
                                                           is_causal=True, scale=attn.scaling)
    out = out.transpose(1, 2).reshape(bsz, q_len, -1)
    return attn.o_proj(out), None


def install(model):
    """Patch every ``model.model.layers[i].self_attn`` (or ``model.layers[i]``); returns ``restore()``."""
    originals = []
    layers = model.model.layers if hasattr(model, "model") else model.layers
    for layer in layers:
        attn = layer.self_attn
        original = attn.forward
        module = inspect.getmodule(attn.__class__)
        originals.append((attn, original))

        def forward(self, hidden_states, position_embeddings=None, attention_mask=None, past_key_values=None,
                    _original=original, _module=module, **kwargs):
            loop_idx = kwargs.pop("loop_idx", 0)
            connected = hasattr(past_key_values, "append_for_attention")
            if not connected or past_key_values.arm == "OFFICIAL":
                w.require(loop_idx == 0, "Looped slots need a connection cache")
                return _original(hidden_states, position_embeddings=position_embeddings, attention_mask=attention_mask,
                                 past_key_values=past_key_values, **kwargs)
            cache_position = kwargs.pop("cache_position", None)
            if hidden_states.shape[1] != 1:
                return prefill(self, _module, hidden_states, position_embeddings, past_key_values, loop_idx,
                               cache_position)
            return decode(self, _module, hidden_states, position_embeddings, past_key_values, loop_idx,
                          cache_position)

        attn.forward = MethodType(forward, attn)

    def restore():
        for attn, original in originals:
            attn.forward = original

    return restore


class LoopedDecoder(torch.nn.Module):
    """A looped decoder: ``loops`` passes over one stack of transformers decoder layers.

    ``config`` is a transformers LlamaConfig (SwiGLU MLP, RMSNorm, RoPE). Weights are
    shared across loops, and each (loop, layer) pair has its own KV slot in the cache.
    The packed cache's slot count and kv-head count come from ``w.LAYERS`` and
    ``w.HEADS``, which the constructor sets, as the reference fixes them per model.
    """

    def __init__(self, config, loops):
        super().__init__()
        from transformers.models.llama import modeling_llama as m
        self.config, self.loops = config, loops
        self.embed = torch.nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = torch.nn.ModuleList([m.LlamaDecoderLayer(config, i) for i in range(config.num_hidden_layers)])
        self.norm = m.LlamaRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.lm_head = torch.nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.rotary = m.LlamaRotaryEmbedding(config)
        w.LAYERS = config.num_hidden_layers
        w.HEADS = config.num_key_value_heads

    @torch.no_grad()
    def forward(self, input_ids, cache, start):
        """Logits [1, T, vocab] of tokens input_ids [1, T] at positions start..start+T-1."""
        h = self.embed(input_ids)
        pos = torch.arange(start, start + input_ids.shape[1], device=input_ids.device)[None]
        emb = self.rotary(h, pos)
        for loop in range(self.loops):
            for layer in self.layers:
                h = layer(h, attention_mask=None, position_ids=pos, past_key_values=cache, position_embeddings=emb,
                          cache_position=pos[0], loop_idx=loop)
        return self.lm_head(self.norm(h))

    @torch.no_grad()
    def generate_teacher_forced(self, prompt, forced, cache):
        """Prefill ``prompt`` [1, P], then decode the tokens of ``forced`` [1, S] one by one.

        Returns the logits of every decode step [S, vocab]. The cache is sealed after
        prefill and after each step by the packed cache's own policy.
        """
        self(prompt, cache, 0)
        cache.post_prefill()
        out = []
        for i in range(forced.shape[1]):
            out.append(self(forced[:, i:i + 1], cache, prompt.shape[1] + i)[0, -1])
            cache.post_decode()
        return torch.stack(out)
