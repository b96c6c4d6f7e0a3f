"""Batched GQA decode scores over a per-channel quantised K cache (the K1c kernel's contract).

Mirrors ``triton_decode_scores(q, tstore, n_q, n_kv, head_dim)``
(experiments/kernels/phase_k1c_triton_fused_kernel.py:252-283). ``tstore`` is the
reference's dict:
- ``code`` uint8 [B, T, n_kv*D], or fp16 K for FP16;
- ``min`` / ``step`` fp16 [B, n_kv*D];
- ``eff_norm`` fp16 [B, n_kv, T] for NSN;
- flags ``is_fp16`` / ``is_nsn``.
The result is fp32 scores [B, n_q, T]. The work runs in libnsnkv.so
(``nsnkv_k1c_scores``), which reads each K byte once for all query heads of its kv head.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import primitives as w


def triton_decode_scores(q, tstore, n_q, n_kv, head_dim):
    L.require_cuda()
    B, T = q.shape[0], tstore["T"]
    w.require(tuple(q.shape) == (B, n_q, head_dim) and q.dtype == torch.float16, "K1c query layout")
    recipe = 0 if tstore["is_fp16"] else (2 if tstore["is_nsn"] else 1)
    code = tstore["code"].contiguous()
    w.require(tuple(code.shape) == (B, T, n_kv * head_dim), "K1c code layout")
    mn = tstore.get("min")
    st = tstore.get("step")
    en = tstore.get("eff_norm")
    out = torch.empty((B, n_q, T), dtype=torch.float32, device=q.device)
    # contiguous copies stay referenced until the launch is enqueued
    qc, mn, st, en = (None if t is None else t.contiguous() for t in (q, mn, st, en))
    L.check(L.load().nsnkv_k1c_scores(recipe, B, n_q, n_kv, T, head_dim, L.ptr(qc), L.ptr(code), L.ptr(mn),
                                      L.ptr(st), L.ptr(en), L.ptr(out), L.stream_handle(q.device)),
            "nsnkv_k1c_scores")
    return out


decode_scores = triton_decode_scores
