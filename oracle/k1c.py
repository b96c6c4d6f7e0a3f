"""CPU oracle for the K1c batched decode scores.  TEST INFRASTRUCTURE ONLY.

Restates, with torch CPU ops:
- the input generation and cache layouts of
  experiments/kernels/phase_k1c_triton_fused_kernel.py: _quant_codes_over_tokens :63-69,
  kivi_store :91-93, nsn_store :96-106, _make_inputs :133-149, make_triton_store :172-197;
- its fp32 gate reference, _torch_decode_scores :152-168 on the fp16 store widened to fp32.
The restatement is pinned by the sha256 of the reference's own stores and by its
recorded fp32 gate scores (tests/golden, tests/test_oracle_golden.py).  Only tests use it.
"""
from __future__ import annotations

import math

import torch

SEED = 20260510
EPS = 1e-12
RENORM_EPS = 1e-8
MODELS = {"gemma": dict(n_kv=8, head_dim=256, n_q=32), "qwen": dict(n_kv=8, head_dim=128, n_q=32)}


def _codes_over_tokens(x, bits):
    levels = (1 << bits) - 1
    lo = x.amin(dim=1, keepdim=True)
    hi = x.amax(dim=1, keepdim=True)
    step = ((hi - lo).float() / levels).clamp(min=EPS).to(x.dtype)
    code = ((x - lo).float() / step.float()).round().clamp(0, levels).to(x.dtype)
    return code, lo, step


def make_store(model, B, T, bits, recipe, dtype=torch.float16):
    """(q fp16 [B,n_q,D], tstore dict as the kernel reads it, fp32 reference store)."""
    n_kv, D, n_q = model["n_kv"], model["head_dim"], model["n_q"]
    g = torch.Generator(device="cpu").manual_seed(SEED)
    q = torch.randn(B, n_q, D, generator=g, dtype=torch.float32).to(dtype)
    k = torch.randn(B, T, n_kv * D, generator=g, dtype=torch.float32)
    if recipe == "fp16":
        kf = k.to(dtype)
        return q, dict(code=kf.contiguous(), is_fp16=True, is_nsn=False, T=T, n_kv=n_kv, head_dim=D), \
            dict(kfp16=kf.float())
    if recipe == "kivi":
        code, lo, step = _codes_over_tokens(k, bits)
        ref = dict(code=code.to(dtype), min=lo.to(dtype), step=step.to(dtype))
    else:
        x = k.reshape(B, T, n_kv, D).float()
        norm = x.norm(dim=-1, keepdim=True).clamp(min=EPS)
        d = x / norm
        code, lo, step = _codes_over_tokens(d, bits)
        dq = code * step + lo
        eff = norm / dq.norm(dim=-1, keepdim=True).clamp(min=RENORM_EPS)
        ref = dict(code=code.reshape(B, T, n_kv * D).to(dtype), min=lo.reshape(B, 1, n_kv * D).to(dtype),
                   step=step.reshape(B, 1, n_kv * D).to(dtype), eff_norm=eff.reshape(B, T, n_kv).to(dtype))
    t = dict(code=ref["code"].round().clamp(0, 255).to(torch.uint8).contiguous(), is_fp16=False,
             is_nsn=recipe == "nsn", min=ref["min"].squeeze(1).contiguous(), step=ref["step"].squeeze(1).contiguous(),
             T=T, n_kv=n_kv, head_dim=D)
    if recipe == "nsn":
        t["eff_norm"] = ref["eff_norm"].transpose(1, 2).contiguous()
    return q, t, {kk: v.float() for kk, v in ref.items()}


def gate_scores(q, ref32, recipe, model):
    """_torch_decode_scores on the fp32-widened store: fp32 scores [B, n_q, T]."""
    n_kv, D, n_q = model["n_kv"], model["head_dim"], model["n_q"]
    B = q.shape[0]
    if recipe == "fp16":
        kdq = ref32["kfp16"]
    elif recipe == "kivi":
        kdq = ref32["code"] * ref32["step"] + ref32["min"]
    else:
        T = ref32["code"].shape[1]
        dq = (ref32["code"] * ref32["step"] + ref32["min"]).reshape(B, T, n_kv, D)
        kdq = (ref32["eff_norm"].unsqueeze(-1) * dq).reshape(B, T, n_kv * D)
    T = kdq.shape[1]
    kdq = kdq.reshape(B, T, n_kv, D)
    qx = q.float().reshape(B, n_kv, n_q // n_kv, D)
    return (torch.einsum("bnrd,btnd->bnrt", qx, kdq) / math.sqrt(D)).reshape(B, n_q, T)
