"""CPU PyTorch port of the reference's bridge decode path (timed CPU baseline).

TEST/BASELINE INFRASTRUCTURE ONLY: used by ``bench.py``'s ``cpu_baseline`` leg and
``--impl reference`` arm, never by the product.  It restates, with the same torch
CPU operators, what the reference's bridge does for one decode query:

  restore_group(g, float16)  = nsn_decode(unpack3(codes), metas, fp16)
        (experiments/nb06/source/loop_kv_nb06_codec.py:36-38,
         loop_kv_nb06_primitives.py:57-66: d = m + s*q; y = n * d / max(||d||, eps);
         0 where n == 0; cast)
  torch.cat((restored, tail), dim=2)          (loop_kv_nb06_kernel.py:167-168)
  repeat_kv + F.scaled_dot_product_attention  (loop_kv_nb06_kernel.py:156-174)

The reference itself cannot be imported on the GPU box (it is not shipped), so
this port is the "reference" CPU arm; its arithmetic is pinned to the reference
by tests/test_oracle_golden.py (same restore bits, same SDPA call).
"""
from __future__ import annotations

import torch

EPS = 1e-12


def unpack3(payload: torch.Tensor, shape) -> torch.Tensor:
    """INT3 3-byte groups -> uint8 codes (loop_kv_nb06_codec.py:17-26)."""
    n = 1
    for x in shape:
        n *= x
    a = payload.reshape(-1)
    if a.numel() % 3:
        a = torch.cat((a, torch.zeros(3 - a.numel() % 3, dtype=torch.uint8)))
    a = a.reshape(-1, 3)
    x, y, z = a[:, 0], a[:, 1], a[:, 2]
    vals = (x & 7, (x >> 3) & 7, ((x >> 6) | (y << 2)) & 7, (y >> 1) & 7, (y >> 4) & 7,
            ((y >> 7) | (z << 1)) & 7, (z >> 2) & 7, (z >> 5) & 7)
    return torch.stack(vals, -1).reshape(-1)[:n].reshape(shape).contiguous()


def unpack_bits(payload: torch.Tensor, shape, bits: int) -> torch.Tensor:
    if bits == 3:
        return unpack3(payload, shape)
    n = 1
    for x in shape:
        n *= x
    b = payload.reshape(-1).to(torch.int64)
    b = torch.cat((b, torch.zeros(2, dtype=torch.int64)))
    pos = torch.arange(n, dtype=torch.int64) * bits
    v = (b[pos // 8] | (b[pos // 8 + 1] << 8)) >> (pos % 8)
    return (v & ((1 << bits) - 1)).to(torch.uint8).reshape(shape)


def nsn_decode(q, metas, dtype):
    n, m, s = (t.float().contiguous() for t in metas)
    d = (m + s * q.float().contiguous()).contiguous()
    y = n * (d / torch.linalg.vector_norm(d, dim=-1, keepdim=True).clamp_min(EPS))
    return torch.where(n == 0, torch.zeros_like(y), y).to(dtype)


def restore_group(codes, metas, dtype, bits=3):
    b, h, n, _ = codes.shape
    q = unpack_bits(codes, (b, h, n, 64, 128), bits)
    return nsn_decode(q, metas, dtype).reshape(b, h, n * 64, 128)


def repeat_kv(x, n_rep):
    b, h, t, d = x.shape
    if n_rep == 1:
        return x
    return x[:, :, None, :, :].expand(b, h, n_rep, t, d).reshape(b, h * n_rep, t, d)


def bridge_decode(q, k_codes, k_metas, k_tail, v_codes, v_metas, v_tail, bits=3):
    """q [1,hq,1,128]; codes [1,h,n,cb]; tails [1,h,t,128] -> out [1,1,hq,128] (q.dtype)."""
    dtype = q.dtype
    kf = torch.cat((restore_group(k_codes, k_metas, dtype, bits), k_tail), 2)
    vf = torch.cat((restore_group(v_codes, v_metas, dtype, bits), v_tail), 2)
    rep = q.shape[1] // kf.shape[1]
    out = torch.nn.functional.scaled_dot_product_attention(q, repeat_kv(kf, rep), repeat_kv(vf, rep))
    return out.transpose(1, 2).contiguous()
