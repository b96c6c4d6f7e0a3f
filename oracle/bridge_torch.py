"""CPU PyTorch port of the reference's bridge decode path (timed CPU baseline).

TEST/BASELINE INFRASTRUCTURE ONLY: used by ``bench.py``'s ``cpu_baseline`` leg and
``--impl reference`` arm, never by the product.  It restates, with the same torch
CPU operators, what the reference does for one decode step of one sequence:

  restore_group(g, float16)  = nsn_decode(unpack3(codes), metas, fp16)
        (experiments/nb06/source/loop_kv_nb06_codec.py:36-38,
         loop_kv_nb06_primitives.py:57-66: d = m + s*q; y = n * d / max(||d||, eps);
         0 where n == 0; cast)
  torch.cat((restored, tail), dim=2)          (loop_kv_nb06_kernel.py:167-168)
  repeat_kv + F.scaled_dot_product_attention  (loop_kv_nb06_kernel.py:156-174)
  the cache append: torch.cat of the new token onto the native tail, and when a tail
  reaches 64 tokens encode_group of those 64 (nsn_encode :37-55 + pack3, codec :6-15,
  :28-34) appended to the packed group with torch.cat (append_group, codec :40-45)

The reference itself cannot be imported on the GPU box (it is not shipped), so
this port is the "reference" CPU arm.  tests/test_oracle_golden.py pins it to the
reference's recorded outputs: bridge_decode reproduces every recorded SDPA output bit
for bit, nsn_encode + pack3 every recorded encode.
"""
from __future__ import annotations

import torch

EPS = 1e-12
BLOCK = 64


def nsn_encode(x, bits=3):
    """loop_kv_nb06_primitives.py:37-55 with torch CPU operators: per-token fp32 norm,
    directions, per-channel min / (max - min) / (2^bits - 1), rounded codes, fp16 metas.
    Returns (q uint8 [..., 64, 128], (n, m, s) fp16); the reference's non-finite checks
    raise ValueError here."""
    a = x.float()
    n = torch.linalg.vector_norm(a, dim=-1, keepdim=True)
    d = a / n.clamp_min(EPS)
    m = d.amin(dim=-2, keepdim=True)
    mx = d.amax(dim=-2, keepdim=True)
    s = (mx - m) / ((1 << bits) - 1)
    denom = torch.where(s == 0, torch.ones_like(s), s)
    q = torch.round((d - m) / denom).clamp(0, (1 << bits) - 1).to(torch.uint8)
    q = torch.where(s == 0, torch.zeros_like(q), q)
    metas = tuple(t.to(torch.float16) for t in (n, m, s))
    if not all(bool(torch.isfinite(t).all()) for t in metas):
        raise ValueError("non-finite fp16 metadata")
    return q, metas


def pack3(q):
    """INT3 codes -> LSB-first bytes, eight codes in three bytes (loop_kv_nb06_codec.py:6-15)."""
    n = q.numel()
    a = q.contiguous().reshape(-1)
    if n % 8:
        a = torch.cat((a, torch.zeros(8 - n % 8, dtype=torch.uint8)))
    a = a.reshape(-1, 8)
    b0 = a[:, 0] | (a[:, 1] << 3) | (a[:, 2] << 6)
    b1 = (a[:, 2] >> 2) | (a[:, 3] << 1) | (a[:, 4] << 4) | (a[:, 5] << 7)
    b2 = (a[:, 5] >> 1) | (a[:, 6] << 2) | (a[:, 7] << 5)
    return torch.stack((b0, b1, b2), -1).reshape(-1)[:(n * 3 + 7) // 8].clone()


def encode_group(x):
    """x [1, h, n, 64, 128] -> (codes [1, h, n, 3072], metas) (loop_kv_nb06_codec.py:28-34, headers omitted)."""
    q, metas = nsn_encode(x, 3)
    b, h, n = q.shape[:3]
    return pack3(q).reshape(b, h, n, 64 * 128 * 3 // 8), tuple(m.contiguous().clone() for m in metas)


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


class BridgeSequence:
    """One sequence of the batched decode under the benchmark's cfg2 policy, the reference way.

    Holds the packed K and V groups and the native tails as torch CPU tensors.  step()
    appends the new token to the tails (torch.cat), attends with the bridge, and seals a
    tail that reached 64 tokens: encode_group of it, torch.cat onto the groups."""

    def __init__(self, k_codes, k_metas, k_tail, v_codes, v_metas, v_tail):
        self.k = [k_codes, k_metas, k_tail]
        self.v = [v_codes, v_metas, v_tail]

    def step(self, q, k_new, v_new):
        """q [1, hq, 1, 128]; k_new / v_new [1, h, 1, 128] -> out [1, 1, hq, 128]."""
        for st, new in ((self.k, k_new), (self.v, v_new)):
            st[2] = torch.cat((st[2], new), 2)
        out = bridge_decode(q, self.k[0], self.k[1], self.k[2], self.v[0], self.v[1], self.v[2])
        if self.k[2].shape[2] >= BLOCK:
            for st in (self.k, self.v):
                h = st[2].shape[1]
                codes, metas = encode_group(st[2][:, :, :BLOCK].reshape(1, h, 1, BLOCK, 128))
                st[0] = torch.cat((st[0], codes), 2)
                st[1] = tuple(torch.cat((a, b), 2) for a, b in zip(st[1], metas))
                st[2] = st[2][:, :, BLOCK:].contiguous()
        return out
