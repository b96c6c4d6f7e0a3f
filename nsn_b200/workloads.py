"""Seeded synthetic inputs for the five configurations of the packed-KV path.

There is no public dataset on this path: the reference measures on K/V blocks
captured from its own model runs, which are not available here.  These
generators stand in for them with the shapes, sizes and value distributions
the benchmark specification names:

  cfg0  seed 0: K,V [1,8,1024,128] fp16 = N(0,1) x per-token lognormal(0,0.5);
        K has 4 fixed outlier channels x8; q [1,32,1,128] N(0,1); 16 INT3 blocks,
        0-token tail, GQA 32:8.
  cfg1  seed 1: 511 INT3 blocks + 64-token fp16 tail, GQA 32:8, q N(0,1)/sqrt(128).
  cfg2  seed 2: batch 64, GQA 32:8, per-sequence blocks U{32..256}, tail U[0,63].
  cfg4  seed 4: GQA 64:8, 2047 INT5 blocks + 64 tail, K 8 outlier channels x8,
        V per-token lognormal(0,1) norms.

Two backends: ``np_*`` (NumPy ``default_rng``; used for golden fixtures and
CPU-sized parity cases) and ``torch_*`` (a seeded ``torch.Generator`` on the
target device; used for the full-size benchmark and GPU property tests).  The
two backends draw different numbers from the same distributions.
"""
from __future__ import annotations

import math

import numpy as np

BLOCK = 64
DIM = 128

K_OUTLIERS_4 = (3, 37, 71, 105)
K_OUTLIERS_8 = (3, 19, 37, 53, 71, 87, 105, 121)

CONFIGS = {
    0: dict(name="cfg0-cpu-reference", seed=0, hq=32, h=8, blocks=16, tail=0, bits=3,
            k_outliers=K_OUTLIERS_4, v_sigma=0.5, q_scale=1.0),
    1: dict(name="cfg1-single-seq-32k", seed=1, hq=32, h=8, blocks=511, tail=64, bits=3,
            k_outliers=K_OUTLIERS_4, v_sigma=0.5, q_scale=1.0 / math.sqrt(128)),
    2: dict(name="cfg2-batched-64", seed=2, hq=32, h=8, batch=64, min_blocks=32, max_blocks=256,
            max_tail=63, bits=3, k_outliers=K_OUTLIERS_4, v_sigma=0.5, q_scale=1.0 / math.sqrt(128)),
    4: dict(name="cfg4-long-131k-int5", seed=4, hq=64, h=8, blocks=2047, tail=64, bits=5,
            k_outliers=K_OUTLIERS_8, v_sigma=1.0, q_scale=1.0 / math.sqrt(128)),
}


def np_kv(rng, shape, outliers=(), sigma=0.5, dtype=np.float16):
    """N(0,1) entries times a per-token lognormal(0, sigma) magnitude; outlier channels x8."""
    x = rng.standard_normal(shape, dtype=np.float32)
    mag = rng.lognormal(0.0, sigma, size=shape[:-1] + (1,)).astype(np.float32)
    x = x * mag
    if outliers:
        x[..., list(outliers)] *= 8
    return x.astype(dtype)


def np_config(cfg: int, heads=None, blocks=None, tail=None):
    """K, V [1,H,T,128] fp16 and q [1,Hq,1,128] fp16 for a single-sequence config.

    ``heads``/``blocks``/``tail`` shrink the config for CPU-sized parity runs
    (the distributions are unchanged).
    """
    c = CONFIGS[cfg]
    rng = np.random.default_rng(c["seed"])
    h = heads or c["h"]
    group = c["hq"] // c["h"]
    nb = c["blocks"] if blocks is None else blocks
    t = c["tail"] if tail is None else tail
    total = nb * BLOCK + t
    k = np_kv(rng, (1, h, total, DIM), c["k_outliers"], 0.5)
    v = np_kv(rng, (1, h, total, DIM), (), c["v_sigma"])
    q = (rng.standard_normal((1, h * group, 1, DIM), dtype=np.float32) * np.float32(c["q_scale"])).astype(np.float16)
    return k, v, q, nb, t


def np_cfg2_lengths(batch=None, seed=None):
    """Per-sequence (sealed blocks, tail tokens) for the batched config."""
    c = CONFIGS[2]
    rng = np.random.default_rng(c["seed"] if seed is None else seed)
    b = batch or c["batch"]
    blocks = rng.integers(c["min_blocks"], c["max_blocks"] + 1, size=b)
    tails = rng.integers(0, c["max_tail"] + 1, size=b)
    return blocks.astype(np.int64), tails.astype(np.int64)


def torch_kv(gen, shape, outliers=(), sigma=0.5, dtype=None, device="cuda"):
    """Device-side twin of ``np_kv`` drawn from a seeded torch.Generator."""
    import torch
    dtype = dtype or torch.float16
    x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    mag = torch.empty(shape[:-1] + (1,), device=device, dtype=torch.float32).log_normal_(0.0, sigma, generator=gen)
    x.mul_(mag)
    if outliers:
        x[..., list(outliers)] *= 8
    return x.to(dtype)
