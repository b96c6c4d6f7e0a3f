"""GPU parity of the K1c batched decode-score kernel (experiments/kernels/phase_k1c_triton_fused_kernel.py).

On the reference's own stores (rebuilt by the pinned oracle) the scores must pass the
reference's gate (rel-max <= 1e-2 against its fp32 scores) with room to spare: the
kernel computes in fp32, so it is held to rel-max <= 1e-5.  A larger cell (batch 8,
2048 tokens, head_dim 256) is checked against the oracle's fp32 scores.
"""
import numpy as np
import pytest
import torch

import golden_util as G

pytestmark = pytest.mark.gpu


def _cuda_store(t):
    return {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in t.items()}


def _rel(got, want):
    return float((got - want).abs().max() / want.abs().max().clamp(min=1e-6))


@pytest.mark.parametrize("cell", G.index()["k1c"]["cells"], ids=lambda c: c["key"])
def test_k1c_scores_pass_the_reference_gate(cell):
    from nsn_b200.k1c import triton_decode_scores
    from oracle import k1c
    model = k1c.MODELS[cell["model"]]
    q, tstore, _ = k1c.make_store(model, cell["B"], cell["T"], cell["bits"], cell["recipe"])
    got = triton_decode_scores(q.cuda(), _cuda_store(tstore), model["n_q"], model["n_kv"], model["head_dim"]).cpu()
    want = torch.from_numpy(G.get(cell["key"] + "_scores"))
    rel = _rel(got, want)
    assert rel <= G.index()["k1c"]["gate_tol"] and rel <= 1e-5, rel


@pytest.mark.parametrize("recipe", ["nsn", "kivi", "fp16"])
def test_k1c_scores_large_cell(recipe):
    from nsn_b200.k1c import triton_decode_scores
    from oracle import k1c
    model = k1c.MODELS["gemma"]
    q, tstore, ref32 = k1c.make_store(model, 8, 2048, 5, recipe)
    want = k1c.gate_scores(q, ref32, recipe, model)
    got = triton_decode_scores(q.cuda(), _cuda_store(tstore), model["n_q"], model["n_kv"], model["head_dim"]).cpu()
    assert _rel(got, want) <= 1e-5
