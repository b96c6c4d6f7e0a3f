"""GPU checks of the batched looped-decoder driver (nsn_b200.looped.PagedLoopedDecoder).

The driver is the model's own projections, norms and MLP around one PagedKVCache per
(loop, layer) slot.  Its attention is checked against the reference bridge end to end:
a second driver runs the same model and caches, but takes each decode step's attention
from the bridge arithmetic (restore_group of the slot's exported groups in the cache
dtype, then SDPA in fp32 over the restored rows, the native tail and the new token;
experiments/nb06/source/loop_kv_nb06_kernel.py:156-174) while the caches advance through
the same nsnkv_paged_step.  The two drivers' logits agree to the attention parity bar
carried through the layers.  A CUDA-graph replay of the decode step gives the eager
step's logits.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def small_model(loops=2, layers=2, hidden=256, heads=2, kv_heads=2):
    from transformers import LlamaConfig
    from nsn_b200 import adapter
    cfg = LlamaConfig(vocab_size=512, hidden_size=hidden, intermediate_size=512, num_hidden_layers=layers,
                      num_attention_heads=heads, num_key_value_heads=kv_heads, head_dim=128,
                      max_position_embeddings=1024, rope_theta=10000.0, attn_implementation="sdpa")
    torch.manual_seed(7)
    return adapter.LoopedDecoder(cfg, loops=loops).cuda().half().eval()


def bridge_driver_class():
    from nsn_b200 import codec
    from nsn_b200.looped import PagedLoopedDecoder

    class BridgeDriver(PagedLoopedDecoder):
        """Decode attention from the bridge over each slot's cache; the cache still steps."""

        def _attend(self, cache, q, k, v):
            B = q.shape[0]
            outs = []
            for b in range(B):
                kg, kt, vg, vt = cache.export_groups(b)
                ks = [codec.restore_group(kg, self.dtype)[0]] if kg is not None else []
                vs = [codec.restore_group(vg, self.dtype)[0]] if vg is not None else []
                kk = torch.cat(ks + [kt[0], k[b, :, None]], 1).float()  # [h, T, 128]
                vv = torch.cat(vs + [vt[0], v[b, :, None]], 1).float()
                rep = self.hq // self.h
                kk, vv = kk.repeat_interleave(rep, 0), vv.repeat_interleave(rep, 0)
                s = torch.einsum("jd,jtd->jt", q[b].float(), kk) / np.sqrt(128.0)
                outs.append(torch.einsum("jt,jtd->jd", torch.softmax(s, -1), vv).to(self.dtype))
            cache.step(q, k, v)
            return torch.stack(outs)

    return BridgeDriver


@pytest.mark.parametrize("heads,kv_heads", [(2, 2), (4, 2)])
def test_driver_matches_bridge_driver(heads, kv_heads):
    from nsn_b200.looped import PagedLoopedDecoder
    model = small_model(heads=heads, kv_heads=kv_heads)
    B, P, steps = 3, 100, 70
    gen = torch.Generator(device="cpu").manual_seed(11)
    ids = torch.randint(0, 512, (B, P + steps), generator=gen).cuda()
    kern = PagedLoopedDecoder(model, B, P + steps)
    ref = bridge_driver_class()(model, B, P + steps)
    la, lb = kern.prefill(ids[:, :P]), ref.prefill(ids[:, :P])
    assert torch.equal(la, lb)  # the same prefill path
    worst = 0.0
    for t in range(steps):
        la = kern.step(ids[:, P + t]).float()
        lb = ref.step(ids[:, P + t]).float()
        err = (la - lb).abs().max().item() / max(lb.abs().max().item(), 1e-6)
        worst = max(worst, err)
    kern.check()
    ref.check()
    # both sets of caches sealed the same blocks
    assert kern.caches[0].n_blocks.cpu().tolist() == [(P + steps) // 64] * B
    assert worst < 2e-2, worst


def test_graph_replay_matches_eager_steps():
    from nsn_b200.looped import PagedLoopedDecoder
    model = small_model()
    B, P, steps = 2, 120, 40
    gen = torch.Generator(device="cpu").manual_seed(12)
    ids = torch.randint(0, 512, (B, P + steps), generator=gen).cuda()
    eager = PagedLoopedDecoder(model, B, P + steps)
    graph = PagedLoopedDecoder(model, B, P + steps)
    eager.prefill(ids[:, :P])
    graph.prefill(ids[:, :P])
    for t in range(3):  # eager warm-up steps on both, then the capture
        eager.step(ids[:, P + t])
        graph.step(ids[:, P + t])
    graph.capture()
    for t in range(3, steps):
        a = eager.step(ids[:, P + t]).float()
        b = graph.replay(ids[:, P + t]).float()
        err = (a - b).abs().max().item() / max(a.abs().max().item(), 1e-6)
        assert err < 1e-3, (t, err)
    torch.cuda.synchronize()
    graph.sync_counters()
    for ce, cg in zip(eager.caches, graph.caches):
        assert torch.equal(ce.n_blocks, cg.n_blocks) and torch.equal(ce.tail_len, cg.tail_len)
        assert list(ce.host_blocks) == list(cg.host_blocks) and list(ce.host_tail) == list(cg.host_tail)
    graph.release()
    eager.check()
    graph.check()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_layer_ops_match_the_llama_modules(dtype):
    """nsnkv_add_rmsnorm, nsnkv_rope_split and nsnkv_swiglu against the transformers
    modules they replace at decode: RoPE and SwiGLU bit for bit; the RMSNorm within one unit
    of the dtype (its fp32 sum of squares runs in another order than torch's mean)."""
    from transformers.models.llama import modeling_llama as m
    from nsn_b200.looped import add_rmsnorm, rope_split, swiglu
    torch.manual_seed(5)
    rows, dim, hq, h, inter = 4, 2048, 16, 4, 5632
    x = torch.randn(rows, dim, device="cuda").to(dtype)
    r = torch.randn(rows, dim, device="cuda").to(dtype)
    norm = m.LlamaRMSNorm(dim, eps=1e-5).cuda().to(dtype)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(dim, device="cuda") + 0.5)
        res, y = add_rmsnorm(x, r, norm.weight, norm.variance_epsilon)
        assert torch.equal(res, x + r)
        want = norm(x + r)
        ulp = (want.float().abs() * (2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7)).clamp_min(1e-6)
        assert ((y.float() - want.float()).abs() <= ulp).all()
        res0, y0 = add_rmsnorm(x, None, norm.weight, norm.variance_epsilon)
        assert res0.data_ptr() == x.data_ptr()
        assert ((y0.float() - norm(x).float()).abs() <= (norm(x).float().abs() * 2.0 ** -7).clamp_min(1e-6)).all()
        # RoPE at one position for every row
        qkv = torch.randn(rows, (hq + 2 * h) * 128, device="cuda").to(dtype)
        cfg = m.LlamaConfig(hidden_size=dim, num_attention_heads=hq, num_key_value_heads=h, head_dim=128,
                            rope_theta=10000.0, max_position_embeddings=4096)
        rot = m.LlamaRotaryEmbedding(cfg).cuda()
        cos, sin = rot(qkv[:, None], torch.tensor([[777]], device="cuda"))
        q, k, v = rope_split(qkv, cos.reshape(-1), sin.reshape(-1), hq, h)
        q4 = qkv[:, :hq * 128].view(rows, 1, hq, 128).transpose(1, 2)
        k4 = qkv[:, hq * 128:(hq + h) * 128].view(rows, 1, h, 128).transpose(1, 2)
        qr, kr = m.apply_rotary_pos_emb(q4, k4, cos, sin)
        assert torch.equal(q, qr[:, :, 0]) and torch.equal(k, kr[:, :, 0])
        assert torch.equal(v, qkv[:, (hq + h) * 128:].view(rows, h, 128))
        # SwiGLU
        gu = torch.randn(rows, 2 * inter, device="cuda").to(dtype) * 3
        want = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
        assert torch.equal(swiglu(gu), want)


@pytest.mark.parametrize("fixed", [False, True])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("m,n,k", [(4, 6144, 2048), (1, 2048, 5632), (8, 512, 256), (3, 32000, 2048)])
def test_gemv_rows_matches_linear(dtype, m, n, k, fixed):
    """nsnkv_gemv_rows against torch's linear (fp32 accumulation in both, different order),
    with and without NSNKV_GEMV_FIXED_WEIGHTS (weight loads before the programmatic wait)."""
    from nsn_b200.looped import linear_rows
    torch.manual_seed(m * 7 + k)
    x = torch.randn(m, k, device="cuda").to(dtype)
    w = (torch.randn(n, k, device="cuda") / np.sqrt(k)).to(dtype)
    got = linear_rows(x, w, fixed).float()
    want = (x.double() @ w.double().t())
    tol = (2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7) * want.abs() + 1e-3
    assert ((got.double() - want).abs() <= tol).all(), (got.double() - want).abs().max().item()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_layer_chain_back_to_back_equals_synchronised(dtype):
    """The layer kernels launch with programmatic dependent launch, and the GEMV with fixed
    weights loads weight rows before its wait.  A decode layer's chain enqueued back to back
    (each kernel reading what the one before it wrote) gives the same bits as the same chain
    with a device synchronise after every op, over 20 repetitions."""
    from nsn_b200.looped import add_rmsnorm, linear_rows, rope_split, swiglu
    torch.manual_seed(21)
    rows, dim, hq, h, inter = 4, 2048, 16, 16, 5632
    wqkv = (torch.randn((hq + 2 * h) * 128, dim, device="cuda") / np.sqrt(dim)).to(dtype)
    wo = (torch.randn(dim, hq * 128, device="cuda") / np.sqrt(hq * 128)).to(dtype)
    wgu = (torch.randn(2 * inter, dim, device="cuda") / np.sqrt(dim)).to(dtype)
    wd = (torch.randn(dim, inter, device="cuda") / np.sqrt(inter)).to(dtype)
    ln = (torch.rand(dim, device="cuda") + 0.5).to(dtype)
    cos = torch.cos(torch.arange(128, device="cuda") * 0.01).to(dtype)
    sin = torch.sin(torch.arange(128, device="cuda") * 0.01).to(dtype)

    def chain(h0, sync):
        s = torch.cuda.synchronize if sync else (lambda: None)
        res, x = add_rmsnorm(h0, None, ln, 1e-5); s()
        qkv = linear_rows(x, wqkv, True); s()
        q, k, v = rope_split(qkv, cos, sin, hq, h); s()
        a = linear_rows(q.reshape(rows, -1), wo, True); s()
        h2, x2 = add_rmsnorm(a, res, ln, 1e-5); s()
        gu = linear_rows(x2, wgu, True); s()
        y = linear_rows(swiglu(gu), wd, True); s()
        return torch.cat([h2.flatten(), k.flatten(), v.flatten(), y.flatten()])

    with torch.no_grad():
        for rep in range(20):
            h0 = torch.randn(rows, dim, device="cuda").to(dtype)
            want = chain(h0, True)
            got = chain(h0, False)
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), want.view(torch.int16)), rep
