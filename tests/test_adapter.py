"""Model adapter (install / make_cache / LoopedDecoder).

CPU: install() leaves an HF model bit-identical under the 'OFFICIAL' arm and restore()
removes the patch.  GPU: a looped decoder (shared-weight layers, one packed-cache slot
per (loop, layer)) decodes the same teacher-forced tokens with the fused packed arm
and with the reference bridge arm; every fused attention call matches the bridge on
the same packed data, the cache seals blocks by the reference policy, and the logits
of the two runs agree.
"""
import pytest
import torch

from oracle import nsn_oracle as O


def tiny_llama(heads=4, kv_heads=2, layers=2, head_dim=128, vocab=384, inter=768):
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=vocab, hidden_size=heads * head_dim, intermediate_size=inter,
                       num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=kv_heads,
                       head_dim=head_dim, max_position_embeddings=4096, rope_theta=10000.0,
                       attn_implementation="sdpa")


def test_install_official_arm_is_transparent_on_cpu():
    from transformers import LlamaForCausalLM
    from nsn_b200 import adapter
    torch.manual_seed(0)
    cfg = tiny_llama(heads=2, kv_heads=1, layers=2, head_dim=32, vocab=97, inter=64)
    model = LlamaForCausalLM(cfg).eval()
    ids = torch.randint(0, 97, (1, 12))
    with torch.no_grad():
        want = model(ids).logits
        restore = adapter.install(model)
        cache = adapter.make_cache()("OFFICIAL")
        assert cache.bits is None
        got = model(ids).logits
        restore()
        again = model(ids).logits
    assert torch.equal(got, want) and torch.equal(again, want)
    assert all(layer.self_attn.forward.__func__ is type(layer.self_attn).forward for layer in model.model.layers)


@pytest.mark.gpu
def test_looped_decoder_fused_matches_bridge():
    from nsn_b200 import adapter
    from nsn_b200 import kernel as K
    cfg = tiny_llama()
    loops, prompt_len, steps = 2, 150, 80
    torch.manual_seed(3)
    model = adapter.LoopedDecoder(cfg, loops).cuda().half().eval()
    gen = torch.Generator(device="cuda").manual_seed(3)
    prompt = torch.randint(0, cfg.vocab_size, (1, prompt_len), generator=gen, device="cuda")
    forced = torch.randint(0, cfg.vocab_size, (1, steps), generator=gen, device="cuda")
    restore = adapter.install(model)
    try:
        Cache = adapter.make_cache()
        fused = Cache("GQA_FUSED", loops)
        calls, seen = [], [0]

        def capture(slot, data, out):
            # every 7th decode call, across all steps (the cache replaces, never mutates, its tensors)
            if seen[0] % 7 == 0:
                calls.append((slot, data, out))
            seen[0] += 1

        fused.capture = capture
        logits_fused = model.generate_teacher_forced(prompt, forced, fused)
        bridge = Cache("TORCH_SDPA", loops)
        logits_bridge = model.generate_teacher_forced(prompt, forced, bridge)
        stepwise = Cache("GQA_FUSED", loops, checks="step")
        logits_step = model.generate_teacher_forced(prompt, forced, stepwise)
    finally:
        restore()
    slots = cfg.num_hidden_layers * loops
    assert all(fused.connections[s] == steps for s in range(slots))
    total = prompt_len + steps
    # reference policy: prefill keeps a tail of at least 64; decode seals one block at tail 128
    want_compressed = ((prompt_len - 64) // 64) * 64
    cur = want_compressed
    for i in range(1, steps + 1):
        if prompt_len + i - cur >= 128:
            cur += 64
    assert all(fused.compressed[s] == cur for s in range(slots)), (fused.compressed, cur)
    assert all(fused.get_seq_length(s) == total for s in range(slots))
    assert calls
    for slot, data, out in calls:
        want = K.pipeline("TORCH_SDPA", data)
        ok, err = O.within_tolerance(out.float().cpu().numpy(), want.float().cpu().numpy(), *O.TOLERANCE["float16"])
        assert ok, (slot, err)
    # reading the device status once per step changes nothing but the host syncs
    assert torch.equal(logits_step, logits_fused)
    # the fused and bridge runs differ only in the attention arithmetic
    assert torch.isfinite(logits_fused).all()
    scale = logits_bridge.float().abs().max().item()
    assert (logits_fused.float() - logits_bridge.float()).abs().max().item() <= 2e-2 * scale
