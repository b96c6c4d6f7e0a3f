"""Fused packed-KV decode attention: the reference's VF01 / NB06 operator surface.

Mirrors experiments/ac08/source/loop_kv_vf01_kernel.py:117-158 (MHA) and
experiments/nb06/source/loop_kv_nb06_kernel.py:131-191 (GQA):

  restore_v(g, tail)                  bridge reconstruction of full-length V (:120-126)
  launch(g, kt, q, vg, vt, trace)     fused attention -> (out, context, score, v) (:128-139)
  pipeline(arm, (g, kt, q, vg, vt))   structural -> input_finite -> attention -> output (:141-158)
  repeat_kv / reference / sdpa        the torch bridge arm (nb06 :156-174)

Arms: 'V_FUSED' / 'GQA_FUSED' (packed K and V consumed in one fused kernel),
'TILE_MATERIALIZE' / 'TILE_SDPA' / 'RF01_MATERIALIZE' (restore kernel writes full
K and V, then the same attention kernel reads them as native rows),
'TORCH_SDPA' (restore kernel + torch.cat + repeat_kv + torch SDPA).
The GQA group is hq / h of the inputs (the reference's NB06 hard-codes 48:8).
``LAST_STAGE`` is maintained as in the reference; non-finite inputs found by the
fused kernel raise NumericalFailure at stage 'input_finite'.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import checks
from . import primitives as w
from .codec import restore_group

LAST_STAGE = "idle"
attention_launch_count = 0
FUSED_ARMS = ("V_FUSED", "GQA_FUSED")
TILE_ARMS = ("TILE_MATERIALIZE", "TILE_SDPA", "RF01_MATERIALIZE")

_workspace_cache: dict = {}


def workspace(nbytes: int, device) -> torch.Tensor:
    """Reusable scratch for the split-KV partials, one buffer per (device, current stream).

    Calls on one stream run in order, so they can share a buffer; calls on different
    streams get different buffers and never race on the partials.  A buffer that grows is
    replaced on its own stream only, where every earlier call has been ordered before the
    caching allocator can hand the old memory out again.
    """
    device = torch.device(device)
    stream = torch.cuda.current_stream(device)
    key = (str(device), stream.cuda_stream)
    buf = _workspace_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspace_cache[key] = buf
    return buf


def decode_attention(q, k_pool, v_pool, *, h, bits, blk_stride_head, blk_stride_page, n_blocks, max_blocks,
                     k_tail=None, v_tail=None, tail_stride_seq=0, tail_stride_head=0, tail_len=0, max_tail=0,
                     block_table=None, k_new=None, v_new=None, out=None, out_f32=None, lse=None, status=None,
                     ws=None, blk_bytes=None, exact=False, blocks_total=0):
    """Direct binding of nsnkv_decode_attn (nsnkv_decode_attn_alpha when both pools carry
    "alpha" or their arrays are fields of block records).

    q [B, hq, 128]; k_pool/v_pool dicts of codes/norm/min/scale tensors, plus the
    per-token renorm factors "alpha" (fp32, 64 per block) when the cache keeps them
    (or None when max_blocks == 0); n_blocks/tail_len either ints (same for every
    sequence) or int32 CUDA tensors [B].  blk_bytes: the block stride of the
    codes / min / scale / alpha arrays (None: read from the tensors' strides, 0: dense).
    With renorm factors, K rows are rounded to the cache dtype as the reference bridge
    rounds them unless ``exact`` (then K and V are both the exact fp32 restore);
    ``blocks_total`` (the sum of n_blocks, when known) sizes their kernel's chunks.
    Returns (out, status).
    """
    L.require_cuda()
    B, hq = q.shape[0], q.shape[1]
    dev = q.device
    if out is None:
        out = torch.empty((B, hq, 128), dtype=q.dtype, device=dev)
    if status is None:
        status = L.status_tensor(dev)
    lib = L.load()
    need = lib.nsnkv_decode_attn_workspace_bytes(B, hq, h, max_blocks, max_tail)
    if ws is None:
        ws = workspace(need, dev)
    nb_t = n_blocks if isinstance(n_blocks, torch.Tensor) else None
    tl_t = tail_len if isinstance(tail_len, torch.Tensor) else None
    kp = k_pool or {}
    vp = v_pool or {}
    if blk_bytes is None:
        blk_bytes = 0
        if max_blocks:
            blk_bytes = w.blk_bytes_of(kp, bits)
            w.require(w.blk_bytes_of(vp, bits) == blk_bytes, "K and V pool layouts")
    blocks = (L.ptr(kp.get("codes")), L.ptr(kp.get("norm")), L.ptr(kp.get("min")), L.ptr(kp.get("scale")),
              L.ptr(vp.get("codes")), L.ptr(vp.get("norm")), L.ptr(vp.get("min")), L.ptr(vp.get("scale")))
    has_alpha = kp.get("alpha") is not None and vp.get("alpha") is not None
    orders = (int(kp.get("code_order", 0)), int(vp.get("code_order", 0)))
    w.require(orders in ((0, 0), (2, 1)), "pool code orders (K paired halves with V paired rows, or neither)")
    rec_order = int(orders == (2, 1))
    w.require(not rec_order or has_alpha, "the block records' code orders need the renorm-factor path")
    w.require(not exact or has_alpha, "exact attention needs the renorm factors")
    if has_alpha or blk_bytes:
        entry, name = lib.nsnkv_decode_attn_alpha, "nsnkv_decode_attn_alpha"
        alphas = (L.ptr(kp["alpha"]), L.ptr(vp["alpha"])) if has_alpha else (L.ptr(None), L.ptr(None))
        flags = (L.ATTN_RECORD_ORDER if rec_order else 0) | (L.ATTN_EXACT if exact else 0)
        blocks = blocks + alphas + (int(blk_bytes), flags)
    else:
        entry, name = lib.nsnkv_decode_attn, "nsnkv_decode_attn"
    counts = (L.ptr(nb_t), 0 if nb_t is not None else int(n_blocks), int(max_blocks))
    if name == "nsnkv_decode_attn_alpha":
        counts = counts + (int(blocks_total),)
    rc = entry(
        B, hq, h, bits, L.DTYPE_CODE[q.dtype], L.ptr(q), *blocks,
        blk_stride_head, blk_stride_page, L.ptr(block_table), block_table.shape[-1] if block_table is not None else 0,
        *counts, L.ptr(k_tail), L.ptr(v_tail), tail_stride_seq, tail_stride_head,
        L.ptr(tl_t), 0 if tl_t is not None else int(tail_len), int(max_tail),
        L.ptr(k_new), L.ptr(v_new), L.ptr(out), L.ptr(out_f32), L.ptr(lse),
        L.ptr(ws), ws.numel(), L.ptr(status), L.stream_handle(dev))
    L.check(rc, name)
    return out, status


def group_pool(g, h):
    """Pool view of a reference-layout group [1, h, n, ...] (block (j, i) at j * head stride + i)."""
    return dict(codes=g["codes"], norm=g["metas"][0], min=g["metas"][1], scale=g["metas"][2])


def _raise_status(st: int, stage_input="input_finite"):
    global LAST_STAGE
    if st & L.ST_INPUT_NONFINITE:
        LAST_STAGE = stage_input
        raise w.NumericalFailure("VF01 nonfinite raw input")
    if st & (L.ST_OUTPUT_NONFINITE | L.ST_META_OVERFLOW | L.ST_META_UNDERFLOW):
        raise w.NumericalFailure("VF01 nonfinite fused intermediate/output")
    if st & L.ST_TIMEOUT:
        raise w.IntegrityError("VF01 device wait timed out")
    if st:
        raise w.IntegrityError(f"VF01 device status {st:#x}")


def restore_v(g, tail):
    """Full-length reconstruction [1, h, C + t, 128] in the tail dtype (restore kernel + tail copy)."""
    h = tail.shape[1]
    if g is None:
        return tail.clone()
    b, hh, n, cb = g["codes"].shape
    y = w.restore_blocks(g["codes"].reshape(hh, n, cb), tuple(m.reshape(hh, n, *m.shape[-2:]) for m in g["metas"]),
                         tail.dtype, bits=cb * 8 // (w.BLOCK * w.DIM), tail=tail.reshape(h, tail.shape[2], 128))
    return y.reshape(1, h, n * 64 + tail.shape[2], 128)


def launch(g, kt, q, vg, vt, trace=False, check=True, status=None):
    """Fused attention over packed K/V groups plus native tails.

    Returns (out [1,1,hq,128] in q.dtype, context fp32 [1,hq,1,128], score, v);
    score/v are the diagnostic fp32 scores [1,hq,T] and restored V when trace.
    With ``check=False`` the device status is left in ``status`` (ORed into it when
    given) for the caller to read later.
    """
    h = kt.shape[1]
    hq = q.shape[1]
    n = 0 if g is None else g["codes"].shape[2]
    t = kt.shape[2]
    bits = 3 if g is None else g["codes"].shape[-1] * 8 // (w.BLOCK * w.DIM)
    ctx = torch.empty((1, hq, 1, 128), dtype=torch.float32, device=q.device)
    stride = n
    if g is not None:  # groups may be views with spare capacity between heads (PackedCache)
        stride = checks.head_stride_blocks(g)
        if checks.head_stride_blocks(vg) != stride:
            g, vg = ({"codes": x["codes"].contiguous(), "metas": tuple(m.contiguous() for m in x["metas"])}
                     for x in (g, vg))
            stride = n
    out, status = decode_attention(
        q.reshape(1, hq, 128), group_pool(g, h) if g is not None else None,
        group_pool(vg, h) if vg is not None else None, h=h, bits=bits, blk_stride_head=stride, blk_stride_page=1,
        n_blocks=n, max_blocks=n, k_tail=kt if t else None, v_tail=vt if t else None,
        tail_stride_seq=h * t, tail_stride_head=t, tail_len=t, max_tail=t, out_f32=ctx.reshape(1, hq, 128),
        status=status, blk_bytes=0)
    if check:
        _raise_status(int(status.item()))
    out = out.reshape(1, 1, hq, 128)
    score = v = None
    if trace:
        kfull = restore_v(g, kt).float()
        v = restore_v(vg, vt)
        rep = hq // h
        score = (torch.matmul(q.float(), repeat_kv(kfull, rep).transpose(-2, -1)).squeeze(-2) * w_scale())
    return out, ctx, score, v


def w_scale():
    return 0.08838834764831845


def repeat_kv(hidden_states, n_rep):
    """[b, h, T, d] -> [b, h*n_rep, T, d]; query head j reads kv head j // n_rep."""
    batch, num_key_value_heads, slen, head_dim = hidden_states.shape
    if n_rep == 1:
        return hidden_states
    hidden_states = hidden_states[:, :, None, :, :].expand(batch, num_key_value_heads, n_rep, slen, head_dim)
    return hidden_states.reshape(batch, num_key_value_heads * n_rep, slen, head_dim)


def reference(g, tail):
    """Torch bridge reconstruction: restore_group(g) concatenated with the tail."""
    return tail if g is None else torch.cat((restore_group(g, tail.dtype), tail), dim=2)


def sdpa(q, key, value):
    rep = q.shape[1] // key.shape[1]
    key = repeat_kv(key, rep)
    value = repeat_kv(value, rep)
    out = torch.nn.functional.scaled_dot_product_attention(q, key, value, attn_mask=None, dropout_p=0.0,
                                                           is_causal=False)
    return out.transpose(1, 2).contiguous()


def tile_attention(kfull, vfull, q, check=True):
    """Attention over fully materialised K/V [1,h,T,128] with the same kernel (raw-row chunks)."""
    h, T = kfull.shape[1], kfull.shape[2]
    hq = q.shape[1]
    ctx = torch.empty((1, hq, 1, 128), dtype=torch.float32, device=q.device)
    out, status = decode_attention(q.reshape(1, hq, 128), None, None, h=h, bits=3, blk_stride_head=0,
                                   blk_stride_page=0, n_blocks=0, max_blocks=0, k_tail=kfull, v_tail=vfull,
                                   tail_stride_seq=h * T, tail_stride_head=T, tail_len=T, max_tail=T,
                                   out_f32=ctx.reshape(1, hq, 128))
    if check:
        _raise_status(int(status.item()))
    return out.reshape(1, 1, hq, 128), ctx


def pipeline(arm, data, trace=False):
    global LAST_STAGE, attention_launch_count
    g, kt, q, vg, vt = data
    LAST_STAGE = "structural"
    checks.structural(g, kt, q, vg, vt)
    LAST_STAGE = "input_finite"
    score = v = ctx = None
    if arm in FUSED_ARMS:
        LAST_STAGE = "attention"
        attention_launch_count += 1
        out, ctx, score, v = launch(g, kt, q, vg, vt, trace=trace)
    elif arm in TILE_ARMS:
        LAST_STAGE = "restore"
        kfull = restore_v(g, kt)
        v = restore_v(vg, vt)
        LAST_STAGE = "attention"
        attention_launch_count += 1
        out, ctx = tile_attention(kfull, v, q)
    elif arm == "TORCH_SDPA":
        LAST_STAGE = "restore"
        key = reference(g, kt)
        v = reference(vg, vt)
        for x in (q, key, v):
            if not bool(torch.isfinite(x).all()):
                LAST_STAGE = "input_finite"
                raise w.NumericalFailure("VF01 nonfinite raw input")
        LAST_STAGE = "attention"
        attention_launch_count += 1
        out = sdpa(q, key, v)
    else:
        raise w.IntegrityError("Unknown VF01 arm")
    LAST_STAGE = "output"
    if not bool(torch.isfinite(out).all()):
        raise w.NumericalFailure("Nonfinite VF01 output")
    LAST_STAGE = "returned"
    return (out, ctx, score, v) if trace else out
