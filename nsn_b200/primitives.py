"""NSN arithmetic on the GPU: the operator surface of the reference's primitives module.

Mirrors experiments/nb06/source/loop_kv_nb06_primitives.py (names, argument
meaning, return values and error behaviour) with every computation done by
libnsnkv.so on the tensor's CUDA device:

  pack_codes             :15-24  LSB-first bitstream (CUDA pack kernel)
  unpack_codes_reference :26-35  its inverse (CUDA unpack kernel)
  nsn_encode             :37-55  fused encoder kernel, bit-exact codes and fp16 metadata
  nsn_decode             :57-66  restore kernel, bit-exact reconstruction
  nsn_qdq                :68-70
  planned_bytes          :72-81  byte accounting (host arithmetic)

Errors: ``NumericalFailure`` for non-finite input, fp16 metadata overflow or
nonzero-to-zero underflow and non-finite reconstruction (same messages as the
reference); ``ContractError`` (a ValueError, like the reference's ``require``)
for shape/dtype/range contract violations.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib as L

BLOCK = 64
DIM = 128
HEADS = 8
LAYERS = 22
EPS = 1e-12


class NumericalFailure(RuntimeError):
    pass


class IntegrityError(RuntimeError):
    pass


class ContractError(ValueError):
    pass


def require(ok, message):
    if not ok:
        raise ContractError(message)


def _status_to_error(status: int, input_msg: str, meta=True, output_msg="Nonfinite NSN reconstruction"):
    if status & L.ST_INPUT_NONFINITE:
        raise NumericalFailure(input_msg)
    if meta and status & L.ST_META_OVERFLOW:
        raise NumericalFailure("FP16 metadata overflow/nonfinite")
    if meta and status & L.ST_META_UNDERFLOW:
        raise NumericalFailure("Nonzero FP16 norm/step underflow")
    if status & L.ST_OUTPUT_NONFINITE:
        raise NumericalFailure(output_msg)
    if status & L.ST_TIMEOUT:
        raise IntegrityError("device wait timed out")
    if status:
        raise IntegrityError(f"device status {status:#x}")


def code_bytes(bits: int) -> int:
    return BLOCK * DIM * bits // 8


def norm_order_of(x: torch.Tensor) -> int:
    """0 when torch's CPU reference reduces this tensor's rows in 8-lane order, 1 when sequentially.

    The reference widens with ``x.float()`` (strides preserved for dense tensors)
    and reduces the last axis; rows whose channels are not contiguous are summed
    sequentially.
    """
    return 0 if x.shape[-1] <= 1 or x.stride(-1) == 1 else 1


# ------------------------------------------------------------------ packing
def pack_codes(codes, bits: int):
    """LSB-first bitstream of uint8 codes.  NumPy/bytes in -> bytes out (as the
    reference); a CUDA tensor in -> CUDA uint8 tensor out.  Packing runs on the GPU."""
    as_bytes = not isinstance(codes, torch.Tensor)
    t = torch.as_tensor(np.asarray(codes, dtype=np.uint8).reshape(-1)).cuda() if as_bytes else codes
    require(bits in (3, 4, 5) and t.dtype == torch.uint8, "Invalid packed code")
    L.require_cuda()
    t = t.contiguous().reshape(-1)
    out = torch.empty((t.numel() * bits + 7) // 8, dtype=torch.uint8, device=t.device)
    status = L.status_tensor(t.device)
    L.check(L.load().nsnkv_pack(L.ptr(t), t.numel(), bits, L.ptr(out), L.ptr(status), L.stream_handle(t.device)),
            "pack_codes")
    require(int(status.item()) == 0, "Invalid packed code")
    return out.cpu().numpy().tobytes() if as_bytes else out


def unpack_codes(payload, count: int, bits: int):
    """Inverse of pack_codes (the reference's scalar ``unpack_codes_reference``).
    bytes/NumPy in -> NumPy uint8 out; CUDA tensor in -> CUDA tensor out."""
    as_np = not isinstance(payload, torch.Tensor)
    if as_np:
        payload = torch.as_tensor(np.frombuffer(bytes(payload), np.uint8).copy()).cuda()
    require(bits in (3, 4, 5) and payload.dtype == torch.uint8 and payload.numel() >= (count * bits + 7) // 8,
            "packed payload shape")
    L.require_cuda()
    out = torch.empty(count, dtype=torch.uint8, device=payload.device)
    payload = payload.contiguous()  # referenced until the launch is enqueued
    L.check(L.load().nsnkv_unpack(L.ptr(payload), count, bits, L.ptr(out),
                                  L.stream_handle(payload.device)), "unpack_codes")
    return out.cpu().numpy() if as_np else out


unpack_codes_reference = unpack_codes


# ------------------------------------------------------------------ encode / decode
def encode_blocks(x: torch.Tensor, bits: int, *, packed=True, unpacked=False, headers_start=None,
                  out=None, out_row_stride=None, out_offset=0, check=True):
    """Fused NSN encoder over x [..., 64, 128] (any layout, fp16/bf16/fp32, CUDA).

    Returns a dict with 'codes' (packed, [..., code_bytes]) and/or 'q' (unpacked
    [..., 64, 128] uint8), 'metas' = (n [...,64,1], m [...,1,128], s [...,1,128])
    fp16 and optionally 'headers' [..., 12].  With ``out`` (a dict of pool tensors
    codes/norm/min/scale[/headers]) the blocks are written there instead, block
    (row, i) at row*out_row_stride + out_offset + i, rows = the leading dims but
    the last block axis.
    """
    require(x.ndim >= 2 and tuple(x.shape[-2:]) == (BLOCK, DIM), "NSN block shape")
    require(bits in (3, 4, 5), "NSN bits")
    require(x.dtype in L.DTYPE_CODE, "NSN input dtype")
    L.require_cuda()
    order = norm_order_of(x)
    lead = tuple(x.shape[:-2])
    nblk = int(np.prod(lead)) if lead else 1
    bpr = lead[-1] if len(lead) >= 1 else 1
    rows = nblk // bpr if bpr else 0
    xc = x.contiguous()
    dev = x.device
    status = L.status_tensor(dev)
    res = {}
    if out is None:
        codes = torch.empty(lead + (code_bytes(bits),), dtype=torch.uint8, device=dev) if packed else None
        n = torch.empty(lead + (BLOCK, 1), dtype=torch.float16, device=dev)
        m = torch.empty(lead + (1, DIM), dtype=torch.float16, device=dev)
        s = torch.empty(lead + (1, DIM), dtype=torch.float16, device=dev)
        hdr = torch.empty(lead + (12,), dtype=torch.uint8, device=dev) if headers_start is not None else None
        stride, offset = bpr, 0
    else:
        codes, n, m, s = out["codes"], out["norm"], out["min"], out["scale"]
        hdr = out.get("headers") if headers_start is not None else None
        stride, offset = (out_row_stride if out_row_stride is not None else bpr), out_offset
    blk = 0 if out is None else blk_bytes_of(out, bits)
    q = torch.empty(lead + (BLOCK, DIM), dtype=torch.uint8, device=dev) if unpacked else None
    if nblk:
        L.check(L.load().nsnkv_encode_blocks_strided(
            L.ptr(xc), L.DTYPE_CODE[x.dtype], rows, bpr, bits, order, L.ptr(codes), L.ptr(q), L.ptr(n), L.ptr(m),
            L.ptr(s), L.ptr(hdr), int(headers_start or 0), stride, offset, blk,
            int(out.get("code_order", 0)) if out is not None else 0, L.ptr(status), L.stream_handle(dev)),
            "nsnkv_encode_blocks")
        if out is not None and out.get("alpha") is not None and codes is not None:
            block_renorm(out, bits, rows, bpr, stride, offset)
    if check:
        st = int(status.item())
        _status_to_error(st, "Nonfinite input to NSN")
    else:
        res["status"] = status
    res.update(codes=codes, q=q, metas=(n, m, s), headers=hdr)
    return res


def pair_rows(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Packed blocks [..., code_bytes] in the reference's row order -> paired rows.

    Paired rows (the V codes of the paged cache's block records): the packed rows of
    tokens 2j and 2j+1 interleaved at 16 bits, 32-bit word j*8*bits + k = [row 2j
    half k | row 2j+1 half k].  The same bytes in another order.
    """
    lead = tuple(codes.shape[:-1])
    require(codes.dtype == torch.uint8 and codes.shape[-1] == code_bytes(bits), "packed block shape")
    h = codes.contiguous().view(torch.int16).reshape(lead + (BLOCK // 2, 2, 8 * bits))
    return h.transpose(-1, -2).contiguous().view(torch.uint8).reshape(lead + (code_bytes(bits),))


def unpair_rows(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Inverse of pair_rows: paired rows -> the reference's packed row order."""
    lead = tuple(codes.shape[:-1])
    require(codes.dtype == torch.uint8 and codes.shape[-1] == code_bytes(bits), "packed block shape")
    h = codes.contiguous().view(torch.int16).reshape(lead + (BLOCK // 2, 8 * bits, 2))
    return h.transpose(-1, -2).contiguous().view(torch.uint8).reshape(lead + (code_bytes(bits),))


def pair_halves(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Packed blocks [..., code_bytes] in the reference's row order -> paired halves.

    Paired halves (the K codes of the paged cache's block records): in each token row,
    each 32-code group (2*bits 16-bit halves: A = the first bits, B = the rest) stored
    as 32-bit words [A half m | B half m], m < bits.
    """
    lead = tuple(codes.shape[:-1])
    require(codes.dtype == torch.uint8 and codes.shape[-1] == code_bytes(bits), "packed block shape")
    h = codes.contiguous().view(torch.int16).reshape(lead + (BLOCK * 4, 2, bits))
    return h.transpose(-1, -2).contiguous().view(torch.uint8).reshape(lead + (code_bytes(bits),))


def unpair_halves(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Inverse of pair_halves."""
    lead = tuple(codes.shape[:-1])
    require(codes.dtype == torch.uint8 and codes.shape[-1] == code_bytes(bits), "packed block shape")
    h = codes.contiguous().view(torch.int16).reshape(lead + (BLOCK * 4, bits, 2))
    return h.transpose(-1, -2).contiguous().view(torch.uint8).reshape(lead + (code_bytes(bits),))


def to_code_order(codes: torch.Tensor, bits: int, order: int) -> torch.Tensor:
    """The reference's row order -> code order 0 (unchanged), 1 (paired rows) or 2 (paired halves)."""
    require(order in (0, 1, 2), "code order")
    return codes if order == 0 else pair_rows(codes, bits) if order == 1 else pair_halves(codes, bits)


def from_code_order(codes: torch.Tensor, bits: int, order: int) -> torch.Tensor:
    """Inverse of to_code_order."""
    require(order in (0, 1, 2), "code order")
    return codes if order == 0 else unpair_rows(codes, bits) if order == 1 else unpair_halves(codes, bits)


def blk_bytes_of(pool, bits: int) -> int:
    """Block stride (bytes) shared by a pool's codes / min / scale / alpha arrays.

    0 when every array is dense (code_bytes, 256, 256 and 256 bytes per block); the
    common stride when they are fields of block records (the paged cache's layout for
    INT3 fp16 caches, see nsnkv_encode_blocks_strided).  Norms are always dense.
    """
    per = {"codes": code_bytes(bits), "min": DIM, "scale": DIM, "alpha": BLOCK}
    found = set()
    dense = True
    for key, e in per.items():
        t = pool.get(key)
        if t is None:
            continue
        try:
            v = t.view(-1, e)
        except RuntimeError:
            raise ContractError(f"pool {key} layout") from None
        require(v.stride(1) == 1, f"pool {key} layout")
        if v.shape[0] <= 1:
            continue
        sb = v.stride(0) * t.element_size()
        found.add(sb)
        dense = dense and sb == e * t.element_size()
    nrm = pool.get("norm")
    require(nrm is None or nrm.is_contiguous(), "pool norm layout")
    if dense:
        return 0
    require(len(found) == 1, "pool block strides")
    sb = found.pop()
    require(sb % 16 == 0 and sb >= code_bytes(bits), "pool block strides")
    return sb


def block_renorm(pool, bits: int, rows: int, blocks_per_row: int, row_stride: int, offset: int = 0):
    """Fill pool["alpha"] (fp32, 64 per block) for blocks (r, i) at r*row_stride + offset + i.

    alpha_t = n_t / max(||d_t||, 1e-12) with d = min + scale * code, 0 when n_t == 0:
    the per-token factor of nsn_decode (loop_kv_nb06_primitives.py:57-66) that
    nsnkv_decode_attn_alpha reads instead of recomputing ||d||.
    """
    require(all(pool[k].is_cuda for k in ("codes", "norm", "min", "scale", "alpha")), "renorm pools on CUDA")
    require(pool["alpha"].dtype == torch.float32, "renorm alpha dtype")
    if rows and blocks_per_row:
        L.check(L.load().nsnkv_block_renorm(
            bits, rows, blocks_per_row, L.ptr(pool["codes"]), L.ptr(pool["norm"]), L.ptr(pool["min"]),
            L.ptr(pool["scale"]), row_stride, offset, L.ptr(pool["alpha"]), blk_bytes_of(pool, bits),
            int(pool.get("code_order", 0)), L.stream_handle(pool["codes"].device)),
            "nsnkv_block_renorm")


def nsn_encode(x: torch.Tensor, bits: int):
    """(q uint8 [...,64,128], (n fp16 [...,64,1], m fp16 [...,1,128], s fp16 [...,1,128]))."""
    r = encode_blocks(x, bits, packed=False, unpacked=True)
    return r["q"], r["metas"]


def restore_blocks(codes, metas, dtype, *, bits=3, unpacked=False, tail=None, check=True, out=None):
    """Reconstruct [R, nb, ...] blocks (+ optional tail [R, t, 128]) into [R, nb*64 + t, 128] of dtype."""
    n, m, s = metas
    require(dtype in L.DTYPE_CODE, "restore dtype")
    L.require_cuda()
    if unpacked:
        lead = tuple(codes.shape[:-2])
    else:
        lead = tuple(codes.shape[:-1])
        require(codes.shape[-1] == code_bytes(bits), "packed block bytes")
    nblk = int(np.prod(lead)) if lead else 1
    bpr = lead[-1] if lead else 1
    rows = nblk // bpr if bpr else (tail.shape[0] if tail is not None else 0)
    t = 0 if tail is None else tail.shape[-2]
    dev = (codes if codes is not None else tail).device
    if out is None:
        out = torch.empty((rows, bpr * BLOCK + t, DIM), dtype=dtype, device=dev)
    status = L.status_tensor(dev)
    if tail is not None:
        require(tail.dtype == dtype and tail.is_contiguous(), "tail dtype/layout")
    # contiguous copies of strided inputs stay referenced until the launch is enqueued (a
    # temporary freed earlier could be handed to the next copy before the kernel reads it)
    codes, n, m, s = (None if x is None else x.contiguous() for x in (codes, n, m, s))
    L.check(L.load().nsnkv_restore(
        L.ptr(codes), int(unpacked), L.ptr(n), L.ptr(m), L.ptr(s), rows, bpr, bits, L.ptr(tail), t, L.DTYPE_CODE[dtype],
        L.ptr(out), L.ptr(status), L.stream_handle(dev)), "nsnkv_restore")
    if check:
        _status_to_error(int(status.item()), "Nonfinite NSN reconstruction", meta=False)
    return out


def nsn_decode(q: torch.Tensor, metas, dtype):
    """Reconstruction n * d/max(||d||, eps) with d = m + s*q, 0 where n == 0, cast to dtype."""
    require(q.dtype == torch.uint8 and q.ndim >= 2 and tuple(q.shape[-2:]) == (BLOCK, DIM), "NSN codes shape")
    y = restore_blocks(q, metas, dtype, unpacked=True, bits=5)
    return y.reshape(q.shape)


def nsn_qdq(x: torch.Tensor, bits: int):
    q, meta = nsn_encode(x, bits)
    return nsn_decode(q, meta, x.dtype)


def planned_bytes(shape, compressed_tokens, bits):
    """KV bytes: codes, fp16 metadata, native tail and 12-byte block headers (:72-81)."""
    b, h, length, d = shape
    require(compressed_tokens % BLOCK == 0 and 0 <= compressed_tokens <= length, "Block accounting")
    if bits is None:
        return {"codes": 0, "metadata": 0, "native": b * h * length * d * 2, "block_headers": 0}
    blocks = b * h * (compressed_tokens // BLOCK)
    return {"codes": blocks * ((BLOCK * d * bits + 7) // 8),
            "metadata": blocks * (BLOCK * 2 + d * 4),
            "native": b * h * (length - compressed_tokens) * d * 2, "block_headers": blocks * 12}
