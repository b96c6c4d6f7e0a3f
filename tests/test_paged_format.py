"""Sequence container format of the paged cache, on CPU.

A sequence in the reference's layout (packed groups with '<QHBB' headers plus native
tails, built here with the oracle's encoder) survives sequence_to_bytes /
sequence_from_bytes unchanged.  Its size after the preamble is what the reference's
planned_bytes counts for K and V.  Corrupted headers and truncated input are rejected.
"""
import numpy as np
import pytest
import torch

from oracle import nsn_oracle as O


def _reference_sequence(h=2, n=3, t=17, bits=3, seed=5):
    from nsn_b200 import checks
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(2):
        x = rng.standard_normal((1, h, n * 64 + t, 128)).astype(np.float16)
        q, nn, m, s, st = O.nsn_encode(x[:, :, :n * 64].astype(np.float32).reshape(1, h, n, 64, 128), bits)
        codes = np.frombuffer(O.pack_codes(q, bits), np.uint8).reshape(1, h, n, -1).copy()
        g = dict(codes=torch.from_numpy(codes),
                 metas=tuple(torch.from_numpy(a.copy()) for a in (nn, m, s)),
                 headers=checks.expected_headers(n, h, bits, 0, "cpu").contiguous())
        out += [g, torch.from_numpy(x[:, :, n * 64:].copy())]
    return out[0], out[1], out[2], out[3]


def _same(a, b):
    return a.dtype == b.dtype and tuple(a.shape) == tuple(b.shape) and torch.equal(a.view(torch.uint8) if a.dtype == torch.uint8 else a.view(torch.int16), b.view(torch.uint8) if b.dtype == torch.uint8 else b.view(torch.int16))


@pytest.mark.parametrize("bits", [3, 5])
def test_sequence_container_round_trip_and_size(bits):
    from nsn_b200 import primitives as w
    from nsn_b200.paged import sequence_from_bytes, sequence_to_bytes
    h, n, t = 2, 3, 17
    kg, kt, vg, vt = _reference_sequence(h, n, t, bits)
    blob = sequence_to_bytes(kg, kt, vg, vt)
    planned = w.planned_bytes((1, h, n * 64 + t, 128), n * 64, bits)
    assert len(blob) == 24 + 2 * sum(planned.values())
    kg2, kt2, vg2, vt2 = sequence_from_bytes(blob)
    for a, b in ((kg, kg2), (vg, vg2)):
        assert _same(a["codes"], b["codes"]) and _same(a["headers"], b["headers"])
        for x, y in zip(a["metas"], b["metas"]):
            assert _same(x, y)
    assert _same(kt, kt2) and _same(vt, vt2)


def test_sequence_container_without_sealed_blocks():
    from nsn_b200.paged import sequence_from_bytes, sequence_to_bytes
    kt = torch.randn(1, 2, 9, 128).half()
    vt = torch.randn(1, 2, 9, 128).half()
    kg, kt2, vg, vt2 = sequence_from_bytes(sequence_to_bytes(None, kt, None, vt))
    assert kg is None and vg is None and torch.equal(kt2, kt) and torch.equal(vt2, vt)


def test_sequence_container_rejects_corruption():
    from nsn_b200 import primitives as w
    from nsn_b200.paged import sequence_from_bytes, sequence_to_bytes
    blob = bytearray(sequence_to_bytes(*_reference_sequence()))
    with pytest.raises(w.ContractError):
        sequence_from_bytes(bytes(blob[:-1]))
    bad = bytearray(blob)
    bad[24 + 8] = 63  # first block header's token count
    with pytest.raises(w.ContractError):
        sequence_from_bytes(bytes(bad))
    bad = bytearray(blob)
    bad[:8] = b"NOTNSNKV"
    with pytest.raises(w.ContractError):
        sequence_from_bytes(bytes(bad))


def test_block_record_pools_layout():
    """The paged cache's block records: K fields then V fields per (head, page), views in the pool dicts."""
    from nsn_b200 import primitives as w
    from nsn_b200.paged import block_record_pools
    rec, kp, vp = block_record_pools(2, 5, 3, "cpu")
    assert tuple(rec.shape) == (2, 5, 7680)
    assert w.blk_bytes_of(kp, 3) == 7680 and w.blk_bytes_of(vp, 3) == 7680
    base = rec.data_ptr()
    offs = {k: kp[k].data_ptr() - base for k in ("codes", "min", "scale", "alpha")}
    assert offs == {"codes": 0, "min": 3072, "scale": 3328, "alpha": 3584}
    assert vp["codes"].data_ptr() - base == 3840 and vp["alpha"].data_ptr() - base == 3840 + 3584
    # writes through the views land in the records
    kp["alpha"][1, 3, 5] = 2.5
    vp["min"][0, 4, 127] = 1.0
    assert rec[1, 3, 3584 + 20:3584 + 24].view(torch.float32).item() == 2.5
    assert rec[0, 4, 3840 + 3072 + 254:3840 + 3072 + 256].view(torch.float16).item() == 1.0
    assert kp["norm"].is_contiguous() and tuple(kp["norm"].shape) == (2, 5, 64)


def test_blk_bytes_of_dense_and_rejected_layouts():
    from nsn_b200 import primitives as w
    from nsn_b200.paged import block_record_pools
    dense = dict(codes=torch.zeros((2, 4, 3072), dtype=torch.uint8), norm=torch.zeros((2, 4, 64), dtype=torch.float16),
                 min=torch.zeros((2, 4, 128), dtype=torch.float16), scale=torch.zeros((2, 4, 128), dtype=torch.float16),
                 alpha=torch.zeros((2, 4, 64), dtype=torch.float32))
    assert w.blk_bytes_of(dense, 3) == 0
    _, kp, _ = block_record_pools(2, 4, 3, "cpu")
    mixed = dict(kp, codes=dense["codes"])  # dense codes with record metadata
    with pytest.raises(w.ContractError):
        w.blk_bytes_of(mixed, 3)
    bad = dict(dense, min=torch.zeros((2, 128, 4), dtype=torch.float16).transpose(1, 2))
    with pytest.raises(w.ContractError):
        w.blk_bytes_of(bad, 3)


@pytest.mark.parametrize("bits", [3, 4, 5])
def test_pair_rows_layout_and_round_trip(bits):
    """Paired rows: word j*8*bits + k = [row 2j half k | row 2j+1 half k]; unpair_rows inverts it."""
    from nsn_b200 import primitives as w
    from nsn_b200.paged import block_record_pools
    rng = np.random.default_rng(bits)
    cb = w.code_bytes(bits)
    codes = torch.from_numpy(rng.integers(0, 256, size=(2, 3, cb), dtype=np.uint8))
    p = w.pair_rows(codes, bits)
    assert p.shape == codes.shape and torch.equal(w.unpair_rows(p, bits), codes)
    rows = codes.view(torch.int16).reshape(2, 3, 64, 8 * bits)
    words = p.view(torch.int32).reshape(2, 3, 32, 8 * bits)
    j, k = 5, 7
    want = (rows[..., 2 * j, k].to(torch.int32) & 0xFFFF) | (rows[..., 2 * j + 1, k].to(torch.int32) << 16)
    assert torch.equal(words[..., j, k], want)
    ph = w.pair_halves(codes, bits)
    assert torch.equal(w.unpair_halves(ph, bits), codes)
    halves = codes.view(torch.int16).reshape(2, 3, 64, 4, 2 * bits)  # [row, group, half]
    hw = ph.view(torch.int32).reshape(2, 3, 64, 4, bits)
    r, gi, m = 9, 2, bits - 1
    want = (halves[..., r, gi, m].to(torch.int32) & 0xFFFF) | (halves[..., r, gi, bits + m].to(torch.int32) << 16)
    assert torch.equal(hw[..., r, gi, m], want)
    for order in (0, 1, 2):
        assert torch.equal(w.from_code_order(w.to_code_order(codes, bits, order), bits, order), codes)
    _, kp, vp = block_record_pools(1, 2, 3, "cpu")
    assert kp["code_order"] == 2 and vp["code_order"] == 1
