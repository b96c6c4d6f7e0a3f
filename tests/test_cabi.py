"""CPU-side checks of the C-ABI boundary: the library loads and exports every
entry point include/nsnkv.h declares, with the argument counts the binding uses.
No compute call is made (there is no GPU here)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_functions():
    text = (ROOT / "include" / "nsnkv.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = {}
    for m in re.finditer(r"\b(int|int64_t)\s+(nsnkv_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a for a in m.group(3).split(",") if a.strip() and a.strip() != "void"]
        decls[m.group(2)] = len(args)
    return decls


def test_header_declares_entry_points():
    decls = header_functions()
    for name in ("nsnkv_encode_blocks", "nsnkv_restore", "nsnkv_pack", "nsnkv_unpack", "nsnkv_decode_attn",
                 "nsnkv_seal_full_tails", "nsnkv_merge_shards", "nsnkv_merge_shard_records"):
        assert name in decls


def test_library_exports_every_declared_symbol():
    from nsn_b200 import _lib, build
    build.build()
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    decls = header_functions()
    for name in decls:
        assert hasattr(lib, name), name
    sig = {n: len(a) for n, _, a in _lib.SIGNATURES}
    assert set(sig) == set(decls), set(sig) ^ set(decls)
    for name, n in decls.items():
        assert sig[name] == n, (name, sig[name], n)


def test_host_only_entry_points():
    from nsn_b200 import _lib
    lib = _lib.load()
    assert lib.nsnkv_version() >= 1
    assert [lib.nsnkv_block_code_bytes(b) for b in (2, 3, 4, 5, 6)] == [0, 3072, 4096, 5120, 0]
    assert lib.nsnkv_decode_attn_workspace_bytes(1, 32, 8, 511, 64) > 0
    assert lib.nsnkv_decode_attn_workspace_bytes(0, 32, 8, 511, 64) == 0


def test_argument_errors_return_before_launch():
    """Invalid arguments are rejected on the host with NSNKV_ERR_ARG (no device touched)."""
    from nsn_b200 import _lib
    lib = _lib.load()
    P = ctypes.c_void_p
    # bits out of range
    assert lib.nsnkv_pack(P(16), 8, 2, P(16), P(16), P(None)) == _lib.ERR_ARG
    assert lib.nsnkv_unpack(P(16), 8, 6, P(16), P(None)) == _lib.ERR_ARG
    # misaligned input pointer
    assert lib.nsnkv_encode_blocks(P(3), 0, 1, 1, 3, 0, P(16), P(None), P(16), P(16), P(16), P(None), 0, 1, 0,
                                   P(16), P(None)) == _lib.ERR_ARG
    # hq not a multiple of h
    assert lib.nsnkv_decode_attn(1, 30, 8, 3, 0, P(16), *([P(16)] * 8), 1, 1, P(None), 0, P(None), 1, 1,
                                 P(16), P(16), 64, 64, P(None), 1, 1, P(None), P(None), P(16), P(None), P(None),
                                 P(16), 1 << 30, P(16), P(None)) == _lib.ERR_ARG
    # empty work is a no-op
    assert lib.nsnkv_pack(P(None), 0, 3, P(None), P(None), P(None)) == _lib.OK


def test_paged_plan_descriptor_and_host_checks():
    """nsnkv_paged_plan_create validates the descriptor on the host (no device touched), and
    nsnkv_paged_step rejects a step that would need a page beyond max_blocks before it
    launches anything."""
    import numpy as np
    from nsn_b200 import _lib
    lib = _lib.load()
    assert ctypes.sizeof(_lib.PagedDesc) == 256  # the C layout of nsnkv_paged_desc on x86-64
    batch, hq, h, max_blocks = 3, 8, 2, 4
    nb = np.array([0, 4, 2], np.int32)
    tl = np.array([5, 62, 0], np.int32)
    fake = 1 << 20  # a 16-byte aligned address that is never dereferenced here
    ws = lib.nsnkv_decode_attn_workspace_bytes(batch, hq, h, max_blocks, 63)

    def desc(**kw):
        d = dict(struct_bytes=ctypes.sizeof(_lib.PagedDesc), batch=batch, hq=hq, h=h, bits=3, dtype=_lib.F16,
                 flags=_lib.ATTN_RECORD_ORDER, max_blocks=max_blocks, blk_bytes=7680, blk_stride_head=12,
                 blk_stride_page=1, table_stride=max_blocks, tail_stride_seq=h * 64, tail_stride_head=64,
                 workspace_bytes=ws, host_n_blocks=nb.ctypes.data, host_tail_len=tl.ctypes.data)
        for f in ("k_codes", "k_norm", "k_min", "k_scale", "k_alpha", "v_codes", "v_norm", "v_min", "v_scale",
                  "v_alpha", "block_table", "n_blocks", "tail_len", "k_tail", "v_tail", "seq_counters", "workspace",
                  "status"):
            d[f] = fake
        d.update(kw)
        return _lib.PagedDesc(**d)

    def create(**kw):
        handle = ctypes.c_void_p()
        return lib.nsnkv_paged_plan_create(ctypes.byref(desc(**kw)), ctypes.byref(handle)), handle

    assert create(struct_bytes=200)[0] == _lib.ERR_ARG
    assert create(hq=7)[0] == _lib.ERR_ARG
    assert create(k_alpha=None)[0] == _lib.ERR_ARG  # one factor array without the other
    assert create(k_alpha=None, v_alpha=None)[0] == _lib.ERR_ARG  # flags need the factors
    assert create(workspace_bytes=ws - 1)[0] == _lib.ERR_ARG
    assert create(tail_stride_head=63)[0] == _lib.ERR_ARG
    tl[2] = 64
    assert create()[0] == _lib.ERR_ARG  # a host counter out of range
    tl[2] = 0
    rc, handle = create()
    assert rc == _lib.OK and handle.value
    P = ctypes.c_void_p
    assert lib.nsnkv_paged_step(handle, P(None), P(fake), P(fake), P(fake), P(None), P(None)) == _lib.ERR_ARG
    # sequence 1 holds max_blocks pages and a tail of 62: one more token fits, a second would not
    tl[1] = 63
    assert lib.nsnkv_paged_step(handle, P(fake), P(fake), P(fake), P(fake), P(None), P(None)) == _lib.ERR_TOO_LARGE
    assert list(nb) == [0, 4, 2] and list(tl) == [5, 63, 0]  # unchanged by a rejected step
    # the host-buffer step: the same checks, before any staging is made (no device touched)
    assert lib.nsnkv_paged_step_host(handle, P(None), P(fake), P(None), P(None)) == _lib.ERR_ARG
    assert lib.nsnkv_paged_step_host(P(None), P(fake), P(fake), P(None), P(None)) == _lib.ERR_ARG
    assert lib.nsnkv_paged_step_host(handle, P(fake), P(fake), P(None), P(None)) == _lib.ERR_TOO_LARGE
    assert lib.nsnkv_paged_plan_destroy(handle) == _lib.OK
    assert lib.nsnkv_paged_plan_destroy(P(None)) == _lib.ERR_ARG


def test_layer_op_argument_errors():
    """The fused layer ops reject bad shapes, dtypes and null pointers before launching."""
    from nsn_b200 import _lib
    lib = _lib.load()
    P = ctypes.c_void_p
    f = P(1 << 20)
    assert lib.nsnkv_add_rmsnorm(4, 8193, _lib.F16, f, None, f, 1e-5, None, f, None) == _lib.ERR_ARG
    assert lib.nsnkv_add_rmsnorm(4, 2048, _lib.F32, f, None, f, 1e-5, None, f, None) == _lib.ERR_ARG
    assert lib.nsnkv_add_rmsnorm(4, 2048, _lib.F16, None, None, f, 1e-5, None, f, None) == _lib.ERR_ARG
    assert lib.nsnkv_add_rmsnorm(4, 2048, _lib.F16, f, None, f, -1.0, None, f, None) == _lib.ERR_ARG
    assert lib.nsnkv_add_rmsnorm(0, 2048, _lib.F16, f, None, f, 1e-5, None, f, None) == _lib.OK  # nothing to do
    assert lib.nsnkv_rope_split(4, 0, 2, _lib.F16, f, f, f, 0, f, f, f, None) == _lib.ERR_ARG
    assert lib.nsnkv_rope_split(4, 16, 4, _lib.F16, f, None, f, 0, f, f, f, None) == _lib.ERR_ARG
    assert lib.nsnkv_rope_split(70000, 16, 4, _lib.F16, f, f, f, 0, f, f, f, None) == _lib.ERR_ARG
    assert lib.nsnkv_swiglu(4, 0, _lib.F16, f, f, None) == _lib.ERR_ARG
    assert lib.nsnkv_swiglu(4, 5632, _lib.BF16, None, f, None) == _lib.ERR_ARG
    fw = _lib.GEMV_FIXED_WEIGHTS
    assert lib.nsnkv_gemv_rows(9, 512, 256, _lib.F16, f, f, f, fw, None) == _lib.ERR_ARG  # m > 8
    assert lib.nsnkv_gemv_rows(4, 510, 256, _lib.F16, f, f, f, fw, None) == _lib.ERR_ARG  # n % 8
    assert lib.nsnkv_gemv_rows(4, 512, 200, _lib.F16, f, f, f, fw, None) == _lib.ERR_ARG  # k % 256
    assert lib.nsnkv_gemv_rows(4, 512, 256, _lib.F16, f, f, f, 2, None) == _lib.ERR_ARG  # unknown flag
    assert lib.nsnkv_gemv_rows(4, 512, 256, _lib.F16, P(8), f, f, fw, None) == _lib.ERR_ARG  # misaligned x
    assert lib.nsnkv_gemv_rows(0, 512, 256, _lib.F16, f, f, f, fw, None) == _lib.OK  # nothing to do
