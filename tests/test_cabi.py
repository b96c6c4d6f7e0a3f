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
