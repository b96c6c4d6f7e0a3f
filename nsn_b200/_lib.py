"""ctypes binding of libnsnkv.so (the C ABI declared in include/nsnkv.h).

There is no fallback: if the library is missing or CUDA is unavailable every
operator raises.  Tensors are passed as raw device pointers together with the
current torch CUDA stream.
"""
from __future__ import annotations

import ctypes
from ctypes import c_int, c_int32, c_int64, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libnsnkv.so"

OK = 0
ERR_ARG = -1
ERR_LAUNCH = -2
ERR_UNSUPPORTED = -3
ERR_CUDA = -4
ERR_TOO_LARGE = -5
NOALLOC_SCRATCH_BYTES = 16 << 20

ST_INPUT_NONFINITE = 1
ST_META_OVERFLOW = 2
ST_META_UNDERFLOW = 4
ST_OUTPUT_NONFINITE = 8
ST_TIMEOUT = 32
ST_CAPACITY = 64

ATTN_RECORD_ORDER = 1  # nsnkv_decode_attn_alpha flags
ATTN_EXACT = 2
GEMV_FIXED_WEIGHTS = 1

F16, BF16, F32 = 0, 1, 2
DTYPE_CODE = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}

# (name, restype, argtypes) for every exported symbol of include/nsnkv.h
P = c_void_p
SIGNATURES = [
    ("nsnkv_version", c_int, []),
    ("nsnkv_block_code_bytes", c_int64, [c_int]),
    ("nsnkv_encode_blocks", c_int, [P, c_int, c_int64, c_int64, c_int, c_int, P, P, P, P, P, P, c_int64, c_int64,
                                    c_int64, P, P]),
    ("nsnkv_encode_blocks_strided", c_int, [P, c_int, c_int64, c_int64, c_int, c_int, P, P, P, P, P, P, c_int64,
                                            c_int64, c_int64, c_int64, c_int, P, P]),
    ("nsnkv_restore", c_int, [P, c_int, P, P, P, c_int64, c_int64, c_int, P, c_int64, c_int, P, P, P]),
    ("nsnkv_pack", c_int, [P, c_int64, c_int, P, P, P]),
    ("nsnkv_unpack", c_int, [P, c_int64, c_int, P, P]),
    ("nsnkv_decode_attn", c_int, [c_int64, c_int, c_int, c_int, c_int, P,
                                  P, P, P, P, P, P, P, P,
                                  c_int64, c_int64, P, c_int64,
                                  P, c_int32, c_int32,
                                  P, P, c_int64, c_int64,
                                  P, c_int32, c_int32,
                                  P, P, P, P, P, P, c_int64, P, P]),
    ("nsnkv_decode_attn_workspace_bytes", c_int64, [c_int64, c_int, c_int, c_int32, c_int32]),
    ("nsnkv_decode_attn_alpha", c_int, [c_int64, c_int, c_int, c_int, c_int, P,
                                        P, P, P, P, P, P, P, P, P, P, c_int64, c_int,
                                        c_int64, c_int64, P, c_int64,
                                        P, c_int32, c_int32, c_int64,
                                        P, P, c_int64, c_int64,
                                        P, c_int32, c_int32,
                                        P, P, P, P, P, P, c_int64, P, P]),
    ("nsnkv_block_renorm", c_int, [c_int, c_int64, c_int64, P, P, P, P, c_int64, c_int64, P, c_int64, c_int, P]),
    ("nsnkv_decode_attn_noalloc", c_int, [c_int64, c_int, c_int, c_int, c_int, P,
                                          P, P, P, P, P, P, P, P,
                                          c_int64, c_int64, P, c_int64,
                                          P, c_int32, c_int32,
                                          P, P, c_int64, c_int64,
                                          P, c_int32, c_int32,
                                          P, P, P, P, P, P, P]),
    ("nsnkv_seal_full_tails", c_int, [c_int64, c_int, c_int, c_int, P, P, c_int64, c_int64, P, P, c_int, P, c_int64,
                                      P, P, P, P, P, P, P, P, c_int64, c_int64, P, P]),
    ("nsnkv_seal_full_tails_alpha", c_int, [c_int64, c_int, c_int, c_int, P, P, c_int64, c_int64, P, P, c_int, P,
                                            c_int64, P, P, P, P, P, P, P, P, P, P, c_int64, c_int, P, c_int64,
                                            c_int64, P, P]),
    ("nsnkv_paged_plan_create", c_int, [P, P]),
    ("nsnkv_paged_step", c_int, [P, P, P, P, P, P, P]),
    ("nsnkv_paged_step_host", c_int, [P, P, P, P, P]),
    ("nsnkv_paged_plan_last_launches", c_int, [P]),
    ("nsnkv_paged_plan_destroy", c_int, [P]),
    ("nsnkv_add_rmsnorm", c_int, [c_int64, c_int, c_int, P, P, P, ctypes.c_float, P, P, P]),
    ("nsnkv_rope_split", c_int, [c_int64, c_int, c_int, c_int, P, P, P, c_int64, P, P, P, P]),
    ("nsnkv_swiglu", c_int, [c_int64, c_int, c_int, P, P, P]),
    ("nsnkv_gemv_rows", c_int, [c_int, c_int, c_int, c_int, P, P, P, c_int, P]),
    ("nsnkv_peer_area_words", c_int64, [c_int, c_int]),
    ("nsnkv_peer_merge_records", c_int, [c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P]),
    ("nsnkv_merge_shards", c_int, [c_int, c_int64, P, P, c_int, P, P, P, P, P]),
    ("nsnkv_merge_shard_records", c_int, [c_int, c_int64, P, c_int64, c_int, P, P, P, P, P]),
    ("nsnkv_int3asym_scratch_bytes", c_int64, [c_int64, c_int64, c_int]),
    ("nsnkv_int3asym_encode", c_int, [P, c_int, c_int64, c_int64, c_int, c_int, P, P, P, P, P, c_int64, P, P]),
    ("nsnkv_int3asym_decode", c_int, [P, P, P, P, c_int64, c_int64, c_int, P, P]),
    ("nsnkv_k1c_scores", c_int, [c_int, c_int64, c_int, c_int, c_int64, c_int, P, P, P, P, P, P, P]),
]


class PagedDesc(ctypes.Structure):
    """nsnkv_paged_desc (include/nsnkv.h), field for field."""
    _fields_ = [("struct_bytes", c_int64), ("batch", c_int64),
                ("hq", c_int32), ("h", c_int32), ("bits", c_int32), ("dtype", c_int32),
                ("flags", c_int32), ("max_blocks", c_int32),
                ("k_codes", P), ("k_norm", P), ("k_min", P), ("k_scale", P), ("k_alpha", P),
                ("v_codes", P), ("v_norm", P), ("v_min", P), ("v_scale", P), ("v_alpha", P),
                ("blk_bytes", c_int64), ("blk_stride_head", c_int64), ("blk_stride_page", c_int64),
                ("block_table", P), ("table_stride", c_int64),
                ("n_blocks", P), ("tail_len", P),
                ("k_tail", P), ("v_tail", P),
                ("tail_stride_seq", c_int64), ("tail_stride_head", c_int64),
                ("seq_counters", P), ("workspace", P), ("workspace_bytes", c_int64), ("status", P),
                ("host_n_blocks", P), ("host_tail_len", P)]


_lib = None


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero code."""


def load():
    """Load (and on first use, build if needed) libnsnkv.so; raise if impossible."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        from . import build
        build.build()
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols():
    return [name for name, _, _ in SIGNATURES]


def ptr(t) -> c_void_p:
    if t is None:
        return c_void_p(None)
    if not t.is_cuda:
        raise NativeError("nsnkv operators take CUDA tensors only (no CPU path)")
    return c_void_p(t.data_ptr())


def stream_handle(device=None) -> c_void_p:
    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check(rc: int, what: str):
    if rc != OK:
        names = {ERR_ARG: "invalid argument", ERR_LAUNCH: "launch failed", ERR_UNSUPPORTED: "unsupported",
                 ERR_CUDA: "CUDA runtime error", ERR_TOO_LARGE: "exceeds fixed capacity"}
        raise NativeError(f"{what}: {names.get(rc, rc)}")


def require_cuda():
    if not torch.cuda.is_available():
        raise NativeError("nsnkv needs a CUDA device; there is no CPU fallback")
    load()


def status_tensor(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)
