"""nsn_b200: B200-native (sm_100a) implementation of NSN's packed-KV hot path.

Modules mirror the reference's operator surface:
  primitives  nsn_encode / nsn_decode / nsn_qdq / pack_codes / planned_bytes
  core        nsn_int3_qdq
  codec       pack3 / unpack3 / encode_group / restore_group / append_group
  packed      make_packed_cache (64-token block cache over an HF-style base)
  kernel      restore_v / launch / pipeline (fused packed-KV decode attention)
  paged       PagedKVCache (batched paged cache: append + attend + seal)
  splitkv     sequence-split decode across GPUs with a log-sum-exp merge
All compute runs in libnsnkv.so (include/nsnkv.h); there is no CPU fallback.
"""
from . import primitives  # noqa: F401
from .primitives import (BLOCK, DIM, ContractError, IntegrityError, NumericalFailure, nsn_decode,  # noqa: F401
                         nsn_encode, nsn_qdq, pack_codes, planned_bytes, unpack_codes)

__version__ = "0.1.0"
