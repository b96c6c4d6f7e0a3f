"""PackedCache: per-slot 64-token block cache with the reference's sealing policy.

The observable behaviour is that of the reference's PK01 cache
(experiments/nb06/source/loop_kv_nb06_packed.py:5-61, the cache half of
experiments/ac08/source/loop_kv_pk01_cache.py:76-132), kept exactly because model
adapters and the reference's own tests drive it:

* ``update(key, value, slot, cache_kwargs)`` appends to the slot's native tail and
  returns the slot's whole K and V (restored blocks + tail); before a slot's first seal
  the HF base cache's own ``update`` runs.
* ``compress_to(target)`` moves tokens [start, target) of every slot out of the tails
  into 64-token blocks; every slot must be at the same ``start`` and keep at least 64
  tail tokens past ``target``.
* ``post_prefill`` seals down to a tail of 64..127 tokens; ``post_decode`` seals one
  block whenever the tail reaches 128.
* The same coordinates, checks and error messages.  ``w.LAYERS`` / ``w.HEADS`` are read
  at call time (tests and LoopedDecoder set them).

The storage is this library's own.  Each (slot, K|V) stream keeps its sealed blocks in
a BlockRun: device arrays with spare capacity (codes [H, cap, 3072], norm / min / scale,
headers) that the fused encoder writes in place, so a seal costs the new blocks only;
the reference re-copies the stream's whole packed history with ``torch.cat`` on every
seal (append_group, loop_kv_nb06_codec.py:40-45).  ``packed[(slot, kv)]`` serves the
reference's group dict (codes [1,H,n,3072], metas, headers) as views of the first n
blocks of a run: block-strided along the block axis, with the run's capacity as the
head stride, which the attention entry points accept.

For batched serving use ``nsn_b200.paged.PagedKVCache`` (page pool + block table,
seal-at-64, no host sync per step).
"""
from __future__ import annotations

from collections import Counter

import torch

from . import primitives as w
from .codec import restore_group


class BlockRun:
    """The sealed blocks of one (slot, K|V) stream, in arrays that grow by doubling."""

    def __init__(self, heads: int, device, bits: int = 3):
        self.heads, self.device, self.bits = heads, device, bits
        self.n = 0
        self.cap = 0
        self.arrays = None

    def _reserve(self, need: int):
        if need <= self.cap:
            return
        cap = max(need, 2 * self.cap, 4)
        h, dev = self.heads, self.device
        grown = dict(codes=torch.empty((h, cap, w.code_bytes(self.bits)), dtype=torch.uint8, device=dev),
                     norm=torch.empty((h, cap, w.BLOCK), dtype=torch.float16, device=dev),
                     min=torch.empty((h, cap, w.DIM), dtype=torch.float16, device=dev),
                     scale=torch.empty((h, cap, w.DIM), dtype=torch.float16, device=dev),
                     headers=torch.empty((h, cap, 12), dtype=torch.uint8, device=dev))
        if self.n:
            for key, arr in grown.items():
                arr[:, :self.n].copy_(self.arrays[key][:, :self.n])
        self.arrays, self.cap = grown, cap

    def seal(self, tokens: torch.Tensor, start: int):
        """Encode tokens [1, H, 64*k, 128] as k more blocks whose headers count from token `start`."""
        k = tokens.shape[2] // w.BLOCK
        self._reserve(self.n + k)
        x = tokens[0].reshape(self.heads, k, w.BLOCK, w.DIM)
        w.encode_blocks(x, self.bits, out=self.arrays, out_row_stride=self.cap, out_offset=self.n,
                        headers_start=start)
        self.n += k

    def group(self):
        """The reference's group dict over the sealed blocks, as views (None when empty)."""
        if not self.n:
            return None
        a, n = self.arrays, self.n
        return dict(codes=a["codes"][None, :, :n],
                    metas=(a["norm"][None, :, :n, :, None], a["min"][None, :, :n, None, :],
                           a["scale"][None, :, :n, None, :]),
                    headers=a["headers"][None, :, :n])


class PackedGroups:
    """Read-only mapping (slot, 'K'|'V') -> group dict over a cache's block runs."""

    def __init__(self):
        self.runs = {}

    def get(self, key, default=None):
        run = self.runs.get(key)
        g = run.group() if run is not None else None
        return default if g is None else g

    def __getitem__(self, key):
        g = self.get(key)
        if g is None:
            raise KeyError(key)
        return g

    def __contains__(self, key):
        return self.get(key) is not None

    def keys(self):
        return [k for k, run in self.runs.items() if run.n]

    def values(self):
        return [self[k] for k in self.keys()]

    def items(self):
        return [(k, self[k]) for k in self.keys()]

    def __len__(self):
        return len(self.keys())

    def __bool__(self):
        return len(self) > 0

    def clear(self):
        self.runs.clear()


def seal_target_after_prefill(length: int) -> int:
    """Sealed-token target that leaves a tail of 64..127 tokens (0 below 128 tokens)."""
    return max(0, (length - w.BLOCK) // w.BLOCK * w.BLOCK)


def seal_target_after_decode(length: int, sealed: int) -> int:
    """One more block once the tail holds 128 tokens, else unchanged."""
    return sealed + w.BLOCK if length - sealed >= 2 * w.BLOCK else sealed


def make_packed_cache(base):
    """A PackedCache class over the HF-style cache class `base` (key_cache / value_cache lists)."""

    class PackedCache(base):
        def __init__(self, r, bits=3):
            super().__init__()
            w.require(bits in (None, 3), "PK01 supports native/3bit only")
            self.r, self.bits = r, bits
            self.packed = PackedGroups()
            self.compressed = {}          # slot -> sealed tokens
            self.calls = Counter()        # slot -> update calls
            self.encoded_blocks = Counter()
            self.restore_observer = None  # callable(slot, k, v) after each packed update

        # ---- sizes
        def _slots(self):
            return w.LAYERS * self.r

        def _tails(self, kv):
            return self.key_cache if kv == "K" else self.value_cache

        def get_seq_length(self, layer_idx=0):
            slot = 0 if layer_idx is None else layer_idx
            tails = self.key_cache
            if not 0 <= slot < len(tails) or tails[slot] is None:
                return 0
            return self.compressed.get(slot, 0) + tails[slot].shape[-2]

        # ---- reads
        def materialize(self, slot, kv):
            """Restored blocks followed by the native tail, [1, H, length, 128] in the tail dtype."""
            tail = self._tails(kv)[slot]
            g = self.packed.get((slot, kv))
            return tail if g is None else torch.cat((restore_group(g, tail.dtype), tail), -2)

        # ---- writes
        def _append(self, key, value, slot, cache_kwargs):
            """Check one update's coordinates and append its tokens to the slot.

            Before the slot's first seal the base cache takes them and its result is
            returned; afterwards they join the native tails here and None is returned."""
            length = self.get_seq_length(slot)
            ok = (0 <= slot < self._slots() and key.shape == value.shape and tuple(key.shape[:2]) == (1, w.HEADS)
                  and key.shape[-1] == w.DIM)
            w.require(ok, "Packed KV coordinates")
            pos = (cache_kwargs or {}).get("cache_position")
            if pos is not None:
                want = torch.arange(length, length + key.shape[-2], device=pos.device)
                w.require(torch.equal(pos, want), "Packed append position")
            self.calls[slot] += 1
            if not self.compressed.get(slot, 0):
                return super().update(key, value, slot, cache_kwargs)  # nothing sealed yet: the base route
            for kv, new in (("K", key), ("V", value)):
                tails = self._tails(kv)
                tails[slot] = torch.cat((tails[slot], new), -2)
            self._seen_tokens = self.get_seq_length(slot)
            return None

        def update(self, key, value, layer_idx, cache_kwargs=None):
            base_result = self._append(key, value, layer_idx, cache_kwargs)
            if base_result is not None:
                return base_result
            k, v = self.materialize(layer_idx, "K"), self.materialize(layer_idx, "V")
            if self.restore_observer is not None:
                self.restore_observer(layer_idx, k, v)
            return k, v

        def compress_to(self, target):
            """Seal tokens [start, target) of every slot (start = the current sealed count)."""
            if self.bits is None:
                return
            start = self.compressed.get(0, 0)
            w.require(target >= start and (target - start) % w.BLOCK == 0, "Block overlap/ordering")
            count = target - start
            if not count:
                return
            for slot in range(self._slots()):
                w.require(self.compressed.get(slot, 0) == start and self.get_seq_length(slot) >= target + w.BLOCK,
                          "Tail/compressed divergence")
                for kv in ("K", "V"):
                    tails = self._tails(kv)
                    run = self.packed.runs.get((slot, kv))
                    if run is None:
                        run = self.packed.runs[(slot, kv)] = BlockRun(w.HEADS, tails[slot].device, self.bits)
                    run.seal(tails[slot][:, :, :count], start)
                    tails[slot] = tails[slot][:, :, count:].contiguous().clone()
                self.compressed[slot] = target
                self.encoded_blocks[slot] += count // w.BLOCK

        def post_prefill(self):
            self.compress_to(seal_target_after_prefill(self.get_seq_length()))

        def post_decode(self):
            if self.bits is not None:
                sealed = self.compressed.get(0, 0)
                self.compress_to(seal_target_after_decode(self.get_seq_length(), sealed))

        def reorder_cache(self, *args, **kwargs):
            raise w.IntegrityError("PK01 beam reorder not supported")

        def clear(self):
            self.key_cache.clear()
            self.value_cache.clear()
            self._seen_tokens = 0
            for state in (self.packed, self.compressed, self.calls, self.encoded_blocks):
                state.clear()

    return PackedCache
