"""nsnkv_decode_attn_noalloc: the allocation-free decode attention entry point.

Some callers cannot allocate device memory: a serving loop that must never call
into an allocator (cudaMalloc can synchronise the device), or a host runtime that
has no access to the caching allocator the workspace normally comes from.  They
call nsnkv_decode_attn_noalloc, which keeps the split-KV partials in a fixed
16 MiB device array inside the library instead of a caller-provided workspace.

This test calls both entry points through the C ABI on the same inputs, twice in
a row with different inputs, and checks that the allocation-free results match
the workspace-based ones: within the attention tolerance used by the other
tests, and in fact bit for bit, because the kernels are the same.  The file is
named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import nsn_oracle as O

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p


def _ptr(t):
    return P(None) if t is None else P(t.data_ptr())


def _case(seed, h, group, nb, t):
    from nsn_b200 import codec, workloads
    rng = np.random.default_rng(seed)
    total = nb * 64 + t
    k = torch.from_numpy(workloads.np_kv(rng, (1, h, total, 128), workloads.K_OUTLIERS_4, 0.5)).cuda()
    v = torch.from_numpy(workloads.np_kv(rng, (1, h, total, 128), (), 0.5)).cuda()
    q = torch.from_numpy(rng.standard_normal((1, h * group, 128)).astype(np.float16)).cuda()
    g = codec.encode_group(k[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0)
    vg = codec.encode_group(v[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0)
    return dict(h=h, hq=h * group, nb=nb, t=t, q=q, g=g, vg=vg,
                kt=k[:, :, nb * 64:].contiguous(), vt=v[:, :, nb * 64:].contiguous())


def _args(c):
    g, vg = c["g"], c["vg"]
    return [1, c["hq"], c["h"], 3, 0, _ptr(c["q"]),
            _ptr(g["codes"]), _ptr(g["metas"][0]), _ptr(g["metas"][1]), _ptr(g["metas"][2]),
            _ptr(vg["codes"]), _ptr(vg["metas"][0]), _ptr(vg["metas"][1]), _ptr(vg["metas"][2]),
            c["nb"], 1, P(None), 0, P(None), c["nb"], c["nb"],
            _ptr(c["kt"]), _ptr(c["vt"]), c["h"] * c["t"], c["t"], P(None), c["t"], c["t"], P(None), P(None)]


def _run(lib, c, noalloc):
    out = torch.empty((1, c["hq"], 128), dtype=torch.float16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = P(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = lib.nsnkv_decode_attn_noalloc(*_args(c), _ptr(out), P(None), P(None), _ptr(status), stream)
    else:
        need = lib.nsnkv_decode_attn_workspace_bytes(1, c["hq"], c["h"], c["nb"], c["t"])
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        rc = lib.nsnkv_decode_attn(*_args(c), _ptr(out), P(None), P(None), _ptr(ws), need, _ptr(status), stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out.float().cpu().numpy()


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from nsn_b200 import _lib
    lib = _lib.load()
    cases = [_case(7, 8, 4, 96, 33), _case(8, 2, 8, 5, 64)]  # the second call is smaller than the first
    for c in cases:
        want = _run(lib, c, noalloc=False)
        got = _run(lib, c, noalloc=True)
        ok, err = O.within_tolerance(got, want, *O.TOLERANCE["float16"])
        assert ok, err
        assert np.array_equal(got, want)


def test_noalloc_rejects_requests_beyond_its_scratch():
    from nsn_b200 import _lib
    lib = _lib.load()
    need = lib.nsnkv_decode_attn_workspace_bytes(64, 32, 8, 4096, 63)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    c = _case(9, 8, 4, 2, 3)
    args = _args(c)
    args[0], args[1], args[2] = 64, 32, 8
    args[20] = 4096  # max_blocks
    rc = lib.nsnkv_decode_attn_noalloc(*args, P(None), P(None), P(None), P(None), P(None))
    assert rc == _lib.ERR_TOO_LARGE
