"""The allocation-free int8 linear entry point (dav2cuda_linear_int8_noalloc).

It serves callers whose host application owns the device heap or runs on a
real-time path, and therefore cannot pass a workspace. Its scratch is a
fixed 16 MiB device array inside the library, shared by every call on a
device. This file is collected last so that a run stopping at the first
failure has run everything else first; it also passes alone in a fresh
process. Each case calls the new entry point twice in a row (the array keeps
the previous call's contents) and compares it with dav2cuda_linear_int8 given
a caller workspace: both compute int8 codes and integer dot products, so
the results must be identical (tolerance 0).
"""
import numpy as np
import pytest

import oracle
from devbuf import call, dev, empty, finish, host, ptr

pytestmark = pytest.mark.gpu


def _problem(seed, rows, k, n):
    r = np.random.default_rng(seed)
    x = r.standard_normal((rows, k)).astype(np.float32)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float32)
    b = r.standard_normal(n).astype(np.float32)
    pw, sw = oracle.pack_weight_s8(w)
    return x, pw, sw, b


@pytest.mark.parametrize("rows,k,n,gelu", [(1370, 384, 1536, 1), (257, 1024, 1024, 0), (64, 20, 9, 0)])
def test_noalloc_matches_workspace_entry_point(cuda, dav2lib, rows, k, n, gelu):
    limit = dav2lib.dav2cuda_linear_int8_noalloc_scratch_limit()
    assert limit == 16 << 20
    for call_index in range(2):  # two calls in a row share the static scratch
        x, pw, sw, b = _problem(1000 * call_index + rows, rows, k, n)
        dx, dw, ds, db = dev(cuda, x), dev(cuda, pw.view(np.int32)), dev(cuda, sw), dev(cuda, b)
        ws = dav2lib.dav2cuda_linear_int8_workspace_size(rows, k, n)
        wsb = empty(cuda, (ws,), np.uint8)
        want = empty(cuda, (rows, n))
        got = empty(cuda, (rows, n))
        call(dav2lib, "dav2cuda_linear_int8", ptr(want), ptr(dx), ptr(dw), ptr(ds), ptr(db), rows, k, n, gelu,
             ptr(wsb), ws, None)
        call(dav2lib, "dav2cuda_linear_int8_noalloc", ptr(got), ptr(dx), ptr(dw), ptr(ds), ptr(db), rows, k, n, gelu,
             None)
        w_host, g_host = host(want), host(got)
        finish(cuda, dav2lib)
        assert np.array_equal(g_host, w_host)


def test_noalloc_rejects_oversized_problems(cuda, dav2lib):
    rows, k = 65536, 1024  # needs 64 MiB of codes
    assert dav2lib.dav2cuda_linear_int8_workspace_size(rows, k, 16) > dav2lib.dav2cuda_linear_int8_noalloc_scratch_limit()
    before = dav2lib.dav2cuda_launch_count(0)
    rc = dav2lib.dav2cuda_linear_int8_noalloc(None, None, None, None, None, rows, k, 16, 0, None)
    assert rc == 1
    assert b"16 MiB" in dav2lib.dav2cuda_last_error()
    assert dav2lib.dav2cuda_launch_count(0) == before
