"""The allocation-free embedding gather, tb_b200_embedding_host_ids_static.

It is for callers that cannot allocate device memory when they gather --
an engine whose device memory belongs to another allocator, or a per-token
decode step that must not take cudaMalloc's implicit synchronisation -- so
its scratch is a fixed device array inside the library instead of an
allocation.  These checks call it through the C ABI and compare it with the
allocating entry point, tb_b200_embedding_host_ids: the gather is a byte
copy, so the two must agree bit for bit, on two calls in a row (the second
call reuses the array the first one left behind).  This file is collected
last so a failure here does not stop the rest of the suite; it must also pass
on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

import tb_b200 as T
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _gather(fn, ids, table_dev, dim, vocab, dtype_code, device):
    import torch
    out = torch.full((ids.size, dim), -7.0, device=device).to(table_dev.dtype)
    rc = fn(dtype_code, ids.size, dim, vocab, ids.ctypes.data, T.ptr(table_dev), T.ptr(out), None)
    torch.cuda.synchronize()
    return rc, out


@pytest.mark.parametrize("is_bf16", [False, True])
def test_static_scratch_gather_matches_allocating_gather(cuda, is_bf16):
    import torch
    L = T.lib()
    rng = np.random.default_rng(2024)
    vocab, dim = 32000, 4096
    table = rng.standard_normal((vocab, dim), dtype=np.float32) * np.float32(0.02)
    if is_bf16:
        table = O.f32_to_bf16(table)
        table_dev = torch.from_numpy(table.view(np.int16)).view(torch.bfloat16).to(cuda)
    else:
        table_dev = torch.from_numpy(table).to(cuda)
    code = T.BF16 if is_bf16 else T.F32
    for n in (4096, 777):  # two calls in a row: the second reuses the array
        ids = np.ascontiguousarray(rng.integers(0, vocab, n), dtype=np.int32)
        rc_a, ref = _gather(L.tb_b200_embedding_host_ids, ids, table_dev, dim, vocab, code, cuda)
        rc_s, got = _gather(L.tb_b200_embedding_host_ids_static, ids, table_dev, dim, vocab,
                            code, cuda)
        assert rc_a == 0 and rc_s == 0, T.last_error()
        assert torch.equal(got.view(torch.int16) if is_bf16 else got,
                           ref.view(torch.int16) if is_bf16 else ref)
        want = O.embedding(ids, table)
        have = got.view(torch.int16).cpu().numpy().view(np.uint16) if is_bf16 else got.cpu().numpy()
        assert np.array_equal(have, want)


def test_static_scratch_gather_limits(cuda):
    import torch
    L = T.lib()
    table = torch.zeros((10, 8), device=cuda)
    out = torch.full((4, 8), 3.0, device=cuda)
    too_many = np.zeros(65537, np.int32)
    big = torch.empty((65537, 8), device=cuda)
    assert L.tb_b200_embedding_host_ids_static(T.F32, too_many.size, 8, 10,
                                               too_many.ctypes.data, T.ptr(table), T.ptr(big),
                                               None) == 9
    assert "TB_B200_STATIC_MAX_TOKENS" in T.last_error()
    bad = np.array([1, 2, 10, 3], np.int32)  # 10 is outside [0, vocab)
    assert L.tb_b200_embedding_host_ids_static(T.F32, 4, 8, 10, bad.ctypes.data, T.ptr(table),
                                               T.ptr(out), None) == 8
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())  # nothing was queued
