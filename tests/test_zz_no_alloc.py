"""The allocation-free sort entry point (fgs_sort_pairs_static), through the C ABI.

It serves callers that cannot allocate device memory at the time they sort
(for instance a host application that lends plug-ins a fixed GPU memory
budget and forbids allocations after start-up). It must give exactly the
results of fgs_sort_pairs, which sorts with caller-provided workspace, and it
must keep doing so on the next call, since every call reuses the same fixed
scratch area. This file is collected last so that a failure here cannot hide
the other tests in a run that stops at the first failure.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fastgs_core_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_KEYS = 1048576  # FGS_SORT_STATIC_MAX_KEYS in include/fastgs_b200.h


def _p(t):
    return C.c_void_p(t.data_ptr())


def _keys(n, seed, dev):
    rng = np.random.default_rng(seed)
    tiles = rng.integers(0, 8160, n).astype(np.uint64)
    depth = rng.uniform(0.2, 60, n).astype(np.float32).view(np.uint32).astype(np.uint64)
    depth[::9] = depth[0]  # ties: the sort must keep input order
    keys = (tiles << np.uint64(32)) | depth
    vals = rng.permutation(n).astype(np.uint32)
    return torch.from_numpy(keys).to(dev), torch.from_numpy(vals).to(dev)


def _sort_with_workspace(keys, vals, key_bits):
    L = _lib.lib()
    n = keys.numel()
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    nbytes = int(L.fgs_sort_workspace_bytes(n, key_bits))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=keys.device)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(L.fgs_sort_pairs(n, key_bits, _p(keys), _p(vals), _p(ko), _p(vo), _p(ws), nbytes, st),
               "sort_pairs")
    return ko, vo


def _sort_static(keys, vals, key_bits):
    L = _lib.lib()
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(L.fgs_sort_pairs_static(keys.numel(), key_bits, _p(keys), _p(vals), _p(ko), _p(vo), st),
               "sort_pairs_static")
    return ko, vo


def test_static_sort_matches_workspace_sort_twice(cuda_dev):
    # two calls in a row (different sizes and data) against the allocating entry point
    for n, seed, bits in ((300_000, 1, 45), (MAX_KEYS, 2, 45)):
        keys, vals = _keys(n, seed, cuda_dev)
        want_k, want_v = _sort_with_workspace(keys, vals, bits)
        got_k, got_v = _sort_static(keys, vals, bits)
        torch.cuda.synchronize()
        assert torch.equal(got_k, want_k) and torch.equal(got_v, want_v)


def test_static_sort_rejects_oversize(cuda_dev):
    L = _lib.lib()
    st = L.fgs_sort_pairs_static(MAX_KEYS + 1, 45, None, None, None, None, None)
    assert st == _lib.FGS_ERR_CAPACITY
    assert b"at most" in L.fgs_last_error()


def test_static_sort_allocates_nothing(cuda_dev):
    # after a first call (which looks the scratch up), a full-size call leaves
    # the device's free memory exactly where it was
    keys, vals = _keys(MAX_KEYS, 3, cuda_dev)
    _sort_static(keys, vals, 45)
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    L = _lib.lib()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(L.fgs_sort_pairs_static(MAX_KEYS, 45, _p(keys), _p(vals), _p(ko), _p(vo), st),
               "sort_pairs_static")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert L.fgs_sort_status(None, st) == _lib.FGS_OK
