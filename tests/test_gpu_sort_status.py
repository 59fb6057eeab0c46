"""The sort's bounded look-back wait reports FGS_ERR_TIMEOUT (through the C ABI).

Every wait in the onesweep sort is bounded. The test hooks make the first
partition publish nothing (a flag that nothing sets), so the next partition's
wait runs out after a short poll limit; the kernel then flags the timeout,
stops waiting, and the last pass replaces the output with its safe form
(all-ones keys, the input values). Nothing faults: the test checks that
fgs_sort_status reports the timeout, that every store stayed inside the
output (guard words around it are untouched), and that with the hooks reset
the same workspace sorts correctly and reports FGS_OK.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from fastgs_core_b200 import _lib

pytestmark = pytest.mark.gpu

GUARD = 4096


def _p(t):
    return C.c_void_p(t.data_ptr())


def _st():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _keys(n, seed, dev):
    rng = np.random.default_rng(seed)
    tiles = rng.integers(0, 8160, n).astype(np.uint64)
    depth = rng.uniform(0.2, 60, n).astype(np.float32).view(np.uint32).astype(np.uint64)
    keys = (tiles << np.uint64(32)) | depth
    return torch.from_numpy(keys).to(dev), torch.arange(n, dtype=torch.int32, device=dev).to(torch.uint32)


@pytest.fixture
def hooks():
    L = _lib.lib()
    yield L
    assert L.fgs_sort_set_test_hooks(0, 0) == _lib.FGS_OK


def test_lookback_timeout_is_reported(hooks, cuda_dev):
    L = hooks
    n, bits = 200_000, 45
    keys, vals = _keys(n, 5, cuda_dev)
    sentinel_k = torch.full((n + 2 * GUARD,), 0x5A5A5A5A5A5A5A5A, dtype=torch.int64, device=cuda_dev)
    sentinel_v = torch.full((n + 2 * GUARD,), 0x7B7B7B7B, dtype=torch.int32, device=cuda_dev)
    ko = sentinel_k.clone()
    vo = sentinel_v.clone()
    nbytes = int(L.fgs_sort_workspace_bytes(n, bits))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda_dev)
    ko_p = C.c_void_p(ko.data_ptr() + 8 * GUARD)
    vo_p = C.c_void_p(vo.data_ptr() + 4 * GUARD)

    # first partition withholds its prefix; waits give up after 2000 polls
    assert L.fgs_sort_set_test_hooks(2000, 1) == _lib.FGS_OK
    assert L.fgs_sort_pairs(n, bits, _p(keys), _p(vals), ko_p, vo_p, _p(ws), nbytes, _st()) == _lib.FGS_OK
    assert L.fgs_sort_status(_p(ws), _st()) == _lib.FGS_ERR_TIMEOUT
    assert b"gave up" in L.fgs_last_error()
    torch.cuda.synchronize()
    for buf, sent in ((ko, sentinel_k), (vo, sentinel_v)):
        assert torch.equal(buf[:GUARD], sent[:GUARD]) and torch.equal(buf[-GUARD:], sent[-GUARD:])
    # the safe output of a timed-out sort: all-ones keys, the input values in order
    assert bool((ko[GUARD:GUARD + n] == -1).all())
    assert torch.equal(vo[GUARD:GUARD + n], vals.view(torch.int32))

    # the static (allocation-free) sort reports through a NULL workspace
    ks, vs = torch.empty_like(keys), torch.empty_like(vals)
    assert L.fgs_sort_pairs_static(n, bits, _p(keys), _p(vals), _p(ks), _p(vs), _st()) == _lib.FGS_OK
    assert L.fgs_sort_status(None, _st()) == _lib.FGS_ERR_TIMEOUT

    # hooks off: the same workspace sorts correctly and the status clears
    assert L.fgs_sort_set_test_hooks(0, 0) == _lib.FGS_OK
    assert L.fgs_sort_pairs(n, bits, _p(keys), _p(vals), ko_p, vo_p, _p(ws), nbytes, _st()) == _lib.FGS_OK
    assert L.fgs_sort_status(_p(ws), _st()) == _lib.FGS_OK
    assert L.fgs_sort_pairs_static(n, bits, _p(keys), _p(vals), _p(ks), _p(vs), _st()) == _lib.FGS_OK
    assert L.fgs_sort_status(None, _st()) == _lib.FGS_OK
    kn = keys.cpu().numpy()
    order = np.argsort(kn, kind="stable")
    got_k = ko[GUARD:GUARD + n].cpu().numpy().view(np.uint64)
    assert np.array_equal(got_k, kn[order])
    assert np.array_equal(vo[GUARD:GUARD + n].cpu().numpy().view(np.uint32), order.astype(np.uint32))
    assert np.array_equal(ks.cpu().numpy(), kn[order])


def test_trainer_raises_on_sort_timeout(hooks, cuda_dev):
    from fastgs_core_b200 import synthetic as S
    from fastgs_core_b200.train import Trainer

    L = hooks
    scene, cam = S.small_scene(3, 60_000, 3, 640, 480, log_scale_mu=-2.5)
    tr = Trainer(scene, cuda_dev)
    tr.activate()
    tr.render_view(cam, sort_only=True)
    tr.check_sort_status()  # no timeout
    want = [t.clone() for t in tr.last_sorted]
    # both sorts of the view (depth order, tile bits) time out; the binning
    # stops after the tile sort, so nothing consumes the safe fallback output
    assert L.fgs_sort_set_test_hooks(2000, 1) == _lib.FGS_OK
    tr.render_view(cam, sort_only=True)
    with pytest.raises(RuntimeError, match="gave up"):
        tr.check_sort_status()
    assert bool((tr.last_sorted[0].view(torch.int64) == -1).all())
    assert L.fgs_sort_set_test_hooks(0, 0) == _lib.FGS_OK
    tr.render_view(cam, sort_only=True)
    tr.check_sort_status()
    assert torch.equal(tr.last_sorted[0], want[0]) and torch.equal(tr.last_sorted[1], want[1])


def test_api_sort_keys_raises_on_timeout(hooks, cuda_dev):
    import fastgs_core_b200 as fg

    L = hooks
    keys, vals = _keys(100_000, 6, cuda_dev)
    fg.sort_keys(keys, vals, key_bits=45)
    assert L.fgs_sort_set_test_hooks(2000, 1) == _lib.FGS_OK
    with pytest.raises(RuntimeError, match="gave up"):
        fg.sort_keys(keys, vals, key_bits=45)
