"""artlite_moe_dispatch_noalloc: the dispatch for callers that must not allocate device memory while they run (a
serving loop with a memory budget fixed at start-up, code whose device memory a framework's caching allocator owns).
It keeps its scratch in a static device array of the library, so the caller passes device buffers for the inputs and
outputs and the library allocates nothing.

Checked through the C ABI against the existing artlite_moe_dispatch on two calls in a row (the second smaller than
the first, so stale scratch from the first would show), bit-exact: the outputs are integers. Collected last
(test_zz_*) so that a run stopping at the first failure has run every other test; passes alone in a fresh process too.
Device buffers come from torch here (test plumbing; the library itself is torch-free)."""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(lib, ids_dev, n, k, E):
    import torch
    off = torch.full((E + 1,), -1, dtype=torch.int64, device="cuda")
    perm = torch.full((max(n * k, 1),), -1, dtype=torch.int32, device="cuda")
    slot = torch.full((max(n * k, 1),), -1, dtype=torch.int32, device="cuda")
    rc = lib.artlite_moe_dispatch_noalloc(ids_dev.data_ptr(), n, k, E, off.data_ptr(), perm.data_ptr(),
                                          slot.data_ptr(), None)
    assert rc == 0, lib.artlite_moe_last_error().decode()
    return off.cpu().numpy(), perm.cpu().numpy()[:n * k], slot.cpu().numpy()[:n * k]


def test_noalloc_matches_dispatch_twice():
    import torch
    from artlite_b200._lib import lib
    from artlite_b200.moe import plan as P

    lb = lib()
    for n, k, E, seed in ((5000, 8, 128, 1), (37, 6, 64, 2)):
        rng = np.random.default_rng(seed)
        lg = rng.standard_normal((n, E)).astype(np.float32) + np.linspace(0, 2, E, dtype=np.float32)
        ids, _ = P.route(lg, k)
        want = P.dispatch(ids, E)  # the existing entry point
        ids_dev = torch.from_numpy(ids).cuda()
        got = _noalloc(lb, ids_dev, n, k, E)
        for a, b in zip(got, want):
            assert np.array_equal(a, b)


def test_noalloc_allocates_nothing():
    """After a first call on the device (its one-time set-up), further calls leave the device's free memory and the
    caller's allocator untouched."""
    import torch
    from artlite_b200._lib import lib
    from artlite_b200.moe import plan as P

    lb = lib()
    n, k, E = 3000, 8, 128
    lg = np.random.default_rng(7).standard_normal((n, E)).astype(np.float32)
    ids, _ = P.route(lg, k)
    ids_dev = torch.from_numpy(ids).cuda()
    off = torch.empty((E + 1,), dtype=torch.int64, device="cuda")
    perm = torch.empty((n * k,), dtype=torch.int32, device="cuda")
    slot = torch.empty((n * k,), dtype=torch.int32, device="cuda")
    args = (ids_dev.data_ptr(), n, k, E, off.data_ptr(), perm.data_ptr(), slot.data_ptr(), None)
    assert lb.artlite_moe_dispatch_noalloc(*args) == 0  # (warm: the set-up and the kernels' first load)
    torch.cuda.synchronize()
    free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    for _ in range(5):
        assert lb.artlite_moe_dispatch_noalloc(*args) == 0, lb.artlite_moe_last_error().decode()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0 and torch.cuda.memory_allocated() == alloc0


def test_noalloc_reports_bad_expert_id():
    """An expert id outside [0, E) comes back as an error (the device status word), as moe_plan's error case."""
    import torch
    from artlite_b200._lib import lib

    lb = lib()
    ids = np.arange(64, dtype=np.int32).reshape(32, 2) % 8
    ids[5, 1] = 8  # (E = 8)
    ids_dev = torch.from_numpy(ids).cuda()
    off = torch.empty((9,), dtype=torch.int64, device="cuda")
    perm = torch.empty((64,), dtype=torch.int32, device="cuda")
    slot = torch.empty((64,), dtype=torch.int32, device="cuda")
    rc = lb.artlite_moe_dispatch_noalloc(ids_dev.data_ptr(), 32, 2, 8, off.data_ptr(), perm.data_ptr(),
                                         slot.data_ptr(), None)
    assert rc != 0 and b"dispatch_noalloc: expert id 8 of 8" in lb.artlite_moe_last_error()
    ids_dev[5, 1] = 3  # (the next call starts from a cleared status word)
    rc = lb.artlite_moe_dispatch_noalloc(ids_dev.data_ptr(), 32, 2, 8, off.data_ptr(), perm.data_ptr(),
                                         slot.data_ptr(), None)
    assert rc == 0, lb.artlite_moe_last_error().decode()


def test_noalloc_rejects_oversize_and_host_memory():
    """Arguments the static scratch cannot take, or buffers that are not the current device's memory, are rejected
    on the host before anything is launched."""
    from artlite_b200._lib import lib

    lb = lib()
    ids = np.zeros((4, 2), np.int32)
    big_n = 262144 // 128 * 4096 // 8 + 8  # one block of pairs past the static scratch at E = 128
    rc = lb.artlite_moe_dispatch_noalloc(ids.ctypes.data, big_n, 8, 128, ids.ctypes.data, ids.ctypes.data,
                                         ids.ctypes.data, None)
    assert rc != 0 and b"static scratch" in lb.artlite_moe_last_error()
    rc = lb.artlite_moe_dispatch_noalloc(ids.ctypes.data, 1 << 62, 8, 128, ids.ctypes.data, ids.ctypes.data,
                                         ids.ctypes.data, None)  # (n k would wrap a 64-bit count)
    assert rc != 0 and b"static scratch" in lb.artlite_moe_last_error()
    rc = lb.artlite_moe_dispatch_noalloc(ids.ctypes.data, 4, 2, 8, ctypes.c_void_p(ids.ctypes.data),
                                         ids.ctypes.data, ids.ctypes.data, None)
    assert rc != 0 and b"device memory" in lb.artlite_moe_last_error()
    fake = ctypes.c_void_p(0x10000)  # (an address no allocation owns)
    rc = lb.artlite_moe_dispatch_noalloc(fake, 4, 2, 8, fake, fake, fake, None)
    assert rc != 0 and b"device memory" in lb.artlite_moe_last_error()
