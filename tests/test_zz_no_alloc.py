"""The allocation-free sort entry point (gsb_radix_sort_pairs_noalloc) against the
regular one (gsb_radix_sort_pairs, caller-provided workspace), through the C ABI.

Some callers of this library cannot allocate device memory: a host application
that budgets all GPU memory itself and hands a plugin only the buffers of each
call, or a loop that must not reach cudaFree, which synchronizes the device.
gsb_radix_sort_pairs_noalloc serves them: its scratch is a fixed device array
inside the library, shared by every call on a device. These tests run it twice
in a row (the second call finds the first call's leftovers in that array) and
check both results bit for bit against the workspace entry point, since a sort
of integers must be exact. They also check that the call takes no device memory
and that sizes above the fixed maximum are refused.

This file is collected last, so a run that stops at its first failure has run
every other test before it.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from torch_gsplat_bridge_fast import _native as N

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _device_tensors(keys: np.ndarray, vals: np.ndarray):
    k_in = torch.from_numpy(keys.view(np.int64)).to(DEV)
    v_in = torch.from_numpy(vals.view(np.int32)).to(DEV)
    return k_in, v_in, torch.empty_like(k_in), torch.empty_like(v_in)


def _sort_workspace(keys, vals, begin, end):
    L = N.load()
    k_in, v_in, k_out, v_out = _device_tensors(keys, vals)
    status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=DEV)
    ws_n = L.gsb_radix_sort_pairs_workspace_size(keys.size, begin, end)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=DEV)
    N.check(L.gsb_radix_sort_pairs(N.ptr(k_in), N.ptr(v_in), N.ptr(k_out), N.ptr(v_out), keys.size, begin, end,
                                   N.ptr(status), N.ptr(ws), ws_n, N.stream_ptr(DEV)), "gsb_radix_sort_pairs")
    torch.cuda.synchronize()
    assert int(status[N.GSB_STATUS_ERROR]) == 0
    return k_out.cpu().numpy().view(np.uint64), v_out.cpu().numpy().view(np.uint32)


def _free_device_bytes() -> int:
    free, _total = torch.cuda.mem_get_info(DEV)
    return int(free)


def _sort_noalloc(keys, vals, begin, end, check_memory: bool):
    """One call of the allocation-free entry point; with check_memory, asserts
    that neither torch's allocator nor the device lost memory across it."""
    L = N.load()
    k_in, v_in, k_out, v_out = _device_tensors(keys, vals)
    status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    alloc0, reserved0, free0 = torch.cuda.memory_allocated(DEV), torch.cuda.memory_reserved(DEV), _free_device_bytes()
    rc = L.gsb_radix_sort_pairs_noalloc(N.ptr(k_in), N.ptr(v_in), N.ptr(k_out), N.ptr(v_out), keys.size, begin, end,
                                        N.ptr(status), N.stream_ptr(DEV))
    N.check(rc, "gsb_radix_sort_pairs_noalloc")
    torch.cuda.synchronize()
    if check_memory:
        assert torch.cuda.memory_allocated(DEV) == alloc0
        assert torch.cuda.memory_reserved(DEV) == reserved0
        # A workspace of this sort is several MB; the driver's free count moves
        # in 2 MiB pages, so a drop of less than that is not an allocation.
        assert _free_device_bytes() > free0 - (2 << 20)
    assert int(status[N.GSB_STATUS_ERROR]) == 0
    return k_out.cpu().numpy().view(np.uint64), v_out.cpu().numpy().view(np.uint32)


def _keys(n: int, seed: int):
    rng = np.random.default_rng(seed)
    keys = rng.integers(0, 2**63, n, dtype=np.uint64) | (rng.integers(0, 2, n, dtype=np.uint64) << np.uint64(63))
    keys[: n // 3] &= np.uint64(0xFFFF0000FFFF00FF)  # many ties: stability matters
    return keys, np.arange(n, dtype=np.uint32)


@pytest.mark.parametrize("n,begin,end", [(N.GSB_SORT_NOALLOC_MAX_PAIRS, 0, 64), (100_003, 32, 45), (4097, 5, 19)])
def test_noalloc_sort_matches_workspace_sort_twice(n, begin, end):
    keys, vals = _keys(n, seed=n + begin)
    ref_k, ref_v = _sort_workspace(keys, vals, begin, end)
    # Two calls in a row: the second meets the first call's histograms and
    # look-back words in the shared scratch and must clear them itself. The
    # first call on the device also looks up the array's address; memory is
    # checked on the second.
    for call in range(2):
        k, v = _sort_noalloc(keys, vals, begin, end, check_memory=call == 1)
        assert np.array_equal(k, ref_k), f"keys differ on call {call}"
        assert np.array_equal(v, ref_v), f"values differ on call {call}"


def test_noalloc_sort_refuses_sizes_above_its_maximum():
    L = N.load()
    n = N.GSB_SORT_NOALLOC_MAX_PAIRS + 1
    keys, vals = _keys(n, seed=1)
    k_in, v_in, k_out, v_out = _device_tensors(keys, vals)
    status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=DEV)
    rc = L.gsb_radix_sort_pairs_noalloc(N.ptr(k_in), N.ptr(v_in), N.ptr(k_out), N.ptr(v_out), n, 0, 64,
                                        N.ptr(status), N.stream_ptr(DEV))
    assert rc == 4, rc  # GSB_ERR_CAPACITY
    assert b"allocation-free" in L.gsb_status_string(rc)
