"""vs_radix_sort_pairs_static, the sort for callers that cannot allocate device
memory during the call (its temporaries live in a static device array),
checked through the C ABI against vs_radix_sort_pairs on the same inputs, on
two calls in a row.  Sorting is integer work, so the outputs must be equal.
This file is collected last, so it also runs after everything else has used
the device."""
import ctypes

import numpy as np
import pytest
import torch

from vauss_b200 import _native, ops

pytestmark = pytest.mark.gpu

MAX_KEYS = 1 << 20


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _sort(ctx, fn, keys, vals, bits):
    k, v = keys.clone(), vals.clone()
    st = getattr(ctx.lib, fn)(ctx.h, _ptr(k), _ptr(v), k.numel(), bits)
    assert st == 0, ctx.lib.vs_ctx_last_error(ctx.h)
    return k, v


@pytest.mark.parametrize("count,bits", [(MAX_KEYS, 32), (300_001, 20), (5_000, 24), (2048, 7), (1, 32)])
def test_static_sort_matches_allocating_sort(cuda, count, bits):
    ctx = ops.context(cuda)
    rng = np.random.default_rng(count + bits)
    keys = torch.from_numpy(rng.integers(0, 1 << bits, count, dtype=np.uint64).astype(np.uint32).view(np.int32))
    keys = keys.to(cuda)
    vals = torch.arange(count, dtype=torch.int32, device=cuda)
    want_k, want_v = _sort(ctx, "vs_radix_sort_pairs", keys, vals, bits)
    for _ in range(2):
        got_k, got_v = _sort(ctx, "vs_radix_sort_pairs_static", keys, vals, bits)
        torch.cuda.synchronize()
        assert torch.equal(got_k, want_k)
        assert torch.equal(got_v, want_v)
    order = np.argsort(keys.cpu().numpy().view(np.uint32), kind="stable")
    assert np.array_equal(want_v.cpu().numpy(), order.astype(np.int32))


def test_static_sort_rejects_oversize(cuda):
    ctx = ops.context(cuda)
    keys = torch.zeros(MAX_KEYS + 1, dtype=torch.int32, device=cuda)
    vals = torch.zeros_like(keys)
    st = ctx.lib.vs_radix_sort_pairs_static(ctx.h, _ptr(keys), _ptr(vals), MAX_KEYS + 1, 32)
    assert st == 2
    assert b"static scratch limit" in ctx.lib.vs_ctx_last_error(ctx.h)
    with pytest.raises(_native.VsError):
        ctx.check(st)


def test_static_sort_allocates_nothing(cuda):
    """The property the entry point exists for: after a first call (which
    looks the static array up), further calls leave the context's workspace
    and the device's free memory exactly as they were."""
    ctx = ops.context(cuda)
    count = 200_000
    rng = np.random.default_rng(3)
    keys = torch.from_numpy(rng.integers(0, 1 << 31, count, dtype=np.uint64).astype(np.uint32).view(np.int32))
    keys = keys.to(cuda)
    vals = torch.arange(count, dtype=torch.int32, device=cuda)
    assert ctx.lib.vs_radix_sort_pairs_static(ctx.h, _ptr(keys), _ptr(vals), count, 32) == 0
    torch.cuda.synchronize()
    ws = ctx.workspace_bytes
    free0 = torch.cuda.mem_get_info(cuda)[0]
    for _ in range(2):
        assert ctx.lib.vs_radix_sort_pairs_static(ctx.h, _ptr(keys), _ptr(vals), count, 32) == 0
    torch.cuda.synchronize()
    assert ctx.workspace_bytes == ws
    assert torch.cuda.mem_get_info(cuda)[0] == free0
    assert torch.cuda.current_device() == cuda.index
