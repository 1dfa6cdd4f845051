"""The allocation-free radix sort (ns_radix_sort_pairs_noalloc) against the
regular entry point, through the C-ABI.

Callers such as a renderer plugin inside a host engine with a fixed memory
budget, or a binding without a CUDA allocator, cannot hand the sort its
ping-pong buffers; this entry point keeps them in a device array inside the
library. The test checks that it returns exactly what ns_radix_sort_pairs
returns, on two calls in a row (the shared array keeps the previous call's
contents, so the second call must not see stale state), and that sizes above
its 1,048,576-pair limit are refused. It lives in its own file, collected last.
"""
import numpy as np
import pytest
import torch

from nest_b200 import _lib, raster

pytestmark = pytest.mark.gpu

MAX_PAIRS = 1 << 20


def _keys(n, bits, seed):
    rng = np.random.default_rng(seed)
    k = rng.integers(0, 1 << bits, size=n, dtype=np.uint64)
    k[1::5] = k[::5][: len(k[1::5])]  # duplicate keys exercise stability
    return torch.from_numpy(k.view(np.int64)).cuda(), torch.arange(n, dtype=torch.int32).cuda()


def _noalloc(keys, vals, end_bit):
    lib = _lib.load()
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    rc = lib.ns_radix_sort_pairs_noalloc(keys.data_ptr(), vals.data_ptr(), ko.data_ptr(), vo.data_ptr(),
                                         keys.numel(), end_bit, _lib.stream_handle(keys.device))
    return rc, ko, vo


@pytest.mark.parametrize("calls", [[(100_000, 45, 1), (MAX_PAIRS, 45, 2)],
                                   [(MAX_PAIRS, 64, 3), (4097, 13, 4)]])
def test_noalloc_sort_matches_regular_sort_twice(calls):
    for n, bits, seed in calls:
        keys, vals = _keys(n, bits, seed)
        rc, ko, vo = _noalloc(keys, vals, bits)
        assert rc == _lib.NS_OK
        ref_k, ref_v = raster.radix_sort_pairs(keys, vals, end_bit=bits)
        torch.cuda.synchronize()
        assert torch.equal(ko, ref_k) and torch.equal(vo, ref_v)


def test_noalloc_sort_refuses_sizes_above_limit():
    lib = _lib.load()
    rc = lib.ns_radix_sort_pairs_noalloc(None, None, None, None, MAX_PAIRS + 1, 45, None)
    assert rc == _lib.NS_ERR_CAPACITY


@pytest.mark.parametrize("n", [0, 16])
@pytest.mark.parametrize("end_bit", [-1, 65])
def test_noalloc_sort_checks_end_bit_like_regular_sort(n, end_bit):
    """end_bit outside [0, 64] is refused by both entry points, also for n == 0."""
    lib = _lib.load()
    keys, vals = _keys(max(n, 1), 45, 5)
    ko, vo = torch.empty_like(keys), torch.empty_like(vals)
    rc = lib.ns_radix_sort_pairs_noalloc(keys.data_ptr(), vals.data_ptr(), ko.data_ptr(), vo.data_ptr(), n,
                                         end_bit, _lib.stream_handle(keys.device))
    assert rc == _lib.NS_ERR_INVALID
    with pytest.raises(RuntimeError):
        raster.radix_sort_pairs(keys[:n], vals[:n], end_bit=end_bit)
