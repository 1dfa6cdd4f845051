"""GPU parity: RVQ decode (bit-exact) and the onesweep radix sort (exact order)."""
import numpy as np
import pytest
import torch

from nest_b200 import raster, synth
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [200_000])
def test_rvq_config0_bit_exact(n):
    cb, idx = synth.config0(n=n)
    out = raster.rvq_decode(idx.cuda(), cb.cuda()).cpu().numpy()
    ref = oracle.rvq_decode_np(idx.numpy(), cb.numpy())
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("n,K,E,D", [(1, 6, 256, 59), (511, 6, 256, 59), (513, 6, 256, 59),
                                     (100_003, 6, 256, 59), (4097, 1, 256, 59), (3000, 6, 16, 17),
                                     (3000, 4, 256, 32), (3000, 6, 256, 64), (3000, 8, 256, 59),
                                     (2000, 3, 100, 33), (3001, 2, 256, 48), (2999, 5, 256, 40),
                                     (1000, 7, 64, 59), (128, 6, 256, 59), (129 * 128 + 3, 6, 256, 59),
                                     ((1 << 20) + 5, 6, 256, 59)])
def test_rvq_shapes_bit_exact(n, K, E, D):
    g = torch.Generator().manual_seed(n + K + E + D)
    cb = torch.randn(K, E, D, generator=g)
    idx = torch.randint(0, E, (n, K), generator=g).to(torch.uint8)
    out = raster.rvq_decode(idx.cuda(), cb.cuda()).cpu().numpy()
    ref = oracle.rvq_decode_np(idx.numpy(), cb.numpy())
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_rvq_unaligned_output():
    # an output 4 bytes past a 16-byte boundary: rows are written without the bulk copies
    g = torch.Generator().manual_seed(12)
    cb = torch.randn(6, 256, 59, generator=g)
    idx = torch.randint(0, 256, (20_000, 6), generator=g).to(torch.uint8)
    buf = torch.full((20_000 * 59 + 4,), -1.0, device="cuda")
    out = buf[1:1 + 20_000 * 59].view(20_000, 59)
    raster.rvq_decode(idx.cuda(), cb.cuda(), out=out)
    ref = oracle.rvq_decode_np(idx.numpy(), cb.numpy())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert float(buf[0]) == -1.0 and torch.all(buf[1 + 20_000 * 59:] == -1.0)


def test_rvq_unaligned_index_view():
    # a view starting one row in: index bytes at an odd offset take the gather path
    g = torch.Generator().manual_seed(9)
    cb = torch.randn(6, 256, 59, generator=g)
    idx = torch.randint(0, 256, (5001, 6), generator=g).to(torch.uint8)
    dev_idx = idx.cuda()
    view = dev_idx.view(-1)[3:3 + 5000 * 6].view(5000, 6)  # 3-byte offset
    out = raster.rvq_decode(view.contiguous() if not view.is_contiguous() else view, cb.cuda()).cpu().numpy()
    ref = oracle.rvq_decode_np(idx.view(-1)[3:3 + 5000 * 6].view(5000, 6).numpy(), cb.numpy())
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_rvq_negative_zero_and_specials():
    cb = torch.zeros(6, 256, 59)
    cb[0, 0, 0] = -0.0
    cb[1, 1, 1] = float("inf")
    cb[2, 2, 2] = float("nan")
    idx = torch.zeros(8, 6, dtype=torch.uint8)
    idx[1, 1] = 1
    idx[2, 2] = 2
    out = raster.rvq_decode(idx.cuda(), cb.cuda()).cpu().numpy()
    ref = oracle.rvq_decode_np(idx.numpy(), cb.numpy())
    assert np.array_equal(out.view(np.uint32)[:, :2], ref.view(np.uint32)[:, :2])
    assert np.isnan(out[2, 2]) and np.isinf(out[1, 1])
    assert np.signbit(out[0, 0]) == np.signbit(ref[0, 0])  # +0 + -0 = +0 in stage order


def _sort_case(n, bits, dup, seed):
    rng = np.random.default_rng(seed)
    hi = np.uint64(1) << np.uint64(min(bits, 63))
    keys = rng.integers(0, int(hi), size=n, dtype=np.uint64, endpoint=False)
    if dup:
        keys = keys[rng.integers(0, max(1, n // 8), size=n)]
    vals = np.arange(n, dtype=np.uint32)
    kt = torch.from_numpy(keys.view(np.int64)).cuda()
    vt = torch.from_numpy(vals.view(np.int32)).cuda()
    ko, vo = raster.radix_sort_pairs(kt, vt, end_bit=bits)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(ko.cpu().numpy().view(np.uint64), keys[order])
    assert np.array_equal(vo.cpu().numpy().view(np.uint32), vals[order])


@pytest.mark.parametrize("n", [1, 2, 4095, 4096, 4097, 100_000, 1 << 20])
def test_sort_45_bit_keys(n):
    _sort_case(n, 45, dup=True, seed=n)


@pytest.mark.parametrize("bits", [1, 8, 13, 33, 64])
def test_sort_end_bits(bits):
    _sort_case(50_000, bits, dup=False, seed=bits)


def test_sort_binning_like_keys():
    # (tile << 32 | depth bits) with heavy tile repetition, as duplicateWithKeys emits
    rng = np.random.default_rng(5)
    n = 300_000
    tiles = rng.integers(0, 4346, size=n).astype(np.uint64)
    depth = rng.uniform(0.2, 10.0, size=n).astype(np.float32).view(np.uint32).astype(np.uint64)
    keys = (tiles << np.uint64(32)) | depth
    keys[1::3] = keys[::3][: len(keys[1::3])]  # exact duplicates exercise stability
    vals = np.arange(n, dtype=np.uint32)
    ko, vo = raster.radix_sort_pairs(torch.from_numpy(keys.view(np.int64)).cuda(),
                                     torch.from_numpy(vals.view(np.int32)).cuda(), end_bit=45)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(vo.cpu().numpy().view(np.uint32), vals[order])
