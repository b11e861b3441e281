"""Onesweep radix sort on the B200 vs the oracle (stable, bit-exact) and the reference's
C2 golden hash (2^24 Zipf pairs, 8,160 tiles)."""
import hashlib
import os

import numpy as np
import pytest

from gsplat_tt_b200 import scenes
from oracle import display as od

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a)).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def gd():
    from gsplat_tt_b200 import display
    return display


def run(gd, keys, vals, key_bits):
    import torch
    v, k = gd.sort_pairs(torch.from_numpy(keys.view(np.int64)), torch.from_numpy(vals.view(np.int32)),
                         key_bits, return_keys=True)
    return k.cpu().numpy().view(np.uint64), v.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("n", [1, 2, 31, 4095, 4096, 4097, 65539, 1 << 20])
def test_zipf_sizes_vs_oracle(gd, n):
    keys, vals = scenes.c2_pairs(n=n, seed=n)
    ko, vo = od.sort_pairs(keys, vals)
    kg, vg = run(gd, keys, vals, 45)
    np.testing.assert_array_equal(kg, ko)
    np.testing.assert_array_equal(vg, vo)


@pytest.mark.parametrize("bits", [1, 8, 13, 32, 45, 64])
def test_key_widths_and_duplicates(gd, bits):
    rng = np.random.default_rng(bits)
    n = 300_000
    hi = (1 << bits) - 1 if bits < 64 else np.iinfo(np.uint64).max
    keys = rng.integers(0, min(hi, 1 << 63), n, dtype=np.uint64, endpoint=True)
    if bits == 64:
        keys |= rng.integers(0, 2, n, dtype=np.uint64) << np.uint64(63)
    keys[::3] = keys[0]  # heavy duplicates exercise stability
    vals = np.arange(n, dtype=np.uint32)
    ko, vo = od.sort_pairs(keys, vals)
    kg, vg = run(gd, keys, vals, bits)
    np.testing.assert_array_equal(kg, ko)
    np.testing.assert_array_equal(vg, vo)


@pytest.mark.parametrize("bits", [5, 12, 21, 40])
def test_bits_above_key_bits_are_ignored(gd, bits):
    """Keys with set bits above key_bits sort stably on their low key_bits bits only
    (the last pass's digit is narrower than a byte here)."""
    rng = np.random.default_rng(100 + bits)
    n = 200_000
    keys = rng.integers(0, 1 << 62, n, dtype=np.uint64)
    vals = np.arange(n, dtype=np.uint32)
    low = keys & np.uint64((1 << bits) - 1)
    order = np.argsort(low, kind="stable")
    kg, vg = run(gd, keys, vals, bits)
    np.testing.assert_array_equal(vg, vals[order])
    np.testing.assert_array_equal(kg, keys[order])


def run_values(gd, keys, vals, key_bits):
    import torch
    v = gd.sort_pairs(torch.from_numpy(keys.view(np.int64)), torch.from_numpy(vals.view(np.int32)),
                      key_bits)
    return v.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("bits", [33, 40, 45, 48, 57, 64])
def test_values_only_sort_with_narrowed_keys(gd, bits):
    """Without keys_out, a sort of more than 32 key bits narrows its keys to 32 bits once
    the bits below key_bits - 32 are sorted (the later passes move 4-byte keys); the values
    must come out in the full-width stable order. Keys carry set bits above key_bits and
    heavy duplicates; values are a permutation."""
    rng = np.random.default_rng(200 + bits)
    n = 300_000
    keys = rng.integers(0, 1 << 63, n, dtype=np.uint64)
    keys |= rng.integers(0, 2, n, dtype=np.uint64) << np.uint64(63)
    keys[::3] = keys[0]
    vals = rng.permutation(n).astype(np.uint32)
    low = keys if bits == 64 else keys & np.uint64((1 << bits) - 1)
    np.testing.assert_array_equal(run_values(gd, keys, vals, bits),
                                  vals[np.argsort(low, kind="stable")])


@pytest.mark.parametrize("n", [1, 4095, 4097, 65539])
def test_values_only_zipf_sizes_vs_oracle(gd, n):
    keys, vals = scenes.c2_pairs(n=n, seed=n)
    _, vo = od.sort_pairs(keys, vals)
    np.testing.assert_array_equal(run_values(gd, keys, vals, 45), vo)


def test_c2_values_only_matches_reference_golden(gd):
    """The benchmark's call: C2 with values only (narrowed keys after two passes)."""
    G = np.load(os.path.join(GOLDEN, "sort.npz"))
    keys, vals = scenes.c2_pairs()
    assert sha(run_values(gd, keys, vals, 45)) == str(G["sha_sorted_values"])


def test_c2_full_matches_reference_golden(gd):
    G = np.load(os.path.join(GOLDEN, "sort.npz"))
    keys, vals = scenes.c2_pairs()
    kg, vg = run(gd, keys, vals, 45)
    assert sha(vg) == str(G["sha_sorted_values"])
    assert np.all(kg[1:] >= kg[:-1])
    # values are a permutation: the sort must be too
    assert np.bincount(vg, minlength=vals.size).max() == 1


def test_sort_and_bin_c2_ranges(gd):
    G = np.load(os.path.join(GOLDEN, "sort.npz"))
    keys, vals = scenes.c2_pairs()
    tiles = (keys >> np.uint64(32)).astype(np.int64)
    depth = (keys & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
    dv = np.empty(vals.shape[0], np.float32)
    dv[vals] = depth
    s, rg = gd.sort(vals.astype(np.int64), tiles, dv, 120, 68)
    assert sha(s.cpu().numpy().astype(np.uint32)) == str(G["sha_sorted_values"])
    np.testing.assert_array_equal(rg.cpu().numpy(), G["ranges"])


def test_device_logf_reproduces_host_logf():
    """Exhaustive over [2^-30, 2^30]: the device logf used for the opacity-aware k and
    the pair-cull threshold equals the host C library's logf bit for bit."""
    import torch
    from gsplat_tt_b200._lib import lib, check
    lo = np.float32(2.0 ** -30).view(np.uint32)
    hi = np.float32(2.0 ** 30).view(np.uint32)
    chunk = 1 << 26
    bad = 0
    for start in range(int(lo), int(hi) + 1, chunk):
        u = np.arange(start, min(start + chunk, int(hi) + 1), dtype=np.uint32)
        x = u.view(np.float32)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        check(lib.gs_debug_logf_host(xd.data_ptr(), yd.data_ptr(), xd.numel(),
                                     torch.cuda.current_stream().cuda_stream))
        yh = od.logf_array(x)
        bad += int((yd.cpu().numpy().view(np.uint32) != yh.view(np.uint32)).sum())
    assert bad == 0


def test_launch_count_counts_the_sort_kernels(gd):
    """gs_launch_count (the bench's gpu_launches) grows by the sort's kernels: the histogram
    and its scan, then one pass per 8 key bits (here 40 bits: five passes)."""
    from gsplat_tt_b200._lib import lib
    rng = np.random.default_rng(3)
    n = 10000
    keys = rng.integers(0, 1 << 40, n, dtype=np.uint64)
    vals = np.arange(n, dtype=np.uint32)
    run(gd, keys, vals, 40)  # first call: module load and attributes
    c0 = lib.gs_launch_count()
    run(gd, keys, vals, 40)
    launched = lib.gs_launch_count() - c0
    assert launched >= 2 + 5, launched
