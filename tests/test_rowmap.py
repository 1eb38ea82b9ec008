"""Row-mode minibatches: the keyed permutation of the rollout rows.

The kernels and the host evaluate the same function (include/metalgym/
rowmap.h); here the host export mg_minibatch_rows is checked against an
independent Python statement of it and for the properties train() relies on:
a bijection of [0, total) for every total, so that the minibatches of one
epoch partition the rollout rows.
"""
import numpy as np
import pytest

M32 = 0xFFFFFFFF


def mix32(x):
    x ^= x >> 16
    x = (x * 0x7FEB352D) & M32
    x ^= x >> 15
    x = (x * 0x846CA68B) & M32
    x ^= x >> 16
    return x


def feistel(x, half, key):
    mask = (1 << half) - 1
    left, right = x >> half, x & mask
    for k in key:
        f = mix32((right & M32) ^ k) & mask
        left, right = right, left ^ f
    return (left << half) | right


def permute(pos, n, key):
    half = 1
    while (1 << (2 * half)) < n:
        half += 1
    y = feistel(pos, half, key)
    while y >= n:
        y = feistel(y, half, key)
    return y


@pytest.fixture(scope="module")
def hostlib():
    import metalgym_b200

    return metalgym_b200.lib()  # host entry points only: no GPU needed


@pytest.fixture(scope="module")
def rows_fn(hostlib):
    from metalgym_b200.session import minibatch_rows

    return minibatch_rows


@pytest.mark.parametrize("total", [1, 2, 3, 5, 64, 1000, 4097])
def test_matches_python_statement(rows_fn, total):
    key = [0x12345678, 0x9ABCDEF0, 7, 0xFFFFFFFF]
    got = rows_fn(key, 0, total, total)
    want = [permute(p, total, key) for p in range(total)]
    assert got.tolist() == want


@pytest.mark.parametrize("total", [1, 7, 4096, 131072, 16384 * 32 + 5])
def test_is_a_permutation(rows_fn, total):
    rng = np.random.default_rng(total)
    key = [int(x) for x in rng.integers(0, 2**32, 4, dtype=np.uint64)]
    got = rows_fn(key, 0, total, total)
    assert np.array_equal(np.sort(got), np.arange(total, dtype=np.uint64))


def test_minibatches_partition_an_epoch(rows_fn):
    total, B = 4096 * 4, 2048
    key = [1, 2, 3, 4]
    parts = [rows_fn(key, m * B, B, total) for m in range(total // B)]
    allrows = np.concatenate(parts)
    assert np.array_equal(np.sort(allrows), np.arange(total, dtype=np.uint64))
    # slices of the one permutation
    assert np.array_equal(allrows, rows_fn(key, 0, total, total))


def test_keys_change_the_order(rows_fn):
    total = 4096
    a = rows_fn([1, 2, 3, 4], 0, total, total)
    b = rows_fn([1, 2, 3, 5], 0, total, total)
    assert (a != b).mean() > 0.9
    # not close to the identity or a shift
    assert np.abs(np.corrcoef(a.astype(float), np.arange(total))[0, 1]) < 0.1


def test_rejects_ranges_past_the_rollout(hostlib):
    import ctypes as C

    k = (C.c_uint32 * 4)(1, 2, 3, 4)
    out = np.zeros(8, np.uint64)
    rc = hostlib.mg_minibatch_rows(k, 10, 8, 16, out.ctypes.data_as(C.c_void_p))
    assert rc != 0 and b"exceeds" in hostlib.mg_last_error()
