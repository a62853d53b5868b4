"""Host Philox4x32-10 (oracle/rng.py) against the published known-answer vectors and its own layout rules."""
import numpy as np

from oracle import rng


def test_known_answer_vectors():
    for ctr, key, want in rng.KAT:
        got = rng.philox4x32_10(*[np.array([c], np.uint32) for c in ctr], *key)
        assert tuple(int(v[0]) for v in got) == want


def test_element_words_follow_the_block_layout():
    seed, offset = 0x1234_5678_9ABC_DEF0, 0x0000_0003_0000_0007
    w = rng.words(seed, offset, 0, 40)
    for g in range(10):
        blk = rng.philox4x32_10(np.array([g]), np.array([0]), np.array([offset & 0xFFFFFFFF]),
                                np.array([offset >> 32]), seed & 0xFFFFFFFF, seed >> 32)
        assert [int(v[0]) for v in blk] == list(w[4 * g:4 * g + 4])
    # any slice equals the same elements of a longer fill (sharded ranks fill their own rows)
    assert np.array_equal(rng.words(seed, offset, 13, 7), w[13:20])
    # counters past 2^32 blocks use the high counter word
    hi = rng.words(seed, offset, 4 << 32, 4)
    blk = rng.philox4x32_10(np.array([0]), np.array([1]), np.array([offset & 0xFFFFFFFF]),
                            np.array([offset >> 32]), seed & 0xFFFFFFFF, seed >> 32)
    assert [int(v[0]) for v in blk] == list(hi)


def test_uniform_is_in_range_and_float32_exact():
    x = rng.uniform(1, 1, 0, 1 << 16, 0.5, 2.0)
    assert x.dtype == np.float32 and x.min() >= 0.5 and x.max() < 2.0
    u = rng.uniform(7, 0, 0, 1 << 16, 0.0, 1.0)
    # u24 values are multiples of 2^-24 below 1
    assert np.all(u * np.float32(2 ** 24) == np.floor(u * np.float32(2 ** 24))) and u.max() < 1.0
    assert abs(float(u.mean()) - 0.5) < 0.01


def test_normal_moments_and_slices():
    z = rng.normal_f64(4, 0, 0, 1 << 18, 0.0, 1.0)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert np.array_equal(rng.normal_f64(4, 0, 5, 11, 0.0, 1.0), z[5:16])
    # a slice ending inside a block still pairs its last element with the block's next word
    assert np.array_equal(rng.normal_f64(4, 0, 0, 7, 0.0, 1.0), z[:7])
    assert np.array_equal(rng.normal_f64(4, 0, 6, 1, 0.0, 1.0), z[6:7])
    y = rng.normal_f64(4, 10, 0, 1 << 16, 0.5, 2.0)
    assert abs(y.mean() - 0.5) < 0.05 and abs(y.std() - 2.0) < 0.05
    assert np.all(rng.normal_error_bound(y, 0.5, 2.0) > 0)
