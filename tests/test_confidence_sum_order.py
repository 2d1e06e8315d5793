"""The two reduction orders of a vocabulary slab's confidence partial (CPU, float32).

Besides the sum below, both kernels find the slab's maximum and its first index; the last test
emulates both scans (ties, NaN, -inf, all-NaN slabs) and requires the same (value, index).

The lm_head's confidence partial of one token and one 128-row slab includes sum_f exp(v_f - max).
Two kernels compute it (csrc/epilogue.cuh, kEpiConf; csrc/gemm_tc.cu, conf_slab_from_tmem):

* tokens on N: a warp holds the token; lane l adds its four values f = l, l + 32, l + 64, l + 96
  in that order, then the 32 lane sums are combined by an xor butterfly (offsets 16, 8, 4, 2, 1)
  and lane 0's result is stored;
* tokens on M: one thread holds the token's 128 values in TMEM column order; it adds them into 32
  column sums s[f % 32] in ascending f, then halves the array (s[j] += s[j + off] for off = 16, 8,
  4, 2, 1) and stores s[0].

These are the same float32 additions in the same tree, so the results are bit-identical for any
terms; the GPU test (tests/test_gpu_confidence_tiles.py) relies on that.  IEEE addition is
commutative, so a butterfly lane adding its partner's value in either operand order gives the same
bits; numpy float32 arithmetic rounds to nearest like the GPU's fp32 adds.
"""

import numpy as np


def _lane_tree(e: np.ndarray) -> np.float32:
    lanes = [np.float32(0.0) for _ in range(32)]
    for lane in range(32):
        acc = np.float32(0.0)
        for i in range(4):
            acc = np.float32(acc + e[lane + 32 * i])
        lanes[lane] = acc
    for off in (16, 8, 4, 2, 1):
        lanes = [np.float32(lanes[lane] + lanes[lane ^ off]) for lane in range(32)]
    return lanes[0]


def _register_halving(e: np.ndarray) -> np.float32:
    s = [np.float32(0.0) for _ in range(32)]
    for f in range(128):  # groups of 16 columns, ascending
        s[f & 31] = np.float32(s[f & 31] + e[f])
    for off in (16, 8, 4, 2, 1):
        for j in range(off):
            s[j] = np.float32(s[j] + s[j + off])
    return s[0]


def test_orders_are_bit_identical_on_wide_ranges():
    rng = np.random.default_rng(0)
    for trial in range(300):
        scale = 10.0 ** rng.uniform(-8, 8)
        e = (rng.standard_normal(128) ** 2 * scale).astype(np.float32)  # non-negative, like exp()
        if trial % 3 == 0:
            e[rng.integers(0, 128, 5)] = np.float32(1.0)  # a few dominant terms (the maxima)
        if trial % 7 == 0:
            e[rng.integers(0, 128, 40)] = np.float32(0.0)  # rows past the vocabulary add zero
        a, b = _lane_tree(e), _register_halving(e)
        assert a.tobytes() == b.tobytes(), (trial, a, b)


def test_orders_differ_from_a_plain_sequential_sum():
    """The check has teeth: a left-to-right sum of the same terms differs in the last bits for some
    inputs, so matching the tree (not just the value) is what the kernels must do."""
    rng = np.random.default_rng(1)
    differs = 0
    for _ in range(200):
        e = (rng.standard_normal(128) ** 2 * 1e3).astype(np.float32)
        seq = np.float32(0.0)
        for x in e:
            seq = np.float32(seq + x)
        differs += int(seq.tobytes() != _lane_tree(e).tobytes())
    assert differs > 0


def _lane_tree_argmax(v: np.ndarray, f0: int):
    """tokens on N: lane l scans f = l + 32 i, then the xor butterfly merges (value, index) pairs;
    a pair replaces the running one if its value is larger, or equal with a smaller index."""
    best = [np.float32(-np.inf)] * 32
    idx = [0x7FFFFFFF] * 32
    for lane in range(32):
        for i in range(4):
            x, F = v[lane + 32 * i], f0 + lane + 32 * i
            if x > best[lane] or (x == best[lane] and F < idx[lane]):
                best[lane], idx[lane] = x, F
    for off in (16, 8, 4, 2, 1):
        nb, ni = list(best), list(idx)
        for lane in range(32):
            ob, oi = best[lane ^ off], idx[lane ^ off]
            if ob > best[lane] or (ob == best[lane] and oi < idx[lane]):
                nb[lane], ni[lane] = ob, oi
        best, idx = nb, ni
    return best[0], idx[0]


def _register_argmax(v: np.ndarray, f0: int):
    """tokens on M: per group of 16 columns, a NaN-ignoring maximum and the first index holding it
    (reverse scan); groups ascend, and a group replaces the running pair if its maximum is larger,
    or if no index was found yet and it equals the running maximum."""
    best, best_i = np.float32(-np.inf), 0x7FFFFFFF
    for c in range(8):
        g = v[16 * c:16 * c + 16]
        m = g[0]
        for x in g[1:]:
            m = np.float32(np.fmax(m, x))
        mi = 0x7FFFFFFF
        for j in range(15, -1, -1):
            if g[j] == m:
                mi = f0 + 16 * c + j
        if m > best or (best_i == 0x7FFFFFFF and m == best):
            best, best_i = m, mi
    return best, best_i


def test_maximum_and_first_index_agree_with_nan_inf_and_ties():
    rng = np.random.default_rng(2)
    for trial in range(400):
        v = rng.standard_normal(128).astype(np.float32)
        kind = trial % 6
        if kind == 1:  # ties of the maximum across lanes, groups and quarters
            top = np.float32(5.0)
            v[rng.choice(128, 4, replace=False)] = top
        elif kind == 2:  # NaNs never win
            v[rng.choice(128, 10, replace=False)] = np.float32(np.nan)
        elif kind == 3:  # every value -inf: the first index
            v[:] = np.float32(-np.inf)
        elif kind == 4:  # -inf and NaN only
            v[:] = np.float32(-np.inf)
            v[rng.choice(128, 20, replace=False)] = np.float32(np.nan)
        elif kind == 5:  # all NaN: no index
            v[:] = np.float32(np.nan)
        f0 = 128 * int(rng.integers(0, 1187))
        (b1, i1), (b2, i2) = _lane_tree_argmax(v, f0), _register_argmax(v, f0)
        assert i1 == i2, (trial, kind, i1, i2)
        assert (np.isnan(b1) and np.isnan(b2)) or b1 == b2, (trial, kind, b1, b2)
        if kind == 5:
            assert i1 == 0x7FFFFFFF and b1 == -np.inf
