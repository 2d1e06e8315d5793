"""The two summation orders of a vocabulary slab's sum of exponentials (CPU, float32).

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
