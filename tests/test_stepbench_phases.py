"""stepbench --phases: the per-kind medians of the launch stamps (host logic, no GPU).

A launch's stamps are [phases][earliest CTA, latest CTA] in global-timer nanoseconds; 0 or all
ones mean "not reached".  Each phase is reported in microseconds after the launch's first CTA past
its dependency wait (phase 1), as the median over the launches of one kind, and each launch's gap
is measured from the previous stamped launch's last exit.
"""

import json

import numpy as np

from fast_dllm_relax_b200.stepbench import print_phases

UNSET = np.iinfo(np.uint64).max


def _launch(t0, wait_hi, p2, exit_lo, exit_hi):
    st = np.zeros((12, 2), dtype=np.uint64)
    st[1] = [t0, wait_hi]
    st[2] = p2
    st[7] = [exit_lo, exit_hi]
    return st


def test_medians_gaps_and_unreached_phases(capsys):
    stamps = np.stack([
        _launch(1_000, 1_500, [3_000, 4_000], 6_000, 8_000),     # qkv
        _launch(9_000, 9_100, [UNSET, UNSET], 12_000, 13_000),   # attention; phase 2 not reached
        _launch(20_000, 20_200, [22_000, 25_000], 26_000, 29_000),  # qkv again
        _launch(0, 0, [0, 0], 0, 0),                                # never started: skipped
    ])
    kinds = np.array([101, 1, 101, 102], dtype=np.int32)
    print_phases(stamps, kinds)
    out = [json.loads(line) for line in capsys.readouterr().out.splitlines()]
    assert [o["kind"] for o in out] == [101, 1]
    qkv, attn = out
    assert qkv["name"] == "qkv" and qkv["launches"] == 2
    assert qkv["phases_us"]["1"] == [0.0, 0.35]                       # medians of 0.5 and 0.2 us
    assert qkv["phases_us"]["2"] == [2.0, 4.0]                        # medians of (2, 3) and (5, 5)
    assert qkv["phases_us"]["7"] == [5.5, 8.0]
    assert qkv["gap_before_us"] == 7.0                                # 20000 - 13000 ns
    assert attn["gap_before_us"] == 1.0                               # 9000 - 8000 ns
    assert "2" not in attn["phases_us"]                               # never reached
