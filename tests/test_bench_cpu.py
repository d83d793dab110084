"""The bench's work accounting on the CPU (no device): the algorithmic work per step of each
workload equals the reference measurement table's figures (forward = 4*D flops per visible
(query, key) pair, backward = 2.5x forward, causal = top-left, decode = bytes of K, V, q and
out), and the per-kernel attribution that the roofline divides by sums to the step's work."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


@pytest.mark.parametrize("name,amount,unit", [
    ("gpt2_causal_fwd_bwd", 45.141e9, "TFLOP/s"),      # config 3
    ("gpt2_dropout_fwd_bwd", 45.141e9, "TFLOP/s"),     # config 3 with dropout: same products
    ("gpt2_floatmask_fwd_bwd", 90.194e9, "TFLOP/s"),   # config 3 mask variant (non-causal)
    ("nanogpt_causal_fwd_bwd", 11.318e9, "TFLOP/s"),   # config 1
    ("mha_core_fwd_bwd", 3.758e9, "TFLOP/s"),          # config 2 core, dense L x S
    ("long_causal_fwd", 4398.2e9, "TFLOP/s"),          # config 4, forward only
])
def test_step_work_matches_the_measurement_table(name, amount, unit):
    got, u = bench.work(bench.WORKLOADS[name])
    assert u == unit
    assert got == pytest.approx(amount, rel=5e-5)


def test_decode_work_is_the_bytes_read_and_written():
    got, u = bench.work(bench.WORKLOADS["decode_splitkv"])
    assert u == "GB/s"
    assert got == 17_179_869_184 + 2_097_152  # K + V, then q + out


def test_causal_pairs_are_top_left():
    assert bench.pairs_per_head(4, 4, True) == 10
    assert bench.pairs_per_head(4, 6, True) == 10  # rows see keys <= i only
    assert bench.pairs_per_head(6, 4, True) == 10 + 2 * 4  # rows past S see every key
    assert bench.pairs_per_head(3, 5, False) == 15


@pytest.mark.parametrize("name", ["gpt2_causal_fwd_bwd", "gpt2_floatmask_fwd_bwd", "nanogpt_causal_fwd_bwd",
                                  "mha_core_fwd_bwd"])
def test_kernel_attribution_sums_to_the_step(name):
    w = bench.WORKLOADS[name]
    total, _ = bench.work(w)
    fwd = bench.kernel_work(w, "fwd_tc_d64")
    pair = bench.kernel_work(w, "bwd_tc")
    assert fwd + pair == pytest.approx(total)
    assert bench.kernel_work(w, "bwd_dkdv_tc") + bench.kernel_work(w, "bwd_dq_tc") == pytest.approx(pair)
    # the pre-pass and the mask draw carry no algorithmic flops of their own
    assert bench.kernel_work(w, "bwd_prep") == 0.0
    assert bench.kernel_work(w, "dropout_keep_bits") == 0.0
