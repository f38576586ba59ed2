"""bench.py's algorithmic bytes, the numerator of every roofline fraction it
reports, on the CPU.

A single-token step reads each 16-bit weight once -- per layer the self
q, k, v, o (4d^2), the cross q and o (2d^2), fc1 and fc2 (2dF), and the tied
logits' V x d table once a step -- plus each window's cross keys and values
(L x 2 x X x d) and its self keys and values up to the step's position.
These are the per-configuration figures of the benchmark configurations:
weights 56.3 MB (tiny.en), 97.1 (base.en), 278 (small.en), 811 (medium.en),
1 601 (large-v3); cross keys and values 9.2, 18.4, 55.3, 147.5 and 245.8 MB a
window.
"""
import pytest

import bench
from whispereacp_b200.synthetic import CONFIGS

WEIGHT_MB = {"tiny_en_b1": 56.35, "base_en_b1": 97.15, "small_en_b32": 277.84, "medium_en_b64": 810.86,
             "large_v3_b128": 1600.78}
CROSS_MB_A_WINDOW = {"tiny_en_b1": 9.216, "base_en_b1": 18.432, "small_en_b32": 55.296, "medium_en_b64": 147.456,
                     "large_v3_b128": 245.76}


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_a_steps_algorithmic_bytes(name):
    run = CONFIGS[name]
    s = run.shape
    none = bench.step_bytes(run, run.windows, 0.0)
    assert none["weights"] / 1e6 == pytest.approx(WEIGHT_MB[name], abs=0.01)
    # With no self keys, the key and value bytes are the windows' cross rows.
    assert none["kv"] / 1e6 == pytest.approx(run.windows * CROSS_MB_A_WINDOW[name], rel=1e-12)
    # Each self key adds 2 x d 16-bit values a layer and window.
    keys = 113.5
    some = bench.step_bytes(run, run.windows, keys)
    assert some["weights"] == none["weights"]
    assert some["kv"] - none["kv"] == pytest.approx(run.windows * s.layers * 2 * s.width * keys * 2, rel=1e-12)


def test_the_bytes_scale_with_the_windows_of_a_rank():
    run = CONFIGS["medium_en_b64"]
    whole = bench.step_bytes(run, 64, 113.5)
    eighth = bench.step_bytes(run, 8, 113.5)
    # The weights are read once a step however few windows a rank holds.
    assert eighth["weights"] == whole["weights"]
    assert eighth["kv"] * 8 == pytest.approx(whole["kv"], rel=1e-12)
