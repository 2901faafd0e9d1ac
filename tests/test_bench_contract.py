"""Host-side logic of bench.py that needs no GPU."""

import bench


def test_attention_split_keeps_one_wave_of_equal_splits():
    # configuration 4: 4 sequences x 8 KV heads, context growing to 33829
    s = bench.attention_split(32768, 33829, 32)
    assert s % 64 == 0
    n = -(-33829 // s)
    assert n * 32 <= 2 * 148                 # one wave of two CTAs per SM
    assert (n - 1) * s < 33829 <= n * s      # the last split is not nearly empty
    assert s == 3776


def test_attention_split_for_many_pairs_is_a_power_of_two():
    # 32 sequences x 8 heads: more pairs than SMs
    s = bench.attention_split(32768, 33000, 256)
    assert s == 4096
    assert bench.attention_split(2048, 2300, 256) == 512


def test_attention_split_single_pair_and_short_context():
    assert bench.attention_split(128, 300, 12) % 64 == 0
    assert bench.attention_split(128, 300, 12) >= 64
