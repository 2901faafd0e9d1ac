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


def test_json_line_is_alone_on_stdout():
    """Writes to file descriptor 1 from native code (a library banner) land on
    stderr once bench.json_stdout() has run; the JSON line goes to stdout."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    code = (
        "import sys, ctypes\n"
        f"sys.path.insert(0, {str(root)!r})\n"
        "import bench\n"
        "out = bench.json_stdout()\n"
        "libc = ctypes.CDLL(None)\n"
        "libc.puts(b'banner from native code')\n"
        "libc.fflush(None)\n"
        "print('a python print')\n"
        "print('{\"k\": 1}', file=out, flush=True)\n"
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout == '{"k": 1}\n'
    assert "banner from native code" in r.stderr and "a python print" in r.stderr
