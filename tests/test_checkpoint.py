"""safetensors reading / writing and checkpoint directories (reference
draftkv/gpt2.py:25-46, :167-172, draftkv/llama.py:153-156).  The reader is
pinned to what the reference's own reader decodes from the same file
(tests/golden/tiny.safetensors, tests/golden/make_golden.py)."""

import json

import numpy as np
import pytest

from draftkv.checkpoint import load_config, load_dir_weights, load_safetensors, save_safetensors


def test_reader_matches_the_reference_reader(golden_dir):
    got = load_safetensors(golden_dir / "tiny.safetensors")
    want = np.load(golden_dir / "tiny_safetensors_ref.npz")
    assert sorted(k.replace(".", "_") for k in got) == sorted(want.files)
    for k, v in got.items():
        w = want[k.replace(".", "_")]
        assert v.shape == w.shape
        # floats bit-exact (bf16 widened exactly); the reference casts ints to f32
        np.testing.assert_array_equal(np.asarray(v, np.float32), w)
        if v.dtype == np.float32:
            assert np.array_equal(v.view(np.uint32), w.view(np.uint32))


def test_round_trip_and_shards(tmp_path):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    a = rng.standard_normal((64, 32)).astype(np.float32)
    b = torch.from_numpy(rng.standard_normal((16, 8)).astype(np.float32)).to(torch.bfloat16)
    save_safetensors({"x.a": a}, tmp_path / "s1.safetensors")
    save_safetensors({"x.b": b}, tmp_path / "s2.safetensors")
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(
        {"weight_map": {"x.a": "s1.safetensors", "x.b": "s2.safetensors"}}))
    w = load_dir_weights(tmp_path)
    assert np.array_equal(w["x.a"], a)
    assert np.array_equal(w["x.b"], b.float().numpy())
    t = load_dir_weights(tmp_path, device="cpu")          # stored dtypes kept
    assert t["x.b"].dtype == torch.bfloat16 and torch.equal(t["x.b"], b)
    assert t["x.a"].dtype == torch.float32


def test_config_dtype(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"hidden_size": 8, "torch_dtype": "bfloat16"}))
    assert load_config(tmp_path)["dtype"] == "bf16"
    (tmp_path / "config.json").write_text(json.dumps({"n_embd": 8, "torch_dtype": "float32"}))
    cfg = load_config(tmp_path)
    assert cfg["dtype"] == "f32" and cfg["vocab_size"] == 50257
    with pytest.raises(FileNotFoundError):
        load_dir_weights(tmp_path)
