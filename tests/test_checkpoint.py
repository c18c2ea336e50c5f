"""The checkpoint loader: safetensors parsing and validation, per-expert ->
stacked layout (byte-exact, as prepare_model.py stacks on disk), config
admission, and the full tensor set of a tiny OLMoE (no GPU needed)."""
import json
import struct

import numpy as np
import pytest

from trifuse_b200 import checkpoint as ck


def _tiny_config(**over):
    raw = dict(model_type="olmoe", num_hidden_layers=2, hidden_size=128, intermediate_size=64,
               num_attention_heads=2, num_key_value_heads=2, head_dim=64, vocab_size=96, num_experts=4,
               num_experts_per_tok=2, rms_norm_eps=1e-5, rope_theta=10000.0, norm_topk_prob=False,
               tie_word_embeddings=False, quantization={"bits": 4, "group_size": 64, "mode": "affine"})
    raw.update(over)
    return raw


def _tiny_tensors(cfg, rng, per_expert):
    out = {}
    for name, shape in ck.expected_shapes(cfg).items():
        if name.endswith("norm.weight"):
            out[name] = (1 + 0.1 * rng.standard_normal(shape)).astype(np.float16)
        elif name.endswith(".weight"):
            out[name] = rng.integers(0, 2 ** 32, size=shape, dtype=np.uint32)
        else:
            out[name] = (rng.random(shape) * 0.01).astype(np.float16)
    if per_expert:
        for name in [n for n in out if ".mlp.switch_mlp." in n]:
            stacked = out.pop(name)
            layer, proj_part = name.split(".mlp.switch_mlp.")
            for e in range(stacked.shape[0]):
                out[f"{layer}.mlp.experts.{e}.{proj_part}"] = stacked[e]
    return out


def test_stacking_is_byte_exact_and_rejects_missing_experts():
    """Distinct values per (layer, expert) in [2,2] tensors: each stacked
    tensor is the experts' bytes concatenated in expert order (the layout
    pinned by prepare_model.py:190-227, restated)."""
    t, want = {}, {}
    for layer in range(2):
        for proj in ("gate_proj", "up_proj", "down_proj"):
            for part in ("weight", "scales", "biases"):
                dt = np.uint32 if part == "weight" else np.float16
                parts = [np.full((2, 2), layer * 10 + e + 1, dt) for e in range(3)]
                for e, a in enumerate(parts):
                    t[f"model.layers.{layer}.mlp.experts.{e}.{proj}.{part}"] = a
                want[f"model.layers.{layer}.mlp.switch_mlp.{proj}.{part}"] = b"".join(a.tobytes() for a in parts)
    t["model.norm.weight"] = np.array([0.25, -2.0], np.float16)
    out = ck.stack_experts(t, layers=2, experts=3)
    assert len(out) == 19
    for name, raw in want.items():
        assert out[name].tobytes() == raw and out[name].shape == (3, 2, 2)
    assert out["model.norm.weight"].tobytes() == struct.pack("<2e", 0.25, -2.0)
    bad = dict(t)
    del bad["model.layers.0.mlp.experts.1.gate_proj.weight"]
    with pytest.raises(ValueError):
        ck.stack_experts(bad, layers=2, experts=3)


def test_round_trip_per_expert_and_stacked(tmp_path):
    raw = _tiny_config()
    cfg = ck.config_from_json(raw, capacity=32)
    rng = np.random.default_rng(3)
    for per_expert in (True, False):
        d = tmp_path / ("per" if per_expert else "stacked")
        d.mkdir()
        src = _tiny_tensors(cfg, rng, per_expert)
        (d / "config.json").write_text(json.dumps(raw))
        names = sorted(src)
        ck.write_safetensors(d / "model-00001.safetensors", {n: src[n] for n in names[: len(names) // 2]})
        ck.write_safetensors(d / "model-00002.safetensors", {n: src[n] for n in names[len(names) // 2:]},
                             metadata={"format": "mlx"})
        got_cfg, got = ck.load_weights(d, capacity=32)
        assert got_cfg == cfg
        assert set(got) == set(ck.expected_shapes(cfg))
        stacked = ck.stack_experts(src, cfg.layers, cfg.experts)
        for name, t in got.items():
            assert t.numpy().tobytes() == np.ascontiguousarray(stacked[name]).tobytes(), name


def test_loader_rejects_bad_layouts(tmp_path):
    cfg = ck.config_from_json(_tiny_config())
    rng = np.random.default_rng(4)
    src = _tiny_tensors(cfg, rng, False)
    (tmp_path / "config.json").write_text(json.dumps(_tiny_config()))
    extra = dict(src)
    extra["model.layers.0.mlp.extra.weight"] = np.zeros((2, 2), np.uint32)
    ck.write_safetensors(tmp_path / "m.safetensors", extra)
    with pytest.raises(ValueError, match="layout differs"):
        ck.load_weights(tmp_path)
    wrong = dict(src)
    wrong["lm_head.scales"] = wrong["lm_head.scales"].astype(np.float32)
    ck.write_safetensors(tmp_path / "m.safetensors", wrong)
    with pytest.raises(ValueError, match="lm_head.scales"):
        ck.load_weights(tmp_path)
    for over in ({"model_type": "llama"}, {"norm_topk_prob": True},
                 {"quantization": {"bits": 4, "group_size": 32, "mode": "affine"}},
                 {"quantization": {"bits": 4, "group_size": 64, "lm_head": {"bits": 8}}}):
        with pytest.raises(ValueError):
            ck.config_from_json(_tiny_config(**over))


def test_safetensors_header_checks(tmp_path):
    p = tmp_path / "x.safetensors"
    ck.write_safetensors(p, {"a": np.arange(4, dtype=np.uint32), "b": np.ones(2, np.float16)})
    got = ck.read_safetensors(p)
    assert got["a"].tolist() == [0, 1, 2, 3] and got["b"].dtype == np.float16

    def write(header, payload):
        raw = json.dumps(header).encode()
        p.write_bytes(struct.pack("<Q", len(raw)) + raw + payload)

    write({"a": {"dtype": "U32", "shape": [2], "data_offsets": [0, 8]},
           "b": {"dtype": "U32", "shape": [2], "data_offsets": [4, 12]}}, bytes(12))
    with pytest.raises(ValueError, match="gap or overlap"):
        ck.read_safetensors(p)
    write({"a": {"dtype": "U32", "shape": [3], "data_offsets": [0, 8]}}, bytes(8))
    with pytest.raises(ValueError, match="byte count"):
        ck.read_safetensors(p)
    write({"a": {"dtype": "U32", "shape": [2], "data_offsets": [0, 8]}}, bytes(12))
    with pytest.raises(ValueError, match="file size"):
        ck.read_safetensors(p)
