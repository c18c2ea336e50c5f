"""OLMoE checkpoints in the reference's on-disk layout.

A checkpoint directory holds ``config.json`` and one or more
``*.safetensors`` files with MLX affine 4-bit projections (u32 codes, f16
scales and biases, group 64) and f16 RMSNorm weights, named as the
reference's sanitized MLX layout (``tools/export/
export_native_olmoe_target.py:65-98``):

  model.embed_tokens / lm_head / model.layers.{l}.self_attn.{q,k,v,o}_proj /
  model.layers.{l}.mlp.gate (router) / model.layers.{l}.mlp.switch_mlp.
  {gate,up,down}_proj, each as .weight/.scales/.biases, plus
  model.norm.weight and the per-layer input_layernorm, post_attention_layernorm,
  self_attn.q_norm and self_attn.k_norm weights.

Expert tensors may also come one per expert
(``model.layers.{l}.mlp.experts.{e}.{proj}.{weight|scales|biases}``); they
are stacked along a leading expert axis in expert order, byte for byte, as
``tools/export/prepare_model.py:67-106`` does on disk.  Everything here is
host-side: tensors are read through a memory map and bound to a tf_model,
which copies them into its own device arena.
"""
from __future__ import annotations

import json
import math
import re
import struct
from pathlib import Path

import numpy as np
import torch

from .model import Config, Model

# safetensors dtype -> (numpy dtype, bytes per element)
_DTYPES = {"U32": (np.uint32, 4), "F16": (np.float16, 2), "F32": (np.float32, 4), "I32": (np.int32, 4),
           "I64": (np.int64, 8), "U8": (np.uint8, 1), "BF16": (np.uint16, 2)}
_EXPERT = re.compile(r"^model\.layers\.(\d+)\.mlp\.experts\.(\d+)\.(gate_proj|up_proj|down_proj)\."
                     r"(weight|scales|biases)$")
_MAX_HEADER = 16 << 20


def _require(cond, message):
    if not cond:
        raise ValueError(message)


def read_safetensors(path) -> dict:
    """name -> numpy array (read-only view of a memory map) of one
    safetensors file, with the header validated: unique names, known dtypes,
    positive shapes, byte counts matching the shapes, and payload ranges that
    tile the data section exactly (the checks of prepare_model.py:31-64)."""
    path = Path(path)
    size = path.stat().st_size
    with path.open("rb") as f:
        raw_len = f.read(8)
        _require(len(raw_len) == 8, f"{path.name}: missing safetensors header length")
        n = struct.unpack("<Q", raw_len)[0]
        _require(0 < n <= _MAX_HEADER and 8 + n <= size, f"{path.name}: invalid header length {n}")

        def no_dups(pairs):
            out = {}
            for k, v in pairs:
                _require(k not in out, f"{path.name}: duplicate key {k}")
                out[k] = v
            return out

        header = json.loads(f.read(n), object_pairs_hook=no_dups)
    _require(isinstance(header, dict), f"{path.name}: header is not an object")
    entries = {k: v for k, v in header.items() if k != "__metadata__"}
    _require(entries, f"{path.name}: no tensors")
    data_begin = 8 + n
    spans = []
    for name, t in entries.items():
        dtype, shape, off = t.get("dtype"), t.get("shape"), t.get("data_offsets")
        _require(dtype in _DTYPES, f"{path.name}: unsupported dtype {dtype} for {name}")
        _require(isinstance(shape, list) and all(type(x) is int and x > 0 for x in shape),
                 f"{path.name}: invalid shape for {name}")
        _require(isinstance(off, list) and len(off) == 2 and all(type(x) is int and x >= 0 for x in off),
                 f"{path.name}: invalid offsets for {name}")
        _require(off[1] - off[0] == math.prod(shape) * _DTYPES[dtype][1], f"{path.name}: byte count of {name}")
        spans.append((off[0], off[1]))
    cursor = 0
    for a, b in sorted(spans):
        _require(a == cursor and b > a, f"{path.name}: payload gap or overlap")
        cursor = b
    _require(size == data_begin + cursor, f"{path.name}: file size does not match the payload")
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, t in entries.items():
        a, b = t["data_offsets"]
        npdt = _DTYPES[t["dtype"]][0]
        out[name] = mm[data_begin + a:data_begin + b].view(npdt).reshape(t["shape"])
    return out


def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """Write name -> numpy array (u32, f16, f32, i32, i64, u8) as one
    safetensors file, tensors in name order."""
    rev = {np.dtype(v[0]): k for k, v in _DTYPES.items() if k != "BF16"}
    header, blobs, cursor = {}, [], 0
    if metadata:
        header["__metadata__"] = metadata
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        _require(a.dtype in rev, f"unsupported dtype {a.dtype} for {name}")
        nb = a.nbytes
        header[name] = {"dtype": rev[a.dtype], "shape": list(a.shape), "data_offsets": [cursor, cursor + nb]}
        blobs.append(a.tobytes())
        cursor += nb
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((-len(raw)) % 8)
    with Path(path).open("wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for blob in blobs:
            f.write(blob)


def stack_experts(tensors: dict, layers: int, experts: int) -> dict:
    """Replace per-expert tensors by stacked switch_mlp tensors [E, ...] in
    expert order (prepare_model.py:67-106): every (layer, projection,
    part) group must hold all experts 0..E-1 with one shape and dtype (u32
    codes, f16 scales/biases).  Already-stacked inputs pass through."""
    groups, out = {}, {}
    for name, t in tensors.items():
        m = _EXPERT.fullmatch(name)
        if not m:
            _require(".mlp.experts." not in name, f"unrecognized expert tensor {name}")
            out[name] = t
            continue
        layer, expert, proj, part = int(m[1]), int(m[2]), m[3], m[4]
        _require(layer < layers and expert < experts, f"expert tensor out of range: {name}")
        groups.setdefault((layer, proj, part), {})[expert] = t
    if not groups:
        return out
    _require(len(groups) == layers * 9, "expected gate/up/down weight/scales/biases groups for every layer")
    for (layer, proj, part), members in sorted(groups.items()):
        _require(set(members) == set(range(experts)), f"layer {layer} {proj}.{part}: missing experts")
        first = members[0]
        want = np.uint32 if part == "weight" else np.float16
        _require(first.ndim == 2 and first.dtype == want, f"layer {layer} {proj}.{part}: dtype/rank")
        _require(all(members[e].shape == first.shape and members[e].dtype == first.dtype for e in members),
                 f"layer {layer} {proj}.{part}: mismatched expert shapes")
        name = f"model.layers.{layer}.mlp.switch_mlp.{proj}.{part}"
        _require(name not in out, f"{name} given both stacked and per expert")
        out[name] = np.stack([members[e] for e in range(experts)])
    return out


def config_from_json(raw: dict, capacity: int = 4096, act: torch.dtype = torch.float16) -> Config:
    """Config of an OLMoE config.json (admission of export_native_olmoe_target.
    py:27-63 and the quantization contract of :100-116: affine, 4 bits, group
    64 everywhere; top-k weights not renormalised)."""
    _require(raw.get("model_type") == "olmoe", "expected model_type 'olmoe'")
    _require(not raw.get("norm_topk_prob", False), "norm_topk_prob must be false for OLMoE")
    _require(not raw.get("tie_word_embeddings", False), "tied embeddings are not part of this layout")
    q = raw.get("quantization", raw.get("quantization_config"))
    _require(isinstance(q, dict), "config.json needs the MLX quantization map")
    if "quantization" in raw and "quantization_config" in raw:
        _require(raw["quantization"] == raw["quantization_config"], "quantization aliases disagree")
    for name, spec in [("", q)] + [(k, v) for k, v in q.items() if isinstance(v, dict)]:
        bits = spec.get("bits", q.get("bits"))
        group = spec.get("group_size", q.get("group_size"))
        mode = spec.get("mode", q.get("mode", "affine"))
        _require(bits == 4 and group == 64 and mode == "affine",
                 f"only affine 4-bit group-64 weights are supported ({name or 'default'}: {spec})")
    heads = raw["num_attention_heads"]
    hidden = raw["hidden_size"]
    return Config(layers=raw["num_hidden_layers"], hidden=hidden, heads=heads,
                  kv_heads=raw.get("num_key_value_heads", heads), head_dim=raw.get("head_dim", hidden // heads),
                  intermediate=raw["intermediate_size"], vocab=raw["vocab_size"], experts=raw["num_experts"],
                  top_k=raw["num_experts_per_tok"], capacity=capacity, rms_eps=float(raw.get("rms_norm_eps", 1e-5)),
                  rope_theta=float(raw.get("rope_theta", 10000.0)), act=act)


def expected_shapes(cfg: Config) -> dict:
    """name -> shape of every tensor of the layout (codes as u32 words)."""
    H, I, E, V = cfg.hidden, cfg.intermediate, cfg.experts, cfg.vocab
    Wq, Wkv = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    out = {}

    def affine(name, *lead_rows_cols):
        *lead, cols = lead_rows_cols
        out[name + ".weight"] = (*lead, cols // 8)
        out[name + ".scales"] = (*lead, cols // 64)
        out[name + ".biases"] = (*lead, cols // 64)

    affine("model.embed_tokens", V, H)
    affine("lm_head", V, H)
    out["model.norm.weight"] = (H,)
    for layer in range(cfg.layers):
        p = f"model.layers.{layer}."
        out[p + "input_layernorm.weight"] = (H,)
        out[p + "post_attention_layernorm.weight"] = (H,)
        out[p + "self_attn.q_norm.weight"] = (Wq,)
        out[p + "self_attn.k_norm.weight"] = (Wkv,)
        affine(p + "self_attn.q_proj", Wq, H)
        affine(p + "self_attn.k_proj", Wkv, H)
        affine(p + "self_attn.v_proj", Wkv, H)
        affine(p + "self_attn.o_proj", H, Wq)
        affine(p + "mlp.gate", E, H)
        affine(p + "mlp.switch_mlp.gate_proj", E, I, H)
        affine(p + "mlp.switch_mlp.up_proj", E, I, H)
        affine(p + "mlp.switch_mlp.down_proj", E, H, I)
    return out


def load_weights(root, capacity: int = 4096, act: torch.dtype = torch.float16):
    """(Config, name -> CPU torch tensor) of a checkpoint directory; every
    tensor of the layout present with its exact shape and dtype, nothing
    extra (export_native_olmoe_target.py:118-135)."""
    root = Path(root)
    cfg = config_from_json(json.loads((root / "config.json").read_text()), capacity, act)
    paths = sorted(root.glob("*.safetensors"))
    _require(paths, f"no *.safetensors in {root}")
    tensors = {}
    for p in paths:
        for name, t in read_safetensors(p).items():
            _require(name not in tensors, f"tensor {name} appears in two files")
            tensors[name] = t
    tensors = stack_experts(tensors, cfg.layers, cfg.experts)
    want = expected_shapes(cfg)
    missing, extra = sorted(set(want) - set(tensors)), sorted(set(tensors) - set(want))
    _require(not missing and not extra, f"checkpoint layout differs: missing {missing[:6]}, extra {extra[:6]}")
    out = {}
    for name, shape in want.items():
        t = tensors[name]
        dt = np.uint32 if name.endswith(".weight") and not name.endswith("norm.weight") else np.float16
        _require(tuple(t.shape) == shape and t.dtype == dt,
                 f"{name}: {t.dtype}{list(t.shape)} instead of {np.dtype(dt)}{list(shape)}")
        if dt == np.float16:
            _require(bool(np.isfinite(t).all()), f"{name}: non-finite values")
        arr = np.array(t, copy=True, order="C")  # detach from the read-only memory map
        out[name] = torch.from_numpy(arr.view(np.int32) if dt == np.uint32 else arr).view(
            torch.uint32 if dt == np.uint32 else torch.float16)
    return cfg, out


def load_model(root, device: int = 0, capacity: int = 4096, act: torch.dtype = torch.float16) -> Model:
    """A device-resident Model from a checkpoint directory."""
    cfg, weights = load_weights(root, capacity, act)
    return Model(cfg, weights, device=device)
