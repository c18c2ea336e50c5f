"""MLX-affine 4-bit packing and seeded synthetic OLMoE checkpoints (torch).

Model-prep tooling, not the hot path: the bench and tests use it to build
random-init weights with BASELINE's distributions (N(0, 0.02) in bf16, then
affine 4-bit / group 64 with float16 scale and bias) directly on the GPU.
The packing is the one the reference consumes: eight 4-bit codes per uint32,
code j at bits 4j (overlays/executorch/backends/mlx/native_affine_ops.py:
29-36).  Checkpoint names follow the OLMoE exporter's inventory
(tools/export/export_native_olmoe_target.py:66-89), with experts stacked
[E, ...] in expert order as tools/export/prepare_model.py produces.
"""
from __future__ import annotations

import torch

GROUP = 64
BITS = 4


def pack_codes(codes: torch.Tensor) -> torch.Tensor:
    """int codes [..., in] (0..15) -> uint32 [..., in/8]."""
    c = codes.to(torch.int64).reshape(*codes.shape[:-1], codes.shape[-1] // 8, 8)
    shifts = torch.arange(8, device=codes.device, dtype=torch.int64) * 4
    words = (c << shifts).sum(-1)
    return words.to(torch.uint32) if words.device.type == "cpu" else words.to(torch.int64).to(torch.uint32)


def affine_quantize(w: torch.Tensor, group: int = GROUP):
    """fp32/bf16 weights [..., in] -> (q uint32 [..., in/8], scales f16, biases f16).

    Same arithmetic as oracle.affine_quantize: scale = (max - min) / 15 stored
    as f16 (floored at 1e-7 before rounding), bias = min as f16, codes =
    clamp(round_half_even((w - b16) / s16), 0, 15)."""
    w = w.float()
    shape = w.shape
    g = w.reshape(*shape[:-1], shape[-1] // group, group)
    lo = g.amin(-1)
    hi = g.amax(-1)
    scale = (hi - lo) / 15.0
    scale = torch.where(scale > 1e-7, scale, torch.full_like(scale, 1e-7))
    s16 = scale.to(torch.float16)
    b16 = lo.to(torch.float16)
    codes = torch.round((g - b16.float()[..., None]) / s16.float()[..., None])
    codes = codes.clamp(0, 15).reshape(shape)
    return pack_codes(codes), s16.contiguous(), b16.contiguous()


def random_affine(shape, gen: torch.Generator, device, std=0.02, chunk_rows=8192):
    """N(0, std) bf16 weights of `shape` quantized chunk by chunk (bounded memory)."""
    *lead, rows, cols = shape
    n = 1
    for d in lead:
        n *= d
    total = n * rows
    qs, ss, bs = [], [], []
    for r0 in range(0, total, chunk_rows):
        r = min(chunk_rows, total - r0)
        w = (torch.randn((r, cols), generator=gen, device=device) * std).to(torch.bfloat16)
        q, s, b = affine_quantize(w)
        qs.append(q)
        ss.append(s)
        bs.append(b)
    q = torch.cat(qs).reshape(*lead, rows, cols // 8)
    s = torch.cat(ss).reshape(*lead, rows, cols // GROUP)
    b = torch.cat(bs).reshape(*lead, rows, cols // GROUP)
    return q, s, b


def synthetic_olmoe(cfg, seed: int = 20260102, device="cuda"):
    """Random-init OLMoE checkpoint: dict checkpoint-name -> tensor.

    cfg needs layers, hidden, heads, head_dim, intermediate, vocab, experts."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    H, W, I, E, V = cfg.hidden, cfg.heads * cfg.head_dim, cfg.intermediate, cfg.experts, cfg.vocab
    out = {}

    def put(name, shape):
        q, s, b = random_affine(shape, gen, device)
        out[name + ".weight"], out[name + ".scales"], out[name + ".biases"] = q, s, b

    def norm(name, width):
        out[name] = (1.0 + 0.1 * torch.randn(width, generator=gen, device=device)).to(torch.float16)

    put("model.embed_tokens", (V, H))
    put("lm_head", (V, H))
    norm("model.norm.weight", H)
    for layer in range(cfg.layers):
        p = f"model.layers.{layer}."
        norm(p + "input_layernorm.weight", H)
        norm(p + "post_attention_layernorm.weight", H)
        norm(p + "self_attn.q_norm.weight", W)
        norm(p + "self_attn.k_norm.weight", W)
        for n in ("q_proj", "k_proj", "v_proj"):
            put(p + "self_attn." + n, (W, H))
        put(p + "self_attn.o_proj", (H, W))
        put(p + "mlp.gate", (E, H))
        put(p + "mlp.switch_mlp.gate_proj", (E, I, H))
        put(p + "mlp.switch_mlp.up_proj", (E, I, H))
        put(p + "mlp.switch_mlp.down_proj", (E, H, I))
    return out
