#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run where the TriFuse reference checkout is available (by default the
``reference`` directory beside this repository's directory; override with
``TRIFUSE_REFERENCE``)::

    python tests/golden/make_golden.py

The script imports the reference's own torch operator bodies
(``overlays/executorch/backends/mlx/native_affine_ops.py``: dequantize,
native_affine_qmm / gather_qmm / embedding, native_olmoe_softmax /
topk_indices, native_take_along_last) and composes them exactly as the
reference's OLMoE export adapter does (``MoE.forward``,
``tools/export/export_native_olmoe_target.py:200-218``, plus the layer's
residual add at ``:227``).  It also runs the reference's byte-stacking
self-test (``tools/export/prepare_model.py:190-227``).  The outputs are small
``.npz`` files that the CPU tests and the GPU parity tests read; nothing at
test time touches the reference tree.

Attention has no runnable reference operator here (``mlx::rope`` and
``kvcache::update_and_attend`` live in ExecuTorch, which is absent), so the
attention fixture is produced by an independent torch restatement
(``torch.nn.functional.rms_norm`` / ``scaled_dot_product_attention``) and is
labelled as such inside the file.

Inputs are seeded synthetic tensors with BASELINE's distributions: weights
N(0, 0.02) rounded to bf16 then MLX-affine 4-bit/group-64 quantized (by the
oracle's min/max quantizer), activations N(0, 1).
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402

REF = Path(os.environ.get("TRIFUSE_REFERENCE", str(ROOT.parent / "reference")))
OPS_FILE = REF / "overlays/executorch/backends/mlx/native_affine_ops.py"
PREP_FILE = REF / "tools/export/prepare_model.py"


def load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


TORCH_ACT = {"f16": torch.float16, "bf16": torch.bfloat16}


def t_act(x, act):
    return torch.from_numpy(np.asarray(x, np.float32)).to(TORCH_ACT[act])


def n_act(t, act):
    return oracle.act_to_bits(t.float().numpy(), act)


def t_u32(q):
    return torch.from_numpy(np.asarray(q, np.uint32).astype(np.int64)).to(torch.uint32)


def t_f16(x):
    return torch.from_numpy(np.asarray(x, np.float16))


def weights(rng, shape):
    return oracle.round_bf16(rng.standard_normal(shape).astype(np.float32) * np.float32(0.02))


def experts(rng, E, H, I):
    out = {}
    for name, shape in (("gate", (E, I, H)), ("up", (E, I, H)), ("down", (E, H, I))):
        out[name] = oracle.affine_quantize(weights(rng, shape))
    return out


def reference_moe(ops, x, logits, ex, K, act):
    """MoE.forward (export_native_olmoe_target.py:200-218) with B=1, using the
    reference's torch ops; returns the intermediate tensors as numpy."""
    mlx = torch.ops.mlx
    T, H = x.shape
    xt = t_act(x, act).reshape(1, T, H)
    probabilities = mlx.native_olmoe_softmax(t_act(logits, act).reshape(1, T, -1))
    ids = mlx.native_olmoe_topk_indices(probabilities, K)
    scores = mlx.native_take_along_last(probabilities, ids)
    sorted_indices = T * K >= 64
    inputs = xt.unsqueeze(-2).unsqueeze(-2)
    if sorted_indices:
        flat = ids.flatten()
        order = torch.argsort(flat, dim=-1).to(torch.int32)
        inverse = torch.argsort(order, dim=-1).to(torch.int32)
        inputs = torch.index_select(inputs.flatten(0, -3), 0, order // K)
        selected = torch.index_select(flat, 0, order)
    else:
        selected = ids

    def expert(name, inp):
        q, s, b = ex[name]
        return mlx.native_affine_gather_qmm(inp, t_u32(q), t_f16(s), t_f16(b), selected, 64, 4,
                                            sorted_indices)

    up = expert("up", inputs)
    gate = expert("gate", inputs)
    h = torch.nn.functional.silu(gate) * up
    out = expert("down", h)
    if sorted_indices:
        out = torch.index_select(out, 0, inverse).reshape(1, T, K, 1, H)
    moe = (out.squeeze(-2) * scores.unsqueeze(-1)).sum(dim=-2)
    return dict(
        probabilities=n_act(probabilities.reshape(T, -1), act),
        ids=ids.reshape(T, K).numpy().astype(np.int32),
        scores=n_act(scores.reshape(T, K), act),
        moe=n_act(moe.reshape(T, H), act),
        expert_out=n_act(out.reshape(T, K, H), act),
        sorted=np.array(sorted_indices),
    )


def make_moe(ops, name, seed, T, H, I, E, K, act, dense_router=True):
    rng = np.random.default_rng(seed)
    x = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    residual = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    ex = experts(rng, E, H, I)
    if dense_router:
        wr = oracle.to_act(weights(rng, (E, H)), act)
        logits_t = (t_act(x, act).float() @ t_act(wr, act).float().T).to(TORCH_ACT[act])
        router = dict(router_w=oracle.act_to_bits(wr, act))
    else:
        rq, rs, rb = oracle.affine_quantize(weights(rng, (E, H)))
        logits_t = torch.ops.mlx.native_affine_qmm(t_act(x, act), t_u32(rq), t_f16(rs), t_f16(rb), 64, 4)
        router = dict(router_q=rq, router_s=rs, router_b=rb)
    logits = oracle.bits_to_act(n_act(logits_t, act), act)
    ref = reference_moe(ops, x, logits, ex, K, act)
    layer_out = (t_act(residual, act) + t_act(oracle.bits_to_act(ref["moe"], act), act)).float()
    arrays = dict(
        x=oracle.act_to_bits(x, act), residual=oracle.act_to_bits(residual, act),
        logits=n_act(logits_t, act),
        gate_q=ex["gate"][0], gate_s=ex["gate"][1], gate_b=ex["gate"][2],
        up_q=ex["up"][0], up_s=ex["up"][1], up_b=ex["up"][2],
        down_q=ex["down"][0], down_s=ex["down"][1], down_b=ex["down"][2],
        layer_out=oracle.act_to_bits(layer_out.numpy(), act),
        meta=np.array(json.dumps(dict(T=T, H=H, I=I, E=E, K=K, act=act, seed=seed,
                                      dense_router=dense_router))),
        **router, **ref)
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    return arrays


def make_config1(ops):
    """BASELINE config 1 at full geometry (T=32, H=2048, E=64, K=8, I=1024,
    bf16, dense bf16 router), composed from the reference's operators as
    ``MoE.forward`` does.  The inputs are regenerated from a seed at test time
    (``config1_inputs.py``); the fixture keeps the reference's outputs and a
    digest of the inputs."""
    sys.path.insert(0, str(HERE))
    import config1_inputs as c1
    x, residual, ex, wr = c1.generate()
    act = c1.ACT
    logits_t = (t_act(x, act).float() @ t_act(wr, act).float().T).to(TORCH_ACT[act])
    logits = oracle.bits_to_act(n_act(logits_t, act), act)
    ref = reference_moe(ops, x, logits, ex, c1.K, act)
    layer_out = (t_act(residual, act) + t_act(oracle.bits_to_act(ref["moe"], act), act)).float()
    arrays = dict(
        logits=n_act(logits_t, act), probabilities=ref["probabilities"], ids=ref["ids"], scores=ref["scores"],
        moe=ref["moe"], layer_out=oracle.act_to_bits(layer_out.numpy(), act),
        digest=np.array(c1.digest(x, residual, ex, wr)),
        meta=np.array(json.dumps(dict(T=c1.T, H=c1.H, I=c1.I, E=c1.E, K=c1.K, act=act, seed=c1.SEED,
                                      dense_router=True, sorted=bool(ref["sorted"])))))
    np.savez_compressed(HERE / "config1_full.npz", **arrays)


def make_ops(ops):
    """Single-operator fixtures: dequantize, qmm, gather_qmm (both call forms),
    embedding, softmax/top-k on crafted rows with ties, NaN and +-inf."""
    rng = np.random.default_rng(7)
    E, O, H = 6, 64, 256
    q, s, b = oracle.affine_quantize(weights(rng, (E, O, H)))
    deq = ops.dequantize_reference(t_u32(q), t_f16(s), t_f16(b), 64, 4).numpy()
    out = dict(q=q, s=s, b=b, dequant=deq.view(np.uint16))
    for act in ("f16", "bf16"):
        x = oracle.to_act(rng.standard_normal((10, H)).astype(np.float32), act)
        idx = rng.integers(0, E, size=(10,)).astype(np.int32)
        qmm = torch.ops.mlx.native_affine_qmm(t_act(x, act), t_u32(q[0]), t_f16(s[0]), t_f16(b[0]), 64, 4)
        gq = torch.ops.mlx.native_affine_gather_qmm(t_act(x, act).reshape(10, 1, H), t_u32(q), t_f16(s),
                                                   t_f16(b), torch.from_numpy(idx), 64, 4, True)
        # Broadcast call form of the unsorted path: x[1,T,1,1,H] with idx[1,T,K].
        ib = rng.integers(0, E, size=(1, 5, 3)).astype(np.int32)
        gb = torch.ops.mlx.native_affine_gather_qmm(t_act(x[:5], act).reshape(1, 5, 1, 1, H), t_u32(q),
                                                   t_f16(s), t_f16(b), torch.from_numpy(ib), 64, 4, False)
        out.update({f"x_{act}": oracle.act_to_bits(x, act), f"idx_{act}": idx,
                    f"qmm_{act}": n_act(qmm, act), f"gather_{act}": n_act(gq.reshape(10, O), act),
                    f"bidx_{act}": ib.reshape(5, 3), f"gather_bcast_{act}": n_act(gb.reshape(5, 3, O), act)})
    ids = rng.integers(0, O, size=(7,)).astype(np.int64)
    emb = torch.ops.mlx.native_affine_embedding(torch.from_numpy(ids), t_u32(q[0]), t_f16(s[0]),
                                                t_f16(b[0]), 64, 4)
    out.update(emb_ids=ids, emb=emb.numpy().view(np.uint16))
    # Router rows: random, exact ties, NaN, +inf, all-equal.
    for act in ("f16", "bf16"):
        lg = rng.standard_normal((12, 64)).astype(np.float32) * 2
        lg[1, 10:20] = 1.5
        lg[2, :] = 0.25
        lg[3, 5] = np.nan
        lg[4, 7] = np.inf
        lg[5, 40:48] = 3.0
        lg[5, 8:16] = 3.0
        lg[6] = np.round(lg[6] * 2) / 2  # many coarse ties
        lg[7, :] = -np.inf
        lg[7, 3] = 0.0
        lg = oracle.to_act(lg, act)
        lt = t_act(lg, act).reshape(1, 12, 64)
        p = torch.ops.mlx.native_olmoe_softmax(lt)
        k = torch.ops.mlx.native_olmoe_topk_indices(p, 8)
        g = torch.ops.mlx.native_take_along_last(p, k)
        out.update({f"route_logits_{act}": oracle.act_to_bits(lg, act),
                    f"route_probs_{act}": n_act(p.reshape(12, 64), act),
                    f"route_ids_{act}": k.reshape(12, 8).numpy().astype(np.int32),
                    f"route_gates_{act}": n_act(g.reshape(12, 8), act)})
    np.savez_compressed(HERE / "ops.npz", **out)


def make_attention():
    """Independent torch restatement of the attention block math for one
    decode step and one 5-token chunk (not a reference operator)."""
    rng = np.random.default_rng(11)
    Hh, D, L0 = 4, 128, 37
    H = Hh * D
    theta, eps = 10000.0, 1e-5
    out = {"provenance": np.array("torch restatement: F.rms_norm full width, half-split RoPE "
                                  "theta^(-2i/D) in fp32, F.scaled_dot_product_attention in fp32")}
    for T in (1, 5):
        q = rng.standard_normal((T, H)).astype(np.float32)
        k = rng.standard_normal((T, H)).astype(np.float32)
        v = oracle.round_f16(rng.standard_normal((T, H)).astype(np.float32))
        qn_w = oracle.round_f16(1 + 0.1 * rng.standard_normal(H).astype(np.float32))
        kn_w = oracle.round_f16(1 + 0.1 * rng.standard_normal(H).astype(np.float32))
        kc = oracle.round_f16(rng.standard_normal((Hh, L0, D)).astype(np.float32))
        vc = oracle.round_f16(rng.standard_normal((Hh, L0, D)).astype(np.float32))
        qh = torch.from_numpy(q).half()
        kh = torch.from_numpy(k).half()

        def norm(x, w):
            return torch.nn.functional.rms_norm(x.float(), (H,), torch.from_numpy(w).float(), eps).half()

        def rope(x, pos):
            x = x.float().reshape(T, Hh, D)
            inv = torch.from_numpy(oracle.rope_inv_freq(D, theta))
            ang = torch.tensor(pos, dtype=torch.float32)[:, None] * inv
            c, s_ = torch.cos(ang)[:, None], torch.sin(ang)[:, None]
            x1, x2 = x[..., :D // 2], x[..., D // 2:]
            return torch.cat([x1 * c - x2 * s_, x1 * s_ + x2 * c], -1).half()

        pos = list(range(L0, L0 + T))
        qr = rope(norm(qh, qn_w), pos)
        kr = rope(norm(kh, kn_w), pos)
        K = torch.cat([torch.from_numpy(kc).half(), kr.transpose(0, 1)], 1)
        V = torch.cat([torch.from_numpy(vc).half(), torch.from_numpy(v).half().reshape(T, Hh, D).transpose(0, 1)], 1)
        L = L0 + T
        mask = None
        if T > 1:
            mask = torch.arange(L)[None, :] <= (L0 + torch.arange(T))[:, None]
        o = torch.nn.functional.scaled_dot_product_attention(
            qr.transpose(0, 1).float(), K.float(), V.float(), attn_mask=mask, scale=D ** -0.5)
        o = o.transpose(0, 1).reshape(T, H).half()
        out.update({f"t{T}_q": q.astype(np.float16).view(np.uint16),
                    f"t{T}_k": k.astype(np.float16).view(np.uint16),
                    f"t{T}_v": v.astype(np.float16).view(np.uint16),
                    f"t{T}_qn": qn_w.astype(np.float16).view(np.uint16),
                    f"t{T}_kn": kn_w.astype(np.float16).view(np.uint16),
                    f"t{T}_kc": kc.astype(np.float16).view(np.uint16),
                    f"t{T}_vc": vc.astype(np.float16).view(np.uint16),
                    f"t{T}_out": o.numpy().view(np.uint16)})
    out["meta"] = np.array(json.dumps(dict(Hh=Hh, D=D, L0=L0, theta=theta, eps=eps)))
    np.savez_compressed(HERE / "attention.npz", **out)


def main():
    if not OPS_FILE.exists():
        raise SystemExit(f"reference operator file not found: {OPS_FILE}")
    torch.manual_seed(0)
    ops = load(OPS_FILE, "trifuse_native_affine_ops")
    prep = load(PREP_FILE, "trifuse_prepare_model")
    make_ops(ops)
    # Reduced geometry (H=256, I=128, E=8/16): sorted (T*K >= 64) and unsorted paths.
    make_moe(ops, "moe_small_sorted_bf16", 101, T=24, H=256, I=128, E=8, K=4, act="bf16")
    make_moe(ops, "moe_small_unsorted_f16", 102, T=8, H=256, I=128, E=8, K=4, act="f16",
             dense_router=False)
    make_moe(ops, "moe_small_sorted_f16", 103, T=40, H=256, I=128, E=16, K=8, act="f16",
             dense_router=False)
    make_attention()
    # BASELINE config 1 at its full geometry (inputs regenerated from a seed).
    make_config1(ops)
    stack = prep.self_test()
    (HERE / "prepare_model_selftest.json").write_text(json.dumps(stack, indent=1) + "\n")
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
