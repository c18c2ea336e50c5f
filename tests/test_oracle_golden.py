"""Pin the CPU oracle against fixtures produced by the reference's own torch
operators (tests/golden/make_golden.py).  CPU only."""
import json

import numpy as np
import pytest

import oracle
from oracle import bits_to_act

from tests.parity import assert_close


def load(golden_dir, name):
    z = np.load(golden_dir / f"{name}.npz")
    meta = json.loads(str(z["meta"])) if "meta" in z.files else {}
    return z, meta


def test_dequantize_bit_exact(golden_dir):
    z = np.load(golden_dir / "ops.npz")
    ours = oracle.dequantize(z["q"], z["s"], z["b"])
    ref = z["dequant"].view(np.float16).astype(np.float32)
    assert np.array_equal(ours.view(np.uint32), ref.view(np.uint32))


def test_pack_unpack_roundtrip():
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 16, size=(3, 5, 64)).astype(np.uint32)
    assert np.array_equal(oracle.unpack_codes(oracle.pack_codes(codes)), codes)


@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_qmm_and_gather_against_reference(golden_dir, act):
    z = np.load(golden_dir / "ops.npz")
    x = bits_to_act(z[f"x_{act}"], act)
    q, s, b = z["q"], z["s"], z["b"]
    assert_close(oracle.affine_qmm(x, q[0], s[0], b[0], act), bits_to_act(z[f"qmm_{act}"], act), act)
    assert_close(oracle.gather_qmm(x, q, s, b, z[f"idx_{act}"], act), bits_to_act(z[f"gather_{act}"], act), act)
    # Broadcast (unsorted) call form: token t's row is used by each of its K experts.
    ib = z[f"bidx_{act}"]
    rows = np.repeat(x[:5], ib.shape[1], axis=0)
    got = oracle.gather_qmm(rows, q, s, b, ib.reshape(-1), act).reshape(5, ib.shape[1], -1)
    assert_close(got, bits_to_act(z[f"gather_bcast_{act}"], act), act)


def test_embedding_bit_exact(golden_dir):
    z = np.load(golden_dir / "ops.npz")
    got = oracle.affine_embedding(z["emb_ids"], z["q"][0], z["s"][0], z["b"][0], "f16")
    ref = z["emb"].view(np.float16).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_route_bit_exact_with_ties_nan_inf(golden_dir, act):
    z = np.load(golden_dir / "ops.npz")
    logits = bits_to_act(z[f"route_logits_{act}"], act)
    probs = oracle.olmoe_softmax(logits, act)
    ref_p = bits_to_act(z[f"route_probs_{act}"], act)
    same = (probs.view(np.uint32) == ref_p.view(np.uint32)) | (np.isnan(probs) & np.isnan(ref_p))
    assert same.all(), np.argwhere(~same)
    idx, gates = oracle.olmoe_route(logits, 8, act)
    assert np.array_equal(idx, z[f"route_ids_{act}"])
    ref_g = bits_to_act(z[f"route_gates_{act}"], act)
    assert np.array_equal(np.isnan(gates), np.isnan(ref_g))
    assert np.array_equal(np.nan_to_num(gates), np.nan_to_num(ref_g))


@pytest.mark.parametrize("name", ["moe_small_sorted_bf16", "moe_small_unsorted_f16", "moe_small_sorted_f16"])
def test_moe_block_against_reference_composition(golden_dir, name):
    z, m = load(golden_dir, name)
    act, K = m["act"], m["K"]
    x = bits_to_act(z["x"], act)
    res = bits_to_act(z["residual"], act)
    logits = bits_to_act(z["logits"], act)
    # Routing given the reference's logits: bit-exact.
    idx, gates = oracle.olmoe_route(logits, K, act)
    assert np.array_equal(idx, z["ids"])
    assert np.array_equal(gates.view(np.uint32), bits_to_act(z["scores"], act).view(np.uint32))
    assert np.array_equal(oracle.olmoe_softmax(logits, act).view(np.uint32),
                          bits_to_act(z["probabilities"], act).view(np.uint32))
    # The route sort groups experts exactly as the reference's argsort does.
    order, inverse, offsets = oracle.route_sort(idx, m["E"])
    flat = idx.reshape(-1)
    assert np.array_equal(np.sort(flat, kind="stable"), flat[order])
    assert np.array_equal(order[inverse], np.arange(flat.size))
    assert offsets[-1] == flat.size
    # Whole block (given the same logits) within tolerance of the reference.
    ex = {n: (z[f"{n}_q"], z[f"{n}_s"], z[f"{n}_b"]) for n in ("gate", "up", "down")}
    sel = flat[order]
    rows = x[order // K]
    up = oracle.gather_qmm(rows, *ex["up"], sel, act)
    gate = oracle.gather_qmm(rows, *ex["gate"], sel, act)
    h = oracle.swiglu(gate, up, act)
    y = oracle.gather_qmm(h, *ex["down"], sel, act)[inverse].reshape(x.shape[0], K, -1)
    assert_close(y, bits_to_act(z["expert_out"], act), act)
    out = oracle.combine(y, gates, res, act)
    assert_close(out, bits_to_act(z["layer_out"], act), act)


@pytest.mark.parametrize("name", ["moe_small_sorted_bf16", "moe_small_unsorted_f16", "moe_small_sorted_f16"])
def test_router_gemv_matches_reference_linear(golden_dir, name):
    """The oracle's fixed-order router GEMV is within one act ulp of the
    reference's torch linear and, on these fixtures, equal to it bit for bit
    (a flip would name how many logits differ)."""
    z, m = load(golden_dir, name)
    act = m["act"]
    x = bits_to_act(z["x"], act)
    if m["dense_router"]:
        got = oracle.router_logits_dense(x, bits_to_act(z["router_w"], act), act)
    else:
        got = oracle.router_logits_affine(x, z["router_q"], z["router_s"], z["router_b"], act)
    ref = bits_to_act(z["logits"], act)
    assert_close(got, ref, act)
    flips = int((oracle.act_to_bits(got, act) != oracle.act_to_bits(ref, act)).sum())
    assert flips == 0, f"{flips} of {got.size} router logits differ from the reference's linear"


def test_attention_against_torch_restatement(golden_dir):
    z = np.load(golden_dir / "attention.npz")
    m = json.loads(str(z["meta"]))
    Hh, D, L0 = m["Hh"], m["D"], m["L0"]
    cfg = oracle.OLMoEConfig(heads=Hh, head_dim=D, hidden=Hh * D, rms_eps=m["eps"],
                             rope_theta=m["theta"], act="f16")
    for T in (1, 5):
        f = lambda k: z[f"t{T}_{k}"].view(np.float16).astype(np.float32)  # noqa: E731
        q = oracle.rms_norm(f("q"), f("qn"), cfg.rms_eps, "f16")
        k = oracle.rms_norm(f("k"), f("kn"), cfg.rms_eps, "f16")
        pos = np.arange(L0, L0 + T)
        q = oracle.rope(q.reshape(T, Hh, D), pos, cfg.rope_theta, "f16")
        k = oracle.rope(k.reshape(T, Hh, D), pos, cfg.rope_theta, "f16")
        K = np.concatenate([f("kc").reshape(Hh, L0, D), k.transpose(1, 0, 2)], 1)
        V = np.concatenate([f("vc").reshape(Hh, L0, D), f("v").reshape(T, Hh, D).transpose(1, 0, 2)], 1)
        o = oracle.sdpa(q, K, V, cfg.attn_scale, "f16", causal_offset=L0 if T > 1 else None)
        assert_close(o.reshape(T, -1), f("out"), "f16")


def test_reference_stacking_selftest_passed(golden_dir):
    rec = json.loads((golden_dir / "prepare_model_selftest.json").read_text())
    assert rec["status"] == "passed" and rec["missing_expert_rejected"]


def test_quantizer_roundtrip_error_bounded():
    rng = np.random.default_rng(3)
    w = oracle.round_bf16(rng.standard_normal((4, 256)).astype(np.float32) * 0.02)
    q, s, b = oracle.affine_quantize(w)
    deq = oracle.dequantize(q, s, b)
    step = np.repeat(s.astype(np.float32), 64, axis=-1)
    assert np.all(np.abs(deq - w) <= 0.5 * step + 1e-3)


def test_bf16_rounding_matches_torch():
    import torch
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(10000) * 10.0 ** rng.integers(-8, 8, 10000)).astype(np.float32)
    x[:4] = [np.inf, -np.inf, 0.0, -0.0]
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(oracle.round_bf16(x).view(np.uint32), ref.view(np.uint32))


def test_config1_full_geometry_against_reference(golden_dir):
    """BASELINE config 1 at its full geometry (T=32, H=2048, E=64, top-8,
    I=1024, bf16, dense router) against the reference's own operators: the
    inputs are rebuilt from their seed and must hash to the recorded digest;
    routing the reference's logits reproduces its ids and gates bit for bit;
    the oracle's fixed-order router logits are within one ulp of the
    reference's linear (their flips are counted) and its block routes every
    token as the reference does, with the output within tolerance."""
    import sys
    sys.path.insert(0, str(golden_dir))
    import config1_inputs as c1
    z = np.load(golden_dir / "config1_full.npz")
    x, res, ex, wr = c1.generate()
    assert c1.digest(x, res, ex, wr) == str(z["digest"]), "regenerated inputs differ from the reference's"
    act = c1.ACT
    ref_logits = bits_to_act(z["logits"], act)
    probs = oracle.olmoe_softmax(ref_logits, act)
    ids = oracle.olmoe_topk(probs, c1.K)
    assert np.array_equal(ids, z["ids"])
    assert np.array_equal(oracle.act_to_bits(np.take_along_axis(probs, ids, -1), act), z["scores"])
    got = oracle.router_logits_dense(x, wr, act)
    assert_close(got, ref_logits, act)
    flips = int((oracle.act_to_bits(got, act) != z["logits"]).sum())
    assert flips <= 2, f"{flips} of {got.size} router logits differ from the reference's linear"
    out, aux = oracle.moe_block(x, res, ("dense", wr), ex, c1.K, act)
    assert np.array_equal(aux["indices"], z["ids"]), "routing differs from the reference"
    assert np.array_equal(oracle.act_to_bits(aux["gates"], act), z["scores"])
    assert_close(out, bits_to_act(z["layer_out"], act), act)
