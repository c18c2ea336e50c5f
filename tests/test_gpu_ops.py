"""GPU parity of the operator entry points against the CPU oracle and the
reference's golden vectors.  Bit-exact where the oracle says so (RMSNorm,
router GEMV, softmax, rank, route sort, combine); max-abs 2e-2 / mean-rel
5e-3 elsewhere (tests/parity.py)."""
import json

import numpy as np
import pytest
import torch

import oracle
from oracle import bits_to_act
from tests.gpu_util import bits_equal, dev, experts_dev, experts_np, host
from tests.parity import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from trifuse_b200 import ops as _ops
    return _ops


@pytest.mark.parametrize("act", ["f16", "bf16"])
@pytest.mark.parametrize("width", [256, 2048])
def test_rms_norm_bit_exact(ops, act, width):
    rng = np.random.default_rng(1)
    x = oracle.to_act(rng.standard_normal((7, width)).astype(np.float32) * 3, act)
    w = oracle.round_f16(1 + 0.1 * rng.standard_normal(width).astype(np.float32))
    got = host(ops.rms_norm(dev(x, act), dev(w.astype(np.float16)), 1e-5))
    assert bits_equal(got, oracle.rms_norm(x, w, 1e-5, act))


@pytest.mark.parametrize("act,dense,H,T", [("bf16", True, 2048, 32), ("f16", False, 2048, 64),
                                             ("bf16", False, 256, 9), ("f16", True, 512, 5),
                                             ("bf16", False, 2048, 300), ("f16", False, 2048, 2051),
                                             ("bf16", True, 1024, 4099), ("bf16", False, 256, 2500)])
def test_router_bit_exact(ops, act, dense, H, T):
    """Every router launch shape (cluster per token up to 256 tokens, one
    token per block up to 2048, sixteen per block on packed fp32 pairs
    beyond, ragged last block) gives the oracle's logits bit for bit."""
    rng = np.random.default_rng(2)
    E, K = 64, 8
    x = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    wr = oracle.round_bf16(rng.standard_normal((E, H)).astype(np.float32) * 0.02)
    if dense:
        w = oracle.to_act(wr, act)
        ref_logits = oracle.router_logits_dense(x, w, act)
        router = dev(w, act)
    else:
        q, s, b = oracle.affine_quantize(wr)
        ref_logits = oracle.router_logits_affine(x, q, s, b, act)
        router = (dev(q), dev(s), dev(b))
    logits, idx, gates = ops.olmoe_router(dev(x, act), router, K)
    assert bits_equal(host(logits), ref_logits)
    ref_idx, ref_g = oracle.olmoe_route(ref_logits, K, act)
    assert np.array_equal(host(idx), ref_idx)
    assert bits_equal(host(gates), ref_g)


@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_route_against_reference_golden(ops, golden_dir, act):
    z = np.load(golden_dir / "ops.npz")
    logits = bits_to_act(z[f"route_logits_{act}"], act)
    lt = dev(logits, act)
    probs = host(ops.native_olmoe_softmax(lt))
    assert bits_equal(probs, bits_to_act(z[f"route_probs_{act}"], act))
    idx, gates = ops.olmoe_route(lt, 8)
    assert np.array_equal(host(idx), z[f"route_ids_{act}"])
    assert bits_equal(host(gates), bits_to_act(z[f"route_gates_{act}"], act))
    top = ops.native_olmoe_topk_indices(dev(bits_to_act(z[f"route_probs_{act}"], act), act), 8)
    assert np.array_equal(host(top), z[f"route_ids_{act}"])
    took = ops.native_take_along_last(dev(bits_to_act(z[f"route_probs_{act}"], act), act), top)
    assert bits_equal(host(took), bits_to_act(z[f"route_gates_{act}"], act))


@pytest.mark.parametrize("T,K,E", [(0, 8, 64), (1, 8, 64), (3, 8, 64), (128, 8, 64), (129, 8, 64),
                                   (1000, 8, 64), (65536, 8, 64), (37, 4, 16), (100, 8, 256)])
def test_route_sort_matches_stable_argsort(ops, T, K, E):
    rng = np.random.default_rng(3)
    idx = rng.integers(0, E, size=(T, K)).astype(np.int32)
    if T > 10:
        idx[: T // 3] = rng.integers(0, 3, size=(T // 3, K))  # skewed experts
    order, inverse, offsets = ops.moe_route_sort(dev(idx), E)
    ro, ri, rf = oracle.route_sort(idx, E)
    assert np.array_equal(host(order), ro)
    assert np.array_equal(host(inverse), ri)
    assert np.array_equal(host(offsets), rf)


@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_qmm_and_gather_against_reference_golden(ops, golden_dir, act):
    z = np.load(golden_dir / "ops.npz")
    x = bits_to_act(z[f"x_{act}"], act)
    q, s, b = dev(z["q"]), dev(z["s"]), dev(z["b"])
    got = host(ops.native_affine_qmm(dev(x, act), q[0].contiguous(), s[0].contiguous(), b[0].contiguous(), 64, 4))
    assert_close(got, bits_to_act(z[f"qmm_{act}"], act))
    g = ops.native_affine_gather_qmm(dev(x, act).reshape(10, 1, -1), q, s, b, dev(z[f"idx_{act}"]), 64, 4, True)
    assert_close(host(g).reshape(10, -1), bits_to_act(z[f"gather_{act}"], act))
    ib = z[f"bidx_{act}"]
    gb = ops.native_affine_gather_qmm(dev(x[:5], act).reshape(1, 5, 1, 1, -1), q, s, b,
                                      dev(ib.reshape(1, 5, 3)), 64, 4, False)
    assert_close(host(gb).reshape(5, 3, -1), bits_to_act(z[f"gather_bcast_{act}"], act))


# The GEMV stages R rows per warp (R = 8 / 4 / 2 for 1024 / 2048 / 4096
# inputs, 1 when that leaves under 148 blocks): the last two cases take the
# multi-row form with a ragged last block (out not a multiple of 8 warps x R).
@pytest.mark.parametrize("act,T,out,inn", [("f16", 1, 6144, 2048), ("bf16", 3, 2048, 2048),
                                           ("f16", 2, 2048, 1024), ("bf16", 5, 512, 4096),
                                           ("f16", 1, 9500, 1024), ("bf16", 2, 4700, 4096)])
def test_qmm_random_against_oracle(ops, act, T, out, inn):
    rng = np.random.default_rng(4)
    x = oracle.to_act(rng.standard_normal((T, inn)).astype(np.float32), act)
    q, s, b = oracle.affine_quantize(oracle.round_bf16(rng.standard_normal((out, inn)).astype(np.float32) * 0.02))
    got = host(ops.native_affine_qmm(dev(x, act), dev(q), dev(s), dev(b), 64, 4))
    assert_close(got, oracle.affine_qmm(x, q, s, b, act))


def test_embedding_bit_exact(ops, golden_dir):
    z = np.load(golden_dir / "ops.npz")
    got = ops.native_affine_embedding(dev(z["emb_ids"]), dev(z["q"][0]), dev(z["s"][0]), dev(z["b"][0]), 64, 4)
    assert bits_equal(host(got), z["emb"].view(np.float16).astype(np.float32))


def _moe_check(ops, x, res, router_np, router_dev, ex, K, act):
    d = experts_dev(ex)
    out, aux = ops.moe(dev(x, act), dev(res, act), router_dev, d["gate"], d["up"], d["down"], K,
                       return_aux=True)
    ref, raux = oracle.moe_block(x, res, router_np, ex, K, act)
    assert bits_equal(host(aux["logits"]), raux["logits"])
    assert np.array_equal(host(aux["indices"]), raux["indices"])
    assert bits_equal(host(aux["gates"]), raux["gates"])
    assert_close(host(out), ref, ulp_act=act)
    return host(out), host(aux["indices"])


@pytest.mark.parametrize("name", ["moe_small_sorted_bf16", "moe_small_unsorted_f16", "moe_small_sorted_f16"])
def test_moe_block_against_reference_golden(ops, golden_dir, name):
    z = np.load(golden_dir / f"{name}.npz")
    m = json.loads(str(z["meta"]))
    act, K = m["act"], m["K"]
    x = bits_to_act(z["x"], act)
    res = bits_to_act(z["residual"], act)
    ex = {n: (z[f"{n}_q"], z[f"{n}_s"], z[f"{n}_b"]) for n in ("gate", "up", "down")}
    if m["dense_router"]:
        w = bits_to_act(z["router_w"], act)
        router_np, router_dev = ("dense", w), dev(w, act)
    else:
        router_np = ("affine", z["router_q"], z["router_s"], z["router_b"])
        router_dev = (dev(z["router_q"]), dev(z["router_s"]), dev(z["router_b"]))
    out, ids = _moe_check(ops, x, res, router_np, router_dev, ex, K, act)
    # Against the reference's own composition: routing identical on every
    # token, output within tolerance on every token.
    assert np.array_equal(ids, z["ids"]), f"{int((ids != z['ids']).any(axis=1).sum())} tokens routed differently"
    assert_close(out, bits_to_act(z["layer_out"], act), ulp_act=act)


@pytest.mark.parametrize("act,T,dense", [("bf16", 32, True), ("f16", 64, False), ("bf16", 1, False)])
def test_moe_block_config1_geometry(ops, act, T, dense):
    """BASELINE config 1 shapes: H=2048, E=64, K=8, I=1024."""
    rng = np.random.default_rng(20260101)
    H, I, E, K = 2048, 1024, 64, 8
    x = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    res = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    ex = experts_np(rng, E, H, I)
    wr = oracle.round_bf16(rng.standard_normal((E, H)).astype(np.float32) * 0.02)
    if dense:
        w = oracle.to_act(wr, act)
        router_np, router_dev = ("dense", w), dev(w, act)
    else:
        q, s, b = oracle.affine_quantize(wr)
        router_np, router_dev = ("affine", q, s, b), (dev(q), dev(s), dev(b))
    _moe_check(ops, x, res, router_np, router_dev, ex, K, act)


@pytest.mark.parametrize("sorted_ids", [False, True])
def test_expert_hook_gpu_callable(ops, sorted_ids):
    rng = np.random.default_rng(6)
    act, T, H, I, E, N = "f16", 12, 256, 128, 8, 30
    x = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    ex = experts_np(rng, E, H, I)
    tok = rng.integers(0, T, size=N).astype(np.int32)
    eid = rng.integers(0, E, size=N).astype(np.int32)
    if sorted_ids:
        eid = np.sort(eid)
    d = experts_dev(ex)
    out, inverse = ops.expert_gpu(dev(x, act), dev(tok), dev(eid), sorted_ids, d["gate"], d["up"], d["down"])
    order = np.argsort(eid, kind="stable")
    rows = x[tok[order]]
    sel = eid[order]
    h = oracle.swiglu(oracle.gather_qmm(rows, *ex["gate"], sel, act), oracle.gather_qmm(rows, *ex["up"], sel, act), act)
    ref = oracle.gather_qmm(h, *ex["down"], sel, act)
    inv = host(inverse)
    assert np.array_equal(order[inv], np.arange(N))
    assert_close(host(out), ref)
    empty_out, empty_inv = ops.expert_gpu(dev(x, act), dev(tok[:0]), dev(eid[:0]), False, d["gate"], d["up"], d["down"])
    assert empty_out.shape == (0, H) and empty_inv.shape == (0,)


def test_out_of_range_device_ids_are_rejected_before_launch(ops):
    """The mirror range-checks device index arrays on the host (the kernels
    index with them unchecked), like the reference ops' indexing does."""
    rng = np.random.default_rng(9)
    T, H, I, E = 4, 256, 128, 8
    d = experts_dev(experts_np(rng, E, H, I))
    x = dev(rng.standard_normal((T, H)).astype(np.float32), "f16")
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
    with pytest.raises(ValueError, match="expert index out of range"):
        ops.expert_gpu(x, i32([0, 1]), i32([0, E]), False, d["gate"], d["up"], d["down"])
    with pytest.raises(ValueError, match="token index out of range"):
        ops.expert_gpu(x, i32([0, T]), i32([0, 1]), False, d["gate"], d["up"], d["down"])
    with pytest.raises(ValueError, match="expert index out of range"):
        ops.moe_route_sort(i32([[0, -1]]), E)
    with pytest.raises(ValueError, match="expert index out of range"):
        ops.native_affine_gather_qmm(x.reshape(T, 1, H), *d["gate"], i32([0, 1, 2, E]), 64, 4)
    out, inverse = ops.expert_gpu(x, i32([0, T - 1]), i32([0, E - 1]), False, d["gate"], d["up"], d["down"])
    assert out.shape == (2, H) and sorted(host(inverse).tolist()) == [0, 1]


def test_attention_against_torch_golden(ops, golden_dir):
    z = np.load(golden_dir / "attention.npz")
    m = json.loads(str(z["meta"]))
    Hh, D, L0 = m["Hh"], m["D"], m["L0"]
    f = lambda k: z[f"t1_{k}"].view(np.float16).astype(np.float32)  # noqa: E731
    cap = 64
    kc = torch.zeros((1, Hh, cap, D), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    kc[0, :, :L0] = dev(f("kc").reshape(Hh, L0, D), "f16")
    vc[0, :, :L0] = dev(f("vc").reshape(Hh, L0, D), "f16")
    qkv = np.concatenate([f("q"), f("k"), f("v")], axis=1)
    out = ops.attention_decode(dev(qkv, "f16"), dev(f("qn"), "f16"), dev(f("kn"), "f16"),
                               dev(np.array([L0], np.int32)), kc, vc, m["eps"], m["theta"])
    assert_close(host(out), f("out"))


@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_attention_decode_batch_against_oracle(ops, act):
    rng = np.random.default_rng(8)
    B, Hh, D, cap = 3, 16, 128, 700
    W = Hh * D
    positions = np.array([0, 255, 699], np.int32)
    kc = oracle.round_f16(rng.standard_normal((B, Hh, cap, D)).astype(np.float32))
    vc = oracle.round_f16(rng.standard_normal((B, Hh, cap, D)).astype(np.float32))
    qkv = oracle.to_act(rng.standard_normal((B, 3 * W)).astype(np.float32), act)
    qn = oracle.round_f16(1 + 0.1 * rng.standard_normal(W).astype(np.float32))
    kn = oracle.round_f16(1 + 0.1 * rng.standard_normal(W).astype(np.float32))
    kt, vt = dev(kc, "f16"), dev(vc, "f16")
    out = host(ops.attention_decode(dev(qkv, act), dev(qn, "f16"), dev(kn, "f16"), dev(positions), kt, vt,
                                    1e-5, 10000.0))
    for b in range(B):
        p = int(positions[b])
        q = oracle.rms_norm(qkv[b:b + 1, :W], qn, 1e-5, act)
        k = oracle.rms_norm(qkv[b:b + 1, W:2 * W], kn, 1e-5, act)
        q = oracle.rope(q.reshape(1, Hh, D), [p], 10000.0, act)
        k = oracle.rope(k.reshape(1, Hh, D), [p], 10000.0, act)
        kc[b, :, p] = oracle.round_f16(k[0])
        vc[b, :, p] = oracle.round_f16(qkv[b, 2 * W:].reshape(Hh, D))
        ref = oracle.sdpa(q, kc[b, :, :p + 1], vc[b, :, :p + 1], np.float32(D ** -0.5), act)
        assert_close(out[b], ref.reshape(-1))
        # the appended slot holds the oracle's f16 k (rope: tolerance) and v (exact)
        assert_close(host(kt[b, :, p]), kc[b, :, p])
        assert bits_equal(host(vt[b, :, p]), vc[b, :, p])
