"""Parity at the full BASELINE shapes, through the C ABI, against the oracle
and (config 1) against the reference's own operators.

* config 1: one MoE block at its full geometry (T=32, H=2048, E=64, top-8,
  I=1024, bf16, dense bf16 router), inputs rebuilt from their seed and
  checked against the fixture the reference's operators produced;
* config 4: decode attention, B=64, 16 x 128, at KV lengths 4096 and 32768
  (the 16- and 128-split merge paths) on sampled requests;
* config 2: one decode step of the 16-layer OLMoE-1B-7B at B=64 with an
  N(0, 1) f16 cache of 4096 entries, every layer of four requests and
  their logits;
* config 3: a 2048-token prefill through the 16 layers, every layer's
  2048 rows and the last-row logits;
* config 5: 65536 bf16 tokens with the per-expert router-logit bias
  N(0, 1.5), routing of sampled tokens bit-exact and their outputs within
  tolerance.

Costs on the host are bounded by sampling requests / tokens where the
computation is independent per request or per token, and by the oracle's
float32-BLAS attention for the long prefill (checked against its float64
form in tests/test_oracle_consistency.py)."""
import sys

import numpy as np
import pytest
import torch

import oracle
from tests.gpu_util import bits_equal, dev, experts_dev, host
from tests.parity import assert_close, assert_logits_close

pytestmark = pytest.mark.gpu


# ---------------------------------------------------------------- config 1

def test_config1_full_geometry_against_reference(golden_dir):
    from trifuse_b200 import ops
    sys.path.insert(0, str(golden_dir))
    import config1_inputs as c1
    z = np.load(golden_dir / "config1_full.npz")
    x, res, ex, wr = c1.generate()
    assert c1.digest(x, res, ex, wr) == str(z["digest"]), "regenerated inputs differ from the reference's"
    act, K = c1.ACT, c1.K
    d = experts_dev(ex)
    out, aux = ops.moe(dev(x, act), dev(res, act), dev(wr, act), d["gate"], d["up"], d["down"], K,
                       return_aux=True)
    torch.cuda.synchronize()
    # Logits: the fixed order of the oracle bit for bit; within one ulp of the reference's linear.
    logits = host(aux["logits"])
    assert bits_equal(logits, oracle.router_logits_dense(x, wr, act))
    ref_logits = oracle.bits_to_act(z["logits"], act)
    assert_close(logits, ref_logits, act)
    flips = int((oracle.act_to_bits(logits, act) != z["logits"]).sum())
    assert flips <= 2, f"{flips} router logits differ from the reference's linear"
    # Routing and gates identical to the reference's on every token.
    assert np.array_equal(host(aux["indices"]), z["ids"])
    assert np.array_equal(oracle.act_to_bits(host(aux["gates"]), act), z["scores"])
    assert_close(host(out), oracle.bits_to_act(z["layer_out"], act), ulp_act=act)
    # Routing the reference's own logits on the device reproduces its ids and gates.
    ids, gates = ops.olmoe_route(dev(ref_logits, act).reshape(1, c1.T, -1), K)
    assert np.array_equal(host(ids).reshape(c1.T, K), z["ids"])
    assert np.array_equal(oracle.act_to_bits(host(gates).reshape(c1.T, K), act), z["scores"])
    # The expert hook given the reference's routes, combined with its gates.
    flat = torch.from_numpy(z["ids"].reshape(-1).astype(np.int32)).cuda()
    tok = torch.arange(c1.T, dtype=torch.int32, device="cuda").repeat_interleave(K)
    y_sorted, inverse = ops.expert_gpu(dev(x, act), tok, flat, False, d["gate"], d["up"], d["down"])
    gref = dev(oracle.bits_to_act(z["scores"], act), act)
    combined = ops.moe_combine(y_sorted, inverse, gref, dev(res, act))
    assert_close(host(combined), oracle.bits_to_act(z["layer_out"], act), ulp_act=act)
    assert ops.device_error() == 0


# ---------------------------------------------------------------- config 4

@pytest.mark.parametrize("L", [4096, 32768])
def test_config4_attention_full_lengths(L):
    """B=64 rows at position L (L keys in the cache + this step's), all 16
    heads, against the oracle on four sampled requests."""
    from trifuse_b200 import ops
    B, Hh, D = 64, 16, 128
    W = Hh * D
    cap = L + 64
    g = torch.Generator(device="cuda")
    g.manual_seed(20260104 + L)
    kc = torch.empty((B, Hh, cap, D), dtype=torch.float16, device="cuda")
    vc = torch.empty_like(kc)
    for b0 in range(0, B, 8):
        kc[b0:b0 + 8].normal_(generator=g)
        vc[b0:b0 + 8].normal_(generator=g)
    rng = np.random.default_rng(L)
    act = "f16"
    qkv = oracle.to_act(rng.standard_normal((B, 3 * W)).astype(np.float32), act)
    qn = oracle.round_f16(1 + 0.1 * rng.standard_normal(W).astype(np.float32))
    kn = oracle.round_f16(1 + 0.1 * rng.standard_normal(W).astype(np.float32))
    pos = np.full(B, L, np.int32)
    pos[1] = L // 2 + 3  # a shorter row in the same launch
    sample = [0, 1, 37, 63]
    before = {b: (host(kc[b, :, :L + 1]), host(vc[b, :, :L + 1])) for b in sample}
    out = host(ops.attention_decode(dev(qkv, act), dev(qn, "f16"), dev(kn, "f16"), dev(pos), kc, vc, 1e-5,
                                    10000.0))
    torch.cuda.synchronize()
    for b in sample:
        p = int(pos[b])
        K_, V_ = before[b]
        q = oracle.rms_norm(qkv[b:b + 1, :W], qn, 1e-5, act)
        k = oracle.rms_norm(qkv[b:b + 1, W:2 * W], kn, 1e-5, act)
        q = oracle.rope(q.reshape(1, Hh, D), [p], 10000.0, act)
        k = oracle.rope(k.reshape(1, Hh, D), [p], 10000.0, act)
        K_[:, p] = oracle.round_f16(k[0])
        V_[:, p] = oracle.round_f16(qkv[b, 2 * W:].reshape(Hh, D))
        ref = oracle.sdpa(q, K_[:, :p + 1], V_[:, :p + 1], np.float32(D ** -0.5), act)
        assert_close(out[b], ref.reshape(-1))
        assert bits_equal(host(vc[b, :, p]), V_[:, p])
    assert ops.device_error() == 0


# ---------------------------------------------------------------- configs 2 and 3

def _oracle_weights(w, cfg):
    n = lambda k: host(w[k])  # noqa: E731
    aff = lambda p: (n(p + ".weight"), n(p + ".scales").astype(np.float16), n(p + ".biases").astype(np.float16))  # noqa: E731
    layers = []
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        layers.append(dict(
            input_norm=n(p + "input_layernorm.weight"), post_norm=n(p + "post_attention_layernorm.weight"),
            q_norm=n(p + "self_attn.q_norm.weight"), k_norm=n(p + "self_attn.k_norm.weight"),
            q=aff(p + "self_attn.q_proj"), k=aff(p + "self_attn.k_proj"), v=aff(p + "self_attn.v_proj"),
            o=aff(p + "self_attn.o_proj"), router=aff(p + "mlp.gate"),
            experts={e: aff(p + f"mlp.switch_mlp.{e}_proj") for e in ("gate", "up", "down")}))
    return dict(embed=aff("model.embed_tokens"), lm_head=aff("lm_head"), final_norm=n("model.norm.weight"),
                layers=layers)


@pytest.fixture(scope="module")
def olmoe_1b7b():
    """The full random-init OLMoE-1B-7B (16 layers, f16 activations) on the
    device, and its weights on the host for the oracle."""
    from trifuse_b200.model import Config, Model
    from trifuse_b200.quant import synthetic_olmoe
    cfg = Config(capacity=4096 + 64)
    w = synthetic_olmoe(cfg, seed=20260102, device="cuda")
    model = Model(cfg, w)
    ow = _oracle_weights(w, cfg)
    del w
    torch.cuda.empty_cache()
    ocfg = oracle.OLMoEConfig(capacity=cfg.capacity, act="f16")
    yield cfg, model, ow, ocfg
    model.close()


def _routing_report(own, forced):
    """(differing, total) token-layer routing decisions (sets of top-k
    experts): how often the oracle's own router, on its input (the device's
    state), chose differently from the device."""
    diff = total = 0
    for o, f in zip(own, forced):
        o = np.sort(np.asarray(o).reshape(-1, np.asarray(o).shape[-1]), -1)
        f = np.sort(np.asarray(f).reshape(o.shape), -1)
        diff += int((o != f).any(-1).sum())
        total += o.shape[0]
    return diff, total


def test_config2_decode_full_model(olmoe_1b7b):
    """One decode step at B=64 with every request's cache filled N(0, 1) to
    4096 entries, checked layer by layer on four requests.  The device
    records each layer's routing and output hidden states
    (tf_session_capture); the oracle recomputes every layer from the
    device's input to it (so rounding differences cannot compound over the
    16 layers) following the device's routing, and each layer's output must
    meet the layer tolerance.  How often the oracle's own router chose
    differently is counted and must be rare (a top-k decision within
    rounding noise of a tie)."""
    from trifuse_b200 import ops
    from trifuse_b200.model import Session
    cfg, model, ow, ocfg = olmoe_1b7b
    B, L, H = 64, 4096, cfg.hidden
    sess = Session(model, max_batch=B, capacity=cfg.capacity)
    try:
        g = torch.Generator(device="cuda")
        g.manual_seed(20260103)
        for layer in range(cfg.layers):
            for t in sess.kv_tensors(layer):
                for b0 in range(0, B, 16):
                    t[b0:b0 + 16, :, :L].normal_(generator=g)
        sample = [0, 17, 42, 63]
        caches = []
        for layer in range(cfg.layers):
            k, v = sess.kv_tensors(layer)
            caches.append((host(k[sample, :, :L + 1]), host(v[sample, :, :L + 1])))
        rng = np.random.default_rng(2)
        ids = rng.integers(0, cfg.vocab, size=B)
        sess.set_lengths([L] * B)
        routes = torch.full((cfg.layers, B, cfg.top_k), -1, dtype=torch.int32, device="cuda")
        hidden = torch.zeros((cfg.layers, B, H), dtype=torch.float16, device="cuda")
        sess.capture(routes, hidden)
        logits = host(sess.decode(torch.from_numpy(ids).cuda()))
        sess.capture(None)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        assert sess.lengths(B) == [L + 1] * B
    finally:
        sess.close()
    routes, hidden = host(routes), host(hidden)
    assert (routes >= 0).all()
    h = oracle.affine_embedding(ids[sample], *ow["embed"], "f16")
    pos = [L] * len(sample)
    aux = []
    for layer in range(cfg.layers):
        kcs = [caches[layer][0][i] for i in range(len(sample))]
        vcs = [caches[layer][1][i] for i in range(len(sample))]
        out = oracle.decode_layer_batched(h, ow["layers"][layer], ocfg, kcs, vcs, pos, fast=True,
                                          forced=routes[layer][sample], aux_out=aux)
        assert_close(out, hidden[layer][sample], ulp_act="f16")
        h = hidden[layer][sample]
    diff, total = _routing_report([a["own_indices"] for a in aux], [routes[l][sample] for l in range(cfg.layers)])
    assert diff <= max(1, total // 20), f"{diff} of {total} routing decisions differ"
    last = oracle.rms_norm(hidden[-1][sample], ow["final_norm"], ocfg.rms_eps, "f16")
    ref = oracle.affine_qmm(last, *ow["lm_head"], "f16")
    assert_logits_close(logits[sample], ref, "f16")


def test_config3_prefill_full_sequence(olmoe_1b7b):
    """One 2048-token sequence (uniform token ids) through the 16 layers,
    checked layer by layer as in the config-2 test: every layer recomputed
    from the device's input to it, following the device's routing, within
    the layer tolerance on all 2048 rows (the last layer on the last row,
    the only one whose MoE block runs, as in the reference); then the
    last-row logits."""
    from trifuse_b200 import ops
    from trifuse_b200.model import Session
    cfg, model, ow, ocfg = olmoe_1b7b
    T, H = 2048, cfg.hidden
    rng = np.random.default_rng(3)
    ids = rng.integers(0, cfg.vocab, size=T)
    sess = Session(model, max_batch=1, capacity=cfg.capacity, max_prefill_tokens=T)
    routes = torch.full((cfg.layers, T, cfg.top_k), -1, dtype=torch.int32, device="cuda")
    hidden = torch.zeros((cfg.layers, T, H), dtype=torch.float16, device="cuda")
    try:
        sess.capture(routes, hidden)
        logits = host(sess.prefill([0], [torch.from_numpy(ids)]))
        sess.capture(None)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
    finally:
        sess.close()
    routes, hidden = host(routes), host(hidden)
    n = cfg.layers
    forced = [routes[l] for l in range(n - 1)] + [routes[-1][:1]]
    assert all((f >= 0).all() for f in forced)
    positions = np.arange(T)
    h = oracle.affine_embedding(ids, *ow["embed"], "f16")
    aux = []
    for l in range(n):
        kc = np.zeros((ocfg.heads, T, ocfg.head_dim), np.float32)
        vc = np.zeros_like(kc)
        out = oracle.layer_forward(h, ow["layers"][l], ocfg, kc, vc, positions, fast=True, forced=forced[l],
                                   aux_out=aux, last_row_only=l == n - 1)
        gpu = hidden[l] if l < n - 1 else hidden[l][:1]
        assert_close(out, gpu, ulp_act="f16")
        h = hidden[l]
    diff, total = _routing_report([a["own_indices"] for a in aux], forced)
    assert diff <= max(1, total // 20), f"{diff} of {total} routing decisions differ"
    last = oracle.rms_norm(hidden[-1][:1], ow["final_norm"], ocfg.rms_eps, "f16")
    ref = oracle.affine_qmm(last, *ow["lm_head"], "f16")
    assert_logits_close(logits.reshape(1, -1), ref, "f16")


# ---------------------------------------------------------------- config 5

def skewed_router(rng, E, H):
    """Dense bf16 router whose logits carry a per-expert bias N(0, 1.5)
    through the last input column (inputs set x[:, -1] = 1): w[:, -1] = bias,
    the other weights N(0, 0.02).  The reference's router has no bias term,
    so the bias rides on an input column."""
    w = rng.standard_normal((E, H)).astype(np.float32) * np.float32(0.02)
    w[:, -1] = rng.standard_normal(E).astype(np.float32) * np.float32(1.5)
    return oracle.to_act(w, "bf16")


def test_config5_skewed_routing_65536_tokens():
    """The MoE layer on 65536 bf16 tokens with skewed routing on one GPU:
    routing of 4096 sampled tokens bit-exact against the oracle, outputs of
    256 sampled tokens within tolerance (each token's result depends only on
    its own row)."""
    from tests.gpu_util import experts_np
    from trifuse_b200 import ops
    E, K, H, I, T = 64, 8, 2048, 1024, 65536
    rng = np.random.default_rng(20260105)
    ex = experts_np(rng, E, H, I)
    w = skewed_router(rng, E, H)
    d = experts_dev(ex)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    x[:, -1] = 1.0
    res = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    out, aux = ops.moe(x, res, dev(w, "bf16"), d["gate"], d["up"], d["down"], K, return_aux=True)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    idx = host(aux["indices"])
    load = np.bincount(idx.reshape(-1), minlength=E)
    assert load.max() > 3 * load.mean(), "routing is not skewed"
    pick = np.sort(np.random.default_rng(9).choice(T, 4096, replace=False))
    xs = host(x[torch.from_numpy(pick).cuda()])
    ref_logits = oracle.router_logits_dense(xs, w, "bf16")
    assert bits_equal(host(aux["logits"])[pick], ref_logits)
    ref_idx, ref_gates = oracle.olmoe_route(ref_logits, K, "bf16")
    assert np.array_equal(idx[pick], ref_idx)
    assert bits_equal(host(aux["gates"])[pick], ref_gates)
    few = pick[::16]
    ref_out, _ = oracle.moe_block(host(x[torch.from_numpy(few).cuda()]), host(res[torch.from_numpy(few).cuda()]),
                                  ("dense", w), ex, K, "bf16")
    assert_close(host(out)[few], ref_out, ulp_act="bf16")
