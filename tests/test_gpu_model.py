"""End-to-end parity of the device-resident model and session (C ABI
tf_model_* / tf_session_*) against the oracle's model_forward, on a small
random-init OLMoE, plus the session's admission / cancellation rules."""
import numpy as np
import pytest
import torch

import oracle
from tests.gpu_util import host
from tests.parity import assert_close, assert_logits_close

pytestmark = pytest.mark.gpu


def tiny_cfg(act=torch.float16):
    from trifuse_b200.model import Config
    return Config(layers=2, hidden=256, heads=2, kv_heads=2, head_dim=128, intermediate=128, vocab=512,
                  experts=8, top_k=2, capacity=64, act=act)


def oracle_weights(w, cfg):
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
def tiny():
    from trifuse_b200.model import Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    cfg = tiny_cfg()
    w = synthetic_olmoe(cfg, seed=7, device="cuda")
    model = Model(cfg, w)
    sess = Session(model, max_batch=2, capacity=64, max_prefill_tokens=32)
    ocfg = oracle.OLMoEConfig(layers=cfg.layers, hidden=cfg.hidden, heads=cfg.heads, head_dim=cfg.head_dim,
                              intermediate=cfg.intermediate, vocab=cfg.vocab, experts=cfg.experts,
                              top_k=cfg.top_k, capacity=64, act="f16")
    yield cfg, model, sess, oracle_weights(w, cfg), ocfg
    sess.close()
    model.close()


def test_prefill_then_decode_matches_oracle(tiny):
    cfg, model, sess, ow, ocfg = tiny
    sess.reset()
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, size=5), rng.integers(0, cfg.vocab, size=9)]
    caches = [([np.zeros((cfg.heads, 64, cfg.head_dim), np.float32) for _ in range(cfg.layers)],
               [np.zeros((cfg.heads, 64, cfg.head_dim), np.float32) for _ in range(cfg.layers)])
              for _ in range(2)]
    logits = host(sess.prefill([0, 1], prompts))
    for r in range(2):
        ref = oracle.model_forward(prompts[r], ow, ocfg, caches[r][0], caches[r][1], 0)
        assert_logits_close(logits[r], ref, "f16")
    assert sess.lengths(2) == [5, 9]
    # three decode steps, both requests at once, device-side token ids
    for step in range(3):
        toks = rng.integers(0, cfg.vocab, size=2)
        lg = host(sess.decode(torch.tensor(toks, dtype=torch.int64, device="cuda")))
        for r in range(2):
            start = len(prompts[r]) + step
            ref = oracle.model_forward(toks[r:r + 1], ow, ocfg, caches[r][0], caches[r][1], start)
            assert_logits_close(lg[r], ref, "f16")
    assert sess.lengths(2) == [8, 12]
    # host inputs / host output through the same call
    lg = sess.decode(torch.tensor([1, 2], dtype=torch.int64))
    assert lg.device.type == "cpu" and lg.shape == (2, cfg.vocab)


def test_decode_after_large_prefill_matches_oracle():
    """A 16-request prefill (1024 rows: the MoE workspace laid out for 2048
    routes), then decode steps of all 16 requests (32 routes: tensor-core
    expert tiles on the split schedule with the route sort fused into the
    router).  The arrival counters those use must not sit on the prefill's
    data: every decode row matches the oracle."""
    import dataclasses

    from trifuse_b200.model import Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    cfg = dataclasses.replace(tiny_cfg(), capacity=128)
    w = synthetic_olmoe(cfg, seed=29, device="cuda")
    ow = oracle_weights(w, cfg)
    ocfg = oracle.OLMoEConfig(layers=cfg.layers, hidden=cfg.hidden, heads=cfg.heads, head_dim=cfg.head_dim,
                              intermediate=cfg.intermediate, vocab=cfg.vocab, experts=cfg.experts,
                              top_k=cfg.top_k, capacity=128, act="f16")
    model = Model(cfg, w)
    B, T = 16, 64
    sess = Session(model, max_batch=B, capacity=128, max_prefill_tokens=B * T)
    rng = np.random.default_rng(31)
    prompts = [rng.integers(0, cfg.vocab, size=T) for _ in range(B)]
    caches = [([np.zeros((cfg.heads, 128, cfg.head_dim), np.float32) for _ in range(cfg.layers)],
               [np.zeros((cfg.heads, 128, cfg.head_dim), np.float32) for _ in range(cfg.layers)])
              for _ in range(B)]
    try:
        lg = host(sess.prefill(list(range(B)), prompts))
        for r in range(B):
            ref = oracle.model_forward(prompts[r], ow, ocfg, caches[r][0], caches[r][1], 0)
            assert_logits_close(lg[r], ref, "f16")
        for step in range(2):
            toks = rng.integers(0, cfg.vocab, size=B)
            lg = host(sess.decode(torch.tensor(toks, dtype=torch.int64, device="cuda")))
            for r in range(B):
                ref = oracle.model_forward(toks[r:r + 1], ow, ocfg, caches[r][0], caches[r][1], T + step)
                assert_logits_close(lg[r], ref, "f16")
    finally:
        sess.close()
        model.close()


def test_session_admission_rules(tiny):
    from trifuse_b200 import TriFuseError
    cfg, model, sess, ow, ocfg = tiny
    sess.reset()
    sess.set_lengths([3, 3])
    ids = torch.tensor([1, 2], dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError, match="invalid absolute position"):
        sess.decode(ids, positions=[3, 4])
    assert sess.lengths(2) == [3, 3]
    sess.set_lengths([64, 3])
    with pytest.raises(TriFuseError, match="CAPACITY"):
        sess.decode(ids)
    sess.set_lengths([3, 3])
    sess.cancel()
    with pytest.raises(TriFuseError, match="CANCELLED"):
        sess.decode(ids)
    assert sess.lengths(2) == [3, 3]
    sess.reset()
    assert sess.lengths(2) == [0, 0]
    with pytest.raises(ValueError, match="outside the vocabulary"):
        sess.prefill([0, 1], [[1, 2], [3, cfg.vocab]])
    assert sess.lengths(2) == [0, 0]
    out = sess.decode(ids)
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("act", ["f16", "bf16"])
def test_full_geometry_layer_tensor_core_path(act):
    """One layer at OLMoE-1B-7B geometry (H=2048, 16 heads, E=64, K=8,
    I=1024; vocab cut to 4096): prefill rows and a 40-request decode batch
    run the tensor-core QMMs; logits match the oracle."""
    from trifuse_b200.model import Config, Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    tdt = torch.float16 if act == "f16" else torch.bfloat16
    cfg = Config(layers=1, vocab=4096, capacity=64, act=tdt)
    w = synthetic_olmoe(cfg, seed=11, device="cuda")
    model = Model(cfg, w)
    sess = Session(model, max_batch=40, capacity=64, max_prefill_tokens=64)
    ow = oracle_weights(w, cfg)
    ocfg = oracle.OLMoEConfig(layers=1, vocab=4096, capacity=64, act=act)
    rng = np.random.default_rng(3)
    B = 40
    prompts = [rng.integers(0, cfg.vocab, size=n) for n in (20, 12)]
    caches = [([np.zeros((16, 64, 128), np.float32)], [np.zeros((16, 64, 128), np.float32)]) for _ in range(B)]
    lg = host(sess.prefill([0, 1], prompts))
    for r in range(2):
        ref = oracle.model_forward(prompts[r], ow, ocfg, caches[r][0], caches[r][1], 0)
        assert_logits_close(lg[r], ref, act)
    lengths = [20, 12] + [0] * (B - 2)
    toks = rng.integers(0, cfg.vocab, size=B)
    lg = host(sess.decode(torch.tensor(toks, dtype=torch.int64, device="cuda")))
    h = oracle.affine_embedding(toks, *ow["embed"], act)
    out = oracle.decode_layer_batched(h, ow["layers"][0], ocfg, [c[0][0] for c in caches],
                                      [c[1][0] for c in caches], lengths)
    ref = oracle.affine_qmm(oracle.rms_norm(out, ow["final_norm"], ocfg.rms_eps, act), *ow["lm_head"], act)
    assert_logits_close(lg, ref, act)
    from trifuse_b200 import ops
    assert ops.device_error() == 0
    sess.close()
    model.close()


def test_greedy_tokens_kernel_matches_oracle():
    from trifuse_b200 import ops
    rng = np.random.default_rng(31)
    lg = rng.standard_normal((9, 50304)).astype(np.float32)
    lg[1, [100, 40000]] = 9.0            # tie -> lower index
    lg[2, 7] = np.nan
    lg[3, 50303] = np.inf
    lg[4, 0] = -np.inf
    lg[5, :] = 1.0                       # all equal -> index 0
    lg[6, 50303] = 50.0                  # maximum in the last slot
    got = ops.greedy_tokens(torch.from_numpy(lg).cuda())
    assert host(got).tolist() == oracle.greedy_token(lg).tolist()
    assert ops.device_error() == 0


def test_decode_greedy_and_one_ahead_pipeline(tiny):
    """decode_greedy == argmax of decode's logits, and the pipelined
    generation (next step submitted with the device tokens before the host
    reads them) yields the same tokens as a host loop."""
    cfg, model, sess, ow, ocfg = tiny
    prompts = [[3, 7, 11], [5, 1]]

    def host_loop(n):
        sess.reset()
        sess.prefill([0, 1], prompts)
        ids = torch.tensor([9, 4], dtype=torch.int64)
        out = []
        for _ in range(n):
            lg = sess.decode(ids)
            ids = torch.as_tensor(oracle.greedy_token(lg.numpy()), dtype=torch.int64)
            out.append(ids.tolist())
        return out

    want = host_loop(6)
    sess.reset()
    sess.prefill([0, 1], prompts)
    tok = sess.decode_greedy(torch.tensor([9, 4], dtype=torch.int64), tokens=torch.empty(2, dtype=torch.int64))
    assert tok.tolist() == want[0]
    sess.reset()
    sess.prefill([0, 1], prompts)
    got = sess.generate_greedy([9, 4], 6)
    assert got == want
    assert sess.lengths(2) == [3 + 6, 2 + 6]
    assert model_device_error_clear() == 0


def model_device_error_clear():
    from trifuse_b200 import ops
    return ops.device_error()


def test_embedding_reads_row_zero_for_out_of_range_device_ids(tiny):
    """Device ids are not checked on the host: a negative id (the greedy -1
    fed back) reads row 0 like the reference's maximum(token, 0); an id past
    the table reads row 0 and records device error 6."""
    from trifuse_b200 import ops
    from trifuse_b200.quant import random_affine
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    q, s, b = random_affine((64, 256), g, "cuda")
    row0 = ops.native_affine_embedding(torch.tensor([0], device="cuda"), q, s, b, 64, 4)
    import ctypes as C
    from trifuse_b200._lib import check, lib
    from trifuse_b200.ops import affine_desc
    w = affine_desc(q, s, b, 64, 4)
    ids = torch.tensor([-1, 64], dtype=torch.int64, device="cuda")
    y = torch.empty((2, 256), dtype=torch.float16, device="cuda")
    assert ops.device_error(clear=True) == 0
    check(lib().tf_affine_embedding(C.c_void_p(ids.data_ptr()), 2, C.byref(w), 1, C.c_void_p(y.data_ptr()),
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    assert torch.equal(y[0], row0[0]) and torch.equal(y[1], row0[0])
    assert ops.device_error(clear=True) == 6
    assert ops.device_error() == 0


def test_model_from_checkpoint_matches_model_from_tensors(tmp_path):
    """A checkpoint directory written in the reference's layout (experts one
    per tensor, two safetensors files) loads into a model whose logits equal,
    bit for bit, those of the same weights bound directly."""
    import json

    from trifuse_b200 import checkpoint as ck
    from trifuse_b200.model import Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    cfg = tiny_cfg()
    w = synthetic_olmoe(cfg, seed=11, device="cuda")
    src = {k: v.cpu().numpy() if v.dtype != torch.uint32 else v.cpu().view(torch.int32).numpy().view(np.uint32)
           for k, v in w.items()}
    per = {}
    for name, a in src.items():
        if ".mlp.switch_mlp." in name:
            layer, rest = name.split(".mlp.switch_mlp.")
            for e in range(a.shape[0]):
                per[f"{layer}.mlp.experts.{e}.{rest}"] = a[e]
        else:
            per[name] = a
    names = sorted(per)
    ck.write_safetensors(tmp_path / "a.safetensors", {n: per[n] for n in names[::2]})
    ck.write_safetensors(tmp_path / "b.safetensors", {n: per[n] for n in names[1::2]})
    (tmp_path / "config.json").write_text(json.dumps(dict(
        model_type="olmoe", num_hidden_layers=cfg.layers, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
        num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim,
        vocab_size=cfg.vocab, num_experts=cfg.experts, num_experts_per_tok=cfg.top_k, rms_norm_eps=cfg.rms_eps,
        rope_theta=cfg.rope_theta, norm_topk_prob=False, quantization={"bits": 4, "group_size": 64})))
    m1 = Model(cfg, w)
    m2 = ck.load_model(tmp_path, capacity=cfg.capacity)
    out = []
    for m in (m1, m2):
        s = Session(m, max_batch=2, capacity=64, max_prefill_tokens=32)
        s.prefill([0, 1], [[1, 2, 3], [4, 5]])
        out.append(host(s.decode(torch.tensor([7, 8], dtype=torch.int64))))
        s.close()
    m1.close()
    m2.close()
    assert np.array_equal(out[0], out[1])


def test_chunked_prefill_matches_one_shot_and_oracle(tiny):
    """A 29-token prompt in chunks of 8 (3 cache-only chunks + a final one)
    gives the last-row logits of the one-shot prefill and of the oracle, and
    leaves the same KV length; decode continues identically afterwards."""
    cfg, model, sess, ow, ocfg = tiny
    rng = np.random.default_rng(41)
    prompt = rng.integers(0, cfg.vocab, size=29)
    sess.reset()
    one = host(sess.prefill([0], [prompt]))[0]
    after_one = host(sess.decode(torch.tensor([5], dtype=torch.int64)))[0]
    sess.reset()
    chunked = sess.prefill_chunked(0, prompt, chunk=8).numpy()
    assert sess.lengths(1) == [29]
    after_chunked = host(sess.decode(torch.tensor([5], dtype=torch.int64)))[0]
    kc = [np.zeros((cfg.heads, 64, cfg.head_dim), np.float32) for _ in range(cfg.layers)]
    vc = [np.zeros((cfg.heads, 64, cfg.head_dim), np.float32) for _ in range(cfg.layers)]
    ref = oracle.model_forward(prompt, ow, ocfg, kc, vc, 0)
    assert_logits_close(chunked, ref, "f16")
    assert_logits_close(chunked, one, "f16")
    assert_logits_close(after_chunked, after_one, "f16")


def test_chunked_prefill_validates_before_running(tiny):
    from trifuse_b200._lib import TriFuseError
    cfg, model, sess, ow, ocfg = tiny
    sess.reset()
    with pytest.raises((ValueError, TriFuseError)):
        sess.prefill_chunked(0, [1, 2, cfg.vocab], chunk=2)    # last token outside the vocabulary
    assert sess.lengths(1) == [0]                              # nothing ran
    with pytest.raises((ValueError, TriFuseError)):
        sess.prefill_chunked(0, [1, 2, 3], chunk=0)


def test_long_prefill_tiled_attention_matches_oracle():
    """Prompts of 150 and 77 tokens in one prefill call: several 64-row query
    blocks and 64-key tiles per request, partial last blocks, causal masks
    inside tiles; last-row logits against the oracle, then one decode step."""
    import dataclasses

    from trifuse_b200.model import Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    cfg = dataclasses.replace(tiny_cfg(), capacity=256)
    w = synthetic_olmoe(cfg, seed=17, device="cuda")
    ow = oracle_weights(w, cfg)
    ocfg = oracle.OLMoEConfig(layers=cfg.layers, hidden=cfg.hidden, heads=cfg.heads, head_dim=cfg.head_dim,
                              intermediate=cfg.intermediate, vocab=cfg.vocab, experts=cfg.experts,
                              top_k=cfg.top_k, capacity=256, act="f16")
    model = Model(cfg, w)
    sess = Session(model, max_batch=2, capacity=256, max_prefill_tokens=256)
    rng = np.random.default_rng(53)
    prompts = [rng.integers(0, cfg.vocab, size=150), rng.integers(0, cfg.vocab, size=77)]
    try:
        lg = host(sess.prefill([0, 1], prompts))
        caches = [([np.zeros((cfg.heads, 256, cfg.head_dim), np.float32) for _ in range(cfg.layers)],
                   [np.zeros((cfg.heads, 256, cfg.head_dim), np.float32) for _ in range(cfg.layers)])
                  for _ in range(2)]
        for r in range(2):
            ref = oracle.model_forward(prompts[r], ow, ocfg, caches[r][0], caches[r][1], 0)
            assert_logits_close(lg[r], ref, "f16")
        toks = np.array([3, 4])
        lg2 = host(sess.decode(torch.tensor(toks, dtype=torch.int64, device="cuda")))
        for r in range(2):
            ref = oracle.model_forward(toks[r:r + 1], ow, ocfg, caches[r][0], caches[r][1], len(prompts[r]))
            assert_logits_close(lg2[r], ref, "f16")
    finally:
        sess.close()
        model.close()


def test_prefill_attention_blocks_layer_by_layer():
    """Two requests in one prefill call: request 0 continues at position 100
    (its 128-row query blocks straddle the 128-key tiles) with 300 rows,
    request 1 starts fresh with 77 rows (one partial block).  Every layer's
    output rows are recomputed by the oracle from the device's own input to
    that layer and its routing (teacher forcing), with the caches rebuilt the
    same way from the first call, and must agree within the layer tolerance;
    this isolates the prefill attention from routing flips."""
    import dataclasses

    from trifuse_b200.model import Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    cap = 512
    cfg = dataclasses.replace(tiny_cfg(), capacity=cap)
    w = synthetic_olmoe(cfg, seed=23, device="cuda")
    ow = oracle_weights(w, cfg)
    ocfg = oracle.OLMoEConfig(layers=cfg.layers, hidden=cfg.hidden, heads=cfg.heads, head_dim=cfg.head_dim,
                              intermediate=cfg.intermediate, vocab=cfg.vocab, experts=cfg.experts,
                              top_k=cfg.top_k, capacity=cap, act="f16")
    model = Model(cfg, w)
    sess = Session(model, max_batch=2, capacity=cap, max_prefill_tokens=cap)
    rng = np.random.default_rng(71)
    first = rng.integers(0, cfg.vocab, size=100)
    prompts = [rng.integers(0, cfg.vocab, size=300), rng.integers(0, cfg.vocab, size=77)]
    L, H, K = cfg.layers, cfg.hidden, cfg.top_k

    def captured(ids_list, reqs):
        rows = sum(len(x) for x in ids_list)
        routes = torch.full((L, rows, K), -1, dtype=torch.int32, device="cuda")
        hidden = torch.zeros((L, rows, H), dtype=torch.float16, device="cuda")
        sess.capture(routes, hidden)
        sess.prefill(reqs, [torch.from_numpy(x) for x in ids_list])
        sess.capture(None)
        torch.cuda.synchronize()
        return host(routes), host(hidden)

    try:
        r1, h1 = captured([first], [0])
        r2, h2 = captured(prompts, [0, 1])
    finally:
        sess.close()
        model.close()
    caches = [([np.zeros((cfg.heads, cap, cfg.head_dim), np.float32) for _ in range(L)],
               [np.zeros((cfg.heads, cap, cfg.head_dim), np.float32) for _ in range(L)]) for _ in range(2)]

    def run(ids, routes, hidden, req, start, row0):
        """Teacher-forced layers of one request's rows [row0, row0 + n) of a
        captured call; checks them when `hidden` rows are compared."""
        n = len(ids)
        pos = np.arange(start, start + n)
        h = oracle.affine_embedding(ids, *ow["embed"], "f16")
        for l in range(L):
            last = l == L - 1
            forced = routes[l][row0:row0 + n] if not last else None
            out = oracle.layer_forward(h, ow["layers"][l], ocfg, caches[req][0][l], caches[req][1][l], pos,
                                       forced=forced, last_row_only=last)
            if not last:
                assert_close(out, hidden[l][row0:row0 + n], ulp_act="f16")
                h = hidden[l][row0:row0 + n]

    run(first, r1, h1, 0, 0, 0)
    run(prompts[0], r2, h2, 0, 100, 0)
    run(prompts[1], r2, h2, 1, 0, 300)


def test_decode_graph_replay_matches_eager():
    """Decode steps replayed from CUDA graphs give the logits of eager steps
    bit for bit, across a KV length of 256 (a new attention split, so a new
    graph is captured), and the launch counter still counts their kernels."""
    import dataclasses

    from trifuse_b200._lib import lib
    from trifuse_b200.model import Model, Session
    from trifuse_b200.quant import synthetic_olmoe
    cfg = dataclasses.replace(tiny_cfg(), capacity=320)
    model = Model(cfg, synthetic_olmoe(cfg, seed=23, device="cuda"))
    rng = np.random.default_rng(61)
    prompts = [rng.integers(0, cfg.vocab, size=250), rng.integers(0, cfg.vocab, size=240)]
    steps = rng.integers(0, cfg.vocab, size=(12, 2))
    out, counts = [], []
    try:
        for graphs in (False, True):
            sess = Session(model, max_batch=2, capacity=320, max_prefill_tokens=512)
            try:
                sess.graphs(graphs)
                sess.prefill([0, 1], prompts)
                lg, n = [], []
                for t in range(12):
                    c0 = lib().tf_launch_count()
                    lg.append(host(sess.decode(torch.tensor(steps[t], dtype=torch.int64, device="cuda"))))
                    n.append(lib().tf_launch_count() - c0)
                out.append(np.stack(lg))
                counts.append(n)
            finally:
                sess.close()
    finally:
        model.close()
    assert counts[0] == counts[1] and min(counts[0]) > 10 * cfg.layers  # replays count their kernels
    assert np.array_equal(out[0], out[1])
