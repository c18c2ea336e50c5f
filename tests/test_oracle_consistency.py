"""Internal consistency of the oracle's composed paths (CPU, small geometry).

The GPU parity tests use three oracle compositions as their checker: the
batched decode layer (many requests, each at its own position), the
per-request model forward (prefill / decode of one request) and the float32
attention variant that the CPU baseline times.  These tests require them to
agree with each other, so a mismatch on the GPU points at the kernels and
not at a disagreement inside the checker:

* decode_layer_batched == layer_forward applied to each request with T = 1
  (MLXNativeGraniteMoEPrefill.h:433-487 for one token);
* prefill of T tokens, then one decode step == one prefill of T + 1 tokens
  (the causal mask and the KV cache make them the same computation);
* sdpa(fast=True) (float32 BLAS) == sdpa() (float64).
"""
import numpy as np

import oracle
from tests.parity import assert_close


def tiny_cfg():
    return oracle.OLMoEConfig(layers=2, hidden=256, heads=2, head_dim=128, intermediate=128, vocab=512,
                              experts=8, top_k=2, capacity=64, act="f16")


def affine(rng, shape):
    return oracle.affine_quantize(oracle.round_bf16(rng.standard_normal(shape).astype(np.float32) * 0.02))


def norm(rng, n):
    return (1 + 0.1 * rng.standard_normal(n)).astype(np.float16)


def layer_weights(rng, cfg):
    H, W, E, I = cfg.hidden, cfg.heads * cfg.head_dim, cfg.experts, cfg.intermediate
    return dict(input_norm=norm(rng, H), post_norm=norm(rng, H), q_norm=norm(rng, W), k_norm=norm(rng, W),
                q=affine(rng, (W, H)), k=affine(rng, (W, H)), v=affine(rng, (W, H)), o=affine(rng, (H, W)),
                router=affine(rng, (E, H)),
                experts={"gate": affine(rng, (E, I, H)), "up": affine(rng, (E, I, H)),
                         "down": affine(rng, (E, H, I))})


def empty_cache(cfg):
    return np.zeros((cfg.heads, cfg.capacity, cfg.head_dim), np.float32)


def test_batched_decode_layer_equals_per_request_layers():
    rng = np.random.default_rng(31)
    cfg = tiny_cfg()
    layer = layer_weights(rng, cfg)
    lengths = [5, 9, 2]
    B = len(lengths)
    kc, vc = [], []
    for n in lengths:
        k, v = empty_cache(cfg), empty_cache(cfg)
        k[:, :n] = oracle.round_f16(rng.standard_normal((cfg.heads, n, cfg.head_dim)))
        v[:, :n] = oracle.round_f16(rng.standard_normal((cfg.heads, n, cfg.head_dim)))
        kc.append(k)
        vc.append(v)
    h = oracle.to_act(rng.standard_normal((B, cfg.hidden)).astype(np.float32), "f16")
    kb, vb = [k.copy() for k in kc], [v.copy() for v in vc]
    batched = oracle.decode_layer_batched(h, layer, cfg, kb, vb, lengths)
    for b, n in enumerate(lengths):
        k1, v1 = kc[b].copy(), vc[b].copy()
        single = oracle.layer_forward(h[b:b + 1], layer, cfg, k1, v1, np.array([n]))
        # one BLAS call over the batch vs one per row: at most an f16 ulp apart
        assert_close(batched[b], single[0], max_abs=2e-3, mean_rel=1e-4, ulp_act="f16")
        # the appended slot is the same RoPE'd key / value
        np.testing.assert_allclose(kb[b][:, n], k1[:, n], atol=2e-3)
        assert np.array_equal(vb[b][:, n], v1[:, n])
        assert np.array_equal(kb[b][:, :n], kc[b][:, :n])  # earlier slots untouched


def test_prefill_then_decode_equals_one_longer_prefill():
    rng = np.random.default_rng(32)
    cfg = tiny_cfg()
    weights = dict(embed=affine(rng, (cfg.vocab, cfg.hidden)), lm_head=affine(rng, (cfg.vocab, cfg.hidden)),
                   final_norm=norm(rng, cfg.hidden), layers=[layer_weights(rng, cfg) for _ in range(cfg.layers)])
    ids = rng.integers(0, cfg.vocab, size=7)
    ka = [empty_cache(cfg) for _ in range(cfg.layers)]
    va = [empty_cache(cfg) for _ in range(cfg.layers)]
    oracle.model_forward(ids[:6], weights, cfg, ka, va, 0)
    stepped = oracle.model_forward(ids[6:], weights, cfg, ka, va, 6)
    kb = [empty_cache(cfg) for _ in range(cfg.layers)]
    vb = [empty_cache(cfg) for _ in range(cfg.layers)]
    whole = oracle.model_forward(ids, weights, cfg, kb, vb, 0)
    assert_close(stepped, whole, max_abs=2e-3, mean_rel=1e-4)
    assert int(np.argmax(stepped)) == int(np.argmax(whole))
    for layer in range(cfg.layers):
        np.testing.assert_allclose(ka[layer][:, :7], kb[layer][:, :7], atol=2e-3)
        np.testing.assert_allclose(va[layer][:, :7], vb[layer][:, :7], atol=2e-3)
        assert not ka[layer][:, 7:].any()


def test_fast_attention_variant_matches_float64():
    rng = np.random.default_rng(33)
    Hh, D, L = 4, 128, 300
    q = oracle.round_f16(rng.standard_normal((5, Hh, D)))
    K = oracle.round_f16(rng.standard_normal((Hh, L, D)))
    V = oracle.round_f16(rng.standard_normal((Hh, L, D)))
    scale = np.float32(D ** -0.5)
    for offset in (None, L - 5):
        exact = oracle.sdpa(q, K, V, scale, "f16", causal_offset=offset)
        fast = oracle.sdpa(q, K, V, scale, "f16", causal_offset=offset, fast=True)
        assert_close(fast, exact, max_abs=4e-3, mean_rel=1e-3)
