"""Parity of the tcgen05/TMEM 4-bit QMM path (batched decode / prefill
shapes) against the oracle and against the CUDA-core GEMV path."""
import contextlib

import numpy as np
import pytest

import oracle
from tests.gpu_util import bits_equal, dev, experts_dev, experts_np, host
from tests.parity import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from trifuse_b200 import ops as _ops
    return _ops


@contextlib.contextmanager
def path(ops, p):
    ops.set_qmm_path(p)
    try:
        yield
    finally:
        ops.set_qmm_path(0)


@pytest.mark.parametrize("act,T,out,inn", [("f16", 8, 2048, 2048), ("bf16", 16, 6144, 2048),
                                           ("f16", 64, 2048, 1024), ("bf16", 300, 1024, 2048),
                                           ("f16", 77, 50304 // 8, 2048)])
def test_dense_tensor_core_qmm(ops, act, T, out, inn):
    rng = np.random.default_rng(11)
    x = oracle.to_act(rng.standard_normal((T, inn)).astype(np.float32), act)
    q, s, b = oracle.affine_quantize(oracle.round_bf16(rng.standard_normal((out, inn)).astype(np.float32) * 0.02))
    args = (dev(x, act), dev(q), dev(s), dev(b), 64, 4)
    with path(ops, 2):
        tc = host(ops.native_affine_qmm(*args))
    with path(ops, 1):
        gemv = host(ops.native_affine_qmm(*args))
    assert ops.device_error() == 0
    ref = oracle.affine_qmm(x, q, s, b, act)
    assert_close(tc, ref)
    assert_close(tc, gemv)


@pytest.mark.parametrize("act,T,skew", [("bf16", 2, False), ("f16", 12, True), ("f16", 64, False),
                                        ("bf16", 256, False), ("f16", 600, True), ("bf16", 2048, True)])
def test_moe_tensor_core_against_oracle(ops, act, T, skew):
    rng = np.random.default_rng(12)
    H, I, E, K = 2048, 1024, 64, 8
    x = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    res = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    ex = experts_np(rng, E, H, I)
    wr = rng.standard_normal((E, H)).astype(np.float32) * 0.02
    if skew:  # uneven expert loads: router rows with larger norms win more tokens
        wr *= (1 + np.abs(rng.standard_normal((E, 1)).astype(np.float32)) * 3)
    w = oracle.to_act(wr, act)
    d = experts_dev(ex)
    zero = np.zeros_like(res)
    with path(ops, 2):
        out, aux = ops.moe(dev(x, act), dev(res, act), dev(w, act), d["gate"], d["up"], d["down"], K,
                           return_aux=True)
        moe_only = ops.moe(dev(x, act), dev(zero, act), dev(w, act), d["gate"], d["up"], d["down"], K)
    assert ops.device_error() == 0
    ref, raux = oracle.moe_block(x, res, ("dense", w), ex, K, act)
    ref0, _ = oracle.moe_block(x, zero, ("dense", w), ex, K, act)
    assert np.array_equal(host(aux["indices"]), raux["indices"])
    assert_close(host(moe_only), ref0)            # the gather_qmm path's own output
    assert_close(host(out), ref, ulp_act=act)     # with the residual stream
    if T * K >= 16:  # the automatic choice takes the tensor cores from 16 routes on
        auto = ops.moe(dev(x, act), dev(res, act), dev(w, act), d["gate"], d["up"], d["down"], K)
        assert np.array_equal(host(auto), host(out))


def test_expert_hook_tensor_core(ops):
    rng = np.random.default_rng(13)
    act, T, H, I, E, N = "bf16", 200, 2048, 1024, 8, 900
    x = oracle.to_act(rng.standard_normal((T, H)).astype(np.float32), act)
    ex = experts_np(rng, E, H, I)
    tok = rng.integers(0, T, size=N).astype(np.int32)
    eid = rng.integers(0, E, size=N).astype(np.int32)
    d = experts_dev(ex)
    with path(ops, 2):
        out, inverse = ops.expert_gpu(dev(x, act), dev(tok), dev(eid), False, d["gate"], d["up"], d["down"])
    assert ops.device_error() == 0
    order = np.argsort(eid, kind="stable")
    rows = x[tok[order]]
    sel = eid[order]
    h = oracle.swiglu(oracle.gather_qmm(rows, *ex["gate"], sel, act),
                      oracle.gather_qmm(rows, *ex["up"], sel, act), act)
    assert_close(host(out), oracle.gather_qmm(h, *ex["down"], sel, act))


def _dequant_torch(q, s, b):
    """fp16(code * s + b) for packed [out, in/8] uint32 words (torch, fp32 result)."""
    import torch
    out, inw = q.shape[0], q.shape[1] * 8
    qi = q.view(torch.int32).long() & 0xFFFFFFFF
    codes = torch.stack([(qi >> (4 * i)) & 0xF for i in range(8)], -1).reshape(out, inw).float()
    w = codes.view(out, -1, 64) * s.float()[..., None] + b.float()[..., None]
    return w.reshape(out, inw).half().float()


def test_tensor_core_many_tiles_per_block_is_deterministic(ops):
    """Many 256-token tiles per persistent block keep every ring slot busy;
    repeated launches must agree bit for bit and match an fp32 reference
    (a slot released before its shared loads completed once let the next
    TMA fill overtake them)."""
    import torch
    from trifuse_b200.quant import random_affine
    g = torch.Generator(device="cuda")
    g.manual_seed(21)
    w = random_affine((32768, 2048), g, "cuda")
    x = torch.randn(1024, 2048, device="cuda", dtype=torch.float16, generator=g)
    ref = x.float() @ _dequant_torch(*w).t()
    with path(ops, 2):
        ys = [ops.native_affine_qmm(x, *w, 64, 4) for _ in range(3)]
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    for y in ys[1:]:
        assert torch.equal(y, ys[0])
    err = (ys[0].float() - ref).abs()
    assert err.max().item() <= 2e-2 + 4e-3 * ref.abs().max().item()
    assert (err / (ref.abs() + 1)).mean().item() < 1e-3
