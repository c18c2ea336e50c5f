"""tf_moe_forward_noalloc: the MoE block for callers that cannot allocate.

Callers such as a host framework's execute callback (whose device memory
was planned ahead of time) or a serving loop that must not let cudaMalloc
synchronize the device use this entry point: it takes only inputs and
outputs and draws its scratch from a fixed buffer inside the library.  These
tests call it through the C ABI twice in a row (a 64-token decode batch on
the tensor-core path, then a 5-token batch on the CUDA-core path, so the
second call runs over what the first left in the shared buffer) and compare
each result with tf_moe_forward given its own workspace.  This file is
named to be collected last."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle
from tests.gpu_util import dev, experts_dev, experts_np, host
from tests.parity import assert_close


def _args(ops, x, res, out, router, ex):
    return ops.moe_args(x, res, out, router, ex["gate"], ex["up"], ex["down"], 8)


def _inputs(rng, T, act):
    x = oracle.to_act(rng.standard_normal((T, 2048)).astype(np.float32), act)
    res = oracle.to_act(rng.standard_normal((T, 2048)).astype(np.float32), act)
    return dev(x, act), dev(res, act)


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_twice():
    from trifuse_b200 import ops
    from trifuse_b200._lib import check, lib
    rng = np.random.default_rng(20261201)
    act = "bf16"
    ex = experts_dev(experts_np(rng, 64, 2048, 1024))
    rq, rs, rb = oracle.affine_quantize(oracle.round_bf16(rng.standard_normal((64, 2048)).astype(np.float32) * 0.02))
    router = (dev(rq), dev(rs), dev(rb))
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for T in (64, 5):
        x, res = _inputs(rng, T, act)
        got = torch.empty_like(x)
        a = _args(ops, x, res, got, router, ex)
        check(lib().tf_moe_forward_noalloc(C.byref(a), stream))
        want = torch.empty_like(x)
        b = _args(ops, x, res, want, router, ex)
        nb = C.c_size_t()
        check(lib().tf_moe_workspace_size(C.byref(b), C.byref(nb)))
        ws = torch.empty(nb.value, dtype=torch.uint8, device="cuda")
        check(lib().tf_moe_forward(C.byref(b), C.c_void_p(ws.data_ptr()), nb.value, stream))
        torch.cuda.synchronize()
        assert_close(host(got), host(want), ulp_act=act)
        assert torch.isfinite(got.float()).all()
    assert ops.device_error() == 0


def test_noalloc_rejects_batches_beyond_its_buffer():
    """65 tokens need more than the fixed buffer: a clear TF_ERR_CAPACITY,
    decided before any device work (runs without a GPU)."""
    from trifuse_b200._lib import AffineWeight, MoeArgs, lib
    a = MoeArgs()
    a.x = a.residual = a.out = 0x1000
    a.tokens, a.hidden, a.intermediate, a.experts, a.top_k, a.act = 65, 2048, 1024, 64, 8, 2
    a.router.affine = AffineWeight(0x1000, 0x2000, 0x3000, 0, 64, 2048, 64, 4)
    a.gate_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 1024, 2048, 64, 4)
    a.up_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 1024, 2048, 64, 4)
    a.down_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 2048, 1024, 64, 4)
    assert lib().tf_moe_forward_noalloc(C.byref(a), None) == 10  # TF_ERR_CAPACITY
    assert b"fixed buffer" in lib().tf_last_error()


def test_noalloc_buffer_holds_its_largest_batch():
    """The workspace a 64-token OLMoE block needs fits the fixed buffer, for
    both activation dtypes (runs without a GPU)."""
    from trifuse_b200._lib import AffineWeight, MoeArgs, lib
    for act in (1, 2):
        a = MoeArgs()
        a.x = a.residual = a.out = 0x1000
        a.tokens, a.hidden, a.intermediate, a.experts, a.top_k, a.act = 64, 2048, 1024, 64, 8, act
        a.router.affine = AffineWeight(0x1000, 0x2000, 0x3000, 0, 64, 2048, 64, 4)
        a.gate_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 1024, 2048, 64, 4)
        a.up_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 1024, 2048, 64, 4)
        a.down_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 2048, 1024, 64, 4)
        nb = C.c_size_t()
        assert lib().tf_moe_workspace_size(C.byref(a), C.byref(nb)) == 0
        assert 0 < nb.value <= 6 << 20
