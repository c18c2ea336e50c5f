"""tf_moe_forward_noalloc: the MoE block for callers that cannot allocate.

Callers such as a host framework's execute callback (whose device memory
was planned ahead of time) or a serving loop that must not let cudaMalloc
synchronize the device use this entry point: it takes only inputs and
outputs and draws its scratch from a fixed buffer inside the library.  The
GPU test calls it through the C ABI three times in a row, each call running
over what the previous one left in the shared buffer: a 64-token batch (512
routes, tensor-core path), a 1-token batch (8 routes, below the 16-route
cutoff, so the CUDA-core GEMV path and its part of the buffer) and a
5-token batch (40 routes, tensor cores again).  Each result is compared with
tf_moe_forward given its own workspace and with the CPU oracle (routing
bit-exact, output within tolerance).  This file is named to be collected
last."""
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
def test_noalloc_matches_workspace_entry_and_oracle():
    from trifuse_b200 import ops
    from trifuse_b200._lib import check, lib
    rng = np.random.default_rng(20261201)
    act = "bf16"
    ex_np = experts_np(rng, 64, 2048, 1024)
    ex = experts_dev(ex_np)
    rq, rs, rb = oracle.affine_quantize(oracle.round_bf16(rng.standard_normal((64, 2048)).astype(np.float32) * 0.02))
    router = (dev(rq), dev(rs), dev(rb))
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for T in (64, 1, 5):
        x, res = _inputs(rng, T, act)
        got = torch.empty_like(x)
        idx = torch.empty((T, 8), dtype=torch.int32, device="cuda")
        a = ops.moe_args(x, res, got, router, ex["gate"], ex["up"], ex["down"], 8, indices=idx)
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
        ref, raux = oracle.moe_block(host(x), host(res), ("affine", rq, rs, rb), ex_np, 8, act)
        assert np.array_equal(idx.cpu().numpy(), raux["indices"]), f"T={T}: routing differs from the oracle"
        assert_close(host(got), ref, ulp_act=act)
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


def test_noalloc_admits_its_largest_batch():
    """A 64-token OLMoE block (f16 and bf16) passes the fixed buffer's size
    check: the call gets past admission (without a GPU it then stops at the
    device lookup, never with TF_ERR_CAPACITY)."""
    from trifuse_b200._lib import AffineWeight, MoeArgs, lib
    for act in (1, 2):
        a = MoeArgs()
        a.x = a.residual = a.out = 0x1000
        a.tokens, a.hidden, a.intermediate, a.experts, a.top_k, a.act = 64, 2048, 1024, 64, 8, act
        a.router.affine = AffineWeight(0x1000, 0x2000, 0x3000, 0, 64, 2048, 64, 4)
        a.gate_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 1024, 2048, 64, 4)
        a.up_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 1024, 2048, 64, 4)
        a.down_proj = AffineWeight(0x1000, 0x2000, 0x3000, 64, 2048, 1024, 64, 4)
        if torch.cuda.is_available():
            pytest.skip("admission-only check; on a GPU the fake pointers would be used")
        rc = lib().tf_moe_forward_noalloc(C.byref(a), None)
        assert rc != 10 and b"fixed buffer" not in lib().tf_last_error(), lib().tf_last_error()
