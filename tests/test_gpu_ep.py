"""Expert parallelism on GPUs with NCCL: the CUDA kernels (router, route
sort, expert hook gather_qmm, combine) with all-to-all dispatch/return.  One
rank in-process always; two ranks as child processes when the box has two
GPUs.  Each rank's output is checked against the oracle's MoE block."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(rank, T):
    import oracle
    from tests.gpu_util import experts_np
    E, K, H, I = 64, 8, 2048, 1024
    shared = np.random.default_rng(21)
    ex = experts_np(shared, E, H, I)
    wr = shared.standard_normal((E, H)).astype(np.float32) * 0.02
    wr *= 1 + np.abs(shared.standard_normal((E, 1)).astype(np.float32)) * 3   # skewed loads
    w = oracle.to_act(wr, "bf16")
    local = np.random.default_rng(200 + rank)
    x = oracle.to_act(local.standard_normal((T, H)).astype(np.float32), "bf16")
    res = oracle.to_act(local.standard_normal((T, H)).astype(np.float32), "bf16")
    return ex, w, x, res, E, K


def _run_rank(rank, world, T):
    import oracle
    from tests.gpu_util import dev, experts_dev, host
    from tests.parity import assert_close
    from trifuse_b200 import ops
    from trifuse_b200.ep import ExpertParallelMoE, shard_experts
    ex, w, x, res, E, K = _case(rank, T)
    d = experts_dev(ex)
    g, u, dn = shard_experts(d["gate"], d["up"], d["down"], rank, world)
    moe = ExpertParallelMoE(dev(w, "bf16"), g, u, dn, E, K)
    out = host(moe(dev(x, "bf16"), dev(res, "bf16")))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    ref, _ = oracle.moe_block(x, res, ("dense", w), ex, K, "bf16")
    assert_close(out, ref, ulp_act="bf16")
    single = host(ops.moe(dev(x, "bf16"), dev(res, "bf16"), dev(w, "bf16"), d["gate"], d["up"], d["down"], K))
    assert_close(out, single, ulp_act="bf16")


def test_expert_parallel_one_rank_nccl():
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda:0"))
    try:
        _run_rank(0, 1, T=512)
    finally:
        dist.destroy_process_group()


def _child(rank, world, port, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        _run_rank(rank, world, T=384 + 64 * rank)
        msg = "ok"
    except AssertionError as e:  # report, and still take part in teardown
        msg = f"fail: {e}"
    finally:
        dist.destroy_process_group()
    with open(f"{path}.{rank}", "w") as f:
        f.write(msg)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_two_ranks_nccl(tmp_path):
    path = str(tmp_path / "r")
    mp.spawn(_child, args=(2, _free_port(), path), nprocs=2, join=True)
    for r in range(2):
        assert open(f"{path}.{r}").read() == "ok"
