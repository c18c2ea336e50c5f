"""Expert parallelism (config 5's layout) on CPU: world_size 2 and 4 gloo
ranks, each with its own tokens and E/n experts, exchange counts, token rows
and expert outputs with all-to-alls; the result must equal the oracle's
single-process MoE block on each rank's tokens bit for bit (routing and the
combine are per token and an expert row depends only on its input row).
Skewed routing leaves some ranks with no rows to compute."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, skew, path):
    import oracle
    from tests.ep_kernels import OracleKernels
    from tests.gpu_util import experts_np
    from trifuse_b200.ep import ExpertParallelMoE, shard_experts
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, K, H, I = 8, 2, 256, 128
        shared = np.random.default_rng(5)          # same weights on every rank
        ex = experts_np(shared, E, H, I)
        wr = shared.standard_normal((E, H)).astype(np.float32) * 0.05
        if skew:                                   # experts 0-1 win almost every route
            wr[:2] *= 40.0
        w = oracle.to_act(wr, "f16")
        local = np.random.default_rng(100 + rank)  # each rank's own tokens
        T = 9 + 3 * rank
        x = oracle.to_act(local.standard_normal((T, H)).astype(np.float32), "f16")
        res = oracle.to_act(local.standard_normal((T, H)).astype(np.float32), "f16")
        t = lambda a: torch.from_numpy(np.asarray(a))  # noqa: E731
        full = {k: tuple(t(a) for a in v) for k, v in ex.items()}
        g, u, d = shard_experts(full["gate"], full["up"], full["down"], rank, world)
        moe = ExpertParallelMoE(t(w).to(torch.float16), g, u, d, E, K, kernels=OracleKernels())
        out = moe(t(x).to(torch.float16), t(res).to(torch.float16))
        ref, _ = oracle.moe_block(x, res, ("dense", w), ex, K, "f16")
        ok = np.array_equal(out.float().numpy(), np.asarray(ref, np.float32))
        with open(f"{path}.{rank}", "w") as f:
            f.write("ok" if ok else f"mismatch max {np.abs(out.float().numpy() - ref).max()}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,skew", [(2, False), (2, True), (4, True)])
def test_expert_parallel_matches_single_process(tmp_path, world, skew):
    path = str(tmp_path / "result")
    mp.spawn(_worker, args=(world, _free_port(), skew, path), nprocs=world, join=True)
    for r in range(world):
        assert open(f"{path}.{r}").read() == "ok", f"rank {r}"
