"""Expert parallelism (config 5's layout) on CPU: world_size 2, 4 and 8 gloo
ranks, each with its own tokens and E/n experts, exchange counts, token rows
and expert outputs with all-to-alls; the result must equal the oracle's
single-process MoE block on each rank's tokens within the layer tolerance
(routing and the combine are per token and an expert row depends only on its
input row; the oracle's per-expert BLAS matmul may sum a row in a different
order when the expert holds a different number of rows, which is the only
difference, at most one act ulp).  Skewed routing leaves some ranks with no
rows to compute: either a few experts' router rows scaled up, or config 5's
own skew, a per-expert router-logit bias N(0, 1.5) carried by a constant
input column."""
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


def _worker(rank, world, port, skew, path, E=8):
    import oracle
    from tests.ep_kernels import OracleKernels
    from tests.gpu_util import experts_np
    from trifuse_b200.ep import ExpertParallelMoE, shard_experts
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        K, H, I = 2, 256, 128
        shared = np.random.default_rng(5)          # same weights on every rank
        ex = experts_np(shared, E, H, I)
        wr = shared.standard_normal((E, H)).astype(np.float32) * 0.05
        if skew == "rows":                         # experts 0-1 win almost every route
            wr[:2] *= 40.0
        elif skew == "bias":                       # per-expert logit bias N(0, 1.5) on input column H-1
            wr[:, -1] = shared.standard_normal(E).astype(np.float32) * 1.5
        w = oracle.to_act(wr, "f16")
        local = np.random.default_rng(100 + rank)  # each rank's own tokens
        T = 9 + 3 * rank
        xs = local.standard_normal((T, H)).astype(np.float32)
        if skew == "bias":
            xs[:, -1] = 1.0
        x = oracle.to_act(xs, "f16")
        res = oracle.to_act(local.standard_normal((T, H)).astype(np.float32), "f16")
        t = lambda a: torch.from_numpy(np.asarray(a))  # noqa: E731
        full = {k: tuple(t(a) for a in v) for k, v in ex.items()}
        g, u, d = shard_experts(full["gate"], full["up"], full["down"], rank, world)
        moe = ExpertParallelMoE(t(w).to(torch.float16), g, u, d, E, K, kernels=OracleKernels())
        out = moe(t(x).to(torch.float16), t(res).to(torch.float16))
        ref, _ = oracle.moe_block(x, res, ("dense", w), ex, K, "f16")
        from tests.parity import assert_close
        try:
            assert_close(out.float().numpy(), np.asarray(ref, np.float32), ulp_act="f16")
            msg = "ok"
        except AssertionError as e:
            msg = f"mismatch: {e}"
        with open(f"{path}.{rank}", "w") as f:
            f.write(msg)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,skew,E", [(2, None, 8), (2, "rows", 8), (4, "rows", 8), (8, "bias", 64)])
def test_expert_parallel_matches_single_process(tmp_path, world, skew, E):
    path = str(tmp_path / "result")
    mp.spawn(_worker, args=(world, _free_port(), skew, path, E), nprocs=world, join=True)
    for r in range(world):
        assert open(f"{path}.{r}").read() == "ok", f"rank {r}"
