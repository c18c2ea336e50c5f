"""Expert-parallel OLMoE MoE block over a torch.distributed process group.

Rank r of n owns experts [r*E/n, (r+1)*E/n) and the full router; every rank
brings its own tokens.  One call is the reference's moe() (MLXNativeGranite
MoEPrefill.h:627-702) with the expert step spread over the ranks:

  1. route locally: router GEMV + fp32 softmax + stable top-k (a1, a2);
  2. group the routes by expert with the stable route sort (a3); because rank
     = expert // (E/n), the same order groups them by destination rank, and
     the sort offsets give the rows bound for each rank;
  3. exchange the per-rank row counts (all-to-all of integers);
  4. dispatch: all-to-all of the routed token rows (act, hidden wide) and of
     their expert ids (local to the destination rank);
  5. each rank runs its experts on the rows it received (gate/up gather_qmm,
     SwiGLU, down gather_qmm: the expert hook's GPU callable,
     MLXMoEExpertHook.h:25-32) and keeps the received order;
  6. return: the all-to-all in the opposite direction brings every expert
     output back to its route's source rank, in route-sort order;
  7. combine: residual + sum_k gate_k * y_k in k order (a6), the same kernel
     as the single-GPU block.

Dropless: buffers are sized by the exchanged counts, no capacity factor (the
reference never drops).  Routing and the combine are per token, and an
expert's output row depends only on its input row, so the result equals the
single-GPU block on the same tokens up to the expert kernel the row count
selects (tensor cores or CUDA cores, both within the parity tolerance).
The exchanges are NCCL all-to-alls on GPUs (gloo in the CPU tests); the
kernels are pluggable so the data movement can be tested on CPU.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class CudaKernels:
    """The CUDA kernels of this package (the product path)."""

    def route(self, x, router, k, experts):
        from . import ops
        _, idx, gates = ops.olmoe_router(x, router, k, experts)
        return idx, gates

    def route_sort(self, idx, experts):
        from . import ops
        return ops.moe_route_sort(idx, experts)

    def experts(self, rows, expert_ids, gate, up, down):
        """Expert outputs in the received order (the down projection writes
        each row back to its route's position; no un-permute)."""
        from . import ops
        n = rows.shape[0]
        if n == 0:
            return torch.empty_like(rows)
        tok = torch.arange(n, dtype=torch.int32, device=rows.device)
        return ops.expert_gpu_ordered(rows, tok, expert_ids.to(torch.int32), gate, up, down, check_ranges=False)

    def gather_rows(self, x, order, k):
        """Rows x[order // k] in route-sort order (the dispatch send buffer)."""
        from . import ops
        return ops.gather_rows(x, order.to(torch.int32), k)

    def combine(self, y_sorted, inverse, gates, residual):
        from . import ops
        return ops.moe_combine(y_sorted, inverse, gates, residual)


class ExpertParallelMoE:
    """One MoE block with this rank's share of the experts.

    router: dense act [E, H] or 4-bit (q, s, b) [E, ...], the full router.
    gate / up / down: (q, s, b) stacked over this rank's E/n local experts.
    """

    def __init__(self, router, gate, up, down, experts: int, top_k: int, group=None, kernels=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if experts % self.world:
            raise ValueError(f"{experts} experts do not split over {self.world} ranks")
        self.experts, self.top_k = experts, top_k
        self.local = experts // self.world
        if gate[0].shape[0] != self.local:
            raise ValueError(f"rank {self.rank} holds {gate[0].shape[0]} experts, expected {self.local}")
        self.router, self.gate, self.up, self.down = router, gate, up, down
        self.k = kernels or CudaKernels()

    def forward(self, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        K, E, L, n = self.top_k, self.experts, self.local, self.world
        dev = x.device
        idx, gates = self.k.route(x, self.router, K, E)
        order, inverse, offsets = self.k.route_sort(idx, E)
        # rows bound for each rank: routes of experts [r*L, (r+1)*L)
        bounds = offsets.long()[torch.arange(0, E + 1, L, device=offsets.device)]
        send_counts = (bounds[1:] - bounds[:-1]).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        # the one host synchronization of the layer: NCCL takes host split sizes
        sizes = torch.stack([send_counts, recv_counts]).cpu()
        send_sizes, recv_sizes = sizes[0].tolist(), sizes[1].tolist()
        # dispatch token rows (gathered straight into the send buffer) and
        # their destination-local expert ids
        sel = idx.reshape(-1).index_select(0, order.long())
        send_rows = self.k.gather_rows(x, order, K)
        send_eid = (sel % L).to(torch.int32)
        recv_rows = torch.empty((sum(recv_sizes), H), dtype=x.dtype, device=dev)
        recv_eid = torch.empty(sum(recv_sizes), dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_rows, send_rows, recv_sizes, send_sizes, group=self.group)
        dist.all_to_all_single(recv_eid, send_eid, recv_sizes, send_sizes, group=self.group)
        # local experts, rows kept in received order
        y_local = self.k.experts(recv_rows, recv_eid, self.gate, self.up, self.down).contiguous()
        # return every row to its source rank, in that rank's route-sort order
        y_sorted = torch.empty((T * K, H), dtype=x.dtype, device=dev)
        dist.all_to_all_single(y_sorted, y_local, send_sizes, recv_sizes, group=self.group)
        return self.k.combine(y_sorted, inverse, gates, residual)

    __call__ = forward


def shard_experts(gate, up, down, rank: int, world: int):
    """This rank's slice [r*E/n, (r+1)*E/n) of stacked (q, s, b) experts."""
    E = gate[0].shape[0]
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    L = E // world
    sl = slice(rank * L, (rank + 1) * L)
    return tuple(tuple(t[sl].contiguous() for t in w) for w in (gate, up, down))
