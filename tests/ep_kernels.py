"""Oracle-backed kernels for the expert-parallel block's CPU tests: the same
interface as trifuse_b200.ep.CudaKernels, computed with the numpy oracle on
CPU torch tensors (test infrastructure only)."""
import numpy as np
import torch

import oracle

_ACT = {torch.float16: "f16", torch.bfloat16: "bf16"}


def _np(t):
    return t.float().numpy() if t.is_floating_point() else t.numpy()


class OracleKernels:
    def __init__(self, act=torch.float16):
        self.act, self.a = act, _ACT[act]

    def route(self, x, router, k, experts):
        logits = oracle.router_logits_dense(_np(x), _np(router), self.a)
        idx, gates = oracle.olmoe_route(logits, k, self.a)
        return torch.from_numpy(np.asarray(idx, np.int32)), torch.from_numpy(np.asarray(gates, np.float32)).to(self.act)

    def route_sort(self, idx, experts):
        order, inverse, offsets = oracle.route_sort(_np(idx), experts)
        return tuple(torch.from_numpy(np.asarray(a, np.int32)) for a in (order, inverse, offsets))

    def experts(self, rows, expert_ids, gate, up, down):
        r = _np(rows)
        e = _np(expert_ids).astype(np.int64)
        if r.shape[0] == 0:
            return rows.clone()
        g = oracle.gather_qmm(r, *[_np(t) if t.is_floating_point() else t.numpy() for t in gate], e, self.a)
        u = oracle.gather_qmm(r, *[_np(t) if t.is_floating_point() else t.numpy() for t in up], e, self.a)
        h = oracle.swiglu(g, u, self.a)
        y = oracle.gather_qmm(h, *[_np(t) if t.is_floating_point() else t.numpy() for t in down], e, self.a)
        return torch.from_numpy(np.asarray(y, np.float32)).to(self.act)

    def gather_rows(self, x, order, k):
        return x.index_select(0, order.long() // k).contiguous()

    def combine(self, y_sorted, inverse, gates, residual):
        T, K = gates.shape
        y = _np(y_sorted)[_np(inverse).astype(np.int64)].reshape(T, K, -1)
        out = oracle.combine(y, _np(gates), _np(residual), self.a)
        return torch.from_numpy(np.asarray(out, np.float32)).to(self.act)
