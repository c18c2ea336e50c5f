"""Python mirror of the reference's MLX operator surface, backed by the C ABI.

Names, argument meaning and error behaviour follow
``overlays/executorch/backends/mlx/native_affine_ops.py`` (the torch custom
ops ``mlx::native_*`` that TriFuse's OLMoE export lowers onto MLX) plus the
runtime-level pieces of the OLMoE adapter (``olmoe_route``, the route sort,
``moe()``, the expert hook's GPU callable, T1 attention).  Every function
takes CUDA tensors and launches the sm_100a kernels of ``libtrifuse_b200.so``
on the current torch stream; there is no CPU path.  torch is used only to
allocate outputs and scratch.
"""
from __future__ import annotations

import ctypes as C

import torch
from torch import Tensor

from ._lib import (AffineWeight, DTYPE_BF16, DTYPE_F16, MoeArgs, RouterWeight, check, lib)

_ACT = {torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}


def _act(t: Tensor) -> int:
    if t.dtype not in _ACT:
        raise ValueError("activations must be float16 or bfloat16")
    return _ACT[t.dtype]


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("trifuse_b200 ops take CUDA tensors (no CPU path)")


def _check_range(ids: Tensor, limit: int, message: str):
    """ids must lie in [0, limit): the kernels index with them unchecked
    (a host read of the extremes, one synchronization)."""
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= limit):
        raise ValueError(message)


def _ws(nbytes: int, device) -> Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def validate_affine(q, scales, biases, group_size, bits, rank):
    """Same checks and messages as native_affine_ops.py:12-26."""
    if (type(bits) is not int or bits not in (4, 8)
            or type(group_size) is not int or group_size not in (32, 64, 128)):
        raise ValueError("Native affine requires bits4/8 and group32/64/128")
    if q.dtype != torch.uint32 or q.ndim != rank or rank not in (2, 3):
        raise ValueError("Native affine Q must be rank2/3 uint32")
    if (scales.dtype not in (torch.float16, torch.float32) or biases.dtype != scales.dtype
            or scales.shape != biases.shape or scales.ndim != rank
            or q.shape[:-1] != scales.shape[:-1]):
        raise ValueError("Native affine S/B shapes or floating dtypes differ")
    width = q.shape[-1] * (32 // bits)
    if (width % group_size or scales.shape[-1] * group_size != width
            or any(type(d) is not int or d <= 0 for d in q.shape)):
        raise ValueError("Native affine packed/group dimensions differ")
    if scales.dtype != torch.float16:
        raise NotImplementedError("this path consumes float16 scales/biases")
    return width


def affine_desc(q, scales, biases, group_size=64, bits=4) -> AffineWeight:
    width = validate_affine(q, scales, biases, group_size, bits, q.ndim)
    _cuda(q, scales, biases)
    for t in (q, scales, biases):
        if not t.is_contiguous():
            raise ValueError("Native affine Q/S/B must be contiguous")
    stacked = q.ndim == 3
    return AffineWeight(q.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                        q.shape[0] if stacked else 0, q.shape[-2], width, group_size, bits)


def native_affine_qmm(x: Tensor, q: Tensor, scales: Tensor, biases: Tensor, group_size: int,
                      bits: int) -> Tensor:
    """``mlx::native_affine_qmm`` (native_affine_ops.py:39-52)."""
    w = affine_desc(q, scales, biases, group_size, bits)
    if q.ndim != 2:
        raise ValueError("Native affine Q must be rank2/3 uint32")
    if x.ndim < 1 or x.shape[-1] != w.in_features:
        raise ValueError("Native affine QMM input width/dtype differs")
    _cuda(x)
    x2 = x.contiguous().reshape(-1, w.in_features)
    y = torch.empty((*x.shape[:-1], w.out_features), dtype=x.dtype, device=x.device)
    check(lib().tf_affine_qmm(_ptr(x2), x2.shape[0], C.byref(w), _act(x), _ptr(y), _stream()))
    return y


def native_affine_gather_qmm(x: Tensor, q: Tensor, scales: Tensor, biases: Tensor, indices: Tensor,
                             group_size: int, bits: int, sorted_indices: bool = False) -> Tensor:
    """``mlx::native_affine_gather_qmm`` (native_affine_ops.py:55-74).

    Supports the reference's call forms (x[..., 1, H] broadcast against
    indices[...]): batch = broadcast(x.shape[:-2], indices.shape), output
    [*batch, 1, out]."""
    if q.ndim != 3:
        raise ValueError("Native affine Q must be rank2/3 uint32")
    w = affine_desc(q, scales, biases, group_size, bits)
    if indices.dtype not in (torch.int32, torch.int64):
        raise ValueError("Expert indices must be integers")
    if (x.ndim < 2 or x.shape[-1] != w.in_features or type(sorted_indices) is not bool):
        raise ValueError("Native affine expert input differs")
    if x.shape[-2] != 1:
        raise NotImplementedError("gather_qmm rows per expert call must be 1 (the adapter's forms)")
    _cuda(x, indices)
    batch = torch.broadcast_shapes(x.shape[:-2], indices.shape)
    xb = x.contiguous().reshape(-1, w.in_features)
    x_index = torch.arange(xb.shape[0], device=x.device, dtype=torch.int32).reshape(x.shape[:-2])
    x_index = x_index.expand(batch).reshape(-1).contiguous()
    idx = indices.to(torch.int32).expand(batch).reshape(-1).contiguous()
    _check_range(idx, w.experts, "expert index out of range")
    y = torch.empty((*batch, 1, w.out_features), dtype=x.dtype, device=x.device)
    check(lib().tf_affine_gather_qmm(_ptr(xb), xb.shape[0], 1, _ptr(x_index), _ptr(idx), idx.numel(),
                                     C.byref(w), int(sorted_indices), _act(x), _ptr(y), _stream()))
    return y


def native_affine_embedding(indices: Tensor, q: Tensor, scales: Tensor, biases: Tensor,
                            group_size: int, bits: int, out_dtype=torch.float16) -> Tensor:
    """``mlx::native_affine_embedding`` (native_affine_ops.py:77-93); output in
    the scales dtype (float16) unless out_dtype says otherwise."""
    if q.ndim != 2:
        raise ValueError("Native affine Q must be rank2/3 uint32")
    w = affine_desc(q, scales, biases, group_size, bits)
    if indices.dtype not in (torch.int32, torch.int64):
        raise ValueError("Embedding indices must be integers")
    _cuda(indices)
    ids = indices.to(torch.int64).reshape(-1).contiguous()
    if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= w.out_features):
        raise ValueError("embedding index out of range")
    y = torch.empty((*indices.shape, w.in_features), dtype=out_dtype, device=indices.device)
    check(lib().tf_affine_embedding(_ptr(ids), ids.numel(), C.byref(w), _ACT[out_dtype], _ptr(y),
                                    _stream()))
    return y


def greedy_tokens(logits: Tensor) -> Tensor:
    """Greedy next tokens of fp32 logits [..., vocab]: argmax (lowest index on
    ties) where every logit of the row is finite, else -1 (int64); the
    reference's where(all(isfinite(logits)), argmax(logits), -1)
    (patches/executorch.patch:1350-1353)."""
    if logits.dtype != torch.float32:
        raise ValueError("greedy: logits must be float32")
    _cuda(logits)
    V = logits.shape[-1]
    lc = logits.contiguous().reshape(-1, V)
    out = torch.empty(lc.shape[0], dtype=torch.int64, device=logits.device)
    check(lib().tf_greedy_tokens(_ptr(lc), lc.shape[0], V, _ptr(out), _stream()))
    return out.reshape(logits.shape[:-1])


def native_olmoe_softmax(x: Tensor) -> Tensor:
    """``mlx::native_olmoe_softmax`` (native_affine_ops.py:128-138): fp32
    softmax over the last axis, rounded to the storage dtype."""
    _cuda(x)
    E = x.shape[-1]
    xc = x.contiguous()
    p = torch.empty_like(xc)
    check(lib().tf_olmoe_softmax(_ptr(xc), xc.numel() // E, E, _act(x), _ptr(p), _stream()))
    return p


def native_olmoe_topk_indices(x: Tensor, k: int) -> Tensor:
    """``mlx::native_olmoe_topk_indices`` (native_affine_ops.py:141-153):
    stable descending rank (ties to lower id, NaN last), first k, int32."""
    if type(k) is not int or not 0 < k <= x.shape[-1]:
        raise ValueError("Invalid OLMoE top-k")
    _cuda(x)
    E = x.shape[-1]
    xc = x.contiguous()
    out = torch.empty((*x.shape[:-1], k), dtype=torch.int32, device=x.device)
    check(lib().tf_olmoe_topk_indices(_ptr(xc), xc.numel() // E, E, k, _act(x), _ptr(out), _stream()))
    return out


def native_take_along_last(x: Tensor, indices: Tensor) -> Tensor:
    """``mlx::native_take_along_last`` (native_affine_ops.py:115-125)."""
    if (x.ndim < 1 or x.shape[:-1] != indices.shape[:-1]
            or indices.dtype not in (torch.int32, torch.int64)):
        raise ValueError("Native take requires matching leading dimensions and integer indices")
    _cuda(x, indices)
    W, K = x.shape[-1], indices.shape[-1]
    xc = x.contiguous()
    ic = indices.to(torch.int32).contiguous()
    out = torch.empty(indices.shape, dtype=x.dtype, device=x.device)
    check(lib().tf_take_along_last(_ptr(xc), xc.numel() // W, W, _ptr(ic), K, _act(x), _ptr(out),
                                   _stream()))
    return out


def olmoe_route(logits: Tensor, k: int):
    """``olmoe_route`` (MLXOLMoERouter.h:86-120): (indices int32, gates act)."""
    if type(k) is not int or not 0 < k <= logits.shape[-1]:
        raise ValueError("OLMoE router geometry differs")
    _cuda(logits)
    E = logits.shape[-1]
    lc = logits.contiguous()
    idx = torch.empty((*logits.shape[:-1], k), dtype=torch.int32, device=logits.device)
    gates = torch.empty((*logits.shape[:-1], k), dtype=logits.dtype, device=logits.device)
    check(lib().tf_olmoe_route(_ptr(lc), lc.numel() // E, E, k, _act(logits), _ptr(idx), _ptr(gates),
                               _stream()))
    return idx, gates


def router_desc(router) -> RouterWeight:
    """A dense act weight [E,H] or an affine (q, scales, biases) triple."""
    if isinstance(router, Tensor):
        _cuda(router)
        return RouterWeight(router.contiguous().data_ptr(), AffineWeight())
    q, s, b = router
    return RouterWeight(None, affine_desc(q, s, b))


def olmoe_router(x: Tensor, router, k: int, experts: int | None = None):
    """Router GEMV + route (MLXNativeGraniteMoEPrefill.h:631-632):
    returns (logits, indices, gates)."""
    _cuda(x)
    H = x.shape[-1]
    E = router.shape[0] if isinstance(router, Tensor) else router[0].shape[0]
    rw = router_desc(router)
    xc = x.contiguous().reshape(-1, H)
    T = xc.shape[0]
    logits = torch.empty((T, E), dtype=x.dtype, device=x.device)
    idx = torch.empty((T, k), dtype=torch.int32, device=x.device)
    gates = torch.empty((T, k), dtype=x.dtype, device=x.device)
    check(lib().tf_olmoe_router(_ptr(xc), T, H, C.byref(rw), E, k, _act(x), _ptr(logits), _ptr(idx),
                                _ptr(gates), _stream()))
    return logits, idx, gates


def moe_route_sort(indices: Tensor, experts: int):
    """Stable grouping of routes by expert (MLXNativeGraniteMoEPrefill.h:
    666-684): (order, inverse, offsets[E+1]), int32."""
    _cuda(indices)
    idx = indices.to(torch.int32).contiguous()
    _check_range(idx, experts, "expert index out of range")
    T = idx.shape[0] if idx.ndim > 1 else idx.numel()
    K = idx.shape[-1] if idx.ndim > 1 else 1
    n = idx.numel()
    order = torch.empty(n, dtype=torch.int32, device=idx.device)
    inverse = torch.empty(n, dtype=torch.int32, device=idx.device)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device=idx.device)
    nb = C.c_size_t()
    check(lib().tf_moe_route_sort_workspace_size(T, K, experts, C.byref(nb)))
    ws = _ws(nb.value, idx.device)
    check(lib().tf_moe_route_sort(_ptr(idx), T, K, experts, _ptr(order), _ptr(inverse), _ptr(offsets),
                                  _ptr(ws), nb.value, _stream()))
    return order, inverse, offsets


def moe_combine(y_sorted: Tensor, inverse: Tensor, gates: Tensor, residual: Tensor) -> Tensor:
    """Top-k combine + residual (MLXNativeGraniteMoEPrefill.h:688-695): rows of
    y_sorted are in route-sort order, inverse maps each route t*k+j to its row."""
    _cuda(y_sorted, inverse, gates, residual)
    T, K = gates.shape
    H = residual.shape[-1]
    if y_sorted.shape != (T * K, H) or inverse.numel() != T * K or residual.shape != (T, H):
        raise ValueError("moe_combine: shape mismatch")
    if not (y_sorted.dtype == gates.dtype == residual.dtype):
        raise ValueError("moe_combine: y, gates and residual share the activation dtype")
    out = torch.empty_like(residual)
    check(lib().tf_moe_combine(_ptr(y_sorted.contiguous()), _ptr(inverse.to(torch.int32).contiguous()),
                               _ptr(gates.contiguous()), _ptr(residual.contiguous()), T, K, H,
                               _act(residual), _ptr(out), _stream()))
    return out


def moe_args(x, residual, out, router, gate, up, down, top_k, logits=None, indices=None, gates=None):
    H = x.shape[-1]
    T = x.numel() // H
    g = affine_desc(*gate)
    a = MoeArgs()
    a.x, a.residual, a.out = x.data_ptr(), residual.data_ptr(), out.data_ptr()
    a.tokens, a.hidden, a.intermediate = T, H, g.out_features
    a.experts, a.top_k, a.act = g.experts, top_k, _act(x)
    a.router = router_desc(router)
    a.gate_proj, a.up_proj, a.down_proj = g, affine_desc(*up), affine_desc(*down)
    a.logits = logits.data_ptr() if logits is not None else None
    a.indices = indices.data_ptr() if indices is not None else None
    a.gates = gates.data_ptr() if gates is not None else None
    return a


def moe(x: Tensor, residual: Tensor, router, gate, up, down, top_k: int, return_aux=False):
    """One OLMoE sparse-MoE block (``moe()``, MLXNativeGraniteMoEPrefill.h:627-702):
    residual + sum_k gate_k * down(silu(gate(x)) * up(x))."""
    _cuda(x, residual)
    if x.shape != residual.shape or x.dtype != residual.dtype:
        raise ValueError("moe: x and residual must match")
    x = x.contiguous()
    residual = residual.contiguous()
    H = x.shape[-1]
    T = x.numel() // H
    E = gate[0].shape[0]
    out = torch.empty_like(x)
    logits = torch.empty((T, E), dtype=x.dtype, device=x.device) if return_aux else None
    idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device) if return_aux else None
    gates = torch.empty((T, top_k), dtype=x.dtype, device=x.device) if return_aux else None
    a = moe_args(x, residual, out, router, gate, up, down, top_k, logits, idx, gates)
    nb = C.c_size_t()
    check(lib().tf_moe_workspace_size(C.byref(a), C.byref(nb)))
    ws = _ws(nb.value, x.device)
    check(lib().tf_moe_forward(C.byref(a), _ptr(ws), nb.value, _stream()))
    if return_aux:
        return out, dict(logits=logits, indices=idx, gates=gates)
    return out


def expert_gpu(x: Tensor, token_indices: Tensor, expert_ids: Tensor, experts_sorted: bool, gate, up,
               down):
    """The expert hook's ``GPUCallable`` (MLXMoEExpertHook.h:25-32): returns
    (expert-sorted output [N, H], inverse [N])."""
    if (token_indices.ndim != 1 or expert_ids.ndim != 1 or token_indices.shape != expert_ids.shape
            or token_indices.dtype not in (torch.int32,) or expert_ids.dtype not in (torch.int32,)):
        raise ValueError("expert hook route arrays must be parallel integer vectors")
    _cuda(x, token_indices, expert_ids)
    H = x.shape[-1]
    xc = x.contiguous().reshape(-1, H)
    g, u, d = affine_desc(*gate), affine_desc(*up), affine_desc(*down)
    _check_range(expert_ids, g.experts, "expert index out of range")
    _check_range(token_indices, xc.shape[0], "token index out of range")
    n = token_indices.numel()
    out = torch.empty((n, H), dtype=x.dtype, device=x.device)
    inverse = torch.empty(n, dtype=torch.int32, device=x.device)
    nb = C.c_size_t()
    check(lib().tf_moe_expert_workspace_size(n, xc.shape[0], H, g.out_features, g.experts, _act(x),
                                             C.byref(nb)))
    ws = _ws(nb.value, x.device)
    check(lib().tf_moe_expert_gpu(_ptr(xc), xc.shape[0], H, _ptr(token_indices), _ptr(expert_ids), n,
                                  int(experts_sorted), g.out_features, g.experts, C.byref(g), C.byref(u),
                                  C.byref(d), _act(x), _ptr(out), _ptr(inverse), _ptr(ws), nb.value,
                                  _stream()))
    return out, inverse


def expert_gpu_ordered(x: Tensor, token_indices: Tensor, expert_ids: Tensor, gate, up, down,
                       check_ranges: bool = True) -> Tensor:
    """The expert hook's computation with the output rows in the routes' own
    order (row i for route i); no inverse permutation.  check_ranges=False
    skips the host-side index checks (one device-to-host read each) for
    callers whose indices are valid by construction."""
    if (token_indices.ndim != 1 or expert_ids.ndim != 1 or token_indices.shape != expert_ids.shape
            or token_indices.dtype != torch.int32 or expert_ids.dtype != torch.int32):
        raise ValueError("expert hook route arrays must be parallel integer vectors")
    _cuda(x, token_indices, expert_ids)
    H = x.shape[-1]
    xc = x.contiguous().reshape(-1, H)
    g, u, d = affine_desc(*gate), affine_desc(*up), affine_desc(*down)
    if check_ranges:
        _check_range(expert_ids, g.experts, "expert index out of range")
        _check_range(token_indices, xc.shape[0], "token index out of range")
    n = token_indices.numel()
    out = torch.empty((n, H), dtype=x.dtype, device=x.device)
    nb = C.c_size_t()
    check(lib().tf_moe_expert_workspace_size(n, xc.shape[0], H, g.out_features, g.experts, _act(x),
                                             C.byref(nb)))
    ws = _ws(nb.value, x.device)
    check(lib().tf_moe_expert_gpu_ordered(_ptr(xc), xc.shape[0], H, _ptr(token_indices), _ptr(expert_ids), n,
                                          g.out_features, g.experts, C.byref(g), C.byref(u), C.byref(d),
                                          _act(x), _ptr(out), _ptr(ws), nb.value, _stream()))
    return out


def gather_rows(x: Tensor, index: Tensor, div: int = 1) -> Tensor:
    """y[i] = x[index[i] // div] (rows of the activation dtype); index int32
    on the device, in range by the caller's construction."""
    _cuda(x, index)
    if index.dtype != torch.int32 or index.ndim != 1:
        raise ValueError("gather_rows: int32 index vector")
    H = x.shape[-1]
    xc = x.contiguous().reshape(-1, H)
    n = index.numel()
    y = torch.empty((n, H), dtype=x.dtype, device=x.device)
    check(lib().tf_gather_rows(_ptr(xc), xc.shape[0], H, _ptr(index), int(div), n, _act(x), _ptr(y), _stream()))
    return y


def rms_norm(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    """``fast::rms_norm`` as used by the adapter (MLXNativeGraniteMoEPrefill.h:434)."""
    _cuda(x, weight)
    W = x.shape[-1]
    xc = x.contiguous()
    y = torch.empty_like(xc)
    check(lib().tf_rms_norm(_ptr(xc), xc.numel() // W, W, _ptr(weight.contiguous()), eps, _act(x), _ptr(y),
                            _stream()))
    return y


def attention_decode(qkv: Tensor, q_norm: Tensor, k_norm: Tensor, positions: Tensor, k_cache: Tensor,
                     v_cache: Tensor, eps: float, rope_theta: float, scale: float | None = None,
                     max_length: int | None = None) -> Tensor:
    """T1 attention for a batch of requests (MLXNativeGraniteMoEPrefill.h:446-483):
    q/k full-width RMSNorm, RoPE, KV append at positions[b], SDPA.
    k_cache/v_cache: float16 [batch, heads, capacity, head_dim] (updated)."""
    _cuda(qkv, q_norm, k_norm, positions, k_cache, v_cache)
    B, heads, cap, D = k_cache.shape
    if qkv.shape != (B, 3 * heads * D) or v_cache.shape != k_cache.shape:
        raise ValueError("attention: qkv/cache geometry differs")
    if k_cache.dtype != torch.float16 or v_cache.dtype != torch.float16:
        raise ValueError("ordered full-history FP16 KV required")
    scale = D ** -0.5 if scale is None else scale
    max_length = cap if max_length is None else max_length
    pos = positions.to(torch.int32).contiguous()
    out = torch.empty((B, heads * D), dtype=qkv.dtype, device=qkv.device)
    nb = C.c_size_t()
    check(lib().tf_attention_decode_workspace_size(B, heads, cap, C.byref(nb)))
    ws = _ws(nb.value, qkv.device)
    check(lib().tf_attention_decode(_ptr(qkv.contiguous()), B, heads, D, _ptr(q_norm), _ptr(k_norm), eps,
                                    rope_theta, _ptr(pos), max_length, _ptr(k_cache), _ptr(v_cache), cap,
                                    scale, _act(qkv), _ptr(out), _ptr(ws), nb.value, _stream()))
    return out


def set_qmm_path(path: int):
    """0 = automatic, 1 = CUDA-core GEMV only, 2 = tensor cores when eligible."""
    check(lib().tf_set_qmm_path(int(path)))


def device_error(clear: bool = True) -> int:
    """First error code recorded by a device-side bounded wait (0 = none)."""
    return lib().tf_device_error(int(clear))
