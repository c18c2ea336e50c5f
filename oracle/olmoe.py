"""numpy restatement of the OLMoE sparse-MoE forward (CPU oracle; test-only).

Every function names the reference lines it restates.  Paths are relative to
the TriFuse project root.

Numeric contract shared with the CUDA kernels
---------------------------------------------
Activations ("act") are float16 or bfloat16; scales/biases, norm weights and
the KV cache are float16; packed weights are uint32 holding eight 4-bit codes,
code j of a word at bits 4j (``native_affine_ops.py:29-36``).  Inside this
module every act tensor is a float32 array whose values are exactly
representable in the act dtype (``to_act`` rounds to nearest even).

Operations are split into two classes.

* Bit-exact (the CUDA kernels reproduce these results bit for bit):
  RMSNorm (``rms_norm``), the router GEMV (``router_logits_*``), the fp32
  softmax with act-dtype rounding (``olmoe_softmax``), the stable top-k rank
  (``olmoe_topk``), the route sort (``route_sort``) and the weighted combine
  (``combine``).  Their fp32 reduction orders are fixed here and in the
  kernels; the orders are written out in each docstring.
* Tolerance-level (fp32 accumulation in an unspecified order, compared with
  max-abs 2e-2 / mean-relative 5e-3): the affine QMM / gather_qmm products,
  SwiGLU (uses ``exp``), RoPE (uses ``cos``/``sin``) and attention.
"""
from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_POOL = None


def _pmap(fn, items):
    """Map over host threads (numpy releases the GIL inside its kernels)."""
    global _POOL
    items = list(items)
    if len(items) <= 1:
        return [fn(i) for i in items]
    if _POOL is None:
        _POOL = ThreadPoolExecutor(max_workers=os.cpu_count() or 1)
    return list(_POOL.map(fn, items))

F16 = "f16"
BF16 = "bf16"
ACT_DTYPES = (F16, BF16)
GROUP = 64
BITS = 4

# ----------------------------------------------------------------------------
# dtype helpers


def round_bf16(x):
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)).astype(np.uint32)
    out = r.view(np.float32)
    return np.where(np.isnan(x), np.float32(np.nan), out).astype(np.float32)


def round_f16(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def to_act(x, act):
    """Round an fp32 array to the activation dtype (values kept as float32)."""
    if act == F16:
        return round_f16(x)
    if act == BF16:
        return round_bf16(x)
    raise ValueError(f"unknown activation dtype {act!r}")


def act_to_bits(x, act):
    """float32 array holding act values -> uint16 storage bits."""
    x = np.asarray(x, dtype=np.float32)
    if act == F16:
        return x.astype(np.float16).view(np.uint16)
    return (round_bf16(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def bits_to_act(bits, act):
    """uint16 storage bits -> float32 array."""
    bits = np.asarray(bits, dtype=np.uint16)
    if act == F16:
        return bits.view(np.float16).astype(np.float32)
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32(x):
    return np.asarray(x, dtype=np.float32)


# ----------------------------------------------------------------------------
# MLX affine 4-bit packing


def unpack_codes(q, bits=BITS):
    """uint32 [..., in/8] -> int codes [..., in]; code j of a word at bits 4j.

    Restates ``native_affine_ops.py:32-34`` (shift/mask unpack)."""
    q = np.asarray(q, dtype=np.uint32)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * np.uint32(bits))
    codes = (q[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return codes.reshape(*q.shape[:-1], q.shape[-1] * per)


def pack_codes(codes, bits=BITS):
    """int codes [..., in] -> uint32 [..., in/8] (inverse of ``unpack_codes``)."""
    codes = np.asarray(codes, dtype=np.uint32)
    per = 32 // bits
    c = codes.reshape(*codes.shape[:-1], codes.shape[-1] // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * np.uint32(bits))
    return np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32)


def affine_quantize(w, group=GROUP, bits=BITS):
    """Min/max affine quantizer: fp32 weights [..., in] -> (q u32, s f16, b f16).

    Written from the affine formula ``w ~= code * scale + bias`` with 2^bits
    levels per group (``native_affine_ops.py:29-36`` is the matching
    dequantizer).  scale = (max - min) / (2^bits - 1) and bias = min, both
    stored as float16; codes round (w - b16) / s16 to nearest even and clamp.
    MLX's own quantizer is not part of the reference tree; parity does not
    depend on it because oracle and kernels consume identical Q/S/B bytes."""
    w = f32(w)
    shape = w.shape
    g = w.reshape(*shape[:-1], shape[-1] // group, group)
    lo = g.min(axis=-1)
    hi = g.max(axis=-1)
    levels = np.float32((1 << bits) - 1)
    scale = ((hi - lo) / levels).astype(np.float32)
    scale = np.where(scale > np.float32(1e-7), scale, np.float32(1e-7)).astype(np.float32)
    s16 = scale.astype(np.float16)
    b16 = lo.astype(np.float16)
    codes = np.rint((g - b16.astype(np.float32)[..., None]) / s16.astype(np.float32)[..., None])
    codes = np.clip(codes, 0, (1 << bits) - 1).astype(np.uint32).reshape(shape)
    return pack_codes(codes, bits), s16, b16


def dequantize(q, scales, biases, group=GROUP, bits=BITS):
    """fp16-rounded dequantized weights (as float32).

    Restates ``native_affine_ops.py:29-36``: ``codes * scales + biases`` in
    fp32 (separate multiply and add), then cast to the scales dtype (f16)."""
    codes = unpack_codes(q, bits).astype(np.float32)
    s = np.repeat(f32(np.asarray(scales, np.float16)), group, axis=-1)
    b = np.repeat(f32(np.asarray(biases, np.float16)), group, axis=-1)
    return round_f16((codes * s).astype(np.float32) + b)


# ----------------------------------------------------------------------------
# affine QMM family (tolerance-level)


def affine_qmm(x, q, scales, biases, act):
    """y = act(x @ dequant(W)^T), fp32 accumulation.

    Restates ``native_affine_ops.py:39-45`` (``native_affine_qmm``) and the
    adapter's ``linear`` (``MLXNativeGraniteMoEPrefill.h:539-541``)."""
    x = f32(x)
    rows = q.shape[0]
    step = max(256, -(-rows // (os.cpu_count() or 1)))
    y = np.empty((*x.shape[:-1], rows), np.float32)

    def part(r0):
        w = dequantize(q[r0:r0 + step], scales[r0:r0 + step], biases[r0:r0 + step])
        y[..., r0:r0 + step] = x @ w.T

    _pmap(part, range(0, rows, step))
    return to_act(y, act)


def gather_qmm(x_rows, q, scales, biases, indices, act):
    """Row n uses expert ``indices[n]``: y[n] = act(x_rows[n] @ W[indices[n]]^T).

    Restates ``native_affine_ops.py:55-63`` for the flattened (sorted) call
    form ``x[N,1,in] x idx[N]`` of ``MLXNativeGraniteMoEPrefill.h:542-550``.
    Each used expert is dequantized once and multiplied over its rows."""
    x_rows = f32(x_rows)
    indices = np.asarray(indices).astype(np.int64)
    out_dim = q.shape[-2]
    y = np.zeros((x_rows.shape[0], out_dim), dtype=np.float32)

    def one(e):
        sel = np.nonzero(indices == e)[0]
        w = dequantize(q[e], scales[e], biases[e])
        y[sel] = x_rows[sel] @ w.T

    _pmap(one, np.unique(indices))
    return to_act(y, act)


def affine_embedding(ids, q, scales, biases, act):
    """Selected-row dequantization, ``native_affine_ops.py:77-87``; the
    adapter's form is ``MLXNativeGraniteMoEPrefill.h:394-396``."""
    ids = np.asarray(ids).astype(np.int64).reshape(-1)
    w = dequantize(q[ids], scales[ids], biases[ids])
    return to_act(w, act)


# ----------------------------------------------------------------------------
# bit-exact reductions


def _butterfly32(v):
    """xor-shuffle tree over the last axis (32 lanes): offsets 16, 8, 4, 2, 1."""
    lanes = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        v = (v + v[..., lanes ^ off]).astype(np.float32)
    return v[..., 0]


def row_sumsq(x):
    """Sum of squares over the last axis in the kernels' fixed order.

    Order: the row is split into 8-element chunks, chunk t owned by thread t
    (t = 0 .. H/8-1); each thread accumulates ``acc = acc + x*x`` (fp32
    multiply, then fp32 add, starting from 0) over its chunk; each warp of 32
    threads combines with the xor butterfly (16, 8, 4, 2, 1); the warp totals
    are then added left to right.  Requires H % 256 == 0."""
    x = f32(x)
    H = x.shape[-1]
    if H % 256:
        raise ValueError("row reduction requires width % 256 == 0")
    c = x.reshape(*x.shape[:-1], H // 8, 8)
    acc = np.zeros(c.shape[:-1], np.float32)
    for i in range(8):
        acc = (acc + (c[..., i] * c[..., i]).astype(np.float32)).astype(np.float32)
    warps = acc.reshape(*x.shape[:-1], H // 256, 32)
    wt = _butterfly32(warps)
    total = wt[..., 0]
    for w in range(1, H // 256):
        total = (total + wt[..., w]).astype(np.float32)
    return total


def rms_norm(x, weight, eps, act):
    """act((x * r) * w) with r = 1 / sqrt(sumsq / H + eps), all fp32 IEEE.

    Restates ``fast::rms_norm`` at ``MLXNativeGraniteMoEPrefill.h:434, 451-452,
    486, 490`` (``F.rms_norm`` in ``export_native_olmoe_target.py:178``)."""
    x = f32(x)
    H = x.shape[-1]
    ss = row_sumsq(x)
    mean = (ss / np.float32(H)).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt((mean + np.float32(eps)).astype(np.float32))).astype(np.float32)
    w = f32(np.asarray(weight, np.float16))
    y = ((x * r[..., None]).astype(np.float32) * w).astype(np.float32)
    return to_act(y, act)


def _router_dot(x, w):
    """Dot products of rows of x [T, H] with rows of w [E, H] in the router's
    fixed order: lane l (0..31) owns the 8-element chunks c = l + 32 j,
    accumulates ``acc = acc + x*w`` (fp32 multiply then add, from 0) over
    j = 0 .. H/256-1 and i = 0..7, then the lanes reduce with the xor
    butterfly.  Returns fp32 [T, E]."""
    x = f32(x)
    w = f32(w)
    T, H = x.shape
    E = w.shape[0]
    if H % 256:
        raise ValueError("router width must be a multiple of 256")
    J = H // 256
    xc = x.reshape(T, J, 32, 8)  # [T, j, lane, i]; chunk c = j*32 + lane
    wc = w.reshape(E, J, 32, 8)
    acc = np.zeros((T, E, 32), np.float32)
    for j in range(J):
        for i in range(8):
            prod = (xc[:, None, j, :, i] * wc[None, :, j, :, i]).astype(np.float32)
            acc = (acc + prod).astype(np.float32)
    return _butterfly32(acc)


def router_logits_dense(x, w, act):
    """Router GEMV with a dense act-dtype weight [E, H] (BASELINE config 1's
    bf16 router).  Restates ``MoE.gate`` at ``export_native_olmoe_target.py:201``
    with the fixed order of ``_router_dot``; result rounded to act."""
    return to_act(_router_dot(x, w), act)


def router_logits_affine(x, q, scales, biases, act):
    """Router GEMV with the model's 4-bit router (``mlp.gate``, restating
    ``MLXNativeGraniteMoEPrefill.h:631`` / ``native_affine_ops.py:39-45``):
    weights are dequantized to f16 exactly as ``dequantize`` does, then dotted
    in the fixed order of ``_router_dot``; result rounded to act."""
    return to_act(_router_dot(x, dequantize(q, scales, biases)), act)


def olmoe_softmax(logits, act):
    """Full-expert fp32 softmax, result rounded to act.

    Restates ``native_affine_ops.py:128-131`` and the router kernel's softmax
    stage (``MLXOLMoERouter.h:26-62``).  Fixed arithmetic: m = max over the
    row ignoring NaN; e_i = fp32(exp_f64(fp32(l_i - m))); the sum puts expert
    i on lane i % 32, each lane adds its experts in increasing order from 0,
    then the xor butterfly; p_i = e_i / sum (fp32 IEEE division).  A NaN logit
    makes the whole row NaN, as in the reference."""
    x = f32(logits)
    T, E = x.shape
    if E > 64:
        raise ValueError("router supports at most 64 experts")
    with np.errstate(invalid="ignore", over="ignore"):
        masked = np.where(np.isnan(x), np.float32(-np.inf), x)
        m = masked.max(axis=-1)
        d = (x - m[:, None]).astype(np.float32)
        e = np.exp(d.astype(np.float64)).astype(np.float32)
        lanes = np.zeros((T, 32), np.float32)
        for i in range(E):
            lanes[:, i % 32] = (lanes[:, i % 32] + e[:, i]).astype(np.float32)
        s = _butterfly32(lanes)
        p = (e / s[:, None]).astype(np.float32)
    return to_act(p, act)


def olmoe_topk(probs, k):
    """Stable descending rank, NaN last, ties to the lower expert id.

    Restates ``MLXOLMoERouter.h:65-83`` (rank after act rounding) which equals
    ``torch.argsort(-p, stable=True)[..., :k]`` (``native_affine_ops.py:141-146``).
    Returns int32 [T, k] in rank order."""
    p = f32(probs)
    T, E = p.shape
    out = np.zeros((T, k), np.int32)
    for t in range(T):
        row = p[t]
        nan = np.isnan(row)
        key = np.where(nan, np.inf, -row.astype(np.float64))
        order = np.lexsort((np.arange(E), nan, key))
        out[t] = order[:k]
    return out


def olmoe_route(logits, k, act):
    """(indices int32 [T,k], gates act [T,k]): softmax, rank, take.

    Restates ``olmoe_route`` (``MLXOLMoERouter.h:86-120``) and the OLMoE
    branch of ``route`` (``MLXNativeGraniteMoEPrefill.h:596-602``).  No top-k
    renormalisation (``export_native_olmoe_target.py:30``)."""
    p = olmoe_softmax(logits, act)
    idx = olmoe_topk(p, k)
    gates = np.take_along_axis(p, idx.astype(np.int64), axis=-1)
    return idx, gates


def greedy_token(logits):
    """Greedy next token per row of fp32 logits: argmax (first occurrence on
    ties) when every logit of the row is finite, else -1.

    Restates the greedy submission's ``where(all(isfinite(logits)),
    argmax(logits), -1)`` (``patches/executorch.patch:1350-1353``)."""
    lg = np.asarray(logits, np.float32)
    lg2 = lg.reshape(-1, lg.shape[-1])
    ok = np.isfinite(lg2).all(axis=1)
    idx = np.argmax(np.where(np.isfinite(lg2), lg2, -np.inf), axis=1)
    return np.where(ok, idx, -1).astype(np.int64).reshape(lg.shape[:-1])


def route_sort(indices, num_experts):
    """Stable grouping of the flat routes by expert.

    Restates ``MLXNativeGraniteMoEPrefill.h:666-684`` (and the export's
    ``export_native_olmoe_target.py:204-212``): ``order`` is a stable argsort
    of the flat [T*K] expert ids (ties keep flat order), ``inverse`` its
    inverse permutation; ``offsets[e]`` is the first sorted slot of expert e
    (E+1 entries).  The sorted input row of slot j is ``order[j] // K``."""
    flat = np.asarray(indices).reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable").astype(np.int32)
    inverse = np.empty_like(order)
    inverse[order] = np.arange(order.size, dtype=np.int32)
    counts = np.bincount(flat, minlength=num_experts)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return order, inverse, offsets


# ----------------------------------------------------------------------------
# SwiGLU, combine and the MoE block


def silu(x):
    x = f32(x)
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x).astype(np.float32))).astype(np.float32)


def swiglu(gate, up, act):
    """h = act(act(silu(gate)) * up).

    Restates ``F.silu(gate) * up`` (``export_native_olmoe_target.py:215``);
    the adapter's compiled form is ``MLXNativeGraniteMoEPrefill.h:551-565``."""
    return to_act(to_act(silu(gate), act) * f32(up), act)


def combine(expert_out, gates, residual, act):
    """out = act(residual + act(sum_k act(y_k * g_k))); fp32 sum in k order.

    Restates ``MLXNativeGraniteMoEPrefill.h:688-695`` (multiply and sum in the
    activation dtype) / ``export_native_olmoe_target.py:218`` plus the layer's
    residual add (``:227``)."""
    y = f32(expert_out)  # [T, K, H]
    g = f32(gates)[..., None]
    prod = to_act((y * g).astype(np.float32), act)
    acc = prod[:, 0].copy()
    for k in range(1, prod.shape[1]):
        acc = (acc + prod[:, k]).astype(np.float32)
    red = to_act(acc, act)
    return to_act((f32(residual) + red).astype(np.float32), act)


def moe_block(x, residual, router, experts, top_k, act, forced_indices=None):
    """One OLMoE sparse-MoE block; returns (out, aux).

    Restates ``NativeGraniteMoEPrefill::moe`` (``MLXNativeGraniteMoEPrefill.h:
    627-702``) = ``MoE.forward`` + residual (``export_native_olmoe_target.py:
    200-218, 227``).

    ``router`` is ``("dense", w_act[E,H])`` or ``("affine", q, s, b)``;
    ``experts`` is a dict with ``gate``/``up``/``down`` -> (q, s, b) stacked
    [E, ...]."""
    x = f32(x)
    T, H = x.shape
    if router[0] == "dense":
        logits = router_logits_dense(x, router[1], act)
    else:
        logits = router_logits_affine(x, *router[1:], act)
    idx, gates = olmoe_route(logits, top_k, act)
    own = idx
    if forced_indices is not None:
        # Follow a given routing (test harness: the device's choices); the
        # gates are this block's own probabilities at those experts.
        idx = np.asarray(forced_indices, np.int64).reshape(T, top_k)
        gates = np.take_along_axis(olmoe_softmax(logits, act), idx, -1)
    E = experts["gate"][0].shape[0]
    order, inverse, offsets = route_sort(idx, E)
    flat = idx.reshape(-1)
    sel = flat[order]
    rows = x[order // top_k]
    gq, gs, gb = experts["gate"]
    uq, us, ub = experts["up"]
    dq, ds, db = experts["down"]
    up = gather_qmm(rows, uq, us, ub, sel, act)
    gate = gather_qmm(rows, gq, gs, gb, sel, act)
    h = swiglu(gate, up, act)
    y_sorted = gather_qmm(h, dq, ds, db, sel, act)
    y = y_sorted[inverse].reshape(T, top_k, -1)
    out = combine(y, gates, residual, act)
    aux = dict(logits=logits, indices=idx, gates=gates, order=order,
               inverse=inverse, offsets=offsets, h_sorted=h, y_sorted=y_sorted, own_indices=own)
    return out, aux


# ----------------------------------------------------------------------------
# attention (tolerance-level)


def rope_inv_freq(head_dim, theta):
    """fp32 inverse frequencies theta^(-2i/D), i < D/2, computed in float64."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    return (float(theta) ** (-2.0 * i / head_dim)).astype(np.float32)


def rope(x, positions, theta, act):
    """Non-traditional (half-split) RoPE on [..., T, heads, D] act values.

    Restates ``fast::rope(x, D, traditional=false, base, scale=1, offset)``
    (``MLXNativeGraniteMoEPrefill.h:457-458``): for i < D/2 the pair
    (x_i, x_{i+D/2}) rotates by angle = fp32(pos) * inv_freq_i (fp32)."""
    x = f32(x)
    D = x.shape[-1]
    inv = rope_inv_freq(D, theta)
    pos = f32(np.asarray(positions, np.float32))
    ang = (pos[..., None] * inv).astype(np.float32)  # [..., T, D/2]
    c = np.cos(ang.astype(np.float64)).astype(np.float32)[..., None, :]
    s = np.sin(ang.astype(np.float64)).astype(np.float32)[..., None, :]
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    o1 = (x1 * c - x2 * s).astype(np.float32)
    o2 = (x1 * s + x2 * c).astype(np.float32)
    return to_act(np.concatenate([o1, o2], axis=-1), act)


def sdpa(q, K, V, scale, act, causal_offset=None, fast=False):
    """softmax(q K^T * scale) V, output rounded to act.  float64 math by
    default; ``fast`` uses float32 BLAS (the timed CPU-baseline variant).

    q [Tq, Hh, D]; K, V [Hh, L, D] (float16 cache values).  With
    ``causal_offset`` = absolute position of q row 0, key j is visible to row
    t iff j <= causal_offset + t.  Restates
    ``fast::scaled_dot_product_attention`` (``MLXNativeGraniteMoEPrefill.h:
    480-481``)."""
    q = f32(q)
    K = f32(K)
    V = f32(V)
    Tq, Hh, D = q.shape
    L = K.shape[1]
    if fast:
        s = np.matmul(q.transpose(1, 0, 2), K.transpose(0, 2, 1)) * np.float32(scale)  # [Hh, Tq, L]
        if causal_offset is not None:
            t = np.arange(Tq)[:, None]
            j = np.arange(L)[None, :]
            s = np.where(j <= causal_offset + t, s, -np.inf)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        o = np.matmul(p, V).transpose(1, 0, 2)
        return to_act(o.astype(np.float32), act)
    s = np.einsum("thd,hld->htl", q.astype(np.float64), K.astype(np.float64)) * scale
    if causal_offset is not None:
        t = np.arange(Tq)[:, None]
        j = np.arange(L)[None, :]
        s = np.where(j <= causal_offset + t, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    o = np.einsum("htl,hld->thd", p, V.astype(np.float64))
    return to_act(o.astype(np.float32), act)


# ----------------------------------------------------------------------------
# model


class OLMoEConfig:
    """Geometry of ``NativeModelConfig`` (``resident_prefill.h:18-42``) for
    OLMoE (``export_native_olmoe_target.py:27-63``)."""

    def __init__(self, layers=16, hidden=2048, heads=16, head_dim=128,
                 intermediate=1024, vocab=50304, experts=64, top_k=8,
                 rms_eps=1e-5, rope_theta=10000.0, capacity=4096, act=F16):
        self.layers = layers
        self.hidden = hidden
        self.heads = heads
        self.head_dim = head_dim
        self.intermediate = intermediate
        self.vocab = vocab
        self.experts = experts
        self.top_k = top_k
        self.rms_eps = rms_eps
        self.rope_theta = rope_theta
        self.capacity = capacity
        self.act = act

    @property
    def attn_scale(self):
        return np.float32(self.head_dim ** -0.5)


def attention_block(h, layer, cfg, k_cache, v_cache, positions, fast=False):
    """Attention half of one layer for one request (decode or prefill chunk).

    h: act [T, H]; k_cache/v_cache: float32 holding f16 values [Hh, cap, D],
    updated in place at ``positions`` (contiguous from ``start``).  Returns
    act h + o_proj(attn).  Restates ``MLXNativeGraniteMoEPrefill.h:434-485``:
    input RMSNorm, q/k/v QMM, full-width Q/K RMSNorm before the head split,
    RoPE at the absolute positions, KV append, SDPA (causal for T > 1),
    o-proj, residual add."""
    act = cfg.act
    T = h.shape[0]
    D = cfg.head_dim
    Hh = cfg.heads
    start = int(positions[0])
    xn = rms_norm(h, layer["input_norm"], cfg.rms_eps, act)
    q = affine_qmm(xn, *layer["q"], act)
    k = affine_qmm(xn, *layer["k"], act)
    v = affine_qmm(xn, *layer["v"], act)
    q = rms_norm(q, layer["q_norm"], cfg.rms_eps, act)
    k = rms_norm(k, layer["k_norm"], cfg.rms_eps, act)
    q = rope(q.reshape(T, Hh, D), positions, cfg.rope_theta, act)
    k = rope(k.reshape(T, Hh, D), positions, cfg.rope_theta, act)
    k_cache[:, start:start + T] = round_f16(k.transpose(1, 0, 2))
    v_cache[:, start:start + T] = round_f16(v.reshape(T, Hh, D).transpose(1, 0, 2))
    L = start + T
    o = sdpa(q, k_cache[:, :L], v_cache[:, :L], cfg.attn_scale, act,
             causal_offset=start if T > 1 else None, fast=fast)
    proj = affine_qmm(o.reshape(T, Hh * D), *layer["o"], act)
    return to_act(f32(h) + proj, act)


def decode_layer_batched(h, layer, cfg, k_caches, v_caches, positions, fast=False, forced=None, aux_out=None):
    """One layer of batched decode: request b has one new token at absolute
    position positions[b] and its own cache k_caches[b] / v_caches[b]
    ([Hh, cap, D], f16 values, updated in place).  Projections and the MoE
    block run over the batch; attention runs per request.  Same math as
    ``layer_forward`` applied to each request (MLXNativeGraniteMoEPrefill.h:
    433-487 with T = 1)."""
    act = cfg.act
    B = h.shape[0]
    D, Hh = cfg.head_dim, cfg.heads
    W = D * Hh
    xn = rms_norm(h, layer["input_norm"], cfg.rms_eps, act)
    q = affine_qmm(xn, *layer["q"], act)
    k = affine_qmm(xn, *layer["k"], act)
    v = affine_qmm(xn, *layer["v"], act)
    q = rms_norm(q, layer["q_norm"], cfg.rms_eps, act)
    k = rms_norm(k, layer["k_norm"], cfg.rms_eps, act)
    o = np.zeros((B, W), np.float32)
    for b in range(B):
        p = int(positions[b])
        qb = rope(q[b].reshape(1, Hh, D), [p], cfg.rope_theta, act)
        kb = rope(k[b].reshape(1, Hh, D), [p], cfg.rope_theta, act)
        k_caches[b][:, p] = round_f16(kb[0])
        v_caches[b][:, p] = round_f16(v[b].reshape(Hh, D))
        o[b] = sdpa(qb, k_caches[b][:, :p + 1], v_caches[b][:, :p + 1], cfg.attn_scale, act,
                    fast=fast).reshape(-1)
    h = to_act(f32(h) + affine_qmm(o, *layer["o"], act), act)
    post = rms_norm(h, layer["post_norm"], cfg.rms_eps, act)
    out, aux = moe_block(post, h, ("affine",) + tuple(layer["router"]), layer["experts"], cfg.top_k, act,
                         forced_indices=forced)
    if aux_out is not None:
        aux_out.append(aux)
    return out


def layer_forward(h, layer, cfg, k_cache, v_cache, positions, fast=False, forced=None, aux_out=None,
                  last_row_only=False):
    """One decoder layer: attention block, post-attention RMSNorm, MoE block.

    Restates ``MLXNativeGraniteMoEPrefill.h:433-487`` / ``Layer.forward``
    (``export_native_olmoe_target.py:225-227``).  ``last_row_only`` keeps
    the MoE half for the last row (the reference's last layer with T > 1,
    ``MLXNativeGraniteMoEPrefill.h:440-442, 471``; every row still writes
    its K/V).  ``forced`` routes the MoE block's rows to given experts."""
    h = attention_block(h, layer, cfg, k_cache, v_cache, positions, fast=fast)
    if last_row_only:
        h = h[-1:]
    post = rms_norm(h, layer["post_norm"], cfg.rms_eps, cfg.act)
    out, aux = moe_block(post, h, ("affine",) + tuple(layer["router"]), layer["experts"],
                         cfg.top_k, cfg.act, forced_indices=forced)
    if aux_out is not None:
        aux_out.append(aux)
    return out


def model_forward(ids, weights, cfg, k_caches, v_caches, start, fast=False, forced=None, aux_out=None):
    """Embedding -> layers -> final RMSNorm on the last row -> lm_head (fp32).

    Restates ``NativeGraniteMoEPrefill::run`` (``MLXNativeGraniteMoEPrefill.h:
    347-493``) for one request, without the last-query-only shortcut (which
    changes no returned value).  Returns fp32 logits [V] (act-rounded).
    ``fast`` selects the float32-BLAS attention (see ``sdpa``) for long
    sequences.  ``forced`` (a list per layer) routes each layer's MoE rows to
    given experts; the last layer's entry then holds the last row's experts
    only and that layer runs its MoE half for the last row, as the reference
    does.  ``aux_out`` collects each layer's MoE aux (own routing included)."""
    ids = np.asarray(ids).reshape(-1)
    T = ids.size
    positions = np.arange(start, start + T)
    h = affine_embedding(ids, *weights["embed"], cfg.act)
    n = len(weights["layers"])
    for i, layer in enumerate(weights["layers"]):
        h = layer_forward(h, layer, cfg, k_caches[i], v_caches[i], positions, fast=fast,
                          forced=None if forced is None else forced[i], aux_out=aux_out,
                          last_row_only=forced is not None and i == n - 1 and T > 1)
    last = rms_norm(h[-1:], weights["final_norm"], cfg.rms_eps, cfg.act)
    return affine_qmm(last, *weights["lm_head"], cfg.act)[0]
