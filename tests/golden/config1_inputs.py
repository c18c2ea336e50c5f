"""Seeded inputs of BASELINE config 1 at its full geometry.

One OLMoE sparse-MoE block: 32 bf16 tokens N(0, 1), hidden 2048, 64 experts,
top-8, expert intermediate 1024, expert weights N(0, 0.02) rounded to bf16
and MLX-affine 4-bit / group-64 quantized, dense bf16 router N(0, 0.02).

The packed weights (about 226 MB) are too large to commit, so the golden
generator (``make_golden.py``, which runs the reference's own operators on
them) and the GPU parity test both regenerate them from the same seed with
numpy's PCG64 stream; the fixture ``config1_full.npz`` records a SHA-256 of
every generated array so the test can prove it rebuilt the very bytes the
reference consumed.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402

SEED = 20260101
T, H, I, E, K = 32, 2048, 1024, 64, 8
ACT = "bf16"
NAMES = ("gate", "up", "down")


def _weights(rng, shape):
    return oracle.round_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))


def _experts(rng, shape):
    """Quantized [E, out, in] weights, drawn and quantized one expert at a
    time (the same stream as one draw of the whole array, in small arrays)."""
    parts = [oracle.affine_quantize(_weights(rng, shape[1:])) for _ in range(shape[0])]
    return tuple(np.stack([p[i] for p in parts]) for i in range(3))


def generate():
    """(x, residual, experts {name: (q, s, b)}, router_w): act values as float32."""
    rng = np.random.default_rng(SEED)
    x = oracle.to_act(rng.standard_normal((T, H), dtype=np.float32), ACT)
    residual = oracle.to_act(rng.standard_normal((T, H), dtype=np.float32), ACT)
    shapes = {"gate": (E, I, H), "up": (E, I, H), "down": (E, H, I)}
    experts = {n: _experts(rng, shapes[n]) for n in NAMES}
    router_w = oracle.to_act(_weights(rng, (E, H)), ACT)
    return x, residual, experts, router_w


def digest(x, residual, experts, router_w):
    """SHA-256 over every input array's bytes in a fixed order."""
    h = hashlib.sha256()
    h.update(oracle.act_to_bits(x, ACT).tobytes())
    h.update(oracle.act_to_bits(residual, ACT).tobytes())
    for n in NAMES:
        for a in experts[n]:
            h.update(np.ascontiguousarray(a).tobytes())
    h.update(oracle.act_to_bits(router_w, ACT).tobytes())
    return h.hexdigest()
