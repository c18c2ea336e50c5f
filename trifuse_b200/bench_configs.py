"""Measurements of the BASELINE configurations other than the headline decode
(which bench.py times): one JSON line per configuration.

    python -m trifuse_b200.bench_configs [--config 1 3 4 5] [--iters N]
    torchrun --nproc-per-node N -m trifuse_b200.bench_configs --config 5

Each number is device time from CUDA events on the launching stream, after
warm-up, with inputs larger than L2 or a buffer larger than L2 written
between iterations (stated per line).  Work is compared with the algorithmic
bytes (HBM-bound configs) or flops (prefill) and the peaks measured on this
pool (MEASURED_PEAKS.json at the repository root), else the nominal figures.

Inputs follow the synthetic definitions of the benchmark: expert weights
N(0, 0.02) in bf16 quantized to MLX affine 4-bit g64, router N(0, 0.02),
activations N(0, 1), fp16 KV N(0, 1), token ids uniform, and for config 5 a
per-expert router bias N(0, 1.5) (here folded into a dense bf16 router by a
constant input column, see _skewed_router).
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
H, I, E, K, V, D, HEADS = 2048, 1024, 64, 8, 50304, 128, 16
EXPERT_PROJ_BYTES = I * H // 2 + I * (H // 64) * 4


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def timed(fn, iters, flush=None):
    """Mean ms of fn over iters launches (after 3 warm-up calls), with an
    optional L2 flush (outside the timed events) before each."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    s = torch.cuda.current_stream()
    for _ in range(iters):
        if flush is not None:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        fn()
        b.record(s)
        b.synchronize()
        total += a.elapsed_time(b)
    return total / iters


def l2_flusher(device):
    junk = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    return lambda: junk.fill_(1)


def experts(gen, device, n_experts=E):
    from .quant import random_affine
    return {n: random_affine(shape, gen, device) for n, shape in
            (("gate", (n_experts, I, H)), ("up", (n_experts, I, H)), ("down", (n_experts, H, I)))}


def config1(args, dev):
    """One MoE block: T=32 bf16 tokens (or --tokens), dense bf16 router, 64 experts top-8."""
    from . import ops
    g = torch.Generator(device=dev)
    g.manual_seed(20260101)
    ex = experts(g, dev)
    router = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    T = args.tokens
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    res = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    _, aux = ops.moe(x, res, router, ex["gate"], ex["up"], ex["down"], K, return_aux=True)
    unique = int(torch.unique(aux["indices"]).numel())
    ms = timed(lambda: ops.moe(x, res, router, ex["gate"], ex["up"], ex["down"], K), args.iters,
               l2_flusher(dev))
    nbytes = unique * 3 * EXPERT_PROJ_BYTES + T * H * 2 * 2 + E * H * 2
    flops = T * K * 3 * 2 * H * I
    hbm, tf, src = peaks()
    gbs = nbytes / ms / 1e6
    tflops = flops / ms / 1e9
    roof = {"bound": "hbm", "peak": hbm, "frac": gbs / hbm, "peak_source": src} if T <= 256 else \
        {"bound": "tensor", "peak": tf, "frac": tflops / tf, "peak_source": src}
    return {"config": 1, "workload": f"MoE block T={T} bf16, dense bf16 router, E=64 top-8", "ms": ms,
            "unique_experts": unique, "algorithmic_bytes": nbytes, "achieved_gbs": gbs, "achieved_tflops": tflops,
            "roofline": roof, "l2": "flushed (256 MB written) before each iteration"}


def config4(args, dev):
    """Decode attention alone: B=64, 16 x 128, fp16 KV N(0,1), L in {512, 4096, 32768}."""
    from . import ops
    out = []
    g = torch.Generator(device=dev)
    g.manual_seed(20260104)
    hbm, _, src = peaks()
    B = 64
    for L in (512, 4096, 32768):
        cap = L + 64
        k = torch.empty((B, HEADS, cap, D), dtype=torch.float16, device=dev)
        v = torch.empty_like(k)
        for b0 in range(0, B, 8):
            k[b0:b0 + 8].normal_(generator=g)
            v[b0:b0 + 8].normal_(generator=g)
        qkv = torch.randn(B, 3 * HEADS * D, generator=g, device=dev).to(torch.float16)
        qn = (1 + 0.1 * torch.randn(HEADS * D, generator=g, device=dev)).to(torch.float16)
        kn = (1 + 0.1 * torch.randn(HEADS * D, generator=g, device=dev)).to(torch.float16)
        pos = torch.full((B,), L, dtype=torch.int32, device=dev)
        fn = lambda: ops.attention_decode(qkv, qn, kn, pos, k, v, 1e-5, 10000.0)  # noqa: E731
        flush = l2_flusher(dev) if L == 512 else None
        ms = timed(fn, args.iters, flush)
        nbytes = B * HEADS * (L + 1) * D * 2 * 2 + B * 4 * HEADS * D * 2
        gbs = nbytes / ms / 1e6
        out.append({"config": 4, "workload": f"decode attention B=64 L={L} (QK-norm, RoPE, append, SDPA)", "ms": ms,
                    "algorithmic_bytes": nbytes, "achieved_gbs": gbs,
                    "roofline": {"bound": "hbm", "peak": hbm, "frac": gbs / hbm, "peak_source": src},
                    "l2": "flushed before each iteration" if flush else "KV larger than L2"})
        del k, v
        torch.cuda.empty_cache()
    return out


def config3(args, dev):
    """Prefill 8 x 2048 uniform tokens through the 16-layer model (one call)."""
    from .model import Config, Model, Session
    from .quant import synthetic_olmoe
    cfg = Config(capacity=2048 + 64)
    w = synthetic_olmoe(cfg, seed=20260103, device=dev)
    model = Model(cfg, w, device=torch.device(dev).index or 0)
    del w
    torch.cuda.empty_cache()
    sess = Session(model, max_batch=8, capacity=cfg.capacity, max_prefill_tokens=8 * 2048)
    g = torch.Generator()
    g.manual_seed(20260103)
    prompts = [torch.randint(0, V, (2048,), generator=g) for _ in range(8)]

    def run():
        sess.reset()
        sess.prefill(list(range(8)), prompts)

    ms = timed(run, max(1, args.iters // 4))
    T = 8 * 2048
    # per layer: experts (gate, up, down), router, q/k/v/o projections
    layer_flops = T * (K * 3 * 2 * H * I + 2 * H * E + 2 * H * 4 * HEADS * D)
    attn_flops = 8 * HEADS * 4 * D * (2048 * 2049 // 2)
    flops = 16 * layer_flops + 16 * attn_flops + 8 * 2 * H * V
    _, tf, src = peaks()
    achieved = flops / ms / 1e9
    sess.close()
    model.close()
    return {"config": 3, "workload": "prefill 8 x 2048 tokens, OLMoE-1B-7B 4-bit, one session call", "ms": ms,
            "tokens_per_s": T / ms * 1e3, "algorithmic_tflop": flops / 1e12, "achieved_tflops": achieved,
            "roofline": {"bound": "tensor", "peak": tf, "frac": achieved / tf, "peak_source": src},
            "note": "every layer runs all 16384 rows (no last-query-only shortcut); includes host-side "
                    "prefill bookkeeping and the final sync of the session call"}


def _skewed_router(g, dev):
    """Router [E, H+...]: a dense bf16 router whose logits carry a per-expert
    bias N(0, 1.5) through the last input column (x[:, -1] = 1, w[:, -1] =
    bias); the remaining weights are N(0, 0.02)."""
    w = torch.randn(E, H, generator=g, device=dev) * 0.02
    bias = torch.randn(E, generator=g, device=dev) * 1.5
    w[:, -1] = bias
    return w.to(torch.bfloat16)


def config5(args, dev):
    """Expert-parallel MoE prefill: 65536 bf16 tokens in total, skewed routing,
    64/n experts per rank, NCCL all-to-all dispatch and return."""
    import torch.distributed as dist

    from .ep import ExpertParallelMoE, shard_experts
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank = int(os.environ.get("RANK", 0))
    if not dist.is_initialized():
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29541")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=300),
                                device_id=torch.device(dev))
    g = torch.Generator(device=dev)
    g.manual_seed(20260105)          # same weights on every rank
    ex = experts(g, dev)
    router = _skewed_router(g, dev)
    gl, ul, dl = shard_experts(ex["gate"], ex["up"], ex["down"], rank, world)
    del ex
    torch.cuda.empty_cache()
    moe = ExpertParallelMoE(router, gl, ul, dl, E, K)
    T = 65536 // world
    gx = torch.Generator(device=dev)
    gx.manual_seed(7000 + rank)
    x = torch.randn(T, H, generator=gx, device=dev).to(torch.bfloat16)
    x[:, -1] = 1.0
    res = torch.randn(T, H, generator=gx, device=dev).to(torch.bfloat16)

    def step():
        moe(x, res)
        dist.barrier()

    ms = timed(step, max(1, args.iters // 4))
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    flops = 65536 * K * 3 * 2 * H * I
    _, tf, src = peaks()
    achieved = flops / ms / 1e9
    line = {"config": 5, "workload": f"EP MoE layer, 65536 bf16 tokens, skew N(0,1.5), {world} GPU(s), "
                                     f"{E // world} experts each", "n_gpus": world, "ms": ms,
            "tokens_per_s": 65536 / ms * 1e3, "achieved_tflops": achieved,
            "roofline": {"bound": "tensor", "peak": tf * world, "frac": achieved / (tf * world),
                         "peak_source": src}, "timing": "max over ranks, barrier inside each step"}
    dist.destroy_process_group()
    return line if rank == 0 else None


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, nargs="+", default=[1, 4, 3])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--tokens", type=int, default=32, help="config 1: tokens in the MoE block")
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    fns = {1: config1, 3: config3, 4: config4, 5: config5}
    for c in args.config:
        res = fns[c](args, dev)
        for line in (res if isinstance(res, list) else [res]):
            if line is not None:
                print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
