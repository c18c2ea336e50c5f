#!/usr/bin/env python3
"""OLMoE-1B-7B 4-bit batched decode benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--kv-len L]
    python bench.py --impl reference ...      # the CPU reference arm

A step is one decode token for each of B requests through the full 16-layer
random-init OLMoE-1B-7B (4-bit MLX-affine weights, group 64) with an fp16 KV
cache pre-filled with N(0, 1) to length L.  Requests are data parallel: each
rank holds a full replica and its own B requests, no collective on the data
path ("scaling": "weak").  `value` is whole-job tokens/s with inputs resident
in HBM; `e2e` is the same metric through the C-ABI session call with host
token ids in and host fp32 logits out (copies inside the timed region).
The KV cache (B x 16 layers x 2 x 16 x L x 128 x 2 B; 34 GB at B=64) is far
larger than L2, so no flush is needed between steps.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "OLMoE-4bit decode & prefill tok/s per B200; MoE GB/s vs HBM peak"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + written) per algorithmic byte of the attention phase,
# from an ncu capture of attn_split at B=64, L=512 (269.76 MB read + 3.84 MB
# of partials written for 268.96 MB of K/V); both terms grow with the KV
# length, so the ratio carries over to the benchmark's L.
ATTN_TRAFFIC_PER_ALGO_BYTE = (269.763072 + 3.841536) / 268.959744

# Algorithmic bytes per launch of each traced phase (per layer), batch B, KV
# length L (keys read per request = L + 1 including this step's slot).
H, W, I, E, K_TOP, V = 2048, 2048, 1024, 64, 8, 50304
EXPERT_PROJ_BYTES = I * H // 2 + I * (H // 64) * 4  # one expert projection: 1,179,648 B


def phase_bytes(phase, B, L):
    act = 2
    if phase == "attention":
        return B * 16 * (L + 1) * 128 * 2 * 2 + B * 3 * W * act + B * W * act
    if phase == "qkv_proj":
        return 3 * (W * H // 2 + W * (H // 64) * 4) + B * H * act + B * 3 * W * act
    if phase == "o_proj":
        return (H * W // 2 + H * (W // 64) * 4) + B * (W + 2 * H) * act
    if phase in ("moe_gate_up", "moe_down"):
        unique = E * (1 - (1 - K_TOP / E) ** B)
        mult = 2 if phase == "moe_gate_up" else 1
        return unique * mult * EXPERT_PROJ_BYTES
    if phase == "lm_head":
        return V * H // 2 + V * (H // 64) * 4 + B * V * 4
    return None


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms; only the
    samples taken inside the timed window (wall clock) are summarised."""
    FIELDS = ("timestamp,index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.path = Path("/tmp") / f"tf_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        # nvidia-smi needs a moment before its first sample
        time.sleep(0.5)

    def stop(self, t0, t1):
        """Summary of the samples stamped inside [t0, t1] (time.time())."""
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 11:
                continue
            if self.uuid and self.uuid not in parts[2]:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                if not t0 <= ts <= t1:
                    continue
                sm.append(float(parts[3]))
                mx.append(float(parts[4]))
            except ValueError:
                continue
            for n, v in zip(names, parts[7:11]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def build_model(cap, device, layers=16):
    import torch

    from trifuse_b200.model import Config, Model
    from trifuse_b200.quant import synthetic_olmoe
    cfg = Config(capacity=cap, layers=layers)
    w = synthetic_olmoe(cfg, seed=20260102, device=f"cuda:{device}")
    model = Model(cfg, w, device=device)
    del w
    torch.cuda.empty_cache()
    return cfg, model


def decode_session(model, B, L, cap, device, seed=20260103):
    """A session of B requests whose caches hold N(0, 1) f16 keys and values
    in slots [0, L) of every layer."""
    import torch

    from trifuse_b200.model import Session
    sess = Session(model, max_batch=B, capacity=cap)
    g = torch.Generator(device=f"cuda:{device}")
    g.manual_seed(seed)
    for layer in range(model.cfg.layers):
        k, v = sess.kv_tensors(layer)
        for t in (k, v):
            for b0 in range(0, B, 16):
                t[b0:b0 + 16, :, :L].normal_(generator=g)
    torch.cuda.synchronize()
    return sess


def time_steps(sess, ids, logits, steps, warmup, L, B, stream, barrier):
    import torch
    sess.set_lengths([L] * B)
    for i in range(warmup):
        sess.decode(ids[i], logits=logits)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        sess.decode(ids[warmup + i], logits=logits)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1) / steps


def prefill_flops(seqs, T):
    """Algorithmic flops of a prefill of `seqs` sequences of T tokens with the
    reference's semantics (MLXNativeGraniteMoEPrefill.h:440-442, 471): layers
    0-14 run every row; the last layer projects K and V of every row but
    runs Q, attention, o-proj and the MoE block for the last row only; the
    lm_head runs on the last row.  Causal attention counts 4 D flops per
    (query, key) pair at or before the query."""
    D = 16 * 128
    rows = seqs * T
    per_row = K_TOP * 3 * 2 * H * I + 2 * H * E + 4 * 2 * H * W
    attn_seq = 4 * D * (T * (T + 1) // 2)
    full = 15 * (rows * per_row + seqs * attn_seq)
    last = rows * 2 * 2 * H * W + seqs * (per_row - 2 * 2 * H * W + 4 * D * T)
    return full + last + seqs * 2 * H * V


class PhaseRoof:
    """Roofline entries of traced phases from their algorithmic bytes."""

    def __init__(self, peak, peak_kind):
        self.peak, self.peak_kind = peak, peak_kind

    def entry(self, phases, name, nbytes):
        tot, cnt = phases.get(name, (0.0, 0))
        if not (nbytes and cnt):
            return None
        avg_ms = tot / cnt
        achieved = nbytes / (avg_ms / 1000.0) / 1e9
        return {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": self.peak, "unit": "GB/s",
                "frac": achieved / self.peak, "peak_source": self.peak_kind,
                "algorithmic_bytes_per_launch": nbytes, "avg_launch_ms": avg_ms}


def run_prefill(model, cfg, rank, world, device, warmup, iters, barrier, max_over_ranks, bf16_peak, peak_kind):
    """8 sequences of 2048 uniform token ids, data parallel
    over the ranks (sequence i on rank i % world), one session call per rank
    and iteration; tok/s = 16384 / the slowest rank's time."""
    import torch

    from trifuse_b200.model import Session
    seqs_total, T = 8, 2048
    mine = [i for i in range(seqs_total) if i % world == rank]
    g = torch.Generator()
    g.manual_seed(20260103)
    prompts = [torch.randint(0, cfg.vocab, (T,), generator=g) for _ in range(seqs_total)]
    n = len(mine)
    if n == 0:
        # more ranks than sequences: this rank only takes part in the timing barriers
        for _ in range(warmup + iters):
            barrier()
        return None
    sess = Session(model, max_batch=n, capacity=T + 64, max_prefill_tokens=n * T)
    ids_dev = torch.cat([prompts[i] for i in mine]).cuda(device)
    logits_dev = torch.empty((n, cfg.vocab), dtype=torch.float32, device=f"cuda:{device}")
    stream = torch.cuda.current_stream()

    def timed(fn, k):
        for _ in range(warmup):
            sess.reset()
            fn()
        torch.cuda.synchronize()
        barrier()
        total = 0.0
        for _ in range(k):
            sess.reset()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            b.synchronize()
            total += a.elapsed_time(b)
        barrier()
        return max_over_ranks(total / k)

    reqs = list(range(n))
    ms = timed(lambda: sess.prefill_device(reqs, [T] * n, ids_dev, logits_dev), iters)
    e2e_ms = timed(lambda: sess.prefill(reqs, [prompts[i] for i in mine]), iters)
    sess.reset()
    sess.trace(True)
    sess.prefill_device(reqs, [T] * n, ids_dev, logits_dev)
    sess.trace(False)
    phases = {p: round(v[0], 3) for p, v in sess.trace_read().items() if v[1]}
    sess.close()
    flops = prefill_flops(seqs_total, T)
    tflops = flops / (ms / 1000.0) / 1e12
    return {"workload": "prefill 8 x 2048 uniform token ids (config 3), sequence i on rank i % n_gpus",
            "value": seqs_total * T / (ms / 1000.0), "unit": "tok/s", "ms_per_call": ms,
            "scaling": "strong", "sequences_per_gpu": n,
            # whole-job throughput against the peak of every GPU that holds a sequence
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": bf16_peak * min(world, seqs_total),
                         "unit": "TFLOP/s", "frac": tflops / (bf16_peak * min(world, seqs_total)),
                         "peak_source": peak_kind, "algorithmic_tflop": flops / 1e12,
                         "flops": "reference semantics: last layer last-row-only, lm_head on last rows"},
            "e2e": {"value": seqs_total * T / (e2e_ms / 1000.0), "unit": "tok/s", "ms_per_call": e2e_ms,
                    "h2d_bytes_per_step": seqs_total * T * 8, "d2h_bytes_per_step": seqs_total * cfg.vocab * 4},
            "phase_ms_rank0": phases if rank == 0 else None}


def run_sweep(model, cfg, batches, L, rank, world, device, warmup, steps, barrier, max_over_ranks):
    """Decode tok/s at other batch sizes (config 2 sweep), same model and L."""
    import torch
    out = {}
    for B in batches:
        cap = L + 2 * (warmup + steps) + 8
        sess = decode_session(model, B, L, cap, device, seed=20260110 + B)
        g = torch.Generator(device="cuda")
        g.manual_seed(20260104 + rank + B)
        ids = torch.randint(0, cfg.vocab, (warmup + steps, B), device="cuda", generator=g, dtype=torch.int64)
        logits = torch.empty((B, cfg.vocab), dtype=torch.float32, device="cuda")
        ms = max_over_ranks(time_steps(sess, ids, logits, steps, warmup, L, B, torch.cuda.current_stream(), barrier))
        out[f"B={B}"] = {"value": B * world / (ms / 1000.0), "unit": "tok/s", "ms_per_step": ms}
        sess.close()
        del sess
        torch.cuda.empty_cache()
    return out


class CpuWorkload:
    """Random-init weights of one OLMoE decoder layer plus the lm_head and a
    shared N(0,1) K/V block, built once; the oracle's decode layer and head
    are then timed on them (the reference's CPU path, numpy)."""

    def __init__(self, B, L, seed=5):
        import numpy as np

        import oracle
        self.oracle = oracle
        rng = np.random.default_rng(seed)
        self.cfg = oracle.OLMoEConfig(act="f16")

        def rand_affine(shape):
            *lead, rows, cols = shape
            q = rng.integers(0, 2 ** 32, size=(*lead, rows, cols // 8), dtype=np.uint32)
            s = (rng.random((*lead, rows, cols // 64)) * 0.004 + 0.001).astype(np.float16)
            b = (-7.5 * s.astype(np.float32)).astype(np.float16)
            return q, s, b

        norm = lambda n: (1 + 0.1 * rng.standard_normal(n)).astype(np.float16)  # noqa: E731
        self.layer = dict(input_norm=norm(H), post_norm=norm(H), q_norm=norm(W), k_norm=norm(W),
                          q=rand_affine((W, H)), k=rand_affine((W, H)), v=rand_affine((W, H)),
                          o=rand_affine((H, W)), router=rand_affine((E, H)),
                          experts={"gate": rand_affine((E, I, H)), "up": rand_affine((E, I, H)),
                                   "down": rand_affine((E, H, I))})
        self.head = rand_affine((V, H))
        self.final_norm = norm(H)
        # One N(0,1) K and V block shared by every request: the timed math is
        # the same per request and host memory stays bounded.
        k1 = rng.standard_normal((16, L + 1, 128), dtype=np.float32).astype(np.float16).astype(np.float32)
        v1 = rng.standard_normal((16, L + 1, 128), dtype=np.float32).astype(np.float16).astype(np.float32)
        self.kc, self.vc = [k1] * B, [v1] * B
        self.h = oracle.round_f16(rng.standard_normal((B, H)).astype(np.float32))
        self.out = self.h  # the head's input until a layer has run (same shape)
        self.B, self.L = B, L

    def layer_s(self):
        t0 = time.perf_counter()
        self.out = self.oracle.decode_layer_batched(self.h, self.layer, self.cfg, self.kc, self.vc,
                                                    [self.L] * self.B, fast=True)
        return time.perf_counter() - t0

    def head_s(self):
        o = self.oracle
        t0 = time.perf_counter()
        o.affine_qmm(o.rms_norm(self.out, self.final_norm, 1e-5, "f16"), *self.head, "f16")
        return time.perf_counter() - t0


def cpu_sample(B, L, seed=5):
    """One decode layer of the oracle for B requests at KV length L, plus the
    lm_head; returns (seconds for the extrapolated 16-layer step, details)."""
    w = CpuWorkload(B, L, seed)
    layer = w.layer_s()
    head = w.head_s()
    return 16 * layer + head, {"layer_s": layer, "head_s": head}


def cpu_threads():
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        n = max((i.get("num_threads", 1) for i in info), default=1)
        return int(n)
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, rank, world):
    """CPU reference arm: the oracle port of the reference's operators on the
    host cores, same metric/config; rank 0 only.  Each step is a bounded
    sample: one of the 16 decode layers for all B requests (weights built
    once); the lm_head is timed once after warm-up, and a step is estimated
    as 16 x layer + head."""
    if rank != 0:
        return
    w = CpuWorkload(args.batch, args.kv_len)
    for _ in range(args.warmup):
        w.layer_s()
    head = w.head_s() if args.warmup or args.steps else 0.0
    layers = [w.layer_s() for _ in range(args.steps)]
    step_s = 16 * (sum(layers) / max(1, len(layers))) + head
    value = args.batch / step_s
    cores = cpu_threads()
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1000,
            "ms_per_step_kind": "extrapolated: 16 x the mean of the sampled layers + the lm_head",
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": config_keys(args.batch, args.kv_len, world),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"per step one of 16 decode layers for {args.batch} requests at "
                                       f"L={args.kv_len} (numpy oracle, weights built once); lm_head timed "
                                       f"once ({head:.2f}s); step = 16 x mean layer + head"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--kv-len", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill measurement")
    ap.add_argument("--sweep", default="1,16,256", help="decode batch sizes of the sweep ('' = none)")
    ap.add_argument("--layers", type=int, default=16, help="model depth (profiling small cases)")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling run: warm up, then one decode step between cudaProfilerStart/Stop")
    ap.add_argument("--ncu-prefill", action="store_true",
                    help="profiling run: one warm-up config-3 prefill (8 x 2048), then one between "
                         "cudaProfilerStart/Stop")
    args = ap.parse_args()
    rank, local_rank, world = env_rank()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from trifuse_b200 import lib
    assert args.warmup >= 1
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local_rank}"))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(ms):
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        return ms

    B, L = args.batch, args.kv_len
    cap = max(L + 2 * (args.warmup + args.steps) + 8, 2048 + 64)
    cfg, model = build_model(cap, local_rank, args.layers)
    if args.ncu_prefill:
        from trifuse_b200.model import Session
        T, n = 2048, 8
        g = torch.Generator()
        g.manual_seed(20260103)
        ids_dev = torch.randint(0, cfg.vocab, (n * T,), generator=g).cuda(local_rank)
        logits_dev = torch.empty((n, cfg.vocab), dtype=torch.float32, device="cuda")
        psess = Session(model, max_batch=n, capacity=T + 64, max_prefill_tokens=n * T)
        for profiled in (False, True):
            psess.reset()
            torch.cuda.synchronize()
            if profiled:
                torch.cuda.profiler.start()
            psess.prefill_device(list(range(n)), [T] * n, ids_dev, logits_dev)
            torch.cuda.synchronize()
            if profiled:
                torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"ncu_prefill": True, "sequences": n, "tokens": T, "layers": args.layers}))
        psess.close()
        model.close()
        return
    sess = decode_session(model, B, L, cap, local_rank)
    stream = torch.cuda.current_stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(20260104 + rank)
    n_ids = args.warmup + args.steps
    ids = torch.randint(0, cfg.vocab, (n_ids, B), device="cuda", generator=g, dtype=torch.int64)
    logits = torch.empty((B, cfg.vocab), dtype=torch.float32, device="cuda")

    if args.ncu:
        sess.set_lengths([L] * B)
        for i in range(args.warmup):
            sess.decode(ids[i], logits=logits)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        sess.decode(ids[args.warmup], logits=logits)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"ncu_step": True, "batch": B, "kv_len": L, "layers": args.layers}))
        sess.close()
        model.close()
        return

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local_rank).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    hbm_peak, peak_kind = measured_peaks()
    bf16_peak = bf16_peak_tflops()

    # 1) decode, device-resident throughput (the headline value)
    launches0 = lib().tf_launch_count()
    clocks.start()
    w0 = time.time()
    ms = max_over_ranks(time_steps(sess, ids, logits, args.steps, args.warmup, L, B, stream, barrier))
    clk = clocks.stop(w0, time.time())
    launches = (lib().tf_launch_count() - launches0) // (args.steps + args.warmup)
    value = B * world / (ms / 1000.0)

    # 2) phase trace of the same workload: the dominant phase's roofline and
    # the MoE gate/up and down HBM fractions
    n_trace = min(args.steps, 4)
    sess.trace(True)
    time_steps(sess, ids, logits, n_trace, 1, L, B, stream, barrier)  # traces the warm-up step too
    sess.trace(False)
    phases = sess.trace_read()
    dom = max(phases, key=lambda p: phases[p][0])
    pr = PhaseRoof(hbm_peak, peak_kind)
    roof = pr.entry(phases, dom, phase_bytes(dom, B, L))
    if roof is not None:
        if dom == "attention":
            roof["traffic"] = roof["algorithmic_bytes_per_launch"] * ATTN_TRAFFIC_PER_ALGO_BYTE
            roof["traffic_source"] = "ncu dram bytes of attn_split at B=64 L=512, scaled by KV length"
        else:
            roof["traffic"] = None
        for ph in ("moe_gate_up", "moe_down"):
            roof[ph] = pr.entry(phases, ph, phase_bytes(ph, B, L))
    step_phase_ms = {p: round(v[0] / (n_trace + 1), 4) for p, v in phases.items() if v[1]}

    # 3) end to end through the C-ABI call with host buffers
    ids_host = ids.cpu().pin_memory()
    logits_host = torch.empty((B, cfg.vocab), dtype=torch.float32, pin_memory=True)
    e2e_ms = max_over_ranks(time_steps(sess, ids_host, logits_host, args.steps, args.warmup, L, B, stream, barrier))
    e2e = {"value": B * world / (e2e_ms / 1000.0), "unit": "tok/s", "h2d_bytes_per_step": B * (8 + 4),
           "d2h_bytes_per_step": B * cfg.vocab * 4, "ms_per_step": e2e_ms}
    sess.close()
    del sess
    torch.cuda.empty_cache()

    # 4) prefill (config 3) and 5) the decode batch sweep (config 2)
    prefill = None
    if not args.no_prefill and args.layers == 16:
        prefill = run_prefill(model, cfg, rank, world, local_rank, args.warmup, max(3, min(args.steps, 5)),
                              barrier, max_over_ranks, bf16_peak, peak_kind)
    sweep = None
    batches = [int(b) for b in args.sweep.split(",") if b.strip()]
    if batches:
        sweep = run_sweep(model, cfg, batches, L, rank, world, local_rank, args.warmup,
                          max(3, min(args.steps, 10)), barrier, max_over_ranks)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        step_s, det = cpu_sample(B, L)
        cpu = {"value": B / step_s, "unit": "tok/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"one of 16 decode layers + lm_head for {B} requests at L={L} (numpy oracle, "
                         f"layer {det['layer_s']:.2f}s, head {det['head_s']:.2f}s), step = 16 x layer + head "
                         f"(extrapolated)"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic (random-init weights, N(0,1) KV)",
                "config": config_keys(B, L, world),
                "e2e": e2e, "gpu_launches": int(launches), "roofline": roof, "cpu_baseline": cpu,
                "clocks": clk, "phase_ms_per_step": step_phase_ms, "prefill": prefill, "sweep": sweep}
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.destroy_process_group()


def config_keys(B, L, world):
    return {"workload": f"decode B={B}/GPU L={L} OLMoE-1B-7B 4-bit (config 2)",
            "batch_per_gpu": B, "global_batch": B * world, "kv_len": L, "layers": 16,
            "parallelism": f"dp{world} replicas", "l2": "inputs larger than L2 (KV cache)"}


def bf16_peak_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"])
        except Exception:
            pass
    return 1590.0


if __name__ == "__main__":
    main()
