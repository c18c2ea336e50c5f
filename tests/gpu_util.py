"""Helpers for GPU parity tests: numpy oracle arrays <-> CUDA tensors."""
import numpy as np
import torch

TORCH_ACT = {"f16": torch.float16, "bf16": torch.bfloat16}


def dev(x, act=None):
    """numpy -> CUDA tensor; act arrays (float32 holding act values) become act dtype."""
    x = np.asarray(x)
    if act is not None:
        return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(TORCH_ACT[act]).cuda()
    if x.dtype == np.uint32:
        return torch.from_numpy(x.astype(np.int64)).to(torch.uint32).cuda()
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    """CUDA tensor -> numpy (act dtypes as float32)."""
    t = t.detach().cpu()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.float().numpy()
    if t.dtype == torch.uint32:
        return t.to(torch.int64).numpy().astype(np.uint32)
    return t.numpy()


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return np.array_equal(a.view(np.uint32), b.view(np.uint32)) or (
        np.array_equal(np.isnan(a), np.isnan(b))
        and np.array_equal(np.where(np.isnan(a), 0, a).view(np.uint32), np.where(np.isnan(b), 0, b).view(np.uint32)))


def experts_np(rng, E, H, I):
    import oracle
    out = {}
    for name, shape in (("gate", (E, I, H)), ("up", (E, I, H)), ("down", (E, H, I))):
        w = oracle.round_bf16(rng.standard_normal(shape).astype(np.float32) * np.float32(0.02))
        out[name] = oracle.affine_quantize(w)
    return out


def experts_dev(ex):
    return {k: tuple(dev(a) for a in v) for k, v in ex.items()}
