"""Device-resident OLMoE model and per-request sessions over the C ABI.

Mirrors the reference's owner objects: ``Model`` stands for the
NativeGraniteMoEPrefill adapter bound to a loaded checkpoint
(MLXNativeGraniteMoEPrefill.h:157-304) and ``Session`` for the resident
session with its KV cache (TFETResidentSession.h: forward / prefill /
beginRequest / cancel).  All compute happens in libtrifuse_b200.so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ._lib import DTYPE_BF16, DTYPE_F16, HOST_INPUTS, HOST_OUTPUT, OLMoEConfig, TriFuseError, check, lib


@dataclass
class Config:
    """OLMoE geometry (export_native_olmoe_target.py:27-63); defaults are
    OLMoE-1B-7B."""
    layers: int = 16
    hidden: int = 2048
    heads: int = 16
    kv_heads: int = 16
    head_dim: int = 128
    intermediate: int = 1024
    vocab: int = 50304
    experts: int = 64
    top_k: int = 8
    capacity: int = 4096
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    act: torch.dtype = torch.float16

    def c_struct(self) -> OLMoEConfig:
        return OLMoEConfig(self.layers, self.hidden, self.heads, self.kv_heads, self.head_dim,
                           self.intermediate, self.vocab, self.experts, self.top_k, self.capacity,
                           self.rms_eps, self.rope_theta,
                           DTYPE_F16 if self.act == torch.float16 else DTYPE_BF16)


class Model:
    def __init__(self, cfg: Config, weights: dict, device: int = 0):
        self.cfg = cfg
        self.device = device
        h = C.c_void_p()
        c = cfg.c_struct()
        check(lib().tf_model_create(C.byref(c), device, C.byref(h)))
        self.handle = h
        try:
            for name, t in weights.items():
                t = t.contiguous()
                nbytes = t.numel() * t.element_size()
                check(lib().tf_model_bind(h, name.encode(), C.c_void_p(t.data_ptr()), nbytes,
                                          int(t.is_cuda)))
            check(lib().tf_model_finalize(h))
        except Exception:
            lib().tf_model_destroy(h)
            self.handle = None
            raise

    def close(self):
        if self.handle:
            check(lib().tf_model_destroy(self.handle))
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


class Session:
    def __init__(self, model: Model, max_batch: int, capacity: int, max_prefill_tokens: int = 0):
        self.model = model
        self.max_batch = max_batch
        self.capacity = capacity
        h = C.c_void_p()
        check(lib().tf_session_create(model.handle, max_batch, capacity, max_prefill_tokens, C.byref(h)))
        self.handle = h

    def kv(self, layer: int):
        """(k, v) device pointers of one layer: f16 [max_batch][kv_heads][capacity][head_dim]."""
        k, v = C.c_void_p(), C.c_void_p()
        check(lib().tf_session_kv(self.handle, layer, C.byref(k), C.byref(v)))
        return k.value, v.value

    def kv_tensors(self, layer: int):
        """Torch views of one layer's caches (no copy)."""
        cfg = self.model.cfg
        shape = (self.max_batch, cfg.kv_heads, self.capacity, cfg.head_dim)
        out = []
        for ptr in self.kv(layer):
            out.append(_device_view(ptr, shape, torch.float16, self.model.device))
        return out

    def set_lengths(self, lengths):
        arr = (C.c_int32 * len(lengths))(*lengths)
        check(lib().tf_session_set_lengths(self.handle, arr, len(lengths)))

    def lengths(self, batch=None):
        batch = self.max_batch if batch is None else batch
        arr = (C.c_int32 * batch)()
        check(lib().tf_session_get_lengths(self.handle, arr, batch))
        return list(arr)

    def decode(self, token_ids: torch.Tensor, positions=None, logits: torch.Tensor | None = None):
        """One token per request; token_ids int64 [B] (host or device);
        returns fp32 logits [B, vocab] on the same side as `logits` or the ids."""
        B = token_ids.numel()
        ids = token_ids.to(torch.int64).contiguous()
        flags = 0 if ids.is_cuda else HOST_INPUTS
        if logits is None:
            logits = torch.empty((B, self.model.cfg.vocab), dtype=torch.float32,
                                 device=ids.device if ids.is_cuda else "cpu",
                                 pin_memory=not ids.is_cuda)
        if not logits.is_cuda:
            flags |= HOST_OUTPUT
        pos = None
        if positions is not None:
            pos = (C.c_int32 * B)(*[int(p) for p in positions])
        check(lib().tf_session_decode(self.handle, C.c_void_p(ids.data_ptr()), pos, B,
                                      C.c_void_p(logits.data_ptr()), flags,
                                      C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return logits

    def decode_greedy(self, token_ids: torch.Tensor, positions=None, tokens: torch.Tensor | None = None,
                      logits: torch.Tensor | None = None):
        """One decode token per request followed by greedy selection on the
        device: returns int64 tokens [B] (argmax, or -1 for rows with a
        non-finite logit) on the device unless `tokens` is a host tensor.
        token_ids may be the device tokens of the previous greedy step."""
        B = token_ids.numel()
        ids = token_ids.to(torch.int64).contiguous()
        flags = 0 if ids.is_cuda else HOST_INPUTS
        if tokens is None:
            tokens = torch.empty(B, dtype=torch.int64, device=f"cuda:{self.model.device}")
        if not tokens.is_cuda:
            flags |= HOST_OUTPUT
            if logits is not None and logits.is_cuda:
                raise ValueError("decode_greedy: logits and tokens must be on the same side")
        elif logits is not None and not logits.is_cuda:
            raise ValueError("decode_greedy: logits and tokens must be on the same side")
        pos = None
        if positions is not None:
            pos = (C.c_int32 * B)(*[int(p) for p in positions])
        check(lib().tf_session_decode_greedy(self.handle, C.c_void_p(ids.data_ptr()), pos, B,
                                             C.c_void_p(tokens.data_ptr()),
                                             C.c_void_p(logits.data_ptr()) if logits is not None else None,
                                             flags, C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return tokens

    def generate_greedy(self, first_ids, steps: int):
        """Greedy generation with one-ahead submission (the reference's greedy
        pipeline, TFETResidentSession.mm:1113-1189): step t+1 is submitted with
        the device-resident tokens of step t before the host reads them, so
        the host copy of each token overlaps the next step.  Returns the
        tokens as a list of int lists [steps][B]; raises if a step produced
        a non-finite row (-1) or a token outside the vocabulary."""
        dev = f"cuda:{self.model.device}"
        ids = torch.as_tensor(first_ids, dtype=torch.int64).reshape(-1).to(dev)
        B = ids.numel()
        stream = torch.cuda.current_stream()
        bufs = [torch.empty(B, dtype=torch.int64, device=dev) for _ in range(2)]
        host = [torch.empty(B, dtype=torch.int64, pin_memory=True) for _ in range(2)]
        done = [torch.cuda.Event(), torch.cuda.Event()]
        out = []
        prev = None
        for t in range(steps):
            cur = bufs[t & 1]
            self.decode_greedy(ids, tokens=cur)
            host[t & 1].copy_(cur, non_blocking=True)
            done[t & 1].record(stream)
            ids = cur
            if prev is not None:  # read step t-1 while step t runs
                out.append(self._read_tokens(host[prev], done[prev]))
            prev = t & 1
        if prev is not None:
            out.append(self._read_tokens(host[prev], done[prev]))
        return out

    def _read_tokens(self, host: torch.Tensor, event) -> list:
        event.synchronize()
        toks = host.tolist()
        V = self.model.cfg.vocab
        for tok in toks:
            if not 0 <= tok < V:
                raise TriFuseError(9, "Greedy pipeline token outside vocabulary")
        return toks

    def prefill_device(self, requests, counts, ids: torch.Tensor, logits: torch.Tensor | None = None):
        """Prefill with device-resident inputs and outputs: ids int64 [sum(counts)]
        on the device (concatenated per request, checked on the device by the
        embedding), logits f32 [len(requests), vocab] on the device or None
        (cache only).  The call synchronizes its stream before it returns
        (its per-row bookkeeping is staged from host memory)."""
        n = len(requests)
        req = (C.c_int32 * n)(*requests)
        cnt = (C.c_int32 * n)(*counts)
        ids = ids.to(torch.int64).contiguous()
        if not ids.is_cuda or (logits is not None and not logits.is_cuda):
            raise ValueError("prefill_device: ids and logits must be device tensors")
        check(lib().tf_session_prefill(self.handle, req, cnt, n, C.c_void_p(ids.data_ptr()),
                                       C.c_void_p(logits.data_ptr()) if logits is not None else None, 0,
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return logits

    def prefill(self, requests, token_lists, want_logits=True):
        """Prefill several requests; token_lists: list of int64 tensors/lists."""
        counts = [len(t) for t in token_lists]
        ids = torch.cat([torch.as_tensor(t, dtype=torch.int64).cpu() for t in token_lists]).contiguous()
        n = len(requests)
        req = (C.c_int32 * n)(*requests)
        cnt = (C.c_int32 * n)(*counts)
        logits = None
        if want_logits:
            logits = torch.empty((n, self.model.cfg.vocab), dtype=torch.float32)
        check(lib().tf_session_prefill(self.handle, req, cnt, n, C.c_void_p(ids.data_ptr()),
                                       C.c_void_p(logits.data_ptr()) if logits is not None else None,
                                       HOST_INPUTS | HOST_OUTPUT,
                                       C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return logits

    def prefill_chunked(self, request: int, tokens, chunk: int = 128, want_logits: bool = True):
        """One request's prompt in chunks of `chunk` tokens (the reference's
        chunked prefill: cache-only intermediate chunks, logits of the last
        row from the final chunk); returns host fp32 logits [vocab] or None."""
        ids = torch.as_tensor(tokens, dtype=torch.int64).reshape(-1).cpu().contiguous()
        logits = torch.empty(self.model.cfg.vocab, dtype=torch.float32) if want_logits else None
        check(lib().tf_session_prefill_chunked(self.handle, int(request), C.c_void_p(ids.data_ptr()), ids.numel(),
                                               int(chunk),
                                               C.c_void_p(logits.data_ptr()) if logits is not None else None,
                                               HOST_INPUTS | HOST_OUTPUT,
                                               C.c_void_p(torch.cuda.current_stream().cuda_stream)))
        return logits

    def capture(self, indices: torch.Tensor | None, hidden: torch.Tensor | None = None):
        """Diagnostic: write every layer's top-k expert ids (int32 device
        tensor [layers, rows, top_k]) and output hidden states (act device
        tensor [layers, rows, hidden]) of the following forwards; both None
        turns it off."""
        rows = None
        for t, dt in ((indices, torch.int32), (hidden, None)):
            if t is None:
                continue
            if not t.is_cuda or t.dim() != 3 or (dt is not None and t.dtype != dt):
                raise ValueError("capture: device tensors [layers, rows, ...] (int32 indices)")
            if rows is not None and t.shape[1] != rows:
                raise ValueError("capture: indices and hidden disagree on rows")
            rows = t.shape[1]
        check(lib().tf_session_capture(self.handle, C.c_void_p(indices.data_ptr()) if indices is not None else None,
                                       C.c_void_p(hidden.data_ptr()) if hidden is not None else None,
                                       rows or 0))

    def graphs(self, enable: bool):
        """Turn CUDA-graph replay of decode steps on/off (default on)."""
        check(lib().tf_session_graphs(self.handle, int(enable)))

    def trace(self, enable: bool):
        """Turn phase tracing (CUDA events around each forward phase) on/off."""
        check(lib().tf_session_trace(self.handle, int(enable)))

    def trace_read(self):
        """{phase: (total_ms, count)} over traced calls since the last read."""
        n = lib().tf_trace_phases()
        ms = (C.c_float * n)()
        cnt = (C.c_int32 * n)()
        check(lib().tf_session_trace_read(self.handle, ms, cnt))
        return {lib().tf_trace_phase_name(i).decode(): (ms[i], cnt[i]) for i in range(n)}

    def cancel(self):
        check(lib().tf_session_cancel(self.handle))

    def reset(self):
        check(lib().tf_session_reset(self.handle))

    def close(self):
        if self.handle:
            check(lib().tf_session_destroy(self.handle))
            self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


def _device_view(ptr: int, shape, dtype, device: int) -> torch.Tensor:
    """Wrap externally owned device memory as a tensor (lifetime = session)."""
    numel = 1
    for d in shape:
        numel *= d
    esize = torch.empty((), dtype=dtype).element_size()

    class _Holder:
        __cuda_array_interface__ = {
            "shape": (numel * esize,), "typestr": "|u1", "data": (ptr, False), "version": 3,
        }

    raw = torch.as_tensor(_Holder(), device=f"cuda:{device}")
    return raw.view(dtype).reshape(shape)
