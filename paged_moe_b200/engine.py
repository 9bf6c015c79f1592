"""Batched entry points over torch CUDA tensors, calling the C ABI.

These remove the reference's per-row Python loop (verify_decode.py:889-898,
lookup_decode.py:344-356): one call processes every row of a [B, V] batch with
per-row settings and histories.  torch provides device memory and the current
stream; all arithmetic happens in libpm_sample.so.
"""

from __future__ import annotations

import ctypes as C
import threading
from typing import Optional, Sequence, Union

import torch

from . import _lib as L
from .params import ProcessorSettings, SamplerSettings, pack_rows, validate

_ws_lock = threading.Lock()
_ws_cache: dict = {}
_params_cache: dict = {}


def workspace(nbytes: int, device: torch.device, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """A zero-initialised device workspace of at least nbytes for (device, stream).

    The kernels leave their workspace ready for the next call, so one buffer
    per stream is reused; calls on different streams get different buffers.
    """
    stream = stream or torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
        return buf


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return L.PM_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return L.PM_DTYPE_BF16
    raise TypeError(f"logits must be float32 or bfloat16, got {t.dtype}")


def _as_list(x, n, default):
    if x is None:
        return [default] * n
    if isinstance(x, (list, tuple)) and not (isinstance(x, tuple) and hasattr(x, "_fields")):
        if len(x) != n:
            raise ValueError(f"expected {n} per-row settings, got {len(x)}")
        return list(x)
    return [x] * n


class _Keep:
    """Holds tensors whose device pointers a C call uses."""

    def __init__(self):
        self.items = []

    def __call__(self, t):
        if t is not None:
            self.items.append(t)
        return t


def _params_for(dev: torch.device, sampler, processors, B: int, V: int):
    """(device params tensor, flags_any, top_k_max, per_row), cached by settings."""
    single = not isinstance(sampler, (list, tuple)) and not isinstance(processors, (list, tuple))
    if single:
        s = sampler if sampler is not None else SamplerSettings()
        p = processors if processors is not None else ProcessorSettings()
        key = (dev.index, V, s, p)
        hit = _params_cache.get(key)
        if hit is not None:
            return hit
        validate(s, p, V)
        samplers, procs, per_row = [s], [p], False
    else:
        samplers = _as_list(sampler, B, SamplerSettings())
        procs = _as_list(processors, B, ProcessorSettings())
        per_row = len(set(samplers)) > 1 or len(set(procs)) > 1
        key = (dev.index, V, tuple(samplers) if per_row else samplers[0], tuple(procs) if per_row else procs[0])
        hit = _params_cache.get(key)
        if hit is not None:
            return hit
        for s, p in zip(samplers, procs):
            validate(s, p, V)
        if len({p.logit_bias for p in procs}) > 1:
            raise ValueError("logit_bias must be the same for every row of one call")
        if not per_row:
            samplers, procs = samplers[:1], procs[:1]
    raw, flags_any, top_k_max = pack_rows(samplers, procs)
    params = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dev)
    bias = None
    lb = procs[0].logit_bias
    if lb:
        bias = (torch.tensor([t for t, _ in lb], dtype=torch.int32, device=dev),
                torch.tensor([float(v) for _, v in lb], dtype=torch.float32, device=dev), len(lb))
    hit = (params, flags_any, top_k_max, per_row, procs, bias)
    with _ws_lock:
        if len(_params_cache) > 256:
            _params_cache.clear()
        _params_cache[key] = hit
    return hit


def build_rows(logits: torch.Tensor, sampler, processors, history, history_len, mask, keep: _Keep,
               feed: Optional[torch.Tensor] = None, feed_group: int = 0,
               forced: Optional[torch.Tensor] = None) -> L.Rows:
    if logits.dim() != 2:
        raise ValueError("logits must be [rows, vocab]")
    if not logits.is_cuda:
        raise ValueError("logits must be a CUDA tensor")
    if logits.stride(1) != 1:
        logits = keep(logits.contiguous())
    B, V = logits.shape
    dev = logits.device
    params, flags_any, top_k_max, per_row, procs, bias = _params_for(dev, sampler, processors, B, V)
    r = L.Rows()
    r.logits = logits.data_ptr()
    r.dtype = _dtype_code(logits)
    r.rows = B
    r.vocab = V
    r.row_stride = logits.stride(0)
    r.params = params.data_ptr()
    r.params_per_row = 1 if per_row else 0
    r.flags_any = flags_any
    r.top_k_max = top_k_max
    if history is not None and any(p.penalties_on for p in procs):
        h = history
        if h.dim() == 1:
            h = h.unsqueeze(0).expand(B if feed is None else B // feed_group, -1)
        h = keep(h.to(device=dev, dtype=torch.int32).contiguous())
        r.hist = h.data_ptr()
        r.hist_stride = h.shape[1]
        if history_len is not None:
            hl = keep(torch.as_tensor(history_len, dtype=torch.int32, device=dev).contiguous())
            r.hist_len = hl.data_ptr()
    if feed is not None:
        f = keep(feed.to(device=dev, dtype=torch.int32).contiguous())
        r.feed = f.data_ptr()
        r.feed_group = feed_group
        if not r.hist:
            # the feed alone is the history
            dummy = keep(torch.zeros((B // feed_group, 1), dtype=torch.int32, device=dev))
            hl = keep(torch.zeros(B // feed_group, dtype=torch.int32, device=dev))
            r.hist, r.hist_len, r.hist_stride = dummy.data_ptr(), hl.data_ptr(), 1
    if bias is not None:
        r.bias_tokens, r.bias_values, r.n_bias = bias[0].data_ptr(), bias[1].data_ptr(), bias[2]
    if mask is not None:
        m = mask
        if m.dtype not in (torch.int32, torch.uint32):
            raise TypeError("mask must be packed 32-bit words (int32 or uint32)")
        if m.dim() == 1:
            m = m.unsqueeze(0).expand(B, -1)
        m = keep(m.to(dev).contiguous())
        if m.shape[1] < (V + 31) // 32:
            raise ValueError("mask has fewer than ceil(vocab/32) words per row")
        r.mask = m.data_ptr()
        r.mask_stride = m.shape[1]
    if forced is not None:
        f = keep(torch.as_tensor(forced, device=dev).to(torch.int32).reshape(B).contiguous())
        r.forced = f.data_ptr()
    keep(logits)
    return r


def _noise(B: int, V: int, seed: int, offset: int, row_base: int, gumbel, uniform, keep: _Keep, dev):
    n = L.Noise()
    if gumbel is not None or uniform is not None:
        n.mode = L.PM_NOISE_INJECTED
        if gumbel is not None:
            g = keep(gumbel.to(device=dev, dtype=torch.float32).contiguous())
            n.gumbel, n.gumbel_stride = g.data_ptr(), g.shape[1]
        if uniform is not None:
            u = keep(uniform.to(device=dev, dtype=torch.float64).contiguous())
            n.uniform = u.data_ptr()
    else:
        n.mode = L.PM_NOISE_PHILOX
    n.seed = seed & 0xFFFFFFFFFFFFFFFF
    n.offset = offset & 0xFFFFFFFFFFFFFFFF
    n.row_base = row_base
    return n


def sample_rows(logits: torch.Tensor, sampler: Union[SamplerSettings, Sequence[SamplerSettings]] = None,
                processors: Union[ProcessorSettings, Sequence[ProcessorSettings], None] = None,
                history: Optional[torch.Tensor] = None, history_len=None, mask: Optional[torch.Tensor] = None,
                seed: int = 0, offset: int = 0, row_base: int = 0, gumbel: Optional[torch.Tensor] = None,
                uniform: Optional[torch.Tensor] = None, return_lse: bool = False,
                return_logprob: bool = False, survivors: int = 0, return_status: bool = False,
                forced: Optional[torch.Tensor] = None):
    """Processors + log-softmax + sampler for every row, one fused pass.

    Returns a dict with "tokens" [B] int32 (and "lse", "logprob",
    "surv_ids"/"surv_probs"/"n_surv" when asked), all on the logits' device,
    enqueued on the current stream.  "status" [B] is non-zero for a row whose
    settings fell outside the fused path's limits.  forced [B] (-1: none)
    restricts a row to one token (the ThinkBudget hook).
    """
    keep = _Keep()
    lib = L.load()
    dev = logits.device
    r = build_rows(logits, sampler, processors, history, history_len, mask, keep, forced=forced)
    B, V = r.rows, r.vocab
    nz = _noise(B, V, seed, offset, row_base, gumbel, uniform, keep, dev)
    out = L.SampleOut()
    tokens = torch.empty(B, dtype=torch.int32, device=dev)
    out.tokens = tokens.data_ptr()
    res = {"tokens": tokens}
    if return_lse:
        res["lse"] = torch.empty(B, dtype=torch.float32, device=dev)
        out.lse = res["lse"].data_ptr()
    if return_logprob:
        res["logprob"] = torch.empty(B, dtype=torch.float32, device=dev)
        out.token_logprob = res["logprob"].data_ptr()
    if survivors:
        res["surv_ids"] = torch.empty((B, survivors), dtype=torch.int32, device=dev)
        res["surv_probs"] = torch.empty((B, survivors), dtype=torch.float32, device=dev)
        res["n_surv"] = torch.empty(B, dtype=torch.int32, device=dev)
        out.surv_ids = res["surv_ids"].data_ptr()
        out.surv_probs = res["surv_probs"].data_ptr()
        out.n_surv = res["n_surv"].data_ptr()
        out.surv_cap = survivors
    nbytes = lib.pm_sample_workspace_bytes(C.byref(r))
    if nbytes == 0:
        L.check(L.PM_ERR_UNSUPPORTED, "pm_sample_workspace_bytes")
    stream = torch.cuda.current_stream(dev)
    ws = workspace(nbytes, dev, stream)
    rc = lib.pm_sample_rows(C.byref(r), C.byref(nz), C.byref(out), ws.data_ptr(), ws.numel(), stream.cuda_stream)
    L.check(rc, "pm_sample_rows")
    if return_status:
        res["status"] = status_view(ws, r)
    return res


def status_view(ws: torch.Tensor, r: L.Rows) -> torch.Tensor:
    # the status array opens the workspace
    return ws[: 4 * r.rows].view(torch.int32).clone()


def apply_processors(logits: torch.Tensor, processors=None, history=None, history_len=None, mask=None,
                     out: Optional[torch.Tensor] = None, return_status: bool = False):
    """Processed logits (fp32): logit bias, penalties, then the mask.  With
    return_status, (logits, per-row status [B] int32)."""
    keep = _Keep()
    lib = L.load()
    dev = logits.device
    r = build_rows(logits, SamplerSettings(), processors, history, history_len, mask, keep)
    if out is None:
        out = torch.empty((r.rows, r.vocab), dtype=torch.float32, device=dev)
    nbytes = lib.pm_processors_workspace_bytes(C.byref(r))
    stream = torch.cuda.current_stream(dev)
    ws = workspace(nbytes, dev, stream)
    rc = lib.pm_apply_processors(C.byref(r), out.data_ptr(), out.stride(0), ws.data_ptr(), ws.numel(),
                                 stream.cuda_stream)
    L.check(rc, "pm_apply_processors")
    if return_status:
        # the status array opens the workspace; only the penalty prep writes it
        st = status_view(ws, r) if r.hist else torch.zeros(r.rows, dtype=torch.int32, device=dev)
        return out, st
    return out


def logprobs(logits: torch.Tensor, processors=None, history=None, history_len=None, mask=None,
             out: Optional[torch.Tensor] = None):
    """(processed logits - row log-sum-exp, lse) in fp32."""
    keep = _Keep()
    lib = L.load()
    dev = logits.device
    r = build_rows(logits, SamplerSettings(), processors, history, history_len, mask, keep)
    if out is None:
        out = torch.empty((r.rows, r.vocab), dtype=torch.float32, device=dev)
    lse = torch.empty(r.rows, dtype=torch.float32, device=dev)
    nbytes = lib.pm_processors_workspace_bytes(C.byref(r))
    stream = torch.cuda.current_stream(dev)
    ws = workspace(nbytes, dev, stream)
    rc = lib.pm_logprobs(C.byref(r), out.data_ptr(), out.stride(0), lse.data_ptr(), ws.data_ptr(), ws.numel(),
                         stream.cuda_stream)
    L.check(rc, "pm_logprobs")
    return out, lse


def argmax_confidence(logits: torch.Tensor, processors=None, history=None, mask=None):
    """Greedy token and its softmax probability per row: the reduction of
    each MTP draft-chain step (reference pagedmoe/mtp.py:731-746, argmax and
    max(softmax)), in one pass: tokens [B] int32, confidence [B] fp32."""
    res = sample_rows(logits, SamplerSettings(temp=0.0), processors, history=history, mask=mask,
                      return_logprob=True)
    return res["tokens"], torch.exp(res["logprob"])

