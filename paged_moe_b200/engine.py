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
    # the raw handle of the current stream: no Stream object per call
    raw = stream.cuda_stream if stream is not None else torch._C._cuda_getCurrentRawStream(device.index)
    key = (device.index, raw)
    buf = _ws_cache.get(key)
    if buf is not None and buf.numel() >= nbytes:
        return buf
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
        return buf


_size_cache: dict = {}


def cached_size(key, query) -> int:
    """A workspace size that depends only on shapes and settings (key),
    queried from the library once per key."""
    v = _size_cache.get(key)
    if v is None:
        v = int(query())
        with _ws_lock:
            if len(_size_cache) > 1024:
                _size_cache.clear()
            _size_cache[key] = v
    return v


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


_DEFAULT_SAMPLER = SamplerSettings()
_DEFAULT_PROCESSORS = ProcessorSettings()


def _params_for(dev: torch.device, sampler, processors, B: int, V: int):
    """(device params tensor, flags_any, top_k_max, per_row), cached by settings."""
    single = not isinstance(sampler, (list, tuple)) and not isinstance(processors, (list, tuple))
    if single:
        s = sampler if sampler is not None else _DEFAULT_SAMPLER
        p = processors if processors is not None else _DEFAULT_PROCESSORS
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


def device_of(logits: torch.Tensor) -> torch.device:
    """The CUDA device a call on these logits runs on (the current one for
    host logits)."""
    return logits.device if logits.is_cuda else torch.device("cuda", torch.cuda.current_device())


def _gather_reads_host(logits: torch.Tensor, mask) -> bool:
    """Whether the masked gather pass can read these host logits in place:
    pinned (so the device reaches them at the same address), a mask given,
    and values the pass fetches as aligned 4-byte words (fp32, or bf16 rows of
    even stride)."""
    if logits.is_cuda or mask is None or not logits.is_pinned():
        return False
    if mask.is_cuda is False and not mask.is_pinned():
        return False
    if logits.dtype == torch.float32:
        return True
    return logits.dtype == torch.bfloat16 and logits.stride(0) % 2 == 0 and logits.data_ptr() % 4 == 0


class Prepared:
    """The tensors of one call, ready for the C ABI: every one on the call's
    device (host logits and mask only when the masked pass reads them in
    place), contiguous, int32 ids."""

    __slots__ = ("dev", "logits", "params", "flags_any", "top_k_max", "per_row", "procs", "hist", "hist_len",
                 "feed", "feed_group", "bias_tok", "bias_val", "mask", "forced")


def prepare(logits: torch.Tensor, sampler, processors, history, history_len, mask, keep: _Keep,
            feed: Optional[torch.Tensor] = None, feed_group: int = 0,
            forced: Optional[torch.Tensor] = None, allow_host: bool = False) -> Prepared:
    """Logits on a CUDA device are used in place.  With allow_host, pinned
    host logits with a mask stay in host memory when the masked gather pass
    takes them and no row has an unbounded filter: the pass reads the mask and
    the allowed logits over the host link, nothing else; other host logits are
    copied to the device first."""
    if logits.dim() != 2:
        raise ValueError("logits must be [rows, vocab]")
    dev = device_of(logits)
    _dtype_code(logits)
    B, V = logits.shape
    q = Prepared()
    q.dev = dev
    q.params, q.flags_any, q.top_k_max, q.per_row, q.procs, bias = _params_for(dev, sampler, processors, B, V)
    if not logits.is_cuda:
        if not logits.is_pinned():
            raise ValueError("logits must be a CUDA tensor or pinned host memory")
        # in place only when the gather pass is the one reader: rows with an
        # unbounded filter may need the wide pass, which streams whole rows
        in_place = (allow_host and logits.stride(1) == 1 and not (q.flags_any & L.PM_F_UNBOUNDED)
                    and _gather_reads_host(logits, mask))
        if not in_place:
            logits = keep(logits.to(dev, non_blocking=True))
    if logits.stride(1) != 1:
        logits = keep(logits.contiguous())
    q.logits = keep(logits)
    q.hist = q.hist_len = q.feed = q.bias_tok = q.bias_val = q.mask = q.forced = None
    q.feed_group = 0
    if history is not None and any(p.penalties_on for p in q.procs):
        h = history
        if h.dim() == 1:
            h = h.unsqueeze(0).expand(B if feed is None else B // feed_group, -1)
        q.hist = keep(h.to(device=dev, dtype=torch.int32).contiguous())
        if history_len is not None:
            q.hist_len = keep(torch.as_tensor(history_len, dtype=torch.int32, device=dev).contiguous())
    if feed is not None:
        q.feed = keep(feed.to(device=dev, dtype=torch.int32).contiguous())
        q.feed_group = feed_group
        if q.hist is None:
            # the feed alone is the history
            q.hist = keep(torch.zeros((B // feed_group, 1), dtype=torch.int32, device=dev))
            q.hist_len = keep(torch.zeros(B // feed_group, dtype=torch.int32, device=dev))
    if bias is not None:
        q.bias_tok, q.bias_val = bias[0], bias[1]
    if mask is not None:
        m = mask
        if m.dtype not in (torch.int32, torch.uint32):
            raise TypeError("mask must be packed 32-bit words (int32 or uint32)")
        if m.dim() == 1:
            m = m.unsqueeze(0).expand(B, -1)
        if m.is_cuda or logits.is_cuda:
            m = keep(m.to(dev, non_blocking=True).contiguous())
        else:  # host logits read in place: the mask too
            m = keep(m if m.is_contiguous() else m.contiguous().pin_memory())
        if m.shape[1] < (V + 31) // 32:
            raise ValueError("mask has fewer than ceil(vocab/32) words per row")
        q.mask = m
    if forced is not None:
        q.forced = keep(torch.as_tensor(forced, device=dev).to(torch.int32).reshape(B).contiguous())
    return q


def _i64(v: int) -> int:
    """A 64-bit unsigned value as the signed int64 with the same bits."""
    v &= 0xFFFFFFFFFFFFFFFF
    return v - (1 << 64) if v >= (1 << 63) else v


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def build_rows(logits: torch.Tensor, sampler, processors, history, history_len, mask, keep: _Keep,
               feed: Optional[torch.Tensor] = None, feed_group: int = 0,
               forced: Optional[torch.Tensor] = None, allow_host: bool = False) -> L.Rows:
    """The pm_rows struct (ctypes) for a call; see prepare()."""
    q = prepare(logits, sampler, processors, history, history_len, mask, keep, feed, feed_group, forced, allow_host)
    B, V = q.logits.shape
    r = L.Rows()
    r.logits = q.logits.data_ptr()
    r.dtype = _dtype_code(q.logits)
    r.rows = B
    r.vocab = V
    r.row_stride = q.logits.stride(0)
    r.params = q.params.data_ptr()
    r.params_per_row = 1 if q.per_row else 0
    r.flags_any = q.flags_any
    r.top_k_max = q.top_k_max
    if q.hist is not None:
        r.hist, r.hist_stride, r.hist_len = q.hist.data_ptr(), q.hist.shape[1], _ptr(q.hist_len)
    if q.feed is not None:
        r.feed, r.feed_group = q.feed.data_ptr(), q.feed_group
    if q.bias_tok is not None:
        r.bias_tokens, r.bias_values, r.n_bias = q.bias_tok.data_ptr(), q.bias_val.data_ptr(), q.bias_tok.numel()
    if q.mask is not None:
        r.mask, r.mask_stride = q.mask.data_ptr(), q.mask.shape[1]
    r.forced = _ptr(q.forced)
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

    logits [B, V] on a CUDA device, or in pinned host memory: with a mask,
    the masked pass then reads only the mask and the allowed logits from
    host memory (no copy of the rows); without one they are copied first.

    Returns a dict with "tokens" [B] int32 (and "lse", "logprob",
    "surv_ids"/"surv_probs"/"n_surv" when asked), all on the logits' device,
    enqueued on the current stream.  "status" [B] is non-zero for a row whose
    settings fell outside the fused path's limits.  forced [B] (-1: none)
    restricts a row to one token (the ThinkBudget hook).
    """
    keep = _Keep()
    E = L.ext()
    q = prepare(logits, sampler, processors, history, history_len, mask, keep, forced=forced, allow_host=True)
    dev = q.dev
    g = u = None
    if gumbel is not None:
        g = keep(gumbel.to(device=dev, dtype=torch.float32).contiguous())
    if uniform is not None:
        u = keep(uniform.to(device=dev, dtype=torch.float64).contiguous())
    key = ("sample", dev.index, q.logits.shape, q.logits.stride(0), q.logits.dtype, q.per_row, q.flags_any,
           q.top_k_max, None if q.hist is None else q.hist.shape, None if q.mask is None else q.mask.shape)
    nbytes = cached_size(key, lambda: E.sample_workspace_bytes(q.logits, q.params, q.per_row, q.flags_any,
                                                              q.top_k_max, q.hist, q.mask))
    if nbytes == 0:
        L.check(L.PM_ERR_UNSUPPORTED, "pm_sample_workspace_bytes")
    ws = workspace(nbytes, dev)
    out = E.sample_rows(q.logits, q.params, q.per_row, q.flags_any, q.top_k_max, q.hist, q.hist_len, q.bias_tok,
                        q.bias_val, q.mask, q.forced, _i64(seed), _i64(offset), row_base, g, u, return_lse,
                        return_logprob, survivors, ws)
    res = {"tokens": out[0]}
    if return_lse:
        res["lse"] = out[1]
    if return_logprob:
        res["logprob"] = out[2]
    if survivors:
        res["surv_ids"], res["surv_probs"], res["n_surv"] = out[3], out[4], out[5]
    if return_status:
        res["status"] = ws[: 4 * q.logits.shape[0]].view(torch.int32).clone()
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
    dev = device_of(logits)
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
    dev = device_of(logits)
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



def _lmhead_struct(hidden: torch.Tensor, weight: torch.Tensor, keep: _Keep) -> L.LmHead:
    if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
        raise ValueError("hidden must be [tokens, hidden_size] and weight [vocab, hidden_size]")
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("the LM head takes bf16 hidden states and weights")
    if not (hidden.is_cuda and weight.is_cuda) or hidden.device != weight.device:
        raise ValueError("hidden and weight must be on the same CUDA device")
    h = hidden if hidden.stride(1) == 1 and hidden.stride(0) % 8 == 0 else keep(hidden.contiguous())
    w = weight if weight.stride(1) == 1 and weight.stride(0) % 8 == 0 else keep(weight.contiguous())
    s = L.LmHead()
    s.hidden, s.n_tokens, s.hidden_size, s.hidden_stride = h.data_ptr(), h.shape[0], h.shape[1], h.stride(0)
    s.weight, s.weight_stride = w.data_ptr(), w.stride(0)
    return s


def lmhead_logits(hidden: torch.Tensor, weight: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """logits = hidden @ weight.T (bf16 in, fp32 accumulate) on the tensor
    cores: the LM head of the reference's decode step (pagedmoe/
    verify_decode.py:821, :887).  The same kernel as lmhead_sample, so these
    are the logits the fused call samples from."""
    keep = _Keep()
    lib = L.load()
    s = _lmhead_struct(hidden, weight, keep)
    V = weight.shape[0]
    if out is None:
        out = torch.empty((hidden.shape[0], (V + 3) // 4 * 4), dtype=torch.float32, device=hidden.device)[:, :V]
    stream = torch.cuda.current_stream(hidden.device)
    rc = lib.pm_lmhead_logits(C.byref(s), V, out.data_ptr(), out.stride(0), stream.cuda_stream)
    L.check(rc, "pm_lmhead_logits")
    return out


def lmhead_sample(hidden: torch.Tensor, weight: torch.Tensor,
                  sampler: Union[SamplerSettings, Sequence[SamplerSettings]] = None,
                  processors: Union[ProcessorSettings, Sequence[ProcessorSettings], None] = None,
                  history: Optional[torch.Tensor] = None, history_len=None,
                  mask: Optional[torch.Tensor] = None, seed: int = 0, offset: int = 0, row_base: int = 0,
                  gumbel: Optional[torch.Tensor] = None, return_lse: bool = False, return_logprob: bool = False,
                  survivors: int = 0, return_status: bool = False):
    """The LM head fused with the sampler: the tokens (and the other outputs
    of sample_rows) that sample_rows would give on lmhead_logits(hidden,
    weight), with the logits never written to device memory.  Greedy rows and
    rows with top_k (plus temperature, top_p, min_p), the processors (logit
    bias, repetition / presence / frequency penalties over `history`) and an
    optional mask; unbounded top-p / min-p and whole-vocabulary draws raise
    (use lmhead_logits + sample_rows)."""
    keep = _Keep()
    lib = L.load()
    s = _lmhead_struct(hidden, weight, keep)
    dev = hidden.device
    B, V = hidden.shape[0], weight.shape[0]
    # the rows need a [B, V] logits view only for their shape: one row, broadcast
    stand_in = torch.empty((1, V), dtype=torch.float32, device=dev).expand(B, V)
    r = build_rows(stand_in, sampler, processors, history, history_len, mask, keep)
    r.logits = None
    n = _noise(B, V, seed, offset, row_base, gumbel, None, keep, dev)
    o = L.SampleOut()
    tokens = torch.empty(B, dtype=torch.int32, device=dev)
    o.tokens = tokens.data_ptr()
    res = {"tokens": tokens}
    if return_lse:
        res["lse"] = torch.empty(B, dtype=torch.float32, device=dev)
        o.lse = res["lse"].data_ptr()
    if return_logprob:
        res["logprob"] = torch.empty(B, dtype=torch.float32, device=dev)
        o.token_logprob = res["logprob"].data_ptr()
    if survivors:
        res["surv_ids"] = torch.empty((B, survivors), dtype=torch.int32, device=dev)
        res["surv_probs"] = torch.empty((B, survivors), dtype=torch.float32, device=dev)
        res["n_surv"] = torch.empty(B, dtype=torch.int32, device=dev)
        o.surv_ids, o.surv_probs, o.n_surv = (res["surv_ids"].data_ptr(), res["surv_probs"].data_ptr(),
                                              res["n_surv"].data_ptr())
        o.surv_cap = survivors
    nbytes = lib.pm_lmhead_sample_workspace_bytes(C.byref(s), C.byref(r))
    if nbytes == 0:
        L.check(L.PM_ERR_UNSUPPORTED, "pm_lmhead_sample_workspace_bytes")
    stream = torch.cuda.current_stream(dev)
    ws = workspace(nbytes, dev, stream)
    rc = lib.pm_lmhead_sample(C.byref(s), C.byref(r), C.byref(n), C.byref(o), ws.data_ptr(), ws.numel(),
                              stream.cuda_stream)
    L.check(rc, "pm_lmhead_sample")
    if return_status:
        res["status"] = status_view(ws, r)
    return res
