"""Drop-in sampler and logits-processor factories over torch CUDA tensors.

Same keyword signatures and call contracts as mlx-lm 0.31.3's
``mlx_lm.sample_utils.make_sampler`` / ``make_logits_processors``, which the
reference builds its decode steps from (run.py:53, walkthrough/tour.py:396,
pagedmoe/pretrain_sidecar.py:645, and mlx-lm's server after
pagedmoe/server.py:2929-2930):

    sampler(logprobs [N, V]) -> tokens [N]            (verify_decode.py:839, :903)
    proc(tokens [T], logits [1, V]) -> logits [1, V]  (verify_decode.py:830-831)

Inputs are torch tensors on a CUDA device; the work runs in libpm_sample.so.
"""

from __future__ import annotations

import os
import threading
from typing import Callable, List, Optional

import torch

from . import engine
from .params import ProcessorSettings, SamplerSettings

_seed_lock = threading.Lock()


def _fresh_seed() -> int:
    with _seed_lock:
        return int.from_bytes(os.urandom(8), "little")


# per-row status bits that mean the row's result cannot be trusted
_ROW_ERRORS = {
    2: "a penalty window is longer than the library's history cap",
    4: "a logits tile copy did not complete within its wait limit",
}


class StatusCheck:
    """Raises RuntimeError for rows whose status carries an error bit.

    mode True: after every call, one 4-byte device-to-host read (waits for
    the call).  mode "deferred": the read is queued into pinned memory and
    checked at the start of the next call (or by check()), so a pipelined
    decode loop never waits for it.  mode False: no check."""

    def __init__(self, mode=True):
        if mode not in (True, False, "deferred"):
            raise ValueError("check_status must be True, False or 'deferred'")
        self.mode = mode
        self._host = None
        self._event = None
        self._what = ""

    @staticmethod
    def _raise(bits: int, what: str):
        msgs = [m for b, m in _ROW_ERRORS.items() if bits & b]
        if msgs:
            raise RuntimeError(f"{what}: " + "; ".join(msgs))

    def check(self):
        if self._event is not None:
            self._event.synchronize()
            bits = int(self._host[0])
            self._event = None
            self._raise(bits, self._what)

    def after(self, status: torch.Tensor, what: str):
        if self.mode is False or status is None or status.numel() == 0:
            return
        bits = torch.bitwise_and(status, 2).amax() + torch.bitwise_and(status, 4).amax()  # OR of bits 2 and 4
        if self.mode is True:
            self._raise(int(bits.item()), what)
            return
        if self._host is None:
            self._host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._host.copy_(bits.to(torch.int32).reshape(1), non_blocking=True)
        self._event = torch.cuda.Event()
        self._event.record(torch.cuda.current_stream(status.device))
        self._what = what


class Sampler:
    """The callable make_sampler returns.  Each call draws fresh noise: the
    Philox offset advances by one per call (the reference's sampler draws from
    mlx's global random state, verify_decode.py:838).  Rows whose status
    carries an error bit raise RuntimeError (see StatusCheck)."""

    def __init__(self, settings: SamplerSettings, seed: Optional[int] = None, check_status=True):
        self.settings = settings
        self.seed = _fresh_seed() if seed is None else int(seed)
        self.offset = 0
        self._lock = threading.Lock()
        self.status = StatusCheck(check_status)

    def __call__(self, logprobs: torch.Tensor) -> torch.Tensor:
        self.status.check()
        x = logprobs
        squeeze = x.dim() == 1
        if squeeze:
            x = x.unsqueeze(0)
        with self._lock:
            off = self.offset
            self.offset += 1
        res = engine.sample_rows(x, self.settings, seed=self.seed, offset=off, return_status=True)
        self.status.after(res["status"], "sampler")
        tok = res["tokens"]
        return tok[0] if squeeze else tok

    def check(self):
        """Raise now for an error a deferred check has not reported yet."""
        self.status.check()


def make_sampler(temp: float = 0.0, top_p: float = 0.0, min_p: float = 0.0, min_tokens_to_keep: int = 1,
                 top_k: int = 0, xtc_probability: float = 0.0, xtc_threshold: float = 0.0,
                 xtc_special_tokens: Optional[List[int]] = None, *, seed: Optional[int] = None,
                 check_status=True) -> Sampler:
    """A sampler that takes log-probabilities [N, V] and returns tokens [N].

    temp == 0 is argmax.  Otherwise top_k, then top_p, then min_p filter the
    log-probabilities and the categorical draw runs at `temp`.
    """
    if xtc_probability > 0.0:
        raise NotImplementedError("XTC sampling is not part of this build's token-selection path")
    return Sampler(SamplerSettings(temp=float(temp), top_p=float(top_p), min_p=float(min_p),
                                   min_tokens_to_keep=int(min_tokens_to_keep), top_k=int(top_k)), seed=seed,
                   check_status=check_status)


class _Processor:
    """One logits processor: proc(tokens, logits) -> logits (fp32).  Rows
    whose status carries an error bit raise RuntimeError (see StatusCheck)."""

    def __init__(self, settings: ProcessorSettings, name: str, check_status=True):
        self.settings = settings
        self.__name__ = name
        self.status = StatusCheck(check_status)

    def __call__(self, tokens, logits: torch.Tensor) -> torch.Tensor:
        self.status.check()
        x = logits
        squeeze = x.dim() == 1
        if squeeze:
            x = x.unsqueeze(0)
        t = torch.as_tensor(tokens, device=x.device).reshape(-1).to(torch.int32)
        if t.numel() == 0 and not self.settings.logit_bias:
            return logits
        hist = t.unsqueeze(0).expand(x.shape[0], -1) if t.numel() else None
        out, status = engine.apply_processors(x, self.settings, history=hist, return_status=True)
        self.status.after(status, self.__name__)
        return out[0] if squeeze else out


def make_logits_processors(logit_bias: Optional[dict] = None, repetition_penalty: Optional[float] = None,
                           repetition_context_size: Optional[int] = 20, presence_penalty: Optional[float] = None,
                           presence_context_size: Optional[int] = 20, frequency_penalty: Optional[float] = None,
                           frequency_context_size: Optional[int] = 20) -> List[Callable]:
    """The processor list mlx-lm builds: logit bias, repetition, presence,
    frequency (each only when set and non-zero), applied in that order."""
    procs: List[Callable] = []
    if logit_bias:
        procs.append(_Processor(ProcessorSettings.make(logit_bias=logit_bias), "logit_bias_processor"))
    if repetition_penalty and repetition_penalty != 0.0:
        if repetition_penalty < 0 or not isinstance(repetition_penalty, (int, float)):
            raise ValueError(f"penalty must be a non-negative float, got {repetition_penalty}")
        procs.append(_Processor(ProcessorSettings(repetition_penalty=float(repetition_penalty),
                                                  repetition_context_size=int(repetition_context_size or 0)),
                                "repetition_penalty_processor"))
    if presence_penalty and presence_penalty != 0.0:
        procs.append(_Processor(ProcessorSettings(presence_penalty=float(presence_penalty),
                                                  presence_context_size=int(presence_context_size or 0)),
                                "presence_penalty_processor"))
    if frequency_penalty and frequency_penalty != 0.0:
        procs.append(_Processor(ProcessorSettings(frequency_penalty=float(frequency_penalty),
                                                  frequency_context_size=int(frequency_context_size or 0)),
                                "frequency_penalty_processor"))
    return procs
