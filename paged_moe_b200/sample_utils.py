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


class Sampler:
    """The callable make_sampler returns.  Each call draws fresh noise: the
    Philox offset advances by one per call (the reference's sampler draws from
    mlx's global random state, verify_decode.py:838)."""

    def __init__(self, settings: SamplerSettings, seed: Optional[int] = None):
        self.settings = settings
        self.seed = _fresh_seed() if seed is None else int(seed)
        self.offset = 0
        self._lock = threading.Lock()

    def __call__(self, logprobs: torch.Tensor) -> torch.Tensor:
        x = logprobs
        squeeze = x.dim() == 1
        if squeeze:
            x = x.unsqueeze(0)
        with self._lock:
            off = self.offset
            self.offset += 1
        res = engine.sample_rows(x, self.settings, seed=self.seed, offset=off)
        tok = res["tokens"]
        return tok[0] if squeeze else tok


def make_sampler(temp: float = 0.0, top_p: float = 0.0, min_p: float = 0.0, min_tokens_to_keep: int = 1,
                 top_k: int = 0, xtc_probability: float = 0.0, xtc_threshold: float = 0.0,
                 xtc_special_tokens: Optional[List[int]] = None, *, seed: Optional[int] = None) -> Sampler:
    """A sampler that takes log-probabilities [N, V] and returns tokens [N].

    temp == 0 is argmax.  Otherwise top_k, then top_p, then min_p filter the
    log-probabilities and the categorical draw runs at `temp`.
    """
    if xtc_probability > 0.0:
        raise NotImplementedError("XTC sampling is not part of this build's token-selection path")
    return Sampler(SamplerSettings(temp=float(temp), top_p=float(top_p), min_p=float(min_p),
                                   min_tokens_to_keep=int(min_tokens_to_keep), top_k=int(top_k)), seed=seed)


class _Processor:
    """One logits processor: proc(tokens, logits) -> logits (fp32)."""

    def __init__(self, settings: ProcessorSettings, name: str):
        self.settings = settings
        self.__name__ = name

    def __call__(self, tokens, logits: torch.Tensor) -> torch.Tensor:
        x = logits
        squeeze = x.dim() == 1
        if squeeze:
            x = x.unsqueeze(0)
        t = torch.as_tensor(tokens, device=x.device).reshape(-1).to(torch.int32)
        if t.numel() == 0 and not self.settings.logit_bias:
            return logits
        hist = t.unsqueeze(0).expand(x.shape[0], -1) if t.numel() else None
        out = engine.apply_processors(x, self.settings, history=hist)
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
