"""Host-side sampler / processor settings and their per-row C struct.

The settings mirror the keyword arguments of mlx-lm 0.31.3's make_sampler and
make_logits_processors (the reference builds its samplers with them:
run.py:53, walkthrough/tour.py:396, pagedmoe/pretrain_sidecar.py:645; and the
server sets them from pagedmoe/sampling.py:121-135).  Every scalar reaches the
device as the fp32 value mlx-lm's arithmetic would see: Python evaluates
1/temp, 1 - top_p and log(min_p) in double, and mlx then rounds the scalar to
fp32 when it meets an fp32 array.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib as L


def f32(x: float) -> float:
    return float(np.float32(x))


@dataclass(frozen=True)
class SamplerSettings:
    """make_sampler(temp, top_p, min_p, min_tokens_to_keep, top_k) keywords."""
    temp: float = 0.0
    top_p: float = 0.0
    min_p: float = 0.0
    min_tokens_to_keep: int = 1
    top_k: int = 0

    @property
    def greedy(self) -> bool:
        return self.temp == 0

    @property
    def top_p_on(self) -> bool:
        return 0.0 < self.top_p < 1.0

    @property
    def min_p_on(self) -> bool:
        return self.min_p != 0.0

    @property
    def filtered(self) -> bool:
        return not self.greedy and (self.top_k > 0 or self.top_p_on or self.min_p_on)


@dataclass(frozen=True)
class ProcessorSettings:
    """make_logits_processors(logit_bias, repetition_penalty, ...) keywords."""
    logit_bias: Optional[tuple] = None  # ((token, bias), ...) -- hashable form of the dict
    repetition_penalty: Optional[float] = None
    repetition_context_size: int = 20
    presence_penalty: Optional[float] = None
    presence_context_size: int = 20
    frequency_penalty: Optional[float] = None
    frequency_context_size: int = 20

    def __post_init__(self):
        # the device lists are bucketed by token id: ascending, distinct ids
        # (a dict, or pairs in any order, come out the same)
        lb = self.logit_bias
        if lb:
            items = lb.items() if isinstance(lb, dict) else lb
            norm = tuple(sorted((int(t), float(v)) for t, v in items))
            if len({t for t, _ in norm}) != len(norm):
                raise ValueError("logit_bias names a token more than once")
            object.__setattr__(self, "logit_bias", norm)
        elif lb is not None:
            object.__setattr__(self, "logit_bias", None)

    @staticmethod
    def make(logit_bias: Optional[dict] = None, **kw) -> "ProcessorSettings":
        lb = tuple(sorted((int(k), float(v)) for k, v in logit_bias.items())) if logit_bias else None
        return ProcessorSettings(logit_bias=lb, **kw)

    @property
    def rep_on(self) -> bool:
        return bool(self.repetition_penalty) and self.repetition_penalty != 0.0

    @property
    def pres_on(self) -> bool:
        return bool(self.presence_penalty) and self.presence_penalty != 0.0

    @property
    def freq_on(self) -> bool:
        return bool(self.frequency_penalty) and self.frequency_penalty != 0.0

    @property
    def penalties_on(self) -> bool:
        return self.rep_on or self.pres_on or self.freq_on

    @property
    def any_on(self) -> bool:
        return self.penalties_on or bool(self.logit_bias)


def validate(s: SamplerSettings, p: ProcessorSettings, vocab: int) -> None:
    """The argument checks mlx-lm's filters and processors make."""
    if s.min_p_on and not (0.0 <= s.min_p <= 1.0):
        raise ValueError(f"`min_p` has to be a float in the [0, 1] interval, but is {s.min_p}")
    if s.top_k > 0 and not s.top_k < vocab:
        raise ValueError(f"`top_k` has to be an integer in the (0, {vocab}] interval, but is {s.top_k}.")
    if s.min_tokens_to_keep < 1 and s.min_p_on:
        raise ValueError("`min_tokens_to_keep` has to be a positive integer")
    for name in ("repetition_penalty",):
        v = getattr(p, name)
        if v is not None and (not isinstance(v, (int, float)) or v < 0):
            raise ValueError(f"penalty must be a non-negative float, got {v}")


def row_struct(s: SamplerSettings, p: ProcessorSettings) -> L.RowParams:
    r = L.RowParams()
    flags = 0
    if s.greedy:
        flags |= L.PM_F_GREEDY
    else:
        if s.top_p_on:
            flags |= L.PM_F_TOP_P
        if s.min_p_on:
            flags |= L.PM_F_MIN_P
        if (s.top_p_on or s.min_p_on) and s.top_k <= 0:
            flags |= L.PM_F_UNBOUNDED
        if not s.filtered:
            flags |= L.PM_F_FULL
    if p.rep_on:
        flags |= L.PM_F_REP
    if p.pres_on:
        flags |= L.PM_F_PRES
    if p.freq_on:
        flags |= L.PM_F_FREQ
    r.flags = flags
    r.inv_temperature = f32(1.0 / s.temp) if s.temp != 0 else 0.0
    r.top_k = int(s.top_k) if (s.top_k > 0 and not s.greedy) else 0
    r.top_p_comp = f32(1.0 - s.top_p)
    r.log_min_p = f32(math.log(s.min_p)) if s.min_p > 0 else float("-inf")
    r.min_tokens_to_keep = int(s.min_tokens_to_keep)
    r.repetition_penalty = f32(p.repetition_penalty or 0.0)
    r.repetition_context_size = int(p.repetition_context_size)
    r.presence_penalty = f32(p.presence_penalty or 0.0)
    r.presence_context_size = int(p.presence_context_size)
    r.frequency_penalty = f32(p.frequency_penalty or 0.0)
    r.frequency_context_size = int(p.frequency_context_size)
    return r


def pack_rows(samplers: Sequence[SamplerSettings], procs: Sequence[ProcessorSettings]):
    """(bytes of the pm_row_params array, flags_any, top_k_max, per_row)."""
    structs = [row_struct(s, p) for s, p in zip(samplers, procs)]
    arr = (L.RowParams * len(structs))(*structs)
    flags_any = 0
    for st in structs:
        flags_any |= st.flags
    top_k_max = max((st.top_k for st in structs), default=0)
    return bytes(arr), flags_any, top_k_max
