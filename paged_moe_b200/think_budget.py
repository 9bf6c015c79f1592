"""ThinkBudget on the device: closes a reasoning block at a character budget
by forcing the close text one token per step (reference
pagedmoe/think_budget.py:60-109).

The reference builds per-token tables (decoded length, sentence-end flag)
once per tokenizer and evaluates the budget with array ops per row; here the
tables live on the device and one kernel (pm_think_budget) evaluates every
row of a batch, producing the forced token per row that the sampling pass
takes through pm_rows.forced.  `__call__(seq, logits)` keeps the reference's
logits-processor call shape for single rows.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib as L

SLACK_TOKENS = 48  # tokens to wait for a sentence end past the budget (reference think_budget.py:36)
# characters that end a sentence when a decoded piece ends with one of them
# (trailing spaces ignored; reference think_budget.py:37)
_SENTENCE_END = frozenset(".!?:\n")
_DECODE_CHUNK = 8192


class PieceTables:
    """Per-id tables of one tokenizer on one device: how many characters the
    id decodes to, and whether that piece ends a sentence.  Decoding the
    whole vocabulary takes a while (about half a second for 250k ids), so
    the tables are made once per (tokenizer, device) and shared."""

    _cache: Dict[Tuple[int, str], "PieceTables"] = {}

    def __init__(self, lens: torch.Tensor, ends: torch.Tensor):
        self.lens, self.ends = lens, ends

    @classmethod
    def of(cls, tokenizer, device) -> "PieceTables":
        key = (id(tokenizer), str(device))
        hit = cls._cache.get(key)
        if hit is None:
            lens, ends = cls._build(tokenizer)
            hit = cls(torch.from_numpy(lens).to(device), torch.from_numpy(ends).to(device))
            cls._cache[key] = hit
        return hit

    @staticmethod
    def _pieces(tokenizer, lo: int, hi: int) -> List[str]:
        ids = [[i] for i in range(lo, hi)]
        try:
            return list(tokenizer.batch_decode(ids))
        except Exception:  # a tokenizer without a batched decode (or one that refuses an id list)
            return [tokenizer.decode(i) for i in range(lo, hi)]

    @classmethod
    def _build(cls, tokenizer):
        n = max(tokenizer.get_vocab().values()) + 1
        lens = np.zeros(n, dtype=np.int32)
        ends = np.zeros(n, dtype=np.uint8)
        for lo in range(0, n, _DECODE_CHUNK):
            hi = min(n, lo + _DECODE_CHUNK)
            for off, piece in enumerate(cls._pieces(tokenizer, lo, hi)):
                lens[lo + off] = len(piece)
                tail = piece.rstrip(" ")
                ends[lo + off] = bool(tail) and tail[-1] in _SENTENCE_END
        return lens, ends


def piece_tables(tokenizer, device) -> tuple:
    """(decoded length, sentence-end flag) per id, as device tensors."""
    t = PieceTables.of(tokenizer, device)
    return t.lens, t.ends


def _close_sequence(tokenizer, close: str, end_id: int) -> List[int]:
    """The ids the budget forces, one per step: the close text's encoding,
    which must finish on the think end tag (otherwise forcing it would never
    close the block)."""
    ids = list(tokenizer.encode(close, add_special_tokens=False))
    if not ids or ids[-1] != end_id:
        raise ValueError(f"the close text must encode to ids ending with the think end id {end_id}, got {ids}")
    return ids


class ThinkBudget:
    """Closes a reasoning block once it passes `chars` characters: after the
    next sentence end (or `slack` tokens), the close text is forced one token
    per step.  With `open_in_prompt` the template opened the block in the
    prompt and every generated token counts; otherwise counting starts after
    the model's own think start token, and a reply without one is left
    alone."""

    def __init__(self, tokenizer, chars: int, close: str, open_in_prompt: bool = True, device=None,
                 slack: int = SLACK_TOKENS):
        self.device = torch.device("cuda" if device is None else device)
        self.chars = int(chars)
        self.slack = int(slack)
        self.open_in_prompt = bool(open_in_prompt)
        self.end_id = int(tokenizer.think_end_id)
        start = getattr(tokenizer, "think_start_id", None)  # absent: the template has no start tag
        self.start_id = -1 if start is None else int(start)
        self.close_ids = _close_sequence(tokenizer, close, self.end_id)
        self.close = torch.tensor(self.close_ids, dtype=torch.int32, device=self.device)
        self.lens, self.ends = piece_tables(tokenizer, self.device)
        self.base: Optional[int] = None  # sequence length at the first call (the prompt's tail)
        self._budgets: Dict[int, torch.Tensor] = {}

    def forced(self, gen: torch.Tensor, gen_len: Optional[torch.Tensor] = None,
               chars: Optional[Sequence[int]] = None) -> torch.Tensor:
        """Forced token per row (-1: none) for generated ids [B, T] (after the prompt)."""
        g = torch.as_tensor(gen, device=self.device)
        if g.dim() == 1:
            g = g.unsqueeze(0)
        g = g.to(torch.int32).contiguous()
        B, T = g.shape
        gl = None if gen_len is None else torch.as_tensor(gen_len, device=self.device).to(torch.int32).contiguous()
        if chars is not None:
            ch = torch.tensor(list(chars), dtype=torch.int32, device=self.device)
        else:  # one budget for every row: a cached device tensor (no host copy per call)
            ch = self._budgets.get(B)
            if ch is None:
                ch = self._budgets[B] = torch.full((B,), self.chars, dtype=torch.int32, device=self.device)
        out = torch.empty(B, dtype=torch.int32, device=self.device)
        start = -1 if self.open_in_prompt else (self.start_id if self.start_id >= 0 else 0x7fffffff)
        rc = L.load().pm_think_budget(g.data_ptr() if g.numel() else None, None if gl is None else gl.data_ptr(), T,
                                      B, self.lens.data_ptr(), self.ends.data_ptr(), self.lens.numel(),
                                      ch.data_ptr(), self.close.data_ptr(), self.close.numel(), self.end_id, start,
                                      self.slack, out.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        L.check(rc, "pm_think_budget")
        return out

    def __call__(self, seq, logits: torch.Tensor) -> torch.Tensor:
        """The reference processor's call: logits unchanged, or only the forced token kept."""
        seq = torch.as_tensor(seq, device=self.device).reshape(-1)
        if self.base is None:
            self.base = int(seq.shape[0])  # the first call carries the prompt's last token(s)
            return logits
        n = int(seq.shape[0]) - self.base
        if n <= 0:
            return logits
        f = self.forced(seq[self.base:].unsqueeze(0))[0]
        keep = torch.arange(logits.shape[-1], device=logits.device) == f.to(logits.device)
        out = torch.where(keep, logits, torch.full_like(logits, float("-inf")))
        return torch.where(f >= 0, out, logits)
