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

from typing import Optional, Sequence

import torch

from . import _lib as L

SLACK_TOKENS = 48  # reference think_budget.py:36
_ENDS = (".", "!", "?", ":", "\n")  # reference think_budget.py:37
_TABLES: dict = {}


def piece_tables(tokenizer, device) -> tuple:
    """Decoded length and sentence-end flag per id, built once per tokenizer."""
    key = (id(tokenizer), str(device))
    got = _TABLES.get(key)
    if got is not None:
        return got
    n = max(tokenizer.get_vocab().values()) + 1
    ids = [[i] for i in range(n)]
    try:
        pieces = tokenizer.batch_decode(ids)
    except Exception:
        pieces = [tokenizer.decode(i) for i in ids]
    lens = torch.tensor([len(p) for p in pieces], dtype=torch.int32, device=device)
    ends = torch.tensor([p.rstrip(" ").endswith(_ENDS) for p in pieces], dtype=torch.uint8, device=device)
    _TABLES[key] = (lens, ends)
    return lens, ends


class ThinkBudget:
    def __init__(self, tokenizer, chars: int, close: str, open_in_prompt: bool = True, device=None,
                 slack: int = SLACK_TOKENS):
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.chars = int(chars)
        self.open_in_prompt = bool(open_in_prompt)
        self.end_id = int(tokenizer.think_end_id)
        start = getattr(tokenizer, "think_start_id", None)
        self.start_id = int(start) if start is not None else -1
        ids = tokenizer.encode(close, add_special_tokens=False)
        if not ids or ids[-1] != self.end_id:
            raise ValueError("close text must end with the think end tag")
        self.close_ids = list(ids)
        self.close = torch.tensor(ids, dtype=torch.int32, device=self.device)
        self.slack = int(slack)
        self.base: Optional[int] = None
        self.lens, self.ends = piece_tables(tokenizer, self.device)

    def forced(self, gen: torch.Tensor, gen_len: Optional[torch.Tensor] = None,
               chars: Optional[Sequence[int]] = None) -> torch.Tensor:
        """Forced token per row (-1: none) for generated ids [B, T] (after the prompt)."""
        g = torch.as_tensor(gen, device=self.device)
        if g.dim() == 1:
            g = g.unsqueeze(0)
        g = g.to(torch.int32).contiguous()
        B, T = g.shape
        gl = None if gen_len is None else torch.as_tensor(gen_len, device=self.device).to(torch.int32).contiguous()
        ch = torch.tensor(list(chars) if chars is not None else [self.chars] * B, dtype=torch.int32,
                          device=self.device)
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
