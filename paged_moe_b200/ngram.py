"""Batched n-gram drafts on the device (pm_draft_ngram).

The reference drafts one request at a time by rescanning its context in
Python (pagedmoe/lookup_decode.py:184-221 draft_ngram); `draft_ngram_batch`
does every request of a batch in one launch, and `draft_ngram` keeps the
reference's call shape (a token list in, a list out) for single requests.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib as L

NGRAM_MIN = 3  # reference config.py:1289 LOOKUP_NGRAM_MIN
NGRAM_MAX = 8  # reference config.py:1288 LOOKUP_NGRAM_MAX


def draft_ngram_batch(history: torch.Tensor, k: int, history_len: Optional[torch.Tensor] = None,
                      n_min: int = NGRAM_MIN, n_max: int = NGRAM_MAX):
    """history [B, H] int ids on the device (+ lengths [B]).  Returns
    (drafts [B, k] int32 with -1 after each draft, lengths [B], matched n [B])."""
    if history.dim() == 1:
        history = history.unsqueeze(0)
    dev = history.device
    h = history.to(dtype=torch.int32).contiguous()
    B, H = h.shape
    hl = None
    if history_len is not None:
        hl = torch.as_tensor(history_len, device=dev).to(torch.int32).contiguous()
    drafts = torch.empty((B, max(k, 0)), dtype=torch.int32, device=dev)
    lens = torch.empty(B, dtype=torch.int32, device=dev)
    used = torch.empty(B, dtype=torch.int32, device=dev)
    rc = L.load().pm_draft_ngram(h.data_ptr(), None if hl is None else hl.data_ptr(), H, B, k, n_min, n_max,
                                 drafts.data_ptr() if drafts.numel() else None, lens.data_ptr(), used.data_ptr(),
                                 torch.cuda.current_stream(dev).cuda_stream)
    L.check(rc, "pm_draft_ngram")
    return drafts, lens, used


def draft_ngram(tokens, k: int, n_min: int = NGRAM_MIN, n_max: int = NGRAM_MAX, device=None) -> list:
    """The reference's draft_ngram(tokens, k) call shape, on the device."""
    toks = list(tokens)
    if k <= 0 or len(toks) == 0:
        return []
    dev = torch.device(device) if device is not None else torch.device("cuda")
    h = torch.tensor(toks, dtype=torch.int32, device=dev)
    drafts, lens, _ = draft_ngram_batch(h, k, n_min=n_min, n_max=n_max)
    n = int(lens[0].item())
    return drafts[0, :n].tolist()
