"""Draft acceptance of a verify pass, batched over requests.

The reference verifies one request at a time in Python
(pagedmoe/lookup_decode.py:319-373 `_verify`, pagedmoe/verify_decode.py:880-921):
for each of the k + 1 target rows it runs the processors over history + [y] +
drafts[:i], takes log-probabilities, samples, and keeps the drafts while the
samples equal them.  `verify` does that for every request of a batch in one
call of the C ABI (pm_verify): the rows' processors, samples and the accept
scan all run on the device.

mode "match" is the reference's rule.  mode "residual" is speculative
rejection sampling (not in the reference): it needs the draft model's logits
and keeps the target distribution exact at any temperature.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib as L
from .engine import _i64, _Keep, cached_size, prepare, workspace

_MODES = {"match": L.PM_VERIFY_MATCH, "residual": L.PM_VERIFY_RESIDUAL}


def _per_row(x, B: int, K1: int):
    """Per-request settings expanded to the request's k + 1 rows."""
    if isinstance(x, (list, tuple)) and not (isinstance(x, tuple) and hasattr(x, "_fields")):
        if len(x) != B:
            raise ValueError(f"expected {B} per-request settings, got {len(x)}")
        return [s for s in x for _ in range(K1)]
    return x


def verify(target_logits: torch.Tensor, drafts: torch.Tensor, y: torch.Tensor, sampler=None, processors=None,
           history: Optional[torch.Tensor] = None, history_len=None, mask: Optional[torch.Tensor] = None,
           mode: str = "match", draft_logits: Optional[torch.Tensor] = None, seed: int = 0, offset: int = 0,
           row_base: int = 0, gumbel: Optional[torch.Tensor] = None, uniform: Optional[torch.Tensor] = None,
           u_accept: Optional[torch.Tensor] = None, u_residual: Optional[torch.Tensor] = None,
           return_row_tokens: bool = False, return_status: bool = False):
    """Accept drafts against the target rows of a verify pass.

    target_logits  [B, k+1, V] (or [B*(k+1), V]) fp32/bf16 on the device:
                   row i scores drafts[:, i] (i < k) or gives the bonus token.
    drafts [B, k], y [B]: the drafted ids and the token before them.
    history [B, H] (+ history_len [B]): ids the penalties see before y.
    mask [B*(k+1), W] or [B, k+1, W]: packed allowed-token words per row.
    draft_logits [B, k, V] (residual mode): the draft model's logits q.
    gumbel [B*(k+1), V], uniform [B*(k+1), 2], u_accept [B, k], u_residual
    [B]: injected noise; otherwise Philox keyed by (seed, offset, row).

    Returns {"tokens": [B, k+1] int32 (accepted tokens then -1),
    "n_accepted": [B] int32} plus "row_tokens" [B, k+1] and "status"
    [B*(k+1)] when asked.  Enqueued on the current stream.
    """
    if mode not in _MODES:
        raise ValueError(f"mode must be one of {sorted(_MODES)}")
    if not isinstance(drafts, torch.Tensor):
        drafts = torch.as_tensor(drafts)
    if drafts.dim() == 1:
        drafts = drafts.unsqueeze(0)
    B, k = drafts.shape
    K1 = k + 1
    V = target_logits.shape[-1]
    x = target_logits.reshape(B * K1, V)
    dev = x.device
    keep = _Keep()
    if drafts.device != dev or drafts.dtype != torch.int32 or not drafts.is_contiguous():
        drafts = keep(drafts.to(device=dev, dtype=torch.int32).contiguous())
    procs = _per_row(processors, B, K1)
    # the feed (y, then the drafts) extends the history the penalties read;
    # without a penalty nothing reads it
    plist = procs if isinstance(procs, list) else [procs]
    pens = any(p is not None and p.penalties_on for p in plist)
    feed = None
    if pens:
        y = torch.as_tensor(y).reshape(B).to(device=dev, dtype=torch.int32)
        feed = keep(torch.cat([y[:, None], drafts], dim=1).contiguous())
    if mask is not None and mask.dim() == 3:
        mask = mask.reshape(B * K1, -1)
    q = prepare(x, _per_row(sampler, B, K1), procs, history, history_len, mask, keep,
                feed=feed, feed_group=K1 if pens else 0)
    g = None if gumbel is None else keep(gumbel.to(device=dev, dtype=torch.float32).contiguous())
    u = None if uniform is None else keep(uniform.to(device=dev, dtype=torch.float64).contiguous())
    dl = None
    if mode == "residual" and k > 0:
        if draft_logits is None:
            raise ValueError("residual mode needs the draft logits")
        dl = draft_logits.reshape(B * k, V)
        if dl.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError(f"draft_logits must be float32 or bfloat16, got {dl.dtype}")
        if dl.stride(1) != 1:
            dl = dl.contiguous()
        if dl.device != dev:
            raise ValueError("draft_logits must be on the target logits' device")
        keep(dl)
    ua = ur = None
    if u_accept is not None:
        ua = keep(torch.as_tensor(u_accept).to(device=dev, dtype=torch.float64).reshape(B, k).contiguous())
    if u_residual is not None:
        ur = keep(torch.as_tensor(u_residual).to(device=dev, dtype=torch.float64).reshape(B).contiguous())
    E = L.ext()
    m = _MODES[mode]
    key = ("verify", dev.index, q.logits.shape, q.logits.stride(0), q.logits.dtype, q.per_row, q.flags_any,
           q.top_k_max, None if q.hist is None else q.hist.shape, None if q.feed is None else q.feed.shape,
           q.feed_group, None if q.mask is None else q.mask.shape, m, drafts.shape)
    nbytes = cached_size(key, lambda: E.verify_workspace_bytes(q.logits, q.params, q.per_row, q.flags_any,
                                                               q.top_k_max, q.hist, q.feed, q.feed_group, q.mask, m,
                                                               drafts))
    if nbytes == 0:
        L.check(L.PM_ERR_UNSUPPORTED, "pm_verify_workspace_bytes")
    ws = workspace(nbytes, dev)
    out = E.verify(q.logits, q.params, q.per_row, q.flags_any, q.top_k_max, q.hist, q.hist_len, q.feed,
                   q.feed_group, q.bias_tok, q.bias_val, q.mask, _i64(seed), _i64(offset), row_base, g, u, m, drafts,
                   dl, ua, ur, return_row_tokens, ws)
    res = {"tokens": out[0], "n_accepted": out[1]}
    if return_row_tokens:
        res["row_tokens"] = out[2]
    if return_status:
        res["status"] = ws[: 4 * B * K1].view(torch.int32).clone()
    return res
