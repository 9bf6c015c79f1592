"""Vocabulary-sharded sampling (a tensor-parallel LM head leaves every GPU with
a contiguous slice of each row's logits).

Each rank summarizes its slice (pm_shard_summarize: best greedy key, top-K
candidate keys with global ids, tile statistics, per-tile draws for
whole-vocabulary rows), one all-gather brings every summary to every rank,
and the merge (pm_shard_merge) gives every rank the row's tokens -- the same
tokens and log-sum-exp as sampling the unsharded rows.  No reference code:
PagedMoE samples on one device.
"""

from __future__ import annotations

import ctypes as C
import dataclasses
from typing import Optional

import torch

from . import _lib as L
from .engine import _Keep, _noise, _params_for, build_rows, workspace
from .params import ProcessorSettings


def shard_width(vocab_total: int, n_shards: int) -> int:
    """Ids per shard: ceil(V / n) rounded up to whole 1024-token tiles."""
    w = -(-vocab_total // n_shards)
    w = -(-w // 1024) * 1024 if n_shards > 1 else w
    if vocab_total - (n_shards - 1) * w <= 0:
        raise ValueError(f"{vocab_total} ids do not split into {n_shards} tile-aligned shards")
    return w


@dataclasses.dataclass(frozen=True)
class ShardSpec:
    index: int
    n_shards: int
    vocab_total: int
    width: int

    @staticmethod
    def of(index: int, n_shards: int, vocab_total: int) -> "ShardSpec":
        return ShardSpec(index, n_shards, vocab_total, shard_width(vocab_total, n_shards))

    @property
    def lo(self) -> int:
        return self.index * self.width

    @property
    def hi(self) -> int:
        return min(self.lo + self.width, self.vocab_total)

    def c(self) -> L.ShardArgs:
        s = L.ShardArgs()
        s.shard_index, s.n_shards, s.vocab_total, s.shard_width = self.index, self.n_shards, self.vocab_total, self.width
        return s


def _local_processors(p: Optional[ProcessorSettings], spec: ShardSpec):
    """The logit bias of the slice, ids shifted to it (penalty ids stay global)."""
    if p is None or not p.logit_bias:
        return p
    lb = tuple((t - spec.lo, v) for t, v in p.logit_bias if spec.lo <= t < spec.hi) or None
    return dataclasses.replace(p, logit_bias=lb)


def summarize(logits_shard: torch.Tensor, spec: ShardSpec, sampler=None, processors=None, history=None,
              history_len=None, mask: Optional[torch.Tensor] = None, seed: int = 0, offset: int = 0,
              row_base: int = 0, gumbel=None, uniform=None) -> torch.Tensor:
    """This shard's summary [rows * row_bytes] uint8 (enqueued on the current stream).

    logits_shard [B, hi - lo]; mask: the full-vocabulary packed words
    [B, ceil(V/32)] (the slice's words are taken here); gumbel [B, V] over
    the full vocabulary when noise is injected."""
    if logits_shard.shape[-1] != spec.hi - spec.lo:
        raise ValueError(f"shard {spec.index} holds {spec.hi - spec.lo} ids, got {logits_shard.shape[-1]}")
    keep = _Keep()
    if isinstance(processors, (list, tuple)):
        procs = [_local_processors(p, spec) for p in processors]
    else:
        procs = _local_processors(processors, spec)
    if mask is not None:
        mask = mask[..., spec.lo // 32: -(-spec.hi // 32)]
    r = build_rows(logits_shard, sampler, procs, history, history_len, mask, keep)
    nz = _noise(r.rows, spec.vocab_total, seed, offset, row_base, gumbel, uniform, keep, logits_shard.device)
    lib = L.load()
    sh = spec.c()
    nbytes = lib.pm_shard_summary_bytes(C.byref(r), C.byref(sh))
    if nbytes == 0 and r.rows > 0:
        L.check(L.PM_ERR_UNSUPPORTED, "pm_shard_summary_bytes")
    out = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=logits_shard.device)
    wsb = lib.pm_sample_workspace_bytes(C.byref(r))
    stream = torch.cuda.current_stream(logits_shard.device)
    ws = workspace(wsb, logits_shard.device, stream)
    rc = lib.pm_shard_summarize(C.byref(r), C.byref(sh), C.byref(nz), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                stream.cuda_stream)
    L.check(rc, "pm_shard_summarize")
    return out[:nbytes]


def merge(summaries: torch.Tensor, spec: ShardSpec, n_rows: int, sampler=None, processors=None, seed: int = 0,
          offset: int = 0, row_base: int = 0, gumbel=None, uniform=None, return_lse: bool = False,
          return_logprob: bool = False, survivors: int = 0, return_status: bool = False):
    """Tokens of the rows from every shard's summary (concatenated in shard order)."""
    dev = summaries.device
    keep = _Keep()
    params, flags_any, top_k_max, per_row, _, _ = _params_for(dev, sampler, processors, n_rows, spec.vocab_total)
    r = L.Rows()
    r.dtype = L.PM_DTYPE_F32
    r.rows = n_rows
    r.vocab = spec.vocab_total
    r.row_stride = spec.vocab_total
    r.params = params.data_ptr()
    r.params_per_row = 1 if per_row else 0
    r.flags_any = flags_any
    r.top_k_max = top_k_max
    nz = _noise(n_rows, spec.vocab_total, seed, offset, row_base, gumbel, uniform, keep, dev)
    out = L.SampleOut()
    tokens = torch.empty(n_rows, dtype=torch.int32, device=dev)
    out.tokens = tokens.data_ptr()
    res = {"tokens": tokens}
    if return_lse:
        res["lse"] = torch.empty(n_rows, dtype=torch.float32, device=dev)
        out.lse = res["lse"].data_ptr()
    if return_logprob:
        res["logprob"] = torch.empty(n_rows, dtype=torch.float32, device=dev)
        out.token_logprob = res["logprob"].data_ptr()
    if survivors:
        res["surv_ids"] = torch.empty((n_rows, survivors), dtype=torch.int32, device=dev)
        res["surv_probs"] = torch.empty((n_rows, survivors), dtype=torch.float32, device=dev)
        res["n_surv"] = torch.empty(n_rows, dtype=torch.int32, device=dev)
        out.surv_ids, out.surv_probs = res["surv_ids"].data_ptr(), res["surv_probs"].data_ptr()
        out.n_surv, out.surv_cap = res["n_surv"].data_ptr(), survivors
    status = torch.empty(max(n_rows, 1), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    rc = L.load().pm_shard_merge(C.byref(r), C.byref(spec.c()), C.byref(nz), summaries.data_ptr(), C.byref(out),
                                 status.data_ptr(), status.numel() * 4, stream.cuda_stream)
    L.check(rc, "pm_shard_merge")
    keep(summaries)
    if return_status:
        res["status"] = status[:n_rows]
    return res


def gather_summaries(summary: torch.Tensor, group=None) -> torch.Tensor:
    """Every rank's summary, in rank (= shard) order, on every rank."""
    import torch.distributed as dist
    n = dist.get_world_size(group)
    if dist.get_backend(group) == "nccl":
        out = torch.empty(n * summary.numel(), dtype=summary.dtype, device=summary.device)
        dist.all_gather_into_tensor(out, summary, group=group)
        return out
    parts = [torch.empty_like(summary) for _ in range(n)]
    dist.all_gather(parts, summary, group=group)
    return torch.cat(parts)


def _rows_of(x, idx, per_row_dim: int):
    """Rows idx of a per-row argument: a tensor of per_row_dim dimensions
    (fewer: shared by every row), or a sequence of per-row settings."""
    if x is None:
        return None
    if isinstance(x, torch.Tensor):
        return x[idx.to(x.device)] if x.dim() == per_row_dim else x
    if isinstance(x, (list, tuple)):
        return [x[int(i)] for i in idx.tolist()]
    return x


def _finish_wide(res: dict, full_rows, n_rows: int, vocab: int, sampler, processors, history, history_len, mask,
                 seed: int, offset: int, row_base: int, gumbel, uniform, merge_kw: dict) -> dict:
    """Rows the records cannot finish (status bit 1: an unbounded top-p /
    min-p keeps more tokens than the candidate lists hold) get the unsharded
    pass on their whole rows: the same kernels, so the same tokens, log-sum-
    exp and status bits as sampling the unsharded rows.  full_rows(idx) gives
    those rows' [len(idx), V] logits (an all-gather of the flagged rows'
    slices on a process group).  Philox rows keep their own row ids."""
    from . import engine
    st = res.get("status")
    if st is None:
        return res
    # only rows with an unbounded filter can be flagged: no host sync otherwise
    _, flags_any, _, _, _, _ = _params_for(st.device, sampler, processors, n_rows, vocab)
    if not (flags_any & L.PM_F_UNBOUNDED):
        return res
    idx = torch.nonzero(st[:n_rows] & 1).flatten()
    if idx.numel() == 0:
        return res
    rows = full_rows(idx)
    for j, r in enumerate(idx.tolist()):
        one = idx[j:j + 1]
        hl = history_len
        if hl is not None and not isinstance(hl, torch.Tensor):
            hl = torch.as_tensor(hl, dtype=torch.int32)
        sub = engine.sample_rows(
            rows[j:j + 1], _rows_of(sampler, one, 0), _rows_of(processors, one, 0),
            history=_rows_of(history, one, 2), history_len=_rows_of(hl, one, 1), mask=_rows_of(mask, one, 2),
            seed=seed, offset=offset, row_base=row_base + r, gumbel=_rows_of(gumbel, one, 2),
            uniform=_rows_of(uniform, one, 2),
            return_lse=bool(merge_kw.get("return_lse")), return_logprob=bool(merge_kw.get("return_logprob")),
            survivors=int(merge_kw.get("survivors") or 0), return_status=True)
        res["tokens"][r] = sub["tokens"][0]
        res["status"][r] = sub["status"][0]
        for k in ("lse", "logprob", "n_surv"):
            if k in res and k in sub:
                res[k][r] = sub[k][0]
        for k in ("surv_ids", "surv_probs"):
            if k in res and k in sub:
                res[k][r] = sub[k][0]
    return res


def gather_rows(logits_shard: torch.Tensor, idx: torch.Tensor, spec: ShardSpec, group=None) -> torch.Tensor:
    """Rows idx of the full [B, V] logits on every rank: each rank's slice of
    those rows (padded to the shard width), one all-gather, the slices end to
    end."""
    import torch.distributed as dist
    n = dist.get_world_size(group)
    part = torch.zeros((idx.numel(), spec.width), dtype=logits_shard.dtype, device=logits_shard.device)
    part[:, : spec.hi - spec.lo] = logits_shard[idx.to(logits_shard.device)]
    if dist.get_backend(group) == "nccl":
        out = torch.empty((n,) + tuple(part.shape), dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(out, part, group=group)
        parts = list(out.unbind(0))
    else:
        parts = [torch.empty_like(part) for _ in range(n)]
        dist.all_gather(parts, part, group=group)
    cols = []
    for i, p_ in enumerate(parts):
        sp = ShardSpec.of(i, n, spec.vocab_total)
        cols.append(p_[:, : sp.hi - sp.lo])
    return torch.cat(cols, dim=1).contiguous()


def sample_vocab_sharded(logits_shard: torch.Tensor, sampler=None, processors=None, group=None, history=None,
                         history_len=None, mask=None, seed: int = 0, offset: int = 0, row_base: int = 0,
                         gumbel=None, uniform=None, vocab_total: Optional[int] = None, **merge_kw):
    """One step of vocabulary-sharded sampling: this rank (rank r of the group)
    holds ids [r * width, ...) of every row; returns the rows' tokens on every rank."""
    import torch.distributed as dist
    n = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if vocab_total is None:
        raise ValueError("vocab_total is required")
    spec = ShardSpec.of(rank, n, vocab_total)
    s = summarize(logits_shard, spec, sampler, processors, history, history_len, mask, seed, offset, row_base,
                  gumbel, uniform)
    allsum = gather_summaries(s, group)
    want_status = bool(merge_kw.pop("return_status", False))
    B = logits_shard.shape[0]
    res = merge(allsum, spec, B, sampler, processors, seed, offset, row_base, gumbel, uniform, return_status=True,
                **merge_kw)
    res = _finish_wide(res, lambda idx: gather_rows(logits_shard, idx, spec, group), B, vocab_total, sampler,
                       processors, history, history_len, mask, seed, offset, row_base, gumbel, uniform, merge_kw)
    if not want_status:
        res.pop("status", None)
    return res


def emulate(logits: torch.Tensor, n_shards: int, sampler=None, processors=None, history=None, history_len=None,
            mask=None, seed: int = 0, offset: int = 0, row_base: int = 0, gumbel=None, uniform=None, **merge_kw):
    """All shards of [B, V] logits on this device, summaries concatenated as
    the all-gather would: the sharded path without a process group."""
    V = logits.shape[-1]
    parts = []
    for i in range(n_shards):
        spec = ShardSpec.of(i, n_shards, V)
        parts.append(summarize(logits[:, spec.lo:spec.hi], spec, sampler, processors, history, history_len, mask,
                               seed, offset, row_base, gumbel, uniform))
    spec0 = ShardSpec.of(0, n_shards, V)
    want_status = bool(merge_kw.pop("return_status", False))
    B = logits.shape[0]
    res = merge(torch.cat(parts), spec0, B, sampler, processors, seed, offset, row_base, gumbel, uniform,
                return_status=True, **merge_kw)
    res = _finish_wide(res, lambda idx: logits[idx.to(logits.device)], B, V, sampler, processors, history,
                       history_len, mask, seed, offset, row_base, gumbel, uniform, merge_kw)
    if not want_status:
        res.pop("status", None)
    return res
