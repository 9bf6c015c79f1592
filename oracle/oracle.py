"""ctypes driver of pm_oracle.c -- TEST INFRASTRUCTURE ONLY (see package doc).

Host-side parameter rounding here restates how the reference's Python floats
reach mlx-lm's fp32 arithmetic: every scalar becomes an fp32 constant
(1/temp, 1 - top_p and log(min_p) are first evaluated in double, as Python
does, then rounded).
"""

from __future__ import annotations

import ctypes as C
import math
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

__all__ = [
    "lib", "build", "Proc", "Sampler", "expf", "expf_shift", "q52", "exp64", "log64", "philox4x32_10",
    "gumbel_from_word", "u53", "row_lse", "tile_stats", "process", "logprobs", "sample",
    "verify", "bf16_to_f32", "philox_gumbel", "philox_uniform", "window_start",
    "shard_sample", "draft_ngram",
]

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libpm_oracle.so")
_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> str:
    """Compile pm_oracle.c into libpm_oracle.so (make, in this folder)."""
    src = os.path.join(_HERE, "pm_oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


class _Proc(C.Structure):
    _fields_ = [
        ("rep_penalty", C.c_float), ("rep_ctx", C.c_int32), ("rep_on", C.c_int32),
        ("pres_penalty", C.c_float), ("pres_ctx", C.c_int32), ("pres_on", C.c_int32),
        ("freq_penalty", C.c_float), ("freq_ctx", C.c_int32), ("freq_on", C.c_int32),
    ]


class _Sampler(C.Structure):
    _fields_ = [
        ("greedy", C.c_int32), ("inv_temp", C.c_float), ("top_k", C.c_int32),
        ("top_p_on", C.c_int32), ("top_p_comp", C.c_float), ("min_p_on", C.c_int32),
        ("log_min_p", C.c_float), ("min_keep", C.c_int32),
    ]


class _Noise(C.Structure):
    _fields_ = [
        ("mode", C.c_int32), ("gumbel", C.POINTER(C.c_float)), ("uniform", C.POINTER(C.c_double)),
        ("seed", C.c_uint64), ("offset", C.c_uint64), ("row", C.c_uint32),
    ]


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = C.CDLL(_SO)
            P = C.c_void_p
            L.orc_expf.restype = C.c_float
            L.orc_expf.argtypes = [C.c_float]
            L.orc_q52.restype = C.c_uint64
            L.orc_q52.argtypes = [C.c_float]
            L.orc_exp64.restype = C.c_double
            L.orc_exp64.argtypes = [C.c_double]
            L.orc_log64.restype = C.c_double
            L.orc_log64.argtypes = [C.c_double]
            L.orc_philox4x32_10.argtypes = [P, P, P]
            L.orc_gumbel_from_word.restype = C.c_float
            L.orc_gumbel_from_word.argtypes = [C.c_uint32]
            L.orc_u53.restype = C.c_uint64
            L.orc_u53.argtypes = [C.c_uint64, C.c_uint64, C.c_uint32, C.c_uint32]
            L.orc_row_lse.restype = C.c_float
            L.orc_row_lse.argtypes = [P, C.c_int]
            L.orc_tile_stats.argtypes = [P, C.c_int, P, P]
            L.orc_combine_tiles.restype = C.c_float
            L.orc_combine_tiles.argtypes = [P, P, C.c_int]
            L.orc_sample_row.restype = C.c_int
            L.orc_sample_row.argtypes = [P, C.c_int, C.c_float, P, P, P, P, P, C.c_int]
            common = [P, C.c_int, C.c_int, P, C.c_int, P, P, P, P, C.c_int, P, C.c_int]
            L.orc_sample_batch.restype = C.c_int
            L.orc_sample_batch.argtypes = common + [P, C.c_int, P, P, C.c_uint64, C.c_uint64,
                                                    C.c_uint32, P, P, P, P, P, C.c_int]
            L.orc_logprobs_batch.restype = C.c_int
            L.orc_logprobs_batch.argtypes = common + [P, P]
            L.orc_process_batch.restype = C.c_int
            L.orc_process_batch.argtypes = common + [P]
            L.orc_expf_shift.restype = None
            L.orc_expf_shift.argtypes = [P, C.c_int, C.c_float, P]
            _lib = L
    return _lib


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# --------------------------------------------------------------------------
# parameters
# --------------------------------------------------------------------------

def _f32(x: float) -> float:
    return float(np.float32(x))


@dataclass
class Proc:
    """mlx-lm make_logits_processors keyword set (defaults 20, as mlx-lm)."""
    repetition_penalty: Optional[float] = None
    repetition_context_size: int = 20
    presence_penalty: Optional[float] = None
    presence_context_size: int = 20
    frequency_penalty: Optional[float] = None
    frequency_context_size: int = 20
    logit_bias: Optional[dict] = None

    def c(self) -> _Proc:
        s = _Proc()
        s.rep_on = int(bool(self.repetition_penalty) and self.repetition_penalty != 0.0)
        s.rep_penalty = _f32(self.repetition_penalty or 0.0)
        s.rep_ctx = int(self.repetition_context_size)
        s.pres_on = int(bool(self.presence_penalty) and self.presence_penalty != 0.0)
        s.pres_penalty = _f32(self.presence_penalty or 0.0)
        s.pres_ctx = int(self.presence_context_size)
        s.freq_on = int(bool(self.frequency_penalty) and self.frequency_penalty != 0.0)
        s.freq_penalty = _f32(self.frequency_penalty or 0.0)
        s.freq_ctx = int(self.frequency_context_size)
        return s

    def bias_arrays(self):
        if not self.logit_bias:
            return None, None, 0
        toks = np.array(list(self.logit_bias.keys()), dtype=np.int32)
        vals = np.array([_f32(v) for v in self.logit_bias.values()], dtype=np.float32)
        return toks, vals, len(toks)


@dataclass
class Sampler:
    """mlx-lm make_sampler keyword set."""
    temp: float = 0.0
    top_p: float = 0.0
    min_p: float = 0.0
    min_tokens_to_keep: int = 1
    top_k: int = 0

    def c(self) -> _Sampler:
        s = _Sampler()
        s.greedy = int(self.temp == 0)
        s.inv_temp = _f32(1.0 / self.temp) if self.temp != 0 else 0.0
        s.top_k = int(self.top_k) if self.top_k > 0 else 0
        s.top_p_on = int(0.0 < self.top_p < 1.0)
        s.top_p_comp = _f32(1.0 - self.top_p)
        s.min_p_on = int(self.min_p != 0.0)
        s.log_min_p = _f32(math.log(self.min_p)) if self.min_p > 0 else float("-inf")
        s.min_keep = int(self.min_tokens_to_keep)
        return s

    @property
    def filtered(self) -> bool:
        return self.top_k > 0 or 0.0 < self.top_p < 1.0 or self.min_p != 0.0


# --------------------------------------------------------------------------
# scalar helpers (for known-answer tests)
# --------------------------------------------------------------------------

def expf(d: float) -> float:
    return lib().orc_expf(d)


def expf_shift(x: np.ndarray, c: float) -> np.ndarray:
    """expf(fl32(x - c)) of every element (the scalar expf, vectorised in C)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_expf_shift(_p(x), x.size, float(np.float32(c)), _p(out))
    return out


def q52(d: float) -> int:
    return lib().orc_q52(d)


def exp64(d: float) -> float:
    return lib().orc_exp64(d)


def log64(z: float) -> float:
    return lib().orc_log64(z)


def philox4x32_10(ctr: Sequence[int], key: Sequence[int]) -> list:
    c = np.array(ctr, dtype=np.uint32)
    k = np.array(key, dtype=np.uint32)
    o = np.zeros(4, dtype=np.uint32)
    lib().orc_philox4x32_10(_p(c), _p(k), _p(o))
    return [int(v) for v in o]


def gumbel_from_word(w: int) -> float:
    return lib().orc_gumbel_from_word(w)


def u53(seed: int, offset: int, row: int, stream: int) -> int:
    return lib().orc_u53(seed, offset, row, stream)


def philox_gumbel(seed: int, offset: int, row: int, tokens) -> np.ndarray:
    """Gumbel noise the Philox mode draws for (row, token)."""
    out = np.empty(len(tokens), dtype=np.float32)
    key = [seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF]
    for i, t in enumerate(tokens):
        t = int(t)
        w = philox4x32_10([t >> 2, row, offset & 0xFFFFFFFF, (offset >> 32) & 0xFFFFFFFF], key)[t & 3]
        out[i] = gumbel_from_word(w)
    return out


def philox_uniform(seed: int, offset: int, row: int, stream: int) -> float:
    """fp64 uniform in [0,1) the Philox mode draws for (row, stream)."""
    return u53(seed, offset, row, stream) * 2.0 ** -53


def window_start(H: int, ctx: int) -> int:
    if ctx > 0:
        return max(H - ctx, 0)
    if ctx == 0:
        return 0
    return min(-ctx, H)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) to the fp32 values they denote (exact)."""
    return (a.astype(np.uint32) << 16).view(np.float32)


def row_lse(x: np.ndarray) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return lib().orc_row_lse(_p(x), x.shape[-1])


def tile_stats(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    nt = (x.shape[-1] + 1023) // 1024
    m = np.empty(nt, dtype=np.float32)
    s = np.empty(nt, dtype=np.uint64)
    lib().orc_tile_stats(_p(x), x.shape[-1], _p(m), _p(s))
    return m, s


# --------------------------------------------------------------------------
# batched drivers (row ranges on host threads; ctypes drops the GIL)
# --------------------------------------------------------------------------

def _nthreads(n: Optional[int]) -> int:
    return n if n else (os.cpu_count() or 1)


def _prep(logits, hist, hist_len, proc, mask):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = logits.shape
    if hist is not None:
        hist = np.ascontiguousarray(hist, dtype=np.int32)
        if hist.ndim == 1:
            hist = np.broadcast_to(hist, (B, hist.shape[0])).copy()
        hist_len = (np.full(B, hist.shape[1], dtype=np.int32) if hist_len is None
                    else np.ascontiguousarray(hist_len, dtype=np.int32))
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.uint32)
    proc = proc or Proc()
    return logits, B, V, hist, hist_len, proc, mask


def _ranges(B, nthreads):
    n = max(1, min(B, nthreads))
    step = (B + n - 1) // n
    return [(a, min(B, a + step)) for a in range(0, B, step)]


def _sub(a, lo, row_elems):
    if a is None:
        return None
    return a.ctypes.data_as(C.c_void_p).value + lo * row_elems * a.itemsize


def process(logits, hist=None, hist_len=None, proc: Optional[Proc] = None, mask=None, nthreads=None):
    """Processed logits: logit_bias, penalties, then the bitmask."""
    logits, B, V, hist, hist_len, proc, mask = _prep(logits, hist, hist_len, proc, mask)
    out = np.empty_like(logits)
    bt, bv, nb = proc.bias_arrays()
    pc = proc.c()
    L = lib()

    def run(lo, hi):
        L.orc_process_batch(
            _sub(logits, lo, V), hi - lo, V, _sub(hist, lo, hist.shape[1]) if hist is not None else None,
            hist.shape[1] if hist is not None else 0,
            _sub(hist_len, lo, 1) if hist is not None else None, C.byref(pc), _p(bt), _p(bv), nb,
            _sub(mask, lo, mask.shape[1]) if mask is not None else None,
            mask.shape[1] if mask is not None else 0, _sub(out, lo, V))

    with ThreadPoolExecutor(_nthreads(nthreads)) as ex:
        list(ex.map(lambda r: run(*r), _ranges(B, _nthreads(nthreads))))
    return out


def logprobs(logits, hist=None, hist_len=None, proc: Optional[Proc] = None, mask=None, nthreads=None):
    """Processed logits minus their row log-sum-exp; returns (logprobs, lse)."""
    logits, B, V, hist, hist_len, proc, mask = _prep(logits, hist, hist_len, proc, mask)
    out = np.empty_like(logits)
    lse = np.empty(B, dtype=np.float32)
    bt, bv, nb = proc.bias_arrays()
    pc = proc.c()
    L = lib()

    def run(lo, hi):
        L.orc_logprobs_batch(
            _sub(logits, lo, V), hi - lo, V, _sub(hist, lo, hist.shape[1]) if hist is not None else None,
            hist.shape[1] if hist is not None else 0,
            _sub(hist_len, lo, 1) if hist is not None else None, C.byref(pc), _p(bt), _p(bv), nb,
            _sub(mask, lo, mask.shape[1]) if mask is not None else None,
            mask.shape[1] if mask is not None else 0, _sub(out, lo, V), _sub(lse, lo, 1))

    with ThreadPoolExecutor(_nthreads(nthreads)) as ex:
        list(ex.map(lambda r: run(*r), _ranges(B, _nthreads(nthreads))))
    return out, lse


def sample(logits, sampler: Sampler, hist=None, hist_len=None, proc: Optional[Proc] = None, mask=None,
           gumbel=None, uniform=None, seed: int = 0, offset: int = 0, row_base: int = 0,
           surv_cap: int = 0, nthreads=None):
    """Processors, log-sum-exp and sampler for every row.

    Noise: injected when `gumbel` ([B,V] fp32 Gumbel values) and/or `uniform`
    ([B,2] fp64 uniforms) are given, else Philox keyed by (seed, offset) with
    row ids row_base + r.  Returns dict(tokens, lse, surv_ids, surv_probs, n_surv).
    """
    logits, B, V, hist, hist_len, proc, mask = _prep(logits, hist, hist_len, proc, mask)
    injected = gumbel is not None or uniform is not None
    if injected:
        gumbel = (np.zeros((B, V), dtype=np.float32) if gumbel is None
                  else np.ascontiguousarray(gumbel, dtype=np.float32))
        uniform = (np.zeros((B, 2), dtype=np.float64) if uniform is None
                   else np.ascontiguousarray(uniform, dtype=np.float64))
    tokens = np.empty(B, dtype=np.int32)
    lse = np.empty(B, dtype=np.float32)
    sid = np.full((B, surv_cap), -1, dtype=np.int32) if surv_cap else None
    spr = np.zeros((B, surv_cap), dtype=np.float32) if surv_cap else None
    nsv = np.zeros(B, dtype=np.int32)
    bt, bv, nb = proc.bias_arrays()
    pc, sc = proc.c(), sampler.c()
    L = lib()
    errs = []

    def run(lo, hi):
        rc = L.orc_sample_batch(
            _sub(logits, lo, V), hi - lo, V, _sub(hist, lo, hist.shape[1]) if hist is not None else None,
            hist.shape[1] if hist is not None else 0,
            _sub(hist_len, lo, 1) if hist is not None else None, C.byref(pc), _p(bt), _p(bv), nb,
            _sub(mask, lo, mask.shape[1]) if mask is not None else None,
            mask.shape[1] if mask is not None else 0, C.byref(sc), 0 if injected else 1,
            _sub(gumbel, lo, V) if injected else None, _sub(uniform, lo, 2) if injected else None,
            seed, offset, row_base + lo, _sub(tokens, lo, 1), _sub(lse, lo, 1),
            _sub(sid, lo, surv_cap) if surv_cap else None, _sub(spr, lo, surv_cap) if surv_cap else None,
            _sub(nsv, lo, 1), surv_cap)
        if rc:
            errs.append(rc)

    with ThreadPoolExecutor(_nthreads(nthreads)) as ex:
        list(ex.map(lambda r: run(*r), _ranges(B, _nthreads(nthreads))))
    if errs:
        raise RuntimeError(f"oracle sample failed: {errs}")
    return dict(tokens=tokens, lse=lse, surv_ids=sid, surv_probs=spr, n_surv=nsv)


def _sample_one(x: np.ndarray, lse: float, sampler: Sampler, noise: _Noise, surv_cap: int = 0):
    x = np.ascontiguousarray(x, dtype=np.float32)
    tok = np.zeros(1, dtype=np.int32)
    sid = np.full(max(surv_cap, 1), -1, dtype=np.int32)
    spr = np.zeros(max(surv_cap, 1), dtype=np.float32)
    sc = sampler.c()
    n = lib().orc_sample_row(_p(x), x.shape[0], lse, C.byref(sc), C.byref(noise), _p(tok), _p(sid),
                             _p(spr), surv_cap)
    return int(tok[0]), sid[:n] if surv_cap else None, spr[:n] if surv_cap else None


def _noise_for(injected, gumbel_row, uniform_row, seed, offset, row):
    nz = _Noise()
    nz.mode = 0 if injected else 1
    keep = []
    if injected:
        g = np.ascontiguousarray(gumbel_row, dtype=np.float32)
        u = np.ascontiguousarray(uniform_row, dtype=np.float64)
        keep += [g, u]
        nz.gumbel = g.ctypes.data_as(C.POINTER(C.c_float))
        nz.uniform = u.ctypes.data_as(C.POINTER(C.c_double))
    nz.seed, nz.offset, nz.row = seed, offset, row
    return nz, keep


def verify(target, drafts, y, sampler: Sampler, mode: str = "match", draft_logits=None, hist=None,
           hist_len=None, proc: Optional[Proc] = None, mask=None, gumbel=None, uniform=None,
           u_accept=None, u_residual=None, seed: int = 0, offset: int = 0):
    """Draft acceptance over a [B, k+1, V] verify pass.

    mode "match": the reference rule (lookup_decode.py:363-369,
    verify_decode.py:915-921): sample every row with the processors seeing
    history + [y] + drafts[:i] (verify_decode.py:889-898), keep the longest
    prefix whose picks equal the drafts, emit picks[:accepted+1].

    mode "residual": speculative rejection sampling (Leviathan et al. 2023;
    not in the reference).  p_i = the sampler's distribution of target row i
    (survivor probabilities at temperature when a filter is on, else
    expf(fl32(y - lse_y)) with y = fl32(x / temp); one-hot at the argmax
    when temp == 0); q_i = expf(fl32(d - lse(d))) of the raw draft logits.
    Draft i is accepted iff u_i * q_i(d_i) < p_i(d_i) in fp64; at the first
    rejection j the token is drawn from max(fl32(p_j - q_j), 0) by exact
    fixed-point inverse CDF (first id whose inclusive prefix of
    floor(r 2^52) exceeds floor(u_res R)); with every draft accepted the
    bonus is an ordinary sample of row k.

    Returns (tokens [B, k+1] with -1 padding, n_accepted [B]).
    """
    target = np.ascontiguousarray(target, dtype=np.float32)
    B, K1, V = target.shape
    k = K1 - 1
    drafts = np.asarray(drafts, dtype=np.int64).reshape(B, k)
    y = np.asarray(y, dtype=np.int64).reshape(B)
    proc = proc or Proc()
    injected = gumbel is not None or uniform is not None
    tokens = np.full((B, K1), -1, dtype=np.int32)
    nacc = np.zeros(B, dtype=np.int32)
    sc = sampler
    for b in range(B):
        base = [] if hist is None else list(np.asarray(hist[b])[: (hist.shape[1] if hist_len is None else hist_len[b])])
        feed = [int(y[b])] + [int(t) for t in drafts[b]]
        rows = []
        for i in range(K1):
            h = np.array(base + feed[: i + 1], dtype=np.int32)[None, :]
            rows.append(process(target[b, i][None, :], hist=h, proc=proc,
                                mask=None if mask is None else np.asarray(mask)[b, i][None, :], nthreads=1)[0])
        lses = [row_lse(r) for r in rows]

        def draw(i):
            nz, keep = _noise_for(injected, None if not injected else gumbel[b, i],
                                  None if not injected else uniform[b, i], seed, offset, b * K1 + i)
            return _sample_one(rows[i], lses[i], sc, nz, surv_cap=V if sc.filtered and not sc.temp == 0 else 0)

        if mode == "match":
            picks = [draw(i)[0] for i in range(K1)]
            out = []
            for i, t in enumerate(picks):
                out.append(t)
                if i >= k or t != feed[i + 1]:
                    break
            tokens[b, : len(out)] = out
            nacc[b] = len(out) - 1
            continue
        if mode != "residual":
            raise ValueError(mode)
        dl = np.ascontiguousarray(draft_logits[b], dtype=np.float32)

        def p_row(i):
            x = rows[i]
            if sc.temp == 0:
                p = np.zeros(V, dtype=np.float32)
                p[int(np.argmax(x))] = 1.0
                return p
            if sc.filtered:
                _, ids, prs = draw(i)
                p = np.zeros(V, dtype=np.float32)
                p[ids] = prs
                return p
            inv = np.float32(1.0 / sc.temp)
            yv = np.where(np.isfinite(x), x * inv, np.float32(-np.inf)).astype(np.float32)
            ly = np.float32(row_lse(yv))
            return expf_shift(yv, ly)

        def q_row(i):
            d = dl[i]
            c = np.float32(row_lse(d))
            return expf_shift(d, c)

        out = []
        rejected = -1
        for i in range(k):
            d = int(drafts[b, i])
            p, q = p_row(i), q_row(i)
            u = (u_accept[b, i] if u_accept is not None
                 else philox_uniform(seed, offset, b * K1 + i, 2))
            if float(u) * float(q[d]) < float(p[d]):
                out.append(d)
                continue
            rejected = i
            r = np.maximum(p - q, np.float32(0.0)).astype(np.float32)
            # floor(r 2^52) exactly: r <= 1, so the product is exact in fp64
            qr = (r.astype(np.float64) * 2.0 ** 52).astype(np.uint64)
            cum = np.cumsum(qr, dtype=np.uint64)  # the residual mass is at most ~1: no overflow
            R = int(cum[-1]) if V else 0
            if R == 0:
                out.append(draw(i)[0])
            else:
                ures = (u_residual[b] if u_residual is not None
                        else philox_uniform(seed, offset, b * K1 + i, 3))
                u53v = min(int(float(ures) * 2.0 ** 53), 2 ** 53 - 1) if ures > 0 else 0
                tgt = (u53v * R) >> 53
                # the first id whose inclusive prefix exceeds tgt
                tok = int(np.searchsorted(cum, np.uint64(tgt), side="right"))
                out.append(tok if tok < V else V - 1)
            break
        if rejected < 0:
            out.append(draw(k)[0])
        tokens[b, : len(out)] = out
        nacc[b] = len(out) - 1
    return tokens, nacc


def shard_sample(logits_shards: Sequence[np.ndarray], sampler: Sampler, gumbel=None, uniform=None,
                 seed: int = 0, offset: int = 0):
    """Vocab-sharded sampling: the shards are contiguous slices of each row;
    tile statistics restart at every shard boundary and are combined across
    shards in shard order; candidates are taken over the whole row.  When
    every shard but the last holds a multiple of 1024 ids this equals
    sample() on the concatenated row."""
    full = np.concatenate([np.asarray(s, dtype=np.float32) for s in logits_shards], axis=1)
    B, V = full.shape
    lses = []
    for b in range(B):
        ms, ss = [], []
        for s in logits_shards:
            m, q = tile_stats(np.asarray(s[b], dtype=np.float32))
            ms.append(m)
            ss.append(q)
        m = np.ascontiguousarray(np.concatenate(ms))
        q = np.ascontiguousarray(np.concatenate(ss))
        lses.append(lib().orc_combine_tiles(_p(m), _p(q), len(m)))
    toks = np.empty(B, dtype=np.int32)
    injected = gumbel is not None or uniform is not None
    for b in range(B):
        nz, keep = _noise_for(injected, None if not injected else gumbel[b],
                              None if not injected else (uniform[b] if uniform is not None else np.zeros(2)),
                              seed, offset, b)
        toks[b] = _sample_one(full[b], lses[b], sampler, nz)[0]
    return toks, np.array(lses, dtype=np.float32)


def draft_ngram(tokens, k: int, n_min: int = 3, n_max: int = 8):
    """Draft continuation of the longest recent n-gram match (reference
    pagedmoe/lookup_decode.py:184-221): for n from min(n_max, len) down to
    n_min, look for earlier occurrences of the last n tokens that leave at
    least one token after them; the latest occurrence with a full k tokens
    after it wins, else the occurrence with the most tokens after it (the
    earliest); the first n with any occurrence decides.  Returns (draft,
    matched_n) with ([], 0) when nothing matches."""
    toks = [int(t) for t in tokens]
    L = len(toks)
    if k <= 0:
        return [], 0
    for n in range(min(n_max, L), n_min - 1, -1):
        tail = toks[L - n:]
        full, part = None, None
        for s in range(L - n):  # s + n <= L - 1: something follows
            if toks[s:s + n] != tail:
                continue
            if s + n + k <= L:
                full = s  # keep the latest
            elif part is None:
                part = s  # the earliest partial has the longest continuation
        if full is not None:
            return toks[full + n:full + n + k], n
        if part is not None:
            return toks[part + n:L], n
    return [], 0

