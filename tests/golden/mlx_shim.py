"""A numpy stand-in for the parts of `mlx.core` and `mlx_lm.models.cache` that
the reference's token-selection code touches, so that code can run on this
(non-Apple) machine to produce golden fixtures.  Used only by
make_golden.py; nothing at test time imports it.

Arithmetic is numpy's: fp32 arrays stay fp32, and logsumexp is evaluated in
fp64 and rounded to fp32 (MLX's own reduction order cannot be reproduced off
Apple hardware, so fixtures compare log-probabilities with a tolerance).
"""

from __future__ import annotations

import sys
import types

import numpy as np


def install() -> None:
    mx = types.ModuleType("mlx.core")
    mx.uint32, mx.int32, mx.float32, mx.bool_ = np.uint32, np.int32, np.float32, np.bool_
    mx.inf = np.inf

    def array(x, dtype=None):
        return np.array(x, dtype=dtype)

    def zeros(shape, dtype=np.float32):
        return np.zeros(shape, dtype=dtype)

    def argmax(a, axis=None):
        return np.argmax(np.asarray(a), axis=axis)

    def logsumexp(a, axis=None, keepdims=False):
        a64 = np.asarray(a, dtype=np.float64)
        m = np.max(a64, axis=axis, keepdims=True)
        r = m + np.log(np.sum(np.exp(a64 - m), axis=axis, keepdims=True))
        if not keepdims:
            r = np.squeeze(r, axis=axis)
        return r.astype(np.float32)

    mx.array, mx.zeros, mx.argmax, mx.logsumexp = array, zeros, argmax, logsumexp
    mx.concatenate = lambda xs, axis=0: np.concatenate(xs, axis=axis)
    mx.eval = lambda *a, **k: None
    mx.async_eval = lambda *a, **k: None
    mx.where = np.where
    mx.any = np.any
    mx.minimum = np.minimum
    mx.maximum = np.maximum
    mx.cumsum = np.cumsum
    mx.logical_not = np.logical_not

    def arange(*args, dtype=None):
        return np.arange(*args, dtype=dtype)

    mx.arange = arange
    mx.random = types.SimpleNamespace(state=[None])

    mlx = types.ModuleType("mlx")
    mlx.core = mx
    sys.modules["mlx"] = mlx
    sys.modules["mlx.core"] = mx

    cache = types.ModuleType("mlx_lm.models.cache")

    class _BaseCache:
        pass

    class ArraysCache(_BaseCache):
        def __init__(self, n=1):
            self.cache = [None] * n

        def is_trimmable(self):
            return False

    def can_trim_prompt_cache(c):
        return all(x.is_trimmable() for x in c)

    def trim_prompt_cache(c, n):
        return min(x.trim(n) for x in c) if c else 0

    cache._BaseCache, cache.ArraysCache = _BaseCache, ArraysCache
    cache.can_trim_prompt_cache, cache.trim_prompt_cache = can_trim_prompt_cache, trim_prompt_cache
    mlx_lm = types.ModuleType("mlx_lm")
    models = types.ModuleType("mlx_lm.models")
    mlx_lm.models = models
    models.cache = cache
    sys.modules["mlx_lm"] = mlx_lm
    sys.modules["mlx_lm.models"] = models
    sys.modules["mlx_lm.models.cache"] = cache


class TrimCache:
    """A KV cache entry that can always be trimmed (what _verify rewinds)."""

    def __init__(self):
        from mlx_lm.models.cache import _BaseCache  # noqa: F401  (shim)
        self.offset = 0

    def is_trimmable(self):
        return True

    def trim(self, n):
        self.offset -= n
        return n


class ScriptedModel:
    """model(inp, cache=...) -> the logits scripted for the next call, [1, n, V]."""

    def __init__(self, logits_per_call):
        self.calls = list(logits_per_call)

    def __call__(self, inp, cache=None):
        x = self.calls.pop(0)
        n = np.asarray(inp).shape[-1]
        assert x.shape[0] == n, (x.shape, n)
        return x[None, :, :]
