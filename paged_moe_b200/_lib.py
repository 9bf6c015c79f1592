"""ctypes binding of libpm_sample.so (the C ABI declared in include/pm_sample.h).

There is no fallback: if the library is missing or does not load, importing
the package fails with the reason.  The structs below mirror the header field
for field.
"""

from __future__ import annotations

import ctypes as C
import os

from . import build as _build

PM_OK = 0
PM_ERR_ARG = -1
PM_ERR_CUDA = -2
PM_ERR_UNSUPPORTED = -3
PM_ERR_WORKSPACE = -4

PM_DTYPE_F32 = 0
PM_DTYPE_BF16 = 1

PM_NOISE_PHILOX = 0
PM_NOISE_INJECTED = 1

PM_F_GREEDY = 0x1
PM_F_TOP_P = 0x2
PM_F_MIN_P = 0x4
PM_F_REP = 0x10
PM_F_PRES = 0x20
PM_F_FREQ = 0x40
PM_F_UNBOUNDED = 0x100
PM_F_FULL = 0x200

PM_STATIC_SCRATCH_BYTES = 32 << 20

PM_VERIFY_MATCH = 0
PM_VERIFY_RESIDUAL = 1

_ERRORS = {
    PM_ERR_ARG: "invalid argument",
    PM_ERR_CUDA: "CUDA error",
    PM_ERR_UNSUPPORTED: "outside this build's limits",
    PM_ERR_WORKSPACE: "workspace too small",
}


class RowParams(C.Structure):
    _fields_ = [
        ("flags", C.c_uint32), ("inv_temperature", C.c_float), ("top_k", C.c_int32),
        ("top_p_comp", C.c_float), ("log_min_p", C.c_float), ("min_tokens_to_keep", C.c_int32),
        ("repetition_penalty", C.c_float), ("repetition_context_size", C.c_int32),
        ("presence_penalty", C.c_float), ("presence_context_size", C.c_int32),
        ("frequency_penalty", C.c_float), ("frequency_context_size", C.c_int32),
    ]


class Rows(C.Structure):
    _fields_ = [
        ("logits", C.c_void_p), ("dtype", C.c_int32), ("rows", C.c_int64), ("vocab", C.c_int64),
        ("row_stride", C.c_int64), ("params", C.c_void_p), ("params_per_row", C.c_int32),
        ("hist", C.c_void_p), ("hist_len", C.c_void_p), ("hist_stride", C.c_int64),
        ("feed", C.c_void_p), ("feed_group", C.c_int32),
        ("bias_tokens", C.c_void_p), ("bias_values", C.c_void_p), ("n_bias", C.c_int32),
        ("mask", C.c_void_p), ("mask_stride", C.c_int64),
        ("flags_any", C.c_uint32), ("top_k_max", C.c_int32), ("forced", C.c_void_p),
    ]


class Noise(C.Structure):
    _fields_ = [
        ("mode", C.c_int32), ("seed", C.c_uint64), ("offset", C.c_uint64), ("row_base", C.c_uint32),
        ("gumbel", C.c_void_p), ("gumbel_stride", C.c_int64), ("uniform", C.c_void_p),
    ]


class SampleOut(C.Structure):
    _fields_ = [
        ("tokens", C.c_void_p), ("lse", C.c_void_p), ("token_logprob", C.c_void_p),
        ("surv_ids", C.c_void_p), ("surv_probs", C.c_void_p), ("n_surv", C.c_void_p),
        ("surv_cap", C.c_int32),
    ]


class VerifyArgs(C.Structure):
    _fields_ = [
        ("mode", C.c_int32), ("drafts", C.c_void_p), ("n_draft", C.c_int32),
        ("draft_logits", C.c_void_p), ("draft_dtype", C.c_int32), ("draft_row_stride", C.c_int64),
        ("u_accept", C.c_void_p), ("u_residual", C.c_void_p),
        ("tokens", C.c_void_p), ("n_accepted", C.c_void_p), ("row_tokens", C.c_void_p),
    ]


class ShardArgs(C.Structure):
    _fields_ = [
        ("shard_index", C.c_int32), ("n_shards", C.c_int32), ("vocab_total", C.c_int64),
        ("shard_width", C.c_int64),
    ]


class LmHead(C.Structure):
    _fields_ = [
        ("hidden", C.c_void_p), ("n_tokens", C.c_int64), ("hidden_size", C.c_int64),
        ("hidden_stride", C.c_int64), ("weight", C.c_void_p), ("weight_stride", C.c_int64),
    ]


# Exported symbols and their signatures: (restype, argtypes)
_P = C.c_void_p
SIGNATURES = {
    "pm_version": (C.c_char_p, []),
    "pm_selfcheck_ex2": (C.c_int, [C.POINTER(C.c_double)]),
    "pm_last_cuda_error": (C.c_int, []),
    "pm_sample_workspace_bytes": (C.c_size_t, [_P]),
    "pm_sample_rows": (C.c_int, [_P, _P, _P, _P, C.c_size_t, _P]),
    "pm_sample_rows_static": (C.c_int, [_P, _P, _P, _P]),
    "pm_processors_workspace_bytes": (C.c_size_t, [_P]),
    "pm_apply_processors": (C.c_int, [_P, _P, C.c_int64, _P, C.c_size_t, _P]),
    "pm_logprobs": (C.c_int, [_P, _P, C.c_int64, _P, _P, C.c_size_t, _P]),
    "pm_verify_workspace_bytes": (C.c_size_t, [_P, _P]),
    "pm_verify": (C.c_int, [_P, _P, _P, _P, C.c_size_t, _P]),
    "pm_shard_summary_bytes": (C.c_size_t, [_P, _P]),
    "pm_shard_summarize": (C.c_int, [_P, _P, _P, _P, _P, C.c_size_t, _P]),
    "pm_shard_merge": (C.c_int, [_P, _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "pm_think_budget": (C.c_int, [_P, _P, C.c_int64, C.c_int64, _P, _P, C.c_int64, _P, _P, C.c_int32, C.c_int32,
                                  C.c_int32, C.c_int32, _P, _P]),
    "pm_draft_ngram": (C.c_int, [_P, _P, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_int32, _P, _P, _P, _P]),
    "pm_lmhead_logits": (C.c_int, [_P, C.c_int64, _P, C.c_int64, _P]),
    "pm_lmhead_sample_workspace_bytes": (C.c_size_t, [_P, _P]),
    "pm_lmhead_sample": (C.c_int, [_P, _P, _P, _P, _P, C.c_size_t, _P]),
}

_lib = None


def load(build_if_missing: bool = True):
    """The loaded library (built first if it is missing and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.SO
    if build_if_missing:
        try:
            path = _build.build()
        except _build.CompilerMissing as e:  # no nvcc on this machine: the prebuilt file must exist
            if not os.path.exists(path):
                raise ImportError(f"libpm_sample.so is missing and could not be built: {e}") from e
    if not os.path.exists(path):
        raise ImportError(f"libpm_sample.so not found at {path}")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


_ext = None


def ext():
    """The PyTorch extension module over the C ABI (_pm_torch), built first
    when it is missing or older than its sources and a compiler exists."""
    global _ext
    if _ext is not None:
        return _ext
    load()
    try:
        _build.build_ext()
    except _build.CompilerMissing as e:  # no compiler here: the prebuilt module must exist
        if not os.path.exists(_build.ext_path()):
            raise ImportError(f"the _pm_torch extension is missing and could not be built: {e}") from e
    from . import _pm_torch  # noqa: E402  (in-tree module next to libpm_sample.so)
    _ext = _pm_torch
    return _ext


def check(rc: int, what: str) -> None:
    if rc == PM_OK:
        return
    msg = _ERRORS.get(rc, f"status {rc}")
    if rc == PM_ERR_CUDA:
        msg += f" (cudaError {load().pm_last_cuda_error()})"
    if rc == PM_ERR_ARG:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")
