"""The C ABI: every declared entry point is exported, and argument checking
happens before any device work (these calls run without a GPU)."""

import ctypes as C
import os
import re
import subprocess

import pytest

from paged_moe_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pm_sample.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"PM_API[^;(]*?\b(pm_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared()
    for n in ("pm_sample_rows", "pm_sample_workspace_bytes", "pm_apply_processors", "pm_logprobs", "pm_verify",
              "pm_verify_workspace_bytes", "pm_shard_summarize", "pm_shard_merge", "pm_shard_summary_bytes",
              "pm_sample_rows_static", "pm_version"):
        assert n in names, n


def test_library_exports_every_declared_symbol():
    lib = L.load()
    so = L._build.SO
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (pm_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing
    for n in declared():
        assert getattr(lib, n) is not None
    assert lib.pm_version().decode().startswith("pm_sample")


def _rows(**kw):
    r = L.Rows()
    r.logits = 0x1000
    r.dtype = L.PM_DTYPE_F32
    r.rows = 4
    r.vocab = 1000
    r.row_stride = 1000
    r.params = 0x2000
    for k, v in kw.items():
        setattr(r, k, v)
    return r


def test_workspace_query_needs_no_device():
    lib = L.load()
    assert lib.pm_sample_workspace_bytes(C.byref(_rows())) > 0
    assert lib.pm_sample_workspace_bytes(C.byref(_rows(top_k_max=64))) > 0
    assert lib.pm_sample_workspace_bytes(C.byref(_rows(top_k_max=257))) == 0  # beyond the fused path
    assert lib.pm_sample_workspace_bytes(C.byref(_rows(vocab=0))) == 0
    assert lib.pm_sample_workspace_bytes(C.byref(_rows(row_stride=10))) == 0


@pytest.mark.parametrize("bad", [
    dict(logits=None), dict(params=None), dict(dtype=7), dict(mask=0x3000, mask_stride=1),
    dict(feed=0x3000, feed_group=3), dict(n_bias=2), dict(hist=0x3000, hist_stride=0),
])
def test_bad_arguments_fail_before_launch(bad):
    lib = L.load()
    r = _rows(**{k: v for k, v in bad.items()})
    nz = L.Noise()
    nz.mode = L.PM_NOISE_PHILOX
    out = L.SampleOut()
    out.tokens = 0x4000
    rc = lib.pm_sample_rows(C.byref(r), C.byref(nz), C.byref(out), 0x5000, 1 << 30, None)
    assert rc == L.PM_ERR_ARG


def test_small_workspace_is_refused():
    lib = L.load()
    r = _rows()
    nz = L.Noise()
    out = L.SampleOut()
    out.tokens = 0x4000
    need = lib.pm_sample_workspace_bytes(C.byref(r))
    assert lib.pm_sample_rows(C.byref(r), C.byref(nz), C.byref(out), 0x5000, need - 1, None) == L.PM_ERR_WORKSPACE


def test_injected_noise_needs_its_arrays():
    lib = L.load()
    r = _rows(top_k_max=20, flags_any=L.PM_F_TOP_P)
    nz = L.Noise()
    nz.mode = L.PM_NOISE_INJECTED
    out = L.SampleOut()
    out.tokens = 0x4000
    assert lib.pm_sample_rows(C.byref(r), C.byref(nz), C.byref(out), 0x5000, 1 << 30, None) == L.PM_ERR_ARG


def _vargs(**kw):
    v = L.VerifyArgs()
    v.mode = L.PM_VERIFY_MATCH
    v.drafts = 0x6000
    v.n_draft = 3
    v.tokens = 0x7000
    v.n_accepted = 0x8000
    for k, val in kw.items():
        setattr(v, k, val)
    return v


@pytest.mark.parametrize("bad", [
    dict(mode=5), dict(drafts=None), dict(tokens=None), dict(n_accepted=None), dict(n_draft=2),
    dict(mode=L.PM_VERIFY_RESIDUAL), dict(mode=L.PM_VERIFY_RESIDUAL, draft_logits=0x9000, draft_row_stride=10),
    dict(mode=L.PM_VERIFY_RESIDUAL, draft_logits=0x9000, draft_row_stride=1000, draft_dtype=9),
])
def test_verify_checks_arguments_before_launch(bad):
    lib = L.load()
    r = _rows()  # 4 rows = 1 request of k = 3
    nz = L.Noise()
    v = _vargs(**bad)
    rc = lib.pm_verify(C.byref(r), C.byref(nz), C.byref(v), 0x5000, 1 << 30, None)
    assert rc == L.PM_ERR_ARG


def test_verify_feed_group_must_be_k_plus_one():
    lib = L.load()
    r = _rows(feed=0x3000, feed_group=2)
    v = _vargs()
    assert lib.pm_verify(C.byref(r), C.byref(L.Noise()), C.byref(v), 0x5000, 1 << 30, None) == L.PM_ERR_ARG


def test_verify_workspace_query():
    lib = L.load()
    r = _rows()
    match = lib.pm_verify_workspace_bytes(C.byref(r), C.byref(_vargs()))
    res = lib.pm_verify_workspace_bytes(C.byref(r), C.byref(_vargs(mode=L.PM_VERIFY_RESIDUAL)))
    assert match >= lib.pm_sample_workspace_bytes(C.byref(r)) and res > match
    assert lib.pm_verify_workspace_bytes(C.byref(r), C.byref(_vargs(n_draft=2))) == 0
    assert lib.pm_verify(C.byref(r), C.byref(L.Noise()), C.byref(_vargs()), 0x5000, match - 1, None) == \
        L.PM_ERR_WORKSPACE


def _shard(i=0, n=8, V=262144, w=32768):
    s = L.ShardArgs()
    s.shard_index, s.n_shards, s.vocab_total, s.shard_width = i, n, V, w
    return s


def test_shard_layout_and_checks():
    lib = L.load()
    r = _rows(vocab=32768, row_stride=32768, top_k_max=64, flags_any=L.PM_F_TOP_P)
    assert lib.pm_shard_summary_bytes(C.byref(r), C.byref(_shard())) > 0
    assert lib.pm_shard_summary_bytes(C.byref(r), C.byref(_shard(w=30000))) == 0  # not whole tiles
    assert lib.pm_shard_summary_bytes(C.byref(r), C.byref(_shard(i=8))) == 0
    assert lib.pm_shard_summary_bytes(C.byref(r), C.byref(_shard(V=300000, w=37888))) == 0
    nz = L.Noise()
    # a slice of the wrong width is refused before any launch
    r2 = _rows(vocab=1000, row_stride=1000)
    assert lib.pm_shard_summarize(C.byref(r2), C.byref(_shard()), C.byref(nz), 0x9000, 0x5000, 1 << 30, None) == \
        L.PM_ERR_ARG
    out = L.SampleOut()
    out.tokens = 0x4000
    r3 = _rows(vocab=262144, row_stride=262144)
    assert lib.pm_shard_merge(C.byref(r3), C.byref(_shard()), C.byref(nz), 0x9000, C.byref(out), 0x5000, 3,
                              None) == L.PM_ERR_WORKSPACE
