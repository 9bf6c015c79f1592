"""pm_sample_rows_static (the fixed-scratch entry point) against
pm_sample_rows on the same rows, two calls in a row, through the C ABI.

Kept in its own file, collected last, so it runs both alone and after every
other GPU test has used the library."""

import ctypes as C

import numpy as np
import pytest
import torch

from paged_moe_b200 import _lib as L
from paged_moe_b200 import workloads as W
from paged_moe_b200.params import ProcessorSettings, SamplerSettings

pytestmark = pytest.mark.gpu


def _static_call(x, s, p, mask, gumbel, uniform, hist):
    from paged_moe_b200 import engine as E
    keep = E._Keep()
    dev = x.device
    r = E.build_rows(x, s, p, hist, None, mask, keep)
    nz = E._noise(r.rows, r.vocab, 1234, 7, 0, gumbel, uniform, keep, dev)
    out = L.SampleOut()
    tokens = torch.full((r.rows,), -7, dtype=torch.int32, device=dev)
    lse = torch.full((r.rows,), float("nan"), dtype=torch.float32, device=dev)
    out.tokens = tokens.data_ptr()
    out.lse = lse.data_ptr()
    stream = torch.cuda.current_stream(dev)
    rc = L.load().pm_sample_rows_static(C.byref(r), C.byref(nz), C.byref(out), stream.cuda_stream)
    L.check(rc, "pm_sample_rows_static")
    torch.cuda.synchronize()
    return tokens.cpu().numpy(), lse.cpu().numpy()


def _workspace_call(x, s, p, mask, gumbel, uniform, hist):
    from paged_moe_b200 import engine as E
    res = E.sample_rows(x, s, p, history=hist, mask=mask, gumbel=gumbel, uniform=uniform, seed=1234, offset=7,
                        return_lse=True)
    torch.cuda.synchronize()
    return res["tokens"].cpu().numpy(), res["lse"].cpu().numpy()


def _case(seed, B, V, s, p, with_mask, with_hist):
    rng = np.random.default_rng(seed)
    dev = torch.device("cuda")
    x = torch.from_numpy(W.peaked_logits(rng, B, V, 2.0, 9.0, 16)).to(dev)
    mask = torch.from_numpy(W.bitmask(rng, B, V).view(np.int32)).to(dev) if with_mask else None
    hist = torch.from_numpy(rng.integers(0, V, (B, 128)).astype(np.int32)).to(dev) if with_hist else None
    g = torch.from_numpy(W.gumbel(rng, (B, V))).to(dev)
    u = torch.from_numpy(rng.random((B, 2))).to(dev)
    return x, s, p, mask, g, u, hist


def test_static_scratch_matches_workspace_path_two_calls_in_a_row():
    cases = [
        _case(1, 64, 32768, SamplerSettings(temp=1.0, top_k=50, top_p=0.95), ProcessorSettings(), True, False),
        _case(2, 17, 50001, SamplerSettings(temp=0.7, min_p=0.05),
              ProcessorSettings(repetition_penalty=1.1, repetition_context_size=64), False, True),
    ]
    for args in cases:
        t_static, l_static = _static_call(*args)
        t_ws, l_ws = _workspace_call(*args)
        np.testing.assert_array_equal(t_static, t_ws)
        np.testing.assert_array_equal(l_static.view(np.uint32), l_ws.view(np.uint32))
    # and the first case again, after the scratch held the second one's data
    t_again, l_again = _static_call(*cases[0])
    t_ws, l_ws = _workspace_call(*cases[0])
    np.testing.assert_array_equal(t_again, t_ws)
    np.testing.assert_array_equal(l_again.view(np.uint32), l_ws.view(np.uint32))


def test_static_scratch_refuses_rows_beyond_its_size():
    lib = L.load()
    r = L.Rows()
    dev = torch.device("cuda")
    x = torch.zeros((1, 1), device=dev)
    r.logits = x.data_ptr()
    r.params = x.data_ptr()
    r.dtype = L.PM_DTYPE_F32
    r.rows, r.vocab, r.row_stride = 4096, 262144, 262144
    r.flags_any = L.PM_F_TOP_P | L.PM_F_UNBOUNDED
    assert lib.pm_sample_workspace_bytes(C.byref(r)) > L.PM_STATIC_SCRATCH_BYTES
    out = L.SampleOut()
    out.tokens = x.data_ptr()
    rc = lib.pm_sample_rows_static(C.byref(r), C.byref(L.Noise()), C.byref(out), None)
    assert rc == L.PM_ERR_WORKSPACE
