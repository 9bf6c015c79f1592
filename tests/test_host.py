"""Host-side logic: the settings -> fp32 constants mapping, validation in
mlx-lm's terms, and the factory contracts (no GPU needed)."""

import math

import numpy as np
import pytest

from paged_moe_b200 import _lib as L
from paged_moe_b200 import params as P
from paged_moe_b200 import sample_utils as SU


def test_scalars_are_python_double_then_fp32():
    s = P.SamplerSettings(temp=0.7, top_p=0.9, min_p=0.05, top_k=20)
    r = P.row_struct(s, P.ProcessorSettings(repetition_penalty=1.05))
    assert r.inv_temperature == float(np.float32(1 / 0.7))
    assert r.top_p_comp == float(np.float32(1 - 0.9))
    assert r.log_min_p == float(np.float32(math.log(0.05)))
    assert r.repetition_penalty == float(np.float32(1.05))
    assert r.top_k == 20
    assert r.flags & L.PM_F_TOP_P and r.flags & L.PM_F_MIN_P and r.flags & L.PM_F_REP
    assert not r.flags & L.PM_F_GREEDY and not r.flags & L.PM_F_UNBOUNDED


def test_mode_flags():
    g = P.row_struct(P.SamplerSettings(temp=0.0, top_k=20, top_p=0.5), P.ProcessorSettings())
    assert g.flags & L.PM_F_GREEDY and g.top_k == 0  # temp 0 is argmax: filters are not used
    f = P.row_struct(P.SamplerSettings(temp=1.0), P.ProcessorSettings())
    assert f.flags & L.PM_F_FULL
    u = P.row_struct(P.SamplerSettings(temp=1.0, top_p=0.9), P.ProcessorSettings())
    assert u.flags & L.PM_F_UNBOUNDED
    assert not P.row_struct(P.SamplerSettings(temp=1.0, top_p=1.0), P.ProcessorSettings()).flags & L.PM_F_TOP_P
    assert not P.row_struct(P.SamplerSettings(temp=1.0, top_p=0.0), P.ProcessorSettings()).flags & L.PM_F_TOP_P


def test_processor_switches_follow_mlx_lm():
    # make_logits_processors: a penalty is on when truthy and non-zero
    assert not P.ProcessorSettings(repetition_penalty=None).rep_on
    assert not P.ProcessorSettings(repetition_penalty=0.0).rep_on
    assert P.ProcessorSettings(repetition_penalty=1.0).rep_on
    assert P.ProcessorSettings(presence_penalty=-0.5).pres_on


def test_validation_matches_mlx_lm():
    with pytest.raises(ValueError):
        P.validate(P.SamplerSettings(temp=1, min_p=1.5), P.ProcessorSettings(), 100)
    with pytest.raises(ValueError):
        P.validate(P.SamplerSettings(temp=1, top_k=100), P.ProcessorSettings(), 100)
    with pytest.raises(ValueError):
        P.validate(P.SamplerSettings(), P.ProcessorSettings(repetition_penalty=-1.0), 100)
    P.validate(P.SamplerSettings(temp=1, top_k=99, min_p=0.1), P.ProcessorSettings(), 100)


def test_pack_rows_bounds():
    ss = [P.SamplerSettings(temp=1, top_k=10), P.SamplerSettings(temp=1, top_k=64, top_p=0.9),
          P.SamplerSettings(temp=0)]
    raw, flags_any, k = P.pack_rows(ss, [P.ProcessorSettings()] * 3)
    assert len(raw) == 3 * 48 and k == 64 and flags_any & L.PM_F_GREEDY and flags_any & L.PM_F_TOP_P


def test_factories_keep_mlx_lm_signatures():
    import inspect
    sig = inspect.signature(SU.make_sampler)
    assert list(sig.parameters)[:8] == ["temp", "top_p", "min_p", "min_tokens_to_keep", "top_k", "xtc_probability",
                                       "xtc_threshold", "xtc_special_tokens"]
    sig = inspect.signature(SU.make_logits_processors)
    assert list(sig.parameters) == ["logit_bias", "repetition_penalty", "repetition_context_size",
                                    "presence_penalty", "presence_context_size", "frequency_penalty",
                                    "frequency_context_size"]
    assert [p.__name__ for p in SU.make_logits_processors(logit_bias={3: 1.0}, repetition_penalty=1.1,
                                                           presence_penalty=0.5, frequency_penalty=0.2)] == [
        "logit_bias_processor", "repetition_penalty_processor", "presence_penalty_processor",
        "frequency_penalty_processor"]
    assert SU.make_logits_processors(repetition_penalty=0.0) == []
    with pytest.raises(NotImplementedError):
        SU.make_sampler(temp=1.0, xtc_probability=0.5)
    s = SU.make_sampler(temp=0.7, top_p=0.9, seed=5)
    assert s.settings == P.SamplerSettings(temp=0.7, top_p=0.9) and s.seed == 5


def test_import_and_workloads_load_no_product_library():
    """The package and its synthetic workloads import without loading
    libpm_sample.so (the benchmark's reference arm builds its inputs from
    them and must run none of this package's native code)."""
    import subprocess
    import sys
    code = ("import paged_moe_b200, paged_moe_b200.workloads as W\n"
            "W.c3(seed=0, B=2, V=4096)\n"
            "maps = open('/proc/self/maps').read()\n"
            "print('LOADED' if 'libpm_sample' in maps else 'CLEAN')\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                         cwd=__import__("os").path.dirname(__import__("os").path.dirname(__file__)))
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip().endswith("CLEAN"), out.stdout


def test_logit_bias_normalised():
    # the device lists are bucketed by id: pairs in any order (or a dict)
    # become ascending distinct ids; a repeated id is an error
    from paged_moe_b200.params import ProcessorSettings
    a = ProcessorSettings(logit_bias=((3, 4.0), (29999, 2.5), (1000, -3.0)))
    b = ProcessorSettings.make(logit_bias={1000: -3.0, 3: 4.0, 29999: 2.5})
    assert a.logit_bias == ((3, 4.0), (1000, -3.0), (29999, 2.5)) == b.logit_bias
    assert a == b and hash(a) == hash(b)
    with pytest.raises(ValueError):
        ProcessorSettings(logit_bias=((5, 1.0), (5, 2.0)))
