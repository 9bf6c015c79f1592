"""GPU parity of the bracketed statistics.

Rows with top-k and top-p (no min-p, no log-sum-exp output) need the row's
log-sum-exp only to place the top-p cut.  On large batches the streaming
pass then writes approximate tile sums (hardware ex2, fp32 additions), the
merge places the cut from a rigorous bracket around the exact log-sum-exp,
and rows whose cut the bracket cannot decide are finished by the exact pass
(status bit 64).  Every result must still equal the oracle's bit for bit.
"""

import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
from paged_moe_b200 import workloads as W
from paged_moe_b200.params import ProcessorSettings, SamplerSettings
from test_gpu_sample import _oproc, _osamp

pytestmark = pytest.mark.gpu


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_ex2_within_the_error_budget():
    """The hardware 2^a over every fp32 a in [-126, 1]: the bracket's budget
    takes 2^-20; the unit must stay within half of it."""
    from paged_moe_b200 import _lib
    v = C.c_double(-1.0)
    assert _lib.load().pm_selfcheck_ex2(C.byref(v)) == 0
    assert 0.0 < v.value <= 2.0 ** -21, v.value


@pytest.mark.parametrize("bf16", [False, True])
def test_bracketed_rows_match_oracle(bf16):
    """64 rows x 163,840 ids (enough tiles a warp for the bracket), top_k 50,
    top_p 0.95, survivors out: tokens, survivor ids and probabilities."""
    from paged_moe_b200 import engine
    rng = np.random.default_rng(21)
    B, V = 64, 163840
    x = W.peaked_logits(rng, B, V, 2.0, 9.0, 64)
    if bf16:
        xb = W.to_bf16_bits(x)
        x = O.bf16_to_f32(xb)
        xt = _t(xb.view(np.int16)).view(torch.bfloat16)
    else:
        xt = _t(x)
    s = SamplerSettings(temp=1.0, top_k=50, top_p=0.95)
    g = W.gumbel(rng, (B, V))
    ref = O.sample(x, _osamp(s), gumbel=g, seed=3, offset=4, surv_cap=16)
    got = engine.sample_rows(xt, s, gumbel=_t(g), seed=3, offset=4, survivors=16, return_status=True)
    torch.cuda.synchronize()
    st = got["status"].cpu().numpy()
    assert ((st & ~64) == 0).all(), st
    np.testing.assert_array_equal(got["tokens"].cpu().numpy(), ref["tokens"])
    np.testing.assert_array_equal(got["n_surv"].cpu().numpy(), ref["n_surv"])
    for b in range(B):
        n = min(int(ref["n_surv"][b]), 16)
        np.testing.assert_array_equal(got["surv_ids"][b, :n].cpu().numpy(), ref["surv_ids"][b, :n])
        np.testing.assert_array_equal(got["surv_probs"][b, :n].cpu().numpy(), ref["surv_probs"][b, :n])


def _tails(xp: np.ndarray, K: int):
    """Exact top-p tails of a processed row: T - A_r over its top-K in rank
    order, q52 relative to the row's exact log-sum-exp."""
    c = np.float32(O.row_lse(xp))
    order = np.lexsort((np.arange(xp.shape[0]), -xp))[:K]
    q = np.array([O.q52(float(np.float32(xp[i]) - c)) for i in order], dtype=object)
    return np.cumsum(q[::-1])[::-1]


def test_undecided_cut_takes_the_exact_pass():
    """Rows whose top-p threshold sits on one of their exact tails (within
    fp32 rounding, far inside the bracket): the merge cannot place the cut,
    queues the row, and the exact pass finishes it -- with a repetition
    penalty, so the exact pass applies the processors itself."""
    from paged_moe_b200 import engine
    rng = np.random.default_rng(22)
    B, V, K = 64, 163840, 64
    x = W.peaked_logits(rng, B, V, 2.5, 10.0, 32)
    hist = rng.integers(0, V, (B, 96)).astype(np.int32)
    hist[:, -32:] = np.argsort(-x, axis=1)[:, :32]  # penalise some of each row's peaks
    p = ProcessorSettings(repetition_penalty=1.2, repetition_context_size=64)
    xp = O.process(x, hist=hist, proc=_oproc(p))
    undecided = {3, 17, 40, 63}
    samplers = []
    for b in range(B):
        top_p = 0.9
        if b in undecided:
            tails = _tails(xp[b], K)
            r = 2 + b % 5
            top_p = 1.0 - float(tails[r]) / 2.0 ** 52
        samplers.append(SamplerSettings(temp=0.8, top_k=K, top_p=top_p))
    g = W.gumbel(rng, (B, V))
    want = np.empty(B, np.int32)
    for b in range(B):
        r = O.sample(x[b:b + 1], _osamp(samplers[b]), hist=hist[b:b + 1], proc=_oproc(p), gumbel=g[b:b + 1],
                     seed=5, offset=6)
        want[b] = r["tokens"][0]
    got = engine.sample_rows(_t(x), samplers, p, history=_t(hist), gumbel=_t(g), seed=5, offset=6,
                             return_status=True)
    torch.cuda.synchronize()
    st = got["status"].cpu().numpy()
    np.testing.assert_array_equal(got["tokens"].cpu().numpy(), want)
    for b in undecided:
        assert st[b] & 64, (b, st[b])
    assert ((st & ~64) == 0).all(), st


def test_bracketed_c5_full_shape():
    """The C5 workload at its full size (1,024 rows x 262,144 ids, top_k 64,
    top_p 0.9, temp 0.8, Philox noise) through the bracketed path, and the
    same rows with the log-sum-exp asked for (exact statistics throughout):
    the same tokens, equal to the oracle's."""
    from paged_moe_b200 import engine
    d = W.c5(seed=23, B=1024)
    x, s = d["logits"], d["sampler"]
    ref = O.sample(x, _osamp(s), seed=9, offset=1)
    xt = _t(x)
    a = engine.sample_rows(xt, s, seed=9, offset=1, return_status=True)
    e = engine.sample_rows(xt, s, seed=9, offset=1, return_lse=True, return_status=True)
    torch.cuda.synchronize()
    assert ((a["status"].cpu().numpy() & ~64) == 0).all()
    assert (e["status"].cpu().numpy() == 0).all()
    np.testing.assert_array_equal(a["tokens"].cpu().numpy(), ref["tokens"])
    np.testing.assert_array_equal(e["tokens"].cpu().numpy(), ref["tokens"])
    np.testing.assert_array_equal(e["lse"].cpu().numpy().view(np.uint32), ref["lse"].view(np.uint32))
