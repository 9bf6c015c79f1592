"""GPU parity of the verify pass (pm_verify through paged_moe_b200.verify)
against the oracle and the reference fixtures, bit for bit: accepted tokens,
acceptance counts and every row's own sample."""

import json
import os

import numpy as np
import pytest
import torch

import oracle as O
from paged_moe_b200 import workloads as W
from paged_moe_b200.params import ProcessorSettings, SamplerSettings

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = torch.device("cuda")


def _verify():
    from paged_moe_b200 import verify
    return verify


def _osamp(s: SamplerSettings) -> O.Sampler:
    return O.Sampler(temp=s.temp, top_p=s.top_p, min_p=s.min_p, min_tokens_to_keep=s.min_tokens_to_keep,
                     top_k=s.top_k)


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


@pytest.mark.parametrize("case", range(24))
def test_match_mode_reproduces_reference_fixture(case):
    """The reference's own _verify outputs (lookup_decode.py:319-373 run on
    the fixture's logits): greedy sampler, repetition penalty on odd cases."""
    z = np.load(os.path.join(GOLDEN, "verify_greedy.npz"))
    c = json.loads(str(z["meta"]))[case]
    x = z[f"logits_{case}"]
    p = ProcessorSettings()
    if c["processor"]:
        p = ProcessorSettings(repetition_penalty=c["processor"]["repetition_penalty"],
                              repetition_context_size=c["processor"]["repetition_context_size"])
    hist = _t(np.array([c["history"]], dtype=np.int32)) if c["history"] else None
    res = _verify()(_t(x[None]), _t(np.array([c["drafts"]], np.int32)), _t(np.array([c["y"]], np.int32)),
                    SamplerSettings(temp=0.0), p, history=hist, mode="match")
    torch.cuda.synchronize()
    n = int(res["n_accepted"][0]) + 1
    assert int(res["n_accepted"][0]) == c["n_accepted"]
    assert res["tokens"][0, :n].cpu().tolist() == c["tokens"]
    assert (res["tokens"][0, n:] == -1).all()


def _drafts_from_picks(rng, picks, V, k):
    """Drafts equal to the rows' picks for a random prefix, then different."""
    B = picks.shape[0]
    d = np.empty((B, k), dtype=np.int32)
    for b in range(B):
        good = int(rng.integers(0, k + 1))
        for i in range(k):
            d[b, i] = picks[b, i] if i < good else (picks[b, i] + 1 + int(rng.integers(0, V - 1))) % V
    return d


def _run(x, drafts, y, s, p=None, hist=None, hist_len=None, mask=None, mode="match", dl=None, injected=True,
         seed=5, bf16=False):
    p = p or ProcessorSettings()
    B, K1, V = x.shape
    k = K1 - 1
    rng = np.random.default_rng(seed)
    g = W.gumbel(rng, (B, K1, V)) if injected else None
    u = rng.random((B, K1, 2)) if injected else None
    ua = rng.random((B, k)) if injected else None
    ur = rng.random(B) if injected else None
    xo = x
    if bf16:
        bits = W.to_bf16_bits(x)
        xo = O.bf16_to_f32(bits)
        xt = _t(bits.view(np.int16)).view(torch.bfloat16)
    else:
        xt = _t(x)
    proc = O.Proc(repetition_penalty=p.repetition_penalty, repetition_context_size=p.repetition_context_size,
                  presence_penalty=p.presence_penalty, presence_context_size=p.presence_context_size,
                  frequency_penalty=p.frequency_penalty, frequency_context_size=p.frequency_context_size,
                  logit_bias=dict(p.logit_bias) if p.logit_bias else None)
    toks, nacc = O.verify(xo, drafts, y, _osamp(s), mode=mode, draft_logits=dl, hist=hist, hist_len=hist_len,
                          proc=proc, mask=mask, gumbel=g, uniform=u, u_accept=ua, u_residual=ur, seed=99,
                          offset=3)
    res = _verify()(xt, _t(drafts), _t(np.asarray(y, np.int32)), s, p,
                    history=None if hist is None else _t(hist),
                    history_len=None if hist_len is None else _t(np.asarray(hist_len, np.int32)),
                    mask=None if mask is None else _t(mask.view(np.int32)), mode=mode,
                    draft_logits=None if dl is None else _t(dl),
                    gumbel=None if g is None else _t(g.reshape(B * K1, V)),
                    uniform=None if u is None else _t(u.reshape(B * K1, 2)),
                    u_accept=None if ua is None else _t(ua), u_residual=None if ur is None else _t(ur),
                    seed=99, offset=3, return_status=True)
    torch.cuda.synchronize()
    assert (res["status"].cpu().numpy() == 0).all()
    np.testing.assert_array_equal(res["n_accepted"].cpu().numpy(), nacc)
    np.testing.assert_array_equal(res["tokens"].cpu().numpy(), toks)
    return toks, nacc


def _picks(x, s, injected_seed, B, K1, V):
    rng = np.random.default_rng(injected_seed)
    g = W.gumbel(rng, (B, K1, V))
    u = rng.random((B, K1, 2))
    out = O.sample(x.reshape(B * K1, V), _osamp(s), gumbel=g.reshape(B * K1, V), uniform=u.reshape(B * K1, 2))
    return out["tokens"].reshape(B, K1)


@pytest.mark.parametrize("s", [SamplerSettings(temp=0.0), SamplerSettings(temp=0.8, top_k=20, top_p=0.9),
                               SamplerSettings(temp=1.0, min_p=0.05), SamplerSettings(temp=0.7)])
def test_match_mode_batched(s):
    rng = np.random.default_rng(11)
    B, k, V = 7, 4, 5003
    x = W.peaked_logits(rng, B * (k + 1), V, 2.5, 9.0, 6).reshape(B, k + 1, V)
    picks = _picks(x, s, 5, B, k + 1, V)
    drafts = _drafts_from_picks(rng, picks, V, k)
    y = rng.integers(0, V, B).astype(np.int32)
    toks, nacc = _run(x, drafts, y, s)
    assert nacc.max() > 0  # some drafts were accepted


def test_match_mode_with_history_penalties_and_mask():
    rng = np.random.default_rng(12)
    B, k, V = 5, 3, 4100
    x = W.peaked_logits(rng, B * (k + 1), V, 2.0, 8.0, 8).reshape(B, k + 1, V)
    hist = rng.integers(0, V, (B, 300)).astype(np.int32)
    hl = rng.integers(0, 301, B).astype(np.int32)
    mask = W.bitmask(rng, B * (k + 1), V).reshape(B, k + 1, -1)
    p = ProcessorSettings(repetition_penalty=1.2, repetition_context_size=64, presence_penalty=0.4,
                          presence_context_size=32, frequency_penalty=0.2, frequency_context_size=128)
    s = SamplerSettings(temp=0.0)
    drafts = rng.integers(0, V, (B, k)).astype(np.int32)
    y = rng.integers(0, V, B).astype(np.int32)
    _run(x, drafts, y, s, p, hist=hist, hist_len=hl, mask=mask)


def test_match_mode_philox_noise():
    rng = np.random.default_rng(13)
    B, k, V = 4, 3, 3000
    x = W.peaked_logits(rng, B * (k + 1), V, 2.5, 9.0, 4).reshape(B, k + 1, V)
    drafts = rng.integers(0, V, (B, k)).astype(np.int32)
    y = rng.integers(0, V, B).astype(np.int32)
    _run(x, drafts, y, SamplerSettings(temp=0.9, top_k=30), injected=False)
    _run(x, drafts, y, SamplerSettings(temp=0.9), injected=False)


def _draft_side(rng, x, B, k, V, sigma=0.5):
    """q = the target rows plus noise; drafts sampled from softmax(q)."""
    dl = (x[:, :k, :] + rng.standard_normal((B, k, V)).astype(np.float32) * sigma).astype(np.float32)
    drafts = np.empty((B, k), dtype=np.int32)
    for b in range(B):
        for i in range(k):
            q = np.exp(dl[b, i].astype(np.float64) - dl[b, i].max())
            drafts[b, i] = rng.choice(V, p=q / q.sum())
    return dl, drafts


@pytest.mark.parametrize("s", [SamplerSettings(temp=0.0), SamplerSettings(temp=0.8, top_k=20, top_p=0.9),
                               SamplerSettings(temp=1.0), SamplerSettings(temp=0.6, min_p=0.02)])
@pytest.mark.parametrize("bf16", [False, True])
def test_residual_mode(s, bf16):
    rng = np.random.default_rng(21)
    B, k, V = 6, 4, 3000
    x = W.peaked_logits(rng, B * (k + 1), V, 2.5, 6.0, 8).reshape(B, k + 1, V)
    dl, drafts = _draft_side(rng, x, B, k, V)
    y = rng.integers(0, V, B).astype(np.int32)
    _run(x, drafts, y, s, mode="residual", dl=dl, bf16=bf16)


def test_residual_mode_philox_and_processors():
    rng = np.random.default_rng(22)
    B, k, V = 5, 3, 2600
    x = W.peaked_logits(rng, B * (k + 1), V, 2.0, 6.0, 8).reshape(B, k + 1, V)
    dl, drafts = _draft_side(rng, x, B, k, V, sigma=1.0)
    y = rng.integers(0, V, B).astype(np.int32)
    hist = rng.integers(0, V, (B, 50)).astype(np.int32)
    p = ProcessorSettings(repetition_penalty=1.1, repetition_context_size=20, logit_bias=((5, 2.0), (2599, -1.0)))
    for s in (SamplerSettings(temp=1.0), SamplerSettings(temp=0.7, top_k=40)):
        _run(x, drafts, y, s, p, hist=hist, mode="residual", dl=dl, injected=False)


def test_residual_rejects_and_resamples():
    """Drafts the target never picks: every request rejects at row 0 and the
    replacement comes from the residual."""
    rng = np.random.default_rng(23)
    B, k, V = 8, 2, 2048
    x = W.peaked_logits(rng, B * (k + 1), V, 1.0, 12.0, 1).reshape(B, k + 1, V)
    dl = np.zeros((B, k, V), dtype=np.float32)
    drafts = np.argmin(x[:, :k, :], axis=2).astype(np.int32)
    y = np.zeros(B, np.int32)
    for s in (SamplerSettings(temp=1.0), SamplerSettings(temp=1.0, top_k=64), SamplerSettings(temp=0.0)):
        toks, nacc = _run(x, drafts, y, s, mode="residual", dl=dl)
        assert (nacc == 0).all() and (toks[:, 0] >= 0).all()


def test_zero_drafts_is_plain_sampling():
    rng = np.random.default_rng(24)
    B, V = 6, 3000
    x = W.peaked_logits(rng, B, V, 2.5, 9.0, 4).reshape(B, 1, V)
    drafts = np.zeros((B, 0), dtype=np.int32)
    y = rng.integers(0, V, B).astype(np.int32)
    for mode in ("match", "residual"):
        toks, nacc = _run(x, drafts, y, SamplerSettings(temp=0.8, top_k=10), mode=mode,
                          dl=np.zeros((B, 0, V), np.float32))
        assert (nacc == 0).all()
