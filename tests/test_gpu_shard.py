"""Vocabulary-sharded sampling on one GPU (every shard's summary computed
here, concatenated as the all-gather would): bit-exact with the unsharded
pass and with the oracle's sharded restatement."""

import numpy as np
import pytest
import torch

import oracle as O
from paged_moe_b200 import shard as S
from paged_moe_b200 import workloads as W
from paged_moe_b200.params import ProcessorSettings, SamplerSettings
from test_gpu_sample import _osamp

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _both(x, s, n, p=None, hist=None, mask=None, injected=True, seed=3):
    from paged_moe_b200 import engine
    rng = np.random.default_rng(seed)
    B, V = x.shape
    g = W.gumbel(rng, (B, V)) if injected else None
    u = rng.random((B, 2)) if injected else None
    kw = dict(seed=77, offset=5, gumbel=None if g is None else _t(g), uniform=None if u is None else _t(u))
    h = None if hist is None else _t(hist)
    m = None if mask is None else _t(mask.view(np.int32))
    sh = S.emulate(_t(x), n, s, p, history=h, mask=m, return_lse=True, return_status=True, **kw)
    un = engine.sample_rows(_t(x), s, p, history=h, mask=m, return_lse=True, return_status=True, **kw)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in sh.items()}, {k: v.cpu().numpy() for k, v in un.items()}, g, u


@pytest.mark.parametrize("n", [2, 4, 8])
def test_c5_pipeline_matches_unsharded(n):
    rng = np.random.default_rng(50 + n)
    x = W.peaked_logits(rng, 24, 262144, 2.5, 10.0, 32)
    s = SamplerSettings(temp=0.8, top_k=64, top_p=0.9)
    sh, un, g, u = _both(x, s, n)
    assert (sh["status"] == 0).all()
    np.testing.assert_array_equal(sh["tokens"], un["tokens"])
    np.testing.assert_array_equal(sh["lse"].view(np.uint32), un["lse"].view(np.uint32))
    # and the oracle's sharded restatement
    spec = [S.ShardSpec.of(i, n, x.shape[1]) for i in range(n)]
    toks, lses = O.shard_sample([x[:, sp.lo:sp.hi] for sp in spec], _osamp(s), gumbel=g, uniform=u)
    np.testing.assert_array_equal(sh["tokens"], toks)


@pytest.mark.parametrize("s", [SamplerSettings(temp=0.0), SamplerSettings(temp=1.0), SamplerSettings(temp=0.7),
                               SamplerSettings(temp=0.9, min_p=0.1), SamplerSettings(temp=0.9, top_k=20)])
@pytest.mark.parametrize("injected", [True, False])
def test_modes_ragged_last_shard(s, injected):
    rng = np.random.default_rng(60)
    x = W.peaked_logits(rng, 10, 151936, 2.0, 6.0, 16)  # 8 shards of 19,456 ids, the last 15,744
    sh, un, _, _ = _both(x, s, 8, injected=injected)
    ok = sh["status"] == 0
    assert ok.all(), sh["status"]
    np.testing.assert_array_equal(sh["tokens"], un["tokens"])
    if s.temp > 0 and (s.top_k or s.min_p):
        np.testing.assert_array_equal(sh["lse"].view(np.uint32), un["lse"].view(np.uint32))


def test_processors_and_mask_sharded():
    rng = np.random.default_rng(61)
    B, V = 6, 65536
    x = W.peaked_logits(rng, B, V, 2.0, 7.0, 16)
    hist = rng.integers(0, V, (B, 500)).astype(np.int32)
    p = ProcessorSettings(repetition_penalty=1.3, repetition_context_size=256, presence_penalty=0.5,
                          presence_context_size=100, frequency_penalty=0.2, frequency_context_size=500,
                          logit_bias=((3, 4.0), (40000, 3.0), (65535, 5.0)))
    mask = W.bitmask(rng, B, V, n_single=4000)
    for s in (SamplerSettings(temp=0.0), SamplerSettings(temp=0.9, top_k=30, top_p=0.95), SamplerSettings(temp=1.0)):
        sh, un, _, _ = _both(x, s, 4, p=p, hist=hist, mask=mask)
        assert (sh["status"] == 0).all()
        np.testing.assert_array_equal(sh["tokens"], un["tokens"])


def test_survivors_and_logprob_sharded():
    rng = np.random.default_rng(62)
    x = W.peaked_logits(rng, 8, 131072, 2.0, 9.0, 32)
    s = SamplerSettings(temp=0.8, top_k=50, top_p=0.9)
    g = W.gumbel(rng, x.shape)
    from paged_moe_b200 import engine
    sh = S.emulate(_t(x), 4, s, gumbel=_t(g), survivors=50, return_logprob=True)
    un = engine.sample_rows(_t(x), s, gumbel=_t(g), survivors=50, return_logprob=True)
    torch.cuda.synchronize()
    for k in ("tokens", "n_surv", "surv_ids", "surv_probs", "logprob"):
        np.testing.assert_array_equal(sh[k].cpu().numpy(), un[k].cpu().numpy(), err_msg=k)


def test_shard_width_rule():
    assert S.shard_width(262144, 8) == 32768
    assert S.shard_width(151936, 8) == 19456
    with pytest.raises(ValueError):
        S.shard_width(2048, 8)


@pytest.mark.parametrize("n", [2, 4, 8])
@pytest.mark.parametrize("injected", [True, False])
@pytest.mark.parametrize("s", [SamplerSettings(temp=1.0, top_p=0.9), SamplerSettings(temp=0.8, min_p=0.02),
                               SamplerSettings(temp=1.0, top_p=0.5, min_p=0.01)])
def test_unbounded_rows_beyond_the_records(n, injected, s):
    # flat rows: an unbounded top-p / min-p keeps thousands of tokens, more
    # than the records' candidates; those rows are finished on their
    # gathered whole rows and must equal the unsharded pass bit for bit
    rng = np.random.default_rng(70 + n)
    B, V = 12, 65536
    x = (rng.standard_normal((B, V)) * 0.5).astype(np.float32)
    x[3] = W.peaked_logits(rng, 1, V, 2.0, 8.0, 4)[0]  # a peaked row the records do finish
    sh, un, _, _ = _both(x, s, n, injected=injected)
    np.testing.assert_array_equal(sh["tokens"], un["tokens"])
    np.testing.assert_array_equal(sh["lse"].view(np.uint32), un["lse"].view(np.uint32))
    np.testing.assert_array_equal(sh["status"], un["status"])
    assert (sh["status"] & 1).sum() == 0
