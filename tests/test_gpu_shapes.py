"""GPU parity at the benchmark configurations' own shapes, and of the drop-in
callables, bit for bit against the oracle.

* C3: all 256 masked rows of V=163,840 (the headline workload).
* C4: the full [32, 5, 151,552] verify pass, drafts sampled from q, in both
  modes (residual rejection sampling and greedy match).
* C5: more rows than twice the SM count (the one-warp-per-row merge) at
  V=262,144, unsharded and as eight emulated vocabulary shards.
* make_logits_processors(...) objects called as proc(tokens, logits)
  (reference verify_decode.py:830-831), the full log-softmax row
  (verify_decode.py:835, 839) and make_sampler(...)(logprobs).
* The streaming pass's candidate buffer when a row part meets sparse masked
  tiles (offered one value per lane) before a dense masked tile (offered four
  per lane): bf16 rows with an odd stride take that path.
"""

import numpy as np
import pytest
import torch

import oracle as O
from paged_moe_b200 import workloads as W
from paged_moe_b200.params import ProcessorSettings, SamplerSettings
from test_gpu_sample import _oproc, _osamp, assert_same, run_both

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("injected", [True, False])
def test_c3_full_batch(injected):
    d = W.c3(seed=11)
    ref, got = run_both(d["logits"], d["sampler"], mask=d["mask"], seed=5, injected=injected, surv=8)
    assert_same(ref, got, surv=8)


def _c4_both(d, s, mode, injected=True):
    from paged_moe_b200 import verify
    x, dl, drafts, y = d["target"], d["draft_logits"], d["drafts"], d["y"]
    B, K1, V = x.shape
    rng = np.random.default_rng(17)
    g = W.gumbel(rng, (B, K1, V)) if injected else None
    u = rng.random((B, K1, 2)) if injected else None
    ua = d["u_accept"] if injected else None
    ur = d["u_residual"] if injected else None
    toks, nacc = O.verify(x, drafts, y, _osamp(s), mode=mode, draft_logits=dl if mode == "residual" else None,
                          gumbel=g, uniform=u, u_accept=ua, u_residual=ur, seed=99, offset=3)
    res = verify(_t(x), _t(drafts), _t(y), s, mode=mode, draft_logits=_t(dl) if mode == "residual" else None,
                 gumbel=None if g is None else _t(g.reshape(B * K1, V)),
                 uniform=None if u is None else _t(u.reshape(B * K1, 2)),
                 u_accept=None if ua is None else _t(ua), u_residual=None if ur is None else _t(ur),
                 seed=99, offset=3, return_status=True)
    torch.cuda.synchronize()
    assert (res["status"].cpu().numpy() == 0).all()
    np.testing.assert_array_equal(res["n_accepted"].cpu().numpy(), nacc)
    np.testing.assert_array_equal(res["tokens"].cpu().numpy(), toks)
    return toks, nacc


def test_c4a_residual_full_shape():
    d = W.c4(seed=3)
    toks, nacc = _c4_both(d, SamplerSettings(temp=1.0), "residual")
    assert nacc.max() > 0 and nacc.min() < 4  # both accepts and rejections


def test_c4a_residual_filtered_philox():
    d = W.c4(seed=4)
    _c4_both(d, SamplerSettings(temp=0.8, top_k=20, top_p=0.9), "residual", injected=False)


def test_c4b_match_full_shape():
    d = W.c4(seed=5)
    _c4_both(d, SamplerSettings(temp=0.0), "match")


def test_c5_rows_beyond_twice_the_sms():
    """320 rows > 2 x 148 SMs: the one-warp-per-row merge, and the same rows
    as eight vocabulary shards."""
    from paged_moe_b200 import engine, shard
    d = W.c5(seed=6, B=320)
    x, s = d["logits"], d["sampler"]
    B, V = x.shape
    rng = np.random.default_rng(8)
    g = W.gumbel(rng, (B, V))
    ref = O.sample(x, _osamp(s), gumbel=g, seed=1, offset=2)
    kw = dict(gumbel=_t(g), seed=1, offset=2, return_lse=True, return_status=True)
    un = engine.sample_rows(_t(x), s, **kw)
    sh = shard.emulate(_t(x), 8, s, **kw)
    torch.cuda.synchronize()
    for got in (un, sh):
        assert (got["status"].cpu().numpy() == 0).all()
        np.testing.assert_array_equal(got["tokens"].cpu().numpy(), ref["tokens"])
        np.testing.assert_array_equal(got["lse"].cpu().numpy().view(np.uint32), ref["lse"].view(np.uint32))


def test_logits_processors_call_shape():
    """Each processor of make_logits_processors as the reference calls it,
    proc(tokens, logits [1, V]), chained, against the oracle's processors."""
    from paged_moe_b200 import make_logits_processors
    rng = np.random.default_rng(9)
    V = 151936
    x = W.peaked_logits(rng, 1, V, 2.5, 10.0, 32)
    hist = rng.integers(0, V, 300).astype(np.int32)
    hist[-40:] = hist[-80:-40]  # repeats inside every window
    procs = make_logits_processors(logit_bias={7: 1.5, 151935: -2.0}, repetition_penalty=1.3,
                                   repetition_context_size=64, presence_penalty=0.5, presence_context_size=32,
                                   frequency_penalty=0.25, frequency_context_size=128)
    assert [p.__name__ for p in procs] == ["logit_bias_processor", "repetition_penalty_processor",
                                           "presence_penalty_processor", "frequency_penalty_processor"]
    out = _t(x)
    for p in procs:
        out = p(_t(hist), out)
    torch.cuda.synchronize()
    want = O.process(x, hist=hist[None, :], proc=O.Proc(logit_bias={7: 1.5, 151935: -2.0}, repetition_penalty=1.3,
                                                        repetition_context_size=64, presence_penalty=0.5,
                                                        presence_context_size=32, frequency_penalty=0.25,
                                                        frequency_context_size=128))
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("mask_on", [False, True])
def test_logprobs_full_row(mask_on):
    """The row the reference yields: processed logits minus their
    log-sum-exp (verify_decode.py:835, 839), every element."""
    from paged_moe_b200 import engine
    rng = np.random.default_rng(10)
    B, V = 6, 151936
    x = W.peaked_logits(rng, B, V, 2.5, 10.0, 32)
    hist = rng.integers(0, V, (B, 500)).astype(np.int32)
    mask = W.bitmask(rng, B, V) if mask_on else None
    p = ProcessorSettings(repetition_penalty=1.1, repetition_context_size=100)
    lp, lse = engine.logprobs(_t(x), p, history=_t(hist), mask=None if mask is None else _t(mask.view(np.int32)))
    torch.cuda.synchronize()
    want = O.logprobs(x, hist=hist, proc=_oproc(p), mask=mask)
    want_lp = want[0] if isinstance(want, tuple) else want
    np.testing.assert_array_equal(lp.cpu().numpy().view(np.uint32), np.asarray(want_lp).view(np.uint32))


def test_make_sampler_on_logprobs():
    """sampler(logprobs) as verify_decode.py:839 calls it; the Philox offset
    advances by one per call."""
    from paged_moe_b200 import engine, make_sampler
    rng = np.random.default_rng(12)
    B, V = 4, 151936
    x = W.peaked_logits(rng, B, V, 2.5, 10.0, 32)
    lp, _ = engine.logprobs(_t(x))
    lpn = lp.cpu().numpy()
    sampler = make_sampler(temp=0.7, top_p=0.8, top_k=20, seed=4242)
    for call in range(3):
        tok = sampler(lp)
        torch.cuda.synchronize()
        want = O.sample(lpn, O.Sampler(temp=0.7, top_p=0.8, top_k=20), seed=4242, offset=call)["tokens"]
        np.testing.assert_array_equal(tok.cpu().numpy(), want)
    one = make_sampler(temp=0.0)(lp[0])  # a single row [V] gives a scalar token
    assert int(one) == int(np.argmax(lpn[0]))


def _sparse_then_dense_mask(B, V, period, sparse_counts):
    """Tile t of every row: phase t % period < len(sparse_counts) allows the
    first n slots of every lane's 32 (elements 128 j + 4 lane + c with
    4 j + c < n), the last phase allows every token."""
    W_ = (V + 31) // 32
    allowed = np.zeros((B, W_ * 32), dtype=bool)
    e = np.arange(1024)
    slot = (e // 128) * 4 + e % 4
    for t in range(V // 1024):
        ph = t % period
        sel = slot < sparse_counts[ph] if ph < len(sparse_counts) else np.ones(1024, bool)
        allowed[:, t * 1024:(t + 1) * 1024] = sel
    bits = allowed.reshape(B, W_, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    return bits.sum(axis=2).astype(np.uint32)


@pytest.mark.parametrize("top_k,B,V,period,sparse", [
    (50, 4, 262144, 2, (12,)),         # KC = 64: 384 single offers, then a dense tile
    (200, 24, 227328, 3, (12, 7)),     # KC = 256: 384 + 224 single offers, then a dense tile
])
def test_sparse_masked_tiles_before_a_dense_one(top_k, B, V, period, sparse):
    rng = np.random.default_rng(13)
    x = rng.standard_normal((B, V), dtype=np.float32) * np.float32(2.0)
    bits = W.to_bf16_bits(x)
    store = np.zeros((B, V + 1), dtype=np.uint16)  # odd row stride: the streaming pass, not the gather
    store[:, :V] = bits
    mask = _sparse_then_dense_mask(B, V, period, sparse)
    s = SamplerSettings(temp=1.0, top_k=top_k, top_p=0.97)
    g = W.gumbel(rng, (B, V))
    from paged_moe_b200 import engine
    xt = _t(store.view(np.int16)).view(torch.bfloat16)[:, :V]
    assert xt.stride(0) == V + 1
    res = engine.sample_rows(xt, s, mask=_t(mask.view(np.int32)), gumbel=_t(g), return_lse=True, return_status=True,
                             survivors=top_k)
    torch.cuda.synchronize()
    ref = O.sample(O.bf16_to_f32(bits), _osamp(s), mask=mask, gumbel=g, surv_cap=top_k)
    got = {k: v.cpu().numpy() for k, v in res.items()}
    got["lse"] = got["lse"]
    assert (got["status"] == 0).all()
    np.testing.assert_array_equal(got["tokens"], ref["tokens"])
    np.testing.assert_array_equal(got["n_surv"], ref["n_surv"])
    for b in range(B):
        n = int(ref["n_surv"][b])
        np.testing.assert_array_equal(got["surv_ids"][b, :n], ref["surv_ids"][b, :n])
