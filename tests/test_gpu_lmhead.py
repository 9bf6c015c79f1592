"""GPU parity of the LM head on the tensor cores and of its fused sampler.

pm_lmhead_logits is checked against an fp32 torch GEMM of the same bf16
operands (tolerance below: fp32 accumulation in a different order).  The
fused pm_lmhead_sample must give, bit for bit, what pm_sample_rows and the
CPU oracle give on the logits pm_lmhead_logits wrote (the same kernel's
accumulators): tokens, log-sum-exp bits, survivor ids and probabilities.
"""

import numpy as np
import pytest
import torch

import oracle as O
from paged_moe_b200 import workloads as W
from paged_moe_b200.params import SamplerSettings

pytestmark = pytest.mark.gpu


def _eng():
    from paged_moe_b200 import engine
    return engine


def _operands(B, H, V, seed, w_scale=0.05, dup=1):
    g = torch.Generator(device="cpu").manual_seed(seed)
    h = torch.randn((B, H), generator=g).to(torch.bfloat16)
    w = (torch.randn((V // dup + 1, H), generator=g) * w_scale).to(torch.bfloat16)
    if dup > 1:  # every weight row repeated: exact ties between ids
        w = w.repeat_interleave(dup, dim=0)
    w = w[:V].contiguous()
    return h.cuda(), w.cuda()


def _pack(allowed: np.ndarray) -> np.ndarray:
    """Packed mask words [B, ceil(V/32)]: bit v of word v/32; every row keeps id 0."""
    B, V = allowed.shape
    allowed = allowed.copy()
    allowed[:, 0] = True
    pad = np.zeros((B, (V + 31) // 32 * 32), dtype=bool)
    pad[:, :V] = allowed
    return np.packbits(pad, axis=1, bitorder="little").view(np.uint32)


def _gemm_fp32(h, w):
    return h.float() @ w.float().T


@pytest.mark.parametrize("B,H,V", [(128, 512, 2048), (200, 1000, 5003), (7, 64, 300), (256, 2048, 151936)])
def test_logits_match_fp32_gemm(B, H, V):
    h, w = _operands(B, H, V, seed=B + V)
    got = _eng().lmhead_logits(h, w)
    torch.cuda.synchronize()
    ref = _gemm_fp32(h, w)
    # fp32 accumulation of H products in another order: bounded by
    # H 2^-24 sum |h||w|; the tolerance is a quarter of that bound
    bound = (h.float().abs() @ w.float().abs().T) * (H * 2.0 ** -24 / 4) + 1e-30
    err = (got - ref).abs()
    assert bool((err <= bound).all()), float((err / bound).max())
    # and not trivially: the values carry information
    assert float(ref.std()) > 0.02 * H ** 0.5


MODES = {
    "greedy": SamplerSettings(temp=0.0),
    "k50_p95": SamplerSettings(temp=1.0, top_k=50, top_p=0.95),
    "k64_p90": SamplerSettings(temp=0.8, top_k=64, top_p=0.9),
    "k20_minp": SamplerSettings(temp=1.0, top_k=20, min_p=0.05),
    "k1": SamplerSettings(temp=1.0, top_k=1),
    "k200_p99": SamplerSettings(temp=1.2, top_k=200, top_p=0.99),
}


def _fused_vs_unfused(h, w, s, mask=None, seed=3, surv=0, injected=True, want_lse=True):
    eng = _eng()
    B, V = h.shape[0], w.shape[0]
    rng = np.random.default_rng(seed)
    g = torch.from_numpy(W.gumbel(rng, (B, V))).cuda() if injected else None
    mt = None if mask is None else torch.from_numpy(mask.view(np.int32)).cuda()
    logits = eng.lmhead_logits(h, w)
    ref = eng.sample_rows(logits, s, mask=mt, gumbel=g, seed=11, offset=5, return_lse=want_lse, survivors=surv,
                          return_status=True)
    got = eng.lmhead_sample(h, w, s, mask=mt, gumbel=g, seed=11, offset=5, return_lse=want_lse, survivors=surv,
                            return_status=True)
    torch.cuda.synchronize()
    ref = {k: v.cpu().numpy() for k, v in ref.items()}
    got = {k: v.cpu().numpy() for k, v in got.items()}
    assert (got["status"] == 0).all(), got["status"]
    assert ((ref["status"] & ~64) == 0).all(), ref["status"]
    np.testing.assert_array_equal(got["tokens"], ref["tokens"])
    if want_lse:
        np.testing.assert_array_equal(got["lse"].view(np.uint32), ref["lse"].view(np.uint32))
    if surv:
        np.testing.assert_array_equal(got["n_surv"], ref["n_surv"])
        for b in range(B):
            n = min(int(ref["n_surv"][b]), surv)
            np.testing.assert_array_equal(got["surv_ids"][b, :n], ref["surv_ids"][b, :n])
            np.testing.assert_array_equal(got["surv_probs"][b, :n].view(np.uint32),
                                          ref["surv_probs"][b, :n].view(np.uint32))
    return logits, got


@pytest.mark.parametrize("mode", list(MODES))
def test_fused_equals_unfused(mode):
    h, w = _operands(96, 1024, 40000, seed=5)
    _fused_vs_unfused(h, w, MODES[mode], surv=64 if mode != "greedy" else 0)


@pytest.mark.parametrize("mode", ["greedy", "k50_p95", "k20_minp"])
def test_fused_equals_oracle(mode):
    h, w = _operands(24, 512, 20000, seed=9)
    s = MODES[mode]
    B, V = 24, 20000
    rng = np.random.default_rng(21)
    g = W.gumbel(rng, (B, V))
    eng = _eng()
    logits = eng.lmhead_logits(h, w)
    got = eng.lmhead_sample(h, w, s, gumbel=torch.from_numpy(g).cuda(), return_lse=True, return_status=True)
    torch.cuda.synchronize()
    x = np.ascontiguousarray(logits.cpu().numpy())
    ref = O.sample(x, O.Sampler(temp=s.temp, top_p=s.top_p, min_p=s.min_p, min_tokens_to_keep=s.min_tokens_to_keep,
                                top_k=s.top_k), gumbel=g, uniform=None, seed=0, offset=0)
    np.testing.assert_array_equal(got["tokens"].cpu().numpy(), ref["tokens"])
    np.testing.assert_array_equal(got["lse"].cpu().numpy().view(np.uint32), ref["lse"].view(np.uint32))
    assert (got["status"].cpu().numpy() == 0).all()


def test_fused_with_mask():
    h, w = _operands(64, 768, 30000, seed=13)
    rng = np.random.default_rng(4)
    for dens in (0.02, 0.5, 0.0005):
        mask = _pack(rng.random((64, 30000)) < dens)
        for mode in ("greedy", "k50_p95", "k64_p90"):
            _fused_vs_unfused(h, w, MODES[mode], mask=mask, surv=32 if mode != "greedy" else 0)


def test_fused_ties_and_constant_rows():
    # repeated weight rows: exact ties across ids (lowest id wins); a zero
    # hidden row: every logit 0, every slice a tie of 256 values
    h, w = _operands(40, 256, 12000, seed=17, dup=8)
    h[3].zero_()
    h[17].zero_()
    for mode in ("greedy", "k50_p95", "k64_p90", "k200_p99", "k1"):
        _fused_vs_unfused(h, w, MODES[mode], surv=16 if mode != "greedy" else 0)


def test_fused_philox_and_per_row_settings():
    h, w = _operands(50, 512, 33000, seed=23)
    rows = [MODES[m] for m in ("greedy", "k50_p95", "k64_p90", "k20_minp", "k1")] * 10
    _fused_vs_unfused(h, w, rows, injected=False)


def test_fused_full_shape():
    # the LM-head shape of the benchmark: 256 rows, hidden 2048, vocabulary 151,936
    h, w = _operands(256, 2048, 151936, seed=29)
    _fused_vs_unfused(h, w, MODES["k50_p95"], injected=False)
    _fused_vs_unfused(h, w, MODES["greedy"], injected=False)


def test_fused_rejects_what_it_cannot_finish():
    h, w = _operands(8, 64, 1000, seed=31)
    eng = _eng()
    with pytest.raises(RuntimeError):
        eng.lmhead_sample(h, w, SamplerSettings(temp=1.0, top_p=0.9))  # unbounded top-p
    with pytest.raises(RuntimeError):
        eng.lmhead_sample(h, w, SamplerSettings(temp=1.0))  # whole-vocabulary draw


@pytest.mark.parametrize("mode", ["k1", "k200_p99", "k64_p90"])
def test_fused_ties_against_oracle(mode):
    # constant rows (every logit 0) and repeated weight rows, against the oracle
    h, w = _operands(16, 256, 9000, seed=37, dup=8)
    h[2].zero_()
    h[9].zero_()
    s = MODES[mode]
    B, V = 16, 9000
    g = W.gumbel(np.random.default_rng(41), (B, V))
    eng = _eng()
    logits = eng.lmhead_logits(h, w)
    got = eng.lmhead_sample(h, w, s, gumbel=torch.from_numpy(g).cuda(), return_lse=True, survivors=256,
                            return_status=True)
    torch.cuda.synchronize()
    x = np.ascontiguousarray(logits.cpu().numpy())
    ref = O.sample(x, O.Sampler(temp=s.temp, top_p=s.top_p, min_p=s.min_p, min_tokens_to_keep=s.min_tokens_to_keep,
                                top_k=s.top_k), gumbel=g, uniform=None, seed=0, offset=0, surv_cap=256)
    assert (got["status"].cpu().numpy() == 0).all()
    np.testing.assert_array_equal(got["tokens"].cpu().numpy(), ref["tokens"])
    np.testing.assert_array_equal(got["lse"].cpu().numpy().view(np.uint32), ref["lse"].view(np.uint32))
    np.testing.assert_array_equal(got["n_surv"].cpu().numpy(), ref["n_surv"])
    ids = got["surv_ids"].cpu().numpy()
    for b in range(B):
        n = int(ref["n_surv"][b])
        np.testing.assert_array_equal(ids[b, :n], ref["surv_ids"][b, :n])


def test_fused_with_processors():
    # C1's settings (top_k 20, top_p 0.8, repetition over a 256-id window)
    # plus presence, frequency and logit bias, per-row histories
    from paged_moe_b200.params import ProcessorSettings
    eng = _eng()
    h, w = _operands(48, 512, 30000, seed=43)
    rng = np.random.default_rng(44)
    hist = torch.from_numpy(rng.integers(0, 30000, (48, 300)).astype(np.int32)).cuda()
    hist[:, 100:140] = 7  # repeats: frequency counts above one
    hl = torch.from_numpy(rng.integers(1, 301, 48).astype(np.int32)).cuda()
    g = torch.from_numpy(W.gumbel(rng, (48, 30000))).cuda()
    procs = [ProcessorSettings(repetition_penalty=1.05, repetition_context_size=256),
             ProcessorSettings(repetition_penalty=1.3, repetition_context_size=64, presence_penalty=0.5,
                               presence_context_size=100, frequency_penalty=0.2, frequency_context_size=300,
                               logit_bias=((3, 4.0), (29999, 2.5), (1000, -3.0)))]
    for p in procs:
        for s in (SamplerSettings(temp=0.7, top_k=20, top_p=0.8), SamplerSettings(temp=0.0),
                  SamplerSettings(temp=1.0, top_k=64, min_p=0.05)):
            logits = eng.lmhead_logits(h, w)
            ref = eng.sample_rows(logits, s, p, history=hist, history_len=hl, gumbel=g, return_lse=True,
                                  return_status=True)
            got = eng.lmhead_sample(h, w, s, p, history=hist, history_len=hl, gumbel=g, return_lse=True,
                                    return_status=True)
            torch.cuda.synchronize()
            assert (got["status"].cpu() == 0).all(), got["status"]
            np.testing.assert_array_equal(got["tokens"].cpu().numpy(), ref["tokens"].cpu().numpy())
            np.testing.assert_array_equal(got["lse"].cpu().numpy().view(np.uint32),
                                          ref["lse"].cpu().numpy().view(np.uint32))
