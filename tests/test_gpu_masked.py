"""GPU parity of the masked-row gather pass (k_sample_masked) against the
oracle, bit for bit: sparse and dense masks (one and several windows),
processors, every sampler mode, bf16 rows, ragged vocabularies and the
degenerate masks."""

import numpy as np
import pytest
import torch

import oracle as O
from paged_moe_b200 import workloads as W
from paged_moe_b200.params import ProcessorSettings, SamplerSettings
from test_gpu_sample import _osamp, assert_same, run_both

pytestmark = pytest.mark.gpu

MODES = [SamplerSettings(temp=0.0), SamplerSettings(temp=0.9, top_k=40, top_p=0.9),
         SamplerSettings(temp=0.8, min_p=0.05), SamplerSettings(temp=1.0),
         SamplerSettings(temp=0.7, top_p=0.8)]


def _density_mask(rng, B, V, p):
    allowed = rng.random((B, V)) < p
    allowed[np.arange(B), rng.integers(0, V, B)] = True
    W_ = (V + 31) // 32
    pad = np.zeros((B, W_ * 32), dtype=bool)
    pad[:, :V] = allowed
    return (pad.reshape(B, W_, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(2).astype(np.uint32)


@pytest.mark.parametrize("density", [0.002, 0.03, 0.2, 0.7, 1.0])
@pytest.mark.parametrize("s", MODES)
def test_masked_modes_and_densities(density, s):
    rng = np.random.default_rng(int(density * 1000) + 7)
    B, V = 6, 50003
    x = W.peaked_logits(rng, B, V, 2.0, 7.0, 24)
    mask = _density_mask(rng, B, V, density)
    surv = 64 if (s.top_k or s.top_p < 1.0 or s.min_p > 0) and s.temp > 0 else 0
    ref, got = run_both(x, s, mask=mask, surv=surv)
    assert_same(ref, got, surv=surv)


def test_masked_with_processors():
    rng = np.random.default_rng(31)
    B, V = 5, 40000
    x = W.peaked_logits(rng, B, V, 2.0, 6.0, 16)
    mask = _density_mask(rng, B, V, 0.05)
    hist = rng.integers(0, V, (B, 400)).astype(np.int32)
    # history ids that are allowed, so the penalties hit kept tokens
    for b in range(B):
        ids = np.flatnonzero(np.unpackbits(mask[b].view(np.uint8), bitorder="little")[:V])
        hist[b, :200] = rng.choice(ids, 200)
    bias = tuple(sorted({(int(t), float(v)) for t, v in zip(rng.integers(0, V, 30), rng.normal(0, 3, 30))}))
    bias = tuple(dict(bias).items())
    p = ProcessorSettings(logit_bias=bias, repetition_penalty=1.3, repetition_context_size=128,
                          presence_penalty=0.7, presence_context_size=64, frequency_penalty=0.4,
                          frequency_context_size=400)
    for s in MODES:
        ref, got = run_both(x, s, p, hist=hist, mask=mask, surv=32 if s.top_k else 0)
        assert_same(ref, got, surv=32 if s.top_k else 0)


@pytest.mark.parametrize("s", MODES)
def test_masked_bf16(s):
    rng = np.random.default_rng(32)
    B, V = 4, 30000
    bits = W.to_bf16_bits(W.peaked_logits(rng, B, V, 2.0, 8.0, 12))
    mask = _density_mask(rng, B, V, 0.04)
    ref, got = run_both(None, s, mask=mask, bf16=bits)
    assert_same(ref, got)


def test_masked_bf16_odd_stride_takes_the_streaming_pass():
    rng = np.random.default_rng(33)
    B, V = 3, 20001
    bits = W.to_bf16_bits(W.peaked_logits(rng, B, V + 1, 2.0, 8.0, 12))
    mask = _density_mask(rng, B, V, 0.05)
    g = W.gumbel(rng, (B, V))
    s = SamplerSettings(temp=0.9, top_k=20)
    xf = O.bf16_to_f32(bits)[:, :V]
    ref = O.sample(np.ascontiguousarray(xf), _osamp(s), mask=mask, gumbel=g)
    from paged_moe_b200 import engine
    dev = torch.device("cuda")
    xt = torch.from_numpy(bits.view(np.int16)).to(dev).view(torch.bfloat16)[:, :V]  # row stride V + 1 (odd)
    res = engine.sample_rows(xt, s, mask=torch.from_numpy(mask.view(np.int32)).to(dev),
                             gumbel=torch.from_numpy(g).to(dev), return_status=True)
    torch.cuda.synchronize()
    assert (res["status"].cpu().numpy() == 0).all()
    np.testing.assert_array_equal(res["tokens"].cpu().numpy(), ref["tokens"])


@pytest.mark.parametrize("top_k", [20, 200])  # candidate buffers of KC = 64 and KC = 256
def test_masked_streaming_vector_offers_after_one_value_offers(top_k):
    """Masked bf16 rows on the streaming pass (odd row stride).  Even tiles
    give every lane exactly 12 allowed slots (one-value offers, 384 keys, no
    compaction), odd tiles are wholly allowed (vector offers of 256 keys at
    once): a warp whose row part holds such a pair must make room before the
    vector offers.  Tokens equal the oracle's."""
    rng = np.random.default_rng(71)
    B, V = 64, 64 * 1024
    nt = V // 1024
    bits = W.to_bf16_bits(W.peaked_logits(rng, B, V + 1, 2.0, 8.0, 12))
    allowed = np.zeros((B, V), dtype=bool)
    for t in range(1, nt, 2):
        allowed[:, t * 1024:(t + 1) * 1024] = True
    # lane l's slot s of a bf16 tile is element (s // 8) * 256 + 8 l + s % 8
    slots = np.argsort(rng.random((B, nt // 2, 32, 32)), axis=-1)[..., :12]
    lane = np.arange(32)[None, None, :, None]
    tile = np.arange(0, nt, 2)[None, :, None, None]
    idx = tile * 1024 + (slots // 8) * 256 + lane * 8 + slots % 8
    np.put_along_axis(allowed, idx.reshape(B, -1), True, axis=1)
    mask = (allowed.reshape(B, V // 32, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)).sum(2)
    mask = mask.astype(np.uint32)
    g = W.gumbel(rng, (B, V))
    s = SamplerSettings(temp=0.9, top_k=top_k)
    xf = np.ascontiguousarray(O.bf16_to_f32(bits)[:, :V])
    ref = O.sample(xf, _osamp(s), mask=mask, gumbel=g)
    from paged_moe_b200 import engine
    dev = torch.device("cuda")
    xt = torch.from_numpy(bits.view(np.int16)).to(dev).view(torch.bfloat16)[:, :V]  # row stride V + 1 (odd)
    res = engine.sample_rows(xt, s, mask=torch.from_numpy(mask.view(np.int32)).to(dev),
                             gumbel=torch.from_numpy(g).to(dev), return_status=True)
    torch.cuda.synchronize()
    assert (res["status"].cpu().numpy() == 0).all()
    np.testing.assert_array_equal(res["tokens"].cpu().numpy(), ref["tokens"])


def test_masked_degenerate_rows():
    """No allowed token, one allowed token, an allowed token with -inf logit."""
    rng = np.random.default_rng(34)
    B, V = 4, 5003
    x = rng.standard_normal((B, V)).astype(np.float32)
    mask = np.zeros((B, (V + 31) // 32), dtype=np.uint32)
    mask[1, 5002 // 32] |= np.uint32(1 << (5002 % 32))
    mask[2, 7 // 32] |= np.uint32(1 << 7)
    mask[2, 4000 // 32] |= np.uint32(1 << (4000 % 32))
    x[2, 7] = -np.inf
    mask[3] = _density_mask(rng, 1, V, 0.5)[0]
    for s in (SamplerSettings(temp=0.0), SamplerSettings(temp=0.8, top_k=10)):
        ref, got = run_both(x, s, mask=mask, want_lse=False)
        assert_same(ref, got, check_lse=False)
        assert got["tokens"][1] == 5002 and got["tokens"][2] == 4000


def test_c3_masked_philox_many_rows():
    d = W.c3(seed=21, B=40)
    ref, got = run_both(d["logits"], d["sampler"], mask=d["mask"], injected=False, surv=50)
    assert_same(ref, got, surv=50)


@pytest.mark.parametrize("bf16", [False, True])
def test_pinned_host_logits_read_in_place(bf16):
    """Logits and mask left in pinned host memory: the masked pass reads only
    the mask and the allowed logits from there; results equal the device run."""
    from paged_moe_b200 import engine
    rng = np.random.default_rng(41)
    B, V = 12, 163840
    x = W.peaked_logits(rng, B, V, 2.0, 9.0, 64)
    mask = W.bitmask(rng, B, V)
    s = SamplerSettings(temp=1.0, top_k=50, top_p=0.95)
    if bf16:
        xt = torch.from_numpy(W.to_bf16_bits(x).view(np.int16)).view(torch.bfloat16)
    else:
        xt = torch.from_numpy(x)
    mt = torch.from_numpy(mask.view(np.int32))
    kw = dict(seed=9, offset=4, return_lse=True, survivors=8, return_status=True)
    dev = engine.sample_rows(xt.cuda(), s, mask=mt.cuda(), **kw)
    host = engine.sample_rows(xt.pin_memory(), s, mask=mt.pin_memory(), **kw)
    torch.cuda.synchronize()
    assert host["tokens"].is_cuda
    for k in ("tokens", "lse", "surv_ids", "n_surv", "status"):
        assert torch.equal(host[k], dev[k]), k
    ref = O.sample(O.bf16_to_f32(W.to_bf16_bits(x)) if bf16 else x, _osamp(s), mask=mask, seed=9, offset=4)
    np.testing.assert_array_equal(host["tokens"].cpu().numpy(), ref["tokens"])


def test_pinned_host_logits_unbounded_rows_copied():
    """Rows with an unbounded filter (min_p, top_k off) may need the wide
    pass over whole rows: pinned host logits are copied to the device first,
    and the results equal the device run."""
    from paged_moe_b200 import engine
    rng = np.random.default_rng(43)
    B, V = 6, 65536
    x = W.peaked_logits(rng, B, V, 2.0, 9.0, 64)
    mask = W.bitmask(rng, B, V)
    s = SamplerSettings(temp=1.0, min_p=0.02)
    xt = torch.from_numpy(x)
    mt = torch.from_numpy(mask.view(np.int32))
    kw = dict(seed=3, offset=1, return_lse=True, return_status=True)
    dev = engine.sample_rows(xt.cuda(), s, mask=mt.cuda(), **kw)
    host = engine.sample_rows(xt.pin_memory(), s, mask=mt.pin_memory(), **kw)
    torch.cuda.synchronize()
    for k in ("tokens", "lse", "status"):
        assert torch.equal(host[k], dev[k]), k
    ref = O.sample(x, _osamp(s), mask=mask, seed=3, offset=1)
    np.testing.assert_array_equal(host["tokens"].cpu().numpy(), ref["tokens"])
