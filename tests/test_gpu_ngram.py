"""Batched n-gram drafts on the GPU against the reference's own outputs
(tests/golden/draft_ngram.json, made by running lookup_decode.draft_ngram)
and the oracle's restatement on long repetitive histories."""

import json
import os

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _batch(hists, k, n_min=3, n_max=8):
    from paged_moe_b200 import ngram
    H = max(1, max(len(h) for h in hists))
    arr = np.zeros((len(hists), H), dtype=np.int32)
    for i, h in enumerate(hists):
        arr[i, :len(h)] = h
    dev = torch.device("cuda")
    d, n, used = ngram.draft_ngram_batch(torch.from_numpy(arr).to(dev), k,
                                         torch.tensor([len(h) for h in hists], dtype=torch.int32, device=dev),
                                         n_min, n_max)
    torch.cuda.synchronize()
    d, n, used = d.cpu().numpy(), n.cpu().numpy(), used.cpu().numpy()
    return [d[i, :n[i]].tolist() for i in range(len(hists))], used


def test_reference_fixture():
    g = json.load(open(os.path.join(GOLDEN, "draft_ngram.json")))
    by_k = {}
    for c in g["cases"]:
        by_k.setdefault(c["k"], []).append(c)
    for k, cases in by_k.items():
        got, _ = _batch([c["tokens"] for c in cases], k, g["ngram_min"], g["ngram_max"])
        assert got == [c["out"] for c in cases], k


@pytest.mark.parametrize("k", [1, 4, 7])
def test_long_repetitive_histories(k):
    rng = np.random.default_rng(k)
    hists = []
    for b in range(48):
        H = int(rng.integers(0, 3000))
        base = rng.integers(0, 5 + b, size=max(H // 7, 1))
        h = np.tile(base, 8)[:H]
        flip = rng.random(H) < 0.05
        h[flip] = rng.integers(0, 50, size=int(flip.sum()))
        hists.append(h.tolist())
    got, used = _batch(hists, k)
    for b, h in enumerate(hists):
        ref, n = O.draft_ngram(h, k)
        assert got[b] == ref, b
        assert used[b] == n, b


def test_single_request_call_shape():
    from paged_moe_b200 import ngram
    assert ngram.draft_ngram([1, 2, 3, 4, 5, 9, 1, 2, 3], 2) == [4, 5]
    assert ngram.draft_ngram([1, 2], 3) == []
    assert ngram.draft_ngram([5] * 20, 4) == [5, 5, 5, 5]
