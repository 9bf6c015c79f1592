"""The oracle against fixtures produced by the reference's own code
(tests/golden/make_golden.py runs pagedmoe/lookup_decode.py,
think_budget.py and sampling.py on numpy stand-ins for mlx)."""

import json
import os

import numpy as np
import pytest

import oracle as O
from paged_moe_b200 import sampling as S

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load_verify():
    z = np.load(os.path.join(GOLDEN, "verify_greedy.npz"))
    meta = json.loads(str(z["meta"]))
    for i, c in enumerate(meta):
        c["logits"] = z[f"logits_{i}"]
        c["logprobs"] = z[f"logprobs_{i}"]
    return meta


@pytest.mark.parametrize("case", range(24))
def test_greedy_equality_acceptance_matches_reference(case):
    """lookup_decode._verify (reference lookup_decode.py:319-373): sample every
    row with the history that row would have seen, keep the drafts while they
    equal the picks, emit picks[:accepted+1]."""
    c = _load_verify()[case]
    proc = None
    if c["processor"]:
        proc = O.Proc(repetition_penalty=c["processor"]["repetition_penalty"],
                      repetition_context_size=c["processor"]["repetition_context_size"])
    hist = np.array([c["history"]], dtype=np.int32) if c["history"] else None
    toks, nacc = O.verify(c["logits"][None], [c["drafts"]], [c["y"]], O.Sampler(temp=0.0), mode="match",
                          hist=hist, proc=proc)
    n = int(nacc[0]) + 1
    assert list(toks[0, :n]) == c["tokens"]
    assert int(nacc[0]) == c["n_accepted"]
    # the emitted rows' log-probabilities (reference verify_decode.py:899, lookup_decode.py:358)
    feed = [c["y"]] + list(c["drafts"])
    for i in range(n):
        h = np.array([c["history"] + feed[: i + 1]], dtype=np.int32)
        lp, _ = O.logprobs(c["logits"][i][None], hist=h, proc=proc or O.Proc())
        np.testing.assert_allclose(lp[0], c["logprobs"][i], rtol=0, atol=2e-6)


def test_think_budget_force_is_the_mask():
    """ThinkBudget.__call__ (reference think_budget.py:75-109) forces one token
    by where(arange == tok, logits, -inf); the packed bitmask with that one bit
    set gives the same row, and the sampler can only return that token."""
    cases = json.load(open(os.path.join(GOLDEN, "think_budget.json")))
    assert any(c["forced"] for c in cases) and any(not c["forced"] for c in cases)
    for c in cases:
        x = np.array([c["logits"]], dtype=np.float32)
        V = x.shape[1]
        mask = np.zeros((1, (V + 31) // 32), dtype=np.uint32)
        for t in c["allowed"]:
            mask[0, t // 32] |= np.uint32(1 << (t % 32))
        got = O.process(x, mask=mask)
        want = np.full_like(x, -np.inf)
        want[0, c["allowed"]] = x[0, c["allowed"]]
        np.testing.assert_array_equal(got, want)
        if c["forced"]:
            t = c["allowed"][0]
            assert O.sample(x, O.Sampler(temp=0.0), mask=mask)["tokens"][0] == t
            g = np.zeros_like(x)
            assert O.sample(x, O.Sampler(temp=0.7, top_k=20, top_p=0.9), mask=mask, gumbel=g)["tokens"][0] == t


def test_sampling_defaults_match_reference():
    """pagedmoe/sampling.py:56-135 on the same inputs."""
    import tempfile
    g = json.load(open(os.path.join(GOLDEN, "sampling_defaults.json")))
    for f in g["families"]:
        assert S.family_for(f["model_type"], f["name"])[0] == f["family"], f
    for d in g["defaults"]:
        if d["name"] is None:
            out, src = S.defaults_for(None, "")
        else:
            root = os.path.join(tempfile.mkdtemp(), d["name"])
            os.makedirs(root)
            if d["generation_config"] is not None:
                with open(os.path.join(root, "generation_config.json"), "w") as fh:
                    json.dump(d["generation_config"], fh)
            out, src = S.defaults_for(root, d["model_type"])
        assert out == d["defaults"], d
        assert src == d["sources"], d
        assert S.describe(out, src) == d["describe"]
    for fcase in g["fills"]:
        class H:
            pass
        h = H()
        h.temperature, h.top_p, h.top_k, h.min_p = 0.0, 1.0, 0, 0.0
        h.repetition_penalty, h.repetition_context_size = 0.0, 20
        applied = S.fill(h, fcase["body"], fcase["defaults"], argv=fcase["argv"])
        assert applied == fcase["applied"]
        assert vars(h) == fcase["handler"]


def test_ngram_draft_matches_reference():
    """lookup_decode.draft_ngram (reference lookup_decode.py:184-221) on the
    fixture's 209 contexts."""
    g = json.load(open(os.path.join(GOLDEN, "draft_ngram.json")))
    for c in g["cases"]:
        assert O.draft_ngram(c["tokens"], c["k"], g["ngram_min"], g["ngram_max"])[0] == c["out"], c
