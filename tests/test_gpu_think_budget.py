"""Device ThinkBudget against the reference's own outputs
(tests/golden/think_budget.json: ThinkBudget.__call__ on the reference test's
tokenizer stand-in, SLACK_TOKENS = 4) and the forcing hook in the sampling
pass."""

import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


class PieceTok:
    """Same decoded pieces as the fixture's tokenizer stand-in."""

    think_end_id = 127

    def get_vocab(self):
        return {str(i): i for i in range(128)}

    def batch_decode(self, ids):
        return ["</think>" if i == 127 else ("." if i % 7 == 0 else "ab") for (i,) in ids]

    def encode(self, text, add_special_tokens=False):
        return [3, 5, 9, 127]


def _cases():
    return json.load(open(os.path.join(GOLDEN, "think_budget.json")))


def test_forced_tokens_batched():
    from paged_moe_b200.think_budget import ThinkBudget
    cases = _cases()
    tb = ThinkBudget(PieceTok(), 10, "", slack=4)
    T = max(len(c["generated"]) for c in cases)
    gen = np.zeros((len(cases), T), dtype=np.int32)
    for i, c in enumerate(cases):
        gen[i, :len(c["generated"])] = c["generated"]
    f = tb.forced(torch.from_numpy(gen).cuda(), torch.tensor([len(c["generated"]) for c in cases]).cuda(),
                  chars=[c["chars"] for c in cases]).cpu().numpy()
    for i, c in enumerate(cases):
        want = c["allowed"][0] if c["forced"] else -1
        assert f[i] == want, (i, c)
    assert any(c["forced"] for c in cases)


def test_processor_call_shape_matches_fixture():
    from paged_moe_b200.think_budget import ThinkBudget
    for c in _cases():
        tb = ThinkBudget(PieceTok(), c["chars"], "", slack=4)
        x = torch.tensor([c["logits"]], dtype=torch.float32, device="cuda")
        tb(torch.tensor([7]), torch.zeros_like(x))
        out = tb(torch.tensor([7] + c["generated"]), x)
        allowed = torch.nonzero(torch.isfinite(out[0])).flatten().cpu().tolist()
        assert allowed == c["allowed"]


def test_forcing_hook_in_the_sampling_pass():
    from paged_moe_b200 import engine
    from paged_moe_b200.params import ProcessorSettings, SamplerSettings
    rng = np.random.default_rng(3)
    B, V = 6, 50000
    x = torch.from_numpy(rng.standard_normal((B, V)).astype(np.float32)).cuda()
    forced = torch.tensor([-1, 5, 49999, -1, 1234, 7], dtype=torch.int32, device="cuda")
    p = ProcessorSettings(logit_bias=((1234, 2.5),))
    for s in (SamplerSettings(temp=0.0), SamplerSettings(temp=0.9, top_k=20, top_p=0.9), SamplerSettings(temp=1.0)):
        res = engine.sample_rows(x, s, p, forced=forced, return_lse=True, return_logprob=True, survivors=4)
        free = engine.sample_rows(x, s, p, return_lse=True)
        torch.cuda.synchronize()
        tok = res["tokens"].cpu().numpy()
        fo = forced.cpu().numpy()
        for b in range(B):
            if fo[b] >= 0:
                assert tok[b] == fo[b]
                xv = np.float32(x[b, fo[b]].item())
                want = xv + np.float32(2.5) if fo[b] == 1234 else xv
                assert np.float32(res["lse"][b].item()) == want
                assert res["logprob"][b].item() == 0.0
                assert res["surv_ids"][b, 0].item() == fo[b] and res["n_surv"][b].item() == 1
            else:
                assert tok[b] == free["tokens"][b].item()


def test_mtp_argmax_confidence():
    """argmax and max(softmax) of each row (reference mtp.py:731-746)."""
    from paged_moe_b200 import argmax_confidence
    rng = np.random.default_rng(4)
    x = torch.from_numpy((rng.standard_normal((5, 151936)) * 3).astype(np.float32)).cuda()
    tok, conf = argmax_confidence(x)
    torch.cuda.synchronize()
    ref_tok = torch.argmax(x, dim=-1)
    ref_conf = torch.softmax(x.double(), dim=-1).max(dim=-1).values
    assert torch.equal(tok.long(), ref_tok)
    torch.testing.assert_close(conf.double(), ref_conf, rtol=2e-6, atol=0)
