"""Generate the golden fixtures from the reference's own code.

Runs pagedmoe/lookup_decode.py (`_verify`, `draft_ngram`),
pagedmoe/think_budget.py (`ThinkBudget`) and pagedmoe/sampling.py from a
checkout of noahclark556/paged-moe on numpy-backed stand-ins for mlx
(mlx_shim.py: the real mlx is Apple-only), and writes their inputs and
outputs next to this file.  The fixtures are committed; the tests read only
them, never the reference.

    python tests/golden/make_golden.py /path/to/paged-moe
"""

from __future__ import annotations

import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import mlx_shim  # noqa: E402


def rep_processor(penalty: float, ctx: int):
    """mlx-lm's repetition penalty as a plain function of (tokens, logits):
    every distinct id in the last `ctx` tokens, x < 0 ? x * p : x / p."""
    p = np.float32(penalty)

    def proc(tokens, logits):
        toks = np.asarray(tokens).reshape(-1)[-ctx:]
        if toks.size == 0:
            return logits
        out = np.array(logits, dtype=np.float32, copy=True)
        ids = np.unique(toks.astype(np.int64))
        sel = out[:, ids]
        out[:, ids] = np.where(sel < 0, sel * p, sel / p).astype(np.float32)
        return out

    return proc


def gen_verify(lookup_decode, rng):
    cases = []
    V = 512
    for case in range(24):
        k = int(rng.integers(1, 8))
        H = int(rng.integers(0, 40))
        hist = rng.integers(0, V, size=H).tolist()
        y = int(rng.integers(0, V))
        logits = (rng.standard_normal((k + 1, V)) * 2.0).astype(np.float32)
        with_proc = case % 2 == 1
        # drafts: copy the greedy pick for a random prefix, then diverge
        procs = [rep_processor(1.3, 16)] if with_proc else None
        seq = hist + [y]
        draft = []
        n_good = int(rng.integers(0, k + 1))
        for i in range(k):
            row = logits[i:i + 1]
            if procs:
                row = procs[0](np.array(seq, dtype=np.uint32), row)
            best = int(np.argmax(row))
            tok = best if i < n_good else (best + 1 + int(rng.integers(0, V - 1))) % V
            draft.append(tok)
            seq.append(tok)
        model = mlx_shim.ScriptedModel([logits])
        cache = [mlx_shim.TrimCache()]
        out = lookup_decode._verify(model, cache, y, draft, None, procs, hist + [y])
        cases.append(dict(
            V=V, k=k, history=hist, y=y, drafts=draft, logits=logits,
            processor=dict(repetition_penalty=1.3, repetition_context_size=16) if with_proc else None,
            tokens=[int(t) for t, _ in out], n_accepted=len(out) - 1,
            logprobs=np.stack([np.asarray(lp, dtype=np.float32) for _, lp in out]),
        ))
    return cases


def save_verify(cases, path):
    meta = [{k: v for k, v in c.items() if k not in ("logits", "logprobs")} for c in cases]
    arrays = {}
    for i, c in enumerate(cases):
        arrays[f"logits_{i}"] = c["logits"]
        arrays[f"logprobs_{i}"] = c["logprobs"]
    np.savez_compressed(path, meta=json.dumps(meta), **arrays)


def gen_draft_ngram(lookup_decode, config, rng):
    config.LOOKUP_NGRAM_MIN = 3
    config.LOOKUP_NGRAM_MAX = 8
    fixed = [
        ([1, 2, 3, 4, 5, 9, 1, 2, 3], 2), ([1, 2, 3, 4, 5, 9, 1, 2, 3], 1), ([1, 2, 3, 4, 5, 6], 3),
        ([1, 2], 3), ([1, 2, 3, 1, 2, 3], 0), ([3, 4, 9, 2, 3, 4, 7, 7, 7, 2, 3, 4], 1), ([5] * 20, 4),
        ([1, 2, 3, 4, 1, 2, 3], 4), ([7, 7, 7, 7], 4),
    ]
    cases = [dict(tokens=t, k=k, out=lookup_decode.draft_ngram(list(t), k)) for t, k in fixed]
    for _ in range(200):
        n = int(rng.integers(0, 60))
        toks = rng.integers(0, 6, size=n).tolist()
        k = int(rng.integers(0, 9))
        cases.append(dict(tokens=toks, k=k, out=lookup_decode.draft_ngram(list(toks), k)))
    return dict(ngram_min=3, ngram_max=8, cases=cases)


class PieceTok:
    """The reference test's tokenizer stand-in (tests/test_verify_decode.py:206-218)."""

    think_end_id = 127

    def get_vocab(self):
        return {str(i): i for i in range(128)}

    def batch_decode(self, ids):
        return ["</think>" if i == 127 else ("." if i % 7 == 0 else "ab") for (i,) in ids]

    def encode(self, text, add_special_tokens=False):
        return [3, 5, 9, 127]


def gen_think_budget(think_budget, rng):
    think_budget.SLACK_TOKENS = 4
    V = 128
    out = []
    for case in range(40):
        tb = think_budget.ThinkBudget(PieceTok(), int(rng.integers(4, 14)), "")
        first = np.array([7], dtype=np.uint32)
        tb(first, np.zeros((1, V), dtype=np.float32))
        gen = rng.integers(0, 127, size=int(rng.integers(1, 24))).tolist()
        logits = rng.standard_normal((1, V)).astype(np.float32)
        res = np.asarray(tb(np.array([7] + gen, dtype=np.uint32), logits))
        finite = np.isfinite(res[0])
        out.append(dict(chars=tb.chars, generated=gen, logits=logits[0].tolist(),
                        allowed=[int(i) for i in np.nonzero(finite)[0]],
                        forced=bool(finite.sum() == 1)))
    return out


def gen_sampling(sampling):
    def ckpt(name, gen=None):
        d = os.path.join(tempfile.mkdtemp(), name)
        os.makedirs(d)
        if gen is not None:
            with open(os.path.join(d, "generation_config.json"), "w") as f:
                json.dump(gen, f)
        return d

    fam = []
    for mt, name in [("qwen3_5_moe", "whatever"), ("qwen4_exp", ""), ("deepseek_v32", ""), ("glm4_moe", ""),
                     ("gpt_oss", ""), ("minimax_m3", "Qwen-ish-name"), ("custom", "GLM-5.2-4bit"),
                     ("custom", "my-model"), ("mixtral", ""), ("gemma3", ""), ("llama4", ""), ("phi4", ""),
                     ("granite", ""), ("kimi_k2", ""), ("", "Devstral-Small")]:
        fam.append(dict(model_type=mt, name=name, family=sampling.family_for(mt, name)[0]))
    gens = [
        ("PagedMoE-35B", {"temperature": 1.0, "top_p": 0.95, "top_k": 20, "do_sample": True}, "qwen3_5_moe"),
        ("Qwen3-235B-Instruct", {"temperature": 0.7, "top_p": 0.8, "top_k": 20}, "qwen3_moe"),
        ("q", {"temperature": 0.7, "repetition_penalty": 1.1}, "qwen3"),
        ("cad", {"do_sample": False}, "qwen3"), ("z", {"temperature": 0}, "qwen3"), ("x", None, "deepseek_v3"),
        ("my-model", None, "custom"), ("gpt-oss-120b", {"temperature": 1.0, "top_p": 1.0, "top_k": 0,
                                                        "repetition_penalty": 1.0}, "gpt_oss"),
        ("m", {"temperature": "hot", "top_k": True, "top_p": -1}, "minimax"),
        ("mini", {"min_p": 0.05, "temperature": 0.8}, "llama"),
    ]
    defaults = []
    for name, gen, mt in gens:
        out, src = sampling.defaults_for(ckpt(name, gen), mt)
        defaults.append(dict(name=name, generation_config=gen, model_type=mt, defaults=out, sources=src,
                             describe=sampling.describe(out, src)))
    defaults.append(dict(name=None, generation_config=None, model_type="", defaults=sampling.defaults_for(None, "")[0],
                         sources={}, describe=sampling.describe({}, {})))

    class Handler:
        def __init__(self):
            self.temperature, self.top_p, self.top_k, self.min_p = 0.0, 1.0, 0, 0.0
            self.repetition_penalty, self.repetition_context_size = 0.0, 20

    fills = []
    dflt = {"temperature": 0.6, "top_p": 0.95, "top_k": 20, "repetition_penalty": 1.05, "repetition_context_size": 64}
    for body, argv in [({}, []), ({"temperature": 0.0, "repetition_penalty": 1.2}, []),
                       ({}, ["--model", "m", "--temp", "0.2", "--top-k=5"]), ({"top_p": 0.5}, ["--min-p", "0.1"])]:
        h = Handler()
        applied = sampling.fill(h, body, dflt, argv=argv)
        fills.append(dict(body=body, argv=argv, defaults=dflt, applied=applied, handler=vars(h)))
    return dict(families=fam, defaults=defaults, fills=fills)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PAGED_MOE_REFERENCE", "")
    if not ref or not os.path.isdir(os.path.join(ref, "pagedmoe")):
        raise SystemExit("usage: make_golden.py /path/to/paged-moe")
    mlx_shim.install()
    sys.path.insert(0, ref)
    from pagedmoe import config, lookup_decode, sampling, think_budget  # noqa: E402

    rng = np.random.default_rng(20261201)
    save_verify(gen_verify(lookup_decode, rng), os.path.join(HERE, "verify_greedy.npz"))
    with open(os.path.join(HERE, "draft_ngram.json"), "w") as f:
        json.dump(gen_draft_ngram(lookup_decode, config, rng), f)
    with open(os.path.join(HERE, "think_budget.json"), "w") as f:
        json.dump(gen_think_budget(think_budget, rng), f)
    with open(os.path.join(HERE, "sampling_defaults.json"), "w") as f:
        json.dump(gen_sampling(sampling), f, indent=1)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
