"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset is involved: the reference publishes no
numbers for this path, and its configs are defined by distributions).

C1  B=1,     V=151,936 fp32; N(0,1)*2.5, +10 at 32 ids; temp 0.7, top_k 20,
             top_p 0.8, repetition_penalty 1.05 over 256 ids ~ U[0, V)
C2  B=64,    V=151,936 bf16; N(0,1)*3, +8 at 16 ids per row; 4,096-id
             histories ~ bounded Zipf(1.1); presence 0.5, frequency 0.3, argmax
             (second run: min_p 0.05, temp 1.0)
C3  B=256,   V=163,840 fp32; N(0,1)*2, +9 at 64 ids per row; allowed-token
             bitmask of 4 blocks of 512 plus ~1,200 singletons; temp 1,
             top_k 50, top_p 0.95, Gumbel-max draw
C4  [32,5,151,552] fp32 target N(0,1)*2.5, +10 at 8 peaks per position;
             draft logits = target + N(0, 0.5); drafts sampled from the draft
             distribution; per-position uniforms
C5  B=1,024, V=262,144 fp32; N(0,1)*2.5 + 32 peaks; 8 contiguous shards;
             temp 0.8, top_k 64, top_p 0.9
"""

from __future__ import annotations

import numpy as np

from .params import ProcessorSettings, SamplerSettings

CONFIGS = {
    "C1": dict(B=1, V=151936),
    "C2": dict(B=64, V=151936),
    "C3": dict(B=256, V=163840),
    "C4": dict(B=32, K=4, V=151552),
    "C5": dict(B=1024, V=262144, shards=8),
}


def peaked_logits(rng, B: int, V: int, sigma: float, peak: float, n_peaks: int, per_row: bool = True):
    x = rng.standard_normal((B, V), dtype=np.float32) * np.float32(sigma)
    if per_row:
        for b in range(B):
            ids = rng.choice(V, size=n_peaks, replace=False)
            x[b, ids] += np.float32(peak)
    else:
        ids = rng.choice(V, size=n_peaks, replace=False)
        x[:, ids] += np.float32(peak)
    return x


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even."""
    u = x.astype(np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) >> 16).astype(np.uint16)


def zipf_ids(rng, n_rows: int, n: int, V: int, s: float = 1.1) -> np.ndarray:
    """Bounded Zipf(s) over ranks 1..V, rank r -> id r-1."""
    w = np.arange(1, V + 1, dtype=np.float64) ** (-s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    u = rng.random((n_rows, n))
    return np.minimum(np.searchsorted(cdf, u, side="right"), V - 1).astype(np.int32)


def bitmask(rng, B: int, V: int, n_blocks: int = 4, block: int = 512, n_single: int = 1200) -> np.ndarray:
    """Packed allowed-token words [B, ceil(V/32)]: blocks + singletons, >= 1 bit."""
    W = (V + 31) // 32
    allowed = np.zeros((B, V), dtype=bool)
    for b in range(B):
        starts = rng.choice(V - block, size=n_blocks, replace=False)
        for s0 in starts:
            allowed[b, s0:s0 + block] = True
        allowed[b, rng.choice(V, size=n_single, replace=False)] = True
        allowed[b, rng.integers(V)] = True
    pad = np.zeros((B, W * 32), dtype=bool)
    pad[:, :V] = allowed
    bits = pad.reshape(B, W, 32).astype(np.uint64) << np.arange(32, dtype=np.uint64)
    return bits.sum(axis=2).astype(np.uint32)


def gumbel(rng, shape) -> np.ndarray:
    """Injected Gumbel noise: uniforms in fp64, -log(-log u), rounded to fp32."""
    u = rng.random(shape)
    u = np.clip(u, 2.0 ** -53, 1.0 - 2.0 ** -53)
    return (-np.log(-np.log(u))).astype(np.float32)


def c1(seed: int = 0, B: int = 1, V: int = 151936):
    rng = np.random.default_rng(seed)
    x = peaked_logits(rng, B, V, 2.5, 10.0, 32)
    hist = rng.integers(0, V, size=(B, 256), dtype=np.int32)
    s = SamplerSettings(temp=0.7, top_k=20, top_p=0.8)
    p = ProcessorSettings(repetition_penalty=1.05, repetition_context_size=256)
    return dict(logits=x, hist=hist, sampler=s, proc=p)


def c2(seed: int = 0, B: int = 64, V: int = 151936, H: int = 4096, second: bool = False):
    rng = np.random.default_rng(seed)
    x = peaked_logits(rng, B, V, 3.0, 8.0, 16)
    bits = to_bf16_bits(x)
    hist = zipf_ids(rng, B, H, V)
    s = SamplerSettings(temp=1.0, min_p=0.05) if second else SamplerSettings(temp=0.0)
    p = ProcessorSettings(presence_penalty=0.5, presence_context_size=H,
                          frequency_penalty=0.3, frequency_context_size=H)
    return dict(logits_bf16=bits, hist=hist, sampler=s, proc=p)


def c3(seed: int = 0, B: int = 256, V: int = 163840):
    rng = np.random.default_rng(seed)
    x = peaked_logits(rng, B, V, 2.0, 9.0, 64)
    mask = bitmask(rng, B, V)
    s = SamplerSettings(temp=1.0, top_k=50, top_p=0.95)
    return dict(logits=x, mask=mask, sampler=s, proc=ProcessorSettings())


def c4(seed: int = 0, B: int = 32, K: int = 4, V: int = 151552):
    rng = np.random.default_rng(seed)
    tgt = peaked_logits(rng, B * (K + 1), V, 2.5, 10.0, 8).reshape(B, K + 1, V)
    dl = (tgt[:, :K] + rng.standard_normal((B, K, V), dtype=np.float32) * np.float32(0.5)).astype(np.float32)
    # drafts sampled from the draft distribution softmax(dl) by Gumbel-max
    g = gumbel(rng, (B, K, V))
    drafts = np.argmax(dl + g, axis=-1).astype(np.int32)
    y = rng.integers(0, V, size=B, dtype=np.int32)
    u_acc = rng.random((B, K))
    u_res = rng.random(B)
    return dict(target=tgt, draft_logits=dl, drafts=drafts, y=y, u_accept=u_acc, u_residual=u_res)


def c5(seed: int = 0, B: int = 1024, V: int = 262144):
    rng = np.random.default_rng(seed)
    x = peaked_logits(rng, B, V, 2.5, 10.0, 32)
    s = SamplerSettings(temp=0.8, top_k=64, top_p=0.9)
    return dict(logits=x, sampler=s, proc=ProcessorSettings())


class SyntheticTokenizer:
    """A tokenizer stand-in for the ThinkBudget workload: vocabulary `V`,
    piece i decodes to a seeded string of 1..8 characters, every 17th piece
    ends a sentence, and the think end tag is the last id."""

    def __init__(self, V: int = 151936, seed: int = 0):
        rng = np.random.default_rng(seed)
        self.V = V
        self.think_end_id = V - 1
        self._lens = rng.integers(1, 9, V)

    def get_vocab(self):
        return {f"t{i}": i for i in range(self.V)}

    def batch_decode(self, ids):
        out = []
        for (i,) in ids:
            if i == self.think_end_id:
                out.append("</think>")
            else:
                out.append("x" * (int(self._lens[i]) - 1) + ("." if i % 17 == 0 else "a"))
        return out

    def encode(self, text, add_special_tokens=False):
        return [11, 12, 13, self.think_end_id]


def ngram_histories(seed: int = 0, B: int = 32, H: int = 4096, V: int = 151936):
    """[B, H] histories made of repeated spans (so n-gram matches exist):
    each row draws 64-token spans, a third of them copies of earlier spans."""
    rng = np.random.default_rng(seed)
    h = np.empty((B, H), dtype=np.int32)
    for b in range(B):
        pos = 0
        while pos < H:
            n = min(64, H - pos)
            if pos >= 64 and rng.random() < 1 / 3:
                src = int(rng.integers(0, pos - n + 1))
                h[b, pos:pos + n] = h[b, src:src + n]
            else:
                h[b, pos:pos + n] = rng.integers(0, V, n)
            pos += n
    return h
