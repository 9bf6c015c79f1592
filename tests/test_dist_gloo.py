"""The vocabulary-sharded exchange on two CPU ranks (gloo): each rank reduces
its slice of the rows to the record the GPU summary carries (best greedy
key, top-K candidate keys with global ids, tile statistics), the records
travel through paged_moe_b200.shard.gather_summaries, and a merge of the
gathered records reproduces the unsharded oracle's tokens and log-sum-exp.
The GPU kernels themselves are covered by tests/test_gpu_shard.py."""

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

B, V, N, K = 6, 8192, 2, 20


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _keys(x, lo):
    ids = np.arange(x.size, dtype=np.int64) + lo
    fin = np.isfinite(x)
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    o = np.where(u & 0x80000000, ~u & 0xFFFFFFFF, u | 0x80000000)
    k = (o << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - ids.astype(np.uint64))
    return k[fin]


def _record(x_shard, lo):
    """[B, 1 + K + 2 * tiles] uint64: best key, top-K keys (0-padded), tile max bits, tile sums."""
    nt = -(-x_shard.shape[1] // 1024)
    rec = np.zeros((B, 1 + K + 2 * nt), dtype=np.uint64)
    for b in range(B):
        k = np.sort(_keys(x_shard[b], lo))[::-1]
        rec[b, 0] = k[0]
        rec[b, 1:1 + min(K, k.size)] = k[:K]
        m, s = O.tile_stats(x_shard[b])
        rec[b, 1 + K:1 + K + nt] = np.asarray(m, dtype=np.float32).view(np.uint32)
        rec[b, 1 + K + nt:] = np.asarray(s, dtype=np.uint64)
    return rec


def _merge(recs, sampler, g):
    from oracle.oracle import _noise_for, _sample_one
    toks, lses = [], []
    for b in range(B):
        ms, ss, keys = [], [], []
        for r in recs:
            nt = (r.shape[1] - 1 - K) // 2
            ms.append(r[b, 1 + K:1 + K + nt].astype(np.uint32).view(np.float32))
            ss.append(r[b, 1 + K + nt:])
            keys.append(r[b, 1:1 + K])
        m = np.ascontiguousarray(np.concatenate(ms))
        s = np.ascontiguousarray(np.concatenate(ss))
        lse = O.lib().orc_combine_tiles(O.oracle._p(m), O.oracle._p(s), len(m))
        x = np.full(V, -np.inf, dtype=np.float32)
        for k in np.concatenate(keys):
            if k:
                idx = 0xFFFFFFFF - int(k & np.uint64(0xFFFFFFFF))
                o = int(k >> np.uint64(32))
                bits = (o & 0x7FFFFFFF) if (o & 0x80000000) else (~o & 0xFFFFFFFF)
                x[idx] = np.uint32(bits).view(np.float32)
        nz, _ = _noise_for(True, g[b], np.zeros(2), 0, 0, b)
        toks.append(_sample_one(x, np.float32(lse), sampler, nz)[0])
        lses.append(np.float32(lse))
    return np.array(toks), np.array(lses, dtype=np.float32)


def _worker(rank, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=N)
    try:
        from paged_moe_b200 import shard as S
        rng = np.random.default_rng(7)
        x = (rng.standard_normal((B, V)) * 2.0).astype(np.float32)
        g = (-np.log(-np.log(rng.random((B, V))))).astype(np.float32)
        w = V // N
        rec = _record(x[:, rank * w:(rank + 1) * w], rank * w)
        raw = torch.from_numpy(rec.view(np.uint8).reshape(-1).copy())
        got = S.gather_summaries(raw).numpy().view(np.uint64).reshape(N, B, -1)
        sampler = O.Sampler(temp=0.9, top_k=K, top_p=0.9)
        toks, lses = _merge([got[i] for i in range(N)], sampler, g)
        ref = O.sample(x, sampler, gumbel=g, uniform=np.zeros((B, 2)))
        np.testing.assert_array_equal(toks, ref["tokens"])
        np.testing.assert_array_equal(lses.view(np.uint32), ref["lse"].view(np.uint32))
        open(os.path.join(out_dir, f"ok{rank}"), "w").write("ok")
    finally:
        dist.destroy_process_group()


def test_sharded_exchange_two_gloo_ranks():
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(_free_port(), d), nprocs=N, start_method="spawn", join=True)
        assert all(os.path.exists(os.path.join(d, f"ok{r}")) for r in range(N))


def _gather_worker(rank, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=N)
    try:
        from paged_moe_b200 import shard as S
        full = torch.arange(5 * 3000, dtype=torch.float32).reshape(5, 3000)
        spec = S.ShardSpec.of(rank, N, 3000)
        idx = torch.tensor([4, 1, 2])
        got = S.gather_rows(full[:, spec.lo:spec.hi].contiguous(), idx, spec)
        np.save(os.path.join(out_dir, f"g{rank}.npy"), got.numpy())
    finally:
        dist.destroy_process_group()


def test_gather_rows_two_ranks():
    # the whole rows of flagged rows, rebuilt from every rank's slice
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_gather_worker, args=(port, d), nprocs=N, join=True, start_method="spawn")
        full = np.arange(5 * 3000, dtype=np.float32).reshape(5, 3000)
        for r in range(N):
            np.testing.assert_array_equal(np.load(os.path.join(d, f"g{r}.npy")), full[[4, 1, 2]])
