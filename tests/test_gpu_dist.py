"""Vocabulary-sharded sampling across real ranks (one process per GPU, NCCL
all-gather of the summaries): every rank's tokens equal the unsharded pass.
Skipped on machines with fewer than two GPUs."""

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from paged_moe_b200 import engine, shard as S, workloads as W
        from paged_moe_b200.params import SamplerSettings
        rng = np.random.default_rng(5)
        B, V = 64, 262144
        x = W.peaked_logits(rng, B, V, 2.5, 10.0, 32)
        spec = S.ShardSpec.of(rank, world, V)
        s = SamplerSettings(temp=0.8, top_k=64, top_p=0.9)
        xs = torch.from_numpy(np.ascontiguousarray(x[:, spec.lo:spec.hi])).to(dev)
        res = S.sample_vocab_sharded(xs, s, vocab_total=V, seed=9, offset=2, return_lse=True)
        ref = engine.sample_rows(torch.from_numpy(x).to(dev), s, seed=9, offset=2, return_lse=True)
        torch.cuda.synchronize(dev)
        np.testing.assert_array_equal(res["tokens"].cpu().numpy(), ref["tokens"].cpu().numpy())
        np.testing.assert_array_equal(res["lse"].cpu().numpy().view(np.uint32),
                                      ref["lse"].cpu().numpy().view(np.uint32))
        open(os.path.join(out_dir, f"ok{rank}"), "w").write("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_vocab_sharded_over_nccl():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _free_port(), d), nprocs=world, start_method="spawn", join=True)
        assert all(os.path.exists(os.path.join(d, f"ok{r}")) for r in range(world))
