"""Multi-process host logic on CPU: gloo ranks (world size 2 and 4).

The batch-sharding split and the tensor-parallel FFN's sequencing (weight
shards, rank-0 bias/residual placement, one all-reduce) run in child
processes over gloo, with a torch-eager stand-in for the kernel provider; the
result must equal the unsharded oracle block. A rank that dies before the
collective makes the others fail with a timeout instead of hanging."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lunara_b200.runtime.sharding import TPEncoderBlock, batch_shard, shard_ffn_weights
from oracle import inputs, oracle


class CpuOps:
    """The ops interface of lunara_b200.runtime.ops, computed with the oracle in fp32 on CPU."""

    @staticmethod
    def gemm(A, B, C, bias=None, residual=None, activation=None, b_layout="kn", **_):
        C.copy_(oracle.gemm(A, B, bias, activation=activation, residual=residual, b_layout=b_layout))
        return C

    @staticmethod
    def attention(q, k, v, causal=False, scale=None, out=None):
        out.copy_(oracle.attention(q, k, v, causal, scale))
        return out

    @staticmethod
    def layernorm(X, w, b, eps=1e-5, out=None):
        out.copy_(oracle.layernorm(X, w, b, eps))
        return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        x, w = inputs.block_inputs(2, 16, seed=7, hidden=64, ffn=256)
        blk = TPEncoderBlock(w, batch=2, seq=16, num_heads=4, world=world, rank=rank, dtype=torch.float32,
                             device="cpu", ops=CpuOps)
        blk.x.copy_(x.view(-1, 64))
        y = blk.run_kernels().clone()
        ref = oracle.encoder_block(x, w, num_heads=4).view(-1, 64)
        result_q.put((rank, (y - ref).abs().max().item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_ffn_matches_unsharded_block(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    errs = dict(q.get(timeout=10) for _ in range(world))
    assert len(errs) == world and max(errs.values()) < 1e-4, errs


def _shard_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        x, w = inputs.block_inputs(6, 16, seed=8, hidden=64, ffn=256)
        start, size = batch_shard(6, world, rank)
        y = oracle.encoder_block(x[start:start + size], w, num_heads=4)
        gathered = [None] * world
        dist.all_gather_object(gathered, (start, y))
        if rank == 0:
            full = torch.cat([t for _, t in sorted(gathered, key=lambda s: s[0])])
            ref = oracle.encoder_block(x, w, num_heads=4)
            result_q.put((full - ref).abs().max().item())
    finally:
        dist.destroy_process_group()


def test_batch_sharded_replicas_match_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert q.get(timeout=10) < 1e-5


def _dead_rank_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)   # leaves between steps, before the collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        result_q.put("completed")
    except Exception as e:  # the collective must fail, not hang
        result_q.put(type(e).__name__)


def test_rank_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung on a collective with a dead peer"
    assert q.get(timeout=5) != "completed"


@pytest.mark.parametrize("gb,world", [(64, 8), (64, 3), (5, 4), (8, 1)])
def test_batch_shard_partition(gb, world):
    parts = [batch_shard(gb, world, r) for r in range(world)]
    assert sum(s for _, s in parts) == gb
    assert all(parts[i][0] + parts[i][1] == parts[i + 1][0] for i in range(world - 1))
    assert max(s for _, s in parts) - min(s for _, s in parts) <= 1


def test_shard_ffn_weights_reassemble():
    _, w = inputs.block_inputs(1, 4, seed=9, hidden=64, ffn=256)
    shards = [shard_ffn_weights(w, 4, r) for r in range(4)]
    assert torch.equal(torch.cat([s["w_1"] for s in shards]), w["w_1"])
    assert torch.equal(torch.cat([s["w_2"] for s in shards], dim=1), w["w_2"])
    with pytest.raises(ValueError):
        shard_ffn_weights(w, 3, 0)
