"""Multi-GPU paths on 2+ GPUs (skipped with fewer): the tensor-parallel FFN
block (NCCL all-reduce of the FFN2 partials) and batch-sharded replicas, one
process per GPU, checked against the fp32 CPU oracle."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, q):
    import torch.distributed as dist

    from lunara_b200.runtime.sharding import TPEncoderBlock, batch_shard
    from oracle import inputs, oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        x, w = inputs.block_inputs(2, 128, seed=11)
        wh = {k: v.half().float() for k, v in w.items()}
        blk = TPEncoderBlock(w, batch=2, seq=128, num_heads=12, world=world, rank=rank, device=dev)
        blk.x.copy_(x.half().view(-1, 768).to(dev))
        y = blk.run_kernels()
        torch.cuda.synchronize()
        ref = oracle.encoder_block(x.half().float(), wh, num_heads=12).view(-1, 768)
        tp_err = oracle.max_abs(y, ref), oracle.rel_l2(y, ref)
        # batch-sharded replicas of the full block, no collective
        from lunara_b200.runtime.encoder import EncoderBlock
        start, size = batch_shard(4, world, rank)
        xb, wb = inputs.block_inputs(4, 128, seed=12)
        whb = {k: v.half().float() for k, v in wb.items()}
        rb = EncoderBlock(wb, batch=size, seq=128, num_heads=12, device=dev)
        rb.x.copy_(xb[start:start + size].half().reshape(-1, 768).to(dev))
        yb = rb.run_kernels()
        torch.cuda.synchronize()
        refb = oracle.encoder_block(xb[start:start + size].half().float(), whb, num_heads=12).reshape(-1, 768)
        q.put((rank, tp_err, (oracle.max_abs(yb, refb), oracle.rel_l2(yb, refb))))
    finally:
        dist.destroy_process_group()


@needs_two
def test_tp_ffn_and_batch_shards_on_two_gpus():
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs)
    res = [q.get(timeout=10) for _ in range(2)]
    for rank, (tp_abs, tp_rel), (b_abs, b_rel) in res:
        assert tp_abs <= 2e-2 and tp_rel <= 1e-3, (rank, tp_abs, tp_rel)
        assert b_abs <= 2e-2 and b_rel <= 1e-3, (rank, b_abs, b_rel)
