"""GPU parity of the whole BERT-base encoder block (B8 S512 H768, fp16) and of a
short stack against the fp32 CPU oracle, eager launches and CUDA-graph replay."""
import pytest
import torch

from oracle import inputs, oracle
from tests._tol import check_close

pytestmark = pytest.mark.gpu


def _half_roundtrip(w):
    return {k: v.half().float() for k, v in w.items()}


@pytest.mark.parametrize("fuse_layernorm", [True, False])
def test_encoder_block_benchmark_config(fuse_layernorm):
    from lunara_b200.runtime.encoder import EncoderBlock, GraphRunner
    x, w = inputs.block_inputs(8, 512, seed=0)
    xh, wh = x.half(), _half_roundtrip(w)
    ref = oracle.encoder_block(xh.float(), wh, num_heads=12)
    blk = EncoderBlock(w, batch=8, seq=512, num_heads=12, fuse_layernorm=fuse_layernorm)
    blk.x.copy_(xh.view(8 * 512, 768).cuda())
    y = blk.run_kernels().clone()
    check_close(y.view(8, 512, 768), ref, torch.float16, f"encoder block (eager, fused LN {fuse_layernorm})")
    runner = GraphRunner(blk.run_kernels)
    y2 = runner.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "graph replay differs from eager launches"
    runner.release()


def test_encoder_block_bf16_small():
    from lunara_b200.runtime.encoder import EncoderBlock
    x, w = inputs.block_inputs(2, 256, seed=5)
    wb = {k: v.bfloat16().float() for k, v in w.items()}
    ref = oracle.encoder_block(x.bfloat16().float(), wb, num_heads=12)
    blk = EncoderBlock(w, batch=2, seq=256, num_heads=12, dtype=torch.bfloat16)
    blk.x.copy_(x.bfloat16().view(-1, 768).cuda())
    y = blk.run_kernels()
    check_close(y.view(2, 256, 768), ref, torch.bfloat16, "encoder block bf16")


def test_encoder_stack_three_layers():
    from lunara_b200.runtime.encoder import EncoderStack
    x, ws = inputs.stack_inputs(batch=2, seq=128, layers=3, seed=4)
    wh = [_half_roundtrip(w) for w in ws]
    ref = oracle.encoder_stack(x.half().float(), wh, num_heads=12)
    st = EncoderStack(ws, batch=2, seq=128, num_heads=12)
    st.x.copy_(x.half().view(-1, 768).cuda())
    y = st.run_kernels()
    check_close(y.view(2, 128, 768), ref, torch.float16, "3-layer stack")
