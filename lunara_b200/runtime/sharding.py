"""Multi-GPU execution of the encoder workloads: one process per GPU.

Two schemes, both on one node:

* Batch sharding (``batch_shard``): the encoder stack is a function of each
  sequence alone, so every rank holds a full weight replica and runs its own
  slice of the batch. There is no collective on the data path; the only
  cross-rank traffic is the timing reduction outside the timed region.

* Tensor-parallel FFN (``TPEncoderBlock``): the FFN's 3072 hidden units are
  split across ranks -- W1 by output rows ([F/n, Hd]), W2 by input columns
  ([Hd, F/n]) -- so each rank computes GELU(x1 W1_r^T + b1_r) W2_r^T, a
  partial [T, Hd] sum. One all-reduce (sum) over NVLink combines the partials.
  Rank 0's FFN2 epilogue also adds b2 and the residual x1, so the reduced sum
  is already g = f W2^T + b2 + x1 and LayerNorm follows directly.

The kernel provider (``ops``) and the all-reduce are injectable so that the
sequencing can be exercised by CPU ranks over gloo in the tests; on the GPU
they are ``lunara_b200.runtime.ops`` and ``torch.distributed.all_reduce``
(NCCL).
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Optional, Tuple

import torch


def batch_shard(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """(start, size) of this rank's contiguous batch slice; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def shard_ffn_weights(w: Dict[str, torch.Tensor], world: int, rank: int) -> Dict[str, torch.Tensor]:
    """This rank's FFN shard: w_1/b_1 rows and w_2 columns [r*F/n, (r+1)*F/n); the rest replicated."""
    ffn = w["w_1"].shape[0]
    if ffn % world != 0:
        raise ValueError(f"FFN width {ffn} is not divisible by {world} ranks")
    k = ffn // world
    lo, hi = rank * k, (rank + 1) * k
    out = dict(w)
    out["w_1"] = w["w_1"][lo:hi].contiguous()
    out["b_1"] = w["b_1"][lo:hi].contiguous()
    out["w_2"] = w["w_2"][:, lo:hi].contiguous()
    return out


def _default_allreduce(t: torch.Tensor) -> None:
    import torch.distributed as dist
    dist.all_reduce(t, op=dist.ReduceOp.SUM)


class TPEncoderBlock:
    """Encoder block with the FFN split across ``world`` ranks (attention replicated)."""

    def __init__(self, weights: Dict[str, torch.Tensor], batch: int, seq: int, num_heads: int, world: int,
                 rank: int, dtype: torch.dtype = torch.float16, device=None, eps: float = 1e-5,
                 ffn_activation: str = "gelu_tanh", ops=None,
                 allreduce: Optional[Callable[[torch.Tensor], None]] = None):
        if ops is None:
            from lunara_b200.runtime import ops as _ops
            ops = _ops
        self.ops = ops
        self.allreduce = allreduce or _default_allreduce
        self.world, self.rank = world, rank
        self.batch, self.seq, self.heads, self.eps = batch, seq, num_heads, eps
        self.ffn_activation = ffn_activation
        device = torch.device(device) if device is not None else torch.device("cuda")
        shard = shard_ffn_weights(weights, world, rank)
        self.w = {k: v.to(device=device, dtype=dtype).contiguous() for k, v in shard.items()}
        self.hidden = self.w["w_o"].shape[0]
        self.head_dim = self.hidden // num_heads
        T = batch * seq
        e = lambda n: torch.empty(T, n, dtype=dtype, device=device)  # noqa: E731
        self.x, self.qkv, self.attn, self.h = e(self.hidden), e(3 * self.hidden), e(self.hidden), e(self.hidden)
        self.x1, self.f, self.g, self.y = e(self.hidden), e(self.w["w_1"].shape[0]), e(self.hidden), e(self.hidden)
        self.scale = 1.0 / math.sqrt(self.head_dim)

    def run_kernels(self, x: Optional[torch.Tensor] = None) -> torch.Tensor:
        ops, w = self.ops, self.w
        x = self.x if x is None else x
        B, S, H, D = self.batch, self.seq, self.heads, self.head_dim
        ops.gemm(x, w["w_qkv"], self.qkv, bias=w["b_qkv"], b_layout="nk")
        t = self.qkv.view(B, S, 3, H, D)
        q, k, v = (t[:, :, i].permute(0, 2, 1, 3) for i in range(3))
        ops.attention(q, k, v, causal=False, scale=self.scale, out=self.attn.view(B, S, H, D).permute(0, 2, 1, 3))
        ops.gemm(self.attn, w["w_o"], self.h, bias=w["b_o"], residual=x, b_layout="nk")
        ops.layernorm(self.h, w["ln1_w"], w["ln1_b"], self.eps, out=self.x1)
        ops.gemm(self.x1, w["w_1"], self.f, bias=w["b_1"], activation=self.ffn_activation, b_layout="nk")
        lead = self.rank == 0
        ops.gemm(self.f, w["w_2"], self.g, bias=w["b_2"] if lead else None, residual=self.x1 if lead else None,
                 b_layout="nk")
        self.allreduce(self.g)
        ops.layernorm(self.g, w["ln2_w"], w["ln2_b"], self.eps, out=self.y)
        return self.y
