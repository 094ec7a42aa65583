"""GPU parity of the drop-in Python surface the reference's users call.

The reference reaches its kernels only through generated launchers:
``Compiler.compile_transformer`` / ``Compiler.compile`` emit a module, and
``CompiledModel.get_launch_fn(name)`` returns ``{name}_launch`` with the
reference's signatures (lunara/driver.py:55-86, lunara/codegen/
triton_emitter.py:155-174, 296-316, 401-411). These tests run exactly those
generated functions on seeded inputs and compare them with the CPU oracle,
then run ``compiled.benchmark()``, the autotuner and the 12-layer stack.
"""
import math

import pytest
import torch

from lunara_b200.codegen.kernel_emitter import KernelKind
from oracle import inputs, oracle
from tests._tol import check_close

pytestmark = pytest.mark.gpu

BLOCK_NAMES = ["qkv_proj", "flash_attn", "out_proj", "layernorm_attn", "ffn1", "ffn2", "layernorm_ffn"]


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _run_launcher(compiled, spec, B, S, hidden, seed):
    """Call one generated launcher with seeded inputs of its own signature; return (out, ref)."""
    g = _gen(seed)
    fn = compiled.get_launch_fn(spec.name)
    dt = getattr(torch, spec.dtype)
    if spec.kind == KernelKind.GEMM:
        M = B * S
        a = torch.randn(M, hidden, generator=g).to(dt)
        w = (0.05 * torch.randn(hidden, hidden, generator=g)).to(dt)       # [K, N], the launcher's B
        bias = (0.1 * torch.randn(hidden, generator=g)).to(dt) if spec.has_bias else None
        res = torch.randn(M, hidden, generator=g).to(dt) if "residual" in spec.epilogue_ops else None
        c = torch.empty(M, hidden, dtype=dt, device="cuda")
        kw = {"residual": res.cuda()} if res is not None else {}
        out = fn(a.cuda(), w.cuda(), c, bias.cuda() if bias is not None else None, **kw)
        assert out.data_ptr() == c.data_ptr(), "the GEMM launcher writes into the caller's C"
        ref = oracle.gemm(a, w, bias, activation=spec.activation, residual=res)
        return out, ref
    if spec.kind == KernelKind.ATTENTION:
        D = spec.tile.HEAD_DIM
        q, k, v = (torch.randn(B, spec.num_heads, S, D, generator=g).to(dt) for _ in range(3))
        out = fn(q.cuda(), k.cuda(), v.cuda(), causal=spec.is_causal)
        return out, oracle.attention(q, k, v, spec.is_causal)
    if spec.kind == KernelKind.LAYERNORM:
        x = (3.0 * torch.randn(B, S, hidden, generator=g) + 0.5).to(dt)
        w = (1.0 + 0.1 * torch.randn(hidden, generator=g)).to(dt)
        b = (0.1 * torch.randn(hidden, generator=g)).to(dt)
        out = fn(x.cuda(), w.cuda(), b.cuda(), 1e-5)
        return out, oracle.layernorm(x, w, b, 1e-5)
    raise AssertionError(f"unexpected kernel kind {spec.kind}")


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_compile_transformer_launchers_match_oracle(tmp_path, dtype):
    from lunara_b200 import Compiler
    compiled = Compiler(dtype=dtype).compile_transformer(768, 12, 512, output_dir=str(tmp_path))
    assert [s.name for s in compiled.kernel_specs] == BLOCK_NAMES
    tdt = getattr(torch, dtype)
    for i, spec in enumerate(compiled.kernel_specs):
        out, ref = _run_launcher(compiled, spec, 8, 512, 768, seed=100 + i)
        assert out.dtype == tdt
        check_close(out, ref, tdt, f"{dtype} {spec.name}_launch")


def test_compiled_benchmark_returns_finite_times(tmp_path):
    from lunara_b200 import Compiler
    compiled = Compiler(dtype="float16").compile_transformer(768, 12, 512, output_dir=str(tmp_path))
    res = compiled.benchmark(batch_size=8, seq_len=512, n_warmup=2, n_trials=5)
    assert list(res) == BLOCK_NAMES
    for name, ms in res.items():
        assert math.isfinite(ms) and 0.0 < ms < 50.0, (name, ms)


def test_compile_onnx_graph_launchers_match_oracle(tmp_path):
    """Compiler.compile() on an ONNX encoder block (causal mask, tanh GELU), then the launchers
    its graph reader derived: residual-fused GEMMs, causal attention, LayerNorm."""
    from lunara_b200 import Compiler
    from tests.test_onnx_graph import attr_str, bert_block
    path = tmp_path / "encoder_block.onnx"
    path.write_bytes(bert_block(causal=True, act_attrs=[attr_str("approximate", "tanh")]))
    compiled = Compiler(dtype="float16").compile(str(path), output_dir=str(tmp_path / "out"))
    kinds = [s.kind for s in compiled.kernel_specs]
    assert kinds.count(KernelKind.GEMM) == 4 and kinds.count(KernelKind.LAYERNORM) == 2
    seen = set()
    for i, spec in enumerate(compiled.kernel_specs):
        out, ref = _run_launcher(compiled, spec, 2, 256, 768, seed=200 + i)
        check_close(out, ref, torch.float16, f"onnx {spec.name}_launch")
        seen.add((spec.kind, spec.activation, tuple(spec.epilogue_ops), spec.is_causal))
    assert (KernelKind.ATTENTION, None, (), True) in seen
    assert (KernelKind.GEMM, "gelu_tanh", (), False) in seen
    assert (KernelKind.GEMM, None, ("residual",), False) in seen


def test_autotuner_gemm_tuned_config_matches_oracle(tmp_path):
    from lunara_b200.codegen.autotuner import Autotuner, gemm_call_args
    from lunara_b200.runtime import ops
    tuner = Autotuner(cache_path=str(tmp_path / "cache.json"), n_warmup=2, n_trials=5, verbose=False)
    res = tuner.tune_gemm(1024, 768, 768, dtype=torch.float16, b_layout="nk")
    assert res.config.BLOCK_M in (128, 256) and res.latency_ms > 0 and res.tflops > 0
    a, b, bias = inputs.gemm_inputs(1024, 768, 768, seed=41)
    a, w, bias = a.half(), b.t().contiguous().half(), bias.half()          # w as a [N, K] Linear weight
    c = ops.gemm(a.cuda(), w.cuda(), bias=bias.cuda(), activation="gelu_tanh", b_layout="nk",
                 **gemm_call_args(res.config))
    check_close(c, oracle.gemm(a, w.t(), bias, activation="gelu_tanh"), torch.float16, "tuned GEMM")
    # cached: the second call answers from the JSON cache with the same config
    again = Autotuner(cache_path=str(tmp_path / "cache.json"), verbose=False).tune_gemm(
        1024, 768, 768, dtype=torch.float16, b_layout="nk")
    assert again.config == res.config


def test_autotuner_agrees_with_planner_on_out_proj_shape(tmp_path):
    """tune_gemm(4096, 768, 768) (the block's out_proj) against the planner's own choice:
    the planner's default launch is within 10% of the best configuration found."""
    from lunara_b200.codegen.autotuner import Autotuner, _bench
    from lunara_b200.runtime import ops
    tuner = Autotuner(cache_path=str(tmp_path / "cache.json"), n_warmup=3, n_trials=15, verbose=False)
    best = tuner.tune_gemm(4096, 768, 768, dtype=torch.float16, b_layout="nk")
    a = torch.randn(4096, 768, dtype=torch.float16, device="cuda")
    w = torch.randn(768, 768, dtype=torch.float16, device="cuda")
    c = torch.empty(4096, 768, dtype=torch.float16, device="cuda")
    planner_ms = _bench(lambda: ops.gemm(a, w, c, b_layout="nk"), 5, 30)
    assert planner_ms <= 1.10 * best.latency_ms, (planner_ms, best)


def test_attention_tuner_measures_the_kernel(tmp_path):
    from lunara_b200.codegen.autotuner import Autotuner
    res = Autotuner(cache_path=str(tmp_path / "c.json"), verbose=False).tune_attention(2, 12, 512, 512, 64)
    assert res.latency_ms > 0 and res.tflops > 10


def test_twelve_layer_stack_rank_share_matches_oracle():
    """One rank's share of the 8-GPU split of the 12-layer B64 stack: 12 layers at B8 S512,
    independent per-layer weights. Every layer matches the oracle's block on that layer's
    own (GPU-produced) input at the block tolerance, and the 12-layer output matches the
    oracle's 12-layer forward within the stacked bound of tests/_tol.py."""
    from lunara_b200.runtime.encoder import EncoderStack, GraphRunner
    from tests._tol import stack_rel_l2
    x, ws = inputs.stack_inputs(batch=8, seq=512, layers=12, seed=4)
    wh = [{k: v.half().float() for k, v in w.items()} for w in ws]
    st = EncoderStack(ws, batch=8, seq=512, num_heads=12)
    st.x.copy_(x.half().view(-1, 768).cuda())
    cur = st.x
    for i, blk in enumerate(st.blocks):
        nxt = torch.empty_like(cur)
        blk.run_kernels(cur, nxt)
        ref_i = oracle.encoder_block(cur.view(8, 512, 768).float().cpu(), wh[i], num_heads=12)
        check_close(nxt.view(8, 512, 768), ref_i, torch.float16, f"stack layer {i}")
        cur = nxt
    ref = oracle.encoder_stack(x.half().float(), wh, num_heads=12)
    y = st.run_kernels().clone()
    assert torch.equal(y, cur), "the stack's own forward differs from its layers run one by one"
    check_close(y.view(8, 512, 768), ref, torch.float16, "12-layer stack B8 S512",
                rel_l2=stack_rel_l2(torch.float16, 12))
    runner = GraphRunner(st.run_kernels)
    y2 = runner.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "graph replay of the stack differs from eager launches"
    runner.release()
