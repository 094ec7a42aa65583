"""Pin the CPU oracle to the reference's own kernels.

tests/golden/*.npz hold inputs and outputs of the reference's Triton kernels
run under Triton's CPU interpreter (tests/golden/make_golden.py). Every oracle
function must reproduce them; the one deliberate difference (LayerNorm
variance with non-power-of-two rows) is checked to be exactly the reference's
padding term."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    return {k: torch.from_numpy(np.asarray(z[k])) for k in z.files}


def test_golden_fixture_set_complete():
    names = {p.stem for p in GOLDEN.glob("*.npz")}
    expected = {"softmax_f32_6x100", "softmax_f32_4x64", "layernorm_f32_5x64", "layernorm_f32_5x96",
                "eltwise_relu_f32", "eltwise_gelu_f32", "eltwise_sigmoid_f32", "eltwise_identity_f32",
                "attention_float32_full", "attention_float32_causal", "attention_float16_full",
                "attention_float16_causal"}
    assert expected <= names
    assert sum(1 for n in names if n.startswith("gemm_")) >= 9


@pytest.mark.parametrize("name", ["softmax_f32_6x100", "softmax_f32_4x64"])
def test_softmax(name):
    d = load(name)
    torch.testing.assert_close(oracle.softmax(d["x"]), d["y"], rtol=1e-5, atol=1e-7)


def test_layernorm_power_of_two_rows():
    d = load("layernorm_f32_5x64")
    torch.testing.assert_close(oracle.layernorm(d["x"], d["w"], d["b"], float(d["eps"])), d["y"],
                               rtol=1e-5, atol=1e-5)


def test_layernorm_padded_rows_deviation_is_exactly_the_padding_term():
    d = load("layernorm_f32_5x96")
    # The reference's output is reproduced by the restatement with its padding term ...
    torch.testing.assert_close(oracle.layernorm_reference_padded(d["x"], d["w"], d["b"], float(d["eps"])), d["y"],
                               rtol=1e-5, atol=1e-5)
    # ... and differs from the exact LayerNorm the kernels implement (torch agrees with the latter).
    exact = oracle.layernorm(d["x"], d["w"], d["b"], float(d["eps"]))
    torch.testing.assert_close(exact, torch.nn.functional.layer_norm(d["x"], (96,), d["w"], d["b"], 1e-5),
                               rtol=1e-5, atol=1e-5)
    assert (exact - d["y"]).abs().max() > 1e-3


@pytest.mark.parametrize("op", ["relu", "gelu", "sigmoid", "identity"])
def test_elementwise(op):
    d = load(f"eltwise_{op}_f32")
    torch.testing.assert_close(oracle.unary(d["x"], op), d["y"], rtol=1e-5, atol=1e-6)


def test_tanh_matches_torch():
    x = torch.linspace(-6, 6, 1001)
    torch.testing.assert_close(oracle.unary(x, "tanh"), torch.tanh(x))


def test_gelu_tanh_vs_erf_within_published_gap():
    x = torch.randn(100000, generator=torch.Generator().manual_seed(0))
    assert (oracle.gelu_tanh(x) - oracle.gelu_erf(x)).abs().max() < 5e-4


GEMM_CASES = sorted(p.stem for p in GOLDEN.glob("gemm_*.npz"))


@pytest.mark.parametrize("name", GEMM_CASES)
def test_gemm(name):
    d = load(name)
    _, dtype, act, bias = name.split("_")
    act = None if act == "none" else act
    ref = d["c"].float()
    if dtype == "float32":
        out = oracle.gemm(d["a"], d["b"], d.get("bias"), activation=act)
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    else:
        # fp16 template: rounds the accumulator to fp16 before bias / activation
        # (triton_emitter.py:145-147); the oracle rounds once at the end.
        out = oracle.gemm(d["a"], d["b"], d.get("bias"), activation=act)
        assert oracle.rel_l2(out.half(), ref) < 1e-3
        assert (out.half().float() - ref).abs().max() < 2e-2 * max(1.0, ref.pow(2).mean().sqrt().item())


@pytest.mark.parametrize("name", ["attention_float32_full", "attention_float32_causal",
                                  "attention_float16_full", "attention_float16_causal"])
def test_attention(name):
    d = load(name)
    causal = name.endswith("causal")
    out = oracle.attention(d["q"], d["k"], d["v"], causal)
    if d["q"].dtype == torch.float32:
        torch.testing.assert_close(out, d["o"], rtol=1e-4, atol=1e-5)
    else:
        assert oracle.max_abs(out.half(), d["o"]) < 1e-2
        assert oracle.rel_l2(out.half(), d["o"]) < 2e-3


def test_qkv_split_is_a_permutation():
    B, S, H, D = 2, 5, 3, 4
    qkv = torch.arange(B * S * 3 * H * D, dtype=torch.float32).view(B, S, 3 * H * D)
    q, k, v = oracle.qkv_split(qkv, H)
    assert q.shape == (B, H, S, D)
    assert q[1, 2, 3, 0].item() == qkv[1, 3, 0 * H * D + 2 * D].item()
    assert v[0, 1, 4, 3].item() == qkv[0, 4, 2 * H * D + 1 * D + 3].item()


def test_encoder_block_matches_torch_modules():
    """The oracle block equals a block built from torch.nn functional pieces."""
    from oracle import inputs
    x, w = inputs.block_inputs(1, 16, seed=3, hidden=64, ffn=128)
    y = oracle.encoder_block(x, w, num_heads=4)
    F = torch.nn.functional
    qkv = F.linear(x, w["w_qkv"], w["b_qkv"]).view(1, 16, 3, 4, 16).permute(2, 0, 3, 1, 4)
    a = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2]).permute(0, 2, 1, 3).reshape(1, 16, 64)
    h = F.layer_norm(F.linear(a, w["w_o"], w["b_o"]) + x, (64,), w["ln1_w"], w["ln1_b"], 1e-5)
    f = F.gelu(F.linear(h, w["w_1"], w["b_1"]), approximate="tanh")
    ref = F.layer_norm(F.linear(f, w["w_2"], w["b_2"]) + h, (64,), w["ln2_w"], w["ln2_b"], 1e-5)
    torch.testing.assert_close(y, ref, rtol=1e-4, atol=1e-5)
