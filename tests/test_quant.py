"""Quantized weights: repack round trips (CPU) and the dequant-fused tcgen05 GEMM (GPU)."""
import numpy as np
import pytest
import torch

from lightbulb_b200 import ops
from lightbulb_b200.formats import gguf as G
from lightbulb_b200.formats import quant as Q


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_q4k_q80_repack_matches_cpp_dequant():
    from lightbulb_b200 import _native
    torch.manual_seed(0)
    x = torch.randn(6, 512) * 0.05
    for t, fn in ((G.GGML_Q4_K, Q.from_q4_k), (G.GGML_Q8_0, Q.from_q8_0)):
        raw = np.frombuffer(G.quantize(x, t), dtype=np.uint8).copy()
        qw = fn(raw, 6, 512)
        ref = _native.dequantize(t, torch.from_numpy(raw), 6 * 512).view(6, 512)
        assert torch.allclose(qw.dequantize(), ref, atol=2e-3, rtol=1e-2)


def test_awq_repack_and_rows_cols():
    g = torch.Generator().manual_seed(0)
    from lightbulb_b200.formats.awq import awq_dequant, random_awq_linear
    q, z, s = random_awq_linear(256, 512, 128, g)
    w = Q.from_awq(q, z, s, 128)
    ref = awq_dequant(q, z, s, 128)
    assert torch.allclose(w.dequantize(), ref, atol=1e-3, rtol=2e-3)
    assert torch.allclose(w.cols(128, 384).dequantize(), ref[:, 128:384], atol=1e-3, rtol=2e-3)
    gu = Q.interleave_rows(w.rows(slice(0, 128)), w.rows(slice(128, 256)))
    d = gu.dequantize()
    assert torch.allclose(d[64:128], ref[128:192], atol=1e-3, rtol=2e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["awq128", "q4k", "q80"])
@pytest.mark.parametrize("m", [1, 16, 77, 256, 600])
def test_gemm_quant_gpu(kind, m):
    torch.manual_seed(m)
    n, k = 512, 1024
    if kind == "awq128":
        from lightbulb_b200.formats.awq import random_awq_linear
        q, z, s = random_awq_linear(n, k, 128, torch.Generator().manual_seed(1))
        w = Q.from_awq(q, z, s, 128)
    else:
        x = torch.randn(n, k) * 0.05
        t = G.GGML_Q4_K if kind == "q4k" else G.GGML_Q8_0
        raw = np.frombuffer(G.quantize(x, t), dtype=np.uint8).copy()
        w = (Q.from_q4_k if kind == "q4k" else Q.from_q8_0)(raw, n, k)
    a = torch.randn(m, k).to(torch.bfloat16)
    ref = a.float() @ w.dequantize().T
    wd = w.to("cuda")
    out = ops.gemm(a.cuda(), wd)
    torch.cuda.synchronize()
    ops.check_errors()
    # exact dequantisation, bf16 operand and output rounding only (~1.5e-3)
    assert _rel(out.cpu(), ref) < 5e-3
    for sp in (1, 2, 3, 4, 8):
        o2 = ops.gemm_quant(a.cuda(), wd, splits=sp)
        ops.check_errors()
        assert _rel(o2.cpu(), ref) < 5e-3, sp


@pytest.mark.gpu
def test_gemm_quant_swiglu_gpu():
    from lightbulb_b200.formats.awq import random_awq_linear
    gen = torch.Generator().manual_seed(2)
    f, k = 256, 512
    gq = Q.from_awq(*random_awq_linear(f, k, 128, gen), 128)
    uq = Q.from_awq(*random_awq_linear(f, k, 128, gen), 128)
    w = Q.interleave_rows(gq, uq)
    a = (torch.randn(40, k) * 0.1).to(torch.bfloat16)
    ref = torch.nn.functional.silu(a.float() @ gq.dequantize().T) * (a.float() @ uq.dequantize().T)
    out = ops.gemm(a.cuda(), w.to("cuda"), mode=ops.EPI_SWIGLU)
    assert _rel(out.cpu(), ref) < 1e-2
