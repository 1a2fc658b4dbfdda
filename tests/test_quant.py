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


def _awq_weight(n, k, group, seed):
    from lightbulb_b200.formats.awq import random_awq_linear
    q, z, s = random_awq_linear(n, k, group, torch.Generator().manual_seed(seed))
    w = Q.from_awq(q, z, s, group)
    # exact AWQ dequantisation (q - z) * s, the integer-weight kernel's arithmetic
    zz = z.float().repeat_interleave(group, 1)
    ss = w.scales.float().repeat_interleave(group, 1)
    return w, (q.float() - zz) * ss


@pytest.mark.gpu
@pytest.mark.parametrize("m", [1, 5, 16, 17, 32])
@pytest.mark.parametrize("n,k,group", [(512, 1024, 128), (704, 2048, 64), (4096, 4096, 128)])
def test_gemm_quant_int_zero_gpu(m, n, k, group):
    """Small-batch AWQ kernel (weights as exact integers in TMEM, per-group fp32 rescale)
    against the fp32 product with (q - z) * s, at every split of the cluster."""
    torch.manual_seed(m + n)
    w, wref = _awq_weight(n, k, group, m + k)
    assert w.int_zero and ops.use_int_zero_kernel(w)
    a = torch.randn(m, k).to(torch.bfloat16)
    ref = a.float() @ wref.T
    wd = w.to("cuda")
    out = ops.gemm(a.cuda(), wd)
    torch.cuda.synchronize()
    ops.check_errors()
    assert _rel(out.cpu(), ref) < 5e-3
    for sp in (1, 2, 3, 8):
        o2 = ops.gemm_quant(a.cuda(), wd, splits=sp)
        ops.check_errors()
        assert _rel(o2.cpu(), ref) < 5e-3, sp
    f32 = ops.gemm_quant(a.cuda(), wd, mode=ops.EPI_F32)
    ops.check_errors()
    assert _rel(f32.cpu(), ref) < 2e-3


@pytest.mark.gpu
def test_gemm_quant_int_zero_swiglu_and_zero_rows_gpu():
    gen_seed = 5
    f, k = 384, 1024
    gq, gref = _awq_weight(f, k, 128, gen_seed)
    uq, uref = _awq_weight(f, k, 128, gen_seed + 1)
    w = Q.interleave_rows(gq, uq)
    assert w.int_zero
    a = (torch.randn(9, k) * 0.1).to(torch.bfloat16)
    ref = torch.nn.functional.silu(a.float() @ gref.T) * (a.float() @ uref.T)
    out = ops.gemm(a.cuda(), w.to("cuda"), mode=ops.EPI_SWIGLU)
    ops.check_errors()
    assert _rel(out.cpu(), ref) < 1e-2
    # rows padded with scale = offset = 0 (narrow heads) give exact zeros
    pw = gq.pad_head_rows(3, 128, 192)
    o = ops.gemm(a.cuda(), pw.to("cuda")).cpu().float().view(9, 3, 192)
    ops.check_errors()
    assert torch.all(o[:, :, 128:] == 0)
    # deterministic: the same inputs give bit-identical outputs
    o1 = ops.gemm(a.cuda(), gq.to("cuda"))
    o2 = ops.gemm(a.cuda(), gq.to("cuda"))
    assert torch.equal(o1, o2)


def test_int_zero_flag_follows_slicing():
    w, _ = _awq_weight(256, 512, 128, 3)
    assert w.int_zero
    assert w.rows(torch.arange(128)).int_zero and w.cols(0, 256).int_zero
    assert Q.cat_rows([w, w]).int_zero and w.pad_head_rows(2, 128, 160).int_zero
    raw = np.frombuffer(G.quantize(torch.randn(64, 256) * 0.05, G.GGML_Q4_K), dtype=np.uint8).copy()
    assert not Q.from_q4_k(raw, 64, 256).int_zero
