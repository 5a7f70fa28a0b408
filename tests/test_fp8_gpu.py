"""The block-scaled fp8 GEMM (tcgen05 kind::f8f6f4, scales per 128-wide K block) and its activation
quantizer, against fp32 PyTorch references of the same arithmetic."""

import math

import pytest
import torch

from everserve_b200.ops import (KernelOps, dequantize_fp8, interleave_gate_up, quantize_act_fp8,
                                quantize_weight_fp8)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return KernelOps("cuda:0")


def test_activation_quantizer_matches_its_restatement(kops):
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(37, 4096, device="cuda", generator=g) * 3).bfloat16()
    x[3, 128:256] = 0  # an all-zero block keeps scale 1
    q, s = kops.quant_fp8(x)
    qr, sr = quantize_act_fp8(x)
    assert torch.equal(s, sr)
    assert torch.equal(q.view(torch.uint8), qr.view(torch.uint8))


@pytest.mark.parametrize("M,N,K", [(64, 4096, 4096), (5, 1024, 1792), (1, 6144, 4096), (200, 384, 512),
                                   (64, 4096, 14336)])
def test_fp8_gemm_matches_dequantized_oracle(kops, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)
    w8, ws = quantize_weight_fp8(w)
    q, sc = kops.quant_fp8(x)
    y = kops.linear_fp8(x, w8, ws)
    torch.cuda.synchronize()
    assert kops.check_status() == 0
    oracle = dequantize_fp8(q, sc, 1) @ dequantize_fp8(w8, ws, 128).t()
    torch.testing.assert_close(y.float(), oracle, rtol=2e-2, atol=2e-2)
    # and close to the bf16 product it stands for (fp8 rounding of both operands)
    rel = (y.float() - x.float() @ w.t()).norm() / (x.float() @ w.t()).norm()
    assert rel < 0.08, rel


def test_fp8_gemm_residual_and_silu(kops):
    g = torch.Generator(device="cuda").manual_seed(5)
    M, N, K = 48, 3584, 4096
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    gu = torch.randn(N, K, device="cuda", generator=g) / 64
    w8, ws = quantize_weight_fp8(interleave_gate_up(gu))
    q, sc = kops.quant_fp8(x)
    prod = dequantize_fp8(q, sc, 1) @ dequantize_fp8(w8, ws, 128).t()  # interleaved columns
    fused = kops.linear_fp8(x, w8, ws, silu=True)
    v = prod.view(M, N // 128, 2, 64)
    gate, up = v[:, :, 0].reshape(M, N // 2), v[:, :, 1].reshape(M, N // 2)
    torch.testing.assert_close(fused.float(), torch.nn.functional.silu(gate) * up, rtol=3e-2, atol=3e-2)
    r = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    y = kops.linear_fp8(x, w8, ws, residual=r)
    torch.testing.assert_close(y.float(), prod + r.float(), rtol=2e-2, atol=3e-2)
    assert kops.check_status() == 0


def test_fp8_rows_independent_of_batch(kops):
    g = torch.Generator(device="cuda").manual_seed(6)
    w8, ws = quantize_weight_fp8(torch.randn(4096, 4096, device="cuda", generator=g) / 64)
    x = torch.randn(64, 4096, device="cuda", generator=g).bfloat16()
    full = kops.linear_fp8(x, w8, ws)
    assert torch.equal(kops.linear_fp8(x[:9].contiguous(), w8, ws), full[:9])
