"""tcgen05 projection GEMM against a plain PyTorch fp32 reference of the same
op, called through the C ABI (ffwd_b200_gemm_bf16 / ffwd_b200_gemm_tf32) on
device pointers."""

import pytest
import torch

from ffwd_b200 import native

pytestmark = pytest.mark.gpu

SHAPES = [
    # M, N, K, bn
    (1, 128, 64, 128),
    (128, 256, 64, 256),
    (300, 384, 384, 128),
    (777, 1152, 384, 128),
    (1000, 1024, 1024, 256),
    (2049, 4096, 1024, 256),
    (513, 1024, 3072, 256),
]


def _split(t):
    hi = t.to(torch.bfloat16)
    lo = (t - hi.float()).to(torch.bfloat16)
    return hi, lo


@pytest.mark.parametrize("M,N,K,bn", SHAPES)
def test_gemm_bf16_single_pass(M, N, K, bn):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.full((M, N), float("nan"), device="cuda")
    native.gemm_bf16(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, bn)
    ref = x.float() @ w.float().T
    err = (y - ref).abs().max().item()
    # fp32 accumulation over K products of bf16 values: only summation order differs
    assert err <= 1e-5 * K ** 0.5 * ref.abs().max().item() + 1e-4, err


@pytest.mark.parametrize("M,N,K,bn", SHAPES[2:5])
@pytest.mark.parametrize("passes", [2, 3])
def test_gemm_split_bf16(M, N, K, bn, passes):
    g = torch.Generator(device="cuda").manual_seed(M + N + passes)
    xf = torch.randn(M, K, device="cuda", generator=g)
    wf = torch.randn(N, K, device="cuda", generator=g)
    if passes == 2:
        wf = wf.to(torch.bfloat16).float()  # exactly representable weights
    xh, xl = _split(xf)
    wh, wl = _split(wf)
    y = torch.empty(M, N, device="cuda")
    native.gemm_bf16(xh.data_ptr(), wh.data_ptr(), y.data_ptr(), M, N, K, bn,
                     x_lo_ptr=xl.data_ptr(), w_lo_ptr=wl.data_ptr() if passes == 3 else None)
    ref = (xf.double() @ wf.double().T)
    rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 2e-5, rel


def _tf32(t):
    """Round f32 to tf32, ties away from zero (cvt.rna.tf32.f32)."""
    u = t.view(torch.int32)
    return ((u + 0x1000) & -0x2000).view(torch.float32)


@pytest.mark.parametrize("M,N,K,bn", SHAPES)
def test_gemm_tf32(M, N, K, bn):
    g = torch.Generator(device="cuda").manual_seed(M * 3 + N)
    x = _tf32(torch.randn(M, K, device="cuda", generator=g))
    w = _tf32(torch.randn(N, K, device="cuda", generator=g))
    y = torch.full((M, N), float("nan"), device="cuda")
    native.gemm_tf32(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, bn)
    ref = x.double() @ w.double().T
    # tf32 operands are exact in f32: only the f32 accumulation differs
    rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel < 2e-5, rel


def test_gemm_tf32_ignores_low_mantissa_bits():
    """kind::tf32 reads only the tf32 bits of each f32 operand: unrounded inputs
    give the product of their truncations (or roundings), never the exact f32
    product."""
    M, N, K = 256, 256, 1024
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g)
    y = torch.empty(M, N, device="cuda")
    native.gemm_tf32(x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, 256)
    exact = x.double() @ w.double().T
    rel = ((y.double() - exact).abs().max() / exact.abs().max()).item()
    assert 1e-6 < rel < 5e-3, rel
