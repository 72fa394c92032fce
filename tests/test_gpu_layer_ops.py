"""The decoder-layer kernels against the Transformers modules they replace.

``silu_mul`` must equal ``LlamaMLP``'s ``act_fn(gate) * up`` bit for bit;
``add_rmsnorm``'s residual sum must equal torch's ``residual + x`` bit for bit
and its normalised output ``LlamaRMSNorm`` within one unit in the last place
(the mean's summation order is the only difference), almost always exactly.
"""

import pytest
import torch

from inferkernellab_b200 import add_rmsnorm, silu_mul

pytestmark = pytest.mark.gpu

ULP = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}


def _hf_rmsnorm(hidden: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    norm = LlamaRMSNorm(hidden.shape[-1], eps=eps).to(device=hidden.device, dtype=hidden.dtype)
    with torch.no_grad():
        norm.weight.copy_(weight)
        return norm(hidden)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("rows,cols", [(256, 4096), (3, 64), (2048, 4096), (5, 200), (7, 1000)])
def test_add_rmsnorm_matches_llama_rmsnorm(dtype, rows, cols):
    gen = torch.Generator(device="cuda").manual_seed(rows * 7 + cols)
    residual = (torch.randn(rows, cols, device="cuda", generator=gen) * 2).to(dtype)
    x = torch.randn(rows, cols, device="cuda", generator=gen).to(dtype)
    weight = (1 + 0.1 * torch.randn(cols, device="cuda", generator=gen)).to(dtype)
    eps = 1e-6 if cols % 8 == 0 else 1e-5
    want_sum = residual + x
    want = _hf_rmsnorm(want_sum, weight, eps)
    keep = residual.clone()
    out, summed = add_rmsnorm(x, residual, weight, eps)
    torch.cuda.synchronize()
    assert summed.data_ptr() == residual.data_ptr()  # in place by default
    assert torch.equal(summed, want_sum)
    diff = (out.float() - want.float()).abs()
    assert bool((diff <= ULP[dtype] * want.float().abs().clamp_min(1e-3) * 2).all())
    assert (diff == 0).float().mean().item() > 0.99
    # out-of-place residual, and the no-add form
    out2, summed2 = add_rmsnorm(x, keep, weight, eps, residual_out=torch.empty_like(keep))
    assert summed2.data_ptr() != keep.data_ptr() and torch.equal(summed2, want_sum)
    assert torch.equal(out2, out)
    out3, same = add_rmsnorm(None, want_sum, weight, eps)
    assert same.data_ptr() == want_sum.data_ptr()
    assert torch.equal(out3, out)


def test_add_rmsnorm_strided_rows_take_the_scalar_path():
    """Rows that are not 16-byte aligned (odd column offset) still normalise correctly."""
    dtype = torch.bfloat16
    base = torch.randn(6, 130, device="cuda").to(dtype)
    residual = base[:, 1:129]  # row stride 130, start offset 1 element: unaligned
    x = torch.randn(6, 128, device="cuda").to(dtype)
    weight = torch.randn(128, device="cuda").to(dtype)
    want_sum = residual + x
    want = _hf_rmsnorm(want_sum, weight, 1e-6)
    out, summed = add_rmsnorm(x, residual, weight, 1e-6, residual_out=torch.empty_like(x))
    assert torch.equal(summed, want_sum)
    assert torch.allclose(out.float(), want.float(), atol=1e-3, rtol=2 * ULP[dtype])
    sum_view = torch.empty(6, 130, device="cuda", dtype=dtype)[:, 1:129]
    sum_view.copy_(want_sum)
    out_strided, _ = add_rmsnorm(None, sum_view, weight, 1e-6)
    assert torch.equal(out_strided, out)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("rows,inter", [(256, 14336), (3, 128), (2048, 1024), (5, 100)])
def test_silu_mul_bit_exact_against_torch(dtype, rows, inter):
    gen = torch.Generator(device="cuda").manual_seed(rows + inter)
    gate_up = (torch.randn(rows, 2 * inter, device="cuda", generator=gen) * 4).to(dtype)
    gate, up = gate_up[:, :inter], gate_up[:, inter:]
    want = torch.nn.functional.silu(gate) * up
    got = silu_mul(gate_up)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_layer_ops_validate_arguments():
    x = torch.randn(4, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.ones(64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="weight"):
        add_rmsnorm(x, x.clone(), w[:32], 1e-6)
    with pytest.raises(ValueError, match="dtype"):
        add_rmsnorm(x.half(), x.clone(), w, 1e-6)
    with pytest.raises(ValueError, match="equal width"):
        silu_mul(torch.randn(4, 63, device="cuda", dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        silu_mul(torch.randn(4, 64, dtype=torch.bfloat16))
