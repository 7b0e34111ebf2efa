"""The attention softmax's two exponentials, checked directly (B200 only).

The pair kernel takes an eighth of its exponentials off the MUFU unit with a
polynomial on the FMA pipe: n = round(x) by the 1.5 * 2^23 trick, 2^(x - n) by
a degree-3 polynomial fitted for this library, then 2^n applied through the
exponent field.  Through the library's self-check hook (spruce_exp2_selfcheck)
it is compared with exact 2^x (float64 on the host) and with MUFU's ex2.approx
over the range the softmax feeds it, x in [-126, 8]:
  * relative error of the polynomial <= 1e-4 (bf16 P is rounded at 3.9e-3);
  * after rounding both to bf16, as P is stored, they differ by at most 1 ulp.
"""
import numpy as np
import pytest
import torch

from spruce_research_b200 import _lib

pytestmark = pytest.mark.gpu


def _probe(x: torch.Tensor):
    poly = torch.empty_like(x)
    mufu = torch.empty_like(x)
    _lib.check(_lib.load().spruce_exp2_selfcheck(x.data_ptr(), x.numel(), poly.data_ptr(), mufu.data_ptr(),
                                                 _lib.stream_of(x)))
    torch.cuda.synchronize()
    return poly.cpu(), mufu.cpu()


def test_polynomial_exp2_error_bound_and_bf16_agreement_with_mufu():
    gen = torch.Generator().manual_seed(5)
    x = torch.cat([torch.rand(1 << 20, generator=gen) * 134.0 - 126.0,       # uniform over [-126, 8]
                   torch.rand(1 << 18, generator=gen) * 2.0 - 1.0,           # dense near 0 (most softmax args)
                   torch.arange(-126, 9, dtype=torch.float32),               # integers
                   torch.arange(-126, 8, dtype=torch.float32) + 0.5])         # rounding ties of n = round(x)
    poly, mufu = _probe(x.cuda())
    exact = np.exp2(x.double().numpy())
    rel = np.abs(poly.double().numpy() - exact) / exact
    w = int(rel.argmax())
    assert rel.max() <= 1e-4, (f"polynomial exp2 max relative error {rel.max():.3e} at x = {x[w].item()!r} "
                               f"(poly {poly[w].item()!r}, exact {exact[w]!r})")
    pb = poly.to(torch.bfloat16).view(torch.int16).int()
    mb = mufu.to(torch.bfloat16).view(torch.int16).int()
    assert (pb - mb).abs().max().item() <= 1, "bf16-rounded polynomial and MUFU exp2 differ by more than 1 ulp"
