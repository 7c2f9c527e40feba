"""merge_attn_states and the N-way partial merge on the GPU.

Cases follow the reference's tests/test_merge.py; expectations come from the
oracle (oracle/merge.py, pinned to the reference formulas).
"""

import numpy as np
import pytest
import torch

import oracle
from flash_attn_b200._merge import _merge_partials, merge_attn_states

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_pair_merge_strided_and_extreme_lse(device, dtype):
    left = torch.randn((4, 3, 14), device=device).to(dtype)[1:, :, 1::2]
    right = torch.randn((3, 6, 7), device=device).to(dtype)[:, ::2]
    la = torch.tensor([[1000., -1000., -float("inf")], [-float("inf"), 0., 10.], [-float("inf"), -50., 50.]], device=device)
    lb = torch.tensor([[1001., -1001., 0.], [-float("inf"), -float("inf"), 11.], [1., 50., -50.]], device=device)
    lse_base = torch.empty((6, 6), device=device)
    lse = lse_base[::2, 1::2]
    out_base = torch.full((3, 3, 14), 99., device=device, dtype=dtype)
    out = out_base[..., 1::2]
    merge_attn_states(out, left, la, right, lb, lse)
    eo, el = oracle.merge_pair(left.cpu().double().numpy(), la.cpu().numpy(),
                               right.cpu().double().numpy(), lb.cpu().numpy())
    tol = dict(rtol=8e-3, atol=8e-3) if dtype == torch.bfloat16 else dict(rtol=2e-3, atol=2e-6)
    torch.testing.assert_close(out.cpu(), torch.from_numpy(eo).to(dtype), **tol)
    torch.testing.assert_close(lse.cpu(), torch.from_numpy(el).float(), rtol=1e-6, atol=2e-6)
    assert torch.equal(out_base.cpu()[..., ::2], torch.full((3, 3, 7), 99., dtype=dtype))


def test_merge_inplace_and_empty_nan_payload(device):
    left = torch.randn((2, 3, 4), device=device)
    right = torch.randn_like(left)
    la = torch.zeros((3, 2), device=device)
    lb = torch.ones_like(la)
    expected = (left.cpu() + right.cpu() * torch.e) / (1 + torch.e)
    merge_attn_states(left, left, la, right, lb, la)
    torch.testing.assert_close(left.cpu(), expected)
    torch.testing.assert_close(la.cpu(), torch.full((3, 2), torch.log(torch.tensor(1 + torch.e))))
    left.fill_(float("nan"))
    right.fill_(float("nan"))
    la.fill_(-float("inf"))
    lb.fill_(-float("inf"))
    merge_attn_states(left, left, la, right, lb, la)
    assert torch.equal(left.cpu(), torch.zeros_like(left.cpu()))
    assert torch.isneginf(la.cpu()).all()


@pytest.mark.parametrize("splits", [0, 1, 5, 40])
def test_merge_partials_noncontiguous_and_empty(device, splits):
    p = torch.randn((splits, 4, 6, 14), device=device)[:, 1:, ::2, 1::2]
    l = torch.randn((splits, 6, 6), device=device)[:, ::2, 1::2]
    if splits:
        l[:, 0, 1] = -float("inf")
        p[:, 1, 0] = float("nan")
    out, lse = _merge_partials(p, l)
    eo, el = oracle.merge_partials(p.cpu().double().numpy(), l.cpu().double().numpy())
    torch.testing.assert_close(out.cpu(), torch.from_numpy(eo).float(), rtol=1e-5, atol=5e-7)
    torch.testing.assert_close(lse.cpu(), torch.from_numpy(el).float(), rtol=1e-5, atol=5e-7)


def test_merge_partials_into_strided_bf16_out(device):
    p = torch.randn((8, 5, 4, 64), device=device)
    l = torch.randn((8, 4, 5), device=device) * 4
    base = torch.full((5, 4, 128), 7., device=device, dtype=torch.bfloat16)
    out = base[..., ::2]
    out_lse = torch.empty((4, 5), device=device)
    _merge_partials(p, l, out=out, out_lse=out_lse)
    eo, el = oracle.merge_partials(p.cpu().double().numpy(), l.cpu().double().numpy())
    torch.testing.assert_close(out.cpu().double(), torch.from_numpy(eo).to(torch.bfloat16).double(),
                               rtol=8e-3, atol=8e-3)
    np.testing.assert_allclose(out_lse.cpu().numpy(), el, rtol=1e-5, atol=1e-5)
    assert torch.equal(base.cpu()[..., 1::2], torch.full((5, 4, 64), 7., dtype=torch.bfloat16))
