"""Dense-layer epilogue kernels (residual add + RMSNorm, SiLU-and-mul) vs the eager
torch modules they replace, in bf16.

Tolerance: the residual add and SiLU-and-mul have the same rounding points as
torch and must agree exactly (or, for SiLU, within 1 bf16 ulp where exp may
differ); RMSNorm sums squares in a different order than torch's reduction, so
the normalised output may differ by 1 bf16 ulp on a small fraction of elements.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ulps(a, b):
    a, b = a.float(), b.float()
    ulp = torch.clamp(b.abs(), min=1e-30) * 2.0 ** -7
    return ((a - b).abs() / ulp)


@pytest.mark.parametrize("rows,hidden", [(1, 64), (8, 4096), (37, 1536), (300, 8192)])
@pytest.mark.parametrize("with_residual", [False, True])
def test_rmsnorm_matches_module(rows, hidden, with_residual):
    from lastkv_b200 import ops
    from lastkv_b200.hf import RMSNorm

    g = torch.Generator(device="cuda").manual_seed(rows * 7 + hidden)
    x = torch.randn((rows, hidden), generator=g, device="cuda").bfloat16()
    r = torch.randn((rows, hidden), generator=g, device="cuda").bfloat16() * 3
    norm = RMSNorm(hidden, 1e-5).cuda().bfloat16()
    with torch.no_grad():
        norm.weight.copy_(torch.rand(hidden, generator=g, device="cuda") + 0.5)
        if with_residual:
            h_ref = x + r
            h, out = ops.rmsnorm(x, norm.weight.detach(), 1e-5, r)
            torch.testing.assert_close(h, h_ref, rtol=0, atol=0)
        else:
            h_ref = x
            out = ops.rmsnorm(x, norm.weight.detach(), 1e-5)
        ref = norm(h_ref)
    u = _ulps(out, ref)
    frac = (u > 0.5).float().mean().item()
    print(f"rmsnorm rows={rows} hidden={hidden}: max {u.max().item():.2f} ulp, {frac:.4%} differ")
    assert u.max().item() <= 1.01 and frac <= 0.02


def test_rmsnorm_in_place_residual_and_strided_rows():
    from lastkv_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(3)
    big = torch.randn((16, 2 * 512), generator=g, device="cuda").bfloat16()
    x = big[:, :512]  # row stride 1024
    r = torch.randn((16, 512), generator=g, device="cuda").bfloat16()
    w = torch.ones(512, device="cuda", dtype=torch.bfloat16)
    expect = x + r
    h, _ = ops.rmsnorm(x, w, 1e-6, r, residual_out=r)  # in place into the residual
    assert h.data_ptr() == r.data_ptr()
    torch.testing.assert_close(r, expect, rtol=0, atol=0)


@pytest.mark.parametrize("rows,ffn", [(1, 8), (8, 14336), (100, 1024)])
def test_silu_mul_matches_torch(rows, ffn):
    from lastkv_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(rows + ffn)
    gu = (torch.randn((rows, 2 * ffn), generator=g, device="cuda") * 4).bfloat16()
    out = ops.silu_mul(gu)
    ref = torch.nn.functional.silu(gu[:, :ffn]) * gu[:, ffn:]
    u = _ulps(out, ref)
    print(f"silu_mul rows={rows} ffn={ffn}: max {u.max().item():.2f} ulp, exact {(u == 0).float().mean().item():.4%}")
    assert u.max().item() <= 1.01


def test_dense_rejects_bad_shapes():
    from lastkv_b200 import ops
    from lastkv_b200.contract import RMarinBackendContractError

    x = torch.zeros((4, 12), device="cuda", dtype=torch.bfloat16)  # hidden not a multiple of 8
    with pytest.raises(RMarinBackendContractError):
        ops.rmsnorm(x, torch.ones(12, device="cuda", dtype=torch.bfloat16), 1e-6)
    with pytest.raises(RMarinBackendContractError):
        ops.silu_mul(torch.zeros((4, 12), device="cuda", dtype=torch.bfloat16))


@pytest.mark.parametrize("rows,cols", [(8, 128256), (3, 1000), (1, 8), (5, 77)])
def test_argmax_rows_matches_torch(rows, cols):
    from lastkv_b200 import ops

    g = torch.Generator(device="cuda").manual_seed(rows * cols)
    pad = -(-cols // 8) * 8
    buf = torch.randn((rows, pad), generator=g, device="cuda").bfloat16()
    x = buf[:, :cols]  # row stride a multiple of 8, any column count
    x[0, cols // 3] = x[0].max() + 1  # a clear winner
    if rows > 1:
        x[1, :] = 0.5                  # all tied: the first index
    if rows > 2:
        x[2, cols // 2] = float("nan")  # NaN counts as the largest (torch.argmax)
    got = ops.argmax_rows(x)
    torch.testing.assert_close(got, x.argmax(-1), rtol=0, atol=0)
