"""tcgen05 decode GEMM (lkv_decode_gemm) vs a float64 reference and torch's bf16 nn.Linear.

The kernel accumulates in fp32 and rounds once to bf16, like cuBLAS; only the
summation order differs.  Tolerance: every output within 1 bf16 ulp of the
float64 result rounded to bf16 plus the fp32 accumulation bound
(K * 2^-24 * sum |x||w|), and the SiLU-and-mul epilogue bit-exact with the
eager torch ops applied to the kernel's own bf16 GEMM outputs.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(m, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((m, k), generator=g, device="cuda").bfloat16()
    w = (torch.randn((n, k), generator=g, device="cuda") * k ** -0.5).bfloat16()
    return x, w


def _check_plain(y, x, w):
    ref = x.double() @ w.double().T
    bound = k_bound = x.shape[1] * 2.0 ** -24 * (x.double().abs() @ w.double().abs().T)
    ulp = torch.clamp(ref.abs(), min=1e-30) * 2.0 ** -7
    err = (y.double() - ref).abs()
    ok = err <= ulp + k_bound + 1e-30
    assert bool(ok.all()), f"max err/ulp {float((err / ulp).max()):.2f}"
    return bound


@pytest.mark.parametrize("m,n,k", [(1, 128, 64), (8, 6144, 4096), (8, 4096, 4096), (8, 4096, 14336),
                                   (16, 1000, 200), (3, 77, 8), (5, 300, 1032)])
def test_plain_matches_reference(m, n, k):
    from lastkv_b200 import ops

    x, w = _case(m, n, k, m * 1000 + n + k)
    y = ops.decode_gemm(x, w)
    _check_plain(y, x, w)
    lin = torch.nn.functional.linear(x, w)
    diff = (y.float() - lin.float()).abs()
    print(f"m={m} n={n} k={k}: {(diff > 0).float().mean().item():.3%} differ from torch bf16 linear")


@pytest.mark.parametrize("m,f,k", [(8, 14336, 4096), (1, 64, 64), (5, 100, 72), (16, 1536, 1024)])
def test_silu_mul_epilogue(m, f, k):
    from lastkv_b200 import ops

    x, w = _case(m, 2 * f, k, 7 * m + f + k)
    y = ops.decode_gemm(x, w, silu_mul=True)
    gu = ops.decode_gemm(x, w)  # the same accumulations, plain epilogue
    ref = torch.nn.functional.silu(gu[:, :f]) * gu[:, f:]
    torch.testing.assert_close(y, ref, rtol=0, atol=0)
    _check_plain(gu, x, w)


def test_deterministic_and_graph_capturable():
    from lastkv_b200 import ops

    x, w = _case(8, 4096, 14336, 3)  # split-K shape
    a = ops.decode_gemm(x, w)
    b = ops.decode_gemm(x, w)
    torch.testing.assert_close(a, b, rtol=0, atol=0)
    out = torch.empty_like(a)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.decode_gemm(x, w, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.decode_gemm(x, w, out=out)
    x.copy_(torch.randn_like(x.float()).bfloat16())
    g.replay()
    torch.testing.assert_close(out, ops.decode_gemm(x, w), rtol=0, atol=0)


def test_strided_rows_and_rejects():
    from lastkv_b200 import ops
    from lastkv_b200.contract import RMarinBackendContractError

    x, w = _case(4, 256, 512, 11)
    big = torch.zeros((4, 1024), device="cuda", dtype=torch.bfloat16)
    big[:, :512] = x
    y = ops.decode_gemm(big[:, :512], w)  # row stride 1024
    torch.testing.assert_close(y, ops.decode_gemm(x, w), rtol=0, atol=0)
    with pytest.raises(RMarinBackendContractError):
        ops.decode_gemm(torch.zeros((17, 512), device="cuda", dtype=torch.bfloat16), w)
    with pytest.raises(RMarinBackendContractError):
        ops.decode_gemm(x, w[:, :256])
