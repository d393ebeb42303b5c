"""The allocation-free decode entry point, checked against the workspace one.

``lkv_decode_paged_noalloc`` serves callers that cannot allocate device
memory (an engine whose KV-cache pool already owns nearly all of HBM, a C-FFI
host that only passes buffers it owns); its scratch is a static array inside
the library that every call shares.  Two calls in a row, with different
inputs, must each match ``lkv_decode_paged`` - which also proves the second
call does not see the first call's leftover scratch.  The file sorts last so a
stop-at-first-failure run has already run everything else, and it sets up its
own inputs so it also passes alone in a fresh process.
"""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O
from tests.gpu_helpers import assert_close_bf16, make_paged_case

pytestmark = pytest.mark.gpu


def _noalloc(lib, t, out, lse, scale, B, Hq, Hkv, D, err):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.lkv_decode_paged_noalloc(
        t["q"].data_ptr(), t["q"].stride(0), t["pool_k"].data_ptr(), t["pool_v"].data_ptr(), t["pool_k"].shape[0],
        t["bt"].data_ptr(), t["bt"].stride(0), t["seq_k"].data_ptr(), out.data_ptr(), out.stride(0), lse.data_ptr(),
        scale.data_ptr(), B, Hq, Hkv, D, t["bt"].shape[1], D ** -0.5, err.data_ptr(), stream)


def test_noalloc_decode_matches_workspace_decode_on_two_calls():
    from lastkv_b200 import _capi, ops

    lib = _capi.load()
    assert lib.lkv_check_device(torch.cuda.current_device()) == 0
    B, Hq, Hkv, D = 16, 32, 8, 128
    for seed, lens in ((31, [4096] * 8 + [17, 1, 999, 2048, 300, 3000, 16, 4000]), (32, [5] * 16)):
        t, n = make_paged_case(seed, B, Hq, Hkv, D, lens)
        scale_h = np.random.default_rng(seed).uniform(0.5, 1.5, Hq).astype(np.float32)
        scale = torch.from_numpy(scale_h).cuda()
        ref_lse = torch.empty((B, Hq), dtype=torch.float32, device="cuda")
        ref = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], lse=ref_lse, out_scale=scale)
        out = torch.full((B, Hq, D), float("nan"), dtype=torch.bfloat16, device="cuda")
        lse = torch.full((B, Hq), float("nan"), dtype=torch.float32, device="cuda")
        err = torch.full((4,), -1, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        assert _noalloc(lib, t, out, lse, scale, B, Hq, Hkv, D, err) == 0
        torch.cuda.synchronize()
        # lkv_check_device above already loaded the static scratch: the call takes no device memory
        assert torch.cuda.mem_get_info()[0] == free_before
        assert_close_bf16(out.float().cpu().numpy(), ref.float().cpu().numpy(), what=f"noalloc seed {seed}")
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), rtol=1e-5, atol=1e-5)
        assert err.cpu().tolist() == [0, 0, 0, 0]
        # and against the float64 oracle directly, at the bf16 tolerance of every decode test
        want, want_lse = O.paged_attention(n["q"], n["pool_k"], n["pool_v"], n["bt"], n["seq_k"], n["cu"],
                                           scale=D ** -0.5, out_scale=scale_h)
        assert_close_bf16(out.float().cpu().numpy(), want, what=f"noalloc vs oracle seed {seed}")
        np.testing.assert_allclose(lse.cpu().numpy(), want_lse, rtol=1e-4, atol=1e-3)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from lastkv_b200 import _capi

    lib = _capi.load()
    t, _ = make_paged_case(40, 1, 8, 8, 128, [16])
    out = torch.zeros((1, 8, 128), dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros((1, 8), dtype=torch.float32, device="cuda")
    scale = torch.ones(8, dtype=torch.float32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    # batch * heads * (D + 1) * 4 beyond 8 MiB: rejected before any launch
    st = _noalloc(lib, t, out, lse, scale, 5000, 8, 8, 128, err)
    assert st == 6 and lib.lkv_status_string(st).startswith(b"workspace")
