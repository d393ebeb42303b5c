"""The context-parallel combine on one GPU: world = 1 equals the merge kernel,
and a peer that never pushes makes the bounded wait expire into the error word
(the failure-detection path, exercised without any GPU fault: the "peer" is a
local buffer nobody writes, the kernel gives up after its ~2 s limit and the
context stays usable)."""

import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _partial(rows, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    o = torch.randn((rows, D), generator=g, device="cuda")
    lse = torch.randn(rows, generator=g, device="cuda") * 3
    return o, lse


def test_single_rank_equals_merge_kernel():
    from lastkv_b200 import ops

    B, Hq, D = 3, 8, 128
    rows = B * Hq
    sizes = ops.cp_combine_sizes(rows, D, 1)
    o, lse = _partial(rows, D, 1)
    send = torch.zeros(sizes["send_floats"], device="cuda")
    send[: rows * D] = o.flatten()
    send[rows * D: rows * (D + 1)] = lse
    recv = torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda")
    scale = torch.rand(Hq, device="cuda") + 0.5
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    got = ops.cp_combine(send, [recv.data_ptr()], 0, 1, state, rows, D, Hq, out_scale=scale, error_word=err)
    ref = ops.merge_partials(o.view(1, B, Hq, D), lse.view(1, B, Hq), out_scale=scale)
    torch.testing.assert_close(got.view(B, Hq, D), ref.view(B, Hq, D), rtol=0, atol=0)
    assert err.cpu().tolist() == [0, 0, 0, 0]
    assert state.cpu().tolist() == [1, 0]  # epoch advanced once, done counter reset
    ops.cp_combine(send, [recv.data_ptr()], 0, 1, state, rows, D, Hq, out_scale=scale, error_word=err)
    assert state.cpu().tolist() == [2, 0]


def test_missing_peer_times_out_into_error_word():
    from lastkv_b200 import ops

    B, Hq, D = 1, 4, 64
    rows = B * Hq
    sizes = ops.cp_combine_sizes(rows, D, 2)
    o, lse = _partial(rows, D, 2)
    send = torch.zeros(sizes["send_floats"], device="cuda")
    send[: rows * D] = o.flatten()
    send[rows * D: rows * (D + 1)] = lse
    mine = torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda")
    peer = torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda")  # rank 1 never runs
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    t0 = time.time()
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    ops.cp_combine(send, [mine.data_ptr(), peer.data_ptr()], 0, 2, state, rows, D, Hq, error_word=err)
    torch.cuda.synchronize()
    waited = time.time() - t0
    e = err.cpu().tolist()
    assert e[0] == 1 and e[1] == 8, e  # wait timeout, reported by the combine kernel
    assert 1.0 < waited < 30.0, waited
    # this rank's push reached the "peer" buffer: {value, epoch = 1} words
    words = peer.view(2, 2, -1)[1, 0, : rows * D].cpu().numpy().astype(np.uint64)
    assert np.all((words >> np.uint64(32)) == 1)
    vals = (words & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
    np.testing.assert_array_equal(vals, o.flatten().cpu().numpy())
    # the context is still usable
    assert float(torch.ones(4, device="cuda").sum()) == 4.0


def test_fused_decode_push_equals_partial_merge_path():
    """lkv_decode_paged_cp on one rank (the decode kernel merges each unit's splits and
    pushes the rows into the receive buffer; the combine only polls and merges) equals
    decode partial + merge of the packed parts bit for bit, over several calls (epochs)."""
    from lastkv_b200 import ops
    from tests.gpu_helpers import make_paged_case

    B, Hq, Hkv, D = 4, 32, 8, 128
    t, _ = make_paged_case(31, B, Hq, Hkv, D, [3000, 17, 900, 2048])
    scale = torch.rand(Hq, device="cuda") + 0.5
    rows = B * Hq
    sizes = ops.cp_combine_sizes(rows, D, 1)
    recv = torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda")
    state = torch.zeros(ops.decode_cp_state_words(B, Hkv), dtype=torch.int32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws = ops.Workspace.for_decode(B, Hq, D, t["bt"].shape[1], device="cuda")
    po, pl = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], partial=True)
    ref = ops.merge_partials(po.view(1, B, Hq, D), pl.view(1, B, Hq), out_scale=scale)
    for call in range(3):
        got = ops.decode_paged_cp(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], [recv.data_ptr()], 0, 1,
                                  state, out_scale=scale, workspace=ws, error_word=err)
        torch.cuda.synchronize()
        assert err.cpu().tolist() == [0, 0, 0, 0]
        torch.testing.assert_close(got.view(B, Hq, D), ref.view(B, Hq, D), rtol=0, atol=0)
        st = state.cpu().tolist()
        assert st[0] == call + 1 and st[1] == 0 and all(v == 0 for v in st[2:]), st  # arrivals reset


def test_fused_exchange_missing_peer_times_out_into_error_word():
    """lkv_decode_paged_cp with the exchange fused into the decode kernel (no combine launch):
    a second "rank" whose receive buffer nobody fills makes every unit's bounded poll give
    up (~2 s) into the error word, and the context stays usable."""
    from lastkv_b200 import ops
    from tests.gpu_helpers import make_paged_case

    B, Hq, Hkv, D = 2, 8, 2, 128
    t, _ = make_paged_case(41, B, Hq, Hkv, D, [500, 70])
    rows = B * Hq
    sizes = ops.cp_combine_sizes(rows, D, 2)
    mine = torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda")
    peer = torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda")  # rank 1 never runs
    state = torch.zeros(ops.decode_cp_state_words(B, Hkv), dtype=torch.int32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws = ops.Workspace.for_decode(B, Hq, D, t["bt"].shape[1], device="cuda")
    t0 = time.time()
    ops.decode_paged_cp(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], [mine.data_ptr(), peer.data_ptr()],
                        0, 2, state, workspace=ws, error_word=err)
    torch.cuda.synchronize()
    waited = time.time() - t0
    e = err.cpu().tolist()
    assert e[0] == 1 and e[1] == 1 and e[3] >= 2000000, e  # wait timeout, reported by the decode kernel
    assert 1.0 < waited < 30.0, waited
    # this rank's rows reached the "peer" buffer with epoch 1
    words = peer.view(2, 2, -1)[1, 0, : rows * D].cpu().numpy().astype(np.uint64)
    assert np.all((words >> np.uint64(32)) == 1)
    assert float(torch.ones(4, device="cuda").sum()) == 4.0


def _prefill_peer_words(recv, world, rows, D, epoch, parts):
    """Write rank r's partial (o [rows, D], natural-log lse [rows]) into receive slot
    [epoch & 1][r] as {value, epoch} words, as rank r's push would (peers 1..world-1)."""
    part_words = (rows * (D + 1) + 1) // 2 * 2
    slots = recv.view(2, world, -1)[:, :, :part_words]
    for r, (o, lse) in parts.items():
        vals = torch.cat([o.flatten(), lse.flatten()]).contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        slots[epoch & 1, r, : rows * (D + 1)] = vals | (epoch << 32)


@pytest.mark.parametrize("world", [3, 8])
def test_eight_rank_merge_from_arrived_words(world):
    """The rank-order merge with more ranks than one batch of requested words (8 ranks:
    two batches of four): every peer's words are already in this rank's receive buffer
    (written here as their pushes would), so nothing waits on another kernel; the
    combine equals merge_partials over the same parts bit for bit."""
    from lastkv_b200 import ops

    B, Hq, D = 2, 8, 128
    rows = B * Hq
    sizes = ops.cp_combine_sizes(rows, D, world)
    parts = {r: _partial(rows, D, 40 + r) for r in range(world)}
    send = torch.zeros(sizes["send_floats"], device="cuda")
    send[: rows * D] = parts[0][0].flatten()
    send[rows * D: rows * (D + 1)] = parts[0][1]
    mine = torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda")
    peers = [torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda") for _ in range(world - 1)]
    _prefill_peer_words(mine, world, rows, D, 1, {r: parts[r] for r in range(1, world)})
    scale = torch.rand(Hq, device="cuda") + 0.5
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    state = torch.zeros(2, dtype=torch.int32, device="cuda")
    got = ops.cp_combine(send, [mine.data_ptr()] + [p.data_ptr() for p in peers], 0, world, state, rows, D, Hq,
                         out_scale=scale, error_word=err)
    o_all = torch.stack([parts[r][0].view(B, Hq, D) for r in range(world)])
    l_all = torch.stack([parts[r][1].view(B, Hq) for r in range(world)])
    ref = ops.merge_partials(o_all, l_all, out_scale=scale)
    torch.cuda.synchronize()
    assert err.cpu().tolist() == [0, 0, 0, 0]
    torch.testing.assert_close(got.view(B, Hq, D), ref.view(B, Hq, D), rtol=0, atol=0)


def test_fused_decode_eight_ranks_from_arrived_words():
    """lkv_decode_paged_cp as rank 0 of 8 (the decode kernel's own unit merge, push to all
    eight buffers, then the poll-and-merge of two batches of four ranks): the seven peers'
    words are in place before the launch, so the kernel waits on nothing; the output
    equals this rank's partial decode merged with the peers' parts by merge_partials."""
    from lastkv_b200 import ops
    from tests.gpu_helpers import make_paged_case

    world = 8
    B, Hq, Hkv, D = 4, 32, 8, 128
    rows = B * Hq
    t, _ = make_paged_case(37, B, Hq, Hkv, D, [3000, 17, 900, 2048])
    scale = torch.rand(Hq, device="cuda") + 0.5
    sizes = ops.cp_combine_sizes(rows, D, world)
    mine = torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda")
    peers = [torch.zeros(sizes["recv_words"], dtype=torch.int64, device="cuda") for _ in range(world - 1)]
    parts = {r: _partial(rows, D, 70 + r) for r in range(1, world)}
    _prefill_peer_words(mine, world, rows, D, 1, parts)
    state = torch.zeros(ops.decode_cp_state_words(B, Hkv), dtype=torch.int32, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws = ops.Workspace.for_decode(B, Hq, D, t["bt"].shape[1], device="cuda")
    got = ops.decode_paged_cp(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"],
                              [mine.data_ptr()] + [p.data_ptr() for p in peers], 0, world, state,
                              out_scale=scale, workspace=ws, error_word=err)
    po, pl = ops.decode_paged(t["q"], t["pool_k"], t["pool_v"], t["bt"], t["seq_k"], partial=True)
    o_all = torch.stack([po] + [parts[r][0].view(B, Hq, D) for r in range(1, world)])
    l_all = torch.stack([pl] + [parts[r][1].view(B, Hq) for r in range(1, world)])
    ref = ops.merge_partials(o_all, l_all, out_scale=scale)
    torch.cuda.synchronize()
    assert err.cpu().tolist() == [0, 0, 0, 0] and ws.error()[0] == 0
    torch.testing.assert_close(got.view(B, Hq, D), ref.view(B, Hq, D), rtol=0, atol=0)
    # this rank's merged rows reached every peer's buffer with the call's epoch
    for p in peers:
        words = p.view(2, world, -1)[1, 0, : rows * D].cpu().numpy().astype(np.uint64)
        assert np.all((words >> np.uint64(32)) == 1)
