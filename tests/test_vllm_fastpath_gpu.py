"""Serving fast path (prepare + run_layer) on the B200 kernels.

1. The reference's recorded calls: pre-RoPE projections in, attention outputs
   compared with the reference's SDPA outputs (chunked prefill across two
   boundaries, then decode), batch 2.
2. A random multi-step schedule mixing prefill spans and decode steps at
   different positions per sequence, with boundary commits, checked step by
   step against the oracle's merged pool driven with the same inputs.
"""

import numpy as np
import pytest
import torch

from oracle import lastkv_oracle as O
from tests.conftest import golden_calls
from tests.gpu_helpers import assert_close_bf16

pytestmark = pytest.mark.gpu


def _fast(layers, slots, max_tokens, chunk, hkv, hq, d, order=None, max_tokens_step=256):
    from lastkv_b200.vllm_backend import SharedKVFastPath, SharedKVPool

    pool = SharedKVPool(num_layers=layers, num_slots=slots, max_sequence_tokens=max_tokens, chunk_size=chunk,
                        num_kv_heads=hkv, head_dim=d, device="cuda", page_order=order)
    return pool, SharedKVFastPath(pool, max_batch=8, max_tokens=max_tokens_step, num_q_heads=hq)


def test_run_layer_reproduces_reference_calls(small_d128):
    from lastkv_b200.vllm_backend import Span, rope_cos_sin_cache

    data = small_d128
    L, C = int(data["num_layers"]), int(data["chunk"])
    hq, hkv, d = int(data["num_heads"]), int(data["num_kv_heads"]), int(data["head_dim"])
    B, T = data["tokens"].shape
    order = np.random.default_rng(2).permutation(B * (-(-T // 16)))
    pool, fast = _fast(L, B, T, C, hkv, hq, d, order)
    pool.bind_parameters(torch.from_numpy(data["alpha_logits"]), torch.from_numpy(data["v_scale"]), hq)
    fast.register_layers([(torch.from_numpy(data["q_norm_w"][l]).cuda(), torch.from_numpy(data["k_norm_w"][l]).cuda())
                          for l in range(L)], rope_cos_sin_cache(T, d, float(data["rope_theta"])), float(data["eps"]))
    n_checked = 0
    for rec in golden_calls(data):
        layer, start, lq = rec["layer"], rec["start"], rec["lq"]
        if layer == 0:
            assert fast.prepare([Span(b, start, lq) for b in range(B)])
        q = torch.from_numpy(rec["q_proj"].reshape(B * lq, hq * d)).cuda().bfloat16()
        k = torch.from_numpy(rec["k_proj"].reshape(B * lq, hkv * d)).cuda().bfloat16()
        v = torch.from_numpy(rec["v_proj"].reshape(B * lq, hkv * d)).cuda().bfloat16()
        out = torch.empty((B * lq, hq, d), dtype=torch.bfloat16, device="cuda")
        fast.run_layer(layer, q, k, v, out)
        exp = rec["out"].transpose(0, 2, 1, 3).reshape(B * lq, hq, d)
        assert_close_bf16(out.float().cpu().numpy(), exp, what=f"layer {layer} @ {start} x {lq}")
        n_checked += 1
    fast.check_errors()
    assert n_checked == int(data["calln"])


def test_mixed_prefill_decode_schedule_matches_oracle():
    from lastkv_b200.vllm_backend import Span, chunk_aligned_new_tokens, rope_cos_sin_cache

    rng = np.random.default_rng(7)
    L, slots, C, hkv, hq, d = 3, 3, 32, 2, 8, 128
    max_tok = 160
    order = rng.permutation(slots * (max_tok // 16))
    pool, fast = _fast(L, slots, max_tok, C, hkv, hq, d, order)
    alpha_logits = rng.standard_normal((L, hkv)).astype(np.float32)
    v_scale = rng.uniform(0.4, 1.6, (L, hkv)).astype(np.float32)
    pool.bind_parameters(torch.from_numpy(alpha_logits), torch.from_numpy(v_scale), hq)
    fast.register_layers([(None, None)] * L, None, 1e-6)  # use_nope / no qk-norm: inputs are final q/k
    lay = O.PoolLayout(num_layers=L, chunk=C, page=16, num_slots=slots, src_pages=pool.src_pages)
    state = O.PagedLastKV(layout=lay, hkv=hkv, d=d, batch=slots, alpha=O.alpha_from_logits(alpha_logits),
                          v_scale=O.bf16_round(v_scale), bf16=True,
                          src_page_lists=[list(pool.src_table[s]) for s in range(slots)])
    # per-slot request lengths; each step schedules chunk-aligned spans (prefill) or one token (decode)
    target = [150, 70, 100]
    done = [0, 0, 0]
    prompt = [100, 40, 64]
    step = 0
    while any(done[s] < target[s] for s in range(slots)):
        spans = []
        for s in range(slots):
            if done[s] >= target[s]:
                continue
            want = prompt[s] - done[s] if done[s] < prompt[s] else 1
            n = chunk_aligned_new_tokens(done[s], min(want, int(rng.integers(1, 40))), C)
            spans.append(Span(s, done[s], n))
        # the oracle commits the previous boundary at the same point the fast path does
        for sp in spans:
            state.commit_if_boundary(sp.slot, sp.num_computed_tokens)
        fast.prepare(spans)
        T = sum(sp.num_query_tokens for sp in spans)
        for layer in range(L):
            q = O.bf16_round(rng.standard_normal((T, hq, d)))
            k = O.bf16_round(rng.standard_normal((T, hkv, d)))
            v = O.bf16_round(rng.standard_normal((T, hkv, d)))
            out = torch.empty((T, hq, d), dtype=torch.bfloat16, device="cuda")
            fast.run_layer(layer, torch.from_numpy(q).cuda().bfloat16(), torch.from_numpy(k).cuda().bfloat16(),
                           torch.from_numpy(v).cuda().bfloat16(), out)
            got = out.float().cpu().numpy()
            t = 0
            for sp in spans:
                n = sp.num_query_tokens
                state.append(layer, sp.slot, k[t:t + n], v[t:t + n], sp.num_computed_tokens)
                exp = state.attend(layer, sp.slot, q[t:t + n], sp.num_computed_tokens, scale=d ** -0.5)
                assert_close_bf16(got[t:t + n], exp, what=f"step {step} layer {layer} slot {sp.slot}")
                t += n
        for sp in spans:
            done[sp.slot] += sp.num_query_tokens
        step += 1
    fast.check_errors()
    assert step > 10


def test_merged_check_switch_reports_two_pass_agreement(small_d128, monkeypatch, capsys):
    """RMARIN_MERGED_CHECK=1 (the reference's diagnostic switch): every layer call is recomputed
    two-pass (ring pages causal + older shared pages non-causal + LSE merge) and the deviation of
    the merged single call is reported; on the recorded calls it stays at bf16 rounding."""
    from lastkv_b200.vllm_backend import Span, rope_cos_sin_cache

    monkeypatch.setenv("RMARIN_MERGED_CHECK", "1")
    data = small_d128
    L, C = int(data["num_layers"]), int(data["chunk"])
    hq, hkv, d = int(data["num_heads"]), int(data["num_kv_heads"]), int(data["head_dim"])
    B, T = data["tokens"].shape
    pool, fast = _fast(L, B, T, C, hkv, hq, d, np.random.default_rng(3).permutation(B * (-(-T // 16))))
    assert fast.check
    pool.bind_parameters(torch.from_numpy(data["alpha_logits"]), torch.from_numpy(data["v_scale"]), hq)
    fast.register_layers([(torch.from_numpy(data["q_norm_w"][l]).cuda(), torch.from_numpy(data["k_norm_w"][l]).cuda())
                          for l in range(L)], rope_cos_sin_cache(T, d, float(data["rope_theta"])), float(data["eps"]))
    for rec in golden_calls(data):
        layer, start, lq = rec["layer"], rec["start"], rec["lq"]
        if layer == 0:
            assert fast.prepare([Span(b, start, lq) for b in range(B)])
        q = torch.from_numpy(rec["q_proj"].reshape(B * lq, hq * d)).cuda().bfloat16()
        k = torch.from_numpy(rec["k_proj"].reshape(B * lq, hkv * d)).cuda().bfloat16()
        v = torch.from_numpy(rec["v_proj"].reshape(B * lq, hkv * d)).cuda().bfloat16()
        out = torch.empty((B * lq, hq, d), dtype=torch.bfloat16, device="cuda")
        fast.run_layer(layer, q, k, v, out)
    fast.check_errors()
    assert len(fast.check_log) == int(data["calln"])
    worst = max(r["rel"] for r in fast.check_log)
    assert worst < 0.02, fast.check_log
    assert "rmarin_merged_check" in capsys.readouterr().out


def test_plugin_backend_reproduces_reference_calls(small_d128):
    """The same recorded calls through the reference's backend surface: the lean metadata
    builder (vLLM's per-step build -> host prologue) and RMarinFlashInferImpl.forward
    (vLLM's per-layer call) of ``lastkv_b200.vllm_plugin``, with vLLM's modules faked at the
    pinned signatures and the real fast path and kernels underneath."""
    import types

    from lastkv_b200 import vllm_plugin
    from lastkv_b200.vllm_backend import rope_cos_sin_cache
    from tests.test_vllm_plugin_cpu import _fake_runtime, _metadata, _versions

    data = small_d128
    L, C = int(data["num_layers"]), int(data["chunk"])
    hq, hkv, d = int(data["num_heads"]), int(data["num_kv_heads"]), int(data["head_dim"])
    B, T = data["tokens"].shape
    pool, fast = _fast(L, B, T, C, hkv, hq, d, np.random.default_rng(3).permutation(B * (-(-T // 16))))
    pool.bind_parameters(torch.from_numpy(data["alpha_logits"]), torch.from_numpy(data["v_scale"]), hq)
    fast.register_layers([(torch.from_numpy(data["q_norm_w"][l]).cuda(), torch.from_numpy(data["k_norm_w"][l]).cuda())
                          for l in range(L)], rope_cos_sin_cache(T, d, float(data["rope_theta"])), float(data["eps"]))
    vllm_plugin._LEAN_BUILDER = None
    cfg = types.SimpleNamespace(model_config=types.SimpleNamespace(hf_config=types.SimpleNamespace(chunk_size=C)))
    importer, _ = _fake_runtime(config=cfg)
    backend, impl_cls = vllm_plugin.build_vllm_backend_types(importer=importer, version_getter=_versions())
    vllm_plugin.install_fast_path(fast)
    try:
        builder = backend.get_builder_cls()(None, [f"l{l}" for l in range(L)], cfg, "cuda")
        impl = impl_cls(hq, d, d ** -0.5, hkv, None, None, "auto", None, "decoder", None, None)
        md = None
        for rec in golden_calls(data):
            layer, start, lq = rec["layer"], rec["start"], rec["lq"]
            if layer == 0:
                md = builder.build(0, _metadata([lq] * B, [start + lq] * B))
            q = torch.from_numpy(rec["q_proj"].reshape(B * lq, hq * d)).cuda().bfloat16()
            k = torch.from_numpy(rec["k_proj"].reshape(B * lq, hkv * d)).cuda().bfloat16()
            v = torch.from_numpy(rec["v_proj"].reshape(B * lq, hkv * d)).cuda().bfloat16()
            out = torch.full((B * lq + 3, hq * d), float("nan"), dtype=torch.bfloat16, device="cuda")  # padded
            impl.forward(types.SimpleNamespace(rmarin_layer_index=layer), q, k, v, None, md, out)
            exp = rec["out"].transpose(0, 2, 1, 3).reshape(B * lq, hq, d)
            assert_close_bf16(out[: B * lq].view(-1, hq, d).float().cpu().numpy(), exp,
                              what=f"plugin layer {layer} @ {start} x {lq}")
            assert bool((out[B * lq:] == 0).all())
        fast.check_errors()
    finally:
        vllm_plugin.uninstall_fast_path()
        vllm_plugin._LEAN_BUILDER = None


def test_captured_decode_graph_carries_boundary_commits():
    """Uniform decode steps replayed from one CUDA graph (every layer's run_layer):
    the boundary commits of the rows that cross a chunk boundary ride in layer 0's
    append as a device-side row count, so the same graph serves steps with and
    without commits.  Outputs and pools are bit-identical to eager steps with a
    separate blend launch (fuse_commit = False)."""
    from lastkv_b200.vllm_backend import Span

    rng = np.random.default_rng(11)
    L, slots, C, hkv, hq, d = 3, 4, 32, 2, 8, 128
    max_tok = 128
    order = rng.permutation(slots * (max_tok // 16))
    alpha_logits = torch.from_numpy(rng.standard_normal((L, hkv)).astype(np.float32))
    v_scale = torch.from_numpy(rng.uniform(0.4, 1.6, (L, hkv)).astype(np.float32))
    prompt = [30, 31, 20, 45]  # rows cross the boundary at 32 (or 64) at different steps
    steps = 24
    inputs = []  # per call: q, k, v for every layer
    spans_of = []
    for phase in range(1 + steps):
        if phase == 0:
            spans = [Span(s, 0, prompt[s]) if prompt[s] <= C else None for s in range(slots)]
            spans = [sp for sp in spans if sp is not None] + [Span(3, 0, C)]
        else:
            spans = [Span(s, prompt[s] + phase - 1, 1) for s in range(slots)]
        spans_of.append(spans)
    spans_of.insert(1, [Span(3, C, prompt[3] - C)])  # the rest of row 3's prompt
    for spans in spans_of:
        T = sum(sp.num_query_tokens for sp in spans)
        inputs.append([(torch.from_numpy(O.bf16_round(rng.standard_normal((T, hq * d)))).cuda().bfloat16(),
                        torch.from_numpy(O.bf16_round(rng.standard_normal((T, hkv * d)))).cuda().bfloat16(),
                        torch.from_numpy(O.bf16_round(rng.standard_normal((T, hkv * d)))).cuda().bfloat16())
                       for _ in range(L)])

    def run(fuse, graph):
        pool, fast = _fast(L, slots, max_tok, C, hkv, hq, d, order)
        fast.fuse_commit = fuse
        pool.bind_parameters(alpha_logits, v_scale, hq)
        fast.register_layers([(None, None)] * L, None, 1e-6)
        outs = []
        static_in = [[torch.empty_like(t) for t in lay] for lay in inputs[-1]]
        static_out = [torch.empty((slots, hq, d), dtype=torch.bfloat16, device="cuda") for _ in range(L)]
        g = None
        for spans, xs in zip(spans_of, inputs):
            fast.prepare(spans)
            decode = all(sp.num_query_tokens == 1 for sp in spans)
            if graph and decode:
                for l in range(L):
                    for dst, src in zip(static_in[l], xs[l]):
                        dst.copy_(src)
                if g is None:  # captured on the first decode step, then replayed every step
                    g = torch.cuda.CUDAGraph()
                    s = torch.cuda.Stream()
                    s.wait_stream(torch.cuda.current_stream())
                    with torch.cuda.graph(g, stream=s):
                        for l in range(L):
                            fast.run_layer(l, *static_in[l], static_out[l])
                    torch.cuda.current_stream().wait_stream(s)
                g.replay()
                outs.append(torch.stack([o.clone() for o in static_out]))
            else:
                T = sum(sp.num_query_tokens for sp in spans)
                res = []
                for l in range(L):
                    out = torch.empty((T, hq, d), dtype=torch.bfloat16, device="cuda")
                    fast.run_layer(l, *xs[l], out)
                    res.append(out)
                outs.append(torch.stack(res))
        torch.cuda.synchronize()
        fast.check_errors()
        assert pool.committed == [32, 32, 32, 64]
        return [o.cpu() for o in outs], pool.pool_k.cpu(), pool.pool_v.cpu()

    want = run(False, False)
    got = run(True, True)
    for a, b in zip(want[0], got[0]):
        assert torch.equal(a, b)
    assert torch.equal(want[1], got[1]) and torch.equal(want[2], got[2])
