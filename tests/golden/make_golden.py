"""Generate golden vectors from the reference's own HF implementation.

Run in a container that has the reference tree (not needed on the GPU box):

    python tests/golden/make_golden.py --reference <path to LastKV checkout>

It imports ``lastkv.llm`` from ``<reference>/llm/src``, builds two seeded
random-init models and records every attention call of the cached chunk
recurrence (``LastKVAttention.forward``, llm/src/lastkv/llm/modeling.py:98-148):
the pre-RoPE projections, cos/sin, the post-RoPE/RMSNorm query and new K/V
handed to SDPA, and SDPA's output; plus end-to-end logits and greedy tokens.

* ``tiny_ref.npz`` - the reference test suite's own tiny model
  (llm/tests/test_llm_inference.py:18-36, seed 19, head_dim 8, chunk 4).
* ``small_d128.npz`` - the same architecture at head_dim 128, GQA 4:1,
  chunk 16 (one ring = 2 pages of 16), batch 2, so the CUDA kernels can run
  on the identical calls.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np


def build(reference: str):
    sys.path.insert(0, os.path.join(reference, "llm", "src"))
    import torch
    from lastkv.llm import CustomRecurrentMarinAKV254ReuseKVConfig as Config
    from lastkv.llm import CustomRecurrentMarinAKV254ReuseKVForCausalLM as Model

    return torch, Config, Model


def tiny_model(torch, Config, Model):
    # Same construction as llm/tests/test_llm_inference.py:18-36.
    torch.manual_seed(19)
    config = Config(
        hidden_size=32, intermediate_size=48, num_attention_heads=4,
        num_key_value_heads=2, num_hidden_layers=3, head_dim=8,
        vocab_size=71, chunk_size=4, max_position_embeddings=64,
        bos_token_id=1, eos_token_id=None, pad_token_id=0,
        deep_v_scale_init=[[0.3, 0.7], [0.8, 1.2], [1.1, 0.9]],
        rope_theta=500000.0, attn_implementation="sdpa",
    )
    model = Model(config).eval()
    with torch.no_grad():
        for i, layer in enumerate(model.model.layers):
            layer.self_attn.prev_chunk_alphas.copy_(torch.tensor([-1.2 + i * 0.2, 0.8 - i * 0.3]))
            layer.self_attn.q_norm.weight.copy_(torch.linspace(0.7, 1.3, config.head_dim))
            layer.self_attn.k_norm.weight.copy_(torch.linspace(1.2, 0.8, config.head_dim))
    return model


def small_model(torch, Config, Model):
    torch.manual_seed(7)
    config = Config(
        hidden_size=64, intermediate_size=96, num_attention_heads=4,
        num_key_value_heads=1, num_hidden_layers=2, head_dim=128,
        vocab_size=97, chunk_size=16, max_position_embeddings=256,
        bos_token_id=1, eos_token_id=None, pad_token_id=0,
        deep_v_scale_init=[[0.6], [1.3]], rope_theta=500000.0,
        attn_implementation="sdpa", initializer_range=0.08,
    )
    model = Model(config).eval()
    with torch.no_grad():
        for i, layer in enumerate(model.model.layers):
            layer.self_attn.prev_chunk_alphas.copy_(torch.tensor([0.9 - 1.7 * i]))
            layer.self_attn.q_norm.weight.copy_(torch.linspace(0.6, 1.4, config.head_dim))
            layer.self_attn.k_norm.weight.copy_(torch.linspace(1.3, 0.7, config.head_dim))
    return model


class Recorder:
    """Record every SDPA call of LastKVAttention with its pre-RoPE inputs."""

    def __init__(self, torch, model, keep_full: bool):
        self.torch = torch
        self.model = model
        self.keep_full = keep_full
        self.calls = []
        self.pending = {}
        self.handles = []
        for index, layer in enumerate(model.model.layers):
            attn = layer.self_attn
            self.handles.append(attn.register_forward_pre_hook(self._pre(index)))
            for name in ("q_proj", "k_proj", "v_proj"):
                self.handles.append(getattr(attn, name).register_forward_hook(self._proj(name)))
        import torch.nn.functional as F

        self.F = F
        self.orig = F.scaled_dot_product_attention
        F.scaled_dot_product_attention = self._sdpa

    def _pre(self, index):
        def hook(module, args):
            hidden, (cos, sin), cache = args
            self.pending = {"layer": index, "start": cache.seen_tokens,
                            "cos": cos.detach().clone(), "sin": sin.detach().clone()}
        return hook

    def _proj(self, name):
        def hook(module, args, output):
            self.pending[name] = output.detach().clone()
        return hook

    def _sdpa(self, query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, enable_gqa=False):
        out = self.orig(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                        is_causal=is_causal, scale=scale, enable_gqa=enable_gqa)
        lq = query.shape[2]
        rec = dict(self.pending)
        rec.update(q=query.detach().clone(), k_new=key[:, :, -lq:].detach().clone(),
                   v_new=value[:, :, -lq:].detach().clone(), out=out.detach().clone(),
                   key_len=key.shape[2])
        if self.keep_full:
            rec.update(full_k=key.detach().clone(), full_v=value.detach().clone())
        self.calls.append(rec)
        return out

    def close(self):
        self.F.scaled_dot_product_attention = self.orig
        for h in self.handles:
            h.remove()


def params(model):
    cfg = model.config
    layers = model.model.layers
    return {
        "alpha_logits": np.stack([l.self_attn.prev_chunk_alphas.detach().numpy() for l in layers]).astype(np.float32),
        "v_scale": np.stack([l.self_attn.deep_v_scale.detach().numpy() for l in layers]).astype(np.float32),
        "q_norm_w": np.stack([l.self_attn.q_norm.weight.detach().numpy() for l in layers]).astype(np.float32),
        "k_norm_w": np.stack([l.self_attn.k_norm.weight.detach().numpy() for l in layers]).astype(np.float32),
        "eps": np.float32(cfg.rms_norm_eps),
        "chunk": np.int64(cfg.chunk_size),
        "num_heads": np.int64(cfg.num_attention_heads),
        "num_kv_heads": np.int64(cfg.num_key_value_heads),
        "head_dim": np.int64(cfg.head_dim),
        "num_layers": np.int64(cfg.num_hidden_layers),
        "rope_theta": np.float64(cfg.rope_theta if hasattr(cfg, "rope_theta") else cfg.rope_parameters["rope_theta"]),
    }


def flatten_calls(calls, prefix, keep_full):
    out = {}
    out[f"{prefix}n"] = np.int64(len(calls))
    for i, c in enumerate(calls):
        p = f"{prefix}{i}_"
        out[p + "meta"] = np.array([c["layer"], c["start"], c["q"].shape[2], c["key_len"]], dtype=np.int64)
        for name in ("q_proj", "k_proj", "v_proj", "cos", "sin", "q", "k_new", "v_new", "out"):
            out[p + name] = c[name].numpy().astype(np.float32)
        if keep_full:
            out[p + "full_k"] = c["full_k"].numpy().astype(np.float32)
            out[p + "full_v"] = c["full_v"].numpy().astype(np.float32)
    return out


def record_run(torch, model, tokens, segments, keep_full):
    """Run the cached path over ``segments``; return calls and per-segment logits."""
    rec = Recorder(torch, model, keep_full)
    logits = []
    cache, start = None, 0
    try:
        with torch.inference_mode():
            for size in segments:
                res = model(tokens[:, start:start + size], past_key_values=cache, use_cache=True)
                logits.append(res.logits)
                cache = res.past_key_values
                start += size
    finally:
        rec.close()
    return rec.calls, torch.cat(logits, dim=1).numpy().astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.dirname(os.path.abspath(__file__)))
    ap.add_argument("--only", choices=["planner"], default=None,
                    help="regenerate the planner fixtures only (they need neither torch nor a model)")
    args = ap.parse_args()
    if args.only == "planner":
        access_plan_golden(args.reference, args.out)
        history_golden(args.reference, args.out)
        return
    torch, Config, Model = build(args.reference)
    torch.set_num_threads(1)

    # --- tiny: the reference test's own model ------------------------------
    model = tiny_model(torch, Config, Model)
    g = torch.Generator().manual_seed(123)
    tokens = torch.randint(3, 71, (2, 15), generator=g)
    segments = [3, 2, 7, 3]
    calls, logits = record_run(torch, model, tokens, segments, keep_full=True)
    with torch.inference_mode():
        full = model(tokens, use_cache=False).logits.numpy().astype(np.float32)
        gen = model.generate(torch.tensor([[1, 5, 17]]), max_new_tokens=10, do_sample=False, use_cache=True)
    data = {"tokens": tokens.numpy(), "segments": np.array(segments), "logits_incremental": logits,
            "logits_full": full, "generate_prompt": np.array([[1, 5, 17]]), "generate_out": gen.numpy()}
    data.update(params(model))
    data.update(flatten_calls(calls, "call", keep_full=True))
    np.savez_compressed(os.path.join(args.out, "tiny_ref.npz"), **data)
    print("tiny_ref:", len(calls), "calls")

    # --- small_d128: head_dim 128, GQA 4:1, batch 2 -------------------------
    model = small_model(torch, Config, Model)
    g = torch.Generator().manual_seed(321)
    tokens = torch.randint(3, 97, (2, 64), generator=g)
    segments = [37] + [1] * 27  # chunked prefill across two boundaries, then decode
    calls, logits = record_run(torch, model, tokens, segments, keep_full=False)
    state = {f"w_{k}": v.detach().numpy().astype(np.float32) for k, v in model.state_dict().items()}
    with torch.inference_mode():
        gen = model.generate(tokens[:1, :20], max_new_tokens=24, do_sample=False, use_cache=True)
        # the logits that chose each generated token (teacher-forced replay of the output)
        gen_logits = model(gen[:, :-1], use_cache=False).logits[:, 19:].float().numpy()
    data = {"tokens": tokens.numpy(), "segments": np.array(segments), "logits_incremental": logits,
            "generate_prompt": tokens[:1, :20].numpy(), "generate_out": gen.numpy(),
            "generate_logits": gen_logits,
            "hidden_size": np.int64(model.config.hidden_size),
            "intermediate_size": np.int64(model.config.intermediate_size),
            "vocab_size": np.int64(model.config.vocab_size)}
    data.update(params(model))
    data.update(state)
    data.update(flatten_calls(calls, "call", keep_full=False))
    np.savez_compressed(os.path.join(args.out, "small_d128.npz"), **data)
    print("small_d128:", len(calls), "calls")

    # --- config1: the 124M architecture, 512-token prompt + 128 greedy steps --
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from seeded_weights import CONFIG1, nontrivial_alpha, nontrivial_scale, seeded_state

    torch.set_num_threads(os.cpu_count() or 1)
    prompt = torch.randint(0, CONFIG1["vocab_size"], (1, 512), generator=torch.Generator().manual_seed(0))
    out = {"prompt": prompt.numpy()}
    for tag, chunk, nontrivial in (("c4096", 4096, False), ("c128", 128, True)):
        config = Config(**CONFIG1, chunk_size=chunk, max_position_embeddings=4096, bos_token_id=1,
                        eos_token_id=None, pad_token_id=0, attn_implementation="sdpa")
        with torch.device("meta"):
            shapes = {k: tuple(v.shape) for k, v in Model(config).state_dict().items()}
        state = seeded_state(shapes, seed=1, alpha_fn=nontrivial_alpha if nontrivial else None,
                             scale_fn=nontrivial_scale if nontrivial else None)
        model = Model(config).eval()
        missing, unexpected = model.load_state_dict({k: torch.from_numpy(v) for k, v in state.items()}, strict=True)
        with torch.inference_mode():
            gen = model.generate(prompt, max_new_tokens=128, do_sample=False, use_cache=True)
            logits = model(gen[:, :-1], use_cache=False).logits[0, 511:].float()
        top_v, top_i = logits.topk(8, dim=-1)
        out[f"{tag}_tokens"] = gen.numpy()
        out[f"{tag}_top_v"] = top_v.numpy()
        out[f"{tag}_top_i"] = top_i.numpy()
        print(f"config1 {tag}: first tokens {gen[0, 512:520].tolist()}")
    np.savez_compressed(os.path.join(args.out, "config1_124m.npz"), **out)

    wan_golden(args.reference, args.out, torch)
    access_plan_golden(args.reference, args.out)
    history_golden(args.reference, args.out)


def _planner_modules(reference):
    """access_plan.py and reference.py of the reference's vLLM backend, loaded as a
    package of their own (the backend package's __init__ imports vLLM; these two
    modules need neither vLLM nor torch)."""
    import importlib.util
    import types

    pkg_dir = os.path.join(reference, "vllm", "src", "lastkv", "vllm", "backends", "rmarin_flashinfer")
    pkg = types.ModuleType("rmarin_planner")
    pkg.__path__ = [pkg_dir]
    sys.modules["rmarin_planner"] = pkg
    mods = []
    for name in ("access_plan", "reference"):
        spec = importlib.util.spec_from_file_location(f"rmarin_planner.{name}", os.path.join(pkg_dir, name + ".py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod  # its dataclasses resolve the module by name
        spec.loader.exec_module(mod)
        mods.append(mod)
    return mods


def history_golden(reference, out_dir):
    """The reference's executable history oracle (reference.py:342-439,
    resolve_reference_history with SourceScale mode "v") on seeded float values:
    for each (chunk, query position, layer kind) the raw top-layer source K/V, the
    layer's own K/V of recent + current, the per-head alpha logits and value scales,
    and the effective history [older: scaled source | recent: blend | current: local]
    it resolves, in float64.  Written to reference_history.npz."""
    ap, ref = _planner_modules(reference)
    rng = np.random.default_rng(2024)
    hkv, d = 2, 8
    out = {}
    cases = [(4, p) for p in (0, 3, 4, 6, 7, 9, 13)] + [(8, p) for p in (5, 8, 17, 23, 31)] + [(16, 40)]
    for i, (chunk, pos) in enumerate(cases):
        top = i % 2
        cur = (pos // chunk) * chunk
        rec = max(0, cur - chunk)
        src_end = pos + 1 if top else cur  # the top layer also holds its own raw current tokens
        raw_k = rng.standard_normal((src_end, hkv, d)).astype(np.float32).astype(np.float64)
        raw_v = rng.standard_normal((src_end, hkv, d)).astype(np.float32).astype(np.float64)
        loc_k = rng.standard_normal((pos + 1 - rec, hkv, d)).astype(np.float32).astype(np.float64)
        loc_v = rng.standard_normal((pos + 1 - rec, hkv, d)).astype(np.float32).astype(np.float64)
        logits = rng.standard_normal(hkv).astype(np.float32).astype(np.float64)
        scales = rng.uniform(0.3, 1.7, hkv).astype(np.float32).astype(np.float64)
        state = ap.RMarinRequestState.for_query(request_id="r", query_position=pos, chunk_size=chunk,
                                                source_initialized_end=src_end)
        plan = ap.plan_rmarin_access(state, ap.RMarinLayerSpec(layer_index=1 if top else 0, num_layers=2,
                                                              source_layer_index=1))

        def tok(k, v):
            return ref.ReferenceKVToken(key=tuple(map(tuple, k)), value=tuple(map(tuple, v)))

        raw = ref.IndexedReferenceCache.from_mapping(
            request_id="r", entries={t: tok(raw_k[t], raw_v[t]) for t in range(src_end)})
        local = ref.IndexedReferenceCache.from_mapping(
            request_id="r", entries={rec + t: tok(loc_k[t], loc_v[t]) for t in range(pos + 1 - rec)})
        hist = ref.resolve_reference_history(plan, raw_source=raw, same_layer_local=local,
                                             alpha_logits=tuple(logits.tolist()),
                                             source_scale=ref.SourceScale(mode="v", value_scales=tuple(scales)))
        eff_k = np.array([t.effective.key for t in hist.tokens])
        eff_v = np.array([t.effective.value for t in hist.tokens])
        for name, val in (("meta", np.array([chunk, pos, top], np.int64)), ("raw_k", raw_k), ("raw_v", raw_v),
                          ("loc_k", loc_k), ("loc_v", loc_v), ("logits", logits), ("scales", scales),
                          ("eff_k", eff_k), ("eff_v", eff_v)):
            out[f"c{i}_{name}"] = val
    out["n"] = np.int64(len(cases))
    np.savez_compressed(os.path.join(out_dir, "reference_history.npz"), **out)
    print("reference_history:", len(cases), "cases")


def access_plan_golden(reference, out_dir):
    """The reference's dependency-free access planner
    (vllm/src/lastkv/vllm/backends/rmarin_flashinfer/access_plan.py:407-474) over a grid
    of chunk sizes and query positions: each query's older / recent / current token
    ranges and whether a source pass (and so an LSE merge) exists, for the top layer
    and a lower one.  Written to access_plan.npz, rows
    [chunk, position, top, older.start, older.end, recent.start, recent.end,
     current.start, current.end, requires_lse_merge]."""
    ap, _ = _planner_modules(reference)
    rows = []
    for chunk in (4, 16, 32, 64, 1024, 4096):
        if chunk <= 64:
            positions = range(0, 3 * chunk + 3)
        else:
            positions = sorted({0, 1, chunk - 1, chunk, chunk + 1, 2 * chunk - 1, 2 * chunk, 2 * chunk + 1,
                                5 * chunk + 7, 8191, 8192, 8200, 131071})
        for p in positions:
            for top in (0, 1):
                state = ap.RMarinRequestState.for_query(request_id="r", query_position=p, chunk_size=chunk)
                layer = ap.RMarinLayerSpec(layer_index=1 if top else 0, num_layers=2, source_layer_index=1)
                plan = ap.plan_rmarin_access(state, layer)
                rows.append([chunk, p, top, plan.older.start, plan.older.end, plan.recent.start, plan.recent.end,
                             plan.current.start, plan.current.end, int(plan.requires_lse_merge)])
    np.savez_compressed(os.path.join(out_dir, "access_plan.npz"), rows=np.array(rows, dtype=np.int64))
    print("access_plan:", len(rows), "rows")


def _diffusers_stub() -> str:
    """A temporary package exposing the three diffusers names videogen/model.py imports."""
    import tempfile

    root = tempfile.mkdtemp(prefix="diffusers_stub_")
    pkg = os.path.join(root, "diffusers")
    os.makedirs(os.path.join(pkg, "models"))
    open(os.path.join(pkg, "__init__.py"), "w").close()
    open(os.path.join(pkg, "models", "__init__.py"), "w").close()
    with open(os.path.join(pkg, "configuration_utils.py"), "w") as f:
        f.write("class ConfigMixin:\n    pass\n\n\ndef register_to_config(fn):\n    return fn\n")
    with open(os.path.join(pkg, "models", "modeling_utils.py"), "w") as f:
        f.write("import torch\n\n\nclass ModelMixin(torch.nn.Module):\n    pass\n")
    return root


def wan_golden(reference, out_dir, torch):
    """Record the reference Wan block attention (videogen/src/lastkv/videogen/model.py:217-390)
    over six 3-frame blocks of a tiny model: 2 heads x 128, 8 tokens per frame (2 x 4 grid),
    one-frame local prefix; none of the segment boundaries is a multiple of 16."""
    sys.path.insert(0, _diffusers_stub())
    sys.path.insert(0, os.path.join(reference, "videogen", "src"))
    from lastkv.videogen import model as wm
    from lastkv.videogen.cache import allocate_caches

    torch.manual_seed(123)
    cfg = dict(model_type="t2v", patch_size=(1, 2, 2), dim=256, ffn_dim=64, num_heads=2, num_layers=3, text_dim=8,
               text_len=5, freq_dim=16, in_dim=2, out_dim=2, qk_norm=True, cross_attn_norm=True,
               akv_mode="reusekv", v_gap=95, num_frame_per_block=3, force_first_local_kv_tokens=8, eps=1e-6)
    model = wm.AKV2541ReuseKVCausalWanModel(**cfg).eval()
    with torch.no_grad():
        model.prev_block_alphas.normal_()
        for blk in model.blocks:
            blk.self_attn.norm_q.weight.copy_(torch.linspace(0.6, 1.4, 256))
            blk.self_attn.norm_k.weight.copy_(torch.linspace(1.3, 0.7, 256))
    fh, fw, fpb, blocks = 2, 4, 3, 6
    frame_tok = fh * fw
    block_tok = frame_tok * fpb
    caches = allocate_caches(model, 1, block_tok * blocks, block_tok, torch.float32, "cpu", shared=True)
    model._ensure_current_history_caches(caches)
    grid = torch.tensor([[fpb, fh, fw]])
    rec, calls = {}, []
    orig_attention = wm.attention

    def capture(q, k, v, *a, **kw):
        out = orig_attention(q, k, v, *a, **kw)
        rec.update(roped_q=q.detach().clone(), full_k=k.detach().clone(), full_v=v.detach().clone(),
                   out=out.detach().clone())
        return out

    wm.attention = capture
    try:
        hooks = []
        for blk in model.blocks:
            at = blk.self_attn
            hooks.append(at.norm_q.register_forward_hook(lambda m, a, o: rec.__setitem__("qn", o.detach().clone())))
            hooks.append(at.norm_k.register_forward_hook(lambda m, a, o: rec.__setitem__("kn", o.detach().clone())))
            hooks.append(at.v.register_forward_hook(lambda m, a, o: rec.__setitem__("v", o.detach().clone())))
        g = torch.Generator().manual_seed(9)
        with torch.no_grad():
            for n in range(blocks):
                start = n * block_tok
                kvs = []
                for layer, blk in enumerate(model.blocks):
                    model._set_prev_block_alpha(caches[layer], layer, torch.float32, "cpu")
                    x = torch.randn(1, block_tok, 256, generator=g)
                    _, kv = blk.self_attn(x, grid, model.freqs, kv_cache=caches[layer], current_start=start,
                                          num_frame_per_block=fpb, return_current_kv=True)
                    kvs.append(kv)
                    calls.append(dict(layer=layer, start=start, **{k: v.numpy() for k, v in rec.items()}))
                model._update_caches_akv(caches, kvs, None, grid, start_frame=start // frame_tok,
                                         current_start=start)
        for h in hooks:
            h.remove()
    finally:
        wm.attention = orig_attention
    data = {"calln": np.int64(len(calls)), "num_heads": np.int64(2), "head_dim": np.int64(128),
            "frame_h": np.int64(fh), "frame_w": np.int64(fw), "frames_per_block": np.int64(fpb),
            "prefix_tokens": np.int64(8), "num_layers": np.int64(3),
            "prev_block_alphas": model.prev_block_alphas.detach().numpy().astype(np.float32)}
    for i, c in enumerate(calls):
        p = f"call{i}_"
        data[p + "meta"] = np.array([c["layer"], c["start"], block_tok, c["full_k"].shape[1]], dtype=np.int64)
        for k in ("qn", "kn", "v", "roped_q", "out"):
            data[p + k] = c[k].astype(np.float32)
    np.savez_compressed(os.path.join(out_dir, "wan_block_attn.npz"), **data)
    print("wan:", len(calls), "calls; key lengths", sorted({int(c["full_k"].shape[1]) for c in calls}))


if __name__ == "__main__":
    main()
