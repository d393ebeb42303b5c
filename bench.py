#!/usr/bin/env python
"""Shared-KV decode benchmark (the reference's config 2, in its merged paged form).

Workload ("shared_kv_decode_attention"): bf16, batch 64, 32 query heads,
8 KV heads, head_dim 128, 8192 keys per sequence in 16-token pages with a
shuffled page table; chunk 1024, so each layer's block table is the 384 shared
final-layer pages [0, 6144) followed by that layer's 128 ring pages
[6144, 8192).  One step = one decode token for all 64 sequences = 32 layer
calls, each reading the full 2 GiB of K/V once (larger than L2, so no flush is
needed between steps).  Q/K/V ~ N(0, 1) (K stands for post-RoPE keys), seeded.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  ``--impl reference`` times the reference's own
CPU computation of the same layer-step (compose the history with torch.cat and
call torch SDPA on the host cores, llm/src/lastkv/llm/modeling.py:109-146) via
the oracle's restatement; it never touches the GPU.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

CFG = dict(batch=64, q_heads=32, kv_heads=8, head_dim=128, context=8192, page=16, layers=32, chunk=1024)
# Small case for profiler captures only (268 MiB of K/V per call, still > L2); never a bench line.
SMALL = dict(batch=8, layers=2)
METRIC = "decode tokens/s (shared-KV attention, 32 layers)"
UNIT = "tokens/s"


def algo_bytes() -> int:
    """K and V bytes one layer call must read: 2 * B * Hkv * N * D * 2."""
    return 2 * CFG["batch"] * CFG["kv_heads"] * CFG["context"] * CFG["head_dim"] * 2


# DRAM read + write bytes of one decode_splitkv launch, from the small-case ncu capture
# (8 sequences, 2 layers; profiles/decode_splitkv_config2.txt): the mean of two launches,
# 268,590,080 read + 1,920,896 written (split partials leaving L2), scaled by the
# sequences a launch processes (x 8 for config 2's 64); the read bytes scale with the
# sequences, the writes only roughly.
NCU_SMALL_TRAFFIC = 268_590_080 + 1_920_896
NCU_SMALL_BATCH = 8


def traffic_per_launch() -> int:
    return NCU_SMALL_TRAFFIC * CFG["batch"] // NCU_SMALL_BATCH


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 100; e2e8b: 256 - warmup)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--case", default="config2", choices=["config2", "small"],
                    help="small: 8 sequences x 2 layers, for ncu captures")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "cp128k", "e2e8b", "decode_gemm"],
                    help="cp128k: config 4, 128K-context decode sharded over the ranks; "
                         "e2e8b: config 3, the 8B-architecture model end to end; "
                         "decode_gemm: its projections on the decode GEMM vs cuBLAS")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the chunked-prefill tensor-core measurement")
    ap.add_argument("--no-e2e8b", action="store_true", help="skip the 8B end-to-end decode measurement (config 3)")
    ap.add_argument("--wan-kv-splits", type=int, default=None,
                    help="force the Wan attention's key-split count (default: lkv_prefill_split_plan)")
    ap.add_argument("--cp-combine", default="p2p", choices=["p2p", "nccl"],
                    help="cp128k: combine the partials over peer memory (one kernel) or NCCL all-gather + merge")
    ap.add_argument("--cp-eager", action="store_true", help="cp128k: launch per layer instead of a CUDA graph")
    ap.add_argument("--no-cp", action="store_true",
                    help="skip the context-parallel 128K decode measurement (config 4) in the default line")
    ap.add_argument("--e2e-layers", type=int, default=None,
                    help="e2e8b with fewer layers (same per-layer shapes), for profiler captures; never a bench line")
    return ap.parse_args()


def workload_config(n_gpus):
    return {"workload": "shared_kv_decode_attention", "batch_per_gpu": CFG["batch"],
            "global_batch": CFG["batch"] * n_gpus, "q_heads": CFG["q_heads"], "kv_heads": CFG["kv_heads"],
            "head_dim": CFG["head_dim"], "context_tokens": CFG["context"], "page_tokens": CFG["page"],
            "layers_per_step": CFG["layers"], "chunk": CFG["chunk"], "layout": "merged [shared pages | layer ring]",
            "page_table": "shuffled", "l2": "inputs (2 GiB per layer call) larger than L2; no flush",
            "parallelism": f"dp{n_gpus} (batch-sharded replicas, no collective)"}


# ----------------------------------------------------------------- CPU baseline


class CpuLayerStep:
    """The reference's CPU layer-step (torch.cat history + SDPA) on `batch` sequences."""

    def __init__(self, batch: int):
        import torch

        from oracle.lastkv_oracle import reference_layer_step_cpu

        self.fn = reference_layer_step_cpu
        torch.manual_seed(0)
        H, Hq, D, N, C = CFG["kv_heads"], CFG["q_heads"], CFG["head_dim"], CFG["context"], CFG["chunk"]
        deep = N - C  # completed chunks [0, 7168) incl. the recent chunk; current chunk holds 1024 keys
        dt = torch.bfloat16
        self.args = (torch.randn(batch, Hq, 1, D, dtype=dt),
                     torch.randn(batch, H, deep, D, dtype=dt), torch.randn(batch, H, deep, D, dtype=dt),
                     torch.randn(batch, H, C, D, dtype=dt), torch.randn(batch, H, C, D, dtype=dt),
                     torch.randn(batch, H, C, D, dtype=dt), torch.randn(batch, H, C, D, dtype=dt),
                     torch.randn(H), torch.rand(H) + 0.5, C)
        self.threads = torch.get_num_threads()

    def step(self) -> float:
        t0 = time.perf_counter()
        self.fn(*self.args)
        return time.perf_counter() - t0


def cpu_layer_step_sample(seconds: float, batch: int):
    runner = CpuLayerStep(batch)
    runner.step()  # warm
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 3:
        times.append(runner.step())
    return times, runner.threads


def cpu_tokens_per_s(layer_step_s: float, batch: int) -> float:
    return batch / (CFG["layers"] * layer_step_s)


# ----------------------------------------------------------------- output check

# bf16 tolerance of the parity tests (attention outputs vs an fp32/float64 recomputation)
PARITY_TOL = {"max_abs": 2e-2, "rel_l2": 1e-2}


def torch_ref_rows(q_rows, pool_k, pool_v, bt_row, n_keys, scale, out_scale=None):
    """fp32 torch attention of query rows q_rows [R, Hq, D] of one sequence against its
    paged keys; row r sees keys [0, n_keys[r]) (the bench's own outputs are checked
    against this after its timed region)."""
    import torch

    R, Hq, D = q_rows.shape
    Hkv = pool_k.shape[2]
    n_max = int(max(n_keys))
    pages = bt_row[: -(-n_max // 16)].long()
    k = pool_k[pages].float().reshape(-1, Hkv, D)[:n_max]
    v = pool_v[pages].float().reshape(-1, Hkv, D)[:n_max]
    qg = q_rows.float().view(R, Hkv, Hq // Hkv, D)
    s = torch.einsum("rhgd,khd->rhgk", qg, k) * scale
    n = torch.as_tensor(list(n_keys), device=s.device).view(R, 1, 1, 1)
    s = s.masked_fill(torch.arange(n_max, device=s.device).view(1, 1, 1, -1) >= n, float("-inf"))
    o = torch.einsum("rhgk,khd->rhgd", torch.softmax(s, dim=-1), v).reshape(R, Hq, D)
    if out_scale is not None:
        o = o * out_scale.float().view(1, Hq, 1)
    return o


def parity_summary(pairs) -> dict:
    """max-abs and relative L2 over (got, want) pairs of tensors, against PARITY_TOL."""
    import torch

    got = torch.cat([g.float().reshape(-1) for g, _ in pairs])
    want = torch.cat([w.float().reshape(-1) for _, w in pairs])
    max_abs = float((got - want).abs().max())
    rel = float((got - want).norm() / want.norm().clamp_min(1e-12))
    return {"max_abs": max_abs, "rel_l2": rel, "values": int(got.numel()), "tolerance": PARITY_TOL,
            "pass": bool(max_abs <= PARITY_TOL["max_abs"] and rel <= PARITY_TOL["rel_l2"]),
            "reference": "torch fp32 recomputation of sampled rows on the same bf16 inputs"}


# ----------------------------------------------------------------- clocks


class ClockSampler:
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        import tempfile

        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        # nvidia-smi takes about a second to print its first sample, as long as a
        # short timed region: wait for it so the samples cover the region
        t_end = time.perf_counter() + 5.0
        while time.perf_counter() < t_end and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.05)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8 or not self.uuid or self.uuid not in parts[0]:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


# ----------------------------------------------------------------- GPU arm


def build_workload(rank: int, device):
    import torch

    from lastkv_b200 import ops

    B, Hq, H, D, N, L, C, P = (CFG[k] for k in ("batch", "q_heads", "kv_heads", "head_dim", "context", "layers",
                                                  "chunk", "page"))
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    pos = N - 1
    cur = (pos // C) * C
    rec = max(0, cur - C)
    nsrc = rec // P  # 384 shared pages per sequence
    ring_pages = 2 * C // P  # 128
    window_pages = -(-(pos + 1 - rec) // P)  # 128
    ring_stride = ring_pages * B + 1
    src_total = B * nsrc
    num_pages = src_total + L * ring_stride
    pool_k = torch.randn((num_pages, P, H, D), generator=gen, device=device, dtype=torch.bfloat16)
    pool_v = torch.randn((num_pages, P, H, D), generator=gen, device=device, dtype=torch.bfloat16)
    perm = torch.randperm(src_total, generator=gen, device=device).to(torch.int32)
    W = nsrc + window_pages
    bt = torch.empty((B, W), dtype=torch.int32, device=device)
    bt[:, :nsrc] = perm.view(B, nsrc)
    first = (rec // P) % ring_pages
    j = torch.arange(window_pages, device=device)
    bt[:, nsrc:] = (torch.arange(B, device=device)[:, None] * ring_pages + (first + j[None, :]) % ring_pages).to(
        torch.int32)
    nsrc_t = torch.full((B,), nsrc, dtype=torch.int32, device=device)
    ring_base = (src_total + torch.arange(L, device=device) * ring_stride).to(torch.int32)
    bt_all = ops.build_layer_block_tables(bt, nsrc_t, ring_base)
    seq_k = torch.full((B,), pos + 1, dtype=torch.int32, device=device)
    q = torch.randn((L, B, Hq, D), generator=gen, device=device, dtype=torch.bfloat16)
    scale = (torch.rand((L, H), generator=gen, device=device) + 0.5).to(torch.bfloat16).float()
    out_scale = scale.repeat_interleave(Hq // H, dim=1).contiguous()
    out = torch.empty((L, B, Hq, D), dtype=torch.bfloat16, device=device)
    ws = ops.Workspace.for_decode(B, Hq, D, W, device=device)
    return dict(pool_k=pool_k, pool_v=pool_v, bt=bt, nsrc=nsrc_t, ring_base=ring_base, bt_all=bt_all, seq_k=seq_k,
                q=q, out_scale=out_scale, out=out, ws=ws, W=W)


PREFILL = dict(batch=8, q_heads=32, kv_heads=8, head_dim=128, context=8192, chunk=1024)


def prefill_flops(span_start: int, span: int, batch: int, hq: int, d: int) -> int:
    """4 * Hq * D * sum over the span's queries of visible keys (causal, bottom-right)."""
    visible = span * span_start + span * (span + 1) // 2
    return 4 * hq * d * visible * batch


def measure_prefill(device, reps: int = 5, batch: int | None = None):
    """Chunked prefill attention of one layer over an 8192-token prompt (8 x 1024-token spans, batch 8).

    The 8B config's 2048-token prefill calls cross a chunk boundary (C = 1024),
    so each is issued as two chunk-aligned spans, as the reference's HF loop
    splits them (llm/src/lastkv/llm/modeling.py:194-208).
    """
    import torch

    from lastkv_b200 import ops

    B, Hq, H, D, N, C = (PREFILL[k] for k in ("batch", "q_heads", "kv_heads", "head_dim", "context", "chunk"))
    B = batch or B
    gen = torch.Generator(device=device).manual_seed(77)
    pages = N // 16
    pool_k = torch.randn((B * pages + 1, 16, H, D), generator=gen, device=device, dtype=torch.bfloat16)
    pool_v = torch.randn((B * pages + 1, 16, H, D), generator=gen, device=device, dtype=torch.bfloat16)
    bt = torch.randperm(B * pages, generator=gen, device=device).to(torch.int32).view(B, pages)
    q = torch.randn((B * C, Hq, D), generator=gen, device=device, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    err = torch.zeros(4, dtype=torch.int32, device=device)
    cu = torch.arange(0, B * C + 1, C, dtype=torch.int32, device=device)
    seqks = [torch.full((B,), C * (s + 1), dtype=torch.int32, device=device) for s in range(N // C)]

    def layer():
        for s in range(N // C):
            ops.prefill_paged(q, pool_k, pool_v, bt, seqks[s], cu, C, out=out, error_word=err,
                              max_pages=C * (s + 1) // 16)

    for _ in range(2):
        layer()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        layer()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = sum(prefill_flops(C * s, C, B, Hq, D) for s in range(N // C))
    # the last span alone (7168 keys of history + 1024 causal): the steady-state kernel rate
    l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0.record()
    for _ in range(reps):
        ops.prefill_paged(q, pool_k, pool_v, bt, seqks[-1], cu, C, out=out, error_word=err)
    l1.record()
    torch.cuda.synchronize()
    last_ms = l0.elapsed_time(l1) / reps
    last_flops = prefill_flops(N - C, C, B, Hq, D)
    if err.cpu().tolist()[0] != 0:
        raise RuntimeError(f"prefill device error word set: {err.cpu().tolist()}")
    # out holds the last span (7168 keys of history + 1024 causal queries): sampled tokens
    toks = torch.tensor([0, 1, 255, 512, C - 1], device=device)
    pairs = []
    for b in sorted({0, B - 1}):
        rows = b * C + toks
        want = torch_ref_rows(q[rows], pool_k, pool_v, bt[b], (N - C + toks + 1).tolist(), D ** -0.5)
        pairs.append((out[rows], want))
    parity = dict(parity_summary(pairs), rows="last span, 2 sequences x 5 tokens, all heads")
    try:
        peak = float(json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))["bf16_tflops"])
        src = "measured (burst)"
    except (OSError, KeyError, ValueError):
        peak, src = 1590.0, "fallback"
    tf = flops / (ms * 1e-3) / 1e12
    tf_last = last_flops / (last_ms * 1e-3) / 1e12
    return {"workload": f"chunked prefill attention, 1 layer, batch {B} x 8192-token prompt as 8 x 1024-token spans, "
                        "32/8 heads, D 128, shuffled pages", "ms_per_layer": ms, "flops_per_layer": flops,
            "tflops": tf, "frac": tf / peak, "last_span_tflops": tf_last, "last_span_frac": tf_last / peak,
            "peak_tflops": peak, "peak_source": src, "kernel": "prefill_tcgen05_kernel", "parity": parity}


WAN = dict(batch=2, heads=12, head_dim=128, frame_h=30, frame_w=52, frames_per_block=3, max_frames=21,
           prefix_tokens=1560)


def measure_wan(device, reps: int = 5, batch: int | None = None, kv_splits: int | None = None):
    """Wan-1.3B causal block attention (config 5): the last 3-frame block (4680 queries) against the
    full 21-frame history (32760 keys), per layer: fused 3-D-RoPE append + non-causal tcgen05 prefill."""
    import torch

    from lastkv_b200 import ops
    from lastkv_b200.wan import WanSharedKVCache, wan_block_attention

    W = dict(WAN)
    if batch:
        W["batch"] = batch
    B, H, D = W["batch"], W["heads"], W["head_dim"]
    cache = WanSharedKVCache(num_layers=1, batch=B, num_heads=H, head_dim=D, frame_h=W["frame_h"],
                             frame_w=W["frame_w"], frames_per_block=W["frames_per_block"],
                             max_frames=W["max_frames"], prefix_tokens=W["prefix_tokens"], device=device)
    BT = cache.block
    gen = torch.Generator(device=device).manual_seed(5)
    alpha = torch.rand((1, H), generator=gen, device=device)
    blocks = W["max_frames"] // W["frames_per_block"]

    def rnd():
        x = torch.randn((B, BT, H * D), generator=gen, device=device, dtype=torch.float32)
        return (x / x.pow(2).mean(-1, keepdim=True).sqrt()).to(torch.bfloat16)

    q, k, v = rnd(), rnd(), rnd()
    for n in range(blocks - 1):  # build the history block by block
        cache.begin_block(n)
        wan_block_attention(q, k, v, cache, 0)
        cache.commit_block(alpha)
    m = cache.begin_block(blocks - 1)
    S = (blocks - 1) * BT
    flops = 4 * H * D * BT * (S + BT) * B
    wan_block_attention(q, k, v, cache, 0)
    qa = torch.randn((B * BT, H, D), generator=gen, device=device, dtype=torch.bfloat16)
    out = torch.empty_like(qa)

    splits = kv_splits or ops.prefill_split_plan(B, BT, H, H, D, int(m["W"]), False)

    def attn_only():
        ops.prefill_paged(qa, cache.pool_k, cache.pool_v, m["bt"][0], m["seq_k"], m["cu_q"], BT, causal=False,
                          out=out, error_word=cache.error_word, max_pages=m["W"], kv_splits=splits)

    attn_only()
    torch.cuda.synchronize()
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record()
    for _ in range(reps):
        attn_only()
    e[1].record()
    for _ in range(reps):
        wan_block_attention(q, k, v, cache, 0)
    e[2].record()
    torch.cuda.synchronize()
    cache.check_errors()
    attn_ms = e[0].elapsed_time(e[1]) / reps
    layer_ms = e[1].elapsed_time(e[2]) / reps
    attn_only()  # out: the timed call's result again (the layer calls above share the cache, not `out`)
    toks = torch.tensor([0, 1559, 1560, 3000, BT - 1], device=device)
    pairs = []
    for b in range(B):
        rows = b * BT + toks
        nk = int(m["seq_k"][b])
        want = torch_ref_rows(qa[rows], cache.pool_k, cache.pool_v, m["bt"][0][b], [nk] * len(toks), D ** -0.5)
        pairs.append((out[rows], want))
    parity = dict(parity_summary(pairs), rows=f"{B} sequences x 5 block tokens, all heads, non-causal")
    try:
        peak = float(json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))["bf16_tflops"])
        src = "measured (burst)"
    except (OSError, KeyError, ValueError):
        peak, src = 1590.0, "fallback"
    tf = flops / (attn_ms * 1e-3) / 1e12
    return {"workload": f"Wan-1.3B block attention: batch {B}, 12 heads x 128, 4680-token block vs "
                        f"{S + BT} keys ([1560 prefix | shared | blended prev block | block]), non-causal",
            "flops_per_layer": flops, "attn_ms": attn_ms, "tflops": tf, "frac": tf / peak,
            "layer_ms_incl_rope_append": layer_ms, "peak_tflops": peak, "peak_source": src,
            "kernel": "prefill_tcgen05_kernel<128, 1> (non-causal, keys split in one launch) + merge_partials_kernel",
            "kv_splits": splits, "parity": parity}


def measure_commit(device, reps: int = 5):
    """Config 3's chunk-boundary commit (8B shapes: 32 layers, 8 KV heads x 128, chunk 1024,
    batch 8): the step after the boundary's first-layer append with the blend of every
    layer's finished chunk fused in (lkv_rope_norm_append_commit), against the append and
    lkv_blend_chunk as two launches.  The blend is HBM-bound: per page of K or V it reads
    the shared raw page and the ring page and writes the ring page; the raw pages of one
    chunk (a few tens of MB) stay in L2 across the layers."""
    import torch

    from lastkv_b200 import ops

    L, Hq, Hkv, D, C, B = (E2E8B[k] for k in ("layers", "q_heads", "kv_heads", "head_dim", "chunk", "batch"))
    ppc = C // 16
    ring_stride = B * 2 * ppc + 1
    src = B * 2 * ppc
    total = src + L * ring_stride
    gen = torch.Generator(device=device).manual_seed(77)
    pool_k = torch.randn((total, 16, Hkv, D), generator=gen, device=device).to(torch.bfloat16)
    pool_v = torch.randn((total, 16, Hkv, D), generator=gen, device=device).to(torch.bfloat16)
    raw = torch.arange(B * ppc, dtype=torch.int32, device=device).view(B, ppc)
    ring = (src + torch.arange(B, device=device)[:, None] * 2 * ppc
            + torch.arange(ppc, device=device)[None, :]).to(torch.int32).contiguous()
    alpha = torch.rand((L, Hkv), generator=gen, device=device).to(torch.bfloat16).float()
    q = torch.randn((B, Hq * D), generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn((B, Hkv * D), generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn((B, Hkv * D), generator=gen, device=device).to(torch.bfloat16)
    pos = torch.full((B,), C, dtype=torch.int64, device=device)
    cs = torch.randn((C + 1, D), generator=gen, device=device).to(torch.bfloat16)
    w = torch.ones(D, dtype=torch.bfloat16, device=device)
    inv = torch.ones(Hkv, dtype=torch.float32, device=device)
    slot = ((src + torch.arange(B, device=device) * 2 * ppc + ppc) * 16).to(torch.int64)  # second ring half
    flat_k, flat_v = pool_k.view(-1, Hkv, D), pool_v.view(-1, Hkv, D)
    err = torch.zeros(4, dtype=torch.int32, device=device)
    commit = ops.Commit(pool_k, pool_v, raw, ring, ring_stride, alpha)

    def append(c=None):
        ops.rope_norm_append(q, k, v, pos, cs, w, w, 1e-6, inv, slot, flat_k, flat_v, error_word=err, commit=c)

    def separate():
        append()
        ops.blend_chunk(pool_k, pool_v, raw, ring, ring_stride, alpha, error_word=err)

    sms = torch.cuda.get_device_properties(device).multi_processor_count
    count = torch.zeros(1, dtype=torch.int32, device=device)

    def timed(fn, n=reps):
        """Device ms per call: n calls captured in one CUDA graph (no host launch cost), replayed."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(n):
                fn()
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        del g
        return a.elapsed_time(b) / n

    sep_ms = timed(separate)
    fused_ms = timed(lambda: append(commit))
    # the device-count form a captured step carries every step: its cost without a boundary
    # (count 0) and its blend time with one (count = batch), at 2 and 8 commit blocks per SM
    plain_us = timed(append, 50) * 1e3
    dev_count = {}
    for per_sm in (2, 8):
        c = commit._replace(count=count, blocks=per_sm * sms)
        count.fill_(0)
        idle_us = timed(lambda: append(c), 50) * 1e3
        count.fill_(B)
        dev_count[f"{per_sm}_per_sm"] = {"no_boundary_us": idle_us, "no_boundary_extra_us": idle_us - plain_us,
                                         "boundary_ms": timed(lambda: append(c))}
    # parity at these shapes: the fused launch (host row count, then device row count) and
    # the two separate launches from the same starting pools give the same bits
    start_k, start_v = pool_k.clone(), pool_v.clone()
    separate()
    want_k, want_v = pool_k.clone(), pool_v.clone()
    same = {}
    for name, c in (("host_count", commit), ("device_count", commit._replace(count=count, blocks=8 * sms))):
        pool_k.copy_(start_k)
        pool_v.copy_(start_v)
        count.fill_(B)
        append(c)
        same[name] = bool(torch.equal(pool_k, want_k) and torch.equal(pool_v, want_v))
    del start_k, start_v, want_k, want_v
    if int(err[0]):
        raise RuntimeError(f"commit bench: device error word {err.tolist()}")
    page_bytes = 16 * Hkv * D * 2
    # K and V: every layer's ring page read and written, each raw page read once (the other
    # layers' reads of the chunk's 2 x B x ppc raw pages hit L2)
    nbytes = B * ppc * L * 2 * 2 * page_bytes + B * ppc * 2 * page_bytes
    gbs = nbytes / (fused_ms * 1e-3) / 1e9
    try:
        peak = float(json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))["hbm_gbs"])
        src_peak = "measured"
    except (OSError, KeyError, ValueError):
        peak, src_peak = 6650.0, "fallback"
    return {"workload": f"boundary commit, 8B shapes: {L} layers x {B} sequences x {ppc} pages of K and V, "
                        f"fused into the next step's layer-0 append of {B} tokens",
            "fused_ms": fused_ms, "separate_ms": sep_ms, "saved_us": (sep_ms - fused_ms) * 1e3,
            "algorithmic_bytes": nbytes, "achieved_gbs": gbs, "peak_gbs": peak, "frac": gbs / peak,
            "peak_source": src_peak, "l2": f"{nbytes / 1e9:.1f} GB per launch (larger than L2); no flush",
            "append_alone_us": plain_us, "device_count": dev_count,
            "parity": {"fused_equals_separate": same, "pass": all(same.values()),
                       "reference": "append + lkv_blend_chunk as two launches on the same starting pools, "
                                    "every pool byte compared"},
            "kernel": "append_commit_kernel<128> (vs rope_norm_append_kernel<128> + blend_chunk_kernel)"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    from lastkv_b200 import _capi, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    _capi.load()
    _capi.check(_capi.lib().lkv_check_device(local), "lkv_check_device")
    wl = build_workload(rank, device)
    L, B = CFG["layers"], CFG["batch"]
    splits, launches_per_call = ops.decode_plan(B, CFG["q_heads"], CFG["kv_heads"], CFG["head_dim"], wl["W"],
                                                wl["ws"])

    def layer(l):
        # the tables were built at set-up, before any torch launch of the warm-up: ready
        ops.decode_paged(wl["q"][l], wl["pool_k"], wl["pool_v"], wl["bt_all"][l], wl["seq_k"], out=wl["out"][l],
                         out_scale=wl["out_scale"][l], workspace=wl["ws"], max_pages=wl["W"], tables_ready=True)

    def barrier():
        if world > 1:
            dist.barrier()

    uuid = str(torch.cuda.get_device_properties(device).uuid)
    side = {}
    if not args.no_prefill:
        # The tensor-core legs first, before the HBM-bound decode loop has run the GPU
        # into its power cap: each is a short burst, set against the burst GEMM peak,
        # with the SM clocks sampled around the two of them.
        pclk = ClockSampler(uuid)
        pclk.start()
        # the small case (profiler captures) runs the same spans with 2 sequences
        side["prefill"] = measure_prefill(device, batch=None if args.case == "config2" else 2)
        side["wan"] = measure_wan(device, batch=None if args.case == "config2" else 1, kv_splits=args.wan_kv_splits)
        tc_clk = pclk.stop()
        side["prefill"]["clocks"] = side["wan"]["clocks"] = tc_clk
        side["commit"] = measure_commit(device)
        torch.cuda.empty_cache()

    stream = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 0)):
        for l in range(L):
            layer(l)
    torch.cuda.synchronize()

    clocks = ClockSampler(uuid)
    # The layer calls go back to back (no events between them, which would cut the
    # programmatic-dependent-launch overlap of consecutive kernels, as a real decode
    # step has none); the average launch time is the timed region over the calls.
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    t0.record(stream)
    for s in range(args.steps):
        for l in range(L):
            layer(l)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    total_ms = t0.elapsed_time(t1)
    op_ms = [total_ms / (args.steps * L)]
    err = wl["ws"].error()
    if err[0] != 0:
        raise RuntimeError(f"device error word set: {err}")
    # the timed region's own outputs (its last step), sampled sequences of the first and last layer
    D = CFG["head_dim"]
    pairs = []
    for l in (0, L - 1):
        for b in sorted({0, B // 3, 2 * B // 3, B - 1}):
            n = int(wl["seq_k"][b])
            want = torch_ref_rows(wl["q"][l][b:b + 1], wl["pool_k"], wl["pool_v"], wl["bt_all"][l][b], [n],
                                  D ** -0.5, wl["out_scale"][l])
            pairs.append((wl["out"][l][b:b + 1], want))
    decode_parity = dict(parity_summary(pairs), rows=f"layers 0 and {L - 1}, 4 sequences each, all heads")

    # ---- end to end through the public op with host buffers every step
    q_host = torch.empty(wl["q"].shape, dtype=wl["q"].dtype, pin_memory=True)
    q_host.copy_(wl["q"].cpu())
    out_host = torch.empty(wl["out"].shape, dtype=wl["out"].dtype, pin_memory=True)
    bt_host = wl["bt"].cpu().pin_memory()
    nsrc_host = wl["nsrc"].cpu().pin_memory()
    seqk_host = wl["seq_k"].cpu().pin_memory()
    h2d = q_host.numel() * 2 + bt_host.numel() * 4 + nsrc_host.numel() * 4 + seqk_host.numel() * 4
    d2h = out_host.numel() * 2

    # A serving loop: each step's queries are uploaded and its outputs downloaded on a copy
    # stream, overlapping the neighbouring steps' attention (double-buffered q and out);
    # the small per-step tables go in-line on the compute stream.
    # Uploads and downloads go on two streams of their own: on one, the next step's upload
    # would queue behind this step's download, which waits for this step to finish.
    up_stream, down_stream = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
    q_dev = [wl["q"], torch.empty_like(wl["q"])]
    out_dev = [wl["out"], torch.empty_like(wl["out"])]
    ev_h2d = [torch.cuda.Event(), torch.cuda.Event()]
    ev_d2h = [torch.cuda.Event(), torch.cuda.Event()]
    ev_done = [torch.cuda.Event(), torch.cuda.Event()]

    def upload(k):
        with torch.cuda.stream(up_stream):
            up_stream.wait_event(ev_done[k])  # the step that last read q_dev[k] has finished
            q_dev[k].copy_(q_host, non_blocking=True)
            ev_h2d[k].record(up_stream)

    def e2e_step(i, n):
        k = i % 2
        stream.wait_event(ev_h2d[k])
        stream.wait_event(ev_d2h[k])  # the download that last read out_dev[k] has finished
        wl["bt"].copy_(bt_host, non_blocking=True)
        wl["nsrc"].copy_(nsrc_host, non_blocking=True)
        wl["seq_k"].copy_(seqk_host, non_blocking=True)
        ops.build_layer_block_tables(wl["bt"], wl["nsrc"], wl["ring_base"], out=wl["bt_all"])
        # the tables come from the kernel just launched, in the same PDL chain: not "ready"
        for l in range(L):
            ops.decode_paged(q_dev[k][l], wl["pool_k"], wl["pool_v"], wl["bt_all"][l], wl["seq_k"],
                             out=out_dev[k][l], out_scale=wl["out_scale"][l], workspace=wl["ws"], max_pages=wl["W"])
        ev_done[k].record(stream)
        with torch.cuda.stream(down_stream):
            down_stream.wait_event(ev_done[k])
            out_host.copy_(out_dev[k], non_blocking=True)  # this step's result to the host
            ev_d2h[k].record(down_stream)
        if i + 1 < n:
            upload(1 - k)                                   # the next step's queries

    def e2e_run(n):
        upload(0)
        for i in range(n):
            e2e_step(i, n)
        stream.wait_stream(down_stream)  # the last download is part of the run

    e2e_run(max(args.warmup, 1))
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up_stream.wait_event(e0)  # the first upload starts inside the timed region
    down_stream.wait_event(e0)
    e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    vals = torch.tensor([total_ms, e2e_ms, float(np.mean(op_ms))], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms, avg_op_ms = vals.tolist()

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))
        peak, peak_src = float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        peak, peak_src = 6650.0, "fallback"
    achieved = algo_bytes() / (avg_op_ms * 1e-3) / 1e9
    tokens = B * args.steps * world
    line = {
        "metric": METRIC, "value": tokens / (total_ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(world),
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_src,
                     "kernel": "decode op = decode_splitkv_kernel + merge_partials_kernel",
                     "algorithmic_bytes_per_launch": algo_bytes(), "avg_launch_ms": avg_op_ms,
                     "traffic": traffic_per_launch(),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the small case "
                                       "(8 sequences), scaled by the sequences per launch"},
        "attn_hbm_gbs": achieved,
        "parity": decode_parity,
        "clocks": clk,
        "gpu_launches": int(args.steps * L * launches_per_call),
        "kv_splits": splits,
    }
    line.update(side)
    if not args.no_e2e8b:
        # config 3 on the same ranks: the 8B architecture end to end (weak scaling, batch 8 per GPU)
        wl = None
        torch.cuda.empty_cache()
        e = measure_e2e8b(max(E2E8B["decode_tokens"] - 3, 1), 3, world, device)
        line["e2e8b"] = {"metric": e["metric"], "value": e["value"], "unit": e["unit"], "n_gpus": world,
                         "batch_per_gpu": E2E8B["batch"], "layers": E2E8B["layers"],
                         "ms_per_step": e["ms_per_step"], "steps": e["steps"], "e2e": e["e2e"]["value"],
                         "roofline_frac": e["roofline"]["frac"], "achieved_gbs": e["roofline"]["achieved"],
                         "prefill_tokens_per_s": e["prefill"]["tokens_per_s"],
                         "gpu_launches": e["gpu_launches"]}
        if world > 1 and E2E8B["batch"] % world == 0:
            # config 3's own global batch of 8 split over the N GPUs (strong scaling): each rank
            # streams all the weights for 8/N sequences, so tokens/s grows far less than N
            e = measure_e2e8b(max(E2E8B["decode_tokens"] - 3, 1), 3, world, device, batch=E2E8B["batch"] // world)
            line["e2e8b_global8"] = {"metric": e["metric"].replace(f"batch {E2E8B['batch'] // world} per GPU",
                                                                   "global batch 8"),
                                     "value": e["value"], "unit": e["unit"], "n_gpus": world,
                                     "batch_per_gpu": E2E8B["batch"] // world, "global_batch": E2E8B["batch"],
                                     "scaling": "strong", "ms_per_step": e["ms_per_step"],
                                     "e2e": e["e2e"]["value"], "roofline_frac": e["roofline"]["frac"]}
    if not args.no_cp:
        # config 4 on the same ranks: 128K-context decode sharded over all N GPUs (strong scaling)
        wl = None
        torch.cuda.empty_cache()
        c4 = measure_cp(100, 3, world, rank, device, combine=args.cp_combine, eager=args.cp_eager)
        line["cp128k"] = {k: c4[k] for k in ("metric", "value", "unit", "n_gpus", "steps", "ms_per_step",
                                             "scaling", "layer_ms", "hbm_gbs_per_gpu", "hbm_frac_per_gpu",
                                             "combine_bytes_per_rank_per_layer", "parity", "error") if k in c4}
        line["cp128k"]["parallelism"] = c4["config"]["parallelism"]
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        times, threads = cpu_layer_step_sample(args.cpu_seconds, batch=8)
        med = statistics.median(times)
        line["cpu_baseline"] = {"value": cpu_tokens_per_s(med, 8), "unit": UNIT, "cores": threads,
                                "cpu_count": os.cpu_count(),
                                "kind": "port",
                                "sample": f"reference CPU layer-step (torch.cat history + torch SDPA, bf16) on 8 of "
                                          f"64 sequences, {len(times)} reps, median {med * 1e3:.1f} ms; "
                                          f"tokens/s = 8 / (32 layers x median)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import torch

    # torch.distributed.run exports OMP_NUM_THREADS=1 to every rank; rank 0 alone runs
    # this arm, so give it every host core, as the single-process run has.
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    batch = 8
    runner = CpuLayerStep(batch)
    threads = runner.threads
    warm = [runner.step() for _ in range(max(args.warmup, 0))]
    steps = [runner.step() for _ in range(max(args.steps, 1))]
    med = statistics.median(steps)
    value = cpu_tokens_per_s(med, batch)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": med * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": workload_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "cpu_count": cores, "kind": "port",
                         "sample": f"one layer-step of the reference's CPU attention (torch.cat history + torch SDPA "
                                   f"bf16) on {batch} of 64 sequences per step; tokens/s = {batch} / (32 x median)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "warmup_s": [round(x, 4) for x in warm],
    }
    print(json.dumps(line), flush=True)


CP = dict(batch=4, q_heads=32, kv_heads=8, head_dim=128, context=131072, window=2048, layers=32)


def run_cp(args):
    """Config 4 alone (``--workload cp128k``): prints its line (rank 0)."""
    import datetime

    import torch
    import torch.distributed as dist

    from lastkv_b200 import _capi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    _capi.load()
    line = measure_cp(args.steps, args.warmup, world, rank, device, combine=args.cp_combine, eager=args.cp_eager)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _cp_shard_tensors(rank: int, world: int, device):
    """Rank ``rank``'s slice of config 4: its pools, shuffled block table and key count
    (seeded per rank, so any rank can rebuild another's slice for the output check)."""
    import torch

    from lastkv_b200.context_parallel import plan_shard

    B, H, D, N, Wt = (CP[k] for k in ("batch", "kv_heads", "head_dim", "context", "window"))
    sp = plan_shard((N - Wt) // 16, Wt, 16, world, rank)
    pages = (sp.p1 - sp.p0) + sp.ring_pages
    gen = torch.Generator(device=device).manual_seed(300 + rank)
    pool_k = torch.randn((B * pages + 1, 16, H, D), generator=gen, device=device, dtype=torch.bfloat16)
    pool_v = torch.randn((B * pages + 1, 16, H, D), generator=gen, device=device, dtype=torch.bfloat16)
    bt = torch.randperm(B * pages, generator=gen, device=device).to(torch.int32).view(B, pages)
    return pool_k, pool_v, bt, sp.seq_k, pages


def measure_cp(steps: int, warmup: int, world: int, rank: int, device, combine: str = "p2p",
               eager: bool = False) -> dict:
    """Config 4: 128K-context decode, sequence-sharded over the ranks (context parallel).

    Each rank holds a contiguous 1/G slice of every sequence's shared pages (the
    last rank also the 2048-token ring window).  With one rank a layer is the
    plain split-KV decode; with more, each layer is ``lkv_decode_paged_cp`` (the
    decode kernel pushes each unit's merged rows to every rank over peer memory,
    then polls and merges every rank's rows in the same launch) or, with
    ``combine="nccl"``, the partial
    decode + NCCL all-gather + merge.  The queries are the same on every rank (one
    decode token).  After the timed region rank 0 checks sampled rows of its
    output against an fp32 recomputation over all ranks' keys (each rank's slice
    rebuilt from its seed).  All ranks call this together.
    """
    import torch
    import torch.distributed as dist

    from lastkv_b200 import ops
    from lastkv_b200.context_parallel import ContextParallelDecode

    B, Hq, H, D, N, Wt, L = (CP[k] for k in ("batch", "q_heads", "kv_heads", "head_dim", "context", "window",
                                             "layers"))
    pool_k, pool_v, bt, seq_len, pages_mine = _cp_shard_tensors(rank, world, device)
    seq_k = torch.full((B,), seq_len, dtype=torch.int32, device=device)
    qgen = torch.Generator(device=device).manual_seed(299)  # one query token, the same on every rank
    q = torch.randn((L, B, Hq, D), generator=qgen, device=device, dtype=torch.bfloat16)
    scale = (torch.rand((L, Hq), generator=qgen, device=device) + 0.5).to(torch.bfloat16).float()
    out = torch.empty((L, B, Hq, D), dtype=torch.bfloat16, device=device)
    ws = ops.Workspace.for_decode(B, Hq, D, pages_mine, device=device)
    cp = ContextParallelDecode(combine=combine) if world > 1 else None

    def step():
        for l in range(L):
            if cp is None:
                ops.decode_paged(q[l], pool_k, pool_v, bt, seq_k, out=out[l], out_scale=scale[l], workspace=ws,
                                 max_pages=pages_mine, tables_ready=True, l2_keep=True)  # tables written at set-up
            else:
                cp.layer(q[l], pool_k, pool_v, bt, seq_k, out_scale=scale[l], out=out[l], workspace=ws,
                         max_pages=pages_mine, tables_ready=True, l2_keep=True)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(warmup, 1)):
        step()
    torch.cuda.synchronize()
    graph = None
    if not eager:
        # the 32 layer calls of one step as one CUDA graph (the combine's epoch lives on the device)
        barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    # device errors travel with the timing in one all-reduce, so every rank takes the same
    # collective steps whatever happened on one of them
    err_words = [ws.error()] + ([st["error"].cpu().tolist() for st in cp._p2p.values()] if cp is not None else [])
    failed = next((w for w in err_words if w[0] != 0), None)
    t = torch.tensor([e0.elapsed_time(e1), 1.0 if failed else 0.0], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0].item())
    any_failed = bool(t[1].item())
    del graph, run  # a graph holding collectives goes before the process group
    parity = None
    if rank == 0 and not any_failed:
        # the last layer's output of the last step, sequences 0 and B-1, against all ranks' keys
        l = L - 1
        keys = {b: ([], []) for b in (0, B - 1)}
        for r in range(world):
            pk, pv, bt_r, n_r, _ = (pool_k, pool_v, bt, seq_len, None) if r == rank else \
                _cp_shard_tensors(r, world, device)
            for b in keys:
                pg = bt_r[b][: -(-n_r // 16)].long()
                keys[b][0].append(pk[pg].reshape(-1, H, D)[:n_r])
                keys[b][1].append(pv[pg].reshape(-1, H, D)[:n_r])
            del pk, pv
        pairs = []
        for b, (ks, vs) in keys.items():
            k, v = torch.cat(ks).float(), torch.cat(vs).float()
            assert k.shape[0] == N
            qg = q[l][b].float().view(H, Hq // H, D)
            p_ = torch.softmax(torch.einsum("hgd,khd->hgk", qg, k) * D ** -0.5, dim=-1)
            want = torch.einsum("hgk,khd->hgd", p_, v).reshape(Hq, D) * scale[l].view(Hq, 1)
            pairs.append((out[l][b], want))
        parity = dict(parity_summary(pairs), rows=f"last layer, sequences 0 and {B - 1}, all heads, over all "
                                                  f"{world} ranks' keys")
        del keys
    layer_ms = ms / (steps * L)
    bytes_layer = 2 * B * H * N * D * 2
    try:
        peak = float(json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        peak = 6650.0
    mode = ("plain split-KV decode (one GPU)" if cp is None else
            "one decode launch per layer: pushes each unit's merged rows over peer memory, then polls and "
            "LSE-merges every rank's rows"
            if cp.combine == "p2p" else "NCCL all-gather + LSE merge")
    line = {"metric": "context-parallel decode tokens/s (attention only, 32 layers, 128K context)",
            "value": B * steps / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cp128k", "batch": B, "context_tokens": N, "ring_window": Wt, "q_heads": Hq,
                       "kv_heads": H, "head_dim": D, "layers_per_step": L,
                       "parallelism": f"cp{world} (shared pages sharded; {mode})",
                       "launch": "eager per layer" if eager else "one CUDA graph per step"},
            "layer_ms": layer_ms, "attn_bytes_per_layer_total": bytes_layer,
            "hbm_gbs_per_gpu": bytes_layer / world / (layer_ms * 1e-3) / 1e9,
            "hbm_frac_per_gpu": bytes_layer / world / (layer_ms * 1e-3) / 1e9 / peak,
            "combine_bytes_per_rank_per_layer": B * Hq * (D + 1) * 4 if world > 1 else 0,
            "parity": parity}
    if any_failed:
        line["error"] = f"a rank's device error word was set (this rank: {failed})"
    del cp, pool_k, pool_v, out, ws
    torch.cuda.empty_cache()
    return line


E2E8B = dict(layers=32, hidden=4096, q_heads=32, kv_heads=8, head_dim=128, ffn=14336, vocab=128256, chunk=1024,
             batch=8, prompt=8192, prefill_call=2048, decode_tokens=256)
# A 4-layer, 2-sequence, 2048-token version for quick checks and profiler captures; never a bench line.
E2E8B_SMALL = dict(layers=4, batch=2, prompt=2048)


def e2e8b_config():
    from lastkv_b200.hf import LastKVConfig

    c = E2E8B
    return LastKVConfig(hidden_size=c["hidden"], intermediate_size=c["ffn"], num_attention_heads=c["q_heads"],
                        num_key_value_heads=c["kv_heads"], num_hidden_layers=c["layers"], head_dim=c["head_dim"],
                        vocab_size=c["vocab"], chunk_size=c["chunk"], rms_norm_eps=1e-5, rope_theta=500000.0,
                        rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                      "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
                        max_position_embeddings=131072)


def run_e2e8b(args):
    """Config 3: the 8B-architecture model end to end, batch 8 per GPU (weak scaling).

    Random-init bf16 weights (built on the meta device, materialised on the
    GPU, then seeded N(0, 0.02); blend logits ~ N(0, 1), value scales ~ U(0.1, 2)).
    Prefill: 8192 random-token prompts in 2048-token calls (each split at the
    1024-token chunk boundaries, as the reference's chunk loop does), timed
    once after one warm-up call on a scratch cache.  Decode: every step is one
    replay of the CUDA graph of the whole model step (fused append + split-KV
    decode per layer, cuBLAS dense layers, argmax) with the host plan copied in
    from pinned memory and the new ids copied out to pinned memory; warm-up +
    timed steps = the config's 256 decode tokens by default.  Ranks run
    independent replicas (no collective on the data path).
    """
    import datetime

    import torch
    import torch.distributed as dist

    from lastkv_b200 import _capi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    _capi.load()
    _capi.check(_capi.lib().lkv_check_device(local), "lkv_check_device")
    line = measure_e2e8b(args.steps, args.warmup, world, device)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measure_e2e8b(steps: int, warmup: int, world: int, device, batch: int | None = None) -> dict:
    """Config 3 on this rank's GPU (all ranks call it together); returns the bench line.
    ``batch``: sequences on this rank (default: the config's 8)."""
    import torch
    import torch.distributed as dist

    from lastkv_b200 import ops
    from lastkv_b200.hf import LastKVForCausalLM
    from lastkv_b200.runner import GraphDecodeRunner, init_random_

    rank = dist.get_rank() if world > 1 else 0

    class _Args:
        pass

    args = _Args()
    args.steps, args.warmup = steps, warmup
    c = E2E8B
    B, P, call, L = batch or c["batch"], c["prompt"], c["prefill_call"], c["layers"]
    Hkv, D = c["kv_heads"], c["head_dim"]
    cfg = e2e8b_config()
    with torch.device("meta"):
        model = LastKVForCausalLM(cfg)
    model = model.to(torch.bfloat16).to_empty(device=device).eval()
    init_random_(model, seed=1234)
    model.model._alpha = None
    model.fuse_projections_()
    weight_bytes = sum(p.numel() * p.element_size() for n, p in model.named_parameters() if "embed_tokens" not in n)
    gen = torch.Generator(device=device).manual_seed(77 + rank)
    prompt = torch.randint(0, c["vocab"], (B, P), generator=gen, device=device)
    total_tokens = P + args.warmup + args.steps
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.no_grad():
        scratch = model.new_cache(B, call)
        model(prompt[:, :call], scratch, logits_to_keep=1)  # cuBLAS / kernel warm-up, same shapes
        del scratch
        cache = model.new_cache(B, total_tokens + 1)
        runner = GraphDecodeRunner(model, cache)
        torch.cuda.synchronize()
        barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        runner.prefill(prompt, call)
        p1.record(stream)
        torch.cuda.synchronize()
        prefill_ms = p0.elapsed_time(p1)

        runner.capture()
        for _ in range(args.warmup):
            runner.step()
        host_ids = torch.empty((max(args.steps, 1), B), dtype=torch.int64, pin_memory=True)
        torch.cuda.synchronize()
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        clocks = ClockSampler(uuid)
        clocks.start()
        barrier()
        torch.cuda.synchronize()
        first_pos = cache.seen_tokens
        w0 = time.perf_counter()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for i in range(args.steps):
            ids = runner.step()
            host_ids[i].copy_(ids.view(-1), non_blocking=True)
        d1.record(stream)
        torch.cuda.synchronize()
        wall_ms = (time.perf_counter() - w0) * 1e3
        barrier()
        clk = clocks.stop()
    cache.check_errors()
    decode_ms = d0.elapsed_time(d1)
    if not bool(((host_ids[: args.steps] >= 0) & (host_ids[: args.steps] < c["vocab"])).all()):
        raise RuntimeError("decoded ids out of range")
    vals = torch.tensor([decode_ms, wall_ms, prefill_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    decode_ms, wall_ms, prefill_ms = vals.tolist()

    # HBM bytes one step must move: every weight but the embedding table once, plus
    # every layer's keys and values (token p attends to p + 1 keys per sequence)
    kv_bytes = sum(L * B * (first_pos + i + 1) * Hkv * D * 2 * 2 for i in range(args.steps))
    step_bytes = weight_bytes + kv_bytes / max(args.steps, 1)
    ms_step = decode_ms / max(args.steps, 1)
    try:
        peak, peak_src = float(json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        peak, peak_src = 6650.0, "fallback"
    achieved = step_bytes / (ms_step * 1e-3) / 1e9
    splits, per_call = ops.decode_plan(B, c["q_heads"], Hkv, D, cache.pages_per_seq + cache.ring_pages,
                                       cache.workspace)
    # ours per step: block tables + final RMSNorm + argmax + per layer (2 RMSNorm, 4 decode
    # GEMMs [q|k|v, o, gate|up+SiLU, down], append, split-KV decode [+ merge]); the
    # embedding gather, rotary table and LM head (cuBLAS) are torch ops
    launches_per_step = 3 + L * (2 + 4 + 1 + per_call)
    H, F_ = c["hidden"], c["ffn"]
    gemm_plans = {name: ops.decode_gemm_plan(n, k, silu) for name, n, k, silu in
                  (("qkv", (c["q_heads"] + 2 * Hkv) * D, H, False), ("o", c["q_heads"] * D, H, False),
                   ("gate_up", 2 * F_, H, True), ("down", H, F_, False))}
    tokens = B * args.steps * world
    h2d = sum(t.numel() * t.element_size() for k, t in runner._h[0].items()
                                            if k != "done")
    line = {
        "metric": f"end-to-end decode tokens/s (8B architecture, batch {B} per GPU, CUDA-graph steps)",
        "value": tokens / (decode_ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, random prompt ids)",
        "config": {"workload": "e2e8b", "layers": L, "d_model": c["hidden"], "q_heads": c["q_heads"],
                   "kv_heads": Hkv, "head_dim": D, "ffn": c["ffn"], "vocab": c["vocab"], "chunk": c["chunk"],
                   "batch_per_gpu": B, "global_batch": B * world, "prompt_tokens": P,
                   "prefill_call_tokens": call, "decode_positions": [first_pos, first_pos + args.steps],
                   "l2": "16 GB of weights per step (larger than L2); no flush",
                   "parallelism": f"dp{world} (independent replicas, no collective)"},
        "e2e": {"value": tokens / (wall_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": B * 8,
                "timing": "host wall clock around the step loop (plan H2D + graph replay + ids D2H), max over ranks"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": peak_src, "kernel": "whole decode step (weights + shared-KV reads)",
                     "algorithmic_bytes_per_step": int(step_bytes), "weight_bytes": int(weight_bytes),
                     "kv_bytes_per_step": int(kv_bytes / max(args.steps, 1)), "traffic": None},
        "prefill": {"tokens_per_s": B * P * world / (prefill_ms * 1e-3), "ms": prefill_ms,
                    "tokens_per_gpu": B * P},
        "clocks": clk,
        "gpu_launches": int(args.steps * launches_per_step),
        "kv_splits": splits,
        "decode_gemm_plans": gemm_plans,
    }
    del runner, cache, model
    torch.cuda.empty_cache()
    return line


def run_decode_gemm(args):
    """The decode-step projections of the 8B architecture (M = 8 rows) on the tcgen05
    decode GEMM and on cuBLAS (torch), each timed inside a CUDA graph over enough
    weight copies (> 600 MB) that no weight is L2-resident between calls."""
    import torch

    from lastkv_b200 import _capi, ops

    torch.cuda.set_device(0)
    _capi.load()
    c = E2E8B
    H, F_, D = c["hidden"], c["ffn"], c["head_dim"]
    shapes = [("qkv", (c["q_heads"] + 2 * c["kv_heads"]) * D, H, False), ("o", c["q_heads"] * D, H, False),
              ("gate_up_silu", 2 * F_, H, True), ("down", H, F_, False), ("lm_head", c["vocab"], H, False)]
    gen = torch.Generator(device="cuda").manual_seed(5)
    rows = []
    for name, n, k, silu in shapes:
        nbytes = n * k * 2
        copies = max(2, int(600e6 // nbytes) + 1)
        ws = [(torch.randn((n, k), generator=gen, device="cuda") * 0.02).bfloat16() for _ in range(copies)]
        x = torch.randn((8, k), generator=gen, device="cuda").bfloat16()
        res = {}
        for impl in ("ours", "cublas"):
            def run(w):
                if impl == "ours":
                    return ops.decode_gemm(x, w, silu_mul=silu)
                y = torch.nn.functional.linear(x, w)
                return ops.silu_mul(y) if silu else y
            for w in ws:
                run(w)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for w in ws:
                    run(w)
            for _ in range(max(args.warmup, 1)):
                g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = max(args.steps, 1)
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
            res[impl] = {"us": us, "gbs": nbytes / us / 1e3}
            del g
        rows.append({"name": name, "n_rows": n, "k": k, "weight_bytes": nbytes,
                     "plan": ops.decode_gemm_plan(n, k, silu), "ours": res["ours"], "cublas": res["cublas"]})
        del ws
        torch.cuda.empty_cache()
    print(json.dumps({"workload": "decode_gemm", "m": 8, "steps": args.steps, "shapes": rows}), flush=True)


def main():
    args = parse()
    if args.steps is None:
        args.steps = max(E2E8B["decode_tokens"] - args.warmup, 1) if args.workload == "e2e8b" else 100
    if args.case == "small":
        CFG.update(SMALL)
        E2E8B.update(E2E8B_SMALL)
    if args.e2e_layers:
        E2E8B["layers"] = args.e2e_layers
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cp128k":
        run_cp(args)
    elif args.workload == "e2e8b":
        run_e2e8b(args)
    elif args.workload == "decode_gemm":
        run_decode_gemm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
