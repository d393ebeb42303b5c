"""The history the merged form attends to, against the reference's own executable
history oracle (vllm/src/lastkv/vllm/backends/rmarin_flashinfer/reference.py:342-439,
resolve_reference_history; recorded in tests/golden/reference_history.npz by
tests/golden/make_golden.py): older tokens = the top layer's raw K with V x s_l,
the completed chunk = alpha-blend of that scaled source with the layer's own K/V,
the current chunk = the layer's own K/V.

Checked two ways: the HF composition of the oracle (``hf_history``, fp32 like the
reference HF model) within fp32 rounding, and the merged paged form's storage -
shared pages hold raw K/V, rings hold K and V / s_l (the blend taken in those
units), the attention output is multiplied by s_l - whose effective history must
equal the reference's to float64 rounding."""

import os

import numpy as np

from conftest import ROOT
from oracle import lastkv_oracle as O

GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_history.npz")


def _cases():
    data = np.load(GOLDEN)
    for i in range(int(data["n"])):
        yield {k: data[f"c{i}_{k}"] for k in ("meta", "raw_k", "raw_v", "loc_k", "loc_v", "logits", "scales",
                                             "eff_k", "eff_v")}


def _split(c):
    chunk, pos, top = (int(v) for v in c["meta"])
    cur = (pos // chunk) * chunk
    rec = max(0, cur - chunk)
    return chunk, pos, top, cur, rec


def test_fixture_spans_first_chunk_boundaries_and_both_layer_kinds():
    metas = [tuple(int(v) for v in c["meta"]) for c in _cases()]
    assert len(metas) >= 12
    assert {m[2] for m in metas} == {0, 1}
    assert any(m[1] < m[0] for m in metas) and any(m[1] >= 2 * m[0] for m in metas)


def test_hf_composition_matches_reference_history():
    for c in _cases():
        chunk, pos, top, cur, rec = _split(c)
        t = lambda x: np.ascontiguousarray(np.transpose(x, (1, 0, 2))).astype(np.float32)  # [Hkv, T, D]
        deep_k = t(c["raw_k"][:cur]) if cur else None
        deep_v = t(c["raw_v"][:cur]) if cur else None
        prev_k = t(c["loc_k"][: cur - rec]) if cur else None
        prev_v = t(c["loc_v"][: cur - rec]) if cur else None
        k, v = O.hf_history(deep_k, deep_v, prev_k, prev_v, t(c["loc_k"][cur - rec:]), t(c["loc_v"][cur - rec:]),
                            c["logits"].astype(np.float32), c["scales"].astype(np.float32), chunk)
        np.testing.assert_allclose(np.transpose(k, (1, 0, 2)), c["eff_k"], rtol=2e-6, atol=2e-6)
        np.testing.assert_allclose(np.transpose(v, (1, 0, 2)), c["eff_v"], rtol=2e-6, atol=2e-6)


def test_merged_storage_reproduces_reference_history():
    for c in _cases():
        chunk, pos, top, cur, rec = _split(c)
        s = c["scales"][None, :, None]
        a = 1.0 / (1.0 + np.exp(-c["logits"]))[None, :, None]
        # pool contents: shared pages raw; the layer ring K and V / s, the finished chunk blended in those units
        ring_k = c["loc_k"].copy()
        ring_v = c["loc_v"] / s
        n_recent = cur - rec
        ring_k[:n_recent] = a * c["raw_k"][rec:cur] + (1 - a) * ring_k[:n_recent]
        ring_v[:n_recent] = a * c["raw_v"][rec:cur] + (1 - a) * ring_v[:n_recent]
        keys = np.concatenate([c["raw_k"][:rec], ring_k])
        vals = np.concatenate([c["raw_v"][:rec], ring_v]) * s  # the output's x s_l
        np.testing.assert_allclose(keys, c["eff_k"], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(vals, c["eff_v"], rtol=1e-12, atol=1e-12)
