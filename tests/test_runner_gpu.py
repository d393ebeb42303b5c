"""CUDA-graph decode runner == eager greedy decoding on the same model and kernels,
across chunk boundaries (commits between replays), batch 2."""

import numpy as np
import pytest
import torch

from tests.test_hf_model_gpu import build_small

pytestmark = pytest.mark.gpu


def test_graph_decode_matches_eager_generation(small_d128):
    from lastkv_b200.runner import GraphDecodeRunner

    model = build_small(small_d128, fused=True)  # the graph path the 8B bench runs
    prompt = torch.from_numpy(small_d128["tokens"][:, :21]).cuda()
    steps = 40  # from position 21 past the boundaries at 32, 48 and 64 (chunk 16)
    eager = model.generate_greedy(prompt, steps).cpu().numpy()
    cache = model.new_cache(2, 21 + steps + 1)
    runner = GraphDecodeRunner(model, cache)
    with torch.no_grad():
        runner.prefill(prompt, 21)  # the same chunk pieces as generate_greedy
        first = runner.ids.clone()
        runner.capture()
        out = [first]
        for _ in range(steps - 1):
            out.append(runner.step().clone())
    cache.check_errors()
    got = torch.cat(out, 1).cpu().numpy()
    np.testing.assert_array_equal(got, eager[:, 21:])
