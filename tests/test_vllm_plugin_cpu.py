"""The reference's vLLM backend surface (``lastkv_b200.vllm_plugin``) against fake runtimes.

vLLM 0.25 / FlashInfer 0.6.13 (the reference's pins) are not installable here,
so - as the reference's ``importer=`` / ``version_getter=`` injection intends -
fake modules stand in for ``vllm.v1.attention.backends.registry``,
``vllm.v1.attention.backends.flashinfer`` and ``vllm.v1.attention.backend``
with the pinned signatures, and a recording stand-in plays the fast path.
"""

import types

import pytest
import torch


def _fake_runtime(*, forward_params=None, has_custom=True, config=None):
    registered = {}

    class Custom:
        def is_overridden(self):
            return "path" in registered

        def get_path(self):
            return registered.get("path")

    def register_backend(backend, class_path, is_mamba=False):
        registered["path"] = class_path
        registered["backend"] = backend

    registry = types.SimpleNamespace(register_backend=register_backend,
                                     AttentionBackendEnum=types.SimpleNamespace(CUSTOM=Custom() if has_custom else None))

    class FlashInferBackend:
        @staticmethod
        def get_builder_cls():
            return object

        @staticmethod
        def get_impl_cls():
            return object

        @staticmethod
        def get_kv_cache_shape(*a):
            return ()

        @staticmethod
        def get_kv_cache_stride_order():
            return ()

    class FlashInferImpl:
        def __init__(self, num_heads, head_size, scale, num_kv_heads, alibi_slopes, sliding_window, kv_cache_dtype,
                     logits_soft_cap, attn_type, kv_sharing_target_layer_name, sinks):
            self.num_heads, self.head_size = num_heads, head_size

        def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                    output_block_scale=None):
            raise AssertionError("the base forward must not run")

    if forward_params is not None:
        FlashInferImpl.forward = forward_params
    cfg = config if config is not None else types.SimpleNamespace(
        model_config=types.SimpleNamespace(hf_config=types.SimpleNamespace(chunk_size=16)))
    flashinfer = types.SimpleNamespace(FlashInferBackend=FlashInferBackend, FlashInferImpl=FlashInferImpl,
                                       get_current_vllm_config_or_none=lambda: cfg)

    class AttentionMetadataBuilder:
        def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
            pass

    api = types.SimpleNamespace(AttentionMetadataBuilder=AttentionMetadataBuilder,
                                AttentionCGSupport=types.SimpleNamespace(UNIFORM_SINGLE_TOKEN_DECODE="uniform",
                                                                         NEVER="never"))
    modules = {"vllm.v1.attention.backends.registry": registry, "vllm.v1.attention.backends.flashinfer": flashinfer,
               "vllm.v1.attention.backend": api, "torch": torch}
    return modules.__getitem__, registered


def _versions(vllm="0.25.0", fi="0.6.13"):
    return {"vllm": vllm, "flashinfer-python": fi}.__getitem__


@pytest.fixture(autouse=True)
def _fresh_module_state():
    from lastkv_b200 import vllm_plugin

    vllm_plugin._LEAN_BUILDER = None
    vllm_plugin._RUNTIME_TYPES = None
    vllm_plugin.uninstall_fast_path()
    yield
    vllm_plugin._LEAN_BUILDER = None
    vllm_plugin.uninstall_fast_path()


def test_validate_runtime_api_accepts_the_pins_and_rejects_drift():
    from lastkv_b200.vllm_plugin import RMarinVllmCompatibilityError, validate_vllm_runtime_api

    importer, _ = _fake_runtime()
    ev = validate_vllm_runtime_api(importer=importer, version_getter=_versions("0.25.0+cu129"))
    assert ev.vllm_version == "0.25.0+cu129" and ev.register_backend_parameters == ("backend", "class_path",
                                                                                      "is_mamba")
    with pytest.raises(RMarinVllmCompatibilityError, match="pinned to vLLM 0.25.0"):
        validate_vllm_runtime_api(importer=importer, version_getter=_versions("0.22.0"))
    with pytest.raises(RMarinVllmCompatibilityError, match="flashinfer-python 0.6.13"):
        validate_vllm_runtime_api(importer=importer, version_getter=_versions(fi="0.6.11"))

    def new_forward(self, layer, query, key, value, kv_cache, attn_metadata, output):
        pass

    importer2, _ = _fake_runtime(forward_params=new_forward)
    with pytest.raises(RMarinVllmCompatibilityError, match="signature changed"):
        validate_vllm_runtime_api(importer=importer2, version_getter=_versions())
    importer3, _ = _fake_runtime(has_custom=False)
    with pytest.raises(RMarinVllmCompatibilityError, match="CUSTOM is unavailable"):
        validate_vllm_runtime_api(importer=importer3, version_getter=_versions())


class _RecordingFastPath:
    def __init__(self, chunk=16):
        self.pool = types.SimpleNamespace(chunk_size=chunk)
        self.active = False
        self.tokens = 0
        self.calls = []

    def prepare(self, spans, num_reqs_padded=None):
        self.calls.append(("prepare", list(spans), num_reqs_padded))
        self.active = bool(spans)
        self.tokens = sum(s.num_query_tokens for s in spans) if spans else 0
        return self.active

    def prepare_dummy(self, num_reqs):
        self.calls.append(("dummy", num_reqs))
        self.active, self.tokens = True, num_reqs
        return True

    def run_layer(self, layer_index, query, key, value, output):
        self.calls.append(("run_layer", layer_index, tuple(query.shape)))
        output[: self.tokens].fill_(7.0)


def test_backend_types_carry_the_reference_names_and_surface():
    from lastkv_b200.vllm_plugin import BACKEND_CLASS_PATH, build_vllm_backend_types

    importer, _ = _fake_runtime()
    backend, impl = build_vllm_backend_types(importer=importer, version_getter=_versions())
    assert backend.__name__ == "RMarinFlashInferBackend" and impl.__name__ == "RMarinFlashInferImpl"
    assert f"{backend.__module__}.{backend.__name__}" == BACKEND_CLASS_PATH
    assert backend.get_name() == "CUSTOM" and backend.get_impl_cls() is impl
    assert backend.supported_dtypes == [torch.bfloat16] and backend.forward_includes_kv_cache_update
    assert not backend.supports_non_causal() and not backend.supports_sink()
    builder = backend.get_builder_cls()
    assert builder.__name__ == "RMarinLeanMetadataBuilder" and builder._cudagraph_support == "uniform"


def _metadata(q_lens, seq_lens):
    q = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0).tolist()), dtype=torch.int32)
    return types.SimpleNamespace(query_start_loc_cpu=q, seq_lens_cpu=torch.tensor(seq_lens, dtype=torch.int32),
                                 num_reqs=len(q_lens), num_actual_tokens=int(sum(q_lens)), slot_mapping="slots",
                                 max_query_len=max(q_lens))


def test_builder_runs_the_host_prologue_and_the_impl_runs_the_layer():
    from lastkv_b200.vllm_backend import Span
    from lastkv_b200.vllm_plugin import build_vllm_backend_types, install_fast_path

    importer, _ = _fake_runtime()
    backend, impl_cls = build_vllm_backend_types(importer=importer, version_getter=_versions())
    fast = _RecordingFastPath()
    install_fast_path(fast, slot_of_row=lambda i: [5, 2, 9][i])
    builder = backend.get_builder_cls()(None, ["l0"], None, "cpu")
    md = builder.build(0, _metadata([1, 7, 1], [40, 23, 1]))
    assert (md.num_actual_tokens, md.num_decodes, md.num_prefills, md.num_prefill_tokens) == (9, 2, 1, 7)
    assert fast.calls[-1] == ("prepare", [Span(5, 39, 1), Span(2, 16, 7), Span(9, 0, 1)], 3)
    impl = impl_cls(4, 128, 128 ** -0.5, 1, None, None, "auto", None, "decoder", None, None)
    out = torch.full((12, 4 * 128), -1.0)
    layer = types.SimpleNamespace(rmarin_layer_index=3)
    got = impl.forward(layer, torch.zeros(12, 4 * 128), None, None, "ignored", md, out)
    assert got is out and fast.calls[-1] == ("run_layer", 3, (12, 4, 128))
    assert bool((out[:9] == 7.0).all()) and bool((out[9:] == 0.0).all())  # the padded tail is zeroed
    assert bool((impl.forward(layer, None, None, None, None, None, out) == 0).all())  # no metadata: zeros
    with pytest.raises(Exception, match="quantization"):
        impl.forward(layer, None, None, None, None, md, out, output_scale=1.0)
    builder.build_for_cudagraph_capture(_metadata([1, 1], [5, 6]))
    assert fast.calls[-1] == ("dummy", 2)


def test_impl_fails_closed_without_a_prepared_fast_path():
    from lastkv_b200.contract import RMarinBackendContractError
    from lastkv_b200.vllm_plugin import build_vllm_backend_types, install_fast_path

    importer, _ = _fake_runtime()
    _, impl_cls = build_vllm_backend_types(importer=importer, version_getter=_versions())
    impl = impl_cls(4, 128, 0.1, 1, None, None, "auto", None, "decoder", None, None)
    layer = types.SimpleNamespace(rmarin_layer_index=0)
    with pytest.raises(RMarinBackendContractError, match="no fallback"):
        impl.forward(layer, torch.zeros(1, 512), None, None, None, object(), torch.zeros(1, 512))
    install_fast_path(_RecordingFastPath(chunk=32))
    with pytest.raises(RMarinBackendContractError, match="chunk 32"):
        impl_cls(4, 128, 0.1, 1, None, None, "auto", None, "decoder", None, None)
    importer2, _ = _fake_runtime(config=types.SimpleNamespace(model_config=types.SimpleNamespace(hf_config=None)))
    from lastkv_b200 import vllm_plugin

    vllm_plugin.uninstall_fast_path()
    _, impl2 = build_vllm_backend_types(importer=importer2, version_getter=_versions())
    with pytest.raises(RMarinBackendContractError, match="chunk_size"):
        impl2(4, 128, 0.1, 1, None, None, "auto", None, "decoder", None, None)


def test_register_backend_is_idempotent_and_exclusive(monkeypatch):
    from lastkv_b200 import vllm_plugin
    from lastkv_b200.vllm_plugin import (BACKEND_CLASS_PATH, RMarinVllmCompatibilityError,
                                         register_rmarin_attention_backend)

    importer, registered = _fake_runtime()
    register_rmarin_attention_backend(importer=importer, version_getter=_versions())
    assert registered["path"] == BACKEND_CLASS_PATH
    register_rmarin_attention_backend(importer=importer, version_getter=_versions())  # same path: fine
    registered["path"] = "someone.else.Backend"
    with pytest.raises(RMarinVllmCompatibilityError, match="already registered"):
        register_rmarin_attention_backend(importer=importer, version_getter=_versions())
    # the general plugin needs the exclusive selection
    monkeypatch.delenv("VLLM_PLUGINS", raising=False)
    with pytest.raises(RMarinVllmCompatibilityError, match="VLLM_PLUGINS=lastkv"):
        vllm_plugin.vllm_general_plugin()
    monkeypatch.setenv("VLLM_PLUGINS", "lastkv,recurrent_marin")
    with pytest.raises(RMarinVllmCompatibilityError, match="exclusive"):
        vllm_plugin.vllm_general_plugin()


def test_spans_from_metadata_rejects_inconsistent_rows():
    from lastkv_b200.contract import RMarinBackendContractError
    from lastkv_b200.vllm_plugin import spans_from_metadata

    with pytest.raises(RMarinBackendContractError, match="query tokens"):
        spans_from_metadata(_metadata([4], [3]), lambda i: i)
