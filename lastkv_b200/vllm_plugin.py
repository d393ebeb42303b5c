"""The reference's vLLM backend surface, bound to the B200 fast path.

Drop-in for the entry points of
vllm/src/lastkv/vllm/backends/rmarin_flashinfer/vllm_backend.py and
vllm_plugin.py, with the same names, arguments and fail-closed behaviour:

* ``validate_vllm_runtime_api(importer=, version_getter=)`` - the pinned
  vLLM / FlashInfer versions and the signatures this backend binds
  (vllm_backend.py:141-239);
* ``build_vllm_backend_types(importer=, version_getter=)`` -> the
  ``RMarinFlashInferBackend`` / ``RMarinFlashInferImpl`` classes (subclasses
  of vLLM's FlashInfer backend and impl, whose placeholder KV cache vLLM still
  allocates) (vllm_backend.py:592-758); ``get_builder_cls`` returns the lean
  metadata builder (vllm_backend.py:499-589), whose ``build`` runs this
  package's host prologue (``SharedKVFastPath.prepare``, or ``prepare_dummy``
  for warm-up and CUDA-graph capture) once per step, and the impl's
  ``forward`` runs ``SharedKVFastPath.run_layer`` - the fused append kernel
  and the split-KV decode / tcgen05 prefill kernels on the merged pool;
* the module attributes ``RMarinFlashInferBackend`` / ``RMarinFlashInferImpl``
  resolve lazily (vLLM imports backends by class path);
* ``register_rmarin_attention_backend`` / ``vllm_general_plugin`` - register
  ``AttentionBackendEnum.CUSTOM`` to this module's class path
  (vllm_plugin.py:19-94).

The engine's model adapter installs the fast path with ``install_fast_path``
(the reference's ``fastpath.install``, fastpath.py:848-857), giving the
mapping from scheduled rows to session slots.  Nothing here imports vLLM or
FlashInfer at import time; every runtime collaborator comes through
``importer``, so the contract is testable with fakes on the host.
"""

from __future__ import annotations

import inspect
import os
from collections.abc import Callable
from dataclasses import dataclass
from importlib import import_module
from typing import Any

from .contract import RMarinBackendContractError
from .vllm_backend import SharedKVFastPath, Span

PINNED_VLLM_VERSION = "0.25.0"  # runtime_contract.py:27
PINNED_FLASHINFER_VERSION = "0.6.13"  # runtime_contract.py:29
BACKEND_CLASS_PATH = "lastkv_b200.vllm_plugin.RMarinFlashInferBackend"

_REGISTRY_MODULE = "vllm.v1.attention.backends.registry"
_FLASHINFER_BACKEND_MODULE = "vllm.v1.attention.backends.flashinfer"
_BACKEND_API_MODULE = "vllm.v1.attention.backend"

# The callables this backend binds, by parameter name (vllm_backend.py:56-80).
_EXPECTED_REGISTER_PARAMETERS = ("backend", "class_path", "is_mamba")
_EXPECTED_IMPL_INIT_PARAMETERS = ("self", "num_heads", "head_size", "scale", "num_kv_heads", "alibi_slopes",
                                  "sliding_window", "kv_cache_dtype", "logits_soft_cap", "attn_type",
                                  "kv_sharing_target_layer_name", "sinks")
_EXPECTED_IMPL_FORWARD_PARAMETERS = ("self", "layer", "query", "key", "value", "kv_cache", "attn_metadata",
                                     "output", "output_scale", "output_block_scale")


class RMarinVllmCompatibilityError(RMarinBackendContractError):
    """The installed runtime differs from the pinned, audited API."""


@dataclass(frozen=True)
class VllmRuntimeApiEvidence:
    """Runtime identity and the signatures that were checked."""

    vllm_version: str
    flashinfer_version: str
    register_backend_parameters: tuple[str, ...]
    impl_init_parameters: tuple[str, ...]
    impl_forward_parameters: tuple[str, ...]


def _public(version: str, label: str) -> str:
    if not isinstance(version, str) or not version:
        raise RMarinVllmCompatibilityError(f"{label} version is missing")
    return version.split("+", 1)[0]


def _params(fn: Any, label: str) -> tuple[str, ...]:
    try:
        return tuple(inspect.signature(fn).parameters)
    except (TypeError, ValueError) as error:
        raise RMarinVllmCompatibilityError(f"cannot inspect the pinned {label} API; rebuild the integration "
                                           "against the deployed runtime") from error


def _require(fn: Any, expected: tuple[str, ...], label: str) -> tuple[str, ...]:
    seen = _params(fn, label)
    if seen != expected:
        raise RMarinVllmCompatibilityError(f"{label} signature changed: expected {expected}, observed {seen}. "
                                           "Re-pin and validate the backend before use.")
    return seen


def validate_vllm_runtime_api(*, importer: Callable[[str], Any] = import_module,
                              version_getter: Callable[[str], str] | None = None) -> VllmRuntimeApiEvidence:
    """Fail closed unless the runtime is the pinned vLLM / FlashInfer with the bound API."""
    if version_getter is None:
        from importlib.metadata import version as version_getter
    vllm_version = version_getter("vllm")
    fi_version = version_getter("flashinfer-python")
    if _public(vllm_version, "vLLM") != PINNED_VLLM_VERSION:
        raise RMarinVllmCompatibilityError(f"the B200 RMarin backend is pinned to vLLM {PINNED_VLLM_VERSION}, "
                                           f"observed {vllm_version!r}")
    if _public(fi_version, "FlashInfer") != PINNED_FLASHINFER_VERSION:
        raise RMarinVllmCompatibilityError(f"the B200 RMarin backend is pinned to flashinfer-python "
                                           f"{PINNED_FLASHINFER_VERSION}, observed {fi_version!r}")
    registry = importer(_REGISTRY_MODULE)
    backend_module = importer(_FLASHINFER_BACKEND_MODULE)
    try:
        register_backend = registry.register_backend
        custom = registry.AttentionBackendEnum.CUSTOM
        backend_class = backend_module.FlashInferBackend
        impl_class = backend_module.FlashInferImpl
    except AttributeError as error:
        raise RMarinVllmCompatibilityError("the vLLM attention API is missing a pinned symbol; rebuild the "
                                           "integration against the deployed runtime") from error
    reg = _require(register_backend, _EXPECTED_REGISTER_PARAMETERS, "vLLM register_backend")
    init = _require(impl_class.__init__, _EXPECTED_IMPL_INIT_PARAMETERS, "vLLM FlashInferImpl.__init__")
    fwd = _require(impl_class.forward, _EXPECTED_IMPL_FORWARD_PARAMETERS, "vLLM FlashInferImpl.forward")
    for name in ("get_builder_cls", "get_impl_cls", "get_kv_cache_shape", "get_kv_cache_stride_order"):
        if not callable(getattr(backend_class, name, None)):
            raise RMarinVllmCompatibilityError(f"vLLM FlashInferBackend.{name} is unavailable; re-pin and "
                                               "validate the backend")
    if custom is None:
        raise RMarinVllmCompatibilityError("vLLM AttentionBackendEnum.CUSTOM is unavailable")
    return VllmRuntimeApiEvidence(vllm_version, fi_version, reg, init, fwd)


# ---------------------------------------------------------------------- the installed fast path


@dataclass
class _Installed:
    fast: SharedKVFastPath
    slot_of_row: Callable[[int], int]


_INSTALLED: _Installed | None = None


def install_fast_path(fast: SharedKVFastPath, *, slot_of_row: Callable[[int], int] | None = None) -> SharedKVFastPath:
    """Make ``fast`` the fast path the backend's builder and impl use (``fastpath.install``).
    ``slot_of_row(i)``: the session slot of the i-th scheduled request of a step (identity
    by default)."""
    global _INSTALLED
    _INSTALLED = _Installed(fast, slot_of_row or (lambda i: i))
    return fast


def uninstall_fast_path() -> None:
    global _INSTALLED
    _INSTALLED = None


def current_fast_path() -> SharedKVFastPath | None:
    """The installed fast path (``fastpath.current``), or None."""
    return _INSTALLED.fast if _INSTALLED is not None else None


def spans_from_metadata(common_attn_metadata: Any, slot_of_row: Callable[[int], int]) -> list[Span]:
    """The step's per-request spans from vLLM's common attention metadata: query lengths from
    ``query_start_loc_cpu``, total lengths from ``seq_lens_cpu`` (computed = total - query)."""
    q = common_attn_metadata.query_start_loc_cpu
    seq = common_attn_metadata.seq_lens_cpu
    n = int(common_attn_metadata.num_reqs)
    spans = []
    for i in range(n):
        lq = int(q[i + 1]) - int(q[i])
        total = int(seq[i])
        if lq < 1 or total < lq:
            raise RMarinBackendContractError(f"request row {i}: {lq} query tokens of {total}")
        spans.append(Span(slot=int(slot_of_row(i)), num_computed_tokens=total - lq, num_query_tokens=lq))
    return spans


# ---------------------------------------------------------------------- lean metadata and builder


class RMarinLeanMetadata:
    """Per-step attention metadata the impl reads (token accounting and slot mapping only;
    vllm_backend.py:457-496)."""

    __slots__ = ("num_actual_tokens", "slot_mapping", "causal", "use_cascade", "num_decode_tokens",
                 "num_prefill_tokens", "num_decodes", "num_prefills", "num_reqs", "query_start_loc_cpu")

    def __init__(self, *, num_actual_tokens, slot_mapping, num_decode_tokens, num_prefill_tokens, num_decodes,
                 num_prefills, num_reqs, query_start_loc_cpu):
        self.num_actual_tokens = num_actual_tokens
        self.slot_mapping = slot_mapping
        self.causal = True
        self.use_cascade = False
        self.num_decode_tokens = num_decode_tokens
        self.num_prefill_tokens = num_prefill_tokens
        self.num_decodes = num_decodes
        self.num_prefills = num_prefills
        self.num_reqs = num_reqs
        self.query_start_loc_cpu = query_start_loc_cpu


_LEAN_BUILDER: type | None = None


def build_lean_metadata_builder_type(importer: Callable[[str], Any] = import_module) -> type:
    """The metadata builder: no FlashInfer wrapper planning (the B200 kernels ignore vLLM's
    placeholder cache); its ``build`` runs the fast path's host prologue for the step."""
    global _LEAN_BUILDER
    if _LEAN_BUILDER is not None:
        return _LEAN_BUILDER
    api = importer(_BACKEND_API_MODULE)
    base, cg = api.AttentionMetadataBuilder, api.AttentionCGSupport

    class RMarinLeanMetadataBuilder(base):
        # every step's per-layer ops read device buffers only: uniform decode steps replay in graphs
        _cudagraph_support = cg.UNIFORM_SINGLE_TOKEN_DECODE
        reorder_batch_threshold = 1

        def __init__(self, kv_cache_spec: Any, layer_names: Any, vllm_config: Any, device: Any) -> None:
            try:
                super().__init__(kv_cache_spec, layer_names, vllm_config, device)
            except TypeError:
                pass
            self.kv_cache_spec, self.layer_names = kv_cache_spec, layer_names
            self.vllm_config, self.device = vllm_config, device
            self._capture = False

        def _prologue(self, common_attn_metadata: Any, num_reqs: int) -> None:
            inst = _INSTALLED
            if inst is None:
                return
            if self._capture:
                inst.fast.prepare_dummy(num_reqs)
                return
            spans = spans_from_metadata(common_attn_metadata, inst.slot_of_row)
            if not inst.fast.prepare(spans, num_reqs):
                inst.fast.prepare_dummy(num_reqs)

        def build(self, common_prefix_len: int, common_attn_metadata: Any,
                  fast_build: bool = False) -> RMarinLeanMetadata:
            q = common_attn_metadata.query_start_loc_cpu
            num_reqs = int(common_attn_metadata.num_reqs)
            lens = [int(q[i + 1]) - int(q[i]) for i in range(num_reqs)]
            decodes = sum(1 for n in lens if n == 1)
            total = int(common_attn_metadata.num_actual_tokens)
            self._prologue(common_attn_metadata, num_reqs)
            return RMarinLeanMetadata(num_actual_tokens=total, slot_mapping=common_attn_metadata.slot_mapping,
                                      num_decode_tokens=decodes, num_prefill_tokens=total - decodes,
                                      num_decodes=decodes, num_prefills=num_reqs - decodes, num_reqs=num_reqs,
                                      query_start_loc_cpu=q)

        def build_for_cudagraph_capture(self, common_attn_metadata: Any) -> RMarinLeanMetadata:
            self._capture = True
            try:
                return self.build(0, common_attn_metadata)
            finally:
                self._capture = False

    RMarinLeanMetadataBuilder.__module__ = __name__
    _LEAN_BUILDER = RMarinLeanMetadataBuilder
    return RMarinLeanMetadataBuilder


# ---------------------------------------------------------------------- backend and impl


def build_vllm_backend_types(*, importer: Callable[[str], Any] = import_module,
                             version_getter: Callable[[str], str] | None = None) -> tuple[type, type]:
    """``(RMarinFlashInferBackend, RMarinFlashInferImpl)`` after validating the pinned runtime."""
    validate_vllm_runtime_api(importer=importer, version_getter=version_getter)
    backend_module = importer(_FLASHINFER_BACKEND_MODULE)
    torch = importer("torch")
    base_backend, base_impl = backend_module.FlashInferBackend, backend_module.FlashInferImpl
    get_config = getattr(backend_module, "get_current_vllm_config_or_none", None)
    if not callable(get_config):
        raise RMarinVllmCompatibilityError("vLLM does not expose the pinned current-config accessor needed for "
                                           "fail-closed runtime validation")

    class RMarinFlashInferImpl(base_impl):
        """vLLM AttentionImpl running each layer on the installed B200 fast path."""

        can_return_lse_for_decode = False

        def __init__(self, *args: Any, **kwargs: Any) -> None:
            super().__init__(*args, **kwargs)
            vllm_config = get_config()
            if vllm_config is None:
                raise RMarinBackendContractError("RMarin attention was constructed outside vLLM's config context")
            hf = getattr(getattr(vllm_config, "model_config", None), "hf_config", None)
            chunk = getattr(hf, "chunk_size", None)
            if chunk is None:
                raise RMarinBackendContractError("vLLM RMarin model config has no recurrent chunk_size")
            fast = current_fast_path()
            if fast is not None and fast.pool.chunk_size != chunk:
                raise RMarinBackendContractError(f"the installed pool uses chunk {fast.pool.chunk_size}, the model "
                                                 f"{chunk}")
            self.rmarin_vllm_config = vllm_config

        def forward(self, layer: Any, query: Any, key: Any, value: Any, kv_cache: Any, attn_metadata: Any,
                    output: Any, output_scale: Any | None = None, output_block_scale: Any | None = None) -> Any:
            del kv_cache  # the merged shared-KV pool belongs to the fast path
            if attn_metadata is None:
                return output.fill_(0)
            if output_scale is not None or output_block_scale is not None:
                raise RMarinBackendContractError("fused output quantization is not supported")
            fast = current_fast_path()
            if fast is None or not fast.active:
                raise RMarinBackendContractError("the B200 fast path was not installed or not prepared for this "
                                                 "step; there is no fallback attention")
            out = output.view(-1, self.num_heads, self.head_size)
            fast.run_layer(int(layer.rmarin_layer_index), query.view(-1, self.num_heads, self.head_size), key,
                           value, out)
            if int(output.shape[0]) > fast.tokens:
                output[fast.tokens:].fill_(0)
            return output

    class RMarinFlashInferBackend(base_backend):
        """vLLM CUSTOM attention backend on the shared last-layer KV pool (B200 kernels)."""

        supported_dtypes = [torch.bfloat16]
        supported_kv_cache_dtypes = ["auto", "bfloat16"]
        forward_includes_kv_cache_update = True  # the fused append writes the pool

        @staticmethod
        def get_name() -> str:
            return "CUSTOM"

        @staticmethod
        def get_impl_cls() -> type:
            return RMarinFlashInferImpl

        @staticmethod
        def get_builder_cls() -> type:
            return build_lean_metadata_builder_type(importer)

        @classmethod
        def supports_non_causal(cls) -> bool:
            return False

        @classmethod
        def supports_sink(cls) -> bool:
            return False

    for cls in (RMarinFlashInferImpl, RMarinFlashInferBackend):
        cls.__module__ = __name__
    return RMarinFlashInferBackend, RMarinFlashInferImpl


_RUNTIME_TYPES: tuple[type, type] | None = None


def __getattr__(name: str) -> Any:
    """Resolve the class-path targets lazily (vLLM imports ``BACKEND_CLASS_PATH``)."""
    global _RUNTIME_TYPES
    if name in ("RMarinFlashInferBackend", "RMarinFlashInferImpl"):
        if _RUNTIME_TYPES is None:
            _RUNTIME_TYPES = build_vllm_backend_types()
        return _RUNTIME_TYPES[0 if name == "RMarinFlashInferBackend" else 1]
    raise AttributeError(name)


# ---------------------------------------------------------------------- plugin


def register_rmarin_attention_backend(*, importer: Callable[[str], Any] = import_module,
                                      version_getter: Callable[[str], str] | None = None
                                      ) -> VllmRuntimeApiEvidence:
    """Register ``AttentionBackendEnum.CUSTOM`` to this module's backend through vLLM's public
    API; idempotent for this class path, and an error if another backend holds CUSTOM."""
    evidence = validate_vllm_runtime_api(importer=importer, version_getter=version_getter)
    registry = importer(_REGISTRY_MODULE)
    custom = registry.AttentionBackendEnum.CUSTOM
    is_overridden = getattr(custom, "is_overridden", None)
    get_path = getattr(custom, "get_path", None)
    if callable(is_overridden) and is_overridden():
        if not callable(get_path):
            raise RMarinVllmCompatibilityError("vLLM CUSTOM backend is already registered but its class path "
                                               "cannot be inspected")
        seen = get_path()
        if seen != BACKEND_CLASS_PATH:
            raise RMarinVllmCompatibilityError(f"vLLM CUSTOM attention backend is already registered as {seen!r}; "
                                               f"this backend requires {BACKEND_CLASS_PATH!r}")
        return evidence
    registry.register_backend(custom, BACKEND_CLASS_PATH, is_mamba=False)
    if callable(get_path) and get_path() != BACKEND_CLASS_PATH:
        raise RMarinVllmCompatibilityError("vLLM did not retain the registered backend class path")
    return evidence


def vllm_general_plugin() -> None:
    """``vllm.general_plugins`` entry point: requires the exclusive selection VLLM_PLUGINS=lastkv
    (so no other plugin silently owns the CUSTOM backend) and registers the backend.  The
    RMarin model class itself is registered by the reference's model package."""
    configured = os.environ.get("VLLM_PLUGINS")
    selected = {x.strip() for x in configured.split(",") if x.strip()} if configured is not None else set()
    if selected != {"lastkv"}:
        raise RMarinVllmCompatibilityError(f"the RMarin backend requires the exclusive plugin selection "
                                           f"VLLM_PLUGINS=lastkv; observed {configured!r}")
    register_rmarin_attention_backend()


__all__ = ["BACKEND_CLASS_PATH", "PINNED_FLASHINFER_VERSION", "PINNED_VLLM_VERSION", "RMarinLeanMetadata",
           "RMarinVllmCompatibilityError", "VllmRuntimeApiEvidence", "build_lean_metadata_builder_type",
           "build_vllm_backend_types", "current_fast_path", "install_fast_path", "register_rmarin_attention_backend",
           "spans_from_metadata", "uninstall_fast_path", "validate_vllm_runtime_api", "vllm_general_plugin"]
