"""The reference's Hugging Face model surface on the B200 kernels.

Drop-in for ``lastkv.llm`` (llm/src/lastkv/llm/__init__.py,
configuration.py, modeling.py): the same class names, config fields and
validation, state-dict names (strict loading), ``forward`` arguments and
``GenerationMixin`` hooks, so ``model.generate(ids, max_new_tokens=...,
do_sample=False, use_cache=True)`` and ``load_model(...)`` call sites work
unchanged.  The module tree is ``lastkv_b200.hf`` (fused RoPE / norm / append
kernel, split-KV decode and tcgen05 prefill kernels on a bf16 paged cache, or
the fp32 kernels on an fp32 cache for fp32 models); the cache returned in
``past_key_values`` is a ``PagedLastKVCache`` (``get_seq_length``,
``reorder_cache``, ``seen_tokens`` as the reference's ``LastKVCache``), created
on the first call and grown as generation proceeds.

Importing this module registers the config and model with transformers'
``AutoConfig`` / ``AutoModelForCausalLM``, as the reference's package import
does (llm/src/lastkv/llm/__init__.py:9-10).
"""

from __future__ import annotations

import torch
import transformers
from torch import nn
from transformers import AutoConfig, AutoModelForCausalLM, LlamaConfig, PreTrainedModel
from transformers.generation import GenerationMixin
from transformers.modeling_outputs import CausalLMOutputWithPast

from .hf import LastKVConfig, LastKVModel, PagedLastKVCache, RMSNorm

MODEL_TYPE = "custom_recurrent_marin_akv254_reusekv"
_TRANSFORMERS_MAJOR = int(transformers.__version__.split(".")[0])


class CustomRecurrentMarinAKV254ReuseKVConfig(LlamaConfig):
    """The reference's config (configuration.py:13-48): a Llama config plus the chunk
    recurrence fields, with the same checks and messages (the released checkpoints'
    contract: final-layer KV reuse, learnable V-only deep rescale)."""

    model_type = MODEL_TYPE

    def __init__(self, chunk_size=1024, v_gap=95, use_qk_norm=True, use_nope=False, deep_kv_rescale=True,
                 deep_rescale_mode="v", deep_v_scale_init=1.0, deep_scale_frozen=False, **kwargs):
        kwargs.setdefault("architectures", ["CustomRecurrentMarinAKV254ReuseKVForCausalLM"])
        kwargs.pop("akv254_kv_mode", None)
        backend = kwargs.pop("attn_implementation", None)
        super().__init__(**kwargs)
        if type(chunk_size) is not int or chunk_size < 1:
            raise ValueError("chunk_size must be a positive integer")
        if v_gap is None or v_gap < self.num_hidden_layers - 1:
            raise ValueError("This inference implementation requires final-layer KV reuse")
        if deep_rescale_mode != "v" or deep_scale_frozen:
            raise ValueError("The released checkpoints use learnable deep_rescale_mode='v'")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        self.chunk_size = chunk_size
        self.v_gap = v_gap
        self.use_qk_norm = use_qk_norm
        self.use_nope = use_nope
        self.deep_kv_rescale = deep_kv_rescale
        self.deep_rescale_mode = deep_rescale_mode
        self.deep_v_scale_init = deep_v_scale_init
        self.deep_scale_frozen = deep_scale_frozen
        self.akv254_kv_mode = "reusekv"
        self._attn_implementation = backend if backend in ("eager", "sdpa") else "sdpa"


def lastkv_config(config: CustomRecurrentMarinAKV254ReuseKVConfig) -> LastKVConfig:
    """The fields the B200 module tree reads, from a transformers config (rope theta and
    llama3 scaling from ``rope_parameters`` or the older ``rope_theta``/``rope_scaling``)."""
    rope = getattr(config, "rope_parameters", None) or {}
    theta = rope.get("rope_theta", getattr(config, "rope_theta", None))
    if theta is None:
        theta = 10000.0
    rtype = rope.get("rope_type", rope.get("type"))
    scaling = dict(rope) if rtype == "llama3" else getattr(config, "rope_scaling", None)
    if scaling and scaling.get("rope_type", scaling.get("type")) not in ("llama3",):
        scaling = None
    head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
    return LastKVConfig(hidden_size=config.hidden_size, intermediate_size=config.intermediate_size,
                        num_attention_heads=config.num_attention_heads,
                        num_key_value_heads=config.num_key_value_heads,
                        num_hidden_layers=config.num_hidden_layers, head_dim=head_dim,
                        vocab_size=config.vocab_size, chunk_size=config.chunk_size,
                        rms_norm_eps=config.rms_norm_eps, rope_theta=float(theta), rope_scaling=scaling,
                        max_position_embeddings=config.max_position_embeddings,
                        deep_kv_rescale=config.deep_kv_rescale, deep_v_scale_init=config.deep_v_scale_init,
                        use_qk_norm=config.use_qk_norm, use_nope=config.use_nope,
                        attention_bias=config.attention_bias, tie_word_embeddings=config.tie_word_embeddings,
                        initializer_range=config.initializer_range)


class CustomRecurrentMarinAKV254ReuseKVForCausalLM(PreTrainedModel, GenerationMixin):
    """The reference's causal LM (modeling.py:215-293) with its attention on the B200 kernels."""

    config_class = CustomRecurrentMarinAKV254ReuseKVConfig
    base_model_prefix = "model"
    _supports_sdpa = True
    _no_split_modules = ["LastKVDecoderLayer"]
    # the LM head ties to the embedding when config.tie_word_embeddings (transformers 5 names the
    # target; 4.x, the reference's pin, takes the list form)
    _tied_weights_keys = ({"lm_head.weight": "model.embed_tokens.weight"} if _TRANSFORMERS_MAJOR >= 5
                          else ["lm_head.weight"])

    def __init__(self, config):
        super().__init__(config)
        self.model = LastKVModel(lastkv_config(config))
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.post_init()

    def _init_weights(self, module):
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=self.config.initializer_range)
            if isinstance(module, nn.Linear) and module.bias is not None:
                nn.init.zeros_(module.bias)
            if isinstance(module, nn.Embedding) and module.padding_idx is not None:
                module.weight.data[module.padding_idx].zero_()
        elif isinstance(module, RMSNorm):
            nn.init.ones_(module.weight)

    @classmethod
    def _supports_default_dynamic_cache(cls):
        return False  # generate() must pass back the PagedLastKVCache this model returns

    @classmethod
    def from_pretrained(cls, *args, **kwargs):
        """Strict loading: any missing, unexpected or mismatched tensor is an error (modeling.py:243-249)."""
        wants_info = kwargs.pop("output_loading_info", False)
        model, info = super().from_pretrained(*args, output_loading_info=True, **kwargs)
        problems = {key: info[key] for key in ("missing_keys", "unexpected_keys", "mismatched_keys", "error_msgs")
                    if info.get(key)}
        if problems:
            raise ValueError(f"Checkpoint is not a strict LastKV model match: {problems}")
        model.model._alpha = None
        return (model, info) if wants_info else model

    def get_input_embeddings(self):
        return self.model.embed_tokens

    def set_input_embeddings(self, value):
        self.model.embed_tokens = value

    def get_output_embeddings(self):
        return self.lm_head

    def set_output_embeddings(self, value):
        self.lm_head = value

    def prepare_inputs_for_generation(self, input_ids, past_key_values=None, attention_mask=None,
                                      inputs_embeds=None, use_cache=True, position_ids=None, **kwargs):
        """Only the tokens the cache has not seen (modeling.py:265-275)."""
        if past_key_values is not None:
            seen = past_key_values.get_seq_length()
            input_ids = input_ids[:, seen:] if input_ids.shape[1] > seen else input_ids[:, -1:]
            inputs_embeds = None
            if position_ids is not None:
                position_ids = position_ids[:, -input_ids.shape[1]:]
        inputs = {"inputs_embeds": inputs_embeds} if inputs_embeds is not None else {"input_ids": input_ids}
        return {**inputs, "past_key_values": past_key_values, "attention_mask": attention_mask,
                "position_ids": position_ids, "use_cache": use_cache, "logits_to_keep": 1}

    def new_cache(self, batch: int, max_tokens: int, **kw) -> PagedLastKVCache:
        """A paged cache for this model (fp32 for an fp32 model, else bf16)."""
        kw.setdefault("dtype", torch.float32 if self.lm_head.weight.dtype == torch.float32 else torch.bfloat16)
        return PagedLastKVCache(self.model.config, batch, max_tokens, device=self.lm_head.weight.device, **kw)

    def forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None,
                inputs_embeds=None, use_cache=None, return_dict=None, logits_to_keep=0, labels=None,
                output_attentions=False, output_hidden_states=False, **kwargs):
        if labels is not None or output_attentions or output_hidden_states:
            raise ValueError("This release provides inference logits and a KV cache only")
        if kwargs.get("cu_seqlens") is not None:
            raise ValueError("Packed-document inputs are unsupported; process each document separately")
        if (input_ids is None) == (inputs_embeds is None):
            raise ValueError("Provide exactly one of input_ids or inputs_embeds")
        if attention_mask is not None and not bool(torch.all(attention_mask != 0)):
            raise ValueError("LastKV supports unpadded sequences; generate each padded prompt separately")
        if past_key_values is not None and not isinstance(past_key_values, PagedLastKVCache):
            raise TypeError("Use a LastKVCache returned by this model, not a standard Llama cache")
        return_dict = self.config.use_return_dict if return_dict is None else return_dict
        use_cache = self.config.use_cache if use_cache is None else use_cache
        batch, length = (input_ids if input_ids is not None else inputs_embeds).shape[:2]
        if not length:
            raise ValueError("At least one new token is required")
        cache = past_key_values
        if cache is None:
            # sized for the call with room to generate; reserve() doubles it when outgrown
            cache = self.new_cache(batch, max(2 * length, length + 256))
        elif cache.batch != batch:
            raise ValueError("Cache batch does not match the input batch")
        need = cache.seen_tokens + length
        if need > cache.max_tokens:
            cache.reserve(max(need, 2 * cache.max_tokens))
        hidden = self.model(input_ids, cache, inputs_embeds=inputs_embeds, position_ids=position_ids)
        indices = slice(-logits_to_keep, None) if isinstance(logits_to_keep, int) else logits_to_keep
        logits = self.lm_head(hidden[:, indices])
        past = cache if use_cache else None
        if return_dict is False:
            return (logits, past)
        return CausalLMOutputWithPast(logits=logits, past_key_values=past)


AutoConfig.register(MODEL_TYPE, CustomRecurrentMarinAKV254ReuseKVConfig, exist_ok=True)
AutoModelForCausalLM.register(CustomRecurrentMarinAKV254ReuseKVConfig, CustomRecurrentMarinAKV254ReuseKVForCausalLM,
                              exist_ok=True)


def load_model(model_name_or_path="ZefanCai/LastKV-LLM-8B-Base", *, revision=None, device="cuda",
               dtype=torch.float32, attention_backend="sdpa"):
    """Strictly load the original HF tensor names and enable cached inference
    (llm/src/lastkv/llm/__init__.py:13-26).  ``attention_backend`` keeps the reference's
    accepted values; attention runs on the B200 kernels either way, in ``dtype``
    (fp32: the fp32 kernels; bf16: the tensor-core kernels).  ``device`` must be a
    CUDA device (there is no CPU path)."""
    if attention_backend not in ("sdpa", "eager"):
        raise ValueError("attention_backend must be 'sdpa' or 'eager'")
    config = CustomRecurrentMarinAKV254ReuseKVConfig.from_pretrained(model_name_or_path, revision=revision)
    config._attn_implementation = attention_backend
    model = CustomRecurrentMarinAKV254ReuseKVForCausalLM.from_pretrained(
        model_name_or_path, revision=revision, config=config, dtype=dtype,
        attn_implementation=attention_backend, use_safetensors=True,
    )
    model.config.use_cache = True
    model.generation_config.use_cache = True
    return model.to(device).eval()


__all__ = ["CustomRecurrentMarinAKV254ReuseKVConfig", "CustomRecurrentMarinAKV254ReuseKVForCausalLM",
           "PagedLastKVCache", "lastkv_config", "load_model"]
