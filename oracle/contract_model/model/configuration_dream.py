"""DreamConfig for the contract model. Field names and defaults follow
prefilling_dllm_eval/model_cache/dream/configuration_dream.py:30-52. TEST INFRASTRUCTURE (oracle)."""

from __future__ import annotations

import json
import os


class DreamConfig:
    model_type = "Dream"

    def __init__(self, vocab_size=151936, hidden_size=4096, intermediate_size=22016, num_hidden_layers=32,
                 num_attention_heads=32, num_key_value_heads=None, hidden_act="silu", max_position_embeddings=32768,
                 initializer_range=0.02, rms_norm_eps=1e-6, tie_word_embeddings=False, rope_theta=10000.0,
                 rope_scaling=None, attention_dropout=0.0, mask_token_id=151666, pad_token_id=151643,
                 bos_token_id=None, eos_token_id=None, torch_dtype="float32", **kwargs):
        self.vocab_size = vocab_size
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_hidden_layers = num_hidden_layers
        self.num_attention_heads = num_attention_heads
        self.num_key_value_heads = num_key_value_heads if num_key_value_heads is not None else num_attention_heads
        self.hidden_act = hidden_act
        self.max_position_embeddings = max_position_embeddings
        self.initializer_range = initializer_range
        self.rms_norm_eps = rms_norm_eps
        self.tie_word_embeddings = tie_word_embeddings
        self.rope_theta = rope_theta
        self.rope_scaling = rope_scaling
        self.attention_dropout = attention_dropout
        self.mask_token_id = mask_token_id
        self.pad_token_id = pad_token_id
        self.bos_token_id = bos_token_id
        self.eos_token_id = eos_token_id
        self.torch_dtype = torch_dtype
        self.output_attentions = False
        self.output_hidden_states = False
        self.use_return_dict = True
        self.use_cache = False
        for key, value in kwargs.items():
            setattr(self, key, value)

    @classmethod
    def from_pretrained(cls, path, **kwargs):
        with open(os.path.join(path, "config.json")) as handle:
            data = json.load(handle)
        data.pop("model_type", None)
        data.pop("architectures", None)
        data.update(kwargs)
        return cls(**data)

    def to_dict(self):
        return {k: v for k, v in self.__dict__.items() if not k.startswith("_")}
