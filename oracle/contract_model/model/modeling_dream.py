"""CPU Dream model that honours the call contract FastDLLMParallelComp expects of Fast-dLLM v1's
`model/modeling_dream.py` (prefilling_dllm_eval/fastdllm_parallelcomp.py:250-365, 702-729, 1154-1164,
2348-2397). TEST INFRASTRUCTURE (oracle): the product never imports it.

Arithmetic restated from the Dream files the reference vendors,
prefilling_dllm_eval/model_cache/dream/model_dream.py: RMSNorm in fp32 (:117-131), rotary cos/sin in fp32 then
cast (:208-236), rotate_half RoPE (:239-264), q/k/v projections with bias and o without (:326-329), GQA by
repeat_kv (:282-291), scores / sqrt(d) + additive mask, softmax in fp32 cast back (:374-383), SwiGLU (:277-278),
pre-norm residual layer (:689-711), final norm + untied lm_head (:945, 1013).

Cache contract (inferred from the reference's call sites, since Fast-dLLM v1 itself is absent): a layer's
past_key_value is (K, V) shaped [B, S, Hkv*D] holding UN-rotated keys; position_ids cover past + current keys and
RoPE is applied after concatenation; with dual_cache the current tokens REPLACE the cache slots flagged by
replace_position and attend the whole cache (later MASK slots included); present = the full (K, V).
"""

from __future__ import annotations

import json
import logging
import math
import os
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .configuration_dream import DreamConfig

logger = logging.getLogger(__name__)
if not hasattr(logger, "warning_once"):
    logger.warning_once = logger.warning  # the reference's patched forward calls logger.warning_once


@dataclass
class BaseModelOutputWithPast:
    last_hidden_state: torch.Tensor = None
    hidden_states: Optional[tuple] = None
    attentions: Optional[tuple] = None
    past_key_values: Optional[list] = None


@dataclass
class MaskedLMOutput:
    logits: torch.Tensor = None
    past_key_values: Optional[list] = None
    hidden_states: Optional[tuple] = None
    attentions: Optional[tuple] = None


class DreamRMSNorm(nn.Module):
    def __init__(self, hidden_size, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, hidden_states):
        input_dtype = hidden_states.dtype
        hidden_states = hidden_states.to(torch.float32)
        variance = hidden_states.pow(2).mean(-1, keepdim=True)
        hidden_states = hidden_states * torch.rsqrt(variance + self.variance_epsilon)
        return self.weight * hidden_states.to(input_dtype)


class DreamRotaryEmbedding(nn.Module):
    """Default (unscaled) rotary table; yarn scaling re-initialises it through __init__(config=...)."""

    def __init__(self, config: DreamConfig = None, **_unused):
        super().__init__()
        self.config = config
        head_dim = config.hidden_size // config.num_attention_heads
        base = float(config.rope_theta)
        inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
        self.attention_scaling = 1.0
        scaling = getattr(config, "rope_scaling", None)
        if scaling and scaling.get("rope_type", scaling.get("type")) == "yarn":
            inv_freq, self.attention_scaling = _yarn_inv_freq(head_dim, base, float(scaling["factor"]),
                                                              int(scaling["original_max_position_embeddings"]))
        self.register_buffer("inv_freq", inv_freq, persistent=False)

    @torch.no_grad()
    def forward(self, x, position_ids):
        inv = self.inv_freq[None, :, None].float().expand(position_ids.shape[0], -1, 1)
        pos = position_ids[:, None, :].float()
        freqs = (inv @ pos).transpose(1, 2)
        emb = torch.cat((freqs, freqs), dim=-1)
        cos = emb.cos() * self.attention_scaling
        sin = emb.sin() * self.attention_scaling
        return cos.to(dtype=x.dtype), sin.to(dtype=x.dtype)


def _yarn_inv_freq(dim, base, factor, original_max, beta_fast=32.0, beta_slow=1.0):
    """Published YaRN frequency blend (Peng et al. 2023), as in transformers' `_compute_yarn_parameters`."""
    pos_freqs = base ** (torch.arange(0, dim, 2).float() / dim)
    extrapolation, interpolation = 1.0 / pos_freqs, 1.0 / (factor * pos_freqs)

    def correction_dim(rot):
        return (dim * math.log(original_max / (rot * 2 * math.pi))) / (2 * math.log(base))

    low = max(math.floor(correction_dim(beta_fast)), 0)
    high = min(math.ceil(correction_dim(beta_slow)), dim - 1)
    if low == high:
        high += 0.001
    ramp = torch.clamp((torch.arange(dim // 2, dtype=torch.float32) - low) / (high - low), 0, 1)
    extrapolation_factor = 1 - ramp
    inv_freq = interpolation * (1 - extrapolation_factor) + extrapolation * extrapolation_factor
    attention_factor = 0.1 * math.log(factor) + 1.0 if factor > 1 else 1.0
    return inv_freq, attention_factor


def rotate_half(x):
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


class DreamMLP(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.gate_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DreamAttention(nn.Module):
    def __init__(self, config: DreamConfig, layer_idx: int):
        super().__init__()
        self.layer_idx = layer_idx
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = self.hidden_size // self.num_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads
        self.q_proj = nn.Linear(self.hidden_size, self.num_heads * self.head_dim, bias=True)
        self.k_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=True)
        self.v_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=True)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, self.hidden_size, bias=False)

    def forward(self, hidden_states, attention_mask=None, position_embeddings=None, past_key_value=None,
                output_attentions=False, use_cache=False, dual_cache=False, replace_position=None):
        bsz, q_len, _ = hidden_states.shape
        q = self.q_proj(hidden_states)
        k_cur = self.k_proj(hidden_states)  # [B, q, Hkv*D], un-rotated: this is what the cache keeps
        v_cur = self.v_proj(hidden_states)

        if past_key_value is not None:
            past_k, past_v = past_key_value
            if dual_cache and replace_position is not None:
                idx = replace_position[0].nonzero(as_tuple=True)[0]
                k_all, v_all = past_k.clone(), past_v.clone()
                k_all[:, idx] = k_cur
                v_all[:, idx] = v_cur
                q_slots = idx
            else:
                k_all = torch.cat([past_k, k_cur], dim=1)
                v_all = torch.cat([past_v, v_cur], dim=1)
                q_slots = torch.arange(k_all.shape[1] - q_len, k_all.shape[1], device=hidden_states.device)
        else:
            k_all, v_all = k_cur, v_cur
            q_slots = torch.arange(q_len, device=hidden_states.device)
        k_len = k_all.shape[1]

        cos, sin = position_embeddings  # [1 or B, k_len, D]: positions of every key, past and current
        if cos.shape[1] != k_len:
            raise ValueError(f"position_ids must cover all {k_len} keys, got {cos.shape[1]}")
        qh = q.view(bsz, q_len, self.num_heads, self.head_dim).transpose(1, 2)
        kh = k_all.view(bsz, k_len, self.num_key_value_heads, self.head_dim).transpose(1, 2)
        vh = v_all.view(bsz, k_len, self.num_key_value_heads, self.head_dim).transpose(1, 2)
        cos_k, sin_k = cos.unsqueeze(1), sin.unsqueeze(1)
        cos_q, sin_q = cos[:, q_slots].unsqueeze(1), sin[:, q_slots].unsqueeze(1)
        qh = (qh * cos_q) + (rotate_half(qh) * sin_q)
        kh = (kh * cos_k) + (rotate_half(kh) * sin_k)

        if self.num_key_value_groups > 1:
            kh = kh[:, :, None].expand(bsz, self.num_key_value_heads, self.num_key_value_groups, k_len, self.head_dim)
            kh = kh.reshape(bsz, self.num_heads, k_len, self.head_dim)
            vh = vh[:, :, None].expand(bsz, self.num_key_value_heads, self.num_key_value_groups, k_len, self.head_dim)
            vh = vh.reshape(bsz, self.num_heads, k_len, self.head_dim)

        attn_weights = torch.matmul(qh, kh.transpose(2, 3)) / math.sqrt(self.head_dim)
        if attention_mask is not None and not isinstance(attention_mask, str):
            attn_weights = attn_weights + attention_mask[:, :, :, :k_len].to(attn_weights.dtype)
        attn_weights = F.softmax(attn_weights, dim=-1, dtype=torch.float32).to(qh.dtype)
        attn_output = torch.matmul(attn_weights, vh)
        attn_output = attn_output.transpose(1, 2).reshape(bsz, q_len, self.hidden_size)
        attn_output = self.o_proj(attn_output)
        present = (k_all, v_all) if use_cache else None
        return attn_output, (attn_weights if output_attentions else None), present


class DreamDecoderLayer(nn.Module):
    def __init__(self, config: DreamConfig, layer_idx: int):
        super().__init__()
        self.self_attn = DreamAttention(config, layer_idx)
        self.mlp = DreamMLP(config)
        self.input_layernorm = DreamRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = DreamRMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, hidden_states, attention_mask=None, position_ids=None, past_key_value=None, output_attentions=False,
                use_cache=False, cache_position=None, position_embeddings=None, dual_cache=False, replace_position=None):
        residual = hidden_states
        hidden_states = self.input_layernorm(hidden_states)
        hidden_states, attn, present = self.self_attn(
            hidden_states, attention_mask=attention_mask, position_embeddings=position_embeddings,
            past_key_value=past_key_value, output_attentions=output_attentions, use_cache=use_cache,
            dual_cache=dual_cache, replace_position=replace_position)
        hidden_states = residual + hidden_states
        residual = hidden_states
        hidden_states = self.post_attention_layernorm(hidden_states)
        hidden_states = self.mlp(hidden_states)
        hidden_states = residual + hidden_states
        outputs = (hidden_states,)
        if output_attentions:
            outputs += (attn,)
        if use_cache:
            outputs += (present,)
        return outputs


class DreamBaseModel(nn.Module):
    def __init__(self, config: DreamConfig):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([DreamDecoderLayer(config, i) for i in range(config.num_hidden_layers)])
        self.norm = DreamRMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.rotary_emb = DreamRotaryEmbedding(config=config)
        self.gradient_checkpointing = False

    def forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None, inputs_embeds=None,
                use_cache=None, output_attentions=None, output_hidden_states=None, return_dict=None, cache_position=None,
                dual_cache=False, replace_position=None):
        """Upstream behaviour (positions regenerated from the cache length); the reference replaces this method with
        its explicit-position forward (fastdllm_parallelcomp.py:236-365), which is the one the hot path runs."""
        use_cache = bool(use_cache)
        hidden = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
        past = past_key_values[0][0].shape[1] if past_key_values is not None else 0
        if position_ids is None:
            n = past if (dual_cache and past_key_values is not None) else past + hidden.shape[1]
            position_ids = torch.arange(n, device=hidden.device).unsqueeze(0)
        pos_emb = self.rotary_emb(hidden, position_ids)
        presents = [] if use_cache else None
        attns = () if output_attentions else None
        for i, layer in enumerate(self.layers):
            out = layer(hidden, attention_mask=attention_mask, position_ids=position_ids,
                        past_key_value=past_key_values[i] if past_key_values is not None else None,
                        output_attentions=bool(output_attentions), use_cache=use_cache, position_embeddings=pos_emb,
                        dual_cache=dual_cache, replace_position=replace_position)
            hidden = out[0]
            if output_attentions:
                attns += (out[1],)
            if use_cache:
                presents.append(out[2 if output_attentions else 1])
        hidden = self.norm(hidden)
        return BaseModelOutputWithPast(last_hidden_state=hidden, attentions=attns, past_key_values=presents)


class DreamModel(nn.Module):
    def __init__(self, config: DreamConfig):
        super().__init__()
        self.config = config
        self.model = DreamBaseModel(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.generation_config = None

    @classmethod
    def from_pretrained(cls, path, config=None, torch_dtype=None, trust_remote_code=False, **_unused):
        from safetensors.torch import load_file

        config = config if config is not None else DreamConfig.from_pretrained(path)
        model = cls(config)
        state = load_file(os.path.join(path, "model.safetensors"))
        missing, unexpected = model.load_state_dict(state, strict=False)
        if missing or unexpected:
            raise RuntimeError(f"checkpoint mismatch: missing={missing} unexpected={unexpected}")
        if isinstance(torch_dtype, torch.dtype):
            model = model.to(torch_dtype)
        return model

    def forward(self, input_ids=None, attention_mask=None, position_ids=None, past_key_values=None, use_cache=None,
                output_attentions=None, return_dict=True, dual_cache=False, replace_position=None, **_unused):
        out = self.model(input_ids=input_ids, attention_mask=attention_mask, position_ids=position_ids,
                         past_key_values=past_key_values, use_cache=use_cache, output_attentions=output_attentions,
                         return_dict=True, dual_cache=dual_cache, replace_position=replace_position)
        logits = self.lm_head(out.last_hidden_state)
        return MaskedLMOutput(logits=logits, past_key_values=out.past_key_values, attentions=out.attentions)


def init_weights_(model: DreamModel, seed: int = 0) -> None:
    """Seeded HF-style init (prefilling_dllm_eval/model_cache/dream/model_dream.py:735-745): N(0, initializer_range)
    for linears and embeddings, zero biases, unit norms — drawn in a fixed parameter order from one generator."""
    g = torch.Generator().manual_seed(seed)
    std = model.config.initializer_range
    for name, p in model.named_parameters():
        with torch.no_grad():
            if name.endswith("layernorm.weight") or name.endswith("norm.weight"):
                p.fill_(1.0)
            elif name.endswith(".bias"):
                p.zero_()
            else:
                p.copy_(torch.randn(p.shape, generator=g, dtype=torch.float32) * std)
