"""Dream / LLaDA-architecture transformer over a paged KV pool, GPU only.

Every step of a layer goes through the sm_100a kernels in `ops`: the linear layers (QKV with bias, O, gate-up with SiLU·mul
fused into its epilogue, down, LM head) on the tcgen05 GEMM kernel, RMSNorm with the residual add, RoPE in place on the
fused QKV output, KV page writes and attention over [selected prefix pages ‖ new rows] — 9 launches per layer (+ the
split-KV merge for decode shapes). Only the embedding gather is torch. A float32 model (the CPU-parity toy) keeps torch's
fp32 GEMM: the tensor cores would round its operands to tf32. Arithmetic follows the Dream model the
reference vendors (prefilling_dllm_eval/model_cache/dream/model_dream.py:117-131 RMSNorm in fp32, :208-264 rotate-half
RoPE with fp32 tables, :326-329 biased q/k/v, :277-278 SwiGLU, :689-711 pre-norm residual) and the engine's own
restatement (prefilling_dllm_engine/prefilling_dllm/models/dream.py:26-237). Keys are stored in pages AFTER RoPE, like
the engine does (models/dream.py:88-101 → attention_v4.py:330-331), so a page is valid for exactly the positions it was
written with.
"""

from __future__ import annotations

import gc

import json
import os
import threading
from collections import deque
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import ops


@dataclass
class DreamArch:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_position_embeddings: int = 131072
    mask_token_id: int = 151666
    bos_token_id: Optional[int] = 151643
    eos_token_id: Optional[int] = 151643
    initializer_range: float = 0.02
    attention_bias: bool = True   # Dream: biased q/k/v; LLaDA-8B: none
    logit_shift: bool = True      # Dream predicts token p from logits[p-1]; LLaDA does not shift

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_pretrained(cls, path: str) -> "DreamArch":
        with open(os.path.join(path, "config.json")) as handle:
            data = json.load(handle)
        names = {f for f in cls.__dataclass_fields__}
        return cls(**{k: v for k, v in data.items() if k in names})

    @classmethod
    def toy(cls) -> "DreamArch":
        """The CPU-runnable toy: 2 layers, hidden 256, 4 query / 2 KV heads of 64, MLP 688, vocabulary 1024."""
        return cls(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=2, num_attention_heads=4,
                   num_key_value_heads=2, rope_theta=1e6, max_position_embeddings=32768, mask_token_id=1023,
                   bos_token_id=1, eos_token_id=2)

    @classmethod
    def dream_7b(cls) -> "DreamArch":
        return cls(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                   num_attention_heads=28, num_key_value_heads=4, rope_theta=1e6, mask_token_id=151666,
                   bos_token_id=151643, eos_token_id=151643)

    @classmethod
    def llada_8b(cls) -> "DreamArch":
        return cls(vocab_size=126464, hidden_size=4096, intermediate_size=12288, num_hidden_layers=32,
                   num_attention_heads=32, num_key_value_heads=32, rope_theta=500000.0, rms_norm_eps=1e-5,
                   mask_token_id=126336, bos_token_id=126080, eos_token_id=126081, attention_bias=False, logit_shift=False)


class PageAllocator:
    """Free-list page allocator with reference counts and a whole-prompt prefix cache.

    Same behaviour as _PrefixPageAllocator (prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:88-167): FIFO free
    list, RuntimeError when pages run out, prefixes keyed by a 64-bit hash of the prompt ids, `evict_one` drops a
    cached prefix nobody uses. Thread-safe (prefill may run on the pd-prefetch thread while decode runs on the main one).
    """

    def __init__(self, num_pages: int, page_size: int):
        self.num_pages = int(num_pages)
        self.page_size = int(page_size)
        self.free_pages = deque(range(self.num_pages))
        self.page_ref_count = [0] * self.num_pages
        self.hash_to_prefix: Dict[int, "CachedPrefix"] = {}
        self._lock = threading.RLock()

    @staticmethod
    def compute_prompt_hash(prompt_ids: Sequence[int]) -> int:
        import numpy as np

        data = np.array(list(prompt_ids), dtype=np.int64).tobytes()
        try:
            import xxhash

            return xxhash.xxh64(data).intdigest()
        except ImportError:  # same role, different 64-bit hash
            import hashlib

            return int.from_bytes(hashlib.blake2b(data, digest_size=8).digest(), "little")

    @property
    def num_free_pages(self) -> int:
        with self._lock:
            return len(self.free_pages)

    def allocate_pages(self, n: int) -> List[int]:
        with self._lock:
            if n > len(self.free_pages):
                raise RuntimeError(f"Cannot allocate {n} pages, only {len(self.free_pages)} free")
            pages = [self.free_pages.popleft() for _ in range(n)]
            for p in pages:
                self.page_ref_count[p] = 1
            return pages

    def ref_pages(self, pages: Sequence[int]) -> None:
        with self._lock:
            for p in pages:
                self.page_ref_count[p] += 1

    def release_pages(self, pages: Sequence[int]) -> None:
        with self._lock:
            for p in pages:
                self.page_ref_count[p] -= 1
                if self.page_ref_count[p] == 0:
                    self.free_pages.append(p)

    def lookup_prefix(self, prompt_ids: Sequence[int]):
        with self._lock:
            return self.hash_to_prefix.get(self.compute_prompt_hash(prompt_ids))

    def register_prefix(self, prompt_ids, page_ids, prompt_len, last_context_logit):
        with self._lock:
            h = self.compute_prompt_hash(prompt_ids)
            entry = CachedPrefix(prompt_hash=h, page_ids=list(page_ids), prompt_len=prompt_len,
                                 last_context_logit=last_context_logit.detach(), ref_count=0)
            self.hash_to_prefix[h] = entry
            return entry

    def release_prefix(self, prompt_ids) -> None:
        with self._lock:
            entry = self.hash_to_prefix.get(self.compute_prompt_hash(prompt_ids))
            if entry is not None:
                entry.ref_count -= 1

    def evict_one(self) -> bool:
        with self._lock:
            for h, entry in list(self.hash_to_prefix.items()):
                if entry.ref_count <= 0:
                    self.release_pages(entry.page_ids)
                    del self.hash_to_prefix[h]
                    return True
            return False

    def ensure_free(self, n: int) -> None:
        """Evict unused cached prefixes until n pages are free (or nothing is left to evict)."""
        while self.num_free_pages < n:
            if not self.evict_one():
                break


@dataclass
class CachedPrefix:
    prompt_hash: int
    page_ids: List[int]
    prompt_len: int
    last_context_logit: torch.Tensor
    ref_count: int = 1


def slots_for(page_ids: Sequence[int], start_token: int, num_tokens: int, page_size: int) -> List[int]:
    """Pool slots of logical tokens [start_token, start_token + num_tokens) laid over `page_ids`."""
    return [page_ids[t // page_size] * page_size + t % page_size for t in range(start_token, start_token + num_tokens)]


class PagedDreamModel:
    """Weights + paged KV pool + forward. One instance per device."""

    def __init__(self, arch: DreamArch, state: Dict[str, torch.Tensor], *, device, dtype: torch.dtype,
                 num_pages: int, page_size: int = 256):
        if not torch.cuda.is_available():
            raise RuntimeError("PagedDreamModel needs a CUDA device; there is no CPU path")
        self.arch = arch
        self.device = torch.device(device)
        self.dtype = dtype
        self.page_size = int(page_size)
        self.num_pages = int(num_pages)
        a = arch
        dev, dt = self.device, dtype

        def get(name):
            return state[name].to(device=dev, dtype=dt).contiguous()

        # bf16 / fp16 models run their linear layers on the tcgen05 GEMM kernel; fp32 models on torch's fp32 GEMM
        self.tensor_core_linear = dtype in (torch.bfloat16, torch.float16)
        self.embed = get("model.embed_tokens.weight")
        self.final_norm = get("model.norm.weight")
        self.lm_head = get("lm_head.weight") if "lm_head.weight" in state else self.embed
        self.layers = []
        for i in range(a.num_hidden_layers):
            p = f"model.layers.{i}."
            wqkv = torch.cat([get(p + "self_attn.q_proj.weight"), get(p + "self_attn.k_proj.weight"), get(p + "self_attn.v_proj.weight")], dim=0)
            bqkv = None
            if a.attention_bias and (p + "self_attn.q_proj.bias") in state:
                bqkv = torch.cat([get(p + "self_attn.q_proj.bias"), get(p + "self_attn.k_proj.bias"), get(p + "self_attn.v_proj.bias")], dim=0)
            gate, up = get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")
            if self.tensor_core_linear:
                # rows interleaved (2i = gate_i, 2i + 1 = up_i): the GEMM epilogue then holds each (gate, up) pair together
                wgu = torch.stack([gate, up], dim=1).reshape(2 * gate.shape[0], gate.shape[1]).contiguous()
            else:
                wgu = torch.cat([gate, up], dim=0).contiguous()
            del gate, up
            self.layers.append(dict(
                ln1=get(p + "input_layernorm.weight"), ln2=get(p + "post_attention_layernorm.weight"),
                wqkv=wqkv.contiguous(), bqkv=bqkv, wo=get(p + "self_attn.o_proj.weight"), wgu=wgu,
                wd=get(p + "mlp.down_proj.weight")))
        self.inv_freq = (1.0 / (a.rope_theta ** (torch.arange(0, a.head_dim, 2, dtype=torch.int64).float() / a.head_dim))).to(dev)
        self.rope_attention_scaling = 1.0      # YaRN's factor on cos / sin (1 without scaling)
        # pool [2 (k,v), layers, pages, page_size, Hkv, D] — same shape as the engine's kv_cache (engine/model_runner.py:557-567)
        self.kv_cache = torch.zeros((2, a.num_hidden_layers, self.num_pages, self.page_size, a.num_key_value_heads, a.head_dim),
                                    dtype=dt, device=dev)
        self.allocator = PageAllocator(self.num_pages, self.page_size)
        self.scale = a.head_dim ** -0.5

    # ---- construction helpers ----
    @classmethod
    def from_pretrained(cls, path: str, *, device, dtype: torch.dtype, num_pages: int, page_size: int = 256, arch: Optional[DreamArch] = None):
        from safetensors.torch import load_file

        arch = arch or DreamArch.from_pretrained(path)
        files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
        state: Dict[str, torch.Tensor] = {}
        for name in files:
            state.update(load_file(os.path.join(path, name)))
        return cls(arch, state, device=device, dtype=dtype, num_pages=num_pages, page_size=page_size)

    @classmethod
    def random_init(cls, arch: DreamArch, *, device, dtype: torch.dtype, num_pages: int, page_size: int = 256, seed: int = 0):
        """Seeded N(0, initializer_range) linears/embeddings, unit norms, zero biases, generated ON the device layer by
        layer (a 7B random model never exists on the host). Not bit-identical to a CPU-seeded checkpoint: use
        from_pretrained when weights must match another implementation."""
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        a = arch
        std = a.initializer_range

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std).to(dtype)

        kv = a.num_key_value_heads * a.head_dim
        state = {"model.embed_tokens.weight": w(a.vocab_size, a.hidden_size), "lm_head.weight": w(a.vocab_size, a.hidden_size),
                 "model.norm.weight": torch.ones(a.hidden_size, device=dev, dtype=dtype)}
        for i in range(a.num_hidden_layers):
            p = f"model.layers.{i}."
            state[p + "self_attn.q_proj.weight"] = w(a.hidden_size, a.hidden_size)
            state[p + "self_attn.k_proj.weight"] = w(kv, a.hidden_size)
            state[p + "self_attn.v_proj.weight"] = w(kv, a.hidden_size)
            if a.attention_bias:
                state[p + "self_attn.q_proj.bias"] = torch.zeros(a.hidden_size, device=dev, dtype=dtype)
                state[p + "self_attn.k_proj.bias"] = torch.zeros(kv, device=dev, dtype=dtype)
                state[p + "self_attn.v_proj.bias"] = torch.zeros(kv, device=dev, dtype=dtype)
            state[p + "self_attn.o_proj.weight"] = w(a.hidden_size, a.hidden_size)
            state[p + "mlp.gate_proj.weight"] = w(a.intermediate_size, a.hidden_size)
            state[p + "mlp.up_proj.weight"] = w(a.intermediate_size, a.hidden_size)
            state[p + "mlp.down_proj.weight"] = w(a.hidden_size, a.intermediate_size)
            state[p + "input_layernorm.weight"] = torch.ones(a.hidden_size, device=dev, dtype=dtype)
            state[p + "post_attention_layernorm.weight"] = torch.ones(a.hidden_size, device=dev, dtype=dtype)
        return cls(arch, state, device=dev, dtype=dtype, num_pages=num_pages, page_size=page_size)

    # ---- pieces ----
    def apply_yarn_rope_scaling(self, factor: float, original_max_position_embeddings: Optional[int] = None,
                                beta_fast: float = 32.0, beta_slow: float = 1.0) -> None:
        """YaRN context extension (Peng et al. 2023) as the reference applies it (prefilling_dllm_eval/fastdllm_parallelcomp.py
        :539-553: rope_scaling = {rope_type: yarn, factor, original_max_position_embeddings}, the rotary table rebuilt): the
        high-frequency dimensions keep their frequency, the low-frequency ones are divided by `factor`, a linear ramp between the
        dimensions that complete `beta_fast` and `beta_slow` rotations within the original context blends the two, and cos / sin
        are multiplied by 0.1 ln(factor) + 1. Pages written before the call keep their old rotation."""
        if factor <= 1.0:
            return
        import math

        a = self.arch
        dim, base = a.head_dim, float(a.rope_theta)
        original = int(original_max_position_embeddings or a.max_position_embeddings)
        pos_freqs = base ** (torch.arange(0, dim, 2).float() / dim)
        extrapolation, interpolation = 1.0 / pos_freqs, 1.0 / (factor * pos_freqs)

        def correction_dim(rotations: float) -> float:
            return (dim * math.log(original / (rotations * 2 * math.pi))) / (2 * math.log(base))

        low = max(math.floor(correction_dim(beta_fast)), 0)
        high = min(math.ceil(correction_dim(beta_slow)), dim - 1)
        if low == high:
            high += 0.001
        keep = 1 - torch.clamp((torch.arange(dim // 2, dtype=torch.float32) - low) / (high - low), 0, 1)
        self.inv_freq = (interpolation * (1 - keep) + extrapolation * keep).to(self.device)
        self.rope_attention_scaling = 0.1 * math.log(factor) + 1.0
        self.__dict__.pop("_step_graphs", None)        # captured steps hold no tables, but shapes may change with longer contexts

    def apply_linear_rope_scaling(self, factor: float) -> None:
        """Position interpolation as the reference applies it to its LLaDA backend (prefilling_dllm_eval/fastdllm_parallelcomp.py
        :555-690, scaling type "linear"): positions are divided by `factor` before they meet the unchanged frequencies; no
        attention scaling. Pages written before the call keep their old rotation."""
        if factor <= 1.0:
            return
        self.rope_position_divisor = float(factor)
        self.__dict__.pop("_step_graphs", None)

    def _rope_tables(self, positions: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        positions = positions.float()
        divisor = getattr(self, "rope_position_divisor", 1.0)
        if divisor != 1.0:
            positions = positions / divisor
        freqs = positions.unsqueeze(-1) * self.inv_freq.unsqueeze(0)  # [T, D/2] fp32
        emb = torch.cat((freqs, freqs), dim=-1)
        cos, sin = emb.cos(), emb.sin()
        if self.rope_attention_scaling != 1.0:
            cos, sin = cos * self.rope_attention_scaling, sin * self.rope_attention_scaling
        return cos.to(self.dtype).unsqueeze(1), sin.to(self.dtype).unsqueeze(1)  # [T, 1, D]

    def layer_cache(self, layer: int) -> Tuple[torch.Tensor, torch.Tensor]:
        return self.kv_cache[0, layer], self.kv_cache[1, layer]

    def plane_pools(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """(K pool, V pool) of ALL layers, each seen as one unified cache of layers * pages pages: one slot mapping or page list
        then addresses every layer at once (slot of token t of layer l: (l * pages + page_id) * page_size + offset)."""
        kv = self.kv_cache
        shape = (kv.shape[1] * kv.shape[2], kv.shape[3], kv.shape[4], kv.shape[5])
        return kv[0].view(shape), kv[1].view(shape)

    def all_layer_slots(self, page_ids: Sequence[int], start: int, n: int) -> torch.Tensor:
        """int32 [n * layers] slots in `plane_pools()` of cache tokens [start, start + n) laid over `page_ids`, token-major
        (row index = token * layers + layer)."""
        base = torch.tensor(slots_for(page_ids, start, n, self.page_size), dtype=torch.int64, device=self.device)
        layers = self.arch.num_hidden_layers
        offs = torch.arange(layers, dtype=torch.int64, device=self.device) * (self.num_pages * self.page_size)
        return (base.view(-1, 1) + offs.view(1, -1)).reshape(-1).to(torch.int32)

    # ---- forward ----
    @torch.inference_mode()
    def forward(self, ids: torch.Tensor, positions: torch.Tensor, *, cu_seqlens: torch.Tensor, max_query_len: int,
                slot_mapping: Optional[torch.Tensor] = None, block_table: Optional[torch.Tensor] = None,
                seq_lens: Optional[torch.Tensor] = None, max_seq_len: int = 0, causal: bool = False,
                logit_rows: Optional[torch.Tensor] = None, want_logits: bool = True,
                capture_qk_layers: Optional[Sequence[int]] = None, store_after_attention: bool = False,
                store_unrotated_k: bool = False, new_row_mask: Optional[torch.Tensor] = None, on_layer_stored=None,
                attention_fn=None):
        """Packed forward of `ids` [T] (several sequences delimited by cu_seqlens) at RoPE `positions` [T].

        slot_mapping [T] int32 (optional): where each row's K/V goes in the pool (-1 = do not store).
        store_after_attention: write the rows' K/V only after the layer's attention has read the pool, for a forward whose
        target slots still hold keys that this same forward must attend (committing a finished block over stale slots).
        store_unrotated_k: the K written to the pool is the projection BEFORE the rotary embedding (attention over the rows
        themselves still uses rotated keys); the caller rotates the stored rows later with `rope_rows` — per-head
        eviction assigns positions only after compaction.
        new_row_mask: bool [rows, rows] visibility among the new rows of ONE sequence (row i sees new row j iff True); the
        cached context stays fully visible. None = all visible (or the causal rule).
        block_table / seq_lens (optional): cached context each sequence attends before its own rows.
        causal: scoring mask (row sees itself and earlier rows); otherwise rows see each other bidirectionally.
        logit_rows: indices of the rows whose logits are wanted (LM head runs on those rows only).
        capture_qk_layers: layers whose rotated (q, k) are returned for the eviction scorer.
        on_layer_stored: callable(layer index), invoked right after a layer's K/V rows were written to pages (their final
        values in a forward that stores before attention): lets a transfer of layer l overlap the compute of layer l + 1.
        attention_fn: callable(layer index, run, out) that takes the place of a layer's attention call. `run(out, mask=...,
        block_table=..., seq_lens=..., max_seq_len=...)` performs the standard call of this forward into `out` [rows, Hq, D] with
        any of its mask / cached-context arguments replaced; the callable must leave the layer's result in `out`. For attention
        variants that are compositions of standard calls (sparse key masks, corrections from a second pass over other pages).
        Returns (logits or None, {layer: (q, k)}).
        """
        a = self.arch
        hq, hkv, d = a.num_attention_heads, a.num_key_value_heads, a.head_dim
        if store_unrotated_k and store_after_attention:
            raise ValueError("store_unrotated_k and store_after_attention are not combined by any caller")
        x = self.embed[ids]                                              # [T, hidden], the residual stream
        cos, sin = self._rope_tables(positions)
        cos2, sin2 = cos.reshape(-1, d), sin.reshape(-1, d)
        captured = {}
        capture = set(capture_qk_layers) if capture_qk_layers is not None else ()
        # A forward that is run only for the (q, k) of some layers — the eviction scorer's, which by default reads the first layer —
        # ends at the last of them: nothing after it is returned or stored.
        ends_at = max(capture) if capture and not want_logits and slot_mapping is None and on_layer_stored is None else None
        total = ids.numel()
        attn_out = torch.empty((total, hq, d), dtype=self.dtype, device=self.device)
        eps = a.rms_norm_eps
        delta = None                                                     # output of the previous sub-block, not yet added to x
        fused_rope_store = self.dtype in (torch.bfloat16, torch.float16) and d % 16 == 0
        for li, w in enumerate(self.layers):
            h = ops.add_rmsnorm(x, w["ln1"], eps, delta)                 # x += delta; h = norm(x)
            qkv = self._linear(h, w["wqkv"], w["bqkv"]).view(total, hq + 2 * hkv, d)
            q, k, v = qkv[:, :hq], qkv[:, hq:hq + hkv], qkv[:, hq + hkv:]   # strided views of one buffer: no copies
            k_cache, v_cache = self.layer_cache(li)
            if fused_rope_store:
                # rotation of the q and k heads and the page write of k and v in ONE launch (the write waits when it must follow attention)
                write_now = slot_mapping is not None and not store_after_attention
                ops.rope_store(qkv, cos2, sin2, hq, hkv, k_cache if write_now else None, v_cache if write_now else None,
                               slot_mapping if write_now else None, k_before_rotation=store_unrotated_k)
            else:
                if slot_mapping is not None and store_unrotated_k:
                    ops.store_kvcache_unified_layout(k, v, k_cache, v_cache, slot_mapping, "diffusion_lm")
                ops.rope_inplace(qkv[:, :hq + hkv], cos2, sin2)              # q and k heads are adjacent: one launch
                if slot_mapping is not None and not store_after_attention and not store_unrotated_k:
                    ops.store_kvcache_unified_layout(k, v, k_cache, v_cache, slot_mapping, "diffusion_lm")
            if li in capture:
                captured[li] = (q.contiguous(), k.contiguous())
                if li == ends_at:
                    return None, captured
            def run_attention(out, mask=new_row_mask, block_table=block_table, seq_lens=seq_lens, max_seq_len=max_seq_len,
                              q=q, k=k, v=v, k_cache=k_cache, v_cache=v_cache):
                if block_table is not None:
                    ops.paged_attention(q, k, v, out, cu_seqlens_q=cu_seqlens, max_query_len=max_query_len, key_cache=k_cache,
                                        value_cache=v_cache, block_table=block_table, seq_lens=seq_lens, max_seq_len=max_seq_len,
                                        sm_scale=self.scale, causal=causal, bidirectional=True, mask=mask)
                else:
                    ops.paged_attention(q, k, v, out, cu_seqlens_q=cu_seqlens, max_query_len=max_query_len,
                                        sm_scale=self.scale, causal=causal, bidirectional=True, mask=mask)

            if attention_fn is None:
                run_attention(attn_out)
            else:
                attention_fn(li, run_attention, attn_out)
            if slot_mapping is not None and store_after_attention:
                ops.store_kvcache_unified_layout(k, v, k_cache, v_cache, slot_mapping, "diffusion_lm")
            if on_layer_stored is not None and slot_mapping is not None:
                on_layer_stored(li)
            proj = self._linear(attn_out.view(total, hq * d), w["wo"])
            h = ops.add_rmsnorm(x, w["ln2"], eps, proj)                  # x += attention output; h = norm(x)
            if self.tensor_core_linear:
                delta = ops.linear(ops.linear(h, w["wgu"], silu_mul_interleaved=True, weights_at_rest=True), w["wd"], weights_at_rest=True)   # SiLU(gate)·up in the GEMM epilogue
            else:
                delta = F.linear(ops.silu_mul(F.linear(h, w["wgu"])), w["wd"])
        if delta is not None:
            x = x + delta
        logits = None
        if want_logits:
            rows = x if logit_rows is None else x.index_select(0, logit_rows)
            logits = self._linear(ops.add_rmsnorm(rows.contiguous(), self.final_norm, eps), self.lm_head)
        return logits, captured

    def _linear(self, x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        return ops.linear(x, weight, bias, weights_at_rest=True) if self.tensor_core_linear else F.linear(x, weight, bias)

    def rope_rows(self, page_ids, start: int, positions: Sequence[int]) -> None:
        """Rotate the un-rotated K rows `[start, start + len(positions))` of `page_ids` in place, in every layer."""
        if not positions:
            return
        cos, sin = self._rope_tables(torch.tensor(list(positions), dtype=torch.long, device=self.device))
        for layer in range(self.arch.num_hidden_layers):
            ops.rope_pages(self.layer_cache(layer)[0], page_ids, start, cos, sin)

    def block_step_runner(self, *, block_len: int, positions: Sequence[int], ctx_page_ids: Sequence[int], ctx_len: int,
                          mask_token_id: int, threshold: float, last_logit: Optional[torch.Tensor], shift: bool,
                          softmax_dtype: Optional[torch.dtype], store_slots: Optional[Sequence[int]] = None,
                          use_graph: bool = True) -> "BlockStepRunner":
        """One denoise step = forward of the block rows against `ctx_len` cached tokens + the unmask kernel, repeated
        with identical shapes until the block is full. Returns a runner whose `.block` (int64 [block_len]) the caller
        fills with the initial ids; `.run()` performs a step and returns the number of MASK slots left."""
        request = dict(positions=positions, ctx_page_ids=ctx_page_ids, ctx_len=ctx_len, last_logit=last_logit, store_slots=store_slots)
        return BlockStepRunner(self, block_len=block_len, requests=[request], mask_token_id=mask_token_id, threshold=threshold,
                               shift=shift, softmax_dtype=softmax_dtype, use_graph=use_graph)

    def batched_step_runner(self, *, block_len: int, requests: Sequence[dict], mask_token_id: int, threshold: float, shift: bool,
                            softmax_dtype: Optional[torch.dtype], use_graph: bool = True) -> "BlockStepRunner":
        """The same step for the blocks of several requests at once (`.blocks[i]`, `.remaining[i]`)."""
        return BlockStepRunner(self, block_len=block_len, requests=list(requests), mask_token_id=mask_token_id, threshold=threshold,
                               shift=shift, softmax_dtype=softmax_dtype, use_graph=use_graph)

    # ---- small tensor helpers ----
    def ids_tensor(self, ids: Sequence[int]) -> torch.Tensor:
        return torch.tensor(list(ids), dtype=torch.long, device=self.device)

    def i32(self, values: Sequence[int]) -> torch.Tensor:
        return torch.tensor(list(values), dtype=torch.int32, device=self.device)



def denoise_blocks(model: "PagedDreamModel", cache, *, suffix_pos_start: int, last_logit: torch.Tensor, first_token, tail_in_cache: int,
                   max_new: int, block_length: int, mask_id: int, threshold: float, softmax_dtype: Optional[torch.dtype], use_graph: bool,
                   fixed_steps_per_block: Optional[int] = None, fill_most_confident=None, steps_out: Optional[List[int]] = None,
                   pick_first_token=None, threshold_step=None) -> List[int]:
    """Fast-dLLM dual-cache block loop over a paged cache (reference eval class prefilling_dllm_eval/fastdllm_parallelcomp.py
    :2932-2998, :2399-2441), shared by the eval-class runtime and the engine's multi-block decode.

    `cache`: a handle with `page_ids`, `length` (valid tokens: prompt, finished blocks and `tail_in_cache` later-block MASK
    slots; updated here) and `slots(start, n)`. Layout while block b is active: [prompt ‖ finished blocks ‖ MASK slots of the
    later blocks]; the active block's rows are the new rows of every forward, so they replace their own slots by
    construction (the LAST block is returned but never written to the cache). After the block is committed its K/V take the place of the first later-MASK slots and the later slots are
    recomputed by the next block's suffix initialisation (reference :2368-2397).
    `first_token`: the first token of block 0 when the prefill already produced it together with the later-MASK slots
    (full_prompt_mask mode); None = every block starts with a suffix initialisation.
    `softmax_dtype`: None = probabilities in the model dtype (eval class), torch.float32 = the engine's rule.
    `fixed_steps_per_block`: None = confidence-threshold denoising; an int = the fixed-step diffusion sampler (reference
    _denoise_block_diffusion :2443-2510): step i of n transfers int(masks * (1 - t[i+1] / t[i])) of the most confident slots
    through `fill_most_confident(logits, block, last_logit, count)`, t = linspace(1, 1e-3, n + 1), the last step all that is left.
    `steps_out`: when given, the number of denoise forwards of every block is appended.
    `pick_first_token(last_logit) -> 0-d tensor`: the first token of a block (default: arg-max, which is what any greedy sampler
    returns). `threshold_step(logits, block, last_logit) -> MASK slots left`: replaces the fused forward + unmask step of the
    confidence-threshold loop by an eager forward followed by this callable (samplers that the unmask kernel does not cover)."""
    import math

    arch = model.arch
    dev = model.device

    def forward(ids_t, positions, ctx_len, *, store_slots=None, logit_rows=None, want_logits=True, store_after_attention=False):
        n = int(ids_t.numel())
        kwargs = {}
        if ctx_len > 0:
            kwargs = dict(block_table=model.i32(cache.page_ids).view(1, -1), seq_lens=model.i32([ctx_len + n]), max_seq_len=ctx_len + n)
        return model.forward(ids_t, torch.tensor(list(positions), dtype=torch.long, device=dev), cu_seqlens=model.i32([0, n]), max_query_len=n,
                             slot_mapping=None if store_slots is None else model.i32(store_slots), causal=False,
                             logit_rows=None if logit_rows is None else model.ids_tensor(logit_rows), want_logits=want_logits,
                             store_after_attention=store_after_attention, **kwargs)

    n0 = cache.length - tail_in_cache          # prompt (+ query) tokens
    num_blocks = max(1, math.ceil(max_new / block_length))
    generated: List[int] = []
    tail_len = tail_in_cache
    for b in range(num_blocks):
        start = b * block_length
        blen = min(block_length, max_new - start)
        if blen <= 0:
            break
        done = n0 + start                       # prompt + finished blocks
        block_pos = list(range(suffix_pos_start + start, suffix_pos_start + start + blen))
        later = max_new - start - blen          # MASK slots of the blocks after this one
        if first_token is None or b > 0:
            # suffix initialisation (reference :2368-2397): forward all remaining MASKs against prompt + finished blocks; the
            # later blocks' K/V go behind the finished ones, the active block's rows are not stored. Dream reads the block's first
            # token from the last context logit; an un-shifted architecture (LLaDA) from the first MASK slot's own row of this
            # forward, which therefore runs even when no later block is left.
            first_logit = last_logit
            if later > 0 or not arch.logit_shift:
                suffix_pos = list(range(suffix_pos_start + start, suffix_pos_start + start + blen + later))
                slots = ([-1] * blen + cache.slots(done, later)) if later > 0 else None
                out, _ = forward(torch.full((blen + later,), mask_id, dtype=torch.long, device=dev), suffix_pos, done, store_slots=slots,
                                 logit_rows=None if arch.logit_shift else [0], want_logits=not arch.logit_shift)
                if not arch.logit_shift:
                    first_logit = out[0]
            tail_len = later
            # softmax is monotone: a greedy sampler's first token is the arg-max of the logit
            first = torch.argmax(first_logit) if pick_first_token is None else pick_first_token(first_logit)
        else:
            first = first_token
        ctx = done + tail_len
        runner = model.block_step_runner(block_len=blen, positions=block_pos, ctx_page_ids=cache.page_ids, ctx_len=ctx, mask_token_id=mask_id,
                                         threshold=float(threshold), last_logit=last_logit, shift=arch.logit_shift, softmax_dtype=softmax_dtype,
                                         use_graph=bool(use_graph))
        block = runner.block                      # the step's ids buffer, updated in place by the unmask kernel
        block.fill_(mask_id)
        block[0] = first
        guard = 0
        remaining = blen - 1
        if fixed_steps_per_block is not None:
            steps = int(fixed_steps_per_block)
            timesteps = torch.linspace(1, 1e-3, steps + 1)       # fp32 on the host, the reference's own arithmetic
            for step in range(steps):
                if remaining <= 0:
                    break
                count = int(remaining * (1 - timesteps[step + 1] / timesteps[step])) if step < steps - 1 else remaining
                if count <= 0:
                    continue
                logits, _ = forward(block, block_pos, ctx)
                remaining -= fill_most_confident(logits, block, last_logit, count)
                guard += 1
            remaining = 0
        while remaining > 0:
            guard += 1
            if guard > blen + 8:
                break
            if threshold_step is not None:
                logits, _ = forward(block, block_pos, ctx)
                remaining = int(threshold_step(logits, block, last_logit))
                continue
            remaining = runner.run()   # forward + unmask kernel (a CUDA graph replay from the third step on); one host read
        if steps_out is not None:
            steps_out.append(guard)
        generated.extend(block.tolist())
        if later <= 0:
            break       # the reference commits the last block too (:2764-2771); nothing reads that K/V or logit afterwards
        # commit forward: the finished block's K/V take the first slots behind prompt + finished; its last logit is the next
        # block's "last context logit". The store comes after attention so the later-MASK slots are still seen.
        logits, _ = forward(block, block_pos, ctx, store_slots=cache.slots(done, blen), logit_rows=[blen - 1], store_after_attention=True)
        last_logit = logits[0]
        cache.length = done + blen
        tail_len = 0
    return generated[:max_new]


def denoise_blocks_batched(model: "PagedDreamModel", caches, *, suffix_pos_starts: Sequence[int], last_logits: Sequence[torch.Tensor],
                           max_new: int, block_length: int, mask_id: int, threshold: float, softmax_dtype: Optional[torch.dtype],
                           use_graph: bool, steps_out: Optional[List[List[int]]] = None) -> List[List[int]]:
    """`denoise_blocks` for several requests whose blocks share every forward: the suffix initialisation, each denoise step and
    the commit of block b run once for all requests (rows packed, every request against its own page list and context
    length), so a step reads the model's weights once whatever the number of requests. Confidence-threshold rule only; every
    request generates `max_new` tokens in blocks of `block_length`. `caches[i]`: as in `denoise_blocks` (updated in place).
    Same ids per request as `denoise_blocks` on that request alone. `steps_out[i]`: forwards each block of request i needed."""
    import math

    arch, dev, n_req = model.arch, model.device, len(caches)

    def packed_forward(ids_rows, pos_rows, ctx_lens, *, slot_rows=None, logit_rows=None, want_logits=True, store_after_attention=False):
        lens = [len(p) for p in pos_rows]
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        width = max(len(c.page_ids) for c in caches)
        table = torch.zeros((n_req, width), dtype=torch.int32, device=dev)
        for i, c in enumerate(caches):
            table[i, :len(c.page_ids)] = model.i32(c.page_ids)
        slots = None if slot_rows is None else model.i32([s for row in slot_rows for s in row])
        return model.forward(torch.cat(ids_rows), torch.tensor([p for row in pos_rows for p in row], dtype=torch.long, device=dev),
                             cu_seqlens=model.i32(cu), max_query_len=max(lens), slot_mapping=slots, causal=False,
                             logit_rows=None if logit_rows is None else model.ids_tensor(logit_rows), want_logits=want_logits,
                             store_after_attention=store_after_attention, block_table=table,
                             seq_lens=model.i32([c + n for c, n in zip(ctx_lens, lens)]), max_seq_len=max(ctx_lens) + max(lens))

    prompt_lens = [int(c.length) for c in caches]
    last_logits = list(last_logits)
    generated: List[List[int]] = [[] for _ in range(n_req)]
    num_blocks = max(1, math.ceil(max_new / block_length))
    for b in range(num_blocks):
        start = b * block_length
        blen = min(block_length, max_new - start)
        if blen <= 0:
            break
        later = max_new - start - blen
        done = [n0 + start for n0 in prompt_lens]
        block_pos = [list(range(s0 + start, s0 + start + blen)) for s0 in suffix_pos_starts]
        first_logits = last_logits
        if later > 0 or not arch.logit_shift:     # un-shifted read-out: the first token comes from the first MASK slot's own row
            masks = torch.full((blen + later,), mask_id, dtype=torch.long, device=dev)
            out, _ = packed_forward([masks] * n_req, [list(range(s0 + start, s0 + start + blen + later)) for s0 in suffix_pos_starts], done,
                                    slot_rows=[[-1] * blen + c.slots(d, later) for c, d in zip(caches, done)] if later > 0 else None,
                                    logit_rows=None if arch.logit_shift else [i * (blen + later) for i in range(n_req)],
                                    want_logits=not arch.logit_shift)
            if not arch.logit_shift:
                first_logits = [out[i] for i in range(n_req)]
        requests = [dict(positions=block_pos[i], ctx_page_ids=caches[i].page_ids, ctx_len=done[i] + later, last_logit=last_logits[i])
                    for i in range(n_req)]
        runner = model.batched_step_runner(block_len=blen, requests=requests, mask_token_id=mask_id, threshold=float(threshold),
                                           shift=arch.logit_shift, softmax_dtype=softmax_dtype, use_graph=bool(use_graph))
        for i, block in enumerate(runner.blocks):
            block.fill_(mask_id)
            block[0] = torch.argmax(first_logits[i])
        left, step, needed = [blen - 1] * n_req, 0, [0] * n_req
        while any(x > 0 for x in left):
            step += 1
            if step > blen + 8:
                raise RuntimeError("denoising did not converge: every step must unmask at least one slot")
            runner.run()
            for i, (before, after) in enumerate(zip(left, runner.remaining)):
                if before > 0 and after == 0:
                    needed[i] = step
            left = list(runner.remaining)
        if steps_out is not None:
            for i in range(n_req):
                steps_out[i].append(needed[i])
        for i, block in enumerate(runner.blocks):
            generated[i].extend(block.tolist())
        if later <= 0:
            break       # the last block's K/V and logit are read by nothing
        # commit: the finished blocks' K/V take the first slots behind prompt + finished blocks (stored after attention, which
        # still reads the later-MASK slots there); the last row's logit is the next block's last-context logit
        ctx = [d + later for d in done]
        logits, _ = packed_forward([blk.clone() for blk in runner.blocks], block_pos, ctx,
                                   slot_rows=[c.slots(d, blen) for c, d in zip(caches, done)],
                                   logit_rows=[i * blen + blen - 1 for i in range(n_req)], store_after_attention=True)
        last_logits = [logits[i] for i in range(n_req)]
        for c, d in zip(caches, done):
            c.length = d + blen
    return [g[:max_new] for g in generated]


class _StepGraph:
    """A captured denoise step and the device buffers it reads: per request only their CONTENTS change."""

    def __init__(self, model: "PagedDreamModel", n: int, batch: int, pages: int, has_last: bool, stores: bool):
        dev = model.device
        self.block = torch.zeros(batch * n, dtype=torch.long, device=dev)
        self.positions = torch.zeros(batch * n, dtype=torch.long, device=dev)
        self.table = torch.zeros((batch, pages), dtype=torch.int32, device=dev)
        self.seq_lens = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.last_logit = torch.zeros((batch, model.arch.vocab_size), dtype=model.dtype, device=dev) if has_last else None
        self.slots = torch.full((batch * n,), -1, dtype=torch.int32, device=dev) if stores else None
        self.cu = model.i32([i * n for i in range(batch + 1)])
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.left: Optional[torch.Tensor] = None      # [batch] MASK slots left after the captured step
        self.eager_steps = 0
        self.calls_per_step = 0                       # C-ABI calls the captured step makes (for launch accounting)
        self.host_counts: Optional[torch.Tensor] = None   # pinned [2, batch]: where the counts of the last two replays land


class BlockStepRunner:
    """The inner loop of block denoising: every step launches the same ~11 kernels per layer on the same few rows, so on
    a 7B model a step is bound by launch overhead (hundreds of launches of microseconds each) and by the 15 GB of
    weights it reads, whatever the number of rows. Two consequences:
      * a step is captured into a CUDA graph, once per shape class — (block length, number of requests, context pages
        rounded up to a multiple of four, unmask rule) — and kept with the model; a request only copies its ids,
        positions, page list, context length and last-context logit into the graph's input buffers and replays. The
        first step of a new shape class runs eagerly (it also initialises library handles and grow-only workspaces),
        the second is the capture. Capturing costs about as much as a hundred steps, so it pays from the second
        request on;
      * the blocks of several requests can share a step: their rows are packed into one forward (each with its own
        page list and context length), so the weights are read once for all of them.
    `requests`: one dict per request with `positions`, `ctx_page_ids`, `ctx_len`, `last_logit`, `store_slots`."""

    _PAGE_BUCKET = 4
    _MAX_CACHED = 8

    def __init__(self, model: PagedDreamModel, *, block_len, requests, mask_token_id, threshold, shift, softmax_dtype, use_graph):
        self.m = model
        n, batch = int(block_len), len(requests)
        if batch < 1:
            raise ValueError("no request to step")
        if any(int(r["ctx_len"]) <= 0 for r in requests):
            raise ValueError("block denoising needs a cached context")
        has_last = requests[0].get("last_logit") is not None
        stores = requests[0].get("store_slots") is not None
        if any((r.get("last_logit") is not None) != has_last or (r.get("store_slots") is not None) != stores for r in requests):
            raise ValueError("requests of one step must agree on last_logit / store_slots being given")
        need = [max(1, -(-int(r["ctx_len"]) // model.page_size)) for r in requests]
        pages = -(-max(need) // self._PAGE_BUCKET) * self._PAGE_BUCKET
        key = (n, batch, pages, int(mask_token_id), float(threshold), has_last, bool(shift), softmax_dtype, stores)
        cache = model.__dict__.setdefault("_step_graphs", {})
        entry = cache.pop(key, None) if use_graph else None
        if entry is None:
            with torch.inference_mode(False):
                entry = _StepGraph(model, n, batch, pages, has_last, stores)
        if use_graph:
            cache[key] = entry                      # most recently used last
            while len(cache) > self._MAX_CACHED:
                cache.pop(next(iter(cache)))
        self.e = entry
        self.n, self.batch, self.use_graph = n, batch, bool(use_graph)
        self.blocks = [entry.block[i * n:(i + 1) * n] for i in range(batch)]
        self.block = self.blocks[0]
        self.remaining = [n] * batch
        self._known = [n] * batch            # MASK slots per request after the last step whose counts were read
        self._most_filled = 1                # most slots any step of this block has filled in one request
        self._pending: List[Tuple[torch.cuda.Event, int]] = []   # replays enqueued whose counts were not read yet
        self._slot = 0
        dev = model.device
        entry.positions.copy_(torch.tensor([p for r in requests for p in r["positions"]], dtype=torch.long, device=dev))
        entry.table.zero_()
        for i, r in enumerate(requests):
            ids = list(r["ctx_page_ids"])[:need[i]]
            entry.table[i, : len(ids)].copy_(model.i32(ids))
            if has_last:
                entry.last_logit[i].copy_(r["last_logit"].reshape(-1))
        entry.seq_lens.copy_(model.i32([int(r["ctx_len"]) + n for r in requests]))
        if stores:
            entry.slots.copy_(model.i32([sl for r in requests for sl in r["store_slots"]]))
        self.kwargs = dict(block_table=entry.table, seq_lens=entry.seq_lens, max_seq_len=pages * model.page_size + n)
        self.unmask = dict(mask_token_id=int(mask_token_id), threshold=float(threshold), shift=bool(shift), softmax_dtype=softmax_dtype)

    def _step(self) -> torch.Tensor:
        e, n = self.e, self.n
        logits, _ = self.m.forward(e.block, e.positions, cu_seqlens=e.cu, max_query_len=n, slot_mapping=e.slots, causal=False,
                                   **self.kwargs)
        # one launch for the blocks of all requests
        counts = ops.unmask_step_batched(logits.view(self.batch, n, -1), e.block.view(self.batch, n), last_logit=e.last_logit,
                                         **self.unmask)
        return counts[:, 2]

    def run(self) -> int:
        """One step for every request; returns the total number of MASK slots left (per request: `.remaining`)."""
        e = self.e
        with torch.cuda.device(self.m.device):
            if not self.use_graph or (e.graph is None and e.eager_steps == 0):
                e.eager_steps += 1
                left = self._step()
            else:
                if e.graph is None:
                    graph = torch.cuda.CUDAGraph()
                    # torch keeps ONE default capture stream per process, created on whichever device captured first:
                    # with engines on several GPUs in one process the capture stream has to be this device's own
                    # Python's cycle collector may run at any allocation; if it finalises an older model's graphs or
                    # tensors in the middle of the capture, their cudaFree invalidates it. Collect now, then keep the
                    # collector off until the capture has ended.
                    gc_was_on = gc.isenabled()
                    gc.collect()
                    gc.disable()
                    calls_before = ops.C_ABI_CALLS
                    try:
                        with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=self.m.device)):
                            e.left = self._step()
                    finally:
                        e.calls_per_step = ops.C_ABI_CALLS - calls_before
                        ops.C_ABI_CALLS = calls_before      # capturing records the launches without running them
                        if gc_was_on:
                            gc.enable()
                    e.graph = graph                  # capturing records the launches without running them
                return self._run_replayed()
            self.remaining = left.tolist()           # the one host read of a step
            self._known = list(self.remaining)
            return int(sum(self.remaining))

    def _enqueue_replay(self) -> None:
        """Replay the step and copy its MASK counts to pinned host memory behind it, without waiting."""
        e = self.e
        e.graph.replay()
        ops.C_ABI_CALLS += e.calls_per_step
        if e.host_counts is None:
            e.host_counts = torch.empty((2,) + tuple(e.left.shape), dtype=e.left.dtype, pin_memory=True)
        slot = self._slot
        self._slot ^= 1
        e.host_counts[slot].copy_(e.left, non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        self._pending.append((done, slot))

    def _run_replayed(self) -> int:
        """A replayed step, with the NEXT step already enqueued behind it when the block cannot finish in this one: launching a
        graph of a few hundred nodes and turning the host around take a fraction of a millisecond per step, during which the
        GPU would idle. A step on a block without MASK slots changes nothing, so a step enqueued in vain costs time only; it is
        enqueued only while more slots are left than four times the most any step of this block has filled."""
        e = self.e
        if not self._pending:
            self._enqueue_replay()
        if len(self._pending) < 2 and max(self._known) > 4 * self._most_filled:
            self._enqueue_replay()
        done, slot = self._pending.pop(0)
        done.synchronize()
        new = e.host_counts[slot].tolist()
        self._most_filled = max([self._most_filled] + [b - a for b, a in zip(self._known, new)])
        self._known = self.remaining = new
        return int(sum(new))
