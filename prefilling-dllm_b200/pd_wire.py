"""Wire format and layer-granular streaming of the prompt KV across the prefill/decode boundary.

The reference hands the KV of a prefilled prompt to the decode engine as an in-process `DreamKVSnapshot` of per-layer
tensors, copied layer by layer with blocking `.to()` calls after the prefill has finished
(prefilling_dllm_engine/prefilling_dllm/fastdllm_engine.py:700-781, 845-859); a serialised form and a transfer that
overlaps the prefill are listed as not yet released (README.md:186). This module supplies both:

  * `snapshot_to_bytes` / `snapshot_from_bytes`: one self-describing buffer for a whole snapshot;
  * `KVStreamWriter` / `KVStreamReader`: the same payload as a sequence of messages — HEADER, then groups of LAYERS, then
    TRAILER — produced WHILE the prefill runs. In the joint prefill the K/V rows of layer l are final as soon as layer l's
    page write has run, so the writer, called by the model after every layer, gathers that layer's pages on a side stream
    (ordered after the write by an event) into pinned host memory while the compute stream goes on with layer l + 1; the
    reader scatters each group into its own pages as it arrives, again on a side stream.

Layout of every message: 8-byte magic `PDKVWIRE`, 1-byte type, 4-byte little-endian length of a UTF-8 JSON header, the
header, then the raw payload (little-endian element bytes, K rows of a layer `[prompt_len, Hkv, D]` followed by its V rows,
layers in ascending order; the trailer's payload is the last-context logit). A CRC-32 of the payload is in the header.
"""

from __future__ import annotations

import json
import math
import struct
import zlib
from typing import Callable, Dict, List, Optional

import torch

MAGIC = b"PDKVWIRE"
TYPE_SNAPSHOT, TYPE_HEADER, TYPE_LAYERS, TYPE_TRAILER = 0, 1, 2, 3
_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _dtype_name(dtype: torch.dtype) -> str:
    for name, dt in _DTYPES.items():
        if dt == dtype:
            return name
    raise ValueError(f"unsupported KV dtype {dtype}")


def _raw(t: torch.Tensor) -> bytes:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()


def _tensor(buf: memoryview, dtype: torch.dtype, shape) -> torch.Tensor:
    flat = torch.frombuffer(bytearray(buf), dtype=torch.uint8)
    return flat.view(dtype).view(*shape)


def pack_message(kind: int, header: Dict, payload: bytes = b"") -> bytes:
    header = dict(header, payload_bytes=len(payload), crc32=zlib.crc32(payload) & 0xFFFFFFFF)
    head = json.dumps(header, separators=(",", ":")).encode("utf-8")
    return MAGIC + struct.pack("<BI", kind, len(head)) + head + payload


def unpack_message(message: bytes):
    """(type, header dict, payload memoryview); raises ValueError on a malformed or corrupted message."""
    view = memoryview(message)
    if len(view) < 13 or bytes(view[:8]) != MAGIC:
        raise ValueError("not a PD KV wire message")
    kind, head_len = struct.unpack("<BI", view[8:13])
    if 13 + head_len > len(view):
        raise ValueError("truncated PD KV wire message header")
    header = json.loads(bytes(view[13:13 + head_len]).decode("utf-8"))
    payload = view[13 + head_len:]
    if len(payload) != header.get("payload_bytes") or (zlib.crc32(payload) & 0xFFFFFFFF) != header.get("crc32"):
        raise ValueError("PD KV wire message payload is truncated or corrupted")
    return kind, header, payload


# ------------------------------------------------------------------------------------------------ whole snapshots
def snapshot_to_bytes(snapshot) -> bytes:
    """Serialise a DreamKVSnapshot (any device) into one buffer."""
    layers = len(snapshot.k_by_layer)
    shape, dtype = [0, 0, 0], "bfloat16"
    if layers:
        shape, dtype = list(snapshot.k_by_layer[0].shape), _dtype_name(snapshot.k_by_layer[0].dtype)
    logit = snapshot.last_context_logit
    header = dict(prompt_len=int(snapshot.prompt_len), page_size=int(snapshot.page_size), kv_mode=snapshot.kv_mode, layers=layers,
                  row_shape=shape[1:], dtype=dtype, logit_shape=None if logit is None else list(logit.shape),
                  logit_dtype=None if logit is None else _dtype_name(logit.dtype))
    parts: List[bytes] = []
    for k, v in zip(snapshot.k_by_layer, snapshot.v_by_layer):
        if list(k.shape) != shape or list(v.shape) != shape:
            raise ValueError("snapshot layers disagree in shape")
        parts += [_raw(k), _raw(v)]
    if logit is not None:
        parts.append(_raw(logit))
    return pack_message(TYPE_SNAPSHOT, header, b"".join(parts))


def snapshot_from_bytes(message: bytes, device="cpu"):
    from .engine import DreamKVSnapshot

    kind, header, payload = unpack_message(message)
    if kind != TYPE_SNAPSHOT:
        raise ValueError(f"expected a snapshot message, got type {kind}")
    dtype = _DTYPES[header["dtype"]]
    shape = [header["prompt_len"]] + list(header["row_shape"])
    per = math.prod(shape) * torch.empty((), dtype=dtype).element_size()
    ks, vs, off = [], [], 0
    for _ in range(header["layers"]):
        ks.append(_tensor(payload[off:off + per], dtype, shape).to(device))
        vs.append(_tensor(payload[off + per:off + 2 * per], dtype, shape).to(device))
        off += 2 * per
    logit = None
    if header["logit_shape"] is not None:
        logit = _tensor(payload[off:], _DTYPES[header["logit_dtype"]], header["logit_shape"]).to(device)
    return DreamKVSnapshot(prompt_len=header["prompt_len"], page_size=header["page_size"], kv_mode=header["kv_mode"], k_by_layer=ks,
                           v_by_layer=vs, last_context_logit=logit)


# ------------------------------------------------------------------------------------------------ streaming during the prefill
class KVStreamWriter:
    """Streams the prompt KV of ONE prefill, a group of layers per message, while the prefill is still running.

    Pass it to `FastDLLMDreamEngine.prefill_to_pd_record(..., kv_stream=writer)`: the engine announces the prompt pages
    (`begin`), the model calls `on_layer_stored(layer)` after each layer's page write, the engine ends with `finish(record)`.
    `sink(message: bytes)` receives the messages in order (it runs on the calling thread, when a group's copy has landed on
    the host: at the next group boundary or in `finish`). Full-dense records only: per-head compaction rewrites the pages
    after the prefill."""

    def __init__(self, engine, sink: Callable[[bytes], None], layers_per_message: int = 4):
        self.engine, self.sink, self.group = engine, sink, max(1, int(layers_per_message))
        self.stream = torch.cuda.Stream(device=engine.device)
        self.pending: List[tuple] = []      # (first layer, count, pinned host tensor, event)
        self.page_ids: Optional[List[int]] = None
        self.prompt_len = 0
        self.bytes_sent = 0

    def begin(self, *, prompt_page_ids, prompt_len: int, header: Dict) -> None:
        self.page_ids, self.prompt_len = list(prompt_page_ids), int(prompt_len)
        kv = self.engine.model.kv_cache
        self._emit(pack_message(TYPE_HEADER, dict(header, prompt_len=self.prompt_len, page_size=int(self.engine.page_size), layers=int(kv.shape[1]),
                                                  row_shape=[int(kv.shape[4]), int(kv.shape[5])], dtype=_dtype_name(kv.dtype))))

    def _emit(self, message: bytes) -> None:
        self.bytes_sent += len(message)
        self.sink(message)

    def on_layer_stored(self, layer: int) -> None:
        """Called on the compute stream right after layer `layer` wrote its K/V rows into pages."""
        kv = self.engine.model.kv_cache
        layers = int(kv.shape[1])
        if self.page_ids is None or ((layer + 1) % self.group != 0 and layer + 1 != layers):
            return
        first = (layer // self.group) * self.group
        count = layer + 1 - first
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(self.engine.device))
        from . import ops

        n_pages = math.ceil(self.prompt_len / self.engine.page_size)
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(done)                     # the group's page writes are complete
            pages = int(kv.shape[2])
            base = torch.tensor(self.page_ids[:n_pages], dtype=torch.int32, device=self.engine.device)
            # (k|v, layer) planes of this group in the pool seen as 2 * layers * pages pages: [layer][k, v]
            planes = torch.tensor([p * layers + l for l in range(first, first + count) for p in (0, 1)], dtype=torch.int32, device=self.engine.device)
            ids = (planes.view(-1, 1) * pages + base.view(1, -1)).reshape(-1).contiguous()
            dense = ops.gather_pages(self.engine._layer_pools(), ids, int(ids.numel()) * self.engine.page_size)
            dense = dense.view(count, 2, n_pages * self.engine.page_size, kv.shape[4], kv.shape[5])[:, :, :self.prompt_len]
            host = torch.empty(dense.shape, dtype=dense.dtype, pin_memory=True)
            host.copy_(dense, non_blocking=True)
            landed = torch.cuda.Event()
            landed.record(self.stream)
        self._flush(wait_all=False)
        self.pending.append((first, count, host, landed))

    def _flush(self, wait_all: bool) -> None:
        while self.pending and (wait_all or self.pending[0][3].query()):
            first, count, host, landed = self.pending.pop(0)
            landed.synchronize()
            self._emit(pack_message(TYPE_LAYERS, dict(first_layer=first, count=count), host.view(torch.uint8).numpy().tobytes()))

    def finish(self, record) -> None:
        self._flush(wait_all=True)
        logit = record.last_context_logit
        header = dict(first_token_id=int(record.first_token_id), logit_shape=None if logit is None else list(logit.shape),
                      logit_dtype=None if logit is None else _dtype_name(logit.dtype))
        self._emit(pack_message(TYPE_TRAILER, header, b"" if logit is None else _raw(logit)))
        self.page_ids = None


class KVStreamReader:
    """Receiving side: feed it the writer's messages in order; after the TRAILER `record` is a decode-ready
    DreamPrefillRecord on `engine` (pages allocated at the HEADER, every group scattered into them as it arrives)."""

    def __init__(self, engine):
        self.engine = engine
        self.stream = torch.cuda.Stream(device=engine.device)
        self.header: Optional[Dict] = None
        self.prompt_pages: List[int] = []
        self.block_pages: List[int] = []
        self.layers_seen = 0
        self.record = None
        self._keep: List[torch.Tensor] = []

    def feed(self, message: bytes) -> None:
        from . import ops
        from .engine import DreamPrefillRecord

        kind, header, payload = unpack_message(message)
        eng = self.engine
        kv = eng.model.kv_cache
        if kind == TYPE_HEADER:
            if header["page_size"] != eng.page_size:
                raise ValueError(f"PD KV stream page_size mismatch: stream={header['page_size']}, engine={eng.page_size}")
            if header["layers"] != int(kv.shape[1]) or header["row_shape"] != [int(kv.shape[4]), int(kv.shape[5])] or _DTYPES[header["dtype"]] != kv.dtype:
                raise ValueError("PD KV stream does not match this engine's model (layers / KV heads / head_dim / dtype)")
            if header.get("kv_mode", "full_dense") != "full_dense":
                raise ValueError("PD KV streams carry full_dense records only")
            self.header = header
            self.prompt_pages, self.block_pages = eng._allocate_prompt_and_block_pages(header["prompt_len"], header["decode_len"])
            self.layers_seen = 0
            return
        if self.header is None:
            raise ValueError("PD KV stream: message before the header")
        try:
            if kind == TYPE_LAYERS:
                first, count = int(header["first_layer"]), int(header["count"])
                if first != self.layers_seen:
                    raise ValueError(f"PD KV stream: expected layer {self.layers_seen}, got {first}")
                prompt_len, page = int(self.header["prompt_len"]), eng.page_size
                n_pages = math.ceil(prompt_len / page)
                shape = (count, 2, prompt_len, int(kv.shape[4]), int(kv.shape[5]))
                host = _tensor(payload, kv.dtype, shape).pin_memory()
                layers, pages = int(kv.shape[1]), int(kv.shape[2])
                with torch.cuda.device(eng.device), torch.cuda.stream(self.stream):
                    staged = torch.zeros((count, 2, n_pages * page) + shape[3:], dtype=kv.dtype, device=eng.device)
                    staged[:, :, :prompt_len].copy_(host, non_blocking=True)
                    base = torch.tensor(self.prompt_pages[:n_pages], dtype=torch.int32, device=eng.device)
                    planes = torch.tensor([p * layers + l for l in range(first, first + count) for p in (0, 1)], dtype=torch.int32, device=eng.device)
                    ids = (planes.view(-1, 1) * pages + base.view(1, -1)).reshape(-1).contiguous()
                    ops.scatter_pages(staged.view(-1, shape[3], shape[4]), eng._layer_pools(), ids)
                self._keep += [host, staged]      # alive until the stream has consumed them
                self.layers_seen += count
            elif kind == TYPE_TRAILER:
                if self.layers_seen != int(self.header["layers"]):
                    raise ValueError(f"PD KV stream ended after {self.layers_seen} of {self.header['layers']} layers")
                torch.cuda.current_stream(eng.device).wait_stream(self.stream)      # decode is ordered after the scatters
                self.stream.synchronize()
                self._keep = []
                logit = None
                if header["logit_shape"] is not None:
                    logit = _tensor(payload, _DTYPES[header["logit_dtype"]], header["logit_shape"]).to(eng.device)
                h = self.header
                self.record = DreamPrefillRecord(
                    prompt_ids=list(h["prompt_ids"]), prompt_positions=list(h["prompt_positions"]), suffix_positions=list(h["suffix_positions"]),
                    prompt_len=int(h["prompt_len"]), full_prompt_len=int(h["full_prompt_len"]), decode_len=int(h["decode_len"]),
                    prompt_page_ids=self.prompt_pages, block_page_ids=self.block_pages, first_token_id=int(header["first_token_id"]),
                    last_context_logit=logit, decode_delta_state=None, owns_prompt_pages=True, cached_prefix=None, kv_mode="full_dense")
                self.header = None
            else:
                raise ValueError(f"PD KV stream: unexpected message type {kind}")
        except BaseException:
            eng._prefix_cache.release_pages(self.prompt_pages + self.block_pages)
            self.header, self.prompt_pages, self.block_pages = None, [], []
            raise
