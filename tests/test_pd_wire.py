"""Wire format of the prompt KV (prefilling_dllm_b200.pd_wire): whole snapshots and stream messages, on CPU tensors."""

import pytest
import torch

from prefilling_dllm_b200 import pd_wire
from prefilling_dllm_b200.engine import DreamKVSnapshot


def _snapshot(dtype, with_logit=True, layers=3, prompt_len=37):
    g = torch.Generator().manual_seed(1)
    ks = [torch.randn(prompt_len, 2, 64, generator=g).to(dtype) for _ in range(layers)]
    vs = [torch.randn(prompt_len, 2, 64, generator=g).to(dtype) for _ in range(layers)]
    logit = torch.randn(1024, generator=g).to(dtype) if with_logit else None
    return DreamKVSnapshot(prompt_len=prompt_len, page_size=256, kv_mode="full_dense", k_by_layer=ks, v_by_layer=vs, last_context_logit=logit)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_snapshot_round_trip_is_bit_exact(dtype):
    snap = _snapshot(dtype)
    back = pd_wire.snapshot_from_bytes(pd_wire.snapshot_to_bytes(snap))
    assert (back.prompt_len, back.page_size, back.kv_mode) == (snap.prompt_len, snap.page_size, snap.kv_mode)
    for a, b in zip(snap.k_by_layer + snap.v_by_layer, back.k_by_layer + back.v_by_layer):
        assert a.dtype == b.dtype and torch.equal(a, b)
    assert torch.equal(snap.last_context_logit, back.last_context_logit)


def test_empty_prompt_and_missing_logit():
    snap = _snapshot(torch.bfloat16, with_logit=False, layers=0, prompt_len=0)
    back = pd_wire.snapshot_from_bytes(pd_wire.snapshot_to_bytes(snap))
    assert back.k_by_layer == [] and back.v_by_layer == [] and back.last_context_logit is None and back.prompt_len == 0


def test_corruption_and_truncation_are_detected():
    msg = bytearray(pd_wire.snapshot_to_bytes(_snapshot(torch.bfloat16)))
    msg[-7] ^= 0x40
    with pytest.raises(ValueError, match="corrupted"):
        pd_wire.snapshot_from_bytes(bytes(msg))
    good = pd_wire.snapshot_to_bytes(_snapshot(torch.bfloat16))
    with pytest.raises(ValueError, match="truncated or corrupted"):
        pd_wire.snapshot_from_bytes(good[:-10])
    with pytest.raises(ValueError, match="not a PD KV wire message"):
        pd_wire.snapshot_from_bytes(b"hello world, this is not it")
    kind, header, payload = pd_wire.unpack_message(pd_wire.pack_message(pd_wire.TYPE_LAYERS, dict(first_layer=4, count=2), b"\x01\x02\x03"))
    assert kind == pd_wire.TYPE_LAYERS and header["first_layer"] == 4 and bytes(payload) == b"\x01\x02\x03"
    with pytest.raises(ValueError, match="expected a snapshot"):
        pd_wire.snapshot_from_bytes(pd_wire.pack_message(pd_wire.TYPE_TRAILER, {}, b""))
