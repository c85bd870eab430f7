"""The entry point that brings its own scratch must give exactly what the workspace-taking entry point gives.

Some callers of the unmask step cannot pass device scratch: they have committed all the device memory they may use
(typically to the KV page pool) and must not allocate once the decode loop runs, or they sit behind an interface
that only carries inputs and outputs. pdllm_unmask_step_static serves them from an array inside the library. This
file is collected last on purpose, so a failure here cannot hide another test's result in a run that stops at the
first failure. It calls both entry points through the C-ABI (ctypes), twice in a row, and compares the outputs bit
for bit (ids and counts are integers; the confidences come from the same kernel on the same inputs).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(lib, fn_name, logits, last, ids, mask_id, threshold, conf_dtype, workspace=None):
    dev = logits.device
    block_len, vocab = logits.shape
    counts = torch.full((3,), -1, dtype=torch.int32, device=dev)
    conf = torch.empty(block_len, dtype=torch.float32, device=dev)
    x0 = torch.empty(block_len, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    args = [logits.data_ptr(), logits.stride(0), last.data_ptr(), 0 if logits.dtype == torch.float32 else 1, block_len, vocab, 1,
            ids.data_ptr(), mask_id, threshold, conf_dtype, counts.data_ptr(), conf.data_ptr(), x0.data_ptr()]
    if workspace is not None:
        args += [workspace.data_ptr(), workspace.numel()]
    args.append(stream)
    rc = getattr(lib, fn_name)(*args)
    return rc, counts, conf, x0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_static_scratch_entry_matches_workspace_entry(cuda_device, dtype):
    from prefilling_dllm_b200 import _lib

    lib = _lib.load()
    g = torch.Generator().manual_seed(123)
    block_len, vocab, mask_id = 32, 9001, 9000
    conf_dtype = 0 if dtype == torch.float32 else 1
    ws_bytes = int(lib.pdllm_unmask_workspace_bytes(block_len))
    workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda_device)
    for call in range(2):  # two calls in a row: the second one finds the first one's leftovers in the shared array
        logits = (torch.randn(block_len, vocab, generator=g) * 3).to(dtype).to(cuda_device)
        logits[5, 77] = 40.0  # two slots far above the threshold, so more than the always-accepted top slot is filled
        logits[8, 99] = 40.0
        last = torch.randn(vocab, generator=g).to(dtype).to(cuda_device)
        ids = torch.full((block_len,), mask_id, dtype=torch.int64)
        ids[0] = 3
        ids[10 + call] = 4
        ids_a, ids_b = ids.to(cuda_device), ids.to(cuda_device)
        rc_a, counts_a, conf_a, x0_a = _call(lib, "pdllm_unmask_step", logits, last, ids_a, mask_id, 0.9, conf_dtype, workspace)
        rc_b, counts_b, conf_b, x0_b = _call(lib, "pdllm_unmask_step_static", logits, last, ids_b, mask_id, 0.9, conf_dtype)
        torch.cuda.synchronize(cuda_device)
        assert rc_a == 0 and rc_b == 0, _lib.last_error()
        assert torch.equal(ids_a, ids_b), call
        assert torch.equal(counts_a, counts_b) and int(counts_b[1]) >= 2, call
        assert torch.equal(x0_a, x0_b), call
        assert torch.equal(conf_a, conf_b), call


def test_static_scratch_entry_rejects_blocks_beyond_its_limit(cuda_device):
    from prefilling_dllm_b200 import _lib

    lib = _lib.load()
    block_len, vocab = 65, 128  # the built-in scratch holds 64 slots
    logits = torch.zeros(block_len, vocab, device=cuda_device)
    last = torch.zeros(vocab, device=cuda_device)
    ids = torch.zeros(block_len, dtype=torch.int64, device=cuda_device)
    rc, _, _, _ = _call(lib, "pdllm_unmask_step_static", logits, last, ids, 1, 0.9, 0)
    assert rc == _lib.E_INVALID
    assert "exceeds the built-in scratch" in _lib.last_error()
