"""qtts_lm_forward_noalloc checked against qtts_lm_forward.

Some programs that call this library may not allocate GPU memory while they
run the model: a real-time synthesis thread cannot afford cudaMalloc/cudaFree,
which can stall the whole device, and some host applications hand out all
GPU memory from their own pool allocator.  For them, qtts_lm_forward_noalloc
runs the same forward on device buffers they own, with the kernel's scratch
in one static device array.

Two lms get the same seeded weights and the same rows; one goes through
qtts_lm_forward (host buffers), the other through the no-allocation entry
(device buffers), on two calls in a row (6 rows, then 1 row).  Logits and
normed states must agree within the f32 tolerance of the parity tests.  The
file name makes pytest collect it last.
"""
import numpy as np
import pytest

import qtts
import synth

pytestmark = pytest.mark.gpu

F32_ATOL = 1e-4  # the f32 logits tolerance of tests/test_gpu_parity.py


def test_noalloc_forward_matches_forward(device):
    torch = pytest.importorskip("torch")
    layers, final = synth.stack(71, "talker", 2)
    heads = qtts.QwenLmHeads(device, "talker", synth.HIDDEN, "f32")
    heads.add(synth.talker_head(71))
    ref = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, layers, final, "f32"), heads, 64)
    lm = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, layers, final, "f32"), heads, 64)
    rows = synth.prompt(71, 7)
    dev = torch.device("cuda", 0)
    logits_dev = torch.full((3072,), float("nan"), dtype=torch.float32, device=dev)
    hidden_dev = torch.full((1024,), float("nan"), dtype=torch.float32, device=dev)
    lr, hr = np.zeros(3072, np.float32), np.zeros(1024, np.float32)
    for a, b in ((0, 6), (6, 7)):
        ref.forward(rows[a:b], output=0, logits=lr, hidden=hr)
        x_dev = torch.from_numpy(np.ascontiguousarray(rows[a:b])).to(dev)
        torch.cuda.synchronize()  # the library's stream does not wait for torch's
        lm.forward_noalloc(x_dev.data_ptr(), b - a, 0, logits_dev.data_ptr(), hidden_dev.data_ptr())
        ln, hn = logits_dev.cpu().numpy(), hidden_dev.cpu().numpy()
        assert np.abs(ln - lr).max() <= F32_ATOL, (a, b, np.abs(ln - lr).max())
        assert np.abs(hn - hr).max() <= F32_ATOL, (a, b, np.abs(hn - hr).max())
        assert int(np.argmax(ln)) == int(np.argmax(lr))
        assert lm.length == ref.length == b
    lm.free()
    ref.free()
    heads.free()
