"""qtts_lm_forward_noalloc checked against qtts_lm_forward.

Some programs that call this library may not allocate GPU memory while they
run the model: a real-time synthesis thread cannot afford cudaMalloc/cudaFree,
which can stall the whole device, and some host applications hand out all
GPU memory from their own pool allocator.  For them, qtts_lm_forward_noalloc
runs the same forward on device buffers they own, with the kernel's scratch
in one static device array.

Two lms get the same seeded weights and the same rows; one goes through
qtts_lm_forward (host buffers), the other through the no-allocation entry
(device buffers), on two calls in a row (6 rows, then 1 row), with f32 and
with Q8_0 weights.  Logits and normed states must agree within the
tolerances of the parity tests (1e-4 for f32, 2e-2 for Q8_0).  A warm call
must leave the device's free memory unchanged; calls without a head or a
state use the array's own slots; misaligned buffers and sizes beyond the
array are refused before anything runs.  The file name makes pytest collect
it last.
"""
import numpy as np
import pytest

import qtts
import synth

pytestmark = pytest.mark.gpu

ATOL = {"f32": 1e-4, "q8_0": 2e-2}  # the logits tolerances of tests/test_gpu_parity.py


def _pair(device, dtype, seed=71, max_pos=64):
    layers, final = synth.stack(seed, "talker", 2)
    heads = qtts.QwenLmHeads(device, "talker", synth.HIDDEN, dtype)
    heads.add(synth.talker_head(seed))
    ref = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, layers, final, dtype), heads, max_pos)
    lm = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, layers, final, dtype), heads, max_pos)
    return heads, ref, lm


@pytest.mark.parametrize("dtype", ["f32", "q8_0"])
def test_noalloc_forward_matches_forward(device, dtype):
    torch = pytest.importorskip("torch")
    heads, ref, lm = _pair(device, dtype)
    rows = synth.prompt(71, 9)
    dev = torch.device("cuda", 0)
    logits_dev = torch.full((3072,), float("nan"), dtype=torch.float32, device=dev)
    hidden_dev = torch.full((1024,), float("nan"), dtype=torch.float32, device=dev)
    lr, hr = np.zeros(3072, np.float32), np.zeros(1024, np.float32)
    try:
        for a, b in ((0, 6), (6, 7)):
            ref.forward(rows[a:b], output=0, logits=lr, hidden=hr)
            x_dev = torch.from_numpy(np.ascontiguousarray(rows[a:b])).to(dev)
            torch.cuda.synchronize()  # the library's stream does not wait for torch's
            free0 = torch.cuda.mem_get_info(dev)[0]
            lm.forward_noalloc(x_dev.data_ptr(), b - a, 0, logits_dev.data_ptr(), hidden_dev.data_ptr())
            if a > 0:  # a warm call: the device's free memory is what it was
                assert torch.cuda.mem_get_info(dev)[0] == free0
            ln, hn = logits_dev.cpu().numpy(), hidden_dev.cpu().numpy()
            assert np.abs(ln - lr).max() <= ATOL[dtype], (a, b, np.abs(ln - lr).max())
            assert np.abs(hn - hr).max() <= ATOL[dtype], (a, b, np.abs(hn - hr).max())
            assert int(np.argmax(ln)) == int(np.argmax(lr))
            assert lm.length == ref.length == b
        # no head, no state: the rows still go into the cache (the array's
        # own slots take the outputs), and the next call sees them
        ref.forward(rows[7:8])
        x_dev = torch.from_numpy(np.ascontiguousarray(rows[7:8])).to(dev)
        torch.cuda.synchronize()
        lm.forward_noalloc(x_dev.data_ptr(), 1, 0, None, None)
        ref.forward(rows[8:9], output=0, logits=lr, hidden=hr)
        x_dev = torch.from_numpy(np.ascontiguousarray(rows[8:9])).to(dev)
        torch.cuda.synchronize()
        lm.forward_noalloc(x_dev.data_ptr(), 1, 0, logits_dev.data_ptr(), None)
        ln = logits_dev.cpu().numpy()
        assert np.abs(ln - lr).max() <= ATOL[dtype]
        assert lm.length == ref.length == 9
    finally:
        lm.free()
        ref.free()
        heads.free()


def test_noalloc_refusals(device):
    # checked on the host, before any launch: the lm's length is unchanged
    torch = pytest.importorskip("torch")
    heads, ref, lm = _pair(device, "f32", max_pos=8)
    dev = torch.device("cuda", 0)
    x = torch.zeros((16, 1024), dtype=torch.float32, device=dev)
    out = torch.zeros(3072 + 8, dtype=torch.float32, device=dev)
    try:
        with pytest.raises(qtts.EQwenLm) as e:  # x off the 16-byte boundary
            lm.forward_noalloc(x.data_ptr() + 4, 1, 0, out.data_ptr(), None)
        assert e.value.code == qtts.E_ARG
        with pytest.raises(qtts.EQwenLm) as e:  # logits off the boundary
            lm.forward_noalloc(x.data_ptr(), 1, 0, out.data_ptr() + 4, None)
        assert e.value.code == qtts.E_ARG
        with pytest.raises(qtts.EQwenLm) as e:  # past the cache
            lm.forward_noalloc(x.data_ptr(), 9, 0, out.data_ptr(), None)
        assert e.value.code == qtts.E_CAPACITY
        assert lm.length == 0
    finally:
        lm.free()
        ref.free()
        heads.free()
    # a head wider than the array's logits slot (4096 rows)
    big = qtts.QwenLmHeads(device, "wide", synth.HIDDEN, "f32")
    big.add(synth.normal((4160, 1024), 0.02, 9, 9))
    layers, final = synth.stack(72, "talker", 1)
    lm = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, layers, final, "f32"), big, 8)
    wide = torch.zeros(4160, dtype=torch.float32, device=dev)
    try:
        with pytest.raises(qtts.EQwenLm) as e:
            lm.forward_noalloc(x.data_ptr(), 1, 0, wide.data_ptr(), None)
        assert e.value.code == qtts.E_CAPACITY
        assert lm.length == 0
    finally:
        lm.free()
        big.free()
