"""The failure path of the bounded device waits, on the GPU, without a fault.

Every spin of the batch-1 kernel is bounded and gives up with an error word
that the host reads (the reference bounds its waits and aborts cleanly,
mormot.ai.tts.qwen.pas:541-548).  qtts_lm_set_wait_test makes the grid
barriers of the next launches wait for one arrival more than the grid has --
a flag that nothing sets -- with a short bound (2e7 SM cycles, ~10 ms), so
the wait runs out on its own: the call must return QTTS_E_TIMEOUT naming
where it gave up, append no position, and leave the lm (its KV cache and the
barrier counters) fit for the next call, whose results must match the oracle.
Nothing traps or hangs: the kernel returns by itself and the context stays
usable.
"""
import numpy as np
import pytest

import qtts
import synth
from model_util import Pair, TalkerPair

pytestmark = pytest.mark.gpu

SHORT = 20_000_000  # SM cycles: about 10 ms at 1.9 GHz


def test_forward_wait_runs_out_then_recovers(device):
    pr = Pair(device, 91, "talker", 2, [synth.talker_head(91)], "f32", max_pos=32)
    try:
        x = synth.prompt(91, 7)
        ld, lo = np.zeros(3072, np.float32), np.zeros(3072, np.float32)
        pr.dev.forward(x[:5], output=0, logits=ld)
        pr.ora.forward(x[:5], 0, lo)
        pr.dev.set_wait_test(1, SHORT)
        with pytest.raises(qtts.EQwenLm) as e:
            pr.dev.forward(x[5:6], output=0, logits=ld)
        assert e.value.code == qtts.E_TIMEOUT
        assert "gave up" in str(e.value)
        assert pr.dev.length == 5  # nothing appended
        # twice in a row: the counters were cleared after the first
        with pytest.raises(qtts.EQwenLm) as e:
            pr.dev.forward(x[5:6], output=0, logits=ld)
        assert e.value.code == qtts.E_TIMEOUT
        pr.dev.set_wait_test(0, 0)
        for r in (5, 6):
            pr.dev.forward(x[r:r + 1], output=0, logits=ld)
            pr.ora.forward(x[r:r + 1], 0, lo)
            assert np.abs(ld - lo).max() <= 1e-4
        assert pr.dev.length == 7
    finally:
        pr.free()


def test_frame_wait_runs_out_then_recovers(device):
    # the frame kernel (one cooperative launch per NextFrame): the failed
    # frame returns no codes; the retried frame is the oracle's frame
    tp = TalkerPair(device, 93, 2, 2, "q8_0", max_pos=64)
    try:
        tp.start(synth.prompt(93, 6), synth.text_rows(93, 2), synth.text_rows(93, 1, key=1)[0])
        cd, co = np.zeros(16, np.int32), np.zeros(16, np.int32)
        assert tp.dev.next_frame(cd) and tp.ora.next_frame(co)
        assert np.array_equal(cd, co)
        tp.t.dev.set_wait_test(1, SHORT)
        with pytest.raises(qtts.EQwenLm) as e:
            tp.dev.next_frame(cd)
        assert e.value.code == qtts.E_TIMEOUT
        assert tp.dev.step == 1
        tp.t.dev.set_wait_test(0, 0)
        for _ in range(2):
            assert tp.dev.next_frame(cd) and tp.ora.next_frame(co)
            assert np.array_equal(cd, co)
        assert tp.dev.step == 3
    finally:
        tp.free()
