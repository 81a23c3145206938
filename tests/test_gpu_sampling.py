"""The sampling mode on the device (qtts_sample, qtts_talker_set_sampling)
against the oracle's restated TInferSampler (talker.pas:626-629, 632-638):
the same draw on the same values, and the frame loop with sampling giving
the same codes frame by frame."""
import numpy as np
import pytest

import oracle as O
import synth
from model_util import TalkerPair

pytestmark = pytest.mark.gpu


def test_device_draw_matches_oracle(device):
    rng = np.random.default_rng(5)
    cases = 0
    for n, T, k, p in [(2048, 0.9, 50, 1.0), (3072, 1.0, 64, 0.8), (2048, 0.5, 1, 1.0), (3072, 1.3, 20, 0.95),
                       (700, 0.9, 50, 0.3)]:
        for trial in range(30):
            lg = (rng.standard_normal(n) * rng.uniform(0.5, 4.0)).astype(np.float32)
            if n == 3072:
                lg[2048:] = -np.inf  # ChooseCode0's forbidden control ids
            seed, step, group = int(rng.integers(1 << 62)), trial, trial % 16
            d = device.sample(lg, T, k, p, seed, step, group)
            o = O.sample(lg, T, k, p, O.sample_uniform(seed, step, group))
            assert d == o, (n, T, k, p, trial)
            cases += 1
    assert cases == 150


def test_sampling_arguments_are_checked(device):
    import qtts
    lg = np.zeros(16, np.float32)
    for T, k, p in [(0.0, 5, 1.0), (1.0, 0, 1.0), (1.0, 65, 1.0), (1.0, 5, 0.0), (1.0, 5, 1.5)]:
        with pytest.raises(qtts.EQwenLm):
            device.sample(lg, T, k, p)


@pytest.mark.parametrize("dtype", ["f32", "q8_0"])
def test_sampled_frames_match_oracle(device, dtype):
    # NextFrame in sampling mode (the qwen_tts defaults: temperature 0.9,
    # top_k 50, both choosers), the same seed on both sides: the same codes
    # frame by frame, the first code 0 drawn at start included
    tp = TalkerPair(device, 81, 2, 2, dtype)
    tp.dev.set_sampling(seed=1234)
    tp.ora.set_sampling(seed=1234)
    tp.start(synth.prompt(81, 10), synth.text_rows(81, 2), synth.text_rows(81, 1, key=1)[0])
    cd, co = np.zeros(16, np.int32), np.zeros(16, np.int32)
    for f in range(8):
        md, mo = tp.dev.next_frame(cd), tp.ora.next_frame(co)
        assert md == mo
        if not md:
            break
        assert np.array_equal(cd, co), (f, cd, co)
    tp.free()


def test_sampling_seed_changes_the_codes(device):
    def frames(seed):
        tp = TalkerPair(device, 82, 1, 1, "f32")
        tp.dev.set_sampling(seed=seed)
        tp.start(synth.prompt(82, 6), None, synth.text_rows(82, 1)[0])
        out = tp.dev.run(4)
        tp.free()
        return out

    a, b, c = frames(7), frames(7), frames(8)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)
