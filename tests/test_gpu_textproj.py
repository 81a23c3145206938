"""TQwenTalker.TextProject (talker.pas:390-421) on the device
(qtts_textproj_*) against the oracle, at the real widths (text hidden 2048,
hidden 1024), with a float32 and a BF16 embedding table."""
import numpy as np
import pytest

import oracle as O
import qtts

pytestmark = pytest.mark.gpu


def weights(seed, vocab=2000, th=2048, hidden=1024):
    rng = np.random.default_rng(seed)
    emb = (rng.standard_normal((vocab, th)) * 0.05).astype(np.float32)
    w1 = (rng.standard_normal((th, th)) * 0.02).astype(np.float32)
    b1 = (rng.standard_normal(th) * 0.02).astype(np.float32)
    w2 = (rng.standard_normal((hidden, th)) * 0.02).astype(np.float32)
    b2 = (rng.standard_normal(hidden) * 0.02).astype(np.float32)
    return emb, w1, b1, w2, b2


@pytest.mark.parametrize("table", ["f32", "bf16"])
def test_text_project_matches_oracle(device, table):
    emb, w1, b1, w2, b2 = weights(3)
    if table == "bf16":
        bits = (emb.view(np.uint32) >> 16).astype(np.uint16)  # truncated to BF16
        emb_dev, emb_ora = bits, (bits.astype(np.uint32) << 16).view(np.float32)
    else:
        emb_dev, emb_ora = emb, emb
    tp = qtts.QwenTextProject(device, emb_dev, w1, b1, w2, b2)
    for ids in ([0, 1, 1999], list(range(100, 140)), [7]):
        y = tp.project(ids)
        o = O.text_project(emb_ora, ids, w1, b1, w2, b2)
        assert y.shape == (len(ids), 1024)
        assert np.abs(y - o).max() <= 2e-5 + 1e-5 * np.abs(o).max(), np.abs(y - o).max()
    with pytest.raises(qtts.EQwenLm):
        tp.project([2000])
    with pytest.raises(qtts.EQwenLm):
        tp.project([-1])
    tp.free()
