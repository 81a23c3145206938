"""TQwenTalker.TextProject (talker.pas:390-421) in the oracle against a
float64 numpy statement of the same formula: y = fc2(silu(fc1(e))) with
biases, silu written as the reference writes it (0 below -80)."""
import numpy as np

import oracle as O


def ref(emb, ids, w1, b1, w2, b2):
    e = emb[ids].astype(np.float64)
    h = e @ w1.T.astype(np.float64) + b1
    h = np.where(h < -80.0, 0.0, h / (1.0 + np.exp(-np.clip(h, -80.0, None))))
    return h @ w2.T.astype(np.float64) + b2


def weights(seed, vocab=300, th=256, hidden=128):
    rng = np.random.default_rng(seed)
    emb = rng.standard_normal((vocab, th)).astype(np.float32)
    w1 = (rng.standard_normal((th, th)) * 0.05).astype(np.float32)
    b1 = (rng.standard_normal(th) * 0.1).astype(np.float32)
    w2 = (rng.standard_normal((hidden, th)) * 0.05).astype(np.float32)
    b2 = (rng.standard_normal(hidden) * 0.1).astype(np.float32)
    return emb, w1, b1, w2, b2


def test_oracle_text_project_matches_formula():
    emb, w1, b1, w2, b2 = weights(1)
    ids = np.array([0, 5, 299, 17, 17], np.int32)
    y = O.text_project(emb, ids, w1, b1, w2, b2)
    r = ref(emb, ids, w1, b1, w2, b2)
    assert np.abs(y - r).max() <= 1e-4 * (1 + np.abs(r).max())
    assert np.array_equal(y[3], y[4])


def test_silu_cut_below_minus_80():
    emb, w1, b1, w2, b2 = weights(2)
    b1[:] = -200.0  # every fc1 output far below -80: silu gives 0, y = b2
    y = O.text_project(emb, np.array([3], np.int32), w1, b1, w2, b2)
    assert np.array_equal(y[0], b2)
