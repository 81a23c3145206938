"""The sampling mode of TQwenTalker's choices (TQwenSampling, talker.pas:
60-73; the draw of talker.pas:626-629 and 632-638) in the oracle: the
restated TInferSampler (oracle/qtts_oracle.c) against its definition --
temperature, top-k with ties, the top-p nucleus, the inverse-CDF draw --
and the counter-based uniform stream.  The reference's sampler lives in the
absent mormot2-ai submodule, so these are properties of the restatement, not
golden vectors of the reference (its random stream is not reproducible)."""
import numpy as np

import oracle as O


def softmax(z):
    e = np.exp(z - z.max())
    return e / e.sum()


def draws(logits, n, temperature=1.0, top_k=50, top_p=1.0, seed=5):
    return np.array([O.sample(logits, temperature, top_k, top_p, O.sample_uniform(seed, s, 3)) for s in range(n)])


def test_uniform_stream_is_a_function_of_the_counter():
    u = [O.sample_uniform(9, s, g) for s in range(40) for g in range(16)]
    assert all(0.0 <= v < 1.0 for v in u)
    assert len(set(u)) == len(u)  # no repeats in a short stream
    assert O.sample_uniform(9, 3, 4) == O.sample_uniform(9, 3, 4)
    assert O.sample_uniform(9, 3, 4) != O.sample_uniform(10, 3, 4)
    # roughly uniform
    big = np.array([O.sample_uniform(1, s, 0) for s in range(20000)])
    assert abs(big.mean() - 0.5) < 0.01 and abs((big < 0.25).mean() - 0.25) < 0.01


def test_top_k_one_is_the_maximum_and_ties_are_kept():
    rng = np.random.default_rng(1)
    lg = rng.standard_normal(2048).astype(np.float32)
    for s in range(20):
        assert O.sample(lg, 0.9, 1, 1.0, O.sample_uniform(2, s, 0)) == int(np.argmax(lg))
    # values equal to the top_k-th largest stay (transformers' TopK keeps
    # ties): both halves of a tie at the maximum are drawn
    lg[700] = lg[1500] = lg.max() + 1.0
    assert set(O.sample(lg, 0.9, 1, 1.0, O.sample_uniform(2, s, 0)) for s in range(200)) == {700, 1500}


def test_distribution_is_the_top_k_softmax():
    rng = np.random.default_rng(2)
    lg = (rng.standard_normal(3072) * 2).astype(np.float32)
    T, k, n = 0.9, 50, 30000
    d = draws(lg, n, T, k)
    top = np.argsort(-lg, kind="stable")[:k]
    assert set(d) <= set(top)  # nothing outside the top k
    p = softmax(lg[top].astype(np.float64) / T)
    emp = np.array([(d == i).sum() for i in top]) / n
    assert np.abs(emp - p).max() < 4.0 * np.sqrt(p.max() / n) + 1e-3


def test_top_p_keeps_the_nucleus():
    lg = (-30.0 - 0.01 * np.arange(2048)).astype(np.float32)  # distinct: no ties at the top-k threshold
    lg[[10, 20, 30, 40]] = np.log(np.array([0.5, 0.3, 0.15, 0.05], np.float32))
    # mass before 10: 0, before 20: .5, before 30: .8, before 40: .95
    assert set(draws(lg, 400, 1.0, 50, 0.5)) == {10}
    assert set(draws(lg, 400, 1.0, 50, 0.75)) == {10, 20}
    assert set(draws(lg, 2000, 1.0, 50, 0.9)) == {10, 20, 30}
    assert 40 in set(draws(lg, 4000, 1.0, 4, 1.0))


def test_forbidden_values_are_never_drawn_and_temperature_sharpens():
    rng = np.random.default_rng(3)
    lg = rng.standard_normal(3072).astype(np.float32)
    lg[2048:] = -np.inf  # ChooseCode0's control ids
    d = draws(lg, 3000, 1.0, 64)
    assert d.max() < 2048
    cold = draws(lg, 3000, 0.05, 64)
    assert (cold == int(np.argmax(lg))).mean() > 0.9
    allinf = np.full(100, -np.inf, np.float32)
    assert O.sample(allinf, 1.0, 10, 1.0, 0.3) == 0
    # more ties at the threshold than the 128 candidates kept: the first maximum
    flat = np.zeros(1000, np.float32)
    flat[500] = 1.0
    assert O.sample(flat, 1.0, 10, 1.0, 0.3) == 500


def test_talker_sampling_is_reproducible():
    # the oracle's frame loop with sampling: the same seed gives the same
    # codes, another seed other codes (2-layer stacks, f32)
    import synth
    from model_util import cosine  # noqa: F401  (shared helpers import path)

    def run(seed):
        ls, fn = synth.stack(71, "talker", 1)
        pls, pfn = synth.stack(71, "predictor", 1)
        th = O.OraHeads(synth.HIDDEN, "f32")
        th.add(synth.talker_head(71))
        ph = O.OraHeads(synth.HIDDEN, "f32")
        for h in synth.predictor_heads(71):
            ph.add(h)
        ts, ps = O.OraStack(synth.CONFIG, ls, fn, "f32"), O.OraStack(synth.CONFIG, pls, pfn, "f32")
        tl, pl = O.OraLm(ts, th, 64), O.OraLm(ps, ph, 32)
        t = O.OraTalker(tl, th, pl, ph, synth.codec_embedding(71), synth.predictor_embeddings(71), synth.CODEC_EOS)
        t.set_sampling(seed=seed)
        t.start(synth.prompt(71, 6), None, synth.text_rows(71, 1)[0])
        out = []
        codes = np.zeros(16, np.int32)
        for _ in range(3):
            assert t.next_frame(codes)
            out.append(codes.copy())
        for o in (t, tl, pl, ts, ps, th, ph):
            o.free()
        return np.array(out)

    a, b, c = run(11), run(11), run(12)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)
