"""The prompt of TQwenTalker.Start (talker.pas:488-574) on the host: the
codec ids from the voice and the language (qtts.start_codec_ids), the token
ids read from config.json (qtts.prompt_tokens), and the oracle's rows
(oracle.start_rows) checked against TextProject + AddRow row by row."""
import numpy as np
import pytest

import oracle as O
import qtts

# a talker_config with the keys Start reads (values chosen for the test)
TC = {
    "codec_pad_id": 2148, "codec_bos_id": 2149, "codec_eos_token_id": 2150,
    "codec_think_id": 2154, "codec_nothink_id": 2155, "codec_think_bos_id": 2156, "codec_think_eos_id": 2157,
    "spk_id": {"vivian": 3065, "eric": 2875, "dylan": 2878},
    "codec_language_id": {"chinese": 2055, "english": 2050, "sichuan_dialect": 2062, "beijing_dialect": 2074},
    "spk_is_dialect": {"vivian": False, "eric": "sichuan_dialect", "dylan": "beijing_dialect"},
}
CONFIG = {"tts_bos_token_id": 151672, "tts_eos_token_id": 151673, "tts_pad_token_id": 151671, "talker_config": TC}
PAD, BOS = [2148], [2149]


def test_codec_ids_auto_language():
    assert qtts.start_codec_ids(TC) == [2155, 2156, 2157] + PAD + BOS
    assert qtts.start_codec_ids(TC, "", "Auto") == [2155, 2156, 2157] + PAD + BOS


def test_codec_ids_language_and_voice():
    assert qtts.start_codec_ids(TC, "", "English") == [2154, 2156, 2050, 2157] + PAD + BOS
    assert qtts.start_codec_ids(TC, "Vivian", "english") == [2154, 2156, 2050, 2157, 3065] + PAD + BOS
    # a voice that is no dialect keeps auto
    assert qtts.start_codec_ids(TC, "vivian", "") == [2155, 2156, 2157, 3065] + PAD + BOS


def test_codec_ids_dialect_voice():
    # chinese or auto: the voice's dialect is the language
    assert qtts.start_codec_ids(TC, "Eric", "chinese") == [2154, 2156, 2062, 2157, 2875] + PAD + BOS
    assert qtts.start_codec_ids(TC, "dylan", "auto") == [2154, 2156, 2074, 2157, 2878] + PAD + BOS
    # another language wins over the dialect
    assert qtts.start_codec_ids(TC, "eric", "english") == [2154, 2156, 2050, 2157, 2875] + PAD + BOS


def test_codec_ids_unknown_voice_or_language():
    with pytest.raises(qtts.EQwenLm):
        qtts.start_codec_ids(TC, "nobody", "")
    with pytest.raises(qtts.EQwenLm):
        qtts.start_codec_ids(TC, "", "klingon")


def test_prompt_tokens_from_config():
    t = qtts.prompt_tokens(CONFIG)
    assert (t.tts_bos, t.tts_eos, t.tts_pad, t.codec_pad, t.codec_bos) == (151672, 151673, 151671, 2148, 2149)


def small_weights(seed, vocab=40, th=16, hidden=8, cvocab=30):
    rng = np.random.default_rng(seed)
    f = lambda *s: (rng.standard_normal(s) * 0.3).astype(np.float32)  # noqa: E731
    return f(vocab, th), f(th, th), f(th), f(hidden, th), f(hidden), f(cvocab, hidden)


TOK = {"tts_bos": 1, "tts_eos": 2, "tts_pad": 3, "codec_pad": 4, "codec_bos": 5}


@pytest.mark.parametrize("non_streaming", [False, True])
@pytest.mark.parametrize("n_text", [1, 2, 7])
def test_oracle_start_rows(non_streaming, n_text):
    emb, w1, b1, w2, b2, ce = small_weights(5)
    ids = [10, 11, 12] + list(range(20, 20 + n_text)) + [13, 14, 10, 11, 12]
    codec = [7, 8, 9, 4, 5]
    pf, tr, pad = O.start_rows(emb, w1, b1, w2, b2, ce, TOK, ids, codec, non_streaming)
    proj = lambda t: O.text_project(emb, [t], w1, b1, w2, b2)[0]  # noqa: E731
    expect = [proj(10), proj(11), proj(12), proj(3) + ce[7], proj(3) + ce[8], proj(3) + ce[9], proj(1) + ce[4]]
    text = list(range(20, 20 + n_text))
    if non_streaming:
        expect += [proj(t) + ce[4] for t in text] + [proj(2) + ce[4], proj(3) + ce[5]]
        expect_tr = [proj(3)]
    else:
        expect += [proj(text[0]) + ce[5]]
        expect_tr = [proj(t) for t in text[1:]] + [proj(2)]
    np.testing.assert_array_equal(pf, np.array(expect, np.float32))
    np.testing.assert_array_equal(tr, np.array(expect_tr, np.float32))
    np.testing.assert_array_equal(pad, proj(3))


@pytest.mark.parametrize("non_streaming", [False, True])
@pytest.mark.parametrize("n_text", [1, 2, 7])
def test_library_plan_builds_the_oracle_rows(non_streaming, n_text):
    # qtts_prompt_plan (the library's host logic, no device): the rows it
    # plans, built with the oracle's projections, are the rows of the
    # oracle's step-by-step Start, bit for bit
    emb, w1, b1, w2, b2, ce = small_weights(6)
    ids = [10, 11, 12] + list(range(20, 20 + n_text)) + [13, 14, 10, 11, 12]
    codec = [7, 8, 9, 4, 5] if n_text != 2 else [4, 5]
    tok = qtts.PromptTokens(TOK["tts_bos"], TOK["tts_eos"], TOK["tts_pad"], TOK["codec_pad"], TOK["codec_bos"])
    pre, trail = qtts.prompt_plan(tok, ids, codec, non_streaming)
    opf, otr, _ = O.start_rows(emb, w1, b1, w2, b2, ce, TOK, ids, codec, non_streaming)
    assert pre.shape[0] == opf.shape[0] and trail.shape[0] == otr.shape[0]

    def build(plan):
        rows = O.text_project(emb, plan[:, 0], w1, b1, w2, b2) if len(plan) else np.zeros((0, ce.shape[1]))
        for r, c in enumerate(plan[:, 1]):
            if c >= 0:
                rows[r] += ce[c]
        return rows

    np.testing.assert_array_equal(build(pre), opf)
    np.testing.assert_array_equal(build(trail), otr)


def test_library_plan_checks_counts():
    tok = qtts.PromptTokens(1, 2, 3, 4, 5)
    for ids, codec in (([0] * 8, [4, 5]), ([0] * 9, [5])):
        with pytest.raises(qtts.EQwenLm) as e:
            qtts.prompt_plan(tok, ids, codec)
        assert e.value.code == qtts.E_ARG
