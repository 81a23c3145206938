"""TQwenTalker.Start from token ids with its rows built on the device
(qtts_talker_start_prompt, qtts_talker_prompt_rows; talker.pas:528-592)
against the oracle's restatement of the same rows (oracle.start_rows), then
the frames that follow.

Tolerances: the rows within 2e-5 abs + 1e-5 of the peak (TextProject's
float32 sums in another order, as tests/test_gpu_textproj.py); the talker
started from the device rows matches the oracle started from the same rows
as in tests/test_gpu_parity.py (f32 logits within 1e-4, identical codes)."""
import numpy as np
import pytest

import oracle as O
import qtts
import synth
from model_util import TalkerPair

pytestmark = pytest.mark.gpu

TEXT_VOCAB, TEXT_HIDDEN = 2000, 2048
TOK = {"tts_bos": 1997, "tts_eos": 1998, "tts_pad": 1999, "codec_pad": 2148, "codec_bos": 2149}


def tokens():
    return qtts.PromptTokens(TOK["tts_bos"], TOK["tts_eos"], TOK["tts_pad"], TOK["codec_pad"], TOK["codec_bos"])


def textproj_weights(seed):
    rng = np.random.default_rng(seed)
    emb = (rng.standard_normal((TEXT_VOCAB, TEXT_HIDDEN)) * 0.05).astype(np.float32)
    bits = (emb.view(np.uint32) >> 16).astype(np.uint16)  # the checkpoint's BF16 table
    emb = (bits.astype(np.uint32) << 16).view(np.float32)
    w1 = (rng.standard_normal((TEXT_HIDDEN, TEXT_HIDDEN)) * 0.02).astype(np.float32)
    b1 = (rng.standard_normal(TEXT_HIDDEN) * 0.02).astype(np.float32)
    w2 = (rng.standard_normal((synth.HIDDEN, TEXT_HIDDEN)) * 0.02).astype(np.float32)
    b2 = (rng.standard_normal(synth.HIDDEN) * 0.02).astype(np.float32)
    return bits, emb, w1, b1, w2, b2


def prompt_ids(seed, n_text):
    rng = np.random.default_rng(seed)
    text = [int(v) for v in rng.integers(0, 1990, n_text)]
    return [1990, 1991, 1992] + text + [1993, 1992, 1990, 1991, 1992]


CODEC = [2155, 2156, 2050, 2157, 3065, 2148, 2149]  # think, bos, language, eos, voice, pad, bos


def close(a, b):
    return np.abs(a - b).max() <= 2e-5 + 1e-5 * np.abs(b).max()


@pytest.mark.parametrize("non_streaming", [False, True])
def test_prompt_rows_match_oracle(device, non_streaming):
    bits, emb, w1, b1, w2, b2 = textproj_weights(7)
    tk = TalkerPair(device, 91, 1, 1, "f32")
    tp = qtts.QwenTextProject(device, bits, w1, b1, w2, b2)
    ids = prompt_ids(8, 9)
    pf, tr = tk.dev.prompt_rows(tp, tokens(), ids, CODEC, non_streaming)
    opf, otr, _ = O.start_rows(emb, w1, b1, w2, b2, synth.codec_embedding(91), TOK, ids, CODEC, non_streaming)
    assert pf.shape == opf.shape and tr.shape == otr.shape
    assert pf.shape[0] == (3 + 6 + 10 + 1 if non_streaming else 3 + 6 + 1)
    assert tr.shape[0] == (1 if non_streaming else 9)
    assert close(pf, opf), np.abs(pf - opf).max()
    assert close(tr, otr), np.abs(tr - otr).max()
    # the shortest text (one token) and its single trailing row, tts_eos
    ids1 = prompt_ids(9, 1)
    pf1, tr1 = tk.dev.prompt_rows(tp, tokens(), ids1, CODEC[-2:], non_streaming)
    opf1, otr1, _ = O.start_rows(emb, w1, b1, w2, b2, synth.codec_embedding(91), TOK, ids1, CODEC[-2:],
                                 non_streaming)
    assert pf1.shape == opf1.shape and tr1.shape == otr1.shape == (1, synth.HIDDEN)
    assert close(pf1, opf1) and close(tr1, otr1)
    tp.free()
    tk.free()


@pytest.mark.parametrize("non_streaming", [False, True])
def test_start_prompt_frames_match_oracle(device, non_streaming):
    # Start from ids on the device; the oracle starts from the same rows
    # (read back by qtts_talker_prompt_rows) and tts_pad's projection
    bits, emb, w1, b1, w2, b2 = textproj_weights(11)
    tk = TalkerPair(device, 92, 2, 2, "f32")
    tp = qtts.QwenTextProject(device, bits, w1, b1, w2, b2)
    ids = prompt_ids(12, 5)
    pf, tr = tk.dev.prompt_rows(tp, tokens(), ids, CODEC, non_streaming)
    pad = tp.project([TOK["tts_pad"]])[0]
    lg = np.zeros(synth.TALKER_VOCAB, np.float32)
    hd = np.zeros(synth.HIDDEN, np.float32)
    tk.dev.start_prompt(tp, tokens(), ids, CODEC, non_streaming, lg, hd)
    tk.ora.start(pf, tr, pad)
    assert np.abs(lg - tk.ora.logits()).max() <= 1e-4
    assert tk.t.dev.length == pf.shape[0]
    codes_d = np.zeros(16, np.int32)
    codes_o = np.zeros(16, np.int32)
    frames = tr.shape[0] + 2  # past the trailing text, into tts_pad
    for f in range(frames):
        md = tk.dev.next_frame(codes_d)
        mo = tk.ora.next_frame(codes_o)
        assert md == mo, f"frame {f}: eos on one side only"
        if not md:
            break
        assert np.array_equal(codes_d, codes_o), f"frame {f}: {codes_d} vs {codes_o}"
        assert np.abs(tk.dev.probe()[0] - tk.ora.logits()).max() <= 1e-4
    tp.free()
    tk.free()


def test_start_prompt_checks_its_ids(device):
    bits, emb, w1, b1, w2, b2 = textproj_weights(13)
    tk = TalkerPair(device, 93, 1, 1, "f32")
    tp = qtts.QwenTextProject(device, bits, w1, b1, w2, b2)
    ids = prompt_ids(14, 3)
    for bad_ids, bad_codec in ((ids[:8], CODEC),                  # empty text
                               ([2000] + ids[1:], CODEC),         # text token out of range
                               (ids, [3072, 2148, 2149]),         # codec id out of range
                               (ids, [2149])):                     # no pad / bos
        with pytest.raises(qtts.EQwenLm) as e:
            tk.dev.start_prompt(tp, tokens(), bad_ids, bad_codec)
        assert e.value.code == qtts.E_ARG
    # the talker still starts afterwards
    tk.dev.start_prompt(tp, tokens(), ids, CODEC)
    assert tk.t.dev.length == 3 + 6 + 1
    tp.free()
    tk.free()


def test_batched_start_prompt_matches_oracle(device):
    # qtts_talkers_start_prompt: three utterances (streaming and not, texts of
    # 1, 4 and 9 tokens) started in one call; each oracle talker starts from
    # the oracle's own rows, then the frames are checked as the batched
    # frame loop's (every choice a maximum of the oracle's values)
    from test_gpu_frames import GAP, Rig, frame
    bits, emb, w1, b1, w2, b2 = textproj_weights(17)
    rig = Rig(device, 94, 2, 2, "f32", "f32", nseq=3)
    tp = qtts.QwenTextProject(device, bits, w1, b1, w2, b2)
    prompts = [(prompt_ids(18, 4), CODEC, False), (prompt_ids(19, 1), CODEC[-2:], True),
               (prompt_ids(20, 9), CODEC[:3] + CODEC[-2:], False)]
    seqs = [2, 0, 1]
    rig.dev.start_prompt(tp, tokens(), seqs, prompts)
    ce = synth.codec_embedding(94)
    rows = {}
    for s, (ids, codec, ns) in zip(seqs, prompts):
        pf, tr, pad = O.start_rows(emb, w1, b1, w2, b2, ce, TOK, ids, codec, ns)
        rig.ora[s].start(pf, tr, pad)
        rows[s] = pf.shape[0]
    stats = [0, 0]
    live = list(seqs)
    frames = {s: 0 for s in seqs}
    for _ in range(4):
        _, more = frame(rig, live, GAP[("f32", "f32")], stats)
        for s, m in zip(list(live), more):
            if m:
                frames[s] += 1
            else:
                live.remove(s)  # eos: the utterance is over
    for s in seqs:
        assert rig.tb.length(s) == rows[s] + frames[s]
    assert stats[0] >= 0.9 * stats[1], stats
    tp.free()
    rig.free()
