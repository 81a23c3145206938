"""The oracle (CPU restatement) pinned against the golden fixtures and the
reference's own test protocols.  CPU only."""
import os

import numpy as np
import pytest

import golden_lib as G
import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_q8_0_matches_gguf_bit_exact():
    # TQwenLmHeads writes ggml's quantize_row_q8_0_ref bytes (lm.pas:259-267)
    f = np.load(os.path.join(GOLD, "q8_0_gguf.npz"))
    q = O.quantize_q8_0(f["x"])
    assert np.array_equal(q, f["q"])


def test_q8_0_roundtrip_bound():
    x = G.q8_blocks()
    back = O.dequantize_q8_0(O.quantize_q8_0(x), x.size)
    blocks = x.reshape(-1, 32)
    d = np.abs(blocks).max(axis=1, keepdims=True) / 127
    # half a step, plus 127 times the fp16 rounding of the scale (relative
    # 2^-11, or half the subnormal step 2^-25 for tiny scales)
    rnd = np.maximum(d * 2.0 ** -11, 2.0 ** -25)
    assert np.all(np.abs(back.reshape(-1, 32) - blocks) <= d * 0.5 + 127 * rnd + 1e-30)


def test_q8_0_digest_independent_of_threads():
    # ParallelQ8MatchesSerial (tests/test.tts.qwen.talker.pas:256-305): the
    # same bytes on one thread and on several
    heads = [G.lcg(1000 + g, 64 * 256)[0].reshape(64, 256) for g in range(3)]
    digests = []
    for n in (1, 4):
        O.set_threads(n)
        h = O.OraHeads(256, "q8_0")
        for t in heads:
            h.add(t)
        digests.append(h.digest())
        h.free()
    O.set_threads(os.cpu_count())
    assert digests[0] == digests[1]


def test_crc32c_known_answer():
    # crc32c("123456789") = 0xE3069283 (the Castagnoli check value)
    assert O.crc32c(b"123456789") == 0xE3069283


@pytest.fixture(scope="module")
def small():
    layers, final, head = G.small_model()
    st = O.OraStack(G.SMALL, layers, final, "f32")
    hd = O.OraHeads(G.SMALL["hidden"], "f32")
    hd.add(head)
    yield st, hd
    st.free()
    hd.free()


def test_stack_matches_transformers(small):
    # CpuFloat32MatchesPyTorch (tests/test.tts.qwen.lm.pas:327-331) on a
    # small random stack: states and logits within atol 1e-3 + rtol 1e-4,
    # cosine >= 0.999999
    st, hd = small
    g = np.load(os.path.join(GOLD, "qwen3_small.npz"))
    lm = O.OraLm(st, hd, 64)
    rows = G.small_rows(9)
    L, H = G.SMALL["layers"], G.SMALL["hidden"]
    states = np.zeros((L, 6, H), np.float32)
    normed = np.zeros((6, H), np.float32)
    logits = np.zeros(G.SMALL["vocab"], np.float32)
    hidden = np.zeros(H, np.float32)
    lm.forward(rows[:6], 0, logits, hidden, states, normed)

    def close(a, r):
        assert np.all(np.abs(a - r) <= 1e-3 + 1e-4 * np.abs(r))
        cos = float(np.dot(a.ravel(), r.ravel()) / (np.linalg.norm(a) * np.linalg.norm(r)))
        assert cos >= 0.999999

    close(states[:L - 1], g["states"])
    close(normed, g["normed"])
    close(hidden, g["normed"][-1])
    close(logits, g["logits0"])
    assert O.argmax(logits) == int(np.argmax(g["logits0"]))
    for r in range(3):
        lm.forward(rows[6 + r:7 + r], 0, logits, hidden)
        close(hidden, g["step_normed"][r])
        close(logits, g["step_logits"][r])
    assert lm.length == 9
    lm.free()


def test_argmax_first_maximum():
    # the test's ArgMax uses a strict '>' (tests/test.tts.qwen.lm.pas:109-117)
    x = np.array([0.5, 2.0, -1.0, 2.0, 1.0], np.float32)
    assert O.argmax(x) == 1


def test_choose_code0_processors():
    # ChooseCode0 (talker.pas:595-630)
    vocab, eos = 3072, 2150
    lg = np.zeros(vocab, np.float32)
    lg[2500] = 9.0          # forbidden control id
    lg[eos] = 8.0           # eos, forbidden before 2 frames
    lg[10] = 5.0
    lg[11] = 4.9
    assert O.choose_code0(lg, eos, []) == 10
    assert O.choose_code0(lg, eos, [3, 4]) == eos          # eos allowed from 2 frames on
    lg[eos] = -1.0
    # the penalty applies once per distinct code: 5/1.05 = 4.76 < 4.9
    assert O.choose_code0(lg, eos, [10, 10, 10]) == 11
    lg2 = np.full(vocab, -3.0, np.float32)
    lg2[5] = -1.0
    lg2[6] = -1.04
    # negative logits are multiplied: -1.05 < -1.04
    assert O.choose_code0(lg2, eos, [5, 5]) == 6
    # penalty 1: no change
    assert O.choose_code0(lg2, eos, [5, 5], penalty=1.0) == 5


def test_predictor_protocol_length(small):
    # the predictor protocol: Forward(embed, 2, 0) then 14 x Forward(row, 1,
    # g); afterwards lm.Length = 16 (tests/test.tts.qwen.lm.pas:272-293)
    st, hd = small
    lm = O.OraLm(st, hd, 32)
    rows = G.small_rows(16, seed=5)
    logits = np.zeros(G.SMALL["vocab"], np.float32)
    lm.forward(rows[:2], 0, logits)
    for g in range(1, 15):
        lm.forward(rows[g + 1:g + 2], 0, logits)
    assert lm.length == 16
    lm.reset()
    assert lm.length == 0
    lm.free()


# the reference checkout: $QTTS_REFERENCE, else a `reference` folder beside
# this repository
REF_ROOT = os.environ.get("QTTS_REFERENCE",
                          os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                       "reference"))
REF_DATASET = os.path.join(REF_ROOT, "tests", "data", "infer-ref", "qwen3-tts-lm")


@pytest.mark.skipif(not os.path.isdir(REF_DATASET), reason="reference dataset not present on this machine")
def test_reference_dataset_is_consistent():
    # DatasetIsConsistent (tests/test.tts.qwen.lm.pas:119-145), with our argmax
    # and ChooseCode0: hashes, argmax of each logits row = its code, row 0 of
    # the predictor input = last talker state
    import hashlib
    import json
    man = json.load(open(os.path.join(REF_DATASET, "manifest.json")))
    blob = open(os.path.join(REF_DATASET, "tensors.bin"), "rb").read()
    assert hashlib.sha256(blob).hexdigest() == man["blob"]["sha256"]
    t = {}
    for e in man["tensors"]:
        raw = blob[e["offset"]:e["offset"] + e["bytes"]]
        assert hashlib.sha256(raw).hexdigest() == e["sha256"]
        t[e["name"]] = np.frombuffer(raw, dtype=np.float32 if e["dtype"] == "f32" else np.int32).reshape(e["shape"])
    codes = t["predictor.codes"]
    assert O.argmax(t["talker.logits_last"][:2048]) == codes[0]
    # code 0 through ChooseCode0 with an empty history (talker vocab 3072)
    eos = 2150
    assert O.choose_code0(t["talker.logits_last"], eos, []) == codes[0]
    for g in range(15):
        assert O.argmax(t["predictor.logits"][g]) == codes[g + 1]
    assert np.array_equal(t["predictor.embed"][0], t["talker.norm"][-1])


def test_check_frame_replays_next_frame():
    # ora_talker_check_frame, the checker of the batched frame loop: driven
    # by the oracle's own codes it reproduces NextFrame with zero gaps; a
    # planted non-maximal choice shows a positive gap at that choice only
    import synth
    ls, final = synth.stack(81, "talker", 1)
    pls, pfinal = synth.stack(81, "predictor", 1)
    ts, ps = O.OraStack(synth.CONFIG, ls, final, "q8_0"), O.OraStack(synth.CONFIG, pls, pfinal, "q8_0")
    th, ph = O.OraHeads(synth.HIDDEN, "q8_0"), O.OraHeads(synth.HIDDEN, "q8_0")
    th.add(synth.talker_head(81))
    for h in synth.predictor_heads(81):
        ph.add(h)
    ce, pe = synth.codec_embedding(81), synth.predictor_embeddings(81)
    lms = [O.OraLm(ts, th, 64), O.OraLm(ps, ph, 32), O.OraLm(ts, th, 64), O.OraLm(ps, ph, 32)]
    a = O.OraTalker(lms[0], th, lms[1], ph, ce, pe, synth.CODEC_EOS)
    b = O.OraTalker(lms[2], th, lms[3], ph, ce, pe, synth.CODEC_EOS)
    pad = synth.text_rows(81, 1, key=1)[0]
    for t in (a, b):
        t.start(synth.prompt(81, 6), synth.text_rows(81, 2), pad)
    codes = np.zeros(16, np.int32)
    for f in range(3):
        if f < 2:
            assert a.next_frame(codes)
        else:
            # the margins variant chooses the same codes; every margin is the
            # best value's lead over the next one, so never negative
            more, margins = a.next_frame_margins(codes)
            assert more and np.all(margins >= 0) and margins.shape == (16,)
        more, gap = b.check_frame(codes)
        assert more and np.all(gap == 0), gap
        assert np.array_equal(a.logits(), b.logits())
    # a planted mistake: the second-best code at choice 3 of the next frame
    c = a.next_frame(codes)
    plant = codes.copy()
    assert c
    # any other id than the first maximum of choice 3 has a positive gap
    plant[3] = (codes[3] + 1) % synth.PRED_VOCAB
    more, gap = b.check_frame(plant)
    assert more and gap[3] > 0 and np.all(gap[:3] == 0)
    for t in (a, b):
        t.free()
    for o in lms:
        o.free()
    for o in (ts, ps, th, ph):
        o.free()
