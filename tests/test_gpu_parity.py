"""Parity of the CUDA path (libqtts.so, through the C-ABI) with the oracle on
the same seeded weights and inputs.

Tolerances (north_star of the build, following the reference's
tests/test.tts.qwen.lm.pas:319-336 and test.tts.qwen.vulkan.pas:224-232):
  f32 weights : logits within 1e-4 abs, identical greedy codes; the predictor
                protocol within 1e-4 relative to the peak (ComparePredictor).
  Q8_0 weights: logits within 2e-2 abs and cosine >= 0.9999 against the
                oracle's Q8_0 path (f32 activations).
"""
import os

import numpy as np
import pytest

import golden_lib as G
import oracle as O
import qtts
import synth
from model_util import Pair, TalkerPair, cosine

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
F32_LOGITS_ATOL = 1e-4
Q8_LOGITS_ATOL = 2e-2
Q8_COSINE = 0.9999


def test_device_quantize_matches_gguf(device):
    f = np.load(os.path.join(GOLD, "q8_0_gguf.npz"))
    assert np.array_equal(device.quantize_q8_0(f["x"]), f["q"])


def test_device_quantize_matches_oracle_large(device):
    x = synth.normal((4096, 1024), 0.02, 5, 5)
    assert np.array_equal(device.quantize_q8_0(x), O.quantize_q8_0(x))


@pytest.mark.parametrize("dtype", ["q8_0", "f32"])
def test_heads_digest_matches_oracle(device, dtype):
    # ParallelQ8MatchesSerial / TQwenLmHeads.Digest: the same bytes
    heads = [synth.talker_head(3)] + synth.predictor_heads(3)[:2]
    d = qtts.QwenLmHeads(device, "heads", synth.HIDDEN, dtype)
    o = O.OraHeads(synth.HIDDEN, dtype)
    for h in heads:
        d.add(h)
        o.add(h)
    assert d.count == 3 and d.rows(0) == 3072 and d.rows(2) == 2048
    assert d.digest() == o.digest()
    per = 1024 * 4 if dtype == "f32" else 1024 // 32 * 34
    assert d.bytes == (3072 + 2 * 2048) * per
    d.free()
    o.free()


def test_forward_f32_prefill_and_steps(device):
    pr = Pair(device, 11, "talker", 2, [synth.talker_head(11)], "f32", max_pos=64)
    x = synth.prompt(11, 13)
    ld, lo = np.zeros(3072, np.float32), np.zeros(3072, np.float32)
    hd, ho = np.zeros(1024, np.float32), np.zeros(1024, np.float32)
    # 10 prefill rows (launches of 4 + 4 + 2), then 3 single rows
    pr.dev.forward(x[:10], output=0, logits=ld, hidden=hd)
    pr.ora.forward(x[:10], 0, lo, ho)
    assert np.abs(ld - lo).max() <= F32_LOGITS_ATOL
    assert np.abs(hd - ho).max() <= 1e-4
    assert int(np.argmax(ld)) == O.argmax(lo)
    for r in range(10, 13):
        pr.dev.forward(x[r:r + 1], output=0, logits=ld, hidden=hd)
        pr.ora.forward(x[r:r + 1], 0, lo, ho)
        assert np.abs(ld - lo).max() <= F32_LOGITS_ATOL
        assert np.abs(hd - ho).max() <= 1e-4
    assert pr.dev.length == 13 == pr.ora.length
    pr.dev.reset()
    assert pr.dev.length == 0
    pr.free()


def test_predictor_protocol_lcg_f32(device):
    # ComparePredictor (tests/test.tts.qwen.vulkan.pas:150-222): the 5-layer
    # predictor with its 15 heads, LCG inputs, 2 rows then one per group;
    # relative error (max |diff| / peak) <= 1e-4 with a float32 cache
    pr = Pair(device, 21, "predictor", 5, synth.predictor_heads(21), "f32", max_pos=32)
    seed = 12345
    worst = 0.0
    ld, lo = np.zeros(2048, np.float32), np.zeros(2048, np.float32)
    hd, ho = np.zeros(1024, np.float32), np.zeros(1024, np.float32)
    for g in range(15):
        rows = 2 if g == 0 else 1
        x, seed = synth.lcg_rows(rows, seed)
        pr.dev.forward(x, output=g, logits=ld, hidden=hd)
        pr.ora.forward(x, g, lo, ho)
        worst = max(worst, np.abs(ld - lo).max() / np.abs(lo).max(), np.abs(hd - ho).max() / np.abs(ho).max())
        assert int(np.argmax(ld)) == O.argmax(lo)
    assert worst <= 1e-4, worst
    assert pr.dev.length == 16


def test_forward_q8_matches_oracle(device):
    pr = Pair(device, 31, "talker", 3, [synth.talker_head(31)], "q8_0", max_pos=64)
    x = synth.prompt(31, 7)
    ld, lo = np.zeros(3072, np.float32), np.zeros(3072, np.float32)
    pr.dev.forward(x[:5], output=0, logits=ld)
    pr.ora.forward(x[:5], 0, lo)
    assert np.abs(ld - lo).max() <= Q8_LOGITS_ATOL and cosine(ld, lo) >= Q8_COSINE
    for r in range(5, 7):
        pr.dev.forward(x[r:r + 1], output=0, logits=ld)
        pr.ora.forward(x[r:r + 1], 0, lo)
        assert np.abs(ld - lo).max() <= Q8_LOGITS_ATOL and cosine(ld, lo) >= Q8_COSINE
    pr.free()


def test_capacity_is_an_error(device):
    pr = Pair(device, 41, "talker", 1, [synth.talker_head(41)], "f32", max_pos=8)
    x = synth.prompt(41, 10)
    with pytest.raises(qtts.EQwenLm) as e:
        pr.dev.forward(x)
    assert e.value.code == qtts.E_CAPACITY
    pr.dev.forward(x[:8])
    assert pr.dev.length == 8
    pr.free()


def run_frames(tp, frames, atol, cos_min=None):
    codes_d = np.zeros(16, np.int32)
    codes_o = np.zeros(16, np.int32)
    n = 0
    for f in range(frames):
        md = tp.dev.next_frame(codes_d)
        mo = tp.ora.next_frame(codes_o)
        assert md == mo, f"frame {f}: eos on one side only"
        if not md:
            break
        assert np.array_equal(codes_d, codes_o), f"frame {f}: {codes_d} vs {codes_o}"
        lg, hd = tp.dev.probe()
        lo = tp.ora.logits()
        assert np.abs(lg - lo).max() <= atol, (f, np.abs(lg - lo).max())
        if cos_min:
            assert cosine(lg, lo) >= cos_min
        n += 1
    return n


@pytest.mark.parametrize("dtype", ["f32", "q8_0"])
def test_talker_frames_match_oracle(device, dtype):
    # NextFrame (talker.pas:640-681) on the device against the oracle: the
    # same 16 codes frame by frame, the talker logits within tolerance
    tp = TalkerPair(device, 51, 2, 2, dtype)
    prefill = synth.prompt(51, 12)
    trailing = synth.text_rows(51, 3)
    pad = synth.text_rows(51, 1, key=1)[0]
    lg, hd = tp.start(prefill, trailing, pad)
    assert np.abs(lg - tp.ora.logits()).max() <= (F32_LOGITS_ATOL if dtype == "f32" else Q8_LOGITS_ATOL)
    atol = F32_LOGITS_ATOL if dtype == "f32" else Q8_LOGITS_ATOL
    n = run_frames(tp, 8, atol, None if dtype == "f32" else Q8_COSINE)
    assert n == 8 and tp.dev.step == 8
    assert tp.t.dev.length == 12 + 8 and tp.p.dev.length == 16
    tp.free()


def test_tagged_handoffs_across_the_epoch_wrap(device):
    # The batch-1 kernel passes the QKV rows, the residual stream and, in
    # greedy frames, the argmax keys between its CTAs as words tagged with
    # the launch's epoch, a counter that wraps after 2^22 - 1 launches (the
    # host clears the tagged words before epoch 1 comes round again).
    # Launches on either side of the wrap must equal the oracle's.
    pr = Pair(device, 97, "talker", 2, [synth.talker_head(97)], "q8_0", max_pos=32)
    try:
        with pytest.raises(qtts.EQwenLm):
            pr.dev.set_launch_epoch(1 << 22)
        x = synth.prompt(97, 9)
        ld, lo = np.zeros(3072, np.float32), np.zeros(3072, np.float32)
        pr.dev.set_launch_epoch((1 << 22) - 3)
        for r0, r1 in ((0, 3), (3, 4), (4, 5), (5, 7), (7, 8), (8, 9)):  # epochs 2^22 - 2, 2^22 - 1, 1, 2, 3, 4
            pr.dev.forward(x[r0:r1], output=0, logits=ld)
            pr.ora.forward(x[r0:r1], 0, lo)
            assert np.abs(ld - lo).max() <= Q8_LOGITS_ATOL and cosine(ld, lo) >= Q8_COSINE, (r0, r1)
    finally:
        pr.free()
    # frames: the talker's launches use the talker lm's counter
    tp = TalkerPair(device, 51, 2, 2, "q8_0")
    try:
        tp.start(synth.prompt(51, 12), synth.text_rows(51, 3), synth.text_rows(51, 1, key=1)[0])
        tp.t.dev.set_launch_epoch((1 << 22) - 2)
        assert run_frames(tp, 4, Q8_LOGITS_ATOL, Q8_COSINE) == 4
    finally:
        tp.free()


def test_eos_ends_the_sentence(device):
    # a talker head whose eos row dominates: eos is forbidden for the first
    # 2 frames (talker.pas:610-611), then chosen; NextFrame returns false
    th = synth.talker_head(61)
    th[synth.CODEC_EOS] = th[synth.CODEC_EOS] * 40.0 + 0.05
    tp = TalkerPair(device, 61, 1, 1, "f32", theads=[th])
    tp.start(synth.prompt(61, 4), None, synth.text_rows(61, 1)[0])
    codes = np.zeros(16, np.int32)
    n = 0
    while tp.dev.next_frame(codes):
        n += 1
        assert n < 10
    codes_o = np.zeros(16, np.int32)
    m = 0
    while tp.ora.next_frame(codes_o):
        m += 1
    assert n == m == 2
    assert not tp.dev.next_frame(codes)
    tp.free()


def test_config1_full_f32_frame(device):
    # 28-layer talker + 5-layer predictor, f32, one frame
    # after 128 prior positions of N(0, 1) rows
    tp = TalkerPair(device, 1, 28, 5, "f32", max_pos=256)
    prefill = synth.prompt(1, 128)
    lg, _ = tp.start(prefill, None, synth.text_rows(1, 1)[0])
    assert np.abs(lg - tp.ora.logits()).max() <= F32_LOGITS_ATOL
    assert run_frames(tp, 2, F32_LOGITS_ATOL) == 2
    tp.free()


def test_predictor_protocol_lcg_kv_f16(device):
    # ComparePredictor with aKvF16 (tests/test.tts.qwen.vulkan.pas:150-232):
    # the 5-layer f32 predictor, LCG inputs, 2 rows then one per group, the
    # K/V cache in half floats.  Against the oracle's f32 cache the reference
    # accepts 5e-2 relative (it measured 2.3e-2).  Against the oracle with the
    # same half-float cache (K/V rounded to nearest even as they are
    # appended): 1e-3 relative -- a float32 difference in the last bit can
    # send a K/V element to the neighbouring half (2^-11 of its value), which
    # is why the f32 tolerance (1e-4) is not kept here (measured 1.2e-4).
    ls, final = synth.stack(21, "predictor", 5)
    heads = synth.predictor_heads(21)
    dh = qtts.QwenLmHeads(device, "predictor", synth.HIDDEN, "f32")
    oh = O.OraHeads(synth.HIDDEN, "f32")
    for h in heads:
        dh.add(h)
        oh.add(h)
    dev = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, ls, final, "f32"), dh, 32, kv_dtype="f16")
    ost = O.OraStack(synth.CONFIG, ls, final, "f32")
    o16, o32 = O.OraLm(ost, oh, 32, kv_f16=True), O.OraLm(ost, oh, 32)
    seed = 12345
    worst16 = worst32 = 0.0
    ld = np.zeros(2048, np.float32)
    l16, l32 = np.zeros(2048, np.float32), np.zeros(2048, np.float32)
    hd, h16, h32 = (np.zeros(1024, np.float32) for _ in range(3))
    for g in range(15):
        rows = 2 if g == 0 else 1
        x, seed = synth.lcg_rows(rows, seed)
        dev.forward(x, output=g, logits=ld, hidden=hd)
        o16.forward(x, g, l16, h16)
        o32.forward(x, g, l32, h32)
        worst16 = max(worst16, np.abs(ld - l16).max() / np.abs(l16).max(), np.abs(hd - h16).max() / np.abs(h16).max())
        worst32 = max(worst32, np.abs(ld - l32).max() / np.abs(l32).max(), np.abs(hd - h32).max() / np.abs(h32).max())
    print({"kv_f16_vs_oracle_f16": worst16, "kv_f16_vs_oracle_f32": worst32})
    assert worst16 <= 1e-3, worst16
    assert worst32 <= 5e-2, worst32
    assert dev.length == 16
    dev.free()
    dh.free()
    for o in (o16, o32, ost, oh):
        o.free()


def test_talker_frames_kv_f16(device):
    # NextFrame with both caches in half floats (TQwenTalkerOptions.KvF16,
    # talker.pas:56): Q8_0 stacks, the same 16 codes as the oracle with
    # half-float caches frame by frame, talker logits within 2e-2, cosine 0.9999
    seed = 52
    tls, tf = synth.stack(seed, "talker", 2)
    pls, pf = synth.stack(seed, "predictor", 2)
    th, ph = qtts.QwenLmHeads(device, "t", synth.HIDDEN, "q8_0"), qtts.QwenLmHeads(device, "p", synth.HIDDEN, "q8_0")
    oth, oph = O.OraHeads(synth.HIDDEN, "q8_0"), O.OraHeads(synth.HIDDEN, "q8_0")
    th.add(synth.talker_head(seed))
    oth.add(synth.talker_head(seed))
    for h in synth.predictor_heads(seed):
        ph.add(h)
        oph.add(h)
    tlm = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, tls, tf, "q8_0"), th, 64, kv_dtype="f16")
    plm = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, pls, pf, "q8_0"), ph, 32, kv_dtype="f16")
    ce, pe = synth.codec_embedding(seed), synth.predictor_embeddings(seed)
    tk = qtts.QwenTalker(tlm, plm, ce, pe, synth.CODEC_EOS)
    ots, ops = O.OraStack(synth.CONFIG, tls, tf, "q8_0"), O.OraStack(synth.CONFIG, pls, pf, "q8_0")
    otl, opl = O.OraLm(ots, oth, 64, kv_f16=True), O.OraLm(ops, oph, 32, kv_f16=True)
    ok = O.OraTalker(otl, oth, opl, oph, ce, pe, synth.CODEC_EOS)
    prefill, trailing, pad = synth.prompt(seed, 12), synth.text_rows(seed, 3), synth.text_rows(seed, 1, key=1)[0]
    lg, hd = np.zeros(3072, np.float32), np.zeros(1024, np.float32)
    tk.start(prefill, trailing, pad, lg, hd)
    ok.start(prefill, trailing, pad)
    assert np.abs(lg - ok.logits()).max() <= Q8_LOGITS_ATOL
    cd, co = np.zeros(16, np.int32), np.zeros(16, np.int32)
    for f in range(6):
        assert tk.next_frame(cd) and ok.next_frame(co)
        assert np.array_equal(cd, co), (f, cd, co)
        lg, _ = tk.probe()
        assert np.abs(lg - ok.logits()).max() <= Q8_LOGITS_ATOL and cosine(lg, ok.logits()) >= Q8_COSINE
    tk.free()
    tlm.free()
    plm.free()
    th.free()
    ph.free()
    for o in (ok, otl, opl, ots, ops, oth, oph):
        o.free()
