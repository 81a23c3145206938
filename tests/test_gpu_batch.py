"""The batched path (qtts_batch_*: paged KV cache, tcgen05 projections)
against the oracle, sequence by sequence.

Shapes follow BASELINE.json at reduced size so that the oracle finishes in
seconds: configs[2] (Q8_0, ragged contexts, one-row decode steps, paged KV in
f32 or bf16) and configs[3] (prefill of several long sequences, f32 weights,
fp16 activations and f32 softmax, logits within 2e-3 of the f32 CPU path).
"""
import numpy as np
import pytest

import oracle as O
import qtts
import synth
from model_util import cosine

pytestmark = pytest.mark.gpu


def build(device, seed, layers, dtype, head):
    ls, final = synth.stack(seed, "talker", layers)
    st = qtts.qwen_lm_stack(device, synth.CONFIG, ls, final, dtype)
    heads = qtts.QwenLmHeads(device, "talker", synth.HIDDEN, dtype)
    heads.add(head)
    ost = O.OraStack(synth.CONFIG, ls, final, dtype)
    oh = O.OraHeads(synth.HIDDEN, dtype)
    oh.add(head)
    return st, heads, ost, oh


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_batched_decode_matches_oracle(device, kv):
    # configs[2] in small: 8 utterances with contexts drawn in [50, 300),
    # prefilled through the batch, then 3 one-row decode steps
    rng = np.random.default_rng(5)
    nseq, layers = 8, 3
    head = synth.talker_head(91)
    st, heads, ost, oh = build(device, 91, layers, "q8_0", head)
    b = qtts.QwenBatch(st, heads, max_seqs=nseq, max_tokens=2400, max_pos=400, kv_dtype=kv)
    ctx = rng.integers(50, 300, nseq)
    oras = [O.OraLm(ost, oh, 400) for _ in range(nseq)]
    prompts = [synth.prompt(200 + i, int(c)) for i, c in enumerate(ctx)]
    lg, hd = b.forward(np.arange(nseq), ctx, np.concatenate(prompts))
    atol, cmin = 2e-2, 0.9999  # the north-star Q8_0 tolerance, bf16 pages included
    lo = np.zeros(3072, np.float32)
    ho = np.zeros(1024, np.float32)
    for i in range(nseq):
        oras[i].forward(prompts[i], 0, lo, ho)
        assert np.abs(lg[i] - lo).max() <= atol and cosine(lg[i], lo) >= cmin, (i, np.abs(lg[i] - lo).max())
    for step in range(3):
        x = synth.prompt(300 + step, nseq)
        lg, hd = b.forward(np.arange(nseq), np.ones(nseq, np.int32), x)
        for i in range(nseq):
            oras[i].forward(x[i:i + 1], 0, lo, ho)
            assert np.abs(lg[i] - lo).max() <= atol and cosine(lg[i], lo) >= cmin, (step, i, np.abs(lg[i] - lo).max())
            assert np.abs(hd[i] - ho).max() <= 10 * atol
    for i in range(nseq):
        assert b.length(i) == ctx[i] + 3
    b.reset(3)
    assert b.length(3) == 0
    b.free()
    qtts.stack_destroy(st)
    heads.free()
    for o in oras:
        o.free()


def test_batched_prefill_f32_matches_oracle(device):
    # configs[3] in small: 4 sequences of 256..700 rows, f32 weights; the
    # logits of the last row within 2e-3 of the f32 CPU path
    lens = [256, 333, 512, 700]
    head = synth.talker_head(93)
    st, heads, ost, oh = build(device, 93, 2, "f32", head)
    b = qtts.QwenBatch(st, heads, max_seqs=4, max_tokens=sum(lens), max_pos=800, kv_dtype="f32")
    prompts = [synth.prompt(400 + i, n) for i, n in enumerate(lens)]
    lg, hd = b.forward([2, 0, 3, 1], lens, np.concatenate(prompts))
    lo = np.zeros(3072, np.float32)
    for i, n in enumerate(lens):
        o = O.OraLm(ost, oh, 800)
        o.forward(prompts[i], 0, lo)
        assert np.abs(lg[i] - lo).max() <= 2e-3, (n, np.abs(lg[i] - lo).max())
        o.free()
    b.free()
    qtts.stack_destroy(st)
    heads.free()


def test_batch_mixed_rows_and_errors(device):
    head = synth.talker_head(95)
    st, heads, ost, oh = build(device, 95, 1, "q8_0", head)
    b = qtts.QwenBatch(st, heads, max_seqs=3, max_tokens=64, max_pos=40)
    x = synth.prompt(95, 21)
    lg, _ = b.forward([0, 1, 2], [1, 17, 3], x)
    lo = np.zeros(3072, np.float32)
    for i, (a, c) in enumerate(((0, 1), (1, 18), (18, 21))):
        o = O.OraLm(ost, oh, 40)
        o.forward(x[a:c], 0, lo)
        assert np.abs(lg[i] - lo).max() <= 2e-2 and cosine(lg[i], lo) >= 0.9999
        o.free()
    with pytest.raises(qtts.EQwenLm) as e:
        b.forward([1], [30], synth.prompt(96, 30))        # 17 + 30 > 40 positions
    assert e.value.code == qtts.E_CAPACITY
    with pytest.raises(qtts.EQwenLm) as e:
        b.forward([0, 0], [1, 1], synth.prompt(96, 2))    # the same sequence twice
    assert e.value.code == qtts.E_ARG
    b.free()
    qtts.stack_destroy(st)
    heads.free()


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_prefill_after_context_tensor_cores(device, kv):
    # the tensor-core prefill attention with cached positions before the new
    # rows (L0 > 0), blocks of 128 rows with a ragged last block, and a run
    # of <= 32 rows (CUDA-core path) in the same call
    head = synth.talker_head(97)
    st, heads, ost, oh = build(device, 97, 2, "q8_0", head)
    b = qtts.QwenBatch(st, heads, max_seqs=3, max_tokens=700, max_pos=800, kv_dtype=kv)
    first = [40, 130, 7]
    second = [300, 261, 20]
    p1 = [synth.prompt(500 + i, n) for i, n in enumerate(first)]
    p2 = [synth.prompt(600 + i, n) for i, n in enumerate(second)]
    b.forward([0, 1, 2], first, np.concatenate(p1))
    lg, hd = b.forward([2, 0, 1], [second[2], second[0], second[1]], np.concatenate([p2[2], p2[0], p2[1]]))
    atol, cmin = 2e-2, 0.9999  # the north-star Q8_0 tolerance, bf16 pages included
    lo = np.zeros(3072, np.float32)
    for i, s in enumerate([2, 0, 1]):
        o = O.OraLm(ost, oh, 800)
        o.forward(p1[s], 0, lo)
        o.forward(p2[s], 0, lo)
        assert np.abs(lg[i] - lo).max() <= atol and cosine(lg[i], lo) >= cmin, (s, np.abs(lg[i] - lo).max())
        o.free()
    assert [b.length(s) for s in range(3)] == [340, 391, 27]
    b.free()
    qtts.stack_destroy(st)
    heads.free()
