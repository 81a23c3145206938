"""Generate the full-size parity fixtures of tests/golden from the oracle
(oracle/qtts_oracle.c, the CPU restatement of the reference path), on the
exact inputs bench.py times (synth.config*_* with seed 1):

1. config1_q8_0.npz: the 28-layer talker and the
   5-layer predictor with Q8_0 weights, a 40-row N(0,1) prompt, 156 greedy
   frames (NextFrame, talker.pas:640-681).  codes [156][16]; margins
   [156][16] = each choice's best value minus the next one (after the
   processors of ChooseCode0); logits0 = the talker logits of the prompt.
2. config2_q8_0_b64.npz -- configs[2]: 64 utterances, contexts U(50, 1000)
   filled with N(0,1) rows, the same Q8_0 stacks, 3 greedy frames each:
   ctx [64]; logits0 [64][3072] (after the prefill); codes and margins
   [64][3][16]; logits3 [64][3072] (after the third frame).
3. config3_f32_prefill.npz -- configs[3]: 16 prompts of U(256, 2048) N(0,1)
   rows through the 28-layer talker with f32 weights (one TQwenLm.Forward
   each, lm.pas:391-408): lens [16]; logits [16][3072] and hidden [16][1024]
   of each prompt's last row.

    python tests/golden/make_config_fixtures.py [config1] [config2] [config3]

Takes about 20 minutes on 8 cores (the configs[2] and [3] prefills of ~34k
and ~18k rows through 28 layers dominate).
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "mormot2-qwen-tts_b200"), os.path.join(ROOT, "oracle")]
import oracle as O  # noqa: E402
import synth  # noqa: E402

SEED = 1


class Model:
    """The bench's seeded stacks and heads in the oracle."""

    def __init__(self, dtype, tlayers=28, players=5):
        tl, tf = synth.stack(SEED, "talker", tlayers)
        self.ts = O.OraStack(synth.CONFIG, tl, tf, dtype)
        self.th = O.OraHeads(synth.HIDDEN, dtype)
        self.th.add(synth.talker_head(SEED))
        self.ps = self.ph = None
        if players:
            pl, pf = synth.stack(SEED, "predictor", players)
            self.ps = O.OraStack(synth.CONFIG, pl, pf, dtype)
            self.ph = O.OraHeads(synth.HIDDEN, dtype)
            for h in synth.predictor_heads(SEED):
                self.ph.add(h)
            self.ce = synth.codec_embedding(SEED)
            self.pe = synth.predictor_embeddings(SEED)
        self.pad = synth.text_rows(SEED, 1, key=1)[0]

    def talker(self, max_pos):
        tlm = O.OraLm(self.ts, self.th, max_pos)
        plm = O.OraLm(self.ps, self.ph, 32)
        return tlm, plm, O.OraTalker(tlm, self.th, plm, self.ph, self.ce, self.pe, synth.CODEC_EOS)


def frames(tk, n):
    codes, margins = [], []
    c = np.zeros(16, np.int32)
    for _ in range(n):
        more, m = tk.next_frame_margins(c)
        if not more:
            break
        codes.append(c.copy())
        margins.append(m)
    return np.array(codes, np.int16), np.array(margins, np.float32)


def config1():
    m = Model("q8_0")
    tlm, plm, tk = m.talker(256)
    tk.start(synth.config1_prompt(SEED), None, m.pad)
    logits0 = tk.logits()
    codes, margins = frames(tk, 156)
    np.savez_compressed(os.path.join(HERE, "config1_q8_0.npz"), codes=codes, margins=margins, logits0=logits0)
    print("config1:", codes.shape, "smallest margins", np.sort(margins.ravel())[:4])


def config2():
    m = Model("q8_0")
    ctx = synth.config2_contexts(SEED)
    n = ctx.size
    logits0 = np.zeros((n, synth.TALKER_VOCAB), np.float32)
    logits3 = np.zeros_like(logits0)
    codes = np.zeros((n, 3, 16), np.int16)
    margins = np.zeros((n, 3, 16), np.float32)
    for s in range(n):
        tlm, plm, tk = m.talker(int(ctx[s]) + 8)
        tk.start(synth.config2_prompt(s, int(ctx[s]), SEED), None, m.pad)
        logits0[s] = tk.logits()
        c, g = frames(tk, 3)
        assert c.shape[0] == 3, "eos within 3 frames"
        codes[s], margins[s] = c, g
        logits3[s] = tk.logits()
        for o in (tk, tlm, plm):
            o.free()
        print("config2: utterance", s, "ctx", int(ctx[s]), flush=True)
    np.savez_compressed(os.path.join(HERE, "config2_q8_0_b64.npz"), ctx=ctx, logits0=logits0, codes=codes,
                        margins=margins, logits3=logits3)


def config3():
    m = Model("f32", players=0)
    lens = synth.config3_lengths(SEED)
    logits = np.zeros((lens.size, synth.TALKER_VOCAB), np.float32)
    hidden = np.zeros((lens.size, synth.HIDDEN), np.float32)
    for i, n in enumerate(lens):
        lm = O.OraLm(m.ts, m.th, int(n))
        lm.forward(synth.config3_prompt(i, int(n), SEED), 0, logits[i], hidden[i])
        lm.free()
        print("config3: prompt", i, "rows", int(n), flush=True)
    np.savez_compressed(os.path.join(HERE, "config3_f32_prefill.npz"), lens=lens, logits=logits, hidden=hidden)


if __name__ == "__main__":
    todo = sys.argv[1:] or ["config1", "config2", "config3"]
    for name in todo:
        t0 = time.time()
        globals()[name]()
        print(name, "%.0f s" % (time.time() - t0), flush=True)
