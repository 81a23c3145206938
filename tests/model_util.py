"""Builders shared by the tests: the same seeded synthetic weights given to
the device library (through the C-ABI) and to the oracle."""
import numpy as np

import oracle as O
import qtts
import synth


def cosine(a, b):
    a, b = np.ravel(a).astype(np.float64), np.ravel(b).astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


class Pair:
    """One stack + heads on the device and in the oracle."""

    def __init__(self, device, seed, name, layers, heads, dtype, max_pos=512):
        ls, final = synth.stack(seed, name, layers)
        self.heads_src = heads
        self.dev_heads = qtts.QwenLmHeads(device, name, synth.HIDDEN, dtype)
        self.ora_heads = O.OraHeads(synth.HIDDEN, dtype)
        for h in heads:
            self.dev_heads.add(h)
            self.ora_heads.add(h)
        self.dev = qtts.QwenLm(qtts.qwen_lm_stack(device, synth.CONFIG, ls, final, dtype), self.dev_heads, max_pos)
        self.ora_stack = O.OraStack(synth.CONFIG, ls, final, dtype)
        self.ora = O.OraLm(self.ora_stack, self.ora_heads, max_pos)

    def free(self):
        self.dev.free()
        self.dev_heads.free()
        self.ora.free()
        self.ora_stack.free()
        self.ora_heads.free()


class TalkerPair:
    """Talker + predictor, device and oracle, with the frame loop."""

    def __init__(self, device, seed, tlayers, players, dtype, max_pos=512, eos=synth.CODEC_EOS, theads=None):
        th = [synth.talker_head(seed)] if theads is None else theads
        self.t = Pair(device, seed, "talker", tlayers, th, dtype, max_pos)
        self.p = Pair(device, seed, "predictor", players, synth.predictor_heads(seed), dtype, 32)
        ce = synth.codec_embedding(seed)
        pe = synth.predictor_embeddings(seed)
        self.dev = qtts.QwenTalker(self.t.dev, self.p.dev, ce, pe, eos)
        self.ora = O.OraTalker(self.t.ora, self.t.ora_heads, self.p.ora, self.p.ora_heads, ce, pe, eos)

    def start(self, prefill, trailing, pad):
        lg = np.zeros(synth.TALKER_VOCAB, np.float32)
        hd = np.zeros(synth.HIDDEN, np.float32)
        self.dev.start(prefill, trailing, pad, lg, hd)
        self.ora.start(prefill, trailing, pad)
        return lg, hd

    def free(self):
        self.dev.free()
        self.ora.free()
        self.t.free()
        self.p.free()
