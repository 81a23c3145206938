"""Deterministic inputs of the golden fixtures (test infrastructure).

Weights and rows come from the reference's own pseudo-random generator, the
LCG of ComparePredictor (tests/test.tts.qwen.vulkan.pas:189-198):
    seed := seed * 1664525 + 1013904223;  x := (integer(seed shr 8) / 2^24 - 0.5) * 0.2
computed in float64 and stored as float32.  Integer-only state and one
multiply per value: the same numbers on every machine, so the fixtures need
not store their weights.
"""
import numpy as np

A, C, M = 1664525, 1013904223, 1 << 32
_B = 1024
_AK = np.empty(_B, dtype=np.uint64)
_CK = np.empty(_B, dtype=np.uint64)
_a, _c = 1, 0
for _k in range(_B):
    _a = (_a * A) % M
    _c = (_c * A + C) % M
    _AK[_k], _CK[_k] = _a, _c


def lcg(seed, n, scale=0.2):
    """n values of the reference LCG after `seed` (the first value uses the
    state after one step, as the Pascal loop does); returns (values, state)."""
    nb = (n + _B - 1) // _B
    states = np.empty(nb * _B, dtype=np.uint64)
    s = seed % M
    for b in range(nb):
        blk = (_AK * np.uint64(s) + _CK) % np.uint64(M)
        states[b * _B:(b + 1) * _B] = blk
        s = int(blk[-1])
    states = states[:n]
    vals = ((states >> np.uint64(8)).astype(np.float64) / float(1 << 24) - 0.5) * scale
    return vals.astype(np.float32), int(states[-1]) if n else seed


SMALL = dict(hidden=256, heads=4, kv_heads=2, head_dim=64, intermediate=512, rms_eps=1e-6, rope_theta=1e6,
             layers=2, vocab=96)


def small_model(seed=777):
    """LCG weights of a small Qwen3 stack + head (dims of SMALL)."""
    c = SMALL
    H, q, kv, I = c["hidden"], c["heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"], c["intermediate"]
    shapes = [("wq", (q, H)), ("wk", (kv, H)), ("wv", (kv, H)), ("wo", (H, q)), ("wg", (I, H)), ("wu", (I, H)),
              ("wd", (H, I))]
    s = seed
    layers = []
    for _ in range(c["layers"]):
        L = {}
        for name, shp in shapes:
            v, s = lcg(s, shp[0] * shp[1], 0.2)
            L[name] = v.reshape(shp)
        for name, n in (("in_norm", H), ("post_norm", H), ("q_norm", c["head_dim"]), ("k_norm", c["head_dim"])):
            v, s = lcg(s, n, 0.2)
            L[name] = (1.0 + v).astype(np.float32)
        layers.append(L)
    v, s = lcg(s, H, 0.2)
    final = (1.0 + v).astype(np.float32)
    head, s = lcg(s, c["vocab"] * H, 0.2)
    return layers, final, head.reshape(c["vocab"], H)


def small_rows(rows, seed=4242, scale=2.0):
    v, _ = lcg(seed, rows * SMALL["hidden"], scale)
    return v.reshape(rows, SMALL["hidden"])


def q8_blocks(seed=99, nblocks=48):
    """Q8_0 test blocks: LCG values at several magnitudes plus edge cases
    (zeros, one value, exact halves after scaling, negatives only, tiny)."""
    v, _ = lcg(seed, nblocks * 32, 2.0)
    x = v.reshape(nblocks, 32).copy()
    x[1] *= 1e-3
    x[2] *= 300.0
    x[3] = 0.0
    x[4] = 0.0
    x[4, 7] = -1.5
    x[5] = np.arange(32, dtype=np.float32) - 15.5    # halves after scaling
    x[6] = -np.abs(x[6])
    x[7] = np.float32(1e-30)
    x[8] = np.linspace(-127, 127, 32).astype(np.float32)
    return x.astype(np.float32).reshape(-1)
