"""Seeded synthetic Qwen3-TTS language-model weights and inputs.

There is no checkpoint on this machine: every benchmark and parity run uses
random weights of the real architecture (Qwen3-TTS-12Hz-0.6B talker and code
predictor: hidden 1024, 16 query / 8 KV heads of 128, SwiGLU 3072, RMSNorm eps
1e-6, RoPE theta 1e6).

Distributions: linear weights, heads and code embeddings N(0, 0.02); norm
weights 1 + N(0, 0.02); prompt rows N(0, 1); text rows (trailing, tts_pad)
N(0, 0.02).  Each tensor has its own numpy PCG64 stream keyed by
(seed, stack, layer, tensor), so a stack can be regenerated layer by layer.
"""
import numpy as np

HIDDEN = 1024
HEADS = 16
KV_HEADS = 8
HEAD_DIM = 128
INTER = 3072
EPS = 1e-6
THETA = 1e6
TALKER_VOCAB = 3072
PRED_VOCAB = 2048
GROUPS = 16
# codec_eos_token_id of the synthetic model: a control id in 2048..3071, the
# range ChooseCode0 (talker.pas:607-609) keeps only for eos
CODEC_EOS = 2150
STD = 0.02

CONFIG = dict(hidden=HIDDEN, heads=HEADS, kv_heads=KV_HEADS, head_dim=HEAD_DIM, intermediate=INTER,
              rms_eps=EPS, rope_theta=THETA)

_TENSORS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "in_norm", "post_norm", "q_norm", "k_norm")
_STACK_ID = {"talker": 1, "predictor": 2, "heads": 3, "emb": 4, "text": 5, "prompt": 6}


def _rng(*key):
    return np.random.default_rng(list(key))


def normal(shape, std, *key):
    return (_rng(*key).standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def layer(seed, stack, index):
    """One layer's tensors ([out][in] matrices) of stack 'talker' or 'predictor'."""
    sid = _STACK_ID[stack]
    q, kv = HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM
    shapes = {"wq": (q, HIDDEN), "wk": (kv, HIDDEN), "wv": (kv, HIDDEN), "wo": (HIDDEN, q),
              "wg": (INTER, HIDDEN), "wu": (INTER, HIDDEN), "wd": (HIDDEN, INTER)}
    out = {}
    for t, name in enumerate(_TENSORS):
        if name in shapes:
            out[name] = normal(shapes[name], STD, seed, sid, index, t)
        else:
            n = HEAD_DIM if name in ("q_norm", "k_norm") else HIDDEN
            out[name] = (1.0 + normal((n,), STD, seed, sid, index, t)).astype(np.float32)
    return out


def stack(seed, name, layers):
    """(list of layer dicts, final_norm) of one stack."""
    sid = _STACK_ID[name]
    ls = [layer(seed, name, i) for i in range(layers)]
    final = (1.0 + normal((HIDDEN,), STD, seed, sid, 1000)).astype(np.float32)
    return ls, final


def talker_head(seed, vocab=TALKER_VOCAB):
    return normal((vocab, HIDDEN), STD, seed, _STACK_ID["heads"], 0)


def predictor_heads(seed, groups=GROUPS, vocab=PRED_VOCAB):
    return [normal((vocab, HIDDEN), STD, seed, _STACK_ID["heads"], 1 + g) for g in range(groups - 1)]


def codec_embedding(seed, vocab=TALKER_VOCAB):
    return normal((vocab, HIDDEN), STD, seed, _STACK_ID["emb"], 0)


def predictor_embeddings(seed, groups=GROUPS, vocab=PRED_VOCAB):
    return normal((groups - 1, vocab, HIDDEN), STD, seed, _STACK_ID["emb"], 1)


def prompt(seed, rows, key=0):
    """N(0, 1) embedding rows (a prefill, or the 128 prior positions)."""
    return normal((rows, HIDDEN), 1.0, seed, _STACK_ID["prompt"], key)


def text_rows(seed, rows, key=0):
    """Rows standing for text projections: trailing rows / tts_pad."""
    return normal((rows, HIDDEN), STD, seed, _STACK_ID["text"], key)


def lcg_rows(rows, seed=12345, hidden=HIDDEN):
    """The pseudo-random inputs of the reference's ComparePredictor
    (tests/test.tts.qwen.vulkan.pas:189-198): seed*1664525+1013904223,
    x = (int(seed shr 8)/2^24 - 0.5) * 0.2; returns (rows, next seed)."""
    out = np.empty(rows * hidden, dtype=np.float32)
    s = seed & 0xFFFFFFFF
    for i in range(out.size):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = ((s >> 8) / float(1 << 24) - 0.5) * 0.2
    return out.reshape(rows, hidden), s
