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


# the 12 Hz decoder (TQwenCodec, codec.pas): seeded weights under the
# speech_tokenizer checkpoint's names and PyTorch shapes
CODEC_RATES = (8, 5, 4, 3)


def codec_weights(seed):
    rng = np.random.default_rng(seed)
    W = {}

    def lin(name, *shape, gain=1.0):
        fan_in = int(np.prod(shape[1:]))
        W[name] = (rng.standard_normal(shape) * gain / np.sqrt(fan_in)).astype(np.float32)

    def vec(name, n, mean=0.0, std=0.1):
        W[name] = (mean + rng.standard_normal(n) * std).astype(np.float32)

    for g in range(16):
        p = ("decoder.quantizer.rvq_first.vq.layers.0._codebook" if g == 0
             else f"decoder.quantizer.rvq_rest.vq.layers.{g - 1}._codebook")
        W[p + ".embedding_sum"] = rng.standard_normal((2048, 256)).astype(np.float32)
        W[p + ".cluster_usage"] = rng.uniform(0.5, 4.0, 2048).astype(np.float32)
    W["decoder.quantizer.rvq_rest.vq.layers.3._codebook.cluster_usage"][:5] = 0.0  # the 1e-5 floor
    lin("decoder.quantizer.rvq_first.output_proj.weight", 512, 256, 1, gain=0.5)
    lin("decoder.quantizer.rvq_rest.output_proj.weight", 512, 256, 1, gain=0.2)
    lin("decoder.pre_conv.conv.weight", 1024, 512, 3)
    vec("decoder.pre_conv.conv.bias", 1024)
    p = "decoder.pre_transformer."
    lin(p + "input_proj.weight", 512, 1024)
    vec(p + "input_proj.bias", 512)
    lin(p + "output_proj.weight", 1024, 512)
    vec(p + "output_proj.bias", 1024)
    vec(p + "norm.weight", 512, 1.0)
    for l in range(8):
        q = f"{p}layers.{l}."
        vec(q + "input_layernorm.weight", 512, 1.0)
        vec(q + "post_attention_layernorm.weight", 512, 1.0)
        for n in ("q", "k", "v"):
            lin(q + f"self_attn.{n}_proj.weight", 1024, 512)
        lin(q + "self_attn.o_proj.weight", 512, 1024)
        lin(q + "mlp.gate_proj.weight", 1024, 512)
        lin(q + "mlp.up_proj.weight", 1024, 512)
        lin(q + "mlp.down_proj.weight", 512, 1024)
        vec(q + "self_attn_layer_scale.scale", 512, 0.3)
        vec(q + "mlp_layer_scale.scale", 512, 0.3)
    for i in range(2):
        lin(f"decoder.upsample.{i}.0.conv.weight", 1024, 1024, 2)
        vec(f"decoder.upsample.{i}.0.conv.bias", 1024)
        q = f"decoder.upsample.{i}.1."
        lin(q + "dwconv.conv.weight", 1024, 1, 7)
        vec(q + "dwconv.conv.bias", 1024)
        vec(q + "norm.weight", 1024, 1.0)
        vec(q + "norm.bias", 1024)
        lin(q + "pwconv1.weight", 4096, 1024)
        vec(q + "pwconv1.bias", 4096)
        lin(q + "pwconv2.weight", 1024, 4096)
        vec(q + "pwconv2.bias", 1024)
        vec(q + "gamma", 1024, 0.3)
    lin("decoder.decoder.0.conv.weight", 1536, 1024, 7)
    vec("decoder.decoder.0.conv.bias", 1536)
    for b in range(4):
        cin, cout, rate = 1536 >> b, 1536 >> (b + 1), CODEC_RATES[b]
        q = f"decoder.decoder.{b + 1}.block."
        vec(q + "0.alpha", cin)
        vec(q + "0.beta", cin)
        lin(q + "1.conv.weight", cin, cout, 2 * rate, gain=0.7)
        vec(q + "1.conv.bias", cout)
        for r in range(3):
            u = f"{q}{r + 2}."
            vec(u + "act1.alpha", cout)
            vec(u + "act1.beta", cout)
            lin(u + "conv1.conv.weight", cout, cout, 7, gain=0.5)
            vec(u + "conv1.conv.bias", cout)
            vec(u + "act2.alpha", cout)
            vec(u + "act2.beta", cout)
            lin(u + "conv2.conv.weight", cout, cout, 1, gain=0.5)
            vec(u + "conv2.conv.bias", cout)
    vec("decoder.decoder.5.alpha", 96)
    vec("decoder.decoder.5.beta", 96)
    lin("decoder.decoder.6.conv.weight", 1, 96, 7, gain=0.3)
    vec("decoder.decoder.6.conv.bias", 1, 0.0, 0.01)
    return W


# The inputs of the benchmark workloads (BASELINE.json configs[1]-[3]), shared
# by bench.py and by the full-size parity fixtures, so that the parity tests
# check exactly what is timed.  `rank` offsets the draws of a replica.
def config1_prompt(seed=1, rows=40, rank=0):
    """the N(0, 1) prompt of the streaming utterance."""
    return prompt(seed + 100 + rank, rows)


def config2_contexts(seed=1, n=64, lo=50, hi=1000, rank=0):
    """per-utterance context lengths, uniform in [lo, hi]."""
    return np.random.default_rng(seed + 7 + rank).integers(lo, hi + 1, n)


def config2_prompt(s, rows, seed=1):
    """the N(0, 1) rows that fill utterance s's context."""
    return prompt(seed + 1000 + s, rows)


def config4_lengths(seed=1, n=1024, lo=20, hi=80):
    """the prompt rows of every utterance of the box (utterance
    u: entry u), uniform in [lo, hi]."""
    return np.random.default_rng(seed + 13).integers(lo, hi + 1, n)


def config4_prompt(u, rows, seed=1):
    """the N(0, 1) prompt rows of utterance u."""
    return prompt(seed + 3000 + u, rows)


def config3_lengths(seed=1, n=16, lo=256, hi=2048, rank=0):
    """prefill prompt lengths, uniform in [lo, hi]."""
    return np.random.default_rng(seed + 11 + rank).integers(lo, hi + 1, n)


def config3_prompt(i, rows, seed=1):
    """the N(0, 1) rows of prompt i."""
    return prompt(seed + 2000 + i, rows)
