"""ctypes wrapper of liboracle.so, the CPU restatement of the reference's
per-frame language-model path (qtts_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, as the checker.  The product
(libqtts.so and the package) never imports it.

Objects follow the reference: OraStack (QwenLmStack, lm.pas:174-179),
OraHeads (TQwenLmHeads, lm.pas:64-100), OraLm (TQwenLm, lm.pas:102-143),
OraTalker (TQwenTalker.Start/NextFrame, talker.pas:471-681), OraCodec (the
12 Hz decoder TQwenCodec, codec.pas; qtts_codec_oracle.c).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, Q8_0 = 0, 1
ACT_F32, ACT_Q8_0 = 0, 1


class OraConfig(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_int), ("hidden", ctypes.c_int), ("heads", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("inter", ctypes.c_int),
                ("eps", ctypes.c_float), ("theta", ctypes.c_float), ("dtype", ctypes.c_int)]


class OraLayerSrc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("in_norm", "post_norm", "q_norm", "k_norm",
                                                "wq", "wk", "wv", "wo", "wg", "wu", "wd")]


P = ctypes.c_void_p


def build():
    """Compile liboracle.so with the Makefile next to this file."""
    subprocess.run(["make", "-C", HERE, "-s"], check=True)


def _load():
    if not os.path.exists(LIB_PATH):
        build()
    lib = ctypes.CDLL(LIB_PATH)
    sig = {
        "ora_set_threads": (None, [ctypes.c_int]),
        "ora_get_threads": (ctypes.c_int, []),
        "ora_set_act_mode": (None, [ctypes.c_int]),
        "ora_quantize_q8_0": (None, [P, ctypes.c_int64, P]),
        "ora_dequantize_q8_0": (None, [P, ctypes.c_int64, P]),
        "ora_crc32c": (ctypes.c_uint32, [ctypes.c_uint32, P, ctypes.c_size_t]),
        "ora_stack_create": (P, [ctypes.POINTER(OraConfig), ctypes.POINTER(OraLayerSrc), P]),
        "ora_stack_free": (None, [P]),
        "ora_heads_create": (P, [ctypes.c_int, ctypes.c_int]),
        "ora_heads_add": (ctypes.c_int, [P, P, ctypes.c_int]),
        "ora_heads_digest": (ctypes.c_uint32, [P]),
        "ora_heads_free": (None, [P]),
        "ora_lm_create": (P, [P, ctypes.c_int]),
        "ora_lm_free": (None, [P]),
        "ora_lm_reset": (None, [P]),
        "ora_lm_length": (ctypes.c_int, [P]),
        "ora_lm_set_kv_f16": (None, [P, ctypes.c_int]),
        "ora_lm_forward": (ctypes.c_int, [P, P, ctypes.c_int, P, ctypes.c_int, P, P, P, P]),
        "ora_argmax": (ctypes.c_int, [P, ctypes.c_int]),
        "ora_choose_code0": (ctypes.c_int, [P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, ctypes.c_float, P]),
        "ora_talker_create": (P, [P, P, P, P, P, ctypes.c_int, P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_float]),
        "ora_talker_free": (None, [P]),
        "ora_codec_create": (P, [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(P),
                                 ctypes.POINTER(ctypes.c_int64)]),
        "ora_codec_free": (None, [P]),
        "ora_codec_reset": (None, [P]),
        "ora_codec_frames": (ctypes.c_longlong, [P]),
        "ora_codec_decode": (ctypes.c_int, [P, P, ctypes.c_int, P]),
        "ora_codec_error": (ctypes.c_char_p, []),
        "ora_talker_start": (ctypes.c_int, [P, P, ctypes.c_int, P, ctypes.c_int, P]),
        "ora_talker_next_frame": (ctypes.c_int, [P, P]),
        "ora_talker_next_frame_margins": (ctypes.c_int, [P, P, P]),
        "ora_talker_check_frame": (ctypes.c_int, [P, P, P]),
        "ora_talker_check_frame_ranks": (ctypes.c_int, [P, P, P, P]),
        "ora_talker_logits": (P, [P]),
        "ora_talker_set_sampling": (None, [P, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                           ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                           ctypes.c_uint64]),
        "ora_sample": (ctypes.c_int, [P, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                      ctypes.c_float]),
        "ora_sample_uniform": (ctypes.c_float, [ctypes.c_uint64, ctypes.c_int, ctypes.c_int]),
        "ora_text_project": (None, [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P, P, P, P, P]),
        "ora_talker_hidden": (P, [P]),
        "ora_rope_table": (None, [ctypes.c_int, ctypes.c_int, ctypes.c_float, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n):
    lib.ora_set_threads(int(n))


def threads():
    return lib.ora_get_threads()


def set_act_mode(mode):
    lib.ora_set_act_mode(mode)


def quantize_q8_0(x):
    """ggml quantize_row_q8_0_ref: float32 -> blocks of 34 bytes."""
    x = _f32(x).reshape(-1)
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    lib.ora_quantize_q8_0(_p(x), x.size, _p(out))
    return out


def dequantize_q8_0(q, n):
    q = np.ascontiguousarray(q, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    lib.ora_dequantize_q8_0(_p(q), n, _p(out))
    return out


def crc32c(data, crc=0):
    a = np.ascontiguousarray(np.frombuffer(bytes(data), dtype=np.uint8) if isinstance(data, (bytes, bytearray))
                             else data).view(np.uint8)
    return lib.ora_crc32c(crc, _p(a), a.size)


def argmax(x):
    x = _f32(x)
    return lib.ora_argmax(_p(x), x.size)


def choose_code0(logits, eos, history, penalty=1.05):
    lg = _f32(logits)
    h = np.ascontiguousarray(history, dtype=np.int32)
    work = np.empty_like(lg)
    return lib.ora_choose_code0(_p(lg), lg.size, eos, _p(h) if h.size else None, h.size, penalty, _p(work))


def sample_uniform(seed, step, group):
    """u in [0, 1) of draw (step, group) of a stream (seed)."""
    return lib.ora_sample_uniform(seed, step, group)


def sample(work, temperature, top_k, top_p, u):
    """TInferSampler.Next restated (qtts_oracle.c): the index drawn from
    work (logits after the processors) with the uniform u."""
    w = _f32(work)
    return lib.ora_sample(_p(w), w.size, temperature, top_k, top_p, u)


def text_project(emb, ids, w1, b1, w2, b2):
    """TQwenTalker.TextProject restated: [n][hidden] float32."""
    emb, w1, b1, w2, b2 = (_f32(a) for a in (emb, w1, b1, w2, b2))
    i = np.ascontiguousarray(ids, dtype=np.int32)
    vocab, th = emb.shape
    hidden = w2.shape[0]
    y = np.zeros((i.size, hidden), np.float32)
    lib.ora_text_project(_p(emb), vocab, th, hidden, _p(i), i.size, _p(w1), _p(b1), _p(w2), _p(b2), _p(y))
    return y


def start_rows(emb, w1, b1, w2, b2, codec_emb, tokens, ids, codec, non_streaming=False):
    """The rows of TQwenTalker.Start (talker.pas:528-574) restated step by
    step: (prefill, trailing, tts_pad).  tokens: dict with tts_bos, tts_eos,
    tts_pad, codec_pad, codec_bos.  The tts vectors are projections of their
    token ids (talker.pas:339-344); AddRow adds a codec embedding row."""
    ce = _f32(codec_emb)
    proj = lambda t: text_project(emb, list(t), w1, b1, w2, b2)  # noqa: E731
    tts_bos, tts_eos, tts_pad = (proj([tokens[k]])[0] for k in ("tts_bos", "tts_eos", "tts_pad"))
    ids = list(ids)
    n_codec = len(codec)
    text = ids[3:3 + len(ids) - 8]
    n_text = len(text)
    hidden = ce.shape[1]
    if non_streaming:
        rows = 3 + (n_codec - 1) + (n_text + 1) + 1
    else:
        rows = 3 + (n_codec - 1) + 1
    prefill = np.zeros((rows, hidden), np.float32)
    prefill[0:3] = proj(ids[0:3])
    r = 3
    for i in range(n_codec - 1):
        prefill[r] = tts_pad if i < n_codec - 2 else tts_bos
        prefill[r] += ce[codec[i]]
        r += 1
    if non_streaming:
        prefill[r:r + n_text] = proj(text)
        prefill[r + n_text] = tts_eos
        for i in range(n_text + 1):
            prefill[r + i] += ce[tokens["codec_pad"]]
        r += n_text + 1
        prefill[r] = tts_pad
        prefill[r] += ce[tokens["codec_bos"]]
        trailing = tts_pad[None, :].copy()
    else:
        prefill[r] = proj(text[0:1])[0]
        prefill[r] += ce[tokens["codec_bos"]]
        trailing = np.zeros((n_text, hidden), np.float32)
        if n_text > 1:
            trailing[0:n_text - 1] = proj(text[1:])
        trailing[n_text - 1] = tts_eos
    return prefill, trailing, tts_pad


class OraCodec:
    """TQwenCodec (the 12 Hz decoder, codec.pas) on the CPU: weights = dict
    of the checkpoint's tensor names -> float32 arrays (the speech_tokenizer
    model.safetensors, PyTorch layouts).  decode(codes [frames][16]) ->
    frames * 1920 samples; frames of successive calls follow each other."""

    FRAME_SAMPLES = 1920

    def __init__(self, weights):
        self._keep = {k: _f32(v) for k, v in weights.items()}
        names = list(self._keep)
        n = len(names)
        cn = (ctypes.c_char_p * n)(*[k.encode() for k in names])
        cp = (P * n)(*[self._keep[k].ctypes.data for k in names])
        cc = (ctypes.c_int64 * n)(*[self._keep[k].size for k in names])
        self.handle = lib.ora_codec_create(n, cn, cp, cc)
        if not self.handle:
            raise ValueError("oracle codec: " + lib.ora_codec_error().decode())

    def decode(self, codes):
        c = np.ascontiguousarray(codes, dtype=np.int32).reshape(-1, 16)
        pcm = np.zeros(c.shape[0] * self.FRAME_SAMPLES, np.float32)
        if lib.ora_codec_decode(self.handle, _p(c), c.shape[0], _p(pcm)):
            raise ValueError("oracle codec: " + lib.ora_codec_error().decode())
        return pcm

    def reset(self):
        lib.ora_codec_reset(self.handle)

    @property
    def frames(self):
        return lib.ora_codec_frames(self.handle)

    def free(self):
        if self.handle:
            lib.ora_codec_free(self.handle)
            self.handle = None


def rope_table(max_pos, head_dim, theta):
    c = np.empty((max_pos, head_dim // 2), dtype=np.float32)
    s = np.empty_like(c)
    lib.ora_rope_table(max_pos, head_dim, theta, _p(c), _p(s))
    return c, s


class OraStack:
    """QwenLmStack on the CPU: layers = list of dicts (wq..wd [out][in],
    in_norm, post_norm, q_norm, k_norm); dtype 'f32' or 'q8_0'."""

    def __init__(self, config, layers, final_norm, dtype="f32"):
        c = config
        self.cfg = OraConfig(len(layers), c["hidden"], c["heads"], c["kv_heads"], c["head_dim"],
                             c["intermediate"], c["rms_eps"], c["rope_theta"], F32 if dtype == "f32" else Q8_0)
        keep = []
        srcs = (OraLayerSrc * len(layers))()
        for i, L in enumerate(layers):
            arrs = {k: _f32(L[k]) for k in ("in_norm", "post_norm", "q_norm", "k_norm",
                                            "wq", "wk", "wv", "wo", "wg", "wu", "wd")}
            keep.append(arrs)
            for k, a in arrs.items():
                setattr(srcs[i], k, a.ctypes.data)
        fn = _f32(final_norm)
        self.handle = lib.ora_stack_create(ctypes.byref(self.cfg), srcs, _p(fn))
        self.hidden = c["hidden"]
        self.layers = len(layers)

    def free(self):
        if self.handle:
            lib.ora_stack_free(self.handle)
            self.handle = None


class OraHeads:
    def __init__(self, hidden, dtype="f32"):
        self.hidden = hidden
        self.handle = lib.ora_heads_create(hidden, F32 if dtype == "f32" else Q8_0)
        self.rows_ = []

    def add(self, tensor):
        t = _f32(tensor)
        self.rows_.append(t.size // self.hidden)
        return lib.ora_heads_add(self.handle, _p(t), t.size // self.hidden)

    def rows(self, i):
        return self.rows_[i]

    def digest(self):
        return lib.ora_heads_digest(self.handle)

    def free(self):
        if self.handle:
            lib.ora_heads_free(self.handle)
            self.handle = None


class OraLm:
    """TQwenLm on the CPU (the stack is owned by the caller here); kv_f16:
    the cache in half floats (TQwenLm.Create's aKvF16)."""

    def __init__(self, stack, heads, max_pos=4096, kv_f16=False):
        self.stack = stack
        self.heads = heads
        self.hidden = stack.hidden
        self.handle = lib.ora_lm_create(stack.handle, max_pos)
        if kv_f16:
            lib.ora_lm_set_kv_f16(self.handle, 1)

    def reset(self):
        lib.ora_lm_reset(self.handle)

    @property
    def length(self):
        return lib.ora_lm_length(self.handle)

    def forward(self, x, output=0, logits=None, hidden=None, states=None, normed=None):
        x = _f32(x)
        rows = x.size // self.hidden
        rc = lib.ora_lm_forward(self.handle, _p(x), rows, self.heads.handle if self.heads else None, output,
                                _p(logits), _p(hidden), _p(states), _p(normed))
        if rc:
            raise RuntimeError("oracle: KV cache full")

    def free(self):
        if self.handle:
            lib.ora_lm_free(self.handle)
            self.handle = None


class OraTalker:
    """TQwenTalker's frame loop (greedy, or sampling after set_sampling) on
    the CPU."""

    def __init__(self, talker, theads, pred, pheads, codec_emb, pred_emb, eos, penalty=1.05, groups=16):
        self.ce = _f32(codec_emb)
        self.pe = _f32(pred_emb)
        vocab = self.ce.shape[0]
        pvocab = self.pe.shape[1]
        self.groups = groups
        self.handle = lib.ora_talker_create(talker.handle, theads.handle, pred.handle, pheads.handle, _p(self.ce),
                                            vocab, _p(self.pe), pvocab, groups, eos, penalty)
        self.hidden = talker.hidden
        self.vocab = vocab

    def set_sampling(self, do_sample=True, temperature=0.9, top_k=50, top_p=1.0, sub_do_sample=True,
                     sub_temperature=0.9, sub_top_k=50, sub_top_p=1.0, seed=0):
        """TQwenSampling (talker.pas:59-73); defaults of qwen_tts (203-229)."""
        lib.ora_talker_set_sampling(self.handle, int(do_sample), temperature, top_k, top_p, int(sub_do_sample),
                                    sub_temperature, sub_top_k, sub_top_p, seed)

    def start(self, prefill, trailing, tts_pad):
        p = _f32(prefill)
        t = _f32(trailing) if trailing is not None and len(trailing) else None
        rc = lib.ora_talker_start(self.handle, _p(p), p.size // self.hidden, _p(t),
                                  0 if t is None else t.size // self.hidden, _p(_f32(tts_pad)))
        if rc:
            raise RuntimeError("oracle: KV cache full")

    def next_frame(self, codes):
        rc = lib.ora_talker_next_frame(self.handle, _p(codes))
        if rc < 0:
            raise RuntimeError("oracle: KV cache full")
        return rc == 1

    def next_frame_margins(self, codes):
        """next_frame (greedy) with the margin of each choice: returns
        (more, margins), margins[g] = the chosen value minus the next
        largest value of choice g (after the processors)."""
        m = np.zeros(self.groups, np.float32)
        rc = lib.ora_talker_next_frame_margins(self.handle, _p(codes), _p(m))
        if rc < 0:
            raise RuntimeError("oracle: KV cache full")
        return rc == 1, m

    def check_frame(self, codes):
        """The frame whose codes were chosen elsewhere: returns (more, gaps),
        gaps[g] = how far codes[g] falls below the best value of choice g
        (0 when it is a first maximum or a tie)."""
        c = np.ascontiguousarray(codes, dtype=np.int32)
        gap = np.zeros(self.groups, np.float32)
        rc = lib.ora_talker_check_frame(self.handle, _p(c), _p(gap))
        if rc < 0:
            raise RuntimeError("oracle: KV cache full")
        return rc == 1, gap

    def check_frame_ranks(self, codes):
        """check_frame with the rank of each choice among its values (after
        the processors): returns (more, gaps, ranks)."""
        c = np.ascontiguousarray(codes, dtype=np.int32)
        gap = np.zeros(self.groups, np.float32)
        rank = np.zeros(self.groups, np.int32)
        rc = lib.ora_talker_check_frame_ranks(self.handle, _p(c), _p(gap), _p(rank))
        if rc < 0:
            raise RuntimeError("oracle: KV cache full")
        return rc == 1, gap, rank

    def logits(self):
        ptr = lib.ora_talker_logits(self.handle)
        return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), (self.vocab,)).copy()

    def hidden_state(self):
        ptr = lib.ora_talker_hidden(self.handle)
        return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), (self.hidden,)).copy()

    def free(self):
        if self.handle:
            lib.ora_talker_free(self.handle)
            self.handle = None
