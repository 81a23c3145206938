"""Host-side mirror of mormot2-qwen-tts's stack API over libqtts.so (ctypes).

The reference is Object Pascal; its stack API lives in
src/tts/mormot.ai.tts.qwen.lm.pas and its frame loop in
src/tts/mormot.ai.tts.qwen.talker.pas.  This module keeps the same objects,
names, argument meanings and error behaviour on top of the C-ABI of
include/qtts.h, so that the tests read like the reference's own tests:

    QwenVulkan-like device   -> QwenDevice            (lm.pas:43-62)
    QwenLmStack(...)         -> qwen_lm_stack(...)     (lm.pas:149-150, 174-179)
    TQwenLmHeads             -> QwenLmHeads            (lm.pas:64-100)
    TQwenLm                  -> QwenLm                 (lm.pas:102-143)
    TQwenTalker (per frame)  -> QwenTalker             (talker.pas:471-681)
    EQwenLm                  -> EQwenLm

Every failure of the library raises EQwenLm with qtts_last_error(), as the
reference raises EQwenLm (lm.pas:167, 232-234, 345).  There is no CPU path:
if libqtts.so is missing the import fails.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqtts.so")

DTYPE_F32 = 0
DTYPE_Q8_0 = 1
DTYPE_BF16 = 2
DTYPES = {"f32": DTYPE_F32, "q8_0": DTYPE_Q8_0, "bf16": DTYPE_BF16, "f16": 3}

E_ARG, E_OOM, E_CUDA, E_CAPACITY, E_TIMEOUT, E_STATE = 1, 2, 3, 4, 5, 6


class EQwenLm(RuntimeError):
    """A failure of the stack library (the reference's EQwenLm)."""

    def __init__(self, code, message):
        super().__init__(f"qtts error {code}: {message}")
        self.code = code


class StackConfig(ctypes.Structure):
    _fields_ = [("layers", ctypes.c_int32), ("hidden", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float), ("dtype", ctypes.c_int32)]


class LayerSrc(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32)] + [(n, ctypes.c_void_p) for n in (
        "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj",
        "input_norm", "post_norm", "q_norm", "k_norm")]


class TalkerConfig(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_int32), ("pred_vocab", ctypes.c_int32), ("groups", ctypes.c_int32),
                ("codec_eos", ctypes.c_int32), ("repetition_penalty", ctypes.c_float)]


class Sampling(ctypes.Structure):
    """TQwenSampling (talker.pas:60-73)."""
    _fields_ = [("do_sample", ctypes.c_int32), ("temperature", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("top_p", ctypes.c_float), ("sub_do_sample", ctypes.c_int32), ("sub_temperature", ctypes.c_float),
                ("sub_top_k", ctypes.c_int32), ("sub_top_p", ctypes.c_float), ("seed", ctypes.c_uint64)]


class PromptTokens(ctypes.Structure):
    """The token ids around the text in TQwenTalker.Start (talker.pas:256-265)."""
    _fields_ = [("tts_bos", ctypes.c_int32), ("tts_eos", ctypes.c_int32), ("tts_pad", ctypes.c_int32),
                ("codec_pad", ctypes.c_int32), ("codec_bos", ctypes.c_int32)]


def prompt_tokens(config):
    """PromptTokens from a config.json dict (TQwenTalker.Create, talker.pas:
    256-261): tts_*_token_id at the top, codec_*_id in talker_config."""
    tc = config["talker_config"]
    return PromptTokens(config["tts_bos_token_id"], config["tts_eos_token_id"], config["tts_pad_token_id"],
                        tc["codec_pad_id"], tc["codec_bos_id"])


def start_codec_ids(talker_config, speaker="", language=""):
    """The codec ids of TQwenTalker.Start (talker.pas:488-527): think,
    think_bos, language, think_eos (nothink, think_bos, think_eos when the
    language is auto), the voice, then codec_pad and codec_bos.  A dialect
    voice (spk_is_dialect naming a codec language) speaking chinese or auto
    takes that language.  Unknown voice or language: EQwenLm, as Start
    raises."""
    tc = talker_config
    spk = (speaker or "").lower()
    spk_id = -1
    if spk:
        if spk not in tc.get("spk_id", {}):
            raise EQwenLm(E_ARG, "Start: unknown speaker %r" % speaker)
        spk_id = int(tc["spk_id"][spk])
    lang = (language or "").lower() or "auto"
    lang_id = -1
    if lang != "auto":
        if lang not in tc.get("codec_language_id", {}):
            raise EQwenLm(E_ARG, "Start: unknown language %r" % language)
        lang_id = int(tc["codec_language_id"][lang])
    if spk and lang in ("chinese", "auto"):
        d = tc.get("spk_is_dialect", {}).get(spk)
        d = "" if d is None else (str(d).lower() if isinstance(d, bool) else str(d))
        if d not in ("", "false", "true") and d in tc.get("codec_language_id", {}):
            lang_id = int(tc["codec_language_id"][d])
    if lang_id < 0:
        codec = [tc["codec_nothink_id"], tc["codec_think_bos_id"], tc["codec_think_eos_id"]]
    else:
        codec = [tc["codec_think_id"], tc["codec_think_bos_id"], lang_id, tc["codec_think_eos_id"]]
    if spk_id >= 0:
        codec.append(spk_id)
    return codec + [tc["codec_pad_id"], tc["codec_bos_id"]]


P = ctypes.c_void_p
I = ctypes.c_int
PI = ctypes.POINTER(ctypes.c_int)

# name -> argtypes; every entry returns int (0 = ok)
EXPORTS = {
    "qtts_device_open": [I, ctypes.POINTER(P)],
    "qtts_device_name": [P, ctypes.c_char_p, I],
    "qtts_device_bytes": [P, ctypes.POINTER(ctypes.c_int64)],
    "qtts_device_close": [P],
    "qtts_stack_create": [P, ctypes.POINTER(StackConfig), ctypes.POINTER(LayerSrc), P, ctypes.POINTER(P)],
    "qtts_safetensors_open": [ctypes.c_char_p, ctypes.POINTER(P)],
    "qtts_safetensors_count": [P, PI],
    "qtts_safetensors_name": [P, I, ctypes.c_char_p, I],
    "qtts_safetensors_tensor": [P, ctypes.c_char_p, PI, PI, P, ctypes.POINTER(P), ctypes.POINTER(ctypes.c_int64)],
    "qtts_safetensors_close": [P],
    "qtts_stack_create_safetensors": [P, ctypes.POINTER(StackConfig), P, ctypes.c_char_p, ctypes.POINTER(P)],
    "qtts_heads_add_safetensors": [P, P, ctypes.c_char_p, I, PI],
    "qtts_codec_create_safetensors": [P, P, ctypes.POINTER(P)],
    "qtts_codec_reset": [P],
    "qtts_codec_decode": [P, P, I, P],
    "qtts_codec_frames": [P, ctypes.POINTER(ctypes.c_int64)],
    "qtts_codec_destroy": [P],
    "qtts_stack_save": [P, ctypes.c_char_p],
    "qtts_stack_load": [P, ctypes.c_char_p, ctypes.POINTER(P)],
    "qtts_stack_bytes": [P, ctypes.POINTER(ctypes.c_int64)],
    "qtts_stack_destroy": [P],
    "qtts_heads_create": [P, ctypes.c_char_p, I, I, ctypes.POINTER(P)],
    "qtts_heads_add": [P, P, I, I, PI],
    "qtts_heads_digest": [P, ctypes.POINTER(ctypes.c_uint32)],
    "qtts_heads_count": [P, PI],
    "qtts_heads_rows": [P, I, PI],
    "qtts_heads_bytes": [P, ctypes.POINTER(ctypes.c_int64)],
    "qtts_heads_linear": [P, I, P, I, P],
    "qtts_heads_destroy": [P],
    "qtts_lm_create": [P, P, I, ctypes.POINTER(P)],
    "qtts_lm_reset": [P],
    "qtts_lm_forward": [P, P, I, I, P, P],
    "qtts_lm_forward_noalloc": [P, P, I, I, P, P],
    "qtts_lm_length": [P, PI],
    "qtts_lm_set_wait_test": [P, I, ctypes.c_int64],
    "qtts_lm_set_launch_epoch": [P, ctypes.c_uint32],
    "qtts_lm_create_kv": [P, P, I, I, ctypes.POINTER(P)],
    "qtts_lm_destroy": [P],
    "qtts_batch_create": [P, P, I, I, I, I, ctypes.POINTER(P)],
    "qtts_batch_reset": [P, I],
    "qtts_batch_length": [P, I, PI],
    "qtts_batch_forward": [P, I, P, P, P, I, P, P],
    "qtts_batch_destroy": [P],
    "qtts_talker_create": [P, P, ctypes.POINTER(TalkerConfig), P, P, ctypes.POINTER(P)],
    "qtts_talker_start": [P, P, I, P, I, P, P, P],
    "qtts_talker_next_frame": [P, P, PI],
    "qtts_talker_run": [P, I, P, PI],
    "qtts_talker_trace_frame": [P, P, PI, P, I, PI],
    "qtts_talker_stream": [P, ctypes.POINTER(P)],
    "qtts_talker_probe": [P, P, P],
    "qtts_talker_step": [P, PI],
    "qtts_talker_destroy": [P],
    "qtts_talker_set_sampling": [P, ctypes.POINTER(Sampling)],
    "qtts_talkers_set_sampling": [P, ctypes.POINTER(Sampling)],
    "qtts_sample": [P, P, I, ctypes.c_float, I, ctypes.c_float, ctypes.c_uint64, I, I, PI],
    "qtts_talkers_create": [P, P, ctypes.POINTER(TalkerConfig), P, P, ctypes.POINTER(P)],
    "qtts_talkers_start": [P, I, P, P, P, P, P, P],
    "qtts_talkers_start_prompt": [P, P, ctypes.POINTER(PromptTokens), I, P, P, P, P, P, P],
    "qtts_talkers_next_frame": [P, I, P, P, P],
    "qtts_talkers_stream": [P, ctypes.POINTER(P)],
    "qtts_talkers_probe": [P, I, P, P],
    "qtts_talkers_destroy": [P],
    "qtts_quantize_q8_0": [P, P, ctypes.c_int64, P],
    "qtts_textproj_create": [P, I, I, I, I, P, P, P, P, P, ctypes.POINTER(P)],
    "qtts_text_project": [P, P, I, P],
    "qtts_textproj_destroy": [P],
    "qtts_prompt_plan": [ctypes.POINTER(PromptTokens), P, I, P, I, I, P, P, I, PI, PI],
    "qtts_talker_start_prompt": [P, P, ctypes.POINTER(PromptTokens), P, I, P, I, I, P, P],
    "qtts_talker_prompt_rows": [P, P, ctypes.POINTER(PromptTokens), P, I, P, I, I, P, I, P, I, PI, PI],
}


def load_library(path=LIB_PATH):
    """Load libqtts.so and declare its entry points (fails loudly if absent)."""
    if not os.path.exists(path):
        raise EQwenLm(E_ARG, f"{path} is missing: build it (python __graft_entry__.py or make -C {HERE})")
    lib = ctypes.CDLL(path)
    for name, args in EXPORTS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.qtts_last_error.argtypes = []
    lib.qtts_last_error.restype = ctypes.c_char_p
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = load_library()
    return _lib


def check(rc):
    if rc != 0:
        raise EQwenLm(rc, lib().qtts_last_error().decode(errors="replace"))


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def prompt_plan(tokens, ids, codec, non_streaming=False):
    """The rows of TQwenTalker.Start as (text token, codec id or -1) pairs:
    (prefill [rows][2], trailing [trailing_rows][2]), computed by the
    library on the host (qtts_prompt_plan, no device)."""
    i = np.ascontiguousarray(ids, dtype=np.int32)
    c = np.ascontiguousarray(codec, dtype=np.int32)
    rows, tr = ctypes.c_int(), ctypes.c_int()
    check(lib().qtts_prompt_plan(ctypes.byref(tokens), _ptr(i), i.size, _ptr(c), c.size, int(non_streaming), None,
                                 None, 0, ctypes.byref(rows), ctypes.byref(tr)))
    n = rows.value + tr.value
    t_out = np.zeros(n, np.int32)
    c_out = np.zeros(n, np.int32)
    check(lib().qtts_prompt_plan(ctypes.byref(tokens), _ptr(i), i.size, _ptr(c), c.size, int(non_streaming),
                                 _ptr(t_out), _ptr(c_out), n, ctypes.byref(rows), ctypes.byref(tr)))
    plan = np.stack([t_out, c_out], 1)
    return plan[:rows.value], plan[rows.value:]


class QwenDevice:
    """One CUDA device (the role of TQwenVulkan, lm.pas:43-62)."""

    def __init__(self, ordinal=0):
        h = P()
        check(lib().qtts_device_open(ordinal, ctypes.byref(h)))
        self.handle = h

    @property
    def name(self):
        buf = ctypes.create_string_buffer(256)
        check(lib().qtts_device_name(self.handle, buf, 256))
        return buf.value.decode()

    @property
    def device_bytes(self):
        v = ctypes.c_int64()
        check(lib().qtts_device_bytes(self.handle, ctypes.byref(v)))
        return v.value

    def sample(self, work, temperature=0.9, top_k=50, top_p=1.0, seed=0, step=0, group=0):
        """TInferSampler.Next on the device: the index drawn from work
        (logits after the processors) with draw (step, group) of `seed`."""
        w = _f32(work)
        c = ctypes.c_int()
        check(lib().qtts_sample(self.handle, _ptr(w), w.size, temperature, top_k, top_p, seed, step, group,
                                ctypes.byref(c)))
        return c.value

    def quantize_q8_0(self, x):
        """InferQuantizeRowQ8_0Ref on the device: float32 -> ggml blocks."""
        x = _f32(x).reshape(-1)
        out = np.empty(x.size // 32 * 34, dtype=np.uint8)
        check(lib().qtts_quantize_q8_0(self.handle, _ptr(x), x.size, _ptr(out)))
        return out

    def close(self):
        if self.handle:
            check(lib().qtts_device_close(self.handle))
            self.handle = None


class QwenStack:
    """A stack on the device (TDecoderModel from QwenLmStack); owned by the
    QwenLm it is given to."""

    def __init__(self, handle, layers):
        self.handle = handle
        self.layers = layers

    @property
    def bytes(self):
        v = ctypes.c_int64()
        check(lib().qtts_stack_bytes(self.handle, ctypes.byref(v)))
        return v.value


    def save(self, path):
        """The cached blob of the stack (its device bytes, config, norms and
        a crc32c)."""
        check(lib().qtts_stack_save(self.handle, os.fsencode(path)))


def _stack_config(config, layers, dtype):
    return StackConfig(layers, config["hidden"], config["heads"], config["kv_heads"], config["head_dim"],
                       config["intermediate"], config["rms_eps"], config["rope_theta"], DTYPES[dtype])


def qwen_lm_stack_load(device, path):
    """A stack from a blob written by QwenStack.save, without a conversion."""
    h = P()
    check(lib().qtts_stack_load(device.handle, os.fsencode(path), ctypes.byref(h)))
    return QwenStack(h, None)


class SafeTensorsFile:
    """TSafeTensorsFile: a .safetensors file mapped read-only by the library."""

    DTYPE_NAMES = {DTYPE_F32: "F32", DTYPE_BF16: "BF16", 3: "F16", -1: "other"}

    def __init__(self, path):
        h = P()
        check(lib().qtts_safetensors_open(os.fsencode(path), ctypes.byref(h)))
        self.handle = h
        self.path = path

    def names(self):
        n = ctypes.c_int()
        check(lib().qtts_safetensors_count(self.handle, ctypes.byref(n)))
        out = []
        buf = ctypes.create_string_buffer(4096)
        for i in range(n.value):
            check(lib().qtts_safetensors_name(self.handle, i, buf, len(buf)))
            out.append(buf.value.decode())
        return out

    def tensor(self, name):
        """(dtype name, shape, bytes) of the tensor `name`; the bytes are a
        copy of the mapped data."""
        dt, nd = ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 8)()
        data, nb = P(), ctypes.c_int64()
        check(lib().qtts_safetensors_tensor(self.handle, name.encode(), ctypes.byref(dt), ctypes.byref(nd), shape,
                                            ctypes.byref(data), ctypes.byref(nb)))
        raw = ctypes.string_at(data.value, nb.value) if nb.value else b""
        return self.DTYPE_NAMES[dt.value], tuple(shape[i] for i in range(nd.value)), raw

    def close(self):
        if self.handle:
            check(lib().qtts_safetensors_close(self.handle))
            self.handle = None


def qwen_lm_stack_safetensors(device, config, layers, file, prefix, dtype="q8_0"):
    """QwenLmStack (lm.pas:174-179) from a safetensors file: the tensors
    {prefix}layers.{i}.* and {prefix}norm.weight (e.g. prefix
    'talker.model.'), converted on the device to `dtype`."""
    cfg = _stack_config(config, layers, dtype)
    h = P()
    check(lib().qtts_stack_create_safetensors(device.handle, ctypes.byref(cfg), file.handle, prefix.encode(),
                                              ctypes.byref(h)))
    return QwenStack(h, layers)


def qwen_lm_stack(device, config, layers, final_norm, dtype="q8_0"):
    """QwenLmStack (lm.pas:174-179): config = dict of the decoder config
    (layers, hidden, heads, kv_heads, head_dim, intermediate, rms_eps,
    rope_theta); layers = list of dicts with wq wk wv wo wg wu wd ([out][in]
    float32) and in_norm post_norm q_norm k_norm; dtype = weights on the
    device ('f32' or 'q8_0')."""
    cfg = StackConfig(len(layers), config["hidden"], config["heads"], config["kv_heads"], config["head_dim"],
                      config["intermediate"], config["rms_eps"], config["rope_theta"], DTYPES[dtype])
    keep = []
    srcs = (LayerSrc * len(layers))()
    for i, L in enumerate(layers):
        arrs = {k: _f32(L[k]) for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd",
                                        "in_norm", "post_norm", "q_norm", "k_norm")}
        keep.append(arrs)
        s = srcs[i]
        s.dtype = DTYPE_F32
        s.q_proj, s.k_proj, s.v_proj, s.o_proj = (arrs[k].ctypes.data for k in ("wq", "wk", "wv", "wo"))
        s.gate_proj, s.up_proj, s.down_proj = (arrs[k].ctypes.data for k in ("wg", "wu", "wd"))
        s.input_norm, s.post_norm = arrs["in_norm"].ctypes.data, arrs["post_norm"].ctypes.data
        s.q_norm, s.k_norm = arrs["q_norm"].ctypes.data, arrs["k_norm"].ctypes.data
    fn = _f32(final_norm)
    h = P()
    check(lib().qtts_stack_create(device.handle, ctypes.byref(cfg), srcs, _ptr(fn), ctypes.byref(h)))
    return QwenStack(h, len(layers))


class QwenLmHeads:
    """TQwenLmHeads (lm.pas:64-100): output heads [rows][hidden], f32 or Q8_0."""

    def __init__(self, device, name, hidden, dtype="q8_0"):
        self.name = name
        self.hidden = hidden
        self.dtype = dtype
        h = P()
        check(lib().qtts_heads_create(device.handle, name.encode(), hidden, DTYPES[dtype], ctypes.byref(h)))
        self.handle = h

    def add(self, tensor, rows=None):
        """TQwenLmHeads.Add: a [rows][hidden] float32 head; returns its index."""
        t = _f32(tensor)
        rows = t.size // self.hidden if rows is None else rows
        if t.size != rows * self.hidden:
            raise EQwenLm(E_ARG, f"{self.name}: head of {t.size} values instead of [{rows},{self.hidden}]")
        idx = ctypes.c_int()
        check(lib().qtts_heads_add(self.handle, _ptr(t), DTYPE_F32, rows, ctypes.byref(idx)))
        return idx.value

    def add_file(self, file, name, rows):
        """TQwenLmHeads.Add from a safetensors tensor [rows][hidden] (F32 or
        BF16, read in place); returns its index."""
        idx = ctypes.c_int()
        check(lib().qtts_heads_add_safetensors(self.handle, file.handle, name.encode(), rows, ctypes.byref(idx)))
        return idx.value

    def digest(self):
        v = ctypes.c_uint32()
        check(lib().qtts_heads_digest(self.handle, ctypes.byref(v)))
        return v.value

    def linear(self, index, x):
        """TInferBackend.Linear with head `index`: x [rows][hidden] -> [rows][head rows]."""
        x = _f32(x).reshape(-1, self.hidden)
        y = np.empty((x.shape[0], self.rows(index)), np.float32)
        check(lib().qtts_heads_linear(self.handle, index, _ptr(x), x.shape[0], _ptr(y)))
        return y

    @property
    def count(self):
        v = ctypes.c_int()
        check(lib().qtts_heads_count(self.handle, ctypes.byref(v)))
        return v.value

    def rows(self, index):
        v = ctypes.c_int()
        check(lib().qtts_heads_rows(self.handle, index, ctypes.byref(v)))
        return v.value

    @property
    def bytes(self):
        v = ctypes.c_int64()
        check(lib().qtts_heads_bytes(self.handle, ctypes.byref(v)))
        return v.value

    def free(self):
        if self.handle:
            check(lib().qtts_heads_destroy(self.handle))
            self.handle = None


class QwenLm:
    """TQwenLm (lm.pas:102-143): a stack (owned), its heads (not owned) and
    its KV cache."""

    def __init__(self, stack, heads, max_pos=4096, kv_dtype="f32"):
        """kv_dtype "f16": the K/V cache in half floats (TQwenLm.Create's
        aKvF16, lm.pas:122-123)."""
        h = P()
        if kv_dtype == "f32":
            check(lib().qtts_lm_create(stack.handle, heads.handle, max_pos, ctypes.byref(h)))
        else:
            check(lib().qtts_lm_create_kv(stack.handle, heads.handle, max_pos, DTYPES[kv_dtype], ctypes.byref(h)))
        stack.handle = None  # owned by the lm from now on
        self.handle = h
        self.heads = heads
        self.hidden = heads.hidden

    def reset(self):
        check(lib().qtts_lm_reset(self.handle))

    def forward(self, x, rows=None, output=0, logits=None, hidden=None):
        """TQwenLm.Forward(x, aRows, aOutput, aLogits, aHidden): logits and
        hidden are float32 arrays to fill (None: not wanted)."""
        x = _f32(x)
        rows = x.size // self.hidden if rows is None else rows
        check(lib().qtts_lm_forward(self.handle, _ptr(x), rows, output, _ptr(logits), _ptr(hidden)))

    def forward_noalloc(self, x_dev, rows, output=0, logits_dev=None, hidden_dev=None):
        """qtts_lm_forward_noalloc: the same forward on device buffers the
        caller owns (integer device addresses), with no allocation at all:
        for callers that may not allocate device memory while they run."""
        check(lib().qtts_lm_forward_noalloc(self.handle, x_dev, rows, output, logits_dev, hidden_dev))

    @property
    def length(self):
        v = ctypes.c_int()
        check(lib().qtts_lm_length(self.handle, ctypes.byref(v)))
        return v.value

    def set_launch_epoch(self, epoch):
        """qtts_lm_set_launch_epoch: set the epoch counter of this lm's
        tagged handoffs (the next launch uses epoch + 1; at 2^22 - 1 it wraps
        to 1 after the tagged words are cleared)."""
        check(lib().qtts_lm_set_launch_epoch(self.handle, epoch))

    def set_wait_test(self, extra_arrivals, wait_cycles):
        """qtts_lm_set_wait_test: make the grid barriers of the next launches
        wait for an arrival that never comes, bounded by wait_cycles
        (failure-path tests); (0, 0) restores normal operation."""
        check(lib().qtts_lm_set_wait_test(self.handle, extra_arrivals, wait_cycles))

    def free(self):
        if self.handle:
            check(lib().qtts_lm_destroy(self.handle))
            self.handle = None


class QwenBatch:
    """Many sequences through one stack per call (batched decode / prefill),
    paged KV cache; the stack and heads are not owned."""

    def __init__(self, stack, heads, max_seqs, max_tokens, max_pos, kv_dtype="f32"):
        h = P()
        check(lib().qtts_batch_create(stack.handle, heads.handle, max_seqs, max_tokens, max_pos, DTYPES[kv_dtype],
                                      ctypes.byref(h)))
        self.handle = h
        self.heads = heads
        self.hidden = heads.hidden

    def reset(self, seq):
        check(lib().qtts_batch_reset(self.handle, seq))

    def length(self, seq):
        v = ctypes.c_int()
        check(lib().qtts_batch_length(self.handle, seq, ctypes.byref(v)))
        return v.value

    def forward(self, seqs, rows, x, head=0, logits=True, hidden=True):
        """Append rows[i] rows to sequence seqs[i]; returns (logits [n][rows
        of head] or None, hidden [n][hidden] or None)."""
        sq = np.ascontiguousarray(seqs, dtype=np.int32)
        rw = np.ascontiguousarray(rows, dtype=np.int32)
        x = _f32(x)
        n = sq.size
        lg = np.empty((n, self.heads.rows(head)), np.float32) if logits else None
        hd = np.empty((n, self.hidden), np.float32) if hidden else None
        check(lib().qtts_batch_forward(self.handle, n, _ptr(sq), _ptr(rw), _ptr(x), head, _ptr(lg), _ptr(hd)))
        return lg, hd

    def free(self):
        if self.handle:
            check(lib().qtts_batch_destroy(self.handle))
            self.handle = None


def stack_destroy(stack):
    """Free a stack that no lm owns (the batch borrows its stack)."""
    if stack.handle:
        check(lib().qtts_stack_destroy(stack.handle))
        stack.handle = None


class QwenTalker:
    """The per-frame device loop of TQwenTalker (talker.pas:471-681), greedy
    or sampling (set_sampling)."""

    def __init__(self, talker, predictor, codec_emb, pred_emb, eos, vocab=3072, pred_vocab=2048, groups=16,
                 repetition_penalty=1.05):
        cfg = TalkerConfig(vocab, pred_vocab, groups, eos, repetition_penalty)
        ce, pe = _f32(codec_emb), _f32(pred_emb)
        h = P()
        check(lib().qtts_talker_create(talker.handle, predictor.handle, ctypes.byref(cfg), _ptr(ce), _ptr(pe),
                                       ctypes.byref(h)))
        self.handle = h
        self.groups = groups
        self.vocab = vocab
        self.hidden = talker.hidden

    def set_sampling(self, do_sample=True, temperature=0.9, top_k=50, top_p=1.0, sub_do_sample=True,
                     sub_temperature=0.9, sub_top_k=50, sub_top_p=1.0, seed=0):
        """TQwenSampling for the frames that follow (call before start for
        the first code 0); defaults of QwenSamplingFromConfig (talker.pas:
        203-230)."""
        s = Sampling(int(do_sample), temperature, top_k, top_p, int(sub_do_sample), sub_temperature, sub_top_k,
                     sub_top_p, seed)
        check(lib().qtts_talker_set_sampling(self.handle, ctypes.byref(s)))

    def start(self, prefill, trailing, tts_pad, logits=None, hidden=None):
        """The device part of TQwenTalker.Start: prefill rows, trailing text
        rows, tts_pad."""
        p = _f32(prefill)
        t = _f32(trailing) if trailing is not None and len(trailing) else None
        check(lib().qtts_talker_start(self.handle, _ptr(p), p.size // self.hidden, _ptr(t),
                                      0 if t is None else t.size // self.hidden, _ptr(_f32(tts_pad)),
                                      _ptr(logits), _ptr(hidden)))

    def start_prompt(self, textproj, tokens, ids, codec, non_streaming=False, logits=None, hidden=None):
        """TQwenTalker.Start from token ids, the prompt rows built on the
        device: ids = PromptIds(text), codec = start_codec_ids(...),
        tokens = prompt_tokens(config)."""
        i = np.ascontiguousarray(ids, dtype=np.int32)
        c = np.ascontiguousarray(codec, dtype=np.int32)
        check(lib().qtts_talker_start_prompt(self.handle, textproj.handle, ctypes.byref(tokens), _ptr(i), i.size,
                                             _ptr(c), c.size, int(non_streaming), _ptr(logits), _ptr(hidden)))

    def prompt_rows(self, textproj, tokens, ids, codec, non_streaming=False):
        """(prefill, trailing) rows that start_prompt builds (the probes
        talker.prefill.embeds / talker.trailing)."""
        i = np.ascontiguousarray(ids, dtype=np.int32)
        c = np.ascontiguousarray(codec, dtype=np.int32)
        rows, tr = ctypes.c_int(), ctypes.c_int()
        args = (self.handle, textproj.handle, ctypes.byref(tokens), _ptr(i), i.size, _ptr(c), c.size,
                int(non_streaming))
        check(lib().qtts_talker_prompt_rows(*args, None, 0, None, 0, ctypes.byref(rows), ctypes.byref(tr)))
        pf = np.zeros((rows.value, self.hidden), np.float32)
        tt = np.zeros((tr.value, self.hidden), np.float32)
        check(lib().qtts_talker_prompt_rows(*args, _ptr(pf), rows.value, _ptr(tt), tr.value, ctypes.byref(rows),
                                            ctypes.byref(tr)))
        return pf, tt

    def next_frame(self, codes):
        """TQwenTalker.NextFrame: fills codes[groups] (int32); False at eos."""
        more = ctypes.c_int()
        check(lib().qtts_talker_next_frame(self.handle, _ptr(codes), ctypes.byref(more)))
        return bool(more.value)

    def trace_frame(self, codes, cap=8192):
        """next_frame with CTA 0's phase timestamps: returns (more, [(tag, ns)])."""
        more = ctypes.c_int()
        st = np.zeros(cap, np.uint64)
        n = ctypes.c_int()
        check(lib().qtts_talker_trace_frame(self.handle, _ptr(codes), ctypes.byref(more), _ptr(st), cap,
                                            ctypes.byref(n)))
        st = st[:n.value]
        return bool(more.value), [(int(v >> np.uint64(48)), int(v & np.uint64(0xFFFFFFFFFFFF))) for v in st]

    def run(self, frames):
        """Up to `frames` frames back to back; returns codes [n][groups]."""
        out = np.zeros((frames, self.groups), np.int32)
        n = ctypes.c_int()
        check(lib().qtts_talker_run(self.handle, frames, _ptr(out), ctypes.byref(n)))
        return out[:n.value]

    @property
    def stream(self):
        """The cudaStream_t of the talker's kernels (an integer handle)."""
        v = P()
        check(lib().qtts_talker_stream(self.handle, ctypes.byref(v)))
        return v.value or 0

    def probe(self):
        """(logits, hidden) of the last talker forward (Emit 'talker.logits')."""
        lg = np.empty(self.vocab, np.float32)
        hd = np.empty(self.hidden, np.float32)
        check(lib().qtts_talker_probe(self.handle, _ptr(lg), _ptr(hd)))
        return lg, hd

    @property
    def step(self):
        v = ctypes.c_int()
        check(lib().qtts_talker_step(self.handle, ctypes.byref(v)))
        return v.value

    def free(self):
        if self.handle:
            check(lib().qtts_talker_destroy(self.handle))
            self.handle = None


class QwenCodec:
    """TQwenCodec (the 12 Hz decoder, codec.pas) on the device, from the
    speech_tokenizer checkpoint: decode(codes [frames][16]) -> frames * 1920
    samples in [-1, 1]; frames of successive calls follow each other."""

    FRAME_SAMPLES = 1920

    def __init__(self, device, file):
        h = P()
        check(lib().qtts_codec_create_safetensors(device.handle, file.handle, ctypes.byref(h)))
        self.handle = h

    def decode(self, codes):
        c = np.ascontiguousarray(codes, dtype=np.int32).reshape(-1, 16)
        pcm = np.zeros(c.shape[0] * self.FRAME_SAMPLES, np.float32)
        check(lib().qtts_codec_decode(self.handle, _ptr(c), c.shape[0], _ptr(pcm)))
        return pcm

    def reset(self):
        check(lib().qtts_codec_reset(self.handle))

    @property
    def frames(self):
        v = ctypes.c_int64()
        check(lib().qtts_codec_frames(self.handle, ctypes.byref(v)))
        return v.value

    def free(self):
        if self.handle:
            check(lib().qtts_codec_destroy(self.handle))
            self.handle = None


class QwenTextProject:
    """TQwenTalker.TextProject (talker.pas:390-421) on the device: the text
    embedding table (BF16 uint16 rows or float32) and the float32 fc1 / fc2
    with biases."""

    def __init__(self, device, emb, fc1_w, fc1_b, fc2_w, fc2_b):
        if emb.dtype == np.uint16:
            dt, e = DTYPES["bf16"], np.ascontiguousarray(emb)
        else:
            dt, e = DTYPES["f32"], _f32(emb)
        self.w = [_f32(a) for a in (fc1_w, fc1_b, fc2_w, fc2_b)]
        self.hidden = self.w[2].shape[0]
        h = P()
        check(lib().qtts_textproj_create(device.handle, e.shape[0], e.shape[1], self.hidden, dt, _ptr(e),
                                         *(_ptr(a) for a in self.w), ctypes.byref(h)))
        self.handle = h

    def project(self, ids):
        i = np.ascontiguousarray(ids, dtype=np.int32)
        y = np.zeros((i.size, self.hidden), np.float32)
        check(lib().qtts_text_project(self.handle, _ptr(i), i.size, _ptr(y)))
        return y

    def free(self):
        if self.handle:
            check(lib().qtts_textproj_destroy(self.handle))
            self.handle = None


class QwenTalkers:
    """TQwenTalker (greedy) for many utterances at once over a talker batch
    and a predictor batch (not owned); utterance ids are sequence ids."""

    def __init__(self, talker, predictor, codec_emb, pred_emb, eos, vocab=3072, pred_vocab=2048, groups=16,
                 repetition_penalty=1.05):
        cfg = TalkerConfig(vocab, pred_vocab, groups, eos, repetition_penalty)
        ce, pe = _f32(codec_emb), _f32(pred_emb)
        h = P()
        check(lib().qtts_talkers_create(talker.handle, predictor.handle, ctypes.byref(cfg), _ptr(ce), _ptr(pe),
                                        ctypes.byref(h)))
        self.handle = h
        self.groups = groups
        self.vocab = vocab
        self.hidden = talker.hidden

    def set_sampling(self, do_sample=True, temperature=0.9, top_k=50, top_p=1.0, sub_do_sample=True,
                     sub_temperature=0.9, sub_top_k=50, sub_top_p=1.0, seed=0):
        """TQwenSampling for every utterance (utterance s: stream seed + s);
        call before start for the first code 0."""
        s = Sampling(int(do_sample), temperature, top_k, top_p, int(sub_do_sample), sub_temperature, sub_top_k,
                     sub_top_p, seed)
        check(lib().qtts_talkers_set_sampling(self.handle, ctypes.byref(s)))

    def start(self, seqs, prefills, trailings, tts_pad):
        """TQwenTalker.Start for utterances seqs[i]: prefills[i] [rows][hidden],
        trailings[i] [rows][hidden] or None, one tts_pad [hidden]."""
        sq = np.ascontiguousarray(seqs, dtype=np.int32)
        rows = np.array([len(p) for p in prefills], np.int32)
        trs = np.array([0 if t is None else len(t) for t in trailings], np.int32)
        pf = _f32(np.concatenate([np.asarray(p, np.float32) for p in prefills]))
        tl = [np.asarray(t, np.float32) for t in trailings if t is not None and len(t)]
        tr = _f32(np.concatenate(tl)) if tl else None
        check(lib().qtts_talkers_start(self.handle, sq.size, _ptr(sq), _ptr(rows), _ptr(pf), _ptr(trs), _ptr(tr),
                                       _ptr(_f32(tts_pad))))

    def start_prompt(self, textproj, tokens, seqs, prompts):
        """TQwenTalker.Start from token ids for utterances seqs[i], their
        rows built on the device: prompts[i] = (ids, codec, non_streaming)
        as QwenTalker.start_prompt takes them."""
        sq = np.ascontiguousarray(seqs, dtype=np.int32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(p[0], np.int32) for p in prompts]), np.int32)
        codec = np.ascontiguousarray(np.concatenate([np.asarray(p[1], np.int32) for p in prompts]), np.int32)
        n_ids = np.array([len(p[0]) for p in prompts], np.int32)
        n_codec = np.array([len(p[1]) for p in prompts], np.int32)
        ns = np.array([int(p[2]) for p in prompts], np.int32)
        check(lib().qtts_talkers_start_prompt(self.handle, textproj.handle, ctypes.byref(tokens), sq.size, _ptr(sq),
                                              _ptr(ids), _ptr(n_ids), _ptr(codec), _ptr(n_codec), _ptr(ns)))

    def next_frame(self, seqs):
        """TQwenTalker.NextFrame for utterances seqs: returns (codes [n][groups],
        more [n] bool)."""
        sq = np.ascontiguousarray(seqs, dtype=np.int32)
        codes = np.zeros((sq.size, self.groups), np.int32)
        more = np.zeros(sq.size, np.int32)
        check(lib().qtts_talkers_next_frame(self.handle, sq.size, _ptr(sq), _ptr(codes), _ptr(more)))
        return codes, more.astype(bool)

    def probe(self, seq):
        """(logits, hidden) of utterance seq's last talker forward."""
        lg = np.empty(self.vocab, np.float32)
        hd = np.empty(self.hidden, np.float32)
        check(lib().qtts_talkers_probe(self.handle, int(seq), _ptr(lg), _ptr(hd)))
        return lg, hd

    @property
    def stream(self):
        v = P()
        check(lib().qtts_talkers_stream(self.handle, ctypes.byref(v)))
        return v.value or 0

    def free(self):
        if self.handle:
            check(lib().qtts_talkers_destroy(self.handle))
            self.handle = None
