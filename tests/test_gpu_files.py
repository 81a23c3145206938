"""Weights from a BF16 safetensors checkpoint (qtts_stack_create_safetensors,
qtts_heads_add_safetensors: QwenLmStack / TQwenLmHeads.Add of the file,
lm.pas:174-179, 277-308) and the cached blob of a stack (qtts_stack_save /
qtts_stack_load).

The bar is bit-exact: a stack read from the file holds the bytes of a stack
made from the same values as host float32 rows (BF16 widens exactly), so its
logits are identical; the heads have the same crc32c (the check of
ParallelQ8MatchesSerial, tests/test.tts.qwen.talker.pas:256-304); a stack
read back from its blob gives identical logits."""
import numpy as np
import pytest
import torch
from safetensors.torch import save_file

import qtts
import synth

pytestmark = pytest.mark.gpu

NAMES = {"wq": "self_attn.q_proj.weight", "wk": "self_attn.k_proj.weight", "wv": "self_attn.v_proj.weight",
         "wo": "self_attn.o_proj.weight", "wg": "mlp.gate_proj.weight", "wu": "mlp.up_proj.weight",
         "wd": "mlp.down_proj.weight", "in_norm": "input_layernorm.weight",
         "post_norm": "post_attention_layernorm.weight", "q_norm": "self_attn.q_norm.weight",
         "k_norm": "self_attn.k_norm.weight"}


def bf16(a):
    """(torch BF16 tensor, the float32 values it holds)."""
    t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)
    return t, t.float().numpy()


def checkpoint(tmp_path, seed, layers, prefix="talker.model."):
    """A BF16 checkpoint of one stack plus a head; returns the path and the
    float32 values of every tensor."""
    ls, final = synth.stack(seed, "talker", layers)
    tensors, values = {}, []
    for i, L in enumerate(ls):
        v = {}
        for k, n in NAMES.items():
            t, f = bf16(L[k])
            tensors[f"{prefix}layers.{i}.{n}"] = t
            v[k] = f
        values.append(v)
    t, fn = bf16(final)
    tensors[prefix + "norm.weight"] = t
    t, head = bf16(synth.talker_head(seed))
    tensors["talker.codec_head.weight"] = t
    path = tmp_path / "model.safetensors"
    save_file(tensors, str(path))
    return path, values, fn, head


@pytest.mark.parametrize("dtype", ["q8_0", "f32"])
def test_stack_from_file_equals_stack_from_rows(device, tmp_path, dtype):
    path, values, fn, head = checkpoint(tmp_path, 31, 2)
    f = qtts.SafeTensorsFile(path)
    hf = qtts.QwenLmHeads(device, "talker", synth.HIDDEN, dtype)
    hf.add_file(f, "talker.codec_head.weight", synth.TALKER_VOCAB)
    hr = qtts.QwenLmHeads(device, "talker", synth.HIDDEN, dtype)
    hr.add(head)
    assert hf.digest() == hr.digest()
    sf = qtts.qwen_lm_stack_safetensors(device, synth.CONFIG, 2, f, "talker.model.", dtype)
    sr = qtts.qwen_lm_stack(device, synth.CONFIG, values, fn, dtype)
    assert sf.bytes == sr.bytes
    lf = qtts.QwenLm(sf, hf, 64)
    lr = qtts.QwenLm(sr, hr, 64)
    x = synth.prompt(31, 9)
    out = []
    for lm in (lf, lr):
        lg = np.zeros(synth.TALKER_VOCAB, np.float32)
        hd = np.zeros(synth.HIDDEN, np.float32)
        lm.forward(x, logits=lg, hidden=hd)
        out.append((lg, hd))
    assert np.array_equal(out[0][0], out[1][0]) and np.array_equal(out[0][1], out[1][1])
    for o in (lf, lr, hf, hr):
        o.free()
    f.close()


def test_stack_from_file_checks_names_and_shapes(device, tmp_path):
    path, values, fn, head = checkpoint(tmp_path, 32, 1)
    f = qtts.SafeTensorsFile(path)
    for layers, prefix in ((2, "talker.model."),           # layer 1 absent
                           (1, "talker.code_predictor.model.")):  # another stack's prefix
        with pytest.raises(qtts.EQwenLm) as e:
            qtts.qwen_lm_stack_safetensors(device, synth.CONFIG, layers, f, prefix)
        assert e.value.code == qtts.E_ARG
    h = qtts.QwenLmHeads(device, "talker", synth.HIDDEN)
    with pytest.raises(qtts.EQwenLm):
        h.add_file(f, "talker.codec_head.weight", synth.TALKER_VOCAB - 1)  # [rows][hidden] mismatch
    h.free()
    f.close()


@pytest.mark.parametrize("dtype", ["q8_0", "f32"])
def test_blob_round_trip(device, tmp_path, dtype):
    ls, final = synth.stack(33, "talker", 2)
    heads = qtts.QwenLmHeads(device, "talker", synth.HIDDEN, dtype)
    heads.add(synth.talker_head(33))
    s = qtts.qwen_lm_stack(device, synth.CONFIG, ls, final, dtype)
    blob = tmp_path / "talker.qtts"
    s.save(blob)
    s2 = qtts.qwen_lm_stack_load(device, blob)
    assert s2.bytes == s.bytes
    x = synth.prompt(33, 7)
    out = []
    for st in (s, s2):
        lm = qtts.QwenLm(st, heads, 64)
        lg = np.zeros(synth.TALKER_VOCAB, np.float32)
        lm.forward(x, logits=lg)
        out.append(lg)
        lm.free()
    assert np.array_equal(out[0], out[1])
    # a damaged or truncated blob is refused
    raw = bytearray(blob.read_bytes())
    raw[len(raw) // 2] ^= 0x40
    bad = tmp_path / "bad.qtts"
    bad.write_bytes(bytes(raw))
    cut = tmp_path / "cut.qtts"
    cut.write_bytes(blob.read_bytes()[:-100])
    for p in (bad, cut):
        with pytest.raises(qtts.EQwenLm) as e:
            qtts.qwen_lm_stack_load(device, p)
        assert e.value.code == qtts.E_ARG
    heads.free()
