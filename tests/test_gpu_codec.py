"""The 12 Hz decoder on the device (qtts_codec_*: TQwenCodec, src/tts/
mormot.ai.tts.qwen.codec.pas) against its CPU restatement (oracle OraCodec,
itself pinned to a float64 PyTorch restatement in tests/test_codec_oracle.py),
on seeded weights under the checkpoint's names, read from a safetensors file.

Tolerance: samples within 1e-4 abs of the oracle (the products on the
tensor cores at float32 accuracy, 3xTF32, summed in another order; samples
of about +-0.2).  Frames decoded in successive calls
give the samples of one call bit for bit (every output is computed the same
way whatever the rows of a call), also past the 72-frame attention window."""
import json

import numpy as np
import pytest
from safetensors.numpy import save_file

import oracle as O
import qtts
from codec_util import codec_weights

pytestmark = pytest.mark.gpu

ATOL = 1e-4


def test_codec_matches_oracle_and_streams(device, tmp_path):
    w = codec_weights(3)
    path = tmp_path / "codec.safetensors"
    save_file(w, str(path))
    f = qtts.SafeTensorsFile(path)
    dc = qtts.QwenCodec(device, f)
    oc = O.OraCodec(w)
    codes = np.random.default_rng(4).integers(0, 2048, (80, 16)).astype(np.int32)
    codes[7, 3] = -5  # read as 0
    whole = dc.decode(codes)
    ref = oc.decode(codes)
    assert whole.shape == ref.shape == (80 * 1920,)
    err = float(np.abs(whole - ref).max())
    print(json.dumps({"test": "codec_80_frames", "max_abs_sample_diff": err}))
    assert err <= ATOL, err
    assert dc.frames == 80
    dc.reset()
    parts, i = [], 0
    for n in (1, 30, 3, 40, 6):  # the key/value cache compacts past 72 frames
        parts.append(dc.decode(codes[i:i + n]))
        i += n
    assert np.array_equal(np.concatenate(parts), whole)
    bad = codes[:2].copy()
    bad[1, 4] = 2048
    with pytest.raises(qtts.EQwenLm) as e:
        dc.decode(bad)
    assert e.value.code == qtts.E_ARG
    dc.free()
    oc.free()
    f.close()


def test_codec_refuses_an_incomplete_checkpoint(device, tmp_path):
    path = tmp_path / "partial.safetensors"
    save_file({"decoder.pre_conv.conv.bias": np.zeros(1024, np.float32)}, str(path))
    f = qtts.SafeTensorsFile(path)
    with pytest.raises(qtts.EQwenLm) as e:
        qtts.QwenCodec(device, f)
    assert e.value.code == qtts.E_ARG
    f.close()
