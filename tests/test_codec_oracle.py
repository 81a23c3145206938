"""The C restatement of the 12 Hz decoder (oracle OraCodec: TQwenCodec,
src/tts/mormot.ai.tts.qwen.codec.pas) on the CPU, the checker for a device
codec.  No golden vectors of the decoder exist in the reference tree (its
codec tests read a downloaded model), so the restatement is pinned against
an independent float64 PyTorch restatement of the same modules
(tests/codec_util.py) within 1e-5 abs on samples of about +-0.2, and
against the properties the reference states: frames decoded one call after
another give exactly the samples of one call (codec.pas:5-8, bit for bit),
including past the 72-frame attention window; a code changes no sample
before its frame (everything is causal); out-of-range codes are refused,
negative ones read as 0 (codec.pas:895-900)."""
import numpy as np
import pytest

import oracle as O
from codec_util import codec_weights, torch_decode

ATOL = 1e-5


@pytest.fixture(scope="module")
def weights():
    return codec_weights(3)


@pytest.fixture(scope="module")
def codec(weights):
    c = O.OraCodec(weights)
    yield c
    c.free()


def codes_of(seed, frames):
    return np.random.default_rng(seed).integers(0, 2048, (frames, 16)).astype(np.int32)


def test_matches_torch_and_streams_past_the_window(codec, weights):
    codes = codes_of(4, 80)
    codec.reset()
    whole = codec.decode(codes)
    assert whole.shape == (80 * 1920,) and codec.frames == 80
    ref = torch_decode(weights, codes)
    assert np.abs(whole - ref).max() <= ATOL, np.abs(whole - ref).max()
    assert 0.02 < whole.std() and np.abs(whole).max() < 1.0  # real signal, no clamping
    codec.reset()
    parts, i = [], 0
    for n in (1, 30, 3, 40, 6):  # the cache compacts past 72 frames
        parts.append(codec.decode(codes[i:i + n]))
        i += n
    assert np.array_equal(np.concatenate(parts), whole)


def test_a_code_changes_nothing_before_its_frame(codec):
    codes = codes_of(5, 6)
    codec.reset()
    a = codec.decode(codes)
    codes[3, 9] = (codes[3, 9] + 1) % 2048
    codec.reset()
    b = codec.decode(codes)
    first = int(np.argmax(a != b))
    assert first >= 3 * 1920 and np.abs(a - b).max() > 1e-4


def test_codes_out_of_range(codec):
    codes = codes_of(6, 2)
    codec.reset()
    ref = codec.decode(np.where(np.arange(32).reshape(2, 16) == 5, 0, codes))
    neg = codes.copy()
    neg[0, 5] = -7  # read as 0, as torch.clamp(min=0)
    codec.reset()
    assert np.array_equal(codec.decode(neg), ref)
    bad = codes.copy()
    bad[1, 2] = 2048
    with pytest.raises(ValueError):
        codec.decode(bad)


def test_missing_or_misshapen_weights(weights):
    w = dict(weights)
    del w["decoder.decoder.5.alpha"]
    with pytest.raises(ValueError, match="decoder.decoder.5.alpha"):
        O.OraCodec(w)
    w = dict(weights)
    w["decoder.pre_conv.conv.bias"] = w["decoder.pre_conv.conv.bias"][:-1]
    with pytest.raises(ValueError, match="pre_conv"):
        O.OraCodec(w)
