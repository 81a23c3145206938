"""The tcgen05 GEMM (the batched projections) through qtts_heads_linear,
the reference's TInferBackend.Linear on a head (mormot.ai.tts.qwen.lm.pas:
404-406) for many rows at once.

Expected values: numpy in float64 on the same fp16 operands the tensor cores
see (x rounded to fp16; the weights as two fp16 tiles, hi and lo, both
multiplied with x: hi = fp16(w), lo = fp16(w - hi) for f32 weights, hi =
fp16(q*d), lo = q*d - hi for Q8_0, which carry the weight to ~2^-22).  Only
the f32 accumulation order differs, hence the tight tolerance.
"""
import numpy as np
import pytest

import oracle as O
import qtts
import synth

pytestmark = pytest.mark.gpu


def fp16_weights(w, dtype):
    if dtype == "f32":
        hi = w.astype(np.float16)
        lo = (w - hi.astype(np.float32)).astype(np.float16)
        return hi.astype(np.float64) + lo.astype(np.float64)
    q = O.quantize_q8_0(w).reshape(-1, 34)
    d = q[:, :2].copy().view(np.float16).astype(np.float64)        # [blocks, 1]
    qs = q[:, 2:].view(np.int8).astype(np.float64)                  # [blocks, 32]
    return (qs * d).reshape(w.shape)  # hi + lo carry q * d to ~2^-22


@pytest.mark.parametrize("dtype", ["q8_0", "f32"])
@pytest.mark.parametrize("rows", [1, 37, 64, 100, 300])
def test_heads_linear_matches_fp16_reference(device, dtype, rows):
    w = synth.talker_head(81) if dtype == "q8_0" else synth.predictor_heads(81)[0]
    heads = qtts.QwenLmHeads(device, "h", synth.HIDDEN, dtype)
    heads.add(w)
    x = synth.prompt(82, rows)
    y = heads.linear(0, x)
    ref = x.astype(np.float16).astype(np.float64) @ fp16_weights(w, dtype).T
    err = np.abs(y - ref).max()
    assert err <= 1e-4 * max(1.0, np.abs(ref).max()), err
    # and against the f32 oracle's Linear semantics (fp16 operands, ~1e-3 rel)
    exact = x.astype(np.float64) @ (O.dequantize_q8_0(O.quantize_q8_0(w), w.size).reshape(w.shape)
                                    if dtype == "q8_0" else w).astype(np.float64).T
    assert np.abs(y - exact).max() <= 1e-2
    heads.free()
