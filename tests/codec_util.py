"""The 12 Hz decoder (TQwenCodec, codec.pas) for the tests: seeded weights
under the checkpoint's tensor names and shapes (synth.codec_weights: the
speech_tokenizer model.safetensors as codec.pas:644-731 reads it), and an independent
restatement of the whole decoder with PyTorch modules in float64, applied
to the whole sequence at once (no streaming state): causal convolutions as
left padding, transposed convolutions cut on the right by K - s, LayerNorm,
exact GELU, attention with a 72-frame sliding-window mask and rotate-half
RoPE."""
import numpy as np
import torch
import torch.nn.functional as F

from synth import codec_weights  # noqa: F401  (the seeded weights, shared with bench.py)

RATES = (8, 5, 4, 3)
DILATIONS = (1, 3, 9)


def torch_decode(W, codes):
    """codes [frames][16] -> frames * 1920 samples, float64 PyTorch."""
    t = lambda n: torch.from_numpy(W[n]).double()  # noqa: E731
    c = torch.from_numpy(np.asarray(codes, np.int64)).clamp(min=0)
    cb = []
    for g in range(16):
        p = ("decoder.quantizer.rvq_first.vq.layers.0._codebook" if g == 0
             else f"decoder.quantizer.rvq_rest.vq.layers.{g - 1}._codebook")
        cb.append(t(p + ".embedding_sum") / t(p + ".cluster_usage").clamp(min=1e-5)[:, None])
    q1 = cb[0][c[:, 0]]
    q2 = sum(cb[g][c[:, g]] for g in range(1, 16))
    x = q1 @ t("decoder.quantizer.rvq_first.output_proj.weight")[:, :, 0].T + \
        q2 @ t("decoder.quantizer.rvq_rest.output_proj.weight")[:, :, 0].T
    x = x.T[None]

    def cconv(x, name, k, dil=1, groups=1):
        return F.conv1d(F.pad(x, ((k - 1) * dil, 0)), t(name + ".weight"), t(name + ".bias"), dilation=dil,
                        groups=groups)

    def tconv(x, name, k, s):
        y = F.conv_transpose1d(x, t(name + ".weight"), t(name + ".bias"), stride=s)
        return y[..., :y.shape[-1] - (k - s)]

    def snake(x, p):
        a = torch.exp(t(p + ".alpha"))[None, :, None]
        inv = 1.0 / (torch.exp(t(p + ".beta")) + 1e-9)[None, :, None]
        return x + inv * torch.sin(x * a) ** 2

    def rms(h, w):
        return h * torch.rsqrt((h * h).mean(-1, keepdim=True) + 1e-5) * w

    x = cconv(x, "decoder.pre_conv.conv", 3)
    p = "decoder.pre_transformer."
    h = x[0].T @ t(p + "input_proj.weight").T + t(p + "input_proj.bias")
    n_f = h.shape[0]
    inv = torch.tensor([np.float32(1.0 / np.exp(np.log(10000.0) * (2.0 * i / 64))) for i in range(32)],
                       dtype=torch.float64)
    ang = torch.arange(n_f, dtype=torch.float64)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]

    def rope(v):
        a, b = v[..., :32], v[..., 32:]
        return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)

    i = torch.arange(n_f)
    mask = (i[None, :] <= i[:, None]) & (i[None, :] >= i[:, None] - 71)
    for l in range(8):
        q = f"{p}layers.{l}."
        n = rms(h, t(q + "input_layernorm.weight"))
        qq = rope((n @ t(q + "self_attn.q_proj.weight").T).view(n_f, 16, 64))
        kk = rope((n @ t(q + "self_attn.k_proj.weight").T).view(n_f, 16, 64))
        vv = (n @ t(q + "self_attn.v_proj.weight").T).view(n_f, 16, 64)
        s = torch.einsum("qhd,khd->hqk", qq, kk) / 8.0
        s = s.masked_fill(~mask[None], float("-inf")).softmax(-1)
        a = torch.einsum("hqk,khd->qhd", s, vv).reshape(n_f, 1024)
        h = h + t(q + "self_attn_layer_scale.scale") * (a @ t(q + "self_attn.o_proj.weight").T)
        n = rms(h, t(q + "post_attention_layernorm.weight"))
        m = F.silu(n @ t(q + "mlp.gate_proj.weight").T) * (n @ t(q + "mlp.up_proj.weight").T)
        h = h + t(q + "mlp_layer_scale.scale") * (m @ t(q + "mlp.down_proj.weight").T)
    y = rms(h, t(p + "norm.weight")) @ t(p + "output_proj.weight").T + t(p + "output_proj.bias")
    x = y.T[None]
    for u in range(2):
        x = tconv(x, f"decoder.upsample.{u}.0.conv", 2, 2)
        q = f"decoder.upsample.{u}.1."
        r = x
        z = cconv(x, q + "dwconv.conv", 7, groups=1024).transpose(1, 2)
        z = F.layer_norm(z, (1024,), t(q + "norm.weight"), t(q + "norm.bias"), 1e-6)
        z = F.gelu(z @ t(q + "pwconv1.weight").T + t(q + "pwconv1.bias"))
        z = (z @ t(q + "pwconv2.weight").T + t(q + "pwconv2.bias")) * t(q + "gamma")
        x = r + z.transpose(1, 2)
    x = cconv(x, "decoder.decoder.0.conv", 7)
    for b in range(4):
        q = f"decoder.decoder.{b + 1}.block."
        x = snake(x, q + "0")
        x = tconv(x, q + "1.conv", 2 * RATES[b], RATES[b])
        for r in range(3):
            u = f"{q}{r + 2}."
            z = cconv(snake(x, u + "act1"), u + "conv1.conv", 7, DILATIONS[r])
            x = x + cconv(snake(z, u + "act2"), u + "conv2.conv", 1)
    x = cconv(snake(x, "decoder.decoder.5"), "decoder.decoder.6.conv", 7)
    return x[0, 0].clamp(-1.0, 1.0).numpy()
