"""Generate the golden fixtures of tests/golden (run in a container where
the Python references are installed: gguf, transformers, torch).

1. q8_0_gguf.npz: float32 blocks and their Q8_0 bytes from gguf's
   Q8_0.quantize_blocks, "bit-exact with the reference implementation in
   ggml-quants.c" (quantize_row_q8_0_ref), the rule of TQwenLmHeads
   (mormot.ai.tts.qwen.lm.pas:259-267).
2. qwen3_small.npz: a small Qwen3 stack (dims golden_lib.SMALL, LCG weights)
   in transformers' Qwen3Model, float32, eager attention, CPU: the model the
   reference's own golden dataset was made with (tools/tts/qwen_ref.py,
   manifest note of tests/data/infer-ref/qwen3-tts-lm).  6 prefill rows
   (per-layer states, final-norm states, head logits of the last row), then 3
   one-row steps through the KV cache (normed state and logits each), which
   is the TQwenLm.Forward protocol (lm.pas:391-408).

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import golden_lib as G  # noqa: E402


def q8_fixture():
    from gguf.quants import Q8_0
    x = G.q8_blocks()
    q = Q8_0.quantize_blocks(x.reshape(-1, 32)).reshape(-1).astype(np.uint8)
    np.savez_compressed(os.path.join(HERE, "q8_0_gguf.npz"), x=x, q=q)
    print("q8_0_gguf.npz:", x.size, "values,", q.size, "bytes")


def qwen3_fixture():
    import torch
    from transformers import Qwen3Config, Qwen3Model
    from transformers.cache_utils import DynamicCache
    c = G.SMALL
    layers, final, head = G.small_model()
    cfg = Qwen3Config(hidden_size=c["hidden"], num_attention_heads=c["heads"], num_key_value_heads=c["kv_heads"],
                      head_dim=c["head_dim"], intermediate_size=c["intermediate"], num_hidden_layers=c["layers"],
                      rms_norm_eps=c["rms_eps"], vocab_size=8, max_position_embeddings=4096,
                      rope_parameters={"rope_type": "default", "rope_theta": c["rope_theta"]})
    cfg._attn_implementation = "eager"
    m = Qwen3Model(cfg).float().eval()
    sd = {}
    for i, L in enumerate(layers):
        p = f"layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = L["wq"]
        sd[p + "self_attn.k_proj.weight"] = L["wk"]
        sd[p + "self_attn.v_proj.weight"] = L["wv"]
        sd[p + "self_attn.o_proj.weight"] = L["wo"]
        sd[p + "self_attn.q_norm.weight"] = L["q_norm"]
        sd[p + "self_attn.k_norm.weight"] = L["k_norm"]
        sd[p + "mlp.gate_proj.weight"] = L["wg"]
        sd[p + "mlp.up_proj.weight"] = L["wu"]
        sd[p + "mlp.down_proj.weight"] = L["wd"]
        sd[p + "input_layernorm.weight"] = L["in_norm"]
        sd[p + "post_attention_layernorm.weight"] = L["post_norm"]
    sd["norm.weight"] = final
    sd["embed_tokens.weight"] = np.zeros((8, c["hidden"]), np.float32)
    m.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()})
    rows = G.small_rows(9)
    prefill, steps = rows[:6], rows[6:]
    headt = torch.from_numpy(head)
    with torch.no_grad():
        cache = DynamicCache(config=cfg)
        out = m(inputs_embeds=torch.from_numpy(prefill)[None], use_cache=True, past_key_values=cache,
                output_hidden_states=True)
        hs = out.hidden_states
        states = np.stack([hs[i + 1][0].numpy() for i in range(c["layers"] - 1)])
        normed = out.last_hidden_state[0].numpy()
        logits0 = (out.last_hidden_state[0, -1] @ headt.T).numpy()
        cache = out.past_key_values
        step_normed, step_logits = [], []
        for r in range(steps.shape[0]):
            o = m(inputs_embeds=torch.from_numpy(steps[r:r + 1])[None], use_cache=True, past_key_values=cache)
            cache = o.past_key_values
            step_normed.append(o.last_hidden_state[0, -1].numpy())
            step_logits.append((o.last_hidden_state[0, -1] @ headt.T).numpy())
    np.savez_compressed(os.path.join(HERE, "qwen3_small.npz"), states=states.astype(np.float32),
                        normed=normed.astype(np.float32), logits0=logits0.astype(np.float32),
                        step_normed=np.stack(step_normed).astype(np.float32),
                        step_logits=np.stack(step_logits).astype(np.float32),
                        torch_version=np.array(torch.__version__), transformers_version=np.array(
                            __import__("transformers").__version__))
    print("qwen3_small.npz: states", states.shape, "normed", normed.shape, "steps", len(step_normed))


if __name__ == "__main__":
    q8_fixture()
    qwen3_fixture()
