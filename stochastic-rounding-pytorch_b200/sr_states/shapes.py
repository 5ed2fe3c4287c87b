"""Parameter shapes of the model-shaped optimizer workloads (no model code).

Lists of (name, shape) in ``model.parameters()`` order, used by the benchmark
and the distributed tests.  Counts: GPT-2 small 124,439,808 parameters in 148
tensors (tied embeddings); Llama-3-8B 8,030,261,248 in 291; Llama-3-70B
70,553,706,496 in 723 (untied embeddings, RMSNorm vectors).
"""

from __future__ import annotations


def gpt2_small():
    d, ctx, vocab = 768, 1024, 50257
    shapes = [("wte", (vocab, d)), ("wpe", (ctx, d))]
    for i in range(12):
        shapes += [(f"h{i}.ln_1.weight", (d,)), (f"h{i}.ln_1.bias", (d,)),
                   (f"h{i}.attn.c_attn.weight", (d, 3 * d)), (f"h{i}.attn.c_attn.bias", (3 * d,)),
                   (f"h{i}.attn.c_proj.weight", (d, d)), (f"h{i}.attn.c_proj.bias", (d,)),
                   (f"h{i}.ln_2.weight", (d,)), (f"h{i}.ln_2.bias", (d,)),
                   (f"h{i}.mlp.c_fc.weight", (d, 4 * d)), (f"h{i}.mlp.c_fc.bias", (4 * d,)),
                   (f"h{i}.mlp.c_proj.weight", (4 * d, d)), (f"h{i}.mlp.c_proj.bias", (d,))]
    return shapes + [("ln_f.weight", (d,)), ("ln_f.bias", (d,))]


def _llama(layers, d, kv, ffn, vocab=128256):
    shapes = [("embed_tokens", (vocab, d))]
    for i in range(layers):
        shapes += [(f"layers.{i}.input_layernorm", (d,)), (f"layers.{i}.q_proj", (d, d)),
                   (f"layers.{i}.k_proj", (kv, d)), (f"layers.{i}.v_proj", (kv, d)),
                   (f"layers.{i}.o_proj", (d, d)), (f"layers.{i}.post_attention_layernorm", (d,)),
                   (f"layers.{i}.gate_proj", (ffn, d)), (f"layers.{i}.up_proj", (ffn, d)),
                   (f"layers.{i}.down_proj", (d, ffn))]
    return shapes + [("norm", (d,)), ("lm_head", (vocab, d))]


def llama3_8b():
    return _llama(32, 4096, 8 * 128, 14336)


def llama3_70b():
    return _llama(80, 8192, 8 * 128, 28672)


def numel(shape) -> int:
    n = 1
    for s in shape:
        n *= s
    return n


MODELS = {"gpt2": gpt2_small, "llama3-8b": llama3_8b, "llama3-70b": llama3_70b}
