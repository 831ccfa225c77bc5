"""Write random-init model folders in the Cactus layout (config.txt + .weights files).

The benchmark configurations use random-initialised weights of the named architectures
(no network, no checkpoints). File names follow the reference converter
(python/src/converter_llm.py:71-228): token_embeddings, output_norm, [output_weight],
layer_{i}_{attn_q,attn_k,attn_v,attn_output,input_norm,attn_q_norm,attn_k_norm,
ffn_gate,ffn_up,ffn_down,post_attn_norm[,pre_ffn_norm,post_ffn_norm]}.weights.
Weights are float32 N(0, 0.02) from ``numpy.random.default_rng(seed)`` drawn in a fixed
order, quantised with the reference's group rule (cactus_b200.weights).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np

from . import weights as W


@dataclass
class Arch:
    name: str
    model_type: str  # qwen | gemma | smol
    num_layers: int
    hidden_dim: int
    ffn_intermediate_dim: int
    attention_heads: int
    attention_kv_heads: int
    attention_head_dim: int
    vocab_size: int
    rope_theta: float
    layer_norm_eps: float = 1e-6
    tie_word_embeddings: bool = True
    # precision per role: attn, mlp, embed (INT8 | INT4 | FP16)
    precision: dict = field(default_factory=lambda: {"attn": "INT8", "mlp": "INT8", "embed": "INT8"})
    group_size: int = 32


def qwen3_0_6b(group_size=32) -> Arch:
    """Config 2: Qwen3-0.6B shape, INT8 weights."""
    return Arch("qwen3-0.6b", "qwen", 28, 1024, 3072, 16, 8, 128, 151936, 1e6,
                precision={"attn": "INT8", "mlp": "INT8", "embed": "INT8"}, group_size=group_size)


def gemma3_270m(group_size=32) -> Arch:
    """Config 3: Gemma-3-270m shape; INT8 attention, INT4 MLP, FP16 embeddings / lm_head."""
    return Arch("gemma3-270m", "gemma", 18, 640, 2048, 4, 1, 256, 262144, 1e6,
                precision={"attn": "INT8", "mlp": "INT4", "embed": "FP16"}, group_size=group_size)


def llama3_2_1b(group_size=32) -> Arch:
    """Config 4: Llama-3.2-1B shape (model_type smol), INT4 group-32 weights; theta 5e5."""
    return Arch("llama3.2-1b", "smol", 16, 2048, 8192, 32, 8, 64, 128256, 5e5,
                precision={"attn": "INT4", "mlp": "INT4", "embed": "INT4"}, group_size=group_size)


def tiny(model_type="qwen", layers=2, group_size=32, precision=None, vocab=1000, hidden=256, ffn=512,
         heads=4, kv_heads=2, head_dim=64, theta=1e6) -> Arch:
    """Small shapes for fast parity tests."""
    return Arch(f"tiny-{model_type}", model_type, layers, hidden, ffn, heads, kv_heads, head_dim, vocab, theta,
                precision=precision or {"attn": "INT8", "mlp": "INT8", "embed": "INT8"}, group_size=group_size)


def write_config(folder: str, a: Arch):
    lines = [
        f"vocab_size={a.vocab_size}",
        "bos_token_id=1",
        "eos_token_id=2",
        f"num_layers={a.num_layers}",
        f"hidden_dim={a.hidden_dim}",
        f"ffn_intermediate_dim={a.ffn_intermediate_dim}",
        f"attention_heads={a.attention_heads}",
        f"attention_kv_heads={a.attention_kv_heads}",
        f"attention_head_dim={a.attention_head_dim}",
        f"layer_norm_eps={a.layer_norm_eps}",
        f"rope_theta={a.rope_theta}",
        f"tie_word_embeddings={'true' if a.tie_word_embeddings else 'false'}",
        f"model_type={a.model_type}",
        "precision=INT8",
    ]
    with open(os.path.join(folder, "config.txt"), "w") as f:
        f.write("\n".join(lines) + "\n")


def make_model(folder: str, a: Arch, seed: int = 0, norm_std: float = 0.0, std: float = 0.02) -> str:
    """Create (or reuse) a random-init model folder; returns the folder path.

    norm_std > 0 draws norm weights as 1 + N(0, norm_std) (parity tests); 0 keeps them 1.0.
    """
    stamp = os.path.join(folder, ".complete")
    if os.path.exists(stamp):
        return folder
    os.makedirs(folder, exist_ok=True)
    rng = np.random.default_rng(seed)
    G = a.group_size
    H, F, D = a.hidden_dim, a.ffn_intermediate_dim, a.attention_head_dim

    def mat(n, k):
        return rng.standard_normal((n, k), dtype=np.float32) * np.float32(std)

    def norm(n):
        if norm_std > 0:
            return (np.float32(1.0) + rng.standard_normal(n, dtype=np.float32) * np.float32(norm_std))
        return np.ones(n, np.float32)

    def save(name, w, prec):
        W.save_tensor(os.path.join(folder, name), w, prec, G)

    save("token_embeddings.weights", mat(a.vocab_size, H), a.precision["embed"])
    save("output_norm.weights", norm(H), "FP16")
    if not a.tie_word_embeddings:
        save("output_weight.weights", mat(a.vocab_size, H), a.precision["embed"])
    for i in range(a.num_layers):
        p = f"layer_{i}_"
        pa, pm = a.precision["attn"], a.precision["mlp"]
        save(p + "attn_q.weights", mat(a.attention_heads * D, H), pa)
        save(p + "attn_k.weights", mat(a.attention_kv_heads * D, H), pa)
        save(p + "attn_v.weights", mat(a.attention_kv_heads * D, H), pa)
        save(p + "attn_output.weights", mat(H, a.attention_heads * D), pa)
        save(p + "input_norm.weights", norm(H), "FP16")
        if a.model_type in ("qwen", "gemma"):
            save(p + "attn_q_norm.weights", norm(D), "FP16")
            save(p + "attn_k_norm.weights", norm(D), "FP16")
        save(p + "ffn_gate.weights", mat(F, H), pm)
        save(p + "ffn_up.weights", mat(F, H), pm)
        save(p + "ffn_down.weights", mat(H, F), pm)
        save(p + "post_attn_norm.weights", norm(H), "FP16")
        if a.model_type == "gemma":
            save(p + "pre_ffn_norm.weights", norm(H), "FP16")
            save(p + "post_ffn_norm.weights", norm(H), "FP16")
    write_config(folder, a)
    open(stamp, "w").close()
    return folder


def default_model_dir(a: Arch, seed: int = 0, norm_std: float = 0.0) -> str:
    base = os.environ.get("CACTUS_B200_MODELS", os.path.join(os.path.expanduser("~"), ".cache", "cactus_b200"))
    return os.path.join(base, f"{a.name}-g{a.group_size}-s{seed}-n{norm_std}-L{a.num_layers}-V{a.vocab_size}")
