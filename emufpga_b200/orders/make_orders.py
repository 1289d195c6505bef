"""Writes the .order files of the benchmark models beside this script.

    python -m emufpga_b200.orders.make_orders

Each file is the library's consumption order (spm_order_default) for one
model: the [rotating] region in the order a decode step reads it (per layer
q, k, v, o, then the feed-forward or router and expert streams; the LM head
last), then the [resident] tensors (embedding, norm gains, router biases).
Tensor names depend only on the model family, its layer count and whether it
has router biases, so each order is computed from a miniature model with the
same names (few experts, tiny dimensions) instead of the full one.
"""
from __future__ import annotations

import dataclasses
from pathlib import Path

HERE = Path(__file__).resolve().parent

# file name -> recipe name in configs.RECIPES
MODELS = {
    "smollm2-135m.order": "smollm2-q8_0",
    "qwen3-8b.order": "qwen3-8b-q6_k",
    "olmoe-1b-7b.order": "olmoe-q6_k",
    "qwen3-30b-a3b.order": "qwen3-30b-a3b-q5_k",
}


def miniature(recipe):
    """The same tensor names at a size a test can synthesize in a moment."""
    from emufpga_b200._lib import Q8_0

    s = recipe.shape
    small = dataclasses.replace(s, hidden=64, intermediate=64, heads=2, kv_heads=1, head_dim=32, vocab=64,
                                experts=min(s.experts, 4), experts_used=min(s.experts_used, 2),
                                expert_ff=64 if s.experts else 0)
    return recipe.replace(shape=small, layer_type=Q8_0, embed_type=Q8_0, head_type=Q8_0, expert_type=Q8_0)


def order_text(recipe_name: str) -> str:
    import emufpga_b200 as eb
    from emufpga_b200 import configs

    mini = miniature(configs.RECIPES[recipe_name])
    return eb.default_order(mini.shape, eb.synth_gguf(mini))


def main() -> None:
    for name, recipe in MODELS.items():
        (HERE / name).write_text(order_text(recipe))
        print(HERE / name)


if __name__ == "__main__":
    main()
