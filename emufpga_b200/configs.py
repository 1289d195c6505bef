"""The model shapes of the token-loop workloads, and small shapes for tests.

Every workload is random-init: weights N(0, 0.02) from a seeded generator,
quantized by this library's encoders; norm gains 1.  Names follow the
reference's model families (SmolLM2, Qwen3, OLMoE, Qwen3-MoE).
"""
from __future__ import annotations

import dataclasses

from ._lib import F32, LLAMA, OLMOE, Q2_K, Q5_K, Q6_K, Q8_0, QWEN3, QWEN3MOE, ModelCfg, SynthSpec


@dataclasses.dataclass(frozen=True)
class Shape:
    family: int
    layers: int
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    experts: int = 0
    experts_used: int = 0
    expert_ff: int = 0
    tied: bool = False
    rope_base: float = 10000.0
    eps: float = 1e-5

    def cfg(self) -> ModelCfg:
        c = ModelCfg()
        for f in dataclasses.fields(self):
            setattr(c, f.name, int(getattr(self, f.name)) if f.name == "tied" else getattr(self, f.name))
        return c

    @property
    def moe(self) -> bool:
        return self.family in (OLMOE, QWEN3MOE)

    @property
    def q_width(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim


@dataclasses.dataclass(frozen=True)
class Recipe:
    """A synthetic GGUF: shape, block types, seed."""

    shape: Shape
    layer_type: int
    embed_type: int
    head_type: int
    expert_type: int = Q6_K
    seed: int = 0
    sigma: float = 0.02
    zipf_s: float = 0.0
    gain_sigma: float = 0.0

    def spec(self, threads: int = 0) -> SynthSpec:
        s = SynthSpec()
        s.cfg = self.shape.cfg()
        s.layer_type, s.expert_type = self.layer_type, self.expert_type
        s.embed_type, s.head_type = self.embed_type, self.head_type
        s.seed, s.sigma, s.zipf_s, s.gain_sigma, s.threads = self.seed, self.sigma, self.zipf_s, self.gain_sigma, threads
        return s

    def replace(self, **kw) -> "Recipe":
        return dataclasses.replace(self, **kw)


# ---- benchmark model shapes ----
SMOLLM2 = Shape(LLAMA, 30, 576, 1536, 9, 3, 64, 49152, tied=True, rope_base=10000.0, eps=1e-5)
QWEN3_8B = Shape(QWEN3, 36, 4096, 12288, 32, 8, 128, 151936, rope_base=1e6, eps=1e-6)
OLMOE_1B7B = Shape(OLMOE, 16, 2048, 0, 16, 16, 128, 50304, experts=64, experts_used=8, expert_ff=1024,
                   rope_base=10000.0, eps=1e-5)
QWEN3_30B_A3B = Shape(QWEN3MOE, 48, 2048, 0, 32, 4, 128, 151936, experts=128, experts_used=8, expert_ff=768,
                      rope_base=1e6, eps=1e-6)

RECIPES = {
    "smollm2-q8_0": Recipe(SMOLLM2, Q8_0, Q8_0, Q8_0),
    "qwen3-8b-q6_k": Recipe(QWEN3_8B, Q6_K, Q6_K, Q6_K),
    "olmoe-q6_k": Recipe(OLMOE_1B7B, Q6_K, Q6_K, Q6_K, expert_type=Q6_K, zipf_s=1.1),
    "olmoe-q2_k": Recipe(OLMOE_1B7B, Q6_K, Q6_K, Q6_K, expert_type=Q2_K, zipf_s=1.1),
    "qwen3-30b-a3b-q5_k": Recipe(QWEN3_30B_A3B, Q5_K, Q5_K, Q5_K, expert_type=Q5_K, zipf_s=1.1),
}

# The five benchmark workloads (prompt lengths, generated tokens, clients).
WORKLOADS = {
    "smollm2-b1": dict(recipe="smollm2-q8_0", prompts=[32], steps=64, prompt_seed=1),
    "smollm2-b5": dict(recipe="smollm2-q8_0", prompts=[16, 24, 32, 48, 64], steps=128, prompt_seed=2),
    "qwen3-8b-b1": dict(recipe="qwen3-8b-q6_k", prompts=[512], steps=256, prompt_seed=3),
    "qwen3-8b-b4": dict(recipe="qwen3-8b-q6_k", prompts=[512] * 4, steps=256, prompt_seed=4),
    "olmoe-q6_k-b8": dict(recipe="olmoe-q6_k", prompts=[256] * 8, steps=128, prompt_seed=5),
    "olmoe-q2_k-b8": dict(recipe="olmoe-q2_k", prompts=[256] * 8, steps=128, prompt_seed=5),
    "qwen3-30b-b8": dict(recipe="qwen3-30b-a3b-q5_k", prompts=[1024] * 8, steps=256, prompt_seed=6),
}

# ---- small shapes for parity tests (same families and block types) ----
TINY = {
    "llama-q8_0": Recipe(Shape(LLAMA, 2, 64, 128, 4, 2, 16, 96, tied=True), Q8_0, Q8_0, Q8_0, seed=7, gain_sigma=0.1),
    "llama-q6_k": Recipe(Shape(LLAMA, 2, 256, 512, 4, 2, 64, 128, tied=True), Q6_K, Q6_K, Q6_K, seed=8, gain_sigma=0.1),
    "qwen3-q6_k": Recipe(Shape(QWEN3, 2, 256, 512, 4, 2, 64, 160, rope_base=1e6, eps=1e-6), Q6_K, Q6_K, Q6_K, seed=9,
                         gain_sigma=0.1),
    "qwen3-q5_k": Recipe(Shape(QWEN3, 2, 256, 512, 4, 1, 64, 160, rope_base=1e6, eps=1e-6), Q5_K, Q5_K, Q5_K, seed=10,
                         gain_sigma=0.1),
    "qwen3-q2_k": Recipe(Shape(QWEN3, 2, 256, 512, 4, 2, 64, 160, rope_base=1e6, eps=1e-6), Q2_K, Q2_K, Q6_K, seed=11,
                         gain_sigma=0.1),
    # four query heads of 64 per kv head, two kv heads
    "qwen3-g4-q5_k": Recipe(Shape(QWEN3, 2, 256, 512, 8, 2, 64, 160, rope_base=1e6, eps=1e-6), Q5_K, Q5_K, Q5_K,
                            seed=16, gain_sigma=0.1),
    # eight query heads of 128 per kv head (the Qwen3-30B-A3B grouping), two kv heads
    "qwen3-g8-q6_k": Recipe(Shape(QWEN3, 2, 256, 512, 16, 2, 128, 160, rope_base=1e6, eps=1e-6), Q6_K, Q6_K, Q6_K,
                            seed=15, gain_sigma=0.1),
    "olmoe-q6_k": Recipe(Shape(OLMOE, 2, 256, 0, 4, 4, 64, 128, experts=8, experts_used=2, expert_ff=256),
                         Q6_K, Q6_K, Q6_K, expert_type=Q6_K, seed=12, zipf_s=1.1, gain_sigma=0.1),
    "olmoe-q2_k": Recipe(Shape(OLMOE, 2, 256, 0, 4, 4, 64, 128, experts=8, experts_used=2, expert_ff=256),
                         Q6_K, Q6_K, Q6_K, expert_type=Q2_K, seed=14, zipf_s=1.1, gain_sigma=0.1),
    "qwen3moe-q5_k": Recipe(Shape(QWEN3MOE, 2, 256, 0, 4, 2, 64, 128, experts=8, experts_used=2, expert_ff=256,
                                  rope_base=1e6, eps=1e-6), Q5_K, Q5_K, Q5_K, expert_type=Q5_K, seed=13, zipf_s=1.1,
                            gain_sigma=0.1),
}

_MASK = (1 << 64) - 1


def _mix64(z: int) -> int:
    z = (z + 0x9E3779B97F4A7C15) & _MASK
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK
    return z ^ (z >> 31)


def prompt_tokens(seed: int, client: int, length: int, vocab: int) -> list[int]:
    """Seeded uniform token ids (splitmix64 counters), independent per client."""
    key = _mix64(seed * 0x1000193 + client)
    return [_mix64(key ^ i) % vocab for i in range(length)]


def workload_prompts(name: str) -> list[list[int]]:
    w = WORKLOADS[name]
    vocab = RECIPES[w["recipe"]].shape.vocab
    return [prompt_tokens(w["prompt_seed"], i, n, vocab) for i, n in enumerate(w["prompts"])]
