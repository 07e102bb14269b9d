"""Parameter-set shapes and seeded synthetic inputs of the benchmark configurations.

The configurations are GPT-shaped parameter lists (no model runs): tok_emb[V,d],
pos_emb[T,d], then per layer ln1.w[d], ln1.b[d], qkv.W[d,3d], qkv.b[3d], proj.W[d,d],
proj.b[d], ln2.w[d], ln2.b[d], fc.W[d,4d], fc.b[4d], fc2.W[4d,d], fc2.b[d], and finally
ln_f.w[d]. Parameters are split into the two groups the reference training loop uses:
weight decay on tensors with ndim >= 2, none on the rest
(decay_parameter_groups, namitorch/training/runner.py:83-90).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class GPTShape:
    n_layer: int
    d_model: int
    vocab: int
    block: int
    name: str = ""

    def shapes(self) -> list[tuple[str, tuple[int, ...]]]:
        d, v, t = self.d_model, self.vocab, self.block
        out: list[tuple[str, tuple[int, ...]]] = [("tok_emb", (v, d)), ("pos_emb", (t, d))]
        for i in range(self.n_layer):
            p = f"h{i}."
            out += [
                (p + "ln1.w", (d,)), (p + "ln1.b", (d,)),
                (p + "qkv.W", (d, 3 * d)), (p + "qkv.b", (3 * d,)),
                (p + "proj.W", (d, d)), (p + "proj.b", (d,)),
                (p + "ln2.w", (d,)), (p + "ln2.b", (d,)),
                (p + "fc.W", (d, 4 * d)), (p + "fc.b", (4 * d,)),
                (p + "fc2.W", (4 * d, d)), (p + "fc2.b", (d,)),
            ]
        out.append(("ln_f.w", (d,)))
        return out

    def numel(self) -> int:
        return sum(int(np.prod(s)) for _, s in self.shapes())

    def groups(self) -> tuple[list[int], list[int]]:
        """Indices with weight decay (ndim >= 2) and without."""
        shapes = self.shapes()
        decay = [i for i, (_, s) in enumerate(shapes) if len(s) >= 2]
        no_decay = [i for i, (_, s) in enumerate(shapes) if len(s) < 2]
        return decay, no_decay


# BASELINE configurations 0/1 (4-layer), 2 (GPT-2 small), 3 (1.3B).
CONFIG_SMALL = GPTShape(n_layer=4, d_model=256, vocab=4096, block=256, name="gpt-4L-d256")
CONFIG_124M = GPTShape(n_layer=12, d_model=768, vocab=50257, block=1024, name="gpt2-small-124M")
CONFIG_1P3B = GPTShape(n_layer=24, d_model=2048, vocab=50257, block=2048, name="gpt-1.3B")

ADAMW_OPTIONS = {"lr": 3e-4, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.1}

# Config 4: LM-head logits of the fused softmax cross-entropy.
XENT_ROWS = 8192
XENT_CLASSES = 50257


@dataclass
class Workload:
    shape: GPTShape
    params: list[np.ndarray] = field(default_factory=list)


def init_params(shape: GPTShape, seed: int = 0, std: float = 0.02) -> list[np.ndarray]:
    """Parameters ~ N(0, std) as float32, drawn in list order from default_rng(seed)."""
    rng = np.random.default_rng(seed)
    return [rng.normal(0.0, std, s).astype(np.float32) for _, s in shape.shapes()]


def normal_grads(shape: GPTShape, seed: int = 0, std: float = 1e-3) -> list[np.ndarray]:
    """Gradients ~ N(0, std) as float32 (config 0 draws the same ones every step)."""
    rng = np.random.default_rng(seed)
    return [rng.normal(0.0, std, s).astype(np.float32) for _, s in shape.shapes()]


def outlier_grads(shape: GPTShape, seed: int = 0, std: float = 1e-3, outlier_std: float = 1e-1,
                  outlier_fraction: float = 0.01) -> list[np.ndarray]:
    """Config 2 gradients: N(0, std) with a seeded 1 % of elements drawn from N(0, outlier_std)."""
    rng = np.random.default_rng(seed)
    out = []
    for _, s in shape.shapes():
        g = rng.normal(0.0, std, s).astype(np.float32)
        mask = rng.random(s) < outlier_fraction
        g[mask] = rng.normal(0.0, outlier_std, int(mask.sum())).astype(np.float32)
        out.append(g)
    return out


def inf_positions(numel: int, fraction: float = 0.001, seed: int = 0) -> np.ndarray:
    """Config 1: the element indices (of tok_emb) set to +inf at the injection step."""
    rng = np.random.default_rng(seed)
    count = max(1, int(round(numel * fraction)))
    return np.sort(rng.choice(numel, size=count, replace=False))


def xent_inputs(rows: int = XENT_ROWS, classes: int = XENT_CLASSES, seed: int = 0, std: float = 2.0):
    """Config 4: logits N(0, std) (float32, to be rounded to bf16) and int64 targets in [0, C)."""
    rng = np.random.default_rng(seed)
    logits = rng.normal(0.0, std, (rows, classes)).astype(np.float32)
    targets = rng.integers(0, classes, rows, dtype=np.int64)
    return logits, targets
