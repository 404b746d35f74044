"""Seeded synthetic inputs with the shapes and distributions of the Titan-block
workloads (no datasets or checkpoints are used by the path).

Weights and biases ~ N(0, 0.02); LayerNorm gamma = 1 + N(0, 0.02), beta ~
N(0, 0.02); the memory bank ~ N(0, mem_std) with mem_std given per workload
(1/sqrt(hidden) when unstated).  Generator: numpy PCG64 seeded per block.
"""
from __future__ import annotations

import numpy as np

WEIGHT_SHAPES = {
    "w_qkv": lambda H, F, Ms: (3 * H, H), "b_qkv": lambda H, F, Ms: (3 * H,),
    "w_o": lambda H, F, Ms: (H, H), "b_o": lambda H, F, Ms: (H,),
    "w_qm": lambda H, F, Ms: (H, H), "b_qm": lambda H, F, Ms: (H,),
    "w_km": lambda H, F, Ms: (H, H), "b_km": lambda H, F, Ms: (H,),
    "w_vm": lambda H, F, Ms: (H, H), "b_vm": lambda H, F, Ms: (H,),
    "w_om": lambda H, F, Ms: (H, H), "b_om": lambda H, F, Ms: (H,),
    "w_g": lambda H, F, Ms: (H, H), "b_g": lambda H, F, Ms: (H,),
    "w_1": lambda H, F, Ms: (F, H), "b_1": lambda H, F, Ms: (F,),
    "w_2": lambda H, F, Ms: (H, F), "b_2": lambda H, F, Ms: (H,),
}


def block_weights(H: int, F: int, Ms: int, seed: int, mem_std: float | None = None,
                  w_std: float = 0.02) -> dict:
    rng = np.random.default_rng(seed)
    w = {}
    for name, shp in WEIGHT_SHAPES.items():
        w[name] = (rng.standard_normal(shp(H, F, Ms), dtype=np.float32) * np.float32(w_std))
    for ln in ("ln1", "ln2"):
        w[ln + "_g"] = (1.0 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        w[ln + "_b"] = rng.standard_normal(H, dtype=np.float32) * np.float32(0.02)
    std = mem_std if mem_std is not None else 1.0 / np.sqrt(H)
    w["memory"] = rng.standard_normal((Ms, H), dtype=np.float32) * np.float32(std)
    return w


def activations(T: int, H: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((T, H), dtype=np.float32)


def embedding(vocab: int, H: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((vocab, H), dtype=np.float32) * np.float32(0.02)


def tokens(B: int, S: int, vocab: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, vocab, size=(B, S), dtype=np.int32)
