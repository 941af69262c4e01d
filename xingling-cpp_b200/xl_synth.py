"""Seeded synthetic inputs for the XingLing token loop.

The real SFT weights and tokenizer are not available, so every measurement
and parity check runs on:

* a random-init fp32 weight tree in the reference's on-disk format (raw
  little-endian fp32 files, ``scripts/export_weights.py:13-25`` of the
  reference; read by ``Transformer::load``, ``src/transformer.cu:139-146``):
  every Linear weight and bias and the embedding ~ N(0, 0.02), every RMSNorm
  gain 1.0.  Tensor ``i`` of the fixed order below draws from
  ``numpy.random.default_rng(SeedSequence([seed, i]))``, so a tree is
  reproducible on any machine with this numpy;
* prompt ids ``numpy.random.default_rng(seed).integers(0, vocab, n)``;
* sampling uniforms from Philox4x32-10 (Salmon et al., "Parallel random
  numbers: as easy as 1, 2, 3", SC'11) with key = seed and counter = draw
  index, ``u = (x0 >> 8) * 2**-24`` — the same stream the engine's
  ``seed()`` produces, so it can be fed to the oracle and the engine alike.
"""
from __future__ import annotations

import concurrent.futures as cf
import json
import os
from dataclasses import asdict, dataclass

import numpy as np


@dataclass(frozen=True)
class ModelShape:
    layers: int = 16
    hidden: int = 1536
    heads: int = 24
    ffn: int = 4096
    vocab: int = 151669
    max_ctx: int = 768
    rope_base: float = 10000.0

    def engine_kwargs(self) -> dict:
        return dict(layers=self.layers, hidden=self.hidden, heads=self.heads, ffn=self.ffn, vocab=self.vocab,
                    max_ctx=self.max_ctx)

    def weight_bytes(self) -> int:
        return 4 * sum(int(np.prod(s)) for _, s, _ in weight_specs(self))


# The XingLing-0.68B shape of the reference's engine (src/inference.cu:19-28).
FULL = ModelShape()
# Small shapes for quick parity tests (same code paths, fewer / narrower layers).
TINY = ModelShape(layers=2, hidden=256, heads=4, ffn=512, vocab=2048, max_ctx=768)
WIDE2 = ModelShape(layers=2, hidden=1536, heads=24, ffn=4096, vocab=8192, max_ctx=768)

WEIGHT_SEED = 0
WEIGHT_STD = 0.02


def weight_specs(shape: ModelShape) -> list[tuple[str, tuple[int, ...], str]]:
    """(relative path, shape, 'normal' | 'ones') in generation order."""
    H, F = shape.hidden, shape.ffn
    specs: list[tuple[str, tuple[int, ...], str]] = [("embedding/weight.bin", (shape.vocab, H), "normal"),
                                                     ("norm/weight.bin", (H,), "ones")]
    for i in range(shape.layers):
        b = f"blocks/{i}/"
        for name in ("Q", "K", "V", "W"):
            specs.append((b + f"attn/{name}/weight.bin", (H, H), "normal"))
            specs.append((b + f"attn/{name}/bias.bin", (H,), "normal"))
        specs.append((b + "ffn/W1/weight.bin", (F, H), "normal"))
        specs.append((b + "ffn/W1/bias.bin", (F,), "normal"))
        specs.append((b + "ffn/V/weight.bin", (F, H), "normal"))
        specs.append((b + "ffn/V/bias.bin", (F,), "normal"))
        specs.append((b + "ffn/W2/weight.bin", (H, F), "normal"))
        specs.append((b + "ffn/W2/bias.bin", (H,), "normal"))
        specs.append((b + "norm1/weight.bin", (H,), "ones"))
        specs.append((b + "norm2/weight.bin", (H,), "ones"))
    return specs


def make_tensor(index: int, shape: tuple[int, ...], kind: str, seed: int = WEIGHT_SEED,
                std: float = WEIGHT_STD) -> np.ndarray:
    if kind == "ones":
        return np.ones(shape, dtype=np.float32)
    rng = np.random.default_rng(np.random.SeedSequence([seed, index]))
    a = rng.standard_normal(int(np.prod(shape)), dtype=np.float32)
    a *= np.float32(std)
    return a.reshape(shape)


def write_weight_tree(path: str, shape: ModelShape = FULL, seed: int = WEIGHT_SEED, std: float = WEIGHT_STD,
                      threads: int = 8) -> str:
    """Write (or reuse) the seeded tree under `path`; returns `path`."""
    stamp = os.path.join(path, "xl_synth.json")
    meta = {"shape": asdict(shape), "seed": seed, "std": std, "format": "raw-fp32-tree-v1"}
    if os.path.exists(stamp):
        with open(stamp) as f:
            if json.load(f) == meta:
                return path
    os.makedirs(path, exist_ok=True)
    specs = weight_specs(shape)

    def one(i: int) -> None:
        rel, shp, kind = specs[i]
        full = os.path.join(path, rel)
        os.makedirs(os.path.dirname(full), exist_ok=True)
        make_tensor(i, shp, kind, seed, std).tofile(full)

    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(one, range(len(specs))))
    with open(stamp, "w") as f:
        json.dump(meta, f)
    return path


def prompt_ids(seed: int, n: int, vocab: int = FULL.vocab) -> list[int]:
    return [int(v) for v in np.random.default_rng(seed).integers(0, vocab, size=n)]


_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
_LO = np.uint64(0xFFFFFFFF)


def philox4x32_10(counters: np.ndarray, seed: int) -> np.ndarray:
    """First output word of Philox4x32-10 for counter (c, 0, 0, 0), key (seed lo, seed hi)."""
    c = np.asarray(counters, dtype=np.uint64)
    c0 = (c & _LO).astype(np.uint32)
    c1 = (c >> np.uint64(32)).astype(np.uint32)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = np.uint32(seed & 0xFFFFFFFF)
    k1 = np.uint32((seed >> 32) & 0xFFFFFFFF)
    with np.errstate(over="ignore"):
        for _ in range(10):
            p0 = _M0 * c0.astype(np.uint64)
            p1 = _M1 * c2.astype(np.uint64)
            hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & _LO).astype(np.uint32)
            hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & _LO).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
            k0 = np.uint32(k0 + _W0)
            k1 = np.uint32(k1 + _W1)
    return c0


def philox_uniforms(seed: int, n: int, start: int = 0) -> np.ndarray:
    x0 = philox4x32_10(np.arange(start, start + n, dtype=np.uint64), seed)
    return (x0 >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)
