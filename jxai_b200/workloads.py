"""The five decode-attention workloads of the benchmark, and how they shard.

Each workload is one decode step of a model shape whose attention fields come
from the reference's per-architecture rules (src/transformer.cpp:140-179 for
the RoPE style, :2117-2137 for per-layer SWA/rope base): every sequence's cache
holds T-1 seeded N(0,1) rows, the step appends row T-1 and attends over T rows
(SWA layers: the last `window` rows).  Values are synthetic (no checkpoints or
datasets exist for this path); shapes follow the named models.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Sequence

import numpy as np

from .attention import Layer

SEED = 0x6A78616900000001


@dataclass
class Workload:
    name: str
    model: str
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    neox: bool
    lengths: List[int]            # attended length T per sequence (cache holds T-1 rows)
    dtype: str = "f32"
    rope_base: float = 1e4
    rope_base_swa: float = 1e4
    swa_layers: Sequence[int] = ()
    window: int = 0
    sharding: str = "replica"     # replica | sequences | positions
    notes: str = ""
    layers: List[Layer] = field(default_factory=list)

    def __post_init__(self):
        if not self.layers:
            self.layers = [
                Layer(self.head_dim, self.head_dim,
                      self.rope_base_swa if l in self.swa_layers else self.rope_base, l,
                      is_swa=l in self.swa_layers)
                for l in range(self.n_layers)]

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def elem_size(self) -> int:
        return 4 if self.dtype == "f32" else 2

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    def attended(self, T: int, layer: Layer) -> int:
        return min(T, self.window) if (layer.is_swa and self.window > 0) else T

    def kv_read_bytes(self, lengths: Sequence[int] | None = None) -> int:
        """Algorithmic KV bytes one step reads: sum over sequences and layers of
        attended rows x kv_dim x 2 (K and V) x element size."""
        lengths = self.lengths if lengths is None else lengths
        rows = sum(self.attended(T, L) for T in lengths for L in self.layers)
        return rows * self.kv_dim * 2 * self.elem_size

    def other_bytes(self, n_seqs: int | None = None) -> int:
        """Non-cache traffic of a step: q/k/v reads, appended rows, output."""
        n = len(self.lengths) if n_seqs is None else n_seqs
        per = (self.q_dim * 4 * 2            # q read + out write
               + self.kv_dim * 4 * 2         # k, v inputs read
               + self.kv_dim * self.elem_size * 2)  # appended K and V rows
        return n * self.n_layers * per

    def describe(self) -> dict:
        return {"workload": self.name, "model_shape": self.model, "layers": self.n_layers,
                "heads": self.n_heads, "kv_heads": self.n_kv_heads, "head_dim": self.head_dim,
                "n_seqs": len(self.lengths), "T": (self.lengths[0] if len(set(self.lengths)) == 1
                                                   else [min(self.lengths), max(self.lengths)]),
                "kv_dtype": self.dtype, "rope": "neox" if self.neox else "interleaved",
                "window": self.window, "swa_layers": len(self.swa_layers)}


def c3_lengths(n: int = 256, lo: int = 128, hi: int = 8192, seed: int = SEED) -> List[int]:
    """Ragged lengths T_i ~ U[lo, hi] (inclusive) drawn from the benchmark seed."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(lo, hi, size=n, endpoint=True)]


def make(name: str, dtype: str | None = None) -> Workload:
    name = name.lower()
    if name in ("c1", "qwen2.5-0.5b"):
        w = Workload("c1", "Qwen2.5-0.5B", 24, 14, 2, 64, True, [512], rope_base=1e6,
                     notes="CPU-runnable reference case")
    elif name in ("c2", "llama-3.2-1b"):
        w = Workload("c2", "Llama-3.2-1B", 16, 32, 8, 64, False, [4096], rope_base=5e5)
    elif name in ("c3", "llama-3.2-1b-batched"):
        w = Workload("c3", "Llama-3.2-1B", 16, 32, 8, 64, False, c3_lengths(), rope_base=5e5,
                     sharding="sequences")
    elif name in ("c4", "mistral-7b"):
        w = Workload("c4", "Mistral-7B", 32, 32, 8, 128, False, [131072], rope_base=1e6,
                     sharding="positions")
    elif name in ("c5", "gemma-3-1b"):
        swa = [l for l in range(26) if l % 6 != 5]  # 5 local : 1 global (layers 5, 11, 17, 23 global)
        w = Workload("c5", "Gemma-3-1B", 26, 4, 1, 256, True, [16384] * 64, rope_base=1e6,
                     rope_base_swa=1e4, swa_layers=swa, window=512, sharding="sequences")
    else:
        raise ValueError(f"unknown workload {name!r}")
    if dtype:
        w.dtype = dtype
    return w


def lpt_partition(lengths: Sequence[int], n_parts: int, cost=None) -> List[List[int]]:
    """Greedy longest-processing-time assignment of sequences to n_parts ranks,
    balancing the summed cost (default: the length).  Returns sorted index lists."""
    cost = cost or (lambda T: T)
    order = sorted(range(len(lengths)), key=lambda i: (-cost(lengths[i]), i))
    loads = [0] * n_parts
    parts: List[List[int]] = [[] for _ in range(n_parts)]
    for i in order:
        r = min(range(n_parts), key=lambda j: (loads[j], j))
        parts[r].append(i)
        loads[r] += cost(lengths[i])
    return [sorted(p) for p in parts]


def position_shards(T: int, n_parts: int) -> List[tuple]:
    """Contiguous position ranges [begin, end) of one long sequence, one per rank."""
    return [(T * r // n_parts, T * (r + 1) // n_parts) for r in range(n_parts)]


def rank_kv_bytes(w: Workload, mode: str, rank: int, world: int, shift: int = 0) -> int:
    """KV bytes one rank reads in a step `shift` tokens after the workload's
    first (every sequence then one row longer).  mode: "replica" (every rank
    the whole workload), "sequences" (the LPT share of the sequences) or
    "positions" (one sequence sharded by position; rows past the first step's
    shard ends belong to the last rank, which holds the newest positions)."""
    if mode == "positions":
        T0 = w.lengths[0]
        T = T0 + shift
        b, e = position_shards(T0, world)[rank]
        end = T if rank == world - 1 else min(e, T)
        rows = sum(max(0, end - max(b, T - w.attended(T, L))) for L in w.layers)
        return rows * w.kv_dim * 2 * w.elem_size
    if mode == "sequences":
        local = [w.lengths[i] for i in lpt_partition(w.lengths, world)[rank]]
    else:
        local = list(w.lengths)
    return w.kv_read_bytes([t + shift for t in local])
