"""Host-side workload logic of the BASELINE configurations: seeded shapes, the
pooled KV-cache layout, and how work is split across the GPUs of one box.

No kernel runs here; bench.py and the tests use these functions to lay out
buffers and to decide which rank owns which sequences / images / KV heads.

KV pool layout (the device-resident replacement of qkn_decoder.c:172-220):
sequence s owns rows [base_s, base_s + layers*cap_s); layer l of sequence s starts
at row base_s + l*cap_s, and position p of that layer is row base_s + l*cap_s + p,
the same ((layer*max)+pos) addressing as qkn_decoder.c:212-220 with a per-sequence
max.  Each row is n_kv_heads*head_dim wide: bf16 for K, fp16 for V.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

# BASELINE configs (shapes only; see BASELINE.json "configs")
CFG2 = dict(n_seqs=256, len_lo=1024, len_hi=8192, layers=28, n_heads=16, n_kv_heads=8, head_dim=128,
            theta=1e6)
CFG1 = dict(prefill=512, decode_steps=128, hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128, theta=1e6,
            eps=1e-6)
CFG3 = dict(images=128, patches=1024, layers=12, n_heads=12, head_dim=64)
CFG4 = dict(batch=32, prefix=320, suffix=128, layers=18, n_heads=8, n_kv_heads=1, head_dim=256, theta=1e4)
CFG5 = dict(batch=4, seq=32768, n_heads=16, n_kv_heads=8, head_dim=128, theta=1e6, layers=28)


def decode_lengths(n_seqs: int, lo: int, hi: int, seed: int = 0) -> np.ndarray:
    """KV lengths drawn uniformly from [lo, hi] with a seeded generator (cfg 2)."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=n_seqs).astype(np.int32)


@dataclass
class PoolLayout:
    lengths: np.ndarray       # [n_seqs] attended length before the step's append
    caps: np.ndarray          # [n_seqs] rows per layer reserved for each sequence
    base: np.ndarray          # [n_seqs] first pool row of each sequence
    layers: int
    rows: int                 # total pool rows

    def row0(self, layer: int) -> np.ndarray:
        """Pool row of position 0 of `layer` for every sequence."""
        return (self.base + layer * self.caps).astype(np.int64)

    def kv_bytes(self, kv_dim: int, extra_tokens: int = 0) -> int:
        """Algorithmic K+V bytes one decode step reads over all layers (2-byte elements)."""
        return int((self.lengths.astype(np.int64) + extra_tokens).sum()) * self.layers * kv_dim * 2 * 2


def pool_layout(lengths: np.ndarray, layers: int, reserve: int = 1) -> PoolLayout:
    """Contiguous per-sequence slabs with `reserve` free rows per layer for appends."""
    lengths = np.asarray(lengths, np.int32)
    caps = lengths.astype(np.int64) + reserve
    sizes = caps * layers
    base = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)
    return PoolLayout(lengths=lengths, caps=caps, base=base, layers=layers, rows=int(sizes.sum()))


def shard_by_bytes(lengths: np.ndarray, world: int) -> list[np.ndarray]:
    """Greedy longest-first bin packing of sequences onto `world` ranks by KV bytes.

    Returns, per rank, the indices of the sequences it owns.  Every sequence goes
    to exactly one rank; no data crosses ranks (decode attention of a sequence
    needs only its own cache)."""
    order = np.argsort(-np.asarray(lengths, np.int64), kind="stable")
    load = np.zeros(world, np.int64)
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = int(np.argmin(load))
        owned[r].append(int(i))
        load[r] += int(lengths[i])
    return [np.array(sorted(o), np.int64) for o in owned]


def shard_evenly(n_items: int, world: int, rank: int) -> range:
    """Contiguous block of items (images of cfg 3, sequences of cfg 4) for `rank`."""
    per = (n_items + world - 1) // world
    lo = min(n_items, rank * per)
    return range(lo, min(n_items, lo + per))


def kv_head_groups(n_kv_heads: int, world: int, rank: int) -> range:
    """KV heads owned by `rank` when long prefill is split by KV-head group (cfg 5)."""
    if n_kv_heads % world != 0:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {world} ranks")
    per = n_kv_heads // world
    return range(rank * per, (rank + 1) * per)


def causal_flops(seq_q: int, seq_k: int, n_heads: int, head_dim: int, q_offset: int = 0) -> int:
    """4*hd FLOPs per visible (query, key) pair per Q head (QK^T + PV), causal mask."""
    pairs = 0
    for i in range(seq_q):
        pairs += max(0, min(q_offset + i + 1, seq_k))
    return 4 * head_dim * n_heads * pairs


def causal_flops_square(L: int, n_heads: int, head_dim: int) -> int:
    return 4 * head_dim * n_heads * (L * (L + 1) // 2)


def prefix_lm_flops(seq: int, prefix: int, n_heads: int, head_dim: int) -> int:
    pairs = prefix * prefix + sum(i + 1 for i in range(prefix, seq))
    return 4 * head_dim * n_heads * pairs


def full_flops(seq: int, n_heads: int, head_dim: int) -> int:
    return 4 * head_dim * n_heads * seq * seq
