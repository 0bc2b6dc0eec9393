"""Multi-GPU work split for the attention path: independent (sequence, KV-head) units over ranks.

Attention of one sequence and one KV head (with its G query heads) reads nothing another unit writes, so a batch
can be split over GPUs with no exchange step: every rank runs its own units through the same C ABI (a head subset
of a sequence is a pointer offset plus a smaller head count; strides are unchanged), and a collective is only
needed to gather results. Units are packed onto ranks longest-processing-time first under a two-roofline cost
model (tensor-core FLOPs for prefill, HBM bytes for decode), which keeps the slowest rank close to the mean.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass, field


@dataclass(frozen=True)
class Unit:
    seq: int            # sequence index in the batch
    kv_head: int        # first KV head of the unit (the unit covers their G query heads each)
    tokens: int         # query tokens (1 for decode)
    start: int          # absolute position of the first query token (decode: context length - 1)
    group: int          # query heads per KV head (G)
    head_dim: int = 64
    kv_heads: int = 1   # consecutive KV heads in the unit

    @property
    def flops(self) -> float:
        """QKᵀ + P·V FLOPs of the visible (query, key) pairs: Σ_t 4·d·(start + t + 1), times G and the KV heads."""
        T, s = self.tokens, self.start
        return self.kv_heads * self.group * 4.0 * self.head_dim * (T * s + T * (T + 1) / 2.0)

    @property
    def kv_bytes(self) -> float:
        """f16 K and V rows this unit reads once."""
        return self.kv_heads * (self.start + self.tokens) * self.head_dim * 2.0 * 2.0

    def cost(self, tflops: float = 1000.0, hbm_gbs: float = 6000.0) -> float:
        """Seconds under the slower of the tensor-core and HBM rooflines."""
        return max(self.flops / (tflops * 1e12), self.kv_bytes / (hbm_gbs * 1e9))


@dataclass
class Plan:
    ranks: list[list[Unit]] = field(default_factory=list)
    loads: list[float] = field(default_factory=list)

    @property
    def imbalance(self) -> float:
        """max load / mean load (1.0 = perfect)."""
        mean = sum(self.loads) / max(1, len(self.loads))
        return max(self.loads) / mean if mean > 0 else 1.0


def units_for_batch(seq_tokens: list[int], seq_starts: list[int], n_heads: int, n_kv_heads: int,
                    head_dim: int = 64) -> list[Unit]:
    """Every (sequence, KV head) unit of a batch."""
    if n_kv_heads <= 0 or n_heads % n_kv_heads:
        raise ValueError("n_heads must be a positive multiple of n_kv_heads")
    if len(seq_tokens) != len(seq_starts):
        raise ValueError("seq_tokens and seq_starts differ in length")
    g = n_heads // n_kv_heads
    return [Unit(s, h, int(t), int(st), g, head_dim) for s, (t, st) in enumerate(zip(seq_tokens, seq_starts))
            for h in range(n_kv_heads)]


def head_group_units(seq_tokens: list[int], seq_starts: list[int], n_kv_heads: int, kv_heads_per_unit: int,
                     group: int = 1, head_dim: int = 64, first_seq: int = 0) -> list[Unit]:
    """Units of `kv_heads_per_unit` consecutive KV heads (a divisor of n_kv_heads) per sequence: the same split as
    units_for_batch, coarser, so that a rank's units all have one head count and run as one call."""
    if n_kv_heads % kv_heads_per_unit:
        raise ValueError("kv_heads_per_unit must divide n_kv_heads")
    return [Unit(first_seq + s, h, int(t), int(st), group, head_dim, kv_heads_per_unit)
            for s, (t, st) in enumerate(zip(seq_tokens, seq_starts)) for h in range(0, n_kv_heads, kv_heads_per_unit)]


def partition(units: list[Unit], n_ranks: int, tflops: float = 1000.0, hbm_gbs: float = 6000.0) -> Plan:
    """Longest-processing-time-first packing of units onto n_ranks (deterministic: ties go to the lower rank,
    equal-cost units keep their input order)."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    order = sorted(range(len(units)), key=lambda i: (-units[i].cost(tflops, hbm_gbs), i))
    heap = [(0.0, r) for r in range(n_ranks)]
    plan = Plan([[] for _ in range(n_ranks)], [0.0] * n_ranks)
    for i in order:
        load, r = heapq.heappop(heap)
        u = units[i]
        plan.ranks[r].append(u)
        load += u.cost(tflops, hbm_gbs)
        plan.loads[r] = load
        heapq.heappush(heap, (load, r))
    for r in range(n_ranks):  # run each rank's units in (sequence, head) order: contiguous head ranges
        plan.ranks[r].sort(key=lambda u: (u.seq, u.kv_head))
    return plan


def head_ranges(units: list[Unit]) -> list[tuple[int, int, int]]:
    """Collapse one rank's units into (seq, first_kv_head, n_kv_heads) runs of consecutive KV heads, each of which
    is one ABI call (pointer offset to the first head, n_heads = n_kv_heads * G)."""
    runs: list[tuple[int, int, int]] = []
    for u in sorted(units, key=lambda u: (u.seq, u.kv_head)):
        if runs and runs[-1][0] == u.seq and runs[-1][1] + runs[-1][2] == u.kv_head:
            s, h0, n = runs[-1]
            runs[-1] = (s, h0, n + u.kv_heads)
        else:
            runs.append((u.seq, u.kv_head, u.kv_heads))
    return runs
