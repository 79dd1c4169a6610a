"""Partition of one decode session over the GPUs of a node (expert
parallelism + split-KV along the sequence).

* Experts: rank r holds experts [r*E/W, (r+1)*E/W) of every layer; the router
  runs on every rank and each rank computes only its own selected experts.
* KV cache: the context capacity is cut into super-chunks of 64 blocks x 256
  tokens (16,384 tokens) and rank r holds a contiguous range of them, so every
  super-chunk partial is computed whole on one rank and the final merge over
  super-chunks in order is the single-GPU merge, bit for bit.
* Dense weights, the embedding and the lm_head are replicated.

Reference: BASELINE configs 2 and 4 (split-KV with an LSE combine, experts
expert-parallel); the merge rule is megakernel.py:276-318.
"""
from __future__ import annotations

from dataclasses import dataclass

BLOCK_TOKENS = 256
SUPER_BLOCKS = 64
SUPER_TOKENS = BLOCK_TOKENS * SUPER_BLOCKS
MAX_WORLD = 8


def split_range(n: int, parts: int, i: int) -> tuple[int, int]:
    """Balanced contiguous split of [0, n) into `parts` ranges (the first
    n % parts ranges get one more element)."""
    q, r = divmod(n, parts)
    lo = i * q + min(i, r)
    return lo, lo + q + (1 if i < r else 0)


@dataclass(frozen=True)
class ShardPlan:
    world: int
    rank: int
    n_experts: int
    capacity: int     # global context capacity (tokens)
    expert_lo: int
    expert_hi: int
    super_lo: int
    super_hi: int

    @property
    def n_super(self) -> int:
        return -(-self.capacity // SUPER_TOKENS)

    @property
    def token_base(self) -> int:
        return self.super_lo * SUPER_TOKENS

    @property
    def token_end(self) -> int:
        return min(self.capacity, self.super_hi * SUPER_TOKENS)

    @property
    def local_capacity(self) -> int:
        """KV slots this rank allocates (at least one block, even when it
        holds no super-chunk)."""
        n = self.token_end - self.token_base
        return max(BLOCK_TOKENS, -(-n // BLOCK_TOKENS) * BLOCK_TOKENS) if n > 0 else BLOCK_TOKENS

    def owns_position(self, pos: int) -> bool:
        return self.token_base <= pos < self.token_end

    def owns_expert(self, e: int) -> bool:
        return self.expert_lo <= e < self.expert_hi


def plan(world: int, rank: int, n_experts: int, capacity: int) -> ShardPlan:
    if not 1 <= world <= MAX_WORLD:
        raise ValueError(f"world size must be 1..{MAX_WORLD}")
    if not 0 <= rank < world:
        raise ValueError("rank outside the world")
    if n_experts % world:
        raise ValueError("the expert count must divide evenly over the ranks")
    if capacity <= 0 or capacity % BLOCK_TOKENS:
        raise ValueError(f"capacity must be a positive multiple of {BLOCK_TOKENS}")
    per = n_experts // world
    n_super = -(-capacity // SUPER_TOKENS)
    s_lo, s_hi = split_range(n_super, world, rank)
    return ShardPlan(world, rank, n_experts, capacity, rank * per, (rank + 1) * per, s_lo, s_hi)


def owner_of_position(plans: list[ShardPlan], pos: int) -> int:
    for p in plans:
        if p.owns_position(pos):
            return p.rank
    raise ValueError(f"position {pos} outside the capacity")
