"""Prompt-prefix reuse across requests (reference engine/src/rec_mlx/prefix.py:10-118).

A `PromptCache` remembers the prompt tokens whose K/V a `KVStorage` holds,
the logits after the last of them, and checkpoints taken before each prefill
chunk.  `select_prefix` keeps the longest reusable part for a new prompt:
the whole cache when the new prompt extends it, else the latest checkpoint
at or below the common prefix (prefix.py:83-118).  The reference's
checkpoints also copy the sliding-window rings; here a sliding-window layer
keeps every row like the others and reads only its window, so no row is
ever overwritten by a later position, and a checkpoint is a position and
its logits.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass, field

from .errors import PrefillCancelled  # noqa: F401  (re-exported, as the reference's module does)


@dataclass
class LayerCache:
    """One layer's cache tensors (codes, scales and biases of K and V)."""

    tensors: dict

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors.values())


@dataclass
class Checkpoint:
    position: int
    logits: object


@dataclass
class PromptCache:
    tokens: list[int]
    storage: object
    logits: object | None = None
    checkpoints: list[Checkpoint] = field(default_factory=list)

    def fork(self) -> "PromptCache":
        """A copy of the bookkeeping over the same storage (prefix.py:29-38)."""
        return PromptCache(self.tokens[:], self.storage, self.logits, self.checkpoints[:])

    def advance(self, tokens, logits) -> None:
        previous = len(self.tokens)
        self.tokens.extend(int(t) for t in tokens)
        self.logits = logits
        if len(self.tokens) // 8192 != previous // 8192:
            logging.info("Prefill progress: %d tokens processed", len(self.tokens))

    def checkpoint(self) -> None:
        """Keeps the latest checkpoint and adds one at the current length
        (prefix.py:48-65)."""
        if not self.tokens:
            return
        self.checkpoints = self.checkpoints[-1:]
        self.checkpoints.append(Checkpoint(len(self.tokens), self.logits))

    @property
    def layers(self) -> list["LayerCache"]:
        """One view per layer of the cache the prompt's K/V sit in, each with
        its `nbytes` (the reference's per-layer caches, prefix.py:22-27,
        whose sliding layers' bytes engine.py:323-329 sums)."""
        return [LayerCache(tensors) for tensors in self.storage.cache.layers]

    @property
    def checkpoint_bytes(self) -> int:
        return sum(int(c.logits.numel() * c.logits.element_size()) for c in self.checkpoints if c.logits is not None)


def select_prefix(prefix: PromptCache | None, tokens):
    """(prefix or None, common prefix length) for a new prompt
    (prefix.py:83-118): a cache the prompt does not fully extend is rolled
    back to its latest checkpoint at or below the common prefix, or dropped
    when there is none."""
    common = 0
    if prefix is not None:
        for previous, current in zip(prefix.tokens, tokens):
            if previous != current:
                break
            common += 1
        if common != len(prefix.tokens):
            checkpoint = next((c for c in reversed(prefix.checkpoints) if c.position <= common), None)
            if checkpoint is None:
                prefix = None
            else:
                prefix.tokens = prefix.tokens[: checkpoint.position]
                prefix.logits = checkpoint.logits
                prefix.checkpoints = [c for c in prefix.checkpoints if c.position < checkpoint.position]
    cached = 0 if prefix is None else len(prefix.tokens)
    logging.info("Prefill: prompt=%d common_prefix=%d reused=%d new=%d", len(tokens), common, cached,
                 len(tokens) - cached)
    return prefix, common
