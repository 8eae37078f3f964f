"""Kept prefixes of prompts (crates/graph/src/prompt.rs:1-21, :352-420, :587-633): the keys and
values a prompt's leading positions left in its slot, copied out of the decoder's cache into
device memory, so that a later prompt that begins with the same positions copies them back into
its slot and runs only the rest. A position here is a row of input embedding (the backbone's
input), so a prefix is matched by the bits of its rows. The copy is exact and the prefill of the
rest reads exactly those keys and values, so a request that starts from a kept prefix comes out
bit for bit as it does from its whole prompt.

Within a byte budget, the least recently used prefixes are dropped first."""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np


@dataclasses.dataclass(eq=False)  # kept prefixes compare by identity
class Kept:
    bits: np.ndarray  # [count][hidden] uint32: the rows' bits
    mem: object       # device memory holding the prefix's keys and values
    bytes: int
    used: int


class PromptCache:
    def __init__(self, decoder, budget: int, alloc=None):
        """`alloc(bytes)` gives device memory for a prefix (the package's Memory on the decoder's
        context by default)."""
        self.decoder = decoder
        self.budget = budget
        self.alloc = alloc
        self.bytes = 0
        self.clock = 0
        self.kept: list[Kept] = []

    def _bits(self, rows: np.ndarray) -> np.ndarray:
        return np.ascontiguousarray(rows, dtype=np.float32).reshape(len(rows), -1).view(np.uint32)

    def shared(self, rows: np.ndarray) -> tuple[Optional[Kept], int]:
        """The kept prefix `rows` begins with the most positions of, and how many (at most
        len(rows) - 1: the last position always runs, its output being the next input)."""
        bits = self._bits(rows)
        best, n = None, 0
        for k in self.kept:
            m = min(len(k.bits), len(bits))
            same = np.all(k.bits[:m] == bits[:m], axis=1)
            s = m if same.all() else int(np.argmin(same))
            if s > n:
                best, n = k, s
        return best, min(n, len(rows) - 1)

    def restore(self, slot: int, rows: np.ndarray) -> int:
        """Copies the longest kept prefix of `rows` into `slot`; the positions it covers (0 for
        none), from which the prompt runs."""
        k, n = self.shared(rows)
        if k is None or n == 0:
            return 0
        self.clock += 1
        k.used = self.clock
        self.decoder.copy_in(slot, n, k.mem)
        return n

    def keep(self, slot: int, rows: np.ndarray) -> bool:
        """Keeps positions [0, len(rows)) of `slot` (written by the prompt `rows`) as a prefix,
        dropping the least recently used ones to make room; False when it cannot fit or is
        already kept."""
        bits = self._bits(rows)
        for k in self.kept:
            if len(k.bits) >= len(bits) and np.array_equal(k.bits[:len(bits)], bits):
                return False
        need = self.decoder.prefix_bytes(len(rows))
        if need > self.budget:
            return False
        while self.bytes + need > self.budget:
            old = min(self.kept, key=lambda k: k.used)
            self.kept.remove(old)
            self.bytes -= old.bytes
        if self.alloc is None:
            from . import Memory  # the package's device memory

            mem = Memory(self.decoder.ctx, need)
        else:
            mem = self.alloc(need)
        self.decoder.copy_out(slot, len(rows), mem)
        self.clock += 1
        self.kept.append(Kept(bits.copy(), mem, need, self.clock))
        self.bytes += need
        return True
