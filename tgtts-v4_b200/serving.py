"""Synthetic request streams for the serving configurations, and the loop that drives a Server
with them (the generator's admit-between-steps pattern, crates/graph/src/generator.rs:189-352).

Config 3: `slots` requests at once, contexts uniform in [64, 2048] (seed 2), each finishing after a
uniform 32-512 steps and replaced by a request with a fresh 128-position prompt.
Config 5: requests with prompts uniform in [64, 1024] and decodes uniform in [64, 768] (seed 3),
Poisson arrivals, spread over the GPUs by a least-loaded rule every rank computes alike.

Prompts are rows of one seeded N(0, 1) pool (bf16-valued), at seeded offsets: the same stream on
every run, with no generation inside a timed loop.
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np


@dataclasses.dataclass
class Req:
    id: int
    len: int
    steps: int
    offset: int  # first row of its prompt in the pool
    arrival: float = 0.0


class Pool:
    """Seeded N(0, 1) rows (rounded to bf16 values) that prompts are cut from."""

    def __init__(self, hidden: int, rows: int, seed: int):
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((rows, hidden), dtype=np.float32)
        u = x.view(np.uint32).astype(np.uint64)
        self.rows = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)

    def prompt(self, r: Req) -> np.ndarray:
        return self.rows[r.offset:r.offset + r.len]


class ContinuousStream:
    """Config 3's stream: the first `slots` requests with contexts in `ctx`, then refills of
    `refill` positions; lifetimes in `life` (inclusive bounds)."""

    def __init__(self, hidden: int, slots: int = 64, seed: int = 2, ctx=(64, 2048), life=(32, 512),
                 refill: int = 128):
        self.rng = np.random.default_rng(seed)
        self.slots, self.ctx, self.life, self.refill = slots, ctx, life, refill
        self.pool = Pool(hidden, ctx[1] + 256, seed + 100)
        self.next_id = 0

    def _req(self, n: int) -> Req:
        r = Req(self.next_id, n, int(self.rng.integers(self.life[0], self.life[1] + 1)),
                int(self.rng.integers(0, self.pool.rows.shape[0] - n + 1)))
        self.next_id += 1
        return r

    def initial(self) -> list[Req]:
        return [self._req(int(self.rng.integers(self.ctx[0], self.ctx[1] + 1))) for _ in range(self.slots)]

    def replacement(self) -> Req:
        return self._req(self.refill)


def poisson_requests(n: int, hidden: int, seed: int = 3, prompt=(64, 1024), decode=(64, 768),
                     rate: float = 4096.0) -> tuple[list[Req], Pool]:
    """Config 5's requests: prompt and decode lengths uniform (inclusive), arrivals a Poisson
    process of `rate` requests per second from t = 0."""
    rng = np.random.default_rng(seed)
    pool = Pool(hidden, prompt[1] + 256, seed + 100)
    t = np.cumsum(rng.exponential(1.0 / rate, n))
    out = []
    for i in range(n):
        ln = int(rng.integers(prompt[0], prompt[1] + 1))
        out.append(Req(i, ln, int(rng.integers(decode[0], decode[1] + 1)),
                       int(rng.integers(0, pool.rows.shape[0] - ln + 1)), float(t[i])))
    return out, pool


def assign_least_loaded(reqs: list[Req], gpus: int) -> list[list[Req]]:
    """Each arrival, in order, to the GPU with the least work assigned so far (prompt + decode
    positions), ties to the lower index: the same split on every rank without a message."""
    load = [0] * gpus
    out: list[list[Req]] = [[] for _ in range(gpus)]
    for r in reqs:
        g = min(range(gpus), key=lambda i: (load[i], i))
        out[g].append(r)
        load[g] += r.len + r.steps
    return out


class Driver:
    """Runs a Server over a request source: admits waiting requests into free slots between steps
    (all admissions of a step in one start), steps every request under way, and frees finished
    slots. Keeps the host's own count of each slot's steps left, so a step needs no query."""

    def __init__(self, server, pool: Pool, slots: int):
        self.server, self.pool, self.slots = server, pool, slots
        self.owner: dict[int, Req] = {}
        self.left: dict[int, int] = {}
        self.outputs: dict[int, list[np.ndarray]] = {}
        self.decoded = 0
        self.prefilled = 0
        self.steps = 0

    def free_slots(self) -> list[int]:
        return [s for s in range(self.slots) if s not in self.owner]

    def admit(self, reqs: list[Req]) -> None:
        if not reqs:
            return
        free = self.free_slots()
        assert len(reqs) <= len(free)
        plan = []
        for r, s in zip(reqs, free):
            self.owner[s] = r
            self.left[s] = r.steps
            plan.append((s, r.len, r.steps))
            self.prefilled += r.len
        self.server.start(plan, np.concatenate([self.pool.prompt(r) for r in reqs]))

    def step(self, read: bool = False, keep: Optional[set] = None) -> list[Req]:
        """One step; returns the requests that finished with it. With `read`, keeps the outputs of
        the requests in `keep` (all when None) in `outputs` by request id."""
        slots, out = self.server.step(read=read)
        self.steps += 1
        self.decoded += len(slots)
        done = []
        for i, s in enumerate(slots):
            r = self.owner[s]
            if read and (keep is None or r.id in keep):
                self.outputs.setdefault(r.id, []).append(out[i].copy())
            self.left[s] -= 1
            if self.left[s] == 0:
                done.append(r)
        for r in done:
            s = next(k for k, v in self.owner.items() if v is r)
            self.server.finish(s)
            del self.owner[s]
            del self.left[s]
        return done
