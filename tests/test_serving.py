"""The serving workloads' host logic on the CPU: seeded request streams, the least-loaded split
over GPUs that every rank computes alike, the driver's admit/step/finish loop against a fake
server, and the split and max-over-ranks timing across two gloo ranks."""

import os
import socket

import numpy as np
import torch.multiprocessing as mp

import __graft_entry__ as entry

entry.load_package()  # as tgtts_v4_b200, also in the spawned ranks, which import this module
from tgtts_v4_b200 import serving  # noqa: E402


def test_streams_are_seeded_and_within_their_bounds():
    a, pool_a = serving.poisson_requests(300, 64, seed=3)
    b, _ = serving.poisson_requests(300, 64, seed=3)
    assert [(r.len, r.steps, r.offset, r.arrival) for r in a] == [(r.len, r.steps, r.offset, r.arrival) for r in b]
    assert all(64 <= r.len <= 1024 and 64 <= r.steps <= 768 for r in a)
    assert all(r.offset + r.len <= pool_a.rows.shape[0] for r in a)
    arrivals = np.array([r.arrival for r in a])
    assert np.all(np.diff(arrivals) >= 0)
    # bf16-valued rows: the low 16 bits are zero.
    assert np.all(pool_a.rows.view(np.uint32) & 0xFFFF == 0)
    c3 = serving.ContinuousStream(64, slots=8)
    first = c3.initial()
    assert len(first) == 8 and all(64 <= r.len <= 2048 and 32 <= r.steps <= 512 for r in first)
    assert c3.replacement().len == 128


def test_least_loaded_split_covers_every_request_once_and_balances():
    reqs, _ = serving.poisson_requests(2048, 16, seed=3)
    for gpus in (1, 2, 4, 8):
        parts = serving.assign_least_loaded(reqs, gpus)
        ids = sorted(r.id for p in parts for r in p)
        assert ids == list(range(2048))
        loads = [sum(r.len + r.steps for r in p) for p in parts]
        assert max(loads) - min(loads) <= 1024 + 768  # within one request's work


class FakeServer:
    """Records what the driver asks of a server; each step runs every held request with steps left."""

    def __init__(self, slots, hidden):
        self.slots, self.hidden = slots, hidden
        self.held = {}  # slot -> steps left
        self.started = []

    def start(self, plan, x):
        assert x.shape == (sum(n for _, n, _ in plan), self.hidden)
        for slot, n, steps in plan:
            assert slot not in self.held
            self.held[slot] = steps
        self.started.append(plan)

    def step(self, read=False):
        slots = sorted(s for s, left in self.held.items() if left > 0)
        for s in slots:
            self.held[s] -= 1
        out = np.tile(np.array(slots, np.float32)[:, None], (1, self.hidden)) if read else None
        return slots, out

    def finish(self, slot):
        del self.held[slot]


def test_driver_admits_into_free_slots_and_frees_finished_ones():
    stream = serving.ContinuousStream(16, slots=4, seed=2, ctx=(4, 20), life=(1, 5), refill=3)
    fake = FakeServer(4, 16)
    drv = serving.Driver(fake, stream.pool, 4)
    drv.admit(stream.initial())
    assert sorted(drv.owner) == [0, 1, 2, 3]
    finished = []
    for _ in range(30):
        done = drv.step(read=True)
        finished += done
        drv.admit([stream.replacement() for _ in done])
        assert len(drv.owner) == 4
    # Every finished request ran exactly its steps, and its outputs were kept.
    for r in finished:
        assert len(drv.outputs[r.id]) == r.steps
    assert drv.decoded == sum(len(v) for v in drv.outputs.values())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    reqs, _ = serving.poisson_requests(512, 16, seed=3)
    mine = serving.assign_least_loaded(reqs, world)[rank]
    ids = torch.zeros(512, dtype=torch.int64)
    ids[[r.id for r in mine]] = 1
    dist.all_reduce(ids)
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    q.put((rank, ids.tolist(), float(t.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_split_the_requests_and_take_the_max_time():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ids, tmax in got:
        assert ids == [1] * 512  # every request on exactly one rank
        assert tmax == 2.0


class FakeDecoder:
    """A decoder's prefix copies recorded on the host: bytes per position, and what went where."""

    def __init__(self, per_position=100):
        self.per = per_position
        self.ops = []

    def prefix_bytes(self, n):
        return n * self.per

    def copy_out(self, slot, n, mem):
        self.ops.append(("out", slot, n, mem))

    def copy_in(self, slot, n, mem):
        self.ops.append(("in", slot, n, mem))


def test_prompt_cache_matches_the_longest_prefix_and_keeps_to_its_budget():
    from tgtts_v4_b200.prompt_cache import PromptCache

    dec = FakeDecoder()
    cache = PromptCache(dec, budget=100 * 50, alloc=lambda n: ("mem", n))
    rng = np.random.default_rng(1)
    a = rng.standard_normal((30, 4), dtype=np.float32)
    assert cache.keep(0, a[:20]) and cache.bytes == 2000
    assert not cache.keep(0, a[:10])  # a prefix of a kept one
    assert cache.keep(1, a)  # a longer one
    k, n = cache.shared(np.concatenate([a[:25], rng.standard_normal((5, 4), dtype=np.float32)]))
    assert n == 25 and len(k.bits) == 30
    assert cache.shared(a[:12])[1] == 11  # the last position always runs
    assert cache.restore(3, a[:12]) == 11 and dec.ops[-1][:3] == ("in", 3, 11)
    assert cache.shared(rng.standard_normal((8, 4), dtype=np.float32))[1] == 0
    # Past the budget the least recently used goes: the restore above used a[:20] (the first of
    # the two that share 12 rows with it), so the whole of a, kept before it, goes.
    b = rng.standard_normal((10, 4), dtype=np.float32)
    assert cache.keep(2, b) and cache.bytes <= cache.budget
    assert [len(k.bits) for k in cache.kept] == [20, 10]
    assert not cache.keep(0, rng.standard_normal((60, 4), dtype=np.float32))  # larger than the budget
