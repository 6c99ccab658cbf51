"""CPU model of the fused NVLink KV-slab exchange's protocol (aubier_b200/csrc/m4b_exchange.cu,
merge_exchange_wvb_kernel), run under random schedules.

Per exchange, every (head, column block) CTA of every GPU: reads its block's exchange count c from
its own memory; stores its record into slot [rank] of half (c + 1) & 1 of every GPU's receive buffer,
each value as one 8-byte word tagged with epoch c + 1; polls its own receive buffer until every
rank's word of that half carries epoch c + 1; merges; stores the count c + 1.  A GPU's next
exchange (the next kernel on its stream) starts only after all of its CTAs of this one have
finished.  Stores to another GPU land asynchronously and in any order.

Checked in every schedule: a poll never finds a word from a LATER exchange than the one it waits for
(that would mean a half was reused while a peer still needed it, and the poll would never end); the
values merged are the ones published for that exchange; every exchange finishes on every GPU.
The planted mistake -- one receive half instead of two -- must be caught.
"""
import random

import pytest


class ProtocolError(AssertionError):
    pass


class Exchange:
    def __init__(self, world, blocks, exchanges, rng, halves=2):
        self.G, self.B, self.E, self.rng, self.halves = world, blocks, exchanges, rng, halves
        # recv[g][half][r][b] = (epoch, value) as seen in GPU g's memory
        self.recv = [[[[(0, None)] * blocks for _ in range(world)] for _ in range(halves)]
                     for _ in range(world)]
        self.count = [[0] * blocks for _ in range(world)]
        self.stores = []                      # stores in flight: (g, half, r, b, epoch, value)
        self.kernel = [0] * world             # exchanges started on each GPU
        self.done_blocks = [0] * world        # CTAs of the current exchange finished
        self.ctas = {}                        # (g, b) -> generator of the running CTA
        self.merged = {}

    def value(self, r, b, e):
        return (r, b, e)                      # what rank r publishes for block b at exchange e

    def cta(self, g, b):
        c = self.count[g][b]
        e = c + 1
        half = e % self.halves
        for p in range(self.G):               # the record into slot [g] of every GPU
            self.stores.append((p, half, g, b, e, self.value(g, b, e)))
        yield
        got = {}
        while len(got) < self.G:               # poll the own buffer, all ranks' words at once
            for r in range(self.G):
                if r in got:
                    continue
                ep, v = self.recv[g][half][r][b]
                if ep > e:
                    raise ProtocolError(f"GPU {g} block {b} waits for exchange {e} but finds "
                                        f"rank {r}'s word of exchange {ep}")
                if ep == e:
                    if v != self.value(r, b, e):
                        raise ProtocolError("a word carries the epoch but not its value")
                    got[r] = v
            if len(got) < self.G:
                yield
        self.merged[(g, b, e)] = tuple(got[r] for r in range(self.G))
        self.count[g][b] = e

    def start_kernel(self, g):
        self.kernel[g] += 1
        self.done_blocks[g] = 0
        for b in range(self.B):
            self.ctas[(g, b)] = self.cta(g, b)

    def run(self, max_steps=500000):
        for g in range(self.G):
            self.start_kernel(g)
        for _ in range(max_steps):
            moves = [("cta", k) for k in self.ctas] + [("store", j) for j in range(len(self.stores))]
            if not moves:
                break
            kind, x = self.rng.choice(moves)
            if kind == "store":
                p, half, r, b, ep, v = self.stores.pop(x)
                self.recv[p][half][r][b] = (ep, v)
                continue
            try:
                next(self.ctas[x])
            except StopIteration:
                del self.ctas[x]
                g = x[0]
                self.done_blocks[g] += 1
                if self.done_blocks[g] == self.B and self.kernel[g] < self.E:
                    self.start_kernel(g)       # the next kernel on this GPU's stream
        else:
            raise ProtocolError("deadlock: polls never see their records")
        for g in range(self.G):
            for b in range(self.B):
                if self.count[g][b] != self.E:
                    raise ProtocolError(f"GPU {g} block {b} finished {self.count[g][b]} exchanges")
                for e in range(1, self.E + 1):
                    want = tuple(self.value(r, b, e) for r in range(self.G))
                    if self.merged[(g, b, e)] != want:
                        raise ProtocolError("merged the wrong exchange's records")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_protocol_holds_under_random_schedules(world):
    rng = random.Random(100 + world)
    for blocks in (1, 2, 4):
        for _ in range(60):
            Exchange(world, blocks, 7, rng).run()


def test_planted_single_receive_half_is_caught():
    rng = random.Random(9)
    caught = 0
    for _ in range(200):
        try:
            Exchange(2, 2, 6, rng, halves=1).run()
        except ProtocolError:
            caught += 1
    assert caught > 0
