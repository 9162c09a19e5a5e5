"""Host-side model checker of the cross-GPU synchronisation protocol of csrc/fused_ar.cu.

The reference argued the correctness of its barrier-free all-gather in prose
(docs/method_design.md:37-67: Q1 arrival via flag, Q2 no overwrite by epoch parity, Q3 stale data
rejected by epoch) and tested it with one interleaving test (exp/M16_epoch_fix/test_interleave.py).
Here the protocol itself is executed step by step by simulated ranks under random and adversarial
schedules, with the invariants checked on every memory operation:

* a sender never overwrites a landing cell that still holds unconsumed data (no lost update),
* a receiver only accepts data of its own call (no stale read),
* a staged input is never overwritten while a peer may still read it for an older call,
* every rank finishes every call (no deadlock), with different grid sizes per call and any mix of
  variants (one CUDA graph per batch size, replayed in any order).

The NVSwitch multicast variants are modelled with their multicast barriers (one add into every rank's
counter per block, a wait for world x calls on the local copy) and, for the two-shot form, the
multicast store of h into every rank's buffer, which must not overwrite a slice a rank has not read.
The layer-boundary pair of csrc/fused_gemm.cu is modelled as one call of two kernels per rank
(variant FG): the push GEMM's CTAs store column groups of every row into land1 of every rank (its
own included) under the call's epoch without advancing it; after that kernel completes, the consumer
GEMM's CTAs each take one piece of columns from all sources (clearing the cells), stage it, publish a
flag tagged with the epoch, and the CTAs of a split wait for all pieces of their split (and, for the
row norms, of every split) before reading the staged activation; the epoch advances when the
consumer kernel completes.

Each simulated memory cell stores (epoch, payload) or FILL, standing for the Lamport -0 sentinel.
The unit of interleaving is one memory operation; blocks of one rank are modelled for the
barrier-based variants because their barriers are per block.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field

FILL = None

L1S, L2S, P1S, P2S = 1, 2, 5, 6
NV1S, NV2S = 3, 4  # NVSwitch multicast: stage + multicast barrier, in-switch reduce (+ multicast store)
L1SX = 7  # one-shot push whose landing cells get their sentinel back only after the row is finished
FG = 100  # gemm_push + ar_norm_gemm (layer-boundary fusion)
FG_COLS = 12  # modelled column groups of the pushed rows


class ProtocolViolation(AssertionError):
    pass


@dataclass
class Call:
    variant: int
    blocks: int
    rows: int
    splits: int = 1  # FG: split-K count of the consumer (its CTAs = blocks x splits pieces)


@dataclass
class Memory:
    world: int
    nslots: int = 2  # landing slots by epoch parity (1 = a deliberately broken protocol)
    land1: dict = field(default_factory=dict)   # (owner, slot, src, row) -> (epoch, value) | FILL
    rs: dict = field(default_factory=dict)      # (owner, slot, src, row)
    ag: dict = field(default_factory=dict)      # (owner, slot, src, row)
    agp: dict = field(default_factory=dict)     # (owner, slot, src, row) -> epoch tag (never cleared)
    stage: dict = field(default_factory=dict)   # (owner, parity, row) -> epoch
    flags: dict = field(default_factory=dict)   # (owner, block, src) -> count
    fg_land: dict = field(default_factory=dict)  # (owner, slot, src, row, col) -> (epoch, value) | FILL
    act: dict = field(default_factory=dict)      # (owner, col) -> epoch of the staged activation
    pflags: dict = field(default_factory=dict)   # (owner, piece) -> epoch tag
    nvcnt: dict = field(default_factory=dict)    # (owner, block, k) -> multicast barrier counter
    hbuf: dict = field(default_factory=dict)     # (owner, row, slice) -> (epoch, value) | FILL (multicast h)


def value(rank: int, epoch: int, row: int) -> int:
    """Distinct payload per (sender, call, row): a stale or foreign value never matches."""
    return (epoch * 1000003 + rank * 7919 + row) & 0xFFFFFFFF


class Rank:
    """One simulated GPU: a generator of steps; a step returns False while it must wait."""

    def __init__(self, rank: int, mem: Memory, calls: list[Call], seed: int = 0):
        self.rank, self.mem, self.calls = rank, mem, calls
        self.rng = random.Random(seed * 131 + rank)
        self.epoch = 0
        self.flag_calls: dict[int, int] = {}
        self.nv_calls: dict[tuple, int] = {}
        self.done = False
        self.gen = self._run()
        self.results: list[dict] = []

    # ---- helpers -------------------------------------------------------------------------
    def _put(self, table: dict, key, val):
        if table.get(key, FILL) is not FILL:
            raise ProtocolViolation(f"rank {self.rank} overwrites unconsumed cell {key}: {table[key]}")
        table[key] = val

    def _peek(self, table: dict, key, epoch: int):
        """Read a landing cell without giving it back (the restore comes later in the same call)."""
        v = table.get(key, FILL)
        if v is FILL:
            return None
        if v[0] != epoch:
            raise ProtocolViolation(f"rank {self.rank} call {epoch} reads stale cell {key}: {v}")
        return v

    def _restore(self, table: dict, key, epoch: int):
        v = table.get(key, FILL)
        if v is FILL or v[0] != epoch:
            raise ProtocolViolation(f"rank {self.rank} call {epoch} restores cell {key} holding {v}")
        table[key] = FILL

    def _take(self, table: dict, key, epoch: int):
        v = table.get(key, FILL)
        if v is FILL:
            return None
        if v[0] != epoch:
            raise ProtocolViolation(f"rank {self.rank} call {epoch} reads stale cell {key}: {v}")
        table[key] = FILL
        return v

    # ---- the protocol ---------------------------------------------------------------------
    def _run(self):
        for call in self.calls:
            e = self.epoch + 1  # every block reads the same epoch; the last block advances it
            got: dict = {}
            blocks = [] if call.variant == FG else [self._block(call, e, b, got) for b in range(call.blocks)]
            live = list(blocks)
            while live:
                g = self.rng.choice(live)
                try:
                    yield next(g)
                except StopIteration:
                    live.remove(g)
            if call.variant == FG:
                yield from self._fused_boundary(call, e, got)
            expect = call.rows * self.mem.world * (FG_COLS if call.variant == FG else 1)
            if len(got) != expect:
                raise ProtocolViolation(f"rank {self.rank} call {e}: {len(got)} of {expect} row pieces")
            for key, v in got.items():
                src, row = key[0], key[1]
                if v != value(src, e, row * FG_COLS + (key[2] if len(key) > 2 else 0) if call.variant == FG
                              else row):
                    raise ProtocolViolation(f"rank {self.rank} call {e}: wrong payload from {src} row {row}")
            self.results.append(dict(epoch=e, n=len(got)))
            self.epoch = e
            yield True
        self.done = True

    def _block(self, call: Call, e: int, b: int, got: dict):
        """One CTA of this rank: rows b, b + blocks, ... (all phases use the same rows)."""
        W = self.mem.world
        slot = e % self.mem.nslots
        rows = range(b, call.rows, call.blocks)
        if call.variant == L1S:
            for row in rows:
                for i in range(1, W):
                    self._put(self.mem.land1, ((self.rank + i) % W, slot, self.rank, row),
                              (e, value(self.rank, e, row)))
                    yield True
            for row in rows:
                for src in range(W):
                    if src == self.rank:
                        got[(src, row)] = value(src, e, row)
                        continue
                    while (v := self._take(self.mem.land1, (self.rank, slot, src, row), e)) is None:
                        yield False
                    got[(src, row)] = v[1]
                    yield True
        elif call.variant == L1SX:
            for row in rows:
                for i in range(1, W):
                    self._put(self.mem.land1, ((self.rank + i) % W, slot, self.rank, row),
                              (e, value(self.rank, e, row)))
                    yield True
            for row in rows:
                for src in range(W):
                    if src == self.rank:
                        got[(src, row)] = value(src, e, row)
                        continue
                    while (v := self._peek(self.mem.land1, (self.rank, slot, src, row), e)) is None:
                        yield False
                    got[(src, row)] = v[1]
                    yield True
                yield True  # the row sum, the outputs; then the row's cells get their sentinel back
                for src in range(W):
                    if src != self.rank:
                        self._restore(self.mem.land1, (self.rank, slot, src, row), e)
                        yield True
        elif call.variant in (L2S, P2S):
            if call.variant == L2S:
                for row in rows:
                    for dst in range(W):
                        if dst != self.rank:
                            self._put(self.mem.rs, (dst, slot, self.rank, row), (e, value(self.rank, e, row)))
                            yield True
            else:
                yield from self._stage_and_barrier(e, b, rows)
            for row in rows:
                for src in range(W):
                    if src == self.rank:
                        continue
                    if call.variant == L2S:
                        while self._take(self.mem.rs, (self.rank, slot, src, row), e) is None:
                            yield False
                    else:
                        self._read_stage(src, e, row)
                    yield True
                for dst in range(W):
                    self._put(self.mem.ag, (dst, slot, self.rank, row), (e, value(self.rank, e, row)))
                    self.mem.agp[(dst, slot, self.rank, row)] = e
                    yield True
            for row in rows:
                for src in range(W):
                    while (v := self._take(self.mem.ag, (self.rank, slot, src, row), e)) is None:
                        yield False
                    while self.mem.agp.get((self.rank, slot, src, row)) != e:
                        yield False
                    got[(src, row)] = v[1]
                    yield True
        elif call.variant == P1S:
            yield from self._stage_and_barrier(e, b, rows)
            for row in rows:
                for src in range(W):
                    self._read_stage(src, e, row)
                    got[(src, row)] = value(src, e, row)
                    yield True
        elif call.variant == NV1S:
            yield from self._stage_and_nv_barrier(e, b, rows, 0)
            for row in rows:  # multimem.ld_reduce: every rank's staged row, summed in the switch
                for src in range(W):
                    self._read_stage(src, e, row)
                    got[(src, row)] = value(src, e, row)
                yield True
        elif call.variant == NV2S:
            yield from self._stage_and_nv_barrier(e, b, rows, 0)
            for row in rows:  # owned slice: reduce in the switch, multicast-store h to every rank
                for src in range(W):
                    self._read_stage(src, e, row)
                for owner in range(W):
                    self._put(self.mem.hbuf, (owner, row, self.rank), (e, value(self.rank, e, row)))
                yield True
            yield from self._nv_barrier(b, 1)
            for row in rows:
                for sl in range(W):
                    v = self._take(self.mem.hbuf, (self.rank, row, sl), e)
                    if v is None:
                        raise ProtocolViolation(f"rank {self.rank} call {e}: h slice {sl} of row {row} missing "
                                                "after the second barrier")
                    got[(sl, row)] = v[1]
                    yield True
        else:
            raise ValueError(call.variant)

    def _interleave(self, gens):
        live = list(gens)
        while live:
            g = self.rng.choice(live)
            try:
                yield next(g)
            except StopIteration:
                live.remove(g)

    def _fused_boundary(self, call: Call, e: int, got: dict):
        """gemm_push (call.blocks CTAs) then, after it completes, ar_norm_gemm (blocks x splits CTAs)."""
        W, slot, C = self.mem.world, e % self.mem.nslots, FG_COLS

        def push(b):
            for row in range(call.rows):
                for col in range(b, C, call.blocks):
                    for i in range(W):  # own heap first, then the peers
                        self._put(self.mem.fg_land, ((self.rank + i) % W, slot, self.rank, row, col),
                                  (e, value(self.rank, e, row * C + col)))
                        yield True

        yield from self._interleave(push(b) for b in range(call.blocks))
        tiles, S = call.blocks, call.splits
        span = [(r * C // S, (r + 1) * C // S) for r in range(S)]

        def consumer(t, r):
            c0, c1 = span[r]
            lo, hi = c0 + (c1 - c0) * t // tiles, c0 + (c1 - c0) * (t + 1) // tiles
            for row in range(call.rows):  # this CTA's piece: columns [lo, hi) of every row
                for col in range(lo, hi):
                    for src in range(W):
                        while (v := self._take(self.mem.fg_land, (self.rank, slot, src, row, col), e)) is None:
                            yield False
                        got[(src, row, col)] = v[1]
                        yield True
            for col in range(lo, hi):
                self.mem.act[(self.rank, col)] = e
                yield True
            self.mem.pflags[(self.rank, r * tiles + t)] = e
            yield True
            # TMA producer of split r: all pieces of the split, then the staged activation
            for tt in range(tiles):
                while self.mem.pflags.get((self.rank, r * tiles + tt)) != e:
                    yield False
            for col in range(c0, c1):
                if self.mem.act.get((self.rank, col)) != e:
                    raise ProtocolViolation(f"rank {self.rank} call {e} split {r} reads activation col {col} "
                                            f"of call {self.mem.act.get((self.rank, col))}")
                yield True

        yield from self._interleave(consumer(t, r) for t in range(tiles) for r in range(S))

    def _stage_and_barrier(self, e: int, b: int, rows):
        """Copy this block's rows into stage[parity], then block b's flag barrier."""
        W = self.mem.world
        for row in rows:
            self.mem.stage[(self.rank, e % self.mem.nslots, row)] = e
            yield True
        bc = self.flag_calls.get(b, 0) + 1
        self.flag_calls[b] = bc
        for peer in range(W):
            self.mem.flags[(peer, b, self.rank)] = bc
            yield True
        for peer in range(W):
            while self.mem.flags.get((self.rank, b, peer), 0) < bc:
                yield False

    def _nv_barrier(self, b: int, k: int):
        """Multicast barrier k of block b: one add to every rank's counter, wait for world x calls locally."""
        W = self.mem.world
        calls = self.nv_calls.get((b, k), 0) + 1
        self.nv_calls[(b, k)] = calls
        for owner in range(W):  # multimem.red: the switch adds to every rank's copy
            self.mem.nvcnt[(owner, b, k)] = self.mem.nvcnt.get((owner, b, k), 0) + 1
        yield True
        while self.mem.nvcnt.get((self.rank, b, k), 0) < calls * W:
            yield False

    def _stage_and_nv_barrier(self, e: int, b: int, rows, k: int):
        for row in rows:
            self.mem.stage[(self.rank, e % self.mem.nslots, row)] = e
            yield True
        yield from self._nv_barrier(b, k)

    def _read_stage(self, src: int, e: int, row: int):
        got = self.mem.stage.get((src, e % self.mem.nslots, row))
        if got != e:
            raise ProtocolViolation(f"rank {self.rank} call {e} reads stage of {src} row {row} holding call {got}")

    def step(self) -> bool:
        if self.done:
            return False
        try:
            return next(self.gen)
        except StopIteration:
            self.done = True
            return True


def simulate(world: int, calls: list[Call], seed: int = 0, max_steps: int = 2_000_000,
             slow_rank: int | None = None, slow_factor: int = 20, nslots: int = 2) -> dict:
    """Run all ranks under a random schedule. `slow_rank` is scheduled `slow_factor` times less often."""
    mem = Memory(world, nslots)
    ranks = [Rank(r, mem, calls, seed) for r in range(world)]
    rng = random.Random(seed)
    weights = [1.0 if r != slow_rank else 1.0 / slow_factor for r in range(world)]
    steps = 0
    idle = 0
    while not all(r.done for r in ranks):
        live = [r for r in ranks if not r.done]
        r = rng.choices(live, weights=[weights[x.rank] for x in live])[0]
        progressed = r.step()
        idle = 0 if progressed else idle + 1
        steps += 1
        if idle > 50 * world * world + 1000:
            raise ProtocolViolation(f"deadlock: epochs {[x.epoch for x in ranks]}")
        if steps > max_steps:
            raise ProtocolViolation("step budget exhausted")
    leftovers = [k for t in (mem.land1, mem.rs, mem.ag, mem.fg_land, mem.hbuf) for k, v in t.items() if v is not FILL]
    if leftovers:
        raise ProtocolViolation(f"landing cells not restored to the sentinel: {leftovers[:4]}")
    return dict(steps=steps, epochs=[r.epoch for r in ranks])


def random_calls(n: int, seed: int, variants=(L1S, L2S, P1S, P2S, L1SX), rows=(1, 3, 8), blocks=(1, 2, 4),
                 splits=(1, 2, 3)) -> list[Call]:
    rng = random.Random(seed)
    return [Call(rng.choice(variants), rng.choice(blocks), rng.choice(rows), rng.choice(splits)) for _ in range(n)]


# ---------------------------------------------------------------------------------------------------
# Row sums across a thread-block cluster without a release-ordered barrier (csrc/fused_ar.cu,
# row_sum_xch): C CTAs each own one word slot per row parity in their shared memory. For row `it` a
# CTA stores (tag it + 1, its partial) into its own slot it % 2, then polls every peer's slot it % 2
# until the tag matches and adds the C partials in CTA order. The words start at tag 0 (cleared before
# a barrier that every CTA passes before its first poll). The model checks, under random schedules and
# slow CTAs, that a CTA never overwrites a slot that a peer has not yet read for the older row, that
# every read returns the partial of the right CTA and row, and that all CTAs compute the same sums.


def cluster_partial(cta: int, it: int) -> int:
    return cta * 1000 + it


def simulate_cluster_exchange(C: int, rows: int, seed: int = 0, slow: int | None = None, slow_factor: int = 20,
                              nslots: int = 2, max_steps: int = 1_000_000) -> dict:
    rng = random.Random(seed)
    words = {(c, s): (0, None) for c in range(C) for s in range(nslots)}   # (cta, slot) -> (tag, value)
    read_upto = {(r, c): -1 for r in range(C) for c in range(C)}          # last row r read from c
    sums: dict[int, list[int]] = {r: [] for r in range(C)}

    def cta(r: int):
        for it in range(rows):
            slot = it % nslots
            for peer in range(C):  # overwriting slot it % 2 needs every peer done with row it - nslots
                if peer != r and it - nslots >= 0 and read_upto[(peer, r)] < it - nslots:
                    raise ProtocolViolation(f"CTA {r} overwrites row {it - nslots} in slot {slot} before CTA {peer} "
                                            f"read it")
            words[(r, slot)] = (it + 1, cluster_partial(r, it))
            yield True
            vals = []
            for c in range(C):
                if c == r:
                    vals.append(cluster_partial(r, it))
                    continue
                while (w := words[(c, slot)])[0] != it + 1:
                    yield False
                if w[1] != cluster_partial(c, it):
                    raise ProtocolViolation(f"CTA {r} row {it} read {w} from CTA {c}")
                read_upto[(r, c)] = it
                vals.append(w[1])
                yield True
            sums[r].append(sum(vals))

    gens = {r: cta(r) for r in range(C)}
    weights = {r: (1.0 / slow_factor if r == slow else 1.0) for r in range(C)}
    steps = idle = 0
    while gens:
        live = list(gens)
        r = rng.choices(live, weights=[weights[x] for x in live])[0]
        try:
            progressed = next(gens[r])
        except StopIteration:
            del gens[r]
            progressed = True
        idle = 0 if progressed else idle + 1
        steps += 1
        if idle > 100 * C * C + 1000:
            raise ProtocolViolation("deadlock in the cluster exchange")
        if steps > max_steps:
            raise ProtocolViolation("step budget exhausted")
    if any(sums[r] != sums[0] for r in range(C)):
        raise ProtocolViolation("CTAs disagree on the row sums")
    return dict(steps=steps, sums=sums[0])
