"""The synchronisation protocol of the quantized GEMM (`qlinear_kernel`,
mlx-lean-moe_b200/csrc/gdn_qlinear.cu), checked on the CPU as a
discrete-event model over random schedules.

Roles, as in the kernel:

- producer: per K-block kb, the x tile and the packed weights into stage
  kb % 3 (one barrier, Q_FULL), once stage kb - 3 is released by the MMA and
  by every dequantizing warp (Q_EMPTY: one commit plus one arrival per warp);
  with scales by TMA, a tile of scales (and biases) per 2^sshift K-blocks into
  one of two buffers, once every warp is done with the tile two before
  (Q_SCEMPTY, one arrival per warp);
- dequantizing warps, each on its own rows and at its own pace: for kb, the
  scales (Q_SCFULL at the tile's first K-block), the packed weights (Q_FULL)
  and the B buffer kb % 2 (Q_BEMPTY of kb - 2), then its rows of B, arriving
  on Q_BFULL, Q_EMPTY and, at a tile's last K-block, Q_SCEMPTY; after the
  loop, the epilogue reads the accumulators (Q_ACC) and stages the output
  over the x and weight rings;
- MMA issuer: per kb, after Q_FULL and Q_BFULL (every warp's rows), the
  product into the accumulators, committing Q_EMPTY and Q_BEMPTY; Q_ACC after
  the last.

Barriers count arrivals: a phase completes when its count is reached.  Every
arrival is checked to land in the phase it is meant for (a fast warp must not
count towards a slow warp's phase), every parity wait to find its barrier at
the awaited phase or one past it, and every buffer access to find the data it
needs with no copy or product in flight against it.  The model runs three
dequantizing warps (the kernel has sixteen; the protocol is the same for any
count of two or more).  A variant whose warps skip the wait for Q_BEMPTY is
checked to fail.
"""

from __future__ import annotations

import random

import pytest


class ProtocolError(AssertionError):
    pass


A_STAGES, B_STAGES = 3, 2


class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.done, self.arrived = name, count, 0, 0

    def arrive(self, phase):
        if phase != self.done:
            raise ProtocolError(f"arrival meant for phase {phase} of {self.name} at phase {self.done}")
        self.arrived += 1
        if self.arrived == self.count:
            self.arrived = 0
            self.done += 1


class QLinear:
    def __init__(self, nk, rng, warps=3, sshift=1, scale_tma=True, skip=None):
        self.nk, self.rng, self.warps, self.sshift, self.scale_tma = nk, rng, warps, sshift, scale_tma
        self.skip = skip or set()
        self.bar = {}
        for s in range(A_STAGES):
            self.bar[f"FULL{s}"] = Barrier(f"FULL{s}", 1)
            self.bar[f"EMPTY{s}"] = Barrier(f"EMPTY{s}", 1 + warps)
        for s in range(B_STAGES):
            self.bar[f"BFULL{s}"] = Barrier(f"BFULL{s}", warps)
            self.bar[f"BEMPTY{s}"] = Barrier(f"BEMPTY{s}", 1)
        for s in range(2):
            self.bar[f"SCFULL{s}"] = Barrier(f"SCFULL{s}", 1)
            self.bar[f"SCEMPTY{s}"] = Barrier(f"SCEMPTY{s}", warps)
        self.bar["ACC"] = Barrier("ACC", 1)
        self.tag, self.copies, self.pipe = {}, [], []
        self.roles = [self.producer(), self.issuer()] + [self.dequant(w) for w in range(warps)]
        self.pending = [None] * len(self.roles)
        self.finished = [False] * len(self.roles)

    # -- waits and accesses --------------------------------------------------
    def parity(self, name, phase):
        d = self.bar[name].done
        if not phase <= d <= phase + 1:
            raise ProtocolError(f"parity wait for phase {phase} of {name} at {d} completed phases")
        return (d & 1) != (phase & 1)

    def in_flight(self):
        for bufs, _, _, _ in self.copies:
            for b in bufs:
                yield b, "w"
        for op in self.pipe:
            if op[0] == "mma":
                for b in op[1]:
                    yield b, "r"
                yield "ACC", "w"

    def access(self, buffer, mode, what):
        for b, m in self.in_flight():
            if b == buffer and (mode == "w" or m == "w"):
                raise ProtocolError(f"{what}: {buffer} ({mode}) while in flight ({m})")

    def expect(self, buffer, tag, what):
        self.access(buffer, "r", what)
        if self.tag.get(buffer) != tag:
            raise ProtocolError(f"{what}: {buffer} holds {self.tag.get(buffer)}, not {tag}")

    def write(self, buffer, tag, what):
        self.access(buffer, "w", what)
        self.tag[buffer] = tag

    def copy(self, buffers, tag, barrier, phase):
        for b in buffers:
            self.access(b, "w", f"copy of {tag}")
            self.tag.pop(b, None)
        self.copies.append((buffers, tag, barrier, phase))

    def step_engines(self):
        if self.copies and (not self.pipe or self.rng.random() < 0.5):
            bufs, tag, bar, phase = self.copies.pop(self.rng.randrange(len(self.copies)))
            for b in bufs:
                self.tag[b] = tag
            self.bar[bar].arrive(phase)
        else:
            op = self.pipe.pop(0)
            if op[0] == "mma":
                self.tag["ACC"] = ("ACC", op[2])
            else:
                self.bar[op[1]].arrive(op[2])

    # -- roles ---------------------------------------------------------------
    def producer(self):
        for kb in range(self.nk):
            s = kb % A_STAGES
            if self.scale_tma and kb % (1 << self.sshift) == 0:
                tile = kb >> self.sshift
                if tile >= 2:
                    yield ("wait", f"SCEMPTY{tile & 1}", tile // 2 - 1)
                self.copy([f"SC{tile & 1}"], ("SC", tile), f"SCFULL{tile & 1}", tile // 2)
                yield None
            if kb >= A_STAGES:
                yield ("wait", f"EMPTY{s}", kb // A_STAGES - 1)
            self.copy([f"A{s}", f"W{s}"], ("AW", kb), f"FULL{s}", kb // A_STAGES)
            yield None

    def issuer(self):
        for kb in range(self.nk):
            s, sb = kb % A_STAGES, kb % B_STAGES
            yield ("wait", f"FULL{s}", kb // A_STAGES)
            yield ("wait", f"BFULL{sb}", kb // B_STAGES)
            self.expect(f"A{s}", ("AW", kb), f"MMA {kb}")
            for w in range(self.warps):
                self.expect(f"B{sb}.{w}", ("B", kb), f"MMA {kb}")
            self.pipe.append(("mma", [f"A{s}"] + [f"B{sb}.{w}" for w in range(self.warps)], kb))
            self.pipe.append(("commit", f"EMPTY{s}", kb // A_STAGES))
            self.pipe.append(("commit", f"BEMPTY{sb}", kb // B_STAGES))
            yield None
        self.pipe.append(("commit", "ACC", 0))

    def dequant(self, w):
        per_tile = 1 << self.sshift
        for kb in range(self.nk):
            s, sb = kb % A_STAGES, kb % B_STAGES
            tile, in_tile = kb >> self.sshift, kb % per_tile
            if self.scale_tma and in_tile == 0:
                yield ("wait", f"SCFULL{tile & 1}", tile // 2)
            yield ("wait", f"FULL{s}", kb // A_STAGES)
            if kb >= B_STAGES and "bempty" not in self.skip:
                yield ("wait", f"BEMPTY{sb}", kb // B_STAGES - 1)
            if self.scale_tma:
                self.expect(f"SC{tile & 1}", ("SC", tile), f"warp {w} scales of K-block {kb}")
            self.expect(f"W{s}", ("AW", kb), f"warp {w} weights of K-block {kb}")
            self.write(f"B{sb}.{w}", ("B", kb), f"warp {w} rows of B for K-block {kb}")
            self.bar[f"BFULL{sb}"].arrive(kb // B_STAGES)
            self.bar[f"EMPTY{s}"].arrive(kb // A_STAGES)
            if self.scale_tma and (in_tile == per_tile - 1 or kb == self.nk - 1):
                self.bar[f"SCEMPTY{tile & 1}"].arrive(tile // 2)
            yield None
        # epilogue: the accumulators, then the output staged over the x and weight rings
        yield ("wait", "ACC", 0)
        self.expect("ACC", ("ACC", self.nk - 1), f"warp {w} epilogue")
        for s in range(A_STAGES):
            self.access(f"A{s}", "w", f"warp {w} output staging")
            self.access(f"W{s}", "w", f"warp {w} output staging")

    # -- scheduler -----------------------------------------------------------
    def run(self, max_steps=100000):
        for _ in range(max_steps):
            if all(self.finished) and not (self.copies or self.pipe):
                return
            runnable = [r for r, w in enumerate(self.pending)
                        if not self.finished[r] and (w is None or self.parity(w[1], w[2]))]
            options = runnable + (["engine"] if (self.copies or self.pipe) else [])
            if not options:
                raise ProtocolError("deadlock: every role waits and nothing is in flight")
            pick = self.rng.choice(options)
            if pick == "engine":
                self.step_engines()
                continue
            try:
                self.pending[pick] = next(self.roles[pick])
            except StopIteration:
                self.finished[pick] = True
                self.pending[pick] = None
        raise ProtocolError("no progress within the step budget")


@pytest.mark.parametrize("scale_tma,sshift", [(False, 0), (True, 0), (True, 1), (True, 2)])
@pytest.mark.parametrize("nk", [1, 2, 3, 4, 7, 12])
def test_qlinear_pipeline_protocol_holds_over_random_schedules(nk, scale_tma, sshift):
    for seed in range(60):
        QLinear(nk, random.Random(seed * 131 + nk), sshift=sshift, scale_tma=scale_tma).run()


def test_the_model_flags_dequantizing_warps_that_skip_the_wait_for_b():
    flagged = 0
    for seed in range(300):
        try:
            QLinear(6, random.Random(seed), skip={"bempty"}).run()
        except ProtocolError:
            flagged += 1
    assert flagged > 0
