"""The synchronisation protocol of the tcgen05 attention prefill
(`attn_tc_kernel`, mlx-lean-moe_b200/csrc/gdn_attention.cu), checked on the CPU
as a discrete-event model over random schedules.

Roles, as in the kernel (the two softmax warp groups meet at named barriers,
so they act as one role here):

- producer: Q once, then K_i and V_(i-1) in that order; a K (V) buffer is
  refilled once S (P V) of the tile two before has completed (K_EMPTY,
  V_EMPTY);
- MMA issuer: S_j = Q K_j^T into S buffer j % 2, then O += P_(j-1) V_(j-1);
  commits S_FULL, K_EMPTY after S and PV_DONE, V_EMPTY (and O_FULL after the
  last one) after P V;
- softmax: at head_dim 256 first copies Q into TMEM (after Q_FULL; then
  QT_READY, which the issuer waits for instead of Q_FULL); waits S_FULL, may rescale O (waits for the product of the tile
  before on PV_DONE), writes P over its S buffer, arrives P_READY; at the end
  waits O_FULL and reads O.

The asynchronous engines: TMA copies land in any order at random times;
tensor-core products run in issue order, and a commit arrives once every
product issued before it is done.  A wait is an mbarrier parity wait: it
passes when the barrier's completed-phase count differs in parity from the
awaited phase.  Such a wait is only sound while the count is the awaited
phase or one past it, so every evaluation checks that, and every buffer
access checks that no copy or product still reads or writes it.

A variant with the final wait for O on PV_DONE by parity (how the kernel
first waited) is checked to fail: with the softmax fast enough, the product of
the second-last tile can still be pending there.
"""

from __future__ import annotations

import random

import pytest


class ProtocolError(AssertionError):
    pass


class Barrier:
    def __init__(self, name):
        self.name = name
        self.done = 0  # completed phases

    def complete(self):
        self.done += 1


class Model:
    def __init__(self, ntiles, rng, final_on_pv_done=False, q_in_tmem=False):
        self.ntiles, self.rng, self.final_on_pv_done, self.q_in_tmem = ntiles, rng, final_on_pv_done, q_in_tmem
        names = ["Q_FULL", "QT_READY", "PV_DONE", "O_FULL"] + [f"{n}{b}" for n in
                                                   ("K_FULL", "V_FULL", "K_EMPTY", "V_EMPTY", "S_FULL", "P_READY")
                                                   for b in (0, 1)]
        self.bar = {n: Barrier(n) for n in names}
        self.tma = []     # in-flight copies: (buffer, tile, barrier)
        self.pipe = []    # issued products and commits, in order
        self.buf = {}     # buffer -> tile it holds, once complete
        self.pv_done = 0  # P V products completed
        self.pv_issued = 0
        self.roles = [self.producer(), self.issuer(), self.softmax()]
        self.finished = [False] * 3
        self.pending = [None] * 3

    # -- access checks -------------------------------------------------------
    def busy(self, buffer):
        """True while a copy writes `buffer` or a product still uses it."""
        if any(b == buffer for b, _, _ in self.tma):
            return True
        return any(op[0] == "mma" and buffer in op[2] for op in self.pipe)

    def check_free(self, buffer, what):
        if self.busy(buffer):
            raise ProtocolError(f"{what}: {buffer} is still in use")

    def check_holds(self, buffer, tile, what):
        if self.busy(buffer) or self.buf.get(buffer) != tile:
            raise ProtocolError(f"{what}: {buffer} does not hold tile {tile} yet ({self.buf.get(buffer)})")

    # -- waits ---------------------------------------------------------------
    def parity_wait(self, name, phase):
        """Evaluates a parity wait for `phase` of barrier `name`."""
        done = self.bar[name].done
        if not phase <= done <= phase + 1:
            raise ProtocolError(f"parity wait for phase {phase} of {name} evaluated at {done} completed phases")
        return (done & 1) != (phase & 1)

    # -- engines -------------------------------------------------------------
    def issue_copy(self, buffer, tile, barrier):
        self.check_free(buffer, f"copy of tile {tile}")
        self.buf.pop(buffer, None)
        self.tma.append((buffer, tile, barrier))

    def issue_mma(self, label, reads, writes, effect=None):
        """Products run in issue order, so one product's output is complete
        before a later one reads it; the roles check copies and the softmax's
        accesses before they issue."""
        for b in reads:
            if any(c[0] == b for c in self.tma):
                raise ProtocolError(f"{label} reads {b} while a copy writes it")
        self.pipe.append(("mma", label, set(reads) | set(writes), effect))

    def commit(self, barrier):
        self.pipe.append(("commit", barrier))

    def step_engines(self):
        """Lands one copy or retires the oldest pipe entry, at random."""
        choices = []
        if self.tma:
            choices.append("tma")
        if self.pipe:
            choices.append("pipe")
        if not choices:
            return False
        if self.rng.choice(choices) == "tma":
            i = self.rng.randrange(len(self.tma))
            buffer, tile, barrier = self.tma.pop(i)
            self.buf[buffer] = tile
            self.bar[barrier].complete()
        else:
            op = self.pipe.pop(0)
            if op[0] == "mma":
                if op[3]:
                    op[3]()
            else:
                self.bar[op[1]].complete()
        return True

    # -- roles (generators yielding ("wait", barrier, phase) or None) ---------
    def producer(self):
        self.issue_copy("Q", 0, "Q_FULL")
        yield None
        for i in range(self.ntiles + 1):
            if i < self.ntiles:
                b = i & 1
                if i >= 2:
                    yield ("wait", f"K_EMPTY{b}", (i >> 1) - 1)
                self.issue_copy(f"K{b}", i, f"K_FULL{b}")
                yield None
            if i >= 1:
                v = i - 1
                b = v & 1
                if v >= 2:
                    yield ("wait", f"V_EMPTY{b}", (v >> 1) - 1)
                self.issue_copy(f"V{b}", v, f"V_FULL{b}")
                yield None

    def issuer(self):
        q_src = "QT" if self.q_in_tmem else "Q"
        yield ("wait", "QT_READY" if self.q_in_tmem else "Q_FULL", 0)
        self.check_holds(q_src, 0, "S products")
        for j in range(self.ntiles + 1):
            if j < self.ntiles:
                b = j & 1
                yield ("wait", f"K_FULL{b}", j >> 1)
                self.check_holds(f"K{b}", j, f"S_{j}")
                # S_j overwrites S buffer b: the P V product of tile j - 2
                # must have been issued before it (the pipe runs in order)
                if j >= 2 and self.pv_issued < j - 1:
                    raise ProtocolError(f"S_{j} issued before O += P_{j - 2} V_{j - 2}")
                self.issue_mma(f"S_{j}", [q_src, f"K{b}"], [f"S{b}"],
                               effect=lambda b=b, j=j: self.buf.__setitem__(f"S{b}", ("S", j)))
                self.commit(f"S_FULL{b}")
                self.commit(f"K_EMPTY{b}")
                yield None
            if j >= 1:
                jp = j - 1
                b = jp & 1
                yield ("wait", f"P_READY{b}", jp >> 1)
                yield ("wait", f"V_FULL{b}", jp >> 1)
                if self.buf.get(f"S{b}") != ("P", jp):
                    raise ProtocolError(f"O += P_{jp} V_{jp} issued before P_{jp} is written")
                self.check_holds(f"V{b}", jp, f"P_{jp} V_{jp}")
                self.pv_issued += 1
                self.issue_mma(f"PV_{jp}", [f"S{b}", f"V{b}"], ["O"],
                               effect=lambda: setattr(self, "pv_done", self.pv_done + 1))
                self.commit("PV_DONE")
                self.commit(f"V_EMPTY{b}")
                if j == self.ntiles:
                    self.commit("O_FULL")
                yield None

    def softmax(self):
        if self.q_in_tmem:  # head_dim 256: Q rows copied into TMEM, then QT_READY
            yield ("wait", "Q_FULL", 0)
            self.check_holds("Q", 0, "Q into TMEM")
            self.buf["QT"] = 0
            self.bar["QT_READY"].complete()
            yield None
        for j in range(self.ntiles):
            b = j & 1
            yield ("wait", f"S_FULL{b}", j >> 1)
            if self.buf.get(f"S{b}") != ("S", j) or self.busy(f"S{b}"):
                raise ProtocolError(f"softmax reads S_{j} before it is complete")
            if j >= 1 and self.rng.random() < 0.5:  # the row maximum grew: rescale O
                yield ("wait", "PV_DONE", j - 1)
                if self.pv_done < j or any(op[0] == "mma" and "O" in op[2] for op in self.pipe):
                    raise ProtocolError(f"rescale at tile {j} with a product of O pending")
            if self.busy(f"S{b}"):
                raise ProtocolError(f"P_{j} written over S buffer {b} while a product uses it")
            self.buf[f"S{b}"] = ("P", j)
            self.bar[f"P_READY{b}"].complete()
            yield None
        if self.final_on_pv_done:
            yield ("wait", "PV_DONE", self.ntiles - 1)
        else:
            yield ("wait", "O_FULL", 0)
        if self.pv_done < self.ntiles:
            raise ProtocolError(f"O read with {self.ntiles - self.pv_done} products pending")
        for b in (0, 1):  # O / l is staged over the K buffers
            self.check_free(f"K{b}", "output staging")

    # -- scheduler -----------------------------------------------------------
    def run(self, max_steps=20000):
        for _ in range(max_steps):
            if all(self.finished) and not self.tma and not self.pipe:
                return
            runnable = []
            for r in range(3):
                if self.finished[r]:
                    continue
                w = self.pending[r]
                if w is None or self.parity_wait(w[1], w[2]):
                    runnable.append(r)
            engines = bool(self.tma or self.pipe)
            options = runnable + (["engine"] if engines else [])
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


@pytest.mark.parametrize("q_in_tmem", [False, True])
@pytest.mark.parametrize("ntiles", [1, 2, 3, 4, 5, 7])
def test_attention_pipeline_protocol_holds_over_random_schedules(ntiles, q_in_tmem):
    for seed in range(300):
        Model(ntiles, random.Random(seed * 31 + ntiles), q_in_tmem=q_in_tmem).run()


def test_the_model_flags_a_final_parity_wait_on_the_shared_product_barrier():
    """The form the kernel first had: O awaited by the parity of the last
    phase of PV_DONE.  Some schedule must reach that wait with the barrier two
    phases short (or read O with a product pending)."""
    flagged = 0
    for seed in range(400):
        try:
            Model(4, random.Random(seed), final_on_pv_done=True).run()
        except ProtocolError:
            flagged += 1
    assert flagged > 0
