"""The synchronisation protocol of the chunked gated-delta scan
(`chunk_scan_kernel`, mlx-lean-moe_b200/csrc/gdn_chunked.cu), checked on the
CPU as a discrete-event model over random schedules.

Roles, as in the kernel (each warp group meets at its named barrier, so each
acts as one role here):

- producer: five streams in chunk order, polled with non-blocking tests: K_c
  with the gates into buffer c % 2 (free once U_(c-2) is done: K_EMPTY), Q_c
  (Q_EMPTY), V_c (V_EMPTY), T_c (T_EMPTY), P_c (P_EMPTY);
- converter: [K;Q~]_c into the fp32 operand tile once K_c, Q_c have landed
  and [X|Y]_(c-1) has read the tile (X_DONE); arrives Q_EMPTY, KQ_READY;
- MMA issuer: per chunk [X|Y]_c = S [K;Q~]_c^T (after KQ_READY, U_DONE of c-1,
  Y_FREE of c-2), the first half of O_(c-1) (after P_FULL, DR_READY), Delta_c
  = R^T T^T (after T_FULL, R_READY), the second half of O_(c-1) (then
  OU_DONE, P_EMPTY), U_c: S += Delta'^T K (after DD_READY; then U_DONE,
  K_EMPTY); the two halves of the last O after the loop;
- epilogue: S_0 into TMEM (S_INIT); per chunk beta V (after K_FULL for the
  gates, V_FULL), R over X (after X_DONE; R_READY, V_EMPTY), gamma S in
  place, Delta' hi / lo over R (after D_DONE; DD_READY), Delta rounded in
  place (DR_READY); the final state after U_DONE of the last chunk;
- output: per chunk Y + O (after OU_DONE of its parity), Y_FREE, then the
  staged tile leaves by an asynchronous store that must have read the staging
  buffer before the next chunk is staged; gated (the fused block), the z tile
  of chunk c is awaited on Z_FULL before the norm and z of chunk c + 1 is
  requested into the same tile after it.

Engines: copies land in any order at random times; products retire in issue
order and a commit arrives once every product issued before it is done.  Each
buffer (TMEM regions X, Y, Delta of each parity, S; shared-memory tiles) is
tagged with the data it holds; every access checks the tag it needs and that
no copy or product in flight conflicts with it, and every parity wait or test
checks that its barrier is at the awaited phase or one past it.  Variants
with a step of the protocol taken out (the converter not waiting for
[X|Y]_(c-1), the issuer not waiting for Y_FREE) are checked to fail.
"""

from __future__ import annotations

import random

import pytest


class ProtocolError(AssertionError):
    pass


BARRIERS = (["Z_FULL", "KQ_READY", "Q_FULL", "Q_EMPTY", "V_FULL", "V_EMPTY", "T_FULL", "T_EMPTY", "P_FULL", "P_EMPTY",
             "S_INIT", "X_DONE", "R_READY", "D_DONE", "DD_READY", "DR_READY", "U_DONE"] +
            [f"{n}{b}" for n in ("K_FULL", "K_EMPTY", "OU_DONE", "Y_FREE") for b in (0, 1)])


class Scan:
    def __init__(self, nch, rng, skip=None, gated=False):
        self.nch, self.rng, self.skip, self.gated = nch, rng, skip or set(), gated
        self.done = {n: 0 for n in BARRIERS}
        self.tag = {}        # buffer -> data it holds
        self.copies = []     # in flight: (buffer, tag, barrier)
        self.pipe = []       # ("mma", reads, writes, effect) or ("commit", barrier), in issue order
        self.stores = []     # output stores in flight: they read the staging buffer
        self.roles = [self.producer(), self.converter(), self.issuer(), self.epilogue(), self.output()]
        self.pending = [None] * len(self.roles)
        self.finished = [False] * len(self.roles)

    # -- barriers ------------------------------------------------------------
    def arrive(self, name):
        self.done[name] += 1

    def parity(self, name, phase):
        d = self.done[name]
        if not phase <= d <= phase + 1:
            raise ProtocolError(f"parity wait for phase {phase} of {name} at {d} completed phases")
        return (d & 1) != (phase & 1)

    # -- accesses ------------------------------------------------------------
    def in_flight(self):
        for b, _, _ in self.copies:
            yield b, "w"
        for op in self.pipe:
            if op[0] == "mma":
                for b in op[1]:
                    yield b, "r"
                for b in op[2]:
                    yield b, "w"
        for _ in self.stores:
            yield "STAGE", "r"

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

    def copy(self, buffer, tag, barrier):
        self.access(buffer, "w", f"copy of {tag}")
        self.tag.pop(buffer, None)
        self.copies.append((buffer, tag, barrier))

    def mma(self, what, needs, writes, effect):
        """needs: {buffer: tag} read (checked at issue: a product reads its
        operands after the barrier that says they are complete); writes: the
        buffers it writes; effect: the tags once it retires."""
        for b, t in needs.items():
            if any(c[0] == b for c in self.copies):
                raise ProtocolError(f"{what} reads {b} while a copy writes it")
            # products run in order: an operand still to be written by an
            # earlier product holds what the last such product leaves
            writers = [op for op in self.pipe if op[0] == "mma" and b in op[2]]
            held = writers[-1][3].get(b) if writers else self.tag.get(b)
            if held != t:
                raise ProtocolError(f"{what}: {b} will hold {held}, not {t}")
        self.pipe.append(("mma", set(needs), set(writes), effect))

    def commit(self, barrier):
        self.pipe.append(("commit", barrier))

    def step_engines(self):
        options = (["copy"] if self.copies else []) + (["pipe"] if self.pipe else []) + \
                  (["store"] if self.stores else [])
        pick = self.rng.choice(options)
        if pick == "copy":
            b, t, bar = self.copies.pop(self.rng.randrange(len(self.copies)))
            self.tag[b] = t
            self.arrive(bar)
        elif pick == "pipe":
            op = self.pipe.pop(0)
            if op[0] == "mma":
                for b, t in op[3].items():
                    self.tag[b] = t
            else:
                self.arrive(op[1])
        else:
            self.stores.pop(0)

    # -- roles ---------------------------------------------------------------
    def producer(self):
        nxt = [0] * 5
        while any(c < self.nch for c in nxt):
            ready = []
            for s, c in enumerate(nxt):
                if c >= self.nch:
                    continue
                if s == 0:
                    ok = c < 2 or self.parity(f"K_EMPTY{c & 1}", (c >> 1) - 1)
                else:
                    ok = c < 1 or self.parity(["", "Q_EMPTY", "V_EMPTY", "T_EMPTY", "P_EMPTY"][s], c - 1)
                if ok:
                    ready.append(s)
            if not ready:
                yield ("poll",)
                continue
            s = self.rng.choice(ready)
            c = nxt[s]
            if s == 0:
                self.copy(f"K{c & 1}", ("K", c), f"K_FULL{c & 1}")
            else:
                name = "QVTP"[s - 1]
                self.copy(name, (name, c), f"{name}_FULL")
            nxt[s] = c + 1
            yield None

    def converter(self):
        for c in range(self.nch):
            yield ("wait", f"K_FULL{c & 1}", c >> 1)
            yield ("wait", "Q_FULL", c)
            if c > 0 and "converter_x_done" not in self.skip:
                yield ("wait", "X_DONE", c - 1)
            self.expect(f"K{c & 1}", ("K", c), "converter")
            self.expect("Q", ("Q", c), "converter")
            self.write("KQ", ("KQ", c), "converter")
            self.arrive("Q_EMPTY")
            self.arrive("KQ_READY")
            yield None

    def issuer(self):
        yield ("wait", "S_INIT", 0)

        def issue_o(c, part):
            if part == 0:
                yield ("wait", "P_FULL", c)
                yield ("wait", "DR_READY", c)
            b = c & 1
            self.mma(f"O_{c} half {part}", {f"D{b}": ("Dr", c), "P": ("P", c),
                                             f"Y{b}": ("Y", c) if part == 0 else ("O0", c)},
                     [f"Y{b}"], {f"Y{b}": ("O0", c) if part == 0 else ("O1", c)})
            if part == 1:
                self.commit(f"OU_DONE{b}")
                self.commit("P_EMPTY")
            yield None

        for c in range(self.nch):
            b = c & 1
            yield ("wait", "KQ_READY", c)
            if c > 0:
                yield ("wait", "U_DONE", c - 1)
            if c >= 2 and "issuer_y_free" not in self.skip:
                yield ("wait", f"Y_FREE{b}", (c >> 1) - 1)
            self.mma(f"XY_{c}", {"S": ("S", c), "KQ": ("KQ", c)}, [f"X{b}", f"Y{b}"],
                     {f"X{b}": ("X", c), f"Y{b}": ("Y", c)})
            self.commit("X_DONE")
            yield None
            if c > 0:
                yield from issue_o(c - 1, 0)
            yield ("wait", "T_FULL", c)
            yield ("wait", "R_READY", c)
            self.mma(f"Delta_{c}", {f"X{b}": ("R", c), "T": ("T", c)}, [f"D{b}"], {f"D{b}": ("D", c)})
            self.commit("D_DONE")
            self.commit("T_EMPTY")
            yield None
            if c > 0:
                yield from issue_o(c - 1, 1)
            yield ("wait", "DD_READY", c)
            self.mma(f"U_{c}", {f"X{b}": ("DD", c), f"K{b}": ("K", c), "S": ("gS", c)}, ["S"], {"S": ("S", c + 1)})
            self.commit("U_DONE")
            self.commit(f"K_EMPTY{b}")
            yield None
        if self.nch > 0:
            yield from issue_o(self.nch - 1, 0)
            yield from issue_o(self.nch - 1, 1)

    def epilogue(self):
        self.write("S", ("S", 0), "S_0")
        self.arrive("S_INIT")
        yield None
        for c in range(self.nch):
            b = c & 1
            yield ("wait", f"K_FULL{b}", c >> 1)
            yield ("wait", "V_FULL", c)
            self.expect(f"K{b}", ("K", c), "beta V (gates)")
            self.expect("V", ("V", c), "beta V")
            yield ("wait", "X_DONE", c)
            self.expect(f"X{b}", ("X", c), "R")
            self.write(f"X{b}", ("R", c), "R")
            self.arrive("R_READY")
            self.arrive("V_EMPTY")
            yield None
            self.expect(f"K{b}", ("K", c), "gamma (gates)")
            self.expect("S", ("S", c), "gamma S")
            self.write("S", ("gS", c), "gamma S")
            yield None
            yield ("wait", "D_DONE", c)
            self.expect(f"K{b}", ("K", c), "Delta' (gates)")
            self.expect(f"D{b}", ("D", c), "Delta'")
            self.write(f"X{b}", ("DD", c), "Delta' over R")
            self.arrive("DD_READY")
            self.write(f"D{b}", ("Dr", c), "Delta rounded")
            self.arrive("DR_READY")
            yield None
        if self.nch > 0:
            yield ("wait", "U_DONE", self.nch - 1)
        self.expect("S", ("S", self.nch), "final state")

    def output(self):
        if self.gated and self.nch > 0:  # z of chunk 0 at once, by the output leader
            self.copy("Z", ("Z", 0), "Z_FULL")
        for c in range(self.nch):
            b = c & 1
            yield ("wait", f"OU_DONE{b}", c >> 1)
            self.expect(f"Y{b}", ("O1", c), "output of Y + O")
            # the previous tile's store has read the staging buffer
            while self.stores:
                yield ("poll",)
            self.arrive(f"Y_FREE{b}")
            self.write("STAGE", ("y", c), "staging")
            if self.gated:  # gated norm with z in place, then z of the next chunk into its tile
                yield ("wait", "Z_FULL", c)
                self.expect("Z", ("Z", c), "gated norm")
                self.write("STAGE", ("out", c), "gated norm")
                if c + 1 < self.nch:
                    self.copy("Z", ("Z", c + 1), "Z_FULL")
            self.stores.append(c)
            yield None

    # -- scheduler -----------------------------------------------------------
    def run(self, max_steps=200000):
        for _ in range(max_steps):
            if all(self.finished) and not (self.copies or self.pipe or self.stores):
                return
            runnable = []
            for r, w in enumerate(self.pending):
                if self.finished[r]:
                    continue
                if w is None or (w[0] == "wait" and self.parity(w[1], w[2])):
                    runnable.append(r)
                elif w[0] == "poll":
                    runnable.append(r)  # a polling role re-tests on its next step
            engines = bool(self.copies or self.pipe or self.stores)
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


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("nch", [1, 2, 3, 5, 8])
def test_scan_pipeline_protocol_holds_over_random_schedules(nch, gated):
    for seed in range(150):
        Scan(nch, random.Random(seed * 97 + nch), gated=gated).run()


@pytest.mark.parametrize("step", ["converter_x_done", "issuer_y_free"])
def test_the_model_flags_a_missing_step_of_the_protocol(step):
    flagged = 0
    for seed in range(300):
        try:
            Scan(5, random.Random(seed), skip={step}).run()
        except ProtocolError:
            flagged += 1
    assert flagged > 0
