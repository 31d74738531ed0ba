"""The barrier protocol of the 64-key-tile attention kernel (csrc/attn_fwd64.cu), on CPU.

A model of the kernel's roles -- the K/V producer, the Q producer, one MMA-issuing thread per
query tile and the two softmax warpgroups -- written as coroutines that wait on and arrive
at mbarriers with the hardware's phase/parity semantics (try_wait.parity succeeds once the
phase of that parity has completed, so a barrier advanced by two phases before its waiter
looks incomplete again).  TMA loads and each issuer's tensor-core operations
complete asynchronously and in issue order, and every commit arrives when the operations
before it are done.  Random interleavings over segment lists (the units and slices a CTA
walks) check that the protocol never deadlocks and never lets a read see the wrong data:
S_i, both P_i buffers, O_i (rescale and epilogue), the Q buffer and every K/V ring slot.
The kernel's waits are bounded, so a protocol error on the GPU ends in ANIMA_ERR_TIMEOUT;
this model is where such errors are found first (it found the two-phase p_full advance that
led to one p_full barrier per P buffer).  The model mirrors the kernel by hand: a change to
the kernel's barrier sequence must be made here too."""
import random

import pytest


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self, n=1):
        self.pending -= n
        assert self.pending >= 0
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity):  # try_wait.parity semantics
        return (self.phase & 1) != parity


STAGES = 8
RESCALE = 0.2


def run(segs, seed):
    rnd = random.Random(seed)
    B = {}
    def bar(name, c):
        B[name] = Bar(c)
    bar("q_full", 1); bar("q_empty", 2)
    for s in range(STAGES):
        bar(f"kvf{s}", 1); bar(f"kve{s}", 2)
    for i in range(2):
        for nm, c in (("s_full", 1), ("s_free", 1), ("pf0_", 1), ("pf1_", 1), ("pvd0_", 1), ("pvd1_", 1), ("o_full", 1), ("o_empty", 1)):
            bar(f"{nm}{i}", c)
    # shadow state
    kv = [None] * STAGES        # item held by each slot
    qbuf = [None]               # segment held by Q
    S = [None, None]            # step held in S_i
    P = [[None, None], [None, None]]  # step held in P_i[buf]
    O = [[], []]                # steps accumulated in O_i (current segment)
    seg_of_step = []
    for a, n in enumerate(segs):
        seg_of_step += [a] * n
    starts = []
    g = 0
    for n in segs:
        starts.append(g); g += n
    tensor_q = [[], []]         # pending tensor ops of each issuing thread (in order)
    tma_q = []                  # pending TMA loads

    def commit(name, i):
        tensor_q[i].append(("commit", name))

    # ---- roles as generators yielding ("wait", bar, parity) or None (a step)
    def kv_producer():
        item = 0
        for a, n in enumerate(segs):
            for j in range(n):
                for kind in range(2):
                    slot, rnd_ = item % STAGES, item // STAGES
                    yield ("wait", f"kve{slot}", (rnd_ & 1) ^ 1)
                    tma_q.append(("kv", slot, item))
                    item += 1
                    yield None

    def q_producer():
        for a, n in enumerate(segs):
            if a > 0:
                yield ("wait", "q_empty", (a - 1) & 1)
            tma_q.append(("q", a))
            yield None

    def mma(i):
        g = 0
        for a, n in enumerate(segs):
            pa = (a - 1) & 1
            yield ("wait", "q_full", a & 1)
            ik = 2 * g
            yield ("wait", f"kvf{ik % STAGES}", (ik // STAGES) & 1)
            if g > 0:
                yield ("wait", f"s_free{i}", (g - 1) & 1)
            tensor_q[i].append(("qk", i, g, ik % STAGES)); commit(f"s_full{i}", i)
            commit(f"kve{ik % STAGES}", i)
            if n == 1:
                commit("q_empty", i)
            for jj in range(n):
                gj = g + jj
                ik, iv = 2 * (gj + 1), 2 * gj + 1
                more = jj + 1 < n
                pg = gj & 1
                if more:
                    yield ("wait", f"kvf{ik % STAGES}", (ik // STAGES) & 1)
                    yield ("wait", f"s_free{i}", pg)
                    tensor_q[i].append(("qk", i, gj + 1, ik % STAGES)); commit(f"s_full{i}", i)
                    commit(f"kve{ik % STAGES}", i)
                    if jj + 2 == n:
                        commit("q_empty", i)
                yield ("wait", f"kvf{iv % STAGES}", (iv // STAGES) & 1)
                yield ("wait", f"pf{gj & 1}_{i}", (gj >> 1) & 1)
                if jj == 0 and a > 0:
                    yield ("wait", f"o_empty{i}", pa)
                tensor_q[i].append(("pv", i, gj, iv % STAGES, gj & 1, jj > 0)); commit(f"pvd{gj & 1}_{i}", i)
                commit(f"kve{iv % STAGES}", i)
                if not more:
                    commit(f"o_full{i}", i)
                yield None
            g += n

    def softmax(i):
        g = 0
        for a, n in enumerate(segs):
            for jj in range(n):
                yield ("wait", f"s_full{i}", g & 1)
                assert S[i] == g, f"softmax{i} reads S step {S[i]} expected {g}"
                yield None  # S in registers
                B[f"s_free{i}"].arrive()
                yield None  # exp work
                if g >= 2:  # P buffer g&1 was last read by PV(g-2)
                    yield ("wait", f"pvd{g & 1}_{i}", ((g - 2) >> 1) & 1)
                if jj > 0 and rnd.random() < RESCALE:  # a rescale of O needs PV(g-1) done
                    yield ("wait", f"pvd{(g - 1) & 1}_{i}", ((g - 1) >> 1) & 1)
                    assert O[i] and O[i][-1] == g - 1, f"rescale before PV {g-1}: {O[i]}"
                # P buffer g&1 must not be pending for PV(g-2)
                assert P[i][g & 1] is None or P[i][g & 1] <= g - 2
                P[i][g & 1] = g
                B[f"pf{g & 1}_{i}"].arrive()
                g += 1
                yield None
            yield ("wait", f"o_full{i}", a & 1)
            seg_steps = list(range(starts[a], starts[a] + n))
            assert O[i] == seg_steps, f"epilogue O{i} {O[i]} expected {seg_steps}"
            yield None
            B[f"o_empty{i}"].arrive()
            yield None

    roles = {"kv": kv_producer(), "q": q_producer(), "mma0": mma(0), "mma1": mma(1),
             "sm0": softmax(0), "sm1": softmax(1)}
    state = {k: None for k in roles}  # pending wait
    finished = set()

    def engine_step():
        acted = False
        if tma_q and rnd.random() < 0.5:
            op = tma_q.pop(0)
            if op[0] == "kv":
                _, slot, item = op
                kv[slot] = item
                B[f"kvf{slot}"].arrive()
            else:
                qbuf[0] = op[1]
                B["q_full"].arrive()
            acted = True
        qs = [q for q in tensor_q if q]
        if qs and rnd.random() < 0.5:
            op = rnd.choice(qs).pop(0)
            if op[0] == "commit":
                B[op[1]].arrive()
            elif op[0] == "qk":
                _, i, gstep, slot = op
                assert kv[slot] == 2 * gstep, f"QK{i}({gstep}) reads K item {kv[slot]}"
                assert qbuf[0] == seg_of_step[gstep], f"QK reads Q of seg {qbuf[0]}"
                S[i] = gstep
            else:
                _, i, gstep, slot, buf, acc = op
                assert kv[slot] == 2 * gstep + 1, f"PV{i}({gstep}) reads V item {kv[slot]}"
                assert P[i][buf] == gstep, f"PV{i}({gstep}) reads P {P[i][buf]}"
                if acc:
                    O[i].append(gstep)
                else:
                    O[i][:] = [gstep]
            acted = True
        return acted

    for it in range(10 ** 6):
        runnable = []
        for k, r in roles.items():
            if k in finished:
                continue
            w = state[k]
            if w is None or B[w[1]].done(w[2]):
                runnable.append(k)
        if not runnable and not tma_q and not any(tensor_q):
            if len(finished) == len(roles):
                return True
            raise RuntimeError(f"deadlock: waits {[(k, state[k]) for k in roles if k not in finished]}")
        if runnable and (not (tma_q or any(tensor_q)) or rnd.random() < 0.6):
            k = rnd.choice(runnable)
            try:
                y = next(roles[k])
                state[k] = y if (y and y[0] == "wait") else None
            except StopIteration:
                finished.add(k)
        else:
            engine_step()
    raise RuntimeError("no progress")




CASES = [[1], [2], [3], [4, 4], [1, 1, 1], [5, 1, 3], [2, 7, 2, 1], [8] * 5, [16, 16, 3],
         [1, 2, 1, 2, 1], [9, 1]]


@pytest.mark.parametrize("segs", CASES, ids=lambda s: "-".join(map(str, s)))
def test_protocol_completes_without_hazards(segs):
    for seed in range(60):
        assert run(segs, seed)
