"""The barrier protocol of the default attention kernel (csrc/attn_fwd.cu), on CPU.

A model of the kernel's roles -- the K/V producer, the Q producer, the single MMA-issuing
thread and the two softmax warpgroups -- written as coroutines that wait on and arrive at
mbarriers with the hardware's phase/parity semantics (try_wait.parity succeeds once the
phase of that parity has completed).  TMA loads and the MMA thread's tensor-core operations
complete asynchronously, the latter in issue order, and every commit arrives when the
operations issued before it are done.  The kernel's correctness rests on that order: P_i is
written over S_i's columns, so the QK^T_i(j+1) that rewrites them must execute after the
PV_i(j) that reads P_i(j), and the softmax's rescale of O_i relies on PV_i(j-1) having run
before S_i(j) arrives.  Random interleavings over segment lists (the units and slices a CTA
walks) check that the protocol never deadlocks and that every read sees the right data: the
scores (read once, and again by the rare re-check of the running max), P, O (rescale and
epilogue), the Q buffer and every K/V ring slot.  The model mirrors the kernel's barrier
sequence by hand: a change to one must be made in the other."""
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


STAGES = 4          # K/V ring slots of the 128-key kernel
RECHECK = 0.2       # share of steps whose running max is re-checked (S read again)
RESCALE = 0.2       # share of those that rescale O


def run(segs, seed):
    rnd = random.Random(seed)
    B = {}

    def bar(name, c):
        B[name] = Bar(c)
    bar("q_full", 1); bar("q_empty", 1)
    for s in range(STAGES):
        bar(f"kvf{s}", 1); bar(f"kve{s}", 1)
    for i in range(2):
        for nm in ("s_full", "p_full", "o_full", "o_empty"):
            bar(f"{nm}{i}", 1)
    kv = [None] * STAGES        # item held by each ring slot
    qbuf = [None]               # segment whose Q tiles are loaded
    SP = [None, None]           # S_i / P_i columns: ("S", step) or ("P", step)
    O = [[], []]                # steps accumulated in O_i (current segment)
    seg_of_step, starts, g = [], [], 0
    for a, n in enumerate(segs):
        seg_of_step += [a] * n
        starts.append(g)
        g += n
    tensor_q = []               # the MMA thread's pending tensor-core operations, in order
    tma_q = []

    def commit(name):
        tensor_q.append(("commit", name))

    def kv_producer():
        item = 0
        for n in segs:
            for _ in range(n):
                for _kind in range(2):
                    slot = item % STAGES
                    yield ("wait", f"kve{slot}", ((item // STAGES) & 1) ^ 1)
                    tma_q.append(("kv", slot, item))
                    item += 1
                    yield None

    def q_producer():
        for a in range(len(segs)):
            if a > 0:
                yield ("wait", "q_empty", (a - 1) & 1)
            tma_q.append(("q", a))
            yield None

    def mma():
        g = 0
        for a, n in enumerate(segs):
            pa = (a - 1) & 1
            yield ("wait", "q_full", a & 1)
            for jj in range(n):
                ik = 2 * g
                yield ("wait", f"kvf{ik % STAGES}", (ik // STAGES) & 1)
                if jj == 0:
                    for i in range(2):
                        tensor_q.append(("qk", i, g, ik % STAGES)); commit(f"s_full{i}")
                    commit(f"kve{ik % STAGES}")
                else:
                    iv, pp = 2 * (g - 1) + 1, (g - 1) & 1
                    yield ("wait", f"kvf{iv % STAGES}", (iv // STAGES) & 1)
                    yield ("wait", "p_full0", pp)
                    if jj == 1 and a > 0:
                        yield ("wait", "o_empty0", pa)
                    tensor_q.append(("pv", 0, g - 1, iv % STAGES, jj > 1))
                    tensor_q.append(("qk", 0, g, ik % STAGES)); commit("s_full0")
                    yield ("wait", "p_full1", pp)
                    if jj == 1 and a > 0:
                        yield ("wait", "o_empty1", pa)
                    tensor_q.append(("pv", 1, g - 1, iv % STAGES, jj > 1))
                    commit(f"kve{iv % STAGES}")
                    tensor_q.append(("qk", 1, g, ik % STAGES)); commit("s_full1")
                    commit(f"kve{ik % STAGES}")
                if jj == n - 1:
                    commit("q_empty")
                g += 1
                yield None
            iv, pp = 2 * (g - 1) + 1, (g - 1) & 1
            yield ("wait", f"kvf{iv % STAGES}", (iv // STAGES) & 1)
            yield ("wait", "p_full0", pp)
            if n == 1 and a > 0:
                yield ("wait", "o_empty0", pa)
            tensor_q.append(("pv", 0, g - 1, iv % STAGES, n > 1)); commit("o_full0")
            yield ("wait", "p_full1", pp)
            if n == 1 and a > 0:
                yield ("wait", "o_empty1", pa)
            tensor_q.append(("pv", 1, g - 1, iv % STAGES, n > 1)); commit("o_full1")
            commit(f"kve{iv % STAGES}")

    def softmax(i):
        g = 0
        for a, n in enumerate(segs):
            for jj in range(n):
                yield ("wait", f"s_full{i}", g & 1)
                assert SP[i] == ("S", g), f"softmax{i} reads {SP[i]} expected S{g}"
                yield None  # exp pass
                if jj > 0 and rnd.random() < RECHECK:
                    assert SP[i] == ("S", g), f"softmax{i} re-reads {SP[i]} expected S{g}"
                    if rnd.random() < RESCALE:
                        assert O[i] and O[i][-1] == g - 1, f"rescale before PV {g - 1}: {O[i]}"
                    yield None
                SP[i] = ("P", g)
                B[f"p_full{i}"].arrive()
                g += 1
                yield None
            yield ("wait", f"o_full{i}", a & 1)
            want = list(range(starts[a], starts[a] + n))
            assert O[i] == want, f"epilogue O{i} {O[i]} expected {want}"
            yield None
            B[f"o_empty{i}"].arrive()
            yield None

    roles = {"kv": kv_producer(), "q": q_producer(), "mma": mma(), "sm0": softmax(0),
             "sm1": softmax(1)}
    state = {k: None for k in roles}
    finished = set()

    def engine_step():
        if tma_q and rnd.random() < 0.5:
            op = tma_q.pop(0)
            if op[0] == "kv":
                kv[op[1]] = op[2]
                B[f"kvf{op[1]}"].arrive()
            else:
                qbuf[0] = op[1]
                B["q_full"].arrive()
        if tensor_q and rnd.random() < 0.5:
            op = tensor_q.pop(0)
            if op[0] == "commit":
                B[op[1]].arrive()
            elif op[0] == "qk":
                _, i, step, slot = op
                assert kv[slot] == 2 * step, f"QK{i}({step}) reads K item {kv[slot]}"
                assert qbuf[0] == seg_of_step[step], f"QK{i}({step}) reads Q of seg {qbuf[0]}"
                assert SP[i] is None or SP[i][0] == "P" and SP[i][1] < step and \
                    pv_ran[i] == SP[i][1], f"QK{i}({step}) overwrites {SP[i]} before its PV"
                SP[i] = ("S", step)
            else:
                _, i, step, slot, acc = op
                assert kv[slot] == 2 * step + 1, f"PV{i}({step}) reads V item {kv[slot]}"
                assert SP[i] == ("P", step), f"PV{i}({step}) reads {SP[i]}"
                if acc:
                    O[i].append(step)
                else:
                    O[i][:] = [step]
                pv_ran[i] = step

    pv_ran = [None, None]
    for _ in range(10 ** 6):
        runnable = [k for k in roles if k not in finished and
                    (state[k] is None or B[state[k][1]].done(state[k][2]))]
        if not runnable and not tma_q and not tensor_q:
            if len(finished) == len(roles):
                return True
            raise RuntimeError(f"deadlock: {[(k, state[k]) for k in roles if k not in finished]}")
        if runnable and (not (tma_q or tensor_q) or rnd.random() < 0.6):
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
