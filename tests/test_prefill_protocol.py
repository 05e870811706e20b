"""Host-side model of the mbarrier protocol of the tcgen05 prefill attention kernel
(``csrc/attention_prefill.cu``): every role is a sequence of waits (barrier, parity) and
arrivals, executed until all roles finish or none can move.  Checks that the FIFO
operand ring, the raw page ring and the S/P buffers never deadlock and that no parity
wait passes more than one phase early (the hazard of a ring with two fillers)."""
import pytest

K_SLOTS, K_RAW = 6, 3


def use_k(i, c):
    return c if i == 0 else 8 * i - 4 + c


def use_v(i, c, n):
    return 8 * n - 4 + c if i == n - 1 else 8 * i + 8 + c


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def passes(self, parity):
        # mbarrier try_wait.parity: true once the phase with this parity has completed
        return (self.phase & 1) != parity


def run(nh, nf):
    n = nh + nf
    B = {}
    for s in range(K_SLOTS):
        B["full", s] = Bar(1)
        B["empty", s] = Bar(1)
    for r in range(K_RAW):
        B["raw_full", r] = Bar(1)
        B["raw_empty", r] = Bar(1)
    for b in range(2):
        B["s_full", b] = Bar(1)
        B["s_free", b] = Bar(1)
        B["p_full", b] = Bar(4)
    early = []

    def W(key, parity, need):
        return ("wait", key, parity, need)  # need = completions the waiter relies on

    def A(key, times=1):
        return ("arrive", key, times)

    def producer():  # raw INT2 pages only
        for i in range(nh):
            rs = i % K_RAW
            if i >= K_RAW:
                yield W(("raw_empty", rs), ((i // K_RAW) - 1) & 1, i // K_RAW)
            yield A(("raw_full", rs))

    def converters():  # the single filler of the operand ring
        for i in range(n + 1):
            for part in range(2):
                ti = i if part == 0 else i - 1
                if ti < 0 or (part == 0 and i >= n):
                    continue
                hist = ti < nh
                rs = ti % K_RAW
                if part == 0 and hist:
                    yield W(("raw_full", rs), (ti // K_RAW) & 1, ti // K_RAW + 1)
                for c in range(4):
                    u = use_k(ti, c) if part == 0 else use_v(ti, c, n)
                    s = u % K_SLOTS
                    if u >= K_SLOTS:
                        yield W(("empty", s), ((u // K_SLOTS) - 1) & 1, u // K_SLOTS)
                    yield A(("full", s))
                if part == 1 and hist:
                    yield A(("raw_empty", rs))

    def mma():
        for i in range(n + 1):
            if i < n:
                b = i & 1
                if i >= 2:
                    yield W(("s_free", b), ((i >> 1) - 1) & 1, i >> 1)
                for c in range(4):
                    u = use_k(i, c)
                    yield W(("full", u % K_SLOTS), (u // K_SLOTS) & 1, u // K_SLOTS + 1)
                    yield A(("empty", u % K_SLOTS))
                yield A(("s_full", b))
            if i >= 1:
                j = i - 1
                b = j & 1
                yield W(("p_full", b), (j >> 1) & 1, (j >> 1) + 1)
                for c in range(4):
                    u = use_v(j, c, n)
                    yield W(("full", u % K_SLOTS), (u // K_SLOTS) & 1, u // K_SLOTS + 1)
                    yield A(("empty", u % K_SLOTS))
                yield A(("s_free", b))

    def softmax():
        for i in range(n):
            b = i & 1
            yield W(("s_full", b), (i >> 1) & 1, (i >> 1) + 1)
            yield A(("p_full", b), 4)
        if n > 0:
            yield W(("s_free", (n - 1) & 1), ((n - 1) >> 1) & 1, ((n - 1) >> 1) + 1)

    roles = {"producer": producer(), "converters": converters(), "mma": mma(), "softmax": softmax()}
    cur = {k: next(g, None) for k, g in roles.items()}
    while True:
        moved = False
        for k, g in roles.items():
            while cur[k] is not None:
                act = cur[k]
                if act[0] == "wait":
                    bar = B[act[1]]
                    if not bar.passes(act[2]):
                        break
                    if bar.phase < act[3]:
                        early.append((k, act))
                else:
                    for _ in range(act[2]):
                        B[act[1]].arrive()
                cur[k] = next(g, None)
                moved = True
        if all(v is None for v in cur.values()):
            return None, early
        if not moved:
            return cur, early


@pytest.mark.parametrize("nh", range(0, 12))
@pytest.mark.parametrize("nf", range(1, 5))
def test_prefill_pipeline_has_no_deadlock_or_early_wait(nh, nf):
    stuck, early = run(nh, nf)
    assert stuck is None, f"deadlock: {stuck}"
    assert not early, f"parity wait passed early: {early[:3]}"
