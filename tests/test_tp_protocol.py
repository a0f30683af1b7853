"""A randomized interleaving simulation of the tensor-parallel residual exchange
(k_merge_q8_tp in syrinx_b200/csrc/gemv_q8.cu), on the CPU.

Each rank runs its exchange kernels in stream order (kernel e+1 starts only after kernel e
completed). In a kernel, one thread per slot (token, row) the exchange carries: reads and
bumps the slot's epoch, stores the 8-byte word {value, epoch} into parity (epoch % 2) of
every peer's receive region, then polls its own region until every peer's word for the
slot carries its epoch. Exchanges carry different slot subsets (decode steps carry token 0
only, prefill chunks carry many tokens). A random scheduler interleaves single steps of all
runnable threads of all ranks. The checks: every value read is the peer's value of the same
exchange (no stale word is ever accepted), and every run finishes (no deadlock)."""
import random

import pytest


def simulate(n_ranks, n_slots, n_exch, seed):
    rng = random.Random(seed)
    # which slots each exchange carries: all, or a prefix (token 0 rows), like M=8 / M=1 merges
    carries = [list(range(n_slots)) if rng.random() < 0.4 else list(range(rng.randint(1, n_slots)))
               for _ in range(n_exch)]
    value = lambda r, e, s: (r * 1000003 + e * 1009 + s * 7919) & 0xFFFFFFFF
    rx = [[[[(0, 0)] * n_slots for _ in range(n_ranks)] for _ in range(2)] for _ in range(n_ranks)]  # [dst][par][src][slot]
    epochs = [[0] * n_slots for _ in range(n_ranks)]
    k_next = [0] * n_ranks  # next kernel per rank
    running = [None] * n_ranks  # per rank: {slot: thread state} of the running kernel
    errors = []

    def start(r):
        e = k_next[r]
        running[r] = {s: {"pc": 0, "ep": None, "q": 0, "tot": 0} for s in carries[e]}

    for r in range(n_ranks):
        start(r)
    steps = 0
    while any(k_next[r] < n_exch for r in range(n_ranks)):
        steps += 1
        if steps > 200000:
            raise AssertionError("deadlock: no progress")
        cands = [(r, s) for r in range(n_ranks) if k_next[r] < n_exch for s, t in running[r].items() if t["pc"] < 3]
        if not cands:  # every thread of the running kernels is done: kernels complete
            for r in range(n_ranks):
                if k_next[r] < n_exch and all(t["pc"] == 3 for t in running[r].values()):
                    k_next[r] += 1
                    if k_next[r] < n_exch:
                        start(r)
            continue
        r, s = rng.choice(cands)
        t = running[r][s]
        e = k_next[r]
        if t["pc"] == 0:  # bump the slot epoch, store the word to every peer
            t["ep"] = epochs[r][s] + 1
            epochs[r][s] = t["ep"]
            for p in range(n_ranks):
                if p != r:
                    rx[p][t["ep"] & 1][r][s] = (value(r, e, s), t["ep"])
            t["pc"] = 1
        elif t["pc"] == 1:  # poll the peers in rank order
            q = t["q"]
            if q == r:
                t["q"] += 1
            else:
                v, ep = rx[r][t["ep"] & 1][q][s]
                if ep == t["ep"]:
                    if v != value(q, e, s):
                        errors.append((r, e, s, q))
                    t["q"] += 1
            if t["q"] >= n_ranks:
                t["pc"] = 2
        else:
            t["pc"] = 3
        # kernels whose threads are all done complete at once
        if all(x["pc"] == 3 for x in running[r].values()):
            k_next[r] += 1
            if k_next[r] < n_exch:
                start(r)
    return errors


@pytest.mark.parametrize("n_ranks", [2, 3, 4])
@pytest.mark.parametrize("seed", range(12))
def test_exchange_never_accepts_a_stale_word(n_ranks, seed):
    assert simulate(n_ranks, n_slots=6, n_exch=40, seed=seed) == []


def test_per_cta_epochs_would_accept_stale_words():
    """The counter-example that made the epoch per slot: with one epoch counter per CTA
    and the CTA owning different rows in decode and prefill exchanges, an old word can
    carry the epoch a receiver waits for. Slot 1 is carried by CTA 0 in a prefill-like
    exchange and by CTA 1 in decode-like ones; CTA 0's counter runs ahead of slot 1's
    history, so after two decode exchanges CTA 1's expected epoch equals a stale one."""
    # slot 1's words: exchange A (CTA 0, epoch 1), then decode exchanges (CTA 1, epochs 1, 2)
    history = [("A", 1), ("D1", 1), ("D2", 2)]
    # the decode exchange D1 expects epoch 1 in parity 1, where exchange A left epoch 1
    stale = {(ep & 1, ep): ex for ex, ep in history[:1]}
    assert stale.get((1 & 1, 1)) == "A"  # D1 would accept A's word: per-CTA epochs are unsafe
