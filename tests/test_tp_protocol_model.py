"""A CPU model of the fused TP all-reduce's exchange protocol.

``needle_b200/csrc/tp_allreduce.cuh`` moves data between ranks without flags:
receive and gather slots start as a sentinel, a reader waits until a slot
holds data, consumes it and writes the sentinel back, and the two halves of
every slot array alternate by the parity of a per-row-index call counter
(one counter per receive role).  This model runs the same steps for every
rank, CTA role and row index under a randomised scheduler -- any interleaving
of the ranks' steps, each rank starting a call only after its previous call
ended (stream order) -- over call sequences that mix the kernel's three
launch shapes (two CTAs per row index, one CTA per index, one CTA looping over
several indices).  Every run must finish (no wait that never ends) with every
rank holding the right residual and output rows.

It checks the protocol, not the CUDA code: the steps below mirror the
kernel's and must be kept in step with it.
"""
import random

import pytest

SENT = None  # the sentinel


class Rank:
    def __init__(self, W, slot_rows, max_idx=64):
        mk = lambda: [[[SENT] * slot_rows for _ in range(W)] for _ in range(2)]
        self.recv = mk()      # [half][sender][index]: partial sums pushed to this owner
        self.gh = mk()        # [half][owner][index]: gathered residual rows
        self.go = mk()        # [half][owner][index]: gathered normalised rows
        self.epochs = [[0] * max_idx for _ in range(2)]  # [role][index]
        self.res = {}
        self.out = {}


def kernel_tasks(R, rank, W, T, split, G, partial, sync_counters=True):
    """One rank's kernel for one call, as one generator per CTA; every
    ``yield`` is a point where the CTA can be descheduled, a wait is a loop
    of yields."""
    per = -(-T // W)
    me = R[rank]

    def wait(arr, i, j, k):
        while arr[i][j][k] is SENT:
            yield

    def cta(role, first):
        for b in range(first, per, G):
            e = me.epochs[role][b]
            par = e & 1
            nq = min(W, (T - 1 - b) // per + 1)            # owners with a row at index b
            if role == 0:
                for q in range(nq):                        # reduce-scatter push
                    R[q].recv[par][rank][b] = partial[rank][q * per + b]
                    yield
                row = rank * per + b
                if row < T:                                # owner of this row
                    for p in range(W):
                        yield from wait(me.recv, par, p, b)
                    s = 0
                    for p in range(W):                     # rank order
                        s += me.recv[par][p][b]
                        me.recv[par][p][b] = SENT          # reset for two calls later
                    h = me.res[row] + s
                    for p in range(W):                     # all-gather push
                        R[p].gh[par][rank][b] = h
                        R[p].go[par][rank][b] = ("norm", h)
                        yield
                for q in range(nq):                        # gathered residual rows
                    yield from wait(me.gh, par, q, b)
                    me.res[q * per + b] = me.gh[par][q][b]
                    me.gh[par][q][b] = SENT
                if not split:                              # ... and normalised rows
                    for q in range(nq):
                        yield from wait(me.go, par, q, b)
                        me.out[q * per + b] = me.go[par][q][b]
                        me.go[par][q][b] = SENT
            else:                                          # role 1: normalised rows
                for q in range(nq):
                    yield from wait(me.go, par, q, b)
                    me.out[q * per + b] = me.go[par][q][b]
                    me.go[par][q][b] = SENT
            me.epochs[role][b] = e + 1
            if not split and sync_counters:
                me.epochs[1][b] = e + 1                    # keep the roles' counters in step
            yield

    tasks = [cta(0, c) for c in range(G)]
    if split:
        tasks += [cta(1, c) for c in range(G)]
    return tasks


def run(W, calls, cap, seed, sync_counters=True, max_steps=400_000):
    """Run ``calls`` (row counts per call) on W ranks with ``cap`` resident
    CTAs per GPU; returns normally only if every call finished correctly."""
    rnd = random.Random(seed)
    slot_rows = -(-max(calls) // W)
    R = [Rank(W, slot_rows) for _ in range(W)]
    n = max(calls)
    res0 = {t: 1000 * t for t in range(n)}
    for r in range(W):
        R[r].res = dict(res0)
    parts = [[[(c + 1) * (r + 1) + t for t in range(T)] for r in range(W)]
             for c, T in enumerate(calls)]
    state = [0] * W
    live = {}
    steps = 0
    while True:
        for r in range(W):                     # stream order: next call after the last ended
            if r not in live and state[r] < len(calls):
                c = state[r]
                T = calls[c]
                per = -(-T // W)
                split = 2 * per <= cap
                G = per if split else min(per, cap)
                live[r] = kernel_tasks(R, r, W, T, split, G, parts[c], sync_counters)
        if not live:
            break
        r = rnd.choice(list(live))
        i = rnd.randrange(len(live[r]))
        try:
            next(live[r][i])
        except StopIteration:
            live[r].pop(i)
            if not live[r]:
                del live[r]
                state[r] += 1
        steps += 1
        if steps > max_steps:
            raise AssertionError(f"no progress: ranks stuck in calls {state}")
    res = dict(res0)
    for c, T in enumerate(calls):
        for t in range(T):
            res[t] += sum(parts[c][r][t] for r in range(W))
    for r in range(W):
        assert R[r].res == res, r
        for t in range(calls[-1]):
            assert R[r].out[t] == ("norm", res[t]), (r, t)


# 6 resident CTAs per GPU: 2*per <= 6 splits, per in (3, 6] takes one CTA per
# row index, per > 6 loops over indices inside a CTA
CALLS = lambda W: [2 * W, 5 * W, W + 1, 9 * W, 3 * W, 1, 7 * W, 2 * W, 2 * W, 4 * W + 1, 3]


@pytest.mark.parametrize("W", [2, 3, 4])
@pytest.mark.parametrize("seed", range(3))
def test_protocol_mixed_launch_shapes(W, seed):
    run(W, CALLS(W), cap=6, seed=seed)


def test_protocol_model_detects_counter_drift():
    """Without advancing the second role's counter in calls that do not split,
    the roles disagree on the slot half later and a wait never ends."""
    with pytest.raises(AssertionError, match="no progress"):
        run(2, [20, 4, 4, 20, 4], cap=6, seed=0, sync_counters=False, max_steps=100_000)
