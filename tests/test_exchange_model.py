"""A model check of the per-level histogram exchange's receive-area reuse (CPU only).

peer_kernels.cu exchanges each level's histogram between ranks with pushes into the
receivers' receive areas, split into two halves by the exchange's epoch parity:
  one-shot (2 ranks): push the whole histogram to every peer, signal, wait for every
      rank's signal, then read the received copies;
  two-shot (3+ ranks): push slice r to rank r, signal, wait, read the copies of this
      rank's slice and push the sums, signal again, wait again.
Ranks run ahead of one another between exchanges (the rest of the level loop does not
synchronise them). This model runs W ranks through a sequence of exchanges of growing and
shrinking sizes under many random interleavings and checks that no push lands on a
receive-area vector that a slower rank has not yet read for an earlier exchange. The
layout the library uses (halves fixed for the fit) passes at every rank count; halves
that scale with each exchange's size fail for the one-shot, which shows the check can see
the hazard, and pass for the two-shot, whose second barrier orders the reuse.
"""
import random

import pytest


def layout_fixed(half):
    return lambda parity, q, stride: parity * half + q * stride


def layout_scaled(W):
    return lambda parity, q, stride: (parity * W + q) * stride


def run(W, sizes, layout, seed):
    """sizes: vectors per exchange. Returns the first overwrite-before-read, or None."""
    rng = random.Random(seed)
    one_shot = W == 2
    signals = [[0] * W for _ in range(W)]    # signals[r][q]: epoch rank q signalled to r
    departs = [[0] * W for _ in range(W)]
    pending = [dict() for _ in range(W)]      # receive vector -> epoch still to be read
    plans = []
    for r in range(W):
        steps = []
        for e, n in enumerate(sizes, start=1):
            stride = n if one_shot else (n + W - 1) // W
            par = e & 1
            # push: the vectors this rank writes into every other rank's receive area
            steps.append(("push", e, [(t, layout(par, r, stride) + j)
                                      for t in range(W) if t != r
                                      for j in range(stride)]))
            steps.append(("signal", e))
            steps.append(("wait", e))
            steps.append(("read", e, [layout(par, q, stride) + j
                                      for q in range(W) if q != r for j in range(stride)]))
            if not one_shot:
                steps.append(("depart", e))
                steps.append(("wait_depart", e))
            steps.append(("other_work", e))   # the rest of the level: no receive access
        plans.append(steps)
    pos = [0] * W
    while any(pos[r] < len(plans[r]) for r in range(W)):
        ready = []
        for r in range(W):
            if pos[r] >= len(plans[r]):
                continue
            st = plans[r][pos[r]]
            if st[0] == "wait" and min(signals[r]) < st[1]:
                continue
            if st[0] == "wait_depart" and min(departs[r]) < st[1]:
                continue
            ready.append(r)
        assert ready, "the schedule deadlocked"
        r = rng.choice(ready)
        st = plans[r][pos[r]]
        pos[r] += 1
        if st[0] == "push":
            for t, v in st[2]:
                if v in pending[t] and pending[t][v] < st[1]:
                    return (r, t, v, pending[t][v], st[1])
                pending[t][v] = st[1]
        elif st[0] == "signal":
            for t in range(W):
                signals[t][r] = st[1]
        elif st[0] == "depart":
            for t in range(W):
                departs[t][r] = st[1]
        elif st[0] == "read":
            for v in st[2]:
                if pending[r].get(v) == st[1]:
                    del pending[r][v]
    return None


# vectors per exchange: a depth-6 tree's levels (1, 1, 2, 4, 8, 16 groups), the per-tree
# scale exchange does not use the receive area, then the next tree
SIZES = [4, 4, 8, 16, 32, 64, 4, 4, 8, 16]


@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_fixed_halves_never_overwrite_unread_copies(W):
    one_shot = W == 2
    big = max(SIZES)
    half = W * (big if one_shot else (big + W - 1) // W)
    for seed in range(300):
        assert run(W, SIZES, layout_fixed(half), seed) is None


def test_size_scaled_halves_can_overwrite_in_the_one_shot():
    """The one-shot ends without a second barrier: with halves that scale with each
    exchange, a fast rank's next (larger) copies reach vectors a slow rank still has to
    read."""
    hits = [run(2, SIZES, layout_scaled(2), seed) for seed in range(300)]
    assert any(h is not None for h in hits)


@pytest.mark.parametrize("W", [3, 4])
def test_two_shot_departure_barrier_orders_reuse(W):
    """The two-shot's second barrier ends every rank's exchange only after all ranks have
    read their copies, so even size-scaled halves would be safe there."""
    for seed in range(300):
        assert run(W, SIZES, layout_scaled(W), seed) is None


def run_full(W, trees, depth, seed, small_layout_parity=True):
    """Both exchange kinds of a fit in their real order: per tree one small exchange (the
    scale maxima: every rank stores into slot [parity][me] of every rank, signal, wait,
    read all slots), then per level the histogram exchange; with 3+ ranks its sums are
    pushed into every rank's reduced copy, which the split scan reads after the exchange.
    Returns the first overwrite-before-read of any resource, or None."""
    rng = random.Random(seed)
    one_shot = W == 2
    sizes = [4 << max(d - 1, 0) for d in range(depth)]
    big = max(sizes, default=1)
    half = W * (big if one_shot else (big + W - 1) // W)
    signals = [[0] * W for _ in range(W)]
    departs = [[0] * W for _ in range(W)]
    pending = [dict() for _ in range(W)]  # (resource, index) -> epoch still to be read
    plans = []
    for r in range(W):
        steps, e = [], 0
        for _t in range(trees):
            e += 1
            par = (e & 1) if small_layout_parity else 0
            steps.append(("push", e, [(t, ("slot", par, r)) for t in range(W)]))
            steps.append(("signal", e))
            steps.append(("wait", e))
            steps.append(("read", e, [("slot", par, q) for q in range(W)]))
            for n in sizes:
                e += 1
                par = e & 1
                stride = n if one_shot else (n + W - 1) // W
                steps.append(("push", e, [(t, ("recv", par * half + r * stride + j))
                                          for t in range(W) if t != r for j in range(stride)]))
                steps.append(("signal", e))
                steps.append(("wait", e))
                steps.append(("read", e, [("recv", par * half + q * stride + j)
                                          for q in range(W) if q != r for j in range(stride)]))
                if not one_shot:
                    lo = r * stride
                    steps.append(("push", e, [(t, ("sum", v)) for t in range(W)
                                              for v in range(lo, min(n, lo + stride))]))
                    steps.append(("depart", e))
                    steps.append(("wait_depart", e))
                    steps.append(("read", e, [("sum", v) for v in range(n)]))  # split scan
        plans.append(steps)
    pos = [0] * W
    while any(pos[r] < len(plans[r]) for r in range(W)):
        ready = [r for r in range(W) if pos[r] < len(plans[r]) and not (
            (plans[r][pos[r]][0] == "wait" and min(signals[r]) < plans[r][pos[r]][1]) or
            (plans[r][pos[r]][0] == "wait_depart" and min(departs[r]) < plans[r][pos[r]][1]))]
        assert ready, "the schedule deadlocked"
        r = rng.choice(ready)
        st = plans[r][pos[r]]
        pos[r] += 1
        if st[0] == "push":
            for t, key in st[2]:
                if key in pending[t] and pending[t][key] < st[1]:
                    return (r, t, key, pending[t][key], st[1])
                pending[t][key] = st[1]
        elif st[0] == "signal":
            for t in range(W):
                signals[t][r] = st[1]
        elif st[0] == "depart":
            for t in range(W):
                departs[t][r] = st[1]
        elif st[0] == "read":
            for key in st[2]:
                if pending[r].get(key) == st[1]:
                    del pending[r][key]
    return None


@pytest.mark.parametrize("W", [2, 3, 4, 8])
def test_fit_sequence_never_overwrites_unread_data(W):
    """Small slots, receive area and reduced copy together, over two depth-6 trees."""
    for seed in range(150):
        assert run_full(W, trees=2, depth=6, seed=seed) is None


def test_small_slots_need_their_parity():
    """Back-to-back small exchanges (the GOSS radix passes) have no other barrier between
    them: without the parity doubling a fast rank's next values could overwrite slots a
    slower rank has not read; the model sees it (depth 0: small exchanges only)."""
    hits = [run_full(2, trees=4, depth=0, seed=s, small_layout_parity=False)
            for s in range(300)]
    assert any(h is not None for h in hits)
    for s in range(300):
        assert run_full(2, trees=4, depth=0, seed=s) is None
