"""Race model of k_persistent_smem's face exchange (CPU, no GPU).

The shared-memory persistent kernel keeps every block of the grid in one
CTA's shared memory and exchanges only faces: at the end of step s a block
stores its faces of p_{s+1} into its neighbours' exchange rows as words
(tag = s + 1, value), then waits for the words of its own rows to show that
tag and reads them.  Rows alternate between two parities, (s + 1) & 1, and a
block never waits for a neighbour to finish reading: the claim is that by the
time it overwrites a row of step s+2, the reader has already consumed the
row of step s, because the writer itself waited for that reader's faces of
step s+1, which the reader stores only after its reads of step s.

This test runs that protocol with one Python thread per block on a small
block grid, with random yields between every word, and checks that every
word a block reads carries exactly the value its neighbour computed for that
step.  With one parity instead of two (the mistake planted in the model) a
fast writer overwrites rows before they are read, and the check must see it.
"""
import random
import threading
import time

import pytest

NEIGHBOURS = ((0, -1), (0, 1), (-1, 0), (1, 0))  # (dz, dy): below / above in y and z


def run_model(yblocks, zblocks, steps, words, parities, seed, timeout_s=20.0):
    """Returns the list of mismatches (block, step, side, word, got, want)."""
    nblk = yblocks * zblocks
    # rows[(parity, receiver, side)] = list of (tag, value) words
    rows = {}
    for p in range(parities):
        for b in range(nblk):
            for side in range(4):
                rows[(p, b, side)] = [(0, None)] * words
    bad = []
    lock = threading.Lock()
    deadline = time.monotonic() + timeout_s

    def nb_of(b, side):
        yb, zb = b % yblocks, b // yblocks
        dz, dy = NEIGHBOURS[side]
        y2, z2 = yb + dy, zb + dz
        if 0 <= y2 < yblocks and 0 <= z2 < zblocks:
            return z2 * yblocks + y2
        return None

    def value(b, s, side_of_writer, w):
        return (b, s, side_of_writer, w)

    def block(b):
        rng = random.Random(seed * 7919 + b)
        for s in range(steps):
            # "compute" p_{s+1}, then store each face into the neighbour's row
            # that holds it (the writer's side s_w lands on the reader's side
            # s_w ^ 1: my face below in y is the halo above of the block below)
            par = (s + 1) % parities
            tag = s + 1
            for side in range(4):
                nb = nb_of(b, side)
                if nb is None:
                    continue
                row = rows[(par, nb, side ^ 1)]
                for w in range(words):
                    if rng.random() < 0.3:
                        time.sleep(0)
                    row[w] = (tag, value(b, tag, side, w))
            # receive this step's faces: wait (bounded) for each word's tag
            for side in range(4):
                nb = nb_of(b, side)
                if nb is None:
                    continue
                row = rows[(par, b, side)]
                for w in range(words):
                    while True:
                        t, v = row[w]
                        if t == tag:
                            break
                        if t > tag or time.monotonic() > deadline:
                            # a newer word already replaced the one this step needs
                            with lock:
                                bad.append((b, s, side, w, (t, v), tag))
                            return
                        time.sleep(0)
                    want = value(nb, tag, side ^ 1, w)
                    if v != want:
                        with lock:
                            bad.append((b, s, side, w, v, want))
                    if rng.random() < 0.3:
                        time.sleep(0)

    threads = [threading.Thread(target=block, args=(b,)) for b in range(nblk)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout_s + 5)
    return bad


@pytest.mark.parametrize("yblocks,zblocks", [(2, 1), (3, 2), (4, 4), (1, 5)])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_two_parities_never_overwrite_an_unread_face(yblocks, zblocks, seed):
    bad = run_model(yblocks, zblocks, steps=12, words=6, parities=2, seed=seed)
    assert not bad, bad[:5]


def test_model_catches_a_single_parity():
    """With one parity a block can store step s+2's faces before its
    neighbour has read step s+1's: the model has to report it."""
    found = False
    for seed in range(1, 40):
        if run_model(4, 1, steps=30, words=4, parities=1, seed=seed, timeout_s=5.0):
            found = True
            break
    assert found
