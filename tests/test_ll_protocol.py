"""Line protocol of the low-latency kernel (CPU): epochs and a threaded model of the exchange.

The kernel (csrc/kernels/ll.cu) stores every 8 payload bytes with the launch's epoch into the
peers' line buffers of parity epoch & 1 and polls its own lines until they carry that epoch; no
flag or barrier separates launches. Its correctness rests on the epoch sequence
(csrc/kernels/ll_epoch.h, shared with the bcclLLEpoch hook checked here): never 0, the value of
a line that was never written; the other parity than the previous launch's, so a rank writes a
parity again only two launches later, after every peer has read it; and no repeat within 2^32 - 2
launches. The model runs ranks as threads doing back-to-back launches with random stalls, with
the launch counter started just before the 32-bit wrap, and checks that every value read belongs
to the reader's current launch.
"""
import random
import threading
import time

from originccl_b200 import _native

PERIOD = (1 << 32) - 2


def epoch(seq):
    return _native.lib().bcclLLEpoch(seq)


def test_epochs_never_zero_and_alternate_parity_across_the_wrap():
    rng = random.Random(3)
    starts = [0, 1, PERIOD - 5, 2 * PERIOD - 5, (1 << 32) - 3, (1 << 40) + 17] + [rng.randrange(1 << 62) for _ in range(50)]
    for s0 in starts:
        prev = epoch(s0)
        assert prev != 0
        for s in range(s0 + 1, s0 + 12):
            e = epoch(s)
            assert e != 0 and e < (1 << 32) - 1
            assert (e & 1) != (prev & 1), (s, prev, e)
            prev = e
    assert epoch(0) == 1 and epoch(PERIOD - 1) == PERIOD and epoch(PERIOD) == 1
    # the 32-bit truncation of seq + 1 (the scheme this replaces) gives 0 at the wrap
    assert ((1 << 32) - 1 + 1) & 0xFFFFFFFF == 0 and epoch((1 << 32) - 1) != 0


def _run_model(nranks, nlines, launches, seq0, seed, epoch_of=None):
    """Ranks as threads; buf[owner][parity][src][line] = (value, epoch), zero-initialised. Launch
    k moves 1 + (k * 7) % nlines lines (the same on every rank, as a collective's size is), so
    some launches read lines that no earlier launch wrote."""
    epoch_of = epoch_of or epoch
    buf = [[[[(0, 0)] * nlines for _ in range(nranks)] for _ in range(2)] for _ in range(nranks)]
    errors = []

    def rank(r):
        rng = random.Random(seed * 100 + r)
        for k in range(launches):
            e = epoch_of(seq0 + k)
            par = e & 1
            lines = 1 + (k * 7) % nlines
            for q in range(nranks):
                if q == r:
                    continue
                for i in range(lines):
                    buf[q][par][r][i] = (1000000 * k + 1000 * r + i, e)  # one store: value with its epoch
                    if rng.random() < 0.05:
                        time.sleep(0)
            for q in range(nranks):
                if q == r:
                    continue
                for i in range(lines):
                    deadline = time.monotonic() + 10.0
                    while True:
                        v, got = buf[r][par][q][i]
                        if got == e:
                            break
                        if time.monotonic() > deadline:
                            errors.append(f"rank {r} launch {k}: line {i} from {q} never arrived")
                            return
                        time.sleep(0)
                    if v != 1000000 * k + 1000 * q + i:
                        errors.append(f"rank {r} launch {k}: line {i} from {q} holds {v}")
            if rng.random() < 0.3:
                time.sleep(rng.random() * 1e-3)  # a slow rank falls behind its peers

    threads = [threading.Thread(target=rank, args=(r,)) for r in range(nranks)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    return errors


def test_threaded_exchange_across_the_epoch_wrap():
    for nranks, seed in ((2, 1), (3, 2), (4, 3)):
        errors = _run_model(nranks, nlines=8, launches=40, seq0=PERIOD - 20, seed=seed)
        assert not errors, errors[:5]


def test_model_catches_an_epoch_that_wraps_to_zero():
    # seq + 1 truncated to 32 bits: launch 2^32 - 1 gets epoch 0 and takes never-written lines
    # (zero) for data. Launches before it move few lines, the one at the wrap the most.
    errors = _run_model(2, nlines=64, launches=12, seq0=(1 << 32) - 10, seed=4,
                        epoch_of=lambda s: (s + 1) & 0xFFFFFFFF)
    assert errors


def test_threaded_exchange_from_a_fresh_communicator():
    errors = _run_model(3, nlines=5, launches=30, seq0=0, seed=9)
    assert not errors, errors[:5]
