"""Schedule of the native device Send/Recv (CPU): the chunk plan the kernel walks.

The kernel (csrc/kernels/p2p_native.cu) and these hooks share one cursor (csrc/kernels/p2p_sched.h);
the checks are the invariants the protocol relies on: sender and receiver derive the same channel
count from the pair's total bytes, every byte of every operation travels exactly once, chunk g of
the pair's FIFO sequence goes to channel g % nch, and each channel carries its chunks in sequence
order (its message numbers). Parity: the reference's P2P keeps one FIFO per directed pair
(OriginCCL src/topology/topology_p2p.cpp:50-58, tests/regression/test_p2p.cpp:312, the repeated-peer FIFO case).
"""
import ctypes
import random

from originccl_b200 import _native

CHUNK = 64 << 10


def plan(sizes, nch, ch):
    lib = _native.lib()
    n = len(sizes)
    cap = sum((s + CHUNK - 1) // CHUNK for s in sizes) + 1
    b = (ctypes.c_ulonglong * max(n, 1))(*sizes)
    op = (ctypes.c_int * cap)()
    off = (ctypes.c_ulonglong * cap)()
    ln = (ctypes.c_ulonglong * cap)()
    k = lib.bcclP2pPlan(b, n, nch, ch, cap, op, off, ln)
    assert k >= 0
    return [(op[i], off[i], ln[i]) for i in range(k)]


def test_channels_follow_total_bytes():
    lib = _native.lib()
    assert lib.bcclP2pChannels(0) == 1
    assert lib.bcclP2pChannels(1) == 1
    assert lib.bcclP2pChannels(256 << 10) == 1
    assert lib.bcclP2pChannels((256 << 10) + 1) == 2
    assert lib.bcclP2pChannels(1 << 30) == 8
    prev = 1
    for b in range(0, 4 << 20, 37 << 10):
        c = lib.bcclP2pChannels(b)
        assert prev <= c <= 8
        prev = c


def test_every_byte_travels_once_in_fifo_order():
    rng = random.Random(5)
    lib = _native.lib()
    for _ in range(60):
        sizes = [rng.choice([1, 2, 17, CHUNK - 1, CHUNK, CHUNK + 1, 3 * CHUNK + 5, rng.randrange(1, 2 << 20)])
                 for _ in range(rng.randrange(1, 9))]
        nch = lib.bcclP2pChannels(sum(sizes))
        # pair-wide chunk numbering in FIFO order
        number = {}
        g = 0
        for i, s in enumerate(sizes):
            for k in range((s + CHUNK - 1) // CHUNK):
                number[(i, k * CHUNK)] = g
                g += 1
        covered = [0] * len(sizes)
        seen = set()
        for ch in range(nch):
            last = -1
            for i, off, ln in plan(sizes, nch, ch):
                g = number[(i, off)]
                assert g % nch == ch
                assert g > last  # message order follows the sequence
                last = g
                assert 0 < ln <= CHUNK and off + ln <= sizes[i]
                assert (i, off) not in seen
                seen.add((i, off))
                covered[i] += ln
        assert covered == sizes
        assert len(seen) == len(number)


def test_bad_arguments_are_rejected():
    lib = _native.lib()
    b = (ctypes.c_ulonglong * 1)(10)
    o = (ctypes.c_int * 1)()
    u = (ctypes.c_ulonglong * 1)()
    assert lib.bcclP2pPlan(b, 1, 0, 0, 1, o, u, u) == -1
    assert lib.bcclP2pPlan(b, 1, 9, 0, 1, o, u, u) == -1
    assert lib.bcclP2pPlan(b, 1, 2, 2, 1, o, u, u) == -1
