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


def _roles(rank, world, tasks):
    """(dir, peer) groups in the order DeviceEngine::RunNativeP2p builds them."""
    lib = _native.lib()
    out = []
    for d in (0, 1):
        for q in range(world):
            if q == rank:
                continue
            ops = [t for t in tasks if t[1] == q and t[0] == d]
            total = sum(len(t[2]) for t in ops)
            if total:
                nch = lib.bcclP2pChannels(total)
                out += [(d, q, ch, nch, ops) for ch in range(nch)]
    return out


def test_protocol_model_over_launches():
    """The kernel's per-CTA protocol, one thread per CTA on every rank: sender waits until the
    slot's previous message was consumed, fills the slot, raises posted; receiver waits for
    posted, drains the slot, raises consumed. Counters carry over between launches whose channel
    counts differ. The model checks that no slot is overwritten before it is drained and that
    every receive buffer ends up equal to the matching send."""
    import threading

    slots = 4
    world = 3
    rng = random.Random(11)
    lock = threading.Condition()
    posted, consumed, sent, recvd = {}, {}, {}, {}
    inbox, full = {}, set()
    errors = []

    def wait(cond):
        with lock:
            if not lock.wait_for(cond, timeout=20):
                errors.append("wait timed out")
                return False
        return True

    def cta(rank, d, peer, ch, nch, ops):
        src, dst = (rank, peer) if d == 0 else (peer, rank)
        key = (src, dst, ch)
        msg = (sent if d == 0 else recvd).get(key, 0)
        sizes = [len(o[2]) for o in ops]
        for i, off, ln in plan(sizes, nch, ch):
            slot = (src, dst, ch, msg % slots)
            if d == 0:
                if msg >= slots and not wait(lambda: consumed.get(key, 0) >= msg + 1 - slots):
                    return
                with lock:
                    if slot in full:
                        errors.append(f"slot {slot} overwritten before it was drained")
                    inbox[slot] = bytes(ops[i][2][off:off + ln])
                    full.add(slot)
                    posted[key] = msg + 1
                    lock.notify_all()
            else:
                if not wait(lambda: posted.get(key, 0) >= msg + 1):
                    return
                with lock:
                    ops[i][2][off:off + ln] = inbox[slot]
                    full.discard(slot)
                    consumed[key] = msg + 1
                    lock.notify_all()
            msg += 1
        (sent if d == 0 else recvd)[key] = msg

    for launch in range(6):
        # matched operations: for every ordered pair a FIFO list of sizes
        pairs = {(a, b): [rng.choice([1, 3, CHUNK, CHUNK + 7, 5 * CHUNK + 1, rng.randrange(1, 40 * CHUNK)])
                          for _ in range(rng.randrange(0, 4))] for a in range(world) for b in range(world) if a != b}
        tasks = {r: [] for r in range(world)}
        expect = []
        for (a, b), sizes in pairs.items():
            for n in sizes:
                payload = bytearray(rng.getrandbits(8) for _ in range(min(n, 64))) * (n // 64 + 1)
                payload = payload[:n]
                out = bytearray(n)
                tasks[a].append((0, b, payload))
                tasks[b].append((1, a, out))
                expect.append((out, bytes(payload)))
        threads = [threading.Thread(target=cta, args=(r,) + role) for r in range(world)
                   for role in _roles(r, world, tasks[r])]
        for t in threads:
            t.start()
        for t in threads:
            t.join(60)
        assert not errors, (launch, errors[:3])
        assert all(bytes(o) == e for o, e in expect), launch
    assert sent == recvd  # both sides of every channel agree on its message count
