"""The torchrun-mode control plane (engine/control_plane.py): rank 0 publishes pickled calls in a
shared-memory segment that the other ranks poll.  Separate processes on the CPU; failures are
made on the host (a reader that never reads, a writer that exits)."""
import multiprocessing as mp
import os
import time

import numpy as np
import pytest

from hilda_vllm_b200.engine.control_plane import SLOTS, ControlPlaneError, ShmChannel


def _reader(name, rank, world, n, out, delay):
    time.sleep(delay)  # a late reader must still see every message
    ch = ShmChannel.attach(name, rank, world)
    got = []
    for _ in range(n):
        method, args = ch.recv()
        got.append((method, int(args[0]), int(args[1].sum())))
    ch.close()
    out.put((rank, got))


def test_every_reader_gets_every_call_in_order():
    ctx = mp.get_context("spawn")
    world, n = 4, 300
    ch = ShmChannel.create(world, size=1 << 20)
    out = ctx.Queue()
    procs = [ctx.Process(target=_reader, args=(ch.name, r, world, n, out, 0.5 if r == 3 else 0.0))
             for r in range(1, world)]
    for p in procs:
        p.start()
    want = []
    for i in range(n):
        payload = np.full(1 + (i * 997) % 50000, i % 251, np.uint8)  # up to ~50 KB
        ch.send("step", i, payload)
        want.append(("step", i, int(payload.sum())))
    res = dict(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    ch.close()
    assert set(res) == {1, 2, 3}
    for r in res:
        assert res[r] == want, r


def test_message_larger_than_segment_is_rejected():
    ch = ShmChannel.create(1, size=4096)
    with pytest.raises(ControlPlaneError, match="exceeds"):
        ch.send("big", np.zeros(10000, np.uint8))
    ch.send("small", 1)  # the channel stays usable
    ch.close()


def _silent_reader(name, ready):
    ShmChannel.attach(name, 1, 2)
    ready.set()
    time.sleep(30)  # never reads


def test_writer_gives_up_when_a_reader_stops_reading():
    ctx = mp.get_context("spawn")
    ch = ShmChannel.create(2, size=1 << 16)
    ready = ctx.Event()
    p = ctx.Process(target=_silent_reader, args=(ch.name, ready))
    p.start()
    assert ready.wait(60)
    for i in range(SLOTS):  # the writer may run SLOTS messages ahead of a reader
        ch.send("early", i, timeout_s=0.5)
    t0 = time.monotonic()
    with pytest.raises(ControlPlaneError, match=r"ranks \[1\] did not read"):
        ch.send("one too many", 2, timeout_s=0.5)
    assert time.monotonic() - t0 < 20
    p.terminate()
    p.join(timeout=30)
    ch.close()


def _short_writer(q):
    ch = ShmChannel.create(2, size=1 << 16)
    q.put(ch.name)
    time.sleep(1.0)
    os._exit(0)  # leaves without sending (segment name stays, tracker cleans it later)


def test_reader_notices_a_writer_that_is_gone():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_short_writer, args=(q,))
    p.start()
    name = q.get(timeout=60)
    ch = ShmChannel.attach(name, 1, 2)
    p.join(timeout=30)
    t0 = time.monotonic()
    with pytest.raises(ControlPlaneError, match="is gone"):
        ch.recv()
    assert time.monotonic() - t0 < 30
    ch.close()
