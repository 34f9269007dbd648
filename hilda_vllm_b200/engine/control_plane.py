"""Rank-0 -> other-ranks call broadcast through one shared-memory segment, for tensor-parallel
ranks that share a host but not a parent process (launched by torchrun).

The reference's spawn mode (mini_vllm/engine/model_runner.py:52-65, 96-124) writes each pickled
call into a SharedMemory block and wakes the ranks with multiprocessing Events inherited from the
parent.  Ranks started by torchrun cannot inherit events; a pickled-object broadcast over a gloo
group costs ~0.7 ms per step at 2 ranks and ~1.2 ms at 8 (measured on the CPU), which is on every
decode step's critical path.  Here the ranks poll a sequence number instead:

  header (little-endian uint64 words)
    [0] seq      messages published so far
    [3] writer   process id of rank 0 (readers give up if it disappears)
    [8 + r]      ack of rank r: the number of messages it has finished reading
    [72 + k]     payload bytes of the message in slot k (k < SLOTS)
    [72 + SLOTS + k]  crc32 of that payload
  payload: SLOTS slots of equal size after the header; message i lives in slot i % SLOTS

Writer: message i may reuse its slot once every reader has acked message i - SLOTS, so rank 0 can
run up to SLOTS calls ahead of the slowest rank (a decode step then never waits for the other
ranks to wake up and read the previous one); it writes payload, length and crc, then seq = i + 1.
Reader: waits until seq moves past what it has read, copies the slot, checks the crc (on a weakly
ordered CPU it may see the new seq before the payload; it then reads again), unpickles, acks.
Waits spin for a while (a rank waiting for its next step should wake at once), then yield, then
back off with short sleeps, so an idle rank does not hold a core at 100 %.
"""
from __future__ import annotations

import mmap
import os
import pickle
import time
import zlib
from multiprocessing.shared_memory import SharedMemory

import numpy as np

SLOTS = 8
HEADER_WORDS = 8 + 64 + 2 * SLOTS  # fixed words, one ack per rank (up to 64 ranks), slot lengths and crcs
LEN_OFF = 8 + 64
CRC_OFF = LEN_OFF + SLOTS
PAYLOAD_OFF = HEADER_WORDS * 8
DEFAULT_BYTES = 8 << 20  # SLOTS x 1 MB; the largest call (prefill metadata of 16384 tokens) is ~0.35 MB


class ControlPlaneError(RuntimeError):
    pass


def _pid_alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    return True


class ShmChannel:
    """Single writer (rank 0), world - 1 readers.  `name` is rank 0's segment, created by
    ShmChannel.create and opened by the others with ShmChannel.attach."""

    def __init__(self, buf: memoryview, size: int, name: str, rank: int, world: int, owner: bool, closer):
        assert 1 <= world <= 64
        self.buf, self.rank, self.world, self.owner = buf, rank, world, owner
        self._name, self._closer = name, closer
        self.hdr = np.ndarray((HEADER_WORDS,), dtype=np.uint64, buffer=buf)
        self.slot_bytes = ((size - PAYLOAD_OFF) // SLOTS) & ~63
        self.capacity = self.slot_bytes
        # A reader starts from 0, so one that attaches after the first message still reads it
        # (the writer cannot move past a message until every reader has acked it).
        self.seen = 0

    @classmethod
    def create(cls, world: int, size: int = DEFAULT_BYTES) -> "ShmChannel":
        """Rank 0: a new segment (tracked by Python, so it is removed even if rank 0 dies)."""
        name = f"hilda_b200_{os.getpid()}_{time.monotonic_ns() & 0xFFFFFFFF:x}"
        shm = SharedMemory(name=name, create=True, size=PAYLOAD_OFF + size)

        def closer():
            shm.close()
            try:
                shm.unlink()
            except FileNotFoundError:
                pass

        ch = cls(shm.buf, shm.size, shm.name, 0, world, True, closer)
        ch.hdr[:] = 0
        ch.hdr[3] = os.getpid()
        return ch

    @classmethod
    def attach(cls, name: str, rank: int, world: int) -> "ShmChannel":
        """Ranks > 0: map rank 0's segment directly (not through SharedMemory, whose resource
        tracker would remove the segment when this rank exits)."""
        fd = os.open("/dev/shm/" + name.lstrip("/"), os.O_RDWR)
        try:
            size = os.fstat(fd).st_size
            mm = mmap.mmap(fd, size)
        finally:
            os.close(fd)
        view = memoryview(mm)

        def closer():
            view.release()
            mm.close()

        return cls(view, size, name, rank, world, False, closer)

    @property
    def name(self) -> str:
        return self._name

    # -------------------------------------------------------------- waiting
    @staticmethod
    def _pause(spins: int) -> None:
        if spins < 200_000:
            return
        time.sleep(0 if spins < 400_000 else 0.0002)

    # -------------------------------------------------------------- writer
    def send(self, method: str, *args, timeout_s: float = 120.0) -> None:
        assert self.owner
        data = pickle.dumps([method, *args], protocol=pickle.HIGHEST_PROTOCOL)
        if len(data) > self.capacity:
            raise ControlPlaneError(f"control-plane message of {len(data)} bytes exceeds the {self.capacity}-byte "
                                    "segment")
        seq = int(self.hdr[0])
        acks = self.hdr[8 + 1:8 + self.world]
        need = seq - SLOTS + 1  # every reader must have read message seq - SLOTS (this slot's last)
        t0, spins = time.monotonic(), 0
        while self.world > 1 and int(acks.min()) < need:
            spins += 1
            self._pause(spins)
            if spins % 4096 == 0 and time.monotonic() - t0 > timeout_s:
                late = [r + 1 for r, a in enumerate(acks.tolist()) if a < need]
                raise ControlPlaneError(f"ranks {late} did not read control message {need - 1} within {timeout_s} s")
        k = seq % SLOTS
        off = PAYLOAD_OFF + k * self.slot_bytes
        self.buf[off:off + len(data)] = data
        self.hdr[LEN_OFF + k] = len(data)
        self.hdr[CRC_OFF + k] = zlib.crc32(data)
        self.hdr[0] = seq + 1

    # -------------------------------------------------------------- readers
    def recv(self):
        assert not self.owner
        writer = int(self.hdr[3])
        spins = 0
        k = self.seen % SLOTS
        off = PAYLOAD_OFF + k * self.slot_bytes
        while True:
            if int(self.hdr[0]) > self.seen:
                n = int(self.hdr[LEN_OFF + k])
                crc = int(self.hdr[CRC_OFF + k])
                data = bytes(self.buf[off:off + n])
                # The writer cannot reuse this slot before this reader acks it, so a crc match is
                # this message (a mismatch: published fields not all visible yet, read again).
                if n <= self.slot_bytes and zlib.crc32(data) == crc:
                    break
                continue
            spins += 1
            self._pause(spins)
            if spins % 8192 == 0 and not _pid_alive(writer):
                raise ControlPlaneError(f"rank 0 (pid {writer}) is gone")
        self.seen += 1
        method, *args = pickle.loads(data)
        self.hdr[8 + self.rank] = self.seen
        return method, args

    def close(self) -> None:
        self.hdr = None
        self._closer()
