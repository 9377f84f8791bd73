"""Control-plane channels of tensor-parallel serving: rank 0 sends each engine step's plan (new requests, aborts, stop)
to the other ranks of the node before the step.

``ShmChannel`` (default): one shared-memory segment per job, one writer (rank 0), one message in flight. The writer
puts the pickled message and its header (length, final-part flag, CRC-32 over sequence number, header and payload)
in place, then bumps the sequence number; each reader waits for the next sequence number, checks the CRC (so a message
seen half-written on a weakly ordered CPU is read again, not used), copies it out and acknowledges it in its own slot.
The writer waits for every acknowledgement before reusing the buffer. A message larger than the buffer goes in parts.
Readers busy-wait (yielding) for the first 16 ms of a wait, the engine-input spin of the reference's launcher
(code/kit/REPRODUCE.md:321), then poll every 0.5 ms. Every wait is bounded by ``timeout_s`` and raises
``TimeoutError``, so a rank whose peer went away ends with an error. The segment's name goes out once over the CPU
process group. vLLM, the reference's engine, sends its scheduler output to the workers through a shared-memory
broadcast queue for the same reason: a per-step collective over sockets costs milliseconds.

``GlooChannel``: ``broadcast_object_list`` over the CPU group (ranks on several hosts).
"""

from __future__ import annotations

import pickle
import struct
import time
import zlib

_HDR = 64                       # [seq u64][len u64][crc u32][final u8] ... payload at _HDR
_SPIN_S = 0.016


def _untrack(shm) -> None:
    """A reader must not unlink the writer's segment at exit (the resource tracker would on Python < 3.13)."""
    try:
        from multiprocessing import resource_tracker
        resource_tracker.unregister(shm._name, "shared_memory")
    except Exception:  # pragma: no cover - tracker internals differ between versions
        pass


def _pause(t0: float) -> None:
    time.sleep(0 if time.monotonic() - t0 < _SPIN_S else 0.0005)


def _crc(seq: int, n: int, final: int, payload) -> int:
    return zlib.crc32(payload, zlib.crc32(struct.pack("<QQB", seq, n, final)))


class ShmChannel:
    def __init__(self, group, timeout_s: float = 60.0, capacity: int = 4 << 20):
        import torch.distributed as dist
        from multiprocessing import shared_memory
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = timeout_s
        self.cap = capacity
        self.ack_off = _HDR + capacity
        size = self.ack_off + 8 * self.world
        box = [None]
        if self.rank == 0:
            self.shm = shared_memory.SharedMemory(create=True, size=size)     # zero-filled
            box = [self.shm.name]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0), group=group)
        if self.rank != 0:
            self.shm = shared_memory.SharedMemory(name=box[0])
            _untrack(self.shm)
        dist.barrier(group=group)                 # every reader is attached before the first message
        self.seq = 0

    def _acked(self, seq: int) -> bool:
        buf = self.shm.buf
        return all(struct.unpack_from("<Q", buf, self.ack_off + 8 * r)[0] >= seq for r in range(1, self.world))

    def publish(self, obj) -> None:
        data = pickle.dumps(obj, protocol=pickle.HIGHEST_PROTOCOL)
        parts = [data[i:i + self.cap] for i in range(0, len(data), self.cap)] or [b""]
        for i, part in enumerate(parts):
            t0 = time.monotonic()
            while not self._acked(self.seq):
                if time.monotonic() - t0 > self.timeout_s:
                    raise TimeoutError(f"control plane: a rank did not take message {self.seq} "
                                       f"within {self.timeout_s:.0f} s")
                _pause(t0)
            final = int(i == len(parts) - 1)
            seq = self.seq + 1
            buf = self.shm.buf
            buf[_HDR:_HDR + len(part)] = part
            struct.pack_into("<QIB", buf, 8, len(part), _crc(seq, len(part), final, part), final)
            struct.pack_into("<Q", buf, 0, seq)
            self.seq = seq

    def receive(self):
        parts = []
        while True:
            want = self.seq + 1
            t0 = time.monotonic()
            while True:
                buf = self.shm.buf
                if struct.unpack_from("<Q", buf, 0)[0] >= want:
                    n, crc, final = struct.unpack_from("<QIB", buf, 8)
                    if n <= self.cap:
                        part = bytes(buf[_HDR:_HDR + n])
                        if _crc(want, n, final, part) == crc:
                            break
                if time.monotonic() - t0 > self.timeout_s:
                    raise TimeoutError(f"control plane: no message {want} from rank 0 within {self.timeout_s:.0f} s")
                _pause(t0)
            self.seq = want
            struct.pack_into("<Q", buf, self.ack_off + 8 * self.rank, want)
            parts.append(part)
            if final:
                return pickle.loads(b"".join(parts))

    def close(self) -> None:
        self.shm.close()
        if self.rank == 0:
            try:
                self.shm.unlink()
            except FileNotFoundError:  # pragma: no cover
                pass


class GlooChannel:
    def __init__(self, group):
        import torch.distributed as dist
        self.group = group
        self.src = dist.get_global_rank(group, 0)

    def _bcast(self, obj):
        import torch.distributed as dist
        box = [obj]
        dist.broadcast_object_list(box, src=self.src, group=self.group)
        return box[0]

    def publish(self, obj) -> None:
        self._bcast(obj)

    def receive(self):
        return self._bcast(None)

    def close(self) -> None:
        pass
