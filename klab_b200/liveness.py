"""Host-side failure detection for the column-sharded chain.

The chain's ranks exchange data through bounded device waits on monotonic epoch
flags: a kernel that waits longer than its limit records a status code and returns,
it never hangs. What the devices cannot tell is *why* a peer stopped. Between
token steps, StepGuard answers that on the host, before any rank launches the next
step (a rank leaves only between steps, with nothing of its own in flight):

  * every rank posts the epoch it is about to run under `<prefix>/<rank>` in a
    torch.distributed Store (the same store the process group rendezvous uses);
  * each rank then waits, at most `timeout` seconds, until every rank has posted
    the epoch; epochs compare like the device flags, as a signed 32-bit
    difference (`epoch_reached`), so they may wrap;
  * the outcome is one exception per failure kind:
      PeerLost       a rank said it left (`leave()`, e.g. on shutdown);
      PeerLate       a rank has not reached the epoch within the bound (a crashed
                     or hung rank looks like this too);
      StaleEpoch     a rank is two or more epochs behind: it restarted or missed
                     steps, so its buffers do not belong to this step;
      CorruptEpoch   a rank's record is not an epoch, or it is two or more epochs
                     ahead, which no healthy rank can be (it waits for everyone);
  * after a step, `check_device()` reads the device status word and raises
    DeviceWaitExpired when a kernel gave up a bounded wait.
"""

from __future__ import annotations

import time

_WRAP = 1 << 32
LEFT = b"left"


def epoch_reached(flag: int, target: int) -> bool:
    """The device comparison of a flag with a target epoch: (int32)(flag - target) >= 0."""
    return ((flag - target) % _WRAP) < (1 << 31)


def epoch_distance(flag: int, target: int) -> int:
    """flag - target as a signed 32-bit difference."""
    d = (flag - target) % _WRAP
    return d - _WRAP if d >= (1 << 31) else d


class PeerFailure(RuntimeError):
    """A peer rank cannot take part in the next step."""

    def __init__(self, message, rank, epoch):
        super().__init__(message)
        self.rank, self.epoch = rank, epoch


class PeerLost(PeerFailure):
    pass


class PeerLate(PeerFailure):
    pass


class StaleEpoch(PeerFailure):
    pass


class CorruptEpoch(PeerFailure):
    pass


class DeviceWaitExpired(RuntimeError):
    """A kernel gave up a bounded wait on a flag or a copy (device status word)."""

    def __init__(self, status):
        super().__init__(f"a kernel gave up a bounded wait (device status {status})")
        self.status = status


class StepGuard:
    """Bounded host-side agreement on the next step's epoch among `world` ranks."""

    def __init__(self, store, rank, world, timeout=1.0, prefix="klab/step", poll=0.002):
        if not (0 <= rank < world):
            raise ValueError("rank must be in [0, world)")
        if not timeout > 0:
            raise ValueError("timeout must be positive")
        self.store, self.rank, self.world = store, rank, world
        self.timeout, self.prefix, self.poll = float(timeout), prefix, poll

    def _key(self, rank):
        return f"{self.prefix}/{rank}"

    def post(self, epoch):
        self.store.set(self._key(self.rank), str(int(epoch) % _WRAP))

    def leave(self):
        """Tell the other ranks that this one has left (they raise PeerLost)."""
        self.store.set(self._key(self.rank), LEFT)

    def _read(self, rank):
        key = self._key(rank)
        if not self.store.check([key]):
            return None
        return self.store.get(key)

    def enter(self, epoch):
        """Post `epoch`, then wait (bounded) until every rank has reached it."""
        epoch = int(epoch) % _WRAP
        self.post(epoch)
        deadline = time.monotonic() + self.timeout
        pending = [r for r in range(self.world) if r != self.rank]
        while True:
            still = []
            for r in pending:
                raw = self._read(r)
                if raw is None:
                    still.append((r, None))
                    continue
                if raw == LEFT:
                    raise PeerLost(f"rank {r} left before epoch {epoch}", r, epoch)
                try:
                    value = int(raw.decode() if isinstance(raw, bytes) else raw)
                except (ValueError, UnicodeDecodeError):
                    raise CorruptEpoch(f"rank {r} posted {raw!r}, not an epoch", r, epoch) from None
                if not 0 <= value < _WRAP:
                    raise CorruptEpoch(f"rank {r} posted {value}, outside 32 bits", r, epoch)
                d = epoch_distance(value, epoch)
                if d >= 2:
                    raise CorruptEpoch(f"rank {r} is {d} epochs ahead of {epoch}", r, epoch)
                if d <= -2:
                    raise StaleEpoch(f"rank {r} is at epoch {value}, {-d} behind {epoch}", r, epoch)
                if d < 0:
                    still.append((r, value))
            if not still:
                return
            if time.monotonic() >= deadline:
                r, value = still[0]
                seen = "nothing" if value is None else f"epoch {value}"
                raise PeerLate(f"rank {r} did not reach epoch {epoch} within {self.timeout:.3f} s ({seen})", r,
                               epoch)
            pending = [r for r, _ in still]
            time.sleep(self.poll)

    @staticmethod
    def check_device(status_fn=None):
        """Raise DeviceWaitExpired when the current device's status word is set (and clear it)."""
        if status_fn is None:
            from . import _native

            status_fn = _native.device_status
        status = status_fn()
        if status:
            raise DeviceWaitExpired(status)
