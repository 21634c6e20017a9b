"""Failure detection for one-process-per-GPU jobs.

The reference has none: `torchrun --standalone` without restarts, no watchdog, and a dead rank leaves
the others inside a collective until NCCL's own timeout (`train_gpt.py:54-64`).  The fused NVLink
kernels of this framework wait on flags that peers write, so a missing peer must be noticed on the
*host* before the next launch, and a wait that does start must end by itself.  Three layers:

1. `HealthMonitor` - a key-value store of its own (TCPStore on 127.0.0.1 / MASTER_ADDR, separate from
   the process group so that a wedged collective cannot block it).  Every rank publishes a step
   counter and a wall-clock heartbeat; `pre_step()` is called before each step's launches and raises
   `RankFailure` naming the ranks that reported an error, stopped beating, or fell behind.
2. `guard()` - context manager around a step: an exception on this rank is published to the store
   before it propagates, so that the peers' next `pre_step()` fails fast instead of timing out.
3. `check_device()` - reads the device status word that every bounded device-side wait sets on
   expiry (csrc/optim.cu `peer_barrier_kernel`, csrc/gemm_sm100.cuh mbarrier waits) and raises
   `DeviceWaitTimeout`; the CUDA context stays usable.

Nothing here faults, traps or hangs a device: failures are raised, published or timed out on the host.
"""
from __future__ import annotations

import contextlib
import datetime
import os
import threading
import time

import torch
import torch.distributed as dist


class RankFailure(RuntimeError):
    def __init__(self, ranks, reason: str):
        self.ranks, self.reason = sorted(ranks), reason
        super().__init__(f"rank(s) {self.ranks}: {reason}")


class DeviceWaitTimeout(RuntimeError):
    pass


class HealthMonitor:
    """`store` may be any `torch.distributed.Store`; by default rank 0 hosts a TCPStore on
    MASTER_PORT + 17.  Keys: `hb/<rank>` = "<step> <unix time>", `fail/<rank>` = reason."""

    def __init__(self, rank: int, world_size: int, store=None, port: int | None = None, beat_timeout_s: float = 30.0,
                 step_timeout_s: float = 120.0, connect_timeout_s: float = 60.0):
        self.rank, self.world = rank, world_size
        self.beat_timeout_s, self.step_timeout_s = beat_timeout_s, step_timeout_s
        if store is None:
            host = os.environ.get("MASTER_ADDR", "127.0.0.1")
            port = port or int(os.environ.get("MASTER_PORT", "29500")) + 17
            store = dist.TCPStore(host, port, world_size, is_master=(rank == 0),
                                  timeout=datetime.timedelta(seconds=connect_timeout_s), wait_for_workers=False)
        self.store = store
        self.step = -1
        self._stop = threading.Event()
        self._thread = None
        self.failure: RankFailure | None = None
        self._t0 = time.time()
        self.beat(-1)

    # ---- publishing ------------------------------------------------------------------------------
    def beat(self, step: int | None = None):
        if step is not None:
            self.step = step
        self.store.set(f"hb/{self.rank}", f"{self.step} {time.time():.3f}")

    def report_failure(self, reason: str):
        self.store.set(f"fail/{self.rank}", reason[:500])

    # ---- observing -------------------------------------------------------------------------------
    def _read(self, r: int):
        key = f"hb/{r}"
        if not self.store.check([key]):
            return None
        s, t = self.store.get(key).decode().split()
        return int(s), float(t)

    def scan(self, min_step: int | None = None) -> RankFailure | None:
        """One pass over the peers' keys; returns the failure seen, if any (does not wait)."""
        failed = {r: self.store.get(f"fail/{r}").decode() for r in range(self.world)
                  if r != self.rank and self.store.check([f"fail/{r}"])}
        if failed:
            return RankFailure(failed, "reported: " + "; ".join(f"[{r}] {m}" for r, m in sorted(failed.items())))
        now = time.time()
        silent = []
        for r in range(self.world):
            if r == self.rank:
                continue
            hb = self._read(r)
            # a peer that has not published yet gets the same grace period, counted from our own start
            if now - (hb[1] if hb is not None else self._t0) > self.beat_timeout_s:
                silent.append(r)
        if silent:
            return RankFailure(silent, f"no heartbeat for more than {self.beat_timeout_s:.1f}s")
        return None

    def pre_step(self, step: int):
        """Publish `step`, then wait (bounded) until every peer has reached it.  Call between steps,
        with none of this rank's kernels or collectives in flight that wait on a peer."""
        if self.failure is not None:
            raise self.failure
        self.beat(step)
        t0 = time.time()
        while True:
            f = self.scan()
            if f is not None:
                self.failure = f
                raise f
            behind = [r for r in range(self.world) if r != self.rank and (self._read(r) or (-2, 0))[0] < step]
            if not behind:
                return
            if time.time() - t0 > self.step_timeout_s:
                self.failure = RankFailure(behind, f"did not reach step {step} within {self.step_timeout_s:.1f}s")
                raise self.failure
            time.sleep(0.005)

    # ---- background liveness ----------------------------------------------------------------------
    def start(self, interval_s: float = 1.0):
        """Heartbeat thread: keeps `hb/<rank>` fresh while the main thread is inside a long step and
        records the first peer failure in `self.failure` for the next `pre_step()`."""
        def loop():
            while not self._stop.wait(interval_s):
                try:
                    self.beat()
                    f = self.scan()
                    if f is not None and self.failure is None:
                        self.failure = f
                except Exception as e:                                  # the store's host is gone
                    if self.failure is None:
                        self.failure = RankFailure([0], f"health store unreachable: {e}")
                    return
        self._thread = threading.Thread(target=loop, daemon=True, name="mng-health")
        self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    @contextlib.contextmanager
    def guard(self):
        try:
            yield self
        except RankFailure:
            raise
        except BaseException as e:
            with contextlib.suppress(Exception):
                self.report_failure(f"{type(e).__name__}: {e}")
            raise


def check_device(device=None):
    """Raises DeviceWaitTimeout if a kernel's bounded wait expired since the last check (synchronises)."""
    if not torch.cuda.is_available():
        return
    from ..ops import native
    like = torch.empty(1, device=device or "cuda")
    word = native.lib().status_tensor(like)
    code = int(word.item())
    if code:
        word.zero_()
        raise DeviceWaitTimeout(f"device status word {code}: a bounded wait on a peer flag or barrier expired")


def monitor_from_env(env) -> HealthMonitor | None:
    """MNG_HEALTH=1 switches the monitor on for multi-rank jobs (MNG_HEALTH_TIMEOUT seconds per step)."""
    if os.environ.get("MNG_HEALTH", "0") != "1" or env.world_size == 1:
        return None
    t = float(os.environ.get("MNG_HEALTH_TIMEOUT", "120"))
    return HealthMonitor(env.rank, env.world_size, step_timeout_s=t, beat_timeout_s=max(10.0, t / 4)).start()
