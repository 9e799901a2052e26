"""Step watchdog for tensor-parallel steps.

The reference wraps every TP forward in a timeout (NEURON_TP_STEP_TIMEOUT_S = 120 s);
on expiry it aborts the NCCL communicator on a separate thread and arms a deadman: if
the abort does not return within NEURON_TP_ABORT_DEADLINE_S = 60 s, the process logs
and exits with status 70 so the service manager restarts it (tp/mod.rs:326-498).

Here a single monitor thread watches `step()` scopes. On a timeout it calls
`on_timeout` (abort the communicators / poison the model) in a helper thread and, if
that does not finish within `abort_deadline_s`, calls `on_deadman` (default:
`os._exit(70)`). All decisions are host-side, so the logic is testable without a GPU.
"""
from __future__ import annotations

import os
import threading
import time
from contextlib import contextmanager
from typing import Callable

EXIT_DEADMAN = 70


class StepTimeout(RuntimeError):
    pass


class StepWatchdog:
    def __init__(self, timeout_s: float | None = None, abort_deadline_s: float | None = None,
                 on_timeout: Callable[[], None] | None = None, on_deadman: Callable[[], None] | None = None,
                 poll_s: float = 0.05):
        self.timeout_s = timeout_s if timeout_s is not None else float(os.environ.get("HELEXA_TP_STEP_TIMEOUT_S", 120))
        self.abort_deadline_s = abort_deadline_s if abort_deadline_s is not None else \
            float(os.environ.get("HELEXA_TP_ABORT_DEADLINE_S", 60))
        self.on_timeout = on_timeout or (lambda: None)
        self.on_deadman = on_deadman or (lambda: os._exit(EXIT_DEADMAN))
        self.poll_s = poll_s
        self._started: float | None = None
        self._name = ""
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self.fired = threading.Event()
        self.deadman_fired = threading.Event()
        self._thread = threading.Thread(target=self._run, name="helexa-watchdog", daemon=True)
        self._thread.start()

    @contextmanager
    def step(self, name: str = "step"):
        if self.fired.is_set():
            raise StepTimeout("communicator was aborted by the watchdog")
        with self._lock:
            self._started, self._name = time.monotonic(), name
        try:
            yield
        finally:
            with self._lock:
                self._started = None
        if self.fired.is_set():
            raise StepTimeout(f"{name} exceeded {self.timeout_s}s and was aborted")

    def _run(self):
        while not self._stop.wait(self.poll_s):
            with self._lock:
                st = self._started
            if st is None or self.fired.is_set() or time.monotonic() - st <= self.timeout_s:
                continue
            self.fired.set()
            done = threading.Event()

            def abort():
                try:
                    self.on_timeout()
                finally:
                    done.set()

            threading.Thread(target=abort, name="helexa-watchdog-abort", daemon=True).start()
            if not done.wait(self.abort_deadline_s):
                self.deadman_fired.set()
                self.on_deadman()

    def close(self):
        self._stop.set()
        self._thread.join(1.0)
