"""Supervision of the multi-process jobs the command line launches (tensor-parallel calibration).

The launcher (``torch.distributed.run``) and its workers run in a process group of their own. The supervisor waits for
the launcher with a time limit; when the limit passes, the launcher fails, or the user interrupts, it terminates the
whole group (SIGTERM, then SIGKILL after a grace period), so no worker survives holding a GPU or a port. Files the
workers wrote stay where they are: a failed calibration keeps its partial measurements, and the caller writes its
success artefacts (``serve.sh``) only when the job exited 0. The reference's CLI supervises its serving engine the same
way (``eagle_harness/cli.py:144-174``).
"""

from __future__ import annotations

import os
import signal
import socket
import subprocess
import sys
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence


@dataclass(frozen=True)
class Outcome:
    code: int
    timed_out: bool = False
    interrupted: bool = False

    @property
    def ok(self) -> bool:
        return self.code == 0 and not self.timed_out and not self.interrupted


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def torchrun(nproc: int, module: str, args: Sequence[str], *, port: Optional[int] = None) -> List[str]:
    """``python -m torch.distributed.run`` of ``module`` on ``nproc`` local ranks (one per GPU)."""
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(nproc),
            "--master-addr", "127.0.0.1", "--master-port", str(port or free_port()), "-m", module, *args]


def _signal_group(pgid: int, sig: int) -> bool:
    try:
        os.killpg(pgid, sig)
        return True
    except ProcessLookupError:
        return False


def stop_group(proc: subprocess.Popen, grace: float = 10.0) -> None:
    """End every process of the group that ``proc`` leads (it was started in a session of its own)."""
    if _signal_group(proc.pid, signal.SIGTERM):
        try:
            proc.wait(grace)
        except subprocess.TimeoutExpired:
            pass
        _signal_group(proc.pid, signal.SIGKILL)
    proc.wait()


def supervise(cmd: Sequence[str], *, timeout: Optional[float] = None, grace: float = 10.0,
              env: Optional[Dict[str, str]] = None) -> Outcome:
    """Run ``cmd`` in a new process group and wait at most ``timeout`` seconds; the group is ended on a time-out, on
    a failure (stragglers) and on an interrupt."""
    proc = subprocess.Popen(list(cmd), start_new_session=True, env=env)
    try:
        code = proc.wait(timeout=timeout)
    except subprocess.TimeoutExpired:
        stop_group(proc, grace)
        return Outcome(124, timed_out=True)
    except KeyboardInterrupt:
        stop_group(proc, grace)
        return Outcome(130, interrupted=True)
    if code != 0:
        stop_group(proc, grace)
    return Outcome(code)
