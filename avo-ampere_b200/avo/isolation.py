"""Child-process runner for scoring workers.

Contract with the reference's scorer and CLI (``avo/isolation.py`` there): a worker prints
its result as one line ``AVO_RESULT_JSON=<json object>`` on stdout, and the parent gets a
record with ``ok``, ``returncode``, ``timed_out``, ``payload`` and the tails of both
output streams.  A crash, a non-zero exit or a timeout of the child becomes a record with
``ok == False``; it never takes the parent down.

This runner starts the child in its own session and, on timeout, ends the whole process
group (a worker that spawned ranks or compiler processes leaves none behind).
"""

from __future__ import annotations

import json
import os
import signal
import subprocess
import sys
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any

RESULT_PREFIX = "AVO_RESULT_JSON="
TAIL_CHARS = 4000


@dataclass(frozen=True)
class IsolatedResult:
    returncode: int | None
    timed_out: bool
    payload: dict[str, Any] | None
    stdout_tail: str = field(repr=False)
    stderr_tail: str = field(repr=False)

    @property
    def ok(self) -> bool:
        """The child exited 0 in time and printed a result object."""
        return not self.timed_out and self.returncode == 0 and self.payload is not None

    def as_dict(self) -> dict[str, Any]:
        record = asdict(self)
        record["ok"] = self.ok
        return record


def extract_payload(stdout: str) -> dict[str, Any] | None:
    """The result object of the last ``AVO_RESULT_JSON=`` line, or None if that line is
    missing, not JSON, or not an object."""
    lines = [ln for ln in stdout.splitlines() if ln.startswith(RESULT_PREFIX)]
    if not lines:
        return None
    try:
        value = json.loads(lines[-1][len(RESULT_PREFIX):])
    except ValueError:
        return None
    return value if isinstance(value, dict) else None


def print_result(payload: dict[str, Any]) -> None:
    """Worker side of the contract: emit the result line and flush."""
    sys.stdout.write(RESULT_PREFIX + json.dumps(payload, sort_keys=True) + "\n")
    sys.stdout.flush()


def module_worker_args(*args: str) -> list[str]:
    """Command line that runs ``python -m avo <args>`` with this interpreter."""
    return [sys.executable, "-m", "avo", *args]


def _as_text(data: str | bytes | None) -> str:
    if data is None:
        return ""
    if isinstance(data, bytes):
        return data.decode("utf-8", errors="replace")
    return data


def _kill_group(proc: subprocess.Popen) -> None:
    try:
        os.killpg(proc.pid, signal.SIGKILL)
    except (ProcessLookupError, PermissionError):
        proc.kill()


def run_json_worker(args: list[str], *, timeout_s: float, cwd: Path | None = None,
                    env: dict[str, str] | None = None) -> IsolatedResult:
    """Run ``args`` to completion or until ``timeout_s`` seconds pass."""
    proc = subprocess.Popen(args, cwd=cwd, env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                            start_new_session=True)
    try:
        out, err = proc.communicate(timeout=timeout_s)
    except subprocess.TimeoutExpired:
        _kill_group(proc)
        out, err = proc.communicate()
        return IsolatedResult(None, True, None, _as_text(out)[-TAIL_CHARS:], _as_text(err)[-TAIL_CHARS:])
    stdout, stderr = _as_text(out), _as_text(err)
    return IsolatedResult(proc.returncode, False, extract_payload(stdout),
                          stdout[-TAIL_CHARS:], stderr[-TAIL_CHARS:])
