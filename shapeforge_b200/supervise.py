"""Supervised evaluation: one worker process per candidate evaluation, heartbeats, deadlines.

Restates the supervision of tcenv/evaluate.py ``supervise`` (:1143) and tcenv/v2_worker.py
``run_bounded_v2`` (:450): the parent owns every deadline, the worker only overwrites one
heartbeat record (the reference's fixed 22-byte form, :mod:`shapeforge_b200.heartbeat`) through the
backend's compile / launch hooks and the GPU lock's wait hooks:

* ``C`` — compiling: the worker is killed when one compile is older than ``compile_deadline_s``;
* ``B`` — inside a GPU launch (or a synchronising call): killed when older than ``launch_deadline_s``;
* ``W`` — queued for the GPU lock: that time does not count toward the evaluation's ``timeout``;
* ``E`` — anything else (the evaluation's own time counts).

The worker runs in its own process group and the parent kills the whole group (the kernel then
releases the worker's GPU lock).  A kill is the typed status ``timeout`` (with the reason
``compile`` / ``launch`` / ``timeout``), a worker that exits without a report is ``crash``, a worker
whose callable raised reports ``runtime_error``.  Nothing here faults or hangs a GPU: the B200
kernels' own waits are bounded; supervision is the outer bound for candidate code that is not.

The worker is ``python -m shapeforge_b200.supervise <request.json>``; the request names a callable
``"module:function"`` taking the payload's ``args`` and returning a JSON-able report.
"""

from __future__ import annotations

import importlib
import json
import os
import signal
import subprocess
import sys
import tempfile
import time
import traceback
from pathlib import Path
from typing import Any, Mapping

from .heartbeat import HeartbeatFile, read

COMPILE_DEADLINE_S = 600.0
LAUNCH_DEADLINE_S = 10.0
KILL_WAIT_S = 10.0


Heartbeat = HeartbeatFile
read_heartbeat = read


def popen_group(cmd: list[str], **kw: Any) -> subprocess.Popen:
    """Start ``cmd`` as the leader of a new process group (killable as a whole)."""
    return subprocess.Popen(cmd, start_new_session=True, **kw)


def kill_group(proc: subprocess.Popen) -> None:
    if proc.poll() is None:
        try:
            os.killpg(proc.pid, signal.SIGKILL)
        except (ProcessLookupError, PermissionError):
            pass
    try:
        proc.wait(timeout=KILL_WAIT_S)
    except subprocess.TimeoutExpired:
        pass


def supervise(proc: subprocess.Popen, hb_path: str | Path, *, launch_deadline_s: float, timeout: float,
              compile_deadline_s: float = COMPILE_DEADLINE_S, poll_s: float = 0.05) -> str:
    """Wait for ``proc``; kill its group when a compile, a launch or the whole evaluation (lock
    waits excluded) is too old.  Returns "" when it exited by itself, else the reason."""
    t0 = last = time.monotonic()
    paused = 0.0
    while proc.poll() is None:
        time.sleep(poll_s)
        now = time.monotonic()
        hb = read_heartbeat(hb_path)
        if hb and hb[0] == "W":
            paused += now - last
        last = now
        reason = ""
        if hb and hb[0] == "C" and time.time() - hb[1] > compile_deadline_s:
            reason = "compile"
        elif hb and hb[0] == "B" and time.time() - hb[1] > launch_deadline_s:
            reason = "launch"
        elif now - t0 - paused > timeout:
            reason = "timeout"
        if reason:
            kill_group(proc)
            return reason
    return ""


def run_bounded(target: str, args: Mapping[str, Any] | None = None, *, timeout: float,
                launch_deadline_s: float = LAUNCH_DEADLINE_S, compile_deadline_s: float = COMPILE_DEADLINE_S,
                env: Mapping[str, str] | None = None) -> dict[str, Any]:
    """Run ``target`` (``"module:function"``) with ``args`` in a supervised worker; return its report
    or the typed failure."""
    root_dir = Path(__file__).resolve().parents[1]
    with tempfile.TemporaryDirectory(prefix="sf_worker_") as td:
        root = Path(td)
        req = {"target": target, "args": dict(args or {}), "out": str(root / "report.json"), "heartbeat": str(root / "heartbeat")}
        (root / "request.json").write_text(json.dumps(req), encoding="utf-8")
        penv = dict(os.environ, **(env or {}))
        penv["PYTHONPATH"] = str(root_dir) + os.pathsep + penv.get("PYTHONPATH", "")
        with open(root / "stderr.txt", "w") as err:
            proc = popen_group([sys.executable, "-m", "shapeforge_b200.supervise", str(root / "request.json")], stdout=err,
                               stderr=err, env=penv, cwd=str(root_dir))
            try:
                reason = supervise(proc, req["heartbeat"], launch_deadline_s=launch_deadline_s, timeout=timeout,
                                   compile_deadline_s=compile_deadline_s)
            finally:
                kill_group(proc)
        tail = (root / "stderr.txt").read_text(errors="replace")[-2000:]
        if reason:
            return {"status": "timeout", "reason": reason, "stderr_tail": tail}
        out = root / "report.json"
        if not out.is_file():
            return {"status": "crash", "returncode": proc.returncode, "stderr_tail": tail}
        return json.loads(out.read_text(encoding="utf-8"))


def _worker_main(request_path: str) -> int:
    req = json.loads(Path(request_path).read_text(encoding="utf-8"))
    hb = HeartbeatFile(req["heartbeat"])
    hb.mark("E")
    hb.install()  # compiles C, launches B, lock waits W (excluded from the timeout)
    module, func = req["target"].split(":")
    try:
        report = getattr(importlib.import_module(module), func)(heartbeat=hb, **req["args"])
    except Exception as exc:  # noqa: BLE001 - the candidate's failure, typed
        report = {"status": "runtime_error", "detail": f"{type(exc).__name__}: {exc}", "traceback": traceback.format_exc()[-4000:]}
    hb.mark("E")
    tmp = Path(req["out"] + ".tmp")
    tmp.write_text(json.dumps(report), encoding="utf-8")
    os.replace(tmp, req["out"])
    return 0


if __name__ == "__main__":
    raise SystemExit(_worker_main(sys.argv[1]))
