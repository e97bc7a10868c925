"""Portfolio shards evaluated one GPU per shard: one worker process per device of the node.

The reference's portfolio runner measures a portfolio's benchmark points one after another on
its one device (tcenv/taskcontract/portfolio_runner.py:888).  The points are independent, so on a
B200 node they are dealt to the GPUs by a longest-processing-time balance over each point's size
(``point_cost``), and each GPU gets one spawned worker process whose ``CUDA_VISIBLE_DEVICES`` is
pinned to it before CUDA initialises.  A worker builds, runs, verifies and times its points with
``portfolio_pack.measure`` (each timing under its own GPU's lock, ``gpulock`` keys locks by the
physical GPU), and sends its shard runs back; the parent merges them, in the order of the domain,
into the list one ``portfolio_pack.performance`` report is made from.  No collective is involved.

What a worker needs besides the parent and the points (input generation, the timing baseline and
the verifier) comes from a *recipe*: ``"package.module:function"`` plus keyword arguments, called
inside the worker and returning ``{"make_inputs": ..., "baseline": ..., "verify": ...}`` as
``portfolio_pack.measure`` takes them, so nothing unpicklable crosses the process boundary.
"""

from __future__ import annotations

import importlib
import os
import time
import traceback
from typing import Any, Mapping, Sequence

DEFAULT_MEASURE = "shapeforge_b200.portfolio_pack:measure"


class FanoutError(RuntimeError):
    """A worker failed (its traceback is the message) or did not answer in time."""


def _resolve(path: str):
    mod, _, name = path.partition(":")
    if not mod or not name:
        raise ValueError(f"expected 'package.module:function', got {path!r}")
    return getattr(importlib.import_module(mod), name)


def point_cost(point: Any) -> float:
    """Size of a shard point for the balance: the product of its integer symbols (a list, such as
    varlen sequence lengths, counts by its sum)."""
    cost = 1.0
    for v in point.names.values():
        if isinstance(v, bool):
            continue
        if isinstance(v, int):
            cost *= max(1, v)
        elif isinstance(v, (list, tuple)) and all(isinstance(x, int) for x in v):
            cost *= max(1, sum(v))
    return cost


def device_masks(count: int | None = None) -> list[str]:
    """``CUDA_VISIBLE_DEVICES`` value of each worker: this process's visible GPUs, one each."""
    mask = os.environ.get("CUDA_VISIBLE_DEVICES")
    if mask is not None and mask.strip():
        entries = [e.strip() for e in mask.split(",") if e.strip()]
    else:
        if count is None:
            import torch

            count = torch.cuda.device_count()
        entries = [str(i) for i in range(count)]
    return entries if count is None else entries[:count]


def _worker(mask: str, job: Mapping[str, Any], conn) -> None:
    os.environ["CUDA_VISIBLE_DEVICES"] = mask  # before anything in this process initialises CUDA
    try:
        from .portfolio_pack import Parent

        recipe = _resolve(job["recipe"])(**job["recipe_kwargs"])
        measure = _resolve(job["measure"])
        parent = Parent.from_json(job["parent_json"])
        runs = measure(parent, job["opspec"], job["points"], reps=job["reps"], **recipe)
        conn.send(("ok", mask, runs))
    except BaseException:  # noqa: BLE001 - every failure is reported to the parent
        conn.send(("error", mask, traceback.format_exc()))
    finally:
        conn.close()


def measure_on_gpus(parent: Any, opspec: Mapping[str, Any], points: Sequence[Any], *, recipe: str,
                    recipe_kwargs: Mapping[str, Any] | None = None, devices: Sequence[str] | None = None, reps: int = 15,
                    measure: str = DEFAULT_MEASURE, timeout_s: float = 3600.0) -> list[Any]:
    """Measure the benchmark points of ``points`` with one worker per GPU; returns the shard runs
    in domain order (one per benchmark point).

    ``devices`` are the workers' ``CUDA_VISIBLE_DEVICES`` values (default: every GPU this process
    sees, ``device_masks()``); at most one worker per benchmark point is started.  ``timeout_s``
    bounds the whole fan-out: a worker that has not answered by then is killed and reported."""
    import multiprocessing as mp

    bench = [p for p in points if p.usage == "benchmark"]
    if not bench:
        return []
    masks = list(devices) if devices is not None else device_masks()
    if not masks:
        raise FanoutError("no GPU to run on")
    masks = masks[: len(bench)]
    parts = balance(points, len(masks))
    ctx = mp.get_context("spawn")
    procs = []
    for mask, part in zip(masks, parts):
        if not part:
            continue
        job = {"recipe": recipe, "recipe_kwargs": dict(recipe_kwargs or {}), "measure": measure, "parent_json": parent.to_json(),
               "opspec": dict(opspec), "points": [bench[i] for i in part], "reps": int(reps)}
        recv, send = ctx.Pipe(duplex=False)
        proc = ctx.Process(target=_worker, args=(mask, job, send), daemon=True)
        proc.start()
        send.close()
        procs.append((mask, proc, recv))
    results: dict[str, Any] = {}
    errors = []
    deadline = time.monotonic() + timeout_s  # one limit for the whole fan-out, not per worker
    for mask, proc, recv in procs:
        try:
            if not recv.poll(max(0.0, deadline - time.monotonic())):
                errors.append(f"GPU {mask}: no answer within {timeout_s:.0f} s")
                proc.kill()
                continue
            status, _, payload = recv.recv()
        except EOFError:
            status, payload = "error", f"worker exited with code {proc.exitcode} before answering"
        finally:
            proc.join(timeout=60)
        if status == "ok":
            for run in payload:
                results[run.point.instance_key] = run
        else:
            errors.append(f"GPU {mask}:\n{payload}")
    if errors:
        raise FanoutError("portfolio worker failed:\n" + "\n".join(errors))
    missing = [p.instance_key for p in bench if p.instance_key not in results]
    if missing:
        raise FanoutError(f"no shard run for {missing}")
    return [results[p.instance_key] for p in bench]


def balance(points: Sequence[Any], workers: int) -> list[list[int]]:
    """The assignment ``measure_on_gpus`` uses: benchmark-point indices per worker."""
    from .shard import lpt_assign

    bench = [p for p in points if p.usage == "benchmark"]
    return lpt_assign([point_cost(p) for p in bench], max(1, min(workers, len(bench)))) if bench else []


