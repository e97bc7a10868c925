"""int32 block-program evaluator of the sem_int tasks (test infrastructure only).

Restates ``evaluate`` of tasks/sem_int_1/reference.py:148-233 (identical in sem_int_2..7): the
program document's statements are evaluated element-wise in int64 over blocks of ``block``
elements, values of the kinds listed in ``rules.wrap_kinds`` wrap to int32 two's complement,
``sum``/``min``/``max`` reduce over each block, ``loop`` wraps the product of every round, and
the final projection XORs the ``final`` values and adds ``idx & index_mask`` with a wrap.
"""

from __future__ import annotations

import numpy as np

_CMP = {"<": np.less, ">": np.greater, "<=": np.less_equal, ">=": np.greater_equal, "==": np.equal, "!=": np.not_equal}


def wrap(v: np.ndarray) -> np.ndarray:
    """int64 -> int32 two's complement, kept in int64."""
    return ((np.asarray(v, dtype=np.int64) + (1 << 31)) & 0xFFFFFFFF) - (1 << 31)


def evaluate(document: dict, x: np.ndarray, y: np.ndarray, k: int) -> np.ndarray:
    rules = document["rules"]
    block = int(document["block"])
    wrap_kinds = set(rules["wrap_kinds"])
    hash_shift, loop_shift = int(rules["hash_shift"]), int(rules["loop_shift"])
    index_mask, mod_mask = int(rules["index_mask"]), int(rules["mod_mask"])
    n = x.size
    p = n // block
    env = {
        "xv": np.asarray(x, dtype=np.int64).reshape(p, block),
        "yv": np.asarray(y, dtype=np.int64).reshape(p, block),
        "idx": wrap(np.arange(n, dtype=np.int64).reshape(p, block)),
        "K": np.full((p, 1), int(k), dtype=np.int64),
    }

    def w(kind, v):
        return wrap(v) if kind in wrap_kinds else v

    for st in document["statements"]:
        kind, dst = st["kind"], st["dst"]
        a = env[st["a"]] if "a" in st else None
        if kind in ("bin", "sbin"):
            b = env[st["b"]] if st.get("b") else np.int64(st["const"])
            op = st["op"]
            r = {"+": lambda: a + b, "-": lambda: a - b, "*": lambda: a * b, "^": lambda: a ^ b, "&": lambda: a & b,
                 "|": lambda: a | b}[op]()
            env[dst] = w(kind, r)
        elif kind == "shl":
            env[dst] = w(kind, a << int(st["const"]))
        elif kind == "shr":
            env[dst] = w(kind, a >> int(st["const"]))
        elif kind == "mod":
            env[dst] = w(kind, (a & mod_mask) % int(st["const"]))
        elif kind == "where":
            env[dst] = w(kind, np.where(_CMP[st["op"]](a, env[st["b"]]), env[st["c"]], env[st["d"]]))
        elif kind == "neg":
            env[dst] = w(kind, -a)
        elif kind == "hash":
            env[dst] = w(kind, (a ^ (a >> hash_shift)) * int(st["const"]))
        elif kind == "loop":
            acc = a
            b = env[st["b"]]
            for _ in range(int(st["rounds"])):
                acc = wrap(wrap(acc * int(st["const"])) + b) ^ (acc >> loop_shift)
            env[dst] = w(kind, acc)
        elif kind == "sum":
            env[dst] = w(kind, a.sum(axis=1, keepdims=True))
        elif kind == "max":
            env[dst] = w(kind, a.max(axis=1, keepdims=True))
        elif kind == "min":
            env[dst] = w(kind, a.min(axis=1, keepdims=True))
        else:
            raise ValueError(f"unknown statement kind {kind!r}")
    res = env[document["final"][0]]
    for name in document["final"][1:]:
        res = res ^ env[name]
    res = wrap(res + (env["idx"] & index_mask))
    return res.reshape(-1).astype(np.int32)
