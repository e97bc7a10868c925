"""Integer / predicate expressions over a task's symbols: portfolio guards and launch geometry.

One evaluator for both uses, with the rules of the reference's geometry plane
(tcenv/track/expr.py, module docstring and ``evaluate``), so that a guard or a grid means the same
thing on the B200 as in the reference's portfolio documents:

* a *term* is an integer, a name, a text expression (``"ceil_div(N, 256) + 1"``), a one-key
  mapping (``{"ceil_div": ["N", 256]}``) or a prefix list (``["eq", "K", 4096]``);
* text uses ``+ - * /``, parentheses, integer literals, names and calls of the closed function
  set: ``ceil_div``, ``trunc_div``, ``rem``, ``min``, ``max`` (integers), ``gt ge lt le eq ne``
  (comparisons) and ``and or not`` (predicates);
* ``/`` is exact integer division (an inexact or zero divisor is an error); ``trunc_div`` and
  ``rem`` truncate toward zero (the remainder has the dividend's sign); ``ceil_div`` needs a
  positive divisor;
* every expression is statically typed (``int`` or ``bool``), a name the caller does not supply
  is an error, and nothing is ever defaulted.

``digest`` hashes a canonical form (commutative operands sorted, nested ``and``/``or``/``+``/``*``
/``min``/``max`` flattened), so two spellings of one guard share a digest.
"""

from __future__ import annotations

import hashlib
import json
import re
from dataclasses import dataclass
from typing import Any, Mapping, Union

INT = "int"
BOOL = "bool"

# name -> (min args, max args or None)
FUNCTIONS: dict[str, tuple[int, int | None]] = {
    "ceil_div": (2, 2), "trunc_div": (2, 2), "rem": (2, 2), "min": (1, None), "max": (1, None),
    "gt": (2, 2), "ge": (2, 2), "lt": (2, 2), "le": (2, 2), "eq": (2, 2), "ne": (2, 2),
    "and": (2, None), "or": (2, None), "not": (1, 1),
}
OPERATORS = ("+", "-", "*", "/")
COMPARISONS = frozenset({"gt", "ge", "lt", "le", "eq", "ne"})
PREDICATES = COMPARISONS | {"and", "or", "not"}
_FLATTEN = frozenset({"and", "or", "+", "*", "min", "max"})
_COMMUTATIVE = _FLATTEN | {"eq", "ne"}
_NAME = re.compile(r"[A-Za-z_][A-Za-z0-9_]*")
_TOKEN = re.compile(r"\s*(?:(\d+)|([A-Za-z_][A-Za-z0-9_]*)|(.))")


class ExprError(ValueError):
    """A term that does not parse, is ill-typed, or cannot be evaluated on the given names."""


@dataclass(frozen=True)
class Num:
    value: int


@dataclass(frozen=True)
class Name:
    name: str


@dataclass(frozen=True)
class Apply:
    func: str
    args: tuple


Node = Union[Num, Name, Apply]


# ---- parsing ----------------------------------------------------------------------------------


def parse(term: Any, where: str = "term") -> Node:
    if isinstance(term, bool):
        raise ExprError(f"{where}: a boolean literal is not a term (write a comparison)")
    if isinstance(term, int):
        return Num(int(term))
    if isinstance(term, str):
        text = term.strip()
        if not text:
            raise ExprError(f"{where}: empty expression")
        return Name(text) if _NAME.fullmatch(text) else _Text(text, where).parse()
    if isinstance(term, Mapping):
        if len(term) != 1:
            raise ExprError(f"{where}: a function mapping needs exactly one key, got {sorted(term)}")
        (func, args), = term.items()
        return _apply(str(func), args if isinstance(args, (list, tuple)) else [args], where)
    if isinstance(term, (list, tuple)):
        if not term or not isinstance(term[0], str):
            raise ExprError(f"{where}: a prefix list starts with a function or operator name")
        return _apply(term[0], list(term[1:]), where)
    raise ExprError(f"{where}: {type(term).__name__} is not a term")


def _apply(func: str, args: list, where: str) -> Node:
    nodes = tuple(a if isinstance(a, (Num, Name, Apply)) else parse(a, f"{where}.{func}[{i}]") for i, a in enumerate(args))
    if func in OPERATORS:
        if len(nodes) == 1 and func == "-":
            return Apply("-", nodes)
        if len(nodes) == 1 and func == "+":
            return nodes[0]
        if len(nodes) != 2:
            raise ExprError(f"{where}: operator {func!r} takes two operands, got {len(nodes)}")
        return Apply(func, nodes)
    if func not in FUNCTIONS:
        raise ExprError(f"{where}: unknown function {func!r}; the closed set is {sorted(FUNCTIONS)}")
    lo, hi = FUNCTIONS[func]
    if len(nodes) < lo or (hi is not None and len(nodes) > hi):
        raise ExprError(f"{where}: {func}() takes {lo}..{hi if hi is not None else 'n'} arguments, got {len(nodes)}")
    return Apply(func, nodes)


class _Text:
    """Recursive descent over ``sum := product (('+'|'-') product)*``, ``product := unary
    (('*'|'/') unary)*``, ``unary := '-' unary | atom``, ``atom := INT | NAME | NAME '(' args ')'
    | '(' sum ')'``."""

    def __init__(self, text: str, where: str) -> None:
        self.text, self.where = text, where
        self.tokens: list[tuple[str, str]] = []
        pos = 0
        while pos < len(text):
            m = _TOKEN.match(text, pos)
            if m is None or m.end() == pos:
                break
            pos = m.end()
            num, name, sym = m.groups()
            if num is not None:
                self.tokens.append(("num", num))
            elif name is not None:
                self.tokens.append(("name", name))
            elif sym is not None and sym.strip():
                if sym not in "+-*/(),":
                    raise ExprError(f"{where}: unexpected character {sym!r} in `{text}`")
                self.tokens.append(("sym", sym))
        self.i = 0

    def _peek(self) -> tuple[str, str] | None:
        return self.tokens[self.i] if self.i < len(self.tokens) else None

    def _take(self, want: str | None = None) -> tuple[str, str]:
        tok = self._peek()
        if tok is None:
            raise ExprError(f"{self.where}: `{self.text}` ends early")
        if want is not None and tok[1] != want:
            raise ExprError(f"{self.where}: `{self.text}` expected {want!r}, got {tok[1]!r}")
        self.i += 1
        return tok

    def parse(self) -> Node:
        node = self._sum()
        if self._peek() is not None:
            raise ExprError(f"{self.where}: trailing {self._peek()[1]!r} in `{self.text}`")
        return node

    def _sum(self) -> Node:
        node = self._product()
        while self._peek() in (("sym", "+"), ("sym", "-")):
            op = self._take()[1]
            node = Apply(op, (node, self._product()))
        return node

    def _product(self) -> Node:
        node = self._unary()
        while self._peek() in (("sym", "*"), ("sym", "/")):
            op = self._take()[1]
            node = Apply(op, (node, self._unary()))
        return node

    def _unary(self) -> Node:
        if self._peek() == ("sym", "-"):
            self._take()
            return Apply("-", (self._unary(),))
        return self._atom()

    def _atom(self) -> Node:
        kind, val = self._take()
        if kind == "num":
            return Num(int(val))
        if kind == "name":
            if self._peek() == ("sym", "("):
                self._take("(")
                args: list[Node] = []
                if self._peek() != ("sym", ")"):
                    args.append(self._sum())
                    while self._peek() == ("sym", ","):
                        self._take(",")
                        args.append(self._sum())
                self._take(")")
                return _apply(val, args, self.where)
            return Name(val)
        if val == "(":
            node = self._sum()
            self._take(")")
            return node
        raise ExprError(f"{self.where}: unexpected {val!r} in `{self.text}`")


# ---- typing and evaluation ----------------------------------------------------------------------


def kind(node: Node) -> str:
    if isinstance(node, (Num, Name)):
        return INT
    want = BOOL if node.func in ("and", "or", "not") else INT
    for i, arg in enumerate(node.args):
        if kind(arg) != want:
            raise ExprError(f"{node.func}() argument {i} must be {'a predicate' if want == BOOL else 'an integer'}")
    return BOOL if node.func in PREDICATES else INT


def names(node: Node) -> set[str]:
    if isinstance(node, Name):
        return {node.name}
    if isinstance(node, Num):
        return set()
    out: set[str] = set()
    for a in node.args:
        out |= names(a)
    return out


def _div_trunc(a: int, b: int) -> int:
    q = abs(a) // abs(b)
    return -q if (a < 0) != (b < 0) else q


def evaluate(node: Node, env: Mapping[str, int]) -> int | bool:
    if isinstance(node, Num):
        return node.value
    if isinstance(node, Name):
        if node.name not in env:
            raise ExprError(f"name {node.name!r} is not declared here; declared: {sorted(env)}")
        v = env[node.name]
        if isinstance(v, bool) or not isinstance(v, int):
            raise ExprError(f"name {node.name!r} is not an integer")
        return v
    f = node.func
    # Every operand is evaluated (no short circuit): an operand that cannot be evaluated makes
    # the whole guard an error, whatever the other operands say.
    v = [evaluate(a, env) for a in node.args]
    if f == "and":
        return all(v)
    if f == "or":
        return any(v)
    if f == "not":
        return not v[0]
    if f in COMPARISONS:
        a, b = v
        return {"gt": a > b, "ge": a >= b, "lt": a < b, "le": a <= b, "eq": a == b, "ne": a != b}[f]
    if f == "+":
        return v[0] + v[1]
    if f == "-":
        return -v[0] if len(v) == 1 else v[0] - v[1]
    if f == "*":
        return v[0] * v[1]
    if f == "/":
        if v[1] == 0 or v[0] % v[1] != 0:
            raise ExprError(f"{v[0]} / {v[1]} is not an exact integer division")
        return v[0] // v[1]
    if f == "ceil_div":
        if v[1] <= 0:
            raise ExprError("ceil_div() needs a positive divisor")
        return -((-v[0]) // v[1])
    if f in ("trunc_div", "rem"):
        if v[1] == 0:
            raise ExprError(f"{f}() divisor is zero")
        q = _div_trunc(v[0], v[1])
        return q if f == "trunc_div" else v[0] - q * v[1]
    if f == "min":
        return min(v)
    if f == "max":
        return max(v)
    raise ExprError(f"unknown function {f!r}")  # parse() closes the set


def evaluate_term(term: Any, env: Mapping[str, int], *, expect: str = INT, where: str = "term") -> int | bool:
    node = parse(term, where)
    got = kind(node)
    if got != expect:
        raise ExprError(f"{where}: expected a{'n' if expect == INT else ''} {expect} expression, got {got}")
    return evaluate(node, env)


# ---- canonical form -----------------------------------------------------------------------------


def canonical(node: Node) -> Any:
    """Prefix-list document with nested associative calls flattened and commutative operands
    sorted by their JSON text."""
    if isinstance(node, Num):
        return node.value
    if isinstance(node, Name):
        return node.name
    args = []
    for a in node.args:
        c = canonical(a)
        if node.func in _FLATTEN and isinstance(c, list) and c[0] == node.func:
            args.extend(c[1:])
        else:
            args.append(c)
    if node.func in _COMMUTATIVE:
        args.sort(key=lambda x: json.dumps(x, sort_keys=True))
    return [node.func, *args]


def digest(term: Any, where: str = "guard") -> str:
    node = parse(term, where)
    doc = json.dumps(canonical(node), sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(doc.encode()).hexdigest()


def guard(term: Any, where: str = "guard") -> Node:
    """Parse a guard: the term must be a predicate."""
    node = parse(term, where)
    if kind(node) != BOOL:
        raise ExprError(f"{where}: a guard must be a predicate, got an integer expression")
    return node
