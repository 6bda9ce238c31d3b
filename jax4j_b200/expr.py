"""Elementwise expression trees (core/tensor/expr/Expr.java:25-35).

A fused chain is a DAG of Input / Unary / Binary / Scalar nodes over equal-length leaf buffers,
exactly the unit FusingBackend hands to ComputeBackend.fused. Nodes are immutable and compared
by identity, as the reference's records are used.

`postfix` flattens an expression into the int32 program the engine and the oracle both read:
  [0, input] | [1, op] (unary) | [2, op] (binary) | [3, op, lo32, hi32] (scalar, double value)
Shared sub-expressions are emitted once per use (the reference's CPU evaluator also recomputes
them); the engine's code generator deduplicates them by structure.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

OPS = ["ADD", "SUB", "MUL", "DIV", "MAX", "MIN", "NEG", "EXP", "LOG", "SQRT", "RSQRT", "TANH",
       "SIGMOID", "RELU", "ABS", "SIGN"]
OP = {name: i for i, name in enumerate(OPS)}
BINARY_OPS = set(OPS[:6])
UNARY_OPS = set(OPS[6:])


class Expr:
    __slots__ = ()

    def __hash__(self):
        return id(self)

    def __eq__(self, other):
        return self is other


@dataclass(frozen=True, eq=False)
class Input(Expr):
    index: int


@dataclass(frozen=True, eq=False)
class Unary(Expr):
    op: str
    a: Expr


@dataclass(frozen=True, eq=False)
class Binary(Expr):
    op: str
    a: Expr
    b: Expr


@dataclass(frozen=True, eq=False)
class Scalar(Expr):
    op: str
    a: Expr
    value: float


def postfix(expr: Expr) -> list[int]:
    out: list[int] = []

    def walk(e: Expr):
        if isinstance(e, Input):
            out.extend((0, e.index))
        elif isinstance(e, Unary):
            walk(e.a)
            out.extend((1, OP[e.op]))
        elif isinstance(e, Binary):
            walk(e.a)
            walk(e.b)
            out.extend((2, OP[e.op]))
        elif isinstance(e, Scalar):
            walk(e.a)
            lo, hi = struct.unpack("<ii", struct.pack("<d", float(e.value)))
            out.extend((3, OP[e.op], lo, hi))
        else:
            raise TypeError(f"not an expression: {e!r}")

    walk(expr)
    return out


def remap(expr: Expr, mapping: dict[int, int], memo: dict | None = None) -> Expr:
    """Rewrites input indices (FusingBackend.reindex, FusingBackend.java:338-365)."""
    memo = {} if memo is None else memo
    got = memo.get(id(expr))
    if got is not None:
        return got
    if isinstance(expr, Input):
        r = Input(mapping[expr.index])
    elif isinstance(expr, Unary):
        r = Unary(expr.op, remap(expr.a, mapping, memo))
    elif isinstance(expr, Binary):
        r = Binary(expr.op, remap(expr.a, mapping, memo), remap(expr.b, mapping, memo))
    else:
        r = Scalar(expr.op, remap(expr.a, mapping, memo), expr.value)
    memo[id(expr)] = r
    return r


def from_postfix(prog: list[int]) -> Expr:
    """The expression a postfix program encodes (inverse of `postfix`)."""
    stack: list[Expr] = []
    i = 0
    while i < len(prog):
        kind = prog[i]
        if kind == 0:
            stack.append(Input(prog[i + 1]))
            i += 2
        elif kind == 1:
            stack.append(Unary(OPS[prog[i + 1]], stack.pop()))
            i += 2
        elif kind == 2:
            b, a = stack.pop(), stack.pop()
            stack.append(Binary(OPS[prog[i + 1]], a, b))
            i += 2
        elif kind == 3:
            value = struct.unpack("<d", struct.pack("<ii", prog[i + 2], prog[i + 3]))[0]
            stack.append(Scalar(OPS[prog[i + 1]], stack.pop(), value))
            i += 4
        else:
            raise ValueError(f"bad postfix word {kind} at {i}")
    if len(stack) != 1:
        raise ValueError("postfix program does not reduce to one expression")
    return stack[0]
