"""TEST INFRASTRUCTURE: a sequential interpreter of the Julia subset STADE's
generators write (the `_b.jl` / `_d.jl` / `_hv.jl` sweeps and their
initstacks functions), on numpy arrays.

It is the checker for the .cu emitter (stade.jl_b200/emitter): it runs a
generated sweep exactly as Julia would, statement by statement in loop order,
with Julia's integer division family (div truncates, mod takes the divisor's
sign), literal powers x^2 = x * x (Base.literal_pow), column-major
multi-dimensional indexing and 1-based subscripts. Float64 runs in Python
floats (IEEE double, one rounding per operation, libm functions); Float32
runs in numpy float32 scalars. It shares no code with the emitter.
"""
from __future__ import annotations

import math
import re

import numpy as np

_TOK = re.compile(r"""
    (?P<nl>\n|;)
  | (?P<ws>[ \t\r]+)
  | (?P<com>\#[^\n]*)
  | (?P<num>(?:\d+\.\d*|\.\d+|\d+)(?:[eEf][+-]?\d+)?)
  | (?P<name>[A-Za-z_@][A-Za-z0-9_!]*)
  | (?P<op>==|!=|<=|>=|&&|\|\||\+=|-=|\*=|/=|[-+*/^()\[\],=<>!:{}%])
""", re.X)


def tokenize(src):
    out, line, pos = [], 1, 0
    while pos < len(src):
        m = _TOK.match(src, pos)
        if not m:
            raise SyntaxError(f"line {line}: unexpected {src[pos]!r}")
        kind = m.lastgroup
        text = m.group()
        pos = m.end()
        if kind == "nl":
            if out and out[-1][0] != "nl":
                out.append(("nl", "\n", line))
            if text == "\n":
                line += 1
        elif kind in ("ws", "com"):
            continue
        else:
            out.append((kind, text, line))
            # a numeric literal coefficient (`0.5x`, `2(a + b)`) multiplies
            if kind == "num" and pos < len(src) and (src[pos].isalpha() or src[pos] in "_("):
                out.append(("op", "jux", line))
    out.append(("nl", "\n", line))
    out.append(("eof", "", line))
    return out


class _P:
    def __init__(self, toks):
        self.t, self.p = toks, 0

    def peek(self, o=0):
        return self.t[min(self.p + o, len(self.t) - 1)]

    def next(self):
        tok = self.t[self.p]
        self.p += 1
        return tok

    def op(self, s):
        k, v, _ = self.peek()
        return k == "op" and v == s

    def kw(self, s):
        k, v, _ = self.peek()
        return k == "name" and v == s

    def expect(self, s):
        if not self.op(s):
            raise SyntaxError(f"line {self.peek()[2]}: expected {s!r}, got {self.peek()[1]!r}")
        self.next()

    def nl(self):
        while self.peek()[0] == "nl":
            self.next()

    # program
    def funcs(self):
        fs = {}
        self.nl()
        while self.peek()[0] != "eof":
            if self.kw("function"):
                self.next()
                name = self.next()[1]
                self.expect("(")
                params = []
                while not self.op(")"):
                    params.append(self.next()[1])
                    if self.op(","):
                        self.next()
                self.next()
                body = self.block(("end",))
                self.next()
                fs[name] = (params, body)
            else:
                self.next()
            self.nl()
        return fs

    def block(self, stops):
        out = []
        while True:
            self.nl()
            if any(self.kw(s) for s in stops):
                return out
            out.append(self.stmt())

    def stmt(self):
        if self.peek()[1].startswith("@"):
            self.next()
            return self.stmt()
        if self.kw("for"):
            self.next()
            var = self.next()[1]
            self.next()  # = or in
            a = self.arith()
            self.expect(":")
            b = self.arith()
            if self.op(":"):
                self.next()
                lo, step, hi = a, b, self.arith()
            else:
                lo, step, hi = a, ("num", 1), b
            body = self.block(("end",))
            self.next()
            return ("for", var, lo, step, hi, body)
        if self.kw("while"):
            self.next()
            c = self.expr()
            body = self.block(("end",))
            self.next()
            return ("while", c, body)
        if self.kw("if"):
            self.next()
            return self.if_tail()
        if self.kw("return"):
            self.next()
            if self.peek()[0] == "nl" or self.kw("end"):
                return ("return", None)
            if self.kw("nothing"):
                self.next()
                return ("return", None)
            e = self.expr()
            if self.op(","):
                items = [e]
                while self.op(","):
                    self.next()
                    items.append(self.expr())
                e = ("tuple", items)
            return ("return", e)
        lhs = self.postfix()
        if self.op("="):
            self.next()
            return ("assign", lhs, self.expr())
        for op in ("+=", "-=", "*=", "/="):
            if self.op(op):
                self.next()
                return ("assign", lhs, ("bin", op[0], lhs, self.expr()))
        raise SyntaxError(f"line {self.peek()[2]}: bad statement")

    def if_tail(self):
        c = self.expr()
        then = self.block(("elseif", "else", "end"))
        els = []
        if self.kw("elseif"):
            self.next()
            els = [self.if_tail()]
            return ("if", c, then, els)
        if self.kw("else"):
            self.next()
            els = self.block(("end",))
        self.next()
        return ("if", c, then, els)

    def expr(self):
        l = self.land()
        while self.op("||"):
            self.next()
            l = ("bin", "||", l, self.land())
        return l

    def land(self):
        l = self.cmp()
        while self.op("&&"):
            self.next()
            l = ("bin", "&&", l, self.cmp())
        return l

    def cmp(self):
        l = self.arith()
        for op in ("==", "!=", "<=", ">=", "<", ">"):
            if self.op(op):
                self.next()
                return ("bin", op, l, self.arith())
        return l

    def arith(self):
        l = self.term()
        while self.op("+") or self.op("-"):
            op = self.next()[1]
            l = ("bin", op, l, self.term())
        return l

    def term(self):
        l = self.unary()
        while self.op("*") or self.op("/") or self.op("%"):
            op = self.next()[1]
            l = ("bin", op, l, self.unary())
        return l

    def unary(self):
        if self.op("-") or self.op("!") or self.op("+"):
            op = self.next()[1]
            e = self.unary()
            if op == "+":
                return e
            if op == "-" and e[0] == "num":
                return ("num", -e[1])
            return ("un", op, e)
        return self.power()

    def power(self):
        b = self.postfix()
        if b[0] == "num" and self.op("jux"):   # binds tighter than * and /, looser than ^
            self.next()
            return ("bin", "*", b, self.power())
        if self.op("^"):
            self.next()
            return ("bin", "^", b, self.unary())
        return b

    def postfix(self):
        e = self.primary()
        while True:
            if self.op("[") and e[0] == "var":
                self.next()
                idx = []
                while not self.op("]"):
                    idx.append(self.expr())
                    if self.op(","):
                        self.next()
                self.next()
                e = ("ref", e[1], idx)
            elif self.op("{") and e[0] == "var":
                self.next()
                ty = self.next()[1]
                self.expect("}")
                e = ("curly", ty)
            elif self.op("(") and e[0] in ("var", "curly"):
                self.next()
                args = []
                while not self.op(")"):
                    args.append(self.expr())
                    if self.op(","):
                        self.next()
                self.next()
                e = ("alloc", e[1], args) if e[0] == "curly" else ("call", e[1], args)
            else:
                return e

    def primary(self):
        k, v, line = self.next()
        if k == "num":
            if re.fullmatch(r"\d+", v):
                return ("num", int(v))
            return ("num", float(v.replace("f", "e")))
        if k == "name":
            if v in ("true", "false"):
                return ("num", 1 if v == "true" else 0)
            return ("var", v)
        if k == "op" and v == "(":
            e = self.expr()
            if self.op(","):
                items = [e]
                while self.op(","):
                    self.next()
                    if self.op(")"):
                        break
                    items.append(self.expr())
                self.expect(")")
                return ("tuple", items)
            self.expect(")")
            return e
        raise SyntaxError(f"line {line}: unexpected {v!r}")


class _Return(Exception):
    def __init__(self, value):
        self.value = value


def _jdiv(a, b):
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b > 0) else -q


def _fmax(a, b):
    if a != a:
        return a
    if b != b:
        return b
    if a == b:
        return b if math.copysign(1.0, float(a)) < 0 else a
    return a if a > b else b


def _fmin(a, b):
    if a != a:
        return a
    if b != b:
        return b
    if a == b:
        return a if math.copysign(1.0, float(a)) < 0 else b
    return a if a < b else b


class Interp:
    """Runs functions of one Julia source. precision 64 or 32; dims maps a
    multi-dimensional array's name to its leading extents (Julia expressions
    in the call's integer arguments)."""

    _FUN64 = dict(sqrt=math.sqrt, exp=math.exp, log=math.log, tanh=math.tanh, sin=math.sin,
                  cos=math.cos, tan=math.tan, sinh=math.sinh, cosh=math.cosh,
                  log2=math.log2, log10=math.log10, expm1=math.expm1, log1p=math.log1p,
                  atan=math.atan, asin=math.asin, acos=math.acos)

    def __init__(self, source, precision=64, dims=None):
        self.funcs = _P(tokenize(source)).funcs()
        self.f32 = precision == 32
        self.dims_src = dims or {}

    def _flt(self, x):
        return np.float32(x) if self.f32 else float(x)

    def call(self, name, *args):
        params, body = self.funcs[name]
        if len(args) != len(params):
            raise TypeError(f"{name} takes {len(params)} arguments, got {len(args)}")
        env = dict(zip(params, args))
        self.dims = {}
        for a, exprs in self.dims_src.items():
            self.dims[a] = [int(self.ev(_P(tokenize(e)).expr(), env)) for e in exprs]
        try:
            self.run(body, env)
        except _Return as r:
            return r.value
        return None

    def initstacks(self, name, *args):
        """Runs initstacks_<k> (closed-form sizes, or a Tier-B sizing loop
        filling prefix tables and totals); returns what it returns, arrays
        zero-filled where it does not write them."""
        params, body = self.funcs[name]
        env = dict(zip(params, args))
        self.dims = {}
        try:
            self.run(body, env)
        except _Return as r:
            v = r.value
            return () if v is None else (v if isinstance(v, tuple) else (v,))
        return ()

    def _off(self, name, idx, env):
        ix = [int(self.ev(i, env)) for i in idx]
        if len(ix) == 1:
            return ix[0] - 1
        d = self.dims[name]
        off, stride = ix[0] - 1, 1
        for k in range(1, len(ix)):
            stride *= d[k - 1]
            off += (ix[k] - 1) * stride
        return off

    def run(self, body, env):
        for st in body:
            k = st[0]
            if k == "assign":
                lhs, val = st[1], self.ev(st[2], env)
                if lhs[0] == "var":
                    env[lhs[1]] = val
                else:
                    o = self._off(lhs[1], lhs[2], env)
                    if o < 0:
                        raise IndexError(f"{lhs[1]}[{o + 1}]")
                    env[lhs[1]][o] = val
            elif k == "for":
                _, var, lo, step, hi, b = st
                lo, step, hi = int(self.ev(lo, env)), int(self.ev(step, env)), int(self.ev(hi, env))
                for v in range(lo, hi + (1 if step > 0 else -1), step):
                    env[var] = v
                    self.run(b, env)
            elif k == "while":
                while self.ev(st[1], env):
                    self.run(st[2], env)
            elif k == "if":
                self.run(st[2] if self.ev(st[1], env) else st[3], env)
            elif k == "return":
                e = st[1]
                if e is None:
                    raise _Return(None)
                if e[0] == "tuple":
                    raise _Return(tuple(self.ev(x, env) for x in e[1]))
                raise _Return(self.ev(e, env))

    def ev(self, e, env):
        k = e[0]
        if k == "alloc":   # Vector{T}(undef, n)
            n = max(0, int(self.ev(e[2][1], env)))
            return np.zeros(n, np.int64 if "Int" in e[1] else
                            (np.float32 if self.f32 else np.float64))
        if k == "num":
            return e[1] if isinstance(e[1], int) else self._flt(e[1])
        if k == "var":
            return env[e[1]]
        if k == "ref":
            o = self._off(e[1], e[2], env)
            if o < 0:
                raise IndexError(f"{e[1]}[{o + 1}]")
            v = env[e[1]][o]
            return int(v) if env[e[1]].dtype.kind == "i" else (v if self.f32 else float(v))
        if k == "un":
            v = self.ev(e[2], env)
            return (not v) if e[1] == "!" else -v
        if k == "bin":
            op = e[1]
            if op == "&&":
                return self.ev(e[2], env) and self.ev(e[3], env)
            if op == "||":
                return self.ev(e[2], env) or self.ev(e[3], env)
            a, b = self.ev(e[2], env), self.ev(e[3], env)
            if op == "+":
                return a + b
            if op == "-":
                return a - b
            if op == "*":
                return a * b
            if op == "/":
                return self._flt(a) / self._flt(b)
            if op == "%":
                return a - b * _jdiv(a, b)
            if op == "^":
                if e[3][0] == "num" and isinstance(e[3][1], int):
                    n = e[3][1]
                    if n == 2:
                        return a * a
                    if n == 3:
                        return a * a * a
                    if n == 1:
                        return a
                    if n == 0:
                        return 1 if isinstance(a, int) else self._flt(1.0)
                    if n == -1 and not isinstance(a, int):
                        return self._flt(1.0) / a
                    if isinstance(a, int) and n > 0:
                        return a ** n
                return self._flt(math.pow(float(a), float(b)))
            return {"==": a == b, "!=": a != b, "<": a < b, ">": a > b, "<=": a <= b,
                    ">=": a >= b}[op]
        if k == "call":
            name, args = e[1], [self.ev(x, env) for x in e[2]]
            if name == "length":
                return int(np.asarray(args[0]).size)
            if name == "div":
                return _jdiv(args[0], args[1])
            if name == "mod":
                return args[0] % args[1]
            if name == "rem":
                return args[0] - args[1] * _jdiv(args[0], args[1])
            if name in ("max", "min"):
                if all(isinstance(a, int) for a in args):
                    return max(args) if name == "max" else min(args)
                f = _fmax if name == "max" else _fmin
                acc = self._flt(args[0])
                for a in args[1:]:
                    acc = f(acc, self._flt(a))
                return acc
            if name == "abs":
                return abs(args[0]) if isinstance(args[0], int) else self._flt(abs(args[0]))
            if name == "sign":
                a = args[0]
                if isinstance(a, int):
                    return (a > 0) - (a < 0)
                return self._flt(1.0 if a > 0 else (-1.0 if a < 0 else a))
            if name in ("Float64", "Float32", "float"):
                return self._flt(args[0])
            if name in ("Int", "Int64"):
                return int(args[0])
            if name == "ifelse":
                return args[1] if args[0] else args[2]
            if name in self._FUN64:
                if self.f32:
                    return getattr(np, {"asin": "arcsin", "acos": "arccos",
                                        "atan": "arctan"}.get(name, name))(np.float32(args[0]))
                return self._FUN64[name](float(args[0]))
            raise NameError(f"function {name} is not in the subset")
        raise ValueError(f"cannot evaluate {e!r}")
