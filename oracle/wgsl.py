"""A small interpreter for the compute-shader subset of WGSL that the
reference's llama runtime uses (src/lib/llama-wgsl-runtime.ts): test
infrastructure that runs the reference's own shader text on the CPU, so the
C oracle's restatement of each kernel can be checked against it
(tests/golden/make_wgsl_golden.py writes the vectors it produces).  It is
not part of the product and nothing in the product imports it.

Supported: struct declarations; module-scope `var` in the storage, uniform
and workgroup address spaces (with @group/@binding); functions with
parameters and return values; `let`, `var`, `const`; assignment and the
compound operators; `if`/`else`, `for`, `loop`, `while`, `break`,
`continue`, `return`; the scalar types u32, i32, f32 and bool, vec2/3/4 and
fixed or runtime-sized arrays; the builtins select, min, max, clamp, abs,
floor, exp, pow, sin, cos, sqrt, inverseSqrt, tanh, unpack2x16float,
workgroupBarrier and the type conversions.

Semantics: every f32 operation is rounded to IEEE single (numpy float32);
u32 arithmetic wraps at 2^32 and i32 at 2^31; shift counts are taken modulo
32.  Transcendental builtins are evaluated in double and rounded once (the
WGSL specification leaves their last bits to the implementation, so results
through them are compared with a tolerance).  A dispatch runs each
workgroup's invocations as generators, advancing every one of them up to
its next workgroupBarrier before any passes it.
"""
from __future__ import annotations

import math
import re
from typing import Any, Dict, List, Optional, Tuple

import numpy as np

# ---------------------------------------------------------------------------
# Lexer

_TOKEN = re.compile(r"""
    (?P<ws>\s+|//[^\n]*|/\*.*?\*/)
  | (?P<num>0[xX][0-9a-fA-F]+[iu]?|(?:\d+\.\d*|\.\d+|\d+)(?:[eE][+-]?\d+)?[fhiu]?)
  | (?P<id>[A-Za-z_][A-Za-z0-9_]*)
  | (?P<op><<=|>>=|->|&&|\|\||<<|>>|<=|>=|==|!=|\+=|-=|\*=|/=|%=|&=|\|=|\^=|\+\+|--|[-+*/%&|^~!<>=(){}\[\],;:.@])
""", re.VERBOSE | re.DOTALL)


def tokenize(src: str) -> List[Tuple[str, str]]:
    out, i = [], 0
    while i < len(src):
        m = _TOKEN.match(src, i)
        if not m:
            raise SyntaxError(f"WGSL: cannot read {src[i:i + 20]!r}")
        i = m.end()
        kind = m.lastgroup
        if kind != "ws":
            out.append((kind, m.group(kind)))
    out.append(("eof", ""))
    return out


# ---------------------------------------------------------------------------
# Types: ("scalar", name) | ("vec", n, elem) | ("array", elem, count or None)
# | ("struct", name)

SCALARS = ("u32", "i32", "f32", "bool")


class Parser:
    def __init__(self, src: str):
        self.t = tokenize(src)
        self.i = 0

    # token helpers
    def peek(self, k: int = 0) -> Tuple[str, str]:
        return self.t[self.i + k]

    def next(self) -> Tuple[str, str]:
        tok = self.t[self.i]
        self.i += 1
        return tok

    def accept(self, v: str) -> bool:
        if self.t[self.i][1] == v and self.t[self.i][0] in ("op", "id"):
            self.i += 1
            return True
        return False

    def expect(self, v: str) -> None:
        if not self.accept(v):
            raise SyntaxError(f"WGSL: expected {v!r}, found {self.peek()[1]!r}")

    def ident(self) -> str:
        kind, v = self.next()
        if kind != "id":
            raise SyntaxError(f"WGSL: expected a name, found {v!r}")
        return v

    # module
    def module(self) -> Dict[str, Any]:
        mod = {"structs": {}, "vars": [], "fns": {}, "consts": []}
        while self.peek()[0] != "eof":
            attrs = self.attributes()
            kw = self.peek()[1]
            if kw == "struct":
                self.next()
                name = self.ident()
                self.expect("{")
                fields = []
                while not self.accept("}"):
                    self.attributes()
                    fname = self.ident()
                    self.expect(":")
                    fields.append((fname, self.type_()))
                    self.accept(",")
                self.accept(";")
                mod["structs"][name] = fields
            elif kw == "var":
                self.next()
                space = access = None
                if self.accept("<"):
                    space = self.ident()
                    if self.accept(","):
                        access = self.ident()
                    self.expect(">")
                name = self.ident()
                ty = None
                if self.accept(":"):
                    ty = self.type_()
                init = self.expr() if self.accept("=") else None
                self.expect(";")
                mod["vars"].append({"name": name, "space": space or "private", "access": access, "type": ty,
                                    "init": init, "attrs": attrs})
            elif kw in ("const", "override", "let"):
                self.next()
                name = self.ident()
                ty = self.type_() if self.accept(":") else None
                self.expect("=")
                mod["consts"].append((name, ty, self.expr()))
                self.expect(";")
            elif kw == "fn":
                self.next()
                name = self.ident()
                self.expect("(")
                params = []
                while not self.accept(")"):
                    pattrs = self.attributes()
                    pname = self.ident()
                    self.expect(":")
                    params.append((pname, self.type_(), pattrs))
                    self.accept(",")
                ret = None
                if self.accept("->"):
                    self.attributes()
                    ret = self.type_()
                mod["fns"][name] = {"params": params, "ret": ret, "body": self.block(), "attrs": attrs}
            else:
                raise SyntaxError(f"WGSL: unexpected {kw!r} at module scope")
        return mod

    def attributes(self) -> Dict[str, list]:
        attrs = {}
        while self.accept("@"):
            name = self.ident()
            args = []
            if self.accept("("):
                while not self.accept(")"):
                    args.append(self.expr())
                    self.accept(",")
            attrs[name] = args
        return attrs

    def type_(self) -> tuple:
        name = self.ident()
        if name in SCALARS:
            return ("scalar", name)
        m = re.fullmatch(r"vec([234])([fiu]?)", name)
        if m:
            n = int(m.group(1))
            if m.group(2):
                return ("vec", n, {"f": "f32", "i": "i32", "u": "u32"}[m.group(2)])
            self.expect("<")
            elem = self.type_()[1]
            self.expect(">")
            return ("vec", n, elem)
        if name == "array":
            self.expect("<")
            elem = self.type_()
            count = None
            if self.accept(","):
                count = self.expr(7)     # above the comparisons: '>' closes the type
            self.expect(">")
            return ("array", elem, count)
        if name == "atomic":
            raise SyntaxError("WGSL: atomics are not supported")
        return ("struct", name)

    # statements
    def block(self) -> list:
        self.expect("{")
        body = []
        while not self.accept("}"):
            body.append(self.statement())
        return body

    def statement(self) -> tuple:
        kw = self.peek()[1]
        if kw == "{":
            return ("block", self.block())
        if kw in ("let", "var", "const"):
            self.next()
            if kw == "var" and self.accept("<"):
                self.ident()
                self.expect(">")
            name = self.ident()
            ty = self.type_() if self.accept(":") else None
            init = self.expr() if self.accept("=") else None
            self.expect(";")
            return ("decl", kw, name, ty, init)
        if kw == "if":
            self.next()
            cond = self.expr()
            then = self.block()
            other = None
            if self.accept("else"):
                other = [self.statement()] if self.peek()[1] == "if" else self.block()
            return ("if", cond, then, other)
        if kw == "for":
            self.next()
            self.expect("(")
            init = None if self.peek()[1] == ";" else self.simple_statement()
            self.expect(";")
            cond = None if self.peek()[1] == ";" else self.expr()
            self.expect(";")
            upd = None if self.peek()[1] == ")" else self.simple_statement()
            self.expect(")")
            return ("for", init, cond, upd, self.block())
        if kw == "while":
            self.next()
            cond = self.expr()
            return ("for", None, cond, None, self.block())
        if kw == "loop":
            self.next()
            return ("for", None, None, None, self.block())
        if kw in ("break", "continue"):
            self.next()
            if kw == "break" and self.accept("if"):
                cond = self.expr()
                self.expect(";")
                return ("if", cond, [("break",)], None)
            self.expect(";")
            return (kw,)
        if kw == "return":
            self.next()
            val = None if self.peek()[1] == ";" else self.expr()
            self.expect(";")
            return ("return", val)
        st = self.simple_statement()
        self.expect(";")
        return st

    def simple_statement(self) -> tuple:
        kw = self.peek()[1]
        if kw in ("let", "var", "const"):
            self.next()
            name = self.ident()
            ty = self.type_() if self.accept(":") else None
            init = self.expr() if self.accept("=") else None
            return ("decl", kw, name, ty, init)
        if kw == "_" and self.peek(1)[1] == "=":
            self.next()
            self.next()
            return ("expr", self.expr())
        lhs = self.expr()
        op = self.peek()[1]
        if op in ("=", "+=", "-=", "*=", "/=", "%=", "&=", "|=", "^=", "<<=", ">>="):
            self.next()
            return ("assign", op, lhs, self.expr())
        if op in ("++", "--"):
            self.next()
            return ("assign", "+=" if op == "++" else "-=", lhs, ("lit", "aint", 1))
        return ("expr", lhs)

    # expressions, by precedence
    _BIN = [("||",), ("&&",), ("|",), ("^",), ("&",), ("==", "!="), ("<", ">", "<=", ">="), ("<<", ">>"),
            ("+", "-"), ("*", "/", "%")]

    def expr(self, level: int = 0) -> tuple:
        if level == len(self._BIN):
            return self.unary()
        lhs = self.expr(level + 1)
        while self.peek()[0] == "op" and self.peek()[1] in self._BIN[level]:
            op = self.next()[1]
            lhs = ("bin", op, lhs, self.expr(level + 1))
        return lhs

    def unary(self) -> tuple:
        if self.peek()[0] == "op" and self.peek()[1] in ("-", "!", "~", "&", "*"):
            op = self.next()[1]
            return ("un", op, self.unary())
        return self.postfix(self.primary())

    def primary(self) -> tuple:
        kind, v = self.next()
        if kind == "num":
            return _literal(v)
        if v == "(":
            e = self.expr()
            self.expect(")")
            return e
        if kind == "id":
            if v in ("true", "false"):
                return ("lit", "bool", v == "true")
            targs = None
            if self.peek()[1] == "<" and v in ("vec2", "vec3", "vec4", "array", "bitcast"):
                self.next()
                targs = self.type_()
                if self.accept(","):
                    self.expr(7)
                self.expect(">")
            if self.accept("("):
                args = []
                while not self.accept(")"):
                    args.append(self.expr())
                    self.accept(",")
                return ("call", v, targs, args)
            return ("name", v)
        raise SyntaxError(f"WGSL: unexpected {v!r}")

    def postfix(self, e: tuple) -> tuple:
        while True:
            if self.accept("["):
                e = ("index", e, self.expr())
                self.expect("]")
            elif self.accept("."):
                e = ("member", e, self.ident())
            else:
                return e


def _literal(v: str) -> tuple:
    s = v.lower()
    if s.startswith("0x"):
        suffix = s[-1] if s[-1] in "iu" else ""
        n = int(s[2:-1] if suffix else s[2:], 16)
        return ("lit", {"": "aint", "i": "i32", "u": "u32"}[suffix], n)
    if s[-1] in "fh":
        return ("lit", "f32", float(s[:-1]))
    if s[-1] in "iu":
        return ("lit", "i32" if s[-1] == "i" else "u32", int(s[:-1]))
    if "." in s or "e" in s:
        return ("lit", "afloat", float(s))
    return ("lit", "aint", int(s))


# ---------------------------------------------------------------------------
# Values: scalars are (type, value) with type u32 / i32 / f32 / bool / aint /
# afloat; vectors are ("vec", elem, [values]); arrays are Arr; structs are
# ("struct", name, {field: value}).

M32 = 0xFFFFFFFF
F32 = np.float32


def _i32(v: int) -> int:
    v &= M32
    return v - (1 << 32) if v & 0x80000000 else v


def _cast(t: str, v) -> Any:
    """Value v (any scalar representation) as scalar type t."""
    if t == "u32":
        if isinstance(v, (float, np.floating)):
            f = float(v)
            return 0 if math.isnan(f) or f <= 0 else (M32 if f >= 4294967295.0 else int(f))
        return int(v) & M32
    if t == "i32":
        if isinstance(v, (float, np.floating)):
            f = float(v)
            if math.isnan(f):
                return 0
            return max(-2147483648, min(2147483647, int(f)))
        return _i32(int(v))
    if t == "f32":
        return F32(v)
    if t == "bool":
        return bool(v)
    raise TypeError(t)


class Arr:
    """An array of scalars (numpy backing) or of composite values (list)."""

    def __init__(self, elem: tuple, data):
        self.elem = elem
        self.data = data

    def get(self, i: int):
        if self.elem[0] == "scalar":
            t = self.elem[1]
            v = self.data[i]
            return (t, F32(v) if t == "f32" else (bool(v) if t == "bool" else int(v)))
        return self.data[i]

    def set(self, i: int, val) -> None:
        if self.elem[0] == "scalar":
            self.data[i] = _cast(self.elem[1], val[1])
        else:
            self.data[i] = val


class StructArr:
    """An array of structs of 32-bit scalar fields over a numpy uint32 buffer
    (field j of element i is word i * fields + j), written in place."""

    def __init__(self, name: str, fields: list, words: np.ndarray):
        self.name = name
        self.fields = fields
        self.words = words

    def get(self, i: int):
        nf = len(self.fields)
        out = {}
        for j, (f, t) in enumerate(self.fields):
            w = self.words[i * nf + j:i * nf + j + 1]
            v = w.view(np.float32)[0] if t[1] == "f32" else (w.view(np.int32)[0] if t[1] == "i32" else w[0])
            out[f] = (t[1], F32(v) if t[1] == "f32" else int(v))
        return ("struct", self.name, out)

    def set(self, i: int, val) -> None:
        nf = len(self.fields)
        for j, (f, t) in enumerate(self.fields):
            v = val[2][f][1]
            w = self.words[i * nf + j:i * nf + j + 1]
            if t[1] == "f32":
                w.view(np.float32)[0] = F32(v)
            elif t[1] == "i32":
                w.view(np.int32)[0] = _i32(int(v))
            else:
                w[0] = int(v) & M32


class _Return(Exception):
    def __init__(self, val):
        self.val = val


class _Break(Exception):
    pass


class _Continue(Exception):
    pass


class Shader:
    """One parsed WGSL module.  run() dispatches its compute entry point."""

    def __init__(self, src: str):
        self.mod = Parser(src).module()
        self.consts: Dict[str, Any] = {}
        for name, ty, e in self.mod["consts"]:
            v = self.eval(e, [{}])
            self.consts[name] = self.coerce(v, ty) if ty else self.concrete(v)

    # -- type helpers ----------------------------------------------------------
    def zero(self, ty: tuple, scopes=None):
        if ty[0] == "scalar":
            return (ty[1], _cast(ty[1], 0))
        if ty[0] == "vec":
            return ("vec", ty[2], [_cast(ty[2], 0)] * ty[1])
        if ty[0] == "array":
            n = self.eval(ty[2], scopes or [{}])[1]
            if ty[1][0] == "scalar":
                dt = {"f32": np.float32, "u32": np.uint32, "i32": np.int32, "bool": np.bool_}[ty[1][1]]
                return Arr(ty[1], np.zeros(int(n), dtype=dt))
            return Arr(ty[1], [self.zero(ty[1], scopes) for _ in range(int(n))])
        fields = self.mod["structs"][ty[1]]
        return ("struct", ty[1], {f: self.zero(t, scopes) for f, t in fields})

    @staticmethod
    def concrete(v):
        if isinstance(v, tuple) and v[0] == "aint":
            return ("i32", _i32(v[1]))
        if isinstance(v, tuple) and v[0] == "afloat":
            return ("f32", F32(v[1]))
        return v

    def coerce(self, v, ty: Optional[tuple]):
        if ty is None:
            return self.concrete(v)
        if ty[0] == "scalar" and isinstance(v, tuple) and v[0] in ("aint", "afloat", "u32", "i32", "f32", "bool"):
            return (ty[1], _cast(ty[1], v[1]))
        return v

    # -- expressions -----------------------------------------------------------
    def lookup(self, name: str, scopes: list):
        for sc in reversed(scopes):
            if name in sc:
                return sc[name]
        if name in self.consts:
            return self.consts[name]
        if name in self.globals:
            return self.globals[name]
        raise NameError(f"WGSL: unknown name {name}")

    def eval(self, e: tuple, scopes: list):
        k = e[0]
        if k == "lit":
            return (e[1], e[2])
        if k == "name":
            v = self.lookup(e[1], scopes)
            return v[0] if isinstance(v, list) else v      # var cells are one-element lists
        if k == "bin":
            return self.binop(e[1], self.eval(e[2], scopes), self.eval(e[3], scopes)) if e[1] not in ("&&", "||") \
                else self.logic(e, scopes)
        if k == "un":
            return self.unop(e[1], self.eval(e[2], scopes))
        if k == "index":
            base = self.eval(e[1], scopes)
            i = int(self.eval(e[2], scopes)[1])
            if isinstance(base, (Arr, StructArr)):
                return base.get(i)
            if base[0] == "vec":
                return (base[1], base[2][i])
            raise TypeError("WGSL: indexing a non-array")
        if k == "member":
            base = self.eval(e[1], scopes)
            if base[0] == "vec":
                return (base[1], base[2]["xyzw".index(e[2])]) if len(e[2]) == 1 else \
                    ("vec", base[1], [base[2]["xyzw".index(c)] for c in e[2]])
            return base[2][e[2]]
        if k == "call":
            return self.call(e[1], e[2], [self.eval(a, scopes) for a in e[3]], scopes)
        raise TypeError(f"WGSL: expression {k}")

    def logic(self, e, scopes):
        a = self.eval(e[2], scopes)[1]
        if e[1] == "&&":
            return ("bool", bool(a) and bool(self.eval(e[3], scopes)[1]))
        return ("bool", bool(a) or bool(self.eval(e[3], scopes)[1]))

    @staticmethod
    def _unify(a, b) -> str:
        ta, tb = a[0], b[0]
        if ta == tb:
            return ta
        if ta in ("aint", "afloat"):
            return tb if not (ta == "afloat" and tb == "aint") else "afloat"
        if tb in ("aint", "afloat"):
            return ta
        raise TypeError(f"WGSL: mixed {ta} and {tb}")

    def binop(self, op: str, a, b):
        if a[0] == "vec" or b[0] == "vec":
            n = len(a[2]) if a[0] == "vec" else len(b[2])
            elem = a[1] if a[0] == "vec" else b[1]
            av = a[2] if a[0] == "vec" else [a[1]] * n
            bv = b[2] if b[0] == "vec" else [b[1]] * n
            res = [self.binop(op, (elem, x), (elem, y)) for x, y in zip(av, bv)]
            return ("vec", res[0][0], [r[1] for r in res])
        t = self._unify(a, b)
        x, y = a[1], b[1]
        if op in ("==", "!=", "<", ">", "<=", ">="):
            if t == "f32":
                x, y = F32(x), F32(y)
            r = {"==": x == y, "!=": x != y, "<": x < y, ">": x > y, "<=": x <= y, ">=": x >= y}[op]
            return ("bool", bool(r))
        if t == "bool":
            return ("bool", {"&": x and y, "|": x or y, "^": x != y}[op])
        if t == "f32" or t == "afloat":
            x, y = (F32(x), F32(y)) if t == "f32" else (float(x), float(y))
            if op == "+":
                r = x + y
            elif op == "-":
                r = x - y
            elif op == "*":
                r = x * y
            elif op == "/":
                with np.errstate(divide="ignore", invalid="ignore"):
                    r = x / y if (t == "f32" or y != 0) else math.copysign(math.inf, x)
            elif op == "%":
                r = x - y * (F32(math.trunc(x / y)) if t == "f32" else math.trunc(x / y))
            else:
                raise TypeError(f"WGSL: {op} on floats")
            return (t, F32(r) if t == "f32" else r)
        # integers
        x, y = int(x), int(y)
        if op in ("<<", ">>"):
            sh = y & 31
            if t == "u32":
                return (t, (x << sh) & M32 if op == "<<" else (x & M32) >> sh)
            if t == "i32":
                return (t, _i32(x << sh) if op == "<<" else (x >> sh))
            return (t, x << y if op == "<<" else x >> y)
        if op == "/":
            r = x if y == 0 else (abs(x) // abs(y)) * (1 if (x >= 0) == (y >= 0) else -1)
        elif op == "%":
            r = 0 if y == 0 else x - y * ((abs(x) // abs(y)) * (1 if (x >= 0) == (y >= 0) else -1))
        else:
            r = {"+": x + y, "-": x - y, "*": x * y, "&": x & y, "|": x | y, "^": x ^ y}[op]
        if t == "u32":
            r &= M32
        elif t == "i32":
            r = _i32(r)
        return (t, r)

    def unop(self, op: str, a):
        if a[0] == "vec":
            return ("vec", a[1], [self.unop(op, (a[1], v))[1] for v in a[2]])
        t, v = a
        if op == "-":
            if t == "f32":
                return (t, F32(-v))
            return (t, _i32(-v) if t == "i32" else (-v) & M32 if t == "u32" else -v)
        if op == "!":
            return ("bool", not v)
        if op == "~":
            return (t, (~v) & M32 if t == "u32" else _i32(~v))
        raise TypeError(f"WGSL: unary {op}")

    def call(self, name: str, targs, args, scopes):
        f = _BUILTINS.get(name)
        if f is not None:
            return f(self, args)
        m = re.fullmatch(r"vec([234])([fiu]?)", name)
        if m:
            n = int(m.group(1))
            elem = {"f": "f32", "i": "i32", "u": "u32"}.get(m.group(2)) or (targs[1] if targs else None)
            flat = []
            for a in args:
                if a[0] == "vec":
                    flat += [(a[1], v) for v in a[2]]
                else:
                    flat.append(a)
            if elem is None:
                elem = self.concrete(flat[0])[0]
            if len(flat) == 1:
                flat = flat * n
            return ("vec", elem, [_cast(elem, v[1]) for v in flat])
        if name in SCALARS:
            return (name, _cast(name, args[0][1]))
        if name in self.mod["structs"]:
            return ("struct", name, {f: self.coerce(a, t) for (f, t), a in zip(self.mod["structs"][name], args)})
        fn = self.mod["fns"].get(name)
        if fn is None:
            raise NameError(f"WGSL: unknown function {name}")
        gen = self.invoke(fn, args)
        try:
            next(gen)
        except StopIteration as s:
            return s.value
        raise RuntimeError("WGSL: workgroupBarrier inside a function called from an expression")

    # -- statements (generators: they yield at workgroupBarrier) --------------
    def invoke(self, fn, args):
        scope = {p[0]: [self.coerce(a, p[1])] for p, a in zip(fn["params"], args)}
        try:
            yield from self.exec_block(fn["body"], [scope])
        except _Return as r:
            return self.coerce(r.val, fn["ret"]) if r.val is not None else None
        return None

    def exec_block(self, body, scopes):
        scopes = scopes + [{}]
        for st in body:
            yield from self.exec(st, scopes)

    def assign(self, lhs, val, scopes):
        k = lhs[0]
        if k == "name":
            cell = self.lookup(lhs[1], scopes)
            if not isinstance(cell, list):
                raise TypeError(f"WGSL: assignment to non-variable {lhs[1]}")
            old = cell[0]
            cell[0] = self.coerce(val, (("scalar", old[0]) if old[0] in SCALARS else None)) \
                if isinstance(old, tuple) and old[0] in SCALARS else val
            return
        if k == "index":
            base = self.eval(lhs[1], scopes)
            i = int(self.eval(lhs[2], scopes)[1])
            if isinstance(base, (Arr, StructArr)):
                base.set(i, val)
            elif base[0] == "vec":
                base[2][i] = _cast(base[1], val[1])
                self.assign(lhs[1], base, scopes)
            return
        if k == "member":
            base = self.eval(lhs[1], scopes)
            if base[0] == "vec":
                base[2]["xyzw".index(lhs[2])] = _cast(base[1], val[1])
            else:
                old = base[2][lhs[2]]
                base[2][lhs[2]] = self.coerce(val, ("scalar", old[0])) if old[0] in SCALARS else val
            # the value read may be a copy (an element of a struct array):
            # store it back through its own place
            if lhs[1][0] != "name" or isinstance(self.lookup(lhs[1][1], scopes), list):
                self.assign(lhs[1], base, scopes)
            return
        raise TypeError("WGSL: bad assignment target")

    def exec(self, st, scopes):
        k = st[0]
        if k == "decl":
            _, kw, name, ty, init = st
            val = self.eval(init, scopes) if init is not None else self.zero(ty, scopes)
            val = self.coerce(val, ty)
            if isinstance(val, tuple) and val[0] == "vec":
                val = ("vec", val[1], list(val[2]))
            scopes[-1][name] = [val] if kw == "var" else val
        elif k == "assign":
            _, op, lhs, rhs = st
            val = self.eval(rhs, scopes)
            if op != "=":
                val = self.binop(op[:-1], self.eval(lhs, scopes), val)
            self.assign(lhs, val, scopes)
        elif k == "expr":
            e = st[1]
            if e[0] == "call" and e[1] in ("workgroupBarrier", "storageBarrier"):
                yield "barrier"
            else:
                self.eval(e, scopes)
        elif k == "if":
            if self.eval(st[1], scopes)[1]:
                yield from self.exec_block(st[2], scopes)
            elif st[3] is not None:
                yield from self.exec_block(st[3], scopes)
        elif k == "for":
            _, init, cond, upd, body = st
            scopes = scopes + [{}]
            if init is not None:
                yield from self.exec(init, scopes)
            while cond is None or self.eval(cond, scopes)[1]:
                try:
                    yield from self.exec_block(body, scopes)
                except _Break:
                    break
                except _Continue:
                    pass
                if upd is not None:
                    yield from self.exec(upd, scopes)
        elif k == "block":
            yield from self.exec_block(st[1], scopes)
        elif k == "return":
            raise _Return(self.eval(st[1], scopes) if st[1] is not None else None)
        elif k == "break":
            raise _Break()
        elif k == "continue":
            raise _Continue()
        else:
            raise TypeError(f"WGSL: statement {k}")

    # -- dispatch ----------------------------------------------------------------
    def run(self, entry: str, groups: Tuple[int, int, int], buffers: Dict[str, Any]) -> None:
        """Dispatch `entry` over `groups` workgroups.  buffers maps each
        module-scope storage / uniform variable name to a numpy array (storage
        array of scalars, written in place) or a dict of struct fields
        (uniform)."""
        self.globals = {}
        for v in self.mod["vars"]:
            if v["space"] in ("storage", "uniform"):
                b = buffers[v["name"]]
                ty = v["type"]
                if ty[0] == "array" and ty[1][0] == "struct":
                    self.globals[v["name"]] = StructArr(ty[1][1], self.mod["structs"][ty[1][1]], b)
                elif ty[0] == "array":
                    self.globals[v["name"]] = Arr(ty[1], b)
                else:
                    fields = dict(self.mod["structs"][ty[1]])
                    self.globals[v["name"]] = ("struct", ty[1],
                                               {f: (fields[f][1], _cast(fields[f][1], b[f])) for f in fields})
        fn = self.mod["fns"][entry]
        ws = [int(self.eval(a, [{}])[1]) for a in fn["attrs"]["workgroup_size"]] + [1, 1]
        wx, wy, wz = ws[0], ws[1], ws[2]
        for gz in range(groups[2]):
            for gy in range(groups[1]):
                for gx in range(groups[0]):
                    for v in self.mod["vars"]:
                        if v["space"] in ("workgroup", "private"):
                            self.globals[v["name"]] = [self.zero(v["type"])]
                    invs = []
                    for lz in range(wz):
                        for ly in range(wy):
                            for lx in range(wx):
                                b = {"local_invocation_id": ("vec", "u32", [lx, ly, lz]),
                                     "workgroup_id": ("vec", "u32", [gx, gy, gz]),
                                     "global_invocation_id": ("vec", "u32", [gx * wx + lx, gy * wy + ly, gz * wz + lz]),
                                     "num_workgroups": ("vec", "u32", list(groups)),
                                     "local_invocation_index": ("u32", lx + wx * (ly + wy * lz))}
                                args = [b[p[2]["builtin"][0][1]] for p in fn["params"]]
                                invs.append(self.invoke(fn, args))
                    live = invs
                    while live:
                        nxt = []
                        for g in live:
                            try:
                                next(g)
                                nxt.append(g)
                            except StopIteration:
                                pass
                        live = nxt


def _f1(fn):
    """A float builtin applied per element, evaluated in double and rounded."""
    def apply(sh, args):
        a = args[0]
        if a[0] == "vec":
            return ("vec", "f32", [F32(fn(float(v))) for v in a[2]])
        return ("f32", F32(fn(float(a[1]))))
    return apply


def _safe(fn):
    def g(x):
        try:
            return fn(x)
        except (ValueError, OverflowError):
            return math.nan if not math.isinf(x) else fn(math.copysign(1e308, x))
    return g


def _minmax(pick):
    def apply(sh, args):
        a, b = args
        t = Shader._unify(a, b)
        if t == "f32":
            return ("f32", F32(pick(F32(a[1]), F32(b[1]))))
        return (t, pick(a[1], b[1]))
    return apply


def _unpack2x16float(sh, args):
    bits = int(args[0][1]) & M32
    h = np.array([bits & 0xFFFF, bits >> 16], dtype=np.uint16).view(np.float16).astype(np.float32)
    return ("vec", "f32", [F32(h[0]), F32(h[1])])


def _select(sh, args):
    f, t, c = args
    return t if c[1] else f


def _clamp(sh, args):
    lo = _minmax(max)(sh, [args[0], args[1]])
    return _minmax(min)(sh, [lo, args[2]])


def _abs(sh, args):
    a = args[0]
    if a[0] == "f32":
        return ("f32", F32(abs(a[1])))
    return (a[0], abs(a[1]) if a[0] != "i32" else _i32(abs(a[1])))


def _pow(sh, args):
    x, y = float(args[0][1]), float(args[1][1])
    try:
        r = math.pow(x, y)
    except (ValueError, OverflowError):
        r = math.nan if x < 0 else math.inf
    return ("f32", F32(r))


_BUILTINS = {
    "select": _select,
    "min": _minmax(min),
    "max": _minmax(max),
    "clamp": _clamp,
    "abs": _abs,
    "floor": _f1(math.floor),
    "exp": _f1(_safe(math.exp)),
    "sin": _f1(math.sin),
    "cos": _f1(math.cos),
    "tanh": _f1(math.tanh),
    "sqrt": _f1(_safe(math.sqrt)),
    "inverseSqrt": _f1(_safe(lambda x: 1.0 / math.sqrt(x))),
    "pow": _pow,
    "unpack2x16float": _unpack2x16float,
}


def extract_shaders(ts_source: str) -> Dict[str, str]:
    """The `const NAME_WGSL = /* wgsl */ \\`...\\`` shader strings of a
    TypeScript source file, by name."""
    return dict(re.findall(r"const (\w+_WGSL) = /\* wgsl \*/ `(.*?)`;", ts_source, re.S))
