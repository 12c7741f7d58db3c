"""A small interpreter for the TypeScript/JavaScript subset of the reference's CPU functions.

Used only by tests/golden/gen_golden.py, here where the reference source is mounted, to
execute the reference's own ``attentionCpu`` / ``ropeCpu`` / ``ropeFactorsCpu`` /
``rmsnormCpu`` source text (src/lib/webgpu/kernels.ts) and record their outputs as golden
fixtures.  No JavaScript engine exists in this image, so this stands in for one.

JS semantics kept:
  * a number is an IEEE double (Python float); ``/`` by zero gives +-Infinity / NaN;
  * a ``Float32Array`` element store rounds to f32 (numpy float32), a load widens to double;
  * ``Math.*`` and ``**`` map to the C library (Python's math module / float pow);
  * ``a ?? b``, default parameters, arrow closures, ``let``/``const`` block scope,
    compound assignment, ``++``/``--``, ``for``/``if``/``return``, growable ``[]`` arrays.
TypeScript type annotations (``: T``, ``?: T``, ``: T[]``, return types) are skipped.
Anything outside this subset raises ``SyntaxError``/``NotImplementedError``.
"""
from __future__ import annotations

import math
import re

import numpy as np

UNDEF = object()

_TOKEN_RE = re.compile(r"""
    (?P<ws>\s+|//[^\n]*|/\*.*?\*/)
  | (?P<num>(?:\d+\.\d*|\.\d+|\d+)(?:[eE][+-]?\d+)?)
  | (?P<id>[A-Za-z_$][A-Za-z0-9_$]*)
  | (?P<str>'[^']*'|"[^"]*")
  | (?P<op>\?\?|\*\*=|\*\*|=>|===|!==|==|!=|<=|>=|&&|\|\||\+\+|--|\+=|-=|\*=|/=|\?\.|[-+*/%<>=!?:;,.(){}\[\]|&])
""", re.S | re.X)


def tokenize(src):
    out, pos = [], 0
    while pos < len(src):
        m = _TOKEN_RE.match(src, pos)
        if not m:
            raise SyntaxError(f"bad char at {pos}: {src[pos:pos+20]!r}")
        pos = m.end()
        kind = m.lastgroup
        if kind == "ws":
            continue
        out.append((kind, m.group(kind)))
    out.append(("eof", None))
    return out


class Parser:
    def __init__(self, src):
        self.t = tokenize(src)
        self.i = 0

    def peek(self, k=0):
        return self.t[self.i + k]

    def next(self):
        tok = self.t[self.i]
        self.i += 1
        return tok

    def at(self, val, k=0):
        return self.t[self.i + k][1] == val and self.t[self.i + k][0] in ("op", "id")

    def expect(self, val):
        tok = self.next()
        if tok[1] != val:
            raise SyntaxError(f"expected {val!r}, got {tok!r}")
        return tok

    # --- TypeScript annotations -------------------------------------------------------
    def skip_type(self):
        depth = 0
        while True:
            kind, val = self.peek()
            if kind == "id":
                self.next()
            elif val == "<":
                depth += 1
                self.next()
            elif val == ">" and depth:
                depth -= 1
                self.next()
            elif val == "[" and self.at("]", 1):
                self.next()
                self.next()
            elif val in ("|", ",") and depth:
                self.next()
            elif val == "|":
                self.next()
            else:
                return

    # --- statements --------------------------------------------------------------------
    def program(self):
        body = []
        while self.peek()[0] != "eof":
            body.append(self.statement())
        return ("block", body)

    def params(self):
        self.expect("(")
        ps = []
        while not self.at(")"):
            name = self.next()[1]
            if self.at("?"):
                self.next()
            if self.at(":"):
                self.next()
                self.skip_type()
            default = None
            if self.at("="):
                self.next()
                default = self.assign()
            ps.append((name, default))
            if self.at(","):
                self.next()
        self.expect(")")
        return ps

    def statement(self):
        kind, val = self.peek()
        if val == "function":
            self.next()
            name = self.next()[1]
            ps = self.params()
            if self.at(":"):
                self.next()
                self.skip_type()
            return ("fundecl", name, ps, self.block())
        if val in ("const", "let", "var"):
            st = self.declaration()
            if self.at(";"):
                self.next()
            return st
        if val == "for":
            self.next()
            self.expect("(")
            init = None
            if not self.at(";"):
                init = self.declaration() if self.peek()[1] in ("const", "let", "var") else ("expr", self.expr())
            self.expect(";")
            test = None if self.at(";") else self.expr()
            self.expect(";")
            update = None if self.at(")") else self.expr()
            self.expect(")")
            return ("for", init, test, update, self.statement())
        if val == "if":
            self.next()
            self.expect("(")
            cond = self.expr()
            self.expect(")")
            then = self.statement()
            other = None
            if self.at("else"):
                self.next()
                other = self.statement()
            return ("if", cond, then, other)
        if val == "return":
            self.next()
            e = None if self.at(";") or self.at("}") else self.expr()
            if self.at(";"):
                self.next()
            return ("return", e)
        if val == "{":
            return self.block()
        if val == ";":
            self.next()
            return ("block", [])
        e = self.expr()
        if self.at(";"):
            self.next()
        return ("expr", e)

    def declaration(self):
        self.next()  # const / let / var
        decls = []
        while True:
            name = self.next()[1]
            if self.at(":"):
                self.next()
                self.skip_type()
            init = None
            if self.at("="):
                self.next()
                init = self.assign()
            decls.append((name, init))
            if self.at(","):
                self.next()
                continue
            return ("decl", decls)

    def block(self):
        self.expect("{")
        body = []
        while not self.at("}"):
            body.append(self.statement())
        self.expect("}")
        return ("block", body)

    # --- expressions -------------------------------------------------------------------
    def expr(self):
        e = self.assign()
        while self.at(","):
            self.next()
            e = ("seq", e, self.assign())
        return e

    def is_arrow(self):
        if self.peek()[0] == "id" and self.at("=>", 1):
            return True
        if not self.at("("):
            return False
        depth, j = 0, self.i
        while True:
            val = self.t[j][1]
            if val == "(":
                depth += 1
            elif val == ")":
                depth -= 1
                if depth == 0:
                    break
            j += 1
        return self.t[j + 1][1] == "=>" or (self.t[j + 1][1] == ":" and "=>" in [x[1] for x in self.t[j + 1:j + 8]])

    def assign(self):
        if self.is_arrow():
            if self.peek()[0] == "id":
                ps = [(self.next()[1], None)]
            else:
                ps = self.params()
                if self.at(":"):
                    self.next()
                    self.skip_type()
            self.expect("=>")
            body = self.block() if self.at("{") else ("return", self.assign())
            return ("arrow", ps, body)
        lhs = self.cond()
        if self.peek()[1] in ("=", "+=", "-=", "*=", "/=", "**="):
            op = self.next()[1]
            return ("assign", op, lhs, self.assign())
        return lhs

    def cond(self):
        c = self.binary(0)
        if self.at("?"):
            self.next()
            a = self.assign()
            self.expect(":")
            b = self.assign()
            return ("cond", c, a, b)
        return c

    _PREC = [("??",), ("||",), ("&&",), ("===", "!==", "==", "!="), ("<", ">", "<=", ">="), ("+", "-"), ("*", "/", "%")]

    def binary(self, level):
        if level == len(self._PREC):
            return self.exponent()
        e = self.binary(level + 1)
        while self.peek()[0] == "op" and self.peek()[1] in self._PREC[level]:
            op = self.next()[1]
            e = ("bin", op, e, self.binary(level + 1))
        return e

    def exponent(self):
        base = self.unary()
        if self.at("**"):
            self.next()
            return ("bin", "**", base, self.exponent())
        return base

    def unary(self):
        if self.peek()[0] == "op" and self.peek()[1] in ("-", "+", "!"):
            op = self.next()[1]
            return ("unary", op, self.unary())
        if self.peek()[1] in ("++", "--"):
            op = self.next()[1]
            return ("preinc", op, self.unary())
        return self.postfix()

    def postfix(self):
        e = self.call()
        if self.peek()[1] in ("++", "--"):
            op = self.next()[1]
            return ("postinc", op, e)
        return e

    def call(self):
        if self.at("new"):
            self.next()
            callee = self.primary()
            while self.at("."):
                self.next()
                callee = ("member", callee, ("str", self.next()[1]))
            args = self.args() if self.at("(") else []
            e = ("new", callee, args)
        else:
            e = self.primary()
        while True:
            if self.at("."):
                self.next()
                e = ("member", e, ("str", self.next()[1]))
            elif self.at("["):
                self.next()
                idx = self.expr()
                self.expect("]")
                e = ("member", e, idx)
            elif self.at("("):
                e = ("call", e, self.args())
            else:
                return e

    def args(self):
        self.expect("(")
        out = []
        while not self.at(")"):
            out.append(self.assign())
            if self.at(","):
                self.next()
        self.expect(")")
        return out

    def primary(self):
        kind, val = self.next()
        if kind == "num":
            return ("num", float(val))
        if kind == "str":
            return ("str", val[1:-1])
        if kind == "id":
            if val == "true":
                return ("num", True)
            if val == "false":
                return ("num", False)
            return ("name", val)
        if val == "(":
            e = self.expr()
            self.expect(")")
            return e
        if val == "[":
            items = []
            while not self.at("]"):
                items.append(self.assign())
                if self.at(","):
                    self.next()
            self.expect("]")
            return ("array", items)
        raise SyntaxError(f"unexpected {kind} {val!r}")


class F32Array:
    """Float32Array: f32 storage, double loads."""

    def __init__(self, n_or_data):
        if isinstance(n_or_data, (int, float)):
            self.a = np.zeros(int(n_or_data), np.float32)
        else:
            self.a = np.array(n_or_data, dtype=np.float32)

    def get(self, i):
        i = int(i)
        return float(self.a[i]) if 0 <= i < self.a.size else UNDEF

    def set(self, i, v):
        i = int(i)
        if 0 <= i < self.a.size:
            self.a[i] = np.float32(v)  # double -> f32, round to nearest even

    @property
    def length(self):
        return float(self.a.size)


class JSArray:
    def __init__(self, items):
        self.items = list(items)

    def get(self, i):
        i = int(i)
        return self.items[i] if 0 <= i < len(self.items) else UNDEF

    def set(self, i, v):
        i = int(i)
        while len(self.items) <= i:
            self.items.append(UNDEF)
        self.items[i] = v

    @property
    def length(self):
        return float(len(self.items))


def _div(a, b):
    if b == 0:
        if a == 0 or math.isnan(a):
            return math.nan
        return math.copysign(math.inf, a) * math.copysign(1.0, b)
    return a / b


class _Return(Exception):
    def __init__(self, v):
        self.v = v


class Env:
    def __init__(self, parent=None):
        self.vars = {}
        self.parent = parent

    def lookup(self, name):
        e = self
        while e is not None:
            if name in e.vars:
                return e
            e = e.parent
        raise NameError(name)


class Closure:
    def __init__(self, params, body, env, interp):
        self.params, self.body, self.env, self.interp = params, body, env, interp

    def __call__(self, *args):
        env = Env(self.env)
        for i, (name, default) in enumerate(self.params):
            v = args[i] if i < len(args) else UNDEF
            if v is UNDEF and default is not None:
                v = self.interp.eval(default, env)
            env.vars[name] = v
        try:
            self.interp.exec(self.body, env)
        except _Return as r:
            return r.v
        return UNDEF


_MATH = {
    "exp": math.exp, "tanh": math.tanh, "sqrt": lambda x: math.sqrt(x) if x >= 0 else math.nan,
    "floor": lambda x: float(math.floor(x)), "cos": math.cos, "sin": math.sin, "abs": abs,
    "max": lambda *a: max(a) if a else -math.inf, "min": lambda *a: min(a) if a else math.inf,
    "log": lambda x: math.log(x) if x > 0 else (-math.inf if x == 0 else math.nan), "PI": math.pi,
    "round": lambda x: float(math.floor(x + 0.5)),
}


class Interpreter:
    def __init__(self):
        self.glob = Env()
        self.glob.vars.update({"Math": _MATH, "Infinity": math.inf, "NaN": math.nan, "undefined": UNDEF,
                               "Float32Array": F32Array})

    def load(self, src):
        for st in Parser(src).program()[1]:  # top level shares the global scope
            self.exec(st, self.glob)

    def call(self, name, *args):
        return self.glob.vars[name](*args)

    # statements
    def exec(self, node, env):
        kind = node[0]
        if kind == "block":
            inner = Env(env)
            for st in node[1]:
                self.exec(st, inner)
        elif kind == "fundecl":
            env.vars[node[1]] = Closure(node[2], node[3], env, self)
        elif kind == "decl":
            for name, init in node[1]:
                env.vars[name] = UNDEF if init is None else self.eval(init, env)
        elif kind == "expr":
            self.eval(node[1], env)
        elif kind == "for":
            loop = Env(env)
            if node[1] is not None:
                self.exec(node[1], loop)
            while node[2] is None or self.truthy(self.eval(node[2], loop)):
                self.exec(node[4], Env(loop))
                if node[3] is not None:
                    self.eval(node[3], loop)
        elif kind == "if":
            if self.truthy(self.eval(node[1], env)):
                self.exec(node[2], env)
            elif node[3] is not None:
                self.exec(node[3], env)
        elif kind == "return":
            raise _Return(UNDEF if node[1] is None else self.eval(node[1], env))
        else:
            raise NotImplementedError(kind)

    @staticmethod
    def truthy(v):
        if v is UNDEF or v is None:
            return False
        if isinstance(v, float):
            return not (v == 0 or math.isnan(v))
        return bool(v)

    def get_member(self, obj, key):
        if isinstance(obj, dict):
            return obj[key]
        if key == "length":
            return obj.length
        return obj.get(key)

    def store(self, target, value, env):
        if target[0] == "name":
            env.lookup(target[1]).vars[target[1]] = value
        elif target[0] == "member":
            obj = self.eval(target[1], env)
            obj.set(self.eval(target[2], env), value)
        else:
            raise NotImplementedError(target[0])

    def binop(self, op, a, b):
        if op == "+":
            return a + b
        if op == "-":
            return a - b
        if op == "*":
            return a * b
        if op == "/":
            return _div(a, b)
        if op == "**":
            try:
                return math.pow(a, b)
            except (OverflowError, ValueError):
                return a ** b if a >= 0 else math.nan
        if op == "%":
            return math.fmod(a, b)
        if op == "<":
            return a < b
        if op == ">":
            return a > b
        if op == "<=":
            return a <= b
        if op == ">=":
            return a >= b
        if op in ("===", "=="):
            return a == b
        if op in ("!==", "!="):
            return a != b
        raise NotImplementedError(op)

    def eval(self, node, env):
        kind = node[0]
        if kind == "num":
            return node[1]
        if kind == "str":
            return node[1]
        if kind == "name":
            return env.lookup(node[1]).vars[node[1]]
        if kind == "array":
            return JSArray([self.eval(x, env) for x in node[1]])
        if kind == "member":
            return self.get_member(self.eval(node[1], env), self.eval(node[2], env))
        if kind == "call":
            fn = self.eval(node[1], env)
            return fn(*[self.eval(a, env) for a in node[2]])
        if kind == "new":
            cls = self.eval(node[1], env)
            return cls(*[self.eval(a, env) for a in node[2]])
        if kind == "arrow":
            return Closure(node[1], node[2], env, self)
        if kind == "unary":
            v = self.eval(node[2], env)
            if node[1] == "-":
                return -v
            if node[1] == "+":
                return float(v)
            return not self.truthy(v)
        if kind in ("postinc", "preinc"):
            old = self.eval(node[2], env)
            new = old + 1 if node[1] == "++" else old - 1
            self.store(node[2], new, env)
            return old if kind == "postinc" else new
        if kind == "assign":
            op, target, rhs = node[1], node[2], node[3]
            if op == "=":
                v = self.eval(rhs, env)
            else:
                v = self.binop(op[:-1], self.eval(target, env), self.eval(rhs, env))
            self.store(target, v, env)
            return v
        if kind == "cond":
            return self.eval(node[2] if self.truthy(self.eval(node[1], env)) else node[3], env)
        if kind == "seq":
            self.eval(node[1], env)
            return self.eval(node[2], env)
        if kind == "bin":
            op = node[1]
            if op == "??":
                a = self.eval(node[2], env)
                return self.eval(node[3], env) if a is UNDEF or a is None else a
            if op == "&&":
                a = self.eval(node[2], env)
                return self.eval(node[3], env) if self.truthy(a) else a
            if op == "||":
                a = self.eval(node[2], env)
                return a if self.truthy(a) else self.eval(node[3], env)
            return self.binop(op, self.eval(node[2], env), self.eval(node[3], env))
        raise NotImplementedError(kind)


def extract_function(source: str, name: str) -> str:
    """Return the text of top-level ``function name(...) {...}`` from a TS file, by brace matching."""
    m = re.search(r"^function\s+" + re.escape(name) + r"\s*\(", source, re.M)
    if not m:
        raise KeyError(name)
    start = m.start()
    i = source.index("{", source.index(")", m.end()))
    # skip a `): Type {` return annotation: the first '{' after the parameter list's ')'.
    depth = 0
    for j in range(i, len(source)):
        if source[j] == "{":
            depth += 1
        elif source[j] == "}":
            depth -= 1
            if depth == 0:
                return source[start:j + 1]
    raise SyntaxError("unbalanced braces in " + name)
