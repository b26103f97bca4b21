"""A compact reader for `.tl` source that produces ABI statements.

It accepts the statement and expression forms the reference grammar defines
(src/frontend/lexer.zig, src/frontend/parser.zig) that the execution backend
lowers: `domain`, `sparse`, equations with every index form and accumulation
operator, queries `T?`, `save` / `load`, and `backward L wrt P, ...`.
Precedence follows the reference parser: the implicit product binds loosest
(parser.zig:485-500), so `Q[q,d] K[k,d] / 8.0` is `Q * (K / 8.0)`; then
`+ -`, then `* / ^`, then unary minus.  A `(` followed by an identifier is a
relation reference, not a group (parser.zig:688-697).

The reader is host-side convenience (the CLI and its Zig frontend stay the
reference's); what crosses the ABI is the lowered `Statement` array.
"""
import ctypes as C
import re

from . import abi

KEYWORDS = {
    "step", "softmax", "relu", "sigmoid", "tanh", "exp", "log", "abs", "sqrt", "sin", "cos",
    "norm", "lnorm", "concat", "embed", "sparse", "domain", "import", "export", "as", "if",
    "else", "for", "in", "true", "false", "save", "load", "backward", "tucker", "wrt",
}
NONLINEARITIES = {"step", "softmax", "relu", "sigmoid", "tanh", "exp", "log", "abs", "sqrt",
                  "sin", "cos", "norm", "lnorm", "concat"}

_TOKEN_RE = re.compile(r"""
    (?P<comment>//[^\n]*)
  | (?P<newline>\n)
  | (?P<ws>[ \t\r]+)
  | (?P<float>\d+\.\d+(?:[eE][+-]?\d+)?|\d+[eE][+-]?\d+)
  | (?P<integer>\d+)
  | (?P<string>"[^"]*")
  | (?P<accum>(?:max|min|avg)=(?!=))
  | (?P<ident>[A-Za-z_][A-Za-z0-9_]*)
  | (?P<op>\+=|\*=|==|!=|<=|>=|[=\[\](),.'?+\-*/^<>&|!:])
""", re.VERBOSE)


class ParseError(ValueError):
    pass


def tokenize(src):
    toks = []
    pos = 0
    while pos < len(src):
        m = _TOKEN_RE.match(src, pos)
        if not m:
            raise ParseError(f"unexpected character {src[pos]!r} at offset {pos}")
        kind = m.lastgroup
        text = m.group(kind)
        pos = m.end()
        if kind in ("ws", "comment"):
            continue
        if kind == "ident" and text in KEYWORDS:
            kind = "kw"
        if kind == "string":
            text = text[1:-1]  # the backend strips the quotes (the reference keeps them)
        toks.append((kind, text))
    toks.append(("eof", ""))
    return toks


# ----------------------------------------------------------------------------
# Expression trees (a tuple form of src/frontend/ast.zig Expr)
# ----------------------------------------------------------------------------
#   ("ref", name, [index, ...])        index = (kind, name, value, value2)
#   ("lit", float)
#   ("prod", left, right)              implicit product
#   ("bin", op, left, right)           op in + - * / ^ < > <= >= == != & |
#   ("neg", e) / ("not", e)
#   ("nl", func, arg, temperature or None)
#   ("group", e)


class Parser:
    def __init__(self, src):
        self.toks = tokenize(src)
        self.i = 0

    def peek(self, k=0):
        return self.toks[min(self.i + k, len(self.toks) - 1)]

    def advance(self):
        t = self.toks[self.i]
        self.i += 1
        return t

    def check(self, kind, text=None):
        t = self.peek()
        return t[0] == kind and (text is None or t[1] == text)

    def match(self, kind, text=None):
        if self.check(kind, text):
            self.advance()
            return True
        return False

    def expect(self, kind, text=None, what=""):
        if not self.check(kind, text):
            raise ParseError(f"expected {what or text or kind}, got {self.peek()}")
        return self.advance()

    def parse(self):
        stmts = []
        while not self.check("eof"):
            if self.match("newline"):
                continue
            stmts.append(self.statement())
        return stmts

    def end_of_statement(self):
        if not (self.match("newline") or self.check("eof")):
            raise ParseError(f"unexpected {self.peek()} at end of statement")

    def statement(self):
        if self.match("kw", "domain"):
            name = self.expect("ident")[1]
            size = None
            if self.match("op", ":"):
                if self.check("integer"):
                    size = int(self.advance()[1])
                else:
                    self.expect("ident")
            self.end_of_statement()
            return ("domain", name, size)
        if self.match("kw", "sparse"):
            name = self.expect("ident")[1]
            idx = []
            close = "]" if self.match("op", "[") else (self.expect("op", "(") and ")")
            while True:
                iname = self.expect("ident")[1]
                dom = None
                if self.match("op", ":"):
                    dom = self.expect("ident")[1]
                idx.append((abi.IX_NAME, dom or iname, 0, 0))
                if not self.match("op", ","):
                    break
            self.expect("op", close)
            self.end_of_statement()
            return ("sparse", name, idx)
        if self.check("kw", "save") or self.check("kw", "load"):
            kw = self.advance()[1]
            name = self.expect("ident")[1]
            path = self.expect("string")[1]
            self.end_of_statement()
            return (kw, name, path)
        if self.match("kw", "backward"):
            loss = self.expect("ident")[1]
            self.expect("kw", "wrt")
            params = [self.expect("ident")[1]]
            while self.match("op", ","):
                params.append(self.expect("ident")[1])
            self.end_of_statement()
            return ("backward", loss, params)
        lhs = self.tensor_ref()
        if self.match("op", "?"):
            self.end_of_statement()
            return ("query", lhs)
        if self.check("accum"):
            op = self.advance()[1]
        else:
            op = self.expect("op", what="accumulation operator")[1]
            if op not in ("=", "+=", "*="):
                raise ParseError(f"expected accumulation operator, got {op!r}")
        rhs = self.expr()
        self.end_of_statement()
        return ("eq", lhs, op, rhs)

    def tensor_ref(self):
        name = self.expect("ident")[1]
        idx = []
        if self.match("op", "["):
            idx = self.indices()
            self.expect("op", "]")
        elif self.check("op", "("):
            self.advance()
            idx = self.indices()
            self.expect("op", ")")
        return ("ref", name, idx)

    def indices(self):
        out = [self.index()]
        while self.match("op", ","):
            out.append(self.index())
        return out

    def index(self):
        if self.match("op", "*"):
            return (abi.IX_VIRTUAL, self.expect("ident")[1], 0, 0)
        if self.match("op", "/"):
            return (abi.IX_NORMALIZE, self.expect("ident")[1], 0, 0)
        if self.check("integer"):
            v = int(self.advance()[1])
            if self.match("op", ":"):
                e = int(self.expect("integer")[1])
                return (abi.IX_SLICE, "", v, e)
            return (abi.IX_CONST, "", v, 0)
        name = self.expect("ident", what="index")[1]
        if self.match("op", "'"):
            return (abi.IX_PRIMED, name, 0, 0)
        if self.match("op", "."):
            return (abi.IX_NORMALIZE, name, 0, 0)
        if self.match("op", "+"):
            return (abi.IX_ADD, name, int(self.expect("integer")[1]), 0)
        if self.match("op", "-"):
            return (abi.IX_SUB, name, int(self.expect("integer")[1]), 0)
        if self.match("op", "/"):
            return (abi.IX_DIV, name, int(self.expect("integer")[1]), 0)
        return (abi.IX_NAME, name, 0, 0)

    # implicit product: lowest precedence, left-assoc binary products
    def expr(self):
        left = self.additive()
        while self.check("ident") or (self.check("kw") and self.peek()[1] in NONLINEARITIES | {"embed"}):
            right = self.additive()
            left = ("prod", left, right)
        return left

    def additive(self):
        left = self.multiplicative()
        while True:
            if self.match("op", "+"):
                left = ("bin", "+", left, self.multiplicative())
            elif self.match("op", "-"):
                left = ("bin", "-", left, self.multiplicative())
            else:
                return left

    def multiplicative(self):
        left = self.unary()
        while True:
            if self.match("op", "*"):
                left = ("bin", "*", left, self.unary())
            elif self.match("op", "/"):
                left = ("bin", "/", left, self.unary())
            elif self.match("op", "^"):
                left = ("bin", "^", left, self.unary())
            elif self.peek()[0] == "op" and self.peek()[1] in ("<", ">", "<=", ">=", "==", "!=", "&", "|"):
                op = self.advance()[1]
                left = ("bin", op, left, self.unary())
            else:
                return left

    def unary(self):
        if self.match("op", "-"):
            return ("neg", self.unary())
        if self.match("op", "!"):
            return ("not", self.unary())
        return self.primary()

    def primary(self):
        t = self.peek()
        if t[0] == "kw" and t[1] in NONLINEARITIES:
            func = self.advance()[1]
            self.expect("op", "(")
            arg = self.expr()
            temp = None
            if func == "sigmoid" and self.match("op", ","):
                temp = float(self.advance()[1])
            self.expect("op", ")")
            return ("nl", func, arg, temp)
        if t == ("op", "(") and self.peek(1)[0] != "ident":
            self.advance()
            e = self.expr()
            self.expect("op", ")")
            return ("group", e)
        if t[0] == "ident":
            return self.tensor_ref()
        if t[0] in ("integer", "float"):
            self.advance()
            return ("lit", float(t[1]))
        if self.match("kw", "true"):
            return ("lit", 1.0)
        if self.match("kw", "false"):
            return ("lit", 0.0)
        if t[0] == "string":
            self.advance()
            return ("lit", 0.0)
        raise ParseError(f"expected expression, got {t}")


def parse(src):
    return Parser(src).parse()


# ----------------------------------------------------------------------------
# Lowering to ABI structs
# ----------------------------------------------------------------------------
_BINOPS = {"+": abi.OP_ADD, "-": abi.OP_SUB, "*": abi.OP_MUL, "/": abi.OP_DIV, "^": abi.OP_POW,
           ">": abi.OP_GT, "<": abi.OP_LT, ">=": abi.OP_GE, "<=": abi.OP_LE, "==": abi.OP_EQ,
           "!=": abi.OP_NE, "&": abi.OP_AND, "|": abi.OP_OR}


def _fill_ref(dst, ref):
    _, name, idx = ref
    if len(idx) > abi.TL_MAX_RANK:
        raise ParseError(f"{name}: more than {abi.TL_MAX_RANK} indices")
    dst.tensor = name.encode()
    dst.rank = len(idx)
    for k, (kind, iname, v, v2) in enumerate(idx):
        dst.idx[k].kind = kind
        dst.idx[k].name = iname.encode()
        dst.idx[k].value = v
        dst.idx[k].value2 = v2


def lower_equation(eq_tuple, dst=None):
    """Lower ("eq", lhs, op, rhs) into an abi.Equation."""
    _, lhs, op, rhs = eq_tuple
    eq = dst if dst is not None else abi.Equation()
    _fill_ref(eq.lhs, lhs)
    eq.accum = abi.ACC[op]
    refs = []
    code = []

    def emit(e):
        kind = e[0]
        if kind == "ref":
            if len(refs) >= abi.TL_MAX_REFS:
                raise ParseError("too many tensor references in one equation")
            refs.append(e)
            code.append((abi.OP_REF, len(refs) - 1, 0, 0.0))
        elif kind == "lit":
            code.append((abi.OP_LIT, 0, 0, e[1]))
        elif kind == "prod":
            emit(e[1])
            emit(e[2])
            code.append((abi.OP_PROD, 2, 0, 0.0))
        elif kind == "bin":
            emit(e[2])
            emit(e[3])
            code.append((_BINOPS[e[1]], 0, 0, 0.0))
        elif kind == "neg":
            emit(e[1])
            code.append((abi.OP_NEG, 0, 0, 0.0))
        elif kind == "not":
            emit(e[1])
            code.append((abi.OP_NOT, 0, 0, 0.0))
        elif kind == "nl":
            emit(e[2])
            temp = e[3]
            code.append((abi.OP_NL, abi.NL[e[1]], 1 if temp is not None else 0,
                         temp if temp is not None else 0.0))
        elif kind == "group":
            emit(e[1])
        else:
            raise ParseError(f"cannot lower {kind}")

    emit(rhs)
    if len(code) > abi.TL_MAX_CODE:
        raise ParseError("right-hand side too long")
    eq.n_refs = len(refs)
    for k, r in enumerate(refs):
        _fill_ref(eq.refs[k], r)
    eq.n_code = len(code)
    for k, (o, a, a2, v) in enumerate(code):
        eq.code[k].op = o
        eq.code[k].arg = a
        eq.code[k].arg2 = a2
        eq.code[k].value = v
    return eq


class Program:
    """A lowered program: an abi.Statement array plus the host buffers it points at.

    `inputs` maps tensor names to numpy arrays (f64) fed at the program's
    `load Name "..."` statements; `sparse_inputs` maps sparse tensor names to
    (rows, cols, vals-or-None) COO triples fed right after their `sparse`
    declaration.
    """

    def __init__(self, src, inputs=None, sparse_inputs=None):
        import numpy as np
        self.src = src
        self.parsed = parse(src)
        self._keep = []
        inputs = inputs or {}
        sparse_inputs = sparse_inputs or {}
        items = []
        for st in self.parsed:
            items.append(st)
            if st[0] == "sparse" and st[1] in sparse_inputs:
                items.append(("sparse_load", st[1]))
        self.stmts = (abi.Statement * max(1, len(items)))()
        self.n = len(items)
        for k, st in enumerate(items):
            s = self.stmts[k]
            kind = st[0]
            if kind == "domain":
                s.kind = abi.STMT_DOMAIN
                s.name = st[1].encode()
                s.size = st[2] if st[2] is not None else -1
            elif kind == "sparse":
                s.kind = abi.STMT_SPARSE
                s.name = st[1].encode()
                _fill_ref(s.sparse, ("ref", st[1], st[2]))
            elif kind == "sparse_load":
                rows, cols, vals = sparse_inputs[st[1]]
                rows = np.ascontiguousarray(rows, dtype=np.int64)
                cols = np.ascontiguousarray(cols, dtype=np.int64)
                self._keep += [rows, cols]
                s.kind = abi.STMT_SPARSE_LOAD
                s.name = st[1].encode()
                s.size = len(rows)
                s.coo_rows = rows.ctypes.data_as(C.POINTER(C.c_int64))
                s.coo_cols = cols.ctypes.data_as(C.POINTER(C.c_int64))
                if vals is not None:
                    vals = np.ascontiguousarray(vals, dtype=np.float64)
                    self._keep.append(vals)
                    s.host_data = vals.ctypes.data_as(C.POINTER(C.c_double))
            elif kind in ("save", "load"):
                s.kind = abi.STMT_SAVE if kind == "save" else abi.STMT_LOAD
                s.name = st[1].encode()
                s.path = st[2].encode()
                if kind == "load" and st[1] in inputs:
                    arr = np.ascontiguousarray(inputs[st[1]], dtype=np.float64)
                    self._keep.append(arr)
                    s.host_data = arr.ctypes.data_as(C.POINTER(C.c_double))
            elif kind == "backward":
                s.kind = abi.STMT_BACKWARD
                s.name = st[1].encode()
                if len(st[2]) > abi.TL_MAX_PARAMS:
                    raise ParseError("too many backward parameters")
                s.n_params = len(st[2])
                for j, p in enumerate(st[2]):
                    s.params[j].value = p.encode()
            elif kind == "query":
                s.kind = abi.STMT_QUERY
                s.name = st[1][1].encode()
                _fill_ref(s.sparse, st[1])
            elif kind == "eq":
                s.kind = abi.STMT_EQUATION
                lower_equation(st, s.eq)
            else:
                raise ParseError(kind)

    def equations(self):
        return [s.eq for s in self.stmts[: self.n] if s.kind == abi.STMT_EQUATION]
