"""A sandboxed interpreter for the JavaScript subset that scene coders write, with a three.js object model.

The reference executes each candidate module (`export default function generate(THREE) { ... }`) in a Node
worker with a 5 s timeout and a 256 MB heap cap, then serialises the returned Object3D tree to three.js
JSON (pipeline_service/modules/js_checker/validator/execute.js:46-47, serialize_worker.mjs). Node is not part
of this framework, so candidates run here instead: a tokenizer, a recursive-descent parser and a
tree-walking evaluator for ES2020 statements and expressions (let/const/var, functions and arrows with
default/rest/destructured parameters, objects, arrays, spread, template literals, for/for-of/for-in/while,
optional chaining, `??`), and a `THREE` namespace implemented natively (Object3D tree, primitive and
buffer geometries with baked transforms, materials, Color, Vector2/3, Euler, Matrix4, InstancedMesh,
MathUtils). Budgets replace the worker limits: an evaluation-step budget and a wall-clock deadline
(timeout), and caps on array lengths and string sizes (heap).

Isolation: JS values never reach Python attributes. Host objects answer only the property names their
tables list, so no Python internals (`__class__`, builtins) are reachable from a candidate.

`run_module(source)` -> `ModuleResult(root, error)`; `to_scene_json(root)` -> the scene JSON that
`phung5_b200.render.scene` rasterises.
"""
from __future__ import annotations

import json
import math
import re
import struct
import time
import uuid as _uuid
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Tuple

# --------------------------------------------------------------------------------------------------- errors


class JSError(Exception):
    """A JavaScript-level error (syntax, type, reference, or a thrown value)."""

    def __init__(self, kind: str, msg: str):
        super().__init__(f"{kind}: {msg}")
        self.kind = kind
        self.msg = msg


class JSBudget(JSError):
    pass


class _Break(Exception):
    def __init__(self, label=None):
        self.label = label


class _Continue(Exception):
    def __init__(self, label=None):
        self.label = label


class _Return(Exception):
    def __init__(self, value):
        self.value = value


class _Throw(Exception):
    def __init__(self, value):
        self.value = value


class _Undefined:
    _inst = None

    def __new__(cls):
        if cls._inst is None:
            cls._inst = super().__new__(cls)
        return cls._inst

    def __repr__(self):
        return "undefined"


UNDEF = _Undefined()

# ---------------------------------------------------------------------------------------------------- lexer

_PUNCT = sorted("""
>>>= ... === !== **= <<= >>= >>> &&= ||= ??= => == != <= >= && || ?? ?. ++ -- += -= *= /= %= &= |= ^= ** << >>
{ } ( ) [ ] ; , < > + - * / % & | ^ ! ~ ? : = . @ #
""".split(), key=len, reverse=True)
_KEYWORDS = {"var", "let", "const", "function", "return", "if", "else", "for", "while", "do", "break", "continue",
             "new", "true", "false", "null", "undefined", "typeof", "instanceof", "in", "of", "export", "default",
             "import", "class", "this", "throw", "try", "catch", "finally", "switch", "case", "void", "delete",
             "async", "await", "yield"}
_ID_START = re.compile(r"[A-Za-z_$]")
_ID_RE = re.compile(r"[A-Za-z0-9_$]*")
_NUM_RE = re.compile(r"0[xX][0-9a-fA-F_]+|0[bB][01_]+|0[oO][0-7_]+|(?:\d[\d_]*\.?[\d_]*|\.\d[\d_]*)(?:[eE][+-]?\d+)?")


@dataclass
class Tok:
    kind: str       # num, str, tpl, id, kw, p (punct), eof
    val: Any
    pos: int
    nl: bool = False  # a line break precedes this token


def tokenize(src: str) -> List[Tok]:
    toks: List[Tok] = []
    i, n, nl = 0, len(src), False
    while i < n:
        c = src[i]
        if c in " \t\r\f\v﻿":
            i += 1
            continue
        if c == "\n":
            nl = True
            i += 1
            continue
        if src.startswith("//", i):
            j = src.find("\n", i)
            i = n if j < 0 else j
            continue
        if src.startswith("/*", i):
            j = src.find("*/", i + 2)
            if j < 0:
                raise JSError("SyntaxError", "unterminated comment")
            nl = nl or "\n" in src[i:j]
            i = j + 2
            continue
        start = i
        if c.isdigit() or (c == "." and i + 1 < n and src[i + 1].isdigit()):
            m = _NUM_RE.match(src, i)
            text = m.group(0).replace("_", "")
            if text[:2].lower() == "0x":
                v = float(int(text[2:], 16))
            elif text[:2].lower() == "0b":
                v = float(int(text[2:], 2))
            elif text[:2].lower() == "0o":
                v = float(int(text[2:], 8))
            else:
                v = float(text)
            i = m.end()
            if i < n and src[i] == "n":
                raise JSError("SyntaxError", "BigInt literals are not supported")
            toks.append(Tok("num", v, start, nl))
        elif c in "'\"":
            s, i = _read_string(src, i + 1, c)
            toks.append(Tok("str", s, start, nl))
        elif c == "`":
            parts, i = _read_template(src, i + 1)
            toks.append(Tok("tpl", parts, start, nl))
        elif _ID_START.match(c) or ord(c) > 127:
            m = _ID_RE.match(src, i + 1)
            j = m.end()
            while j < n and ord(src[j]) > 127:
                j += 1
            word = src[i:j]
            i = j
            toks.append(Tok("kw" if word in _KEYWORDS else "id", word, start, nl))
        else:
            for p in _PUNCT:
                if src.startswith(p, i):
                    if p == "?." and i + 2 < n and src[i + 2].isdigit():
                        continue   # `a ?.5 : b` is a conditional
                    toks.append(Tok("p", p, start, nl))
                    i += len(p)
                    break
            else:
                raise JSError("SyntaxError", f"unexpected character {c!r} at {i}")
        nl = False
    toks.append(Tok("eof", None, n, nl))
    return toks


_ESC = {"n": "\n", "t": "\t", "r": "\r", "b": "\b", "f": "\f", "v": "\v", "0": "\0"}


def _read_string(src, i, q):
    out, n = [], len(src)
    while i < n:
        c = src[i]
        if c == q:
            return "".join(out), i + 1
        if c == "\\":
            i += 1
            e = src[i] if i < n else ""
            if e == "u":
                if src[i + 1] == "{":
                    j = src.index("}", i)
                    out.append(chr(int(src[i + 2:j], 16)))
                    i = j + 1
                else:
                    out.append(chr(int(src[i + 1:i + 5], 16)))
                    i += 5
                continue
            if e == "x":
                out.append(chr(int(src[i + 1:i + 3], 16)))
                i += 3
                continue
            if e == "\n":
                i += 1
                continue
            out.append(_ESC.get(e, e))
            i += 1
            continue
        if c == "\n":
            raise JSError("SyntaxError", "unterminated string")
        out.append(c)
        i += 1
    raise JSError("SyntaxError", "unterminated string")


def _read_template(src, i):
    """-> ([str | expression-source], end)."""
    parts, buf, n = [], [], len(src)
    while i < n:
        c = src[i]
        if c == "`":
            parts.append("".join(buf))
            return parts, i + 1
        if c == "\\":
            e = src[i + 1]
            buf.append(_ESC.get(e, e))
            i += 2
            continue
        if c == "$" and i + 1 < n and src[i + 1] == "{":
            parts.append("".join(buf))
            buf = []
            depth, j = 1, i + 2
            while j < n and depth:
                if src[j] == "{":
                    depth += 1
                elif src[j] == "}":
                    depth -= 1
                elif src[j] in "'\"":
                    _, j = _read_string(src, j + 1, src[j])
                    continue
                elif src[j] == "`":
                    _, j = _read_template(src, j + 1)
                    continue
                j += 1
            parts.append(("expr", src[i + 2:j - 1]))
            i = j
            continue
        buf.append(c)
        i += 1
    raise JSError("SyntaxError", "unterminated template literal")


# --------------------------------------------------------------------------------------------------- parser
# AST nodes are tuples: (tag, ...). Patterns: ("id", name) | ("objpat", [(key, pattern, default)], rest)
# | ("arrpat", [(pattern | None, default)], rest) .

_BINPREC = {"??": 1, "||": 2, "&&": 3, "|": 4, "^": 5, "&": 6, "==": 7, "!=": 7, "===": 7, "!==": 7,
            "<": 8, ">": 8, "<=": 8, ">=": 8, "instanceof": 8, "in": 8, "<<": 9, ">>": 9, ">>>": 9,
            "+": 10, "-": 10, "*": 11, "/": 11, "%": 11, "**": 12}
_ASSIGN = {"=", "+=", "-=", "*=", "/=", "%=", "**=", "<<=", ">>=", ">>>=", "&=", "|=", "^=", "&&=", "||=", "??="}


class Parser:
    def __init__(self, src: str):
        self.t = tokenize(src)
        self.i = 0
        self.no_in = False

    # token helpers
    @property
    def cur(self) -> Tok:
        return self.t[self.i]

    def peek(self, k=1) -> Tok:
        return self.t[min(self.i + k, len(self.t) - 1)]

    def at(self, val, kind=None) -> bool:
        c = self.cur
        return c.val == val and c.kind in ((kind,) if kind else ("p", "kw"))

    def eat(self, val, kind=None) -> bool:
        if self.at(val, kind):
            self.i += 1
            return True
        return False

    def expect(self, val):
        if not self.eat(val):
            c = self.cur
            raise JSError("SyntaxError", f"expected {val!r} but found {c.val!r} at {c.pos}")

    def ident(self) -> str:
        c = self.cur
        if c.kind == "id" or (c.kind == "kw" and c.val in ("of", "async", "await", "yield", "undefined")):
            self.i += 1
            return c.val
        raise JSError("SyntaxError", f"expected an identifier, found {c.val!r} at {c.pos}")

    def semi(self):
        if self.eat(";"):
            return
        c = self.cur
        if c.nl or c.kind == "eof" or self.at("}"):
            return
        raise JSError("SyntaxError", f"unexpected token {c.val!r} at {c.pos}")

    # program
    def program(self):
        body = []
        while self.cur.kind != "eof":
            body.append(self.statement(top=True))
        return ("block", body)

    def statement(self, top=False):
        c = self.cur
        if c.kind == "p":
            if c.val == "{":
                return self.block()
            if c.val == ";":
                self.i += 1
                return ("empty",)
        if c.kind == "kw":
            v = c.val
            if v in ("var", "let", "const"):
                d = self.declaration()
                self.semi()
                return d
            if v == "function":
                return self.function_decl()
            if v == "async" and self.peek().val == "function":
                raise JSError("SyntaxError", "async functions are not supported")
            if v == "return":
                self.i += 1
                if self.at(";") or self.at("}") or self.cur.nl or self.cur.kind == "eof":
                    self.eat(";")
                    return ("return", None)
                e = self.expression()
                self.semi()
                return ("return", e)
            if v == "if":
                self.i += 1
                self.expect("(")
                test = self.expression()
                self.expect(")")
                cons = self.statement()
                alt = self.statement() if self.eat("else") else None
                return ("if", test, cons, alt)
            if v == "for":
                return self.for_stmt()
            if v == "while":
                self.i += 1
                self.expect("(")
                test = self.expression()
                self.expect(")")
                return ("while", test, self.statement())
            if v == "do":
                self.i += 1
                body = self.statement()
                self.expect("while")
                self.expect("(")
                test = self.expression()
                self.expect(")")
                self.eat(";")
                return ("dowhile", body, test)
            if v in ("break", "continue"):
                self.i += 1
                label = None
                if self.cur.kind == "id" and not self.cur.nl:
                    label = self.cur.val
                    self.i += 1
                self.semi()
                return (v, label)
            if v == "throw":
                self.i += 1
                e = self.expression()
                self.semi()
                return ("throw", e)
            if v == "try":
                return self.try_stmt()
            if v == "switch":
                return self.switch_stmt()
            if v == "export":
                if not top:
                    raise JSError("SyntaxError", "export inside a block")
                self.i += 1
                if self.eat("default"):
                    if self.at("function"):
                        f = self.function_expr()
                        self.eat(";")
                        return ("export_default", f)
                    e = self.assign()
                    self.semi()
                    return ("export_default", e)
                if self.at("function"):
                    f = self.function_decl()
                    return ("export_named", f, f[1])
                if self.cur.val in ("const", "let", "var"):
                    d = self.declaration()
                    self.semi()
                    return ("export_decl", d)
                raise JSError("SyntaxError", "unsupported export form")
            if v == "import":
                raise JSError("SyntaxError", "import statements are not allowed (THREE is passed to generate)")
            if v == "class":
                node = self.class_def(need_name=True)
                return ("classdecl", node[1], node)
        if c.kind == "id" and self.peek().kind == "p" and self.peek().val == ":":
            self.i += 2
            return ("labeled", c.val, self.statement())
        e = self.expression()
        self.semi()
        return ("expr", e)

    def block(self):
        self.expect("{")
        body = []
        while not self.at("}"):
            if self.cur.kind == "eof":
                raise JSError("SyntaxError", "unexpected end of input")
            body.append(self.statement())
        self.i += 1
        return ("block", body)

    def declaration(self):
        kind = self.cur.val
        self.i += 1
        decls = []
        while True:
            target = self.pattern()
            init = self.assign() if self.eat("=") else None
            if init is None and kind == "const" and not (self.at("of") or self.at("in")):
                raise JSError("SyntaxError", "missing initializer in const declaration")
            decls.append((target, init))
            if not self.eat(","):
                break
        return ("decl", kind, decls)

    def pattern(self):
        if self.eat("{"):
            props, rest = [], None
            while not self.at("}"):
                if self.eat("..."):
                    rest = self.ident()
                    break
                if self.eat("["):
                    key = self.assign()
                    self.expect("]")
                    key = ("computed", key)
                else:
                    c = self.cur
                    if c.kind in ("str", "num"):
                        self.i += 1
                        key = _prop_key(c.val)
                    else:
                        key = c.val
                        self.i += 1
                if self.eat(":"):
                    target = self.pattern()
                else:
                    target = ("id", key)
                default = self.assign() if self.eat("=") else None
                props.append((key, target, default))
                if not self.eat(","):
                    break
            self.expect("}")
            return ("objpat", props, rest)
        if self.eat("["):
            elems, rest = [], None
            while not self.at("]"):
                if self.at(","):
                    self.i += 1
                    elems.append((None, None))
                    continue
                if self.eat("..."):
                    rest = self.pattern()
                    break
                target = self.pattern()
                default = self.assign() if self.eat("=") else None
                elems.append((target, default))
                if not self.eat(","):
                    break
            self.expect("]")
            return ("arrpat", elems, rest)
        return ("id", self.ident())

    def params(self):
        self.expect("(")
        ps, rest = [], None
        while not self.at(")"):
            if self.eat("..."):
                rest = self.pattern()
                break
            target = self.pattern()
            default = self.assign() if self.eat("=") else None
            ps.append((target, default))
            if not self.eat(","):
                break
        self.expect(")")
        return ps, rest

    def function_decl(self):
        self.expect("function")
        if self.eat("*"):
            raise JSError("SyntaxError", "generators are not supported")
        name = self.ident()
        ps, rest = self.params()
        body = self.block()
        return ("fundecl", name, ("func", name, ps, rest, body, False))

    def function_expr(self):
        self.expect("function")
        if self.eat("*"):
            raise JSError("SyntaxError", "generators are not supported")
        name = self.ident() if not self.at("(") else None
        ps, rest = self.params()
        body = self.block()
        return ("func", name, ps, rest, body, False)

    def for_stmt(self):
        self.expect("for")
        if self.at("await"):
            raise JSError("SyntaxError", "for await is not supported")
        self.expect("(")
        init = None
        if self.cur.val in ("var", "let", "const") and self.cur.kind == "kw":
            kind = self.cur.val
            save = self.i
            self.i += 1
            target = self.pattern()
            if self.at("of") or self.at("in"):
                op = self.cur.val
                self.i += 1
                it = self.assign() if op == "of" else self.expression()
                self.expect(")")
                return ("forof" if op == "of" else "forin", kind, target, it, self.statement())
            self.i = save
            self.no_in = True
            init = self.declaration()
            self.no_in = False
        elif not self.at(";"):
            save = self.i
            self.no_in = True
            e = self.expression()
            self.no_in = False
            if self.at("of") or self.at("in"):
                self.i = save
                target = self.pattern()
                op = self.cur.val
                self.i += 1
                it = self.assign() if op == "of" else self.expression()
                self.expect(")")
                return ("forof" if op == "of" else "forin", None, target, it, self.statement())
            init = ("expr", e)
        self.expect(";")
        test = None if self.at(";") else self.expression()
        self.expect(";")
        update = None if self.at(")") else self.expression()
        self.expect(")")
        return ("for", init, test, update, self.statement())

    def try_stmt(self):
        self.expect("try")
        body = self.block()
        param, handler, fin = None, None, None
        if self.eat("catch"):
            if self.eat("("):
                param = self.pattern()
                self.expect(")")
            handler = self.block()
        if self.eat("finally"):
            fin = self.block()
        return ("try", body, param, handler, fin)

    def switch_stmt(self):
        self.expect("switch")
        self.expect("(")
        disc = self.expression()
        self.expect(")")
        self.expect("{")
        cases = []
        while not self.eat("}"):
            if self.eat("default"):
                test = None
            else:
                self.expect("case")
                test = self.expression()
            self.expect(":")
            body = []
            while not (self.at("case") or self.at("default") or self.at("}")):
                body.append(self.statement())
            cases.append((test, body))
        return ("switch", disc, cases)

    # expressions
    def expression(self):
        e = self.assign()
        if self.at(","):
            seq = [e]
            while self.eat(","):
                seq.append(self.assign())
            return ("seq", seq)
        return e

    def _arrow_ahead(self) -> bool:
        """At `(`: is this the parameter list of an arrow function?"""
        depth, j = 0, self.i
        while j < len(self.t):
            tk = self.t[j]
            if tk.kind == "p" and tk.val in "([{" and len(tk.val) == 1:
                depth += 1
            elif tk.kind == "p" and tk.val in ")]}" and len(tk.val) == 1:
                depth -= 1
                if depth == 0:
                    nx = self.t[j + 1]
                    return nx.kind == "p" and nx.val == "=>" and not nx.nl
            elif tk.kind == "eof":
                return False
            j += 1
        return False

    def arrow_body(self, ps, rest):
        if self.at("{"):
            body = self.block()
            return ("func", None, ps, rest, body, True)
        save = self.no_in
        self.no_in = False
        e = self.assign()
        self.no_in = save
        return ("func", None, ps, rest, ("block", [("return", e)]), True)

    def assign(self):
        c = self.cur
        if c.kind == "kw" and c.val == "async" and (self.peek().val == "(" or self.peek().kind == "id"):
            raise JSError("SyntaxError", "async functions are not supported")
        if (c.kind == "id" or (c.kind == "kw" and c.val in ("of",))) and self.peek().val == "=>" and self.peek().kind == "p":
            self.i += 2
            return self.arrow_body([(("id", c.val), None)], None)
        if self.at("(") and self._arrow_ahead():
            ps, rest = self.params()
            self.expect("=>")
            return self.arrow_body(ps, rest)
        left = self.conditional()
        if self.cur.kind == "p" and self.cur.val in _ASSIGN:
            op = self.cur.val
            self.i += 1
            right = self.assign()
            if op == "=" and left[0] in ("object", "array"):
                return ("assign_pat", _to_pattern(left), right)
            if left[0] not in ("ident", "member"):
                raise JSError("SyntaxError", "invalid assignment target")
            return ("assign", op, left, right)
        return left

    def conditional(self):
        test = self.binary(0)
        if self.eat("?"):
            save = self.no_in
            self.no_in = False
            cons = self.assign()
            self.no_in = save
            self.expect(":")
            alt = self.assign()
            return ("cond", test, cons, alt)
        return test

    def binary(self, minp):
        left = self.unary()
        while True:
            c = self.cur
            op = c.val
            if not ((c.kind == "p" or (c.kind == "kw" and op in ("instanceof", "in"))) and op in _BINPREC):
                return left
            if op == "in" and self.no_in:
                return left
            p = _BINPREC[op]
            if p < minp:            # binds looser than the operator whose right operand this is
                return left
            self.i += 1
            right = self.binary(p if op == "**" else p + 1)
            if op in ("&&", "||", "??"):
                left = ("logic", op, left, right)
            else:
                left = ("bin", op, left, right)

    def unary(self):
        c = self.cur
        if c.kind == "p" and c.val in ("!", "-", "+", "~"):
            self.i += 1
            return ("unary", c.val, self.unary())
        if c.kind == "p" and c.val in ("++", "--"):
            self.i += 1
            return ("update", c.val, True, self.unary())
        if c.kind == "kw" and c.val in ("typeof", "void", "delete"):
            self.i += 1
            return ("unary", c.val, self.unary())
        if c.kind == "kw" and c.val == "await":
            raise JSError("SyntaxError", "await is not supported")
        return self.postfix()

    def postfix(self):
        e = self.call_member(self.primary())
        c = self.cur
        if c.kind == "p" and c.val in ("++", "--") and not c.nl:
            self.i += 1
            return ("update", c.val, False, e)
        return e

    def args(self):
        out = []
        self.expect("(")
        while not self.at(")"):
            if self.eat("..."):
                out.append(("spread", self.assign()))
            else:
                out.append(self.assign())
            if not self.eat(","):
                break
        self.expect(")")
        return out

    def call_member(self, e, allow_call=True):
        while True:
            c = self.cur
            if c.kind == "p" and c.val == ".":
                self.i += 1
                name = self.cur
                if name.kind not in ("id", "kw"):
                    raise JSError("SyntaxError", f"bad property name at {name.pos}")
                self.i += 1
                e = ("member", e, ("lit", name.val), False, False)
            elif c.kind == "p" and c.val == "?.":
                self.i += 1
                if self.at("("):
                    e = ("call", e, self.args(), True)
                elif self.eat("["):
                    k = self.expression()
                    self.expect("]")
                    e = ("member", e, k, True, True)
                else:
                    name = self.cur
                    self.i += 1
                    e = ("member", e, ("lit", name.val), True, False)
            elif c.kind == "p" and c.val == "[":
                self.i += 1
                k = self.expression()
                self.expect("]")
                e = ("member", e, k, False, True)
            elif c.kind == "p" and c.val == "(" and allow_call:
                e = ("call", e, self.args(), False)
            elif c.kind == "tpl":
                raise JSError("SyntaxError", "tagged templates are not supported")
            else:
                return e

    def primary(self):
        c = self.cur
        k = c.kind
        if k == "num" or k == "str":
            self.i += 1
            return ("lit", c.val)
        if k == "tpl":
            self.i += 1
            parts = [p if isinstance(p, str) else Parser(p[1]).expression_only() for p in c.val]
            return ("tpl", parts)
        if k == "id" and c.val != "super":
            self.i += 1
            return ("ident", c.val)
        if k in ("kw", "id"):
            v = c.val
            if v == "true" or v == "false":
                self.i += 1
                return ("lit", v == "true")
            if v == "null":
                self.i += 1
                return ("lit", None)
            if v == "undefined":
                self.i += 1
                return ("lit", UNDEF)
            if v == "function":
                return self.function_expr()
            if v == "new":
                self.i += 1
                if self.at("."):
                    raise JSError("SyntaxError", "new.target is not supported")
                callee = self.call_member(self.primary(), allow_call=False)
                a = self.args() if self.at("(") else []
                return ("new", callee, a)
            if v == "this":
                self.i += 1
                return ("this",)
            if v in ("of", "async"):
                self.i += 1
                return ("ident", v)
            if v == "class":
                return self.class_def(need_name=False)
            if v == "super":
                self.i += 1
                if self.at("("):
                    return ("super_call", self.args())
                if self.eat("."):
                    name = self.cur
                    self.i += 1
                    return ("super_member", ("lit", name.val))
                if self.eat("["):
                    k = self.expression()
                    self.expect("]")
                    return ("super_member", k)
                raise JSError("SyntaxError", "'super' must be called or followed by a property")
            if v == "import":
                raise JSError("SyntaxError", "dynamic import is not allowed")
        if k == "p":
            v = c.val
            if v == "(":
                self.i += 1
                save = self.no_in
                self.no_in = False
                e = self.expression()
                self.no_in = save
                self.expect(")")
                return e
            if v == "[":
                self.i += 1
                items = []
                while not self.at("]"):
                    if self.at(","):
                        self.i += 1
                        items.append(("lit", UNDEF))
                        continue
                    if self.eat("..."):
                        items.append(("spread", self.assign()))
                    else:
                        items.append(self.assign())
                    if not self.eat(","):
                        break
                self.expect("]")
                return ("array", items)
            if v == "{":
                return self.object_lit()
        raise JSError("SyntaxError", f"unexpected token {c.val!r} at {c.pos}")

    def class_def(self, need_name: bool):
        """class [Name] [extends Expr] { constructor / methods / get / set / static / fields }"""
        self.expect("class")
        name = None
        if self.cur.kind == "id":
            name = self.cur.val
            self.i += 1
        elif need_name:
            raise JSError("SyntaxError", "class declaration needs a name")
        parent = None
        if self.eat("extends", "id"):
            parent = self.call_member(self.primary())
        self.expect("{")
        members = []          # (kind, static, key, value): kind method | get | set | field | ctor
        while not self.eat("}"):
            if self.eat(";"):
                continue
            static = False
            if self.at("static", "id") and self.peek().val not in ("(", "=", ";", "}"):
                self.i += 1
                static = True
            kind = "method"
            if self.cur.val in ("get", "set") and self.cur.kind in ("id", "kw") and \
                    self.peek().val not in ("(", "=", ";", "}"):
                kind = self.cur.val
                self.i += 1
            if self.cur.kind == "p" and self.cur.val == "#":
                raise JSError("SyntaxError", "private class members are not supported")
            if self.eat("["):
                key = ("computed", self.assign())
                self.expect("]")
            else:
                c = self.cur
                if c.kind not in ("id", "kw", "str", "num"):
                    raise JSError("SyntaxError", f"bad class member name {c.val!r} at {c.pos}")
                self.i += 1
                key = _prop_key(c.val) if c.kind in ("str", "num") else c.val
            if self.at("("):
                ps, rest = self.params()
                body = self.block()
                fn = ("func", key if isinstance(key, str) else None, ps, rest, body, False)
                if key == "constructor" and not static and kind == "method":
                    members.append(("ctor", False, key, fn))
                else:
                    members.append((kind, static, key, fn))
            else:
                value = self.assign() if self.eat("=") else None
                self.semi()
                members.append(("field", static, key, value))
        return ("class", name, parent, members)

    def object_lit(self):
        self.expect("{")
        props = []
        while not self.at("}"):
            if self.eat("..."):
                props.append(("spread", self.assign()))
            else:
                c = self.cur
                accessor = None
                if c.kind in ("id", "kw") and c.val in ("get", "set") and \
                        self.peek().kind in ("id", "kw", "str", "num") and self.peek().val not in (",", ":", "(", "}"):
                    accessor = c.val
                    self.i += 1
                    c = self.cur
                if self.eat("["):
                    key = ("computed", self.assign())
                    self.expect("]")
                elif c.kind in ("id", "kw"):
                    self.i += 1
                    key = c.val
                elif c.kind in ("str", "num"):
                    self.i += 1
                    key = _prop_key(c.val)
                else:
                    raise JSError("SyntaxError", f"bad object key {c.val!r} at {c.pos}")
                if accessor is not None:
                    ps, rest = self.params()
                    body = self.block()
                    props.append((accessor, key, ("func", None, ps, rest, body, False)))
                elif self.eat(":"):
                    props.append(("kv", key, self.assign()))
                elif self.at("("):
                    ps, rest = self.params()
                    body = self.block()
                    props.append(("kv", key, ("func", key if isinstance(key, str) else None, ps, rest, body, False)))
                elif self.at("="):       # shorthand with default: only valid as a pattern
                    self.i += 1
                    props.append(("shorthand_default", key, self.assign()))
                else:
                    props.append(("kv", key, ("ident", key)))
            if not self.eat(","):
                break
        self.expect("}")
        return ("object", props)

    def expression_only(self):
        e = self.expression()
        if self.cur.kind != "eof":
            raise JSError("SyntaxError", "bad template expression")
        return e


def _prop_key(v) -> str:
    return _to_str(v) if not isinstance(v, str) else v


def _to_pattern(node):
    tag = node[0]
    if tag == "ident":
        return ("id", node[1])
    if tag == "member":
        return ("memberpat", node)
    if tag == "array":
        elems, rest = [], None
        for it in node[1]:
            if it[0] == "spread":
                rest = _to_pattern(it[1])
            elif it == ("lit", UNDEF):
                elems.append((None, None))
            elif it[0] == "assign" and it[1] == "=":
                elems.append((_to_pattern(it[2]), it[3]))
            else:
                elems.append((_to_pattern(it), None))
        return ("arrpat", elems, rest)
    if tag == "object":
        props, rest = [], None
        for p in node[1]:
            if p[0] == "spread":
                rest = p[1][1]
            elif p[0] == "shorthand_default":
                props.append((p[1], ("id", p[1]), p[2]))
            else:
                val = p[2]
                if val[0] == "assign" and val[1] == "=":
                    props.append((p[1], _to_pattern(val[2]), val[3]))
                else:
                    props.append((p[1], _to_pattern(val), None))
        return ("objpat", props, rest)
    if tag == "assign_pat":
        return node[1]
    raise JSError("SyntaxError", "invalid destructuring target")


# ---------------------------------------------------------------------------------------------- value model


class JSObject:
    """A plain JS object: ordered own properties and an optional prototype (another JSObject)."""
    __slots__ = ("props", "proto")
    cls_name = "Object"

    def __init__(self, props: Optional[dict] = None, proto: Optional["JSObject"] = None):
        self.props = {} if props is None else props
        self.proto = proto

    def js_get(self, key: str):
        return self.props.get(key, UNDEF)

    def js_set(self, key: str, value):
        self.props[key] = value

    def js_keys(self) -> List[str]:
        return list(self.props.keys())

    def js_has(self, key: str) -> bool:
        return key in self.props


class JSArray:
    __slots__ = ("items",)
    cls_name = "Array"

    def __init__(self, items: Optional[list] = None):
        self.items = [] if items is None else items


class TypedArray(JSArray):
    """Float32Array, Uint16Array, ...: a fixed-length array whose elements are stored converted to its element
    type (float32 rounding, modular integers, clamped bytes). A BufferAttribute holds the module's own typed
    array, so writes through either are seen by both, as in three.js."""
    __slots__ = ("kind",)

    def __init__(self, kind: str, items: Optional[list] = None, coerced: bool = False):
        super().__init__([] if items is None else (items if coerced else _typed_values(kind, items)))
        self.kind = kind

    @property
    def cls_name(self):
        return self.kind


class JSFunction:
    __slots__ = ("name", "params", "rest", "body", "env", "arrow", "this", "props", "home")

    def __init__(self, name, params, rest, body, env, arrow, this=UNDEF):
        self.name, self.params, self.rest, self.body = name, params, rest, body
        self.env, self.arrow, self.this = env, arrow, this
        self.props = {}
        self.home = None          # class methods: the object they were defined on (for `super.x`)


class Accessor:
    """A getter / setter pair stored as a property value (object literals and classes)."""
    __slots__ = ("get", "set")

    def __init__(self, get=None, set=None):
        self.get, self.set = get, set


class JSClass:
    """A class: constructor, prototype object (methods and accessors), parent (a class, a host constructor
    such as THREE.Group, or None), instance field initialisers, and static members in `props`."""
    __slots__ = ("name", "ctor", "proto", "parent", "fields", "props", "env")

    def __init__(self, name, ctor, proto, parent, fields, env):
        self.name, self.ctor, self.proto, self.parent, self.fields, self.env = name, ctor, proto, parent, fields, env
        self.props = {}


class Native:
    """A host function: fn(this, args) -> value. `ctor` builds for `new` (and is used when callable as class)."""
    __slots__ = ("name", "fn", "ctor", "props")

    def __init__(self, name: str, fn: Optional[Callable] = None, ctor: Optional[Callable] = None,
                 props: Optional[dict] = None):
        self.name, self.fn, self.ctor = name, fn, ctor
        self.props = props or {}


class Env:
    __slots__ = ("vars", "parent", "consts")

    def __init__(self, parent: Optional["Env"] = None):
        self.vars: Dict[str, Any] = {}
        self.parent = parent
        self.consts: set = set()

    def lookup(self, name):
        e = self
        while e is not None:
            if name in e.vars:
                return e
            e = e.parent
        return None

    def get(self, name):
        e = self.lookup(name)
        if e is None:
            raise _Throw(_error_obj("ReferenceError", f"{name} is not defined"))
        v = e.vars[name]
        if v is _TDZ:
            raise _Throw(_error_obj("ReferenceError", f"cannot access {name} before initialization"))
        return v

    def set(self, name, value):
        e = self.lookup(name)
        if e is None:
            raise _Throw(_error_obj("ReferenceError", f"{name} is not defined"))
        if name in e.consts:
            raise _Throw(_error_obj("TypeError", f"assignment to constant variable {name}"))
        e.vars[name] = value

    def declare(self, name, value, const=False):
        self.vars[name] = value
        if const:
            self.consts.add(name)


_TDZ = object()
_MISSING = object()


def _mine(ex, labels) -> bool:
    """A break / continue belongs to this loop: unlabeled, or naming one of the loop's labels."""
    return ex.label is None or ex.label in labels


def _error_obj(kind, msg):
    return JSObject({"name": kind, "message": msg})


def _num_to_str(v: float) -> str:
    if v != v:
        return "NaN"
    if v in (math.inf, -math.inf):
        return "Infinity" if v > 0 else "-Infinity"
    if v == int(v) and abs(v) < 1e21:
        return str(int(v))
    r = repr(v)
    if "e" in r:
        m, e = r.split("e")
        e = int(e)
        return f"{m}e{'+' if e > 0 else '-'}{abs(e)}"
    return r


def _to_str(v) -> str:
    if isinstance(v, str):
        return v
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, float):
        return _num_to_str(v)
    if isinstance(v, int):
        return str(v)
    if v is None:
        return "null"
    if v is UNDEF:
        return "undefined"
    if isinstance(v, JSArray):
        return ",".join("" if x is None or x is UNDEF else _to_str(x) for x in v.items)
    if isinstance(v, (JSFunction, Native)):
        return f"function {getattr(v, 'name', '') or ''}() {{ [code] }}"
    if isinstance(v, JSClass):
        return f"class {v.name} {{ }}"
    if isinstance(v, Host):
        return v.to_string()
    if isinstance(v, JSObject):
        return "[object Object]"
    return str(v)


def _to_num(v) -> float:
    if isinstance(v, bool):
        return 1.0 if v else 0.0
    if isinstance(v, (int, float)):
        return float(v)
    if v is None:
        return 0.0
    if v is UNDEF:
        return math.nan
    if isinstance(v, str):
        s = v.strip()
        if not s:
            return 0.0
        try:
            if s[:2].lower() == "0x":
                return float(int(s, 16))
            return float(s)
        except ValueError:
            return math.nan
    if isinstance(v, JSArray):
        if not v.items:
            return 0.0
        if len(v.items) == 1:
            return _to_num(v.items[0])
    return math.nan


def _truthy(v) -> bool:
    if isinstance(v, bool):
        return v
    if isinstance(v, float):
        return v != 0.0 and v == v
    if isinstance(v, int):
        return v != 0
    if isinstance(v, str):
        return v != ""
    return not (v is None or v is UNDEF)


def _typeof(v) -> str:
    if v is UNDEF:
        return "undefined"
    if isinstance(v, bool):
        return "boolean"
    if isinstance(v, (int, float)):
        return "number"
    if isinstance(v, str):
        return "string"
    if isinstance(v, (JSFunction, Native, JSClass)):
        return "function"
    return "object"


def _strict_eq(a, b) -> bool:
    ta, tb = _typeof(a), _typeof(b)
    if ta != tb:
        return False
    if ta == "number":
        return float(a) == float(b)
    if ta in ("string", "boolean", "undefined"):
        return a == b
    return a is b


def _loose_eq(a, b) -> bool:
    if (a is None or a is UNDEF) and (b is None or b is UNDEF):
        return True
    if a is None or a is UNDEF or b is None or b is UNDEF:
        return False
    ta, tb = _typeof(a), _typeof(b)
    if ta == tb:
        return _strict_eq(a, b)
    if ta in ("number", "string", "boolean") and tb in ("number", "string", "boolean"):
        return _to_num(a) == _to_num(b)
    return False


def _to_int32(v) -> int:
    x = _to_num(v)
    if x != x or x in (math.inf, -math.inf):
        return 0
    x = int(x) & 0xFFFFFFFF
    return x - (1 << 32) if x >= (1 << 31) else x


def _index(v) -> Optional[int]:
    if isinstance(v, (int, float)) and not isinstance(v, bool):
        f = float(v)
        if f == f and f == int(f) and f >= 0:
            return int(f)
    if isinstance(v, str) and v.isdigit():
        return int(v)
    return None


# ----------------------------------------------------------------------------------------------- interpreter


@dataclass
class Limits:
    steps: int = 20_000_000
    seconds: float = 5.0
    array_len: int = 2_000_000
    string_len: int = 4_000_000


class Interp:
    def __init__(self, limits: Optional[Limits] = None, seed: int = 0):
        self.lim = limits or Limits()
        self.steps = 0
        self.deadline = time.monotonic() + self.lim.seconds
        self.rng_state = (seed * 2654435761 + 0x9E3779B9) & 0xFFFFFFFF or 1
        self.globals = Env()
        self.exports: Dict[str, Any] = {}
        _install_globals(self)

    # budget
    def tick(self):
        self.steps += 1
        if self.steps > self.lim.steps:
            raise JSBudget("RangeError", f"step budget of {self.lim.steps} exceeded")
        if (self.steps & 0x3FFF) == 0 and time.monotonic() > self.deadline:
            raise JSBudget("RangeError", f"execution exceeded {self.lim.seconds:.1f}s")

    def random(self) -> float:
        """xorshift32: deterministic Math.random for reproducible candidates."""
        x = self.rng_state
        x ^= (x << 13) & 0xFFFFFFFF
        x ^= x >> 17
        x ^= (x << 5) & 0xFFFFFFFF
        self.rng_state = x & 0xFFFFFFFF
        return self.rng_state / 4294967296.0

    # statements
    def run_program(self, prog):
        env = self.globals
        self.hoist(prog[1], env)
        for st in prog[1]:
            name = _intrinsic_name(st)
            if name is not None:
                env.declare(name, _INTRINSICS[name][1](self), const=True)
                continue
            self.exec(st, env)

    def hoist(self, body, env):
        for st in body:
            tag = st[0]
            if tag == "fundecl":
                env.declare(st[1], self.make_func(st[2], env))
            elif tag == "export_named" and st[1][0] == "fundecl":
                env.declare(st[2], self.make_func(st[1][2], env))
            elif tag == "decl" and st[1] == "var":
                for target, _ in st[2]:
                    for nm in _pattern_names(target):
                        if nm not in env.vars:
                            env.declare(nm, UNDEF)
            elif tag == "decl":
                for target, _ in st[2]:
                    for nm in _pattern_names(target):
                        env.vars[nm] = _TDZ
            elif tag == "classdecl":
                env.vars[st[1]] = _TDZ

    def make_func(self, node, env, this=UNDEF):
        _, name, ps, rest, body, arrow = node
        return JSFunction(name, ps, rest, body, env, arrow, this)

    def exec_block(self, body, env):
        self.hoist(body, env)
        for st in body:
            self.exec(st, env)

    def exec(self, st, env, labels=()):
        self.tick()
        tag = st[0]
        if tag == "expr":
            self.eval(st[1], env)
        elif tag == "decl":
            kind = st[1]
            for target, init in st[2]:
                v = UNDEF if init is None else self.eval(init, env)
                if kind == "var" and init is None:
                    continue
                self.bind(target, v, env, kind)
        elif tag == "return":
            raise _Return(UNDEF if st[1] is None else self.eval(st[1], env))
        elif tag == "if":
            if _truthy(self.eval(st[1], env)):
                self.exec(st[2], Env(env) if st[2][0] == "block" else env) if st[2][0] != "block" \
                    else self.exec_block(st[2][1], Env(env))
            elif st[3] is not None:
                if st[3][0] == "block":
                    self.exec_block(st[3][1], Env(env))
                else:
                    self.exec(st[3], env)
        elif tag == "block":
            self.exec_block(st[1], Env(env))
        elif tag == "for":
            self.exec_for(st, env, labels)
        elif tag == "forof":
            self.exec_forof(st, env, labels)
        elif tag == "forin":
            _, kind, target, it, body = st
            obj = self.eval(it, env)
            keys = _own_keys(obj)
            for k in keys:
                self.tick()
                loop = Env(env)
                if kind is None:
                    self.assign_pattern(target, k, env)
                else:
                    self.bind(target, k, loop, kind)
                try:
                    self.exec_body(body, loop)
                except _Break as b:
                    if _mine(b, labels):
                        break
                    raise
                except _Continue as c:
                    if _mine(c, labels):
                        continue
                    raise
        elif tag == "while":
            while _truthy(self.eval(st[1], env)):
                self.tick()
                try:
                    self.exec_body(st[2], Env(env))
                except _Break as b:
                    if _mine(b, labels):
                        break
                    raise
                except _Continue as c:
                    if _mine(c, labels):
                        continue
                    raise
        elif tag == "dowhile":
            while True:
                self.tick()
                try:
                    self.exec_body(st[1], Env(env))
                except _Break as b:
                    if _mine(b, labels):
                        break
                    raise
                except _Continue as c:
                    if not _mine(c, labels):
                        raise
                if not _truthy(self.eval(st[2], env)):
                    break
        elif tag == "break":
            raise _Break(st[1] if len(st) > 1 else None)
        elif tag == "continue":
            raise _Continue(st[1] if len(st) > 1 else None)
        elif tag == "labeled":
            inner = st[2]
            if inner[0] in ("for", "forof", "forin", "while", "dowhile"):
                self.exec(inner, env, labels + (st[1],))
            else:
                try:
                    self.exec(inner, env)
                except _Break as b:
                    if b.label != st[1]:
                        raise
        elif tag == "classdecl":
            env.declare(st[1], self.make_class(st[2], env))
        elif tag == "fundecl":
            pass   # hoisted
        elif tag == "empty":
            pass
        elif tag == "throw":
            raise _Throw(self.eval(st[1], env))
        elif tag == "try":
            self.exec_try(st, env)
        elif tag == "switch":
            self.exec_switch(st, env)
        elif tag == "export_default":
            v = self.eval(st[1], env)
            self.exports["default"] = v
        elif tag == "export_named":
            self.exports[st[2]] = env.get(st[2])
        elif tag == "export_decl":
            self.exec(st[1], env)
            for target, _ in st[1][2]:
                for nm in _pattern_names(target):
                    self.exports[nm] = env.get(nm)
        else:
            raise JSError("SyntaxError", f"unsupported statement {tag}")

    def exec_body(self, st, env):
        if st[0] == "block":
            self.exec_block(st[1], env)
        else:
            self.exec(st, env)

    def exec_for(self, st, env, labels=()):
        _, init, test, update, body = st
        loop_env = Env(env)
        per_iter = init is not None and init[0] == "decl" and init[1] in ("let", "const")
        if init is not None:
            if init[0] == "decl":
                self.hoist([init], loop_env)
            self.exec(init, loop_env)
        while True:
            self.tick()
            if test is not None and not _truthy(self.eval(test, loop_env)):
                break
            it_env = Env(loop_env)
            if per_iter:   # closures capture a per-iteration copy of let bindings
                it_env = Env(env)
                it_env.vars.update(loop_env.vars)
                it_env.consts = set(loop_env.consts)
            try:
                self.exec_body(body, Env(it_env))
            except _Break as b:
                if _mine(b, labels):
                    break
                raise
            except _Continue as c:
                if not _mine(c, labels):
                    raise
            if per_iter:
                loop_env.vars.update({k: it_env.vars[k] for k in loop_env.vars})
            if update is not None:
                self.eval(update, loop_env)

    def exec_forof(self, st, env, labels=()):
        _, kind, target, it, body = st
        seq = self.iterate(self.eval(it, env))
        for v in seq:
            self.tick()
            loop = Env(env)
            if kind is None:
                self.assign_pattern(target, v, env)
            else:
                self.bind(target, v, loop, kind)
            try:
                self.exec_body(body, loop)
            except _Break as b:
                if _mine(b, labels):
                    break
                raise
            except _Continue as c:
                if _mine(c, labels):
                    continue
                raise

    def exec_try(self, st, env):
        _, body, param, handler, fin = st
        try:
            self.exec_block(body[1], Env(env))
        except (_Throw, JSError) as ex:
            if isinstance(ex, JSBudget) or handler is None:
                raise
            val = ex.value if isinstance(ex, _Throw) else _error_obj(ex.kind, ex.msg)
            henv = Env(env)
            if param is not None:
                self.bind(param, val, henv, "let")
            self.exec_block(handler[1], henv)
        finally:
            if fin is not None:
                self.exec_block(fin[1], Env(env))

    def exec_switch(self, st, env):
        _, disc, cases = st
        d = self.eval(disc, env)
        senv = Env(env)
        matched = False
        try:
            for pass_default in (False, True):
                for test, body in cases:
                    if not matched:
                        if test is None:
                            if not pass_default:
                                continue
                        elif pass_default or not _strict_eq(d, self.eval(test, senv)):
                            continue
                        matched = True
                    for s in body:
                        self.exec(s, senv)
                if matched:
                    break
        except _Break as b:
            if b.label is not None:
                raise

    def iterate(self, v) -> list:
        if isinstance(v, JSArray):
            return list(v.items)
        if isinstance(v, str):
            return list(v)
        if isinstance(v, Host) and v.iterable() is not None:
            return v.iterable()
        raise _Throw(_error_obj("TypeError", f"{_typeof(v)} is not iterable"))

    # binding
    def bind(self, target, value, env, kind):
        tag = target[0]
        if tag == "id":
            env.declare(target[1], value, const=(kind == "const"))
        elif tag == "objpat":
            self.destructure_obj(target, value, lambda p, v: self.bind(p, v, env, kind), env)
        elif tag == "arrpat":
            self.destructure_arr(target, value, lambda p, v: self.bind(p, v, env, kind), env)
        else:
            raise JSError("SyntaxError", "invalid binding")

    def assign_pattern(self, target, value, env):
        tag = target[0]
        if tag == "id":
            env.set(target[1], value)
        elif tag == "memberpat":
            m = target[1]
            self.put(self.eval(m[1], env), self.member_key(m, env), value)
        elif tag == "objpat":
            self.destructure_obj(target, value, lambda p, v: self.assign_pattern(p, v, env), env)
        elif tag == "arrpat":
            self.destructure_arr(target, value, lambda p, v: self.assign_pattern(p, v, env), env)

    def destructure_obj(self, target, value, put, env):
        if value is None or value is UNDEF:
            raise _Throw(_error_obj("TypeError", "cannot destructure undefined"))
        used = []
        for key, pat, default in target[1]:
            k = _to_str(self.eval(key[1], env)) if isinstance(key, tuple) else key
            used.append(k)
            v = self.get(value, k)
            if v is UNDEF and default is not None:
                v = self.eval(default, env)
            put(pat, v)
        if target[2] is not None:
            rest = JSObject({k: self.get(value, k) for k in _own_keys(value) if k not in used})
            put(("id", target[2]), rest)

    def destructure_arr(self, target, value, put, env):
        items = self.iterate(value)
        for i, (pat, default) in enumerate(target[1]):
            if pat is None:
                continue
            v = items[i] if i < len(items) else UNDEF
            if v is UNDEF and default is not None:
                v = self.eval(default, env)
            put(pat, v)
        if target[2] is not None:
            put(target[2], JSArray(items[len(target[1]):]))

    # calls
    def call(self, f, this, args, super_fn=None):
        self.tick()
        if isinstance(f, JSFunction):
            env = Env(f.env)
            if not f.arrow:
                env.declare("this", this if this is not UNDEF else f.this)
                env.declare("arguments", JSArray(list(args)))
                if f.home is not None:
                    env.declare("%home", f.home)
                if super_fn is not None:
                    env.declare("%super", _nat("super", lambda i, t, x, _e=env: super_fn(x, _e)))
            for i, (pat, default) in enumerate(f.params):
                v = args[i] if i < len(args) else UNDEF
                if v is UNDEF and default is not None:
                    v = self.eval(default, env)
                self.bind(pat, v, env, "let")
            if f.rest is not None:
                self.bind(f.rest, JSArray(list(args[len(f.params):])), env, "let")
            try:
                self.exec_block(f.body[1], env)
            except _Return as r:
                return r.value
            return UNDEF
        if isinstance(f, Native):
            if f.fn is None:
                raise _Throw(_error_obj("TypeError", f"class constructor {f.name} cannot be invoked without 'new'"))
            return f.fn(self, this, list(args))
        if isinstance(f, JSClass):
            raise _Throw(_error_obj("TypeError", f"class constructor {f.name} cannot be invoked without 'new'"))
        raise _Throw(_error_obj("TypeError", f"{_to_str(f)[:40]} is not a function"))

    def construct(self, f, args, new_target=None):
        self.tick()
        if isinstance(f, JSClass):
            return self.construct_class(f, list(args), new_target or f)
        if isinstance(f, Native) and f.ctor is not None:
            obj = f.ctor(self, list(args))
            if new_target is not None and isinstance(obj, JSObject):
                obj.proto = new_target.proto
            return obj
        if isinstance(f, JSFunction) and not f.arrow:
            obj = JSObject(proto=new_target.proto if new_target is not None else self.fn_prototype(f))
            r = self.call(f, obj, args)
            return r if isinstance(r, (JSObject, JSArray, Host)) else obj
        raise _Throw(_error_obj("TypeError", f"{getattr(f, 'name', _typeof(f))} is not a constructor"))

    @staticmethod
    def fn_prototype(f: JSFunction) -> JSObject:
        p = f.props.get("prototype")
        if not isinstance(p, JSObject):
            p = JSObject()
            f.props["prototype"] = p
        return p

    def make_class(self, node, env) -> JSClass:
        _, name, parent_e, members = node
        parent = None
        if parent_e is not None:
            parent = self.eval(parent_e, env)
            if parent is not None and not isinstance(parent, (JSClass, Native, JSFunction)):
                raise _Throw(_error_obj("TypeError", "class extends value is not a constructor"))
        cenv = Env(env)
        proto = JSObject(proto=parent.proto if isinstance(parent, JSClass) else
                         (self.fn_prototype(parent) if isinstance(parent, JSFunction) else None))
        cls = JSClass(name or "", None, proto, parent, [], cenv)
        if name:
            cenv.declare(name, cls, const=True)
        for kind, static, key, value in members:
            k = _to_str(self.eval(key[1], cenv)) if isinstance(key, tuple) else key
            target = cls.props if static else proto.props
            if kind == "ctor":
                cls.ctor = self.make_func(value, cenv)
                cls.ctor.home = proto
            elif kind == "field":
                if static:
                    fenv = Env(cenv)
                    fenv.declare("this", cls)
                    cls.props[k] = UNDEF if value is None else self.eval(value, fenv)
                else:
                    cls.fields.append((k, value))
            else:
                fn = self.make_func(value, cenv)
                fn.home = cls if static else proto
                if kind == "method":
                    target[k] = fn
                else:
                    acc = target.get(k)
                    if not isinstance(acc, Accessor):
                        acc = Accessor()
                        target[k] = acc
                    if kind == "get":
                        acc.get = fn
                    else:
                        acc.set = fn
        return cls

    def init_fields(self, cls: JSClass, obj) -> None:
        for k, value in cls.fields:
            fenv = Env(cls.env)
            fenv.declare("this", obj)
            fenv.declare("%home", cls.proto)
            self.put(obj, k, UNDEF if value is None else self.eval(value, fenv))

    def construct_class(self, cls: JSClass, args, nt: JSClass):
        parent = cls.parent
        if parent is None:
            obj = JSObject(proto=nt.proto)
            self.init_fields(cls, obj)
            if cls.ctor is not None:
                r = self.call(cls.ctor, obj, args)
                if isinstance(r, (JSObject, JSArray)):
                    return r
            return obj
        made = []

        def do_super(sargs, fenv):
            if made:
                raise _Throw(_error_obj("ReferenceError", "super constructor may only be called once"))
            o = self.construct(parent, sargs, new_target=nt)
            made.append(o)
            if fenv is not None:
                fenv.vars["this"] = o
            self.init_fields(cls, o)
            return UNDEF
        if cls.ctor is None:
            do_super(list(args), None)
            return made[0]
        r = self.call(cls.ctor, _TDZ, args, super_fn=do_super)
        if isinstance(r, (JSObject, JSArray)):
            return r
        if not made:
            raise _Throw(_error_obj("ReferenceError", "derived class constructor must call super()"))
        return made[0]

    def proto_get(self, proto, key: str, receiver):
        """Property `key` found on a prototype chain starting at `proto` (accessors called on `receiver`)."""
        depth = 0
        while proto is not None and depth < 64:
            v = proto.props.get(key, _MISSING)
            if v is not _MISSING:
                if isinstance(v, Accessor):
                    return UNDEF if v.get is None else self.call(v.get, receiver, [])
                return v
            proto = proto.proto
            depth += 1
        return _MISSING

    def proto_setter(self, proto, key: str):
        depth = 0
        while proto is not None and depth < 64:
            v = proto.props.get(key, _MISSING)
            if v is not _MISSING:
                return v if isinstance(v, Accessor) else None
            proto = proto.proto
            depth += 1
        return None

    # property access
    def get(self, obj, key):
        if isinstance(obj, JSArray):
            idx = _index(key)
            if idx is not None:
                return obj.items[idx] if idx < len(obj.items) else UNDEF
            if isinstance(obj, TypedArray):
                return _typed_method(self, obj, _to_str(key))
            return _array_method(self, obj, _to_str(key))
        if isinstance(obj, Host):
            k = _to_str(key)
            if obj.proto is not None and k not in obj.props:       # a class built on a host object
                w = self.proto_get(obj.proto, k, obj)
                if w is not _MISSING:
                    return w
            return obj.js_get(self, k)
        if isinstance(obj, JSObject):
            k = _to_str(key)
            v = obj.props.get(k, _MISSING)
            if v is _MISSING:
                if obj.proto is not None:
                    v = self.proto_get(obj.proto, k, obj)
                if v is _MISSING:
                    return _OBJECT_PROTO[k](self, obj) if k in _OBJECT_PROTO else UNDEF
            if isinstance(v, Accessor):
                return UNDEF if v.get is None else self.call(v.get, obj, [])
            return v
        if isinstance(obj, JSClass):
            k = _to_str(key)
            c = obj
            while isinstance(c, JSClass):
                if k in c.props:
                    v = c.props[k]
                    return self.call(v.get, obj, []) if isinstance(v, Accessor) and v.get else v
                c = c.parent
            if isinstance(c, (Native, JSFunction)) and k in c.props:
                return c.props[k]
            if k == "name":
                return obj.name
            if k == "prototype":
                return obj.proto
            if k in ("call", "apply", "bind"):
                return _function_method(self, obj, k)
            return UNDEF
        if isinstance(obj, str):
            idx = _index(key)
            if idx is not None:
                return obj[idx] if idx < len(obj) else UNDEF
            return _string_method(self, obj, _to_str(key))
        if isinstance(obj, (int, float)) and not isinstance(obj, bool):
            return _number_method(self, float(obj), _to_str(key))
        if isinstance(obj, (JSFunction, Native)):
            k = _to_str(key)
            if k in obj.props:
                return obj.props[k]
            if k == "prototype" and isinstance(obj, JSFunction) and not obj.arrow:
                return self.fn_prototype(obj)
            if k == "name":
                return obj.name or ""
            if k in ("call", "apply", "bind"):
                return _function_method(self, obj, k)
            return UNDEF
        if obj is None or obj is UNDEF:
            raise _Throw(_error_obj("TypeError", f"cannot read properties of {_to_str(obj)} (reading '{_to_str(key)}')"))
        return UNDEF

    def put(self, obj, key, value):
        if isinstance(obj, TypedArray):
            idx = _index(key)
            if idx is not None and idx < len(obj.items):
                obj.items[idx] = _typed_value(obj.kind, value)
            return                                      # out-of-range indices and length are ignored
        if isinstance(obj, JSArray):
            idx = _index(key)
            if idx is not None:
                if idx >= self.lim.array_len:
                    raise JSBudget("RangeError", "array too large")
                if idx >= len(obj.items):
                    obj.items.extend([UNDEF] * (idx + 1 - len(obj.items)))
                obj.items[idx] = value
                return
            if _to_str(key) == "length":
                n = int(_to_num(value))
                if n > self.lim.array_len:
                    raise JSBudget("RangeError", "array too large")
                del obj.items[n:]
                obj.items.extend([UNDEF] * (n - len(obj.items)))
                return
            raise _Throw(_error_obj("TypeError", f"cannot set property {_to_str(key)} of an array"))
        if isinstance(obj, Host):
            k = _to_str(key)
            if obj.proto is not None and k not in obj.props:
                acc = self.proto_setter(obj.proto, k)
                if acc is not None:
                    if acc.set is not None:
                        self.call(acc.set, obj, [value])
                    return
            obj.js_set(self, k, value)
            return
        if isinstance(obj, JSObject):
            k = _to_str(key)
            cur = obj.props.get(k, _MISSING)
            if cur is _MISSING and obj.proto is not None:
                cur = self.proto_setter(obj.proto, k) or _MISSING
            if isinstance(cur, Accessor):
                if cur.set is not None:
                    self.call(cur.set, obj, [value])
                return
            obj.props[k] = value
            return
        if isinstance(obj, (JSFunction, Native, JSClass)):
            obj.props[_to_str(key)] = value
            return
        if obj is None or obj is UNDEF:
            raise _Throw(_error_obj("TypeError", f"cannot set properties of {_to_str(obj)}"))
        # primitives: silently ignored (sloppy mode)

    def member_key(self, node, env):
        k = node[2]
        return k[1] if k[0] == "lit" else self.eval(k, env)

    # expressions
    def eval(self, e, env):
        tag = e[0]
        if tag == "lit":
            return e[1]
        if tag == "ident":
            return env.get(e[1])
        if tag == "member":
            obj = self.eval(e[1], env)
            if e[3] and (obj is None or obj is UNDEF):
                return UNDEF
            return self.get(obj, self.member_key(e, env))
        if tag == "call":
            callee = e[1]
            if callee[0] == "super_member":
                this = self.eval(("this",), env)
                f = self.super_get(self.member_super_key(callee, env), env, this)
                return self.call(f, this, self.eval_args(e[2], env))
            if callee[0] == "member":
                this = self.eval(callee[1], env)
                if callee[3] and (this is None or this is UNDEF):
                    return UNDEF
                f = self.get(this, self.member_key(callee, env))
            else:
                this = UNDEF
                f = self.eval(callee, env)
            if e[3] and (f is None or f is UNDEF):
                return UNDEF
            if f is UNDEF or f is None:
                name = callee[2][1] if callee[0] == "member" and callee[2][0] == "lit" else \
                    (callee[1] if callee[0] == "ident" else "expression")
                raise _Throw(_error_obj("TypeError", f"{name} is not a function"))
            return self.call(f, this, self.eval_args(e[2], env))
        if tag == "bin":
            return self.binop(e[1], self.eval(e[2], env), self.eval(e[3], env))
        if tag == "logic":
            a = self.eval(e[2], env)
            op = e[1]
            if op == "&&":
                return self.eval(e[3], env) if _truthy(a) else a
            if op == "||":
                return a if _truthy(a) else self.eval(e[3], env)
            return self.eval(e[3], env) if (a is None or a is UNDEF) else a
        if tag == "assign":
            return self.assign(e, env)
        if tag == "assign_pat":
            v = self.eval(e[2], env)
            self.assign_pattern(e[1], v, env)
            return v
        if tag == "unary":
            op = e[1]
            if op == "typeof":
                if e[2][0] == "ident" and env.lookup(e[2][1]) is None:
                    return "undefined"
                return _typeof(self.eval(e[2], env))
            if op == "delete":
                t = e[2]
                if t[0] == "member":
                    obj = self.eval(t[1], env)
                    if isinstance(obj, JSObject) and not isinstance(obj, Host):
                        obj.props.pop(_to_str(self.member_key(t, env)), None)
                return True
            v = self.eval(e[2], env)
            if op == "!":
                return not _truthy(v)
            if op == "-":
                return -_to_num(v)
            if op == "+":
                return _to_num(v)
            if op == "~":
                return float(~_to_int32(v))
            if op == "void":
                return UNDEF
        if tag == "update":
            _, op, prefix, target = e
            old = _to_num(self.eval(target, env))
            new = old + (1.0 if op == "++" else -1.0)
            self.store(target, new, env)
            return new if prefix else old
        if tag == "cond":
            return self.eval(e[2], env) if _truthy(self.eval(e[1], env)) else self.eval(e[3], env)
        if tag == "array":
            out = []
            for it in e[1]:
                if it[0] == "spread":
                    out.extend(self.iterate(self.eval(it[1], env)))
                else:
                    out.append(self.eval(it, env))
            if len(out) > self.lim.array_len:
                raise JSBudget("RangeError", "array too large")
            return JSArray(out)
        if tag == "object":
            obj = JSObject()
            for p in e[1]:
                if p[0] == "spread":
                    src = self.eval(p[1], env)
                    for k in _own_keys(src):
                        obj.props[k] = self.get(src, k)
                elif p[0] == "shorthand_default":
                    raise JSError("SyntaxError", "invalid shorthand property initializer")
                elif p[0] in ("get", "set"):
                    key = p[1]
                    k = _to_str(self.eval(key[1], env)) if isinstance(key, tuple) else key
                    acc = obj.props.get(k)
                    if not isinstance(acc, Accessor):
                        acc = Accessor()
                        obj.props[k] = acc
                    fn = self.make_func(p[2], env)
                    if p[0] == "get":
                        acc.get = fn
                    else:
                        acc.set = fn
                else:
                    key = p[1]
                    k = _to_str(self.eval(key[1], env)) if isinstance(key, tuple) else key
                    v = self.eval(p[2], env)
                    if isinstance(v, JSFunction) and not v.arrow:
                        v.this = obj
                    obj.props[k] = v
            return obj
        if tag == "func":
            return self.make_func(e, env)
        if tag == "class":
            return self.make_class(e, env)
        if tag == "super_call":
            sup = env.lookup("%super")
            if sup is None:
                raise JSError("SyntaxError", "'super' call outside a derived constructor")
            return self.call(sup.vars["%super"], UNDEF, self.eval_args(e[1], env))
        if tag == "super_member":
            this = self.eval(("this",), env)
            return self.super_get(self.member_super_key(e, env), env, this)
        if tag == "new":
            return self.construct(self.eval(e[1], env), self.eval_args(e[2], env))
        if tag == "tpl":
            s = "".join(p if isinstance(p, str) else _to_str(self.eval(p, env)) for p in e[1])
            if len(s) > self.lim.string_len:
                raise JSBudget("RangeError", "string too large")
            return s
        if tag == "seq":
            v = UNDEF
            for x in e[1]:
                v = self.eval(x, env)
            return v
        if tag == "this":
            ev = env.lookup("this")
            if ev is None:
                return UNDEF
            v = ev.vars["this"]
            if v is _TDZ:
                raise _Throw(_error_obj("ReferenceError", "must call super constructor before accessing 'this'"))
            return v
        if tag == "spread":
            raise JSError("SyntaxError", "unexpected spread")
        raise JSError("SyntaxError", f"unsupported expression {tag}")

    def member_super_key(self, node, env):
        k = node[1]
        return _to_str(k[1] if k[0] == "lit" else self.eval(k, env))

    def super_get(self, key: str, env, this):
        h = env.lookup("%home")
        if h is None:
            raise JSError("SyntaxError", "'super' outside a method")
        home = h.vars["%home"]
        if isinstance(home, JSClass):                         # static method: the parent class's statics
            return self.get(home.parent, key) if home.parent is not None else UNDEF
        v = self.proto_get(home.proto, key, this) if home.proto is not None else _MISSING
        if v is _MISSING:
            # a host parent (e.g. THREE.Group): its own methods, not the subclass's overrides
            return this.js_get(self, key) if isinstance(this, Host) else UNDEF
        return v

    def eval_args(self, args, env):
        out = []
        for a in args:
            if a[0] == "spread":
                out.extend(self.iterate(self.eval(a[1], env)))
            else:
                out.append(self.eval(a, env))
        return out

    def store(self, target, value, env):
        if target[0] == "ident":
            env.set(target[1], value)
        elif target[0] == "member":
            self.put(self.eval(target[1], env), self.member_key(target, env), value)
        else:
            raise JSError("SyntaxError", "invalid assignment target")

    def assign(self, e, env):
        _, op, target, rhs = e
        if op == "=":
            v = self.eval(rhs, env)
            if isinstance(v, JSFunction) and v.name is None and target[0] == "ident":
                v.name = target[1]
            self.store(target, v, env)
            return v
        if target[0] == "member":
            obj = self.eval(target[1], env)
            key = self.member_key(target, env)
            cur = self.get(obj, key)
        else:
            obj = key = None
            cur = env.get(target[1])
        if op in ("&&=", "||=", "??="):
            keep = {"&&=": not _truthy(cur), "||=": _truthy(cur), "??=": not (cur is None or cur is UNDEF)}[op]
            if keep:
                return cur
            v = self.eval(rhs, env)
        else:
            v = self.binop(op[:-1], cur, self.eval(rhs, env))
        if target[0] == "member":
            self.put(obj, key, v)
        else:
            env.set(target[1], v)
        return v

    def binop(self, op, a, b):
        if op == "+":
            if isinstance(a, str) or isinstance(b, str) or _is_objlike(a) or _is_objlike(b):
                s = _to_str(a) + _to_str(b)
                if len(s) > self.lim.string_len:
                    raise JSBudget("RangeError", "string too large")
                return s
            return _to_num(a) + _to_num(b)
        if op == "-":
            return _to_num(a) - _to_num(b)
        if op == "*":
            return _to_num(a) * _to_num(b)
        if op == "/":
            x, y = _to_num(a), _to_num(b)
            if y == 0:
                if x == 0 or x != x:
                    return math.nan
                return math.copysign(math.inf, x) * math.copysign(1.0, y)
            return x / y
        if op == "%":
            x, y = _to_num(a), _to_num(b)
            if y == 0 or x != x or y != y or x in (math.inf, -math.inf):
                return math.nan
            return math.fmod(x, y)
        if op == "**":
            x, y = _to_num(a), _to_num(b)
            try:
                r = x ** y
                return r if isinstance(r, float) else math.nan
            except (OverflowError, ZeroDivisionError):
                return math.inf
        if op in ("===", "!=="):
            r = _strict_eq(a, b)
            return r if op == "===" else not r
        if op in ("==", "!="):
            r = _loose_eq(a, b)
            return r if op == "==" else not r
        if op in ("<", ">", "<=", ">="):
            if isinstance(a, str) and isinstance(b, str):
                x, y = a, b
            else:
                x, y = _to_num(a), _to_num(b)
                if x != x or y != y:
                    return False
            return {"<": x < y, ">": x > y, "<=": x <= y, ">=": x >= y}[op]
        if op == "&":
            return float(_to_int32(a) & _to_int32(b))
        if op == "|":
            return float(_to_int32(a) | _to_int32(b))
        if op == "^":
            return float(_to_int32(a) ^ _to_int32(b))
        if op == "<<":
            return float(_to_int32(_to_int32(a) << (_to_int32(b) & 31)))
        if op == ">>":
            return float(_to_int32(a) >> (_to_int32(b) & 31))
        if op == ">>>":
            return float((_to_int32(a) & 0xFFFFFFFF) >> (_to_int32(b) & 31))
        if op == "instanceof":
            if isinstance(b, (JSClass, JSFunction)):
                target = b.proto if isinstance(b, JSClass) else self.fn_prototype(b)
                p = a.proto if isinstance(a, JSObject) else None
                depth = 0
                while p is not None and depth < 64:
                    if p is target:
                        return True
                    p, depth = p.proto, depth + 1
                return False
            if isinstance(b, Native) and isinstance(a, Host):
                return a.is_instance(b.name)
            if isinstance(b, Native) and b.name in TYPED_BYTES:
                return isinstance(a, TypedArray) and a.kind == b.name
            if isinstance(b, Native) and b.name == "Array":
                return isinstance(a, JSArray) and not isinstance(a, TypedArray)
            if isinstance(b, Native) and b.name == "Object":
                return isinstance(a, (JSObject, JSArray, Host))
            return False
        if op == "in":
            k = _to_str(a)
            if isinstance(b, JSArray):
                i = _index(a)
                return i is not None and i < len(b.items)
            if isinstance(b, Host):
                return b.js_get(self, k) is not UNDEF
            if isinstance(b, JSObject):
                return k in b.props
            raise _Throw(_error_obj("TypeError", "cannot use 'in' on a primitive"))
        raise JSError("SyntaxError", f"unsupported operator {op}")


def _is_index_key(k: str) -> bool:
    return k.isdigit() and (k == "0" or k[0] != "0") and int(k) < 4294967295


def _is_objlike(v):
    return isinstance(v, (JSObject, JSArray)) and not isinstance(v, Host) or isinstance(v, JSArray)


def _pattern_names(p) -> List[str]:
    tag = p[0]
    if tag == "id":
        return [p[1]]
    out = []
    if tag == "objpat":
        for _, t, _ in p[1]:
            out += _pattern_names(t)
        if p[2] is not None:
            out.append(p[2])
    elif tag == "arrpat":
        for t, _ in p[1]:
            if t is not None:
                out += _pattern_names(t)
        if p[2] is not None:
            out += _pattern_names(p[2])
    return out


def _own_keys(v) -> List[str]:
    if isinstance(v, JSArray):
        return [str(i) for i in range(len(v.items))]
    if isinstance(v, Host):
        return v.own_keys()
    if isinstance(v, JSObject):
        keys = list(v.props.keys())
        idx = [k for k in keys if _is_index_key(k)]
        if not idx:
            return keys
        # integer-like keys first, ascending, then the others in insertion order
        return sorted(idx, key=int) + [k for k in keys if not _is_index_key(k)]
    if isinstance(v, str):
        return [str(i) for i in range(len(v))]
    return []


# -------------------------------------------------------------------------------------------- builtin library


def _nat(name, fn):
    return Native(name, fn=fn)


def _arg(args, i, default=UNDEF):
    return args[i] if i < len(args) else default


def _num_arg(args, i, default=0.0):
    v = _arg(args, i)
    return default if v is UNDEF else _to_num(v)


def _flat(items, depth: float) -> list:
    out = []
    for v in items:
        if isinstance(v, JSArray) and depth >= 1:
            out.extend(_flat(v.items, depth - 1))
        else:
            out.append(v)
    return out


def _array_method(it: Interp, arr: JSArray, name: str):
    a = arr.items
    if name == "length":
        return float(len(a))

    def cb(f, *xs):
        return it.call(f, UNDEF, list(xs))

    m: Dict[str, Callable] = {
        "push": lambda i, t, x: (a.extend(x), _check_len(it, a), float(len(a)))[-1],
        "pop": lambda i, t, x: a.pop() if a else UNDEF,
        "shift": lambda i, t, x: a.pop(0) if a else UNDEF,
        "unshift": lambda i, t, x: (a.__setitem__(slice(0, 0), x), float(len(a)))[-1],
        "map": lambda i, t, x: JSArray([cb(x[0], v, float(k), arr) for k, v in enumerate(list(a))]),
        "forEach": lambda i, t, x: ([cb(x[0], v, float(k), arr) for k, v in enumerate(list(a))], UNDEF)[-1],
        "filter": lambda i, t, x: JSArray([v for k, v in enumerate(list(a)) if _truthy(cb(x[0], v, float(k), arr))]),
        "some": lambda i, t, x: any(_truthy(cb(x[0], v, float(k), arr)) for k, v in enumerate(list(a))),
        "every": lambda i, t, x: all(_truthy(cb(x[0], v, float(k), arr)) for k, v in enumerate(list(a))),
        "find": lambda i, t, x: next((v for k, v in enumerate(list(a)) if _truthy(cb(x[0], v, float(k), arr))), UNDEF),
        "findIndex": lambda i, t, x: float(next((k for k, v in enumerate(list(a)) if _truthy(cb(x[0], v, float(k), arr))), -1)),
        "indexOf": lambda i, t, x: float(next((k for k, v in enumerate(a) if _strict_eq(v, _arg(x, 0))), -1)),
        "includes": lambda i, t, x: any(_strict_eq(v, _arg(x, 0)) or (_num_nan(v) and _num_nan(_arg(x, 0))) for v in a),
        "join": lambda i, t, x: (_to_str(x[0]) if x and x[0] is not UNDEF else ",").join(
            "" if v is None or v is UNDEF else _to_str(v) for v in a),
        "slice": lambda i, t, x: JSArray(a[_slice_idx(x, 0, len(a), 0):_slice_idx(x, 1, len(a), len(a))]),
        "concat": lambda i, t, x: JSArray(a + [w for y in x for w in (y.items if isinstance(y, JSArray) else [y])]),
        "reverse": lambda i, t, x: (a.reverse(), arr)[-1],
        "fill": lambda i, t, x: (_fill(a, x), arr)[-1],
        "reduce": lambda i, t, x: _reduce(it, arr, x),
        "sort": lambda i, t, x: (_sort(it, a, x), arr)[-1],
        "splice": lambda i, t, x: _splice(a, x),
        "flat": lambda i, t, x: JSArray(_flat(list(a), _num_arg(x, 0, 1.0))),
        "flatMap": lambda i, t, x: JSArray([w for k, v in enumerate(list(a))
                                            for r in [cb(x[0], v, float(k), arr)]
                                            for w in (r.items if isinstance(r, JSArray) else [r])]),
        "keys": lambda i, t, x: JSArray([float(k) for k in range(len(a))]),
        "values": lambda i, t, x: JSArray(list(a)),
        "entries": lambda i, t, x: JSArray([JSArray([float(k), v]) for k, v in enumerate(a)]),
        "at": lambda i, t, x: (a[int(_num_arg(x, 0))] if -len(a) <= int(_num_arg(x, 0)) < len(a) else UNDEF),
        "toString": lambda i, t, x: _to_str(arr),
    }
    f = m.get(name)
    return _nat(name, f) if f is not None else UNDEF


def _num_nan(v):
    return isinstance(v, float) and v != v


def _check_len(it, a):
    if len(a) > it.lim.array_len:
        raise JSBudget("RangeError", "array too large")


def _slice_idx(x, i, n, default):
    v = _arg(x, i)
    if v is UNDEF:
        return default
    k = int(_to_num(v)) if _to_num(v) == _to_num(v) else 0
    return max(0, n + k) if k < 0 else min(k, n)


def _fill(a, x):
    n = len(a)
    lo, hi = _slice_idx(x, 1, n, 0), _slice_idx(x, 2, n, n)
    for k in range(lo, hi):
        a[k] = _arg(x, 0)


def _reduce(it, arr, x):
    a = list(arr.items)
    k = 0
    if len(x) > 1:
        acc = x[1]
    else:
        if not a:
            raise _Throw(_error_obj("TypeError", "reduce of empty array with no initial value"))
        acc, k = a[0], 1
    for j in range(k, len(a)):
        acc = it.call(x[0], UNDEF, [acc, a[j], float(j), arr])
    return acc


def _sort(it, a, x):
    import functools
    f = _arg(x, 0)
    if f is UNDEF:
        a.sort(key=_to_str)
    else:
        a.sort(key=functools.cmp_to_key(lambda p, q: (lambda r: -1 if r < 0 else (1 if r > 0 else 0))(
            _to_num(it.call(f, UNDEF, [p, q])))))


def _splice(a, x):
    n = len(a)
    start = _slice_idx(x, 0, n, 0)
    cnt = n - start if len(x) < 2 else max(0, min(int(_to_num(x[1])), n - start))
    removed = a[start:start + cnt]
    a[start:start + cnt] = x[2:]
    return JSArray(removed)


def _string_method(it, s: str, name: str):
    if name == "length":
        return float(len(s))
    m = {
        "toUpperCase": lambda i, t, x: s.upper(),
        "toLowerCase": lambda i, t, x: s.lower(),
        "trim": lambda i, t, x: s.strip(),
        "slice": lambda i, t, x: s[_slice_idx(x, 0, len(s), 0):_slice_idx(x, 1, len(s), len(s))],
        "substring": lambda i, t, x: _substring(s, x),
        "substr": lambda i, t, x: _substr(s, x),
        "at": lambda i, t, x: (lambda k: s[k] if 0 <= k < len(s) else UNDEF)(
            int(_num_arg(x, 0)) + (len(s) if _num_arg(x, 0) < 0 else 0)),
        "lastIndexOf": lambda i, t, x: float(s.rfind(_to_str(_arg(x, 0)))),
        "trimStart": lambda i, t, x: s.lstrip(),
        "trimEnd": lambda i, t, x: s.rstrip(),
        "concat": lambda i, t, x: s + "".join(_to_str(v) for v in x),
        "localeCompare": lambda i, t, x: float((s > _to_str(_arg(x, 0))) - (s < _to_str(_arg(x, 0)))),
        "charAt": lambda i, t, x: s[int(_num_arg(x, 0))] if 0 <= int(_num_arg(x, 0)) < len(s) else "",
        "charCodeAt": lambda i, t, x: float(ord(s[int(_num_arg(x, 0))])) if 0 <= int(_num_arg(x, 0)) < len(s) else math.nan,
        "indexOf": lambda i, t, x: float(s.find(_to_str(_arg(x, 0)), max(0, int(_num_arg(x, 1))))),
        "includes": lambda i, t, x: _to_str(_arg(x, 0)) in s,
        "startsWith": lambda i, t, x: s.startswith(_to_str(_arg(x, 0))),
        "endsWith": lambda i, t, x: s.endswith(_to_str(_arg(x, 0))),
        "split": lambda i, t, x: _split(s, x),
        "repeat": lambda i, t, x: _repeat(it, s, int(_num_arg(x, 0))),
        "padStart": lambda i, t, x: _pad(it, s, x, True),
        "padEnd": lambda i, t, x: _pad(it, s, x, False),
        "replace": lambda i, t, x: s.replace(_to_str(_arg(x, 0)), _to_str(_arg(x, 1)), 1),
        "replaceAll": lambda i, t, x: s.replace(_to_str(_arg(x, 0)), _to_str(_arg(x, 1))),
        "toString": lambda i, t, x: s,
    }
    f = m.get(name)
    return _nat(name, f) if f is not None else UNDEF


def _substring(s, x):
    n = len(s)

    def clamp(v):
        v = _to_num(v)
        return 0 if v != v else int(max(0, min(n, v)))
    a = clamp(_arg(x, 0, 0.0))
    b = n if len(x) < 2 or x[1] is UNDEF else clamp(x[1])
    return s[min(a, b):max(a, b)]


def _substr(s, x):
    n = len(s)
    a = int(_num_arg(x, 0))
    a = max(0, n + a) if a < 0 else min(a, n)
    ln = n - a if len(x) < 2 or x[1] is UNDEF else max(0, int(_num_arg(x, 1)))
    return s[a:a + ln]


def _split(s, x):
    sep = _arg(x, 0)
    lim = _arg(x, 1)
    if sep is UNDEF:
        parts = [s]
    elif _to_str(sep) == "":
        parts = list(s)
    else:
        parts = s.split(_to_str(sep))
    if lim is not UNDEF:
        parts = parts[:max(0, int(_to_num(lim)))]
    return JSArray(parts)


def _pad(it, s, x, start):
    n = int(_num_arg(x, 0))
    fill = _to_str(_arg(x, 1, " "))
    if n <= len(s) or fill == "":
        return s
    if n > it.lim.string_len:
        raise JSBudget("RangeError", "string too large")
    k = n - len(s)
    pad = (fill * (k // len(fill) + 1))[:k]
    return pad + s if start else s + pad


def _to_fixed(v: float, digits: int) -> str:
    """Number.prototype.toFixed: the exact binary value rounded half away from zero (JS picks the larger n on a
    tie, applied to the magnitude)."""
    from decimal import ROUND_HALF_UP, Decimal
    if v != v:
        return "NaN"
    if abs(v) >= 1e21 or math.isinf(v):
        return _num_to_str(v)
    d = max(0, min(100, digits))
    q = Decimal(v if v != 0 else 0.0).quantize(Decimal(1).scaleb(-d), rounding=ROUND_HALF_UP)
    return f"{q:f}"             # a negative value that rounds to zero keeps its sign, as in JS ("-0.00")


def _radix_str(v: float, radix: int) -> str:
    if radix == 10 or v != v or math.isinf(v):
        return _num_to_str(v)
    digits = "0123456789abcdefghijklmnopqrstuvwxyz"
    neg, v = v < 0, abs(v)
    ip, fp = int(v), v - int(v)
    out = ""
    while True:
        out = digits[ip % radix] + out
        ip //= radix
        if ip == 0:
            break
    if fp:
        out += "."
        for _ in range(52):
            fp *= radix
            dgt = int(fp)
            out += digits[dgt]
            fp -= dgt
            if not fp:
                break
    return ("-" if neg else "") + out


def _repeat(it, s, n):
    if n < 0 or len(s) * n > it.lim.string_len:
        raise JSBudget("RangeError", "invalid repeat count")
    return s * n


def _number_method(it, v: float, name: str):
    if name == "toFixed":
        return _nat(name, lambda i, t, x: _to_fixed(v, int(_num_arg(x, 0))))
    if name == "toString":
        return _nat(name, lambda i, t, x: _radix_str(v, max(2, min(36, int(_num_arg(x, 0, 10.0))))))
    if name == "toPrecision":
        return _nat(name, lambda i, t, x: f"{v:.{int(_num_arg(x, 0))}g}")
    return UNDEF


def _function_method(it, f, name):
    if name == "call":
        return _nat(name, lambda i, t, x: it.call(f, _arg(x, 0), x[1:]))
    if name == "apply":
        return _nat(name, lambda i, t, x: it.call(f, _arg(x, 0), it.iterate(_arg(x, 1)) if len(x) > 1 and x[1] is not UNDEF else []))
    return _nat(name, lambda i, t, x: _nat("bound", lambda i2, t2, y: it.call(f, _arg(x, 0), x[1:] + y)))


_OBJECT_PROTO = {
    "hasOwnProperty": lambda it, o: _nat("hasOwnProperty", lambda i, t, x: _to_str(_arg(x, 0)) in o.props),
    "toString": lambda it, o: _nat("toString", lambda i, t, x: "[object Object]"),
}


def _install_globals(it: Interp):
    g = it.globals
    rnd = it.random

    def mfn(f):
        return lambda i, t, x: f(*[_to_num(v) for v in x])

    def safe(f):
        def w(*a):
            try:
                return float(f(*a))
            except (ValueError, OverflowError, ZeroDivisionError):
                return math.nan
        return w

    math_props = {
        "PI": math.pi, "E": math.e, "SQRT2": math.sqrt(2), "LN2": math.log(2), "LN10": math.log(10),
        "SQRT1_2": math.sqrt(0.5), "LOG2E": 1 / math.log(2), "LOG10E": 1 / math.log(10),
    }
    for nm, f in {"sin": math.sin, "cos": math.cos, "tan": math.tan, "asin": math.asin, "acos": math.acos,
                  "atan": math.atan, "sqrt": math.sqrt, "exp": math.exp, "log": math.log, "log2": math.log2,
                  "log10": math.log10, "cbrt": lambda v: math.copysign(abs(v) ** (1 / 3), v), "sinh": math.sinh,
                  "cosh": math.cosh, "tanh": math.tanh, "abs": abs, "atan2": math.atan2,
                  "floor": lambda v: float(math.floor(v)) if math.isfinite(v) else v,
                  "ceil": lambda v: float(math.ceil(v)) if math.isfinite(v) else v,
                  "round": lambda v: float(math.floor(v + 0.5)) if math.isfinite(v) else v,
                  "trunc": lambda v: float(math.trunc(v)) if math.isfinite(v) else v,
                  "sign": lambda v: v if v != v else float((v > 0) - (v < 0)),
                  "pow": lambda a, b: a ** b, "hypot": lambda *v: math.hypot(*v),
                  "fround": _fround}.items():
        math_props[nm] = _nat(nm, mfn(safe(f)))
    math_props["min"] = _nat("min", lambda i, t, x: min([_to_num(v) for v in x], default=math.inf))
    math_props["max"] = _nat("max", lambda i, t, x: max([_to_num(v) for v in x], default=-math.inf))
    math_props["random"] = _nat("random", lambda i, t, x: rnd())
    g.declare("Math", JSObject(math_props))
    g.declare("NaN", math.nan)
    g.declare("Infinity", math.inf)
    g.declare("undefined", UNDEF)
    g.declare("parseFloat", _nat("parseFloat", lambda i, t, x: _parse_float(_to_str(_arg(x, 0)))))
    g.declare("parseInt", _nat("parseInt", lambda i, t, x: _parse_int(_to_str(_arg(x, 0)), _arg(x, 1))))
    g.declare("isNaN", _nat("isNaN", lambda i, t, x: _to_num(_arg(x, 0)) != _to_num(_arg(x, 0))))
    g.declare("isFinite", _nat("isFinite", lambda i, t, x: math.isfinite(_to_num(_arg(x, 0)))))
    g.declare("Number", Native("Number", fn=lambda i, t, x: _to_num(_arg(x, 0, 0.0)), props={
        "isFinite": _nat("isFinite", lambda i, t, x: isinstance(_arg(x, 0), float) and math.isfinite(x[0])),
        "isInteger": _nat("isInteger", lambda i, t, x: isinstance(_arg(x, 0), float) and math.isfinite(x[0]) and x[0] == int(x[0])),
        "EPSILON": 2.0 ** -52, "MAX_SAFE_INTEGER": 2.0 ** 53 - 1, "MAX_VALUE": 1.7976931348623157e308,
        "POSITIVE_INFINITY": math.inf, "NEGATIVE_INFINITY": -math.inf, "NaN": math.nan,
        "parseFloat": _nat("parseFloat", lambda i, t, x: _parse_float(_to_str(_arg(x, 0))))}))
    g.declare("String", Native("String", fn=lambda i, t, x: _to_str(_arg(x, 0, "")), props={
        "fromCharCode": _nat("fromCharCode", lambda i, t, x: "".join(chr(int(_to_num(c)) & 0xFFFF) for c in x)),
        "fromCodePoint": _nat("fromCodePoint", lambda i, t, x: "".join(chr(int(_to_num(c))) for c in x))}))
    g.declare("Boolean", Native("Boolean", fn=lambda i, t, x: _truthy(_arg(x, 0, False))))

    def array_ctor(i, x):
        if len(x) == 1 and isinstance(x[0], float):
            n = int(x[0])
            if n > it.lim.array_len or n < 0:
                raise JSBudget("RangeError", "invalid array length")
            return JSArray([UNDEF] * n)
        return JSArray(list(x))

    def array_from(i, t, x):
        src = _arg(x, 0)
        f = _arg(x, 1)
        if isinstance(src, (JSArray, str)) or isinstance(src, Host):
            items = it.iterate(src)
        else:
            n = int(_to_num(it.get(src, "length"))) if isinstance(src, JSObject) else 0
            if n > it.lim.array_len or n < 0:
                raise JSBudget("RangeError", "invalid array length")
            items = [it.get(src, float(k)) for k in range(n)]
        if f is not UNDEF:
            items = [it.call(f, UNDEF, [v, float(k)]) for k, v in enumerate(items)]
        return JSArray(items)

    g.declare("Array", Native("Array", fn=lambda i, t, x: array_ctor(i, x), ctor=array_ctor, props={
        "isArray": _nat("isArray", lambda i, t, x: isinstance(_arg(x, 0), JSArray) and
                        not isinstance(_arg(x, 0), TypedArray)),
        "from": _nat("from", array_from),
        "of": _nat("of", lambda i, t, x: JSArray(list(x)))}))
    g.declare("Object", Native("Object", fn=lambda i, t, x: JSObject(), ctor=lambda i, x: JSObject(), props={
        "keys": _nat("keys", lambda i, t, x: JSArray(_own_keys(_arg(x, 0)))),
        "values": _nat("values", lambda i, t, x: JSArray([it.get(x[0], k) for k in _own_keys(x[0])])),
        "entries": _nat("entries", lambda i, t, x: JSArray([JSArray([k, it.get(x[0], k)]) for k in _own_keys(x[0])])),
        "assign": _nat("assign", lambda i, t, x: _assign(it, x)),
        "freeze": _nat("freeze", lambda i, t, x: _arg(x, 0)),
        "fromEntries": _nat("fromEntries", lambda i, t, x: JSObject({_to_str(it.get(p, 0.0)): it.get(p, 1.0)
                                                                       for p in it.iterate(_arg(x, 0))}))}))
    g.declare("console", JSObject({k: _nat(k, lambda i, t, x: UNDEF) for k in ("log", "warn", "error", "info", "debug")}))
    g.declare("Error", Native("Error", fn=lambda i, t, x: _error_obj("Error", _to_str(_arg(x, 0, ""))),
                              ctor=lambda i, x: _error_obj("Error", _to_str(_arg(x, 0, "")))))
    for cls in ("Float32Array", "Uint16Array", "Uint32Array", "Int32Array", "Uint8Array", "Float64Array", "Int16Array",
                "Uint8ClampedArray", "Int8Array"):
        g.declare(cls, _typed_array_ctor(it, cls))
    for kind in ("TypeError", "RangeError"):
        g.declare(kind, Native(kind, fn=lambda i, t, x, _k=kind: _error_obj(_k, _to_str(_arg(x, 0, ""))),
                               ctor=lambda i, x, _k=kind: _error_obj(_k, _to_str(_arg(x, 0, "")))))
    for nm in ("BigInt", "ArrayBuffer", "DataView", "BigInt64Array", "BigUint64Array"):
        def unsupported(i, *a, _n=nm):
            raise _Throw(_error_obj("TypeError", f"{_n} is not supported by the module checker"))
        g.declare(nm, Native(nm, fn=lambda i, t, x, _u=unsupported: _u(i), ctor=lambda i, x, _u=unsupported: _u(i)))
    num = g.vars["Number"].props
    num.update({
        "parseInt": _nat("parseInt", lambda i, t, x: _parse_int(_to_str(_arg(x, 0)), _arg(x, 1))),
        "isNaN": _nat("isNaN", lambda i, t, x: isinstance(_arg(x, 0), float) and x[0] != x[0]),
        "isSafeInteger": _nat("isSafeInteger", lambda i, t, x: isinstance(_arg(x, 0), float) and math.isfinite(x[0])
                              and x[0] == int(x[0]) and abs(x[0]) <= 2.0 ** 53 - 1),
        "MIN_VALUE": 5e-324, "MIN_SAFE_INTEGER": -(2.0 ** 53 - 1)})
    g.declare("JSON", JSObject({
        "parse": _nat("parse", lambda i, t, x: _json_parse(_to_str(_arg(x, 0)))),
        "stringify": _nat("stringify", lambda i, t, x: _json_stringify(it, _arg(x, 0), _arg(x, 2)))}))
    g.declare("Map", Native("Map", ctor=lambda i, x: JSMap(it, _arg(x, 0))))
    g.declare("Set", Native("Set", ctor=lambda i, x: JSSet(it, _arg(x, 0))))
    counter = [0]

    def symbol(i, t, x):
        counter[0] += 1
        return f"@@symbol({_to_str(_arg(x, 0, ''))})#{counter[0]}"
    g.declare("Symbol", Native("Symbol", fn=symbol, props={"iterator": "@@iterator"}))


def _json_parse(text: str):
    try:
        v = json.loads(text)
    except (ValueError, RecursionError) as e:
        raise _Throw(_error_obj("SyntaxError", f"JSON.parse: {str(e)[:80]}"))

    def conv(o):
        if isinstance(o, dict):
            return JSObject({str(k): conv(w) for k, w in o.items()})
        if isinstance(o, list):
            return JSArray([conv(w) for w in o])
        if isinstance(o, bool) or o is None or isinstance(o, str):
            return o
        return float(o)
    return conv(v)


def _json_stringify(it, v, indent):
    seen = set()

    def conv(o):
        if o is None or isinstance(o, (bool, str)):
            return o
        if isinstance(o, (int, float)):
            f = float(o)
            return None if not math.isfinite(f) else (int(f) if f == int(f) and abs(f) < 2 ** 53 else f)
        if isinstance(o, (JSFunction, Native, JSClass)) or o is UNDEF:
            return _SKIP
        if id(o) in seen:
            raise _Throw(_error_obj("TypeError", "converting circular structure to JSON"))
        seen.add(id(o))
        try:
            if isinstance(o, JSArray):
                return [None if (c := conv(w)) is _SKIP else c for w in o.items]
            if isinstance(o, Vec):
                return {c: conv(w) for c, w in zip(o.comps, o.v())}
            out = {}
            for k in _own_keys(o):
                c = conv(it.get(o, k))
                if c is not _SKIP:
                    out[k] = c
            return out
        finally:
            seen.discard(id(o))
    r = conv(v)
    if r is _SKIP:
        return UNDEF
    ind = None
    if isinstance(indent, float) and indent > 0:
        ind = min(10, int(indent))
    elif isinstance(indent, str) and indent:
        ind = indent[:10]
    return json.dumps(r, indent=ind, separators=None if ind else (",", ":"), ensure_ascii=False)


_SKIP = object()


def _mkey(v):
    """SameValueZero key of a Map / Set entry."""
    if isinstance(v, bool):
        return ("b", v)
    if isinstance(v, (int, float)):
        f = float(v)
        return ("nan",) if f != f else ("n", f + 0.0)
    if isinstance(v, str):
        return ("s", v)
    if v is None:
        return ("null",)
    if v is UNDEF:
        return ("undef",)
    return ("o", id(v))


TYPED_BYTES = {"Float32Array": 4, "Float64Array": 8, "Int8Array": 1, "Uint8Array": 1, "Uint8ClampedArray": 1,
               "Int16Array": 2, "Uint16Array": 2, "Int32Array": 4, "Uint32Array": 4}
_TYPED_INT = {"Int8Array": (8, True), "Uint8Array": (8, False), "Int16Array": (16, True), "Uint16Array": (16, False),
              "Int32Array": (32, True), "Uint32Array": (32, False)}


def _fround(v: float) -> float:
    try:
        return struct.unpack("f", struct.pack("f", v))[0]
    except OverflowError:
        return math.copysign(math.inf, v)


def _typed_value(kind: str, v) -> float:
    """One element stored into a typed array of `kind` (ECMAScript's ToInt8 ... ToUint32, ToUint8Clamp, and float32
    rounding)."""
    x = _to_num(v)
    if kind == "Float64Array":
        return x
    if kind == "Float32Array":
        return _fround(x)
    if kind == "Uint8ClampedArray":
        return 0.0 if x != x else float(round(min(255.0, max(0.0, x))))      # ties to even
    if not math.isfinite(x):
        return 0.0
    bits, signed = _TYPED_INT[kind]
    n = int(x) % (1 << bits)
    return float(n - (1 << bits) if signed and n >= 1 << (bits - 1) else n)


def _typed_values(kind: str, vals) -> list:
    """_typed_value over a sequence, vectorised for the large buffers geometry code builds."""
    import numpy as np
    a = np.asarray([_to_num(v) if not isinstance(v, float) else v for v in vals], dtype=np.float64)
    if kind == "Float64Array":
        return a.tolist()
    if kind == "Float32Array":
        with np.errstate(over="ignore"):
            return a.astype(np.float32).astype(np.float64).tolist()
    if kind == "Uint8ClampedArray":
        return np.round(np.clip(np.nan_to_num(a, nan=0.0), 0.0, 255.0)).tolist()
    bits, signed = _TYPED_INT[kind]
    a = np.trunc(np.where(np.isfinite(a), a, 0.0))
    m = float(1 << bits)
    a = np.mod(a, m)
    if signed:
        a = np.where(a >= m / 2, a - m, a)
    return (a + 0.0).tolist()


def _typed_from(it, kind: str, src, fn=UNDEF) -> TypedArray:
    if isinstance(src, (int, float)) and not isinstance(src, bool):
        n = int(src) if src == src else 0
        if n < 0 or n > it.lim.array_len:
            raise JSBudget("RangeError", "invalid typed array length")
        return TypedArray(kind, [0.0] * n, coerced=True)
    if src is UNDEF or src is None:
        return TypedArray(kind, [], coerced=True)
    if isinstance(src, (JSArray, JSMap, JSSet, str)):
        vals = list(it.iterate(src))
    else:                                               # an array-like object: {length: n, 0: ..., 1: ...}
        n = _to_num(it.get(src, "length"))
        n = int(n) if n == n and n > 0 else 0
        if n > it.lim.array_len:
            raise JSBudget("RangeError", "invalid typed array length")
        vals = [it.get(src, float(k)) for k in range(n)]
    if fn is not UNDEF:
        vals = [it.call(fn, UNDEF, [v, float(k)]) for k, v in enumerate(vals)]
    return TypedArray(kind, vals)


def _typed_array_ctor(it, cls):
    return Native(cls, ctor=lambda i, x: _typed_from(it, cls, _arg(x, 0, 0.0)),
                  props={"from": _nat("from", lambda i, t, x: _typed_from(it, cls, _arg(x, 0), _arg(x, 1))),
                         "of": _nat("of", lambda i, t, x: TypedArray(cls, list(x))),
                         "BYTES_PER_ELEMENT": float(TYPED_BYTES[cls])})


_TYPED_SAME_KIND = ("map", "filter", "slice")
_TYPED_ABSENT = ("push", "pop", "shift", "unshift", "splice", "concat", "flat", "flatMap")


def _typed_method(it, arr: TypedArray, name: str):
    """Typed-array members: set / subarray / BYTES_PER_ELEMENT / byteLength, map / filter / slice returning the
    same kind, fill converting its value, sort numeric by default; no push / pop / splice / concat (fixed length).
    subarray returns a copy of the range (three.js modules read it; a write through it does not reach the
    parent array)."""
    a = arr.items
    if name == "BYTES_PER_ELEMENT":
        return float(TYPED_BYTES[arr.kind])
    if name == "byteLength":
        return float(len(a) * TYPED_BYTES[arr.kind])
    if name in _TYPED_ABSENT:
        return UNDEF
    if name == "set":
        def set_(i, t, x):
            src, off = _arg(x, 0), int(_num_arg(x, 1, 0.0))
            vals = list(it.iterate(src)) if isinstance(src, JSArray) else []
            if off < 0 or off + len(vals) > len(a):
                raise _Throw(_error_obj("RangeError", "offset is out of bounds"))
            a[off:off + len(vals)] = [_typed_value(arr.kind, v) for v in vals]
            return UNDEF
        return _nat("set", set_)
    if name == "subarray":
        return _nat("subarray", lambda i, t, x: TypedArray(
            arr.kind, a[_slice_idx(x, 0, len(a), 0):_slice_idx(x, 1, len(a), len(a))], coerced=True))
    if name == "fill":
        def fill(i, t, x):
            _fill(a, [_typed_value(arr.kind, _arg(x, 0))] + list(x[1:]))
            return arr
        return _nat("fill", fill)
    if name == "sort":
        def sort(i, t, x):
            if _arg(x, 0) is UNDEF:
                a.sort(key=lambda v: (v != v, v))       # numeric, NaN last
            else:
                _sort(it, a, x)
            return arr
        return _nat("sort", sort)
    m = _array_method(it, arr, name)
    if name in _TYPED_SAME_KIND and isinstance(m, Native):
        inner = m.fn
        return _nat(name, lambda i, t, x: (lambda r: TypedArray(arr.kind, r.items) if isinstance(r, JSArray) else r)(
            inner(i, t, x)))
    return m


def _assign(it, x):
    tgt = _arg(x, 0)
    for src in x[1:]:
        if src is None or src is UNDEF:
            continue
        for k in _own_keys(src):
            it.put(tgt, k, it.get(src, k))
    return tgt


def _parse_float(s: str) -> float:
    m = re.match(r"\s*[+-]?(\d+\.?\d*(e[+-]?\d+)?|\.\d+(e[+-]?\d+)?|Infinity)", s, re.I)
    if not m:
        return math.nan
    return float(m.group(0))


def _parse_int(s: str, radix) -> float:
    s = s.strip()
    r = 10 if radix is UNDEF else int(_to_num(radix))
    sign = -1 if s.startswith("-") else 1
    s = s.lstrip("+-")
    if (r in (0, 16) or radix is UNDEF) and s[:2].lower() == "0x":
        s, r = s[2:], 16
    r = r or 10
    digits = "0123456789abcdefghijklmnopqrstuvwxyz"[:r]
    out = ""
    for ch in s.lower():
        if ch not in digits:
            break
        out += ch
    return float(sign * int(out, r)) if out else math.nan


# --------------------------------------------------------------------------------------------- three.js model


class Host(JSObject):
    """A native object. Subclasses list readable/writable properties; everything else is an expando dict."""
    __slots__ = ()
    cls_name = "Host"
    bases: Tuple[str, ...] = ()

    def js_get(self, it, key):
        v = self.props.get(key, UNDEF)
        if v is not UNDEF:
            return v
        m = getattr(type(self), "js_methods", {}).get(key)
        if m is not None:
            return _nat(key, lambda i, t, x, _m=m, _s=self: _m(_s, i, x))
        return self.get_special(it, key)

    def get_special(self, it, key):
        if key == "type":
            return self.cls_name
        if key == "isObject3D":
            return isinstance(self, Object3D) or UNDEF
        return UNDEF

    def js_set(self, it, key, value):
        if self.set_special(it, key, value):
            return
        self.props[key] = value

    def set_special(self, it, key, value) -> bool:
        return False

    def own_keys(self):
        return list(self.props.keys())

    def iterable(self):
        return None

    def is_instance(self, name):
        return name == self.cls_name or name in self.bases

    def to_string(self):
        return f"[object {self.cls_name}]"


class Vec(Host):
    """Vector2 / Vector3 / Euler: numeric components held in props."""
    __slots__ = ("comps", "kind")

    def __init__(self, comps=("x", "y", "z"), vals=None, cls_name="Vector3"):
        super().__init__({c: float(v) for c, v in zip(comps, vals or [0.0] * len(comps))})
        self.comps = comps
        self.kind = cls_name
        self.props["is" + cls_name] = True
        if cls_name == "Euler":
            self.props["order"] = "XYZ"

    @property
    def cls_name(self):
        return self.kind

    def is_instance(self, name):
        return name == self.kind

    def v(self):
        return [_to_num(self.props[c]) for c in self.comps]

    def setv(self, vals):
        for c, x in zip(self.comps, vals):
            self.props[c] = float(x)
        return self

    def set_special(self, it, key, value):
        if key in self.comps:
            self.props[key] = _to_num(value)
            return True
        return False


def _vec_methods():
    def new_like(s, vals):
        n = Vec(s.comps, vals, s.kind)
        if s.kind == "Euler":
            n.props["order"] = _order(s)
        return n

    def copy_from(s, x):
        s.setv(other(x, s))
        if s.kind == "Euler" and isinstance(_arg(x, 0), Vec) and _arg(x, 0).kind == "Euler":
            s.props["order"] = _order(_arg(x, 0))
        return s

    def set_all(s, x):
        s.setv([_num_arg(x, k) for k in range(len(s.comps))])
        if s.kind == "Euler" and isinstance(_arg(x, 3), str) and _arg(x, 3) in _ORDERS:
            s.props["order"] = _arg(x, 3)               # Euler.set(x, y, z, order)
        return s

    def other(x, s):
        o = _arg(x, 0)
        if not isinstance(o, Vec):
            raise _Throw(_error_obj("TypeError", f"{s.kind} method expects a vector"))
        return o.v()

    def length(s):
        return math.sqrt(sum(c * c for c in s.v()))

    return {
        "set": lambda s, i, x: set_all(s, x),
        "setScalar": lambda s, i, x: s.setv([_num_arg(x, 0)] * len(s.comps)),
        "copy": lambda s, i, x: copy_from(s, x),
        "clone": lambda s, i, x: new_like(s, s.v()),
        "add": lambda s, i, x: s.setv([a + b for a, b in zip(s.v(), other(x, s))]),
        "sub": lambda s, i, x: s.setv([a - b for a, b in zip(s.v(), other(x, s))]),
        "addScalar": lambda s, i, x: s.setv([a + _num_arg(x, 0) for a in s.v()]),
        "multiplyScalar": lambda s, i, x: s.setv([a * _num_arg(x, 0) for a in s.v()]),
        "divideScalar": lambda s, i, x: s.setv([a / (_num_arg(x, 0) or math.inf) for a in s.v()]),
        "multiply": lambda s, i, x: s.setv([a * b for a, b in zip(s.v(), other(x, s))]),
        "addVectors": lambda s, i, x: s.setv([a + b for a, b in zip(_arg(x, 0).v(), _arg(x, 1).v())]),
        "subVectors": lambda s, i, x: s.setv([a - b for a, b in zip(_arg(x, 0).v(), _arg(x, 1).v())]),
        "negate": lambda s, i, x: s.setv([-a for a in s.v()]),
        "length": lambda s, i, x: length(s),
        "lengthSq": lambda s, i, x: sum(c * c for c in s.v()),
        "normalize": lambda s, i, x: s.setv([a / (length(s) or 1.0) for a in s.v()]),
        "setLength": lambda s, i, x: s.setv([a / (length(s) or 1.0) * _num_arg(x, 0) for a in s.v()]),
        "dot": lambda s, i, x: sum(a * b for a, b in zip(s.v(), other(x, s))),
        "cross": lambda s, i, x: s.setv(_cross(s.v(), other(x, s))),
        "crossVectors": lambda s, i, x: s.setv(_cross(_arg(x, 0).v(), _arg(x, 1).v())),
        "distanceTo": lambda s, i, x: math.sqrt(sum((a - b) ** 2 for a, b in zip(s.v(), other(x, s)))),
        "lerp": lambda s, i, x: s.setv([a + (b - a) * _num_arg(x, 1) for a, b in zip(s.v(), other(x, s))]),
        "lerpVectors": lambda s, i, x: s.setv([a + (b - a) * _num_arg(x, 2) for a, b in zip(_arg(x, 0).v(), _arg(x, 1).v())]),
        "equals": lambda s, i, x: s.v() == other(x, s),
        "toArray": lambda s, i, x: JSArray(s.v()),
        "fromArray": lambda s, i, x: s.setv([_to_num(v) for v in it_items(_arg(x, 0))][int(_num_arg(x, 1)):]),
        "applyAxisAngle": lambda s, i, x: s.setv(_rot_axis(s.v(), other(x, s), _num_arg(x, 1))),
        "applyEuler": lambda s, i, x: s.setv(_mat3_apply(_rot_mat(_arg(x, 0)), s.v())),
        "applyMatrix4": lambda s, i, x: s.setv(_mat4_point(_arg(x, 0).m, s.v())),
        "rotateAround": lambda s, i, x: s.setv(_rot2(s.v(), _arg(x, 0).v(), _num_arg(x, 1))),
        "angle": lambda s, i, x: math.atan2(s.v()[1], s.v()[0]) % (2 * math.pi),
        "setX": lambda s, i, x: _set_comp(s, 0, _num_arg(x, 0)),
        "setY": lambda s, i, x: _set_comp(s, 1, _num_arg(x, 0)),
        "setZ": lambda s, i, x: _set_comp(s, 2, _num_arg(x, 0)),
        "setW": lambda s, i, x: _set_comp(s, 3, _num_arg(x, 0)),
        "setComponent": lambda s, i, x: _set_comp(s, int(_num_arg(x, 0)), _num_arg(x, 1)),
        "getComponent": lambda s, i, x: s.v()[int(_num_arg(x, 0))] if 0 <= int(_num_arg(x, 0)) < len(s.comps) else UNDEF,
        "addScaledVector": lambda s, i, x: s.setv([a + b * _num_arg(x, 1) for a, b in zip(s.v(), other(x, s))]),
        "distanceToSquared": lambda s, i, x: sum((a - b) ** 2 for a, b in zip(s.v(), other(x, s))),
        "manhattanLength": lambda s, i, x: sum(abs(a) for a in s.v()),
        "min": lambda s, i, x: s.setv([min(a, b) for a, b in zip(s.v(), other(x, s))]),
        "max": lambda s, i, x: s.setv([max(a, b) for a, b in zip(s.v(), other(x, s))]),
        "clamp": lambda s, i, x: s.setv([max(lo, min(hi, a)) for a, lo, hi in zip(s.v(), _arg(x, 0).v(), _arg(x, 1).v())]),
        "clampScalar": lambda s, i, x: s.setv([max(_num_arg(x, 0), min(_num_arg(x, 1), a)) for a in s.v()]),
        "floor": lambda s, i, x: s.setv([float(math.floor(a)) for a in s.v()]),
        "ceil": lambda s, i, x: s.setv([float(math.ceil(a)) for a in s.v()]),
        "round": lambda s, i, x: s.setv([float(math.floor(a + 0.5)) for a in s.v()]),
        "applyQuaternion": lambda s, i, x: s.setv(_mat3_apply(_arg(x, 0).r, s.v())),
        "applyMatrix3": lambda s, i, x: s.setv(_mat3_apply(_arg(x, 0).m, s.v()[:3])),
        "transformDirection": lambda s, i, x: s.setv(_unit(_mat3_apply([r[:3] for r in _arg(x, 0).m[:3]], s.v()))),
        "angleTo": lambda s, i, x: _angle_to(s.v(), other(x, s)),
        "projectOnVector": lambda s, i, x: s.setv(_project(s.v(), other(x, s))),
        "projectOnPlane": lambda s, i, x: s.setv([a - b for a, b in zip(s.v(), _project(s.v(), other(x, s)))]),
        "reflect": lambda s, i, x: s.setv([a - 2 * sum(p * q for p, q in zip(s.v(), other(x, s))) * b
                                          for a, b in zip(s.v(), other(x, s))]),
        "setFromSpherical": lambda s, i, x: s.setv(_from_spherical(*_arg(x, 0).rpt())),
        "setFromSphericalCoords": lambda s, i, x: s.setv(_from_spherical(_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2))),
        "setFromCylindrical": lambda s, i, x: s.setv(_from_cylindrical(*_arg(x, 0).rty())),
        "setFromCylindricalCoords": lambda s, i, x: s.setv(_from_cylindrical(_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2))),
        "setFromMatrixPosition": lambda s, i, x: s.setv([_arg(x, 0).m[r][3] for r in range(3)]),
        "setFromQuaternion": lambda s, i, x: _set_rot(s, _arg(x, 0).cur()),
        "setFromRotationMatrix": lambda s, i, x: _set_rot(s, _rot_part(_arg(x, 0).m)),
        "setFromVector3": lambda s, i, x: s.setv(_arg(x, 0).v()[:3]),
        "setFromMatrixScale": lambda s, i, x: s.setv([math.sqrt(sum(_arg(x, 0).m[r][c] ** 2 for r in range(3)))
                                                      for c in range(3)]),
        "setFromMatrixColumn": lambda s, i, x: s.setv([_arg(x, 0).m[r][int(_num_arg(x, 1))] for r in range(3)]),
    }


def it_items(v):
    return v.items if isinstance(v, JSArray) else []


def _set_comp(s, k, val):
    if 0 <= k < len(s.comps):
        s.props[s.comps[k]] = float(val)
    return s


def _unit(v):
    n = math.sqrt(sum(a * a for a in v)) or 1.0
    return [a / n for a in v]


def _angle_to(a, b):
    den = math.sqrt(sum(x * x for x in a) * sum(y * y for y in b))
    if den == 0:
        return math.pi / 2
    return math.acos(max(-1.0, min(1.0, sum(x * y for x, y in zip(a, b)) / den)))


def _project(v, onto):
    den = sum(x * x for x in onto)
    if den == 0:
        return [0.0] * len(v)
    k = sum(x * y for x, y in zip(v, onto)) / den
    return [k * x for x in onto]


def _from_spherical(r, phi, theta):
    """three.js spherical coordinates: polar angle phi from +y, azimuth theta around y from +z."""
    sp = math.sin(phi) * r
    return [sp * math.sin(theta), math.cos(phi) * r, sp * math.cos(theta)]


def _from_cylindrical(r, theta, y):
    return [r * math.sin(theta), y, r * math.cos(theta)]


Vec.js_methods = _vec_methods()


def _cross(a, b):
    return [a[1] * b[2] - a[2] * b[1], a[2] * b[0] - a[0] * b[2], a[0] * b[1] - a[1] * b[0]]


def _rot2(p, c, ang):
    x, y = p[0] - c[0], p[1] - c[1]
    cs, sn = math.cos(ang), math.sin(ang)
    return [c[0] + x * cs - y * sn, c[1] + x * sn + y * cs]


def _rot_axis(v, axis, ang):
    n = math.sqrt(sum(a * a for a in axis)) or 1.0
    k = [a / n for a in axis]
    cs, sn = math.cos(ang), math.sin(ang)
    kxv = _cross(k, v)
    kdv = sum(a * b for a, b in zip(k, v))
    return [v[j] * cs + kxv[j] * sn + k[j] * kdv * (1 - cs) for j in range(3)]


def _axis_rot(axis, a):
    c, s = math.cos(a), math.sin(a)
    if axis == "X":
        return [[1.0, 0.0, 0.0], [0.0, c, -s], [0.0, s, c]]
    if axis == "Y":
        return [[c, 0.0, s], [0.0, 1.0, 0.0], [-s, 0.0, c]]
    return [[c, -s, 0.0], [s, c, 0.0], [0.0, 0.0, 1.0]]


def _euler_mat(e, order="XYZ"):
    """Rotation matrix of Euler angles (x, y, z) applied in `order` (three.js: for "XYZ", R = Rx * Ry * Rz)."""
    if order not in _ORDERS:
        order = "XYZ"
    ang = {"X": e[0], "Y": e[1], "Z": e[2]}
    m = [[1.0, 0.0, 0.0], [0.0, 1.0, 0.0], [0.0, 0.0, 1.0]]
    for ax in order:
        m = _mat_mul(m, _axis_rot(ax, ang[ax]))
    return m


_ORDERS = ("XYZ", "YXZ", "ZXY", "ZYX", "YZX", "XZY")


def _order(e) -> str:
    o = e.props.get("order", "XYZ") if isinstance(e, Vec) else "XYZ"
    return o if o in _ORDERS else "XYZ"


def _rot_mat(e):
    """Rotation matrix of an Euler vector in its own order (a plain vector: XYZ)."""
    return _euler_mat(e.v() if isinstance(e, Vec) else list(e), _order(e))


def _set_rot(e, m):
    """Write a rotation matrix into an Euler vector, in the vector's order; returns the vector."""
    e.setv(_mat3_to_euler(m, _order(e)))
    return e


def _mat3_apply(m, v):
    return [sum(m[r][k] * v[k] for k in range(3)) for r in range(3)]


def _mat3_to_euler(m, order="XYZ"):
    """Euler angles (x, y, z) in `order` of a rotation matrix (the inverse of _euler_mat; at gimbal lock the
    first-applied free angle takes the whole rotation)."""
    def cl(v):
        return max(-1.0, min(1.0, v))
    lim = 0.9999999
    if order == "YXZ":
        x = math.asin(-cl(m[1][2]))
        if abs(m[1][2]) < lim:
            return [x, math.atan2(m[0][2], m[2][2]), math.atan2(m[1][0], m[1][1])]
        return [x, math.atan2(-m[2][0], m[0][0]), 0.0]
    if order == "ZXY":
        x = math.asin(cl(m[2][1]))
        if abs(m[2][1]) < lim:
            return [x, math.atan2(-m[2][0], m[2][2]), math.atan2(-m[0][1], m[1][1])]
        return [x, 0.0, math.atan2(m[1][0], m[0][0])]
    if order == "ZYX":
        y = math.asin(-cl(m[2][0]))
        if abs(m[2][0]) < lim:
            return [math.atan2(m[2][1], m[2][2]), y, math.atan2(m[1][0], m[0][0])]
        return [0.0, y, math.atan2(-m[0][1], m[1][1])]
    if order == "YZX":
        z = math.asin(cl(m[1][0]))
        if abs(m[1][0]) < lim:
            return [math.atan2(-m[1][2], m[1][1]), math.atan2(-m[2][0], m[0][0]), z]
        return [0.0, math.atan2(m[0][2], m[2][2]), z]
    if order == "XZY":
        z = math.asin(-cl(m[0][1]))
        if abs(m[0][1]) < lim:
            return [math.atan2(m[2][1], m[1][1]), math.atan2(m[0][2], m[0][0]), z]
        return [math.atan2(-m[1][2], m[2][2]), 0.0, z]
    y = math.asin(cl(m[0][2]))
    if abs(m[0][2]) < lim:
        return [math.atan2(-m[1][2], m[2][2]), y, math.atan2(-m[0][1], m[0][0])]
    return [math.atan2(m[2][1], m[1][1]), y, 0.0]


def _mat_mul(a, b):
    n = len(a)
    return [[sum(a[r][k] * b[k][c] for k in range(n)) for c in range(n)] for r in range(n)]


def _mat4_point(m, v):
    """m: row-major 4x4 list; v: 3 coords."""
    w = m[3][0] * v[0] + m[3][1] * v[1] + m[3][2] * v[2] + m[3][3]
    w = w or 1.0
    return [(m[r][0] * v[0] + m[r][1] * v[1] + m[r][2] * v[2] + m[r][3]) / w for r in range(3)]


def _compose(pos, rot, scl, order="XYZ"):
    r = _euler_mat(rot, order)
    return [[r[0][0] * scl[0], r[0][1] * scl[1], r[0][2] * scl[2], pos[0]],
            [r[1][0] * scl[0], r[1][1] * scl[1], r[1][2] * scl[2], pos[1]],
            [r[2][0] * scl[0], r[2][1] * scl[1], r[2][2] * scl[2], pos[2]],
            [0.0, 0.0, 0.0, 1.0]]


def _m3to4(r):
    return [list(r[0]) + [0.0], list(r[1]) + [0.0], list(r[2]) + [0.0], [0.0, 0.0, 0.0, 1.0]]


def _det4(m):
    import numpy as np
    return float(np.linalg.det(np.asarray(m, dtype=np.float64)))


def _inv4(m):
    import numpy as np
    a = np.asarray(m, dtype=np.float64)
    if abs(np.linalg.det(a)) < 1e-300:
        return [[0.0] * 4 for _ in range(4)]
    return np.linalg.inv(a).tolist()


def _decompose(m, pos, quat, scl):
    sx, sy, sz = (math.sqrt(sum(m[r][c] ** 2 for r in range(3))) for c in range(3))
    if _det4(m) < 0:
        sx = -sx
    if isinstance(pos, Vec):
        pos.setv([m[0][3], m[1][3], m[2][3]])
    if isinstance(scl, Vec):
        scl.setv([sx, sy, sz])
    if isinstance(quat, Quaternion):
        ss = (sx or 1.0, sy or 1.0, sz or 1.0)
        quat.put([[m[r][c] / ss[c] for c in range(3)] for r in range(3)])
    return None


def _look4(m, eye, target, up):
    """Rotation part of three.js's Matrix4.lookAt: the z axis points from target to eye."""
    z = [a - b for a, b in zip(eye, target)]
    if sum(v * v for v in z) == 0:
        z = [0.0, 0.0, 1.0]
    z = _unit(z)
    x = _cross(up, z)
    if sum(v * v for v in x) == 0:
        z = _unit([z[0] + 1e-4, z[1], z[2]])
        x = _cross(up, z)
    x = _unit(x)
    y = _cross(z, x)
    out = [row[:] for row in m]
    for r in range(3):
        out[r][0], out[r][1], out[r][2] = x[r], y[r], z[r]
    return out


def _ident4():
    return [[1.0 if r == c else 0.0 for c in range(4)] for r in range(4)]


class Matrix4(Host):
    __slots__ = ("m",)
    cls_name = "Matrix4"

    def __init__(self, m=None):
        super().__init__({"isMatrix4": True})
        self.m = m or _ident4()

    def get_special(self, it, key):
        if key == "elements":
            return JSArray([self.m[r][c] for c in range(4) for r in range(4)])
        return super().get_special(it, key)

    def _rot(self, axis, a):
        cs, sn = math.cos(a), math.sin(a)
        m = _ident4()
        i, j = {"x": (1, 2), "y": (2, 0), "z": (0, 1)}[axis]
        m[i][i], m[i][j], m[j][i], m[j][j] = cs, -sn, sn, cs
        self.m = m
        return self

    js_methods = {
        "identity": lambda s, i, x: (setattr(s, "m", _ident4()), s)[-1],
        "copy": lambda s, i, x: (setattr(s, "m", [row[:] for row in _arg(x, 0).m]), s)[-1],
        "clone": lambda s, i, x: Matrix4([row[:] for row in s.m]),
        "makeTranslation": lambda s, i, x: (setattr(s, "m", _compose(
            _arg(x, 0).v() if isinstance(_arg(x, 0), Vec) else [_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2)],
            [0, 0, 0], [1, 1, 1])), s)[-1],
        "makeScale": lambda s, i, x: (setattr(s, "m", _compose([0, 0, 0], [0, 0, 0],
                                                                [_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2)])), s)[-1],
        "makeRotationX": lambda s, i, x: s._rot("x", _num_arg(x, 0)),
        "makeRotationY": lambda s, i, x: s._rot("y", _num_arg(x, 0)),
        "makeRotationZ": lambda s, i, x: s._rot("z", _num_arg(x, 0)),
        "makeRotationFromEuler": lambda s, i, x: (setattr(s, "m", _m3to4(_rot_mat(_arg(x, 0)))), s)[-1],
        "makeRotationFromQuaternion": lambda s, i, x: (setattr(s, "m", _m3to4(_arg(x, 0).cur())), s)[-1],
        "makeRotationAxis": lambda s, i, x: (setattr(s, "m", _m3to4(_axis_mat(_arg(x, 0).v(), _num_arg(x, 1)))), s)[-1],
        "invert": lambda s, i, x: (setattr(s, "m", _inv4(s.m)), s)[-1],
        "transpose": lambda s, i, x: (setattr(s, "m", [list(c) for c in zip(*s.m)]), s)[-1],
        "determinant": lambda s, i, x: _det4(s.m),
        "decompose": lambda s, i, x: _decompose(s.m, _arg(x, 0), _arg(x, 1), _arg(x, 2)) or s,
        "lookAt": lambda s, i, x: (setattr(s, "m", _look4(s.m, _arg(x, 0).v(), _arg(x, 1).v(), _arg(x, 2).v())), s)[-1],
        "extractRotation": lambda s, i, x: (setattr(s, "m", _m3to4(_rot_part(_arg(x, 0).m))), s)[-1],
        "scale": lambda s, i, x: (setattr(s, "m", [[s.m[r][c] * (_arg(x, 0).v()[c] if c < 3 else 1.0) for c in range(4)]
                                                   for r in range(4)]), s)[-1],
        "getMaxScaleOnAxis": lambda s, i, x: max(math.sqrt(sum(s.m[r][c] ** 2 for r in range(3))) for c in range(3)),
        "makeBasis": lambda s, i, x: (setattr(s, "m", [[_arg(x, 0).v()[r], _arg(x, 1).v()[r], _arg(x, 2).v()[r], 0.0]
                                                       for r in range(3)] + [[0.0, 0.0, 0.0, 1.0]]), s)[-1],
        "compose": lambda s, i, x: (setattr(s, "m", _compose(_arg(x, 0).v(), _quat_or_euler(_arg(x, 1)), _arg(x, 2).v())), s)[-1],
        "multiply": lambda s, i, x: (setattr(s, "m", _mat_mul(s.m, _arg(x, 0).m)), s)[-1],
        "premultiply": lambda s, i, x: (setattr(s, "m", _mat_mul(_arg(x, 0).m, s.m)), s)[-1],
        "multiplyMatrices": lambda s, i, x: (setattr(s, "m", _mat_mul(_arg(x, 0).m, _arg(x, 1).m)), s)[-1],
        "setPosition": lambda s, i, x: (_set_pos(s.m, _arg(x, 0).v() if isinstance(_arg(x, 0), Vec)
                                                 else [_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2)]), s)[-1],
    }


def _set_pos(m, p):
    m[0][3], m[1][3], m[2][3] = p


class Quaternion(Host):
    """A rotation, held as a 3x3 matrix. An object's `quaternion` is a live view of its rotation: reads come from
    the object's Euler angles and every change is written back to them."""
    __slots__ = ("r", "owner")
    cls_name = "Quaternion"

    def __init__(self, r=None, owner=None):
        super().__init__({"isQuaternion": True})
        self.r = r or _euler_mat([0, 0, 0])
        self.owner = owner

    def cur(self):
        if self.owner is not None:
            self.r = _rot_mat(self.owner.props["rotation"])
        return self.r

    def put(self, r):
        self.r = [list(map(float, row)) for row in r]
        if self.owner is not None:
            _set_rot(self.owner.props["rotation"], (self.r))
        return self

    def get_special(self, it, key):
        if key in ("x", "y", "z", "w"):
            return _m2q(self.cur())["xyzw".index(key)]
        return super().get_special(it, key)

    def set_special(self, it, key, value):
        if key in ("x", "y", "z", "w"):
            q = list(_m2q(self.cur()))
            q["xyzw".index(key)] = _to_num(value)
            self.put(_q2m(q))
            return True
        return False

    js_methods = {
        "set": lambda s, i, x: s.put(_q2m([_num_arg(x, k) for k in range(4)])),
        "setFromEuler": lambda s, i, x: s.put(_rot_mat(_arg(x, 0))),
        "setFromAxisAngle": lambda s, i, x: s.put(_axis_mat(_arg(x, 0).v(), _num_arg(x, 1))),
        "setFromUnitVectors": lambda s, i, x: s.put(_between(_arg(x, 0).v(), _arg(x, 1).v())),
        "setFromRotationMatrix": lambda s, i, x: s.put(_rot_part(_arg(x, 0).m)),
        "identity": lambda s, i, x: s.put(_euler_mat([0, 0, 0])),
        "multiply": lambda s, i, x: s.put(_mat_mul(s.cur(), _arg(x, 0).cur())),
        "premultiply": lambda s, i, x: s.put(_mat_mul(_arg(x, 0).cur(), s.cur())),
        "multiplyQuaternions": lambda s, i, x: s.put(_mat_mul(_arg(x, 0).cur(), _arg(x, 1).cur())),
        "slerp": lambda s, i, x: s.put(_q2m(_slerp(_m2q(s.cur()), _m2q(_arg(x, 0).cur()), _num_arg(x, 1)))),
        "slerpQuaternions": lambda s, i, x: s.put(_q2m(_slerp(_m2q(_arg(x, 0).cur()), _m2q(_arg(x, 1).cur()),
                                                              _num_arg(x, 2)))),
        "invert": lambda s, i, x: s.put([list(c) for c in zip(*s.cur())]),
        "conjugate": lambda s, i, x: s.put([list(c) for c in zip(*s.cur())]),
        "normalize": lambda s, i, x: s,
        "angleTo": lambda s, i, x: 2 * math.acos(min(1.0, abs(sum(a * b for a, b in zip(_m2q(s.cur()),
                                                                                        _m2q(_arg(x, 0).cur())))))),
        "dot": lambda s, i, x: sum(a * b for a, b in zip(_m2q(s.cur()), _m2q(_arg(x, 0).cur()))),
        "toArray": lambda s, i, x: JSArray(list(_m2q(s.cur()))),
        "fromArray": lambda s, i, x: s.put(_q2m([_to_num(i.get(_arg(x, 0), float(int(_num_arg(x, 1, 0.0)) + k)))
                                                 for k in range(4)])),
        "length": lambda s, i, x: 1.0,                  # held as a rotation: always a unit quaternion
        "lengthSq": lambda s, i, x: 1.0,
        "equals": lambda s, i, x: isinstance(_arg(x, 0), Quaternion) and all(
            abs(a - b) < 1e-12 for a, b in zip(_m2q(s.cur()), _m2q(_arg(x, 0).cur()))),
        "rotateTowards": lambda s, i, x: _rotate_towards(s, _arg(x, 0), _num_arg(x, 1)),
        "clone": lambda s, i, x: Quaternion([row[:] for row in s.cur()]),
        "copy": lambda s, i, x: s.put([row[:] for row in _arg(x, 0).cur()]),
    }


def _rotate_towards(q: "Quaternion", target, step: float):
    """Turn q toward target by at most `step` radians (slerp by step / angle)."""
    a, b = _m2q(q.cur()), _m2q(target.cur())
    angle = 2 * math.acos(min(1.0, abs(sum(p * r for p, r in zip(a, b)))))
    if angle == 0:
        return q
    return q.put(_q2m(_slerp(a, b, min(1.0, step / angle))))


def _m2q(m):
    """Unit quaternion (x, y, z, w) of a rotation matrix (the largest-diagonal branch is taken for stability)."""
    t = m[0][0] + m[1][1] + m[2][2]
    if t > 0:
        s = 0.5 / math.sqrt(t + 1.0)
        q = ((m[2][1] - m[1][2]) * s, (m[0][2] - m[2][0]) * s, (m[1][0] - m[0][1]) * s, 0.25 / s)
    elif m[0][0] > m[1][1] and m[0][0] > m[2][2]:
        s = 2.0 * math.sqrt(max(1e-30, 1.0 + m[0][0] - m[1][1] - m[2][2]))
        q = (0.25 * s, (m[0][1] + m[1][0]) / s, (m[0][2] + m[2][0]) / s, (m[2][1] - m[1][2]) / s)
    elif m[1][1] > m[2][2]:
        s = 2.0 * math.sqrt(max(1e-30, 1.0 + m[1][1] - m[0][0] - m[2][2]))
        q = ((m[0][1] + m[1][0]) / s, 0.25 * s, (m[1][2] + m[2][1]) / s, (m[0][2] - m[2][0]) / s)
    else:
        s = 2.0 * math.sqrt(max(1e-30, 1.0 + m[2][2] - m[0][0] - m[1][1]))
        q = ((m[0][2] + m[2][0]) / s, (m[1][2] + m[2][1]) / s, 0.25 * s, (m[1][0] - m[0][1]) / s)
    return q


def _q2m(q):
    x, y, z, w = q
    n = math.sqrt(x * x + y * y + z * z + w * w) or 1.0
    x, y, z, w = x / n, y / n, z / n, w / n
    return [[1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
            [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
            [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)]]


def _slerp(a, b, t):
    d = sum(p * q for p, q in zip(a, b))
    if d < 0:
        b, d = [-v for v in b], -d
    if d > 0.9995:
        return [p + (q - p) * t for p, q in zip(a, b)]
    th = math.acos(d)
    sa, sb = math.sin((1 - t) * th) / math.sin(th), math.sin(t * th) / math.sin(th)
    return [p * sa + q * sb for p, q in zip(a, b)]


def _between(a, b):
    """Rotation matrix taking the unit vector a onto the unit vector b."""
    a, b = _unit(a), _unit(b)
    c = sum(p * q for p, q in zip(a, b))
    if c < -0.999999:                               # opposite: half a turn about any perpendicular axis
        axis = _cross([1.0, 0.0, 0.0], a)
        if sum(v * v for v in axis) < 1e-12:
            axis = _cross([0.0, 1.0, 0.0], a)
        return _axis_mat(_unit(axis), math.pi)
    v = _cross(a, b)
    k = 1.0 / (1.0 + c)
    vx = [[0.0, -v[2], v[1]], [v[2], 0.0, -v[0]], [-v[1], v[0], 0.0]]
    vx2 = _mat_mul(vx, vx)
    return [[(1.0 if r == q else 0.0) + vx[r][q] + k * vx2[r][q] for q in range(3)] for r in range(3)]


def _rot_part(m4):
    """The rotation of a 4x4 transform (its upper 3x3 with the column scales divided out)."""
    cols = [[m4[r][c] for r in range(3)] for c in range(3)]
    cols = [_unit(c) for c in cols]
    return [[cols[c][r] for c in range(3)] for r in range(3)]


def _quat_copy(q):
    return Quaternion([row[:] for row in q.cur()])


def _axis_mat(axis, ang):
    cols = [_rot_axis(e, axis, ang) for e in ([1, 0, 0], [0, 1, 0], [0, 0, 1])]
    return [[cols[c][r] for c in range(3)] for r in range(3)]


def _quat_or_euler(q):
    if isinstance(q, Quaternion):
        return _mat3_to_euler(q.cur())
    if isinstance(q, Vec):
        return q.v()
    return [0.0, 0.0, 0.0]


_NAMED_COLORS = {"white": 0xFFFFFF, "black": 0x000000, "red": 0xFF0000, "green": 0x008000, "blue": 0x0000FF,
                 "yellow": 0xFFFF00, "orange": 0xFFA500, "purple": 0x800080, "gray": 0x808080, "grey": 0x808080,
                 "brown": 0xA52A2A, "pink": 0xFFC0CB, "cyan": 0x00FFFF, "magenta": 0xFF00FF, "silver": 0xC0C0C0,
                 "gold": 0xFFD700, "navy": 0x000080, "teal": 0x008080, "maroon": 0x800000, "olive": 0x808000,
                 "lime": 0x00FF00, "beige": 0xF5F5DC, "tan": 0xD2B48C, "skyblue": 0x87CEEB, "darkgreen": 0x006400,
                 "forestgreen": 0x228B22, "saddlebrown": 0x8B4513, "sienna": 0xA0522D, "ivory": 0xFFFFF0,
                 "khaki": 0xF0E68C, "coral": 0xFF7F50, "salmon": 0xFA8072, "chocolate": 0xD2691E,
                 "darkgray": 0xA9A9A9, "darkgrey": 0xA9A9A9, "lightgray": 0xD3D3D3, "lightgrey": 0xD3D3D3,
                 "dimgray": 0x696969, "wheat": 0xF5DEB3, "crimson": 0xDC143C, "indigo": 0x4B0082, "violet": 0xEE82EE}


def _srgb_to_linear(c: float) -> float:
    """The sRGB transfer function's inverse (IEC 61966-2-1)."""
    return c * 0.0773993808 if c < 0.04045 else (c * 0.9478672986 + 0.0521327014) ** 2.4


def _linear_to_srgb(c: float) -> float:
    return c * 12.92 if c < 0.0031308 else 1.055 * (c ** 0.41666) - 0.055


class Color(Host):
    """r, g, b in three.js's working colour space, linear sRGB: hex values, CSS strings and the sRGB colour-space
    arguments are converted on the way in, getHex / getStyle / the scene JSON's hex convert back, and
    setRGB / setHSL / setScalar / arithmetic work on the linear components (as three.js's colour management
    does)."""
    __slots__ = ()
    cls_name = "Color"

    def __init__(self, r=1.0, g=1.0, b=1.0):
        super().__init__({"r": r, "g": g, "b": b, "isColor": True})

    def rgb(self):
        return [_to_num(self.props[c]) for c in "rgb"]

    def srgb(self):
        return [_linear_to_srgb(c) for c in self.rgb()]

    def set_srgb(self, r, g, b):
        return self.set_rgb(_srgb_to_linear(r), _srgb_to_linear(g), _srgb_to_linear(b))

    def set_any(self, x):
        a = _arg(x, 0)
        if len(x) >= 3:
            return self.set_rgb(_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2))
        if isinstance(a, Color):
            return self.set_rgb(*a.rgb())
        if isinstance(a, (int, float)) and not isinstance(a, bool):
            h = int(a) & 0xFFFFFF
            return self.set_srgb(((h >> 16) & 255) / 255, ((h >> 8) & 255) / 255, (h & 255) / 255)
        if isinstance(a, str):
            s = a.strip().lower()
            if s.startswith("#"):
                s = s[1:]
                if len(s) == 3:
                    s = "".join(ch * 2 for ch in s)
                try:
                    h = int(s[:6], 16)
                except ValueError:
                    return self
                return self.set_any([float(h)])
            m = re.match(r"rgba?\(\s*(\d+)\s*,\s*(\d+)\s*,\s*(\d+)\s*(,\s*[\d.]+\s*)?\)", s)
            if m:
                return self.set_srgb(*(min(255, int(g)) / 255 for g in m.groups()[:3]))
            m = re.match(r"hsla?\(\s*([\d.]+)\s*,\s*([\d.]+)%\s*,\s*([\d.]+)%\s*(,\s*[\d.]+\s*)?\)", s)
            if m:
                return self.set_hsl(float(m.group(1)) / 360, float(m.group(2)) / 100, float(m.group(3)) / 100, True)
            if s in _NAMED_COLORS:
                return self.set_any([float(_NAMED_COLORS[s])])
        return self

    def set_rgb(self, r, g, b):
        self.props.update({"r": float(r), "g": float(g), "b": float(b)})
        return self

    def set_hsl(self, h, s, l, srgb=False):
        h = h % 1.0
        s = min(max(s, 0.0), 1.0)
        l = min(max(l, 0.0), 1.0)
        put = self.set_srgb if srgb else self.set_rgb
        if s == 0:
            return put(l, l, l)
        p = l * (1 + s) if l <= 0.5 else l + s - l * s
        q = 2 * l - p

        def hue(t):
            t %= 1.0
            if t < 1 / 6:
                return q + (p - q) * 6 * t
            if t < 1 / 2:
                return p
            if t < 2 / 3:
                return q + (p - q) * 6 * (2 / 3 - t)
            return q
        return put(hue(h + 1 / 3), hue(h), hue(h - 1 / 3))

    def get_hsl(self, srgb=False):
        r, g, b = self.srgb() if srgb else self.rgb()
        mx, mn = max(r, g, b), min(r, g, b)
        l = (mx + mn) / 2
        if mx == mn:
            return 0.0, 0.0, l
        d = mx - mn
        s = d / (2 - mx - mn) if l > 0.5 else d / (mx + mn)
        if mx == r:
            h = (g - b) / d + (6 if g < b else 0)
        elif mx == g:
            h = (b - r) / d + 2
        else:
            h = (r - g) / d + 4
        return h / 6, s, l

    def hex(self) -> int:
        """The sRGB hex value (getHex)."""
        r, g, b = (int(math.floor(max(0.0, min(255.0, c * 255)) + 0.5)) for c in self.srgb())
        return (r << 16) | (g << 8) | b

    def set_special(self, it, key, value):
        if key in ("r", "g", "b"):
            self.props[key] = _to_num(value)
            return True
        return False

    js_methods = {
        "set": lambda s, i, x: s.set_any(x),
        "setHex": lambda s, i, x: s.set_any([float(int(_num_arg(x, 0)))]),
        "setRGB": lambda s, i, x: (s.set_srgb if _arg(x, 3) == "srgb" else s.set_rgb)(
            _num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2)),
        "setHSL": lambda s, i, x: s.set_hsl(_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2), _arg(x, 3) == "srgb"),
        "getRGB": lambda s, i, x: (lambda t, c: (t.props.update({"r": c[0], "g": c[1], "b": c[2]}), t)[-1])(
            _arg(x, 0) if isinstance(_arg(x, 0), (JSObject, Color)) else JSObject(),
            s.srgb() if _arg(x, 1) == "srgb" else s.rgb()),
        "convertSRGBToLinear": lambda s, i, x: s.set_srgb(*s.rgb()),
        "convertLinearToSRGB": lambda s, i, x: s.set_rgb(*s.srgb()),
        "copySRGBToLinear": lambda s, i, x: s.set_srgb(*_arg(x, 0).rgb()),
        "copyLinearToSRGB": lambda s, i, x: s.set_rgb(*_arg(x, 0).srgb()),
        "setStyle": lambda s, i, x: s.set_any(x[:1]),
        "setScalar": lambda s, i, x: s.set_rgb(*[_num_arg(x, 0)] * 3),
        "getHex": lambda s, i, x: float(s.hex()),
        "getHexString": lambda s, i, x: f"{s.hex():06x}",
        "getStyle": lambda s, i, x: f"rgb({','.join(str(int(math.floor(c * 255 + 0.5))) for c in s.srgb())})",
        "getHSL": lambda s, i, x: _hsl_out(s, _arg(x, 0), _arg(x, 1) == "srgb"),
        "offsetHSL": lambda s, i, x: (lambda h: s.set_hsl(h[0] + _num_arg(x, 0), h[1] + _num_arg(x, 1),
                                                         h[2] + _num_arg(x, 2)))(s.get_hsl()),
        "clone": lambda s, i, x: Color(*s.rgb()),
        "copy": lambda s, i, x: s.set_rgb(*_arg(x, 0).rgb()),
        "multiplyScalar": lambda s, i, x: s.set_rgb(*[c * _num_arg(x, 0) for c in s.rgb()]),
        "multiply": lambda s, i, x: s.set_rgb(*[a * b for a, b in zip(s.rgb(), _arg(x, 0).rgb())]),
        "add": lambda s, i, x: s.set_rgb(*[a + b for a, b in zip(s.rgb(), _arg(x, 0).rgb())]),
        "addScalar": lambda s, i, x: s.set_rgb(*[c + _num_arg(x, 0) for c in s.rgb()]),
        "lerp": lambda s, i, x: s.set_rgb(*[a + (b - a) * _num_arg(x, 1) for a, b in zip(s.rgb(), _arg(x, 0).rgb())]),
        "lerpColors": lambda s, i, x: s.set_rgb(*[a + (b - a) * _num_arg(x, 2)
                                                  for a, b in zip(_arg(x, 0).rgb(), _arg(x, 1).rgb())]),
        "equals": lambda s, i, x: s.rgb() == _arg(x, 0).rgb(),
    }


def _hsl_out(c, target, srgb=False):
    h, s, l = c.get_hsl(srgb)
    o = target if isinstance(target, JSObject) else JSObject()
    o.props.update({"h": h, "s": s, "l": l})
    return o


# geometries: record type + params + baked transforms; triangulated only at serialisation

_GEOM_PARAMS = {
    "BoxGeometry": ("width", "height", "depth", "widthSegments", "heightSegments", "depthSegments"),
    "SphereGeometry": ("radius", "widthSegments", "heightSegments", "phiStart", "phiLength", "thetaStart", "thetaLength"),
    "CylinderGeometry": ("radiusTop", "radiusBottom", "height", "radialSegments", "heightSegments", "openEnded",
                         "thetaStart", "thetaLength"),
    "ConeGeometry": ("radius", "height", "radialSegments", "heightSegments", "openEnded", "thetaStart", "thetaLength"),
    "PlaneGeometry": ("width", "height", "widthSegments", "heightSegments"),
    "CircleGeometry": ("radius", "segments", "thetaStart", "thetaLength"),
    "RingGeometry": ("innerRadius", "outerRadius", "thetaSegments", "phiSegments", "thetaStart", "thetaLength"),
    "TorusGeometry": ("radius", "tube", "radialSegments", "tubularSegments", "arc"),
    "TorusKnotGeometry": ("radius", "tube", "tubularSegments", "radialSegments", "p", "q"),
    "CapsuleGeometry": ("radius", "length", "capSegments", "radialSegments"),
    "IcosahedronGeometry": ("radius", "detail"),
    "OctahedronGeometry": ("radius", "detail"),
    "TetrahedronGeometry": ("radius", "detail"),
    "DodecahedronGeometry": ("radius", "detail"),
    "LatheGeometry": ("points", "segments", "phiStart", "phiLength"),
    "TubeGeometry": ("path", "tubularSegments", "radius", "radialSegments", "closed"),
    "ExtrudeGeometry": ("shapes", "options"),
    "ShapeGeometry": ("shapes", "curveSegments"),
}
_GEOM_DEFAULTS = {
    "BoxGeometry": (1, 1, 1, 1, 1, 1), "SphereGeometry": (1, 32, 16, 0, 2 * math.pi, 0, math.pi),
    "CylinderGeometry": (1, 1, 1, 32, 1, False, 0, 2 * math.pi), "ConeGeometry": (1, 1, 32, 1, False, 0, 2 * math.pi),
    "PlaneGeometry": (1, 1, 1, 1), "CircleGeometry": (1, 32, 0, 2 * math.pi),
    "RingGeometry": (0.5, 1, 32, 1, 0, 2 * math.pi), "TorusGeometry": (1, 0.4, 12, 48, 2 * math.pi),
    "TorusKnotGeometry": (1, 0.4, 64, 8, 2, 3), "CapsuleGeometry": (1, 1, 4, 8), "IcosahedronGeometry": (1, 0),
    "OctahedronGeometry": (1, 0), "TetrahedronGeometry": (1, 0), "DodecahedronGeometry": (1, 0),
    "LatheGeometry": (None, 12, 0, 2 * math.pi), "TubeGeometry": (None, 64, 1, 8, False),
    "ExtrudeGeometry": (None, None), "ShapeGeometry": (None, 12),
}


class Geometry(Host):
    """A three.js geometry. Primitives stay parametric (tessellated when the scene is serialised) until a module
    touches their vertex data (`attributes`, `getAttribute`, `setAttribute`, `index`, `setIndex`); then they are
    baked once into explicit position / normal / index (and, for planes, uv) buffers, as three.js primitives
    always are, and the module edits those."""
    __slots__ = ("gtype", "params", "xform", "buffer", "id_", "baked")
    cls_name = "BufferGeometry"
    bases = ("BufferGeometry",)

    def __init__(self, gtype="BufferGeometry", params=None):
        super().__init__({"isBufferGeometry": True})
        self.gtype = gtype
        self.params = params or {}
        self.xform = _ident4()
        self.buffer: Dict[str, Any] = {}
        self.id_ = _uuid.uuid4().hex
        self.baked = False

    def get_special(self, it, key):
        if key == "type":
            return self.gtype
        if key == "parameters":
            return JSObject({k: v for k, v in self.params.items()})
        if key == "attributes":
            _bake(self)
            return JSObject({k: v for k, v in self.buffer.items() if k != "__index"})
        if key == "index":
            _bake(self)
            return self.buffer.get("__index", None)
        if key == "uuid":
            return self.id_
        return super().get_special(it, key)

    def is_instance(self, name):
        return name in (self.gtype, "BufferGeometry")

    def apply(self, m):
        """Transforms move explicit vertex buffers at once (as three.js's applyMatrix4 does, normals by the
        inverse transpose); parametric primitives keep the transform until they are tessellated."""
        pos = self.buffer.get("position")
        if not (isinstance(pos, BufferAttribute) and pos.item == 3):
            self.xform = _mat_mul(m, self.xform)
            return self
        import torch
        mt = torch.tensor(m, dtype=torch.float64)
        v = torch.tensor(pos.array, dtype=torch.float64).view(-1, 3)
        pos.array = ((v @ mt[:3, :3].t()) + mt[:3, 3]).reshape(-1).tolist()
        nrm = self.buffer.get("normal")
        if isinstance(nrm, BufferAttribute) and nrm.item == 3 and nrm is not pos:
            nm = torch.linalg.inv(mt[:3, :3]).t() if abs(float(torch.det(mt[:3, :3]))) > 1e-30 else mt[:3, :3]
            n = torch.tensor(nrm.array, dtype=torch.float64).view(-1, 3) @ nm.t()
            nrm.array = (n / n.norm(dim=1, keepdim=True).clamp(min=1e-30)).reshape(-1).tolist()
        return self

    js_methods = {
        "translate": lambda s, i, x: s.apply(_compose([_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2)], [0, 0, 0], [1, 1, 1])),
        "scale": lambda s, i, x: s.apply(_compose([0, 0, 0], [0, 0, 0], [_num_arg(x, 0, 1.0), _num_arg(x, 1, 1.0), _num_arg(x, 2, 1.0)])),
        "rotateX": lambda s, i, x: s.apply(_compose([0, 0, 0], [_num_arg(x, 0), 0, 0], [1, 1, 1])),
        "rotateY": lambda s, i, x: s.apply(_compose([0, 0, 0], [0, _num_arg(x, 0), 0], [1, 1, 1])),
        "rotateZ": lambda s, i, x: s.apply(_compose([0, 0, 0], [0, 0, _num_arg(x, 0)], [1, 1, 1])),
        "applyMatrix4": lambda s, i, x: s.apply(_arg(x, 0).m),
        "center": lambda s, i, x: _geom_center(s),
        "computeVertexNormals": lambda s, i, x: _compute_normals(s),
        "clone": lambda s, i, x: _geom_clone(s),
        "dispose": lambda s, i, x: UNDEF,
        "setAttribute": lambda s, i, x: (_bake(s), s.buffer.__setitem__(_to_str(_arg(x, 0)), _arg(x, 1)), s)[-1],
        "getAttribute": lambda s, i, x: (_bake(s), s.buffer.get(_to_str(_arg(x, 0)), UNDEF))[-1],
        "deleteAttribute": lambda s, i, x: (_bake(s), s.buffer.pop(_to_str(_arg(x, 0)), None), s)[-1],
        "setIndex": lambda s, i, x: (_bake(s), s.buffer.__setitem__("__index", _index_attr(i, _arg(x, 0))), s)[-1],
        "addGroup": lambda s, i, x: (s.props.setdefault("groups", JSArray()).items.append(JSObject(
            {"start": _num_arg(x, 0), "count": _num_arg(x, 1), "materialIndex": _num_arg(x, 2)})), UNDEF)[-1],
        "clearGroups": lambda s, i, x: (s.props.__setitem__("groups", JSArray()), UNDEF)[-1],
        "setDrawRange": lambda s, i, x: (s.props.__setitem__("drawRange", JSObject(
            {"start": _num_arg(x, 0), "count": _num_arg(x, 1, math.inf)})), UNDEF)[-1],
        "toNonIndexed": lambda s, i, x: _non_indexed(s),
        "computeBoundingBox": lambda s, i, x: (s.props.__setitem__("boundingBox", _geom_box(s)), UNDEF)[-1],
        "computeBoundingSphere": lambda s, i, x: (s.props.__setitem__("boundingSphere", _geom_sphere(s)), UNDEF)[-1],
        "setFromPoints": lambda s, i, x: (s.buffer.__setitem__("position", BufferAttribute(
            [c for p in it_items(_arg(x, 0)) for c in (p.v() + [0.0])[:3]], 3)), s)[-1],
    }


def _index_attr(it, idx):
    """setIndex's argument as three.js stores it: an array becomes a Uint16 (or, above 65535, Uint32) attribute."""
    if isinstance(idx, JSArray) and not isinstance(idx, TypedArray):
        vals = [_to_num(v) for v in it.iterate(idx)]
        return BufferAttribute(vals, 1, "Uint32Array" if any(v > 65535 for v in vals) else "Uint16Array")
    if isinstance(idx, TypedArray):
        return BufferAttribute(idx, 1)
    return idx if isinstance(idx, BufferAttribute) else None


def _compute_normals(g: Geometry):
    """computeVertexNormals: area-weighted sums of the face normals around each vertex of the position buffer
    (indexed geometry shares them across faces; non-indexed geometry gets flat normals), written into the existing
    normal attribute when it has the right size."""
    _bake(g)
    pos = g.buffer.get("position")
    if not (isinstance(pos, BufferAttribute) and pos.item == 3):
        return UNDEF
    v, f = geometry_mesh(g)
    vals = _vertex_normals(v, f).reshape(-1).tolist()
    nrm = g.buffer.get("normal")
    if isinstance(nrm, BufferAttribute) and nrm.item == 3 and len(nrm.array) == len(vals) and nrm is not pos:
        nrm.array = vals
    else:
        g.buffer["normal"] = BufferAttribute(vals, 3)
    return UNDEF


def _non_indexed(g: Geometry) -> Geometry:
    """A copy with three vertices per triangle (positions only), as three.js's toNonIndexed."""
    v, f = geometry_mesh(g)
    return _baked(g.gtype if g.gtype != "BufferGeometry" else "BufferGeometry", v[f.reshape(-1)].tolist())


def _geom_box(g: Geometry):
    v, _ = geometry_mesh(g)
    b = Box3()
    if v.shape[0]:
        b.props["min"].setv(v.min(0).values.tolist())
        b.props["max"].setv(v.max(0).values.tolist())
    return b


def _geom_sphere(g: Geometry):
    v, _ = geometry_mesh(g)
    sp = Sphere()
    if v.shape[0]:
        c = ((v.min(0).values + v.max(0).values) / 2)
        sp.props["center"].setv(c.tolist())
        sp.props["radius"] = float((v - c).norm(dim=1).max())
    return sp


def _geom_clone(g: Geometry) -> Geometry:
    n = Geometry(g.gtype, dict(g.params))
    n.xform = [row[:] for row in g.xform]
    n.buffer = {k: (BufferAttribute(list(v.array), v.item, v.data.kind) if isinstance(v, BufferAttribute) else v)
                for k, v in g.buffer.items()}
    n.baked = g.baked
    return n


PLANE_MAX_SEGMENTS = 512


def _plane_grid(width: float, height: float, gx: int, gy: int):
    """Vertices, faces and uvs of a width x height plane of gx x gy cells in the xy plane, facing +z: rows of
    gx + 1 vertices from the top edge (y = height / 2) down, two triangles per cell, counter-clockwise."""
    import torch
    xs = torch.arange(gx + 1, dtype=torch.float32) * (width / gx) - width / 2
    ys = height / 2 - torch.arange(gy + 1, dtype=torch.float32) * (height / gy)
    v = torch.stack([xs[None, :].expand(gy + 1, -1), ys[:, None].expand(-1, gx + 1),
                     torch.zeros(gy + 1, gx + 1)], -1).reshape(-1, 3)
    uv = torch.stack([(torch.arange(gx + 1, dtype=torch.float32) / gx)[None, :].expand(gy + 1, -1),
                      (1 - torch.arange(gy + 1, dtype=torch.float32) / gy)[:, None].expand(-1, gx + 1)], -1)
    top = (torch.arange(gy)[:, None] * (gx + 1) + torch.arange(gx)[None, :]).reshape(-1)   # cell's top-left
    bot = top + gx + 1
    f = torch.cat([torch.stack([top, bot, top + 1], 1), torch.stack([bot, bot + 1, top + 1], 1)])
    return v, f, uv.reshape(-1, 2)


def _vertex_normals(v, f):
    import torch
    n = torch.zeros_like(v)
    if f.numel():
        fn = torch.cross(v[f[:, 1]] - v[f[:, 0]], v[f[:, 2]] - v[f[:, 0]], dim=1)    # area-weighted
        for k in range(3):
            n.index_add_(0, f[:, k], fn)
    return n / n.norm(dim=1, keepdim=True).clamp(min=1e-12)


_NON_INDEXED = {"ExtrudeGeometry", "PolyhedronGeometry", "TetrahedronGeometry", "OctahedronGeometry",
                "IcosahedronGeometry", "DodecahedronGeometry"}


def _bake(g: Geometry) -> None:
    """Turn a parametric primitive into explicit buffers (transform applied), once."""
    if g.baked or g.gtype == "BufferGeometry":
        return
    import torch
    uv = None
    if g.gtype == "PlaneGeometry":
        def seg(k):
            q = g.params.get(k, 1)
            return max(1, min(PLANE_MAX_SEGMENTS, int(_to_num(q)) if q not in (UNDEF, None) else 1))
        def num(k):
            q = g.params.get(k, 1)
            return float(_to_num(q)) if q not in (UNDEF, None) else 1.0
        v, f, uv = _plane_grid(num("width"), num("height"), seg("widthSegments"), seg("heightSegments"))
        m = torch.tensor(g.xform, dtype=torch.float32)
        v = (torch.cat([v, torch.ones(v.shape[0], 1)], 1) @ m.t())[:, :3]
    else:
        v, f = geometry_mesh(g)
    nrm = _vertex_normals(v, f)
    indexed = g.gtype not in _NON_INDEXED
    if not indexed and f.numel():
        # three.js builds these without an index: three vertices of their own per triangle; the polyhedra with
        # detail > 0 keep smooth (shared) normals, the rest are flat
        smooth = g.gtype != "ExtrudeGeometry" and int(_to_num(g.params.get("detail", 0) or 0)) > 0
        flat = f.reshape(-1)
        nrm = nrm[flat] if smooth else _vertex_normals(v[flat], torch.arange(flat.numel()).view(-1, 3))
        v = v[flat]
    g.buffer.setdefault("position", BufferAttribute(v.reshape(-1).tolist(), 3))
    g.buffer.setdefault("normal", BufferAttribute(nrm.reshape(-1).tolist(), 3))
    if uv is not None:
        g.buffer.setdefault("uv", BufferAttribute(uv.reshape(-1).tolist(), 2))
    if indexed:
        g.buffer.setdefault("__index", BufferAttribute(f.reshape(-1).tolist(), 1, "Uint32Array"))
    g.xform = _ident4()
    g.baked = True


def _geom_center(g: Geometry):
    v, _ = geometry_mesh(g)
    if v.shape[0]:
        c = (v.min(0).values + v.max(0).values) / 2
        g.apply(_compose([-float(c[0]), -float(c[1]), -float(c[2])], [0, 0, 0], [1, 1, 1]))
    return g


class BufferAttribute(Host):
    """A vertex attribute over a typed array. The array is the module's own (`new BufferAttribute(arr, 3)` keeps
    `arr`, and `attribute.array` returns it), so element writes through either reach the geometry."""
    __slots__ = ("data", "item")
    cls_name = "BufferAttribute"

    def __init__(self, array, item_size, kind: str = "Float32Array"):
        super().__init__({"isBufferAttribute": True})
        self.data = array if isinstance(array, TypedArray) else TypedArray(kind, list(array))
        self.item = max(1, int(item_size))

    @property
    def array(self) -> list:
        return self.data.items

    @array.setter
    def array(self, vals) -> None:
        self.data.items = _typed_values(self.data.kind, vals)

    def get_special(self, it, key):
        if key == "count":
            return float(len(self.array) // max(self.item, 1))
        if key == "itemSize":
            return float(self.item)
        if key == "array":
            return self.data
        return super().get_special(it, key)

    def _set(self, i, k, v):
        j = int(i) * self.item + k
        if 0 <= j < len(self.array):
            self.array[j] = _typed_value(self.data.kind, v)
        return self

    def _get(self, i, k):
        j = int(i) * self.item + k
        return self.array[j] if 0 <= j < len(self.array) else UNDEF

    js_methods = {
        "setXYZ": lambda s, i, x: (s._set(_num_arg(x, 0), 0, _num_arg(x, 1)), s._set(_num_arg(x, 0), 1, _num_arg(x, 2)),
                                   s._set(_num_arg(x, 0), 2, _num_arg(x, 3)))[-1],
        "setXY": lambda s, i, x: (s._set(_num_arg(x, 0), 0, _num_arg(x, 1)), s._set(_num_arg(x, 0), 1, _num_arg(x, 2)))[-1],
        "setX": lambda s, i, x: s._set(_num_arg(x, 0), 0, _num_arg(x, 1)),
        "setY": lambda s, i, x: s._set(_num_arg(x, 0), 1, _num_arg(x, 1)),
        "setZ": lambda s, i, x: s._set(_num_arg(x, 0), 2, _num_arg(x, 1)),
        "getX": lambda s, i, x: s._get(_num_arg(x, 0), 0),
        "getY": lambda s, i, x: s._get(_num_arg(x, 0), 1),
        "getZ": lambda s, i, x: s._get(_num_arg(x, 0), 2),
        "setUsage": lambda s, i, x: (s.props.__setitem__("usage", _arg(x, 0)), s)[-1],
    }


class Material(Host):
    __slots__ = ("mtype",)
    cls_name = "Material"

    def __init__(self, mtype, params: Optional[JSObject] = None):
        super().__init__({"isMaterial": True, "color": Color(1, 1, 1), "opacity": 1.0, "transparent": False,
                          "side": 0.0, "visible": True, "wireframe": False})
        self.mtype = mtype
        if isinstance(params, JSObject):
            for k, v in params.props.items():
                self.js_set(None, k, v)

    def chain(self):
        return _MAT_CHAIN.get(self.mtype, (self.mtype,))

    def get_special(self, it, key):
        if key == "type":
            return self.mtype
        if key.startswith("is") and key[2:] in self.chain() and key not in self.props:
            return True                                 # isMeshStandardMaterial, isLineBasicMaterial ...
        return super().get_special(it, key)

    def is_instance(self, name):
        return name == "Material" or name in self.chain()

    def set_special(self, it, key, value):
        if key in ("color", "emissive", "specular", "sheenColor", "attenuationColor"):
            c = Color(0, 0, 0)
            c.set_any([value])
            self.props[key] = c
            return True
        return False

    js_methods = {
        "clone": lambda s, i, x: _mat_clone(s),
        "dispose": lambda s, i, x: UNDEF,
        "setValues": lambda s, i, x: ([s.js_set(i, k, v) for k, v in _arg(x, 0).props.items()], UNDEF)[-1],
    }


def _mat_clone(m: Material):
    n = Material(m.mtype)
    for k, v in m.props.items():
        n.props[k] = Color(*v.rgb()) if isinstance(v, Color) else v
    return n


class Texture(Host):
    """A texture over the module's data array (DataTexture keeps the array it is given, so texels written after
    construction count): its data size in bytes (a typed array's byteLength, as the texture-data limit counts
    it; 0 for a plain array, which has none) and the mean texel colour (the renders tint a mapped surface by it;
    texel values are read as 8-bit or float channels of an RGBA / RGB / RG / R layout)."""
    __slots__ = ("src", "ch", "scale", "size")
    cls_name = "Texture"

    def __init__(self, src=None, ch: int = 4, scale: float = 255.0, size=(0.0, 0.0), data_texture: bool = False):
        super().__init__({"isTexture": True, "repeat": Vec(("x", "y"), [1, 1], "Vector2"),
                          "offset": Vec(("x", "y"), [0, 0], "Vector2"), "colorSpace": "", "needsUpdate": False})
        if data_texture:
            self.props["isDataTexture"] = True
        self.src, self.ch, self.scale, self.size = src, ch, scale, size

    def get_special(self, it, key):
        if key == "image":
            return JSObject({"data": self.src if self.src is not None else None,
                             "width": self.size[0], "height": self.size[1]})
        return super().get_special(it, key)

    @property
    def nbytes(self) -> int:
        return len(self.src.items) * TYPED_BYTES[self.src.kind] if isinstance(self.src, TypedArray) else 0

    @property
    def mean(self):
        """Raw mean texel RGB in [0, 1] of the data as it is now, or None."""
        data = self.src.items if isinstance(self.src, JSArray) else []
        ch = self.ch
        n = len(data) // ch
        if not n:
            return None
        step = max(1, n // 4096)                  # a sample of the texels is enough for the mean
        acc = [0.0, 0.0, 0.0]
        cnt = 0
        for k in range(0, n, step):
            px = [_to_num(data[k * ch + c]) / self.scale for c in range(ch)]
            rgb = px[:3] if ch >= 3 else [px[0]] * 3
            acc = [a + (max(0.0, min(1.0, v)) if v == v else 0.0) for a, v in zip(acc, rgb)]
            cnt += 1
        return [a / cnt for a in acc]

    def linear_mean(self):
        mean = self.mean
        if mean is None:
            return None
        if self.props.get("colorSpace") == "srgb":
            return [c ** 2.2 for c in mean]
        return list(mean)

    js_methods = {"clone": lambda s, i, x: _texture_clone(s), "dispose": lambda s, i, x: UNDEF}


def _texture_clone(t: Texture) -> Texture:
    """clone shares the image data, as three.js's does; settings are copied."""
    n = Texture(t.src, t.ch, t.scale, t.size, data_texture=bool(t.props.get("isDataTexture")))
    for k, v in t.props.items():
        n.props[k] = Vec(v.comps, v.v(), v.kind) if isinstance(v, Vec) else v
    return n


def _data_texture(x):
    """DataTexture(data, width, height, format, type)."""
    data = _arg(x, 0) if x else None
    fmt = _num_arg(x, 3, 1023.0)
    ch = {1023.0: 4, 1022.0: 3, 1030.0: 2, 1028.0: 1, 1024.0: 1}.get(fmt, 4)
    typ = _num_arg(x, 4, 1009.0)
    scale = 255.0 if typ in (1009.0, 1010.0) else 1.0
    return Texture(data if isinstance(data, JSArray) else None, ch, scale, (_num_arg(x, 1, 1.0), _num_arg(x, 2, 1.0)),
                   data_texture=True)


# three.js class chains below Object3D: an object answers is<Class> and instanceof for each
_OBJ_CHAIN = {"InstancedMesh": ("InstancedMesh", "Mesh"), "LineSegments": ("LineSegments", "Line"),
              "LineLoop": ("LineLoop", "Line")}
_MAT_CHAIN = {"MeshPhysicalMaterial": ("MeshPhysicalMaterial", "MeshStandardMaterial"),
              "LineDashedMaterial": ("LineDashedMaterial", "LineBasicMaterial")}


class Object3D(Host):
    __slots__ = ("otype", "id_", "quat_")
    cls_name = "Object3D"

    def __init__(self, otype="Object3D", geometry=None, material=None):
        super().__init__({"isObject3D": True, "name": "", "visible": True, "castShadow": False,
                          "receiveShadow": False, "userData": JSObject(), "parent": None,
                          "position": Vec(("x", "y", "z"), None, "Vector3"),
                          "rotation": Vec(("x", "y", "z"), None, "Euler"),
                          "scale": Vec(("x", "y", "z"), [1, 1, 1], "Vector3"),
                          "children": JSArray(), "matrix": Matrix4(), "matrixAutoUpdate": True})
        self.otype = otype
        self.id_ = _uuid.uuid4().hex
        if geometry is not None:
            self.props["geometry"] = geometry
        if material is not None:
            self.props["material"] = material

    def chain(self):
        return _OBJ_CHAIN.get(self.otype, (self.otype,))

    def get_special(self, it, key):
        if key == "type":
            return self.otype
        if key == "uuid":
            return self.id_
        if key.startswith("is") and key[2:] in self.chain() and key not in self.props:
            return True                                 # isMesh, isInstancedMesh, isLine, isLineSegments, isGroup ...
        if key == "quaternion":
            if getattr(self, "quat_", None) is None:
                self.quat_ = Quaternion(owner=self)
            return self.quat_
        if key == "matrixWorld":
            return Matrix4(_world4(self))
        if key == "up":
            return Vec(("x", "y", "z"), [0, 1, 0], "Vector3")
        return super().get_special(it, key)

    def is_instance(self, name):
        return name == "Object3D" or name in self.chain()

    def set_special(self, it, key, value):
        if key in ("position", "rotation", "scale"):
            raise _Throw(_error_obj("TypeError", f"cannot assign to read only property '{key}' of object"))
        return False

    def composed(self):
        return _compose(self.props["position"].v(), self.props["rotation"].v(), self.props["scale"].v(),
                        _order(self.props["rotation"]))

    def local(self):
        """The local matrix three.js renders with: composed from position / rotation / scale, or, once the module
        sets matrixAutoUpdate = false, the `matrix` it holds (kept by updateMatrix or written directly)."""
        m = self.props.get("matrix")
        if self.props.get("matrixAutoUpdate", True) is False and isinstance(m, Matrix4):
            return [row[:] for row in m.m]
        return self.composed()

    def children(self) -> list:
        return self.props["children"].items

    def add(self, objs):
        for o in objs:
            if not isinstance(o, Object3D):
                raise _Throw(_error_obj("TypeError", "add() expects Object3D instances"))
            if o is self:
                continue
            old = o.props.get("parent")
            if isinstance(old, Object3D):
                old.children()[:] = [c for c in old.children() if c is not o]
            o.props["parent"] = self
            self.children().append(o)
        return self

    def rotate_local(self, axis, ang):
        r = _rot_mat(self.props["rotation"])
        a = {"x": [1, 0, 0], "y": [0, 1, 0], "z": [0, 0, 1]}[axis]
        _set_rot(self.props["rotation"], (_mat_mul(r, _axis_mat(a, ang))))
        return self

    def look_at(self, target):
        p = self.props["position"].v()
        f = [t - q for t, q in zip(target, p)]
        n = math.sqrt(sum(c * c for c in f)) or 1.0
        z = [c / n for c in f]                      # objects look down +z
        up = [0.0, 1.0, 0.0] if abs(z[1]) < 0.999 else [0.0, 0.0, 1.0]
        x = _cross(up, z)
        xn = math.sqrt(sum(c * c for c in x)) or 1.0
        x = [c / xn for c in x]
        y = _cross(z, x)
        m = [[x[0], y[0], z[0]], [x[1], y[1], z[1]], [x[2], y[2], z[2]]]
        _set_rot(self.props["rotation"], (m))
        return self

    js_methods = {
        "add": lambda s, i, x: s.add(x),
        "remove": lambda s, i, x: (s.children().__setitem__(slice(None), [c for c in s.children() if all(c is not o for o in x)]), s)[-1],
        "clear": lambda s, i, x: (s.children().clear(), s)[-1],
        "rotateX": lambda s, i, x: s.rotate_local("x", _num_arg(x, 0)),
        "rotateY": lambda s, i, x: s.rotate_local("y", _num_arg(x, 0)),
        "rotateZ": lambda s, i, x: s.rotate_local("z", _num_arg(x, 0)),
        # world axis: the rotation composes on the left (the object turns about a world-space axis through its
        # own origin; its position is unchanged)
        "rotateOnWorldAxis": lambda s, i, x: (_set_rot(s.props["rotation"], (_mat_mul(
            _axis_mat(_arg(x, 0).v(), _num_arg(x, 1)), _rot_mat(s.props["rotation"])))), s)[-1],
        "rotateOnAxis": lambda s, i, x: (_set_rot(s.props["rotation"], (_mat_mul(_rot_mat(s.props["rotation"]),
                                                                                         _axis_mat(_arg(x, 0).v(), _num_arg(x, 1))))), s)[-1],
        "translateX": lambda s, i, x: (s.props["position"].setv(_add3(s.props["position"].v(), _mat3_apply(_rot_mat(s.props["rotation"]), [_num_arg(x, 0), 0, 0]))), s)[-1],
        "translateY": lambda s, i, x: (s.props["position"].setv(_add3(s.props["position"].v(), _mat3_apply(_rot_mat(s.props["rotation"]), [0, _num_arg(x, 0), 0]))), s)[-1],
        "translateZ": lambda s, i, x: (s.props["position"].setv(_add3(s.props["position"].v(), _mat3_apply(_rot_mat(s.props["rotation"]), [0, 0, _num_arg(x, 0)]))), s)[-1],
        "lookAt": lambda s, i, x: s.look_at(_arg(x, 0).v() if isinstance(_arg(x, 0), Vec) else [_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2)]),
        "updateMatrix": lambda s, i, x: (setattr(s.props["matrix"], "m", s.composed()), UNDEF)[-1],
        "updateMatrixWorld": lambda s, i, x: UNDEF,
        "traverse": lambda s, i, x: (_traverse(i, s, _arg(x, 0)), UNDEF)[-1],
        "clone": lambda s, i, x: _obj_clone(i, s),
        "copy": lambda s, i, x: _copy_obj(i, s, _arg(x, 0), _arg(x, 1) is UNDEF or _truthy(_arg(x, 1)))
        if isinstance(_arg(x, 0), Object3D) else s,
        "getObjectByName": lambda s, i, x: _find_name(s, _to_str(_arg(x, 0))),
        "setMatrixAt": lambda s, i, x: (s.props.setdefault("__inst", {}).__setitem__(int(_num_arg(x, 0)), [row[:] for row in _arg(x, 1).m]), UNDEF)[-1],
        "setColorAt": lambda s, i, x: _set_color_at(s, int(_num_arg(x, 0)), _arg(x, 1)),
        "getColorAt": lambda s, i, x: (_arg(x, 1).set_rgb(*s.props.get("__icol", {}).get(int(_num_arg(x, 0)), (1.0, 1.0, 1.0)))
                                       if isinstance(_arg(x, 1), Color) else None, UNDEF)[-1],
        "getMatrixAt": lambda s, i, x: (setattr(_arg(x, 1), "m", [row[:] for row in s.props.get("__inst", {}).get(int(_num_arg(x, 0)), _ident4())]), UNDEF)[-1],
        "applyMatrix4": lambda s, i, x: _apply_obj_matrix(s, _arg(x, 0).m),
        "applyQuaternion": lambda s, i, x: (_set_rot(s.props["rotation"], (_mat_mul(
            _arg(x, 0).cur(), _rot_mat(s.props["rotation"])))), s)[-1],
        "setRotationFromEuler": lambda s, i, x: (s.props["rotation"].setv(_arg(x, 0).v()), s.props["rotation"].props.__setitem__(
            "order", _order(_arg(x, 0))), UNDEF)[-1],
        "setRotationFromQuaternion": lambda s, i, x: (_set_rot(s.props["rotation"], (_arg(x, 0).cur())), UNDEF)[-1],
        "setRotationFromMatrix": lambda s, i, x: (_set_rot(s.props["rotation"], (_rot_part(_arg(x, 0).m))), UNDEF)[-1],
        "setRotationFromAxisAngle": lambda s, i, x: (_set_rot(s.props["rotation"], (_axis_mat(
            _arg(x, 0).v(), _num_arg(x, 1)))), UNDEF)[-1],
        "getWorldPosition": lambda s, i, x: _target_vec(x).setv([_world4(s)[r][3] for r in range(3)]),
        "getWorldScale": lambda s, i, x: _target_vec(x).setv([math.sqrt(sum(_world4(s)[r][c] ** 2 for r in range(3)))
                                                              for c in range(3)]),
        "getWorldQuaternion": lambda s, i, x: (_arg(x, 0) if isinstance(_arg(x, 0), Quaternion) else Quaternion()).put(
            _rot_part(_world4(s))),
        "getWorldDirection": lambda s, i, x: _target_vec(x).setv(_unit([_world4(s)[r][2] for r in range(3)])),
        "localToWorld": lambda s, i, x: _arg(x, 0).setv(_mat4_point(_world4(s), _arg(x, 0).v())),
        "worldToLocal": lambda s, i, x: _arg(x, 0).setv(_mat4_point(_inv4(_world4(s)), _arg(x, 0).v())),
        "attach": lambda s, i, x: _attach(s, _arg(x, 0)),
        "removeFromParent": lambda s, i, x: _remove_from_parent(s),
        "getObjectById": lambda s, i, x: UNDEF,
        "computeBoundingSphere": lambda s, i, x: UNDEF,
        "computeBoundingBox": lambda s, i, x: UNDEF,
    }


def _set_color_at(o: "Object3D", k: int, c):
    """InstancedMesh.setColorAt: the instance's colour (linear), which multiplies the material colour; the first
    call creates `instanceColor`, as three.js does, so `instanceColor.needsUpdate = true` works after it."""
    if isinstance(c, Color) and 0 <= k < max(0, int(_to_num(o.props.get("count", 0)))):
        o.props.setdefault("__icol", {})[k] = tuple(c.rgb())
        if not isinstance(o.props.get("instanceColor"), JSObject):
            o.props["instanceColor"] = JSObject({"needsUpdate": False, "isInstancedBufferAttribute": True})
    return UNDEF


def _add3(a, b):
    return [p + q for p, q in zip(a, b)]


def _target_vec(x):
    t = _arg(x, 0)
    return t if isinstance(t, Vec) else Vec(("x", "y", "z"), [0.0, 0.0, 0.0], "Vector3")


def _world4(o: "Object3D"):
    m = o.local()
    p = o.props.get("parent")
    depth = 0
    while isinstance(p, Object3D) and depth < 64:
        m = _mat_mul(p.local(), m)
        p = p.props.get("parent")
        depth += 1
    return m


def _remove_from_parent(o: "Object3D"):
    p = o.props.get("parent")
    if isinstance(p, Object3D):
        kids = p.children()
        kids[:] = [c for c in kids if c is not o]
    o.props["parent"] = None
    return o


def _attach(new_parent: "Object3D", o):
    """Reparent `o` under `new_parent` keeping its world transform."""
    if not isinstance(o, Object3D):
        return new_parent
    local = _mat_mul(_inv4(_world4(new_parent)), _world4(o))
    _remove_from_parent(o)
    new_parent.add([o])
    sx, sy, sz = (math.sqrt(sum(local[r][c] ** 2 for r in range(3))) or 1.0 for c in range(3))
    o.props["position"].setv([local[0][3], local[1][3], local[2][3]])
    o.props["scale"].setv([sx, sy, sz])
    _set_rot(o.props["rotation"], ([[local[r][c] / (sx, sy, sz)[c] for c in range(3)] for r in range(3)]))
    return new_parent


def _apply_obj_matrix(o: Object3D, m):
    full = _mat_mul(m, o.local())
    pos = [full[0][3], full[1][3], full[2][3]]
    sc = [math.sqrt(sum(full[r][c] ** 2 for r in range(3))) for c in range(3)]
    rot = [[full[r][c] / (sc[c] or 1.0) for c in range(3)] for r in range(3)]
    o.props["position"].setv(pos)
    o.props["scale"].setv(sc)
    _set_rot(o.props["rotation"], (rot))
    return o


def _traverse(it, o, f):
    it.call(f, UNDEF, [o])
    for c in list(o.children()):
        _traverse(it, c, f)


def _find_name(o, name):
    if o.props.get("name") == name:
        return o
    for c in o.children():
        r = _find_name(c, name)
        if r is not UNDEF:
            return r
    return UNDEF


def _copy_obj(it, n: Object3D, o: Object3D, recursive: bool = True) -> Object3D:
    """Object3D.copy: n takes o's transform (rotation order included), name, flags, a deep copy of userData and
    (recursive) clones of o's children; geometry and material are shared, as three.js shares them."""
    for k, v in o.props.items():
        if k in ("children", "parent", "matrix"):
            continue
        if k in ("position", "rotation", "scale"):
            n.props[k].setv(v.v())
            if k == "rotation":
                n.props[k].props["order"] = _order(v)
        elif k == "userData":
            n.props[k] = _user_data_copy(it, v)
        elif k == "__inst":
            n.props[k] = {i: [row[:] for row in m] for i, m in v.items()}
        else:
            n.props[k] = v
    if recursive:
        for c in o.children():
            n.add([_obj_clone(it, c)])
    return n


def _user_data_copy(it, v):
    """three.js copies userData through JSON; data JSON cannot hold (a cycle, e.g. a stored object) is copied
    shallowly instead of throwing."""
    if not isinstance(v, JSObject):
        return v
    try:
        text = _json_stringify(it, v, None)
        return _json_parse(text) if isinstance(text, str) else JSObject()
    except _Throw:
        return JSObject(dict(v.props))


def _obj_clone(it, o: Object3D) -> Object3D:
    return _copy_obj(it, Object3D(o.otype, o.props.get("geometry"), o.props.get("material")), o)


class Shape(Host):
    """Shape / Path: a list of segments (points from moveTo / lineTo, quadratic and cubic Beziers, arcs and
    ellipses, splines, closePath) sampled as three.js's CurvePath.getPoints(divisions) samples them: each curve at
    `divisions` steps (ellipses and arcs at twice that, splines at that times their point count), a point equal to
    the one before it skipped. getPoints() and the shape geometries use 12 (ExtrudeGeometry's and ShapeGeometry's
    curveSegments when given)."""
    __slots__ = ("segs", "holes_")
    cls_name = "Shape"

    def __init__(self, pts=None):
        super().__init__({})
        self.segs: List[Tuple[str, Any]] = [("pt", list(p.v()[:2])) for p in pts] if pts else []
        self.holes_: List["Shape"] = []

    def get_special(self, it, key):
        if key == "holes":
            return _HolesProxy(self)
        if key == "currentPoint":
            return Vec(("x", "y"), self.current(), "Vector2")
        return super().get_special(it, key)

    @property
    def pts(self) -> List[List[float]]:
        return self.sample(12)

    def current(self) -> List[float]:
        out = self.sample(1)
        return out[-1] if out else [0.0, 0.0]

    def sample(self, n: int) -> List[List[float]]:
        n = max(1, min(int(n), 256))
        out: List[List[float]] = []

        def push(p):
            p = [float(p[0]), float(p[1])]
            if not out or out[-1] != p:
                out.append(p)
        for kind, d in self.segs:
            sx, sy = out[-1] if out else (0.0, 0.0)
            if kind == "pt":
                push(d)
            elif kind == "quad":
                cx, cy, ex, ey = d
                for k in range(0 if not out else 1, n + 1):
                    t = k / n
                    push([(1 - t) ** 2 * sx + 2 * (1 - t) * t * cx + t * t * ex,
                          (1 - t) ** 2 * sy + 2 * (1 - t) * t * cy + t * t * ey])
            elif kind == "bez":
                c1x, c1y, c2x, c2y, ex, ey = d
                for k in range(0 if not out else 1, n + 1):
                    t = k / n
                    u = 1 - t
                    push([u ** 3 * sx + 3 * u * u * t * c1x + 3 * u * t * t * c2x + t ** 3 * ex,
                          u ** 3 * sy + 3 * u * u * t * c1y + 3 * u * t * t * c2y + t ** 3 * ey])
            elif kind == "ell":
                for k in range(2 * n + 1):
                    push(_ellipse_point(d, k / (2 * n)))
            elif kind == "spline":
                pts = ([[sx, sy]] if out else []) + d
                if len(pts) >= 2:
                    c = Curve("catmull", pts, dim=2)
                    m = n * len(pts)
                    for k in range(0 if not out else 1, m + 1):
                        push(c.point(k / m))
            elif kind == "close" and len(out) > 1 and out[-1] != out[0]:
                out.append(list(out[0]))
        return out

    def _quad(self, x):
        self.segs.append(("quad", tuple(_num_arg(x, k) for k in range(4))))
        return self

    def _bez(self, x):
        self.segs.append(("bez", tuple(_num_arg(x, k) for k in range(6))))
        return self

    def _arc(self, x, absolute):
        cx, cy, r, a0, a1 = (_num_arg(x, k) for k in range(5))
        if not absolute:
            px, py = self.current()
            cx, cy = cx + px, cy + py
        self.segs.append(("ell", {"aX": cx, "aY": cy, "xRadius": r, "yRadius": r, "aStartAngle": a0,
                                  "aEndAngle": a1, "aClockwise": _truthy(_arg(x, 5, False)), "aRotation": 0.0}))
        return self

    def _ellipse(self, x, absolute):
        """absellipse / ellipse(aX, aY, xRadius, yRadius, aStartAngle, aEndAngle, aClockwise, aRotation)."""
        names = ("aX", "aY", "xRadius", "yRadius", "aStartAngle", "aEndAngle", "aClockwise", "aRotation")
        defaults = (0.0, 0.0, 1.0, 1.0, 0.0, 2 * math.pi, False, 0.0)
        p = {}
        for k, (nm, d) in enumerate(zip(names, defaults)):
            v = _arg(x, k)
            p[nm] = d if v is UNDEF else (_truthy(v) if nm == "aClockwise" else _to_num(v))
        if not absolute:
            px, py = self.current()
            p["aX"] += px
            p["aY"] += py
        self.segs.append(("ell", p))
        return self

    def _spline(self, x):
        self.segs.append(("spline", [q.v()[:2] for q in it_items(_arg(x, 0)) if isinstance(q, Vec)]))
        return self

    def _vecs(self, x, key_index=0):
        n = _arg(x, key_index)
        return JSArray([Vec(("x", "y"), p, "Vector2") for p in self.sample(12 if n is UNDEF else _to_num(n))])

    js_methods = {
        "absellipse": lambda s, i, x: s._ellipse(x, True),
        "ellipse": lambda s, i, x: s._ellipse(x, False),
        "splineThru": lambda s, i, x: s._spline(x),
        "getSpacedPoints": lambda s, i, x: s._vecs(x),
        "extractPoints": lambda s, i, x: (lambda n: JSObject({
            "shape": JSArray([Vec(("x", "y"), p, "Vector2") for p in s.sample(n)]),
            "holes": JSArray([JSArray([Vec(("x", "y"), p, "Vector2") for p in h.sample(n)]) for h in s.holes_])}))(
            12 if _arg(x, 0) is UNDEF else _to_num(_arg(x, 0))),
        "moveTo": lambda s, i, x: (s.segs.append(("pt", [_num_arg(x, 0), _num_arg(x, 1)])), s)[-1],
        "lineTo": lambda s, i, x: (s.segs.append(("pt", [_num_arg(x, 0), _num_arg(x, 1)])), s)[-1],
        "quadraticCurveTo": lambda s, i, x: s._quad(x),
        "bezierCurveTo": lambda s, i, x: s._bez(x),
        "absarc": lambda s, i, x: s._arc(x, True),
        "arc": lambda s, i, x: s._arc(x, False),
        "closePath": lambda s, i, x: (s.segs.append(("close", None)), s)[-1],
        "getPoints": lambda s, i, x: s._vecs(x),
        "setFromPoints": lambda s, i, x: (setattr(s, "segs", [("pt", list(p.v()[:2])) for p in it_items(_arg(x, 0))]),
                                          s)[-1],
    }


class _HolesProxy(Host):
    __slots__ = ("shape",)

    def __init__(self, shape):
        super().__init__({})
        self.shape = shape

    def get_special(self, it, key):
        if key == "length":
            return float(len(self.shape.holes_))
        k = _index(key)
        if k is not None:
            return self.shape.holes_[k] if k < len(self.shape.holes_) else UNDEF
        return super().get_special(it, key)

    def iterable(self):
        return list(self.shape.holes_)

    js_methods = {"push": lambda s, i, x: (s.shape.holes_.extend(v for v in x if isinstance(v, Shape)),
                                           float(len(s.shape.holes_)))[-1]}


class Curve(Host):
    """getPoint(t), t in [0, 1], of the curve classes: 3D CatmullRomCurve3 / LineCurve3 / QuadraticBezierCurve3 /
    CubicBezierCurve3; 2D EllipseCurve / ArcCurve / LineCurve / SplineCurve / QuadraticBezierCurve /
    CubicBezierCurve (same formulas on two components); "custom" = THREE.Curve subclassed by the module (its own
    getPoint is called); "path" = CurvePath (its curves in sequence, equal shares of t); "poly" = points sampled
    from a custom curve (piecewise linear)."""
    __slots__ = ("kind_", "ctrl", "closed", "dim", "interp", "params")
    cls_name = "Curve"

    def __init__(self, kind, ctrl, closed=False, dim=3, interp=None, params=None):
        super().__init__({})
        self.kind_, self.ctrl, self.closed, self.dim, self.interp = kind, ctrl, closed, dim, interp
        self.params = params or {}
        if kind == "path":
            self.props["curves"] = JSArray(list(ctrl))

    def vec(self, p):
        return Vec(("x", "y", "z")[:self.dim], list(p)[:self.dim], "Vector3" if self.dim == 3 else "Vector2")

    def point(self, t):
        c = self.ctrl
        if self.kind_ == "custom":
            f = self.interp.get(self, "getPoint") if self.interp is not None else UNDEF
            if not isinstance(f, (JSFunction, Native)) or isinstance(f, Native) and f.name == "getPoint":
                raise _Throw(_error_obj("TypeError", "THREE.Curve subclass must implement getPoint(t)"))
            r = self.interp.call(f, self, [float(t), self.vec([0.0] * self.dim)])
            if not isinstance(r, Vec):
                raise _Throw(_error_obj("TypeError", "getPoint must return a vector"))
            return r.v()
        if self.kind_ == "path":
            curves = [k for k in it_items(self.props.get("curves")) if isinstance(k, Curve)]
            if not curves:
                return [0.0] * self.dim
            f = min(max(t, 0.0), 1.0) * len(curves)
            k = min(int(f), len(curves) - 1)
            return curves[k].point(f - k)
        if self.kind_ == "poly":
            n = len(c) - 1
            f = min(max(t, 0.0), 1.0) * n
            k = min(int(f), max(n - 1, 0))
            w = f - k
            return [a + (b - a) * w for a, b in zip(c[k], c[min(k + 1, n)])]
        if self.kind_ == "ellipse":
            return _ellipse_point(self.params, t)
        if self.kind_ == "line":
            return [a + (b - a) * t for a, b in zip(c[0], c[1])]
        if self.kind_ == "quad":
            u = 1 - t
            return [u * u * a + 2 * u * t * b + t * t * d for a, b, d in zip(*c)]
        if self.kind_ == "cubic":
            u = 1 - t
            return [u ** 3 * a + 3 * u * u * t * b + 3 * u * t * t * d + t ** 3 * e for a, b, d, e in zip(*c)]
        # centripetal-free uniform Catmull-Rom through the control points
        n = len(c)
        if n == 1:
            return list(c[0])
        segs = n if self.closed else n - 1
        f = t * segs
        k = min(int(f), segs - 1)
        w = f - k

        def P(j):
            return c[j % n] if self.closed else c[max(0, min(n - 1, j))]
        p0, p1, p2, p3 = P(k - 1), P(k), P(k + 1), P(k + 2)
        return [0.5 * (2 * b + (-a + d) * w + (2 * a - 5 * b + 4 * d - e) * w * w + (-a + 3 * b - 3 * d + e) * w ** 3)
                for a, b, d, e in zip(p0, p1, p2, p3)]

    def points(self, n):
        n = max(1, min(int(n), 4096))
        return JSArray([self.vec(self.point(k / n)) for k in range(n + 1)])

    def arc_table(self, n=200):
        """Cumulative chord lengths at t = k / n (three.js's arcLengthDivisions = 200)."""
        pts = [self.point(k / n) for k in range(n + 1)]
        acc = [0.0]
        for a, b in zip(pts, pts[1:]):
            acc.append(acc[-1] + math.sqrt(sum((p - q) ** 2 for p, q in zip(a, b))))
        return acc

    def u_to_t(self, u, acc=None):
        """three.js's getUtoTmapping: the t at which the arc length is u of the whole."""
        acc = acc or self.arc_table()
        n = len(acc) - 1
        total = acc[-1]
        if total <= 0:
            return u
        target = min(max(u, 0.0), 1.0) * total
        lo, hi = 0, n
        while lo < hi:                                  # first sample whose length reaches the target
            mid = (lo + hi) // 2
            if acc[mid] < target:
                lo = mid + 1
            else:
                hi = mid
        if acc[lo] == target or lo == 0:
            return lo / n
        seg = acc[lo] - acc[lo - 1]
        return (lo - 1 + ((target - acc[lo - 1]) / seg if seg > 0 else 0.0)) / n

    def tangent(self, t):
        """three.js's Curve.getTangent: the normalised difference of the points 1e-4 either side (clamped)."""
        a, b = self.point(max(0.0, t - 1e-4)), self.point(min(1.0, t + 1e-4))
        d = [q - p for p, q in zip(a, b)]
        n = math.sqrt(sum(c * c for c in d)) or 1.0
        return self.vec([c / n for c in d])

    js_methods = {
        "getPoint": lambda s, i, x: s.vec(s.point(_num_arg(x, 0))),
        "getPointAt": lambda s, i, x: s.vec(s.point(s.u_to_t(_num_arg(x, 0)))),
        "getPoints": lambda s, i, x: s.points(_num_arg(x, 0, 12.0 if s.kind_ == "path" else 5.0)),
        "getSpacedPoints": lambda s, i, x: (lambda n, tab: JSArray([s.vec(s.point(s.u_to_t(k / n, tab)))
                                                                    for k in range(n + 1)]))(
            max(1, min(int(_num_arg(x, 0, 5.0)), 4096)), s.arc_table()),
        "getTangent": lambda s, i, x: s.tangent(_num_arg(x, 0)),
        "getTangentAt": lambda s, i, x: s.tangent(s.u_to_t(_num_arg(x, 0))),
        "getUtoTmapping": lambda s, i, x: s.u_to_t(_num_arg(x, 0)),
        "getLength": lambda s, i, x: _curve_length(s),
        "add": lambda s, i, x: (s.props["curves"].items.append(_arg(x, 0)), UNDEF)[-1] if s.kind_ == "path" else UNDEF,
    }


def _ellipse_point(p, t):
    """A point of an ellipse arc (centre, radii, start / end angle, direction, rotation about the centre)."""
    cx, cy, rx, ry = p["aX"], p["aY"], p["xRadius"], p["yRadius"]
    a0, a1, cw, rot = p["aStartAngle"], p["aEndAngle"], p["aClockwise"], p["aRotation"]
    two_pi = 2 * math.pi
    delta = a1 - a0
    same = abs(delta) < 1e-12
    while delta < 0:
        delta += two_pi
    while delta > two_pi:
        delta -= two_pi
    if delta < 1e-12:
        delta = 0.0 if same else two_pi
    if cw and not same:
        delta = -two_pi if delta == two_pi else delta - two_pi
    ang = a0 + t * delta
    x, y = cx + rx * math.cos(ang), cy + ry * math.sin(ang)
    if rot:
        c, s_ = math.cos(rot), math.sin(rot)
        dx, dy = x - cx, y - cy
        x, y = dx * c - dy * s_ + cx, dx * s_ + dy * c + cy
    return [x, y]


def _curve_length(c: "Curve", n: int = 200) -> float:
    pts = [c.point(k / n) for k in range(n + 1)]
    return sum(math.sqrt(sum((a - b) ** 2 for a, b in zip(p, q))) for p, q in zip(pts, pts[1:]))


def _ctor(cls_name, build):
    return Native(cls_name, ctor=lambda it, x: build(it, x))


def _geom_ctor(gtype):
    names = _GEOM_PARAMS[gtype]
    defaults = _GEOM_DEFAULTS[gtype]

    def build(it, x):
        params = {}
        for k, nm in enumerate(names):
            v = _arg(x, k)
            params[nm] = defaults[k] if v is UNDEF else (_to_num(v) if isinstance(v, (int, float, bool)) and not isinstance(v, bool) else v)
        path = params.get("path")
        if gtype == "TubeGeometry" and isinstance(path, Curve) and path.kind_ in ("custom", "path"):
            n = max(1, min(int(_to_num(params.get("tubularSegments") or 64)), 256))
            pts = [list(path.point(k / n)) + [0.0] * (3 - path.dim) for k in range(n + 1)]
            params["path"] = Curve("poly", pts)
        return Geometry(gtype, params)
    return Native(gtype, ctor=build)


def world_bbox(root: "Object3D", precise: bool = False):
    """World-space (min, max) of every object with a geometry under `root` (its own transform included), or None,
    by three.js's Box3.setFromObject: each geometry's bounding box (all of its positions) has its eight corners
    moved by the object's world matrix (so a rotated object contributes the box around its rotated box, not around
    its vertices); an InstancedMesh contributes its instances' boxes. `precise` uses every vertex instead
    (setFromObject(object, true); instanced meshes stay boxes). Invisible objects count, as in three.js."""
    import numpy as np
    lo, hi = np.full(3, np.inf), np.full(3, -np.inf)
    corners = np.array([[x, y, z, 1.0] for x in (0, 1) for y in (0, 1) for z in (0, 1)])

    def box_points(bmin, bmax, m):
        pts = np.where(corners[:, :3] > 0, bmax, bmin)
        return pts @ m[:3, :3].T + m[:3, 3]

    def walk(o, parent, depth):
        w = parent @ np.asarray(o.local(), dtype=np.float64)
        g = o.props.get("geometry")
        if isinstance(g, Geometry):
            v = geometry_mesh(g)[0].double().numpy()
            if len(v):
                if o.otype == "InstancedMesh":
                    gmin, gmax = v.min(0), v.max(0)
                    inst = o.props.get("__inst", {})
                    n = max(0, int(_to_num(o.props.get("count", 0))))
                    mats = [np.asarray(inst.get(k, _ident4()), dtype=np.float64) for k in range(min(n, 1 << 16))]
                    if mats:
                        ip = np.concatenate([box_points(gmin, gmax, mk) for mk in mats])
                        p = box_points(ip.min(0), ip.max(0), w)
                    else:
                        p = np.zeros((0, 3))
                elif precise:
                    p = v @ w[:3, :3].T + w[:3, 3]
                else:
                    p = box_points(v.min(0), v.max(0), w)
                if len(p):
                    lo[:] = np.minimum(lo, p.min(0))
                    hi[:] = np.maximum(hi, p.max(0))
        if depth < 64:
            for c in o.children():
                walk(c, w, depth + 1)
    walk(root, np.eye(4), 0)
    return None if not (np.isfinite(lo).all() and np.isfinite(hi).all()) else (lo.tolist(), hi.tolist())


class Box3(Host):
    """THREE.Box3 subset: setFromObject (world bounds of an object's meshes), getCenter, getSize, isEmpty."""
    cls_name = "Box3"

    def __init__(self):
        super().__init__({"min": Vec(("x", "y", "z"), [math.inf] * 3, "Vector3"),
                          "max": Vec(("x", "y", "z"), [-math.inf] * 3, "Vector3"), "isBox3": True})

    def set_from(self, o, precise=False):
        bb = world_bbox(o, precise) if isinstance(o, Object3D) else None
        self.props["min"].setv(bb[0] if bb else [math.inf] * 3)
        self.props["max"].setv(bb[1] if bb else [-math.inf] * 3)
        return self

    def empty(self):
        return any(a > b for a, b in zip(self.props["min"].v(), self.props["max"].v()))

    def expand(self, p):
        lo, hi = self.props["min"], self.props["max"]
        lo.setv([min(a, b) for a, b in zip(lo.v(), p)])
        hi.setv([max(a, b) for a, b in zip(hi.v(), p)])
        return self

    def set_pts(self, pts):
        self.props["min"].setv([math.inf] * 3)
        self.props["max"].setv([-math.inf] * 3)
        for q in pts:
            self.expand(q.v()[:3])
        return self

    def copy_from(self, o):
        self.props["min"].setv(o.props["min"].v())
        self.props["max"].setv(o.props["max"].v())
        return self

    js_methods = {
        "setFromObject": lambda s, i, x: s.set_from(_arg(x, 0), _truthy(_arg(x, 1, False))),
        "setFromPoints": lambda s, i, x: s.set_pts(it_items(_arg(x, 0))),
        "set": lambda s, i, x: (s.props["min"].setv(_arg(x, 0).v()), s.props["max"].setv(_arg(x, 1).v()), s)[-1],
        "expandByPoint": lambda s, i, x: s.expand(_arg(x, 0).v()),
        "expandByScalar": lambda s, i, x: (s.props["min"].setv([a - _num_arg(x, 0) for a in s.props["min"].v()]),
                                           s.props["max"].setv([a + _num_arg(x, 0) for a in s.props["max"].v()]), s)[-1],
        "expandByObject": lambda s, i, x: (lambda b: s if b.empty() else s.expand(b.props["min"].v()).expand(
            b.props["max"].v()))(Box3().set_from(_arg(x, 0), _truthy(_arg(x, 1, False)))),
        "union": lambda s, i, x: s.expand(_arg(x, 0).props["min"].v()).expand(_arg(x, 0).props["max"].v()),
        "containsPoint": lambda s, i, x: all(a <= p <= b for a, p, b in zip(s.props["min"].v(), _arg(x, 0).v(),
                                                                             s.props["max"].v())),
        "makeEmpty": lambda s, i, x: s.set_pts([]),
        "clone": lambda s, i, x: Box3().copy_from(s),
        "copy": lambda s, i, x: s.copy_from(_arg(x, 0)),
        "isEmpty": lambda s, i, x: s.empty(),
        "getCenter": lambda s, i, x: _arg(x, 0).setv([0.0] * 3 if s.empty() else
                                                     [(a + b) / 2 for a, b in zip(s.props["min"].v(), s.props["max"].v())]),
        "getSize": lambda s, i, x: _arg(x, 0).setv([0.0] * 3 if s.empty() else
                                                   [b - a for a, b in zip(s.props["min"].v(), s.props["max"].v())]),
    }


def _buffer_attribute(it, x, kind):
    """new BufferAttribute(typedArray, itemSize) keeps the module's typed array and rejects a plain array, as
    three.js does; new Float32BufferAttribute(arrayOrLength, itemSize) (and the other typed kinds) copies into a
    fresh typed array of its kind."""
    src, item = _arg(x, 0), _num_arg(x, 1, 3.0)
    if kind is None:
        if not isinstance(src, TypedArray):
            raise _Throw(_error_obj("TypeError", "THREE.BufferAttribute: array should be a Typed Array."))
        return BufferAttribute(src, item)
    return BufferAttribute(_typed_from(it, kind, src), item)


def _vec_ctor(name, comps):
    def make(it, x):
        v = Vec(comps, [_num_arg(x, k) for k in range(len(comps))], name)
        if name == "Euler" and isinstance(_arg(x, 3), str) and _arg(x, 3) in _ORDERS:
            v.props["order"] = _arg(x, 3)               # new Euler(x, y, z, order)
        return v
    return Native(name, ctor=make)


def make_three(it: Interp) -> JSObject:
    mats = ("MeshStandardMaterial", "MeshPhysicalMaterial", "MeshBasicMaterial", "MeshLambertMaterial",
            "MeshPhongMaterial", "MeshToonMaterial", "MeshNormalMaterial", "MeshMatcapMaterial",
            "LineBasicMaterial", "LineDashedMaterial", "PointsMaterial", "SpriteMaterial")
    three: Dict[str, Any] = {}
    for g in _GEOM_PARAMS:
        three[g] = _geom_ctor(g)
    three["BufferGeometry"] = Native("BufferGeometry", ctor=lambda i, x: Geometry())
    for m in mats:
        three[m] = Native(m, ctor=lambda i, x, _m=m: Material(_m, _arg(x, 0) if x else None))
    three["BufferAttribute"] = Native("BufferAttribute", ctor=lambda i, x: _buffer_attribute(i, x, None))
    for cls in ("Float32BufferAttribute", "Uint16BufferAttribute", "Uint32BufferAttribute", "Int32BufferAttribute",
                "Uint8BufferAttribute", "Int8BufferAttribute", "Int16BufferAttribute"):
        three[cls] = Native(cls, ctor=lambda i, x, _k=cls.replace("BufferAttribute", "Array"): _buffer_attribute(i, x, _k))
    three["Group"] = Native("Group", ctor=lambda i, x: Object3D("Group"))
    three["Box3"] = Native("Box3", ctor=lambda i, x: Box3())
    three["Object3D"] = Native("Object3D", ctor=lambda i, x: Object3D("Object3D"))
    three["Scene"] = Native("Scene", ctor=lambda i, x: Object3D("Group"))
    for t in ("Mesh", "LineSegments", "Line", "LineLoop", "Points", "Sprite"):
        three[t] = Native(t, ctor=lambda i, x, _t=t: Object3D(_t, _arg(x, 0) if x else Geometry(),
                                                               _arg(x, 1) if len(x) > 1 else Material("MeshBasicMaterial")))
    three["InstancedMesh"] = Native("InstancedMesh", ctor=lambda i, x: _instanced(x))
    three["Vector2"] = _vec_ctor("Vector2", ("x", "y"))
    three["Vector3"] = _vec_ctor("Vector3", ("x", "y", "z"))
    three["Euler"] = _vec_ctor("Euler", ("x", "y", "z"))
    three["Matrix4"] = Native("Matrix4", ctor=lambda i, x: Matrix4())
    three["Quaternion"] = Native("Quaternion", ctor=lambda i, x: Quaternion())
    three["Color"] = Native("Color", ctor=lambda i, x: Color().set_any(x) if x else Color())
    three["Shape"] = Native("Shape", ctor=lambda i, x: Shape(it_items(_arg(x, 0)) if x else None))
    three["Path"] = Native("Path", ctor=lambda i, x: Shape(it_items(_arg(x, 0)) if x else None))
    three["CatmullRomCurve3"] = Native("CatmullRomCurve3", ctor=lambda i, x: Curve(
        "catmull", [p.v() for p in it_items(_arg(x, 0))], _truthy(_arg(x, 1, False))))
    three["LineCurve3"] = Native("LineCurve3", ctor=lambda i, x: Curve("line", [_arg(x, 0).v(), _arg(x, 1).v()]))
    three["QuadraticBezierCurve3"] = Native("QuadraticBezierCurve3", ctor=lambda i, x: Curve(
        "quad", [_arg(x, k).v() for k in range(3)]))
    three["CubicBezierCurve3"] = Native("CubicBezierCurve3", ctor=lambda i, x: Curve(
        "cubic", [_arg(x, k).v() for k in range(4)]))
    for t in ("Texture", "CanvasTexture"):
        three[t] = Native(t, ctor=lambda i, x: Texture())
    three["DataTexture"] = Native("DataTexture", ctor=lambda i, x: _data_texture(x))
    _install_spec_members(it, three)
    for name, val in THREE_CONSTANTS.items():
        three[name] = val
    rnd = it.random
    three["MathUtils"] = JSObject({
        "degToRad": _nat("degToRad", lambda i, t, x: _num_arg(x, 0) * math.pi / 180),
        "radToDeg": _nat("radToDeg", lambda i, t, x: _num_arg(x, 0) * 180 / math.pi),
        "clamp": _nat("clamp", lambda i, t, x: max(_num_arg(x, 1), min(_num_arg(x, 2), _num_arg(x, 0)))),
        "lerp": _nat("lerp", lambda i, t, x: _num_arg(x, 0) + (_num_arg(x, 1) - _num_arg(x, 0)) * _num_arg(x, 2)),
        "mapLinear": _nat("mapLinear", lambda i, t, x: _num_arg(x, 3) + (_num_arg(x, 0) - _num_arg(x, 1)) *
                          (_num_arg(x, 4) - _num_arg(x, 3)) / ((_num_arg(x, 2) - _num_arg(x, 1)) or 1.0)),
        "smoothstep": _nat("smoothstep", lambda i, t, x: _smoothstep(_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2))),
        "randFloat": _nat("randFloat", lambda i, t, x: _num_arg(x, 0) + rnd() * (_num_arg(x, 1) - _num_arg(x, 0))),
        "randFloatSpread": _nat("randFloatSpread", lambda i, t, x: _num_arg(x, 0) * (0.5 - rnd())),
        "randInt": _nat("randInt", lambda i, t, x: float(math.floor(_num_arg(x, 0) + rnd() * (_num_arg(x, 1) - _num_arg(x, 0) + 1)))),
        "seededRandom": _nat("seededRandom", lambda i, t, x: rnd()),
        "euclideanModulo": _nat("euclideanModulo", lambda i, t, x: (_num_arg(x, 0) % _num_arg(x, 1)) if _num_arg(x, 1) else math.nan),
        "inverseLerp": _nat("inverseLerp", lambda i, t, x: ((_num_arg(x, 2) - _num_arg(x, 0)) / (_num_arg(x, 1) - _num_arg(x, 0)))
                            if _num_arg(x, 0) != _num_arg(x, 1) else 0.0),
        "damp": _nat("damp", lambda i, t, x: _num_arg(x, 0) + (_num_arg(x, 1) - _num_arg(x, 0)) *
                     (1 - math.exp(-_num_arg(x, 2) * _num_arg(x, 3)))),
        "pingpong": _nat("pingpong", lambda i, t, x: _num_arg(x, 1, 1.0) - abs(
            (_num_arg(x, 0) % (2 * _num_arg(x, 1, 1.0))) - _num_arg(x, 1, 1.0))),
        "smootherstep": _nat("smootherstep", lambda i, t, x: (lambda u: u * u * u * (u * (u * 6 - 15) + 10))(
            min(1.0, max(0.0, (_num_arg(x, 0) - _num_arg(x, 1)) / ((_num_arg(x, 2) - _num_arg(x, 1)) or 1.0))))),
        "isPowerOfTwo": _nat("isPowerOfTwo", lambda i, t, x: (lambda v: v > 0 and v == int(v) and (int(v) & (int(v) - 1)) == 0)(
            _num_arg(x, 0))),
        "ceilPowerOfTwo": _nat("ceilPowerOfTwo", lambda i, t, x: float(2 ** math.ceil(math.log2(max(_num_arg(x, 0), 1e-300))))),
        "floorPowerOfTwo": _nat("floorPowerOfTwo", lambda i, t, x: float(2 ** math.floor(math.log2(max(_num_arg(x, 0), 1e-300))))),
        "DEG2RAD": math.pi / 180, "RAD2DEG": 180 / math.pi})
    return JSObject(three)


# three.js's public enum values (its constants module): sides, wrapping, filters, texel types and formats,
# colour spaces, blending modes, buffer usages, shading
THREE_CONSTANTS = {
    "FrontSide": 0.0, "BackSide": 1.0, "DoubleSide": 2.0,
    "RepeatWrapping": 1000.0, "ClampToEdgeWrapping": 1001.0, "MirroredRepeatWrapping": 1002.0,
    "NearestFilter": 1003.0, "NearestMipmapNearestFilter": 1004.0, "NearestMipmapLinearFilter": 1005.0,
    "LinearFilter": 1006.0, "LinearMipmapNearestFilter": 1007.0, "LinearMipmapLinearFilter": 1008.0,
    "UnsignedByteType": 1009.0, "ByteType": 1010.0, "ShortType": 1011.0, "UnsignedShortType": 1012.0,
    "IntType": 1013.0, "UnsignedIntType": 1014.0, "FloatType": 1015.0, "HalfFloatType": 1016.0,
    "AlphaFormat": 1021.0, "RGBFormat": 1022.0, "RGBAFormat": 1023.0, "RedFormat": 1028.0, "RGFormat": 1030.0,
    "NoColorSpace": "", "SRGBColorSpace": "srgb", "LinearSRGBColorSpace": "srgb-linear",
    "NoBlending": 0.0, "NormalBlending": 1.0, "AdditiveBlending": 2.0, "SubtractiveBlending": 3.0,
    "MultiplyBlending": 4.0,
    "StaticDrawUsage": 35044.0, "DynamicDrawUsage": 35048.0, "StreamDrawUsage": 35040.0,
    "FlatShading": 1.0, "SmoothShading": 2.0, "LuminanceFormat": 1024.0,
}


def _smoothstep(x, lo, hi):
    if x <= lo:
        return 0.0
    if x >= hi:
        return 1.0
    t = (x - lo) / (hi - lo)
    return t * t * (3 - 2 * t)


def _instanced(x):
    o = Object3D("InstancedMesh", _arg(x, 0), _arg(x, 1))
    o.props["count"] = _num_arg(x, 2)
    o.props["__inst"] = {}
    o.props["instanceMatrix"] = JSObject({"needsUpdate": False})
    return o


# ---------------------------------------------------------------------------------- triangulation & export


def geometry_mesh(g: Geometry):
    """-> (vertices [V, 3] float32 tensor, faces [F, 3] int64) with the geometry's baked transform applied."""
    import torch

    from ..render import scene as S
    p = g.params
    t = "BufferGeometry" if g.baked else g.gtype

    def n(key, d=0.0):
        v = p.get(key, d)
        return _to_num(v) if v is not UNDEF and v is not None else d

    if t == "BoxGeometry":
        v, f = S._box(n("width", 1), n("height", 1), n("depth", 1))
    elif t in ("SphereGeometry",):
        v, f = S._sphere(n("radius", 1), min(int(n("widthSegments", 32)), 64), min(int(n("heightSegments", 16)), 48),
                         n("phiStart", 0.0), n("phiLength", 2 * math.pi), n("thetaStart", 0.0), n("thetaLength", math.pi))
    elif t in ("IcosahedronGeometry", "OctahedronGeometry", "TetrahedronGeometry", "DodecahedronGeometry"):
        v, f = _platonic(t, n("radius", 1), int(n("detail", 0)))
    elif t == "CylinderGeometry":
        v, f = S._cylinder(n("radiusTop", 1), n("radiusBottom", 1), n("height", 1), min(int(n("radialSegments", 32)), 64),
                           min(int(n("heightSegments", 1)), 32), _truthy(p.get("openEnded", False)),
                           n("thetaStart", 0.0), n("thetaLength", 2 * math.pi))
    elif t == "ConeGeometry":
        v, f = S._cone(n("radius", 1), n("height", 1), min(int(n("radialSegments", 32)), 64),
                       min(int(n("heightSegments", 1)), 32), _truthy(p.get("openEnded", False)),
                       n("thetaStart", 0.0), n("thetaLength", 2 * math.pi))
    elif t == "PlaneGeometry":
        v, f = S._plane(n("width", 1), n("height", 1))
    elif t == "CircleGeometry":
        v, f = _fan(n("radius", 1), 0.0, min(int(n("segments", 32)), 96), n("thetaStart", 0), n("thetaLength", 2 * math.pi))
    elif t == "RingGeometry":
        v, f = _fan(n("outerRadius", 1), n("innerRadius", 0.5), min(int(n("thetaSegments", 32)), 96),
                    n("thetaStart", 0), n("thetaLength", 2 * math.pi))
    elif t == "TorusGeometry":
        v, f = S._torus(n("radius", 1), n("tube", 0.4), min(int(n("radialSegments", 12)), 32),
                        min(int(n("tubularSegments", 48)), 96), n("arc", 2 * math.pi))
    elif t == "CapsuleGeometry":
        r, L = n("radius", 1), n("length", 1)
        prof = [(r * math.sin(math.pi / 2 * k / 6), L / 2 + r * math.cos(math.pi / 2 * k / 6)) for k in range(7)]
        prof += [(r * math.cos(math.pi / 2 * k / 6), -L / 2 - r * math.sin(math.pi / 2 * k / 6)) for k in range(7)]
        v, f = S._lathe([(0.0, L / 2 + r)] + prof + [(0.0, -L / 2 - r)], min(int(n("radialSegments", 8)) * 2, 48))
    elif t == "LatheGeometry":
        pts = [q.v()[:2] for q in it_items(p.get("points"))] or [[0, 0], [1, 0]]
        v, f = S._lathe([(a, b) for a, b in pts], min(max(int(n("segments", 12)), 3), 96), n("phiStart", 0.0),
                        n("phiLength", 2 * math.pi))
    elif t == "TorusKnotGeometry":
        v, f = _knot(n("radius", 1), n("tube", 0.4), min(int(n("tubularSegments", 64)), 128),
                     min(int(n("radialSegments", 8)), 16), n("p", 2), n("q", 3))
    elif t == "TubeGeometry":
        path = p.get("path")
        if not isinstance(path, Curve):
            raise _Throw(_error_obj("TypeError", "TubeGeometry needs a Curve path"))
        v, f = _tube(path, min(int(n("tubularSegments", 64)), 256), n("radius", 1), min(int(n("radialSegments", 8)), 24))
    elif t in ("ExtrudeGeometry", "ShapeGeometry"):
        from . import extrude as X
        shapes = p.get("shapes")
        shapes = it_items(shapes) if isinstance(shapes, JSArray) else [shapes]
        opts = p.get("options")
        o = opts.props if isinstance(opts, JSObject) else {}

        def opt(key, d):
            v = o.get(key, UNDEF)
            return d if v is UNDEF or v is None else v
        segs = int(_to_num(opt("curveSegments", 12))) if t == "ExtrudeGeometry" else int(n("curveSegments", 12))
        if t == "ExtrudeGeometry":
            depth = _to_num(opt("depth", opt("amount", 1.0)))
            bevel = _truthy(opt("bevelEnabled", True))
            thick = _to_num(opt("bevelThickness", 0.2))
            size = _to_num(opt("bevelSize", thick - 0.1))
            kw = dict(depth=depth, bevel=bevel, thickness=thick, size=size, offset=_to_num(opt("bevelOffset", 0.0)),
                      segments=int(_to_num(opt("bevelSegments", 3))))
        else:
            kw = dict(depth=0.0, bevel=False)
        vs, fs, off = [], [], 0
        for sh in shapes:
            if isinstance(sh, Shape) and len(sh.sample(segs)) >= 3:
                holes = [h.sample(segs) for h in sh.holes_]
                vv, ff = X.extrude(sh.sample(segs), [h for h in holes if len(h) >= 3], **kw)
                if vv:
                    vs += vv
                    fs += [(a + off, b + off, c + off) for a, b, c in ff]
                    off += len(vv)
        v = torch.tensor(vs, dtype=torch.float32).view(-1, 3)
        f = torch.tensor(fs, dtype=torch.long).view(-1, 3)
    elif t == "BufferGeometry":
        pos = g.buffer.get("position")
        if not isinstance(pos, BufferAttribute) or pos.item < 2:
            v, f = torch.zeros(0, 3), torch.zeros(0, 3, dtype=torch.long)
        else:
            arr = torch.tensor(pos.array, dtype=torch.float32).view(-1, pos.item)
            v = torch.zeros(arr.shape[0], 3)
            v[:, :min(3, pos.item)] = arr[:, :3]
            idx = g.buffer.get("__index")
            if isinstance(idx, BufferAttribute):
                ia = idx.array
            elif isinstance(idx, JSArray):
                ia = [_to_num(q) for q in idx.items]
            else:
                ia = list(range(v.shape[0]))
            ia = [int(q) for q in ia[: len(ia) // 3 * 3]]
            f = torch.tensor(ia, dtype=torch.long).view(-1, 3) if ia else torch.zeros(0, 3, dtype=torch.long)
            if f.numel() and (f.max() >= v.shape[0] or f.min() < 0):
                raise _Throw(_error_obj("RangeError", "index out of range in BufferGeometry"))
    else:
        raise _Throw(_error_obj("TypeError", f"unsupported geometry {t}"))
    m = torch.tensor(g.xform, dtype=torch.float32)
    if v.shape[0]:
        v = torch.cat([v.float(), torch.ones(v.shape[0], 1)], 1) @ m.t()
        v = v[:, :3]
    return v.float(), f.long()


def _fan(r_out, r_in, seg, t0, tl):
    import torch
    seg = max(seg, 3)
    verts, faces = [], []
    for k in range(seg + 1):
        a = t0 + tl * k / seg
        verts.append((r_out * math.cos(a), r_out * math.sin(a), 0.0))
        verts.append((r_in * math.cos(a), r_in * math.sin(a), 0.0))
    for k in range(seg):
        a, b, c, d = 2 * k, 2 * k + 1, 2 * k + 2, 2 * k + 3
        faces += [(a, c, b), (b, c, d)]
    return torch.tensor(verts, dtype=torch.float32), torch.tensor(faces)


def _knot(R, r, tseg, rseg, p, q):
    import torch

    def c(u):
        qu = q * u
        cs = math.cos(qu)
        return [R * (2 + cs) * 0.5 * math.cos(p * u), R * (2 + cs) * 0.5 * math.sin(p * u), R * math.sin(qu) * 0.5]
    ctrl = [c(2 * math.pi * k / tseg) for k in range(tseg)]
    return _tube(Curve("catmull", ctrl, True), tseg, r, rseg)


def _tube(curve: Curve, tseg, radius, rseg):
    import torch
    tab = curve.arc_table()
    pts = [curve.point(curve.u_to_t(k / tseg, tab)) for k in range(tseg + 1)]     # equal arc lengths, as three.js
    verts, faces = [], []
    prev_n = None
    for k, pt in enumerate(pts):
        a = pts[max(k - 1, 0)]
        b = pts[min(k + 1, len(pts) - 1)]
        tng = [y - x for x, y in zip(a, b)]
        tn = math.sqrt(sum(x * x for x in tng)) or 1.0
        tng = [x / tn for x in tng]
        ref = prev_n or ([0.0, 1.0, 0.0] if abs(tng[1]) < 0.9 else [1.0, 0.0, 0.0])
        nrm = _cross(_cross(tng, ref), tng)
        nn = math.sqrt(sum(x * x for x in nrm)) or 1.0
        nrm = [x / nn for x in nrm]
        prev_n = nrm
        bn = _cross(tng, nrm)
        for j in range(rseg):
            ang = 2 * math.pi * j / rseg
            verts.append([pt[i] + radius * (math.cos(ang) * nrm[i] + math.sin(ang) * bn[i]) for i in range(3)])
    for k in range(tseg):
        for j in range(rseg):
            a, b = k * rseg + j, k * rseg + (j + 1) % rseg
            faces += [(a, b, b + rseg), (a, b + rseg, a + rseg)]
    return torch.tensor(verts, dtype=torch.float32), torch.tensor(faces)


@dataclass
class ModuleResult:
    root: Any = None
    error: Optional[str] = None
    steps: int = 0
    seconds: float = 0.0
    texture_bytes: int = 0


# Module-level `const NAME = ...` declarations that the interpreter runs natively when the statement's syntax tree
# equals a registered source exactly: the helpers that mechanical repairs insert, whose per-texel loops a JS engine
# runs in milliseconds and this tree-walker in tens of seconds. The native must compute what the source computes.
_INTRINSICS: Dict[str, Tuple[str, Callable]] = {}
_INTRINSIC_AST: Dict[str, Any] = {}


def register_intrinsic(name: str, source: str, native: Callable) -> None:
    """source: one `const name = ...;` statement; native(interp) -> the value bound to name."""
    _INTRINSICS[name] = (source, native)
    _INTRINSIC_AST.pop(name, None)


def _intrinsic_name(st) -> Optional[str]:
    if not (st[0] == "decl" and st[1] == "const" and len(st[2]) == 1 and st[2][0][0][0] == "id"):
        return None
    name = st[2][0][0][1]
    if name not in _INTRINSICS:
        return None
    if name not in _INTRINSIC_AST:
        _INTRINSIC_AST[name] = Parser(_INTRINSICS[name][0]).program()[1][0]
    return name if _INTRINSIC_AST[name] == st else None


def run_module(source: str, limits: Optional[Limits] = None, seed: int = 0) -> ModuleResult:
    """Evaluate a module and call its default export with THREE. Never raises for JS-level failures."""
    t0 = time.monotonic()
    it = Interp(limits, seed)
    try:
        prog = Parser(source).program()
        it.run_program(prog)
        gen = it.exports.get("default")
        if gen is None:
            gen = it.exports.get("generate")
        if gen is None:
            ev = it.globals.lookup("generate")
            gen = ev.vars["generate"] if ev is not None else None
        if not isinstance(gen, (JSFunction, Native)):
            return ModuleResult(error="NO_DEFAULT_EXPORT: module must `export default function generate(THREE)`",
                                steps=it.steps, seconds=time.monotonic() - t0)
        root = it.call(gen, UNDEF, [make_three(it)])
        return ModuleResult(root=root, steps=it.steps, seconds=time.monotonic() - t0)
    except JSBudget as e:
        kind = "TIMEOUT" if ("budget" in e.msg or "exceeded" in e.msg) else "HEAP"   # time / steps, or memory
        return ModuleResult(error=f"{kind}: {e.msg}", steps=it.steps, seconds=time.monotonic() - t0)
    except JSError as e:
        return ModuleResult(error=f"{e.kind}: {e.msg}", steps=it.steps, seconds=time.monotonic() - t0)
    except _Throw as e:
        v = e.value
        msg = f"{_to_str(v.props.get('name', 'Error'))}: {_to_str(v.props.get('message', ''))}" \
            if isinstance(v, JSObject) and not isinstance(v, Host) else f"Uncaught {_to_str(v)}"
        return ModuleResult(error=f"RUNTIME: {msg}", steps=it.steps, seconds=time.monotonic() - t0)
    except (_Break, _Continue, _Return):
        return ModuleResult(error="SyntaxError: illegal break/continue/return", steps=it.steps,
                            seconds=time.monotonic() - t0)
    except RecursionError:
        return ModuleResult(error="RangeError: maximum call stack size exceeded", steps=it.steps,
                            seconds=time.monotonic() - t0)


def _col_major(m):
    return [m[r][c] for c in range(4) for r in range(4)]


def _tri_groups(g: "Geometry", n_tris: int) -> Dict[int, List[int]]:
    """Material index -> triangle indices: explicit groups (addGroup, in index units), else three.js's groups of
    a box (one per face: +x, -x, +y, -y, +z, -z) or a cylinder / cone (side, top cap, bottom cap), else one
    group 0."""
    out: Dict[int, List[int]] = {}
    groups = g.props.get("groups")
    if isinstance(groups, JSArray) and groups.items:
        for gr in groups.items:
            st, cnt = int(_to_num(gr.js_get("start"))), _to_num(gr.js_get("count"))
            cnt = n_tris * 3 - st if not math.isfinite(cnt) else int(cnt)
            mi = int(_to_num(gr.js_get("materialIndex")))
            out.setdefault(mi, []).extend(range(max(0, st // 3), min(n_tris, (st + cnt) // 3)))
        return out
    if not g.baked and g.gtype == "BoxGeometry" and n_tris == 12:
        for pair, mi in enumerate((5, 4, 3, 2, 0, 1)):        # our face order: -z, +z, -y, +y, +x, -x
            out[mi] = [2 * pair, 2 * pair + 1]
        return out
    if not g.baked and g.gtype in ("CylinderGeometry", "ConeGeometry"):
        R = max(3, min(int(_to_num(g.params.get("radialSegments", 32))), 64))
        Hs = max(1, min(int(_to_num(g.params.get("heightSegments", 1))), 32))
        side = 2 * R * Hs
        out[0] = list(range(min(side, n_tris)))
        caps = list(range(side, n_tris))
        rt = _to_num(g.params.get("radiusTop", 1.0)) if g.gtype == "CylinderGeometry" else 0.0
        k = 1
        while caps:
            out[k] = caps[:R]
            caps = caps[R:]
            k += 1
        if rt <= 0 and 1 in out and 2 not in out:             # a cone's only cap is the bottom (group 2)
            out[2] = out.pop(1)
        return out
    return {0: list(range(n_tris))}


def to_scene_json(root: Object3D, max_depth: int = 64) -> dict:
    """Object3D tree -> the scene JSON of render/scene.py (geometries baked to BufferGeometry where needed)."""
    geoms: Dict[int, dict] = {}
    mats: Dict[Any, dict] = {}

    meshes: Dict[int, tuple] = {}

    def mesh_of(g: Geometry):
        if id(g) not in meshes:
            meshes[id(g)] = geometry_mesh(g)
        return meshes[id(g)]

    def geom_ref(g: Geometry, group: Optional[int] = None, tris=None) -> str:
        key = (id(g), group)
        if key not in geoms:
            v, f = mesh_of(g)
            if tris is not None:
                f = f[tris]
            attrs = {"position": {"itemSize": 3, "type": "Float32Array", "array": v.reshape(-1).tolist()}}
            col = g.buffer.get("color")
            if isinstance(col, BufferAttribute) and col.item >= 3 and len(col.array) // col.item == v.shape[0]:
                attrs["color"] = {"itemSize": 3, "type": "Float32Array",
                                  "array": [c for k in range(v.shape[0]) for c in col.array[k * col.item:k * col.item + 3]]}
            geoms[key] = {"uuid": g.id_ + f"-{len(geoms)}", "type": "BufferGeometry",
                          "data": {"attributes": attrs,
                                   "index": {"type": "Uint32Array", "array": f.reshape(-1).tolist()}}}
        return geoms[key]["uuid"]

    def mat_ref(m) -> Optional[str]:
        if isinstance(m, JSArray):
            m = next((x for x in m.items if isinstance(x, Material)), None)
        if not isinstance(m, Material):
            return None
        key = id(m)
        if key not in mats:
            col = m.props.get("color")
            mats[key] = {"uuid": f"m{len(mats)}", "type": m.mtype,
                         "color": col.hex() if isinstance(col, Color) else 0xCCCCCC,
                         "opacity": _to_num(m.props.get("opacity", 1.0))}
            if _truthy(m.props.get("vertexColors", False)):
                mats[key]["vertexColors"] = True
            tex = m.props.get("map")
            if isinstance(tex, Texture) and tex.linear_mean() is not None:
                mats[key]["mapMean"] = tex.linear_mean()
            if m.mtype in ("MeshStandardMaterial", "MeshPhysicalMaterial"):
                mats[key]["roughness"] = _to_num(m.props.get("roughness", 1.0))
                mats[key]["metalness"] = _to_num(m.props.get("metalness", 0.0))
        return mats[key]["uuid"]

    def tinted(mid: str, rgb) -> str:
        """A copy of material `mid` whose colour is multiplied by an instance colour (linear)."""
        key = (mid, tuple(round(c, 6) for c in rgb))
        if key not in mats:
            base = next(v for v in mats.values() if v["uuid"] == mid)
            c = Color()
            c.set_any([float(base.get("color", 0xFFFFFF))])
            c.set_rgb(*[a * b for a, b in zip(c.rgb(), rgb)])
            mats[key] = dict(base, uuid=f"{mid}-{len(mats)}", color=c.hex())
        return mats[key]["uuid"]

    def node(o: Object3D, depth: int) -> dict:
        if depth > max_depth:
            raise ValueError("scene depth limit exceeded")
        d = {"uuid": o.id_, "type": o.otype, "matrix": _col_major(o.local()), "children": []}
        if not _truthy(o.props.get("visible", True)):
            d["visible"] = False
            return d
        g = o.props.get("geometry")
        if isinstance(g, Geometry) and o.otype in ("Mesh", "InstancedMesh"):
            gid, mid = geom_ref(g), mat_ref(o.props.get("material"))
            if o.otype == "InstancedMesh":
                count = int(_to_num(o.props.get("count", 0)))
                inst = o.props.get("__inst", {})
                icol = o.props.get("__icol", {})
                for k in range(count):
                    mk = mid if k not in icol else tinted(mid, icol[k])
                    d["children"].append({"uuid": f"{o.id_}-{k}", "type": "Mesh", "geometry": gid, "material": mk,
                                          "matrix": _col_major(inst.get(k, _ident4())), "children": []})
            elif isinstance(o.props.get("material"), JSArray):
                # one material per geometry group: a sub-mesh per group (three.js draws each group with its
                # material; a geometry without groups takes the first material here)
                mlist = o.props["material"].items
                for grp, tris in _tri_groups(g, mesh_of(g)[1].shape[0]).items():
                    m = mlist[grp] if 0 <= grp < len(mlist) else None
                    if isinstance(m, Material) and tris:
                        d["children"].append({"uuid": f"{o.id_}-g{grp}", "type": "Mesh",
                                              "geometry": geom_ref(g, grp, tris), "material": mat_ref(m),
                                              "matrix": _col_major(_ident4()), "children": []})
            else:
                d["geometry"], d["material"] = gid, mid
        for c in o.children():
            d["children"].append(node(c, depth + 1))
        return d

    obj = node(root, 0)
    return {"metadata": {"version": 4.6, "type": "Object", "generator": "phung5_b200.app.jsvm"},
            "geometries": list(geoms.values()), "materials": list(mats.values()), "object": obj}


# ------------------------------------------------------------------------------------------------------------
# the rest of the specification's THREE members: math helpers, 2D / custom curves and paths, polyhedra, edge and
# wireframe geometries, more attribute types and interleaved buffers
# ------------------------------------------------------------------------------------------------------------

def _v3(vals=(0.0, 0.0, 0.0)):
    return Vec(("x", "y", "z"), list(vals), "Vector3")


def _v2(vals=(0.0, 0.0)):
    return Vec(("x", "y"), list(vals), "Vector2")


def _vec_or(x, k, dim=3):
    v = _arg(x, k)
    return v.v()[:dim] if isinstance(v, Vec) else [0.0] * dim


def _target(x, k, dim=3):
    t = _arg(x, k)
    return t if isinstance(t, Vec) else (_v3() if dim == 3 else _v2())


class _Shape3(Host):
    """A math object whose state is a few vector / number properties (Sphere, Plane, Ray, Line3, Triangle, Box2,
    Spherical, Cylindrical); `fields` lists them for clone / copy."""
    __slots__ = ("kind",)
    fields: Tuple[str, ...] = ()

    def __init__(self, kind, props):
        super().__init__(dict(props, **{"is" + kind: True}))
        self.kind = kind

    @property
    def cls_name(self):
        return self.kind

    def is_instance(self, name):
        return name == self.kind

    def clone_(self):
        return type(self)(**{f: (self.props[f].v() if isinstance(self.props[f], Vec) else self.props[f])
                             for f in self.fields})

    def copy_(self, o):
        for f in self.fields:
            if isinstance(self.props[f], Vec):
                self.props[f].setv(o.props[f].v())
            else:
                self.props[f] = o.props[f]
        return self


class Sphere(_Shape3):
    fields = ("center", "radius")

    def __init__(self, center=(0.0, 0.0, 0.0), radius=-1.0):
        super().__init__("Sphere", {"center": _v3(center), "radius": float(radius)})

    def from_points(self, pts):
        vs = [p.v() for p in pts if isinstance(p, Vec)]
        if not vs:
            return self
        c = [(min(a) + max(a)) / 2 for a in zip(*vs)]
        self.props["center"].setv(c)
        self.props["radius"] = max(math.dist(c, v) for v in vs)
        return self

    js_methods = {
        "set": lambda s, i, x: (s.props["center"].setv(_vec_or(x, 0)), s.props.__setitem__("radius", _num_arg(x, 1)), s)[-1],
        "setFromPoints": lambda s, i, x: s.from_points(it_items(_arg(x, 0))),
        "clone": lambda s, i, x: s.clone_(),
        "copy": lambda s, i, x: s.copy_(_arg(x, 0)),
        "isEmpty": lambda s, i, x: _to_num(s.props["radius"]) < 0,
        "containsPoint": lambda s, i, x: math.dist(_vec_or(x, 0), s.props["center"].v()) <= _to_num(s.props["radius"]),
        "distanceToPoint": lambda s, i, x: math.dist(_vec_or(x, 0), s.props["center"].v()) - _to_num(s.props["radius"]),
        "translate": lambda s, i, x: (s.props["center"].setv([a + b for a, b in zip(s.props["center"].v(), _vec_or(x, 0))]), s)[-1],
    }


class Plane(_Shape3):
    fields = ("normal", "constant")

    def __init__(self, normal=(1.0, 0.0, 0.0), constant=0.0):
        super().__init__("Plane", {"normal": _v3(normal), "constant": float(constant)})

    def dist(self, p):
        return sum(a * b for a, b in zip(self.props["normal"].v(), p)) + _to_num(self.props["constant"])

    def from_coplanar(self, a, b, c):
        n = _unit(_cross([q - p for p, q in zip(b, c)], [q - p for p, q in zip(b, a)]))
        self.props["normal"].setv(n)
        self.props["constant"] = -sum(x * y for x, y in zip(a, n))
        return self

    js_methods = {
        "set": lambda s, i, x: (s.props["normal"].setv(_vec_or(x, 0)), s.props.__setitem__("constant", _num_arg(x, 1)), s)[-1],
        "setComponents": lambda s, i, x: (s.props["normal"].setv([_num_arg(x, k) for k in range(3)]),
                                          s.props.__setitem__("constant", _num_arg(x, 3)), s)[-1],
        "setFromNormalAndCoplanarPoint": lambda s, i, x: (s.props["normal"].setv(_vec_or(x, 0)), s.props.__setitem__(
            "constant", -sum(a * b for a, b in zip(_vec_or(x, 1), _vec_or(x, 0)))), s)[-1],
        "setFromCoplanarPoints": lambda s, i, x: s.from_coplanar(_vec_or(x, 0), _vec_or(x, 1), _vec_or(x, 2)),
        "normalize": lambda s, i, x: (lambda n: (s.props["normal"].setv([a / n for a in s.props["normal"].v()]),
                                                 s.props.__setitem__("constant", _to_num(s.props["constant"]) / n), s)[-1])(
            math.sqrt(sum(a * a for a in s.props["normal"].v())) or 1.0),
        "negate": lambda s, i, x: (s.props["normal"].setv([-a for a in s.props["normal"].v()]),
                                   s.props.__setitem__("constant", -_to_num(s.props["constant"])), s)[-1],
        "distanceToPoint": lambda s, i, x: s.dist(_vec_or(x, 0)),
        "projectPoint": lambda s, i, x: _target(x, 1).setv([p - s.dist(_vec_or(x, 0)) * n for p, n in zip(
            _vec_or(x, 0), s.props["normal"].v())]),
        "clone": lambda s, i, x: s.clone_(),
        "copy": lambda s, i, x: s.copy_(_arg(x, 0)),
    }


class Ray(_Shape3):
    fields = ("origin", "direction")

    def __init__(self, origin=(0.0, 0.0, 0.0), direction=(0.0, 0.0, -1.0)):
        super().__init__("Ray", {"origin": _v3(origin), "direction": _v3(direction)})

    js_methods = {
        "set": lambda s, i, x: (s.props["origin"].setv(_vec_or(x, 0)), s.props["direction"].setv(_vec_or(x, 1)), s)[-1],
        "at": lambda s, i, x: _target(x, 1).setv([o + d * _num_arg(x, 0) for o, d in zip(
            s.props["origin"].v(), s.props["direction"].v())]),
        "clone": lambda s, i, x: s.clone_(),
        "copy": lambda s, i, x: s.copy_(_arg(x, 0)),
    }


class Line3(_Shape3):
    fields = ("start", "end")

    def __init__(self, start=(0.0, 0.0, 0.0), end=(0.0, 0.0, 0.0)):
        super().__init__("Line3", {"start": _v3(start), "end": _v3(end)})

    def ab(self):
        return self.props["start"].v(), self.props["end"].v()

    js_methods = {
        "set": lambda s, i, x: (s.props["start"].setv(_vec_or(x, 0)), s.props["end"].setv(_vec_or(x, 1)), s)[-1],
        "getCenter": lambda s, i, x: _target(x, 0).setv([(a + b) / 2 for a, b in zip(*s.ab())]),
        "delta": lambda s, i, x: _target(x, 0).setv([b - a for a, b in zip(*s.ab())]),
        "distance": lambda s, i, x: math.dist(*s.ab()),
        "distanceSq": lambda s, i, x: math.dist(*s.ab()) ** 2,
        "at": lambda s, i, x: _target(x, 1).setv([a + (b - a) * _num_arg(x, 0) for a, b in zip(*s.ab())]),
        "clone": lambda s, i, x: s.clone_(),
        "copy": lambda s, i, x: s.copy_(_arg(x, 0)),
    }


class Triangle(_Shape3):
    fields = ("a", "b", "c")

    def __init__(self, a=(0.0, 0.0, 0.0), b=(0.0, 0.0, 0.0), c=(0.0, 0.0, 0.0)):
        super().__init__("Triangle", {"a": _v3(a), "b": _v3(b), "c": _v3(c)})

    def abc(self):
        return self.props["a"].v(), self.props["b"].v(), self.props["c"].v()

    def normal_(self):
        a, b, c = self.abc()
        return _cross([q - p for p, q in zip(b, c)], [q - p for p, q in zip(b, a)])

    js_methods = {
        "set": lambda s, i, x: (s.props["a"].setv(_vec_or(x, 0)), s.props["b"].setv(_vec_or(x, 1)),
                                s.props["c"].setv(_vec_or(x, 2)), s)[-1],
        "getNormal": lambda s, i, x: _target(x, 0).setv(_unit(s.normal_())),
        "getArea": lambda s, i, x: 0.5 * math.sqrt(sum(a * a for a in s.normal_())),
        "getMidpoint": lambda s, i, x: _target(x, 0).setv([sum(t) / 3 for t in zip(*s.abc())]),
        "clone": lambda s, i, x: s.clone_(),
        "copy": lambda s, i, x: s.copy_(_arg(x, 0)),
    }


class Box2(_Shape3):
    fields = ("min", "max")

    def __init__(self, min=(math.inf, math.inf), max=(-math.inf, -math.inf)):
        super().__init__("Box2", {"min": _v2(min), "max": _v2(max)})

    def expand(self, p):
        lo, hi = self.props["min"], self.props["max"]
        lo.setv([_mn(a, b) for a, b in zip(lo.v(), p)])
        hi.setv([_mx(a, b) for a, b in zip(hi.v(), p)])
        return self

    def empty(self):
        return any(a > b for a, b in zip(self.props["min"].v(), self.props["max"].v()))

    js_methods = {
        "set": lambda s, i, x: (s.props["min"].setv(_vec_or(x, 0, 2)), s.props["max"].setv(_vec_or(x, 1, 2)), s)[-1],
        "setFromPoints": lambda s, i, x: (s.props["min"].setv([math.inf] * 2), s.props["max"].setv([-math.inf] * 2),
                                          [s.expand(p.v()[:2]) for p in it_items(_arg(x, 0))], s)[-1],
        "expandByPoint": lambda s, i, x: s.expand(_vec_or(x, 0, 2)),
        "makeEmpty": lambda s, i, x: (s.props["min"].setv([math.inf] * 2), s.props["max"].setv([-math.inf] * 2), s)[-1],
        "isEmpty": lambda s, i, x: s.empty(),
        "getSize": lambda s, i, x: _target(x, 0, 2).setv([0.0, 0.0] if s.empty() else
                                                         [b - a for a, b in zip(s.props["min"].v(), s.props["max"].v())]),
        "getCenter": lambda s, i, x: _target(x, 0, 2).setv([0.0, 0.0] if s.empty() else
                                                           [(a + b) / 2 for a, b in zip(s.props["min"].v(), s.props["max"].v())]),
        "containsPoint": lambda s, i, x: all(a <= p <= b for a, p, b in zip(s.props["min"].v(), _vec_or(x, 0, 2),
                                                                             s.props["max"].v())),
        "clone": lambda s, i, x: s.clone_(),
        "copy": lambda s, i, x: s.copy_(_arg(x, 0)),
    }


def _mn(a, b):
    return a if a < b else b


def _mx(a, b):
    return a if a > b else b


class Spherical(_Shape3):
    fields = ("radius", "phi", "theta")

    def __init__(self, radius=1.0, phi=0.0, theta=0.0):
        super().__init__("Spherical", {"radius": float(radius), "phi": float(phi), "theta": float(theta)})

    def rpt(self):
        return _to_num(self.props["radius"]), _to_num(self.props["phi"]), _to_num(self.props["theta"])

    def from_xyz(self, x, y, z):
        r = math.sqrt(x * x + y * y + z * z)
        self.props["radius"] = r
        self.props["theta"] = math.atan2(x, z) if r else 0.0
        self.props["phi"] = math.acos(max(-1.0, min(1.0, y / r))) if r else 0.0
        return self

    js_methods = {
        "set": lambda s, i, x: (s.props.update(radius=_num_arg(x, 0), phi=_num_arg(x, 1), theta=_num_arg(x, 2)), s)[-1],
        "setFromVector3": lambda s, i, x: s.from_xyz(*_vec_or(x, 0)),
        "setFromCartesianCoords": lambda s, i, x: s.from_xyz(_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2)),
        "makeSafe": lambda s, i, x: (s.props.__setitem__("phi", max(1e-6, min(math.pi - 1e-6, _to_num(s.props["phi"])))), s)[-1],
        "clone": lambda s, i, x: s.clone_(),
        "copy": lambda s, i, x: s.copy_(_arg(x, 0)),
    }


class Cylindrical(_Shape3):
    fields = ("radius", "theta", "y")

    def __init__(self, radius=1.0, theta=0.0, y=0.0):
        super().__init__("Cylindrical", {"radius": float(radius), "theta": float(theta), "y": float(y)})

    def rty(self):
        return _to_num(self.props["radius"]), _to_num(self.props["theta"]), _to_num(self.props["y"])

    def from_xyz(self, x, y, z):
        self.props.update(radius=math.sqrt(x * x + z * z), theta=math.atan2(x, z), y=float(y))
        return self

    js_methods = {
        "set": lambda s, i, x: (s.props.update(radius=_num_arg(x, 0), theta=_num_arg(x, 1), y=_num_arg(x, 2)), s)[-1],
        "setFromVector3": lambda s, i, x: s.from_xyz(*_vec_or(x, 0)),
        "setFromCartesianCoords": lambda s, i, x: s.from_xyz(_num_arg(x, 0), _num_arg(x, 1), _num_arg(x, 2)),
        "clone": lambda s, i, x: s.clone_(),
        "copy": lambda s, i, x: s.copy_(_arg(x, 0)),
    }


class Matrix3(Host):
    __slots__ = ("m",)
    cls_name = "Matrix3"

    def __init__(self, m=None):
        super().__init__({"isMatrix3": True})
        self.m = m or [[1.0, 0.0, 0.0], [0.0, 1.0, 0.0], [0.0, 0.0, 1.0]]

    def get_special(self, it, key):
        if key == "elements":
            return JSArray([self.m[r][c] for c in range(3) for r in range(3)])
        return super().get_special(it, key)

    def put(self, m):
        self.m = [list(map(float, row)) for row in m]
        return self

    def det(self):
        m = self.m
        return (m[0][0] * (m[1][1] * m[2][2] - m[1][2] * m[2][1]) - m[0][1] * (m[1][0] * m[2][2] - m[1][2] * m[2][0]) +
                m[0][2] * (m[1][0] * m[2][1] - m[1][1] * m[2][0]))

    def inv(self):
        d = self.det()
        if d == 0:
            return self.put([[0.0] * 3 for _ in range(3)])
        m = self.m
        cof = [[(m[(r + 1) % 3][(c + 1) % 3] * m[(r + 2) % 3][(c + 2) % 3] -
                 m[(r + 1) % 3][(c + 2) % 3] * m[(r + 2) % 3][(c + 1) % 3]) for c in range(3)] for r in range(3)]
        return self.put([[cof[c][r] / d for c in range(3)] for r in range(3)])

    js_methods = {
        "set": lambda s, i, x: s.put([[_num_arg(x, 3 * r + c) for c in range(3)] for r in range(3)]),
        "identity": lambda s, i, x: s.put([[1.0 if r == c else 0.0 for c in range(3)] for r in range(3)]),
        "copy": lambda s, i, x: s.put(_arg(x, 0).m),
        "clone": lambda s, i, x: Matrix3([row[:] for row in s.m]),
        "multiply": lambda s, i, x: s.put(_mat_mul(s.m, _arg(x, 0).m)),
        "premultiply": lambda s, i, x: s.put(_mat_mul(_arg(x, 0).m, s.m)),
        "multiplyMatrices": lambda s, i, x: s.put(_mat_mul(_arg(x, 0).m, _arg(x, 1).m)),
        "multiplyScalar": lambda s, i, x: s.put([[a * _num_arg(x, 0) for a in row] for row in s.m]),
        "determinant": lambda s, i, x: s.det(),
        "invert": lambda s, i, x: s.inv(),
        "transpose": lambda s, i, x: s.put([list(col) for col in zip(*s.m)]),
        "setFromMatrix4": lambda s, i, x: s.put([row[:3] for row in _arg(x, 0).m[:3]]),
        "makeRotation": lambda s, i, x: s.put([[math.cos(_num_arg(x, 0)), -math.sin(_num_arg(x, 0)), 0.0],
                                               [math.sin(_num_arg(x, 0)), math.cos(_num_arg(x, 0)), 0.0],
                                               [0.0, 0.0, 1.0]]),
        "makeScale": lambda s, i, x: s.put([[_num_arg(x, 0), 0.0, 0.0], [0.0, _num_arg(x, 1), 0.0], [0.0, 0.0, 1.0]]),
        "makeTranslation": lambda s, i, x: s.put([[1.0, 0.0, _num_arg(x, 0)], [0.0, 1.0, _num_arg(x, 1)],
                                                  [0.0, 0.0, 1.0]]),
        "toArray": lambda s, i, x: JSArray([s.m[r][c] for c in range(3) for r in range(3)]),
        "fromArray": lambda s, i, x: s.put([[_to_num(it_items(_arg(x, 0))[3 * c + r]) for c in range(3)]
                                            for r in range(3)]),
    }


class InterleavedBuffer(Host):
    __slots__ = ("array", "stride")
    cls_name = "InterleavedBuffer"

    def __init__(self, array, stride):
        super().__init__({"isInterleavedBuffer": True, "stride": float(stride)})
        self.array, self.stride = [float(_to_num(a)) for a in array], max(1, int(stride))

    def get_special(self, it, key):
        if key == "count":
            return float(len(self.array) // self.stride)
        if key == "array":
            return JSArray(list(self.array))
        return super().get_special(it, key)


def _interleaved_attr(x):
    """An attribute view of an interleaved buffer, copied out into a plain attribute (edits do not write back)."""
    ib, item, off = _arg(x, 0), max(1, int(_num_arg(x, 1, 3.0))), int(_num_arg(x, 2, 0.0))
    if not isinstance(ib, InterleavedBuffer):
        raise _Throw(_error_obj("TypeError", "InterleavedBufferAttribute needs an InterleavedBuffer"))
    n = len(ib.array) // ib.stride
    return BufferAttribute([ib.array[r * ib.stride + off + k] for r in range(n) for k in range(item)
                            if r * ib.stride + off + k < len(ib.array)], item)


def _baked(gtype, verts, faces=None, params=None):
    g = Geometry(gtype, params or {})
    g.buffer["position"] = BufferAttribute([float(c) for v in verts for c in v], 3)
    if faces is not None:
        g.buffer["__index"] = BufferAttribute([float(i) for f in faces for i in f], 1, "Uint32Array")
    g.baked = True
    return g


_PHI = (1 + math.sqrt(5)) / 2
_PLATONIC_VERTS = {
    "TetrahedronGeometry": [(1, 1, 1), (-1, -1, 1), (-1, 1, -1), (1, -1, -1)],
    "OctahedronGeometry": [(1, 0, 0), (-1, 0, 0), (0, 1, 0), (0, -1, 0), (0, 0, 1), (0, 0, -1)],
    "IcosahedronGeometry": [(sx, sy * _PHI, 0) for sx in (-1, 1) for sy in (-1, 1)] +
                           [(0, sx, sy * _PHI) for sx in (-1, 1) for sy in (-1, 1)] +
                           [(sy * _PHI, 0, sx) for sx in (-1, 1) for sy in (-1, 1)],
    "DodecahedronGeometry": [(a, b, c) for a in (-1, 1) for b in (-1, 1) for c in (-1, 1)] +
                            [(0, a / _PHI, b * _PHI) for a in (-1, 1) for b in (-1, 1)] +
                            [(a / _PHI, b * _PHI, 0) for a in (-1, 1) for b in (-1, 1)] +
                            [(a * _PHI, 0, b / _PHI) for a in (-1, 1) for b in (-1, 1)],
}


def _subdivided_sphere_mesh(pts, tris, radius, detail):
    """Split every triangle into (detail + 1)^2 and push every vertex out to the sphere of the radius."""
    n = detail + 1
    verts, faces = [], []
    for a, b, c in tris:
        a, b, c = pts[a], pts[b], pts[c]
        grid = {}
        for r in range(n + 1):
            for k in range(n + 1 - r):
                q = [a[j] + (b[j] - a[j]) * r / n + (c[j] - a[j]) * k / n for j in range(3)]
                grid[(r, k)] = len(verts)
                verts.append([x * radius for x in _unit(q)])
        for r in range(n):
            for k in range(n - r):
                faces.append((grid[(r, k)], grid[(r + 1, k)], grid[(r, k + 1)]))
                if k + 1 <= n - r - 1:
                    faces.append((grid[(r + 1, k)], grid[(r + 1, k + 1)], grid[(r, k + 1)]))
    return verts, faces


def _platonic(gtype, radius, detail):
    """A Platonic solid inscribed in the sphere of the radius (its faces triangulated from the convex hull of
    its vertices), optionally subdivided toward the sphere."""
    import torch
    from scipy.spatial import ConvexHull
    pts = [list(map(float, q)) for q in _PLATONIC_VERTS[gtype]]
    hull = ConvexHull(pts)
    verts, faces = _subdivided_sphere_mesh(pts, [tuple(int(i) for i in t) for t in hull.simplices],
                                           radius, max(0, min(int(detail), 5)))
    return torch.tensor(verts, dtype=torch.float32), torch.tensor(faces, dtype=torch.long).view(-1, 3)


def _polyhedron(x):
    """PolyhedronGeometry(vertices, indices, radius, detail): every face split into (detail + 1)^2 triangles,
    every vertex pushed out to the sphere of the radius."""
    vs = [float(_to_num(a)) for a in it_items(_arg(x, 0))]
    ids = [int(_to_num(a)) for a in it_items(_arg(x, 1))]
    radius, detail = _num_arg(x, 2, 1.0), max(0, min(int(_num_arg(x, 3, 0.0)), 6))
    pts = [vs[k:k + 3] for k in range(0, len(vs) - 2, 3)]
    verts, faces = [], []
    for f in range(0, len(ids) - 2, 3):
        try:
            a, b, c = (pts[ids[f + j]] for j in range(3))
        except IndexError:
            raise _Throw(_error_obj("RangeError", "PolyhedronGeometry index out of range"))
        n = detail + 1
        grid = {}
        for r in range(n + 1):
            for k in range(n + 1 - r):
                w_b, w_c = r / n, k / n
                p = [a[j] + (b[j] - a[j]) * w_b + (c[j] - a[j]) * w_c for j in range(3)]
                grid[(r, k)] = len(verts)
                verts.append([q * radius for q in _unit(p)])
        for r in range(n):
            for k in range(n - r):
                faces.append((grid[(r, k)], grid[(r + 1, k)], grid[(r, k + 1)]))
                if k + 1 <= n - r - 1:
                    faces.append((grid[(r + 1, k)], grid[(r + 1, k + 1)], grid[(r, k + 1)]))
    return _baked("PolyhedronGeometry", verts, faces, {"radius": radius, "detail": float(detail)})


def _edge_segments(geom, threshold_deg=None):
    """Line segments of a geometry's triangle edges: every edge (wireframe), or only edges whose two faces bend by
    more than `threshold_deg` plus open edges (EdgesGeometry). Vertices are merged by position first."""
    if not isinstance(geom, Geometry):
        raise _Throw(_error_obj("TypeError", "expected a geometry"))
    v, f = geometry_mesh(geom)
    key = {}
    remap = []
    for p in v.tolist():
        k = tuple(round(c, 5) for c in p)
        remap.append(key.setdefault(k, len(key)))
    pos = list(key.keys())
    edges = {}
    for tri in f.tolist():
        a, b, c = (remap[t] for t in tri)
        n = _cross([q - p for p, q in zip(pos[a], pos[b])], [q - p for p, q in zip(pos[a], pos[c])])
        if sum(t * t for t in n) == 0:
            continue
        n = _unit(n)
        for e in ((a, b), (b, c), (c, a)):
            edges.setdefault(tuple(sorted(e)), []).append(n)
    out = []
    cos_t = None if threshold_deg is None else math.cos(math.radians(threshold_deg))
    for (a, b), ns in edges.items():
        if cos_t is None or len(ns) == 1 or sum(p * q for p, q in zip(ns[0], ns[1])) <= cos_t:
            out += [pos[a], pos[b]]
    return out


def _install_spec_members(it: "Interp", three: Dict[str, Any]) -> None:
    three["Vector4"] = _vec_ctor("Vector4", ("x", "y", "z", "w"))
    three["Matrix3"] = Native("Matrix3", ctor=lambda i, x: Matrix3())
    three["Box2"] = Native("Box2", ctor=lambda i, x: Box2(_vec_or(x, 0, 2) if x else (math.inf,) * 2,
                                                          _vec_or(x, 1, 2) if len(x) > 1 else (-math.inf,) * 2))
    three["Sphere"] = Native("Sphere", ctor=lambda i, x: Sphere(_vec_or(x, 0), _num_arg(x, 1, -1.0)))
    three["Plane"] = Native("Plane", ctor=lambda i, x: Plane(_vec_or(x, 0) if x else (1.0, 0.0, 0.0), _num_arg(x, 1)))
    three["Ray"] = Native("Ray", ctor=lambda i, x: Ray(_vec_or(x, 0), _vec_or(x, 1) if len(x) > 1 else (0.0, 0.0, -1.0)))
    three["Line3"] = Native("Line3", ctor=lambda i, x: Line3(_vec_or(x, 0), _vec_or(x, 1)))
    three["Triangle"] = Native("Triangle", ctor=lambda i, x: Triangle(_vec_or(x, 0), _vec_or(x, 1), _vec_or(x, 2)))
    three["Spherical"] = Native("Spherical", ctor=lambda i, x: Spherical(_num_arg(x, 0, 1.0), _num_arg(x, 1), _num_arg(x, 2)))
    three["Cylindrical"] = Native("Cylindrical", ctor=lambda i, x: Cylindrical(_num_arg(x, 0, 1.0), _num_arg(x, 1),
                                                                               _num_arg(x, 2)))
    three["Curve"] = Native("Curve", ctor=lambda i, x: Curve("custom", [], interp=it))
    three["CurvePath"] = Native("CurvePath", ctor=lambda i, x: Curve("path", [], interp=it))

    def ellipse(x, arc=False):
        if arc:                     # ArcCurve(aX, aY, aRadius, aStartAngle, aEndAngle, aClockwise)
            names = ("aX", "aY", "xRadius", "aStartAngle", "aEndAngle", "aClockwise")
            d = {n: _arg(x, k) for k, n in enumerate(names)}
            d["yRadius"] = d["xRadius"]
            d["aRotation"] = 0.0
        else:
            names = ("aX", "aY", "xRadius", "yRadius", "aStartAngle", "aEndAngle", "aClockwise", "aRotation")
            d = {n: _arg(x, k) for k, n in enumerate(names)}
        defaults = {"aX": 0.0, "aY": 0.0, "xRadius": 1.0, "yRadius": 1.0, "aStartAngle": 0.0,
                    "aEndAngle": 2 * math.pi, "aClockwise": False, "aRotation": 0.0}
        p = {k: (defaults[k] if v is UNDEF else (_truthy(v) if k == "aClockwise" else _to_num(v))) for k, v in d.items()}
        return Curve("ellipse", [], dim=2, params=p)
    three["EllipseCurve"] = Native("EllipseCurve", ctor=lambda i, x: ellipse(x))
    three["ArcCurve"] = Native("ArcCurve", ctor=lambda i, x: ellipse(x, arc=True))
    three["LineCurve"] = Native("LineCurve", ctor=lambda i, x: Curve("line", [_vec_or(x, 0, 2), _vec_or(x, 1, 2)], dim=2))
    three["QuadraticBezierCurve"] = Native("QuadraticBezierCurve", ctor=lambda i, x: Curve(
        "quad", [_vec_or(x, k, 2) for k in range(3)], dim=2))
    three["CubicBezierCurve"] = Native("CubicBezierCurve", ctor=lambda i, x: Curve(
        "cubic", [_vec_or(x, k, 2) for k in range(4)], dim=2))
    three["SplineCurve"] = Native("SplineCurve", ctor=lambda i, x: Curve(
        "catmull", [p.v()[:2] for p in it_items(_arg(x, 0)) if isinstance(p, Vec)] or [[0.0, 0.0]], dim=2))
    three["PolyhedronGeometry"] = Native("PolyhedronGeometry", ctor=lambda i, x: _polyhedron(x))
    three["EdgesGeometry"] = Native("EdgesGeometry", ctor=lambda i, x: _baked(
        "EdgesGeometry", _edge_segments(_arg(x, 0), _num_arg(x, 1, 1.0))))
    three["WireframeGeometry"] = Native("WireframeGeometry", ctor=lambda i, x: _baked(
        "WireframeGeometry", _edge_segments(_arg(x, 0))))
    three["InterleavedBuffer"] = Native("InterleavedBuffer", ctor=lambda i, x: InterleavedBuffer(
        i.iterate(_arg(x, 0)) if isinstance(_arg(x, 0), JSArray) else [], _num_arg(x, 1, 3.0)))
    three["InterleavedBufferAttribute"] = Native("InterleavedBufferAttribute", ctor=lambda i, x: _interleaved_attr(x))


class JSMap(Host):
    __slots__ = ("d",)
    cls_name = "Map"

    def __init__(self, it, src=UNDEF):
        super().__init__({})
        self.d: Dict[Any, Tuple[Any, Any]] = {}
        if src is not UNDEF and src is not None:
            for e in it.iterate(src):
                self.d[_mkey(it.get(e, 0.0))] = (it.get(e, 0.0), it.get(e, 1.0))

    def get_special(self, it, key):
        if key == "size":
            return float(len(self.d))
        return super().get_special(it, key)

    def iterable(self):
        return [JSArray([k, v]) for k, v in self.d.values()]

    def own_keys(self):
        return []

    def _each(self, it, f):
        for k, v in list(self.d.values()):
            it.call(f, UNDEF, [v, k, self])
        return UNDEF

    js_methods = {
        "get": lambda s, i, x: s.d.get(_mkey(_arg(x, 0)), (None, UNDEF))[1],
        "set": lambda s, i, x: (s.d.__setitem__(_mkey(_arg(x, 0)), (_arg(x, 0), _arg(x, 1))), s)[-1],
        "has": lambda s, i, x: _mkey(_arg(x, 0)) in s.d,
        "delete": lambda s, i, x: s.d.pop(_mkey(_arg(x, 0)), None) is not None,
        "clear": lambda s, i, x: (s.d.clear(), UNDEF)[-1],
        "forEach": lambda s, i, x: s._each(i, _arg(x, 0)),
        "keys": lambda s, i, x: JSArray([k for k, _ in s.d.values()]),
        "values": lambda s, i, x: JSArray([v for _, v in s.d.values()]),
        "entries": lambda s, i, x: JSArray(s.iterable()),
    }


class JSSet(Host):
    __slots__ = ("d",)
    cls_name = "Set"

    def __init__(self, it, src=UNDEF):
        super().__init__({})
        self.d: Dict[Any, Any] = {}
        if src is not UNDEF and src is not None:
            for v in it.iterate(src):
                self.d[_mkey(v)] = v

    def get_special(self, it, key):
        if key == "size":
            return float(len(self.d))
        return super().get_special(it, key)

    def iterable(self):
        return list(self.d.values())

    def own_keys(self):
        return []

    def _each(self, it, f):
        for v in list(self.d.values()):
            it.call(f, UNDEF, [v, v, self])
        return UNDEF

    js_methods = {
        "add": lambda s, i, x: (s.d.__setitem__(_mkey(_arg(x, 0)), _arg(x, 0)), s)[-1],
        "has": lambda s, i, x: _mkey(_arg(x, 0)) in s.d,
        "delete": lambda s, i, x: s.d.pop(_mkey(_arg(x, 0)), _SKIP) is not _SKIP,
        "clear": lambda s, i, x: (s.d.clear(), UNDEF)[-1],
        "forEach": lambda s, i, x: s._each(i, _arg(x, 0)),
        "keys": lambda s, i, x: JSArray(s.iterable()),
        "values": lambda s, i, x: JSArray(s.iterable()),
        "entries": lambda s, i, x: JSArray([JSArray([v, v]) for v in s.iterable()]),
    }
