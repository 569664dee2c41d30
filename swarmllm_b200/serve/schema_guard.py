"""JSON-Schema-constrained decoding: the output stays a prefix of a JSON value
that the request's `response_format` json_schema accepts.

`SchemaPrefix` is an incremental recogniser like `json_guard.JsonPrefix`, but
every value is checked against the schema that applies at its place: the
allowed types, object keys (`properties`, `required`, `additionalProperties`),
array items and item counts (`items`, `minItems`, `maxItems`), `enum` /
`const` values, integers versus numbers, string `pattern`s (regex_guard.py:
the ECMA subset without back-references or look-around), the fixed-shape
`format`s (date, time, date-time, uuid, ipv4, email), `minLength` /
`maxLength`, numeric ranges (`minimum` / `maximum` and their exclusive forms;
a bounded number is written without an exponent, and a prefix is live only
while some completion of it lies in the range), and `anyOf` / `oneOf`
alternatives.  It is a set of deterministic parsers, one per alternative
still open: a character is accepted if at least one parser takes it.  A parser
never takes a character after which the value could not be completed (a ','
with no unseen allowed key left, a '}' with a required key missing, a ']' short
of minItems), so decoding cannot paint itself into a corner.  Whitespace
between tokens is limited to one character (or a newline and up to 8 blanks
of indentation), and none before the value: JSON allows any amount, but a
sampler that may always add a blank can stall on it forever.

Reference behaviour: structured replies through a grammar compiled from the
schema (src/inference/reply_grammar.rs:90,156).
"""
from __future__ import annotations

import json
from decimal import Decimal

from .regex_guard import FORMAT_PATTERNS, compile_pattern

_WS = " \t\n\r"
_DIGITS = "0123456789"

# expectation between tokens
_VALUE, _OBJ_FIRST, _OBJ_KEY, _COLON, _AFTER, _ARR_FIRST, _DONE = range(7)
# inside a token
_NONE, _STR, _ESC, _UNI, _NUM, _LIT, _ENUM = range(7)
# number sub-states
_N_SIGN, _N_ZERO, _N_INT, _N_DOT, _N_FRAC, _N_E, _N_ESIGN, _N_EXP = range(8)
_NUM_END_OK = (_N_ZERO, _N_INT, _N_FRAC, _N_EXP)


def _types(schema: dict) -> set | None:
    """The JSON types a schema allows, or None for any."""
    t = schema.get("type")
    if isinstance(t, str):
        return {t}
    if isinstance(t, list):
        return set(t)
    if "properties" in schema or "required" in schema:
        return {"object"}
    if "items" in schema:
        return {"array"}
    return None


def _alternatives(schema) -> list[dict]:
    """A schema with anyOf / oneOf expanded into its alternatives (each merged
    with the schema's own keywords)."""
    if not isinstance(schema, dict):
        return [{}]
    for key in ("anyOf", "oneOf"):
        alts = schema.get(key)
        if isinstance(alts, list) and alts:
            base = {k: v for k, v in schema.items() if k != key}
            out = []
            for a in alts:
                for sub in _alternatives(a if isinstance(a, dict) else {}):
                    out.append({**base, **sub})
            return out
    return [schema]


class _Obj:
    __slots__ = ("schema", "seen", "key")

    def __init__(self, schema: dict):
        self.schema, self.seen, self.key = schema, set(), ""

    def copy(self):
        c = _Obj(self.schema)
        c.seen, c.key = set(self.seen), self.key
        return c

    @property
    def props(self) -> dict:
        p = self.schema.get("properties")
        return p if isinstance(p, dict) else {}

    @property
    def closed(self) -> bool:
        """Only the listed properties may appear."""
        return self.schema.get("additionalProperties") is False

    def key_ok(self, prefix: str, full: bool) -> bool:
        if prefix in self.seen and full:
            return False
        if not self.closed:
            return True
        names = [k for k in self.props if k not in self.seen]
        return any(k == prefix for k in names) if full else any(k.startswith(prefix)
                                                                for k in names)

    def can_add(self) -> bool:
        return not self.closed or any(k not in self.seen for k in self.props)

    def can_close(self) -> bool:
        req = self.schema.get("required") or []
        return all(r in self.seen for r in req)

    def value_schema(self) -> dict:
        if self.key in self.props:
            return self.props[self.key]
        ap = self.schema.get("additionalProperties")
        return ap if isinstance(ap, dict) else {}


class _Arr:
    __slots__ = ("schema", "n")

    def __init__(self, schema: dict):
        self.schema, self.n = schema, 0

    def copy(self):
        c = _Arr(self.schema)
        c.n = self.n
        return c

    def item_schema(self) -> dict:
        it = self.schema.get("items")
        return it if isinstance(it, dict) else {}

    def can_close(self) -> bool:
        return self.n >= int(self.schema.get("minItems", 0))

    def can_add(self) -> bool:
        mx = self.schema.get("maxItems")
        return mx is None or self.n < int(mx)


class _Parser:
    """One deterministic parse under one choice of anyOf / oneOf alternatives."""

    __slots__ = ("stack", "exp", "tok", "key", "uni", "num", "integer", "lit", "lpos",
                 "cands", "text", "pending", "ws", "nl", "scon", "sst", "slen", "uhex", "nrule", "ntext")

    def __init__(self):
        self.stack: list = []
        self.exp = _VALUE
        self.tok = _NONE
        self.key = False
        self.uni = 0
        self.num = _N_INT
        self.integer = False
        self.lit, self.lpos = "", 0
        self.cands: list[str] = []      # enum / const texts the current value may still be
        self.text = ""
        self.pending: dict = {}        # schema of the next value to start
        self.ws = 0                    # blanks read since the last token
        self.nl = False                # ... the first of them a newline
        self.scon = None               # _StrRule of the string being read, if any
        self.sst = None                # its patterns' NFA state sets
        self.slen = 0                  # characters of the string so far
        self.uhex = ""                 # hex digits of a \u escape
        self.nrule = None              # _NumRule of the number being read, if any
        self.ntext = ""                # ... its text so far

    def copy(self) -> "_Parser":
        c = _Parser.__new__(_Parser)
        c.stack = [f.copy() for f in self.stack]
        for f in ("exp", "tok", "key", "uni", "num", "integer", "lit", "lpos", "text",
                  "pending", "ws", "nl", "scon", "sst", "slen", "uhex", "nrule", "ntext"):
            setattr(c, f, getattr(self, f))
        c.cands = list(self.cands)
        return c

    @property
    def done(self) -> bool:
        return self.exp == _DONE and self.tok == _NONE

    def _end_value(self):
        if self.stack and isinstance(self.stack[-1], _Arr):
            self.stack[-1].n += 1
        self.exp = _AFTER if self.stack else _DONE

    # -------------------------------------------------------------- branching
    def feed_char(self, c: str) -> list["_Parser"]:
        """The parsers that result from reading c (empty: rejected)."""
        if self.tok == _NONE and self.exp in (_VALUE, _ARR_FIRST) and c not in _WS and \
                not (self.exp == _ARR_FIRST and c == "]"):
            out = []
            for alt in _alternatives(self.pending):
                p = self.copy()
                p.ws = 0
                if p._start_value(c, alt):
                    out.append(p)
            return out
        return [self] if self._char(c) else []

    # -------------------------------------------------------------- values
    def _start_value(self, c: str, schema: dict) -> bool:
        for k in ("enum", "const"):
            if k in schema:
                vals = schema[k] if k == "enum" else [schema[k]]
                self.cands = [json.dumps(v, separators=(",", ":")) for v in vals]
                self.text = ""
                self.tok = _ENUM
                return self._enum_char(c)
        types = _types(schema)
        ok = lambda t: types is None or t in types
        if c == "{" and ok("object"):
            self.stack.append(_Obj(schema))
            self.exp = _OBJ_FIRST
            return True
        if c == "[" and ok("array"):
            self.stack.append(_Arr(schema))
            self.exp = _ARR_FIRST
            self.pending = self.stack[-1].item_schema()
            return True
        if c == '"' and ok("string"):
            self.tok, self.key = _STR, False
            self.scon = _StrRule.of(schema)
            self.slen = 0
            self.sst = self.scon.start() if self.scon is not None else None
            return True
        if (c == "-" or c in _DIGITS) and (ok("number") or ok("integer")):
            self.integer = types is not None and "number" not in types
            self.nrule = _NumRule.of(schema, self.integer)
            if self.nrule is not None and not self.nrule.viable(c):
                return False
            self.tok = _NUM
            self.ntext = c
            self.num = _N_SIGN if c == "-" else (_N_ZERO if c == "0" else _N_INT)
            return True
        for lit, t in (("true", "boolean"), ("false", "boolean"), ("null", "null")):
            if c == lit[0] and ok(t):
                self.tok, self.lit, self.lpos = _LIT, lit, 1
                return True
        return False

    def _enum_char(self, c: str) -> bool:
        t = self.text + c
        live = [s for s in self.cands if s.startswith(t)]
        if live:
            self.text, self.cands = t, live
            return True
        if self.text in self.cands:      # the value ended; c belongs to what follows
            self.tok = _NONE
            self._end_value()
            return self._char(c)
        return False

    # -------------------------------------------------------------- characters
    def _char(self, c: str) -> bool:
        t = self.tok
        if t == _ENUM:
            return self._enum_char(c)
        if t == _STR:
            return self._str_char(c)
        if t == _ESC:
            if c == "u":
                self.tok, self.uni, self.uhex = _UNI, 4, ""
                return True
            if c in '"\\/bfnrt':
                self.tok = _STR
                return self._str_value_char(_JSON_ESC[c])
            return False
        if t == _UNI:
            if c not in "0123456789abcdefABCDEF":
                return False
            self.uni -= 1
            self.uhex += c
            if self.uni == 0:
                self.tok = _STR
                return self._str_value_char(chr(int(self.uhex, 16)))
            return True
        if t == _LIT:
            if c != self.lit[self.lpos]:
                return False
            self.lpos += 1
            if self.lpos == len(self.lit):
                self.tok = _NONE
                self._end_value()
            return True
        if t == _NUM:
            n = self.num
            if self.nrule is not None and (c in _DIGITS or c == "."):
                if not self.nrule.viable(self.ntext + c):
                    return False
            if c in _DIGITS:
                self.ntext += c
                if n == _N_SIGN:
                    self.num = _N_ZERO if c == "0" else _N_INT
                elif n == _N_ZERO:
                    return False
                elif n == _N_DOT:
                    self.num = _N_FRAC
                elif n in (_N_E, _N_ESIGN):
                    self.num = _N_EXP
                return True
            if not self.integer:
                if c == "." and n in (_N_ZERO, _N_INT):
                    self.num = _N_DOT
                    self.ntext += c
                    return True
                if c in "eE" and n in (_N_ZERO, _N_INT, _N_FRAC) and self.nrule is None:
                    self.num = _N_E
                    return True
                if c in "+-" and n == _N_E:
                    self.num = _N_ESIGN
                    return True
            if n not in _NUM_END_OK:
                return False
            if self.nrule is not None and not self.nrule.contains(Decimal(self.ntext)):
                return False
            self.tok = _NONE
            self.nrule = None
            self._end_value()
            if not self.stack:
                return c in _WS
        # between tokens
        if c in _WS:
            # one blank, or a newline and up to 8 blanks of indentation
            if self.exp == _VALUE and not self.stack:
                return False
            if self.ws >= 1 and not (self.ws < 9 and self.nl and c in " \t"):
                return False
            if self.ws == 0:
                self.nl = c == "\n"
            self.ws += 1
            return True
        self.ws = 0
        e = self.exp
        if e in (_DONE, _VALUE):
            return False                  # values start in feed_char
        if e == _ARR_FIRST:
            if c == "]" and self.stack[-1].can_close():
                self.stack.pop()
                self._end_value()
                return True
            return False
        if e in (_OBJ_FIRST, _OBJ_KEY):
            top = self.stack[-1]
            if c == '"' and top.can_add():
                self.tok, self.key, top.key = _STR, True, ""
                return True
            if e == _OBJ_FIRST and c == "}" and top.can_close():
                self.stack.pop()
                self._end_value()
                return True
            return False
        if e == _COLON:
            if c == ":":
                self.exp = _VALUE
                self.pending = self.stack[-1].value_schema()
                return True
            return False
        if e == _AFTER:
            top = self.stack[-1]
            if c == ",":
                if isinstance(top, _Obj):
                    if not top.can_add():
                        return False
                    self.exp = _OBJ_KEY
                else:
                    if not top.can_add():
                        return False
                    self.exp = _VALUE
                    self.pending = top.item_schema()
                return True
            if c == "}" and isinstance(top, _Obj) and top.can_close():
                self.stack.pop()
                self._end_value()
                return True
            if c == "]" and isinstance(top, _Arr) and top.can_close():
                self.stack.pop()
                self._end_value()
                return True
            return False
        return False

    def _str_char(self, c: str) -> bool:
        if self.key:
            top = self.stack[-1]
            if c == '"':
                if not top.key_ok(top.key, True):
                    return False
                top.seen.add(top.key)
                self.tok = _NONE
                self.exp = _COLON
                return True
            if c == "\\" or ord(c) < 0x20:
                return False              # keys are plain names here
            if not top.key_ok(top.key + c, False):
                return False
            top.key += c
            return True
        if c == '"':
            if self.scon is not None and not self.scon.complete(self.sst, self.slen):
                return False
            self.tok = _NONE
            self.scon = self.sst = None
            self._end_value()
        elif c == "\\":
            if self.scon is not None and self.escapes_blocked():
                return False
            self.tok = _ESC
        elif ord(c) < 0x20:
            return False
        else:
            return self._str_value_char(c)
        return True

    def escapes_blocked(self) -> bool:
        """No escape can start when the string is already at maxLength."""
        return self.scon.max_len is not None and self.slen >= self.scon.max_len

    def _str_value_char(self, ch: str) -> bool:
        """One decoded character of a string value, against its rules."""
        if self.scon is None:
            return True
        r = self.scon
        if r.max_len is not None and self.slen >= r.max_len:
            return False
        nxt = r.step(self.sst, ch)
        if nxt is None:
            return False
        self.sst, self.slen = nxt, self.slen + 1
        return True


_JSON_ESC = {'"': '"', "\\": "\\", "/": "/", "b": "\b", "f": "\f", "n": "\n", "r": "\r",
             "t": "\t"}


class _StrRule:
    """The constraints on one string value: patterns (`pattern` and a
    fixed-shape `format`, all of which must match) and the length bounds."""

    __slots__ = ("pats", "min_len", "max_len")

    @staticmethod
    def of(schema: dict) -> "_StrRule | None":
        pats = []
        for src in (schema.get("pattern"), FORMAT_PATTERNS.get(schema.get("format"))):
            if isinstance(src, str):
                p = compile_pattern(src)
                if p is not None:
                    pats.append(p)
        mn, mx = schema.get("minLength"), schema.get("maxLength")
        mn = mn if isinstance(mn, int) and mn > 0 else 0
        mx = mx if isinstance(mx, int) and mx >= 0 else None
        if not pats and not mn and mx is None:
            return None
        r = _StrRule()
        r.pats, r.min_len, r.max_len = tuple(pats), mn, mx
        return r

    def start(self):
        return tuple(p.start() for p in self.pats)

    def step(self, states, ch: str):
        out = []
        for p, st in zip(self.pats, states):
            n = p.step(st, ch)
            if not n:
                return None
            out.append(n)
        return tuple(out)

    def complete(self, states, n: int) -> bool:
        return n >= self.min_len and all(p.accepts(st) for p, st in zip(self.pats, states))


_NUM_PREFIX = __import__("re").compile(r"-?(\d+(\.\d*)?)?$")


def _dec(v):
    return Decimal(str(v)) if isinstance(v, (int, float)) and not isinstance(v, bool) else None


class _NumRule:
    """`minimum` / `maximum` (inclusive) and `exclusiveMinimum` /
    `exclusiveMaximum` (numbers, or draft-4 booleans) of one number."""

    __slots__ = ("lo", "lo_ex", "hi", "hi_ex", "integer")

    @staticmethod
    def of(schema: dict, integer: bool) -> "_NumRule | None":
        lo, hi = _dec(schema.get("minimum")), _dec(schema.get("maximum"))
        lo_ex = hi_ex = False
        xmin, xmax = schema.get("exclusiveMinimum"), schema.get("exclusiveMaximum")
        if xmin is True:
            lo_ex = lo is not None
        elif _dec(xmin) is not None and (lo is None or _dec(xmin) >= lo):
            lo, lo_ex = _dec(xmin), True
        if xmax is True:
            hi_ex = hi is not None
        elif _dec(xmax) is not None and (hi is None or _dec(xmax) <= hi):
            hi, hi_ex = _dec(xmax), True
        if lo is None and hi is None:
            return None
        r = _NumRule()
        r.lo, r.lo_ex, r.hi, r.hi_ex, r.integer = lo, lo_ex, hi, hi_ex, integer
        return r

    def contains(self, x: Decimal) -> bool:
        if self.lo is not None and (x < self.lo or (self.lo_ex and x == self.lo)):
            return False
        if self.hi is not None and (x > self.hi or (self.hi_ex and x == self.hi)):
            return False
        return True

    def _meets(self, a: Decimal, a_in: bool, b: Decimal | None, b_in: bool) -> bool:
        """Does the value interval from a to b (None: unbounded above) meet
        the allowed range?  a_in / b_in: whether the ends belong to it."""
        lo, lo_in = (a, a_in)
        if self.lo is not None and (self.lo > lo or (self.lo == lo and self.lo_ex)):
            lo, lo_in = self.lo, not self.lo_ex
        hi, hi_in = (b, b_in)
        if self.hi is not None and (hi is None or self.hi < hi or (self.hi == hi and self.hi_ex)):
            hi, hi_in = self.hi, not self.hi_ex
        if hi is None:
            return True
        return lo < hi or (lo == hi and lo_in and hi_in)

    def viable(self, text: str) -> bool:
        """Some completion of the number prefix `text` (sign, digits, an
        optional '.' and fraction digits) lies in the range."""
        if not _NUM_PREFIX.match(text):
            return True                    # not number syntax: the parser refuses it
        neg = text.startswith("-")
        body = text[1:] if neg else text
        if body == "":                     # just the sign: any magnitude
            return self._side(neg, [(Decimal(0), True, None, False)])
        ip, dot, fp = body.partition(".")
        if dot:
            a = Decimal(ip + "." + (fp or "0"))
            step = Decimal(1).scaleb(-len(fp)) if fp else Decimal(1)
            return self._side(neg, [(a, True, a + step, False)])
        I = Decimal(ip)
        if I == 0:                         # "0" or "0.xxx"
            return self._side(neg, [(Decimal(0), True, Decimal(0) if self.integer else Decimal(1),
                                     self.integer)])
        ivs = []
        bound = max(abs(v) for v in (self.lo, self.hi) if v is not None)
        m = 0
        while True:
            a = I.scaleb(m)
            b = (I + 1).scaleb(m)
            ivs.append((a, True, b - 1 if self.integer else b, self.integer))
            if a > bound:
                break
            m += 1
            if m > 400:
                break
        return self._side(neg, ivs)

    def _side(self, neg: bool, ivs) -> bool:
        """Magnitude intervals, mapped to values (negated for a '-' prefix)."""
        for a, a_in, b, b_in in ivs:
            if not neg:
                if self._meets(a, a_in, b, b_in):
                    return True
            else:
                lo, lo_in = (-b, b_in) if b is not None else (None, False)
                if lo is None:             # unbounded below
                    if self.lo is None:
                        return True
                    if self._meets(self.lo, not self.lo_ex, -a, a_in):
                        return True
                    continue
                if self._meets(lo, lo_in, -a, a_in):
                    return True
        return False


class SchemaPrefix:
    """The set of parses still open; same interface as json_guard.JsonPrefix
    (copy, feed, done)."""

    def __init__(self, schema: dict | None):
        p = _Parser()
        p.pending = schema if isinstance(schema, dict) else {}
        self.parsers = [p]
        self.top_object = True

    def copy(self) -> "SchemaPrefix":
        c = SchemaPrefix.__new__(SchemaPrefix)
        c.parsers = [p.copy() for p in self.parsers]
        c.top_object = self.top_object
        return c

    @property
    def done(self) -> bool:
        return any(p.done for p in self.parsers)

    def feed(self, s: str) -> bool:
        ps = self.parsers
        for ch in s:
            nxt = []
            for p in ps:
                nxt.extend(p.feed_char(ch))
            if not nxt:
                return False
            ps = nxt[:64]                 # alternatives still open (bounded)
        self.parsers = ps
        return True
