"""Prefix recognition for the regular expressions of JSON Schema `pattern`.

A pattern is parsed into a small syntax tree and compiled into a Thompson
NFA; a string is a live prefix while the set of NFA states it reaches is not
empty, and complete when that set holds the accepting state.  Every state of
an NFA built this way can still reach acceptance (character classes are
never empty), so a prefix the set accepts can always be finished.

Syntax (the ECMA-262 subset JSON Schema patterns use): literals and escaped
metacharacters, `.`, classes `[...]` / `[^...]` with ranges, `\\d \\w \\s`
and their negations, groups `( )` / `(?: )`, alternation `|`, quantifiers
`* + ? {n} {n,} {n,m}` (a trailing `?` for laziness is read and ignored, as
laziness does not change which strings match), and `^` / `$` at the ends.
JSON Schema patterns are not anchored: without `^` the match may start
anywhere (a leading `.*`), without `$` it may end anywhere.  Back-references,
look-around and anchors in the middle are not supported: `compile_pattern`
raises `Unsupported` and the caller leaves the pattern unenforced.

Reference behaviour: structured replies through a grammar compiled from the
schema (src/inference/reply_grammar.rs:90,156).
"""
from __future__ import annotations

MAX_STATES = 20000


class Unsupported(ValueError):
    pass


# a character set: (negated, ((lo, hi), ...)) over code points
_DIGIT = ((ord("0"), ord("9")),)
_WORD = ((ord("0"), ord("9")), (ord("A"), ord("Z")), (ord("a"), ord("z")), (ord("_"), ord("_")))
_SPACE = tuple((ord(c), ord(c)) for c in " \t\n\r\f\v") + ((0xA0, 0xA0), (0x2028, 0x2029))
_ANY_BUT_NL = (True, ((10, 10), (13, 13)))
_ESCAPES = {"n": "\n", "t": "\t", "r": "\r", "f": "\f", "v": "\v", "0": "\0"}


def _in(cs, ch: str) -> bool:
    neg, ranges = cs
    o = ord(ch)
    hit = any(lo <= o <= hi for lo, hi in ranges)
    return hit != neg


class _Reader:
    def __init__(self, s: str):
        self.s, self.i = s, 0

    def peek(self):
        return self.s[self.i] if self.i < len(self.s) else None

    def take(self):
        c = self.peek()
        if c is None:
            raise Unsupported("pattern ends early")
        self.i += 1
        return c


def _class_escape(c: str):
    """The set of an escape inside or outside a class, or None for a literal."""
    if c in "dD":
        return (c == "D", _DIGIT)
    if c in "wW":
        return (c == "W", _WORD)
    if c in "sS":
        return (c == "S", _SPACE)
    return None


def _escape_char(r: _Reader) -> str:
    c = r.take()
    if c in _ESCAPES:
        return _ESCAPES[c]
    if c == "u":
        h = "".join(r.take() for _ in range(4))
        try:
            return chr(int(h, 16))
        except ValueError:
            raise Unsupported("bad \\u escape") from None
    if c == "x":
        h = r.take() + r.take()
        try:
            return chr(int(h, 16))
        except ValueError:
            raise Unsupported("bad \\x escape") from None
    if c.isalnum():
        raise Unsupported(f"escape \\{c}")     # \b, \1, \p{..}, ...
    return c


def _parse_class(r: _Reader):
    neg = r.peek() == "^"
    if neg:
        r.take()
    ranges, first = [], True
    while True:
        c = r.take()
        if c == "]" and not first:
            break
        first = False
        if c == "\\":
            e = r.peek()
            cs = _class_escape(e) if e is not None else None
            if cs is not None:
                r.take()
                if cs[0]:
                    raise Unsupported("negated escape inside a class")
                ranges.extend(cs[1])
                continue
            c = _escape_char(r)
        lo = ord(c)
        if r.peek() == "-" and r.i + 1 < len(r.s) and r.s[r.i + 1] != "]":
            r.take()
            d = r.take()
            if d == "\\":
                d = _escape_char(r)
            hi = ord(d)
            if hi < lo:
                raise Unsupported("reversed range")
            ranges.append((lo, hi))
        else:
            ranges.append((lo, lo))
    return ("set", (neg, tuple(ranges)))


def _parse_alt(r: _Reader, depth: int):
    items = [_parse_seq(r, depth)]
    while r.peek() == "|":
        r.take()
        items.append(_parse_seq(r, depth))
    return items[0] if len(items) == 1 else ("alt", items)


def _parse_seq(r: _Reader, depth: int):
    items = []
    while True:
        c = r.peek()
        if c is None or c == "|" or (c == ")" and depth > 0):
            break
        atom = _parse_atom(r, depth)
        items.append(_parse_quant(r, atom))
    return ("cat", items)


def _parse_atom(r: _Reader, depth: int):
    c = r.take()
    if c == "(":
        if r.peek() == "?":
            r.take()
            if r.take() != ":":
                raise Unsupported("look-around or named group")
        node = _parse_alt(r, depth + 1)
        if r.take() != ")":
            raise Unsupported("unbalanced group")
        return node
    if c == "[":
        return _parse_class(r)
    if c == ".":
        return ("set", _ANY_BUT_NL)
    if c == "\\":
        e = r.peek()
        cs = _class_escape(e) if e is not None else None
        if cs is not None:
            r.take()
            return ("set", cs)
        ch = _escape_char(r)
        return ("set", (False, ((ord(ch), ord(ch)),)))
    if c in "^$":
        raise Unsupported("anchor inside the pattern")
    if c in "*+?{" :
        if c == "{" and not _looks_like_count(r):
            return ("set", (False, ((ord(c), ord(c)),)))
        raise Unsupported("quantifier without an operand")
    if c == ")":
        raise Unsupported("unbalanced group")
    return ("set", (False, ((ord(c), ord(c)),)))


def _looks_like_count(r: _Reader) -> bool:
    j = r.s.find("}", r.i)
    if j < 0:
        return False
    body = r.s[r.i:j]
    parts = body.split(",")
    return 1 <= len(parts) <= 2 and parts[0].isdigit() and all(p.isdigit() or p == "" for p in parts[1:])


def _parse_quant(r: _Reader, atom):
    while True:
        c = r.peek()
        if c == "*":
            lo, hi = 0, None
        elif c == "+":
            lo, hi = 1, None
        elif c == "?":
            lo, hi = 0, 1
        elif c == "{" and _looks_like_count_at(r):
            r.take()
            j = r.s.index("}", r.i)
            parts = r.s[r.i:j].split(",")
            r.i = j
            lo = int(parts[0])
            hi = lo if len(parts) == 1 else (int(parts[1]) if parts[1] else None)
            if hi is not None and hi < lo:
                raise Unsupported("bad count")
        else:
            return atom
        r.take()
        if r.peek() == "?":        # lazy: the same strings match
            r.take()
        atom = ("rep", atom, lo, hi)


def _looks_like_count_at(r: _Reader) -> bool:
    save = r.i
    r.i += 1
    ok = _looks_like_count(r)
    r.i = save
    return ok


class _Nfa:
    """Thompson NFA: per state, its character edges and its epsilon edges."""

    def __init__(self):
        self.edges: list[list] = []     # [(charset, next)]
        self.eps: list[list[int]] = []

    def state(self) -> int:
        if len(self.edges) >= MAX_STATES:
            raise Unsupported("pattern too large")
        self.edges.append([])
        self.eps.append([])
        return len(self.edges) - 1

    def build(self, node) -> tuple[int, int]:
        kind = node[0]
        if kind == "set":
            a, b = self.state(), self.state()
            self.edges[a].append((node[1], b))
            return a, b
        if kind == "cat":
            a = b = self.state()
            for it in node[1]:
                s, e = self.build(it)
                self.eps[b].append(s)
                b = e
            return a, b
        if kind == "alt":
            a, b = self.state(), self.state()
            for it in node[1]:
                s, e = self.build(it)
                self.eps[a].append(s)
                self.eps[e].append(b)
            return a, b
        # rep: lo mandatory copies, then (hi - lo) optional ones or a loop
        _, sub, lo, hi = node
        a = b = self.state()
        for _ in range(lo):
            s, e = self.build(sub)
            self.eps[b].append(s)
            b = e
        if hi is None:
            s, e = self.build(sub)
            self.eps[b].append(s)
            self.eps[e].append(s)
            end = self.state()
            self.eps[b].append(end)
            self.eps[e].append(end)
            return a, end
        end = self.state()
        for _ in range(hi - lo):
            s, e = self.build(sub)
            self.eps[b].append(s)
            self.eps[b].append(end)
            b = e
        self.eps[b].append(end)
        return a, end


class Pattern:
    """A compiled pattern: `start()` gives the state set before any
    character, `step(states, ch)` the set after one (empty: dead), and
    `accepts(states)` whether the string so far matches."""

    def __init__(self, source: str):
        self.source = source
        s = source
        anchored_start = s.startswith("^")
        if anchored_start:
            s = s[1:]
        anchored_end = s.endswith("$") and not s.endswith("\\$")
        if anchored_end:
            s = s[:-1]
        r = _Reader(s)
        tree = _parse_alt(r, 0)
        if r.peek() is not None:
            raise Unsupported("unbalanced group")
        anything = ("rep", ("set", (True, ())), 0, None)
        parts = ([] if anchored_start else [anything]) + [tree] + ([] if anchored_end else [anything])
        self.nfa = _Nfa()
        self.s0, self.acc = self.nfa.build(("cat", parts))
        self._start = self._closure({self.s0})

    def _closure(self, states) -> frozenset:
        out, todo = set(states), list(states)
        eps = self.nfa.eps
        while todo:
            for n in eps[todo.pop()]:
                if n not in out:
                    out.add(n)
                    todo.append(n)
        return frozenset(out)

    def start(self) -> frozenset:
        return self._start

    def step(self, states: frozenset, ch: str) -> frozenset:
        edges = self.nfa.edges
        nxt = {n for s in states for cs, n in edges[s] if _in(cs, ch)}
        return self._closure(nxt) if nxt else frozenset()

    def accepts(self, states: frozenset) -> bool:
        return self.acc in states

    def fullmatch(self, text: str) -> bool:
        st = self.start()
        for ch in text:
            st = self.step(st, ch)
            if not st:
                return False
        return self.accepts(st)


# JSON Schema `format` values with a fixed shape, as anchored patterns
FORMAT_PATTERNS = {
    "date": r"^\d{4}-(0[1-9]|1[0-2])-(0[1-9]|[12]\d|3[01])$",
    "time": r"^([01]\d|2[0-3]):[0-5]\d:([0-5]\d|60)(\.\d+)?([Zz]|[+-]([01]\d|2[0-3]):[0-5]\d)$",
    "date-time": r"^\d{4}-(0[1-9]|1[0-2])-(0[1-9]|[12]\d|3[01])[Tt ]([01]\d|2[0-3]):[0-5]\d:"
                 r"([0-5]\d|60)(\.\d+)?([Zz]|[+-]([01]\d|2[0-3]):[0-5]\d)$",
    "uuid": r"^[0-9a-fA-F]{8}-[0-9a-fA-F]{4}-[0-9a-fA-F]{4}-[0-9a-fA-F]{4}-[0-9a-fA-F]{12}$",
    "ipv4": r"^((25[0-5]|2[0-4]\d|1\d\d|[1-9]?\d)\.){3}(25[0-5]|2[0-4]\d|1\d\d|[1-9]?\d)$",
    "email": r"^[A-Za-z0-9._%+-]+@[A-Za-z0-9-]+(\.[A-Za-z0-9-]+)+$",
}

_CACHE: dict[str, Pattern | None] = {}


def compile_pattern(source: str) -> Pattern | None:
    """The compiled pattern, or None when it uses syntax outside the subset
    (it is then left unenforced).  Compiled patterns are cached."""
    if source not in _CACHE:
        try:
            _CACHE[source] = Pattern(source)
        except (Unsupported, IndexError, ValueError):
            _CACHE[source] = None
    return _CACHE[source]
