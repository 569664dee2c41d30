"""JSON-constrained decoding for `response_format` json_object / json_schema.

`JsonPrefix` is an incremental JSON recogniser: it accepts text one character
at a time and refuses the first character after which no completion to a
valid JSON value exists.  `JsonConstraint` applies it per request inside the
engine step: of the sampled row's candidates (the drawn token first, then the
others by logit) it keeps the first whose text leaves the output a valid JSON
prefix; the end-of-sequence token is allowed only once the top-level value is
complete, and forced then.  The output is therefore always a prefix of valid
JSON, and valid JSON when the model stops on its own.  With a json_schema the
recogniser is schema_guard.SchemaPrefix, which also enforces the schema's
types, keys, required properties, items, enums and alternatives.

Reference behaviour: reply grammar via llguidance (src/inference/reply_grammar.rs:156,240).
"""
from __future__ import annotations

_WS = " \t\n\r"
_LITERALS = ("true", "false", "null")

# expectation states
_VALUE, _OBJ_FIRST, _OBJ_KEY, _COLON, _AFTER, _ARR_FIRST, _DONE = range(7)
# token states
_NONE, _STR, _ESC, _UNI, _NUM, _LIT = range(6)
# number sub-states
_N_SIGN, _N_ZERO, _N_INT, _N_DOT, _N_FRAC, _N_E, _N_ESIGN, _N_EXP = range(8)
_NUM_END_OK = (_N_ZERO, _N_INT, _N_FRAC, _N_EXP)


class JsonPrefix:
    __slots__ = ("stack", "exp", "tok", "key", "uni", "num", "lit", "lpos", "top_object")

    def __init__(self, top_object: bool = True):
        self.stack: list[str] = []      # open containers: '{' or '['
        self.exp = _VALUE
        self.tok = _NONE
        self.key = False                # the string being read is an object key
        self.uni = 0                    # hex digits left in a \\u escape
        self.num = _N_INT
        self.lit = ""
        self.lpos = 0
        self.top_object = top_object

    def copy(self) -> "JsonPrefix":
        c = JsonPrefix.__new__(JsonPrefix)
        c.stack = list(self.stack)
        for f in ("exp", "tok", "key", "uni", "num", "lit", "lpos", "top_object"):
            setattr(c, f, getattr(self, f))
        return c

    @property
    def done(self) -> bool:
        """A complete top-level value has been read (only whitespace may follow)."""
        return self.exp == _DONE and self.tok == _NONE

    def _end_value(self):
        self.exp = _AFTER if self.stack else _DONE

    def feed(self, s: str) -> bool:
        for ch in s:
            if not self._char(ch):
                return False
        return True

    def _char(self, c: str) -> bool:
        t = self.tok
        if t == _STR:
            if c == '"':
                self.tok = _NONE
                if self.key:
                    self.exp = _COLON
                else:
                    self._end_value()
            elif c == "\\":
                self.tok = _ESC
            elif ord(c) < 0x20:
                return False
            return True
        if t == _ESC:
            if c == "u":
                self.tok, self.uni = _UNI, 4
            elif c in '"\\/bfnrt':
                self.tok = _STR
            else:
                return False
            return True
        if t == _UNI:
            if c not in "0123456789abcdefABCDEF":
                return False
            self.uni -= 1
            if self.uni == 0:
                self.tok = _STR
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
            if c.isdigit():
                if n == _N_SIGN:
                    self.num = _N_ZERO if c == "0" else _N_INT
                elif n == _N_ZERO:
                    return False            # no leading zeros
                elif n == _N_DOT:
                    self.num = _N_FRAC
                elif n in (_N_E, _N_ESIGN):
                    self.num = _N_EXP
                return True
            if c == "." and n in (_N_ZERO, _N_INT):
                self.num = _N_DOT
                return True
            if c in "eE" and n in (_N_ZERO, _N_INT, _N_FRAC):
                self.num = _N_E
                return True
            if c in "+-" and n == _N_E:
                self.num = _N_ESIGN
                return True
            if n not in _NUM_END_OK:
                return False
            self.tok = _NONE               # the number ended; c starts what follows
            self._end_value()
            if not self.stack:             # a top-level number is closed by anything
                return c in _WS
        # between tokens
        if c in _WS:
            return True
        e = self.exp
        if e == _DONE:
            return False
        if e in (_VALUE, _ARR_FIRST):
            if e == _ARR_FIRST and c == "]":
                self.stack.pop()
                self._end_value()
                return True
            top = not self.stack
            if top and self.top_object and c != "{":
                return False
            if c == "{":
                self.stack.append("{")
                self.exp = _OBJ_FIRST
            elif c == "[":
                self.stack.append("[")
                self.exp = _ARR_FIRST
            elif c == '"':
                self.tok, self.key = _STR, False
            elif c == "-" or c.isdigit():
                self.tok = _NUM
                self.num = _N_SIGN if c == "-" else (_N_ZERO if c == "0" else _N_INT)
            else:
                for lit in _LITERALS:
                    if lit[0] == c:
                        self.tok, self.lit, self.lpos = _LIT, lit, 1
                        return True
                return False
            return True
        if e in (_OBJ_FIRST, _OBJ_KEY):
            if c == '"':
                self.tok, self.key = _STR, True
                return True
            if e == _OBJ_FIRST and c == "}":
                self.stack.pop()
                self._end_value()
                return True
            return False
        if e == _COLON:
            if c == ":":
                self.exp = _VALUE
                return True
            return False
        if e == _AFTER:
            top = self.stack[-1]
            if c == ",":
                self.exp = _OBJ_KEY if top == "{" else _VALUE
                return True
            if (c == "}" and top == "{") or (c == "]" and top == "["):
                self.stack.pop()
                self._end_value()
                return True
            return False
        return False


class JsonConstraint:
    """Per-request state of JSON-constrained decoding (JSON syntax, or a JSON
    schema when one is given)."""

    def __init__(self, piece, eos_id: int, top_object: bool = True, schema: dict | None = None):
        self.piece = piece              # token id -> its text
        self.eos = eos_id
        self.schema = schema
        if schema is not None:
            from .schema_guard import SchemaPrefix
            self.state = SchemaPrefix(schema)
        else:
            self.state = JsonPrefix(top_object)

    def fresh(self) -> "JsonConstraint":
        """The same constraint from the start (one per request)."""
        return JsonConstraint(self.piece, self.eos, self.state.top_object, self.schema)

    def allowed(self, tok: int) -> bool:
        if tok == self.eos:
            return self.state.done
        if self.state.done:
            return False
        s = self.piece(tok)
        return bool(s) and self.state.copy().feed(s)

    def choose(self, drawn: int, candidates) -> int | None:
        """The drawn token if allowed, else the first allowed candidate (the
        candidates come in descending logit order); None if none is."""
        if self.state.done and self.eos >= 0:
            return self.eos
        if self.allowed(drawn):
            return drawn
        for t in candidates:
            t = int(t)
            if self.allowed(t):
                return t
        return None

    def accept(self, tok: int):
        if tok != self.eos:
            self.state.feed(self.piece(tok))
