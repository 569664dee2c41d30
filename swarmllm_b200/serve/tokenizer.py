"""Tokenizers built from GGUF vocab metadata, plus a byte-level fallback.

* ``BPETokenizer``   GPT-2 style byte-level BPE (``tokenizer.ggml.model ==
                     "gpt2"``: Llama-3, Qwen, gpt-oss): tokens + merges ranks.
* ``SPMTokenizer``   SentencePiece-style unigram/BPE by scores
                     (``tokenizer.ggml.model == "llama"``): greedy
                     highest-score merge of "▁"-prefixed pieces, byte fallback.
* ``ByteTokenizer``  1 byte = 1 token id (+ offset), for random-init models
                     whose GGUF carries no vocabulary.

Reference: src/inference/tokenizer.rs:160,603,712,810 (BPE, SPM, Gemma-4).
The benchmarks feed token ids directly; tokenizers serve the HTTP API.
"""
from __future__ import annotations

import re

try:   # \p{L} / \p{N} classes for the pre-tokenizer patterns
    import regex as _rx
except ImportError:  # pragma: no cover -- the stdlib fallback keeps one pattern
    _rx = None


def _bytes_to_unicode() -> dict[int, str]:
    """The reversible byte -> printable-unicode map of byte-level BPE
    (published with GPT-2)."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + \
        list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return dict(zip(bs, (chr(c) for c in cs)))


class ByteTokenizer:
    def __init__(self, vocab_size: int = 32000, offset: int = 3, bos_id: int = 1, eos_id: int = 2):
        self.vocab_size, self.offset = vocab_size, offset
        self.bos_id, self.eos_id = bos_id, eos_id

    def encode(self, text: str, add_bos: bool = True) -> list[int]:
        ids = [b + self.offset for b in text.encode("utf-8")]
        return ([self.bos_id] if add_bos else []) + ids

    def decode(self, ids) -> str:
        bs = bytes(int(i) - self.offset for i in ids if self.offset <= int(i) < self.offset + 256)
        return bs.decode("utf-8", errors="replace")

    def token_str(self, i: int) -> str:
        return self.decode([i])


# Pre-tokenizer patterns (the public definitions of each tokenizer family: a
# BPE vocabulary only reproduces its training splits with the same pattern).
_APOS = r"(?:'[sS]|'[tT]|'[rR][eE]|'[vV][eE]|'[mM]|'[lL][lL]|'[dD])"
_PAT_GPT2 = r"'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+"
_PAT_LLAMA3 = (_APOS + r"|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"
               r"|\s*[\r\n]+|\s+(?!\S)|\s+")
_PAT_QWEN2 = (_APOS + r"|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"
              r"|\s*[\r\n]+|\s+(?!\S)|\s+")
# Qwen 3.5: combining marks stay with their letters
_PAT_QWEN35 = (_APOS + r"|[^\r\n\p{L}\p{N}]?[\p{L}\p{M}]+|\p{N}| ?[^\s\p{L}\p{M}\p{N}]+[\r\n]*"
               r"|\s*[\r\n]+|\s+(?!\S)|\s+")
_UP, _LO = r"[\p{Lu}\p{Lt}\p{Lm}\p{Lo}\p{M}]", r"[\p{Ll}\p{Lm}\p{Lo}\p{M}]"
# GPT-4o / o200k (gpt-oss, Llama 4): case runs split, digits in threes
_PAT_GPT4O = (r"[^\r\n\p{L}\p{N}]?" + _UP + "*" + _LO + "+" + _APOS + "?"
              r"|[^\r\n\p{L}\p{N}]?" + _UP + "+" + _LO + "*" + _APOS + "?"
              r"|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n/]*|\s*[\r\n]+|\s+(?!\S)|\s+")
# Mistral tekken: as GPT-4o without the contractions, single digits
_PAT_TEKKEN = (r"[^\r\n\p{L}\p{N}]?" + _UP + "*" + _LO + "+"
               r"|[^\r\n\p{L}\p{N}]?" + _UP + "+" + _LO + "*"
               r"|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n/]*|\s*[\r\n]+|\s+(?!\S)|\s+")

# tokenizer.ggml.pre -> patterns applied in sequence (each re-splits the
# previous pass's pieces)
PRE_TOKENIZERS = {
    **{k: (_PAT_LLAMA3,) for k in ("llama3", "llama-v3", "llama-bpe", "smaug-bpe", "dbrx",
                                   "falcon3", "pixtral", "glm4", "chatglm-bpe")},
    **{k: (_PAT_QWEN2,) for k in ("qwen2", "deepseek-r1-qwen", "stablelm2", "megrez", "hunyuan")},
    "qwen35": (_PAT_QWEN35,),
    **{k: (_PAT_GPT4O,) for k in ("gpt-4o", "llama4", "minimax-m2")},
    "tekken": (_PAT_TEKKEN,),
    **{k: (_PAT_GPT2,) for k in ("gpt-2", "gpt2", "phi-2", "olmo", "mpt", "roberta-bpe")},
    "default": (r"[\p{P}\$\+<=>\^~\|]+", _PAT_GPT2, r"\p{N}+", r"[0-9][0-9][0-9]"),
    **{k: (r"\p{N}", _PAT_GPT2) for k in ("starcoder", "refact", "command-r", "smollm")},
    "whitespace": (r"\S+|\s+",),
}


def pre_split(text: str, patterns) -> list[str]:
    """Split `text` by each compiled pattern in turn; the text between
    matches stays as its own piece, so nothing is dropped."""
    pieces = [text]
    for pat in patterns:
        out = []
        for piece in pieces:
            pos = 0
            for m in pat.finditer(piece):
                if m.start() > pos:
                    out.append(piece[pos:m.start()])
                if m.end() > m.start():
                    out.append(m.group())
                pos = m.end()
            if pos < len(piece):
                out.append(piece[pos:])
        pieces = out
    return pieces


class BPETokenizer:
    adds_bos = True   # the file's rule, set by from_gguf_metadata (adds_bos)
    # fallback pre-tokenizer (Llama 3 style) when the regex module is missing
    PAT = re.compile(r"""'(?:[sdmt]|ll|ve|re)| ?[^\W\d_]+| ?\d{1,3}| ?[^\s\w]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+""",
                     re.UNICODE)

    def __init__(self, tokens: list[str], merges: list[str], bos_id: int = -1, eos_id: int = -1,
                 token_types: list[int] | None = None, pre: str | None = None):
        """`pre`: the GGUF `tokenizer.ggml.pre` name (Llama 3's pattern when
        absent or unknown)."""
        self.pre = pre if pre in PRE_TOKENIZERS else "llama3"
        self.patterns = (tuple(_rx.compile(p) for p in PRE_TOKENIZERS[self.pre])
                         if _rx is not None else (self.PAT,))
        self.tokens = tokens
        self.vocab = {t: i for i, t in enumerate(tokens)}
        self.ranks = {}
        for r, m in enumerate(merges):
            a, _, b = m.partition(" ")
            self.ranks[(a, b)] = r
        self.b2u = _bytes_to_unicode()
        self.u2b = {v: k for k, v in self.b2u.items()}
        self.bos_id, self.eos_id = bos_id, eos_id
        self.special = {t: i for i, t in enumerate(tokens)
                        if token_types and token_types[i] in (3, 4)}  # control / user-defined
        self._cache: dict[str, list[int]] = {}
        self.vocab_size = len(tokens)

    def _bpe(self, word: str) -> list[int]:
        if word in self._cache:
            return self._cache[word]
        parts = list(word)
        while len(parts) > 1:
            best, bi = None, -1
            for i in range(len(parts) - 1):
                r = self.ranks.get((parts[i], parts[i + 1]))
                if r is not None and (best is None or r < best):
                    best, bi = r, i
            if best is None:
                break
            parts[bi:bi + 2] = [parts[bi] + parts[bi + 1]]
        ids = []
        for p in parts:
            if p in self.vocab:
                ids.append(self.vocab[p])
            else:  # unknown piece: fall back to its bytes
                ids.extend(self.vocab.get(ch, 0) for ch in p)
        self._cache[word] = ids
        return ids

    def encode(self, text: str, add_bos: bool = True) -> list[int]:
        ids = [self.bos_id] if (add_bos and self.adds_bos and self.bos_id >= 0) else []
        # split out special tokens first
        if self.special:
            pat = "(" + "|".join(re.escape(s) for s in sorted(self.special, key=len, reverse=True)) + ")"
            chunks = re.split(pat, text)
        else:
            chunks = [text]
        for ch in chunks:
            if not ch:
                continue
            if ch in self.special:
                ids.append(self.special[ch])
                continue
            for w in pre_split(ch, self.patterns):
                ids.extend(self._bpe("".join(self.b2u[b] for b in w.encode("utf-8"))))
        return ids

    def decode(self, ids) -> str:
        out = bytearray()
        for i in ids:
            i = int(i)
            if i < 0 or i >= len(self.tokens) or i in (self.bos_id, self.eos_id):
                continue
            t = self.tokens[i]
            if t in self.special:
                out += t.encode()
                continue
            for ch in t:
                b = self.u2b.get(ch)
                if b is not None:
                    out.append(b)
                else:
                    out += ch.encode()
        return out.decode("utf-8", errors="replace")

    def token_str(self, i: int) -> str:
        return self.decode([i])


class SPMTokenizer:
    """SentencePiece-style BPE over the whole text (a dummy-prefix '▁', spaces
    as '▁'): the highest-scoring adjacent pair that is a vocabulary entry merges
    first, leftmost among equals, with a heap of candidate pairs over a linked
    list of symbols (O(n log n)); pieces outside the vocabulary fall back to
    byte tokens <0xNN>.  Control and user-defined tokens (token types 3 / 4)
    in the text are matched whole first, as the BPE tokenizer does."""
    adds_bos = True   # the file's rule, set by from_gguf_metadata (adds_bos)

    def __init__(self, tokens: list[str], scores: list[float], bos_id: int = 1, eos_id: int = 2,
                 token_types: list[int] | None = None):
        self.tokens, self.scores = tokens, scores
        self.vocab = {t: i for i, t in enumerate(tokens)}
        self.bos_id, self.eos_id = bos_id, eos_id
        self.byte_ids = {}
        for i, t in enumerate(tokens):
            m = re.fullmatch(r"<0x([0-9A-Fa-f]{2})>", t)
            if m:
                self.byte_ids[int(m.group(1), 16)] = i
        self.special = {t: i for i, t in enumerate(tokens)
                        if token_types and i < len(token_types) and token_types[i] in (3, 4)
                        and i not in (bos_id, eos_id) and t}
        self.vocab_size = len(tokens)

    def _merge(self, text: str) -> list[int]:
        import heapq
        sym = list(text)
        n = len(sym)
        nxt = list(range(1, n + 1))
        prv = list(range(-1, n - 1))
        alive = [True] * n
        heap = []

        def push(i):
            j = nxt[i]
            if j < n:
                k = self.vocab.get(sym[i] + sym[j])
                if k is not None:
                    heapq.heappush(heap, (-self.scores[k], i, sym[i], sym[j]))
        for i in range(n - 1):
            push(i)
        while heap:
            _, i, a, b = heapq.heappop(heap)
            j = nxt[i] if i < n else n
            # stale: a side merged since this pair was pushed
            if not alive[i] or j >= n or sym[i] != a or sym[j] != b:
                continue
            sym[i] = a + b
            alive[j] = False
            nxt[i] = nxt[j]
            if nxt[j] < n:
                prv[nxt[j]] = i
            if prv[i] >= 0:
                push(prv[i])
            push(i)
        ids = []
        i = 0
        while i < n:
            p = sym[i]
            if p in self.vocab:
                ids.append(self.vocab[p])
            else:
                ids.extend(self.byte_ids.get(b, 0) for b in p.encode("utf-8"))
            i = nxt[i]
        return ids

    def encode(self, text: str, add_bos: bool = True) -> list[int]:
        ids = [self.bos_id] if add_bos and self.adds_bos and self.bos_id >= 0 else []
        if self.special:
            pat = "(" + "|".join(re.escape(t) for t in sorted(self.special, key=len, reverse=True)) + ")"
            chunks = re.split(pat, text)
        else:
            chunks = [text]
        first = True
        for ch in chunks:
            if not ch:
                continue
            if ch in self.special:
                ids.append(self.special[ch])
                first = False
                continue
            # the dummy prefix goes before the text's first piece only
            ids.extend(self._merge(("▁" if first else "") + ch.replace(" ", "▁")))
            first = False
        return ids

    def decode(self, ids) -> str:
        out = bytearray()
        for i in ids:
            i = int(i)
            if i in (self.bos_id, self.eos_id) or not (0 <= i < len(self.tokens)):
                continue
            t = self.tokens[i]
            m = re.fullmatch(r"<0x([0-9A-Fa-f]{2})>", t)
            if m:
                out.append(int(m.group(1), 16))
            else:
                out += t.replace("▁", " ").encode()
        s = out.decode("utf-8", errors="replace")
        return s[1:] if s.startswith(" ") else s

    def token_str(self, i: int) -> str:
        return self.decode([i])


# BPE pre-tokenizers whose prompts start with BOS when the file does not say,
# and those that never take one (llama.cpp's vocabulary rules)
_PRE_ADD_BOS = {"llama3", "llama-v3", "llama-bpe", "falcon3", "falcon-h1", "pixtral", "midm-2.0",
                "lfm2"}
_PRE_NO_BOS = {"glm4", "chatglm-bpe"}


def adds_bos(md: dict) -> bool:
    """Whether a prompt starts with BOS: the file's tokenizer.ggml.add_bos_token
    when present, else yes for a SentencePiece vocabulary and, for a GPT-2
    BPE one, only for the pre-tokenizers that ask for it; a pre-tokenizer
    without BOS overrides the key.  Qwen files, for one, name a BOS id but
    declare add_bos_token false.  Reference: split/gguf_meta.rs:1374."""
    model, pre = md.get("tokenizer.ggml.model"), md.get("tokenizer.ggml.pre", "")
    if pre in _PRE_NO_BOS:
        return False
    declared = md.get("tokenizer.ggml.add_bos_token")
    if declared is not None:
        return bool(declared)
    return model == "llama" or (model == "gpt2" and pre in _PRE_ADD_BOS)


def from_gguf_metadata(md: dict, vocab_size: int):
    model = md.get("tokenizer.ggml.model")
    toks = md.get("tokenizer.ggml.tokens")
    bos = int(md.get("tokenizer.ggml.bos_token_id", -1))
    eos = int(md.get("tokenizer.ggml.eos_token_id", -1))
    tok = None
    if toks and model == "gpt2":
        tok = BPETokenizer(toks, md.get("tokenizer.ggml.merges", []), bos, eos,
                           md.get("tokenizer.ggml.token_type"), md.get("tokenizer.ggml.pre"))
    elif toks and model == "llama":
        tok = SPMTokenizer(toks, md.get("tokenizer.ggml.scores", [0.0] * len(toks)), bos, eos,
                           md.get("tokenizer.ggml.token_type"))
    if tok is None:
        return ByteTokenizer(vocab_size)
    tok.adds_bos = adds_bos(md)
    return tok
