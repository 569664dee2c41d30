

def test_pre_tokenizer_patterns_by_family():
    """tokenizer.ggml.pre picks the family's split: Llama 3 groups digits in
    threes, Qwen 2 splits every digit, GPT-4o keeps contractions on the word
    and splits case runs, the GPT-2 list keeps digit runs whole."""
    import regex

    from swarmllm_b200.serve.tokenizer import PRE_TOKENIZERS, pre_split

    def split(name, text):
        return pre_split(text, [regex.compile(p) for p in PRE_TOKENIZERS[name]])
    assert split("llama-bpe", "x 12345") == ["x", " ", "123", "45"]
    assert split("qwen2", "x 123") == ["x", " ", "1", "2", "3"]
    assert split("gpt-4o", "it's HelloWorld") == ["it's", " Hello", "World"]
    assert split("gpt2", "a 12345!!") == ["a", " 12345", "!!"]
    assert split("qwen35", "naïve") == ["naïve"]          # the mark stays on its letter
    for name in PRE_TOKENIZERS:                   # every piece kept: the split is lossless
        t = "Hi  there,\n\n 42 café 你好!? x"
        assert "".join(split(name, t)) == t, name


def test_bpe_tokenizer_uses_the_gguf_pre_name():
    from swarmllm_b200.serve.tokenizer import BPETokenizer, _bytes_to_unicode
    b2u = _bytes_to_unicode()
    toks = [b2u[b] for b in range(256)] + [b2u[ord("1")] + b2u[ord("2")]]
    merges = [f"{b2u[ord('1')]} {b2u[ord('2')]}"]
    q = BPETokenizer(toks, merges, pre="qwen2")
    ll = BPETokenizer(toks, merges, pre="llama-bpe")
    assert q.pre == "qwen2" and ll.pre == "llama-bpe"
    assert len(q.encode("12", add_bos=False)) == 2         # single digits: no merge across them
    assert ll.encode("12", add_bos=False) == [256]         # one piece "12": merged
    assert q.decode(q.encode("a 12 b", add_bos=False)) == "a 12 b"
    assert BPETokenizer(toks, merges, pre="no-such-pre").pre == "llama3"


def _naive_spm(tok, text):
    """The definition: repeatedly merge the best-scoring adjacent pair
    (leftmost among equals) over the whole text; empty text has no pieces."""
    if not text:
        return []
    parts = list("▁" + text.replace(" ", "▁"))
    while True:
        best, bi = None, -1
        for i in range(len(parts) - 1):
            j = tok.vocab.get(parts[i] + parts[i + 1])
            if j is not None and (best is None or tok.scores[j] > best):
                best, bi = tok.scores[j], i
        if best is None:
            break
        parts[bi:bi + 2] = [parts[bi] + parts[bi + 1]]
    out = []
    for p in parts:
        out += [tok.vocab[p]] if p in tok.vocab else [tok.byte_ids.get(b, 0) for b in p.encode()]
    return out


def test_spm_heap_merge_matches_the_definition():
    import random

    from swarmllm_b200.serve.tokenizer import SPMTokenizer
    rng = random.Random(0)
    alpha = "ab c▁"
    pieces = set("abc▁")
    while len(pieces) < 60:
        pieces.add("".join(rng.choice("abc▁") for _ in range(rng.randint(2, 4))))
    toks = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)] + sorted(pieces)
    scores = [0.0] * 259 + [float(rng.randint(-5, 5)) for _ in sorted(pieces)]   # many ties
    tok = SPMTokenizer(toks, scores, 1, 2)
    for _ in range(300):
        text = "".join(rng.choice(alpha) for _ in range(rng.randint(0, 30)))
        assert tok.encode(text, add_bos=False) == _naive_spm(tok, text), text
    assert tok.decode(tok.encode("ab c", add_bos=True)) == "ab c"


def test_spm_special_tokens_stay_whole():
    from swarmllm_b200.serve.tokenizer import SPMTokenizer
    toks = (["<unk>", "<s>", "</s>", "<start_of_turn>"] + [f"<0x{b:02X}>" for b in range(256)]
            + ["▁", "h", "i", "▁h", "hi", "▁hi"])
    types = [2, 3, 3, 3] + [6] * 256 + [1] * 6
    scores = [0.0] * 260 + [0.0, 0.0, 0.0, 1.0, 2.0, 3.0]
    tok = SPMTokenizer(toks, scores, 1, 2, types)
    ids = tok.encode("<start_of_turn>hi", add_bos=False)
    assert ids[0] == 3 and ids[1:] == [tok.vocab["hi"]]
    assert tok.encode("hi", add_bos=False) == [tok.vocab["▁hi"]]


def test_bos_follows_the_files_rule():
    """A prompt starts with BOS as llama.cpp decides it: the declared
    add_bos_token, else SentencePiece yes, GPT-2 BPE only for the
    pre-tokenizers that ask for it; GLM's pre-tokenizer never."""
    from swarmllm_b200.serve.tokenizer import adds_bos, from_gguf_metadata
    spm, bpe = {"tokenizer.ggml.model": "llama"}, {"tokenizer.ggml.model": "gpt2"}
    assert adds_bos(spm) and not adds_bos({**spm, "tokenizer.ggml.add_bos_token": False})
    assert not adds_bos({**bpe, "tokenizer.ggml.pre": "qwen2"})
    assert adds_bos({**bpe, "tokenizer.ggml.pre": "llama-bpe"})
    assert not adds_bos({**bpe, "tokenizer.ggml.pre": "glm4", "tokenizer.ggml.add_bos_token": True})
    toks = ["<|endoftext|>", "a", "b", "ab"]
    md = {**bpe, "tokenizer.ggml.pre": "qwen2", "tokenizer.ggml.tokens": toks,
          "tokenizer.ggml.merges": ["a b"], "tokenizer.ggml.bos_token_id": 0,
          "tokenizer.ggml.eos_token_id": 0, "tokenizer.ggml.add_bos_token": False}
    tok = from_gguf_metadata(md, len(toks))
    assert tok.encode("ab") == [3]
    tok = from_gguf_metadata({**md, "tokenizer.ggml.add_bos_token": True}, len(toks))
    assert tok.encode("ab") == [0, 3]
