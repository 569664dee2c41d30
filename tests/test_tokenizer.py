

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
