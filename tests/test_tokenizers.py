"""Tokenizers beyond byte fallback: byte-level BPE and SentencePiece.

Each test restates one of the reference's tokenizer unit tests
(crates/det-token/src/lib.rs, cited by line) through GGUF tokenizer
metadata, the way Tokenizer::from_gguf (lib.rs:86-132) receives it, and runs
it on every implementation: the C oracle (oracle/ref_token.c) and the
library's own host tokenizer (det_tokenize, which needs no GPU).  A random
cross-check then compares the two on synthetic vocabularies.
"""
import numpy as np
import pytest

from detllm_b200 import synth as S


def gpt2_char(b: int) -> str:
    """gpt2_byte_unicode_token_bytes (lib.rs:1608-1633) as a string."""
    def printable(c):
        return 33 <= c <= 126 or 161 <= c <= 172 or 174 <= c <= 255
    if printable(b):
        return chr(b)
    n = sum(1 for c in range(b) if not printable(c))
    return chr(256 + n)


GPT2_BYTES = [gpt2_char(b) for b in range(256)]
SPACE = "▁"  # the SentencePiece space marker


class Impl:
    def __init__(self, name):
        self.name = name
        if name == "oracle":
            from oracle import oracle as O

            O.build()
            self.kind, self.tok, self.detok, self.err = O.tokenizer_kind, O.tokenize, O.detokenize, O.OracleError
        else:
            import detllm_b200 as D

            self.kind, self.tok, self.detok, self.err = (D.tokenizer_kind, D.tokenize, D.detokenize, D.DetError)

    def tokenize(self, g, data):
        return [int(t) for t in self.tok(g, data)]

    def codec(self, g, data):
        return [int(t) for t in self.tok(g, data, codec=True)]


@pytest.fixture(scope="module", params=["oracle", "product"])
def impl(request):
    return Impl(request.param)


def gguf(tokens, **kw):
    return S.gguf_metadata(S.tokenizer_kvs(tokens, **kw))


def test_bpe_merges_by_rank_then_leftmost_position(impl):  # lib.rs:920-943
    toks = S.byte_tokens() + ["ab", "ba", "aba"]
    ab, aba = 256, 258
    g = gguf(toks, merges=["<0x61> <0x62>", "<0x62> <0x61>", "ab <0x61>"])
    assert impl.kind(g) == "byte_bpe"
    assert impl.tokenize(g, b"ab") == [ab]
    assert impl.tokenize(g, b"aba") == [aba]
    assert impl.tokenize(g, b"baba") == [ord("b"), aba]
    assert impl.detok(g, [aba]) == b"aba"


def rank_scan(tokens, merges, data):
    """tokenize_bpe_by_rank_scan (lib.rs:1576-1606): repeatedly merge the
    leftmost pair of the lowest rank (byte tokens + plain ASCII pieces)."""
    def piece(t):
        return bytes([int(t[3:5], 16)]) if t.startswith("<0x") else t.encode()
    ids_of = {piece(t): i for i, t in enumerate(tokens)}
    ranks = {}
    for r, m in enumerate(merges):
        left, right = m.split(" ")
        ranks[(ids_of[piece(left)], ids_of[piece(right)])] = (r, ids_of[piece(left) + piece(right)])
    ids = [ids_of[bytes([b])] for b in data]
    while True:
        best = None
        for i in range(len(ids) - 1):
            if (ids[i], ids[i + 1]) in ranks:
                r, mid = ranks[(ids[i], ids[i + 1])]
                if best is None or r < best[0]:
                    best = (r, i, mid)
        if best is None:
            return ids
        ids[best[1]] = best[2]
        del ids[best[1] + 1]


def test_bpe_priority_queue_matches_rank_scan(impl):  # lib.rs:946-970
    toks = S.byte_tokens() + ["aa", "aaa", "aaaa", "ab", "ba", "aba", "abab", "baba"]
    merges = ["<0x61> <0x61>", "aa <0x61>", "aaa <0x61>", "<0x61> <0x62>", "<0x62> <0x61>", "ab <0x61>", "ab ab",
              "ba ba"]
    g = gguf(toks, merges=merges)
    for data in [b"aaaaa", b"abababa", b"bababaa", b"aaabaaa"]:
        assert impl.tokenize(g, data) == rank_scan(toks, merges, data), data


def test_bpe_rejects_duplicate_or_malformed_merges(impl):  # lib.rs:973-989
    toks = S.byte_tokens() + ["ab"]
    with pytest.raises(impl.err):
        impl.kind(gguf(toks, merges=["<0x61> <0x62>", "<0x61> <0x62>"]))
    for m in ["<0x61>", "<0x61>  <0x62>", "<0x61> <0x62> extra"]:
        with pytest.raises(impl.err):
            impl.kind(gguf(toks, merges=[m]))


def test_bpe_rejects_duplicate_tokens(impl):  # lib.rs:992-1010
    with pytest.raises(impl.err):  # "A" duplicates <0x41>
        impl.kind(gguf(S.byte_tokens() + ["A"], model="gpt2"))
    with pytest.raises(impl.err):
        impl.kind(gguf(S.byte_tokens() + ["ab", "ab"], model="gpt2"))


def test_from_gguf_prefers_bpe_when_merges_exist(impl):  # lib.rs:1013-1029
    g = gguf(S.byte_tokens() + ["ab"], merges=["<0x61> <0x62>"])
    assert impl.tokenize(g, b"ab") == [256]


def test_from_gguf_uses_gpt2_model_without_merges(impl):  # lib.rs:1032-1052
    g = gguf(GPT2_BYTES, model="gpt2")
    assert impl.kind(g) == "byte_bpe"
    data = b"\x00A \xff\n"
    assert impl.detok(g, impl.tokenize(g, data)) == data


def test_from_gguf_rejects_unknown_model(impl):  # lib.rs:1055-1070
    with pytest.raises(impl.err):
        impl.kind(gguf(S.byte_tokens(), model="unsupported"))


def test_bpe_does_not_emit_control_tokens(impl):  # lib.rs:1075-1100
    toks = S.byte_tokens() + ["ab"]
    types = [6] * len(toks)
    types[256] = 3
    g = gguf(toks, merges=["<0x61> <0x62>"], token_type=types)
    assert impl.tokenize(g, b"ab") == [97, 98]
    assert impl.detok(g, [256]) == b"ab"


def test_byte_fallback_codec_escapes_nonemittable_bytes(impl):  # lib.rs:1120-1147
    types = [6] * 256
    types[0xFF] = 3
    g = gguf(S.byte_tokens(), token_type=types)
    assert impl.kind(g) == "byte_fallback"
    assert impl.codec(g, bytes([0xFE, 0xFF])) == [0xFE, 256 + 0xFF]
    with pytest.raises(impl.err):
        impl.tokenize(g, bytes([0xFF]))
    assert impl.detok(g, [0xFF]) == b"\xff"


HELLO_TOKENS = GPT2_BYTES + ["he", "hel", "hell", "hello", "helloĠ"]
HELLO_MERGES = ["h e", "he l", "hel l", "hell o", "hello Ġ"]


def test_bpe_decodes_gpt2_byte_unicode_tokens(impl):  # lib.rs:1150-1177
    g = gguf(HELLO_TOKENS, merges=HELLO_MERGES)
    assert impl.tokenize(g, b"hello ") == [260]
    assert impl.detok(g, [260]) == b"hello "
    assert impl.tokenize(g, b"\n") == [10]


def test_bpe_round_trips_all_byte_values(impl):  # lib.rs:1180-1202
    g = gguf(HELLO_TOKENS, merges=HELLO_MERGES)
    every = bytes(range(256))
    assert impl.detok(g, impl.tokenize(g, every)) == every
    data = b"\x00hello \xff\nhello "
    assert impl.detok(g, impl.tokenize(g, data)) == data


def test_bpe_partial_byte_seed(impl):  # lib.rs:1205-1247
    g = gguf(GPT2_BYTES[:255] + ["hi"], merges=["h i"])
    assert impl.tokenize(g, b"hi") == [255]
    assert impl.detok(g, [255]) == b"hi"
    with pytest.raises(impl.err):
        impl.tokenize(g, b"\xff")
    # codec symbols escape the byte without a token
    assert impl.codec(g, b"hi\xff!") == [255, 256 + 0xFF, ord("!")]


def spm(tokens, scores=None, model="llama", **kw):
    return gguf(tokens, model=model, scores=scores, **kw)


def test_spm_longest_piece_and_space_marker(impl):  # lib.rs:1283-1297
    toks = S.byte_tokens() + [SPACE + "hello"]
    scores = [0.0] * len(toks)
    scores[256] = 10.0
    g = spm(toks, scores)
    assert impl.kind(g) == "sentencepiece"
    assert impl.tokenize(g, b" hello!") == [256, ord("!")]
    assert impl.detok(g, [256]) == b" hello"


def test_spm_round_trips_all_byte_values(impl):  # lib.rs:1300-1313
    toks = S.byte_tokens() + [SPACE + "hello"]
    scores = [0.0] * len(toks)
    scores[256] = 10.0
    g = spm(toks, scores)
    every = bytes(range(256))
    assert impl.detok(g, impl.tokenize(g, every)) == every
    data = b"\x00 hello\xff\n hello"
    assert impl.detok(g, impl.tokenize(g, data)) == data


def test_spm_duplicate_piece_ties(impl):  # lib.rs:1316-1337
    toks = S.byte_tokens() + [SPACE + "x", SPACE + "x", SPACE + "y", SPACE + "y"]
    scores = [0.0] * len(toks)
    scores[256], scores[257], scores[258], scores[259] = 1.0, 2.0, 3.0, 3.0
    g = spm(toks, scores)
    assert impl.tokenize(g, b" x") == [257]
    assert impl.tokenize(g, b" y") == [258]


def test_spm_rejects_malformed_scores(impl):  # lib.rs:1340-1355, 1524-1563
    toks = S.byte_tokens()
    with pytest.raises(impl.err):
        impl.kind(spm(toks, [0.0] * 255))
    with pytest.raises(impl.err):
        impl.kind(spm(toks, [0.0] * 17 + [float("inf")] + [0.0] * 238))
    with pytest.raises(impl.err):  # scores select SentencePiece without a model key
        impl.kind(spm(toks, [0.0] * 255, model=None))
    with pytest.raises(impl.err):
        impl.kind(spm(toks, [0.0] * 17 + [float("nan")] + [0.0] * 238, model=None))


def test_spm_selection(impl):  # lib.rs:1358-1397
    toks = S.byte_tokens() + [SPACE + "hello"]
    g = spm(toks)  # model "llama", no scores
    assert impl.kind(g) == "sentencepiece"
    assert impl.tokenize(g, b" hello") == [256]
    g = spm(toks, [0.0] * len(toks), model=None)  # scores only
    assert impl.kind(g) == "sentencepiece"
    assert impl.tokenize(g, b" hello") == [256]


def test_spm_control_and_nonemittable_tokens(impl):  # lib.rs:1400-1465
    toks = S.byte_tokens() + [SPACE + "hello"]
    types = [6] * len(toks)
    types[256] = 3
    g = spm(toks, token_type=types)
    assert impl.tokenize(g, b" hello") != [256]
    assert impl.detok(g, [256]) == b" hello"
    types = [6] * 256
    types[0xFF] = 3
    g = spm(S.byte_tokens(), token_type=types)
    assert impl.codec(g, bytes([0xFE, 0xFF])) == [0xFE, 256 + 0xFF]
    with pytest.raises(impl.err):
        impl.tokenize(g, bytes([0xFF]))
    assert impl.detok(g, [0xFF]) == b"\xff"


def test_rejects_bad_token_types(impl):  # lib.rs:1468-1521
    with pytest.raises(impl.err):
        impl.kind(gguf(S.byte_tokens(), token_type=[6] * 255))
    for v in (-1, 0, 7):
        with pytest.raises(impl.err):
            impl.kind(gguf(S.byte_tokens(), token_type=[v] * 256))
    kv = S.tokenizer_kvs(S.byte_tokens()) + [("tokenizer.ggml.token_type", S.GV_ARRAY, (S.GV_U32, [7] * 256))]
    with pytest.raises(impl.err):
        impl.kind(S.gguf_metadata(kv))


@pytest.mark.parametrize("kind", ["spm", "bpe"])
def test_synthetic_vocab_round_trip_and_oracle_agreement(impl, kind):
    """A seeded vocabulary of frequent pieces of Markov text (the one the GPU
    codec tests use): tokens of impl == tokens of the oracle, and
    detokenize(tokenize(x)) == x."""
    from oracle import oracle as O

    g = S.gguf_metadata(S.synthetic_tokenizer_kvs(kind, 700, seed=5))
    data = S.markov_text(4000, seed=5) + bytes(range(256))
    want = O.tokenize(g, data, codec=True)
    got = impl.codec(g, data)
    assert got == [int(t) for t in want]
    assert impl.detok(g, got) == data
    assert len(got) < len(data)  # multi-byte pieces are used


def _random_tokenizer(rng, kind):
    """A random tokenizer GGUF over a small alphabet (so pieces overlap and
    compete).  SentencePiece: canonical byte tokens (sometimes one missing),
    random pieces, some with the space marker, scores with ties and
    duplicates.  BPE: GPT-2 byte tokens and merges that join two existing
    pieces (sometimes an invalid or duplicate merge).  Random token types.
    Invalid vocabularies are allowed: both sides must then refuse them."""
    def enc(bs):
        return "".join(GPT2_BYTES[b] for b in bs)
    alphabet = b"ab c\n"
    if kind == "spm":
        toks = S.byte_tokens()
        if rng.random() < 0.15:
            del toks[int(rng.integers(256))]
        for _ in range(int(rng.integers(5, 60))):
            n = int(rng.integers(2, 6))
            p = "".join(chr(alphabet[int(rng.integers(len(alphabet)))]) for _ in range(n))
            toks.append(SPACE + p[1:] if rng.random() < 0.3 else p)
        kw = {"model": "llama" if rng.random() < 0.7 else None}
        if kw["model"] is None or rng.random() < 0.8:
            kw["scores"] = [float(rng.integers(-3, 3)) for _ in toks]
    else:
        toks = list(GPT2_BYTES)
        known = [bytes([c]) for c in alphabet]
        merges = []
        for _ in range(int(rng.integers(5, 60))):
            a = known[int(rng.integers(len(known)))]
            b = known[int(rng.integers(len(known)))]
            m = a + b
            if m in known or len(m) > 8:
                continue
            known.append(m)
            toks.append(enc(m))
            merges.append(enc(a) + " " + enc(b))
        if rng.random() < 0.1:
            merges.append("a zz")  # a piece that is not a token
        if rng.random() < 0.1 and merges:
            merges.append(merges[0])  # duplicate merge
        if rng.random() < 0.2:
            rng.shuffle(merges)
        kw = {"merges": merges, "model": "gpt2" if rng.random() < 0.5 else None}
    if rng.random() < 0.3:
        kw["token_type"] = [int(rng.choice([1, 1, 1, 6, 3])) for _ in toks]
    return gguf(toks, **kw)


@pytest.mark.parametrize("kind", ["spm", "bpe"])
def test_random_tokenizers_product_matches_oracle(kind):
    """Differential test: the library's tokenizer (C++) against the oracle's
    (C) on random vocabularies and inputs: the same tokenizer kind or the
    same refusal, the same tokens, codec symbols and bytes."""
    import detllm_b200 as D
    from oracle import oracle as O

    O.build()
    rng = np.random.default_rng(17 if kind == "spm" else 18)
    for _ in range(60):
        g = _random_tokenizer(rng, kind)
        try:
            want_kind = O.tokenizer_kind(g)
        except O.OracleError:
            with pytest.raises(D.DetError):
                D.tokenizer_kind(g)
            continue
        assert D.tokenizer_kind(g) == want_kind
        for _ in range(4):
            n = int(rng.integers(0, 200))
            # the alphabet includes the UTF-8 bytes of the space marker U+2581,
            # so literal marker bytes in the input meet the "▁" pieces
            data = bytes(rng.choice(list(b"ab c\n\xff\x00\xe2\x96\x81"), size=n).astype(np.uint8)) if n else b""
            for codec in (False, True):
                try:
                    want = O.tokenize(g, data, codec=codec)
                except O.OracleError:
                    with pytest.raises(D.DetError):
                        D.tokenize(g, data, codec=codec)
                    continue
                got = D.tokenize(g, data, codec=codec)
                assert got.tolist() == want.tolist()
                assert D.detokenize(g, got, byte_escapes=codec) == O.detokenize(g, want, escapes=codec)
