"""Seeded synthetic models and inputs for the benchmark configurations.

No real checkpoints or datasets are available offline, so the benchmark and
the parity tests use random-init weights of the named architectures and
seeded synthetic token / byte streams with the shapes the configurations
name.  Everything here is deterministic in (config, seed).

* weights (libdetsynth.so, csrc/synth.c): N(0, 0.02) values quantised to the
  GGUF block formats det-quant decodes (Q8_0, Q4_0, Q4_K, Q6_K; layouts fixed
  by crates/det-quant/src/lib.rs:506-568); norm weights 1.0; qwen2 QKV biases
  N(0, 0.02); a byte-fallback vocabulary (256 ``<0xNN>`` tokens, then filler
  pieces) so det-token selects ByteFallbackTokenizer (lib.rs:111-130);
* inputs: Zipf(s) token ids over the vocabulary through a seeded permutation,
  and order-2 Markov text over printable ASCII plus '<' / '>' markup.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os

import numpy as np

GT_F32, GT_F16, GT_Q4_0, GT_Q8_0, GT_Q4_K, GT_Q6_K = 0, 1, 2, 8, 12, 14
_LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdetsynth.so")
_lib = None


@dataclasses.dataclass
class ModelSpec:
    arch: str = "llama"             # "llama" (adjacent RoPE) or "qwen2" (split-half RoPE)
    n_layer: int = 2
    d: int = 256
    d_ff: int = 512
    n_head: int = 4
    n_head_kv: int = 2
    vocab: int = 1024
    ctx: int = 512
    rope_base: float = 10000.0
    eps: float = 1e-5
    tied: bool = False
    # ggml types: token_embd, attention (q, k, v, o), ffn gate/up, ffn down, output
    t_embd: int = GT_Q8_0
    t_attn: int = GT_Q8_0
    t_gate_up: int = GT_Q8_0
    t_down: int = GT_Q8_0
    t_out: int = GT_Q8_0
    qkv_bias: bool = False
    seed: int = 1234
    # byte values whose <0xNN> token is marked non-emittable (token type 3),
    # so the codec sends them as byte escapes (det-token lib.rs:150-180)
    escape_bytes: tuple = ()

    @property
    def head_dim(self) -> int:
        return self.d // self.n_head


# The BASELINE configurations (random init; shapes as named there)
CONFIGS = {
    "tinyllama-q8_0": ModelSpec("llama", 22, 2048, 5632, 32, 4, 32000, 2048, 10000.0),
    "tinyllama-q4_k_m": ModelSpec("llama", 22, 2048, 5632, 32, 4, 32000, 2048, 10000.0, t_embd=GT_Q4_K,
                                  t_attn=GT_Q4_K, t_gate_up=GT_Q4_K, t_down=GT_Q6_K, t_out=GT_Q6_K),
    "qwen2.5-0.5b-q8_0": ModelSpec("qwen2", 24, 896, 4864, 14, 2, 151936, 4096, 1000000.0, eps=1e-6, tied=True,
                                   qkv_bias=True),
    "llama3-8b-q4_k": ModelSpec("llama", 32, 4096, 14336, 32, 8, 128256, 8192, 500000.0, t_embd=GT_Q4_K,
                                t_attn=GT_Q4_K, t_gate_up=GT_Q4_K, t_down=GT_Q6_K, t_out=GT_Q6_K),
}


class _Spec(C.Structure):
    _fields_ = [("arch", C.c_int), ("n_layer", C.c_int), ("d", C.c_int), ("d_ff", C.c_int), ("n_head", C.c_int),
                ("n_head_kv", C.c_int), ("vocab", C.c_int), ("ctx", C.c_int), ("rope_base", C.c_float),
                ("eps", C.c_float), ("tied", C.c_int), ("qkv_bias", C.c_int), ("t_embd", C.c_int),
                ("t_attn", C.c_int), ("t_gate_up", C.c_int), ("t_down", C.c_int), ("t_out", C.c_int),
                ("seed", C.c_uint64), ("escape", C.c_uint8 * 32)]


def _synth_lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            raise RuntimeError(f"{_LIB} is missing: build it with `make -C detllm_b200/csrc`")
        L = C.CDLL(_LIB)
        L.synth_gguf.restype = C.c_size_t
        L.synth_gguf.argtypes = [C.POINTER(_Spec), C.c_void_p, C.c_size_t, C.c_int]
        L.synth_markov.restype = C.c_size_t
        L.synth_markov.argtypes = [C.c_void_p, C.c_size_t, C.c_uint64]
        _lib = L
    return _lib


def build_gguf(spec: ModelSpec, threads: int = 0) -> bytes:
    """A GGUF v3 file of `spec` with seeded random-init weights."""
    s = _Spec()
    s.arch = 1 if spec.arch == "qwen2" else 0
    for f in ("n_layer", "d", "d_ff", "n_head", "n_head_kv", "vocab", "ctx", "t_embd", "t_attn", "t_gate_up",
              "t_down", "t_out"):
        setattr(s, f, int(getattr(spec, f)))
    s.rope_base, s.eps = spec.rope_base, spec.eps
    s.tied, s.qkv_bias, s.seed = int(spec.tied), int(spec.qkv_bias), spec.seed
    for b in spec.escape_bytes:
        s.escape[b >> 3] |= 1 << (b & 7)
    L = _synth_lib()
    n = L.synth_gguf(C.byref(s), None, 0, 1)
    buf = np.empty(n, np.uint8)
    got = L.synth_gguf(C.byref(s), buf.ctypes.data, n, threads or min(os.cpu_count() or 1, 32))
    assert got == n
    return buf.tobytes()


def weight_bytes_per_token(spec: ModelSpec) -> int:
    """Algorithmic weight bytes one token's forward streams (all GEMV
    matrices incl. the lm_head; the embedding is one row)."""
    bpw = {GT_F32: 4.0, GT_F16: 2.0, GT_Q8_0: 34 / 32, GT_Q4_0: 18 / 32, GT_Q4_K: 144 / 256, GT_Q6_K: 210 / 256}
    hd = spec.head_dim
    attn = (spec.n_head * hd * spec.d * 2 + spec.n_head_kv * hd * spec.d * 2) * bpw[spec.t_attn]
    ffn = 2 * spec.d_ff * spec.d * bpw[spec.t_gate_up] + spec.d * spec.d_ff * bpw[spec.t_down]
    out = spec.vocab * spec.d * bpw[spec.t_embd if spec.tied else spec.t_out]
    return int(round(spec.n_layer * (attn + ffn) + out))


def zipf_tokens(n: int, vocab: int, s: float = 1.1, seed: int = 7) -> np.ndarray:
    """n token ids with rank ~ Zipf(s) over the vocabulary, mapped through a
    seeded permutation."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** -s
    p /= p.sum()
    r = rng.choice(vocab, size=n, p=p)
    perm = rng.permutation(vocab)
    return perm[r].astype(np.uint32)


def markov_text(n: int, seed: int = 11) -> bytes:
    """n bytes of seeded order-2 Markov text over printable ASCII, newline and
    extra '<' / '>' markup mass."""
    rng = np.random.default_rng(seed)
    alphabet = np.array([*range(0x20, 0x7F), 0x0A], np.uint8)
    k = len(alphabet)
    weights = rng.gamma(0.3, 1.0, size=(k, k, k))
    for ch in (ord("<"), ord(">")):
        weights[:, :, int(np.where(alphabet == ch)[0][0])] += 0.5
    cdf = np.cumsum(weights / weights.sum(axis=2, keepdims=True), axis=2)
    u = rng.random(n)
    out = np.empty(n, np.uint8)
    a, b = 0, 1
    for i in range(n):
        c = min(int(np.searchsorted(cdf[a, b], u[i])), k - 1)
        out[i] = alphabet[c]
        a, b = b, c
    return out.tobytes()


def markov_stream(n: int, seed: int = 16) -> bytes:
    """n bytes of seeded order-2 Markov text (printable ASCII, newline, extra
    '<' / '>' markup mass) from libdetsynth.so: the benchmark's multi-MiB
    input streams, generated in well under a second."""
    buf = np.empty(max(n, 1), np.uint8)
    got = _synth_lib().synth_markov(buf.ctypes.data, n, seed)
    if got != n:
        raise MemoryError("synth_markov failed")
    return buf[:n].tobytes()


# ---- GGUF metadata (tokenizer vocabularies) ---------------------------------
# GGUF v3 value types (det-gguf lib.rs:58-96)
GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STRING, GV_ARRAY, GV_F64 = 4, 5, 6, 7, 8, 9, 12


def _gguf_str(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return len(b).to_bytes(8, "little") + b


def _gguf_value(ty: int, v) -> bytes:
    import struct

    if ty == GV_STRING:
        return _gguf_str(v)
    if ty == GV_U32:
        return struct.pack("<I", v)
    if ty == GV_I32:
        return struct.pack("<i", v)
    if ty == GV_F32:
        return struct.pack("<f", v)
    if ty == GV_BOOL:
        return struct.pack("<B", int(v))
    if ty == GV_F64:
        return struct.pack("<d", v)
    elem, items = v
    body = b"".join(_gguf_value(elem, x) for x in items)
    return struct.pack("<IQ", elem, len(items)) + body


def gguf_metadata(kvs) -> bytes:
    """A GGUF v3 file with metadata only (no tensors): kvs is a list of
    (key, type, value); an array value is (element type, items)."""
    out = b"GGUF" + (3).to_bytes(4, "little") + (0).to_bytes(8, "little") + len(kvs).to_bytes(8, "little")
    for key, ty, v in kvs:
        out += _gguf_str(key) + ty.to_bytes(4, "little") + _gguf_value(ty, v)
    return out + b"\0" * (-len(out) % 32)


def byte_tokens() -> list:
    """The 256 canonical byte-fallback tokens <0x00>..<0xFF>."""
    return [f"<0x{b:02X}>" for b in range(256)]


def tokenizer_kvs(tokens, model=None, merges=None, scores=None, token_type=None) -> list:
    """tokenizer.ggml.* metadata entries for gguf_metadata / with_tokenizer."""
    kv = [("tokenizer.ggml.tokens", GV_ARRAY, (GV_STRING, list(tokens)))]
    if model is not None:
        kv.append(("tokenizer.ggml.model", GV_STRING, model))
    if merges is not None:
        kv.append(("tokenizer.ggml.merges", GV_ARRAY, (GV_STRING, list(merges))))
    if scores is not None:
        kv.append(("tokenizer.ggml.scores", GV_ARRAY, (GV_F32, list(scores))))
    if token_type is not None:
        kv.append(("tokenizer.ggml.token_type", GV_ARRAY, (GV_I32, list(token_type))))
    return kv


def _gpt2_chars() -> list:
    """GPT-2's byte-to-unicode table: printable bytes stand for themselves,
    the other 68 bytes map to code points 256, 257, ... in byte order (the
    decoding det-token applies to BPE token strings, lib.rs:813-839)."""
    def printable(c):
        return 33 <= c <= 126 or 161 <= c <= 172 or 174 <= c <= 255
    out, n = [], 0
    for b in range(256):
        if printable(b):
            out.append(chr(b))
        else:
            out.append(chr(256 + n))
            n += 1
    return out


def _spm_vocab(vocab: int, sample: bytes) -> tuple:
    """SentencePiece-style vocabulary: the 256 byte tokens, then the most
    frequent 2..8-byte pieces of `sample` (a leading space written as U+2581),
    scored by descending frequency x length."""
    counts = {}
    for n in range(2, 9):
        for i in range(len(sample) - n + 1):
            p = sample[i:i + n]
            if b"\n" in p[1:]:
                continue
            counts[p] = counts.get(p, 0) + 1
    ranked = sorted(counts, key=lambda p: (-counts[p] * len(p), p))[: vocab - 256]
    tokens = byte_tokens()
    scores = [0.0] * 256
    for r, p in enumerate(ranked):
        s = p.decode()
        tokens.append("▁" + s[1:] if s.startswith(" ") else s)
        scores.append(-float(r + 1))
    return tokens, scores


def _bpe_vocab(vocab: int, sample: bytes) -> tuple:
    """Byte-level BPE vocabulary: GPT-2 byte tokens, then merges learned on
    `sample` (most frequent adjacent pair first, ties by first occurrence)."""
    chars = _gpt2_chars()
    tokens = list(chars)
    pieces = [bytes([b]) for b in range(256)]
    seq = [pieces[b] for b in sample]
    merges = []
    known = set(pieces)
    while len(tokens) < vocab and len(seq) > 1:
        counts, first = {}, {}
        for i in range(len(seq) - 1):
            pr = (seq[i], seq[i + 1])
            counts[pr] = counts.get(pr, 0) + 1
            first.setdefault(pr, i)
        best = None
        for pr, c in counts.items():
            if pr[0] + pr[1] in known:
                continue
            if best is None or c > counts[best] or (c == counts[best] and first[pr] < first[best]):
                best = pr
        if best is None or counts[best] < 2:
            break
        merged = best[0] + best[1]
        known.add(merged)
        tokens.append("".join(chars[b] for b in merged))
        merges.append("".join(chars[b] for b in best[0]) + " " + "".join(chars[b] for b in best[1]))
        out, i = [], 0
        while i < len(seq):
            if i + 1 < len(seq) and (seq[i], seq[i + 1]) == best:
                out.append(merged)
                i += 2
            else:
                out.append(seq[i])
                i += 1
        seq = out
    while len(tokens) < vocab:  # filler pieces that the merges never produce
        tokens.append(f"<unused{len(tokens)}>")
    return tokens, merges


_VOCABS = {}


def synthetic_tokenizer_kvs(kind: str, vocab: int, seed: int = 5) -> list:
    """tokenizer.ggml.* metadata of a seeded `kind` ("spm" or "bpe")
    vocabulary of exactly `vocab` tokens learned on Markov text."""
    key = (kind, vocab, seed)
    if key not in _VOCABS:
        sample = markov_text(3000, seed=seed)
        if kind == "spm":
            tokens, scores = _spm_vocab(vocab, sample)
            _VOCABS[key] = tokenizer_kvs(tokens, model="llama", scores=scores)
        else:
            tokens, merges = _bpe_vocab(vocab, sample)
            _VOCABS[key] = tokenizer_kvs(tokens, model="gpt2", merges=merges)
    return _VOCABS[key]


def _skip_value(b: bytes, o: int, ty: int) -> int:
    fixed = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
    if ty in fixed:
        return o + fixed[ty]
    if ty == GV_STRING:
        return o + 8 + int.from_bytes(b[o:o + 8], "little")
    if ty == GV_ARRAY:
        et, n = int.from_bytes(b[o:o + 4], "little"), int.from_bytes(b[o + 4:o + 12], "little")
        o += 12
        if et in fixed:
            return o + fixed[et] * n
        for _ in range(n):
            o = _skip_value(b, o, et)
        return o
    raise ValueError(f"GGUF value type {ty}")


def with_tokenizer(gguf: bytes, kvs) -> bytes:
    """`gguf` (v3) with its tokenizer.ggml.* metadata replaced by `kvs`;
    tensor infos and data are kept (tensor offsets are relative to the
    data section, which stays aligned to 32 bytes)."""
    return with_metadata(gguf, kvs, drop=lambda key: key.startswith("tokenizer.ggml."))


def with_metadata(gguf: bytes, kvs, drop=None) -> bytes:
    """`gguf` (v3) with the (key, type, value) entries of `kvs` set (an
    existing entry of the same key is replaced) and the keys for which
    `drop(key)` is true removed; tensor infos and data are kept."""
    assert gguf[:4] == b"GGUF"
    new_keys = {k for k, _, _ in kvs}
    n_t = int.from_bytes(gguf[8:16], "little")
    n_kv = int.from_bytes(gguf[16:24], "little")
    o, keep = 24, []
    for _ in range(n_kv):
        start = o
        klen = int.from_bytes(gguf[o:o + 8], "little")
        key = gguf[o + 8:o + 8 + klen].decode()
        ty = int.from_bytes(gguf[o + 8 + klen:o + 12 + klen], "little")
        o = _skip_value(gguf, o + 12 + klen, ty)
        if key not in new_keys and not (drop and drop(key)):
            keep.append(gguf[start:o])
        if key == "general.alignment":
            raise ValueError("custom alignment is not handled")
    infos_start = o
    for _ in range(n_t):
        nlen = int.from_bytes(gguf[o:o + 8], "little")
        o += 8 + nlen
        nd = int.from_bytes(gguf[o:o + 4], "little")
        o += 4 + 8 * nd + 4 + 8
    infos = gguf[infos_start:o]
    data = gguf[o + (-o % 32):]
    new_kv = b"".join(_gguf_str(k) + t.to_bytes(4, "little") + _gguf_value(t, v) for k, t, v in kvs)
    head = gguf[:8] + n_t.to_bytes(8, "little") + (len(keep) + len(kvs)).to_bytes(8, "little")
    body = head + b"".join(keep) + new_kv + infos
    return body + b"\0" * (-len(body) % 32) + data
