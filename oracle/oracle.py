"""ctypes wrapper of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE.  This module is the parity checker for the B200 library:
only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import it.  The product path (``detllm_b200``) never imports it.

The oracle restates the detllm reference CPU path in C; see oracle/ref.h for
the reference files it follows and the golden vectors that pin it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None


class SymbolRange(C.Structure):
    _fields_ = [("cum", C.c_uint64), ("freq", C.c_uint32), ("pad", C.c_uint32), ("total", C.c_uint64)]


class ModelInfo(C.Structure):
    _fields_ = [
        ("block_count", C.c_uint32), ("embedding_length", C.c_uint32), ("feed_forward_length", C.c_uint32),
        ("head_count", C.c_uint32), ("head_count_kv", C.c_uint32), ("head_dim", C.c_uint32),
        ("rope_dimension_count", C.c_uint32), ("rope_pairing", C.c_uint32),
        ("context_length", C.c_uint32), ("vocab", C.c_uint32),
        ("rms_epsilon", C.c_float), ("attention_scale", C.c_float), ("rope_freq_base", C.c_float),
        ("weight_types", C.c_uint32 * 9), ("has_qkv_bias", C.c_uint32), ("tied_output", C.c_uint32),
    ]


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P, SZ, I, U32, U64, F = C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_uint64, C.c_float
        sig = {
            "ref_expf": (F, [F]),
            "ref_expf_batch": (None, [P, P, SZ]),
            "ref_silu": (F, [F]),
            "ref_exp_f64": (C.c_double, [C.c_double]),
            "ref_ln_f64": (C.c_double, [C.c_double]),
            "ref_sin_f64": (C.c_double, [C.c_double]),
            "ref_cos_f64": (C.c_double, [C.c_double]),
            "ref_dot_f32": (F, [P, P, SZ]),
            "ref_sum_f32": (F, [P, SZ]),
            "ref_sum_squares_f32": (F, [P, SZ]),
            "ref_f16_to_f32": (F, [C.c_uint16]),
            "ref_round_ties_even_i32": (C.c_int32, [F]),
            "ref_sha256": (None, [P, SZ, P]),
            "ref_canary_hash": (None, [P]),
            "ref_runtime_canary_hash": (I, [P]),
            "ref_quant_kernel_hash": (I, [P]),
            "ref_fixture_gguf": (SZ, [I, P, SZ]),
            "ref_set_threads": (None, [I]),
            "ref_set_rowwise_gemv": (None, [I]),
            "ref_model_load": (I, [P, SZ, C.POINTER(P)]),
            "ref_model_free": (None, [P]),
            "ref_model_get_info": (I, [P, C.POINTER(ModelInfo)]),
            "ref_logits": (I, [P, P, SZ, P]),
            "ref_logits_hash": (I, [P, P, SZ, SZ, P]),
            "ref_rope_tables": (I, [P, SZ, P, P]),
            "ref_logits_to_symbol_range": (I, [P, SZ, SZ, I, C.POINTER(SymbolRange)]),
            "ref_decoder_total": (I, [P, SZ, I, C.POINTER(U64)]),
            "ref_decoder_lookup": (I, [P, SZ, I, U64, C.POINTER(U32), C.POINTER(SymbolRange)]),
            "ref_logits_to_cdf": (I, [P, SZ, P, P, C.POINTER(U64)]),
            "ref_range_encode": (I, [P, P, P, SZ, P, SZ, C.POINTER(SZ)]),
            "ref_compress": (I, [P, SZ, P, SZ, U32, C.POINTER(P), C.POINTER(SZ)]),
            "ref_decompress": (I, [P, SZ, P, SZ, C.POINTER(P), C.POINTER(SZ)]),
            "ref_encode_symbols": (I, [P, P, SZ, U32, U32, I, C.POINTER(P), C.POINTER(SZ)]),
            "ref_symbol_ranges_stream": (I, [P, P, SZ, U32, U32, I, P]),
            "ref_next_window_start": (SZ, [SZ, SZ, SZ, SZ]),
            "ref_gguf_parse_status": (I, [C.c_char_p, SZ]),
            "ref_rope_rotate": (I, [P, SZ, SZ, SZ, I, P, P]),
            "ref_softmax": (I, [P, SZ]),
            "ref_rmsnorm": (I, [P, P, SZ, F, P]),
            "ref_quantize_q8a_flat": (I, [P, SZ, P, P]),
            "ref_quantize_q8k_flat": (I, [P, SZ, P, P, P]),
            "ref_free": (None, [P]),
            "ref_tokenizer_kind": (I, [P, SZ, C.POINTER(C.c_int)]),
            "ref_tokenize": (I, [P, SZ, P, SZ, I, C.POINTER(P), C.POINTER(SZ)]),
            "ref_detokenize": (I, [P, SZ, P, SZ, I, C.POINTER(P), C.POINTER(SZ)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class OracleError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: status {code}")
        self.code = code


def _check(code: int, what: str):
    if code != 0:
        raise OracleError(code, what)


def rmsnorm(x, w, eps: float) -> np.ndarray:
    """det-model rmsnorm (lib.rs:2053-2073)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    _check(lib().ref_rmsnorm(_ptr(x), _ptr(w), x.size, eps, _ptr(out)), "rmsnorm")
    return out


def softmax(x) -> np.ndarray:
    """det-model softmax_in_place (lib.rs:2361-2388)."""
    x = np.array(x, np.float32)
    _check(lib().ref_softmax(_ptr(x), x.size), "softmax")
    return x


def rope_rotate(x, heads: int, head_dim: int, cos_row, sin_row, split_half: bool) -> np.ndarray:
    """det-model apply_rope (lib.rs:2011-2051) for one position, with the
    given table row (len(cos_row) rotation pairs per head)."""
    x = np.array(x, np.float32)
    c = np.ascontiguousarray(cos_row, np.float32)
    s = np.ascontiguousarray(sin_row, np.float32)
    _check(lib().ref_rope_rotate(_ptr(x), heads, head_dim, c.size, int(split_half), _ptr(c), _ptr(s)), "rope")
    return x


GGUF_ERRORS = ["ok", "bad magic", "unsupported version", "truncated", "unsupported value type", "invalid utf-8",
               "invalid tensor offset", "invalid tensor shape", "tensor not found", "metadata not found",
               "duplicate metadata key", "duplicate tensor name", "invalid bool", "metadata type mismatch",
               "unsupported tensor type", "alloc"]


def gguf_parse_error(data: bytes) -> str:
    """The det-gguf parse result of a whole file: "ok" or the GgufError
    (restated in oracle/ref_gguf.c)."""
    return GGUF_ERRORS[lib().ref_gguf_parse_status(data, len(data))]


def next_window_start(pos: int, start: int, n_ctx: int, overlap: int) -> int:
    """det-cli next_window_start (main.rs:772-778)."""
    return int(lib().ref_next_window_start(pos, start, n_ctx, overlap))


def set_threads(n: int) -> None:
    lib().ref_set_threads(int(n))


def set_rowwise_gemv(on: bool) -> None:
    """True: every GEMV row goes through the one-row K-quant dot functions
    (ref_dot_q4_k_q8a / ref_dot_q6_k_q8k) instead of the row-group ones."""
    lib().ref_set_rowwise_gemv(int(bool(on)))


def sha256(data: bytes) -> bytes:
    out = (C.c_uint8 * 32)()
    buf = np.frombuffer(data, dtype=np.uint8) if len(data) else np.zeros(1, np.uint8)
    lib().ref_sha256(_ptr(buf), len(data), out)
    return bytes(out)


def canary_hash() -> bytes:
    out = (C.c_uint8 * 32)()
    lib().ref_canary_hash(out)
    return bytes(out)


def runtime_canary_hash() -> bytes:
    out = (C.c_uint8 * 32)()
    _check(lib().ref_runtime_canary_hash(out), "runtime canary")
    return bytes(out)


def quant_kernel_hash() -> bytes:
    out = (C.c_uint8 * 32)()
    _check(lib().ref_quant_kernel_hash(out), "quant kernel hash")
    return bytes(out)


def fixture_gguf(which: str) -> bytes:
    idx = {"tiny-f32": 0, "tiny-qmix": 1}[which]
    n = lib().ref_fixture_gguf(idx, None, 0)
    buf = np.zeros(n, dtype=np.uint8)
    lib().ref_fixture_gguf(idx, _ptr(buf), n)
    return buf.tobytes()


def expf(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().ref_expf_batch(_ptr(x), _ptr(y), x.size)
    return y


def quantize_q8a(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = np.empty(x.size // 32, np.float32)
    q = np.empty(x.size, np.int8)
    _check(lib().ref_quantize_q8a_flat(_ptr(x), x.size, _ptr(d), _ptr(q)), "quantize_q8a")
    return d, q


def quantize_q8k(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = np.empty(x.size // 256, np.float32)
    q = np.empty(x.size, np.int8)
    bs = np.empty(x.size // 16, np.int16)
    _check(lib().ref_quantize_q8k_flat(_ptr(x), x.size, _ptr(d), _ptr(q), _ptr(bs)), "quantize_q8k")
    return d, q, bs


def symbol_range(logits: np.ndarray, symbol: int, byte_escapes: bool = True):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    r = SymbolRange()
    _check(lib().ref_logits_to_symbol_range(_ptr(logits), logits.size, symbol, int(byte_escapes), C.byref(r)),
           "symbol_range")
    return r.cum, r.freq, r.total


def decoder_total(logits: np.ndarray, byte_escapes: bool = True) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    t = C.c_uint64()
    _check(lib().ref_decoder_total(_ptr(logits), logits.size, int(byte_escapes), C.byref(t)), "decoder_total")
    return t.value


def decoder_lookup(logits: np.ndarray, value: int, byte_escapes: bool = True):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    s = C.c_uint32()
    r = SymbolRange()
    _check(lib().ref_decoder_lookup(_ptr(logits), logits.size, int(byte_escapes), value, C.byref(s), C.byref(r)),
           "decoder_lookup")
    return s.value, r.cum, r.freq, r.total


def logits_to_cdf(logits: np.ndarray):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    f = np.empty(logits.size, np.uint32)
    c = np.empty(logits.size, np.uint64)
    t = C.c_uint64()
    _check(lib().ref_logits_to_cdf(_ptr(logits), logits.size, _ptr(f), _ptr(c), C.byref(t)), "logits_to_cdf")
    return f, c, t.value


def _take_bytes(p: C.c_void_p, n: int) -> bytes:
    data = C.string_at(p.value, n) if n else b""
    lib().ref_free(p)
    return data


def compress(model: bytes, data: bytes, n_ctx: int = 0) -> bytes:
    mb = np.frombuffer(model, np.uint8)
    ib = np.frombuffer(data, np.uint8) if data else np.zeros(1, np.uint8)
    out, n = C.c_void_p(), C.c_size_t()
    _check(lib().ref_compress(_ptr(mb), len(model), _ptr(ib), len(data), n_ctx, C.byref(out), C.byref(n)),
           "compress")
    return _take_bytes(out, n.value)


def decompress(model: bytes, dtlz: bytes) -> bytes:
    mb = np.frombuffer(model, np.uint8)
    db = np.frombuffer(dtlz, np.uint8) if dtlz else np.zeros(1, np.uint8)
    out, n = C.c_void_p(), C.c_size_t()
    _check(lib().ref_decompress(_ptr(mb), len(model), _ptr(db), len(dtlz), C.byref(out), C.byref(n)), "decompress")
    return _take_bytes(out, n.value)


TOKENIZER_KINDS = ("byte_fallback", "byte_bpe", "sentencepiece")


def tokenizer_kind(gguf: bytes) -> str:
    """Tokenizer::from_gguf's selection (det-token lib.rs:86-132)."""
    gb = np.frombuffer(gguf, np.uint8)
    k = C.c_int()
    _check(lib().ref_tokenizer_kind(_ptr(gb), len(gguf), C.byref(k)), "tokenizer")
    return TOKENIZER_KINDS[k.value]


def tokenize(gguf: bytes, data: bytes, codec: bool = False) -> np.ndarray:
    """tokenize_bytes of the GGUF's tokenizer, or with codec=True the codec
    symbols (tokens, and vocab + byte for byte escapes)."""
    gb = np.frombuffer(gguf, np.uint8)
    ib = np.frombuffer(data, np.uint8) if data else np.zeros(1, np.uint8)
    out, n = C.c_void_p(), C.c_size_t()
    _check(lib().ref_tokenize(_ptr(gb), len(gguf), _ptr(ib), len(data), int(codec), C.byref(out), C.byref(n)),
           "tokenize")
    return np.frombuffer(_take_bytes(out, 4 * n.value), np.uint32).copy()


def detokenize(gguf: bytes, symbols, escapes: bool = True) -> bytes:
    """The bytes of a token / codec symbol sequence (decode_codec_symbol)."""
    gb = np.frombuffer(gguf, np.uint8)
    s = np.ascontiguousarray(symbols, np.uint32)
    sb = s if s.size else np.zeros(1, np.uint32)
    out, n = C.c_void_p(), C.c_size_t()
    _check(lib().ref_detokenize(_ptr(gb), len(gguf), _ptr(sb), s.size, int(escapes), C.byref(out), C.byref(n)),
           "detokenize")
    return _take_bytes(out, n.value)


class Model:
    """A model loaded by the oracle (F32Llama::from_gguf restated)."""

    def __init__(self, gguf: bytes):
        self._bytes = np.frombuffer(gguf, np.uint8)
        h = C.c_void_p()
        _check(lib().ref_model_load(_ptr(self._bytes), len(gguf), C.byref(h)), "model_load")
        self._h = h
        info = ModelInfo()
        _check(lib().ref_model_get_info(h, C.byref(info)), "model_info")
        self.info = info
        self.vocab = info.vocab

    def close(self):
        if self._h:
            lib().ref_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def logits(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty((t.size, self.vocab), np.float32)
        _check(lib().ref_logits(self._h, _ptr(t), t.size, _ptr(out)), "logits")
        return out

    def logits_hash(self, tokens, chunk: int = 1) -> bytes:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = (C.c_uint8 * 32)()
        _check(lib().ref_logits_hash(self._h, _ptr(t), t.size, chunk, out), "logits_hash")
        return bytes(out)

    def rope_tables(self, positions: int):
        half = self.info.rope_dimension_count // 2
        c = np.empty((positions, half), np.float32)
        s = np.empty((positions, half), np.float32)
        _check(lib().ref_rope_tables(self._h, positions, _ptr(c), _ptr(s)), "rope_tables")
        return c, s

    def encode_symbols(self, symbols, n_ctx: int, overlap: int, byte_escapes: bool = True) -> bytes:
        s = np.ascontiguousarray(symbols, dtype=np.uint32)
        if s.size == 0:
            s = np.zeros(1, np.uint32)[:0]
        out, n = C.c_void_p(), C.c_size_t()
        _check(lib().ref_encode_symbols(self._h, _ptr(s) if s.size else None, s.size, n_ctx, overlap,
                                        int(byte_escapes), C.byref(out), C.byref(n)), "encode_symbols")
        return _take_bytes(out, n.value)

    def symbol_ranges(self, symbols, n_ctx: int, overlap: int, byte_escapes: bool = True) -> np.ndarray:
        s = np.ascontiguousarray(symbols, dtype=np.uint32)
        out = np.zeros((max(s.size, 1), 3), np.uint64)
        raw = (SymbolRange * max(s.size, 1))()
        _check(lib().ref_symbol_ranges_stream(self._h, _ptr(s), s.size, n_ctx, overlap, int(byte_escapes), raw),
               "symbol_ranges")
        for i in range(s.size):
            out[i] = (raw[i].cum, raw[i].freq, raw[i].total)
        return out[: s.size]
