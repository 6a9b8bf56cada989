"""detllm_b200 -- the detllm token loop on NVIDIA B200 (sm_100a).

Python view of ``libdetgpu.so`` (C ABI: ``include/detgpu.h``).  The names
mirror the reference crates so callers read like the reference's own code:

* :class:`Model` -- ``det_model::F32Llama`` (``from_gguf``,
  ``logits_hash_for_tokens_chunked``, ``logits_bytes_for_tokens_chunked``)
* :class:`Session` -- ``RopeTables`` + ``KvCache`` + ``ForwardWorkspace``
  around ``forward_one_with_workspace``, extended to teacher-forced chunks
* :meth:`Session.symbol_ranges` / :meth:`Session.decoder_total` /
  :meth:`Session.decoder_lookup` -- ``det_coder`` logits -> CDF
* :func:`compress` / :func:`decompress` -- ``detllm compress`` / ``decompress``

Every result is bit-identical to the reference CPU path.  There is no CPU
fallback: without the built library or a CUDA device these calls raise.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

__all__ = ["DetError", "Model", "Session", "compress", "decompress", "device_count", "lib", "LIB_PATH"]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdetgpu.so")
_lib = None

# status codes (include/detgpu.h)
OK = 0
ERR_SHAPE = 1
ERR_NONFINITE = 2
ERR_CDF_SYMBOL_OUT_OF_RANGE = 35
ERR_NO_DEVICE = 65


class SymbolRange(C.Structure):
    _fields_ = [("cum", C.c_uint64), ("freq", C.c_uint32), ("reserved", C.c_uint32), ("total", C.c_uint64)]


class Config(C.Structure):
    _fields_ = [
        ("block_count", C.c_uint32), ("embedding_length", C.c_uint32), ("feed_forward_length", C.c_uint32),
        ("head_count", C.c_uint32), ("head_count_kv", C.c_uint32), ("head_dim", C.c_uint32),
        ("rope_dimension_count", C.c_uint32), ("rope_pairing", C.c_uint32),
        ("context_length", C.c_uint32), ("vocab", C.c_uint32),
        ("rms_epsilon", C.c_float), ("attention_scale", C.c_float), ("rope_freq_base", C.c_float),
        ("weight_types", C.c_uint32 * 9), ("has_qkv_bias", C.c_uint32), ("tied_output", C.c_uint32),
    ]


class Stats(C.Structure):
    _fields_ = [("forward_ms", C.c_double), ("cdf_ms", C.c_double), ("launches", C.c_uint64),
                ("h2d_bytes", C.c_uint64), ("d2h_bytes", C.c_uint64), ("tokens", C.c_uint64),
                ("gemm_ms", C.c_double), ("gemm_launches", C.c_uint64), ("gemm_bytes", C.c_double),
                ("gemm_weight_bytes", C.c_double)]

    def as_dict(self) -> dict:
        return {k: getattr(self, k) for k, _ in self._fields_}


class DetError(RuntimeError):
    """A non-zero det_status from the library."""

    def __init__(self, code: int, what: str):
        msg = lib().det_status_string(code).decode() if _lib is not None else str(code)
        super().__init__(f"{what}: {msg} (status {code})")
        self.code = code


def lib():
    """Load libdetgpu.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C detllm_b200/csrc` "
                               "(or __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        P, SZ, I, U32, U64 = C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_uint64
        sig = {
            "det_status_string": (C.c_char_p, [I]),
            "det_device_count": (I, [C.POINTER(I)]),
            "det_model_load": (I, [P, SZ, I, C.POINTER(P)]),
            "det_model_load_tp": (I, [P, SZ, P, I, C.POINTER(P)]),
            "det_model_free": (None, [P]),
            "det_model_info": (I, [P, C.POINTER(Config)]),
            "det_model_sha256": (I, [P, P]),
            "det_session_create": (I, [P, U32, U32, C.POINTER(P)]),
            "det_session_free": (None, [P]),
            "det_session_reset": (I, [P]),
            "det_forward": (I, [P, P, U32, U32, P]),
            "det_symbol_ranges": (I, [P, P, P, U32, I, P]),
            "det_decoder_total": (I, [P, U32, I, C.POINTER(U64)]),
            "det_decoder_lookup": (I, [P, U32, I, U64, C.POINTER(U32), C.POINTER(SymbolRange)]),
            "det_logits_hash": (I, [P, P, SZ, U32, P]),
            "det_compress": (I, [P, P, SZ, U32, C.POINTER(P), C.POINTER(SZ)]),
            "det_decompress": (I, [P, P, SZ, C.POINTER(P), C.POINTER(SZ)]),
            "det_encode_symbols": (I, [P, P, SZ, U32, U32, I, C.POINTER(P), C.POINTER(SZ)]),
            "det_free": (None, [P]),
            "det_tokenizer_kind": (I, [P, SZ, C.POINTER(C.c_int)]),
            "det_tokenize": (I, [P, SZ, P, SZ, I, C.POINTER(P), C.POINTER(SZ)]),
            "det_detokenize": (I, [P, SZ, P, SZ, I, C.POINTER(P), C.POINTER(SZ)]),
            "det_session_stats": (I, [P, C.POINTER(Stats), I]),
            "det_device_expf": (I, [I, P, P, SZ]),
            "det_model_stats": (I, [P, C.POINTER(Stats), I]),
            "det_set_profiling": (I, [I]),
            "det_set_encode_chunk": (I, [U32, C.POINTER(U32)]),
            "det_set_q8_tensor_cores": (I, [I, C.POINTER(I)]),
            "det_model_profile": (I, [P, C.c_char_p, SZ, I]),
            "det_session_gemv_stream": (I, [P, U32, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
            "det_symbol_ranges_noalloc": (I, [P, U32, U32, P, I, P, P]),
            "det_tp_exchange_timeout_selftest": (I, [I]),
            "det_q6k_pipeline_timeout_selftest": (I, [I]),
            "det_add_latency_cycles": (I, [I, C.POINTER(C.c_double)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(code: int, what: str) -> None:
    if code != OK:
        raise DetError(code, what)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _u32(x) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.uint32))
    return a if a.size else np.zeros(1, np.uint32)[:0]


def device_count() -> int:
    n = C.c_int()
    _check(lib().det_device_count(C.byref(n)), "det_device_count")
    return n.value


def _take(p: C.c_void_p, n: int) -> bytes:
    data = C.string_at(p.value, n) if n else b""
    lib().det_free(p)
    return data


class Model:
    """``F32Llama::from_gguf`` on a B200: weights live in device memory."""

    def __init__(self, gguf: bytes, device: int = 0, devices=None):
        """``devices``: a list of CUDA devices for a row-sharded
        (tensor-parallel) model (``det_model_load_tp``; a device may repeat);
        ``device`` is then ``devices[0]``."""
        self._keep = np.frombuffer(gguf, np.uint8)
        h = C.c_void_p()
        if devices is None:
            _check(lib().det_model_load(_ptr(self._keep), len(gguf), device, C.byref(h)), "det_model_load")
            self.devices = [device]
        else:
            devs = np.ascontiguousarray(np.asarray(devices, dtype=np.int32))
            _check(lib().det_model_load_tp(_ptr(self._keep), len(gguf), _ptr(devs), int(devs.size), C.byref(h)),
                   "det_model_load_tp")
            self.devices = [int(d) for d in devs]
            device = self.devices[0]
        self._h = h
        del self._keep
        cfg = Config()
        _check(lib().det_model_info(h, C.byref(cfg)), "det_model_info")
        self.config = cfg
        self.vocab = cfg.vocab
        self.device = device

    @classmethod
    def from_gguf(cls, gguf: bytes, device: int = 0) -> "Model":
        return cls(gguf, device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().det_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def sha256(self) -> bytes:
        out = (C.c_uint8 * 32)()
        _check(lib().det_model_sha256(self._h, out), "det_model_sha256")
        return bytes(out)

    def logits_hash_for_tokens_chunked(self, tokens, chunk: int = 1) -> bytes:
        t = _u32(tokens)
        out = (C.c_uint8 * 32)()
        _check(lib().det_logits_hash(self._h, _ptr(t), t.size, chunk, out), "det_logits_hash")
        return bytes(out)

    def logits_hash_for_tokens(self, tokens) -> bytes:
        return self.logits_hash_for_tokens_chunked(tokens, 1)

    def logits_for_tokens(self, tokens, chunk: int = 64) -> np.ndarray:
        """Logits of every position (``visit_logits_for_tokens_chunked``)."""
        t = _u32(tokens)
        out = np.empty((t.size, self.vocab), np.float32)
        with Session(self, n_ctx=t.size, max_chunk=min(chunk, t.size, 1024)) as s:
            for p in range(0, t.size, s.max_chunk):
                n = min(s.max_chunk, t.size - p)
                out[p:p + n] = s.forward(t[p:p + n], p, want_logits=True)
        return out

    def logits_bytes_for_tokens_chunked(self, tokens, chunk: int = 1) -> bytes:
        return self.logits_for_tokens(tokens, max(chunk, 1)).astype("<f4").tobytes()

    def stats(self, reset: bool = False) -> Stats:
        st = Stats()
        _check(lib().det_model_stats(self._h, C.byref(st), int(reset)), "det_model_stats")
        return st

    def profile(self, reset: bool = False) -> dict:
        """Per-kernel-group device time gathered while profiling was on:
        {group: (launches, milliseconds)}."""
        import json

        buf = C.create_string_buffer(4096)
        _check(lib().det_model_profile(self._h, buf, len(buf), int(reset)), "det_model_profile")
        return {k: (int(v[0]), float(v[1])) for k, v in json.loads(buf.value.decode()).items()}

    def session(self, n_ctx: int, max_chunk: int = 64) -> "Session":
        return Session(self, n_ctx, max_chunk)

    def encode_symbols(self, symbols, n_ctx: int, overlap: int, byte_escapes: bool = True) -> bytes:
        s = _u32(symbols)
        out, n = C.c_void_p(), C.c_size_t()
        _check(lib().det_encode_symbols(self._h, _ptr(s) if s.size else None, s.size, n_ctx, overlap,
                                        int(byte_escapes), C.byref(out), C.byref(n)), "det_encode_symbols")
        return _take(out, n.value)


class Session:
    """One context window on the device (RoPE table, KV cache, workspace)."""

    def __init__(self, model: Model, n_ctx: int, max_chunk: int = 64):
        self.model = model
        h = C.c_void_p()
        _check(lib().det_session_create(model._h, n_ctx, max_chunk, C.byref(h)), "det_session_create")
        self._h = h
        self.n_ctx = n_ctx
        self.max_chunk = min(max_chunk, n_ctx)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().det_session_free(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self) -> None:
        _check(lib().det_session_reset(self._h), "det_session_reset")

    def forward(self, tokens, pos0: int, want_logits: bool = False):
        t = _u32(tokens)
        out = np.empty((t.size, self.model.vocab), np.float32) if want_logits else None
        _check(lib().det_forward(self._h, _ptr(t), t.size, pos0, _ptr(out) if want_logits else None),
               "det_forward")
        return out

    def symbol_ranges(self, symbols, rows=None, byte_escapes: bool = True) -> np.ndarray:
        """(cum, freq, total) per symbol, as ``logits_to_symbol_range_with_byte_escapes``."""
        s = _u32(symbols)
        r = _u32(rows) if rows is not None else None
        out = (SymbolRange * max(s.size, 1))()
        _check(lib().det_symbol_ranges(self._h, _ptr(r) if r is not None else None, _ptr(s), s.size,
                                       int(byte_escapes), out), "det_symbol_ranges")
        return np.array([(out[i].cum, out[i].freq, out[i].total) for i in range(s.size)], np.uint64).reshape(-1, 3)

    def decoder_total(self, row: int, byte_escapes: bool = True) -> int:
        t = C.c_uint64()
        _check(lib().det_decoder_total(self._h, row, int(byte_escapes), C.byref(t)), "det_decoder_total")
        return t.value

    def decoder_lookup(self, row: int, value: int, byte_escapes: bool = True):
        sym = C.c_uint32()
        r = SymbolRange()
        _check(lib().det_decoder_lookup(self._h, row, int(byte_escapes), value, C.byref(sym), C.byref(r)),
               "det_decoder_lookup")
        return sym.value, r.cum, r.freq, r.total

    def gemv_stream(self, reps: int = 20):
        """(ms, bytes) per pass of the one-token weight GEMVs run back to back."""
        ms, by = C.c_double(), C.c_double()
        _check(lib().det_session_gemv_stream(self._h, reps, C.byref(ms), C.byref(by)), "det_session_gemv_stream")
        return ms.value, by.value

    def stats(self, reset: bool = False) -> Stats:
        st = Stats()
        _check(lib().det_session_stats(self._h, C.byref(st), int(reset)), "det_session_stats")
        return st


def set_encode_chunk(chunk: int) -> int:
    """Positions per forward chunk of the codec (16..1024, 0 = default);
    returns the previous value.  The output bytes do not depend on it."""
    prev = C.c_uint32()
    _check(lib().det_set_encode_chunk(int(chunk), C.byref(prev)), "det_set_encode_chunk")
    return prev.value


def set_q8_tensor_cores(enable: bool) -> bool:
    """Chunk GEMM for Q8_0 / Q4_0 weights: True the tcgen05 kernel, False the
    mma.sync kernel (default); returns the previous choice.  Same bits."""
    prev = C.c_int()
    _check(lib().det_set_q8_tensor_cores(int(bool(enable)), C.byref(prev)), "det_set_q8_tensor_cores")
    return bool(prev.value)


def add_latency_cycles(device: int = 0) -> float:
    """Measured cycles of one dependent f32 add on `device` (the floor of
    every ordered chain)."""
    v = C.c_double()
    _check(lib().det_add_latency_cycles(int(device), C.byref(v)), "det_add_latency_cycles")
    return v.value


def set_profiling(enable: bool) -> None:
    """Per-launch CUDA-event timing of the weight GEMV/GEMM kernels."""
    _check(lib().det_set_profiling(int(enable)), "det_set_profiling")


def device_expf(x: np.ndarray, device: int = 0) -> np.ndarray:
    """det-num ``exp_f32`` evaluated by the device kernel (numerics self-test)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    _check(lib().det_device_expf(device, _ptr(x), _ptr(y), x.size), "det_device_expf")
    return y


TOKENIZER_KINDS = ("byte_fallback", "byte_bpe", "sentencepiece")


def tokenizer_kind(gguf: bytes) -> str:
    """``Tokenizer::from_gguf``'s selection for a GGUF's tokenizer metadata
    (host only, no device)."""
    gb = np.frombuffer(gguf, np.uint8)
    k = C.c_int()
    _check(lib().det_tokenizer_kind(_ptr(gb), len(gguf), C.byref(k)), "det_tokenizer_kind")
    return TOKENIZER_KINDS[k.value]


def tokenize(gguf: bytes, data: bytes, codec: bool = False) -> np.ndarray:
    """``tokenize_bytes``, or with codec=True the codec symbols (tokens, and
    vocab + byte for byte escapes), of the GGUF's tokenizer (host only)."""
    gb = np.frombuffer(gguf, np.uint8)
    ib = np.frombuffer(data, np.uint8) if data else np.zeros(1, np.uint8)
    out, n = C.c_void_p(), C.c_size_t()
    _check(lib().det_tokenize(_ptr(gb), len(gguf), _ptr(ib), len(data), int(codec), C.byref(out), C.byref(n)),
           "det_tokenize")
    return np.frombuffer(_take(out, 4 * n.value), np.uint32).copy()


def detokenize(gguf: bytes, symbols, byte_escapes: bool = True) -> bytes:
    """The bytes of a token / codec symbol sequence (host only)."""
    gb = np.frombuffer(gguf, np.uint8)
    s = np.ascontiguousarray(symbols, np.uint32)
    sb = s if s.size else np.zeros(1, np.uint32)
    out, n = C.c_void_p(), C.c_size_t()
    _check(lib().det_detokenize(_ptr(gb), len(gguf), _ptr(sb), s.size, int(byte_escapes), C.byref(out),
                                C.byref(n)), "det_detokenize")
    return _take(out, n.value)


def compress(model: Model, data: bytes, n_ctx: int = 0) -> bytes:
    """``detllm compress``: DTLZ bytes for ``data`` (n_ctx 0 = model context)."""
    buf = np.frombuffer(data, np.uint8) if data else np.zeros(1, np.uint8)
    out, n = C.c_void_p(), C.c_size_t()
    _check(lib().det_compress(model._h, _ptr(buf), len(data), n_ctx, C.byref(out), C.byref(n)), "det_compress")
    return _take(out, n.value)


def decompress(model: Model, dtlz: bytes) -> bytes:
    """``detllm decompress``: restores the bytes, after the canonical re-encode check."""
    buf = np.frombuffer(dtlz, np.uint8) if dtlz else np.zeros(1, np.uint8)
    out, n = C.c_void_p(), C.c_size_t()
    _check(lib().det_decompress(model._h, _ptr(buf), len(dtlz), C.byref(out), C.byref(n)), "det_decompress")
    return _take(out, n.value)
