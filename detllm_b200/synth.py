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
