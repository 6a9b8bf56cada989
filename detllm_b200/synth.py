"""Seeded synthetic models and inputs for the benchmark configurations.

No real checkpoints or datasets are available offline, so the benchmark and
the parity tests use random-init weights of the named architectures and
seeded synthetic token / byte streams with the shapes the configurations
name.  Everything here is deterministic in (config, seed).

* weights: N(0, 0.02) values, quantised to the GGUF block formats that
  det-quant decodes (Q8_0, Q4_0, Q4_K, Q6_K; crates/det-quant/src/lib.rs:
  506-568 fixes the layouts); norm weights 1.0; qwen2 QKV biases N(0, 0.02);
* vocabulary: 256 byte-fallback tokens ``<0xNN>`` followed by filler pieces,
  so det-token selects its ByteFallbackTokenizer (lib.rs:111-130);
* inputs: Zipf(s) token ids over the vocabulary through a seeded permutation,
  and order-2 Markov text over printable ASCII plus '<' / '>' markup.
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np

GT_F32, GT_F16, GT_Q4_0, GT_Q8_0, GT_Q4_K, GT_Q6_K = 0, 1, 2, 8, 12, 14


@dataclasses.dataclass
class ModelSpec:
    arch: str = "llama"             # "llama" (adjacent RoPE) or "qwen2" (split-half RoPE, QKV bias)
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
    # ggml types: token_embd, attn (q,k,v,o), ffn gate/up, ffn down, output
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


def _f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def _f16_val(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


def quant_q8_0(w: np.ndarray) -> bytes:
    """d = f16(amax / 127), q = round(x / d) per 32-block (ggml Q8_0)."""
    b = w.reshape(-1, 32).astype(np.float32)
    amax = np.abs(b).max(axis=1)
    dbits = _f16_bits(amax / 127.0)
    d = _f16_val(dbits)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1.0), 0.0).astype(np.float32)
    q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), np.uint8)
    out[:, 0:2] = dbits.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def quant_q4_0(w: np.ndarray) -> bytes:
    """ggml Q4_0: d = max/-8, q = clip(round(x/d) + 8, 0, 15); low nibbles hold
    elements 0..15, high nibbles 16..31 (det-quant lib.rs:455-466)."""
    b = w.reshape(-1, 32).astype(np.float32)
    idx = np.abs(b).argmax(axis=1)
    mx = b[np.arange(b.shape[0]), idx]
    dbits = _f16_bits(mx / -8.0)
    d = _f16_val(dbits)
    inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1.0), 0.0).astype(np.float32)
    q = np.clip(np.rint(b * inv[:, None]) + 8, 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], 18), np.uint8)
    out[:, 0:2] = dbits.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.tobytes()


def quant_q4_k(w: np.ndarray) -> bytes:
    """Q4_K super-blocks: value = (d*sc)*q - dmin*m with 6-bit (sc, m) per
    32-element sub-block, packed as q4_k_scale_min decodes them
    (det-quant lib.rs:506-529)."""
    b = w.reshape(-1, 8, 32).astype(np.float32)
    mn = np.minimum(b.min(axis=2), 0.0)
    mx = b.max(axis=2)
    scale = (mx - mn) / 15.0
    dmin_bits = _f16_bits(np.maximum(-mn.min(axis=1), 1e-8) / 63.0)
    d_bits = _f16_bits(np.maximum(scale.max(axis=1), 1e-8) / 63.0)
    d, dmin = _f16_val(d_bits), _f16_val(dmin_bits)
    sc = np.clip(np.rint(scale / d[:, None]), 1, 63).astype(np.uint8)
    m = np.clip(np.rint(-mn / dmin[:, None]), 0, 63).astype(np.uint8)
    step = (d[:, None] * sc)[..., None]
    off = (dmin[:, None] * m)[..., None]
    q = np.clip(np.rint((b + off) / step), 0, 15).astype(np.uint8)
    nb = b.shape[0]
    scales = np.zeros((nb, 12), np.uint8)
    for i in range(4):
        scales[:, i] = (sc[:, i] & 63) | ((sc[:, i + 4] >> 4) << 6)
        scales[:, i + 4] = (m[:, i] & 63) | ((m[:, i + 4] >> 4) << 6)
        scales[:, i + 8] = (sc[:, i + 4] & 15) | ((m[:, i + 4] & 15) << 4)
    qs = np.empty((nb, 128), np.uint8)
    for k in range(4):
        qs[:, k * 32:(k + 1) * 32] = q[:, 2 * k] | (q[:, 2 * k + 1] << 4)
    out = np.empty((nb, 144), np.uint8)
    out[:, 0:2] = d_bits.view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dmin_bits.view(np.uint8).reshape(-1, 2)
    out[:, 4:16] = scales
    out[:, 16:] = qs
    return out.tobytes()


def quant_q6_k(w: np.ndarray) -> bytes:
    """Q6_K super-blocks: value = (d*sc)*(q - 32), int8 sc per 16 elements,
    q split into ql (low 4 bits) and qh (high 2 bits) as q6_k_quant reads
    them (det-quant lib.rs:536-568)."""
    x = w.reshape(-1, 256).astype(np.float32)
    nb = x.shape[0]
    # element index i -> (half, part, l): i = half*128 + part*32 + l
    g = x.reshape(nb, 16, 16)  # scale group = i // 16 (scale index = half*8 + l//16 + 2*part)
    amax = np.abs(g).max(axis=2)
    gscale = amax / 31.0
    d_bits = _f16_bits(np.maximum(gscale.max(axis=1), 1e-10) / 127.0)
    d = _f16_val(d_bits)
    sc = np.clip(np.rint(gscale / d[:, None]), 1, 127).astype(np.int8)
    # scale for element i: index half*8 + l//16 + 2*part with i = half*128+part*32+l
    i = np.arange(256)
    half, within = i // 128, i % 128
    part, l = within // 32, within % 32
    sidx = half * 8 + l // 16 + 2 * part
    step = d[:, None] * sc[:, sidx].astype(np.float32)
    q = np.clip(np.rint(x / step) + 32, 0, 63).astype(np.uint8)
    ql = np.zeros((nb, 128), np.uint8)
    qh = np.zeros((nb, 64), np.uint8)
    for hf in range(2):
        for p in range(4):
            qq = q[:, hf * 128 + p * 32: hf * 128 + p * 32 + 32]
            lo, hi = qq & 15, qq >> 4
            base = hf * 64 + (32 if p in (1, 3) else 0)
            if p < 2:
                ql[:, base:base + 32] |= lo
            else:
                ql[:, base:base + 32] |= lo << 4
            qh[:, hf * 32: hf * 32 + 32] |= hi << (2 * p)
    out = np.empty((nb, 210), np.uint8)
    out[:, 0:128] = ql
    out[:, 128:192] = qh
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d_bits.view(np.uint8).reshape(-1, 2)
    return out.tobytes()


def encode_tensor(w: np.ndarray, ty: int) -> bytes:
    if ty == GT_F32:
        return np.asarray(w, "<f4").tobytes()
    if ty == GT_F16:
        return np.asarray(w, np.float16).tobytes()
    return {GT_Q8_0: quant_q8_0, GT_Q4_0: quant_q4_0, GT_Q4_K: quant_q4_k, GT_Q6_K: quant_q6_k}[ty](w)


class _GgufWriter:
    def __init__(self):
        self.kv = []
        self.tensors = []
        self.data = bytearray()

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode()
        return struct.pack("<Q", len(b)) + b

    def u32(self, k, v):
        self.kv.append(self._str(k) + struct.pack("<II", 4, v))

    def f32(self, k, v):
        self.kv.append(self._str(k) + struct.pack("<If", 6, v))

    def string(self, k, v):
        self.kv.append(self._str(k) + struct.pack("<I", 8) + self._str(v))

    def str_array(self, k, vals):
        body = b"".join(self._str(v) for v in vals)
        self.kv.append(self._str(k) + struct.pack("<IIQ", 9, 8, len(vals)) + body)

    def i32_array(self, k, vals):
        self.kv.append(self._str(k) + struct.pack("<IIQ", 9, 5, len(vals)) + np.asarray(vals, "<i4").tobytes())

    def tensor(self, name, dims, ty, payload: bytes):
        while len(self.data) % 32:
            self.data.append(0)
        self.tensors.append((name, dims, ty, len(self.data)))
        self.data += payload

    def bytes(self) -> bytes:
        out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(self.tensors), len(self.kv)))
        for kv in self.kv:
            out += kv
        for name, dims, ty, off in self.tensors:
            out += self._str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
            out += struct.pack("<IQ", ty, off)
        while len(out) % 32:
            out.append(0)
        return bytes(out + self.data)


def vocab_pieces(n: int):
    toks = [f"<0x{b:02X}>" for b in range(256)]
    toks += [f"tok{i}" for i in range(256, n)]
    return toks[:n]


def build_gguf(spec: ModelSpec, progress=None) -> bytes:
    """A GGUF v3 file of `spec` with seeded random-init weights."""
    rng = np.random.default_rng(spec.seed)
    w = _GgufWriter()
    a = spec.arch
    w.string("general.architecture", a)
    w.u32(f"{a}.block_count", spec.n_layer)
    w.u32(f"{a}.embedding_length", spec.d)
    w.u32(f"{a}.feed_forward_length", spec.d_ff)
    w.u32(f"{a}.attention.head_count", spec.n_head)
    w.u32(f"{a}.attention.head_count_kv", spec.n_head_kv)
    w.f32(f"{a}.attention.layer_norm_rms_epsilon", spec.eps)
    w.f32(f"{a}.rope.freq_base", spec.rope_base)
    w.u32(f"{a}.context_length", spec.ctx)
    w.u32(f"{a}.vocab_size", spec.vocab)
    w.str_array("tokenizer.ggml.tokens", vocab_pieces(spec.vocab))
    if spec.escape_bytes:
        types = np.ones(spec.vocab, np.int32)
        types[list(spec.escape_bytes)] = 3
        w.i32_array("tokenizer.ggml.token_type", types)
    hd = spec.head_dim

    def mat(name, rows, cols, ty):
        x = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
        w.tensor(name, [cols, rows], ty, encode_tensor(x, ty))

    def vec(name, n, value=None):
        x = np.full(n, 1.0, np.float32) if value is None else value
        w.tensor(name, [n], GT_F32, np.asarray(x, "<f4").tobytes())

    mat("token_embd.weight", spec.vocab, spec.d, spec.t_embd)
    for l in range(spec.n_layer):
        p = f"blk.{l}."
        vec(p + "attn_norm.weight", spec.d)
        mat(p + "attn_q.weight", spec.n_head * hd, spec.d, spec.t_attn)
        if spec.qkv_bias:
            vec(p + "attn_q.bias", spec.n_head * hd, rng.standard_normal(spec.n_head * hd, np.float32) * 0.02)
        mat(p + "attn_k.weight", spec.n_head_kv * hd, spec.d, spec.t_attn)
        if spec.qkv_bias:
            vec(p + "attn_k.bias", spec.n_head_kv * hd, rng.standard_normal(spec.n_head_kv * hd, np.float32) * 0.02)
        mat(p + "attn_v.weight", spec.n_head_kv * hd, spec.d, spec.t_attn)
        if spec.qkv_bias:
            vec(p + "attn_v.bias", spec.n_head_kv * hd, rng.standard_normal(spec.n_head_kv * hd, np.float32) * 0.02)
        mat(p + "attn_output.weight", spec.d, spec.n_head * hd, spec.t_attn)
        vec(p + "ffn_norm.weight", spec.d)
        mat(p + "ffn_gate.weight", spec.d_ff, spec.d, spec.t_gate_up)
        mat(p + "ffn_up.weight", spec.d_ff, spec.d, spec.t_gate_up)
        mat(p + "ffn_down.weight", spec.d, spec.d_ff, spec.t_down)
        if progress:
            progress(l + 1, spec.n_layer)
    vec("output_norm.weight", spec.d)
    if not spec.tied:
        mat("output.weight", spec.vocab, spec.d, spec.t_out)
    return w.bytes()


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
    for ch in (b"<"[0], b">"[0]):
        weights[:, :, int(np.where(alphabet == ch)[0][0])] += 0.5
    probs = weights / weights.sum(axis=2, keepdims=True)
    cdf = np.cumsum(probs, axis=2)
    out = np.empty(n, np.uint8)
    a, b = 0, 1
    u = rng.random(n)
    for i in range(n):
        c = int(np.searchsorted(cdf[a, b], u[i]))
        c = min(c, k - 1)
        out[i] = alphabet[c]
        a, b = b, c
    return out.tobytes()
