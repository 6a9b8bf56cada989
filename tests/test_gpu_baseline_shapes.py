"""GPU parity at the shapes the benchmark runs.

The other GPU parity tests use small models.  These run the kernels on the
configurations' real widths, vocabularies, window lengths, RoPE bases and
the 1,024-position encode chunk, with the layer count cut to one so that
the CPU oracle finishes in seconds:

* config 2 (TinyLlama-1.1B shape, Q8_0): d 2048, 32/4 heads, FFN 5632,
  V 32,000, n_ctx 2048; logits over two chunks (1,024 + 76 positions) and
  the DTLZ payload of 2,600 symbols (a window rollover with its replay);
* config 3 (the same shape, Q4_K / Q6_K mix, Q4_K embedding): compress of
  Markov bytes through the byte-fallback tokenizer past a rollover, and
  decompress back to the input;
* config 4 (Qwen2.5-0.5B shape): V 151,936 tied, QKV bias, split-half RoPE
  at theta 1e6, n_ctx 4096; logits over two chunks and the payload of
  4,160 symbols (a rollover at 4,096);
* config 5 (Llama-3-8B shape): head_dim 128, 32/8 heads, FFN 14,336,
  V 128,256, Q4_K / Q6_K; logits over two chunks and symbol ranges at the
  full vocabulary;
* config 5's attention and RoPE at full length: head_dim 128, GQA 4,
  theta 5e5, every position of an 8,192 window (chunked and one-position
  forwards) and a payload that rolls the window over.

Every comparison is bit for bit (logits, ranges, DTLZ bytes): the
reference's f32 order is normative, so the tolerance is zero ULP.
"""
import dataclasses
import hashlib

import numpy as np
import pytest

from detllm_b200 import synth as S

pytestmark = pytest.mark.gpu

CHUNK = 1024  # the encode chunk the benchmark and det_encode_symbols use


@pytest.fixture(scope="module")
def D():
    import detllm_b200

    assert detllm_b200.device_count() > 0, "gpu tests need a CUDA device"
    return detllm_b200


def one_layer(name, **kw):
    return dataclasses.replace(S.CONFIGS[name], n_layer=1, **kw)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def chunked_logits(model, toks, n_ctx, visit):
    """Forward `toks` in chunks of CHUNK positions through one session and
    call visit(p0, logits of the chunk, session) after each chunk."""
    with model.session(n_ctx=n_ctx, max_chunk=CHUNK) as s:
        for p in range(0, len(toks), CHUNK):
            visit(p, s.forward(toks[p:p + CHUNK], p, want_logits=True), s)


def gpu_logits_hash(model, toks, n_ctx):
    h = hashlib.sha256()
    chunked_logits(model, toks, n_ctx, lambda p, lg, s: h.update(np.ascontiguousarray(lg, "<f4").tobytes()))
    return h.digest()


@pytest.mark.parametrize("name,n_sym", [("tinyllama-q8_0", 2600), ("qwen2.5-0.5b-q8_0", 4160)])
def test_q8_0_configs_logits_and_payload(D, oracle, name, n_sym):
    spec = one_layer(name)
    g = S.build_gguf(spec)
    om, m = oracle.Model(g), D.Model(g)
    toks = S.zipf_tokens(1100, spec.vocab, seed=17)
    # the oracle's hash covers the same logits in the same order (chunk-invariant)
    assert gpu_logits_hash(m, toks, spec.ctx) == om.logits_hash(toks, 1)
    n_ctx, overlap = spec.ctx, spec.ctx // 4
    syms = S.zipf_tokens(n_sym, spec.vocab + 256, seed=19)  # byte escapes included
    assert m.encode_symbols(syms, n_ctx, overlap) == om.encode_symbols(syms, n_ctx, overlap)


def test_q4_k_m_config_compress_and_decompress(D, oracle):
    spec = one_layer("tinyllama-q4_k_m")
    g = S.build_gguf(spec)
    m = D.Model(g)
    toks = S.zipf_tokens(1100, spec.vocab, seed=23)
    assert gpu_logits_hash(m, toks, spec.ctx) == oracle.Model(g).logits_hash(toks, 1)
    data = S.markov_text(2200, seed=29)  # 2,200 byte tokens: one rollover at n_ctx 2048
    got = D.compress(m, data, spec.ctx)
    assert got == oracle.compress(g, data, spec.ctx)
    assert D.decompress(m, got) == data


def test_llama3_8b_shape_logits_and_ranges(D, oracle):
    spec = one_layer("llama3-8b-q4_k")
    g = S.build_gguf(spec)
    toks = S.zipf_tokens(1060, spec.vocab, seed=31)
    want = oracle.Model(g).logits(toks)
    m = D.Model(g)
    rng = np.random.default_rng(5)
    checked = []

    def visit(p, lg, s):
        diff = np.nonzero(bits(lg) != bits(want[p:p + len(lg)]))
        assert diff[0].size == 0, f"{diff[0].size} logits differ, first at {p + diff[0][0]},{diff[1][0]}"
        rows = rng.integers(0, len(lg), 24).astype(np.uint32)
        syms = rng.integers(0, spec.vocab + 256, 24).astype(np.uint32)
        syms[:3] = [0, spec.vocab - 1, spec.vocab + 255]
        got = s.symbol_ranges(syms, rows, byte_escapes=True)
        for i in range(len(rows)):
            assert tuple(int(v) for v in got[i]) == oracle.symbol_range(want[p + rows[i]], int(syms[i]), True)
        checked.append(len(lg))

    chunked_logits(m, toks, spec.ctx, visit)
    assert checked == [1024, 36]


LONG = S.ModelSpec(n_layer=1, d=512, d_ff=512, n_head=4, n_head_kv=1, vocab=1024, ctx=8192, rope_base=500000.0,
                   t_embd=S.GT_Q4_K, t_attn=S.GT_Q4_K, t_gate_up=S.GT_Q4_K, t_down=S.GT_Q6_K, t_out=S.GT_Q6_K,
                   seed=51)


@pytest.fixture(scope="module")
def long_window(oracle):
    g = S.build_gguf(LONG)
    toks = S.zipf_tokens(8192, LONG.vocab, seed=3)
    return g, toks, oracle.Model(g).logits(toks)


def test_full_window_logits_chunked_and_one_position(D, long_window):
    """head_dim 128, GQA 4, RoPE theta 5e5 at every position 0..8191: the
    1,024-position chunks (tiled attention over up to 8,192 keys), then the
    last 64 positions again as one-position forwards (decode kernels)."""
    g, toks, want = long_window
    m = D.Model(g)
    got = np.empty_like(want)

    def visit(p, lg, s):
        got[p:p + len(lg)] = lg

    chunked_logits(m, toks, LONG.ctx, visit)
    diff = np.nonzero(bits(got) != bits(want))
    assert diff[0].size == 0, f"{diff[0].size} logits differ, first at {diff[0][0]},{diff[1][0]}"
    with m.session(n_ctx=LONG.ctx, max_chunk=CHUNK) as s:
        for p in range(0, 8128, CHUNK):
            n = min(CHUNK, 8128 - p)
            s.forward(toks[p:p + n], p)
        for p in range(8128, 8192):
            lg = s.forward(toks[p:p + 1], p, want_logits=True)
            assert (bits(lg[0]) == bits(want[p])).all(), f"one-position logits differ at {p}"


def test_full_window_payload_with_rollover(D, oracle, long_window):
    g = long_window[0]
    syms = S.zipf_tokens(8400, LONG.vocab + 256, seed=4)
    assert D.Model(g).encode_symbols(syms, 8192, 2048) == oracle.Model(g).encode_symbols(syms, 8192, 2048)
