"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Integer / byte / index results must be bit-exact, and so must every float:
the reference's numerics are normative (fixed reduction order, explicit
rounding), so the tolerance for logits is zero ULP.
"""
import dataclasses
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from detllm_b200 import synth as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def D():
    import detllm_b200

    assert detllm_b200.device_count() > 0, "gpu tests need a CUDA device"
    return detllm_b200


SPECS = {
    "q8_0": S.ModelSpec(n_layer=2, d=256, d_ff=512, n_head=4, n_head_kv=2, vocab=1024, ctx=64),
    "q4k_q6k": S.ModelSpec(n_layer=2, d=256, d_ff=512, n_head=4, n_head_kv=2, vocab=1024, ctx=64,
                           t_embd=S.GT_Q4_K, t_attn=S.GT_Q4_K, t_gate_up=S.GT_Q4_K, t_down=S.GT_Q6_K,
                           t_out=S.GT_Q6_K, seed=5),
    "qwen2_bias_tied_q4_0": S.ModelSpec(arch="qwen2", n_layer=2, d=128, d_ff=256, n_head=2, n_head_kv=1, vocab=600,
                                        ctx=64, tied=True, qkv_bias=True, rope_base=1e6, t_attn=S.GT_Q4_0, seed=9),
    # one-position K-quant kernels: a Q6_K ffn_down 8448 wide (two passes of
    # 32 blocks) and 1000 output rows (a ragged 32-row tile)
    "q4k_q6k_wide_ffn": S.ModelSpec(n_layer=1, d=256, d_ff=8448, n_head=4, n_head_kv=2, vocab=1000, ctx=64,
                                    t_embd=S.GT_Q4_K, t_attn=S.GT_Q4_K, t_gate_up=S.GT_Q4_K, t_down=S.GT_Q6_K,
                                    t_out=S.GT_Q6_K, seed=6),
    # a Q6_K ffn_down wider than 16,384 (65 blocks): the one-position Q6_K
    # kernel that stages no activation pairs
    "q6k_down_65_blocks": S.ModelSpec(n_layer=1, d=256, d_ff=16640, n_head=4, n_head_kv=2, vocab=300, ctx=64,
                                      t_embd=S.GT_Q4_K, t_attn=S.GT_Q4_K, t_gate_up=S.GT_Q4_K, t_down=S.GT_Q6_K,
                                      t_out=S.GT_Q6_K, seed=8),
    "f16_f32_escapes": S.ModelSpec(n_layer=1, d=64, d_ff=128, n_head=2, n_head_kv=2, vocab=300, ctx=32,
                                   t_embd=S.GT_F16, t_attn=S.GT_F32, t_gate_up=S.GT_F16, t_down=S.GT_Q8_0,
                                   t_out=S.GT_F32, escape_bytes=(10, 32, 65), seed=3),
}


# Longer windows: several 64-key tiles, several query blocks per chunk,
# GQA groups of 8 and 7 (a 63-row block) and head_dim 128.
LONG_SPECS = {
    "hd64_gqa8": S.ModelSpec(n_layer=2, d=512, d_ff=256, n_head=8, n_head_kv=1, vocab=512, ctx=320, seed=21),
    "hd64_gqa7_qwen2": S.ModelSpec(arch="qwen2", n_layer=1, d=448, d_ff=256, n_head=7, n_head_kv=1, vocab=400,
                                   ctx=320, qkv_bias=True, rope_base=1e6, seed=22),
    "hd128_gqa2": S.ModelSpec(n_layer=1, d=256, d_ff=256, n_head=2, n_head_kv=1, vocab=512, ctx=320,
                              t_attn=S.GT_Q4_0, seed=23),
    # Q4_K attention / gate / up and embedding, Q6_K down and output: the
    # K-quant chunk path over several row tiles and position groups
    "hd64_q4k_m": S.ModelSpec(n_layer=1, d=512, d_ff=768, n_head=8, n_head_kv=2, vocab=300, ctx=320,
                              t_embd=S.GT_Q4_K, t_attn=S.GT_Q4_K, t_gate_up=S.GT_Q4_K, t_down=S.GT_Q6_K,
                              t_out=S.GT_Q6_K, seed=24),
}


@pytest.fixture(scope="module")
def models():
    return {k: S.build_gguf(v) for k, v in SPECS.items()}


@pytest.fixture(scope="module")
def long_models(oracle):
    out = {}
    for k, spec in LONG_SPECS.items():
        g = S.build_gguf(spec)
        toks = S.zipf_tokens(300, spec.vocab, seed=len(k))
        out[k] = (g, toks, oracle.Model(g).logits(toks))
    return out


@pytest.mark.parametrize("name", list(LONG_SPECS))
@pytest.mark.parametrize("chunk", [1, 37, 128, 300])  # 1: one-position forwards
def test_long_window_logits_bit_exact(D, long_models, name, chunk):
    g, toks, want = long_models[name]
    got = D.Model(g).logits_for_tokens(toks, chunk=chunk)
    diff = np.nonzero(bits(got) != bits(want))
    assert diff[0].size == 0, f"{diff[0].size} logits differ, first at {diff[0][0]},{diff[1][0]}"


@pytest.mark.parametrize("name", ["hd64_gqa8", "hd128_gqa2"])  # Q8_0 everywhere; Q4_0 attention
@pytest.mark.parametrize("chunk", [37, 300])
def test_q8_chunk_gemm_tcgen05_kernel(D, long_models, name, chunk):
    """The tcgen05 chunk GEMM (the alternative to the default mma.sync one)
    gives the same bits; 37 positions leave the second 64-position group of
    the CTA absent."""
    g, toks, want = long_models[name]
    prev = D.set_q8_tensor_cores(True)
    try:
        got = D.Model(g).logits_for_tokens(toks, chunk=chunk)
    finally:
        D.set_q8_tensor_cores(prev)
    diff = np.nonzero(bits(got) != bits(want))
    assert diff[0].size == 0, f"{diff[0].size} logits differ, first at {diff[0][0]},{diff[1][0]}"


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# The child process of test_fused_one_position_forward: DETGPU_FUSED_DECODE is
# read once per process, so the fused path runs in a process of its own.
_FUSED_CHILD = """
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import detllm_b200 as D
from detllm_b200 import synth as S
spec = S.ModelSpec(**json.loads(sys.argv[2]))
toks = np.array(json.loads(sys.argv[3]), np.uint32)
m = D.Model(S.build_gguf(spec))
D.set_profiling(True)
got = m.logits_for_tokens(toks, chunk=1)
D.set_profiling(False)
np.save(sys.argv[4], got)
print(json.dumps(m.profile(reset=True)))
"""


@pytest.mark.parametrize("name", ["hd64_gqa8", "hd64_gqa7_qwen2", "hd128_gqa2"])
def test_fused_one_position_forward(D, long_models, name, tmp_path):
    """DETGPU_FUSED_DECODE=1: models whose weights are all Q8_0 / Q4_0 run
    each one-position forward as one persistent kernel (decode_fused.cu), one
    launch per token, with logits bit-exact against the oracle over score
    lengths 1..120 (two 64-key tiles; GQA groups of 8 and 7, split-half RoPE
    with q/k/v biases, head_dim 128 with Q4_0 attention)."""
    g, toks, want = long_models[name]
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = tmp_path / "logits.npy"
    env = dict(os.environ, DETGPU_FUSED_DECODE="1")
    r = subprocess.run([sys.executable, "-c", _FUSED_CHILD, root, json.dumps(dataclasses.asdict(LONG_SPECS[name])),
                        json.dumps([int(t) for t in toks[:120]]), str(out)],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    prof = json.loads(r.stdout.strip().splitlines()[-1])
    assert prof["decode_fused"][0] == 120, prof
    assert prof["gemm_qkv"][0] == 0 and prof["attention"][0] == 0, prof
    got = np.load(out)
    diff = np.nonzero(bits(got) != bits(want[:120]))
    assert diff[0].size == 0, f"{diff[0].size} logits differ, first at {diff[0][0]},{diff[1][0]}"


def test_add_latency_probe(D):
    """det_add_latency_cycles: one dependent f32 add takes a few cycles (the
    chain floor bench.py reports decode against)."""
    c = D.add_latency_cycles(0)
    assert 1.0 < c < 64.0, c


def test_device_expf_matches_vendored_expf(D, oracle):
    # every 251st bit pattern of the f32 space plus dense sweeps where the
    # algorithm changes branch (expf.rs:47-80) and the softmax/CDF range
    pats = np.arange(0, 2**32, 251, dtype=np.uint64).astype(np.uint32)
    dense = [np.linspace(-104.0, 89.0, 2_000_001, dtype=np.float32).view(np.uint32)]
    for c in (0x42AEAC50, 0x42B17218, 0x42CFF1B5, 0x3EB17218, 0x3F851592, 0x39000000):
        for s in (0, 0x80000000):
            dense.append(np.arange(c - 4096, c + 4096, dtype=np.uint32) | s)
    x = np.concatenate([pats] + dense).view(np.float32)
    got = D.device_expf(x)
    want = oracle.expf(x)
    ok = (bits(got) == bits(want)) | (np.isnan(got) & np.isnan(want))
    assert ok.all(), (x[~ok][:5], got[~ok][:5], want[~ok][:5])


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-qmix"])
@pytest.mark.parametrize("chunk", [1, 2, 3, 6])
def test_fixture_logits_hash(D, goldens, fixtures, name, chunk):
    # testdata/*.logits.sha256 through det_logits_hash
    m = D.Model(fixtures[name])
    h = m.logits_hash_for_tokens_chunked(goldens["tokens"], chunk)
    assert h.hex() == goldens[name.replace("-", "_") + "_logits_sha256"]


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-qmix", "q4k_q6k"])
def test_position_invariance_under_replay(D, goldens, fixtures, models, name):
    # det-model lib.rs:3681-3724, 3761-3796: the logits of position p from
    # continuous one-position forwards equal those of a fresh cache that
    # replays positions 0..p, bit for bit; here the replay also runs as one
    # teacher-forced chunk, whose last row must be the same logits
    g = fixtures[name] if name in fixtures else models[name]
    toks = goldens["tokens"] if name in fixtures else [int(t) for t in S.zipf_tokens(12, SPECS[name].vocab, seed=2)]
    m = D.Model(g)
    with m.session(n_ctx=len(toks), max_chunk=len(toks)) as s:
        cont = [bits(s.forward([t], p, want_logits=True)[0]) for p, t in enumerate(toks)]
        for end in range(len(toks)):
            s.reset()
            for p in range(end + 1):
                lg = s.forward([toks[p]], p, want_logits=True)[0]
            assert (bits(lg) == cont[end]).all(), f"one-position replay differs at {end}"
            s.reset()
            lg = s.forward(toks[:end + 1], 0, want_logits=True)[-1]
            assert (bits(lg) == cont[end]).all(), f"chunked replay differs at {end}"
    m.close()


@pytest.mark.parametrize("name", list(SPECS))
@pytest.mark.parametrize("chunk", [1, 7, 12, 24])  # decode, decode (T <= 8), small-T and chunk GEMM paths
def test_logits_bit_exact(D, oracle, models, name, chunk):
    spec = SPECS[name]
    toks = S.zipf_tokens(24, spec.vocab, seed=hash(name) % 1000)
    want = oracle.Model(models[name]).logits(toks)
    got = D.Model(models[name]).logits_for_tokens(toks, chunk=chunk)
    assert got.shape == want.shape
    diff = np.nonzero(bits(got) != bits(want))
    assert diff[0].size == 0, f"{diff[0].size} logits differ, first at {diff[0][0]},{diff[1][0]}"


@pytest.mark.parametrize("name", ["q8_0", "q4k_q6k"])
def test_symbol_ranges_and_decoder(D, oracle, models, name):
    spec = SPECS[name]
    m = D.Model(models[name])
    toks = S.zipf_tokens(16, spec.vocab, seed=3)
    rng = np.random.default_rng(0)
    with m.session(n_ctx=32, max_chunk=16) as s:
        logits = s.forward(toks, 0, want_logits=True)
        rows = rng.integers(0, 16, 200).astype(np.uint32)
        syms = rng.integers(0, spec.vocab + 256, 200).astype(np.uint32)
        syms[:8] = [0, spec.vocab - 1, spec.vocab, spec.vocab + 255, 1, 2, 3, 4]
        got = s.symbol_ranges(syms, rows, byte_escapes=True)
        for i in range(200):
            assert tuple(int(v) for v in got[i]) == oracle.symbol_range(logits[rows[i]], int(syms[i]), True)
        got_ne = s.symbol_ranges(syms % spec.vocab, rows, byte_escapes=False)
        for i in range(0, 200, 7):
            want = oracle.symbol_range(logits[rows[i]], int(syms[i] % spec.vocab), False)
            assert tuple(int(v) for v in got_ne[i]) == want
        for row in (0, 5, 15):
            total = s.decoder_total(row)
            assert total == oracle.decoder_total(logits[row])
            for value in list(rng.integers(0, total, 40)) + [0, total - 1, total - 256, total - 257]:
                got = s.decoder_lookup(row, int(value))
                assert got == oracle.decoder_lookup(logits[row], int(value))


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-qmix"])
def test_fixture_codec_bytes(D, oracle, goldens, fixtures, name):
    # testdata_cli.rs:220-310 cases + docs/validation.md codec sizes
    m = D.Model(fixtures[name])
    cases = [b"", goldens["tiny_tokens_txt"].encode(), goldens["smoke_input"].encode(),
             "detllm deterministic 圧縮 smoke\n復元一致\n".encode(), bytes(range(256)) + b"detllm"]
    for data in cases:
        got = D.compress(m, data, 8)
        assert got == oracle.compress(fixtures[name], data, 8), (name, len(data))
        assert D.decompress(m, got) == data
    tok = goldens["tiny_tokens_txt"].encode()
    assert len(D.compress(m, tok, 8)) == goldens["tokens_txt_codec"][name]["dtlz"]


@pytest.mark.parametrize("name", list(SPECS))
@pytest.mark.parametrize("n_ctx", [2, 3, 9, 64])  # 2, 3: overlap 0, every window starts empty
def test_codec_bytes_synthetic(D, oracle, models, name, n_ctx):
    spec = SPECS[name]
    n_ctx = min(n_ctx, spec.ctx)
    data = S.markov_text(120, seed=5) + bytes(range(0, 256, 5))
    m = D.Model(models[name])
    got = D.compress(m, data, n_ctx)
    assert got == oracle.compress(models[name], data, n_ctx)
    assert D.decompress(m, got) == data


@pytest.mark.parametrize("name", ["hd64_gqa8", "hd64_q4k_m"])
def test_codec_bytes_long_stream(D, oracle, long_models, name):
    # several windows of 320 positions with 80-position replays: chunk GEMMs
    # over several 64-position groups, tiled attention over several key
    # tiles, and one-token forwards (decode kernels) in decompress
    g = long_models[name][0]
    data = S.markov_text(1500, seed=8)
    m = D.Model(g)
    got = D.compress(m, data, 320)
    assert got == oracle.compress(g, data, 320)
    assert D.decompress(m, got) == data


def test_encode_symbols_streams(D, oracle, models):
    spec = SPECS["q8_0"]
    g = models["q8_0"]
    rng = np.random.default_rng(1)
    m, om = D.Model(g), oracle.Model(g)
    for n_ctx, overlap in ((8, 2), (3, 1), (5, 0), (64, 16)):
        syms = rng.integers(0, spec.vocab + 256, 90).astype(np.uint32)
        assert m.encode_symbols(syms, n_ctx, overlap) == om.encode_symbols(syms, n_ctx, overlap)
        toks = rng.integers(0, spec.vocab, 90).astype(np.uint32)
        assert m.encode_symbols(toks, n_ctx, overlap, False) == om.encode_symbols(toks, n_ctx, overlap, False)


def test_decompress_rejections(D, oracle, fixtures):
    m = D.Model(fixtures["tiny-f32"])
    d = D.compress(m, b"detllm", 8)
    with pytest.raises(D.DetError) as e:
        D.decompress(m, d + b"\0")
    assert e.value.code in (59, 41)
    with pytest.raises(D.DetError) as e:
        D.decompress(D.Model(fixtures["tiny-qmix"]), d)
    assert e.value.code == 58
    with pytest.raises(D.DetError) as e:
        D.decompress(m, d[:40])
    assert e.value.code == 48


def test_codec_calls_from_several_host_threads(D, oracle, models):
    # the reference's model is immutable (&self), so callers may share one
    # model between threads; the library's codec calls share a session
    # cached in the model and run one after another, with the bytes of
    # sequential calls
    import threading

    g = models["q8_0"]
    m = D.Model(g)
    inputs = [S.markov_text(300 + 40 * i, seed=80 + i) for i in range(6)]
    want = [D.compress(m, x, 48) for x in inputs]
    got, back, errors = [None] * len(inputs), [None] * len(inputs), []

    def work(i):
        try:
            got[i] = D.compress(m, inputs[i], 48)
            back[i] = D.decompress(m, got[i])
        except Exception as e:  # reported below
            errors.append(repr(e))

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(inputs))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    assert got == want and back == inputs
    assert want[0] == oracle.compress(g, inputs[0], 48)
    m.close()


def test_encode_rejects_invalid_windows(D, oracle, fixtures):
    # det-cli main.rs:1264-1287: n_ctx 0, overlap == n_ctx and n_ctx above
    # the model's context length fail with the window error, as the oracle does
    m = D.Model(fixtures["tiny-f32"])
    om = oracle.Model(fixtures["tiny-f32"])
    assert m.encode_symbols([0, 1], 3, 1) == om.encode_symbols([0, 1], 3, 1)
    for n_ctx, overlap in [(0, 0), (3, 3), (m.config.context_length + 1, 0)]:
        with pytest.raises(D.DetError) as e:
            m.encode_symbols([0, 1], n_ctx, overlap)
        assert e.value.code == 57, (n_ctx, overlap)
    assert m.encode_symbols([0, 1], 3, 1) == om.encode_symbols([0, 1], 3, 1)  # the model is still usable
    m.close()


def test_nonfinite_is_an_error_like_the_reference(D, oracle):
    # DET-4: an overflowing activation is rejected, not propagated
    spec = S.ModelSpec(n_layer=1, d=64, d_ff=128, n_head=2, n_head_kv=2, vocab=300, ctx=16, t_embd=S.GT_F32,
                       t_attn=S.GT_F32, t_gate_up=S.GT_F32, t_down=S.GT_F32, t_out=S.GT_F32)
    g = bytearray(S.build_gguf(spec))
    # output_norm.weight (the 64 floats just before the last tensor) set to
    # 3e38: the final RMSNorm output overflows wherever |x * r| > 1.14
    n = 300 * 64 * 4
    g[len(g) - n - 256:len(g) - n] = np.full(64, 3e38, "<f4").tobytes()
    g = bytes(g)
    with pytest.raises(oracle.OracleError) as eo:
        oracle.Model(g).logits([1, 2])
    with pytest.raises(D.DetError) as eg:
        D.Model(g).logits_for_tokens([1, 2])
    assert eo.value.code == eg.value.code == 2


# (block bytes, offset of the f16 scale in the block) of the lm_head types
_SCALE_AT = {S.GT_Q8_0: (34, 0), S.GT_Q4_0: (18, 0), S.GT_Q4_K: (144, 0), S.GT_Q6_K: (210, 208), S.GT_F16: (2, 0)}


@pytest.mark.parametrize("t_out", list(_SCALE_AT))
def test_load_rejects_a_nonfinite_scale(D, oracle, t_out):
    """The device repack checks every block scale as the reference's readers
    do: an infinite f16 scale in the last block of output.weight (the last
    tensor of the file) fails the load with the oracle's status."""
    spec = S.ModelSpec(n_layer=1, d=256, d_ff=256, n_head=2, n_head_kv=2, vocab=300, ctx=16, t_out=t_out, seed=4)
    g = bytearray(S.build_gguf(spec))
    block, at = _SCALE_AT[t_out]
    p = len(g) - block + at
    g[p:p + 2] = b"\x00\x7c"  # +inf
    g = bytes(g)
    with pytest.raises(oracle.OracleError) as eo:
        oracle.Model(g).logits([1, 2])
    with pytest.raises(D.DetError) as eg:
        D.Model(g)
    assert eo.value.code == eg.value.code == 2


@pytest.mark.parametrize("kind", ["spm", "bpe"])
def test_codec_bytes_sentencepiece_and_bpe(D, oracle, kind):
    """compress / decompress through a SentencePiece and a byte-level BPE
    vocabulary (multi-byte tokens, det-token lib.rs:328-617) at n_ctx 48 (many
    window rollovers): DTLZ bytes equal to the oracle's, and decompress
    restores the input."""
    spec = S.ModelSpec(n_layer=1, d=128, d_ff=256, n_head=2, n_head_kv=1, vocab=700, ctx=64, seed=41)
    g = S.with_tokenizer(S.build_gguf(spec), S.synthetic_tokenizer_kvs(kind, 700, seed=5))
    data = S.markov_text(600, seed=5) + bytes([0, 255, 10])
    want = oracle.compress(g, data, 48)
    m = D.Model(g)
    got = D.compress(m, data, 48)
    assert got == want
    assert D.decompress(m, got) == data


def test_pipeline_wait_times_out_and_device_recovers(D):
    """The bulk-copy pipeline's bounded mbarrier waits: the tensor-core Q6_K
    chunk GEMM runs with one stage never copied, gives up after its (20 ms)
    bound and reports DET_ERR_TIMEOUT without hanging; the complete launch
    after it, and a K-quant forward through the model, still work."""
    import time

    t = time.time()
    code = D.lib().det_q6k_pipeline_timeout_selftest(0)
    assert code == 67, D.lib().det_status_string(code)  # DET_ERR_TIMEOUT
    assert time.time() - t < 20
    spec = SPECS["q4k_q6k"]
    toks = S.zipf_tokens(24, spec.vocab, seed=2)
    assert D.Model(S.build_gguf(spec)).logits_for_tokens(toks, chunk=24).shape == (24, spec.vocab)
