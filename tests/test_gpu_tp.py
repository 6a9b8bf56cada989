"""Row-sharded tensor parallelism (det_model_load_tp) against one device.

The reference splits every GEMV's output rows over threads
(gemv_rows_parallel, crates/det-model/src/lib.rs:291-321) and asserts that
logits hashes do not depend on the thread count (det-model lib.rs:3727-3759).
The same holds for the split over devices: every logit, logits hash and DTLZ
byte of a G-part model must equal the single-device model's, bit for bit.

Parts may share a GPU (a device repeats in the list), so a 1-GPU box runs
the whole tensor-parallel path -- slicing, exchanges, event ordering and the
multi-device graph -- and a box with several GPUs spreads the parts over them.
"""
import numpy as np
import pytest

from detllm_b200 import synth as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def D():
    import detllm_b200

    assert detllm_b200.device_count() > 0, "gpu tests need a CUDA device"
    return detllm_b200


def devices_for(D, parts):
    n = D.device_count()
    return [p % n for p in range(parts)]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# Sizes chosen so slices are real at 2-4 parts: d 512 = 8 row tiles of 64,
# d_ff 1024, a vocab that is not a multiple of 64 (ragged last slice), and
# 4 KV heads (heads sharded at 2 and 4 parts, replicated at 3).
SPECS = {
    "q8_0": S.ModelSpec(n_layer=2, d=512, d_ff=1024, n_head=8, n_head_kv=4, vocab=1000, ctx=64, seed=31),
    "q4k_q6k": S.ModelSpec(n_layer=2, d=512, d_ff=1024, n_head=8, n_head_kv=4, vocab=1000, ctx=64,
                           t_embd=S.GT_Q4_K, t_attn=S.GT_Q4_K, t_gate_up=S.GT_Q4_K, t_down=S.GT_Q6_K,
                           t_out=S.GT_Q6_K, seed=32),
    "qwen2_bias_tied_q4_0": S.ModelSpec(arch="qwen2", n_layer=2, d=256, d_ff=512, n_head=4, n_head_kv=2,
                                        vocab=700, ctx=64, tied=True, qkv_bias=True, rope_base=1e6,
                                        t_attn=S.GT_Q4_0, seed=33),
    "f16_f32": S.ModelSpec(n_layer=1, d=256, d_ff=384, n_head=4, n_head_kv=2, vocab=300, ctx=64,
                           t_embd=S.GT_F16, t_attn=S.GT_F32, t_gate_up=S.GT_F16, t_down=S.GT_Q8_0,
                           t_out=S.GT_F32, seed=34),
}


@pytest.fixture(scope="module")
def cases(D):
    out = {}
    for k, spec in SPECS.items():
        g = S.build_gguf(spec)
        toks = S.zipf_tokens(40, spec.vocab, seed=len(k) + 3)
        out[k] = (g, toks, {c: D.Model(g).logits_for_tokens(toks, chunk=c) for c in (1, 7, 24)})
    return out


@pytest.mark.parametrize("name", list(SPECS))
@pytest.mark.parametrize("parts", [2, 3, 4])
def test_tp_logits_equal_single_device(D, cases, name, parts):
    g, toks, want = cases[name]
    m = D.Model(g, devices=devices_for(D, parts))
    for chunk in (1, 7, 24):  # decode GEMV, decode (T <= 8) and chunk GEMM kernels
        got = m.logits_for_tokens(toks, chunk=chunk)
        diff = np.nonzero(bits(got) != bits(want[chunk]))
        assert diff[0].size == 0, f"chunk {chunk}: {diff[0].size} logits differ, first at {diff[0][0]},{diff[1][0]}"


def test_tp_logits_match_oracle(D, oracle, cases):
    g, toks, _ = cases["q8_0"]
    want = oracle.Model(g).logits(toks)
    got = D.Model(g, devices=devices_for(D, 2)).logits_for_tokens(toks, chunk=7)
    assert np.array_equal(bits(got), bits(want))


def test_tp_eager_equals_graph(D, cases):
    # profiling turns the CUDA graphs off: the eagerly enqueued multi-part
    # forward must give the same logits
    g, toks, want = cases["q4k_q6k"]
    m = D.Model(g, devices=devices_for(D, 2))
    D.set_profiling(True)
    try:
        got = m.logits_for_tokens(toks, chunk=24)
    finally:
        D.set_profiling(False)
    assert np.array_equal(bits(got), bits(want[24]))


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-qmix"])
def test_tp_fixture_logits_hash(D, goldens, fixtures, name):
    # testdata/*.logits.sha256 at 2 and 3 parts, chunk sizes of the reference test
    for parts in (2, 3):
        m = D.Model(fixtures[name], devices=devices_for(D, parts))
        for chunk in (1, 2, 3, 6):
            h = m.logits_hash_for_tokens_chunked(goldens["tokens"], chunk)
            assert h.hex() == goldens[name.replace("-", "_") + "_logits_sha256"], (parts, chunk)


def test_tp_codec_bytes_with_window_rollover(D, cases):
    spec = S.ModelSpec(n_layer=2, d=512, d_ff=1024, n_head=8, n_head_kv=4, vocab=600, ctx=64, seed=35)
    g = S.build_gguf(spec)
    data = S.markov_text(300, seed=5)
    one = D.compress(D.Model(g), data, 64)
    m = D.Model(g, devices=devices_for(D, 2))
    assert D.compress(m, data, 64) == one
    assert D.decompress(m, one) == data


def test_tp_session_reset_and_reuse(D, cases):
    g, toks, want = cases["q8_0"]
    m = D.Model(g, devices=devices_for(D, 4))
    with m.session(n_ctx=64, max_chunk=8) as s:
        for _ in range(2):
            s.reset()
            got = np.concatenate([s.forward(toks[p:p + 8], p, want_logits=True) for p in range(0, 40, 8)])
            assert np.array_equal(bits(got), bits(want[7][:40]))


def test_tp_rejects_bad_devices(D):
    spec = SPECS["q8_0"]
    g = S.build_gguf(spec)
    with pytest.raises(D.DetError):
        D.Model(g, devices=[])
    with pytest.raises(D.DetError):
        D.Model(g, devices=[0, D.device_count()])
    with pytest.raises(D.DetError):
        D.Model(g, devices=[0] * 9)


def test_tp_exchange_wait_times_out(D):
    # the exchange kernel waits for a peer counter that nothing sets: after
    # its 2 s bound it reports a timeout instead of hanging, and the device
    # keeps working
    import time

    t = time.time()
    code = D.lib().det_tp_exchange_timeout_selftest(0)
    assert code == 67, D.lib().det_status_string(code)  # DET_ERR_TIMEOUT
    assert 1.5 < time.time() - t < 30
    spec = SPECS["q8_0"]
    g = S.build_gguf(spec)
    toks = S.zipf_tokens(8, spec.vocab, seed=1)
    assert D.Model(g).logits_for_tokens(toks, chunk=8).shape == (8, spec.vocab)
