"""Pins the CPU oracle to the reference's own golden vectors and unit KATs.

Every expected value here comes from the reference repository (its committed
fixture hashes, canary constants, validation log and unit tests); see
tests/golden/make_goldens.py.  The oracle is test infrastructure: once it
matches these, it is the checker the GPU parity tests compare against.
"""
import struct

import numpy as np
import pytest


def f32(bits):
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def bits(x):
    return struct.unpack("<I", struct.pack("<f", np.float32(x)))[0]


def abits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_num_canary(oracle, goldens):
    # crates/det-num/src/canary.rs:3-6
    assert oracle.canary_hash().hex() == goldens["num_canary_sha256"]


def test_runtime_canary(oracle, goldens):
    # crates/det-cli/src/main.rs:5-8, 146-224
    assert oracle.runtime_canary_hash().hex() == goldens["runtime_canary_sha256"]


def test_quant_kernel_hash(oracle, goldens):
    # docs/validation.md:345; generator crates/det-cli/src/main.rs:233-388
    assert oracle.quant_kernel_hash().hex() == goldens["quant_kernel_hash"]


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-qmix"])
def test_fixture_gguf_bytes(oracle, goldens, fixtures, name):
    # xtask generate-testdata --check (xtask/src/main.rs:934-973)
    data = fixtures[name]
    key = name.replace("-", "_")
    assert len(data) == goldens[f"{key}_gguf_len"]
    assert oracle.sha256(data).hex() == goldens[f"{key}_gguf_sha256"]


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-qmix"])
@pytest.mark.parametrize("chunk", [1, 2, 3, 6])
def test_fixture_logits_hash(oracle, goldens, fixtures, name, chunk):
    # testdata/*.logits.sha256; chunk invariance det-model lib.rs:3727-3759
    m = oracle.Model(fixtures[name])
    assert m.logits_hash(goldens["tokens"], chunk).hex() == goldens[name.replace("-", "_") + "_logits_sha256"]


@pytest.mark.parametrize("threads", [1, 2, 7, 16])
def test_fixture_hash_thread_invariance(oracle, goldens, fixtures, threads):
    # det-model lib.rs:3727-3759 (threads {1,2,7,16})
    oracle.set_threads(threads)
    try:
        m = oracle.Model(fixtures["tiny-qmix"])
        assert m.logits_hash(goldens["tokens"], 3).hex() == goldens["tiny_qmix_logits_sha256"]
    finally:
        oracle.set_threads(0)


def test_sha256_abc(oracle):
    # crates/det-num/src/hash.rs:149-160
    assert oracle.sha256(b"abc").hex() == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"


def test_expf_anchors(oracle, goldens):
    # crates/det-num/src/math.rs:40-47
    for x, want in goldens["expf_anchors"].items():
        assert bits(oracle.lib().ref_expf(float(x))) == want
    assert bits(oracle.lib().ref_expf(0.0)) == bits(1.0)


def test_f64_anchors(oracle, goldens):
    # crates/det-num/src/math.rs:50-62
    L = oracle.lib()
    for fn, x, want in goldens["f64_anchors"]:
        got = L.ref_exp_f64(x) if fn == "exp_f64" else L.ref_ln_f64(x)
        assert struct.unpack("<Q", struct.pack("<d", got))[0] == want
    assert L.ref_sin_f64(0.0) == 0.0 and L.ref_cos_f64(0.0) == 1.0
    assert L.ref_sin_f64(np.pi / 2) == 1.0
    assert struct.unpack("<Q", struct.pack("<d", L.ref_cos_f64(np.pi / 2)))[0] == 0x3C91A62633145C07
    # vendored_libm/sin.rs test_near_pi
    x = struct.unpack("<d", struct.pack("<Q", 0x400921FB000FD5DD))[0]
    assert struct.unpack("<Q", struct.pack("<d", L.ref_sin_f64(x)))[0] == 0x3EA50D15CED1A4A2


def test_round_and_f16(oracle):
    # det-num round.rs:45-57, f16.rs:40-49
    L = oracle.lib()
    assert [L.ref_round_ties_even_i32(v) for v in (0.5, 1.5, 2.5, -0.5, -1.5, -2.5)] == [0, 2, 2, 0, -2, -2]
    assert bits(L.ref_f16_to_f32(0x0000)) == 0 and bits(L.ref_f16_to_f32(0x8000)) == 0x80000000
    assert L.ref_f16_to_f32(0x3C00) == 1.0 and L.ref_f16_to_f32(0xC000) == -2.0
    assert L.ref_f16_to_f32(0x7BFF) == 65504.0


def test_dot_lane_order(oracle):
    # det-num reduce.rs:44-61
    x = np.array([1, 2, -3, 4, 5.5, -6.25, 7, 8, -9, 10, 11, -12, 13, 14, -15, 16, 17], np.float32)
    y = np.array([0.5, -1, 2, 3, -4, 5, 6, -7, 8, 9, -10, 11, 12, -13, 14, 15, -16], np.float32)
    acc = np.zeros(8, np.float32)
    for i in range(17):
        acc[i % 8] = np.float32(acc[i % 8] + np.float32(x[i] * y[i]))
    want = np.float32(np.float32(np.float32(acc[0] + acc[1]) + np.float32(acc[2] + acc[3])) +
                      np.float32(np.float32(acc[4] + acc[5]) + np.float32(acc[6] + acc[7])))
    got = oracle.lib().ref_dot_f32(x.ctypes.data, y.ctypes.data, 17)
    assert bits(got) == bits(want)


def test_rmsnorm_runs_in_specified_order(oracle):
    # det-model lib.rs:2443-2459: ss by the 8-lane sum of squares, then
    # r = 1 / sqrt(ss / n + eps), out = (x * r) * w, each op rounded to f32
    f = np.float32
    x = np.array([1.0, -2.0, 3.0, -4.0], f)
    w = np.array([0.5, 1.0, 1.5, 2.0], f)
    out = oracle.rmsnorm(x, w, 1e-5)
    sq = x * x
    ss = f(f(sq[0] + sq[1]) + f(sq[2] + sq[3]))  # lanes 4..7 are zero
    r = f(1.0) / np.sqrt(f(f(ss / f(4.0)) + f(1e-5)))
    assert (abits(out) == abits((x * r).astype(f) * w)).all()


def test_softmax_uses_det_exp_and_8lane_sum(oracle):
    # det-model lib.rs:2462-2469
    x = oracle.softmax([1.0, 0.0, -2.0, 3.0, -88.0, 3.0, -1.0, 2.0, 0.5])
    z = np.float32(0.0)
    lanes = [np.float32(0.0)] * 8
    for i, v in enumerate(x):
        lanes[i % 8] = np.float32(lanes[i % 8] + v)
    z = np.float32(np.float32(np.float32(lanes[0] + lanes[1]) + np.float32(lanes[2] + lanes[3])) +
                   np.float32(np.float32(lanes[4] + lanes[5]) + np.float32(lanes[6] + lanes[7])))
    assert abs(float(z) - 1.0) < 1e-6
    assert bits(x[3]) == bits(x[5])


def test_rope_pairs_in_specified_order(oracle):
    # det-model lib.rs:2752-2821: position 1 of a 2-position table with
    # cos (0, 0.5) and sin (1, -0.25)
    c, s = [0.0, 0.5], [1.0, -0.25]
    adj = oracle.rope_rotate([1, 2, 3, 4, 5, 6, 7, 8], 2, 4, c, s, split_half=False)
    assert (abits(adj) == abits(np.array([-2.0, 1.0, 2.5, 1.25, -6.0, 5.0, 5.5, 2.25], np.float32))).all()
    split = oracle.rope_rotate([1, 2, 3, 4], 1, 4, c, s, split_half=True)
    assert (abits(split) == abits(np.array([-3.0, 2.0, 1.0, 1.5], np.float32))).all()
    # a head longer than the rotary pairs keeps its tail
    tail = oracle.rope_rotate([1, 2, 3, 4, 9, -9], 1, 6, c, s, split_half=False)
    assert (abits(tail) == abits(np.array([-2.0, 1.0, 2.5, 1.25, 9.0, -9.0], np.float32))).all()
    tail = oracle.rope_rotate([1, 2, 3, 4, 9, -9], 1, 6, c, s, split_half=True)
    assert (abits(tail) == abits(np.array([-3.0, 2.0, 1.0, 1.5, 9.0, -9.0], np.float32))).all()


def test_q8a_quantize_kat(oracle):
    # det-quant lib.rs:826-842
    d, q = oracle.quantize_q8a(np.zeros(32, np.float32))
    assert bits(d[0]) == 0 and not q.any()
    x = np.zeros(32, np.float32)
    x[0], x[1], x[2], x[3] = 1.0, -1.0, np.float32(0.5) / np.float32(127.0), -np.float32(0.5) / np.float32(127.0)
    d, q = oracle.quantize_q8a(x)
    assert list(q[:4]) == [127, -127, 1, -1]
    with pytest.raises(oracle.OracleError):
        x[3] = np.nan
        oracle.quantize_q8a(x)


def test_q8k_quantize_kat(oracle):
    # det-quant lib.rs:1159-1166
    x = np.zeros(256, np.float32)
    x[0], x[1] = 2.0, -1.0
    d, q, bs = oracle.quantize_q8k(x)
    assert np.signbit(d[0]) and q[0] == -127 and bs[0] == q[:16].astype(np.int16).sum()


def test_cdf_kats(oracle):
    # det-coder cdf.rs:433-470
    f, c, t = oracle.logits_to_cdf(np.array([0.0, 0.0, 0.0, 0.0], np.float32))
    ef = int(np.float32(16777216.0) / np.float32(4)) + 1
    assert list(f) == [ef] * 4 and t == 16777216 + 4
    a = oracle.logits_to_cdf(np.array([0.0, -88.0, -88.0, -0.5], np.float32))
    b = oracle.logits_to_cdf(np.array([0.0, -1000.0, -1.0e30, -0.5], np.float32))
    assert all((x == y).all() if hasattr(x, "all") else x == y for x, y in zip(a, b))
    logits = np.array([1.0, 0.25, -2.0, 3.5], np.float32)
    f, c, t = oracle.logits_to_cdf(logits)
    for s in range(4):
        cum, fr, tot = oracle.symbol_range(logits, s, byte_escapes=True)
        assert (cum, fr, tot) == (c[s], f[s], t + 256)
        for v in (c[s], c[s] + f[s] - 1):
            assert oracle.decoder_lookup(logits, int(v), True) == (s, c[s], f[s], t + 256)
    for s in range(4, 260):
        assert oracle.symbol_range(logits, s, True) == (t + s - 4, 1, t + 256)
    with pytest.raises(oracle.OracleError) as e:
        oracle.symbol_range(np.array([0.0, 1.0], np.float32), 2, byte_escapes=False)
    assert e.value.code == 35


def test_cdf_large_vocab_scalar_reference(oracle):
    # det-coder cdf.rs:568-620 (10,003 LCG logits) against a numpy restatement
    state = 0x123456789ABCDEF0
    vals = []
    for _ in range(10003):
        state = (state * 6364136223846793005 + 1442695040888963407) & (2**64 - 1)
        unit = np.float32(state >> 40) / np.float32(1 << 24)
        vals.append(np.float32(np.float32(unit * np.float32(40.0)) - np.float32(20.0)))
    logits = np.array(vals, np.float32)
    f, c, t = oracle.logits_to_cdf(logits)
    e = oracle.expf(np.maximum(logits - logits.max(), np.float32(-88.0)))
    acc = np.zeros(8, np.float32)
    for i in range(0, len(e) - len(e) % 8, 8):
        acc = (acc + e[i:i + 8]).astype(np.float32)
    for i in range(len(e) - len(e) % 8, len(e)):
        acc[i % 8] = np.float32(acc[i % 8] + e[i])
    z = np.float32(np.float32(np.float32(acc[0] + acc[1]) + np.float32(acc[2] + acc[3])) +
                   np.float32(np.float32(acc[4] + acc[5]) + np.float32(acc[6] + acc[7])))
    want = ((e / z).astype(np.float32) * np.float32(16777216.0)).astype(np.float32).astype(np.uint32) + 1
    assert (f == want).all() and t == int(want.astype(np.uint64).sum())


def test_codec_golden_sizes(oracle, goldens, fixtures):
    # docs/validation.md:1261-1267 and :488-510
    tok = goldens["tiny_tokens_txt"].encode()
    for name, row in goldens["tokens_txt_codec"].items():
        d = oracle.compress(fixtures[name], tok, 8)
        assert len(d) == row["dtlz"] and len(d) - 56 == row["payload"]
        assert oracle.decompress(fixtures[name], d) == tok
    smoke = goldens["smoke_input"].encode()
    d = oracle.compress(fixtures["tiny-f32"], smoke, 8)
    assert len(d) == goldens["smoke_dtlz_len"]


@pytest.mark.parametrize("name", ["tiny-f32", "tiny-qmix"])
def test_codec_round_trips(oracle, fixtures, name):
    # crates/det-cli/tests/testdata_cli.rs:220-310
    cases = [b"", "detllm deterministic 圧縮 smoke\n復元一致\n".encode(), bytes(range(256)) + b"detllm"]
    for data in cases:
        d = oracle.compress(fixtures[name], data, 8)
        assert d[:4] == b"DTLZ" and struct.unpack("<HHII", d[4:8] + d[40:48])[1:] == (1, 8, 2)
        assert struct.unpack("<Q", d[48:56])[0] == len(data)
        assert d[8:40] == oracle.sha256(fixtures[name])
        assert oracle.decompress(fixtures[name], d) == data


def test_window_rolls_over_when_context_reaches_n_ctx(oracle):
    # det-cli main.rs:1289-1304: n_ctx 8, overlap 2
    start, seen = 0, []
    for pos in range(18):
        start = oracle.next_window_start(pos, start, 8, 2)
        seen.append((pos, start, pos - start))
    assert seen[7] == (7, 0, 7)
    assert seen[8] == (8, 6, 2)
    assert seen[13] == (13, 6, 7)
    assert seen[14] == (14, 12, 2)


def test_codec_rejects_invalid_windows(oracle, fixtures):
    # det-cli main.rs:1264-1287: n_ctx 0, overlap == n_ctx, n_ctx above the
    # model's context length all fail with the window error (status 57)
    m = oracle.Model(fixtures["tiny-f32"])
    assert m.encode_symbols([0, 1], 3, 1)
    for n_ctx, overlap in [(0, 0), (3, 3), (m.info.context_length + 1, 0)]:
        with pytest.raises(oracle.OracleError) as e:
            m.encode_symbols([0, 1], n_ctx, overlap)
        assert e.value.code == 57, (n_ctx, overlap)
    m.close()


def test_codec_rejects_noncanonical_and_bad_header(oracle, fixtures):
    # testdata_cli.rs:312-371, file.rs:45-56
    m = fixtures["tiny-f32"]
    d = oracle.compress(m, b"detllm", 8)
    with pytest.raises(oracle.OracleError) as e:
        oracle.decompress(m, d + b"\x00")
    assert e.value.code in (59, 41)
    bad = bytearray(d)
    bad[6] = 2
    with pytest.raises(oracle.OracleError) as e:
        oracle.decompress(m, bytes(bad))
    assert e.value.code == 51
    with pytest.raises(oracle.OracleError) as e:
        oracle.decompress(fixtures["tiny-qmix"], d)
    assert e.value.code == 58


def test_dtlz_header_rejections(oracle, fixtures):
    # det-coder file.rs:111-207 through decompress: each header field is
    # checked before the model hash and the payload
    m = fixtures["tiny-f32"]
    d = oracle.compress(m, b"detllm header", 8)

    def patched(off, fmt, value):
        b = bytearray(d)
        struct.pack_into(fmt, b, off, value)
        return bytes(b)

    cases = [
        (b"", 48), (d[:55], 48),                      # TooShort
        (b"NOPE" + d[4:], 49),                        # BadMagic
        (patched(4, "<H", 2), 50),                    # UnsupportedVersion(VERSION + 1)
        (patched(6, "<H", 1 << 1), 51),               # UnsupportedFlags(FLAG_BYTE_ESCAPES << 1)
        (patched(40, "<I", 0), 52),                   # InvalidContext: n_ctx 0
        (patched(44, "<I", 8), 53),                   # InvalidOverlap: overlap == n_ctx
    ]
    for data, want in cases:
        with pytest.raises(oracle.OracleError) as e:
            oracle.decompress(m, data)
        assert e.value.code == want, (data[:8], want)
    assert oracle.decompress(m, d) == b"detllm header"


def test_range_encoder_rejects_invalid_frequency_ranges(oracle):
    # det-coder range.rs:270-282: cum + freq beyond total (without
    # overflowing), a zero frequency, and a total above 2^31 - 1
    import ctypes as C

    out = np.zeros(64, np.uint8)
    n = C.c_size_t()
    for cum, freq, total in [(2**64 - 1, 1, 8), (0, 0, 8), (8, 1, 8), (0, 1, 1 << 31)]:
        cs, fs, ts = (np.array([v], np.uint64) for v in (cum, freq, total))
        st = oracle.lib().ref_range_encode(cs.ctypes.data, fs.ctypes.data, ts.ctypes.data, 1, out.ctypes.data,
                                           out.size, C.byref(n))
        assert st == 40, (cum, freq, total)
    cs, fs, ts = (np.array([v], np.uint64) for v in (7, 1, 8))
    assert oracle.lib().ref_range_encode(cs.ctypes.data, fs.ctypes.data, ts.ctypes.data, 1, out.ctypes.data,
                                         out.size, C.byref(n)) == 0


def test_range_coder_million_symbols(oracle):
    # det-coder range.rs:327-357 (LCG stream) -- encode through the oracle,
    # decode with a Python restatement of RangeDecoder
    import ctypes as C

    rng = 0xDECAFBAD5EED

    def nxt():
        nonlocal rng
        rng = (rng * 6364136223846793005 + 1442695040888963407) & (2**64 - 1)
        return rng >> 32

    freq = np.array([1 + nxt() % 997 for _ in range(257)], np.uint64)
    cum = np.concatenate([[0], np.cumsum(freq)[:-1]]).astype(np.uint64)
    total = int(cum[-1] + freq[-1])
    syms = np.array([nxt() % 257 for _ in range(100000)], np.int64)
    cs, fs = cum[syms].copy(), freq[syms].copy()
    ts = np.full(len(syms), total, np.uint64)
    cap = len(syms) * 4 + 64
    out = np.zeros(cap, np.uint8)
    n = C.c_size_t()
    assert oracle.lib().ref_range_encode(cs.ctypes.data, fs.ctypes.data, ts.ctypes.data, len(syms),
                                         out.ctypes.data, cap, C.byref(n)) == 0
    data = out[: n.value].tobytes()
    M = 2**64 - 1
    low, code, rng_, pos = 0, 0, M, 0
    for _ in range(8):
        code = (code << 8) | data[pos]
        pos += 1
    for s in syms[:2000]:
        r = rng_ // total
        v = ((code - low) & M) // r
        got = int(np.searchsorted(cum, v, side="right") - 1)
        assert got == s
        low = (low + r * int(cum[got])) & M
        rng_ = r * int(freq[got])
        while True:
            if (low ^ ((low + rng_) & M)) < (1 << 56):
                pass
            elif rng_ < (1 << 48):
                rng_ = ((-low) & M) & ((1 << 48) - 1)
            else:
                break
            code = ((code << 8) | data[pos]) & M
            pos += 1
            low = (low << 8) & M
            rng_ = (rng_ << 8) & M


@pytest.mark.parametrize("threads", [1, 3])
def test_kquant_row_groups_equal_row_by_row(oracle, threads):
    """The oracle's row-group Q4_K / Q6_K GEMV (several rows side by side,
    row-independent values hoisted) gives the same logits bit for bit as the
    one-row functions that restate dot_q4_k_q8a / dot_q6_k_q8k
    (det-quant lib.rs:281-315, :353-397); 1,000 output rows leave a ragged
    last group, d_ff 768 three Q6_K blocks per down row."""
    from detllm_b200 import synth as S

    spec = S.ModelSpec(n_layer=2, d=512, d_ff=768, n_head=8, n_head_kv=2, vocab=1000, ctx=64,
                       t_embd=S.GT_Q4_K, t_attn=S.GT_Q4_K, t_gate_up=S.GT_Q4_K, t_down=S.GT_Q6_K,
                       t_out=S.GT_Q6_K, seed=31)
    g = S.build_gguf(spec)
    toks = S.zipf_tokens(12, spec.vocab, seed=2)
    oracle.set_threads(threads)
    try:
        m = oracle.Model(g)
        fast = m.logits(toks)
        oracle.set_rowwise_gemv(True)
        slow = m.logits(toks)
    finally:
        oracle.set_rowwise_gemv(False)
        oracle.set_threads(0)
    assert (fast.view(np.uint32) == slow.view(np.uint32)).all()
