"""det_symbol_ranges_noalloc against det_symbol_ranges.

The no-allocation entry point serves callers that cannot allocate device
memory inside a call (engines whose memory budget is fixed at start-up,
runtimes whose allocator is not cudaMalloc): they hand it device buffers and
it works in a fixed device array.  Its results are integers, so they must
equal the session entry point's exactly, call after call, although every
call reuses the same array.  This file is collected last so that a stop at the first failure has
already run every other test.
"""
import numpy as np
import pytest

from detllm_b200 import synth as S

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT = 69
MAX_ROWS = 1024
MAX_FLOATS = 1 << 21


@pytest.fixture(scope="module")
def env():
    import torch

    import detllm_b200 as D

    assert D.device_count() > 0 and torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.set_device(0)
    return D, torch


def noalloc(env, logits, symbols, byte_escapes):
    """Run the entry point on device copies of `logits` / `symbols`; returns
    (status, n x 3 array of cum, freq, total, reserved words)."""
    D, torch = env
    n, vocab = logits.shape
    d_logits = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).cuda()
    d_syms = torch.from_numpy(np.ascontiguousarray(symbols, np.uint32).view(np.int32)).cuda()
    d_out = torch.full((n, 3), -1, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    st = D.lib().det_symbol_ranges_noalloc(d_logits.data_ptr(), n, vocab, d_syms.data_ptr(), int(byte_escapes),
                                           d_out.data_ptr(), stream)
    raw = d_out.cpu().numpy().view(np.uint64)
    ranges = np.stack([raw[:, 0], raw[:, 1] & 0xFFFFFFFF, raw[:, 2]], axis=1)
    return st, ranges, raw[:, 1] >> 32


def session_ranges(sess, rows, symbols, byte_escapes):
    return sess.symbol_ranges(symbols, rows, byte_escapes=byte_escapes)


def test_noalloc_matches_session_entry_point_twice(env):
    D, _ = env
    spec = S.ModelSpec(n_layer=2, d=256, d_ff=512, n_head=4, n_head_kv=2, vocab=1024, ctx=64, seed=11)
    m = D.Model(S.build_gguf(spec))
    toks = S.zipf_tokens(24, spec.vocab, seed=4)
    rng = np.random.default_rng(7)
    with m.session(n_ctx=32, max_chunk=24) as s:
        logits = s.forward(toks, 0, want_logits=True)
        # call 1: every row, byte escapes on, symbols across the whole alphabet
        syms1 = rng.integers(0, spec.vocab + 256, 24).astype(np.uint32)
        syms1[:4] = [0, spec.vocab - 1, spec.vocab, spec.vocab + 255]
        st, got1, res1 = noalloc(env, logits, syms1, True)
        assert st == 0, D.lib().det_status_string(st)
        assert (got1 == session_ranges(s, np.arange(24), syms1, True)).all()
        assert (res1 == 0).all()
        # call 2 right after, on fewer rows in another order and without
        # escapes: nothing of call 1 may leak through the shared array
        rows2 = np.array([17, 3, 3, 0, 23, 9, 12], np.uint32)
        syms2 = rng.integers(0, spec.vocab, rows2.size).astype(np.uint32)
        st, got2, _ = noalloc(env, logits[rows2], syms2, False)
        assert st == 0, D.lib().det_status_string(st)
        assert (got2 == session_ranges(s, rows2, syms2, False)).all()


def test_noalloc_errors_and_recovery(env, oracle):
    D, _ = env
    rng = np.random.default_rng(3)
    vocab = 32000
    n = MAX_FLOATS // vocab  # the largest row count that fits the array
    logits = rng.normal(0.0, 3.0, (n, vocab)).astype(np.float32)
    syms = rng.integers(0, vocab + 256, n).astype(np.uint32)
    st, got, _ = noalloc(env, logits, syms, True)
    assert st == 0
    for i in range(0, n, 13):
        assert tuple(int(v) for v in got[i]) == oracle.symbol_range(logits[i], int(syms[i]), True)
    # the reference's own errors come back through the device error word ...
    st, _, _ = noalloc(env, logits[:3], np.array([1, vocab, 2], np.uint32), False)
    assert st == 35  # CdfError::SymbolOutOfRange
    bad = logits[:2].copy()
    bad[1, 77] = np.inf
    st, _, _ = noalloc(env, bad, np.array([1, 2], np.uint32), True)
    assert st == 34  # CdfError::NonFiniteLogit
    # ... and the next call starts clean
    st, again, _ = noalloc(env, logits[:5], syms[:5], True)
    assert st == 0 and (again == got[:5]).all()
    # requests beyond the fixed array are refused before any launch
    lib = D.lib()
    assert lib.det_symbol_ranges_noalloc(8, MAX_ROWS + 1, 16, 8, 1, 8, None) == SCRATCH_LIMIT
    assert lib.det_symbol_ranges_noalloc(8, n + 1, vocab, 8, 1, 8, None) == SCRATCH_LIMIT
