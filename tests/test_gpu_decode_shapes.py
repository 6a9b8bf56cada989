"""GPU parity of the short-forward kernels at the benchmark's real widths.

Decompress runs one position per forward, and the session runs forwards of
2..16 positions through their own kernels (no chunk GEMM).  At the
BASELINE configurations' widths these are:

* config 5 (Llama-3-8B shape, Q4_K / Q6_K): the split Q4_K GEMV (q|k|v with
  6,144 rows, o with 4,096), the one-lane-per-row Q4_K GEMV (gate|up, 28,672
  rows), the MMA Q6_K GEMV (down at K 14,336, the 128,256-row lm_head), the
  one-position attention at head_dim 128, and the generic K-quant kernel for
  2..16 positions;
* config 4 (Qwen2.5-0.5B shape, Q8_0): the decode GEMV (T <= 8) and the
  small GEMM (9..16 positions) with QKV bias and the tied 151,936-row
  lm_head, and the on-device decoder search over 152,192 symbols.

The layer count is cut to one so that the CPU oracle stays cheap.  Logits
are compared bit for bit, and compress / decompress runs across window
rollovers (n_ctx 64) with the DTLZ bytes equal to the oracle's.
"""
import dataclasses

import numpy as np
import pytest

from detllm_b200 import synth as S

pytestmark = pytest.mark.gpu

N_CTX = 64  # window of the round trips: 160 bytes roll it over twice


@pytest.fixture(scope="module")
def D():
    import detllm_b200

    assert detllm_b200.device_count() > 0, "gpu tests need a CUDA device"
    return detllm_b200


@pytest.fixture(scope="module", params=["llama3-8b-q4_k", "qwen2.5-0.5b-q8_0"])
def config(request):
    spec = dataclasses.replace(S.CONFIGS[request.param], n_layer=1)
    return spec, S.build_gguf(spec)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_short_forwards_logits_bit_exact(D, oracle, config):
    """Positions 0..23 one at a time, then forwards of 5 and 11 positions."""
    spec, g = config
    toks = S.zipf_tokens(40, spec.vocab, seed=61)
    want = oracle.Model(g).logits(toks)
    m = D.Model(g)
    with m.session(n_ctx=spec.ctx, max_chunk=16) as s:
        spans = [(p, 1) for p in range(24)] + [(24, 5), (29, 11)]
        for p0, n in spans:
            lg = s.forward(toks[p0:p0 + n], p0, want_logits=True)
            diff = np.nonzero(bits(lg) != bits(want[p0:p0 + n]))
            assert diff[0].size == 0, (f"{diff[0].size} logits differ in the {n}-position forward at {p0}, "
                                       f"first at position {p0 + diff[0][0]}, column {diff[1][0]}")
    m.close()


def test_round_trip_across_rollovers(D, oracle, config):
    """Compress equals the oracle's bytes; decompress (the one-position
    forward, CDF and range decoder on the device) restores the input."""
    spec, g = config
    data = S.markov_text(160, seed=67)
    m = D.Model(g)
    got = D.compress(m, data, N_CTX)
    assert got == oracle.compress(g, data, N_CTX)
    assert D.decompress(m, got) == data
    m.close()
