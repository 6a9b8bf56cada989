"""Model metadata the reference refuses, refused the same way.

`LlamaConfig::from_gguf` / `validate` (crates/det-model/src/lib.rs) reject
GGUF metadata that asks for a decoder feature this forward does not have,
or for values that can make it produce NaN, with a fixed `ModelError`.  The
cases below restate the reference's own tests (det-model :4433-4612,
:4653-4728) on a small synthetic model whose metadata is rewritten:
neutral values load, every other value fails with the reference's error.
The oracle is checked on the CPU; the library (det_model_load through the
C ABI) on a GPU, with the same table.
"""
import math

import numpy as np
import pytest

from detllm_b200 import synth as S

# ModelError order (det-model :48-59)
SHAPE, ARCH, HEAD_LENGTH, FEATURE, ROPE_SCALING, MISSING, GGUF = 1, 3, 4, 5, 6, 7, 8

SPEC = S.ModelSpec(n_layer=1, d=64, d_ff=128, n_head=2, n_head_kv=1, vocab=300, ctx=32, seed=71)
HD = SPEC.d // SPEC.n_head

F32_FEATURE_KEYS = [  # det-model :4577-4589
    "llama.attention.max_alibi_bias", "llama.attention.clamp_kqv", "llama.attention.value_scale",
    "llama.attn_logit_softcapping", "llama.final_logit_softcapping", "llama.logit_scale",
    "llama.embedding_scale", "llama.residual_scale",
]

# (name, metadata entries, expected status: 0 = loads)
CASES = [
    ("neutral features", [("llama.use_parallel_residual", S.GV_BOOL, False),
                          ("llama.attention.causal", S.GV_BOOL, True),
                          ("llama.embedding_length_out", S.GV_U32, SPEC.d),
                          ("llama.attention.sliding_window", S.GV_U32, 0),
                          ("llama.attention.key_length", S.GV_U32, HD),
                          ("llama.attention.value_length", S.GV_U32, HD),
                          ("llama.rope.scaling.type", S.GV_STRING, "none")]
     + [(k, S.GV_F32, -0.0) for k in F32_FEATURE_KEYS], 0),
    ("f64 negative zero", [("llama.attention.max_alibi_bias", S.GV_F64, -0.0)], 0),
    ("key_length", [("llama.attention.key_length", S.GV_U32, 2 * HD)], HEAD_LENGTH),
    ("value_length", [("llama.attention.value_length", S.GV_U32, 2 * HD)], HEAD_LENGTH),
    ("parallel residual", [("llama.use_parallel_residual", S.GV_BOOL, True)], FEATURE),
    ("non-causal", [("llama.attention.causal", S.GV_BOOL, False)], FEATURE),
    ("embedding_length_out", [("llama.embedding_length_out", S.GV_U32, 2 * SPEC.d)], FEATURE),
    ("sliding window", [("llama.attention.sliding_window", S.GV_U32, 128)], FEATURE),
    ("f64 subnormal", [("llama.attention.max_alibi_bias", S.GV_F64, 5e-324)], FEATURE),
    ("linear rope scaling", [("llama.rope.scaling.type", S.GV_STRING, "linear")], ROPE_SCALING),
    ("rms epsilon 0", [("llama.attention.layer_norm_rms_epsilon", S.GV_F32, 0.0)], SHAPE),
    ("rms epsilon -1", [("llama.attention.layer_norm_rms_epsilon", S.GV_F32, -1.0)], SHAPE),
    ("attention scale 0", [("llama.attention.scale", S.GV_F32, 0.0)], SHAPE),
    ("attention scale nan", [("llama.attention.scale", S.GV_F32, math.nan)], SHAPE),
    ("rope base 0", [("llama.rope.freq_base", S.GV_F32, 0.0)], SHAPE),
    ("rope base inf", [("llama.rope.freq_base", S.GV_F32, math.inf)], SHAPE),
    ("rope dims 3", [("llama.rope.dimension_count", S.GV_U32, 3)], SHAPE),
    # metadata of the wrong kind: map_metadata_error and vocab_size (:1668-1692, :2158-2163, :3087-3116)
    ("architecture", [("general.architecture", S.GV_STRING, "gpt2")], ARCH),
    ("head_count as a string", [("llama.attention.head_count", S.GV_STRING, "2")], GGUF),
    ("vocab_size as a string", [("llama.vocab_size", S.GV_STRING, "3")], GGUF),
] + [(k.split(".")[-1], [(k, S.GV_F32, 1.0)], FEATURE) for k in F32_FEATURE_KEYS]

# (name, entries set, keys removed, expected status)
DROPPED = [
    ("no head_count", [], {"llama.attention.head_count"}, MISSING),
    ("no block_count", [], {"llama.block_count"}, MISSING),
    # without a vocab_size key the vocabulary comes from the token list,
    # which must be strings (vocab_size, :1679-1684)
    ("tokens as integers", [("tokenizer.ggml.tokens", S.GV_ARRAY, (S.GV_U32, [0, 1, 2]))],
     {"llama.vocab_size"}, GGUF),
]


@pytest.fixture(scope="module")
def base():
    return S.build_gguf(SPEC)


def variants(base):
    for name, kvs, want in CASES:
        yield name, S.with_metadata(base, kvs), want
    for name, kvs, keys, want in DROPPED:
        yield name, S.with_metadata(base, kvs, drop=lambda k, keys=keys: k in keys), want


def test_oracle_refuses_metadata_like_the_reference(oracle, base):
    for name, g, want in variants(base):
        if want == 0:
            oracle.Model(g).close()
            continue
        with pytest.raises(oracle.OracleError) as e:
            oracle.Model(g)
        assert e.value.code == want, name


def test_oracle_config_defaults_and_attention_scale(oracle):
    # det-model :4377-4430: head_dim = d / heads, attention scale
    # 1 / sqrt(head_dim) (f32 sqrt, then f32 division) unless
    # attention.scale is given, RoPE base 10,000 when the key is absent
    spec = S.ModelSpec(n_layer=1, d=64, d_ff=128, n_head=2, n_head_kv=1, vocab=300, ctx=32, rope_base=5e5, seed=72)
    g = S.build_gguf(spec)
    m = oracle.Model(g)
    assert m.info.head_dim == 32 and m.info.head_count == 2 and m.info.head_count_kv == 1
    assert m.info.block_count == 1 and m.info.embedding_length == 64 and m.info.feed_forward_length == 128
    assert m.info.context_length == 32 and m.vocab == 300
    want = np.float32(1.0) / np.sqrt(np.float32(32.0))
    assert np.float32(m.info.attention_scale).view(np.uint32) == want.view(np.uint32)
    assert m.info.rope_freq_base == 5e5
    base_logits = m.logits([1, 2, 3])
    m.close()
    m = oracle.Model(S.with_metadata(g, [], drop=lambda k: k == "llama.rope.freq_base"))
    assert m.info.rope_freq_base == 10000.0
    m.close()
    m = oracle.Model(S.with_metadata(g, [("llama.attention.scale", S.GV_F32, 0.125)]))
    assert m.info.attention_scale == 0.125
    assert not np.array_equal(m.logits([1, 2, 3]), base_logits)  # the scale reaches the scores
    m.close()


def test_oracle_refuses_token_ids_outside_the_vocabulary(oracle, base):
    # det-model :3153-3175
    m = oracle.Model(base)
    with pytest.raises(oracle.OracleError) as e:
        m.logits_hash([SPEC.vocab], 1)
    assert e.value.code == SHAPE
    with pytest.raises(oracle.OracleError) as e:
        m.logits_hash([0, SPEC.vocab], 1)
    assert e.value.code == SHAPE
    m.close()


@pytest.mark.gpu
def test_library_refuses_metadata_like_the_reference(oracle, base):
    import detllm_b200 as D

    assert D.device_count() > 0, "gpu tests need a CUDA device"
    toks = [1, 2, 3]
    for name, g, want in variants(base):
        if want == 0:
            m = D.Model(g)
            assert m.logits_hash_for_tokens(toks) == oracle.Model(g).logits_hash(toks, 1), name
            m.close()
            continue
        with pytest.raises(D.DetError) as e:
            D.Model(g)
        assert e.value.code == want, name
    # token ids outside the vocabulary (det-model :3153-3175), then the model still works
    m = D.Model(base)
    for bad in ([SPEC.vocab], [0, SPEC.vocab]):
        with pytest.raises(D.DetError) as e:
            m.logits_hash_for_tokens(bad)
        assert e.value.code == SHAPE, bad
    assert m.logits_hash_for_tokens(toks) == oracle.Model(base).logits_hash(toks, 1)
    m.close()
