"""Determinism policy of the sources, checked on the CPU.

The reference keeps its numerics reproducible with a source scan
(`xtask check-determinism`, xtask/src/main.rs:522-660): no platform
transcendentals, no fused multiply-add, no fast-math.  This is the same
policy for CUDA and C sources:

* no call to a platform or CUDA transcendental or approximate intrinsic
  (expf, __expf, __fdividef, rsqrtf, ...) and no approximate or
  flush-to-zero PTX instruction; exp, log, sin and cos come from the
  restated fdlibm routines, and sqrt / division are the IEEE operations;
* every fused multiply-add is one the reference's two roundings cannot
  tell apart (an add written as p * 1 + acc, or a product that is exact),
  and says so in a comment on its line or just above it;
* the builds keep FMA contraction, fast-math and flush-to-zero off.
"""
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PRODUCT = sorted(glob.glob(os.path.join(ROOT, "detllm_b200", "csrc", "*.cu")) +
                 glob.glob(os.path.join(ROOT, "detllm_b200", "csrc", "*.cuh")) +
                 glob.glob(os.path.join(ROOT, "detllm_b200", "csrc", "*.cpp")) +
                 glob.glob(os.path.join(ROOT, "detllm_b200", "csrc", "*.h")))
ORACLE = sorted(glob.glob(os.path.join(ROOT, "oracle", "*.c")) + glob.glob(os.path.join(ROOT, "oracle", "*.h")))

BANNED_CALLS = re.compile(
    r"(?<![\w.])(?:std::)?("
    r"expf|exp|exp2f|exp2|expm1f|expm1|exp10f|logf|log|log2f|log2|log10f|log10|log1pf|log1p|"
    r"sinf|sin|cosf|cos|tanf|tan|sincosf|sincos|powf|pow|tanhf|tanh|erff|erf|"
    r"__expf|__exp10f|__logf|__log2f|__log10f|__sinf|__cosf|__tanf|__sincosf|__powf|__fdividef|"
    r"rsqrtf|rsqrt|__frsqrt_rn|rcbrtf|__frcp_rn|__frcp_rz|__saturatef|fmaf|fma|__fmul_rz)\s*\(")
BANNED_PTX = re.compile(r"\.approx|\.ftz|\b(?:ex2|lg2|sin|cos|rcp|rsqrt|tanh)\.")
FMA_SITE = re.compile(r"fma\.rn|__fmaf_r[nzdu]\s*\(|(?<![\w.])fma2\s*\(")
FMA_HELPER = re.compile(r"^\s*(?:DI|__device__|static)?\s*[\w ]*\bfma2\s*\(\s*(?:float2|unsigned long long)\s+\w+")


def code_lines(path):
    """(line number, code without // comments, full line) of a source file;
    block comments and string-free lines are kept as they are (inline PTX
    lives in strings and is checked on purpose)."""
    out = []
    in_block = False
    for i, line in enumerate(open(path, encoding="utf-8").read().split("\n"), 1):
        code = line
        if in_block:
            if "*/" not in code:
                continue
            code = code.split("*/", 1)[1]
            in_block = False
        while "/*" in code:
            head, rest = code.split("/*", 1)
            if "*/" in rest:
                code = head + rest.split("*/", 1)[1]
            else:
                code, in_block = head, True
                break
        out.append((i, code.split("//", 1)[0], line))
    return out


def test_no_platform_transcendentals_or_approximations():
    bad = []
    for path in PRODUCT + ORACLE:
        for i, code, _ in code_lines(path):
            m = BANNED_CALLS.search(code)
            if m:
                bad.append(f"{os.path.relpath(path, ROOT)}:{i}: {m.group(1)}(")
            if path in PRODUCT and "asm" in code and BANNED_PTX.search(code):
                bad.append(f"{os.path.relpath(path, ROOT)}:{i}: approximate PTX")
    assert not bad, "\n".join(bad)


def test_every_fused_multiply_add_is_exact_and_says_why():
    sites, bad = 0, []
    for path in PRODUCT:
        lines = code_lines(path)
        raw = open(path, encoding="utf-8").read().split("\n")
        for k, (i, code, _) in enumerate(lines):
            if not FMA_SITE.search(code):
                continue
            # the generic packed helpers themselves: callers carry the note
            if FMA_HELPER.search(code) or any(FMA_HELPER.search(c) for _, c, _ in lines[max(0, k - 2):k]):
                continue
            sites += 1
            note = " ".join(raw[max(0, i - 9):i]).lower()
            if "exact" not in note:
                bad.append(f"{os.path.relpath(path, ROOT)}:{i}: {raw[i - 1].strip()}")
    assert sites >= 5, sites  # the exact adds and the Q4_K dequantisation
    assert not bad, "fused multiply-adds without an exactness note:\n" + "\n".join(bad)


def test_builds_keep_contraction_fast_math_and_ftz_off():
    mk = open(os.path.join(ROOT, "detllm_b200", "csrc", "Makefile")).read()
    nv = re.search(r"^NVFLAGS\s*:=(.*?)(?:\n\S|\Z)", mk, re.S | re.M).group(1)
    cxx = re.search(r"^CXXFLAGS\s*:=(.*?)(?:\n\S|\Z)", mk, re.S | re.M).group(1)
    for flag in ("--fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false", "-ffp-contract=off"):
        assert flag in nv, flag
    assert "-ffp-contract=off" in cxx and "-fno-fast-math" in cxx
    assert "use_fast_math" not in mk and "-ffast-math" not in mk and "-Ofast" not in mk
    om = open(os.path.join(ROOT, "oracle", "Makefile")).read()
    assert "-ffp-contract=off" in om and "-fno-fast-math" in om
    assert "-ffast-math" not in om and "-Ofast" not in om
