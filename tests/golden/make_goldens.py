"""Regenerate tests/golden/reference_goldens.json from the reference repository.

Run in the authoring container only (the reference tree is not present on the
GPU box):  python tests/golden/make_goldens.py /path/to/reference

Every value is read as text from the reference's own files: its committed
fixture hashes, its canary constants, the quant-kernel hash and codec sizes
recorded in its validation log, and the SHA-256 of its fixture GGUF files.
The GGUF files themselves are not copied; the oracle regenerates them and the
tests compare SHA-256 digests.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import sys


def _hex_array(text: str, name: str) -> str:
    m = re.search(name + r"[^=]*=\s*\[(.*?)\];", text, re.S)
    if not m:
        raise SystemExit(f"constant {name} not found")
    return "".join(f"{int(v, 16):02x}" for v in re.findall(r"0x([0-9a-fA-F]{2})", m.group(1)))


def main(ref: str) -> None:
    out = {}
    td = os.path.join(ref, "testdata")
    out["tiny_f32_logits_sha256"] = open(os.path.join(td, "tiny-f32.logits.sha256")).read().strip()
    out["tiny_qmix_logits_sha256"] = open(os.path.join(td, "tiny-qmix.logits.sha256")).read().strip()
    out["tokens"] = [int(t) for t in open(os.path.join(td, "tiny.tokens.txt")).read().strip().split(",")]
    out["tiny_tokens_txt"] = open(os.path.join(td, "tiny.tokens.txt"), "rb").read().decode()
    for name in ("tiny-f32", "tiny-qmix"):
        data = open(os.path.join(td, f"{name}.gguf"), "rb").read()
        out[f"{name.replace('-', '_')}_gguf_sha256"] = hashlib.sha256(data).hexdigest()
        out[f"{name.replace('-', '_')}_gguf_len"] = len(data)
    canary = open(os.path.join(ref, "crates/det-num/src/canary.rs")).read()
    out["num_canary_sha256"] = _hex_array(canary, "EXPECTED")
    cli = open(os.path.join(ref, "crates/det-cli/src/main.rs")).read()
    out["runtime_canary_sha256"] = _hex_array(cli, "RUNTIME_CANARY_EXPECTED")
    val = open(os.path.join(ref, "docs/validation.md")).read()
    m = re.search(r"## Quant Kernel Canary.*?```text\s*([0-9a-f]{64})", val, re.S)
    out["quant_kernel_hash"] = m.group(1)
    # Compression smoke (docs/validation.md "Compression Smoke"): 39 input bytes -> 102 DTLZ bytes
    m = re.search(r"\|\s*39\s*\|\s*102\s*\|", val)
    out["smoke_input"] = "detllm deterministic compression smoke\n"
    out["smoke_dtlz_len"] = 102 if m else None
    # token-text fixture row: 12 input bytes -> 19 payload bytes, 75 DTLZ bytes (both fixtures)
    rows = re.findall(r"\| `testdata/(tiny-[a-z0-9]+)\.gguf` \| `[0-9a-f]{64}` \| `[0-9a-f]{64}` \| (\d+) \| (\d+) \| (\d+) \| (\d+) \|", val)
    out["tokens_txt_codec"] = {r[0]: {"input": int(r[1]), "tokens": int(r[2]), "payload": int(r[3]), "dtlz": int(r[4])}
                               for r in rows}
    # expf anchors (det-num/src/math.rs:40-47)
    math_rs = open(os.path.join(ref, "crates/det-num/src/math.rs")).read()
    anchors = re.findall(r"exp_f32\((-?[0-9.]+)\)\.to_bits\(\), (0x[0-9a-f_]+)\)", math_rs)
    out["expf_anchors"] = {a: int(b.replace("_", ""), 16) for a, b in anchors}
    f64 = re.findall(r"(exp_f64|ln_f64)\(([0-9_.]+)\)\.to_bits\(\), (0x[0-9a-f_]+)\)", math_rs)
    out["f64_anchors"] = [[fn, float(x.replace("_", "")), int(b.replace("_", ""), 16)] for fn, x, b in f64]
    json.dump(out, open(os.path.join(os.path.dirname(__file__), "reference_goldens.json"), "w"), indent=1)
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_goldens.py <path of the detllm reference checkout>")
    main(sys.argv[1])
