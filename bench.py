#!/usr/bin/env python3
"""Benchmark: encode tokens/s of the detllm token loop on B200.

Headline workload (the configuration it names for
1/2/4/8 GPUs): a Llama-3-8B-shaped decoder with random-init Q4_K / Q6_K
weights (32 layers, d 4096, 32/8 heads, head_dim 128, FFN 14336, vocab
128256, RoPE theta 5e5), n_ctx 8192, over a seeded 16 MiB order-2 Markov
byte stream cut into 8 independent segments (2 MiB each) that run
segment-parallel: one model replica per GPU, segments dealt round-robin, no
data-path collective.  The byte-fallback tokenizer makes one token per byte.

One step = every rank compresses one segment's first 8,192 bytes (one full
n_ctx window: positions 0..8191, overlap n_ctx / 4) through det_compress:
tokenize -> teacher-forced forward in 1,024-position chunks -> logits ->
CDF ranges -> host range coder -> DTLZ file.  Rank r takes segment
(step * N + r) mod 8, so per-GPU work per step is fixed (weak scaling) and
the 8 segments are covered in turn.

* value: bytes (= tokens) of all ranks / max over ranks of the device time
  of the timed steps (CUDA events on the session stream around the forward
  and CDF kernels).
* e2e: the same tokens / max over ranks of the wall time of the det_compress
  calls, with host bytes in and the DTLZ file out (tokenisation, the token
  upload, the range download and host range coding inside).
* full_stream: the whole 16 MiB stream extrapolated from the measured window
  (every later window forwards the same 8,192 positions: 2,048 replayed,
  6,144 coded), as the reference's bench-file estimate scales a prefix
  (xtask/src/main.rs:2295-2325).
* roofline: the encode step's dominant kernel, the Q4_K chunk GEMM (q|k|v,
  o, gate|up: two thirds of the step), against the FP32 pipe that bounds it
  (the reference's one ordered f32 chain per row: 2 rounded ops per weight
  per position; peak = 148 SMs x 128 lanes x the SM clock measured during
  the timed region, since no FP32 peak is measured by the driver).
* roofline_decode: the headline model's decode weight GEMVs (one token per
  forward), the north-star HBM target: one token's weight GEMV launches back
  to back in a CUDA graph (programmatic dependent launch), algorithmic bytes
  (weights + quantised activations + outputs) / CUDA-event time, against
  the measured HBM copy bandwidth in MEASURED_PEAKS.json.
* configs: BASELINE configs 2-4 at N = 1 (TinyLlama Q8_0 at chunk 1024 and at
  the configuration's literal chunk 64; TinyLlama Q4_K_M compress and
  decompress of Markov bytes; Qwen2.5-0.5B with V 151,936).
* cpu_baseline / --impl reference: the C restatement of the reference CPU
  path (oracle/, all host threads) on a bounded prefix of the same segment;
  the GPU's payload for that prefix is compared with the oracle's
  (parity.payload_equal).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HEADLINE = "llama3-8b-q4_k"
STREAM_BYTES = 16 << 20
N_SEGMENTS = 8
PREFIX = 8192          # bytes (= tokens) of each segment per step: one n_ctx window
HEAD_CTX = 8192
STREAM_SEED = 16
METRIC = "encode tokens/s (logits+CDF+code)"
# DRAM bytes (read + write) per launch of one token's weight GEMVs of
# TinyLlama Q8_0, from one ncu capture
# (profiles/gemv_decode_stream_tinyllama_q8_0_1token_traffic.md)
DECODE_GEMV_TRAFFIC_PER_LAUNCH = {"tinyllama-q8_0": 12.400e6}
FP32_LANES_PER_SM = 128
# DRAM bytes (read + write) of one fused gate|up Q4_K chunk launch of the
# headline model (28,672 rows x K 4,096 x 1,024 positions), from one ncu
# capture (profiles/gemm_q4k_llama3_8b_q4_k_gate_up_T1024.md); the
# algorithmic bytes of that launch are 188.2 MB
ENCODE_Q4K_TRAFFIC_PER_LAUNCH = 102.500e6 + 85.558e6


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_init(gpus):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist

        rank, local = int(os.environ["RANK"]), int(os.environ.get("LOCAL_RANK", os.environ["RANK"]))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        return rank, ws, local
    if gpus > 1:
        raise SystemExit("--gpus > 1 needs torchrun (one rank per GPU)")
    return 0, 1, 0


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def all_max(x, ws):
    from detllm_b200 import segments as G

    return G.max_over_ranks(x, ws, device="cuda")


LAYERS = 0  # --layers: cut the headline model's layer count (profiling captures only)
PROFILE_ANY_LAYERS = False  # --decode-profile: --layers applies to the profiled configuration


def generator_digest():
    """First 8 hex digits of the SHA-256 of the synthetic GGUF generator's
    sources: a cached model file is reused only if the same generator made it."""
    import hashlib

    h = hashlib.sha256()
    for rel in ("detllm_b200/csrc/synth.c", "detllm_b200/synth.py"):
        with open(os.path.join(ROOT, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()[:8]


def model_bytes(config, rank=0, ws=1):
    """The seeded GGUF of `config`, built once per box (rank 0) into /tmp."""
    import dataclasses

    from detllm_b200 import synth as S

    spec = S.CONFIGS[config]
    if LAYERS and (config == HEADLINE or PROFILE_ANY_LAYERS):
        spec = dataclasses.replace(spec, n_layer=LAYERS)
    path = os.path.join(tempfile.gettempdir(),
                        f"detllm_bench_{config}_L{spec.n_layer}_s{spec.seed}_g{generator_digest()}.gguf")
    if rank == 0 and not os.path.exists(path):
        t = time.time()
        data = S.build_gguf(spec)
        with open(path + ".part", "wb") as f:
            f.write(data)
        os.replace(path + ".part", path)
        log(f"built {path} ({len(data) / 1e9:.2f} GB) in {time.time() - t:.1f}s")
    barrier(ws)
    with open(path, "rb") as f:
        return spec, f.read()


def segment_prefixes():
    from detllm_b200 import segments as G
    from detllm_b200 import synth as S

    segs = G.split_stream(S.markov_stream(STREAM_BYTES, seed=STREAM_SEED), N_SEGMENTS)
    return segs, [s[:PREFIX] for s in segs]


class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local):
        self.local = local
        self.p = None

    def __enter__(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.local}", f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *exc):
        if self.p:
            self.p.terminate()
            self.p.wait(timeout=10)

    def summary(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        load = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def decode_probe(model, vocab, n_ctx, n_prefix=1024, n_steps=48):
    """Single-token forwards (the decode path) after an n_prefix-token
    prefix: device time per token with CUDA graphs, then one profiled pass
    that times every weight GEMV launch, then the same GEMV launches back to
    back in one graph (det_session_gemv_stream)."""
    import detllm_b200 as D
    from detllm_b200 import synth as S

    tokens = S.zipf_tokens(n_prefix + 2 * n_steps + 8, vocab, seed=11)
    out = {}
    with model.session(n_ctx=n_ctx, max_chunk=512) as s:
        for p in range(0, n_prefix, 512):
            s.forward(tokens[p:p + 512], p)
        pos = n_prefix
        for _ in range(4):  # warm-up (graph capture for n = 1)
            s.forward(tokens[pos:pos + 1], pos)
            pos += 1
        s.stats(reset=True)
        for _ in range(n_steps):
            s.forward(tokens[pos:pos + 1], pos)
            pos += 1
        st = s.stats(reset=True)
        out["tokens_per_s"] = n_steps / (st.forward_ms / 1000.0)
        out["ms_per_token"] = st.forward_ms / n_steps
        D.set_profiling(True)
        model.profile(reset=True)
        for _ in range(n_steps):
            s.forward(tokens[pos:pos + 1], pos)
            pos += 1
        D.set_profiling(False)
        pr = s.stats(reset=True)
        gms, gbytes = s.gemv_stream(20)
    # per-kernel-group device time of one token (the profiled pass)
    out["kernels_us_per_token"] = {k: round(1000.0 * ms / n_steps, 2)
                                   for k, (n, ms) in model.profile(reset=True).items() if n}
    out["fused"] = int(pr.gemm_launches) == n_steps  # one GEMM-accounted launch per token
    out["gemv_launches_per_token"] = int(pr.gemm_launches) // n_steps
    out["gemv_ms_per_token"] = pr.gemm_ms / n_steps
    out["gemv_gbs_in_forward"] = pr.gemm_bytes / (pr.gemm_ms / 1000.0) / 1e9 if pr.gemm_ms > 0 else None
    out["positions"] = f"{n_prefix}..{pos - 1}"
    out["gemv_stream_ms_per_token"] = gms
    out["gemv_stream_bytes_per_token"] = gbytes
    out["gemv_stream_gbs"] = gbytes / (gms / 1000.0) / 1e9 if gms > 0 else None
    return out


# bytes per weight of the GEMV matrix types (ggml block sizes)
TYPE_BYTES_PER_WEIGHT = {"Q8_0": 34 / 32, "Q4_0": 18 / 32, "Q4_K": 144 / 256, "Q6_K": 210 / 256}


def decode_chain_floor(spec, add_cycles, sm_mhz, hbm_gbs):
    """The floor of one token's weight GEMVs: each launch takes at least its
    bytes at HBM rate and, for a Q4_K matrix, its row chain of K dependent
    adds (det-quant lib.rs:281-315) at the measured latency of one add.
    Q8_0 / Q4_0 / Q6_K rows are chains of K / 32 or K / 256 adds per lane,
    far below their bytes."""
    from detllm_b200 import synth as S

    names = {S.GT_Q8_0: "Q8_0", S.GT_Q4_0: "Q4_0", S.GT_Q4_K: "Q4_K", S.GT_Q6_K: "Q6_K"}
    hd, d = spec.head_dim, spec.d
    qkv_rows = (spec.n_head + 2 * spec.n_head_kv) * hd
    launches = [(spec.t_attn, qkv_rows, d), (spec.t_attn, d, spec.n_head * hd), (spec.t_gate_up, 2 * spec.d_ff, d),
                (spec.t_down, d, spec.d_ff)]
    us = 0.0
    parts = {}
    for t, rows, k in launches:
        name = names.get(t)
        if name is None:
            return None
        mem = rows * k * TYPE_BYTES_PER_WEIGHT[name] / (hbm_gbs * 1e3)  # us
        chain = k * add_cycles / sm_mhz if name == "Q4_K" else 0.0
        parts[f"{name} {rows}x{k}"] = {"us": round(max(mem, chain), 2), "bound": "chain" if chain > mem else "hbm"}
        us += max(mem, chain) * spec.n_layer
    out_t = names.get(spec.t_embd if spec.tied else spec.t_out)
    if out_t is None:
        return None
    us += spec.vocab * d * TYPE_BYTES_PER_WEIGHT[out_t] / (hbm_gbs * 1e3)
    return {"ms_per_token": us / 1000.0, "add_cycles": add_cycles, "sm_mhz": sm_mhz, "per_layer_launch": parts}


def decode_roofline(dec, config, peak, peak_kind, floor=None):
    n = max(dec["gemv_launches_per_token"], 1)
    gbs = dec["gemv_stream_gbs"]
    extra = {}
    if floor:
        extra = {"chain_floor": floor,
                 "frac_of_chain_floor": floor["ms_per_token"] / dec["gemv_stream_ms_per_token"]}
    return {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak if gbs else None, **extra,
            "traffic": DECODE_GEMV_TRAFFIC_PER_LAUNCH.get(config),
            "traffic_unit": "bytes per launch (ncu capture, see profiles/)",
            "kernel": f"decode weight GEMVs, one token's {n} launches back to back ({config})",
            "peak_kind": peak_kind, "launches": n, "ms_per_launch": dec["gemv_stream_ms_per_token"] / n,
            "bytes_per_launch": dec["gemv_stream_bytes_per_token"] / n, "in_forward_gbs": dec["gemv_gbs_in_forward"]}


def encode_roofline(kprof, ops, sm_mhz, n_sms):
    """The Q4_K chunk GEMMs (q|k|v, o, gate|up of the headline model) against
    the FP32 pipe: 2 rounded ops per weight per position (the reference's
    product and chain add), over their kernel time in one profiled step."""
    groups = ("gemm_qkv", "gemm_o", "gemm_gate_up")
    n = sum(kprof.get(g, (0, 0.0))[0] for g in groups)
    ms = sum(kprof.get(g, (0, 0.0))[1] for g in groups)
    if not n or not sm_mhz or ms <= 0:
        return None
    peak = n_sms * FP32_LANES_PER_SM * sm_mhz * 1e6 / 1e12
    achieved = ops / (ms / 1000.0) / 1e12
    return {"bound": "fp32", "achieved": achieved, "peak": peak, "unit": "T lane-ops/s", "frac": achieved / peak,
            "traffic": ENCODE_Q4K_TRAFFIC_PER_LAUNCH,
            "traffic_unit": "DRAM bytes of one fused gate|up launch (ncu capture, see profiles/); "
                            "its algorithmic bytes are 188.2 MB",
            "kernel": "gemm_q4k_kernel (Q4_K x Q8A chunk GEMMs: q|k|v, o, gate|up of one step)",
            "peak_kind": f"nominal: {n_sms} SMs x {FP32_LANES_PER_SM} FP32 lanes x measured {sm_mhz:.0f} MHz",
            "launches": n, "ms": ms, "ops": ops}


def q4k_weight_positions(spec, positions):
    """Q4_K weight x position products of one step's chunk GEMMs (the
    lm_head of the last window position is skipped by the codec, which this
    count ignores)."""
    from detllm_b200 import synth as S

    hd = spec.head_dim
    per_tok = 0
    if spec.t_attn == S.GT_Q4_K:
        per_tok += spec.d * (spec.n_head * hd * 2 + spec.n_head_kv * hd * 2)
    if spec.t_gate_up == S.GT_Q4_K:
        per_tok += 2 * spec.d_ff * spec.d
    return per_tok * spec.n_layer * positions


def full_stream_estimate(seg_len, n_ctx, t_window, ws):
    """Windows of one segment: the first codes n_ctx symbols, every later one
    replays n_ctx / 4 and codes the rest (det-cli next_window_start,
    main.rs:772-778) and forwards the same n_ctx positions."""
    adv = n_ctx - n_ctx // 4
    windows = 1 + max(0, -(-(seg_len - n_ctx) // adv))
    segs_per_rank = -(-N_SEGMENTS // ws)
    est = segs_per_rank * windows * t_window
    return {"bytes": STREAM_BYTES, "segments": N_SEGMENTS, "windows_per_segment": windows,
            "est_s": est, "est_tokens_per_s": STREAM_BYTES / est,
            "method": "measured one-window step time x windows per segment x segments per GPU"}


def oracle_prefix(gguf, prefix_bytes, n_ctx, budget_s=20.0):
    """The CPU oracle on a bounded prefix: (symbols, payload, seconds)."""
    from oracle import oracle as O

    O.build()
    om = O.Model(gguf)
    syms = O.tokenize(gguf, prefix_bytes, codec=True)
    t = time.time()
    om.encode_symbols(syms[:2], n_ctx, n_ctx // 4)
    per = max((time.time() - t) / 2, 1e-4)
    s = int(max(4, min(len(syms), budget_s / per)))
    t = time.time()
    payload = om.encode_symbols(syms[:s], n_ctx, n_ctx // 4)
    dt = time.time() - t
    om.close()
    return syms[:s], payload, dt


def timed(fn, steps, warmup, model=None):
    """Wall time of `steps` calls after `warmup` untimed ones; the model's
    device-time counters are reset after the warm-up."""
    for _ in range(warmup):
        fn()
    if model is not None:
        model.stats(reset=True)
    t = time.perf_counter()
    for _ in range(steps):
        out = fn()
    return time.perf_counter() - t, out


def sub_configs(D, S, peak, peak_kind, add_cycles=None, sm_mhz=None):
    """BASELINE configs 2-4 on this GPU (N = 1): each model built, loaded,
    measured and freed in turn."""
    out = {}
    # config 2: TinyLlama-1.1B Q8_0, 4,096 Zipf tokens, n_ctx 2048
    spec, g = model_bytes("tinyllama-q8_0")
    m = D.Model(g)
    toks = S.zipf_tokens(4096, spec.vocab, seed=7)
    r = {"workload": "tinyllama-q8_0 encode of 4,096 Zipf(1.1) tokens, n_ctx 2048, overlap 512"}
    for chunk in (1024, 64):
        D.set_encode_chunk(chunk)
        wall, _ = timed(lambda: m.encode_symbols(toks, 2048, 512), 3, 1, m)
        st = m.stats(reset=True)
        r[f"chunk{chunk}"] = {"tokens_per_s": 3 * 4096 / ((st.forward_ms + st.cdf_ms) / 1000.0),
                              "e2e_tokens_per_s": 3 * 4096 / wall}
    D.set_encode_chunk(0)
    dec = decode_probe(m, spec.vocab, 2048)
    r["decode"] = dec
    r["roofline"] = decode_roofline(dec, "tinyllama-q8_0", peak, peak_kind,
                                    decode_chain_floor(spec, add_cycles, sm_mhz, peak) if add_cycles and sm_mhz
                                    else None)
    m.close()
    out["tinyllama-q8_0"] = r
    # config 3: TinyLlama Q4_K_M, compress and decompress of Markov bytes
    spec, g = model_bytes("tinyllama-q4_k_m")
    m = D.Model(g)
    data = S.markov_stream(16384, seed=3)
    wall_c, f = timed(lambda: D.compress(m, data, 2048), 2, 1, m)
    st = m.stats(reset=True)
    enc_tps = 2 * len(data) / ((st.forward_ms + st.cdf_ms) / 1000.0)
    small = D.compress(m, data[:1024], 2048)
    t = time.perf_counter()
    back = D.decompress(m, small)
    wall_d = time.perf_counter() - t
    assert back == data[:1024], "config 3 round trip failed"
    dec_tps = 1024 / wall_d
    out["tinyllama-q4_k_m"] = {
        "workload": "tinyllama-q4_k_m: compress of 16 KiB of order-2 Markov bytes (byte-fallback tokens), "
                    "decompress of a 1 KiB prefix, n_ctx 2048",
        "compress_tokens_per_s": enc_tps, "compress_e2e_tokens_per_s": 2 * len(data) / wall_c,
        "decompress_e2e_tokens_per_s": dec_tps, "round_trip_ok": True,
        "est_1mib_round_trip_s": (1 << 20) / enc_tps + (1 << 20) / dec_tps,
        "decode": decode_probe(m, spec.vocab, 2048)}
    m.close()
    # config 4: Qwen2.5-0.5B Q8_0, V 151,936, 8,192 Zipf tokens at n_ctx 4096
    spec, g = model_bytes("qwen2.5-0.5b-q8_0")
    m = D.Model(g)
    toks = S.zipf_tokens(8192, spec.vocab, seed=7)
    wall, _ = timed(lambda: m.encode_symbols(toks, 4096, 1024), 3, 1, m)
    st = m.stats(reset=True)
    out["qwen2.5-0.5b-q8_0"] = {"workload": "qwen2.5-0.5b-q8_0 encode of 8,192 Zipf(1.1) tokens, n_ctx 4096",
                                "tokens_per_s": 3 * 8192 / ((st.forward_ms + st.cdf_ms) / 1000.0),
                                "e2e_tokens_per_s": 3 * 8192 / wall,
                                "decode": decode_probe(m, spec.vocab, 4096)}
    m.close()
    return out


TP_CONFIG = HEADLINE  # the configuration BASELINE.json runs row-sharded


def chunk_probe(model, vocab):
    """Single-stream chunked forwards (the encode path): positions 0..1023
    as warm-up, then 1024..3071 in two 1,024-position chunks, device time."""
    from detllm_b200 import synth as S

    tk = S.zipf_tokens(3072, vocab, seed=13)
    with model.session(n_ctx=HEAD_CTX, max_chunk=1024) as s:
        s.forward(tk[:1024], 0)
        s.stats(reset=True)
        s.forward(tk[1024:2048], 1024)
        s.forward(tk[2048:3072], 2048)
        st = s.stats(reset=True)
    return 2048 / (st.forward_ms / 1000.0)


def tp_probe(D, gguf, spec, devices):
    """Row-sharded tensor parallelism over `devices` from this one process
    (rank 0, after the timed region, while the other ranks wait): single-
    stream decode and chunked-forward tokens/s on one GPU and on all of
    `devices`, and whether the logits hashes of 256 tokens are equal."""
    from detllm_b200 import synth as S

    try:
        toks = S.zipf_tokens(256, spec.vocab, seed=5)
        one = D.Model(gguf, device=devices[0])
        h_one = one.logits_hash_for_tokens_chunked(toks, 64).hex()
        d1 = decode_probe(one, spec.vocab, HEAD_CTX)
        c1 = chunk_probe(one, spec.vocab)
        one.close()
        t = time.time()
        tp = D.Model(gguf, devices=devices)
        load_s = time.time() - t
        h_tp = tp.logits_hash_for_tokens_chunked(toks, 64).hex()
        with tp.session(n_ctx=HEAD_CTX, max_chunk=512) as s:
            tk = S.zipf_tokens(1024 + 60, spec.vocab, seed=11)
            for p in range(0, 1024, 512):
                s.forward(tk[p:p + 512], p)
            for p in range(1024, 1028):
                s.forward(tk[p:p + 1], p)
            s.stats(reset=True)
            for p in range(1028, 1076):
                s.forward(tk[p:p + 1], p)
            st = s.stats(reset=True)
        tps = 48 / (st.forward_ms / 1000.0)
        ctp = chunk_probe(tp, spec.vocab)
        tp.close()
    except Exception as e:  # reported, never fatal to the bench line
        return {"config": TP_CONFIG, "parts": len(devices), "unavailable": f"{type(e).__name__}: {e}"}
    return {"config": TP_CONFIG, "parts": len(devices), "devices": devices, "decode_tokens_per_s": tps,
            "decode_tokens_per_s_1gpu": d1["tokens_per_s"], "speedup": tps / d1["tokens_per_s"],
            "chunk_tokens_per_s": ctp, "chunk_tokens_per_s_1gpu": c1, "chunk_speedup": ctp / c1,
            "logits_hash_equal": h_tp == h_one, "load_s": round(load_s, 1)}


def run_reference(args):
    """The reference arm: the C restatement of the reference CPU path
    (oracle/, all host threads) on the headline configuration, each step a
    bounded prefix of segment 0 (rank 0 only)."""
    rank, ws, local = dist_init(args.gpus)
    if rank != 0:
        return
    spec, gguf = model_bytes(HEADLINE)
    from oracle import oracle as O

    O.build()
    _, prefixes = segment_prefixes()
    syms = O.tokenize(gguf, prefixes[0], codec=True)
    om = O.Model(gguf)
    sample = args.ref_sample
    per = []
    for i in range(args.warmup + args.steps):
        t = time.time()
        om.encode_symbols(syms[:sample], HEAD_CTX, HEAD_CTX // 4)
        if i >= args.warmup:
            per.append(time.time() - t)
    tps = sample * len(per) / sum(per)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(per) / len(per),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+int8",
        "data": "synthetic (seeded random-init weights, order-2 Markov bytes)",
        "config": {"workload": f"{HEADLINE} encode, first {sample} bytes of segment 0 of the 16 MiB stream per step, "
                               f"n_ctx {HEAD_CTX}", "global_batch": sample, "seq_len": HEAD_CTX, "parallelism": "cpu"},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"encode of the first {sample} byte tokens of segment 0 per step"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run(args):
    rank, ws, local = dist_init(args.gpus)
    import detllm_b200 as D
    from detllm_b200 import synth as S

    spec, gguf = model_bytes(HEADLINE, rank, ws)
    segs, prefixes = segment_prefixes()
    t = time.time()
    model = D.Model(gguf, device=local)
    log(f"rank {rank}: model on cuda:{local} in {time.time() - t:.1f}s")
    import torch

    torch.cuda.set_device(local)
    step_i = [0]

    def step():
        seg = (step_i[0] * ws + rank) % N_SEGMENTS
        step_i[0] += 1
        return seg, D.compress(model, prefixes[seg], HEAD_CTX)

    for _ in range(args.warmup):
        step()
    model.stats(reset=True)
    files = {}
    barrier(ws)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            seg, f = step()
            files[seg] = f
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    barrier(ws)
    st = model.stats(reset=True)
    dev_s = (st.forward_ms + st.cdf_ms) / 1000.0
    dev_max, wall_max = all_max(dev_s, ws), all_max(wall, ws)
    clocks = clk.summary()
    # one profiled step: per-kernel-group device time
    D.set_profiling(True)
    model.profile(reset=True)
    D.compress(model, prefixes[rank % N_SEGMENTS], HEAD_CTX)
    D.set_profiling(False)
    model.stats(reset=True)
    kprof = model.profile(reset=True)
    # decode path: a short round trip of this rank's first segment, then the
    # one-token probe and the weight-GEMV stream
    small = D.compress(model, prefixes[rank % N_SEGMENTS][:256], HEAD_CTX)
    round_trip_ok = D.decompress(model, small) == prefixes[rank % N_SEGMENTS][:256]
    dec = decode_probe(model, spec.vocab, HEAD_CTX)
    tpj = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))
        dist.barrier(group=cpu)
        if rank == 0:
            model.close()
            tpj = tp_probe(D, gguf, spec, list(range(ws)))
        dist.barrier(group=cpu)
    if rank != 0:
        model.close()
        return
    total = PREFIX * args.steps * ws
    peak, peak_kind = peaks()
    props = torch.cuda.get_device_properties(local)
    add_cycles = D.add_latency_cycles(local)  # measured: the floor of every ordered chain
    line = {
        "metric": METRIC, "value": total / dev_max, "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dev_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+int8",
        "data": "synthetic (seeded random-init weights, order-2 Markov byte stream)",
        "config": {"workload": f"{HEADLINE} segment-parallel compress: 16 MiB Markov stream in {N_SEGMENTS} segments, "
                               f"each step one segment's first {PREFIX} bytes per GPU (one n_ctx {HEAD_CTX} window, "
                               f"overlap {HEAD_CTX // 4}), chunk 1024",
                   "global_batch": PREFIX * ws, "seq_len": HEAD_CTX, "parallelism": f"segments{ws}",
                   "l2": f"weights {S.weight_bytes_per_token(spec) / 1e9:.2f} GB streamed per chunk > 126 MB L2 "
                         "(no flush)"},
        "e2e": {"value": total / wall_max, "unit": "tokens/s", "h2d_bytes_per_step": st.h2d_bytes // max(args.steps, 1),
                "d2h_bytes_per_step": st.d2h_bytes // max(args.steps, 1)},
        "gpu_launches": int(st.launches),
        "roofline": encode_roofline(kprof, 2.0 * q4k_weight_positions(spec, PREFIX), clocks.get("sm_mhz"),
                                    props.multi_processor_count),
        "roofline_decode": decode_roofline(dec, HEADLINE, peak, peak_kind,
                                           decode_chain_floor(spec, add_cycles, clocks.get("sm_mhz"), peak)
                                           if add_cycles and clocks.get("sm_mhz") else None),
        "full_stream": full_stream_estimate(len(segs[0]), HEAD_CTX, dev_max / args.steps, ws),
        "decode": dec,
        "round_trip_ok": round_trip_ok,
        "kernels": {k: {"launches": n, "ms": round(ms, 3),
                        "share": round(ms / max(sum(v[1] for v in kprof.values()), 1e-9), 4)}
                    for k, (n, ms) in kprof.items() if n},
        "clocks": clocks,
        "tensor_parallel": tpj,
        "payload_bytes": {str(k): len(v) for k, v in sorted(files.items())},
        "weight_bytes_per_token": S.weight_bytes_per_token(spec),
    }
    if ws == 1 and not args.no_cpu_baseline:
        syms, want, dt = oracle_prefix(gguf, prefixes[0], HEAD_CTX)
        got = model.encode_symbols(syms, HEAD_CTX, HEAD_CTX // 4)
        line["cpu_baseline"] = {"value": len(syms) / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"encode of the first {len(syms)} byte tokens of segment 0 (~{dt:.0f}s)"}
        line["parity"] = {"prefix_tokens": len(syms), "payload_equal": got == want, "payload_bytes": len(got)}
    model.close()
    if ws == 1 and not args.no_configs:
        line["configs"] = sub_configs(D, S, peak, peak_kind, add_cycles, clocks.get("sm_mhz"))
    print(json.dumps(line), flush=True)


def run_decode_profile(args):
    """One configuration's one-position forwards for a profiler: a 512-token
    prefill, 6 warm-up tokens, 20 timed tokens (device time printed), then
    `--profile-tokens` more between cudaProfilerStart and cudaProfilerStop, so
    that `ncu --profile-from-start off` sees exactly those launches."""
    import torch

    import detllm_b200 as D
    from detllm_b200 import synth as S

    spec, gguf = model_bytes(args.decode_profile)
    m = D.Model(gguf)
    toks = S.zipf_tokens(600 + args.profile_tokens, spec.vocab, seed=3)
    with m.session(n_ctx=2048, max_chunk=512) as s:
        s.forward(toks[:512], 0)
        pos = 512
        for _ in range(6):
            s.forward(toks[pos:pos + 1], pos)
            pos += 1
        s.stats(reset=True)
        for _ in range(20):
            s.forward(toks[pos:pos + 1], pos)
            pos += 1
        st = s.stats(reset=True)
        torch.cuda.profiler.start()
        for _ in range(args.profile_tokens):
            s.forward(toks[pos:pos + 1], pos)
            pos += 1
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    m.close()
    print(json.dumps({"decode_profile": args.decode_profile, "layers": spec.n_layer, "position": 512,
                      "ms_per_token": st.forward_ms / 20}), flush=True)


def run_chunk_profile(args):
    """One configuration's chunked forwards for a profiler: positions
    0..ctx-1 (`--ctx`, default 1024) in chunks of `--chunk` as warm-up, the
    same positions again timed (device time printed), then between
    cudaProfilerStart and cudaProfilerStop the last chunk once more or, when
    ctx > 1024, the first and the last chunk (attention time grows linearly
    with the chunk's position, so the two together weigh the kernels as a
    whole window does)."""
    import torch

    import detllm_b200 as D
    from detllm_b200 import synth as S

    if args.q8_tensor_cores:
        D.set_q8_tensor_cores(True)
    spec, gguf = model_bytes(args.chunk_profile)
    m = D.Model(gguf)
    ctx = max(args.ctx, 16)
    c = min(args.chunk, 1024, ctx)
    toks = S.zipf_tokens(ctx, spec.vocab, seed=3)
    starts = list(range(0, ctx, c))
    with m.session(n_ctx=ctx, max_chunk=c) as s:
        for p in starts:
            s.forward(toks[p:p + c], p)
        s.stats(reset=True)
        for p in starts:
            s.forward(toks[p:p + c], p)
        st = s.stats(reset=True)
        torch.cuda.profiler.start()
        for p in ([0] if ctx > 1024 else []) + [starts[-1]]:
            s.forward(toks[p:p + c], p)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    m.close()
    print(json.dumps({"chunk_profile": args.chunk_profile, "layers": spec.n_layer, "chunk": c, "ctx": ctx,
                      "q8_tensor_cores": bool(args.q8_tensor_cores),
                      "tokens_per_s": ctx / (st.forward_ms / 1000.0)}), flush=True)


def main():
    global PREFIX, LAYERS, PROFILE_ANY_LAYERS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--ref-sample", type=int, default=4, help="byte tokens per reference step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the BASELINE configs 2-4 sub-benchmarks")
    ap.add_argument("--prefix", type=int, default=PREFIX,
                    help="bytes of each segment per step (default one n_ctx window; smaller is for profiling)")
    ap.add_argument("--layers", type=int, default=0,
                    help="layers of the headline model (default all; fewer only for profiling captures)")
    ap.add_argument("--decode-profile", default=None, metavar="CONFIG",
                    help="only one-position forwards of CONFIG, for a profiler (see run_decode_profile)")
    ap.add_argument("--profile-tokens", type=int, default=1)
    ap.add_argument("--chunk-profile", default=None, metavar="CONFIG",
                    help="only chunked forwards of CONFIG, for a profiler (see run_chunk_profile)")
    ap.add_argument("--chunk", type=int, default=1024)
    ap.add_argument("--ctx", type=int, default=1024,
                    help="with --chunk-profile: positions forwarded (the window); above 1,024 the first and last "
                         "chunks are profiled")
    ap.add_argument("--q8-tensor-cores", action="store_true",
                    help="with --chunk-profile: the tcgen05 Q8_0 / Q4_0 chunk GEMM instead of the mma.sync one")
    args = ap.parse_args()
    PREFIX = args.prefix
    LAYERS = args.layers
    if args.decode_profile:
        PROFILE_ANY_LAYERS = True
        run_decode_profile(args)
        return
    if args.chunk_profile:
        PROFILE_ANY_LAYERS = True
        run_chunk_profile(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
