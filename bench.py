#!/usr/bin/env python3
"""Benchmark: encode tokens/s of the detllm token loop on B200.

Workload: a TinyLlama-1.1B-shaped decoder with
random-init Q8_0 weights (22 layers, d 2048, 32/4 heads, FFN 5632, vocab
32000), 4096 Zipf(1.1) token ids encoded as codec symbols at n_ctx 2048
(overlap 512, one window rollover), forward chunk 1024.  One step = one full
compress of that stream: teacher-forced forward -> logits -> CDF ranges ->
host range coder, through det_encode_symbols.

* value: tokens of all ranks / max over ranks of the device time of the
  timed steps (CUDA events on the session stream: forward + CDF kernels).
* e2e: same tokens / max over ranks of the wall time of the C-ABI calls with
  host buffers (symbols in, payload out; host<->device copies and host range
  coding inside).
* roofline: the decode GEMVs (one token per forward, after a 1024-token
  prefix): one token's weight GEMV launches replayed back to back in a CUDA
  graph (programmatic dependent launch), algorithmic bytes (weights +
  activations + outputs) / CUDA-event time, against the measured HBM copy
  bandwidth in MEASURED_PEAKS.json.  decode.gemv_gbs_in_forward is the same
  ratio for the launches inside real forwards, each bracketed by events.
  With DETGPU_FUSED_DECODE=1 the one-position forward is one persistent
  kernel (decode_fused_kernel) and the roofline is that launch: all weight
  bytes of one token + the KV rows its attention reads, / its event time.
  The chunked encode GEMM is FP32-pipe bound (its exact ordered fold) and
  is reported separately under chunk_gemm with the per-kernel time shares.
* cpu_baseline / --impl reference: the C restatement of the reference CPU
  path (oracle/, all host threads) on a bounded prefix of the same stream.

Multi-GPU (torchrun, one rank per GPU): independent compression segments,
one model replica per GPU, no data-path collective (weak scaling).
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

CONFIG = "tinyllama-q8_0"
N_TOKENS = 4096
N_CTX = 2048
OVERLAP = N_CTX // 4
# --config: BASELINE.json configs 2-4 (tokens per rank, n_ctx)
CONFIG_RUNS = {"tinyllama-q8_0": (4096, 2048), "tinyllama-q4_k_m": (4096, 2048),
               "qwen2.5-0.5b-q8_0": (8192, 4096), "llama3-8b-q4_k": (4096, 8192)}
METRIC = "encode tokens/s (logits+CDF+code)"
# DRAM bytes (read + write) per launch of one token's 89 weight GEMVs of the
# headline config, from one ncu capture
# (profiles/gemv_decode_stream_tinyllama_q8_0_1token_traffic.md)
DECODE_GEMV_TRAFFIC_PER_LAUNCH = 12.400e6
# DRAM bytes (read + write) per launch of the fused one-position kernel, per
# config, from one ncu capture (profiles/decode_fused_tinyllama_q8_0_1token.md)
DECODE_FUSED_TRAFFIC_PER_LAUNCH = {"tinyllama-q8_0": 1146.713e6 + 25.272e6}


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


def model_bytes(rank, ws):
    """Build the seeded GGUF once per box (rank 0), shared through /tmp."""
    from detllm_b200 import synth as S

    spec = S.CONFIGS[CONFIG]
    path = os.path.join(tempfile.gettempdir(), f"detllm_bench_{CONFIG}_s{spec.seed}.gguf")
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


def oracle_sample(spec, gguf, tokens, budget_s=20.0):
    """Time the CPU oracle on a bounded prefix (encode of the first S symbols)."""
    from oracle import oracle as O

    O.build()
    t = time.time()
    om = O.Model(gguf)
    load_s = time.time() - t
    t = time.time()
    om.encode_symbols(tokens[:2], N_CTX, OVERLAP)
    per_tok = max((time.time() - t) / 2, 1e-4)
    s = int(max(4, min(len(tokens), budget_s / per_tok)))
    t = time.time()
    om.encode_symbols(tokens[:s], N_CTX, OVERLAP)
    dt = time.time() - t
    om.close()
    return s, dt, load_s


def decode_tokens_per_s(model, vocab, n_prefix=1024, n_steps=48):
    """Single-token forwards after an n_prefix-token prefix (CUDA graphs):
    device time per token (forward events on the session stream)."""
    from detllm_b200 import synth as S

    tokens = S.zipf_tokens(n_prefix + n_steps + 8, vocab, seed=11)
    with model.session(n_ctx=N_CTX, max_chunk=512) as s:
        for p in range(0, n_prefix, 512):
            s.forward(tokens[p:p + 512], p)
        pos = n_prefix
        for _ in range(4):
            s.forward(tokens[pos:pos + 1], pos)
            pos += 1
        s.stats(reset=True)
        for _ in range(n_steps):
            s.forward(tokens[pos:pos + 1], pos)
            pos += 1
        st = s.stats(reset=True)
    return n_steps / (st.forward_ms / 1000.0), st.forward_ms / n_steps


def run_tp(args):
    """--tp G1,G2,...: row-sharded tensor parallelism in one process over
    devices 0..G-1 (det_model_load_tp): single-stream decode tokens/s,
    chunked encode tokens/s of the config's stream, and the logits hash of
    the first 256 tokens, which must equal the 1-GPU hash.  One JSON line
    per part count."""
    import detllm_b200 as D
    from detllm_b200 import synth as S

    spec, gguf = model_bytes(0, 1)
    tokens = S.zipf_tokens(N_TOKENS, spec.vocab, seed=7)
    ndev = D.device_count()
    ref_hash = None
    for G in [int(x) for x in args.tp.split(",")]:
        if G > ndev:
            log(f"--tp {G}: only {ndev} devices, skipped")
            continue
        t = time.time()
        model = D.Model(gguf, device=0) if G == 1 else D.Model(gguf, devices=list(range(G)))
        load_s = time.time() - t
        h = model.logits_hash_for_tokens_chunked(tokens[:256], 64).hex()
        ref_hash = ref_hash or h
        dec_tps, dec_ms = decode_tokens_per_s(model, spec.vocab)
        for _ in range(args.warmup):
            model.encode_symbols(tokens, N_CTX, OVERLAP)
        model.stats(reset=True)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            model.encode_symbols(tokens, N_CTX, OVERLAP)
        wall = time.perf_counter() - t0
        st = model.stats(reset=True)
        dev_s = (st.forward_ms + st.cdf_ms) / 1000.0
        wb = S.weight_bytes_per_token(spec)
        print(json.dumps({
            "mode": "tensor-parallel", "config": CONFIG, "parts": G, "devices": list(range(G)),
            "decode_tokens_per_s": dec_tps, "decode_ms_per_token": dec_ms,
            "decode_weight_gbs_per_gpu": wb / G / (dec_ms / 1000.0) / 1e9,
            "encode_tokens_per_s": N_TOKENS * args.steps / dev_s,
            "encode_e2e_tokens_per_s": N_TOKENS * args.steps / wall,
            "logits_hash_256": h, "hash_equals_1gpu": h == ref_hash, "load_s": round(load_s, 1),
        }), flush=True)
        model.close()


TP_CONFIG = "llama3-8b-q4_k"  # the configuration BASELINE.json runs row-sharded


def tp_probe(D, devices):
    """Row-sharded tensor parallelism over `devices` from this one process
    (run by rank 0 after the timed region while the other ranks wait), on the
    Llama-3-8B-shaped Q4_K/Q6_K model BASELINE.json names for it:
    single-stream decode tokens/s on one GPU and on all of `devices`, and
    whether the logits hashes of 256 tokens are equal."""
    from detllm_b200 import synth as S

    spec = S.CONFIGS[TP_CONFIG]
    try:
        t = time.time()
        gguf = S.build_gguf(spec)
        build_s = time.time() - t
        toks = S.zipf_tokens(256, spec.vocab, seed=5)
        one = D.Model(gguf, device=devices[0])
        h_one = one.logits_hash_for_tokens_chunked(toks, 64).hex()
        tps1, ms1 = decode_tokens_per_s(one, spec.vocab)
        one.close()
        t = time.time()
        tp = D.Model(gguf, devices=devices)
        load_s = time.time() - t
        h_tp = tp.logits_hash_for_tokens_chunked(toks, 64).hex()
        tps, ms = decode_tokens_per_s(tp, spec.vocab)
        tp.close()
    except Exception as e:  # reported, never fatal to the bench line
        return {"config": TP_CONFIG, "parts": len(devices), "unavailable": f"{type(e).__name__}: {e}"}
    return {"config": TP_CONFIG, "parts": len(devices), "devices": devices, "decode_tokens_per_s": tps,
            "decode_ms_per_token": ms, "decode_tokens_per_s_1gpu": tps1, "decode_ms_per_token_1gpu": ms1,
            "speedup": tps / tps1, "logits_hash_equal": h_tp == h_one,
            "weight_bytes_per_token": S.weight_bytes_per_token(spec), "load_s": round(load_s, 1),
            "build_s": round(build_s, 1)}


def decode_probe(D, model, vocab, n_prefix=1024, n_steps=48):
    """Single-token forwards (the decode path) after a 1024-token prefix:
    device time per token with CUDA graphs, then one profiled pass that times
    every weight GEMV launch (algorithmic bytes / event time)."""
    from detllm_b200 import synth as S

    tokens = S.zipf_tokens(n_prefix + 2 * n_steps + 8, vocab, seed=11)
    out = {}
    with model.session(n_ctx=N_CTX, max_chunk=512) as s:
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
        for _ in range(n_steps):
            s.forward(tokens[pos:pos + 1], pos)
            pos += 1
        D.set_profiling(False)
        pr = s.stats(reset=True)
        gms, gbytes = s.gemv_stream(20)
    # one GEMM-accounted launch per token: the fused one-position kernel ran
    out["fused"] = int(pr.gemm_launches) == n_steps
    out["gemv_launches"] = int(pr.gemm_launches)
    out["gemv_ms_per_token"] = pr.gemm_ms / n_steps
    out["gemv_bytes_per_launch"] = pr.gemm_bytes / max(pr.gemm_launches, 1)
    out["gemv_ms_per_launch"] = pr.gemm_ms / max(pr.gemm_launches, 1)
    out["gemv_gbs_in_forward"] = pr.gemm_bytes / (pr.gemm_ms / 1000.0) / 1e9 if pr.gemm_ms > 0 else None
    out["positions"] = f"{n_prefix}..{pos - 1}"
    # the same launches back to back (one graph, programmatic dependent launch)
    out["gemv_stream_ms_per_token"] = gms
    out["gemv_stream_bytes_per_token"] = gbytes
    out["gemv_stream_gbs"] = gbytes / (gms / 1000.0) / 1e9 if gms > 0 else None
    return out


def roofline(dec, peak, peak_kind):
    """The decode roofline object: the fused one-position kernel when it ran,
    else the per-op weight GEMVs back to back (see the module docstring)."""
    if dec.get("fused"):
        gbs = dec["gemv_gbs_in_forward"]
        return {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                "frac": gbs / peak if gbs else None, "traffic": DECODE_FUSED_TRAFFIC_PER_LAUNCH.get(CONFIG),
                "traffic_unit": "bytes per launch (ncu capture, see profiles/)",
                "kernel": f"decode_fused_kernel: one token's forward (all layers + lm_head) in one launch ({CONFIG})",
                "peak_kind": peak_kind, "launches": 1, "ms_per_launch": dec["gemv_ms_per_launch"],
                "bytes_per_launch": dec["gemv_bytes_per_launch"],
                "bytes": "weights of every matrix + K and V rows read by the attention",
                "per_op_gemv_stream_gbs": dec["gemv_stream_gbs"]}
    n = max(dec["gemv_launches"] // 48, 1)
    return {"bound": "hbm", "achieved": dec["gemv_stream_gbs"], "peak": peak, "unit": "GB/s",
            "frac": dec["gemv_stream_gbs"] / peak if dec["gemv_stream_gbs"] else None,
            "traffic": DECODE_GEMV_TRAFFIC_PER_LAUNCH if CONFIG == "tinyllama-q8_0" else None,
            "traffic_unit": "bytes per launch (ncu capture, see profiles/)",
            "kernel": f"decode weight GEMVs, one token's {n} launches back to back ({CONFIG})",
            "peak_kind": peak_kind, "launches": n, "ms_per_launch": dec["gemv_stream_ms_per_token"] / n,
            "bytes_per_launch": dec["gemv_stream_bytes_per_token"] / n, "in_forward_gbs": dec["gemv_gbs_in_forward"]}


def run_reference(args):
    rank, ws, local = dist_init(args.gpus)
    if rank != 0:
        return
    from detllm_b200 import synth as S

    spec, gguf = model_bytes(0, 1)
    tokens = S.zipf_tokens(N_TOKENS, spec.vocab, seed=7)
    from oracle import oracle as O

    O.build()
    om = O.Model(gguf)
    per = []
    sample = args.ref_sample
    for i in range(args.warmup + args.steps):
        t = time.time()
        om.encode_symbols(tokens[:sample], N_CTX, OVERLAP)
        if i >= args.warmup:
            per.append(time.time() - t)
    tps = sample * len(per) / sum(per)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(per) / len(per),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+int8",
        "data": "synthetic (seeded random-init weights, Zipf tokens)",
        "config": {"workload": f"{CONFIG} encode, first {sample} of {N_TOKENS} Zipf tokens per step, n_ctx {N_CTX}",
                   "global_batch": sample, "seq_len": N_CTX, "parallelism": "cpu"},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"first {sample} tokens of the {N_TOKENS}-token stream per step"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run(args):
    import numpy as np

    rank, ws, local = dist_init(args.gpus)
    import detllm_b200 as D
    from detllm_b200 import synth as S

    spec, gguf = model_bytes(rank, ws)
    tokens = S.zipf_tokens(N_TOKENS, spec.vocab, seed=7 + rank)  # one segment per rank
    t = time.time()
    model = D.Model(gguf, device=local)
    log(f"rank {rank}: model on cuda:{local} in {time.time() - t:.1f}s")
    import torch

    torch.cuda.set_device(local)
    for _ in range(args.warmup):
        model.encode_symbols(tokens, N_CTX, OVERLAP)
    model.stats(reset=True)
    barrier(ws)
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            payload = model.encode_symbols(tokens, N_CTX, OVERLAP)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    barrier(ws)
    st = model.stats(reset=True)
    dev_s = (st.forward_ms + st.cdf_ms) / 1000.0
    dev_max, wall_max = all_max(dev_s, ws), all_max(wall, ws)
    # one profiled step for the per-launch GEMV/GEMM roofline
    D.set_profiling(True)
    model.profile(reset=True)
    model.encode_symbols(tokens, N_CTX, OVERLAP)
    D.set_profiling(False)
    prof = model.stats(reset=True)
    kprof = model.profile(reset=True)
    dec = decode_probe(D, model, spec.vocab)
    # tensor parallelism over all the job's GPUs, from rank 0 alone; the
    # other ranks wait on a CPU (gloo) group, since an NCCL barrier kernel
    # spinning on their GPU would time-slice with rank 0's parts there
    tpj = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))
        dist.barrier(group=cpu)
        if rank == 0:
            tpj = tp_probe(D, list(range(ws)))
        dist.barrier(group=cpu)
    if rank != 0:
        return
    total_tokens = N_TOKENS * args.steps * ws
    peak, peak_kind = peaks()
    achieved = prof.gemm_bytes / (prof.gemm_ms / 1000.0) / 1e9 if prof.gemm_ms > 0 else None
    line = {
        "metric": METRIC, "value": total_tokens / dev_max, "unit": "tokens/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dev_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+int8",
        "data": "synthetic (seeded random-init weights, Zipf(1.1) tokens)",
        "config": {"workload": f"{CONFIG} encode: {N_TOKENS} Zipf tokens per rank, n_ctx {N_CTX}, overlap {OVERLAP}, "
                               f"chunk {os.environ.get('DETGPU_CHUNK', '1024')}", "global_batch": N_TOKENS * ws, "seq_len": N_CTX,
                   "parallelism": f"segments{ws}",
                   "l2": f"weights {S.weight_bytes_per_token(spec) / 1e9:.2f} GB streamed per chunk > 126 MB L2 (no flush)"},
        "e2e": {"value": total_tokens / wall_max, "unit": "tokens/s", "h2d_bytes_per_step": st.h2d_bytes // args.steps,
                "d2h_bytes_per_step": st.d2h_bytes // args.steps},
        "gpu_launches": int(st.launches),
        "roofline": roofline(dec, peak, peak_kind),
        "decode": dec,
        "chunk_gemm": {"bound": "fp32 pipe (exact ordered fold, 4 fp32 ops per weight per position)",
                       "weight_stream_gbs": achieved, "launches": int(prof.gemm_launches),
                       "ms_per_launch": prof.gemm_ms / max(prof.gemm_launches, 1),
                       "bytes_per_launch": prof.gemm_bytes / max(prof.gemm_launches, 1),
                       "share_of_device_time": prof.gemm_ms / max(prof.forward_ms + prof.cdf_ms, 1e-9)},
        "kernels": {k: {"launches": n, "ms": round(ms, 3), "share": round(ms / max(sum(v[1] for v in kprof.values()),
                                                                                  1e-9), 4)}
                    for k, (n, ms) in kprof.items() if n},
        "clocks": clk.summary(),
        "tensor_parallel": tpj,
        "payload_bytes": len(payload),
        "weight_bytes_per_token": S.weight_bytes_per_token(spec),
    }
    if ws == 1 and not args.no_cpu_baseline:
        s, dt, load_s = oracle_sample(spec, gguf, tokens)
        line["cpu_baseline"] = {"value": s / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"encode of the first {s} tokens of the stream (~{dt:.0f}s)"}
    print(json.dumps(line), flush=True)
    model.close()


def main():
    global N_TOKENS, CONFIG, N_CTX, OVERLAP
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--ref-sample", type=int, default=16, help="tokens per reference step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", default=CONFIG, choices=sorted(CONFIG_RUNS),
                    help="model configuration (default: the headline BASELINE config)")
    ap.add_argument("--tp", default=None,
                    help="comma-separated part counts: row-sharded tensor parallelism in one process "
                         "(single-stream decode / encode), instead of the segment-parallel bench")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per rank per step (default: the config's; smaller values are for profiling)")
    args = ap.parse_args()
    CONFIG = args.config
    N_TOKENS, N_CTX = CONFIG_RUNS[CONFIG]
    OVERLAP = N_CTX // 4
    if args.tokens:
        N_TOKENS = args.tokens
    if args.tp:
        run_tp(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
