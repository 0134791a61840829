"""Decode throughput of the B200 engine on the headline benchmark workload, one JSON line.

Default workload (benchmark config 2): Qwen3.5-2B-shaped f16 hybrid decoder (synthetic, seed 1),
batch 1 per GPU, KV cache prefilled to 3968 tokens, then greedy decode steps (one step = one
token of one sequence per GPU) up to the 4096 limit. With N GPUs (torchrun) every rank decodes
its own independent sequence on its own weight replica (weak scaling, no collective on the data
path; NCCL is used only for the barrier and the max-over-ranks timing).

  value   device-resident greedy decode (CUDA-graph replays, GPU argmax feeding the next
          embedding), CUDA events on the engine's stream, max over ranks.
  e2e     the agent's per-token loop through the public API with device sampling:
          qne_step_sample(token, pos) with the reference's default sampling options (temperature
          0.6, top_k 20, top_p 0.95), 8 bytes (token id) in and 8 bytes (token, status) out per
          token. `e2e_host_logits` is the reference agent's own loop: qne_step per token with the
          logits (993 KB f32) read back to pinned host memory and the pick made on the host.
  roofline  the dominant kernel (f16 GEMV, SwiGLU gate_up of all 24 layers) timed live with CUDA
          events: algorithmic bytes per launch / mean launch time vs MEASURED_PEAKS.json.
  cpu_baseline  the CPU oracle (C++ restatement of the reference decoder) on the host cores,
          rank 0 at N=1 only, a bounded sample of decode tokens.

`--impl reference` times the reference's CPU arithmetic (the oracle port: the reference is Rust +
WGSL and cannot be built or run on this box) on the same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen-native-engine_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "decode tok/s (B=1 and B=32/GPU) at 1/2/4/8 B200; GEMV/attn % of HBM BW"
PROMPT, STEPS_MAX = 3968, 128


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path("/tmp") / f"qne_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.1)
        self.proc.terminate()
        self.proc.wait()
        rows = [r.split(",") for r in self.path.read_text().splitlines() if r.strip()]
        sm = [float(r[1]) for r in rows if len(r) >= 9]
        mx = [float(r[2]) for r in rows if len(r) >= 9]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_collectives(dist, world: int, device: str):
    """Barrier and max-over-ranks used around every timed region (one process per GPU; gloo on
    CPU in the tests). Every rank must call them in the same order."""
    import torch

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    return barrier, max_over_ranks


def rank_seed(base: int, rank: int) -> int:
    """Seed of rank `rank`'s synthetic inputs: every replica decodes its own sequences."""
    return base + 1000 * rank


def aggregate_rate(world: int, units_per_rank: int, max_ms: float) -> float:
    """Whole-job throughput: the units all ranks processed over the slowest rank's time."""
    return world * units_per_rank / (max_ms * 1e-3)


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), for the CPU-baseline record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def bench_config(cfg_n: int, prompt_len: int, steps: int, world: int, weight_file_bytes: int) -> dict:
    """The `config` object of the B=1 line, shared by both arms so that they name one workload."""
    from qne import synth
    info = synth.baseline_config(cfg_n)
    size_name = {"0.8b": "0.8B", "2b": "2B"}[info["size"]]
    c = {"workload": f"config {cfg_n}: Qwen3.5-{size_name}-shaped {info['kind']} hybrid decoder "
                     f"(synthetic, seed {info['seed']}), B=1 per GPU, KV prefilled to {prompt_len}, "
                     f"{steps} greedy decode steps",
         "model": f"qwen3.5-{size_name.lower()}-shaped", "global_batch": world, "seq_len": 4096,
         "parallelism": f"replicas x{world}",
         "l2": f"inputs larger than L2 ({weight_file_bytes / 1e9:.2f} GB of weights read per step)"}
    return c


def cpu_oracle_decode(om, prompt_len: int, warmup: int, tokens: int, first_token: int):
    """Times `tokens` greedy oracle steps from the state `om` holds after a prompt of prompt_len
    (snapshot taken by the caller): `warmup` untimed steps, restore, then the timed steps."""
    from oracle import oracle
    tok = first_token
    for i in range(warmup):
        tok = oracle.argmax(om.step(tok, prompt_len + i))
    om.restore()
    tok = first_token
    t0 = time.perf_counter()
    for i in range(tokens):
        tok = oracle.argmax(om.step(tok, prompt_len + i))
    return tokens / (time.perf_counter() - t0)


def cpu_baseline_sample(s, cfg_n: int, prompt_len: int, tokens: int = 48):
    """cpu_baseline leg of our arm (rank 0, N=1): the oracle decoding `tokens` steps at the same
    context as the timed GPU steps, its KV cache and GDN states filled with seeded synthetic history
    (oracle_model_fill_synthetic) instead of a prompt (a step's cost depends on the context length,
    not on the cached values)."""
    from oracle import oracle
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    om.fill_synthetic(prompt_len, 7)
    om.snapshot()
    rate = cpu_oracle_decode(om, prompt_len, 2, tokens, 12345)
    om.close()
    return rate, oracle.threads()


def reference_arm(args, world, rank):
    """`--impl reference`: the reference's decode arithmetic on the host cores (the CPU oracle, a
    restatement of the reference WGSL decoder; the reference itself is Rust + wgpu and cannot run
    here) on the workload of our arm: config 2, the same 3968-token prompt (brought in through the
    oracle's batched CPU prefill, untimed), then `--warmup` untimed steps, a restore, and the timed
    greedy steps from position 3968. Imports only the oracle and the synthetic-model generator: no
    engine code is loaded. Rank 0 alone runs; the other ranks exit without work."""
    if rank != 0:
        return
    from oracle import oracle
    from qne import synth
    cfg_n = args.config
    info = synth.baseline_config(cfg_n)
    steps = args.steps
    prompt_len = min(args.prompt if args.prompt is not None else info["prompt"], 4096 - steps)
    s = synth.build_config(cfg_n)
    om = oracle.OracleModel(s.index_json, s.weights, kv_f16=True)
    prompt = synth.prompt_ids(prompt_len, rank_seed(1, 0))
    t0 = time.perf_counter()
    logits = om.prefill_batched(prompt)
    prefill_s = time.perf_counter() - t0
    om.snapshot()
    rate = cpu_oracle_decode(om, prompt_len, min(args.warmup, 4096 - prompt_len), steps, oracle.argmax(logits))
    cores = oracle.threads()
    om.close()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(rate, 4), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / rate, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16" if info["kind"] == "f16" else "int4 (f32 math)",
        "data": "synthetic",
        "config": bench_config(cfg_n, prompt_len, steps, world, s.weights.nbytes),
        "cpu_baseline": {"value": round(rate, 4), "unit": "tok/s", "cores": cores, "cpu_model": cpu_model(),
                         "kind": "port",
                         "sample": f"{steps} greedy decode steps from position {prompt_len} after the bench's "
                                   f"{prompt_len}-token prompt (CPU restatement of the reference WGSL decoder, "
                                   f"all host threads; prompt through its batched CPU path in {prefill_s:.1f} s, "
                                   f"untimed)"},
        "e2e": {"value": round(rate, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_gemv_family(model, torch, reps: int = 3):
    """Live CUDA-event timing of the SwiGLU gate_up GEMV of every layer (the dominant kernel).
    The stream is first held by a spin kernel so that all launches and events are queued before
    the GPU reaches them: the events then bracket device execution, not host launch overhead.
    Rotating over the 24 layers' matrices (1.2 GB) keeps every launch reading from HBM."""
    import qne
    stream = torch.cuda.current_stream()
    H, I = model.hidden, model.intermediate
    h = torch.randn(H, device="cuda", dtype=torch.float32)
    act = torch.empty(I, device="cuda", dtype=torch.float32)
    mats = [model.matrix(f"layer{i}.gate_up") for i in range(model.layers)]
    norms = [model.tensor_ptr(f"layer{i}.post_norm") for i in range(model.layers)]
    for m, g in zip(mats, norms):  # warm-up
        qne.rmsnorm_gemv(m, h, g, act, "swiglu", stream=stream.cuda_stream)
    torch.cuda.synchronize()
    events = [torch.cuda.Event(enable_timing=True) for _ in range(reps * len(mats) + 1)]
    torch.cuda._sleep(100_000_000)
    events[0].record(stream)
    k = 1
    for _ in range(reps):
        for m, g in zip(mats, norms):
            qne.rmsnorm_gemv(m, h, g, act, "swiglu", stream=stream.cuda_stream)
            events[k].record(stream)
            k += 1
    torch.cuda.synchronize()
    durs = [events[i].elapsed_time(events[i + 1]) for i in range(len(events) - 1)]
    mean_ms = float(np.mean(durs))
    # bytes per weight: f16; block-32 int4 (+ u32 scale pair per 64, u32 zero points per 256);
    # group-64 int4 (+ f16 scale and f16 zero point per 64)
    bpw = {0: 2.0, 1: 0.5 + 4 / 64 + 4 / 256, 2: 0.5 + 4 / 64}[int(mats[0].kind)]
    bytes_per_launch = int(2 * I * H * bpw) + H * 4 + I * 4
    return mean_ms, bytes_per_launch


def profile_step4(args):
    """Small fixed workload for ncu captures: a 2B-shaped decoder cut to 4 layers (32K vocab,
    seed 3), a 16-token prompt, then 8 greedy tokens on the device, through the launch path chosen
    by --path. Launch order: model set-up, 16 prompt tokens, 8 decode tokens."""
    import qne
    from qne import synth
    s = synth.build(2048, 6144, layers=4, vocab=32768, seed=3)
    m = qne.Model(s.index_json, s.weights, any_shape=True)
    if args.path != "auto":
        m.set_fused(args.path == "fused")
    m.prefill(synth.prompt_ids(16, 2, 32768))
    m.decode_async(8)
    m.sync()
    print(json.dumps({"micro": "step4", "fused": m.fused, "dispatches_per_token": m.dispatches_per_token(),
                      "last_token": list(m.last_token())}), flush=True)
    m.close()


def profile_prefill(args):
    """Fixed workload for the prefill launch list: the bench's config (2B f16 by default), its
    3968-token prompt through qne_prefill_chunk, the first 3904 tokens untimed, then the last
    64-token chunk (positions 3904..3967, the longest attention context) plus the LM head inside
    the NVTX range "last_chunk", timed with CUDA events."""
    import torch
    import qne
    from qne import synth
    torch.cuda.set_device(0)
    cfg_info = synth.baseline_config(args.config)
    s = synth.build_config(args.config)
    m = qne.Model(s.index_json, s.weights)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    m.set_stream(stream.cuda_stream)
    n = cfg_info["prompt"]
    prompt = synth.prompt_ids(n, 1)
    c = qne.PREFILL_CHUNK_TOKENS
    m.prefill_chunk(prompt[: n - c], 0, False)
    m.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("last_chunk")
    e0.record(stream)
    m.prefill_chunk(prompt[n - c:], n - c, True)
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(json.dumps({"micro": "prefill", "config": args.config, "batched": m.prefill_batched_supported,
                      "chunk_positions": [n - c, n - 1], "chunk_ms": round(e0.elapsed_time(e1), 3),
                      "last_token": list(m.last_token())}), flush=True)
    m.close()


def micro(args):
    """benchmark config 5: per-kernel microbench (seed 4). Each kernel is timed over enough distinct
    copies of its inputs that every launch reads HBM (> 126 MB L2 per rotation); launches are queued
    behind a spin kernel so CUDA events measure device time. One JSON line per case."""
    import torch
    import qne
    torch.cuda.set_device(0)
    peak, peak_kind = peaks()
    rng = np.random.default_rng(4)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sel = set(args.micro.split(","))
    out = []

    def timed(launch, copies, reps):
        for i in range(copies):
            launch(i)
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda._sleep(50_000_000)
        ev[0].record(stream)
        for r in range(reps):
            for i in range(copies):
                launch(i)
        ev[1].record(stream)
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]) * 1e3 / (reps * copies)  # us per launch

    keep = []
    if sel & {"all", "gemv"}:
        for kind in ("f16", "q4g64"):
            for (K, N) in ((2048, 6144), (6144, 2048), (2048, 4096), (1024, 248320)):
                el = N * K
                nbytes = el * 2 if kind == "f16" else el // 2 + el // 16
                copies = max(1, min(16, int(2.5e8 // nbytes) + 1))
                mats = []
                for c in range(copies):
                    if kind == "f16":
                        w = torch.from_numpy(rng.standard_normal(el, dtype=np.float32).astype(np.float16)).cuda()
                        mats.append(qne.matrix("f16", N, K, w))
                        keep.append(w)
                    else:
                        w = torch.randint(-2**31, 2**31 - 1, (el // 8,), dtype=torch.int32, device="cuda")
                        sc = (torch.rand(el // 64, device="cuda") * 0.01).half()
                        zp = torch.full((el // 64,), 8.0, device="cuda").half()
                        mats.append(qne.matrix("q4g64", N, K, w, sc, zp))
                        keep.extend([w, sc, zp])
                x = torch.randn(K, device="cuda")
                y = torch.empty(N, device="cuda")
                variants = [(0, 2), (1, 1), (2, 2)] if kind == "f16" else [(0, 2), (1, 1), (4, 2)]
                for var, cps in variants:
                    us = timed(lambda i: qne.gemv_ex(mats[i], x, y, "store", var, cps, stream=stream.cuda_stream),
                               copies, max(2, 64 // copies))
                    gbs = nbytes / (us * 1e-6) / 1e9
                    out.append({"micro": "gemv", "kind": kind, "K": K, "N": N, "variant": var, "ctas_per_sm": cps,
                                "us": round(us, 2), "GBs": round(gbs, 1), "frac_of_" + peak_kind: round(gbs / peak, 4),
                                "bytes": nbytes})
                keep.clear()
    if sel & {"all", "gemm", "gemm1"}:
        # the batched GEMM on the decoder's shapes (2B and 0.8B), B = 32 and 8 activation rows;
        # gemm1: only the 0.8B gate_up (SwiGLU) GEMM at B = 32 on the tensor-core kernel (ncu)
        shapes = ((8224, 2048, "store"), (2048, 2048, "accumulate"), (12288, 2048, "swiglu"),
                  (2048, 6144, "accumulate"), (8224, 1024, "store"), (1024, 2048, "accumulate"),
                  (7168, 1024, "swiglu"), (1024, 3584, "accumulate"), (248320, 1024, "store"))
        one = not sel & {"all", "gemm"}
        for (rows, K, epi) in (((7168, 1024, "swiglu"),) if one else shapes):
            nbytes = rows * K * 2
            copies = max(1, min(16, int(2.5e8 // nbytes) + 1))
            mats = []
            for c in range(copies):
                w = torch.from_numpy((rng.standard_normal(rows * K, dtype=np.float32) * 0.05).astype(np.float16)).cuda()
                mats.append(qne.matrix("f16", rows, K, w))
                keep.append(w)
            out_rows = rows // 2 if epi == "swiglu" else rows
            for B in ((32,) if one else (32, 8)):
                x = torch.randn(B, K, device="cuda")
                y = torch.zeros(B, out_rows, device="cuda")
                for impl in (("tcgen05",) if one else ("tcgen05", "mma_sync")):
                    us = timed(lambda i: qne.gemm(mats[i], x, B, y, epi, stream=stream.cuda_stream, impl=impl),
                               copies, max(2, 64 // copies))
                    gbs = nbytes / (us * 1e-6) / 1e9
                    out.append({"micro": "gemm", "impl": impl, "rows": rows, "K": K, "epilogue": epi, "batch": B,
                                "us": round(us, 2), "GBs": round(gbs, 1), "frac_of_" + peak_kind: round(gbs / peak, 4),
                                "bytes": nbytes, "note": "includes qne_gemm's f32 -> hi/lo staging kernel"})
            keep.clear()
    if sel & {"all", "gdn"}:
        for B in (1, 32):
            copies = max(2, int(2.5e8 // (B * 16 * 128 * 128 * 4)) + 1)
            proj = torch.randn(B, 8224, device="cuda")
            conv_w = torch.rand(6144 * 4, device="cuda") - 0.5
            prm = torch.cat([torch.zeros(16), torch.full((16,), -0.5), torch.ones(128)]).cuda()
            states = [torch.randn(B, 16, 128, 128, device="cuda") * 0.1 for _ in range(copies)]
            rings = [torch.zeros(B, 4, 6144, device="cuda") for _ in range(copies)]
            ctr = torch.full((B,), 5, dtype=torch.int32, device="cuda")
            o = torch.empty(B, 2048, device="cuda")
            us = timed(lambda i: qne.gdn_step(proj, rings[i], conv_w, states[i], prm, ctr, o, B,
                                              stream=stream.cuda_stream), copies, 4)
            nbytes = B * 2 * 16 * 128 * 128 * 4
            gbs = nbytes / (us * 1e-6) / 1e9
            out.append({"micro": "gdn", "batch": B, "us": round(us, 2), "GBs": round(gbs, 1),
                        "frac_of_" + peak_kind: round(gbs / peak, 4), "bytes": nbytes,
                        "note": "gdn_step + gated norm (2 launches)"})
    if sel & {"all", "attn"}:
        for B in (1, 32):
            for ctx in (512, 2048, 4096):
                pool_pages = B * 256
                per = pool_pages * 16384 * 2
                copies = max(1, min(24, int(3e8 // (B * ctx * 2048)) + 1))
                pools = [torch.randn(pool_pages * 16384, device="cuda").half() for _ in range(copies)]
                table = torch.randperm(pool_pages, device="cuda", dtype=torch.int64).to(torch.int32)
                proj = torch.randn(B, 5120, device="cuda")
                norms = torch.ones(512, device="cuda")
                pos = torch.full((B,), ctx - 1, dtype=torch.int32, device="cuda")
                o = torch.empty(B, 2048, device="cuda")
                nbytes_s = qne.attention_scratch_bytes(B)
                scratch = torch.zeros(nbytes_s, dtype=torch.uint8, device="cuda")
                us = timed(lambda i: qne.attention_step(proj, norms, 1e7, pools[i], pool_pages, table, pos, o, B,
                                                        scratch, nbytes_s, stream=stream.cuda_stream), copies,
                           max(2, 32 // copies))
                nbytes = B * ctx * 2048
                gbs = nbytes / (us * 1e-6) / 1e9
                out.append({"micro": "attention", "batch": B, "ctx": ctx, "us": round(us, 2), "GBs": round(gbs, 1),
                            "frac_of_" + peak_kind: round(gbs / peak, 4), "bytes": nbytes})
                del pools
    for line in out:
        print(json.dumps(line), flush=True)


def other_config_run(torch, qne, synth, cfg_n: int, rank: int, world: int, barrier, max_over_ranks, warmup: int):
    """benchmark configs 1 (0.8B f16, 128-token prompt, 128 greedy steps) and 3 (2B int4 group-64,
    1024-token prompt, 256 steps) on each rank's own replica, on the default launch path: the prompt
    through qne_prefill_chunk, `warmup` untimed steps, a restore, then the config's steps timed with
    CUDA events (max over ranks). Returns the sub-object of the JSON line (rank 0) or None."""
    info = synth.baseline_config(cfg_n)
    s = synth.build_config(cfg_n)
    model = qne.Model(s.index_json, s.weights, device=torch.cuda.current_device())
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    model.set_stream(stream.cuda_stream)
    steps, prompt_len = info["steps"], info["prompt"]
    prompt = synth.prompt_ids(prompt_len, rank_seed(cfg_n, rank))
    model.prefill_chunk(prompt, 0, True)  # records the chunk graphs
    # the prompt itself, timed (batched chunks; for int4 the tensor-core GEMMs widen the nibbles)
    model.reset()
    model.sync()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    model.prefill_chunk(prompt, 0, True)
    p1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(p0.elapsed_time(p1))
    model.snapshot()
    model.sync()
    if warmup:
        model.decode_async(warmup)
        model.sync()
    model.restore()
    model.sync()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(20_000_000)
    e0.record(stream)
    model.decode_async(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1))
    kv_bytes = 2048 * (model.layers // 4) * (prompt_len + steps / 2)
    state_bytes = (model.layers - model.layers // 4) * (2 * 16 * 128 * 128 * 4 + 2 * 4 * 6144 * 4)
    tok_bytes = model.weight_bytes + kv_bytes + state_bytes + model.vocab * 4
    path = model.path
    model.close()
    if rank != 0:
        return None
    peak, kind = peaks()
    tps = aggregate_rate(world, steps, ms)
    gbs = tok_bytes / (ms / steps * 1e-3) / 1e9
    size_name = {"0.8b": "0.8B", "2b": "2B"}[info["size"]]
    return {"workload": f"config {cfg_n}: Qwen3.5-{size_name}-shaped {info['kind']} hybrid decoder (synthetic, seed "
                        f"{info['seed']}), B=1 per GPU, {prompt_len}-token prompt, {steps} greedy decode steps",
            "value": round(tps, 2), "unit": "tok/s", "n_gpus": world, "ms_per_step": round(ms / steps, 4),
            "launch_path": path, "bytes_per_token": int(tok_bytes),
            "step_roofline": {"achieved_gbs": round(gbs, 1), "peak": peak, "frac": round(gbs / peak, 4),
                              "peak_source": kind},
            "prefill": {"tokens": prompt_len, "ms": round(prefill_ms, 2),
                        "tok_per_s": round(world * prompt_len / (prefill_ms * 1e-3), 1)}}


def batched_run(torch, qne, synth, rank: int, world: int, barrier, max_over_ranks, warmup: int,
                steps: int = 64, batch: int = 32):
    """benchmark config 4: Qwen3.5-0.8B-shaped f16 (seed 3), `batch` independent sequences per GPU
    with context lengths uniform in [256, 4032] (so 64 steps stay within 4096), randomly permuted
    16-token page tables, synthetic history (KV pages, GDN states) written on the device, then
    `steps` greedy steps. Returns a dict for the JSON line (rank 0) or None."""
    s = synth.build_config(4)
    model = qne.Model(s.index_json, s.weights, device=torch.cuda.current_device())
    # A dedicated stream for the engine and the events that time it (the default stream's handle
    # is 0, which the engine reads as "use the model's own stream").
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    model.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(rank_seed(3, rank))
    lens = rng.integers(256, 4096 - steps - warmup, batch, endpoint=True)
    bt = qne.Batch(model, batch)
    bt.set_page_table(rng.permutation(batch * 256).astype(np.uint32))
    for b in range(batch):
        bt.fill_synthetic(b, int(lens[b]), int(rng.integers(0, synth.VOCAB)), rank_seed(3, rank) + b)
    bt.sync()
    if warmup:
        bt.decode_async(warmup)
        bt.sync()
    launches0 = qne.kernel_launches()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(20_000_000)
    torch.cuda.nvtx.range_push("batched_steps")  # the launch-list captures select this range
    e0.record(stream)
    bt.decode_async(steps)
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1))
    launches = qne.kernel_launches() - launches0
    ctx_mean = float(lens.mean()) + warmup + steps / 2
    weights = model.weight_bytes
    per_seq = 18 * (2 * 16 * 128 * 128 * 4 + 4 * 6144 * 4 + 6144 * 4) + 6 * 2048 * ctx_mean + model.vocab * 4
    step_bytes = weights + batch * per_seq
    peak, kind = peaks()
    bt.close()
    model.close()
    if rank != 0:
        return None
    tps = aggregate_rate(world, batch * steps, ms)
    return {"workload": f"config 4: Qwen3.5-0.8B-shaped f16 (seed 3), {batch} sequences per GPU, contexts "
                        f"U[256,{4096 - steps - warmup}] (mean {lens.mean():.0f}), permuted 16-token pages, "
                        f"{steps} greedy steps",
            "value": round(tps, 1), "unit": "tok/s", "n_gpus": world, "ms_per_step": round(ms / steps, 4),
            "bytes_per_step": int(step_bytes),
            "step_roofline": {"achieved_gbs": round(step_bytes / (ms / steps * 1e-3) / 1e9, 1), "peak": peak,
                              "frac": round(step_bytes / (ms / steps * 1e-3) / 1e9 / peak, 4),
                              "peak_source": kind},
            "gpu_launches": int(launches)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt", type=int, default=None, help="context tokens before the timed steps "
                                                            "(default: the config's)")
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3],
                    help="B=1 workload: benchmark config 1 (0.8B f16), 2 (2B f16, the headline) or 3 (2B int4 g64)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--micro", default="", help="config-5 microbench: all | gemv,gdn,attn; "
                                                     "step4 = the small decode workload of the ncu captures; gemm1 = one batched GEMM shape; "
                                                     "prefill = the last 64-token chunk of the bench prompt")
    ap.add_argument("--no-batched", action="store_true", help="skip the config-4 batched decode run")
    ap.add_argument("--no-other-configs", action="store_true", help="skip the config-1 and config-3 decode runs")
    ap.add_argument("--batched-only", action="store_true", help="run only the config-4 batched decode (profiling)")
    ap.add_argument("--batched-steps", type=int, default=64)
    ap.add_argument("--path", default="auto", choices=["auto", "fused", "split"],
                    help="B=1 launch path: one kernel per op (the default) or the fused layer kernels")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    if args.micro == "prefill":
        profile_prefill(args)
        return
    if args.micro == "step4":
        profile_step4(args)
        return
    if args.micro:
        micro(args)
        return
    if args.impl == "reference":
        reference_arm(args, world, rank)
        return

    import torch
    import torch.distributed as dist
    import qne
    from qne import synth

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    barrier, max_over_ranks = make_collectives(dist, world, "cuda")

    if args.batched_only:
        res = batched_run(torch, qne, synth, rank, world, barrier, max_over_ranks, args.warmup, args.batched_steps)
        if rank == 0:
            print(json.dumps({"batched": res}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    steps = args.steps
    cfg_n = args.config
    cfg_info = synth.baseline_config(cfg_n)
    size_name = {"0.8b": "0.8B", "2b": "2B"}[cfg_info["size"]]
    prompt_len = min(args.prompt if args.prompt is not None else cfg_info["prompt"], 4096 - steps)
    if prompt_len < 1 or steps < 1 or args.warmup < 0:
        raise SystemExit("need 1 <= --steps <= 4095")

    s = synth.build_config(cfg_n)
    model = qne.Model(s.index_json, s.weights, device=local)
    if args.path != "auto":
        model.set_fused(args.path == "fused")
    fused = model.fused
    # one dedicated stream for the engine and the CUDA events that time it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    model.set_stream(stream.cuda_stream)
    prompt = synth.prompt_ids(prompt_len, rank_seed(1, rank))
    # Batched prompt processing through the public API (qne_prefill_chunk: 64-token chunks; int4
    # matrices decoded to f16 before each GEMM), timed on the device. An untimed call first builds
    # the chunk runner and the launch graphs of the chunk sizes the prompt uses.
    model.reset()
    chunk = qne.PREFILL_CHUNK_TOKENS
    model.prefill_chunk(prompt[: min(prompt_len, chunk + prompt_len % chunk)], 0, True)
    model.reset()
    model.sync()
    torch.cuda.synchronize()
    barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    model.prefill_chunk(prompt, 0, True)
    p1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(p0.elapsed_time(p1))
    prefill_batched = model.prefill_batched_supported
    model.snapshot()
    model.sync()

    # warm-up, then restore the prefilled state so the timed steps cover positions prompt..prompt+steps
    if args.warmup:
        model.decode_async(min(args.warmup, 4095 - prompt_len))
        model.sync()
    model.restore()
    model.sync()
    torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    launches0 = qne.kernel_launches()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(20_000_000)  # hold the stream while the host queues the steps
    torch.cuda.nvtx.range_push("decode_steps")  # the launch-list captures select this range
    e0.record(stream)
    model.decode_async(steps)
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    launches = qne.kernel_launches() - launches0
    clk = clocks.stop()

    # e2e: host-logits loop through the public API (qne_step + pinned readback + host pick)
    model.restore()
    model.sync()
    tok, pos = model.last_token()
    out = torch.empty(model.vocab, dtype=torch.float32, pin_memory=True).numpy()
    for i in range(min(args.warmup, 2)):
        model.step(tok, pos, out)
    model.restore()
    model.sync()
    tok, pos = model.last_token()
    barrier()
    t0 = time.perf_counter()
    for i in range(steps):
        logits = model.step(tok, pos + i, out)
        tok = int(np.argmax(logits))
    e2e_s = max_over_ranks(time.perf_counter() - t0)

    # e2e: the same loop with the draw on the device (qne_step_sample, reference sampling defaults)
    sampler = qne.Sampler(model, temperature=0.6, top_k=20, top_p=0.95, seed=rank_seed(42, rank))
    model.restore()
    model.sync()
    tok, pos = model.last_token()
    for i in range(min(args.warmup, 2)):
        model.step_sample(sampler, tok, pos)
    model.restore()
    model.sync()
    tok, pos = model.last_token()
    barrier()
    t0 = time.perf_counter()
    for i in range(steps):
        tok = model.step_sample(sampler, tok, pos + i)
    e2e_sampled_s = max_over_ranks(time.perf_counter() - t0)
    sampler.close()

    # the other launch paths on the same state and steps (informational; `value` is the default path)
    paths = {model.path: round(aggregate_rate(world, steps, ms), 2)}
    for other_path in ("token", "layers"):
        if other_path == model.path:
            continue
        default_path = model.path
        try:
            model.set_path(other_path)
        except qne.QneError:
            continue
        model.restore()
        model.sync()
        barrier()
        torch.cuda.synchronize()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(20_000_000)
        q0.record(stream)
        model.decode_async(steps)
        q1.record(stream)
        torch.cuda.synchronize()
        paths[other_path] = round(aggregate_rate(world, steps, max_over_ranks(q0.elapsed_time(q1))), 2)
        model.set_path(default_path)

    # the dominant kernel, timed live
    gemv_ms, gemv_bytes = time_gemv_family(model, torch)
    peak, peak_kind = peaks()
    achieved = gemv_bytes / (gemv_ms * 1e-3) / 1e9

    dispatches = model.dispatches_per_token()
    model_weight_bytes = model.weight_bytes
    model.close()
    batched = None
    if not args.no_batched:
        batched = batched_run(torch, qne, synth, rank, world, barrier, max_over_ranks, args.warmup, args.batched_steps)
    others = {}
    if not args.no_other_configs and cfg_n == 2:
        for other in (1, 3):
            others[f"config{other}"] = other_config_run(torch, qne, synth, other, rank, world, barrier, max_over_ranks,
                                                        args.warmup)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_tokens = 48
        rate, cores = cpu_baseline_sample(s, cfg_n, prompt_len, cpu_tokens)
        cpu = {"value": round(rate, 4), "unit": "tok/s", "cores": cores, "cpu_model": cpu_model(), "kind": "port",
               "sample": f"{cpu_tokens} greedy decode steps of the same {size_name} {cfg_info['kind']} model from "
                         f"position {prompt_len} (KV cache and GDN states filled with seeded synthetic history), "
                         "CPU oracle (C++ restatement of the reference decoder, all host threads)"}

    if rank == 0:
        value = aggregate_rate(world, steps, ms)
        bytes_per_token = model.weight_bytes + 24 * 0  # weights; state/KV listed below
        kv_bytes = 6 * 2048 * (prompt_len + steps / 2)
        state_bytes = 18 * (2 * 16 * 128 * 128 * 4 + 2 * 4 * 6144 * 4)
        tok_bytes = bytes_per_token + kv_bytes + state_bytes + model.vocab * 4
        step_gbs = tok_bytes * value / world / 1e9
        if fused:
            # The fused layer kernel is the whole step: its algorithmic bytes per launch are the
            # token's bytes over the launches, its mean launch time the step time over them.
            roof = {"bound": "hbm", "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(step_gbs / peak, 4), "traffic": None,
                    "kernel": f"layer_kernel (fused decoder layer; {dispatches} launches per token, the last "
                              f"with the LM head)", "peak_source": peak_kind,
                    "mean_launch_us": round(ms / steps / dispatches * 1e3, 2),
                    "bytes_per_launch": int(tok_bytes / dispatches)}
        else:
            # traffic: DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one gate_up
            # launch from a full ncu capture (2B shape, cold L2): 50.38 MB read + 0.024 MB written.
            f16 = cfg_info["kind"] == "f16"
            shape = f"{2 * model.intermediate}x{model.hidden}"
            roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": 50_405_120 if cfg_n == 2 else None,
                    "kernel": (f"gemv_pipe_kernel<RMSNorm, SwiGLU> (gate_up, {shape})" if f16 else
                               f"int4 GEMV <{cfg_info['kind']}, RMSNorm, SwiGLU> (gate_up, {shape})"),
                    "peak_source": peak_kind, "mean_launch_us": round(gemv_ms * 1e3, 2)}
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(ms / steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": bench_config(cfg_n, prompt_len, steps, world, s.weights.nbytes),
            "e2e": {"value": round(aggregate_rate(world, steps, e2e_sampled_s * 1e3), 2), "unit": "tok/s",
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                    "loop": "qne_step_sample: decode step + device sampling (T 0.6, top_k 20, top_p 0.95)"},
            "e2e_host_logits": {"value": round(aggregate_rate(world, steps, e2e_s * 1e3), 2), "unit": "tok/s",
                                "h2d_bytes_per_step": 8, "d2h_bytes_per_step": model.vocab * 4,
                                "loop": "qne_step + logits to pinned host memory + host pick (the reference agent's)"},
            "roofline": roof,
            "step_roofline": {"bytes_per_token": int(tok_bytes), "achieved_gbs": round(tok_bytes * value / world / 1e9, 1),
                              "frac": round(tok_bytes * value / world / 1e9 / peak, 4)},
            "gpu_launches": int(launches),
            "dispatches_per_token": dispatches,
            "launch_paths_tok_s": paths,
            "clocks": clk,
            "cpu_baseline": cpu,
            "batched": batched,
            **others,
            "prefill": {"tokens": prompt_len, "ms": round(prefill_ms, 3),
                        "tok_per_s": round(aggregate_rate(world, prompt_len, prefill_ms), 1),
                        "path": (f"batched: {chunk}-token chunks, tensor-core GEMMs, chunked GDN scan"
                                 + ("" if cfg_info["kind"] == "f16" else ", int4 matrices decoded to f16 per GEMM")
                                 if prefill_batched else "one token per step"),
                        "weight_gbs": (round(model_weight_bytes * -(-prompt_len // chunk) / (prefill_ms * 1e-3) / 1e9, 1)
                                       if prefill_batched else None)},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
