#!/usr/bin/env python
"""Decode benchmark: Qwen3-1.7B-shaped Q4_0 batch-1 greedy decode.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl zero_b200|reference]

A step is one decode step (forward through 28 layers + LM-head argmax) for
one token; K steps are timed after a 16-token prompt prefill.  Prints one
JSON line on rank 0.

  value    tok/s of the K decode steps, device-timed with CUDA events around
           the CUDA-graph replays (weights resident in HBM; the token chain
           stays on the device).  Weights stream 1.12 GB per step, far above
           the 126 MB L2, so no flush is needed between steps.
  e2e      the same metric through the reference-facing C ABI per token
           (zgpu_forward_single_token + zgpu_lm_head_argmax), host token in,
           host token out, host wall clock.
  roofline the dominant kernel: the persistent step kernel's decode launch
           (algorithmic bytes = steps x (1.124 GB of weights + the KV rows
           read) over its CUDA-event duration) vs the measured HBM copy
           bandwidth; plus, at N = 1, the BASELINE config-1 GEMV sweep (four
           Q4_0 shapes, f32 and Q8_0 activations) as a secondary figure.
  cpu_baseline  the CPU oracle's AVX-512-order restatement of the reference
           decode on a persistent pinned pool over the physical host cores,
           on a bounded sample (rank 0, N=1 only).

With --gpus N > 1 (launched under torchrun) the one sequence is decoded
tensor parallel over the N GPUs (strong scaling): every rank holds 1/N of the
rows of each matmul and the stage outputs cross NVLink inside the persistent
step kernel; times are the max over ranks.

Other workloads (--workload), each printing the same kind of line:
  qwen3-8b          BASELINE config 2: cache filled to 4096 tokens, greedy
                    steps; tensor parallel over the torchrun ranks; with
                    --batch 16, sixteen sequences per step (zgpu_decode_batch,
                    one GPU)
  ds2               BASELINE config 3's model (MLA + MoE), one sequence;
                    expert parallel over the torchrun ranks; with --batch 32,
                    the config's 32 concurrent sequences per step
                    (zgpu_ds2_decode_batch)
  prefill           BASELINE config 4: a 2048-token prompt (--batch 8: eight)
  kquant            the GGUF-compat Q4_K / Q6_K GEMVs of one token at
                    Qwen3-1.7B shape, HBM GB/s
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s, Qwen3-1.7B-shape Q4_0 b=1; GEMV HBM GB/s vs ~8 TB/s peak"
PUBLISHED_TOK_S = 194.5      # README.md:29 of the reference (EPYC 9354P, AVX-512, CPU only)
PROMPT_LEN = 16
SEED = 0
# DRAM bytes (read + write) per decode step of the persistent step kernel,
# from one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum of a
# timed decode launch, divided by its steps), together with a digest of the
# kernel sources it was captured on.  When those sources change the figure is
# withheld (roofline.traffic null) until it is captured again.
NCU_TRAFFIC_PER_STEP = 1_125_072_896
NCU_TRAFFIC_SOURCES = ("step.cu", "step.h", "gemv_body.cuh", "attn_body.cuh", "common.cuh", "layout.h")
NCU_TRAFFIC_DIGEST = "3b67d4ac1785f3e7"


def kernel_sources_digest() -> str:
    import hashlib

    h = hashlib.sha256()
    for name in NCU_TRAFFIC_SOURCES:
        h.update((ROOT / "zero_b200" / "csrc" / name).read_bytes())
    return h.hexdigest()[:16]


def measured_traffic_per_step():
    """ncu's DRAM bytes per decode step, or None when the step kernel's
    sources differ from those it was captured on."""
    if NCU_TRAFFIC_PER_STEP and NCU_TRAFFIC_DIGEST and kernel_sources_digest() == NCU_TRAFFIC_DIGEST:
        return NCU_TRAFFIC_PER_STEP
    return None



def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="zero_b200", choices=["zero_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the per-token C-ABI loop")
    ap.add_argument("--no-roofline", action="store_true", help="skip the standalone GEMV sweep")
    ap.add_argument("--workload", default="qwen3", choices=["qwen3", "ds2", "prefill", "qwen3-8b", "kquant"],
                    help="qwen3: BASELINE config 0 (the headline); ds2: the config-3 DeepSeek2 "
                         "MLA+MoE model, one sequence, as a secondary line")
    ap.add_argument("--context", type=int, default=2048, help="ds2: tokens in the cache before decode")
    ap.add_argument("--batch", type=int, default=1, help="prefill: prompts per step (BASELINE config 4: 1 or 8); "
                    "qwen3-8b: sequences decoded together (BASELINE config 2: 1 or 16); "
                    "ds2: sequences decoded together (BASELINE config 3: 32, at most 32)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def physical_cores() -> int:
    try:
        out = subprocess.run(["lscpu", "-p=CORE,SOCKET"], capture_output=True, text=True).stdout
        cores = {tuple(l.split(",")) for l in out.splitlines() if l and not l.startswith("#")}
        if cores:
            return len(cores)
    except OSError:
        pass
    return os.cpu_count() or 1


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs", 6650.0), "bf16_tflops": d.get("bf16_tflops", 1590.0),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                parts = [s.strip() for s in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        except OSError:
            pass
        finally:
            if self.path:
                try:
                    os.unlink(self.path)
                except OSError:
                    pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [int(r[1]) for r in rows]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": int(statistics.median(sm)), "sm_max_mhz": int(rows[0][2]),
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3] not in ("[N/A]", "")),
                "reasons": sorted(reasons)}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


def host_read_gbs(threads: int, mb_per_thread: int = 64) -> float:
    """Read bandwidth of the host's memory with `threads` threads (numpy
    reductions release the GIL), GB/s: the ceiling of the CPU baseline, which
    streams 1.12 GB of weights per decode step."""
    from concurrent.futures import ThreadPoolExecutor

    n = mb_per_thread * (1 << 20) // 8
    bufs = [np.ones(n, np.float64) for _ in range(threads)]
    with ThreadPoolExecutor(threads) as ex:
        list(ex.map(np.sum, bufs))                      # touch
        best = 0.0
        for _ in range(3):
            t0 = time.perf_counter()
            list(ex.map(np.sum, bufs))
            best = max(best, threads * n * 8 / (time.perf_counter() - t0) / 1e9)
    return best


def cpu_decode(cfg, weights, prompt, steps: int, threads: int):
    """Time `steps` decode steps (forward + LM head) of the CPU oracle's AVX-512 path."""
    import oracle as O

    r = O.OracleRun(cfg, weights, PROMPT_LEN + steps + 2, order=O.ORDER_AVX512, threads=threads)
    for i, t in enumerate(prompt):
        r.forward(int(t), i)
    rc, tok, _ = r.lm_head()
    pos = len(prompt)
    t0 = time.perf_counter()
    for _ in range(steps):
        r.forward(tok, pos)
        rc, tok, _ = r.lm_head()
        pos += 1
    dt = time.perf_counter() - t0
    r.close()
    return steps / dt, dt


def cpu_decode_sample(cfg, weights, prompt, steps: int, threads: int):
    """The reference's decode loop on the CPU oracle (AVX-512 order) for a
    short prompt: tok/s of `steps` decode steps after it."""
    import oracle as O

    r = O.OracleRun(cfg, weights, len(prompt) + steps + 2, order=O.ORDER_AVX512, threads=threads)
    for i, t in enumerate(prompt):
        r.forward(int(t), i)
    rc, tok, _ = r.lm_head()
    pos = len(prompt)
    t0 = time.perf_counter()
    for _ in range(steps):
        r.forward(tok, pos)
        rc, tok, _ = r.lm_head()
        pos += 1
    dt = time.perf_counter() - t0
    r.close()
    return steps / dt, dt


def cpu_synth():
    """zero_b200/synth.py loaded by file path, not through the package (whose
    import loads libzgpu), generating through the oracle library's build of
    the same generator: the CPU arms load no GPU code and still get the
    seeded bytes the GPU arm uses."""
    import importlib.util

    import oracle as O

    name = "zero_b200_synth_cpu"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / "zero_b200" / "synth.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    mod.use_generator(O.LIB, "zo_")
    return mod


def synth_module(args):
    """The weight generator: the package's for the GPU arm, the oracle-backed
    copy for the reference arm."""
    if args.impl == "reference":
        return cpu_synth()
    from zero_b200 import synth

    return synth


def run_reference(args, rank):
    """The reference arm: the reference's CPU decode path (restated, AVX-512 order)
    on the host cores, same config and metric."""
    if rank != 0:
        return
    synth = cpu_synth()

    cfg = synth.QWEN3_1_7B
    weights = synth.qwen3_weights(cfg, seed=SEED, x4=False)
    prompt = synth.prompt_ids(cfg, PROMPT_LEN, seed=SEED)
    cores = physical_cores()
    cpu_decode(cfg, weights, prompt, max(1, min(args.warmup, 3)), cores)   # warm-up
    tok_s, dt = cpu_decode(cfg, weights, prompt, args.steps, cores)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * dt / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": round(tok_s / PUBLISHED_TOK_S, 4), "dtype": "f32",
        "data": "synthetic (seeded random-init .smodel v2 weights)",
        "config": {"workload": "qwen3-1.7b-shape q4_0 decode b=1 (BASELINE config 0)",
                   "prompt": PROMPT_LEN, "decode_steps": args.steps, "layers": cfg.n_layers,
                   "hidden": cfg.hidden, "ffn": cfg.ffn, "vocab": cfg.vocab_padded,
                   "parallelism": "cpu threads"},
        "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                         "weights_gbs": round(tok_s * cfg.weight_bytes_per_token() / 1e9, 2),
                         "host_read_gbs": round(host_read_gbs(cores), 2),
                         "sample": f"{args.steps} decode steps after a {PROMPT_LEN}-token prefill, "
                                   f"persistent pinned pool, fused dispatches"},
        "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


DS2_METRIC = "decode tok/s, DeepSeek-V2-Lite-shape MLA+MoE Q4_0, one sequence"


def ds2_cpu_sample(cfg, weights, context: int, steps: int):
    """The reference's own DeepSeek2 step on the host cores: the oracle's
    restatement of its AVX-512 kernel path (inference_avx512.rs:2141-2825:
    every cached latent re-expanded through kv_b twice per layer, matmuls on
    a persistent pinned pool, one participant per physical core), one
    sequence at `context` cached tokens.  The cache rows are seeded (the cost
    depends on the context, not on the values).  Returns (tok/s, seconds,
    threads) over `steps` forward + LM-head steps; the reference decodes
    concurrent sequences one forward at a time, so this is also its batch
    throughput."""
    import oracle as O

    r = O.OracleDs2Run(cfg, weights, context + steps + 1, order=O.ORDER_AVX512, threads=0)
    rng = np.random.default_rng(SEED)
    width = cfg.kv_lora_rank + cfg.rope_dim
    for layer in range(cfg.n_layers):
        r.set_cache_rows(layer, 0, rng.standard_normal((context, width), dtype=np.float32))
    tok = 1
    t0 = time.perf_counter()
    for s in range(steps):
        r.forward(tok, context + s)
        rc, nxt, _ = r.lm_head()
        tok = nxt if rc == 0 else 1
    dt = time.perf_counter() - t0
    threads = r.threads
    r.close()
    return steps / dt, dt, threads


def ds2_reference_line(args, rank, metric, config):
    """The reference arm of the DeepSeek2 lines: ds2_cpu_sample at the line's
    context, min(K, 2) timed steps after one untimed (each takes seconds)."""
    if rank != 0:
        return
    synth = cpu_synth()
    cfg = synth.DS2_V2_LITE
    weights = synth.ds2_weights(cfg, seed=SEED)
    ds2_cpu_sample(cfg, weights, args.context, 1)
    steps = max(1, min(args.steps, 2))
    tok_s, dt, threads = ds2_cpu_sample(cfg, weights, args.context, steps)
    sample = (f"{steps} decode step(s) of one sequence at context {args.context} (cache rows seeded), "
              f"the reference's AVX-512 kernel order restated, {threads} threads, {dt:.1f} s")
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(tok_s, 4), "unit": "tok/s", "n_gpus": 0,
        "steps": steps, "warmup": 1, "ms_per_step": round(1000 * dt / steps, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, same weights)",
        "config": config,
        "cpu_baseline": {"value": round(tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(tok_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_ds2(args, rank, world, local):
    """BASELINE config 3's model (27 layers, MLA kv_lora 512, 64 experts top-6 +
    2 shared, vocab 102400) decoding one sequence: the cache is filled to
    --context tokens by a seeded prompt, then K greedy steps are timed.  The
    config's batch of 32 sequences is --batch 32; under torchrun the experts
    are sharded over the ranks (expert parallelism)."""
    if args.impl == "reference":
        ds2_reference_line(args, rank, DS2_METRIC,
                           {"workload": "deepseek-v2-lite-shape mla+moe q4_0 decode, 1 sequence "
                                        "(BASELINE config 3 model)", "context": args.context,
                            "parallelism": "cpu threads"})
        return
    import torch

    import zero_b200 as zb
    synth = synth_module(args)

    cfg = synth.DS2_V2_LITE
    if world > 1:
        import datetime

        import torch.distributed as dist

        from zero_b200 import tp

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    weights = synth.ds2_weights(cfg, seed=SEED)
    prompt = synth.ds2_prompt_ids(cfg, args.context, seed=SEED)
    ctx = zb.Context(device=local)
    # N > 1: expert parallel, experts [r E/N, (r+1) E/N) on rank r (zgpu_ds2_create_ep)
    model = zb.Ds2Model(ctx, cfg, weights, rank=rank, world=world)
    if world > 1:
        tp.connect(model)
    max_tokens = args.context + args.steps + 2
    kv = model.new_kv(max_tokens)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    barrier()
    model.generate_greedy(kv, prompt[: min(len(prompt), 64)], args.warmup + 1)   # warm-up, graphs captured
    barrier()
    with ClockSampler(physical_gpu_index(local)) as clocks:
        toks, _ = model.generate_greedy(kv, prompt, args.steps + 1)
        barrier()
    perf = model.perf()
    dec_ms = float(perf["decode_ms"])
    if world > 1:
        t = torch.tensor([dec_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dec_ms = float(t.item())
    tok_s = args.steps / (dec_ms / 1000.0)
    # e2e: the per-token C ABI with host token in / token out, a few steps
    n_e2e = min(args.steps, 16)
    pos = args.context + args.steps + 1 - n_e2e - 1
    tok = int(toks[-1])
    t0 = time.perf_counter()
    for i in range(n_e2e):
        model.forward_single_token(kv, tok, pos + i)
        tok, _ = model.lm_head_argmax(want_logits=False)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_tok_s = n_e2e / e2e_s
    peaks = measured_peaks()
    step_w = cfg.weight_bytes_per_token()
    cache_b = sum(cfg.cache_bytes_per_token() * (args.context + i + 1) for i in range(args.steps))
    launch_bytes = args.steps * step_w + cache_b
    gbs = launch_bytes / (dec_ms / 1000.0) / 1e9
    # CPU baseline: the reference's AVX-512 step restated, one step at the
    # line's context (ds2_cpu_sample)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        c_tok_s, dt, threads = ds2_cpu_sample(cfg, weights, args.context, 1)
        cpu = {"value": round(c_tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"one decode step of one sequence at context {args.context} (cache rows seeded), "
                         f"the reference's AVX-512 kernel order restated, {threads} threads, {dt:.1f} s"}
    if rank == 0:
        line = {
            "metric": DS2_METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dec_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init, BASELINE config 3 shapes)",
            "config": {"workload": "deepseek-v2-lite-shape mla+moe q4_0 decode, 1 sequence (BASELINE config 3 model)",
                       "context": args.context, "decode_steps": args.steps, "layers": cfg.n_layers,
                       "experts": f"{cfg.n_experts} routed top-{cfg.top_k} + {cfg.n_shared} shared",
                       "q_lora_rank": cfg.q_lora_rank, "batch": 1,
                       "weight_bytes_per_step": step_w,
                       "l2": "inputs larger than L2 (1.5 GB of weights streamed per step)",
                       "parallelism": f"ep{world} (experts sharded; router, attention, shared experts "
                                      f"replicated)" if world > 1 else "single GPU",
                       "tokens_first": [int(v) for v in toks[:4]]},
            "roofline": {"bound": "hbm", "kernel": "per-op decode kernels (whole step, CUDA graph)",
                         "per": "GPU" if world == 1 else "step (all ranks' bytes over the slowest rank's time)",
                         "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                         "traffic": None, "algorithmic_bytes": launch_bytes,
                         "avg_launch_us": round(dec_ms * 1000 / max(perf["decode_launches"], 1), 2)},
            "e2e": {"value": round(e2e_tok_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 84,
                    "d2h_bytes_per_step": 12},
            "gpu_launches": int(perf["decode_launches"]),
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    kv.close()
    model.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


DS2_BATCH_METRIC = "decode tok/s, DeepSeek-V2-Lite-shape MLA+MoE Q4_0, 32 concurrent sequences, context 2048"


def run_ds2_batch(args, rank, world, local):
    """BASELINE config 3 at its serving shape: --batch sequences (32), each
    with its own MLA cache holding --context tokens, decoded together by
    zgpu_ds2_decode_batch; with N > 1 ranks the experts are sharded (expert
    parallel) and every rank runs the same batch.  One cache is filled by a
    seeded prompt and copied on the device to the others
    (zgpu_mla_kv_copy); each sequence then continues from its own seeded
    token.  A step is one batched greedy step of every sequence."""
    if args.impl == "reference":
        ds2_reference_line(args, rank, DS2_BATCH_METRIC,
                           {"workload": f"deepseek-v2-lite-shape mla+moe q4_0 decode, {args.batch} sequences "
                                        f"(BASELINE config 3)", "context": args.context, "batch": args.batch,
                            "parallelism": "cpu threads (the reference decodes the sequences one forward "
                                           "at a time)"})
        return
    import torch

    import zero_b200 as zb
    synth = synth_module(args)

    cfg = synth.DS2_V2_LITE
    n_seq = args.batch
    if world > 1:
        import datetime

        import torch.distributed as dist

        from zero_b200 import tp

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    weights = synth.ds2_weights(cfg, seed=SEED)
    prompt = synth.ds2_prompt_ids(cfg, args.context, seed=SEED)
    ctx = zb.Context(device=local)
    model = zb.Ds2Model(ctx, cfg, weights, rank=rank, world=world)
    if world > 1:
        tp.connect(model)
    max_tokens = args.context + args.warmup + args.steps + 2
    fill = model.new_kv(max_tokens)
    model.generate_greedy(fill, prompt, 1)        # context tokens into the first cache
    kvs = [fill] + [model.new_kv(max_tokens) for _ in range(n_seq - 1)]
    for kv in kvs[1:]:
        kv.copy_from(fill, args.context)
    tokens = synth.ds2_prompt_ids(cfg, n_seq, seed=SEED + 1)
    pos = np.full(n_seq, args.context, np.uint32)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    barrier()
    for _ in range(args.warmup):
        tokens, _ = model.decode_batch(kvs, tokens, pos, want_logits=False)
        pos = pos + 1
    barrier()
    dev_ms = 0.0
    launches = 0
    first = []
    with ClockSampler(physical_gpu_index(local)) as clocks:
        t0 = time.perf_counter()
        for i in range(args.steps):
            tokens, _ = model.decode_batch(kvs, tokens, pos, want_logits=False)
            pos = pos + 1
            p = model.perf()
            dev_ms += float(p["decode_ms"])
            launches += int(p["decode_launches"])
            if i == 0:
                first = [int(v) for v in tokens[:4]]
        barrier()
        wall_s = time.perf_counter() - t0
    ids, _ = model.batch_expert_ids(n_seq)
    if world > 1:
        t = torch.tensor([dev_ms, wall_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, wall_s = float(t[0].item()), float(t[1].item())
    tok_s = n_seq * args.steps / (dev_ms / 1000.0)
    e2e_tok_s = n_seq * args.steps / wall_s
    # algorithmic bytes of one batched step: every non-expert weight once,
    # the shared experts and the distinct routed experts the batch selected
    # (counted on the last step's ids) once each, n_seq embedding rows, and
    # every sequence's latent cache rows
    q4 = 18 / 32
    H = cfg.hidden
    expert_b = 3 * cfg.expert_ffn * H * q4
    n_moe = cfg.n_layers - cfg.n_dense
    distinct = [len(np.unique(ids[layer])) for layer in range(cfg.n_dense, cfg.n_layers)]
    single_w = cfg.weight_bytes_per_token()
    embd_row = H * (34 / 32 if cfg.embd_quant == "q8_0" else q4)
    step_w = single_w - n_moe * cfg.top_k * expert_b + sum(distinct) * expert_b + (n_seq - 1) * embd_row
    ctx_mean = args.context + args.warmup + (args.steps + 1) / 2
    cache_b = n_seq * cfg.cache_bytes_per_token() * ctx_mean
    step_bytes = step_w + cache_b
    gbs = step_bytes * args.steps / (dev_ms / 1000.0) / 1e9
    peaks = measured_peaks()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        c_tok_s, dt, threads = ds2_cpu_sample(cfg, weights, args.context, 1)
        cpu = {"value": round(c_tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"one decode step of one sequence at context {args.context} (cache rows seeded), "
                         f"the reference's AVX-512 kernel order restated, {threads} threads, {dt:.1f} s "
                         f"(the reference decodes concurrent sequences one forward at a time)"}
    if rank == 0:
        line = {
            "metric": DS2_BATCH_METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init, BASELINE config 3 shapes)",
            "config": {"workload": f"deepseek-v2-lite-shape mla+moe q4_0 decode, {n_seq} sequences "
                                   f"(BASELINE config 3)",
                       "context": args.context, "batch": n_seq, "decode_steps": args.steps,
                       "layers": cfg.n_layers,
                       "experts": f"{cfg.n_experts} routed top-{cfg.top_k} + {cfg.n_shared} shared",
                       "distinct_experts_per_moe_layer": round(sum(distinct) / max(len(distinct), 1), 1),
                       "q_lora_rank": cfg.q_lora_rank,
                       "l2": "inputs larger than L2 (weights and 32 latent caches, several GB per step)",
                       "parallelism": f"ep{world} (experts sharded; router, attention, shared experts "
                                      f"replicated)" if world > 1 else "single GPU",
                       "tokens_first": first},
            "roofline": {"bound": "hbm", "kernel": "per-op decode kernels widened over the batch (CUDA graph)",
                         "per": "GPU" if world == 1 else "step (all ranks' bytes over the slowest rank's time)",
                         "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                         "traffic": None, "algorithmic_bytes_per_step": int(step_bytes),
                         "cache_bytes_per_step": int(cache_b)},
            "e2e": {"value": round(e2e_tok_s, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": n_seq * (4 + 4 + 8), "d2h_bytes_per_step": n_seq * 4 + 4},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    for kv in kvs:
        kv.close()
    model.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


TP_METRIC = "decode tok/s, Qwen3-8B-shape Q4_0 b=1, context 4096, tensor parallel over N GPUs"
TP_CONTEXT = 4096


def run_qwen3_tp(args, rank, world, local):
    """BASELINE config 2 at batch 1: the Qwen3-8B shape, the cache filled to
    4096 seeded tokens, then K greedy steps, tensor parallel over the N GPUs
    of the launch (one rank per GPU; at N = 1 the plain one-GPU model).  The
    stage outputs cross NVLink inside the persistent step kernel (peer stores
    of tagged words), so a step is one kernel per GPU.  Strong scaling: one
    sequence, its weights split N ways."""
    synth = synth_module(args)

    cfg = synth.QWEN3_8B
    n_cpu_prompt, n_cpu_gen = 4, 4
    if args.impl == "reference":
        if rank == 0:
            weights = synth.qwen3_weights(cfg, seed=SEED, x4=False)
            prompt = synth.prompt_ids(cfg, n_cpu_prompt, seed=SEED)
            cores = physical_cores()
            tok_s, dt = cpu_decode_sample(cfg, weights, prompt, n_cpu_gen, cores)
            print(json.dumps({
                "impl": "reference", "metric": TP_METRIC, "value": round(tok_s, 3), "unit": "tok/s",
                "n_gpus": args.gpus, "steps": n_cpu_gen, "warmup": 0, "ms_per_step": round(1000 * dt / n_cpu_gen, 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-init .smodel v2 weights, BASELINE config 2 shapes)",
                "config": {"workload": "qwen3-8b-shape q4_0 decode b=1 (BASELINE config 2)",
                           "parallelism": "cpu threads"},
                "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                                 "sample": f"{n_cpu_gen} decode steps after a {n_cpu_prompt}-token prompt "
                                           f"(context <= {n_cpu_prompt + n_cpu_gen}, not 4096)"},
                "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}), flush=True)
        return
    import datetime

    import torch
    import torch.distributed as dist

    import zero_b200 as zb
    from zero_b200 import tp

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    weights = synth.qwen3_weights(cfg, seed=SEED)
    prompt = synth.prompt_ids(cfg, TP_CONTEXT, seed=SEED)
    ctx = zb.Context(device=local)
    model = zb.Qwen3Model(ctx, cfg, weights, rank=rank, world=world)
    del weights
    if world > 1:
        tp.connect(model)
    max_tokens = TP_CONTEXT + args.steps + 2
    kv = model.new_kv(max_tokens)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    model.generate_greedy(kv, prompt[:16], args.warmup + 1)      # warm-up
    barrier()
    with ClockSampler(physical_gpu_index(local)) as clocks:
        t0 = time.perf_counter()
        toks, _ = model.generate_greedy(kv, prompt, args.steps + 1)
        wall = time.perf_counter() - t0
        barrier()
    perf = model.perf()
    dec_ms = max_over_ranks(float(perf["decode_ms"]))
    fill_ms = max_over_ranks(float(perf["prefill_ms"]))
    wall = max_over_ranks(wall)
    tok_s = args.steps / (dec_ms / 1000.0)
    peaks = measured_peaks()
    # per GPU and step: its weight slice (1/N of the 4.57 GB; the embedding row
    # and norms are whole on every rank) and its kv heads' rows of the cache
    step_bytes = cfg.weight_bytes_per_token() / world
    kv_row_bytes = 2 * (cfg.n_kv_heads // world) * cfg.head_dim * 4 * cfg.n_layers
    kv_bytes = sum(kv_row_bytes * (TP_CONTEXT + i + 1) for i in range(args.steps))
    launch_bytes = args.steps * step_bytes + kv_bytes
    gbs = launch_bytes / (dec_ms / 1000.0) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        del model, kv
        w_plain = synth.qwen3_weights(cfg, seed=SEED, x4=False)
        c_tok_s, c_dt = cpu_decode_sample(cfg, w_plain, prompt[:n_cpu_prompt], n_cpu_gen, physical_cores())
        cpu = {"value": round(c_tok_s, 3), "unit": "tok/s", "cores": physical_cores(), "kind": "port",
               "sample": f"{n_cpu_gen} decode steps after a {n_cpu_prompt}-token prompt (context <= "
                         f"{n_cpu_prompt + n_cpu_gen}, not {TP_CONTEXT}), AVX-512-order restatement, {c_dt:.1f} s"}
    if rank == 0:
        line = {
            "metric": TP_METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dec_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init .smodel v2 weights, BASELINE config 2 shapes)",
            "config": {"workload": "qwen3-8b-shape q4_0 decode b=1 (BASELINE config 2)",
                       "context": TP_CONTEXT, "decode_steps": args.steps, "layers": cfg.n_layers,
                       "hidden": cfg.hidden, "ffn": cfg.ffn, "batch": 1,
                       "parallelism": f"tp{world}" if world > 1 else "single GPU",
                       "context_fill_ms": round(fill_ms, 1),
                       "l2": "inputs larger than L2 (4.57 GB of weights / N per GPU per step)",
                       "tokens_first": [int(v) for v in toks[:4]]},
            "roofline": {"bound": "hbm", "kernel": "persistent step kernel (all decode steps, one launch per GPU)",
                         "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                         "per": "GPU", "traffic": None, "algorithmic_bytes": int(launch_bytes)},
            "e2e": {"value": round((TP_CONTEXT + args.steps) / wall, 2), "unit": "tok/s",
                    "scope": f"zgpu_generate_greedy wall clock: {TP_CONTEXT}-token context fill + "
                             f"{args.steps} greedy steps, tokens processed per second",
                    "h2d_bytes_per_step": 4 * TP_CONTEXT // (TP_CONTEXT + args.steps),
                    "d2h_bytes_per_step": 4},
            "gpu_launches": int(perf["decode_launches"]),
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


BATCH_METRIC = "decode tok/s (all sequences), Qwen3-8B-shape Q4_0, batch B, context 4096"


def run_qwen3_batch(args, rank, world, local):
    """BASELINE config 2 at batch B (16): B sequences, each cache filled to
    4096 seeded tokens (zgpu_prefill_batch, four sequences at a time), then K
    greedy steps of all B sequences at once (zgpu_decode_batch: projections
    and LM head on the exact tensor-core matvec, which multiplies the f32
    activations' integer digits by int8 weight tiles and reproduces the
    single-token GEMV bit for bit; the decode attention with a sequence grid
    dimension).  One GPU; value = B x K tokens over the device time of the K
    steps."""
    synth = synth_module(args)

    cfg = synth.QWEN3_8B
    B = args.batch
    n_cpu_prompt, n_cpu_gen = 4, 4
    if world > 1:
        raise SystemExit("batched decode runs on one GPU")
    if args.impl == "reference":
        weights = synth.qwen3_weights(cfg, seed=SEED, x4=False)
        prompt = synth.prompt_ids(cfg, n_cpu_prompt, seed=SEED)
        cores = physical_cores()
        tok_s, dt = cpu_decode_sample(cfg, weights, prompt, n_cpu_gen, cores)
        print(json.dumps({
            "impl": "reference", "metric": BATCH_METRIC, "value": round(tok_s, 3), "unit": "tok/s",
            "n_gpus": args.gpus, "steps": n_cpu_gen, "warmup": 0, "ms_per_step": round(1000 * dt / n_cpu_gen, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init .smodel v2 weights, BASELINE config 2 shapes)",
            "config": {"workload": f"qwen3-8b-shape q4_0 decode b={B} (BASELINE config 2)",
                       "parallelism": "cpu threads"},
            "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"one sequence: {n_cpu_gen} decode steps after a {n_cpu_prompt}-token "
                                       f"prompt (the reference decodes the sequences of a batch one after "
                                       f"another, so its batch rate is its single-sequence rate)"},
            "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    import torch

    import zero_b200 as zb

    torch.cuda.set_device(local)
    weights = synth.qwen3_weights(cfg, seed=SEED)
    ctx = zb.Context(device=local)
    model = zb.Qwen3Model(ctx, cfg, weights)
    del weights
    max_tokens = TP_CONTEXT + args.warmup + args.steps + 2
    kvs = [model.new_kv(max_tokens) for _ in range(B)]
    prompts = np.stack([synth.prompt_ids(cfg, TP_CONTEXT, seed=SEED + i) for i in range(B)])
    toks = np.empty(B, np.uint32)
    t0 = time.perf_counter()
    for g in range(0, B, 4):
        toks[g:g + 4] = model.prefill_batch(kvs[g:g + 4], prompts[g:g + 4], want_logits=False)[0]
    fill_s = time.perf_counter() - t0
    pos = TP_CONTEXT
    for _ in range(args.warmup):
        toks, _ = model.decode_batch(kvs, toks, np.full(B, pos), want_logits=False)
        pos += 1
    torch.cuda.synchronize()
    dev_ms, gemm_ms, attn_ms, wall = [], [], [], []
    kv_bytes = 0
    kv_row = 2 * cfg.n_kv_heads * cfg.head_dim * 4          # K and V of one token, one layer
    first = []
    with ClockSampler(physical_gpu_index(local)) as clocks:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            toks, _ = model.decode_batch(kvs, toks, np.full(B, pos), want_logits=False)
            wall.append(time.perf_counter() - t0)
            p = model.perf()
            dev_ms.append(p["decode_ms"])
            gemm_ms.append(p["batch_gemm_ms"])
            attn_ms.append(p["batch_attn_ms"])
            kv_bytes += B * (pos + 1) * kv_row * cfg.n_layers
            pos += 1
            if len(first) < 4:
                first.append(int(toks[0]))
    launches = int(model.perf()["decode_launches"])
    K = args.steps
    tok_s = B * K / (sum(dev_ms) / 1000.0)
    peaks = measured_peaks()
    attn_launch_bytes = kv_bytes / (K * cfg.n_layers)
    attn_us = 1000.0 * sum(attn_ms) / (K * cfg.n_layers)
    attn_gbs = attn_launch_bytes / (attn_us / 1e6) / 1e9
    tile_bytes = (cfg.n_layers * ((cfg.q_dim + 2 * cfg.kv_dim) * cfg.hidden + cfg.hidden * cfg.q_dim
                                  + 2 * cfg.ffn * cfg.hidden + cfg.hidden * cfg.ffn)
                  + cfg.vocab_padded * cfg.hidden) * 5 // 4
    # the matvec's weight tiles: per 128 rows x 32 columns, 4 KB of int8, the
    # rows' f32 block scales and int32 row sums (5 KB); every Qwen3-8B row
    # count is a multiple of 128
    gemm_gbs = tile_bytes / (statistics.mean(gemm_ms) / 1000.0) / 1e9
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        for kv in kvs:
            kv.close()
        model.close()
        w_plain = synth.qwen3_weights(cfg, seed=SEED, x4=False)
        c_tok_s, c_dt = cpu_decode_sample(cfg, w_plain, prompts[0][:n_cpu_prompt], n_cpu_gen, physical_cores())
        cpu = {"value": round(c_tok_s, 3), "unit": "tok/s", "cores": physical_cores(), "kind": "port",
               "sample": f"one sequence, {n_cpu_gen} decode steps after a {n_cpu_prompt}-token prompt (context <= "
                         f"{n_cpu_prompt + n_cpu_gen}, not {TP_CONTEXT}), AVX-512-order restatement, {c_dt:.1f} s; "
                         f"the reference decodes a batch's sequences one after another"}
    print(json.dumps({
        "metric": BATCH_METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": 1, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(statistics.mean(dev_ms), 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 (projections: exact int8 digit x int8 weight -> int32 products on tcgen05)",
        "data": "synthetic (seeded random-init .smodel v2 weights, BASELINE config 2 shapes)",
        "config": {"workload": f"qwen3-8b-shape q4_0 decode b={B} (BASELINE config 2)", "batch": B,
                   "context": TP_CONTEXT, "decode_steps": K, "layers": cfg.n_layers,
                   "parallelism": "single GPU", "context_fill_s": round(fill_s, 1),
                   "gemm_ms_per_step": round(statistics.mean(gemm_ms), 4),
                   "attention_ms_per_step": round(statistics.mean(attn_ms), 4),
                   "gemm_tile_gbs": round(gemm_gbs, 1),
                   "l2": f"inputs larger than L2 ({tile_bytes / 1e9:.1f} GB of weight tiles and "
                         f"{B * TP_CONTEXT * cfg.n_layers * 2 * cfg.kv_dim * 4 / 1e9:.0f} GB of KV rows per step)",
                   "tokens_first_seq0": first},
        "roofline": {"bound": "hbm", "kernel": "attn_decode_batch_kernel (one layer, all sequences)",
                     "achieved": round(attn_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(attn_gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "traffic": None, "algorithmic_bytes": int(attn_launch_bytes),
                     "avg_launch_us": round(attn_us, 2)},
        "e2e": {"value": round(B * K / sum(wall), 1), "unit": "tok/s",
                "scope": "zgpu_decode_batch per step with host tokens in and out, host wall clock",
                "h2d_bytes_per_step": 4 * B + 24 * B, "d2h_bytes_per_step": 8 * B},
        "gpu_launches": launches * K,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }), flush=True)
    if cpu is None:
        for kv in kvs:
            kv.close()
        model.close()
    ctx.close()


PREFILL_METRIC = "prefill tok/s, Qwen3-1.7B-shape Q4_0, 2048-token prompt; int8 tensor-core TOPS"
PREFILL_LEN = 2048


def prefill_gemm_ops(cfg, n: int) -> int:
    """Integer multiply-adds x 2 of the projection GEMMs of one n-token prefill
    (QKV, O, gate/up, down per layer; the LM head runs on the last token only)."""
    per_layer = (cfg.q_dim + 2 * cfg.kv_dim) * cfg.hidden + cfg.hidden * cfg.q_dim \
        + 2 * cfg.ffn * cfg.hidden + cfg.hidden * cfg.ffn
    return 2 * n * cfg.n_layers * per_layer


def cpu_prefill(cfg, weights, prompt, threads: int):
    """The reference's prompt loop (forward_single_token per prompt token,
    inference.rs:1938-1999) on the CPU oracle's AVX-512 path."""
    import oracle as O

    r = O.OracleRun(cfg, weights, len(prompt) + 2, order=O.ORDER_AVX512, threads=threads)
    t0 = time.perf_counter()
    for i, t in enumerate(prompt):
        r.forward(int(t), i)
    rc, tok, _ = r.lm_head()
    dt = time.perf_counter() - t0
    r.close()
    return len(prompt) / dt, dt


def run_prefill(args, rank, world, local):
    """BASELINE config 4 at batch 1: a 2048-token seeded prompt through the
    token-parallel prefill (tcgen05 int8 projections, causal attention writing
    the KV cache, LM head on the last token).  A step is one whole prefill."""
    synth = synth_module(args)

    cfg = synth.QWEN3_1_7B
    n_cpu = 64
    if args.impl == "reference":
        if rank == 0:
            weights = synth.qwen3_weights(cfg, seed=SEED, x4=False)
            prompt = synth.prompt_ids(cfg, PREFILL_LEN, seed=SEED)
            cores = physical_cores()
            tok_s, dt = cpu_prefill(cfg, weights, prompt[:n_cpu], cores)
            print(json.dumps({
                "impl": "reference", "metric": PREFILL_METRIC, "value": round(tok_s, 3), "unit": "tok/s",
                "n_gpus": args.gpus, "steps": 1, "warmup": 0, "ms_per_step": round(1000 * dt, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded random-init .smodel v2 weights)",
                "config": {"workload": "qwen3-1.7b-shape q4_0 prefill b=1 (BASELINE config 4)",
                           "prompt": PREFILL_LEN, "parallelism": "cpu threads"},
                "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                                 "sample": f"the first {n_cpu} prompt tokens, one forward_single_token each"},
                "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}), flush=True)
        return
    import torch

    import zero_b200 as zb

    weights = synth.qwen3_weights(cfg, seed=SEED)
    B = args.batch
    prompts = np.stack([synth.prompt_ids(cfg, PREFILL_LEN, seed=SEED + i) for i in range(B)])
    prompt = prompts[0]
    ctx = zb.Context(device=local)
    model = zb.Qwen3Model(ctx, cfg, weights)
    kvs = [model.new_kv(PREFILL_LEN + 8) for _ in range(B)]
    kv = kvs[0]

    def one_step():
        if B == 1:
            return model.prefill(kv, prompt, want_logits=False)[0]
        return int(model.prefill_batch(kvs, prompts, want_logits=False)[0][0])

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    dev_ms, gemm_ms, attn_ms, wall = [], [], [], []
    with ClockSampler(physical_gpu_index(local)) as clocks:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            tok = one_step()
            wall.append(time.perf_counter() - t0)
            p = model.perf()
            dev_ms.append(p["prefill_ms"])
            gemm_ms.append(p["prefill_gemm_ms"])
            attn_ms.append(p["prefill_attn_ms"])
    launches = int(model.perf()["kernel_launches"])
    tok_s = B * PREFILL_LEN / (statistics.mean(dev_ms) / 1000.0)
    e2e_tok_s = B * PREFILL_LEN * args.steps / sum(wall)
    ops = prefill_gemm_ops(cfg, B * PREFILL_LEN)
    g_ms = statistics.mean(gemm_ms)
    tops = ops / (g_ms / 1000.0) / 1e12
    peaks = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cores = physical_cores()
        w_plain = synth.qwen3_weights(cfg, seed=SEED, x4=False)
        c_tok_s, c_dt = cpu_prefill(cfg, w_plain, prompt[:n_cpu], cores)
        cpu = {"value": round(c_tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"the first {n_cpu} prompt tokens through the AVX-512-order restatement of the "
                         f"reference's per-token prompt loop, {c_dt:.1f} s"}
    if rank == 0:
        line = {
            "metric": PREFILL_METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(statistics.mean(dev_ms), 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int8 -> int32 (Q8_0 x Q4_0), f32 elsewhere",
            "data": "synthetic (seeded random-init .smodel v2 weights, BASELINE config 4)",
            "config": {"workload": f"qwen3-1.7b-shape q4_0 prefill b={B} (BASELINE config 4)",
                       "prompt": PREFILL_LEN, "batch": B, "layers": cfg.n_layers,
                       "l2": "inputs larger than L2 (793 MB of projection weights per prefill)",
                       "parallelism": "single GPU", "next_token": int(tok),
                       "gemm_ms": round(g_ms, 3), "attention_ms": round(statistics.mean(attn_ms), 3),
                       "other_ms": round(statistics.mean(dev_ms) - g_ms - statistics.mean(attn_ms), 3)},
            "roofline": {"bound": "tensor", "kernel": "q4q8_mma (tcgen05 int8, all projection GEMMs)",
                         "achieved": round(tops, 1), "peak": round(int8_peak, 1), "unit": "TOPS",
                         "frac": round(tops / int8_peak, 4),
                         "peak_source": f"2 x measured bf16 burst ({peaks['source']}): int8 MMA issues at "
                                        f"twice the bf16 rate",
                         "traffic": None, "algorithmic_ops": ops,
                         "avg_launch_us": round(g_ms * 1000 / (4 * cfg.n_layers), 2)},
            "e2e": {"value": round(e2e_tok_s, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * PREFILL_LEN * B,
                    "d2h_bytes_per_step": 4 * B},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    for k in kvs:
        k.close()
    model.close()
    ctx.close()


KQUANT_METRIC = "K-quant GEMV weight GB/s, one token's matmuls of a Qwen3-1.7B-shape Q4_K/Q6_K model"


def kquant_mats(cfg) -> list[tuple[str, str, int, int]]:
    """(name, quant, rows, cols) of one token's matmuls in a Q4_K_M-style mix:
    Q6_K for the V projection, the FFN down projection and the LM head, Q4_K
    for the rest (the GGUF-compat path's linear_q4k / linear_q6k)."""
    h, q, kv, f = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.ffn
    mats = []
    for i in range(cfg.n_layers):
        mats += [(f"blk.{i}.attn_q", "q4_k", q, h), (f"blk.{i}.attn_k", "q4_k", kv, h),
                 (f"blk.{i}.attn_v", "q6_k", kv, h), (f"blk.{i}.attn_output", "q4_k", h, q),
                 (f"blk.{i}.ffn_gate", "q4_k", f, h), (f"blk.{i}.ffn_up", "q4_k", f, h),
                 (f"blk.{i}.ffn_down", "q6_k", h, f)]
    mats.append(("output", "q6_k", cfg.vocab_padded, h))
    return mats


def kquant_bytes(quant: str, rows: int, cols: int) -> int:
    return rows * (cols // 256) * (144 if quant == "q4_k" else 210)


def cpu_kquant(mats, weights, xs, threads: int, budget_s: float = 20.0):
    """The oracle's linear_q4k / linear_q6k restatement over the matmuls in
    order, rows split across `threads` (ctypes drops the GIL); stops after
    budget_s.  Returns (GB/s, matrices done, seconds)."""
    from concurrent.futures import ThreadPoolExecutor

    import oracle as O

    done, nbytes, t0 = 0, 0, time.perf_counter()
    with ThreadPoolExecutor(threads) as pool:
        for (name, quant, rows, cols), w in zip(mats, weights):
            x = xs[cols]
            per = (rows + threads - 1) // threads
            bpr = kquant_bytes(quant, 1, cols)
            parts = [(r0, min(rows, r0 + per)) for r0 in range(0, rows, per)]
            list(pool.map(lambda p: O.linear_kquant(x, w[p[0] * bpr:p[1] * bpr], cols, p[1] - p[0], quant),
                          parts))
            done += 1
            nbytes += w.nbytes
            if time.perf_counter() - t0 > budget_s:
                break
    dt = time.perf_counter() - t0
    return nbytes / dt / 1e9, done, dt


def run_kquant(args, rank, world, local):
    """The GGUF-compat matmul path at Qwen3-1.7B shape: a step is one token's
    197 GEMVs (28 layers x 7 + the LM head) through zgpu_linear_dispatch_device,
    captured once as a CUDA graph and replayed.  The 1.15 GB of weights is
    far above the 126 MB L2, so no flush is needed between steps."""
    synth = synth_module(args)

    if world > 1:
        raise SystemExit("the kquant workload runs on one GPU")
    cfg = synth.QWEN3_1_7B
    mats = kquant_mats(cfg)
    weights = [synth.kquant(SEED + i, rows, cols, quant) for i, (_, quant, rows, cols) in enumerate(mats)]
    step_bytes = sum(w.nbytes for w in weights)
    rng = np.random.default_rng(SEED)
    xs = {c: rng.standard_normal(c).astype(np.float32) for c in {m[3] for m in mats}}
    cores = physical_cores()
    if args.impl == "reference":
        gbs, done, dt = cpu_kquant(mats, weights, xs, cores)
        sample = f"the first {done} of {len(mats)} matmuls of one step, {dt:.1f} s"
        print(json.dumps({
            "impl": "reference", "metric": KQUANT_METRIC, "value": round(gbs, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": 1, "warmup": 0, "ms_per_step": round(1000 * step_bytes / 1e9 / gbs, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random Q4_K / Q6_K super-blocks)",
            "config": {"workload": "qwen3-1.7b-shape q4_k_m-style decode matmuls b=1", "parallelism": "cpu threads"},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    import torch

    import zero_b200 as zb

    ctx = zb.Context(device=local)
    qt = {"q4_k": zb.Q4_K, "q6_k": zb.Q6_K}
    keys = [ctx.register(w, qt[q], rows, cols) for w, (_, q, rows, cols) in zip(weights, mats)]
    d_x = {c: torch.from_numpy(v).cuda() for c, v in xs.items()}
    d_y = torch.empty(max(m[2] for m in mats), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()

    def sweep(s):
        for key, (_, q, rows, cols) in zip(keys, mats):
            ctx.linear_dispatch_device(d_x[cols].data_ptr(), key, d_y.data_ptr(), cols, rows, qt[q], s)

    with torch.cuda.stream(stream):
        for _ in range(2):
            sweep(stream.cuda_stream)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            sweep(torch.cuda.current_stream().cuda_stream)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu_index(local)) as clocks:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        step_ms = e0.elapsed_time(e1) / args.steps
        # the dominant kernel alone: the Q6_K LM head GEMV (255 MB per launch)
        key, (_, q, rows, cols) = keys[-1], mats[-1]
        reps = 64
        with torch.cuda.stream(stream):
            ctx.linear_dispatch_device(d_x[cols].data_ptr(), key, d_y.data_ptr(), cols, rows, qt[q],
                                       stream.cuda_stream)
            e0.record(stream)
            for _ in range(reps):
                ctx.linear_dispatch_device(d_x[cols].data_ptr(), key, d_y.data_ptr(), cols, rows, qt[q],
                                           stream.cuda_stream)
            e1.record(stream)
        torch.cuda.synchronize()
        lm_us = 1000 * e0.elapsed_time(e1) / reps
    launches = len(mats) * args.steps   # kernels the timed graph replays launch
    # e2e: the reference-facing host-buffer call per matmul (x in, y out every call)
    t0 = time.perf_counter()
    for key, (_, q, rows, cols) in zip(keys, mats):
        ctx.linear_dispatch(xs[cols], key, cols, rows, qt[q])
    e2e_s = time.perf_counter() - t0
    h2d = sum(4 * m[3] for m in mats)
    d2h = sum(4 * m[2] for m in mats)
    peaks = measured_peaks()
    gbs = step_bytes / (step_ms / 1000) / 1e9
    lm_bytes = weights[-1].nbytes + 4 * (mats[-1][3] + mats[-1][2])
    lm_gbs = lm_bytes / (lm_us / 1e6) / 1e9
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        c_gbs, done, dt = cpu_kquant(mats, weights, xs, cores)
        cpu = {"value": round(c_gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"the first {done} of {len(mats)} matmuls of one step through the oracle's "
                         f"linear_q4k / linear_q6k, rows across {cores} threads, {dt:.1f} s"}
    print(json.dumps({
        "metric": KQUANT_METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (weights Q4_K / Q6_K)",
        "data": "synthetic (seeded random Q4_K / Q6_K super-blocks)",
        "config": {"workload": "qwen3-1.7b-shape q4_k_m-style decode matmuls b=1", "matmuls_per_step": len(mats),
                   "weight_bytes_per_step": step_bytes, "tok_s_equivalent": round(1000 / step_ms, 1),
                   "l2": "inputs larger than L2 (1.15 GB of weights per step)", "parallelism": "single GPU",
                   "cuda_graph": True},
        "roofline": {"bound": "hbm", "kernel": "gemv_kquant_kernel<Q6_K> (LM head 151936 x 2048)",
                     "achieved": round(lm_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(lm_gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "traffic": None, "algorithmic_bytes": lm_bytes, "avg_launch_us": round(lm_us, 2)},
        "e2e": {"value": round(step_bytes / e2e_s / 1e9, 2), "unit": "GB/s",
                "scope": "zgpu_linear_dispatch per matmul with host x / y buffers, host wall clock",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }), flush=True)
    ctx.close()


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.workload == "kquant":
        if args.impl != "reference":
            import torch

            torch.cuda.set_device(local)
        run_kquant(args, rank, world, local)
        return
    if args.workload == "ds2":
        if args.impl != "reference":
            import torch

            torch.cuda.set_device(local)
        if args.batch > 1:
            run_ds2_batch(args, rank, world, local)
        else:
            run_ds2(args, rank, world, local)
        return
    if args.workload == "qwen3-8b":
        if args.batch > 1:
            run_qwen3_batch(args, rank, world, local)
        else:
            run_qwen3_tp(args, rank, world, local)
        return
    if args.workload == "prefill":
        if args.impl != "reference":
            import torch

            torch.cuda.set_device(local)
        run_prefill(args, rank, world, local)
        return
    if args.impl == "reference":
        run_reference(args, rank)
        return
    import torch

    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import zero_b200 as zb
    synth = synth_module(args)

    cfg = synth.QWEN3_1_7B
    weights = synth.qwen3_weights(cfg, seed=SEED)
    prompt = synth.prompt_ids(cfg, PROMPT_LEN, seed=SEED)
    ctx = zb.Context(device=local)
    # N > 1: tensor parallel over the N GPUs (one sequence, its weights split
    # N ways: strong scaling); the stage outputs cross NVLink inside the
    # persistent step kernel
    model = zb.Qwen3Model(ctx, cfg, weights, rank=rank, world=world)
    if world > 1:
        from zero_b200 import tp

        tp.connect(model)
    max_tokens = 512
    n_gen_timed = args.steps + 1
    assert PROMPT_LEN + n_gen_timed - 1 <= max_tokens
    kv = model.new_kv(max_tokens)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()

    # warm-up: W decode steps (graphs captured on the first call)
    model.generate_greedy(kv, prompt, args.warmup + 1)
    barrier()
    with ClockSampler(physical_gpu_index(local)) as clocks:
        toks, _ = model.generate_greedy(kv, prompt, n_gen_timed)
        barrier()
    perf = model.perf()
    dec_ms = float(perf["decode_ms"])
    if world > 1:
        t = torch.tensor([dec_ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dec_ms = float(t.item())
    tok_s = args.steps / (dec_ms / 1000.0)
    # kernel launches of this library inside the timed decode steps
    gpu_launches = perf["decode_launches"]

    # ------------------------------------------------ e2e through the C ABI
    e2e_tok_s = None
    if not args.no_e2e:
        kv2 = model.new_kv(max_tokens)
        for i, t in enumerate(prompt):
            model.forward_single_token(kv2, int(t), i)
        tok, _ = model.lm_head_argmax(want_logits=False)
        barrier()
        t0 = time.perf_counter()
        pos = PROMPT_LEN
        for _ in range(args.steps):
            model.forward_single_token(kv2, tok, pos)
            tok, _ = model.lm_head_argmax(want_logits=False)
            pos += 1
        e2e_s = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([e2e_s], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e_tok_s = args.steps / e2e_s
        kv2.close()

    # -------------------------------------- roofline of the dominant kernel
    # The decode steps run as one persistent launch (decode_launches == 1):
    # algorithmic bytes = K steps x (weights 1.124 GB + the KV rows each step
    # reads), duration = the CUDA-event time of that launch (decode_ms).  With
    # the per-op kernels instead, the same bytes over the same device time give
    # the whole-step figure.
    # Tensor parallel (N > 1): per GPU, its 1/N of the weights and the K/V
    # rows of its kv heads, over the slowest rank's launch time.
    peaks = measured_peaks()
    step_bytes = cfg.weight_bytes_per_token() // world
    # a step at position p reads the K and V rows of tokens 0..p-1 and writes row p (f32, all layers)
    kv_row_bytes = 2 * (cfg.n_kv_heads // world) * cfg.head_dim * 4 * cfg.n_layers
    kv_bytes = sum(kv_row_bytes * (PROMPT_LEN + i + 1) for i in range(args.steps))
    launch_bytes = args.steps * step_bytes + kv_bytes
    step_gbs = launch_bytes / (dec_ms / 1000.0) / 1e9
    traffic_step = measured_traffic_per_step() if world == 1 else None
    kv.close()
    model.close()

    # ----------------------------- secondary: the config-1 GEMV sweep (N = 1)
    # The four BASELINE config-1 shapes (Q4_0 weights, 2048->4096, 2048->12288,
    # 6144->2048, 2048->151936) with f32 activations (the reference's GEMV) and
    # with Q8_0 activations; weights rotated over > 2x L2 per sweep, launches
    # captured in a CUDA graph and timed with CUDA events on its stream.
    gemv_sweep = None
    if world == 1 and not args.no_roofline:
        from zero_b200 import microbench

        gemv_sweep = []
        for shp in microbench.CONFIG1_SHAPES:
            o, i = (int(v) for v in shp.split("x"))
            for act in ("f32", "q8"):
                r = microbench.run_shape(ctx, o, i, act, 5, None, torch)
                r["frac"] = round(r["gbs"] / peaks["hbm_gbs"], 4)
                gemv_sweep.append(r)

    # ------------------------------------------------------- CPU baseline
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = physical_cores()
        probe_rate, _ = cpu_decode(cfg, weights, prompt, 1, cores)
        n = int(max(2, min(64, 15.0 * probe_rate)))
        rate, dt = cpu_decode(cfg, weights, prompt, n, cores)
        host_gbs = host_read_gbs(cores)
        cpu = {"value": round(rate, 3), "unit": "tok/s", "cores": cores, "kind": "port",
               "weights_gbs": round(rate * cfg.weight_bytes_per_token() / 1e9, 2),
               "host_read_gbs": round(host_gbs, 2),
               "sample": f"{n} decode steps (forward + LM head) after a {PROMPT_LEN}-token prefill, "
                         f"same seeded weights, AVX-512-order restatement, {dt:.1f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dec_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": round(tok_s / PUBLISHED_TOK_S, 3), "dtype": "f32",
            "data": "synthetic (seeded random-init .smodel v2 weights, BASELINE config 0)",
            "config": {"workload": "qwen3-1.7b-shape q4_0 decode b=1 (BASELINE config 0)",
                       "prompt": PROMPT_LEN, "decode_steps": args.steps, "layers": cfg.n_layers,
                       "hidden": cfg.hidden, "ffn": cfg.ffn, "vocab": cfg.vocab_padded,
                       "weight_bytes_per_step": step_bytes,
                       "l2": "inputs larger than L2 (1.12 GB of weights streamed per step)",
                       "parallelism": f"tp{world} (one sequence; stage outputs exchanged over NVLink "
                                      f"inside the step kernel)" if world > 1 else "single GPU",
                       "tokens_first": [int(v) for v in toks[:4]]},
            "roofline": {"bound": "hbm",
                         "kernel": "step_kernel (persistent decode, one launch for all timed steps)"
                                   if gpu_launches == 1 else "per-op decode kernels (whole step)",
                         "per": "GPU",
                         "achieved": round(step_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(step_gbs / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                         "traffic": (traffic_step * args.steps) if traffic_step else None,
                         "traffic_source": "ncu dram bytes per step x steps" if traffic_step else
                                           "not captured on the current step-kernel sources",
                         "algorithmic_bytes": launch_bytes,
                         "avg_launch_us": round(dec_ms * 1000 / max(gpu_launches, 1), 1),
                         "gemv_sweep_config1": gemv_sweep},
            "e2e": {"value": round(e2e_tok_s, 2) if e2e_tok_s else None, "unit": "tok/s",
                    "h2d_bytes_per_step": 84, "d2h_bytes_per_step": 12},
            "gpu_launches": int(gpu_launches),
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # A rank that fails (a device-wait timeout, an exception) ends at once
        # with a non-zero status, so the launcher stops the other ranks;
        # unwinding normally could block in process-group teardown while its
        # peers wait at their next collective.
        try:
            main()
        except BaseException:
            import traceback

            traceback.print_exc()
            sys.stderr.flush()
            sys.stdout.flush()
            os._exit(1)
    else:
        main()
