"""Standalone GEMV sweep: HBM GB/s of the batch-1 kernels.

    python -m zero_b200.microbench [--shape OUTxIN ...] [--act f32|q8] [--reps R]

For each shape, enough distinct seeded weight copies are registered that one
pass over them streams more than 2x the 126 MB L2, the launches over all
copies are captured into one CUDA graph on a torch stream, and the graph is
replayed `reps` times between CUDA events recorded on that stream.  Prints one
JSON line per shape: average launch time and algorithmic GB/s (weights +
activation + output bytes per launch).

--act f32 runs the reference's f32-activation GEMV (Q4_0X4 weights,
linear_dispatch); --act q8 runs the Q4_0 x Q8_0-activation GEMV.

--tokens T (prefill) times the batched Q4_0 x Q8_0 matmul
on the tcgen05 int8 path instead: T activation rows per launch (quantisation
included), reported as int8 TOPS (2 * rows * in * T per launch) next to the
weight and activation bytes.

--vectors V runs the exact batched matvec (zgpu_linear_dispatch_batch: V f32
rows per call, host buffers) on each shape, for profiling its kernels.

--ds2-batch N decodes N sequences of the
DeepSeek-V2-Lite-shaped model (--layers L of its 27) together with
zgpu_ds2_decode_batch: every sequence's latent cache holds --context seeded
rows (stored once, copied on the device), then --reps steps, each printed
with its device time and the distinct experts of its MoE layers.
"""
from __future__ import annotations

import argparse
import json

import numpy as np

import zero_b200 as zb
from zero_b200 import synth

CONFIG1_SHAPES = ["4096x2048", "12288x2048", "2048x6144", "151936x2048"]
L2_BYTES = 126 * 1024 * 1024


def run_shape(ctx, out_dim: int, in_dim: int, act: str, reps: int, copies: int | None, torch):
    wbytes = out_dim * in_dim * 18 // 32
    n = copies or max(2, -(-2 * L2_BYTES // wbytes))
    keys = []
    for c in range(n):
        w = synth.q4_0(100 + c, out_dim + 7 * in_dim, out_dim, in_dim, 0.02)
        if act == "f32":
            keys.append(ctx.register(synth.pack_x4(w, out_dim, in_dim, "q4_0"), zb.Q4_0X4, out_dim, in_dim))
        else:
            keys.append(ctx.register(w, zb.Q4_0, out_dim, in_dim))
    stream = torch.cuda.Stream()
    sh = stream.cuda_stream
    if act == "f32":
        x = torch.randn(in_dim, device="cuda", dtype=torch.float32)
        xbytes = in_dim * 4
    else:
        xq = ctx.quantize_q8_0(np.random.default_rng(0).standard_normal(in_dim).astype(np.float32))
        x = torch.from_numpy(xq).cuda()
        xbytes = in_dim // 32 * 34
    y = torch.empty(out_dim, device="cuda", dtype=torch.float32)

    def sweep():
        for k in keys:
            if act == "f32":
                ctx.linear_dispatch_device(x.data_ptr(), k, y.data_ptr(), in_dim, out_dim, zb.Q4_0, sh)
            else:
                ctx.linear_q8act_device(x.data_ptr(), k, y.data_ptr(), in_dim, out_dim, sh)

    with torch.cuda.stream(stream):
        sweep()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        sweep()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    ms = e0.elapsed_time(e1) / (reps * n)
    alg = wbytes + xbytes + out_dim * 4
    del graph
    ctx.clear_weights()
    return {"kernel": f"gemv_{'x4_q4_0_f32act' if act == 'f32' else 'q4_0_q8act'}",
            "shape": f"{in_dim}->{out_dim}", "copies": n, "reps": reps,
            "avg_launch_us": round(ms * 1000, 3), "algorithmic_bytes": alg,
            "gbs": round(alg / (ms * 1e-3) / 1e9, 1)}


def run_batch(ctx, out_dim: int, in_dim: int, T: int, reps: int, torch):
    w = synth.q4_0(100, out_dim + 7 * in_dim, out_dim, in_dim, 0.02)
    key = ctx.register(w, zb.Q4_0, out_dim, in_dim)
    stream = torch.cuda.Stream()
    sh = stream.cuda_stream
    x = torch.randn(T, in_dim, device="cuda", dtype=torch.float32)
    y = torch.empty(T, out_dim, device="cuda", dtype=torch.float32)

    def launch():
        ctx.linear_q8act_batch_device(x.data_ptr(), key, y.data_ptr(), T, in_dim, out_dim, sh)

    with torch.cuda.stream(stream):
        launch()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    ms = e0.elapsed_time(e1) / reps
    ops = 2.0 * out_dim * in_dim * T
    del graph
    ctx.clear_weights()
    return {"kernel": "q4q8_mma (tcgen05 kind::i8) + q8_0 quantiser", "shape": f"{in_dim}->{out_dim}",
            "tokens": T, "reps": reps, "avg_launch_us": round(ms * 1000, 2),
            "tops": round(ops / (ms * 1e-3) / 1e12, 2),
            "bytes": out_dim * in_dim * 18 // 32 + T * in_dim * 4 + T * out_dim * 4}


def run_vectors(ctx, out_dim: int, in_dim: int, V: int, reps: int):
    w = synth.q4_0(100, out_dim + 7 * in_dim, out_dim, in_dim, 0.02)
    key = ctx.register(w, zb.Q4_0, out_dim, in_dim)
    x = np.random.default_rng(0).standard_normal((V, in_dim)).astype(np.float32)
    for _ in range(reps):
        ctx.linear_dispatch_batch(x, key, in_dim, out_dim, zb.Q4_0)
    ctx.clear_weights()
    return {"kernel": "dm_gemm (tcgen05 kind::i8 over activation digits)", "shape": f"{in_dim}->{out_dim}",
            "vectors": V, "reps": reps}


def run_ds2_batch(n_seq: int, context: int, layers: int, reps: int):
    cfg = synth.DS2_V2_LITE
    if layers != cfg.n_layers:
        cfg = synth.Ds2Config(**{**cfg.__dict__, "n_layers": layers})
    ctx = zb.Context()
    m = zb.Ds2Model(ctx, cfg, synth.ds2_weights(cfg, seed=0))
    max_tokens = context + reps + 4
    first = m.new_kv(max_tokens)
    rows = synth.f32(1, 2, context * (cfg.kv_lora_rank + cfg.rope_dim), 0.0, 0.5).reshape(context, -1)
    for layer in range(cfg.n_layers):
        for t in range(context):
            first.store_compressed(layer, t, rows[t, :cfg.kv_lora_rank], rows[t, cfg.kv_lora_rank:])
    kvs = [first] + [m.new_kv(max_tokens) for _ in range(n_seq - 1)]
    for kv in kvs[1:]:
        kv.copy_from(first, context)
    tokens = synth.ds2_prompt_ids(cfg, n_seq, seed=1)
    pos = np.full(n_seq, context, np.uint32)
    for s in range(reps):
        tokens, _ = m.decode_batch(kvs, tokens, pos, want_logits=False)
        pos = pos + 1
        ms = m.perf()["decode_ms"]
        ids, _ = m.batch_expert_ids(n_seq)
        distinct = float(np.mean([len(np.unique(ids[layer])) for layer in range(cfg.n_dense, cfg.n_layers)]))
        print(json.dumps({"workload": "ds2 batch", "sequences": n_seq, "context": context, "layers": cfg.n_layers,
                          "step": s, "ms": round(ms, 3), "tok_s": round(n_seq / (ms * 1e-3), 1),
                          "distinct_experts": round(distinct, 1)}), flush=True)
    for kv in kvs:
        kv.close()
    m.close()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", action="append", help="OUTxIN, repeatable (default: config 1 sweep)")
    ap.add_argument("--act", default="f32", choices=["f32", "q8"])
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--copies", type=int, default=None, help="weight copies (default: > 2x L2)")
    ap.add_argument("--tokens", type=int, default=0, help="time the batched tcgen05 matmul over T tokens")
    ap.add_argument("--vectors", type=int, default=0, help="run the exact batched matvec on V rows")
    ap.add_argument("--ds2-batch", type=int, default=0, help="decode N DeepSeek2 sequences together")
    ap.add_argument("--context", type=int, default=2048, help="--ds2-batch: cached rows per sequence")
    ap.add_argument("--layers", type=int, default=27, help="--ds2-batch: layers of the model")
    args = ap.parse_args()
    if args.ds2_batch:
        run_ds2_batch(args.ds2_batch, args.context, args.layers, args.reps)
        return
    import torch

    ctx = zb.Context()
    for s in args.shape or CONFIG1_SHAPES:
        o, i = (int(v) for v in s.lower().split("x"))
        if args.vectors:
            print(json.dumps(run_vectors(ctx, o, i, args.vectors, args.reps)), flush=True)
        elif args.tokens:
            print(json.dumps(run_batch(ctx, o, i, args.tokens, args.reps, torch)), flush=True)
        else:
            print(json.dumps(run_shape(ctx, o, i, args.act, args.reps, args.copies, torch)), flush=True)
    ctx.close()


if __name__ == "__main__":
    main()
