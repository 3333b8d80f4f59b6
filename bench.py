#!/usr/bin/env python
"""Decode tokens/s of voxtral.cpp's decoder KV step on B200.

One "step" = every stream appends one token and attends over its cache in all
decoder layers (fused RoPE + K/V append + GQA flash-decoding attention per
layer, through libvxk.so's C ABI).  Default workload: 64 streams per GPU,
30 layers (Voxtral-Mini-3B decoder shape: 32 q / 8 kv heads x 128), f16 cache
in 16-token pages with a seeded random block table, contexts seeded uniform
in [400, 4096].  Synthetic N(0, 0.5^2) activations.  After the timed region
a sample of the outputs (three streams, first and last layer) is compared
with the CPU oracle and the result is printed in the line's "checked" key.

Multi-GPU: one process per GPU (torchrun).  The job's contexts are drawn once
from the seed and dealt to ranks by longest-processing-time
(vxk_shard.assign_streams); each rank owns its streams' pages (no data-path
collective); timing is max over ranks, and every rank's time is reported.
The default workload has 64 streams per GPU (weak scaling); `--config 3`
(256 realtime streams) and `--config 5` (128 q8_0 streams) fix the job's
total and shard it (strong scaling), running on each GPU the streams that
fit its memory.

`--impl reference` times the CPU restatement of the same path (the reference's
ggml CPU backend cannot be built here: ggml is fetched at configure time and
is absent) on the host cores, on rank 0, over streams taken from the same
seeded context list.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "voxtral.cpp_b200"))
from vxk_shard import assign_streams, gather_over_ranks, max_over_ranks  # noqa: E402

HD, NQ, NKV, BT = 128, 32, 8, 16
CONFIGS = {
    # name: layers, streams per GPU, ctx range, dtype, capacity
    "2": dict(layers=30, streams=64, ctx=(400, 4096), dtype=1, capacity=8192,
              desc="3B decoder, 64 streams/GPU, ctx~U[400,4096], f16 16-token pages, random block table"),
    "3": dict(layers=26, total_streams=256, ctx=(8192, 8192), dtype=1, capacity=8192,
              desc="4B realtime decoder, 256 streams sharded by stream, full 8192-slot sliding rings "
                   "(steady state: one eviction per stream and step)"),
    "5": dict(layers=30, total_streams=128, ctx=(8192, 32768), dtype=8, capacity=32768 + 1024,
              desc="3B decoder, 128 streams sharded by stream, q8_0 cache, ctx~U[8192,32768]"),
    "head": dict(kind="head", rows=64, vocab=131072, dim=3072, dtype=1,
                 desc="greedy head: tied logits (131072 x 3072 f16 embeddings) + argmax for 64 streams/GPU, "
                      "logits written like the reference's decoder_logits"),
    "headq": dict(kind="headq", rows=64, vocab=131072, dim=3072, qtype=14,
                  desc="greedy head over Q6_K tied embeddings (Q4_K_M's tok_embeddings, 131072 x 3072) for 64 "
                       "streams/GPU, logits written like the reference's decoder_logits"),
    "proj": dict(kind="qmm", layers=30, rows=64,
                 mats=(("q", 4096, 3072, 12), ("k", 1024, 3072, 12), ("v", 1024, 3072, 14), ("o", 3072, 4096, 12)),
                 desc="decoder attention projections q/k/v/o of 30 layers for 64 batched streams/GPU, "
                      "Q4_K_M types (attn_q/k/o Q4_K, attn_v Q6_K), distinct weights per layer"),
    "decoder": dict(kind="decoder", layers=26, streams=64, ctx=(400, 4096), dim=3072, hidden=9216, vocab=131072,
                    capacity=8192, dtype=1,
                    desc="whole 4B-realtime decoder step (26 layers, 3072 / 9216, vocab 131072, Q4_K_M weights: "
                         "attn_q/k/o, ffn_w1/w3 Q4_K; attn_v, ffn_w2, tok_embeddings Q6_K) for 64 streams/GPU, "
                         "ctx~U[400,4096] f16 16-token pages: embeddings + audio, norms, time scale, projections, "
                         "attention, SwiGLU FFN, logits + argmax"),
    "encstack": dict(kind="encstack", layers=32, streams=128, heads=20, rows=4, window=750, capacity=878, dtype=30,
                     dim=1280, hidden=5120,
                     desc="whole streaming encoder step (conv stem, 32 layers: RMS norms, q/k/v/o with biases, "
                          "RoPE + ring append + 750-frame window attention, SwiGLU FFN; final norm) for 128 "
                          "streams x 4 new frames, 20 heads x 64, d_model 1280, FFN 5120, Q4_K_M weights, bf16 rings"),
    "4": dict(kind="encoder", layers=32, streams=128, heads=20, rows=4, window=750, capacity=878, dtype=30,
              desc="streaming encoder, 128 streams, 20 heads x 64, 4 new rows per 80 ms chunk, "
                   "750-frame window in an 878-slot bf16 ring (steady state, rings wrapped)"),
}


def run_encoder(args, cfg, world, rank, local, dist, torch, vxk):
    """Config 4: one step = one 80 ms chunk (4 new encoder rows) of every
    stream through every encoder layer (append + tcgen05 window attention; for
    16-bit rings one launch per layer, the append fused into the attention)."""
    L, S, H, P = cfg["layers"], cfg["streams"], cfg["heads"], cfg["rows"]
    W, CAP, HDE = cfg["window"], cfg["capacity"], 64
    pool = vxk.EncPool(device=local, n_layers=L, n_heads=H, head_dim=HDE, window=W, capacity=CAP, max_streams=S,
                       max_new=CAP - W, dtype=cfg["dtype"], max_position=65536)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    streams = [pool.open_stream() for _ in range(S)]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed + rank)
    fill = CAP - W
    fq = torch.randn((S * fill, H, HDE), device="cuda", generator=gen) * 0.5
    fo = torch.empty_like(fq)
    pos = 0
    while pos < CAP + 128:  # wrap every ring so each chunk sees a full 750-frame window
        pool.plan(streams, [fill] * S, sh)
        for layer in range(L):
            pool.layer(layer, fq.data_ptr(), fq.data_ptr(), fq.data_ptr(), fo.data_ptr(), sh)
        pool.commit()
        pos += fill
    torch.cuda.synchronize()
    del fq, fo
    NSETS = 2
    qs = torch.randn((NSETS, L, S * P, H, HDE), device="cuda", generator=gen) * 0.5
    ks = torch.randn((NSETS, L, S * P, H, HDE), device="cuda", generator=gen) * 0.5
    vs = torch.randn((NSETS, L, S * P, H, HDE), device="cuda", generator=gen) * 0.5
    out = torch.empty((L, S * P, H, HDE), device="cuda")

    def step(i):
        pool.plan(streams, [P] * S, sh)
        st = i % NSETS
        for layer in range(L):
            pool.layer(layer, qs[st, layer].data_ptr(), ks[st, layer].data_ptr(), vs[st, layer].data_ptr(),
                       out[layer].data_ptr(), sh)
        pool.commit()

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    props = torch.cuda.get_device_properties(local)
    gpu_id = str(getattr(props, "uuid", local))
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    rank_ms = gather_over_ranks(dist, ms, "cuda")
    ms = max(rank_ms)
    keys = W + P - 1  # union of the chunk's windows
    eb = 4 if cfg["dtype"] == 0 else 2  # ring value bytes (f32 or 16-bit)
    per_stream_layer = keys * H * HDE * eb * 2 + 3 * P * H * HDE * 4 + P * H * HDE * 4 + 2 * P * H * HDE * eb
    bytes_per_layer = S * per_stream_layer
    layer_s = (ms / 1000.0) / (args.steps * L)
    achieved = bytes_per_layer / layer_s / 1e9
    peak, peak_kind = load_peaks()
    flops_per_layer = S * H * P * keys * HDE * 2 * 2
    traffic_ratio, traffic_src = load_traffic(args.config) if not args.cache else (None, None)

    # ---- end to end: per step, pinned host q/k/v of every layer go up on a
    # copy stream (layer l's copy overlaps layer l-1's kernels), the layers
    # run through the public vxk_enc_layer call, and the outputs come back.
    e2e = None
    if not args.no_e2e:
        hq = torch.randn((L, S * P, H, HDE)).mul_(0.5).pin_memory()
        hk = torch.randn((L, S * P, H, HDE)).mul_(0.5).pin_memory()
        hv = torch.randn((L, S * P, H, HDE)).mul_(0.5).pin_memory()
        ho = torch.empty((L, S * P, H, HDE)).pin_memory()
        dq, dk, dv = (torch.empty_like(hq, device="cuda") for _ in range(3))
        # uploads and downloads on two copy streams, so the two PCIe directions
        # overlap; the next step's uploads wait only for the layers that read
        # the staging, its layers for the downloads of their outputs
        copy_stream, down_stream = torch.cuda.Stream(), torch.cuda.Stream()
        up = [torch.cuda.Event() for _ in range(L)]
        done_ev = [torch.cuda.Event() for _ in range(L)]

        def host_step():
            pool.plan(streams, [P] * S, sh)
            copy_stream.wait_stream(stream)
            with torch.cuda.stream(copy_stream):
                for layer in range(L):
                    dq[layer].copy_(hq[layer], non_blocking=True)
                    dk[layer].copy_(hk[layer], non_blocking=True)
                    dv[layer].copy_(hv[layer], non_blocking=True)
                    up[layer].record(copy_stream)
            stream.wait_stream(down_stream)
            for layer in range(L):
                stream.wait_event(up[layer])
                pool.layer(layer, dq[layer].data_ptr(), dk[layer].data_ptr(), dv[layer].data_ptr(),
                           out[layer].data_ptr(), sh)
                done_ev[layer].record(stream)
            with torch.cuda.stream(down_stream):
                for layer in range(L):
                    down_stream.wait_event(done_ev[layer])
                    ho[layer].copy_(out[layer], non_blocking=True)
            pool.commit()

        host_step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        f0.record(stream)
        for _ in range(args.steps):
            host_step()
        stream.wait_stream(down_stream)
        f1.record(stream)
        torch.cuda.synchronize()
        ems = f0.elapsed_time(f1)
        ems = max_over_ranks(dist, ems, "cuda")
        e2e = {"value": round(world * S * args.steps / (ems / 1000.0), 1), "unit": "stream-chunks/s",
               "h2d_bytes_per_step": int(hq.numel() + hk.numel() + hv.numel()) * 4,
               "d2h_bytes_per_step": int(ho.numel()) * 4, "ms_per_step": round(ems / args.steps, 3)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cps, done = encoder_cpu_sample(cfg, args.seed, args.cpu_seconds)
        cpu = {"value": round(cps, 4), "unit": "stream-chunks/s", "cores": 1, "kind": "port",
               "sample": f"{done} stream-layer chunks ({P} rows x {H} heads over a {W}-frame window) of the "
                         f"oracle's window attention on one host thread, scaled to {L} layers"}
    if dist:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": "encoder chunks/s (KV append + windowed attention, 4 rows/chunk)",
            "value": round(world * S * args.steps / (ms / 1000.0), 1),
            "unit": "stream-chunks/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": {30: "bf16 ring, bf16 hi+lo operands, fp32 accumulate",
                      1: "f16 ring, f16 hi+lo operands, fp32 accumulate",
                      0: "f32 ring, fp32 CUDA-core products"}[cfg["dtype"]], "data": "synthetic",
            "config": {"workload": f"config 4: {cfg['desc']}", "layers": L, "streams_per_gpu": S, "heads": H,
                       "parallelism": f"streams sharded, {S}/GPU, no collective",
                       "l2": "inputs larger than L2 (window reads per launch >> 126 MB)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": None if traffic_ratio is None else round(traffic_ratio * bytes_per_layer),
                         "traffic_source": traffic_src and f"{traffic_src} (ncu dram bytes per algorithmic byte, "
                                                           f"scaled to this launch)",
                         "algorithmic_bytes_per_launch": bytes_per_layer,
                         "avg_layer_us": round(layer_s * 1e6, 2),
                         "kernel": "enc_f32_kernel (+ enc_append_kernel)" if cfg["dtype"] == 0
                         else "enc_tc_kernel (K/V append fused: <= 8 rows per stream)",
                         "tensor_tflops": round(flops_per_layer / layer_s / 1e12, 2)},
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": int(args.steps * L * (2 if cfg["dtype"] == 0 else 1)),
            "clocks": clocks.summary(),
        }
        line.update(rank_fields(rank_ms))
        print(json.dumps(line), flush=True)
    pool.close()


def run_head(args, cfg, world, rank, local, dist, torch, vxk):
    """Greedy head: one step = logits of every stream's row over the whole
    vocabulary (written out) and their argmax, through vxk_head_logits_argmax."""
    R, V, D, dt = cfg["rows"], cfg["vocab"], cfg["dim"], cfg["dtype"]
    head = vxk.Head(device=local, dim=D, vocab=V, dtype=dt)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed + rank)
    w = (torch.randn((V, D), device="cuda", generator=gen) * 0.02).to(torch.float16 if dt == 1 else torch.bfloat16)
    NSETS = 4
    xs = torch.randn((NSETS, R, D), device="cuda", generator=gen)
    am = torch.empty((R,), dtype=torch.int32, device="cuda")
    lg = torch.empty((R, V), device="cuda")

    def step(i):
        x = xs[i % NSETS]
        head.logits_argmax(w.data_ptr(), x.data_ptr(), R, am.data_ptr(), lg.data_ptr(), sh)

    for i in range(args.warmup):
        step(i)
    head.sync(sh)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    props = torch.cuda.get_device_properties(local)
    gpu_id = str(getattr(props, "uuid", local))
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
    head.sync(sh)
    rank_ms = gather_over_ranks(dist, e0.elapsed_time(e1), "cuda")
    ms = max(rank_ms)
    step_s = ms / 1000.0 / args.steps
    bytes_per_step = V * D * 2 + R * D * 4 + R * V * 4 + R * 4  # W once, x, logits, argmax
    achieved = bytes_per_step / step_s / 1e9
    peak, peak_kind = load_peaks()
    traffic_ratio, traffic_src = load_traffic(args.config)

    # end to end: x from pinned host memory, argmax back to the host, each step
    e2e = None
    if not args.no_e2e:
        hx = torch.randn((R, D)).pin_memory()
        ha = torch.empty((R,), dtype=torch.int32).pin_memory()
        dx = torch.empty((R, D), device="cuda")

        def host_step():
            dx.copy_(hx, non_blocking=True)
            head.logits_argmax(w.data_ptr(), dx.data_ptr(), R, am.data_ptr(), lg.data_ptr(), sh)
            ha.copy_(am, non_blocking=True)

        host_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            host_step()
        f1.record(stream)
        torch.cuda.synchronize()
        ems = max_over_ranks(dist, f0.elapsed_time(f1), "cuda")
        e2e = {"value": round(world * R * args.steps / (ems / 1000.0), 1), "unit": "rows/s",
               "h2d_bytes_per_step": int(hx.numel()) * 4, "d2h_bytes_per_step": int(ha.numel()) * 4,
               "ms_per_step": round(ems / args.steps, 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cps, done = head_cpu_sample(cfg, args.seed, args.cpu_seconds)
        cpu = {"value": round(cps, 3), "unit": "rows/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{done} steps of 4 rows over a {V // 8}-row slice of the vocabulary "
                         f"(oracle.logits_argmax, float64 BLAS), scaled to {R} rows x {V}"}
    if dist:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": "greedy head rows/s (tied logits + argmax)",
            "value": round(world * R * args.steps / (ms / 1000.0), 1),
            "unit": "rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": ("f16" if dt == 1 else "bf16") + " weights and rows, fp32 accumulate", "data": "synthetic",
            "config": {"workload": f"config head: {cfg['desc']}", "rows_per_gpu": R, "vocab": V, "dim": D,
                       "parallelism": f"rows sharded, {R}/GPU, no collective",
                       "l2": "inputs larger than L2 (805 MB of weights per step)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": None if traffic_ratio is None else round(traffic_ratio * bytes_per_step),
                         "traffic_source": traffic_src and f"{traffic_src} (ncu dram bytes per algorithmic byte, "
                                                           f"scaled to this step)",
                         "algorithmic_bytes_per_launch": bytes_per_step, "avg_step_us": round(step_s * 1e6, 2),
                         "kernel": "head_kernel (+ x conversion and finish)",
                         "tensor_tflops": round(2.0 * R * V * D / step_s / 1e12, 2)},
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": int(args.steps * 3),
            "clocks": clocks.summary(),
        }
        line.update(rank_fields(rank_ms))
        print(json.dumps(line), flush=True)
    head.close()


def qmm_gguf_bytes(n, k, t):
    return n * (k // 32 * 34 if t == 8 else k // 256 * (144 if t == 12 else 210))


def run_qmm(args, cfg, world, rank, local, dist, torch, vxk):
    """Quantized projections: one step = q, k, v (from the same normed rows)
    and o of every layer for the GPU's batch of stream rows, each through
    vxk_qweight_matmul (activation quantization + the int8 tensor-core
    product)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    R, L = cfg["rows"], cfg["layers"]
    rng = np.random.default_rng(args.seed + rank)
    host = {name: vx_oracle.random_qblocks(t, n, k, rng) for name, n, k, t in cfg["mats"]}
    mats = []
    for _ in range(L):  # distinct device copies per layer: the step streams every layer's weights
        mats.append({name: vxk.QWeight(host[name], device=local, type=t, n_rows=n, n_cols=k, max_batch=R)
                     for name, n, k, t in cfg["mats"]})
    dims = {name: (n, k) for name, n, k, _ in cfg["mats"]}
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed + rank)
    x = torch.randn((R, dims["q"][1]), device="cuda", generator=gen)
    att = torch.randn((R, dims["o"][1]), device="cuda", generator=gen)
    ys = {name: torch.empty((R, n), device="cuda") for name, (n, _) in dims.items()}

    def step(s):
        # q, k, v share the normed rows: one quantization and one launch
        # (vxk_qweight_matmul_group); o multiplies the attention output
        for layer in mats:
            vxk.qweight_matmul_group([layer["q"], layer["k"], layer["v"]], x.data_ptr(), R,
                                     [ys["q"].data_ptr(), ys["k"].data_ptr(), ys["v"].data_ptr()], s)
            layer["o"].matmul(att.data_ptr(), R, ys["o"].data_ptr(), s)

    # eager warm-up (raises the kernels' shared-memory limits), then the whole
    # step captured once as a CUDA graph of the C-ABI launches: 120 launches of
    # a few microseconds each are otherwise paced by the host
    step(sh)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap):
        step(cap.cuda_stream)
    stream.wait_stream(cap)
    for _ in range(args.warmup):
        graph.replay()
    mats[0]["q"].sync(sh)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    props = torch.cuda.get_device_properties(local)
    gpu_id = str(getattr(props, "uuid", local))
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    for layer in mats:
        for m in layer.values():
            m.sync(sh)
    rank_ms = gather_over_ranks(dist, e0.elapsed_time(e1), "cuda")
    ms = max(rank_ms)
    step_s = ms / 1000.0 / args.steps
    w_bytes = L * sum(qmm_gguf_bytes(n, k, t) for _, n, k, t in cfg["mats"])
    # x read once for q/k/v (one quantization per group), the attention rows once, every output once
    io_bytes = L * R * 4 * (dims["q"][1] + dims["o"][1] + sum(n for n, _ in dims.values()))
    bytes_per_step = w_bytes + io_bytes
    achieved = bytes_per_step / step_s / 1e9
    peak, peak_kind = load_peaks()
    traffic_ratio, traffic_src = load_traffic(args.config)

    # end to end: the step's rows from pinned host memory, the last o rows back
    e2e = None
    if not args.no_e2e:
        hx = torch.randn((R, dims["q"][1])).pin_memory()
        hy = torch.empty((R, dims["o"][0])).pin_memory()

        def host_step():
            x.copy_(hx, non_blocking=True)
            graph.replay()
            hy.copy_(ys["o"], non_blocking=True)

        host_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            host_step()
        f1.record(stream)
        torch.cuda.synchronize()
        ems = max_over_ranks(dist, f0.elapsed_time(f1), "cuda")
        e2e = {"value": round(world * R * args.steps / (ems / 1000.0), 1), "unit": "tokens/s",
               "h2d_bytes_per_step": int(hx.numel()) * 4, "d2h_bytes_per_step": int(hy.numel()) * 4,
               "ms_per_step": round(ems / args.steps, 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, done = qmm_cpu_sample(cfg, args.seed, args.cpu_seconds)
        cpu = {"value": round(tps, 4), "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": f"{done} single-row products of the k projection (1024 x 3072 Q4_K) by the oracle "
                         f"(oracle/vx_qmm.c, one thread), scaled by weight count to q/k/v/o x {L} layers"}
    if dist:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": "attention-projection tokens/s (q/k/v/o, Q4_K_M, 30 layers)",
            "value": round(world * R * args.steps / (ms / 1000.0), 1),
            "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "Q4_K / Q6_K weights, Q8_K rows, exact integer dots on the tensor cores, fp32 scales",
            "data": "synthetic",
            "config": {"workload": f"config proj: {cfg['desc']}" + ("" if R == 64 else f" (run with {R} rows)"),
                       "rows_per_gpu": R, "layers": L,
                       "parallelism": f"stream rows sharded, {R}/GPU, no collective",
                       "l2": f"inputs larger than L2 ({w_bytes / 1e6:.0f} MB of weights per step)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": None if traffic_ratio is None else round(traffic_ratio * bytes_per_step),
                         "traffic_source": traffic_src and f"{traffic_src} (ncu dram bytes per algorithmic byte, "
                                                           f"scaled to this step)",
                         "algorithmic_bytes_per_launch": bytes_per_step, "avg_step_us": round(step_s * 1e6, 2),
                         "kernel": "qtc_kernel for Q4_K from 17 rows, qmm_kernel otherwise (+ quantization kernels)",
                         "int8_tops": round(2.0 * R * L * sum(n * k for _, n, k, _ in cfg["mats"]) / step_s / 1e12,
                                            2)},
            "cpu_baseline": cpu, "e2e": e2e,
            # per layer: (quantize + product) for q/k/v and for o
            "gpu_launches": int(args.steps * L * 4),
            "launch": "CUDA graph of the step's C-ABI calls (vxk_qweight_matmul_group for q/k/v, "
                      "vxk_qweight_matmul for o), replayed per step",
            "clocks": clocks.summary(),
        }
        line.update(rank_fields(rank_ms))
        print(json.dumps(line), flush=True)
    for layer in mats:
        for m in layer.values():
            m.close()


def qmm_cpu_sample(cfg, seed, seconds):
    """Times the oracle's quantized product on one row of the k projection;
    returns tokens/s scaled by weight count to all projections of all layers."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    rng = np.random.default_rng(seed)
    _, n, k, t = cfg["mats"][1]
    w = vx_oracle.random_qblocks(t, n, k, rng)
    x = rng.standard_normal((1, k)).astype(np.float32)
    vx_oracle.qmatmul(t, w, n, k, x)
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        vx_oracle.qmatmul(t, w, n, k, x)
        done += 1
    el = time.perf_counter() - t0
    per_row = el / done
    scale = sum(nn * kk for _, nn, kk, _ in cfg["mats"]) / (n * k) * cfg["layers"]
    return 1.0 / (per_row * scale), done


def run_headq(args, cfg, world, rank, local, dist, torch, vxk):
    """Greedy head over quantized embeddings: one step = the quantized logits
    product of every stream's row (vxk_qweight) and their argmax, through
    vxk_head_logits_argmax_q."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    R, V, D, t = cfg["rows"], cfg["vocab"], cfg["dim"], cfg["qtype"]
    rng = np.random.default_rng(args.seed + rank)
    w_host = vx_oracle.random_qblocks(t, V, D, rng)
    qw = vxk.QWeight(w_host, device=local, type=t, n_rows=V, n_cols=D, max_batch=R)
    del w_host
    head = vxk.Head(device=local, dim=D, vocab=V, dtype=1)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed + rank)
    NSETS = 4
    xs = torch.randn((NSETS, R, D), device="cuda", generator=gen)
    am = torch.empty((R,), dtype=torch.int32, device="cuda")
    lg = torch.empty((R, V), device="cuda")

    def step(i):
        head.logits_argmax_q(qw, xs[i % NSETS].data_ptr(), R, am.data_ptr(), lg.data_ptr(), sh)

    for i in range(args.warmup):
        step(i)
    qw.sync(sh)
    head.sync(sh)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    props = torch.cuda.get_device_properties(local)
    gpu_id = str(getattr(props, "uuid", local))
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
    qw.sync(sh)
    head.sync(sh)
    rank_ms = gather_over_ranks(dist, e0.elapsed_time(e1), "cuda")
    ms = max(rank_ms)
    step_s = ms / 1000.0 / args.steps
    bytes_per_step = qmm_gguf_bytes(V, D, t) + R * D * 4 + R * V * 4 + R * 4  # W once, x, logits, argmax
    achieved = bytes_per_step / step_s / 1e9
    peak, peak_kind = load_peaks()
    traffic_ratio, traffic_src = load_traffic(args.config)

    e2e = None
    if not args.no_e2e:
        hx = torch.randn((R, D)).pin_memory()
        ha = torch.empty((R,), dtype=torch.int32).pin_memory()
        dx = torch.empty((R, D), device="cuda")

        def host_step():
            dx.copy_(hx, non_blocking=True)
            head.logits_argmax_q(qw, dx.data_ptr(), R, am.data_ptr(), lg.data_ptr(), sh)
            ha.copy_(am, non_blocking=True)

        host_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            host_step()
        f1.record(stream)
        torch.cuda.synchronize()
        ems = max_over_ranks(dist, f0.elapsed_time(f1), "cuda")
        e2e = {"value": round(world * R * args.steps / (ems / 1000.0), 1), "unit": "rows/s",
               "h2d_bytes_per_step": int(hx.numel()) * 4, "d2h_bytes_per_step": int(ha.numel()) * 4,
               "ms_per_step": round(ems / args.steps, 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cps, done = headq_cpu_sample(cfg, args.seed, args.cpu_seconds)
        cpu = {"value": round(cps, 4), "unit": "rows/s", "cores": 1, "kind": "port",
               "sample": f"{done} single-row products over a {V // 64}-row slice of the vocabulary by the oracle "
                         f"(oracle/vx_qmm.c, one thread), scaled to {V} rows"}
    if dist:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": "greedy head rows/s (Q6_K tied logits + argmax)",
            "value": round(world * R * args.steps / (ms / 1000.0), 1),
            "unit": "rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "Q6_K weights, Q8_K rows, exact integer dots on the tensor cores, fp32 scales",
            "data": "synthetic",
            "config": {"workload": f"config headq: {cfg['desc']}", "rows_per_gpu": R, "vocab": V, "dim": D,
                       "parallelism": f"rows sharded, {R}/GPU, no collective",
                       "l2": f"inputs larger than L2 ({qmm_gguf_bytes(V, D, t) / 1e6:.0f} MB of weights per step)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": None if traffic_ratio is None else round(traffic_ratio * bytes_per_step),
                         "traffic_source": traffic_src and f"{traffic_src} (ncu dram bytes per algorithmic byte, "
                                                           f"scaled to this step)",
                         "algorithmic_bytes_per_launch": bytes_per_step, "avg_step_us": round(step_s * 1e6, 2),
                         "kernel": "qtc_kernel (+ quantization, argmax)"},
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": int(args.steps * 4),
            "clocks": clocks.summary(),
        }
        line.update(rank_fields(rank_ms))
        print(json.dumps(line), flush=True)
    head.close()
    qw.close()


def headq_cpu_sample(cfg, seed, seconds):
    """Times the oracle's quantized product on one row over 1/64 of the
    vocabulary; returns rows/s scaled to the full head."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    rng = np.random.default_rng(seed)
    V, D, t = cfg["vocab"] // 64, cfg["dim"], cfg["qtype"]
    w = vx_oracle.random_qblocks(t, V, D, rng)
    x = rng.standard_normal((1, D)).astype(np.float32)
    vx_oracle.qmatmul(t, w, V, D, x)
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        vx_oracle.qmatmul(t, w, V, D, x)
        done += 1
    el = time.perf_counter() - t0
    return done / el / 64.0, done


def head_cpu_sample(cfg, seed, seconds):
    """Times the oracle's greedy head (float64 BLAS on all host cores) on 4
    rows over 1/8 of the vocabulary; returns rows/s scaled to the full head."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    rng = np.random.default_rng(seed)
    V, D = cfg["vocab"] // 8, cfg["dim"]
    w = (rng.standard_normal((V, D), dtype=np.float32) * 0.02).astype(np.float16).view(np.uint16)
    x = rng.standard_normal((4, D)).astype(np.float32)
    vx_oracle.logits_argmax(w, cfg["dtype"], x)
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        vx_oracle.logits_argmax(w, cfg["dtype"], x)
        done += 1
    el = time.perf_counter() - t0
    return 4 * done / el / 8.0, done


def write_decoder_gguf(path, cfg, seed):
    """A seeded Q4_K_M-typed decoder with the reference's tensor names and keys
    (src/voxtral.cpp:1097-1110, 1225-1252), written with the gguf package.
    Returns the host tensors (vx_decoder.Tensor) for the CPU sample."""
    import gguf

    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_decoder as vd
    import vx_oracle

    rng = np.random.default_rng(seed)
    L, D, H, V = cfg["layers"], cfg["dim"], cfg["hidden"], cfg["vocab"]
    gt = {vd.Q4_K: gguf.GGMLQuantizationType.Q4_K, vd.Q6_K: gguf.GGMLQuantizationType.Q6_K}
    w = gguf.GGUFWriter(str(path), "voxtral_realtime") if path else None
    if w is None:  # host tensors only (the CPU arm)
        class _NoWriter:
            def __getattr__(self, name):
                return lambda *a, **k: None
        w = _NoWriter()
    for k, v in (("dim", D), ("n_layers", L), ("n_heads", NQ), ("head_dim", HD), ("hidden_dim", H),
                 ("n_kv_heads", NKV)):
        w.add_int32(f"voxtral.decoder.{k}", v)
    w.add_float32("voxtral.decoder.norm_eps", 1e-5)
    w.add_float32("voxtral.decoder.rope_theta", 1e6)
    w.add_bool("voxtral.ada_rms_norm_t_cond", True)
    tensors = {}

    def mat(name, t, rows, cols):
        blocks = vx_oracle.random_qblocks(t, rows, cols, rng, zero_mean=True)
        tensors[name] = vd.Tensor(t, rows, cols, blocks)
        w.add_tensor(name, blocks, raw_dtype=gt[t])

    def vec(name, n):
        a = rng.uniform(0.8, 1.2, n).astype(np.float32)
        tensors[name] = vd.Tensor(vd.F32, 1, n, a)
        w.add_tensor(name, a)

    mat("tok_embeddings.weight", vd.Q6_K, V, D)
    for l in range(L):
        p = f"dec.blk.{l}."
        mat(p + "attn_q.weight", vd.Q4_K, NQ * HD, D)
        mat(p + "attn_k.weight", vd.Q4_K, NKV * HD, D)
        mat(p + "attn_v.weight", vd.Q6_K, NKV * HD, D)
        mat(p + "attn_o.weight", vd.Q4_K, D, NQ * HD)
        mat(p + "ffn_w1.weight", vd.Q4_K, H, D)
        mat(p + "ffn_w3.weight", vd.Q4_K, H, D)
        mat(p + "ffn_w2.weight", vd.Q6_K, D, H)
        mat(p + "ada0.weight", vd.Q4_K, 32, D)
        a2 = rng.normal(0, 1.0 / np.sqrt(32), (D, 32)).astype(np.float16)
        tensors[p + "ada2.weight"] = vd.Tensor(vd.F16, D, 32, a2)
        w.add_tensor(p + "ada2.weight", a2)
        vec(p + "attn_norm.weight", D)
        vec(p + "ffn_norm.weight", D)
    vec("dec.norm.weight", D)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


def write_encoder_gguf(path, cfg, seed):
    """A seeded Q4_K_M-typed streaming encoder with the reference's tensor names
    and keys (src/voxtral.cpp:1085-1095, 1190-1222), written with the gguf package."""
    import gguf

    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    rng = np.random.default_rng(seed)
    L, D, H, F = cfg["layers"], cfg["dim"], cfg["heads"], cfg["hidden"]
    qd = H * 64
    q4, q6 = gguf.GGMLQuantizationType.Q4_K, gguf.GGMLQuantizationType.Q6_K
    w = gguf.GGUFWriter(str(path), "voxtral_realtime")
    for k, v in (("dim", D), ("n_layers", L), ("n_heads", H), ("head_dim", 64), ("hidden_dim", F), ("n_kv_heads", H)):
        w.add_int32(f"voxtral.encoder.{k}", v)
    w.add_float32("voxtral.encoder.norm_eps", 1e-5)
    w.add_float32("voxtral.encoder.rope_theta", 1e6)

    def mat(name, t, gt, rows, cols):
        w.add_tensor(name, vx_oracle.random_qblocks(t, rows, cols, rng, zero_mean=True), raw_dtype=gt)

    def vec(name, n, lo, hi):
        w.add_tensor(name, rng.uniform(lo, hi, n).astype(np.float32))

    w.add_tensor("enc.conv0.weight", rng.normal(0, 1 / np.sqrt(384), (D, 128, 3)).astype(np.float16))
    vec("enc.conv0.bias", D, -0.1, 0.1)
    w.add_tensor("enc.conv1.weight", rng.normal(0, 1 / np.sqrt(3 * D), (D, D, 3)).astype(np.float16))
    vec("enc.conv1.bias", D, -0.1, 0.1)
    for l in range(L):
        p = f"enc.blk.{l}."
        mat(p + "attn_q.weight", 12, q4, qd, D)
        mat(p + "attn_k.weight", 12, q4, qd, D)
        mat(p + "attn_v.weight", 14, q6, qd, D)
        mat(p + "attn_o.weight", 12, q4, D, qd)
        mat(p + "ffn_w1.weight", 12, q4, F, D)
        mat(p + "ffn_w3.weight", 12, q4, F, D)
        mat(p + "ffn_w2.weight", 14, q6, D, F)
        vec(p + "attn_q.bias", qd, -0.1, 0.1)
        vec(p + "attn_v.bias", qd, -0.1, 0.1)
        vec(p + "attn_o.bias", D, -0.1, 0.1)
        vec(p + "ffn_w2.bias", D, -0.1, 0.1)
        vec(p + "attn_norm.weight", D, 0.8, 1.2)
        vec(p + "ffn_norm.weight", D, 0.8, 1.2)
    vec("enc.norm.weight", D, 0.8, 1.2)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def encoder_cpu_stack_sample(cfg, seed, seconds):
    """Times the oracle's whole encoder step (oracle/vx_decoder.py Encoder: conv stem,
    every layer with fp64 window attention over a prefilled 750-frame history, final
    norm) on one stream's 4-frame chunk, one thread; returns (chunks/s, chunks)."""
    import tempfile

    import gguf

    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_decoder as vd
    import vx_oracle

    path = Path(tempfile.mkdtemp(prefix="vxk_cpu_")) / "enc.gguf"
    write_encoder_gguf(path, cfg, seed)
    r = gguf.GGUFReader(str(path))
    tensors = {}
    for t in r.tensors:
        ne = [int(v) for v in t.shape]
        qt = int(t.tensor_type)
        data = np.asarray(t.data)
        rows = int(np.prod(ne[1:])) if len(ne) > 1 else 1
        cols = ne[0]
        if qt in (vd.Q8_0, vd.Q4_K, vd.Q6_K):
            tensors[t.name] = vd.Tensor(qt, rows, cols, data.reshape(rows, -1).copy())
        elif len(ne) == 3:
            tensors[t.name] = vd.Tensor(qt, ne[2], ne[1] * ne[0], data.reshape(ne[2], ne[1], ne[0]).copy())
        else:
            tensors[t.name] = vd.Tensor(qt, rows, cols, data.copy())
    os.unlink(path)
    H, W, P = cfg["heads"], cfg["window"], cfg["rows"]
    enc = vd.Encoder(tensors, cfg["layers"], H, cache_dtype=cfg["dtype"], window=W)
    rng = np.random.default_rng(seed + 3)
    q0 = W
    rb = H * 64 * 2
    for l in range(cfg["layers"]):
        kk = rng.normal(0, 0.5, (W, H * 64)).astype(np.float32)
        bits = vx_oracle.f32_to_bf16_bits(kk).view(np.uint8).reshape(W, rb)
        for j in range(W):
            enc.hist[(0, l, q0 - W + j)] = (bits[j], bits[(j + 1) % W])
    mel = rng.normal(0, 1, (128, 2 * P + 4)).astype(np.float32)
    done, t0 = 0, time.perf_counter()
    while True:
        enc.forward([(0, q0 + done * P, P, mel)])
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 4:
            break
    return done / el, done


def encoder_weight_bytes(cfg):
    L, D, F, qd = cfg["layers"], cfg["dim"], cfg["hidden"], cfg["heads"] * 64
    q4 = lambda n, k: n * (k // 256) * 144  # noqa: E731
    q6 = lambda n, k: n * (k // 256) * 210  # noqa: E731
    return L * (2 * q4(qd, D) + q6(qd, D) + q4(D, qd) + 2 * q4(F, D) + q6(D, F)) + 2 * (128 * 3 * D + 3 * D * D)


def run_encstack(args, cfg, world, rank, local, dist, torch, vxk):
    """Whole streaming encoder step: one 80 ms chunk (4 new frames) of every
    stream through the conv stem, all layers and the final norm
    (vxk_encoder_forward), rings prefilled so every window holds 750 frames."""
    import tempfile

    L, S, H, P, W, CAP = cfg["layers"], cfg["streams"], cfg["heads"], cfg["rows"], cfg["window"], cfg["capacity"]
    tmpdir = tempfile.mkdtemp(prefix="vxk_bench_")
    path = Path(tmpdir) / f"encoder_{rank}.gguf"
    write_encoder_gguf(path, cfg, args.seed)
    pool = vxk.EncPool(device=local, n_layers=L, n_heads=H, head_dim=64, window=W, capacity=CAP, max_streams=S,
                       max_new=CAP - W, dtype=cfg["dtype"], max_position=65536)
    g = vxk.Gguf(path)
    enc = vxk.Encoder(g, pool, max_rows=S * P)
    g.close()
    os.unlink(path)
    os.rmdir(tmpdir)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    streams = [pool.open_stream() for _ in range(S)]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed + rank)
    fill = CAP - W
    fq = torch.randn((S * fill, H, 64), device="cuda", generator=gen) * 0.5
    fo = torch.empty_like(fq)
    pos = 0
    while pos < CAP + 128:  # wrap every ring so each chunk sees a full 750-frame window
        pool.plan(streams, [fill] * S, sh)
        for layer in range(L):
            pool.layer(layer, fq.data_ptr(), fq.data_ptr(), fq.data_ptr(), fo.data_ptr(), sh)
        pool.commit()
        pos += fill
    torch.cuda.synchronize()
    del fq, fo
    mel = torch.randn((S, 128, 2 * P + 4), device="cuda", generator=gen)
    out = torch.empty((S * P, cfg["dim"]), device="cuda")

    def step():
        pool.plan(streams, [P] * S, sh)
        enc.forward(mel.data_ptr(), out.data_ptr(), sh)
        pool.commit()

    for _ in range(args.warmup):
        step()
    enc.sync(sh)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    props = torch.cuda.get_device_properties(local)
    gpu_id = str(getattr(props, "uuid", local))
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    enc.sync(sh)
    rank_ms = gather_over_ranks(dist, e0.elapsed_time(e1), "cuda")
    ms = max(rank_ms)
    step_s = ms / 1000.0 / args.steps
    w_bytes = encoder_weight_bytes(cfg)
    keys = W + P - 1
    ring_bytes = L * S * keys * H * 64 * 2 * 2
    rows = S * P
    flops = 2 * rows * (w_bytes * 0 + L * (4 * H * 64 * cfg["dim"] + 3 * cfg["dim"] * cfg["hidden"])) \
        + L * S * P * H * keys * 64 * 4
    e2e = None
    if not args.no_e2e:
        hmel = torch.randn((S, 128, 2 * P + 4)).pin_memory()
        hout = torch.empty((S * P, cfg["dim"])).pin_memory()

        def host_step():
            mel.copy_(hmel, non_blocking=True)
            step()
            hout.copy_(out, non_blocking=True)

        host_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            host_step()
        f1.record(stream)
        torch.cuda.synchronize()
        ems = max_over_ranks(dist, f0.elapsed_time(f1), "cuda")
        e2e = {"value": round(world * S * args.steps / (ems / 1000.0), 1), "unit": "stream-chunks/s",
               "h2d_bytes_per_step": int(hmel.numel()) * 4, "d2h_bytes_per_step": int(hout.numel()) * 4,
               "ms_per_step": round(ems / args.steps, 4)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cps, done = encoder_cpu_stack_sample(cfg, args.seed, args.cpu_seconds)
        cpu = {"value": round(cps, 5), "unit": "stream-chunks/s", "cores": 1, "kind": "port",
               "sample": f"{done} chunks of one stream (4 frames, 750-frame window) through the conv stem, all "
                         f"{L} layers and the final norm by the oracle (oracle/vx_decoder.py Encoder, one thread)"}
    if dist:
        dist.barrier()
    if rank == 0:
        peak, peak_kind = load_peaks()
        achieved = (w_bytes + ring_bytes) / step_s / 1e9
        line = {
            "metric": "whole encoder step stream-chunks/s (conv stem + 32 layers + norm, 4 frames per chunk)",
            "value": round(world * S * args.steps / (ms / 1000.0), 1),
            "unit": "stream-chunks/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "Q4_K / Q6_K weights with Q8_K rows, f16 conv operands, bf16 rings, fp32 activations",
            "data": "synthetic",
            "config": {"workload": f"config encstack: {cfg['desc']}", "layers": L, "streams_per_gpu": S,
                       "parallelism": f"streams sharded, {S}/GPU, no collective",
                       "l2": f"inputs larger than L2 ({ring_bytes / 1e6:.0f} MB of ring reads per step)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "algorithmic_bytes_per_step": int(w_bytes + ring_bytes),
                         "tflops": round(flops / step_s / 1e12, 2), "avg_step_us": round(step_s * 1e6, 1),
                         "kernel": "whole step (all kernels); products re-stream their weights per 64-row chunk"},
            "cpu_baseline": cpu, "e2e": e2e,
            # conv stem (2), the first norm (quantizing into layer 0's q/k/v tiles), per layer (q/k/v
            # product, attention with the fused ring append, o quantize + product, norm into the
            # w1/w3 tiles, w1/w3 product, w2 quantize + product, norm)
            "gpu_launches": int(args.steps * (2 + 1 + L * 9)),
            "launch": "eager C-ABI calls per step: vxk_enc_batch_plan, vxk_encoder_forward, vxk_enc_batch_commit",
            "clocks": clocks.summary(),
        }
        line.update(rank_fields(rank_ms))
        print(json.dumps(line), flush=True)
    enc.close()
    pool.close()


def decoder_weight_bytes(cfg):
    """GGUF bytes of every matrix one decoder step streams (all layers + head)."""
    L, D, H, V = cfg["layers"], cfg["dim"], cfg["hidden"], cfg["vocab"]
    q4 = lambda n, k: n * (k // 256) * 144  # noqa: E731
    q6 = lambda n, k: n * (k // 256) * 210  # noqa: E731
    per_layer = (q4(NQ * HD, D) + q4(NKV * HD, D) + q6(NKV * HD, D) + q4(D, NQ * HD) + 2 * q4(H, D) + q6(D, H))
    return L * per_layer + q6(V, D)


def run_decoder(args, cfg, world, rank, local, dist, torch, vxk):
    """Whole decoder step: one step = one token of every stream through the
    embeddings, all layers and the greedy head (vxk_decoder_forward over the
    pool's planned batch), caches prefilled to seeded contexts."""
    import tempfile

    L, S, cap = cfg["layers"], cfg["streams"], cfg["capacity"]
    tmpdir = tempfile.mkdtemp(prefix="vxk_bench_")
    path = Path(tmpdir) / f"decoder_{rank}.gguf"
    tensors = write_decoder_gguf(path, cfg, args.seed)
    rng = np.random.default_rng(args.seed)
    lo, hi = cfg["ctx"]
    ctx_all = rng.integers(lo, hi + 1, size=S * world)
    ctx0 = ctx_all[assign_streams(ctx_all, world, S)[rank]]
    total_steps = args.warmup + args.steps * (1 if args.no_e2e else 2) + 2
    pages = [min(cap // BT, (int(c) + total_steps) // BT + 2) for c in ctx0]
    prefill_chunk = min(int(ctx0.max()), 4096)
    pool = vxk.Pool(device=local, n_layers=L, n_q_heads=NQ, n_kv_heads=NKV, head_dim=HD, block_tokens=BT,
                    capacity=cap, n_blocks=int(sum(pages)) + 64, max_streams=S, max_rows=max(S, prefill_chunk),
                    max_position=int(ctx0.max()) + total_steps + BT + 16, dtype=cfg["dtype"], alloc_seed=1234 + rank)
    g = vxk.Gguf(path)
    dec = vxk.Decoder(g, pool, audio_capacity=256, enc_capacity=0)
    g.close()
    os.unlink(path)
    os.rmdir(tmpdir)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    streams = [pool.open_stream() for _ in range(S)]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed + rank)
    kfill = torch.randn((prefill_chunk, NKV, HD), device="cuda", generator=gen) * 0.5
    vfill = torch.randn((prefill_chunk, NKV, HD), device="cuda", generator=gen) * 0.5
    for s, c in zip(streams, ctx0):
        left = int(c)
        while left > 0:
            n = min(left, prefill_chunk)
            pool.plan([s], [n], sh)
            for layer in range(L):
                pool.append_layer(layer, kfill.data_ptr(), vfill.data_ptr(), sh)
            pool.commit()
            left -= n
    audio = torch.randn((256, cfg["dim"]), device="cuda", generator=gen) * 0.05
    for s in streams:
        dec.write_audio(s, 0, 256, audio.data_ptr(), sh)
    torch.cuda.synchronize()
    del kfill, vfill
    ones = [1] * S
    pos = [int(c) for c in ctx0]
    tok_rng = np.random.default_rng(args.seed + 7 + rank)
    tokens = [int(t) for t in tok_rng.integers(0, cfg["vocab"], S)]
    amax = torch.zeros(S, dtype=torch.int32, device="cuda")

    def step():
        pool.plan(streams, ones, sh)
        dec.forward(tokens, [p % 256 for p in pos], amax.data_ptr(), 0, 0, sh)
        pool.commit()
        for j in range(S):
            pos[j] += 1

    for _ in range(args.warmup):
        step()
    dec.sync(sh)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    props = torch.cuda.get_device_properties(local)
    gpu_id = str(getattr(props, "uuid", local))
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    ctx_sum = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step()
            ctx_sum.append(sum(min(cap, p) for p in pos))
        e1.record(stream)
        torch.cuda.synchronize()
    dec.sync(sh)
    rank_ms = gather_over_ranks(dist, e0.elapsed_time(e1), "cuda")
    ms = max(rank_ms)
    step_s = ms / 1000.0 / args.steps
    w_bytes = decoder_weight_bytes(cfg)
    kv_bytes = L * 4096 * statistics.mean(ctx_sum)
    # per row and layer: x / xn / q / k / v / att / proj / gate / up / ffn fp32 reads and writes, the append
    act_bytes = S * L * 4 * (6 * cfg["dim"] + 3 * NQ * HD + 4 * NKV * HD + 4 * cfg["hidden"]) + S * L * 4096
    bytes_per_step = w_bytes + kv_bytes + act_bytes
    achieved = bytes_per_step / step_s / 1e9
    peak, peak_kind = load_peaks()
    traffic_ratio, traffic_src = load_traffic(args.config)

    e2e = None
    if not args.no_e2e:
        # the serving loop through the public API: tokens from the previous
        # step's argmax read back to the host (4 bytes per stream), as the
        # reference's hot loop does
        host_amax = torch.zeros(S, dtype=torch.int32).pin_memory()
        toks = list(tokens)

        def host_step():
            pool.plan(streams, ones, sh)
            dec.forward(toks, [p % 256 for p in pos], amax.data_ptr(), 0, 0, sh)
            host_amax.copy_(amax, non_blocking=True)
            stream.synchronize()
            pool.commit()
            for j in range(S):
                pos[j] += 1
            toks[:] = [int(t) for t in host_amax.tolist()]

        host_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            host_step()
        f1.record(stream)
        torch.cuda.synchronize()
        ems = max_over_ranks(dist, f0.elapsed_time(f1), "cuda")
        e2e = {"value": round(world * S * args.steps / (ems / 1000.0), 1), "unit": "tokens/s",
               "h2d_bytes_per_step": S * 8 + S * 16, "d2h_bytes_per_step": S * 4,
               "ms_per_step": round(ems / args.steps, 4)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, done, mctx = decoder_cpu_sample(tensors, cfg, int(statistics.mean([int(c) for c in ctx0])),
                                             args.seed, args.cpu_seconds)
        cpu = {"value": round(tps, 5), "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": f"{done} single-token steps of one stream (cache prefilled to ctx {mctx}) through all "
                         f"{L} layers and the head by the oracle (oracle/vx_decoder.py over vx_qmm.c / vx_oracle.c, "
                         f"one thread)"}
    del tensors
    if dist:
        dist.barrier()
    if rank == 0:
        per_layer = 8
        line = {
            "metric": "whole decoder step tokens/s (Q4_K_M, 26 layers + head)",
            "value": round(world * S * args.steps / (ms / 1000.0), 1),
            "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "Q4_K / Q6_K weights with Q8_K rows (exact integer dots), f16 KV cache, fp32 activations",
            "data": "synthetic",
            "config": {"workload": f"config decoder: {cfg['desc']}", "layers": L, "streams_per_gpu": S,
                       "mean_ctx_timed": round(statistics.mean(ctx_sum) / S, 1),
                       "parallelism": f"streams sharded, {S}/GPU, no collective",
                       "l2": f"inputs larger than L2 ({w_bytes / 1e9:.2f} GB of weights per step)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": None if traffic_ratio is None else round(traffic_ratio * bytes_per_step),
                         "traffic_source": traffic_src,
                         "algorithmic_bytes_per_step": round(bytes_per_step),
                         "weight_bytes": w_bytes, "kv_bytes": round(kv_bytes),
                         "avg_step_us": round(step_s * 1e6, 1), "kernel": "whole step (all kernels)"},
            "cpu_baseline": cpu, "e2e": e2e,
            # embed, layer 0's q/k/v quantization, per layer (q/k/v product, attention quantizing
            # its output into the o tiles, o product, norm quantizing into the w1/w3 tiles, w1/w3
            # product, w2 quantize (SwiGLU inside) + product, norm quantizing into the next q/k/v
            # tiles), head (quantize, product, argmax, token ids)
            "gpu_launches": int(args.steps * (1 + 1 + per_layer * L + 4)),
            "launch": "eager C-ABI calls per step: vxk_batch_plan, vxk_decoder_forward, vxk_batch_commit",
            "clocks": clocks.summary(),
        }
        line.update(rank_fields(rank_ms))
        print(json.dumps(line), flush=True)
    dec.close()
    pool.close()


def decoder_cpu_sample(tensors, cfg, ctx, seed, seconds):
    """Times the oracle's whole decoder step on one stream whose cache holds
    ctx random rows; returns (tokens/s, steps, ctx)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_decoder as vd

    rng = np.random.default_rng(seed + 11)
    ref = vd.Decoder(tensors, cfg["layers"], capacity=cfg["capacity"])
    st = ref.stream(0)
    rb = NKV * HD * 2
    for l in range(cfg["layers"]):
        kk = rng.normal(0, 0.5, (ctx, NKV * HD)).astype(np.float16).view(np.uint8).reshape(ctx, rb)
        vv = rng.normal(0, 0.5, (ctx, NKV * HD)).astype(np.float16).view(np.uint8).reshape(ctx, rb)
        st.k[l] = list(kk)
        st.v[l] = list(vv)
    st.next_pos = ctx
    done = 0
    t0 = time.perf_counter()
    while True:
        ref.forward([(0, [int(rng.integers(0, cfg["vocab"]))])],
                    rng.normal(0, 0.05, (1, cfg["dim"])).astype(np.float32))
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 8:
            break
    return done / el, done, ctx


def rank_fields(rank_ms):
    """Every rank's timed-region milliseconds and the slowest rank, which sets
    the job's time (the data plane has no collective)."""
    return {"rank_ms": [round(float(x), 3) for x in rank_ms], "slowest_rank": int(np.argmax(rank_ms))}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["vxk", "reference"], default="vxk")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="2")
    ap.add_argument("--streams", type=int, default=0, help="override streams per GPU")
    ap.add_argument("--layers", type=int, default=0, help="override decoder layers (profiling small cases)")
    ap.add_argument("--vocab", type=int, default=0, help="override the greedy head's vocabulary (profiling)")
    ap.add_argument("--seed", type=int, default=20261201)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--cache", choices=["f16", "q8_0", "f32", "bf16"], default=None,
                    help="override the cache format: decoder configs 2, 3, 5 (f16, q8_0, f32); encoder config 4 "
                         "(bf16, f16, f32)")
    return ap.parse_args()


def algorithmic_bytes(ctx: int, dtype: int) -> int:
    """Bytes one decode token must move in one layer (per-layer figure of the
    unit): K+V window reads + q/k/v fp32 reads + append write + fp32 output."""
    if dtype == 8:
        return 2176 * ctx + 43136
    if dtype == 0:
        return 8192 * ctx + 49152
    return 4096 * ctx + 45056


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


TRAFFIC_PROFILES = {
    "2": "decode_kernel_f16_config2.md",
    "3": "decode_kernel_f16_config2.md",   # same kernel and page format; ratio scaled to config 3
    "5": "decode_kernel_q8_0_config5.md",
    "4": "enc_tc_kernel_config4.md",
    "head": "head_kernel_config_head.md",
    "proj": "qmm_kernel_config_proj.md",
    "headq": "qtc_kernel_config_headq.md",
    "decoder": "decoder_step_config_decoder.md",
}


def load_traffic(config: str):
    """DRAM bytes per algorithmic byte of the dominant kernel, read from the
    `dram_bytes_per_algorithmic_byte:` line of its committed ncu summary
    (dram__bytes_read.sum + dram__bytes_write.sum of one captured launch over
    that launch's algorithmic bytes).  Returns (ratio, file) or (None, None)."""
    name = TRAFFIC_PROFILES.get(config)
    p = ROOT / "profiles" / name if name else None
    if p is None or not p.exists():
        return None, None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_algorithmic_byte:"):
            try:
                return float(line.split(":", 1)[1]), f"profiles/{name}"
            except ValueError:
                break
    return None, None


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            if self.thread:
                self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_sample(layers, ctx0, seed, seconds=None, steps=None, warmup=0, dtype=1):
    """Times the CPU restatement (oracle/vx_cpu_step.c) of the same decode
    step on all host cores, for an f16 (1) or q8_0 (8) cache, over streams
    whose starting contexts are `ctx0`.  Returns (tokens/s, steps done,
    threads, mean context, algorithmic bytes/s)."""
    if dtype not in (1, 8):
        raise ValueError("the CPU step restates the f16 and q8_0 caches only")
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    rng = np.random.default_rng(seed)
    ctx0 = np.asarray(ctx0, dtype=np.int64)
    n_streams = len(ctx0)
    total = (steps or 0) + warmup + 64
    cap = int(ctx0.max()) + total + 16
    if dtype == 8:
        # rows of ggml q8_0 blocks (34 B per 32 values), tiled from quantized noise
        row_b = HD // 32 * 34
        shape = (n_streams, layers, NKV, cap, row_b)
        src = (rng.standard_normal(1 << 20).astype(np.float32) * 0.5)
        block = np.ascontiguousarray(vx_oracle.quantize_q8_0(src), dtype=np.uint8).reshape(-1)
        kc = np.resize(block, int(np.prod(shape))).reshape(shape)
        vc = np.resize(block, int(np.prod(shape))).reshape(shape)
    else:
        shape = (n_streams, layers, NKV, cap, HD)
        block = (rng.standard_normal(1 << 22).astype(np.float32) * 0.5).astype(np.float16).view(np.uint16)
        kc = np.resize(block, int(np.prod(shape))).reshape(shape).view(np.uint8)
        vc = np.resize(block[::-1], int(np.prod(shape))).reshape(shape).view(np.uint8)
    q = rng.standard_normal((n_streams, layers, NQ, HD), dtype=np.float32) * 0.5
    k = rng.standard_normal((n_streams, layers, NKV, HD), dtype=np.float32) * 0.5
    v = rng.standard_normal((n_streams, layers, NKV, HD), dtype=np.float32) * 0.5
    rope = vx_oracle.rope_table(cap + 1, HD, 1e6)
    pos = ctx0.copy()
    win = np.zeros(n_streams, dtype=np.int64)
    threads = os.cpu_count() or 1
    scale = float(np.float32(1.0 / np.sqrt(HD)))
    for _ in range(warmup):
        vx_oracle.cpu_decode_step(dtype, kc, vc, q, k, v, pos, win, rope, scale, threads)
        pos += 1
    done = 0
    nbytes = 0
    t0 = time.perf_counter()
    while True:
        vx_oracle.cpu_decode_step(dtype, kc, vc, q, k, v, pos, win, rope, scale, threads)
        nbytes += layers * sum(algorithmic_bytes(int(p) + 1, dtype) for p in pos)
        pos += 1
        done += 1
        el = time.perf_counter() - t0
        if steps is not None and done >= steps:
            break
        if seconds is not None and el >= seconds:
            break
    el = time.perf_counter() - t0
    return n_streams * done / el, done, threads, float(np.mean(ctx0)), nbytes / el


def cpu_streams(dtype: int) -> int:
    """Streams in the CPU sample: 4, or 2 for the q8_0 config whose contexts
    (up to 32K positions x 30 layers) would otherwise need > 8 GB of host memory."""
    return 2 if dtype == 8 else 4


def sample_contexts(ctx, n):
    """n contexts taken from `ctx` at the centres of n equal quantile bins of
    its sorted order, so the sample's mean context follows the job's."""
    srt = sorted(int(c) for c in ctx)
    return [srt[min(len(srt) - 1, int((i + 0.5) * len(srt) / n))] for i in range(n)]


def job_layout(cfg, seed, world):
    """The decode job: every stream's starting context, drawn once from the
    seed, and the streams each rank owns (longest-processing-time).  Configs
    with `total_streams` fix the job's total (strong scaling); the others have
    `streams` per GPU (weak scaling).  Returns (ctx_all, parts, scaling)."""
    rng = np.random.default_rng(seed)
    lo, hi = cfg["ctx"]
    if cfg.get("total_streams"):
        total = int(cfg["total_streams"])
        per = -(-total // world)
        scaling = "strong"
    else:
        per = int(cfg["streams"])
        total = per * world
        scaling = "weak"
    ctx_all = rng.integers(lo, hi + 1, size=total)
    return ctx_all, assign_streams(ctx_all, world, per), scaling


def decode_config(args, cfg, world, ctx_all, parts, scaling):
    """The `config` object of a decode line: the same for both arms."""
    per = max(len(p) for p in parts)
    par = f"streams sharded by stream, {per}/GPU, no collective"
    return {"workload": f"config {args.config}: {cfg['desc']}", "layers": cfg["layers"],
            "streams_total": int(len(ctx_all)), "streams_per_gpu": per, "global_batch": int(len(ctx_all)),
            "ctx_range": list(cfg["ctx"]), "mean_ctx_job": round(float(np.mean(ctx_all)), 1),
            "scaling": scaling, "parallelism": par,
            "l2": "inputs larger than L2 (KV read per launch >> 126 MB), no flush"}


def encoder_cpu_sample(cfg, seed, seconds):
    """Times the CPU restatement (oracle attention, one thread) of one
    stream-layer of a config-4 chunk; returns stream-chunks/s for all layers."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    rng = np.random.default_rng(seed)
    H, P, W = cfg["heads"], cfg["rows"], cfg["window"]
    keys = W + P - 1
    kr = vx_oracle.f32_to_bf16_bits(rng.standard_normal((keys, H * 64), dtype=np.float32) * 0.5).view(np.uint8)
    vr = vx_oracle.f32_to_bf16_bits(rng.standard_normal((keys, H * 64), dtype=np.float32) * 0.5).view(np.uint8)
    q = rng.standard_normal((H, 64), dtype=np.float32) * 0.5
    scale = float(np.float32(0.125))
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        for j in range(P):  # the chunk's rows, each over its own window
            lo = j
            vx_oracle.attn_row(q, 10000 + j, 1e6, kr[lo:lo + W], vr[lo:lo + W], vx_oracle.BF16, H, scale)
        done += 1
    el = time.perf_counter() - t0
    return done / el / cfg["layers"], done


def run_reference(args, cfg, rank, world):
    if rank != 0:
        return
    if cfg.get("kind") == "head":
        cps, done = head_cpu_sample(cfg, args.seed, 20.0)
        line = {"impl": "reference", "metric": "greedy head rows/s (tied logits + argmax)",
                "value": round(cps, 4), "unit": "rows/s", "n_gpus": args.gpus, "steps": done, "warmup": 1,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16 weights, float64 accumulate", "data": "synthetic",
                "config": {"workload": f"config head: {cfg['desc']}"},
                "cpu_baseline": {"value": round(cps, 4), "unit": "rows/s", "cores": os.cpu_count() or 1,
                                 "kind": "port",
                                 "sample": f"{done} steps of 4 rows over 1/8 of the vocabulary (oracle.logits_argmax, "
                                           f"float64 BLAS), scaled"},
                "e2e": {"value": round(cps, 4), "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if cfg.get("kind") == "headq":
        cps, done = headq_cpu_sample(cfg, args.seed, 20.0)
        line = {"impl": "reference", "metric": "greedy head rows/s (Q6_K tied logits + argmax)",
                "value": round(cps, 4), "unit": "rows/s", "n_gpus": args.gpus, "steps": done, "warmup": 1,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "Q6_K weights, Q8_K rows, exact integer dots", "data": "synthetic",
                "config": {"workload": f"config headq: {cfg['desc']}"},
                "cpu_baseline": {"value": round(cps, 4), "unit": "rows/s", "cores": 1, "kind": "port",
                                 "sample": f"{done} single-row products over 1/64 of the vocabulary by the oracle "
                                           f"(oracle/vx_qmm.c), scaled"},
                "e2e": {"value": round(cps, 4), "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if cfg.get("kind") == "qmm":
        tps, done = qmm_cpu_sample(cfg, args.seed, 20.0)
        line = {"impl": "reference", "metric": "attention-projection tokens/s (q/k/v/o, Q4_K_M, 30 layers)",
                "value": round(tps, 4), "unit": "tokens/s", "n_gpus": args.gpus, "steps": done, "warmup": 1,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "Q4_K / Q6_K weights, Q8_K rows, exact integer dots", "data": "synthetic",
                "config": {"workload": f"config proj: {cfg['desc']}"},
                "cpu_baseline": {"value": round(tps, 4), "unit": "tokens/s", "cores": 1, "kind": "port",
                                 "sample": f"{done} single-row products of the k projection by the oracle "
                                           f"(oracle/vx_qmm.c), scaled by weight count"},
                "e2e": {"value": round(tps, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if cfg.get("kind") == "encstack":
        cps, done = encoder_cpu_stack_sample(cfg, args.seed, 20.0)
        line = {"impl": "reference", "metric": "whole encoder step stream-chunks/s (conv stem + 32 layers + norm, "
                                               "4 frames per chunk)",
                "value": round(cps, 5), "unit": "stream-chunks/s", "n_gpus": args.gpus, "steps": done, "warmup": 0,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "Q4_K / Q6_K weights, Q8_K rows, exact integer dots, fp64 attention", "data": "synthetic",
                "config": {"workload": f"config encstack: {cfg['desc']}"},
                "cpu_baseline": {"value": round(cps, 5), "unit": "stream-chunks/s", "cores": 1, "kind": "port",
                                 "sample": f"{done} chunks of one stream through the stem, every layer and the norm by "
                                           f"the oracle (oracle/vx_decoder.py Encoder, one thread)"},
                "e2e": {"value": round(cps, 5), "unit": "stream-chunks/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if cfg.get("kind") == "decoder":
        tensors = write_decoder_gguf(None, cfg, args.seed)
        rng = np.random.default_rng(args.seed)
        lo, hi = cfg["ctx"]
        mctx = int(rng.integers(lo, hi + 1, size=cfg["streams"]).mean())
        tps, done, mctx = decoder_cpu_sample(tensors, cfg, mctx, args.seed, 20.0)
        line = {"impl": "reference", "metric": "whole decoder step tokens/s (Q4_K_M, 26 layers + head)",
                "value": round(tps, 5), "unit": "tokens/s", "n_gpus": args.gpus, "steps": done, "warmup": 0,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "Q4_K / Q6_K weights, Q8_K rows, exact integer dots, fp64 attention", "data": "synthetic",
                "config": {"workload": f"config decoder: {cfg['desc']}"},
                "cpu_baseline": {"value": round(tps, 5), "unit": "tokens/s", "cores": 1, "kind": "port",
                                 "sample": f"{done} single-token steps of one stream (ctx {mctx}) through every layer "
                                           f"and the head by the oracle (oracle/vx_decoder.py, one thread)"},
                "e2e": {"value": round(tps, 5), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if cfg.get("kind") == "encoder":
        cps, done = encoder_cpu_sample(cfg, args.seed, 20.0)
        line = {"impl": "reference", "metric": "encoder chunks/s (KV append + windowed attention, 4 rows/chunk)",
                "value": round(cps, 4), "unit": "stream-chunks/s", "n_gpus": args.gpus, "steps": done,
                "warmup": 0, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16 ring, fp64 accumulate", "data": "synthetic",
                "config": {"workload": f"config {args.config}: {cfg['desc']}", "layers": cfg["layers"]},
                "cpu_baseline": {"value": round(cps, 4), "unit": "stream-chunks/s", "cores": 1, "kind": "port",
                                 "sample": f"{done} stream-layer chunks of the oracle's window attention, "
                                           f"one thread, scaled to {cfg['layers']} layers"},
                "e2e": {"value": round(cps, 4), "unit": "stream-chunks/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    ctx_all, parts, scaling = job_layout(cfg, args.seed, world)
    sample = sample_contexts(ctx_all[parts[0]], cpu_streams(cfg["dtype"]))
    budget = 150.0
    tps, done, threads, mean_ctx, bps = cpu_sample(cfg["layers"], sample, args.seed, seconds=budget,
                                                   steps=args.steps, warmup=min(args.warmup, 3), dtype=cfg["dtype"])
    line = {
        "impl": "reference",
        "metric": "decode tokens/s (KV append+GQA attn)",
        "value": round(tps, 3),
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": done,
        "warmup": min(args.warmup, 3),
        "ms_per_step": round(1000.0 * len(sample) / tps, 3),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": ("q8_0" if cfg["dtype"] == 8 else "f16") + " cache, fp32 accumulate",
        "data": "synthetic",
        "config": decode_config(args, cfg, world, ctx_all, parts, scaling),
        "bytes_per_s": round(bps, 1),
        "cpu_baseline": {"value": round(tps, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "bytes_per_s": round(bps, 1),
                         "sample": f"{len(sample)} streams of rank 0's share of the job (starting contexts "
                                   f"{sample}, quantile centres of the job's seeded list, mean {mean_ctx:.0f}) x "
                                   f"{cfg['layers']} layers x {done} steps of the CPU restatement "
                                   f"(oracle/vx_cpu_step.c), ggml absent"},
        "e2e": {"value": round(tps, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    cfg = dict(CONFIGS[args.config])
    if args.streams:
        cfg["total_streams" if cfg.get("total_streams") else "streams"] = args.streams
        if cfg.get("kind") == "qmm":
            cfg["rows"] = args.streams
    if args.layers:
        cfg["layers"] = args.layers
    if args.vocab:
        cfg["vocab"] = args.vocab
    if args.cache and "dtype" in cfg and cfg.get("kind") in (None, "encoder"):
        if cfg.get("kind") == "encoder":
            cfg["dtype"] = {"f16": 1, "bf16": 30, "f32": 0}[args.cache]
        else:
            cfg["dtype"] = {"f16": 1, "q8_0": 8, "f32": 0}[args.cache]
        cfg["desc"] += f" ({args.cache} cache)"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    import vxk

    if cfg.get("kind") == "head":
        run_head(args, cfg, world, rank, local, dist, torch, vxk)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    if cfg.get("kind") == "headq":
        run_headq(args, cfg, world, rank, local, dist, torch, vxk)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    if cfg.get("kind") == "qmm":
        run_qmm(args, cfg, world, rank, local, dist, torch, vxk)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    if cfg.get("kind") == "encstack":
        run_encstack(args, cfg, world, rank, local, dist, torch, vxk)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    if cfg.get("kind") == "decoder":
        run_decoder(args, cfg, world, rank, local, dist, torch, vxk)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    if cfg.get("kind") == "encoder":
        run_encoder(args, cfg, world, rank, local, dist, torch, vxk)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    run_decode(args, cfg, world, rank, local, dist, torch, vxk)
    if dist:
        dist.destroy_process_group()


def page_bytes(L: int, dtype: int) -> int:
    """Device bytes of one 16-position page across every layer (K and V)."""
    tile = {1: BT * HD * 2, 0: BT * HD * 4}.get(dtype, BT * HD + BT * (HD // 32) * 2)
    return NKV * 2 * tile * L


def oracle_check(pool, streams, ctx0, qs, ks, vs, out, st, L, dtype, sh):
    """Checker run after the timed region: for three streams (shortest,
    median and longest context) and the first and last layer, the row the
    last timed step appended must equal the CPU oracle's bytes, and the
    step's attention output must be within 2e-3 of the oracle's fp64
    attention over the stream's cache as read back from the device.
    Returns (max abs error, append bytes exact, rows checked)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import vx_oracle

    order = np.argsort(np.asarray(ctx0), kind="stable")
    picks = sorted({int(order[0]), int(order[len(order) // 2]), int(order[-1])})
    scale = float(np.float32(1.0 / np.sqrt(HD)))
    err, exact, n = 0.0, True, 0
    for j in picks:
        r = pool.ring(streams[j])
        pos, lo = r.next_absolute_position - 1, r.oldest_absolute_position
        for layer in sorted({0, L - 1}):
            kb, vb = pool.read_rows(layer, streams[j], lo, pos - lo + 1, sh)
            q = qs[st, layer, j].cpu().numpy()
            wk, wv = vx_oracle.kv_row(ks[st, layer, j].cpu().numpy(), vs[st, layer, j].cpu().numpy(), pos, 1e6,
                                      dtype)
            exact = exact and bool(np.array_equal(kb[-1], wk)) and bool(np.array_equal(vb[-1], wv))
            want = vx_oracle.attn_row(q, pos, 1e6, kb, vb, dtype, NKV, scale)
            err = max(err, float(np.abs(out[layer, j].cpu().numpy() - want).max()))
            n += 1
    return err, exact, n


def run_decode(args, cfg, world, rank, local, dist, torch, vxk):
    L, dtype, cap = cfg["layers"], cfg["dtype"], cfg["capacity"]
    ctx_all, parts, scaling = job_layout(cfg, args.seed, world)
    mine = parts[rank]
    total_steps = args.warmup + args.steps * (1 if args.no_e2e else 2) + 6  # + the 4 per-launch probe steps
    NSETS = 4
    prefill_chunk = int(min(cap, 4096, ctx_all.max()))

    def pages_of(c):
        return min(cap // BT, (int(c) + total_steps) // BT + 2)

    # The rank's streams that fit its memory, taken in index order: the
    # per-step inputs, outputs, host-path staging, split scratch, fill
    # buffers and a 3 GiB margin are set aside first.
    free_b, total_b = torch.cuda.mem_get_info(local)
    n_mine = len(mine)
    max_rows = max(n_mine, prefill_chunk)
    fixed = ((NSETS + 1) * L * n_mine * (NQ + 2 * NKV) * HD * 4
             + (0 if args.no_e2e else L * n_mine * (2 * NQ + 2 * NKV) * HD * 4)
             + max(2048, 8 * max_rows) * NQ * 132 * 4 + 2 * prefill_chunk * NKV * HD * 4 + (3 << 30))
    budget = free_b - fixed
    pb = page_bytes(L, dtype)
    run, used = [], 0
    for i in mine:
        b = pages_of(ctx_all[i]) * pb
        if used + b > budget:
            break
        run.append(i)
        used += b
    if not run:
        raise RuntimeError(f"rank {rank}: no stream fits {free_b / 1e9:.1f} GB of free device memory")
    S = len(run)
    ctx0 = ctx_all[run]
    need_pos = int(ctx0.max()) + total_steps + BT
    n_blocks = int(sum(pages_of(c) for c in ctx0)) + 64
    pool = vxk.Pool(device=local, n_layers=L, n_q_heads=NQ, n_kv_heads=NKV, head_dim=HD, block_tokens=BT,
                    capacity=cap, n_blocks=n_blocks, max_streams=S, max_rows=max(S, prefill_chunk),
                    max_position=need_pos + 16, dtype=dtype, alloc_seed=1234 + rank)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    streams = [pool.open_stream() for _ in range(S)]

    # ---- fill caches to ctx0 (append only; values random) -------------------
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed + rank)
    kfill = torch.randn((prefill_chunk, NKV, HD), device="cuda", generator=gen) * 0.5
    vfill = torch.randn((prefill_chunk, NKV, HD), device="cuda", generator=gen) * 0.5
    for s, c in zip(streams, ctx0):
        left = int(c)
        while left > 0:
            n = min(left, prefill_chunk)
            pool.plan([s], [n], sh)
            for layer in range(L):
                pool.append_layer(layer, kfill.data_ptr(), vfill.data_ptr(), sh)
            pool.commit()
            left -= n
    torch.cuda.synchronize()
    del kfill, vfill

    # ---- per-step inputs resident in HBM (4 rotating sets) -------------------
    qs = torch.randn((NSETS, L, S, NQ, HD), device="cuda", generator=gen) * 0.5
    ks = torch.randn((NSETS, L, S, NKV, HD), device="cuda", generator=gen) * 0.5
    vs = torch.randn((NSETS, L, S, NKV, HD), device="cuda", generator=gen) * 0.5
    out = torch.empty((L, S, NQ, HD), device="cuda")
    ones = [1] * S
    ctx_now = [int(c) for c in ctx0]

    def step(i):
        pool.plan(streams, ones, sh)
        st = i % NSETS
        for layer in range(L):
            pool.decode_layer(layer, qs[st, layer].data_ptr(), ks[st, layer].data_ptr(), vs[st, layer].data_ptr(),
                              out[layer].data_ptr(), sh)
        pool.commit()
        for j in range(S):
            ctx_now[j] = min(cap, ctx_now[j] + 1)

    for i in range(args.warmup):
        step(i)
    pool.sync(sh)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()

    # ---- timed region --------------------------------------------------------
    props = torch.cuda.get_device_properties(local)
    gpu_id = str(getattr(props, "uuid", local))
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    launches0 = pool.stats().kernel_launches
    bytes_per_step = []
    ctx_means = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
            bytes_per_step.append(sum(algorithmic_bytes(c, dtype) for c in ctx_now))
            ctx_means.append(sum(ctx_now) / S)
        end.record(stream)
        torch.cuda.synchronize()
    pool.sync(sh)
    launches = pool.stats().kernel_launches - launches0
    ms_local = start.elapsed_time(end)
    rank_ms = gather_over_ranks(dist, ms_local, "cuda")
    rank_streams = [int(x) for x in gather_over_ranks(dist, float(S), "cuda")]
    ms = max(rank_ms)
    streams_run = sum(rank_streams)
    value = streams_run * args.steps / (ms / 1000.0)

    # ---- sampled check against the CPU oracle (outside the timed region) ----
    chk_err, chk_exact, chk_rows = oracle_check(pool, streams, ctx0, qs, ks, vs, out,
                                                (args.warmup + args.steps - 1) % NSETS, L, dtype, sh)
    chk_err = max_over_ranks(dist, chk_err, "cuda")
    chk_bad = max_over_ranks(dist, 0.0 if chk_exact else 1.0, "cuda")
    checked = {"passed": bool(chk_err <= 2e-3 and chk_bad == 0.0), "max_abs_err": chk_err, "tolerance": 2e-3,
               "append_bit_exact": chk_bad == 0.0, "rows_per_gpu": chk_rows,
               "what": "last timed step: shortest / median / longest-context stream x first / last layer, "
                       "appended row bytes and attention output vs the CPU oracle"}

    # ---- per-launch cross-check: a few more steps with CUDA events around
    # every decode launch (the events keep consecutive layers from overlapping,
    # so this is each launch's own warm duration) --------------------------------
    probe_steps = min(4, args.steps)
    probe_us, probe_bytes = [], []
    for i in range(probe_steps):
        pool.plan(streams, ones, sh)
        st = (args.warmup + args.steps + i) % NSETS
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(L + 1)]
        evs[0].record(stream)
        for layer in range(L):
            pool.decode_layer(layer, qs[st, layer].data_ptr(), ks[st, layer].data_ptr(), vs[st, layer].data_ptr(),
                              out[layer].data_ptr(), sh)
            evs[layer + 1].record(stream)
        pool.commit()
        for j in range(S):
            ctx_now[j] = min(cap, ctx_now[j] + 1)
        torch.cuda.synchronize()
        probe_bytes.append(sum(algorithmic_bytes(c, dtype) for c in ctx_now))
        probe_us += [evs[layer].elapsed_time(evs[layer + 1]) * 1000.0 for layer in range(L)]
    pool.sync(sh)
    probe_launch_us = statistics.mean(probe_us)
    probe_gbs = statistics.mean(probe_bytes) / (probe_launch_us / 1e6) / 1e9

    # ---- roofline of the dominant kernel (decode_kernel) --------------------
    peak, peak_kind = load_peaks()
    bytes_per_launch = statistics.mean(bytes_per_step)  # one layer launch: every stream's token in that layer
    # Consecutive layer launches overlap (programmatic dependent launch), so the
    # per-launch duration is the timed region divided by the decode launches
    # in it (the small plan upload per step is charged to them too).
    avg_launch_s = (ms_local / 1000.0) / (args.steps * L)
    achieved = bytes_per_launch / avg_launch_s / 1e9
    achieved = max_over_ranks(dist, -achieved, "cuda") * -1.0  # the slowest rank's rate
    traffic_ratio, traffic_src = load_traffic(args.config) if not args.cache else (None, None)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "frac_of_nominal_8000": round(achieved / 8000.0, 4),
                "traffic": None if traffic_ratio is None else round(traffic_ratio * bytes_per_launch),
                "traffic_source": traffic_src and f"{traffic_src} (ncu dram bytes per algorithmic byte, "
                                                  f"scaled to this launch)",
                "algorithmic_bytes_per_launch": round(bytes_per_launch),
                "avg_launch_us": round(avg_launch_s * 1e6, 2),
                "event_launch_us": round(probe_launch_us, 2), "event_achieved": round(probe_gbs, 1),
                "event_note": f"{probe_steps} extra steps, CUDA events around each decode launch (no overlap between "
                              f"layers); avg_launch_us is the timed region over its launches",
                "kernel": "decode_kernel<" + {1: "f16", 8: "q8_0", 0: "f32"}[dtype] + ">"}
    job_bytes_per_s = sum(gather_over_ranks(dist, statistics.mean(bytes_per_step) * L, "cuda")) * args.steps / (
        ms / 1000.0)

    # ---- end to end through the host-buffer C-ABI entry point ----------------
    e2e = None
    if not args.no_e2e:
        hq = torch.randn((L, S, NQ, HD)).mul_(0.5).pin_memory()
        hk = torch.randn((L, S, NKV, HD)).mul_(0.5).pin_memory()
        hv = torch.randn((L, S, NKV, HD)).mul_(0.5).pin_memory()
        ho = torch.empty((L, S, NQ, HD)).pin_memory()
        pool.decode_step_host(streams, hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), ho.data_ptr(), sh)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            pool.decode_step_host(streams, hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), ho.data_ptr(), sh)
        e1.record(stream)
        torch.cuda.synchronize()
        ems = max_over_ranks(dist, e0.elapsed_time(e1), "cuda")
        e2e = {"value": round(streams_run * args.steps / (ems / 1000.0), 1), "unit": "tokens/s",
               "h2d_bytes_per_step": int(hq.numel() + hk.numel() + hv.numel()) * 4,
               "d2h_bytes_per_step": int(ho.numel()) * 4, "ms_per_step": round(ems / args.steps, 3)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and dtype in (1, 8):
        sample = sample_contexts(ctx0, cpu_streams(dtype))
        tps, done, threads, mean_ctx, bps = cpu_sample(L, sample, args.seed, seconds=args.cpu_seconds, dtype=dtype)
        cpu = {"value": round(tps, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
               "bytes_per_s": round(bps, 1),
               "sample": f"{len(sample)} streams (starting contexts {sample}: quantile centres of this run's "
                         f"list, mean {mean_ctx:.0f}) x {L} layers x {done} steps, "
                         f"{'q8_0' if dtype == 8 else 'f16'} cache, oracle/vx_cpu_step.c on {threads} host threads"}

    if dist:
        dist.barrier()
    if rank == 0:
        cfg_line = decode_config(args, cfg, world, ctx_all, parts, scaling)
        line = {
            "metric": "decode tokens/s (KV append+GQA attn)",
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": {1: "f16", 8: "q8_0", 0: "f32"}[dtype] + " cache, fp32 accumulate",
            "data": "synthetic",
            "config": cfg_line,
            "streams_run": streams_run,
            "streams_per_rank": rank_streams,
            "fits": streams_run == len(ctx_all),
            "device_memory_gb": round(total_b / 1e9, 1),
            "mean_ctx_timed": round(statistics.mean(ctx_means), 1),
            "rank_ms": [round(x, 3) for x in rank_ms],
            "slowest_rank": int(np.argmax(rank_ms)),
            "bytes_per_s": round(job_bytes_per_s, 1),
            "roofline": roofline,
            "checked": checked,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    pool.close()


if __name__ == "__main__":
    main()
