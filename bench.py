#!/usr/bin/env python
"""Benchmark of the B200 text-embedding + exact-search hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl svl|reference]

One process per GPU (torchrun for N > 1; RANK / LOCAL_RANK / WORLD_SIZE from
the environment).  Rank 0 prints ONE JSON line.

Headline: EmbeddingGemma-2 encoder at the manifest
shapes, random N(0, 0.02) FP32 weights (seed 1234), a batch of 64 sequences
per GPU with lengths ~ U[64, 512] and ids ~ U[2, 262144) (seed 2), batches
split data-parallel with no collective ("weak" scaling: 64 sequences per
GPU, the global batch is 64 * N, balanced by longest-processing-time on the
forward's cost model).  A step is one forward of the GPU's batch producing
768-dim embeddings; value = whole-job embeddings/s, the maximum step time
over ranks timed with CUDA events on the launching stream.

Also reported, nested under "search": exact cosine
top-10 of 1024 queries over a 10,000,000 x 768 N(0,1) corpus row-sharded over
the GPUs (per-GPU top-k merged after an NCCL all-gather), at dim 768 and at
the Matryoshka dim 256.

The CPU baseline (rank 0, N = 1) and `--impl reference` time the C++
restatement of the reference's scalar path (oracle/, bit-identical to it on
the golden fixture) on the host's cores: the reference is Rust and there is
no cargo on this image, so it cannot be built.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
for p in (str(ROOT), str(ROOT / "seldon-vault-lite-rust_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "text embeddings/s (and tokens/s) at b64xs512 on 1/2/4/8 B200; exact-search QPS at 10Mx768"
# DRAM traffic of the encoder's GEMM-family kernels per configs[1] forward
# (8,514 MB read + 834 MB written; profiles/encoder_configs1_launch_list.md)
ENCODER_GEMM_TRAFFIC_BYTES = 9_349_000_000
# ... and of all kernels of that forward (11,693 MB read + 1,098 MB written)
ENCODER_STEP_TRAFFIC_BYTES = 12_791_000_000


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["svl", "reference"], default="svl")
    ap.add_argument("--batch", type=int, default=64, help="sequences per GPU")
    ap.add_argument("--no-search", action="store_true")
    ap.add_argument("--search-rows", type=int, default=10_000_000)
    ap.add_argument("--search-queries", type=int, default=1024)
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tokenizer", action="store_true", help="skip the host tokenizer throughput line")
    ap.add_argument("--no-ingress", action="store_true", help="skip the .svlm cold-start line")
    ap.add_argument("--no-ingest", action="store_true", help="skip the document-ingest line")
    ap.add_argument("--no-extra-encoder", action="store_true",
                    help="skip the fixed b64xs512, configs[2] long-context and split-precision encoder lines")
    ap.add_argument("--no-sweep", action="store_true", help="skip the search query-batch sweep and full ranking")
    ap.add_argument("--no-e2e-pipeline", action="store_true", help="skip the configs[4] ingest-then-query line")
    ap.add_argument("--vocab", type=int, default=0,
                    help="profiling knob: a random model with this many vocabulary rows (token ids folded below it) "
                         "instead of the manifest's 262,144, so a multi-pass ncu capture holds a few GB; the encoder's "
                         "per-token work does not depend on the vocabulary")
    ap.add_argument("--no-encoder", action="store_true",
                    help="search only (a small profiling case; prints the search part of the line)")
    return ap.parse_args()


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ---------------------------------------------------------------- clocks --
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    INTERVAL_MS = 50
    START_TIMEOUT_S = 3.0

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.INTERVAL_MS)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # the timed region starts once the sampler is live: nvidia-smi takes
        # a moment to write its first sample, about a timed region's length
        deadline = time.monotonic() + self.START_TIMEOUT_S
        while self.proc is not None and time.monotonic() < deadline:
            if os.path.getsize(self.path) > 0 or self.proc.poll() is not None:
                break
            time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9:
                    rows.append(f)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i] and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------- helpers --
def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "fallback": True}


def tf32_peak_tflops(torch):
    """cuBLAS TF32 dense throughput measured now (8192^3, best of 10)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(8192, 8192, device="cuda")
    b = torch.randn(8192, 8192, device="cuda")
    for _ in range(3):
        torch.matmul(a, b)
    best = float("inf")
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(10):
        s.record()
        torch.matmul(a, b)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    torch.cuda.empty_cache()
    return 2 * 8192 ** 3 / (best / 1e3) / 1e12


def max_over_ranks(torch, dist, value: float, world: int) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(torch, dist, value: float, world: int) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def workload(cfg, world, rank, per_gpu):
    from svl import dist as sdist
    from svl import synth

    seqs = synth.config2_batch(seed=2, batch=per_gpu * world)
    costs = [cfg.flops_per_sequence(s.size) for s in seqs]
    parts = sdist.balance(costs, world)
    return [seqs[i] for i in parts[rank]], seqs


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def oracle_encoder_sample(cfg, weights, seqs, threads):
    """Times the oracle's forward of `threads` sequences (one per host thread)."""
    import oracle

    m = oracle.OracleModel(cfg, weights)
    from svl.text import pack

    ids, cu = pack(seqs)
    t0 = time.perf_counter()
    m.embed_many(ids, cu, cfg.embedding_dim, threads=threads)
    dt = time.perf_counter() - t0
    m.close()
    return dt


# -------------------------------------------------------------- encoder --
def bench_encoder(args, torch, dist, rank, world, local):
    from svl import synth
    from svl.text import TextModel, pack

    cfg = synth.manifest_config(vocab_size=args.vocab) if args.vocab else synth.manifest_config()
    weights = synth.random_weights(cfg, seed=1234)
    model = TextModel(cfg, weights, device=local)
    mine, _ = workload(cfg, world, rank, args.batch)
    if args.vocab:
        mine = [2 + (s.astype(np.int64) - 2) % (args.vocab - 2) for s in mine]
        mine = [s.astype(np.uint32) for s in mine]
    ids, cu = pack(mine)
    B, T = len(mine), int(cu[-1])
    d_ids = torch.from_numpy(ids.view(np.int32)).cuda()
    d_out = torch.empty((B, cfg.embedding_dim), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def step():
        model.embed_batch_device(d_ids.data_ptr(), cu, cfg.embedding_dim, d_out.data_ptr(), stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    model.check()
    lib = model._lib
    import ctypes

    ms6 = (ctypes.c_double * 6)()
    n6 = (ctypes.c_uint64 * 6)()
    lib.svl_model_profile_read.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.svl_model_profile.argtypes = [ctypes.c_void_p, ctypes.c_int]
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        # one more untimed step: the GPU idled while the sampler started
        step()
        torch.cuda.synchronize()
        lib.svl_model_profile_read(model._h, ms6, n6)  # reset launch counters
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    lib.svl_model_profile_read(model._h, ms6, n6)
    launches = int(sum(n6))
    model.check()
    ms_max = max_over_ranks(torch, dist, ms, world)

    # per-category kernel times (separate pass right after the timed region)
    lib.svl_model_profile(model._h, 1)
    prof_steps = 2
    for _ in range(prof_steps):
        step()
    lib.svl_model_profile_read(model._h, ms6, n6)
    lib.svl_model_profile(model._h, 0)
    cat_ms = [ms6[i] / prof_steps for i in range(6)]

    # end to end through the host API (pinned host ids in, host embeddings out)
    ids_pin = torch.from_numpy(ids.view(np.int32)).pin_memory()
    out_pin = torch.empty((B, cfg.embedding_dim), dtype=torch.float32).pin_memory()
    ids_np, out_np = ids_pin.numpy().view(np.uint32), out_pin.numpy()
    for _ in range(2):
        model.embed_packed(ids_np, cu, cfg.embedding_dim, out_np)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.embed_packed(ids_np, cu, cfg.embedding_dim, out_np)
    e2e_s = max_over_ranks(torch, dist, time.perf_counter() - t0, world)
    assert np.allclose(out_np, d_out.cpu().numpy(), atol=0, rtol=0), "host and device entry points disagree"

    tokens_total = sum_over_ranks(torch, dist, float(T), world)
    flops_rank = sum(cfg.flops_per_sequence(s.size) for s in mine)
    gemm_flops = T * cfg.linear_flops_per_token()
    gemm_flops_f16, gemm_flops_tf32 = (T * x for x in cfg.linear_flops_split_per_token(
        os.environ.get("SVL_GEMM_TF32", "0") != "1" and cfg.hidden_size % 128 == 0 and cfg.hidden_size <= 1024))
    attn_flops = sum(cfg.attention_flops(s.size) for s in mine)
    return dict(cfg=cfg, weights=weights, mine=mine, B=B, T=T, ms=ms, ms_max=ms_max, launches=launches,
                cat_ms=cat_ms, e2e_s=e2e_s, tokens_total=tokens_total, flops_rank=flops_rank,
                gemm_flops=gemm_flops, gemm_flops_f16=gemm_flops_f16, gemm_flops_tf32=gemm_flops_tf32,
                attn_flops=attn_flops, clocks=clk.summary(),
                h2d=int(ids.nbytes + cu.nbytes), d2h=int(B * cfg.embedding_dim * 4), model=model)


def time_encoder(torch, dist, world, model, cfg, seqs, steps, warmup, dim=None):
    """Device time of `steps` forwards of `seqs` on this rank (ids resident in
    HBM, one stream, CUDA events, a barrier first); returns the max over ranks
    in ms, this rank's launches and its clocks."""
    import ctypes

    from svl.text import pack

    dim = dim or cfg.embedding_dim
    ids, cu = pack(seqs)
    d_ids = torch.from_numpy(ids.view(np.int32)).cuda()
    d_out = torch.empty((len(seqs), dim), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def step():
        model.embed_batch_device(d_ids.data_ptr(), cu, dim, d_out.data_ptr(), stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    model.check()
    lib = model._lib
    ms6, n6 = (ctypes.c_double * 6)(), (ctypes.c_uint64 * 6)()
    lib.svl_model_profile_read.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        # one more untimed step: the GPU idled while the sampler started
        step()
        torch.cuda.synchronize()
        lib.svl_model_profile_read(model._h, ms6, n6)  # reset launch counters
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s.record()
        for _ in range(steps):
            step()
        e.record()
        torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    lib.svl_model_profile_read(model._h, ms6, n6)
    model.check()
    return max_over_ranks(torch, dist, ms, world), int(sum(n6)), clk.summary()


def encoder_line(cfg, seqs_rank, tokens_total, n_seqs_total, ms_max, steps, peaks, world):
    """emb/s, tok/s and the whole-step tensor fraction of one encoder workload
    (algorithmic FLOPs: linear + windowed attention, config.flops_per_sequence)."""
    flops = sum(cfg.flops_per_sequence(s.size) for s in seqs_rank)
    step_s = ms_max / steps / 1e3
    tflops = flops / step_s / 1e12
    return {
        "value": round(n_seqs_total / step_s, 2),
        "unit": "embeddings/s",
        "tokens_per_s": round(tokens_total / step_s, 1),
        "ms_per_step": round(ms_max / steps, 3),
        "steps": steps,
        "tflops_per_gpu": round(tflops, 1),
        "whole_step_frac_of_burst": round(tflops / peaks["bf16_tflops"], 3),
        "whole_step_frac_of_sustained": round(tflops / peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]), 3),
        "algorithmic_tflop_per_step_per_gpu": round(flops / 1e12, 4),
        "n_gpus": world,
    }


def bench_fixed_s512(args, torch, dist, rank, world, model, cfg, peaks):
    """The metric's literal point: 64 sequences x 512 tokens per GPU (uniform
    ids, seed 6), weak scaling like the headline."""
    from svl import synth

    rng = np.random.default_rng(6)
    allseqs = [rng.integers(2, cfg.vocab_size, size=512, dtype=np.int64).astype(np.uint32)
               for _ in range(args.batch * world)]
    mine = allseqs[rank * args.batch:(rank + 1) * args.batch]
    ms_max, launches, clocks = time_encoder(torch, dist, world, model, cfg, mine, args.steps, args.warmup)
    out = encoder_line(cfg, mine, 512 * args.batch * world, args.batch * world, ms_max, args.steps, peaks, world)
    out.update({"workload": f"b{args.batch}xs512 per GPU: {args.batch} sequences of 512 tokens, ids U[2,262144) "
                            "(seed 6); 768-dim output; weak scaling",
                "scaling": "weak", "gpu_launches": launches, "clocks": clocks})
    del synth
    return out


def bench_single_query(args, torch, dist, rank, world, model, cfg):
    """one 32-token sequence (the SearchQuery prompt ids,
    23 ids U[2, 262144) seed 0, eos), batch 1 -- the reference's own latency
    benchmark (one SearchQuery input, p50 / p95 of a text embed). Latency of the
    synchronous host-buffer C call (svl_embed_batch: ids copied in, the
    embedding copied out), plus the device time of one forward; every rank
    runs its own (replicas)."""
    from svl import synth
    from svl.text import pack

    if max(synth.SEARCH_QUERY_PREFIX_IDS) >= cfg.vocab_size:
        return {"skipped": "the vocabulary is cut below the SearchQuery prompt ids (a profiling run)"}
    ids = synth.config1_ids(seed=0, vocab=cfg.vocab_size)
    steps = max(args.steps, 20)
    ms_max, launches, clocks = time_encoder(torch, dist, world, model, cfg, [ids], steps, args.warmup)
    packed, cu = pack([ids])
    out = np.empty((1, cfg.embedding_dim), np.float32)
    for _ in range(max(args.warmup, 3)):
        model.embed_packed(packed, cu, cfg.embedding_dim, out)
    lat = []
    for _ in range(100):
        t0 = time.perf_counter()
        model.embed_packed(packed, cu, cfg.embedding_dim, out)
        lat.append((time.perf_counter() - t0) * 1e3)
    p50, p95 = float(np.percentile(lat, 50)), float(np.percentile(lat, 95))
    return {
        "workload": "BASELINE configs[0]: one 32-token sequence (SearchQuery prompt ids + 23 ids U[2,262144), "
                    "seed 0, + eos), batch 1, 768-dim output",
        "unit": "ms",
        "latency_ms_p50": round(p50, 3),
        "latency_ms_p95": round(p95, 3),
        "latency_samples": len(lat),
        "api": "svl_embed_batch (host ids in, host embedding out), one synchronous call per sample",
        "device_ms_per_forward": round(ms_max / steps, 3),
        "steps": steps,
        "gpu_launches": launches,
        "clocks": clocks,
        "reference_published": {"p50_ms": 154.8, "p95_ms": 173.2, "input": "one 15-token SearchQuery input",
                                "hardware": "Apple M2 Pro, NEON path (scalar FP32 path: 1,485 ms p50)",
                                "source": "rapport/2026-11-11_23-08-37/benchmark.md:158-169, "
                                          "docs/benchmarks.md:26-35"},
    }


def bench_long_context(args, torch, dist, rank, world, model, cfg, peaks):
    """8 sequences of 2048 tokens (seed 3) split over the
    GPUs (one per GPU at 8 GPUs): strong scaling, the 512-token window masks
    whole key blocks on 20 of the 24 layers."""
    from svl import synth

    allseqs = synth.config3_batch()
    mine = [allseqs[i] for i in range(rank, len(allseqs), world)]
    if not mine:
        mine = [allseqs[0]]  # more ranks than sequences: idle ranks repeat one (not counted)
    ms_max, launches, clocks = time_encoder(torch, dist, world, model, cfg, mine, args.steps, args.warmup)
    n_total = len(allseqs)
    out = encoder_line(cfg, mine, 2048 * n_total, n_total, ms_max, args.steps, peaks, world)
    out.update({"workload": f"BASELINE configs[2]: 8 x 2048 tokens (seed 3), window 512, "
                            f"{len(mine)} sequence(s) per GPU; 768-dim output",
                "scaling": "strong", "gpu_launches": launches, "clocks": clocks})
    return out


def bench_split_precision(args, torch, dist, rank, world, cfg, weights, mine, peaks, local):
    """Cost of the split precision (svl_model_create_ex, SVL_PRECISION_SPLIT)
    on the headline batch."""
    from svl.text import TextModel

    model = TextModel(cfg, weights, device=local, precision="split")
    steps = max(3, args.steps // 2)
    ms_max, launches, _ = time_encoder(torch, dist, world, model, cfg, mine, steps, args.warmup)
    model.close()
    out = encoder_line(cfg, mine, sum_over_ranks(torch, dist, float(sum(s.size for s in mine)), world),
                       args.batch * world, ms_max, steps, peaks, world)
    out.update({"workload": "the headline configs[1] batch in split precision (hi/lo-split TF32 products over "
                            "every projection, FP32 attention on the CUDA cores)", "gpu_launches": launches})
    return out


def bench_ingest_then_query(args, torch, dist, rank, world, local, model, cfg, comm, peaks):
    """65,536 documents (lengths lognormal, median 200,
    sigma 0.8, clipped to [8, 2048], default_rng(5); ids uniform) embedded
    data-parallel into per-rank shards (svl_ingest_batch, no exchange), then
    4096 queries of 32 tokens (the SearchQuery prefix, 23 uniform ids, eos)
    embedded data-parallel, all-gathered (svl_allgather_rows) and searched
    top-10 over every shard (svl_sharded_search).  Documents/s over the whole
    ingest and queries/s over the query stage, each timed from a barrier to
    the last rank's finish."""
    from functools import lru_cache

    from svl import dist as sdist
    from svl import synth
    from svl.index import VectorIndex
    from svl.text import pack

    lengths = synth.config5_lengths()
    n_docs = int(lengths.size)
    offs = np.concatenate([[0], np.cumsum(lengths)])
    ids_all = np.random.default_rng(55).integers(2, cfg.vocab_size, size=int(offs[-1]), dtype=np.int64)
    ids_all = ids_all.astype(np.uint32)
    flops_of = lru_cache(maxsize=None)(lambda n: cfg.flops_per_sequence(int(n)))
    costs = [flops_of(int(n)) for n in lengths]
    mine = sdist.assign_documents(costs, world)[rank]
    sizes = [len(p) for p in sdist.assign_documents(costs, world)]
    row_offset = sum(sizes[:rank])
    batches, cur, cur_tok = [], [], 0
    for d in mine:
        n = int(lengths[d])
        if cur and (cur_tok + n > 32768 or len(cur) == 256):
            batches.append(cur)
            cur, cur_tok = [], 0
        cur.append(d)
        cur_tok += n
    if cur:
        batches.append(cur)
    dim = cfg.embedding_dim
    stream = torch.cuda.current_stream().cuda_stream
    # each batch's ids and chunk ids packed in pinned host memory; inside the
    # timed region every batch is copied in (asynchronously), embedded at the
    # index dimension (svl_embed_batch_device) and appended with Chunk::new's
    # normalisation (svl_index_append_device), all queued on one stream with
    # no host synchronisation between batches
    packed = []
    for b in batches:
        ids_b, cu_b = pack([ids_all[offs[d]:offs[d + 1]] for d in b])
        packed.append((torch.from_numpy(ids_b.view(np.int32)).pin_memory(), cu_b,
                       torch.from_numpy(np.asarray(b, np.int64)).pin_memory()))
    d_emb = torch.empty((max(len(b) for b in batches), dim), device="cuda")

    def ingest(index, which):
        for ids_h, cu_b, chunk_h in which:
            d_ids = ids_h.to("cuda", non_blocking=True)
            d_chunk = chunk_h.to("cuda", non_blocking=True)
            n = cu_b.size - 1
            model.embed_batch_device(d_ids.data_ptr(), cu_b, dim, d_emb.data_ptr(), stream)
            index.append_device(d_emb.data_ptr(), d_chunk.data_ptr(), n, stream=stream)

    scratch = VectorIndex(dim, sum(cu.size - 1 for _, cu, _ in packed[:2]), device=local)
    ingest(scratch, packed[:2])  # warm-up: workspaces grown, kernels loaded
    torch.cuda.synchronize()
    scratch.check()
    scratch.close()
    index = VectorIndex(dim, len(mine), device=local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ingest(index, packed)
    torch.cuda.synchronize()
    ingest_s = max_over_ranks(torch, dist, time.perf_counter() - t0, world)
    model.check()
    index.check()
    assert len(index) == len(mine)
    doc_flops = sum_over_ranks(torch, dist, float(sum(costs[d] for d in mine)), world)

    # query stage
    Q, k = 4096, 10
    qrng = np.random.default_rng(7)
    prefix = np.asarray(synth.SEARCH_QUERY_PREFIX_IDS, np.uint32)
    queries = [np.concatenate([prefix, qrng.integers(2, cfg.vocab_size, size=23).astype(np.uint32),
                               np.asarray([synth.EOS_ID], np.uint32)]) for _ in range(Q)]
    a, b = sdist.query_slice(Q, world, rank)
    qids, qcu = pack(queries[a:b])
    d_qids = torch.from_numpy(qids.view(np.int32)).cuda()
    d_local = torch.empty((b - a, dim), device="cuda")
    shard = sdist.ShardedIndex(index, row_offset, comm)

    def qstep():
        model.embed_batch_device(d_qids.data_ptr(), qcu, dim, d_local.data_ptr(), stream)
        d_all = comm.allgather_rows(d_local, stream)
        return shard.search(d_all, k, stream)

    for _ in range(args.warmup):
        res = qstep()
    torch.cuda.synchronize()
    model.check()
    index.check()
    if world == 1:  # the merged answer equals the plain index search
        d_all = comm.allgather_rows(d_local, stream)
        torch.cuda.synchronize()
        want = index.search(d_all[:64].cpu().numpy(), k)
        assert np.array_equal(res[1][:64].cpu().numpy().astype(np.uint64), want[1])
        assert np.array_equal(res[0][:64].cpu().numpy(), want[2])
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s.record()
    for _ in range(args.steps):
        qstep()
    e.record()
    torch.cuda.synchronize()
    index.check()
    q_ms = max_over_ranks(torch, dist, s.elapsed_time(e), world) / args.steps
    index.close()
    return {
        "workload": "BASELINE configs[4]: 65,536 documents (lognormal lengths, median 200, sigma 0.8, clipped to "
                    "[8, 2048], seed 5; uniform ids) ingested data-parallel into per-GPU shards, then 4096 "
                    "32-token queries embedded data-parallel, all-gathered and searched top-10 over every shard",
        "docs_per_s": round(n_docs / ingest_s, 1),
        "ingest_s": round(ingest_s, 3),
        "tokens": int(offs[-1]),
        "ingest_tokens_per_s": round(float(offs[-1]) / ingest_s, 1),
        "ingest_tflops_per_gpu": round(doc_flops / world / ingest_s / 1e12, 1),
        "qps": round(Q / (q_ms / 1e3), 1),
        "query_ms_per_batch": round(q_ms, 3),
        "n_gpus": world,
        "docs_per_gpu_max": max(sizes),
        "api": "ingest: per batch (<= 32,768 tokens or 256 documents) pinned host ids copied in, "
               "svl_embed_batch_device, svl_index_append_device, queued without host synchronisation; "
               "queries: svl_embed_batch_device + svl_allgather_rows + svl_sharded_search",
        "timing": "ingest: wall clock from a barrier, max over ranks; queries: CUDA events, max over ranks",
    }


# --------------------------------------------------------------- search --
def bench_search(args, torch, dist, rank, world, local, comm=None, dims=(768, 256)):
    import ctypes

    from svl import dist as sdist
    from svl.index import VectorIndex

    N, Q, k = args.search_rows, args.search_queries, args.k
    r0, r1 = sdist.shard_range(N, world, rank)
    n_local = r1 - r0
    chunk = 1 << 16
    gq = torch.Generator(device="cuda").manual_seed(4)
    queries = torch.randn((Q, 768), generator=gq, device="cuda")
    queries /= queries.norm(dim=1, keepdim=True)
    stream = torch.cuda.current_stream().cuda_stream
    results = {}
    for dim in dims:
        idx = VectorIndex(dim, n_local, device=local)
        c0 = r0 // chunk
        while c0 * chunk < r1:
            g = torch.Generator(device="cuda").manual_seed(3_000_000 + c0)
            block = torch.randn((chunk, 768), generator=g, device="cuda")
            a, b = max(r0, c0 * chunk), min(r1, (c0 + 1) * chunk)
            rows = block[a - c0 * chunk: b - c0 * chunk, :dim].contiguous()
            ids = torch.arange(a, b, dtype=torch.int64, device="cuda")
            idx.append_device(rows.data_ptr(), ids.data_ptr(), b - a, stream=stream)
            c0 += 1
        torch.cuda.synchronize()
        idx.check()
        q = queries[:, :dim].contiguous()
        sharded = sdist.ShardedIndex(idx, r0, comm) if world > 1 else None
        out_rows = torch.empty((Q, k), dtype=torch.int64, device="cuda")
        out_chunk = torch.empty((Q, k), dtype=torch.int64, device="cuda")
        out_scores = torch.empty((Q, k), dtype=torch.float64, device="cuda")
        out_counts = torch.empty((Q,), dtype=torch.int32, device="cuda")

        def step():
            if sharded is not None:
                return sharded.search(q, k, stream=stream)
            idx.search_device(q.data_ptr(), Q, k, out_rows.data_ptr(), out_chunk.data_ptr(), out_scores.data_ptr(),
                              out_counts.data_ptr(), stream=stream)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        idx.check()
        lib = idx._lib
        lib.svl_index_profile.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.svl_index_profile_read.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        ms6 = (ctypes.c_double * 6)()
        n6 = (ctypes.c_uint64 * 6)()
        lib.svl_index_profile_read(idx.handle, ms6, n6)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        lib.svl_index_profile_read(idx.handle, ms6, n6)
        launches = int(sum(n6))
        idx.check()
        ms_max = max_over_ranks(torch, dist, ms, world)
        lib.svl_index_profile(idx.handle, 1)
        for _ in range(2):
            step()
        lib.svl_index_profile_read(idx.handle, ms6, n6)
        lib.svl_index_profile(idx.handle, 0)
        screen_ms = ms6[4] / 2
        rescore_ms = ms6[5] / 2
        # end to end: host queries in, host results out -- the single-GPU host
        # API, or at N > 1 pinned host queries copied in, svl_sharded_search,
        # and the merged results copied back, every step
        e2e_steps = max(1, args.steps // 2)
        if world == 1:
            qh = q.cpu().numpy()
            idx.search(qh, k)
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                idx.search(qh, k)
            e2e_s = time.perf_counter() - t0
        else:
            q_pin = q.cpu().pin_memory()
            res_pin = [torch.empty((Q, k), dtype=t, pin_memory=True) for t in (torch.float64, torch.int64)]

            def e2e_step():
                d_q = q_pin.to("cuda", non_blocking=True)
                sc, ch, _, _ = sharded.search(d_q, k, stream=stream)
                res_pin[0].copy_(sc, non_blocking=True)
                res_pin[1].copy_(ch, non_blocking=True)
                torch.cuda.current_stream().synchronize()

            e2e_step()
            dist.barrier()
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                e2e_step()
            e2e_s = max_over_ranks(torch, dist, time.perf_counter() - t0, world)
        e2e_qps = Q * e2e_steps / e2e_s
        results[dim] = dict(ms=ms, ms_max=ms_max, qps=Q * args.steps / (ms_max / 1e3), screen_ms=screen_ms,
                            rescore_ms=rescore_ms, n_local=n_local, launches=launches, e2e_qps=e2e_qps,
                            idx=idx if dim == dims[0] else None)
        if dim != dims[0]:
            idx.close()
    return results


def bench_search_sweep(args, torch, dist, world, idx, n_local, peaks):
    """The HBM regime of the screen: Q in {1, 8, 32, 64, 128} queries against
    this GPU's whole shard (10M x 768 at one GPU), top-k, no merge.  Bytes per
    batch: the FP16 screening copy (n x 768 x 2) + the queries; the exact
    rescoring reads at most a few hundred FP32 candidate rows per query
    (< 0.1% of the copy) and is not counted."""
    import ctypes

    gq = torch.Generator(device="cuda").manual_seed(4)
    queries = torch.randn((128, 768), generator=gq, device="cuda")
    queries /= queries.norm(dim=1, keepdim=True)
    stream = torch.cuda.current_stream().cuda_stream
    lib = idx._lib
    ms6, n6 = (ctypes.c_double * 6)(), (ctypes.c_uint64 * 6)()
    k = args.k
    out_rows = torch.empty((128, k), dtype=torch.int64, device="cuda")
    out_chunk = torch.empty((128, k), dtype=torch.int64, device="cuda")
    out_scores = torch.empty((128, k), dtype=torch.float64, device="cuda")
    out_counts = torch.empty((128,), dtype=torch.int32, device="cuda")
    rows = []
    steps = max(args.steps, 10)
    for Q in (1, 8, 32, 64, 128):
        q = queries[:Q].contiguous()

        def step():
            idx.search_device(q.data_ptr(), Q, k, out_rows.data_ptr(), out_chunk.data_ptr(), out_scores.data_ptr(),
                              out_counts.data_ptr(), stream=stream)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        idx.check()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s.record()
        for _ in range(steps):
            step()
        e.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(torch, dist, s.elapsed_time(e), world) / steps
        lib.svl_index_profile(idx.handle, 1)
        lib.svl_index_profile_read(idx.handle, ms6, n6)
        for _ in range(3):
            step()
        lib.svl_index_profile_read(idx.handle, ms6, n6)
        lib.svl_index_profile(idx.handle, 0)
        screen_ms, rescore_ms = ms6[4] / 3, ms6[5] / 3
        nbytes = n_local * 768 * 2 + Q * 768 * 2
        rows.append({"queries": Q, "ms_per_batch": round(ms, 4), "qps_per_gpu": round(Q / (ms / 1e3), 1),
                     "screen_ms": round(screen_ms, 4), "rescore_ms": round(rescore_ms, 4),
                     "frac_hbm_batch": round(nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 3),
                     "frac_hbm_screen": round(nbytes / (screen_ms / 1e3) / 1e9 / peaks["hbm_gbs"], 3)
                     if screen_ms > 0 else None,
                     "bytes_per_batch": nbytes})
    return {"rows_per_gpu": n_local, "dim": 768, "k": k, "peak_gbs": peaks["hbm_gbs"],
            "bytes": "FP16 screening copy n x 768 x 2 + queries Q x 768 x 2 (rescored FP32 rows not counted)",
            "timing": "device time per batch (query prep + screen + rescore) with CUDA events, max over ranks; "
                      "screen_ms / rescore_ms from per-launch events in a separate pass",
            "sweep": rows}


def bench_full_rank(args, torch, idx, n_local, peaks):
    """The complete ranking (vector::rank returns every row; Index::search
    slices offset + limit <= 1,001,000 of it, index/mod.rs:21-23): one query,
    k = the whole shard and k = 1,001,000; exact f64 scores of every row
    (N x D x 4 bytes of FP32 rows) then a stable radix sort."""
    gq = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn((1, 768), generator=gq, device="cuda")
    q /= q.norm()
    stream = torch.cuda.current_stream().cuda_stream
    out = {"rows": n_local, "dim": 768, "peak_gbs": peaks["hbm_gbs"],
           "bytes": "N x 768 x 4 (the FP32 rows, each read once by the f64 scoring)"}
    for name, k in (("k_all", n_local), ("k_1001000", min(1_001_000, n_local))):
        o_rows = torch.empty((1, k), dtype=torch.int64, device="cuda")
        o_chunk = torch.empty((1, k), dtype=torch.int64, device="cuda")
        o_scores = torch.empty((1, k), dtype=torch.float64, device="cuda")
        o_counts = torch.empty((1,), dtype=torch.int32, device="cuda")

        def step():
            idx.search_device(q.data_ptr(), 1, k, o_rows.data_ptr(), o_chunk.data_ptr(), o_scores.data_ptr(),
                              o_counts.data_ptr(), stream=stream)

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        idx.check()
        steps = 5
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            step()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / steps
        assert int(o_counts[0].item()) == k
        out[name] = {"k": k, "ms_per_query": round(ms, 3),
                     "frac_hbm": round(n_local * 768 * 4 / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 3)}
        del o_rows, o_chunk, o_scores, o_counts
    return out


def cpu_search_sample(dim, n_rows, n_queries, k, threads):
    """Oracle exact top-k (vector::rank order, f64) of `n_queries` unit queries
    over an `n_rows` sample of an N(0,1) corpus stored as Chunk::new stores it;
    returns queries/s over the sample (scale by sample/corpus rows)."""
    import oracle

    rng = np.random.default_rng(3)
    corpus = rng.standard_normal((n_rows, dim), dtype=np.float32)
    corpus /= np.linalg.norm(corpus.astype(np.float64), axis=1, keepdims=True).astype(np.float32)
    q = rng.standard_normal((n_queries, dim), dtype=np.float32)
    t0 = time.perf_counter()
    oracle.vector_topk(q, corpus, k, threads=threads)
    return n_queries / (time.perf_counter() - t0)


# The JSON line is the only thing on stdout: everything else written to file
# descriptor 1 (NCCL's version banner, library logs) is sent to stderr.
_JSON_OUT = None


def emit(line):
    os.write(_JSON_OUT if _JSON_OUT is not None else 1, (json.dumps(line) + "\n").encode())


def main():
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.dup(1)
    os.dup2(2, 1)
    args = parse_args()
    rank, world, local = env_rank()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    # a real (non-default) stream: the library's *_device calls and the CUDA
    # events that time them must share it (a NULL stream handle would select
    # the handle's own stream, which the events would not see)
    torch.cuda.set_stream(torch.cuda.Stream())
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    peaks = measured_peaks()
    tf32_peak = tf32_peak_tflops(torch)
    from svl import dist as sdist

    # the library's own NCCL communicator (sharded search, query all-gather)
    comm = sdist.NcclComm.from_torch(local) if world > 1 else sdist.NcclComm(local, 1, 0, sdist.NcclComm.unique_id())

    if args.no_encoder:
        sr = bench_search(args, torch, dist, rank, world, local, comm, dims=(768,))
        s = sr[768]
        if rank == 0:
            out = {"mode": "search only", "rows": args.search_rows, "queries": args.search_queries,
                   "k": args.k, "qps": round(s["qps"], 1), "screen_ms": round(s["screen_ms"], 3),
                   "rescore_ms": round(s["rescore_ms"], 3)}
            # the complete ranking of the same shard (a small profiling case of it)
            if world == 1 and not args.no_sweep and s.get("idx") is not None:
                out["full_rank"] = side_measurement(bench_full_rank, args, torch, s["idx"], s["n_local"], peaks)
            emit(out)
        if s.get("idx") is not None:
            s["idx"].close()
        if world > 1:
            dist.barrier()
        comm.close()
        if world > 1:
            dist.destroy_process_group()
        return

    enc = bench_encoder(args, torch, dist, rank, world, local)
    emb_s = args.batch * world * args.steps / (enc["ms_max"] / 1e3)
    tok_s = enc["tokens_total"] * args.steps / (enc["ms_max"] / 1e3)
    gemm_ms = enc["cat_ms"][0]
    gemm_tflops = enc["gemm_flops"] / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    # roofline peak of the GEMM mix: each FLOP at the peak of its operand type
    # (FP16 at the sustained measured dense BF16/FP16 rate -- the GEMMs run
    # inside a continuous multi-millisecond step -- TF32 at cuBLAS TF32
    # measured in this run); peak = total / sum(flops_i / peak_i)
    f16_peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    mix_peak = enc["gemm_flops"] / (enc["gemm_flops_f16"] / f16_peak + enc["gemm_flops_tf32"] / tf32_peak)
    mix_desc = ("all on FP16 operands: MEASURED_PEAKS bf16_tflops_sustained" if not enc["gemm_flops_tf32"] else
                "all on TF32 operands: cuBLAS TF32 8192^3 measured in this run" if not enc["gemm_flops_f16"] else
                "FLOP-weighted FP16 / TF32 mix")
    step_tflops = enc["flops_rank"] / (enc["ms"] / args.steps / 1e3) / 1e12

    line = {
        "metric": METRIC,
        "value": round(emb_s, 2),
        "unit": "embeddings/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(enc["ms_max"] / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32 activations and accumulation; tensor-core operands fp16 with power-of-two row scales "
                 "(the 11-bit significand of tf32)",
        "data": "synthetic: random N(0,0.02) weights at the manifest shapes, uniform token ids",
        "config": {
            "workload": "BASELINE configs[1]: EmbeddingGemma-2 encoder (24 layers, hidden 512, manifest shapes), "
                        f"{args.batch} sequences per GPU, lengths U[64,512] (seed 2), ids U[2,262144); 768-dim output"
                        + (f" [profiling run: vocabulary cut to {args.vocab} rows]" if args.vocab else ""),
            "per_gpu_batch": args.batch,
            "tokens_per_gpu": enc["T"],
            "tokens_per_s": round(tok_s, 1),
            "parallelism": f"dp{world} (sequences LPT-balanced, weights replicated, no collective)",
            "l2": "inputs larger than L2: 1.08 GB of weights and ~2 GB of activations stream per step",
        },
        "kernel_ms_per_step": {n: round(v, 3) for n, v in zip(
            ["gemm", "attention", "norm_rope_residual", "other", "screen", "rescore"], enc["cat_ms"])},
        "encoder_tflops_per_gpu": round(step_tflops, 1),
        # the north star's figure: the whole encoder step (every kernel of the
        # forward) against the tensor roofline, live device time
        "roofline": {
            "kernel": "the encoder step: every kernel of one forward (tcgen05 GEMMs incl. the row-fused o / down / "
                      "per-layer-input kernels, tcgen05 attention, norms), two half-batch streams",
            "bound": "tensor",
            "achieved": round(step_tflops, 1),
            "peak": peaks["bf16_tflops"],
            "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst: the timed region is well under a second)",
            "unit": "TFLOP/s",
            "frac": round(step_tflops / peaks["bf16_tflops"], 3),
            "frac_of_sustained": round(step_tflops / peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]), 3),
            # DRAM bytes (read + written) of all kernels of one forward of this
            # workload, from the one-pass ncu capture summarised in
            # profiles/encoder_configs1_launch_list.md (same command with
            # --vocab 4096, which does not change the per-token work)
            "traffic": ENCODER_STEP_TRAFFIC_BYTES if not args.vocab and not os.environ.get("SVL_ROW_FUSED") else None,
            "traffic_unit": "bytes per step (one forward)",
            "algorithmic_flops_per_step": int(enc["flops_rank"]),
        },
        # the projections alone, from the single-stream per-category pass (the
        # row-fused kernels occupy half the machine there, so this reads low)
        "roofline_gemm": {
            "kernel": "tcgen05 GEMMs, all encoder projections (kind::f16 with power-of-two row scales; kind::tf32 "
                      "with SVL_GEMM_TF32=1), the row-fused kernels' residual epilogues included",
            "bound": "tensor",
            "achieved": round(gemm_tflops, 1) if gemm_tflops else None,
            "peak": round(mix_peak, 1),
            "peak_source": f"{mix_desc} (FP16 FLOPs at {f16_peak}; TF32 at {tf32_peak:.1f}, measured in this run)",
            "unit": "TFLOP/s",
            "frac": round(gemm_tflops / mix_peak, 3) if gemm_tflops else None,
            "frac_of_measured_bf16": round(gemm_tflops / peaks["bf16_tflops"], 3) if gemm_tflops else None,
            "traffic": ENCODER_GEMM_TRAFFIC_BYTES if not args.vocab and not os.environ.get("SVL_ROW_FUSED") else None,
            "traffic_unit": "bytes per step (all GEMM-family launches of one forward)",
            "algorithmic_flops_per_step": int(enc["gemm_flops"]),
            "timing": "per-launch CUDA events in a separate single-stream pass right after the timed region",
        },
        "e2e": {
            "value": round(args.batch * world * args.steps / enc["e2e_s"], 2),
            "unit": "embeddings/s",
            "h2d_bytes_per_step": enc["h2d"],
            "d2h_bytes_per_step": enc["d2h"],
            "api": "svl_embed_batch (pinned host ids and host output, copies inside the timed region)",
        },
        "gpu_launches": enc["launches"],
        "clocks": enc["clocks"],
    }

    if not args.no_ingest:
        line["ingest"] = side_measurement(bench_ingest, enc, args.steps, world)
    # the whole step against the tensor roofline (linear + windowed attention)
    line["encoder_whole_step"] = {
        "tflops_per_gpu": round(step_tflops, 1),
        "frac_of_burst": round(step_tflops / peaks["bf16_tflops"], 3),
        "frac_of_sustained": round(step_tflops / peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]), 3),
        "burst_peak": peaks["bf16_tflops"],
        "note": "algorithmic FLOPs of the step (config.flops_per_sequence: every projection plus QK^T and PV over "
                "the attended window) / device time; peaks from MEASURED_PEAKS.json (dense BF16 cuBLAS)",
    }
    if not args.no_extra_encoder:
        line["fixed_b64_s512"] = side_measurement(bench_fixed_s512, args, torch, dist, rank, world, enc["model"],
                                                  enc["cfg"], peaks)
        line["long_context"] = side_measurement(bench_long_context, args, torch, dist, rank, world, enc["model"],
                                                enc["cfg"], peaks)
        line["single_query"] = side_measurement(bench_single_query, args, torch, dist, rank, world, enc["model"],
                                                enc["cfg"])
        for key in ("fixed_b64_s512", "long_context", "single_query"):
            line["gpu_launches"] += line[key].get("gpu_launches", 0)
    if not args.no_e2e_pipeline:
        line["ingest_then_query"] = side_measurement(bench_ingest_then_query, args, torch, dist, rank, world, local,
                                                     enc["model"], enc["cfg"], comm, peaks)
    if not args.no_extra_encoder:
        line["precision_split"] = side_measurement(bench_split_precision, args, torch, dist, rank, world, enc["cfg"],
                                                   enc["weights"], enc["mine"], peaks, local)

    if not args.no_search:
        enc["model"].close()
        del enc["model"]
        torch.cuda.empty_cache()
        sr = bench_search(args, torch, dist, rank, world, local, comm)
        s768 = sr[768]
        # the index screens an FP16 copy of its rows (kind::f16; SVL_SEARCH_TF32=1: the FP32 rows in TF32)
        screen_f16 = os.environ.get("SVL_SEARCH_TF32", "0") != "1"
        eb = 2 if screen_f16 else 4
        screen_peak = peaks["bf16_tflops_sustained"] if screen_f16 else tf32_peak
        bytes_screen = s768["n_local"] * 768 * eb + args.search_queries * 768 * eb
        flops_screen = 2 * args.search_queries * s768["n_local"] * 768
        line["search"] = {
            "workload": f"BASELINE configs[3]: {args.search_rows} x 768 N(0,1) corpus (unit norm), "
                        f"{args.search_queries} queries, top-{args.k}, row-sharded over {world} GPU(s)",
            "qps": round(s768["qps"], 1),
            "ms_per_batch": round(s768["ms_max"] / args.steps, 3),
            "qps_dim256": round(sr[256]["qps"], 1),
            "ms_per_batch_dim256": round(sr[256]["ms_max"] / args.steps, 3),
            "e2e_qps": round(s768["e2e_qps"], 1) if s768["e2e_qps"] else None,
            "screen_ms": round(s768["screen_ms"], 3),
            "rescore_ms": round(s768["rescore_ms"], 3),
            "gpu_launches": s768["launches"],
            "roofline": {
                "kernel": "screen (tcgen05 " + ("FP16" if screen_f16 else "TF32")
                          + " queries x corpus + fused top-k candidates)",
                "bound": "tensor" if flops_screen / (screen_peak * 1e12) > bytes_screen / (peaks["hbm_gbs"] * 1e9) else "hbm",
                "achieved_gbs": round(bytes_screen / (s768["screen_ms"] / 1e3) / 1e9, 1),
                "peak_gbs": peaks["hbm_gbs"],
                "frac_hbm": round(bytes_screen / (s768["screen_ms"] / 1e3) / 1e9 / peaks["hbm_gbs"], 3),
                "achieved_tflops": round(flops_screen / (s768["screen_ms"] / 1e3) / 1e12, 1),
                "peak_tflops": round(screen_peak, 1),
                "peak_tflops_source": ("MEASURED_PEAKS bf16_tflops_sustained (FP16 operands)" if screen_f16
                                       else "cuBLAS TF32 8192^3 measured in this run"),
                "frac_tensor": round(flops_screen / (s768["screen_ms"] / 1e3) / 1e12 / screen_peak, 3),
                "algorithmic_bytes_per_launch": bytes_screen,
                "algorithmic_flops_per_launch": flops_screen,
            },
        }
        line["gpu_launches"] += s768["launches"]
        if not args.no_sweep:
            line["search"]["hbm_sweep"] = side_measurement(bench_search_sweep, args, torch, dist, world, s768["idx"],
                                                           s768["n_local"], peaks)
            if world == 1:
                line["search"]["full_rank"] = side_measurement(bench_full_rank, args, torch, s768["idx"],
                                                               s768["n_local"], peaks)
        if s768.get("idx") is not None:
            s768["idx"].close()

    if rank == 0 and not args.no_ingress:
        line["ingress"] = side_measurement(bench_ingress, enc["cfg"], enc["weights"], local)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        from svl import synth

        cfg = synth.manifest_config()
        weights = synth.random_weights(cfg, seed=1234)
        mine, _ = workload(cfg, 1, 0, args.batch)
        sample = mine[:threads]
        dt = oracle_encoder_sample(cfg, weights, sample, threads)
        sample_rows = 500_000
        qps_sample = cpu_search_sample(768, sample_rows, threads, args.k, threads)
        if "search" in line:
            line["search"]["cpu_baseline"] = {
                "value": round(qps_sample * sample_rows / args.search_rows, 4),
                "unit": "queries/s at 10M x 768",
                "cores": threads,
                "kind": "port",
                "sample": f"{threads} queries over a {sample_rows}-row sample, scaled by "
                          f"{sample_rows}/{args.search_rows}; oracle f64 vector::rank restatement",
            }
        line["cpu_baseline"] = {
            "value": round(len(sample) / dt, 4),
            "unit": "embeddings/s",
            "cores": threads,
            "kind": "port",
            "sample": f"the first {len(sample)} sequences of the same batch ({sum(s.size for s in sample)} tokens), "
                      f"one per host thread, oracle/ C++ restatement of the scalar path (-O3), {dt:.1f} s",
        }

    if rank == 0 and not args.no_tokenizer:
        line["tokenizer"] = side_measurement(bench_tokenizer, world == 1 and not args.no_cpu_baseline)

    if rank == 0:
        emit(line)
    if world > 1:
        dist.barrier()
    comm.close()
    if world > 1:
        dist.destroy_process_group()


def side_measurement(fn, *args):
    """One of the side lines (front ends, extra workloads): on one GPU a
    failure is reported in its own object instead of costing the headline
    line.  With several ranks it is raised: a rank that skipped ahead would
    meet the others in a different collective, so the job must end instead."""
    try:
        return fn(*args)
    except Exception as exc:  # noqa: BLE001 -- recorded, not hidden
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            raise
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


# ----------------------------------------------------------------- ingest --
def bench_ingest(enc, steps, world):
    """Documents into the device index (svl_ingest_batch: embeddings stay on
    the GPU) against the host path (svl_embed_batch to host memory, then
    svl_index_append), on this rank's configs[1] batch, `steps` batches each;
    every rank runs its own model and index (no collective)."""
    from svl.index import VectorIndex

    model, mine = enc["model"], enc["mine"]
    dim = enc["cfg"].embedding_dim
    chunk = np.arange(len(mine), dtype=np.uint64)
    out = {}
    for name in ("device", "host"):
        index = VectorIndex(dim, len(mine) * (steps + 1), model.device)
        if name == "device":
            index.ingest(model, mine, chunk)  # warm-up
        else:
            index.append(model.embed_batch(mine, dim), chunk)
        t0 = time.perf_counter()
        for s in range(steps):
            ids = chunk + np.uint64((s + 1) * len(mine))
            if name == "device":
                index.ingest(model, mine, ids)
            else:
                index.append(model.embed_batch(mine, dim), ids)
        out[name] = len(mine) * steps / (time.perf_counter() - t0)
        assert len(index) == len(mine) * (steps + 1)
        index.close()
    return {"unit": "documents/s", "value": round(out["device"] * world, 2),
            "host_path": round(out["host"] * world, 2), "per_gpu_batch": len(mine),
            "api": "svl_ingest_batch (host ids in; embeddings appended on the device) vs svl_embed_batch + "
                   "svl_index_append; wall clock per rank, summed over ranks"}


# ---------------------------------------------------------------- ingress --
def bench_ingress(cfg, weights, device):
    """Cold start from a `.svlm` bundle file (src/model/source.rs
    load_text_model): the production-shaped encoder with the bench's random
    weights rounded to BF16 (as the frozen model ships), packed with its
    config.json; timed from the file on disk to a model resident on the GPU
    (read, structural parse, SHA-256 of every section, safetensors parse,
    upload, BF16 -> FP32 widening and the FP16 operand copies on the device)."""
    import struct
    import tempfile

    from svl import bundle, synth
    from svl.bundle import Bundle, SectionInput, SectionRole

    header, blobs, off = {}, [], 0
    for name, arr in weights.items():
        f = np.ascontiguousarray(arr, np.float32)
        u = f.view(np.uint32)  # nearest-even rounding to BF16 (finite values: no 32-bit overflow)
        bits = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(f.shape), "data_offsets": [off, off + len(bits)]}
        blobs.append(bits)
        off += len(bits)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    weights_bytes = struct.pack("<Q", len(h)) + h + b"".join(blobs)
    del blobs
    config = synth.manifest_config_dict()
    config["vocab_size"] = cfg.vocab_size  # the --vocab profiling knob shrinks the tables
    config_bytes = json.dumps(config).encode()
    t0 = time.perf_counter()
    data = Bundle.build([SectionInput("config.json", SectionRole.Config, config_bytes),
                         SectionInput("model.safetensors", SectionRole.Weights, weights_bytes)])
    build_s = time.perf_counter() - t0
    del weights_bytes
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(tmp) / "model.svlm"
        path.write_bytes(data)
        n_bytes = len(data)
        del data
        t0 = time.perf_counter()
        raw = path.read_bytes()
        b = Bundle.parse(raw)
        b.verify()
        verify_s = time.perf_counter() - t0
        del b, raw
        t0 = time.perf_counter()
        model = bundle.load_text_model(path, device)
        model.check()
        cold_s = time.perf_counter() - t0
        fingerprint = model.fingerprint_hex()
        model.close()
    return {
        "unit": "s",
        "value": round(cold_s, 3),
        "metric": "cold start: .svlm file on disk -> encoder resident on the GPU",
        "bundle_bytes": n_bytes,
        "read_parse_verify_s": round(verify_s, 3),
        "verify_gb_per_s": round(n_bytes / verify_s / 1e9, 2),
        "build_s": round(build_s, 3),
        "weights": f"{cfg.num_hidden_layers}-layer manifest shapes, bench random weights rounded to BF16",
        "fingerprint": fingerprint,
        "reference": "7.40 s for the 1.53 GB frozen bundle on an Apple M2 Pro (published, docs/formats.md)",
    }


# ------------------------------------------------------------- tokenizer --
def bench_tokenizer(with_baseline: bool):
    """Host throughput of the text front end (include/svl_tokenizer.h): the
    reference's golden tokenizer corpus, encoded with <bos> / <eos> by the
    reduced tokenizer.json that reproduces the official ids on it (one host
    thread), beside the literal restatement of the reference's merge loop
    (oracle/bpe_ref.py, pure Python) as the CPU port."""
    from svl.tokenizer import Tokenizer

    golden = Path(__file__).resolve().parent / "tests" / "golden" / "tokenizer"
    corpus = [c["text"] for c in json.loads((golden / "golden.json").read_text(encoding="utf-8"))["cases"]]
    doc = (golden / "mini_tokenizer.json").read_text(encoding="utf-8")
    tok = Tokenizer.from_json_str(doc)
    n_bytes = sum(len(t.encode("utf-8")) for t in corpus)
    n_tokens = sum(len(tok.encode(t, True)) for t in corpus)
    reps, dt = 1, 0.0
    while dt < 0.2:
        reps *= 2
        t0 = time.perf_counter()
        for _ in range(reps):
            for t in corpus:
                tok.encode_array(t, True)
        dt = time.perf_counter() - t0
    # one svl_tokenizer_encode_batch call over 64 copies of the corpus, all host threads
    batch = corpus * 64
    tok.encode_batch(batch, True)
    bdt, breps = 0.0, 0
    while bdt < 0.2:
        t0 = time.perf_counter()
        tok.encode_batch(batch, True)
        bdt += time.perf_counter() - t0
        breps += 1
    out = {
        "unit": "tokens/s",
        "value": round(reps * n_tokens / dt, 1),
        "mb_per_s": round(reps * n_bytes / dt / 1e6, 2),
        "threads": 1,
        "sample": f"{len(corpus)} golden-corpus texts ({n_bytes} bytes, {n_tokens} tokens) x {reps}, "
                  f"reduced tokenizer.json; includes the Python call per text",
        "batch": {"value": round(breps * 64 * n_tokens / bdt, 1), "unit": "tokens/s",
                  "threads": os.cpu_count(), "texts_per_call": len(batch),
                  "api": "svl_tokenizer_encode_batch (packed ids + cu_seqlens, as svl_embed_batch takes them)"},
    }
    if with_baseline:
        import oracle.bpe_ref as bpe_ref

        ref = bpe_ref.RefTokenizer(doc)
        t0 = time.perf_counter()
        for t in corpus:
            ref.encode(t, True)
        rdt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": round(n_tokens / rdt, 1), "unit": "tokens/s", "cores": 1, "kind": "port",
                               "sample": "one pass over the same corpus, pure-Python restatement of "
                                         "tokenizer.rs:392-560 (quadratic merge rounds)"}
    return out


# ------------------------------------------------------------- reference --
def run_reference(args, rank, world):
    """The reference's CPU path (the oracle port; the Rust crate cannot be built
    here) on the host cores, on this bench's workload and metric."""
    if rank != 0:
        return
    from svl import synth

    threads = cpu_threads()
    cfg = synth.manifest_config()
    weights = synth.random_weights(cfg, seed=1234)
    mine, _ = workload(cfg, 1, 0, args.batch)
    import oracle
    from svl.text import pack

    m = oracle.OracleModel(cfg, weights)

    def step(i):
        sel = [mine[(i * threads + j) % len(mine)] for j in range(threads)]
        ids, cu = pack(sel)
        t0 = time.perf_counter()
        m.embed_many(ids, cu, cfg.embedding_dim, threads=threads)
        return len(sel), time.perf_counter() - t0

    for i in range(args.warmup):
        step(i)
    n_total, t_total = 0, 0.0
    for i in range(args.steps):
        n, t = step(args.warmup + i)
        n_total += n
        t_total += t
    value = n_total / t_total
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "embeddings/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_total / args.steps * 1e3, 1),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic: random N(0,0.02) weights at the manifest shapes, uniform token ids",
        "config": {"workload": "BASELINE configs[1] batch (lengths U[64,512], seed 2); each step embeds "
                               f"{threads} of its sequences, one per host thread"},
        "cpu_baseline": {"value": round(value, 4), "unit": "embeddings/s", "cores": threads, "kind": "port",
                         "sample": f"{threads} sequences per step from the configs[1] batch; oracle/ C++ "
                                   "restatement of the reference's scalar FP32 path (Rust toolchain absent)"},
        "e2e": {"value": round(value, 4), "unit": "embeddings/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


if __name__ == "__main__":
    main()
