"""Benchmark of the EmbeddingGemma text-encoder forward on B200 GPUs.

Metric: embedded tokens/s at BASELINE config 2 -- 64 texts with lengths
uniform in 32..512 packed by token count (about 17.4k tokens), random-init seed-0 Q8_0
weights of the 24-layer hidden-768 encoder -- on N GPUs, one process per GPU.  Each rank
embeds its own seeded 64-text batch per step (weak scaling: the sequences of a batch are
independent, so the data-parallel shard has no collective).  A token is an input token
including BOS/EOS (Embedding.tokenCount).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`value` times K device-resident forwards (ids already in HBM) with CUDA events, max over
ranks.  `e2e` times the same K steps through the public API with host buffers
(EmbeddingModel.embed on the batch's token ids -> ge_embed_tokens: host->device ids,
device->host pooled vectors inside the timed region).  `e2e_text` does the same from strings
(EmbeddingModel.embed on texts -> ge_embed_texts, tokenisation with the document prefix
inside the timed region) on seeded synthetic texts cut to the batch's lengths, and
`tokenizer` compares the library's tokenizer with the oracle's restatement on one thread.
`e2e_stream` runs K *distinct* seeded config-2 batches through the same API (every step a new
length mix, so a new batch shape: what an embedding service sees), with the CUDA graphs captured
per step beside it.  `workloads` holds device-resident lines for the metric's literal 64 x 512
batch and for config 3 (16 x 2048 + 4 x 8192 tokens), each with its own roofline.  `strong`
times one config-2 batch on all N GPUs through the library's own dispatcher (rank 0 loads the
model on devices 0..N-1 and EmbeddingModel.embed shards the batch's sequences over them, packs
each share, and gathers the vectors on the host) while the other ranks wait: strong scaling.
`roofline` is the forward's largest kernel class against its peak; `step_roofline` is the whole
timed region's algorithmic FLOPs (every GEMM and attention FLOP of the forward) against the
sustained tensor peak.
`--impl reference` times the CPU oracle (the restated CPUReference.forward, the only
runnable form of the reference's path here) on the host cores.

`--config 4` runs BASELINE config 4 instead (32 synthetic 768x768 images per rank through the
vision and text towers, images/s) and `--config 5` BASELINE config 5 (16 clips x 60 s of
Gaussian-noise PCM per rank through the log-mel front end, the audio tower and the text tower,
audio seconds per second), each with the same value / e2e / roofline / cpu_baseline keys.
"""
from __future__ import annotations

import argparse
import csv
import importlib
import io
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PKG = "gemma-embed-swift_b200"


def args_():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, default=2)
    p.add_argument("--arch", default="gemma-embedding")
    p.add_argument("--profile-reps", type=int, default=5)
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="bound of the CPU-baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--legs", choices=["all", "core"], default="all",
                   help="core: only the device-resident steps, the end-to-end steps and the kernel profile "
                        "(for profiler captures)")
    p.add_argument("--q8-sweep", choices=["on", "off"], default="on",
                   help="time the Q8_0 (dequantise in shared memory) and fp16-weight GEMM paths by batch size")
    p.add_argument("--fused-qkv", choices=["on", "off"], default="off",
                   help="q/k/v norms and RoPE in the q/k/v projection's epilogue (GE_LOAD_FUSED_QKV)")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return {"hbm_gbs": m["hbm_gbs"], "bf16_tflops": m["bf16_tflops"],
                "bf16_tflops_sustained": m["bf16_tflops_sustained"], "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), "--query-gpu=" + ",".join(self.FIELDS), "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) == len(self.FIELDS)]
        sm = sorted(float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit())
        mx = max((float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()), default=None)
        reasons = set()
        for r in rows:
            for name, val in zip(["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"], r[5:9]):
                if val.strip() == "Active":
                    reasons.add(name)
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(rows)}


def host_threads() -> int:
    """Every core this process may run on (torchrun sets OMP_NUM_THREADS=1; the CPU arms use all)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(path, seqs, seconds):
    """The CPU oracle on a bounded prefix of the same batch, all host threads."""
    from oracle import binding
    binding.set_threads(host_threads())
    m = binding.OracleModel(path)
    m.forward(seqs[0][:8])  # dequantises and caches every weight matrix outside the timing
    tokens = 0
    done = 0
    t0 = time.perf_counter()
    for s in seqs:
        m.forward(s)
        tokens += len(s)
        done += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    cores = binding.threads()
    m.close()
    return {"value": tokens / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"first {done} of {len(seqs)} texts of the same batch ({tokens} tokens), one pass, {dt:.1f} s"}


def run_reference(a, rank, world):
    """--impl reference: the reference's CPU path (its restated CPUReference) on the host cores."""
    if rank != 0:
        return 0
    synth = importlib.import_module(PKG + ".synthetic")
    from oracle import binding
    path = synth.model_path(a.arch, seed=0)
    seqs = synth.config_sequences(a.config, seed=0)
    binding.set_threads(host_threads())
    m = binding.OracleModel(path)
    m.forward(seqs[0][:8])
    # One step = one text of the batch, in order, cycling: a bounded sample of the workload.
    order = list(range(len(seqs)))
    for i in range(a.warmup):
        m.forward(seqs[order[i % len(order)]])
    tokens = 0
    t0 = time.perf_counter()
    for i in range(a.steps):
        s = seqs[order[(a.warmup + i) % len(order)]]
        m.forward(s)
        tokens += len(s)
    dt = time.perf_counter() - t0
    value = tokens / dt
    cores = binding.threads()
    line = {"impl": "reference", "metric": "embedded tokens/sec (config 2: 64 texts x 32..512 tokens)", "value": value,
            "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": dt * 1000 / a.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config {a.config}", "arch": a.arch, "step": "one text of the seeded batch"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{a.steps} texts of the config-{a.config} batch ({tokens} tokens)"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    m.close()
    return 0


def main():
    a = args_()
    rank, world, local = dist_env()
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group(backend="nccl" if a.impl == "ours" else "gloo",
                                timeout=datetime.timedelta(seconds=300))
    if a.config in (4, 5):
        if a.config == 4:
            rc = run_images_reference(a, rank, world) if a.impl == "reference" else run_images(a, rank, world, local)
        else:
            rc = run_audios_reference(a, rank, world) if a.impl == "reference" else run_audios(a, rank, world, local)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return rc
    if a.impl == "reference":
        rc = run_reference(a, rank, world)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return rc

    import numpy as np
    import torch

    ge = importlib.import_module(PKG)
    synth = importlib.import_module(PKG + ".synthetic")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier()

    # A host-side (gloo) group for waits while rank 0 drives every GPU: an NCCL barrier would
    # leave a kernel spinning on each waiting rank's GPU beside rank 0's work there.
    host_group = dist.new_group(backend="gloo") if dist is not None else None

    # Rank 0 writes the synthetic GGUF first; the others then read the cached file.
    if rank == 0:
        path = synth.model_path(a.arch, seed=0)
    barrier()
    if rank != 0:
        path = synth.model_path(a.arch, seed=0)
    # One packed batch per step: the budget covers the whole config-2 batch (BASELINE: "packed by
    # token count, about 16k tokens per batch"; the reference default of 8192 would cut it in three).
    model = ge.EmbeddingModel.load(path, ge.LoadOptions(devices=(local,), batch_token_budget=BATCH_BUDGET,
                                                        fused_qkv=a.fused_qkv == "on"))
    seqs = synth.config_sequences(a.config, seed=rank)
    tokens, positions, ranges = ge.pack(seqs)
    ntok, nseq = len(tokens), len(ranges)
    od = model.info.output_dimensions

    d_tokens = torch.from_numpy(tokens).cuda()
    d_out = torch.empty((nseq, od), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()  # every kernel of the timed steps runs on this stream

    def step_device():
        model.forward_device(d_tokens, ranges, d_out, stream=stream, device=local)

    for _ in range(max(a.warmup, 3)):
        step_device()
    torch.cuda.synchronize()

    # ---- device-resident throughput
    clocks = ClockSampler(local)
    time.sleep(0.3)
    launches0 = model_launches(model)
    barrier()
    torch.cuda.synchronize()
    # Events between the steps on the same stream give each step's latency (p50, p99).
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.steps + 1)]
    e0, e1 = ev[0], ev[-1]
    e0.record(stream)
    for i in range(a.steps):
        step_device()
        ev[i + 1].record(stream)
    torch.cuda.synchronize()
    step_ms = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(a.steps))
    barrier()
    clock_info = clocks.stop()
    launches = model_launches(model) - launches0
    ms_total = e0.elapsed_time(e1)
    ms_max, tok_sum = reduce_max_sum(dist, ms_total, ntok * a.steps)
    value = tok_sum / (ms_max / 1000.0)

    # ---- per-kernel roofline (rank 0): the kernel class with the largest share of a forward,
    # profiled right after the timed region, at the clocks it ran at
    pk = peaks()
    roofline = None
    prof = []
    if rank == 0:
        prof = model.profile(tokens, ranges, reps=a.profile_reps)
        roofline = top_roofline(prof, pk)
        traffic = NCU_DRAM_BYTES_CONFIG2["bytes"].get(roofline["kernel"]) if a.config == 2 and a.arch == "gemma-embedding" else None
        roofline["traffic"] = traffic
        roofline["traffic_source"] = NCU_DRAM_BYTES_CONFIG2["source"] if traffic else None
    step_roof = step_roofline(prof, pk, a.steps, world, ms_max) if rank == 0 else None

    full = a.legs == "all"
    # ---- end to end through the public API with host buffers: EmbeddingModel.embed on the
    # batch's token ids (one packed batch), Matryoshka 256-d L2-normalised vectors back
    texts = [np.asarray(q, dtype=np.int32) for q in seqs]
    opts = ge.EmbedOptions(max_tokens=max(2048, max(len(q) for q in texts)), dimensions=256)  # no text truncated
    for _ in range(2):
        model.embed(texts, opts)
    barrier()
    torch.cuda.synchronize()
    info0 = model_info(model)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        out = model.embed(texts, opts)
    t1 = time.perf_counter()
    barrier()
    info1 = model_info(model)
    e2e_ms, _ = reduce_max_sum(dist, (t1 - t0) * 1000.0, 0)
    e2e = tok_sum / (e2e_ms / 1000.0)
    # bytes the library copied per step (ids, positions, sequence ranges, attention schedule up;
    # status word and pooled vectors down), counted by the library itself
    h2d = (info1.host_to_device_bytes - info0.host_to_device_bytes) // a.steps
    d2h = (info1.device_to_host_bytes - info0.device_to_host_bytes) // a.steps

    e2e_text, tok_stats, e2e_stream, workloads, strong = None, None, None, {}, None
    if full:
        # ---- end to end from strings: the same lengths as seeded synthetic prose, tokenised inside
        # the timed region (EmbeddingModel.embed on texts with the default document prefix)
        tk = model.tokenizer
        strings = text_batch(synth, tk, [len(q) for q in seqs], seed=1000 + rank)
        sopts = ge.EmbedOptions(max_tokens=opts.max_tokens, dimensions=256)
        for _ in range(2):
            model.embed(strings, sopts)
        barrier()
        t0 = time.perf_counter()
        for _ in range(a.steps):
            sout = model.embed(strings, sopts)
        t1 = time.perf_counter()
        barrier()
        text_tokens = sum(e.token_count for e in sout)
        et_ms, et_tok = reduce_max_sum(dist, (t1 - t0) * 1000.0, text_tokens * a.steps)
        e2e_text = {"value": et_tok / (et_ms / 1000.0), "unit": "tokens/s", "tokens_per_step": et_tok // a.steps,
                    "api": "ge_embed_texts (EmbeddingModel.embed on strings), document prefix, 256-d normalised output"}
        tok_stats = tokenizer_throughput(synth, tk, path) if rank == 0 else None

    if full:
        # ---- a stream of distinct batches through the same API: new lengths (a new batch shape)
        # every step, as an embedding service sees them; graph captures per step beside it
        stream_batches = [[np.asarray(q, dtype=np.int32) for q in synth.config_sequences(2, seed=10_000 + 100 * rank + i)]
                          for i in range(a.steps + 2)]
        for b in stream_batches[:2]:
            model.embed(b, opts)
        barrier()
        c0 = model.counters()
        st_ms, st_tok = [], 0
        t0 = time.perf_counter()
        for b in stream_batches[2:]:
            s0 = time.perf_counter()
            model.embed(b, opts)
            st_ms.append((time.perf_counter() - s0) * 1000.0)
            st_tok += sum(len(q) for q in b)
        t1 = time.perf_counter()
        barrier()
        c1 = model.counters()
        es_ms, es_tok = reduce_max_sum(dist, (t1 - t0) * 1000.0, st_tok)
        st_ms.sort()
        e2e_stream = {"value": es_tok / (es_ms / 1000.0), "unit": "tokens/s", "steps": a.steps,
                      "tokens_per_step": es_tok // a.steps,
                      "graph_captures_per_step": (c1["graph_captures"] - c0["graph_captures"]) / a.steps,
                      "latency_ms_p50": pct(st_ms, 50), "latency_ms_p99": pct(st_ms, 99),
                      "api": "ge_embed_tokens (EmbeddingModel.embed), a distinct seeded config-2 batch every step, "
                             "256-d normalised output"}

    if full:
        # ---- the metric's literal 64 x 512 batch and config 3, device-resident, each with its roofline
        workloads = {}
        if a.config == 2:
            for name, cfg in (("64x512", 4), ("config 3", 3)):
                wseqs = synth.config_sequences(cfg, seed=rank)
                wt, _, wr = ge.pack(wseqs)
                w_tokens = torch.from_numpy(wt).cuda()
                w_out = torch.empty((len(wr), od), dtype=torch.float32, device="cuda")
                wsteps = max(3, min(a.steps, 10))
                for _ in range(3):
                    model.forward_device(w_tokens, wr, w_out, stream=stream, device=local)
                barrier()
                torch.cuda.synchronize()
                wev = [torch.cuda.Event(enable_timing=True) for _ in range(wsteps + 1)]
                wev[0].record(stream)
                for i in range(wsteps):
                    model.forward_device(w_tokens, wr, w_out, stream=stream, device=local)
                    wev[i + 1].record(stream)
                torch.cuda.synchronize()
                w_step = sorted(wev[i].elapsed_time(wev[i + 1]) for i in range(wsteps))
                w_ms, w_tok = reduce_max_sum(dist, wev[0].elapsed_time(wev[-1]), len(wt) * wsteps)
                entry = {"value": w_tok / (w_ms / 1000.0), "unit": "tokens/s", "ms_per_step": w_ms / wsteps,
                         "steps": wsteps, "tokens_per_rank": int(len(wt)), "texts_per_rank": len(wr),
                         "latency_ms_p50": pct(w_step, 50), "latency_ms_p99": pct(w_step, 99)}
                if rank == 0:
                    wprof = model.profile(wt, wr, reps=max(1, a.profile_reps // 2))
                    entry["roofline"] = top_roofline(wprof, peaks())
                workloads[name] = entry
                del w_tokens, w_out
            if a.arch == "gemma-embedding" and rank == 0:
                workloads["gemma-embedding2 config 2"] = eg2_workload(ge, synth, seqs, a.profile_reps)

    if full:
        # ---- strong scaling through the library's dispatcher: rank 0 alone embeds one config-2
        # batch on devices 0..N-1 (sequences sharded longest first onto the least-loaded device,
        # each share packed and run on its own host thread and stream, vectors gathered on the host)
        strong = None
        if world > 1:
            barrier()
            torch.cuda.synchronize()
            # The other ranks wait on the host, with nothing of theirs running on any GPU.
            if rank == 0:
                strong = strong_scaling(ge, path, [np.asarray(q, dtype=np.int32) for q in synth.config_sequences(2, seed=0)],
                                        opts, world, a.steps)
            dist.barrier(group=host_group)
        else:
            strong = {"value": e2e, "unit": "tokens/s", "devices": 1, "note": "one GPU: the e2e measurement"}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(path, seqs, a.cpu_seconds)
    sweeps = full and rank == 0 and world == 1 and a.config == 2 and a.q8_sweep == "on"
    q8 = q8_gemm_sweep(ge, synth, path) if sweeps else None
    gemm_paths = gemm_schedule_sweep() if sweeps else None

    if rank == 0:
        line = {"metric": "embedded tokens/sec (config 2: 64 texts x 32..512 tokens)", "value": value,
                "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": ms_max / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16", "data": "synthetic",
                "config": {"workload": f"config {a.config}", "arch": a.arch, "tokens_per_rank": ntok,
                           "texts_per_rank": nseq, "global_batch_tokens": tok_sum // a.steps,
                           "parallelism": f"dp{world}", "fused_qkv": a.fused_qkv == "on",
                           "l2": "working set larger than L2 (fp16 weights 203 MB + ~0.5 GB of activations per step)"},
                "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "api": "ge_embed_tokens (EmbeddingModel.embed), 256-d normalised output"},
                "e2e_text": e2e_text, "e2e_stream": e2e_stream, "strong": strong, "workloads": workloads,
                "q8_gemm": q8, "gemm_schedules": gemm_paths,
                "tokenizer": tok_stats,
                "gpu_launches": int(launches), "clocks": clock_info, "roofline": roofline, "step_roofline": step_roof,
                "cpu_baseline": cpu, "latency_ms_p50": pct(step_ms, 50), "latency_ms_p99": pct(step_ms, 99),
                "kernels": [{k: (round(v, 5) if isinstance(v, float) else v) for k, v in p.items()} for p in prof]}
        print(json.dumps(line), flush=True)
    model.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


# dram__bytes_read.sum + dram__bytes_write.sum per launch of each kernel class, from one
# `ncu --set full` capture of one config-2 layer (cold caches: reads include operands a normal
# run finds in L2).  The capture belongs to the kernels of the commit named in "source"; a
# kernel changed since then needs a new capture.
NCU_DRAM_BYTES_CONFIG2 = {
    "source": "ncu --set full on layer 6 of a config-2 forward: the GEMMs at commit 8909a33 (CTA pairs), the "
              "q/k/v norm, attention and residual kernels at commit dc778e8",
    "bytes": {"gemm_qkv": 36.83e6, "gemm_o": 33.54e6, "gemm_gate_up": 40.26e6, "gemm_down": 50.74e6,
              "qkv_norm_rope": 58.00e6, "attention_sliding": 52.73e6, "residual_attn": 100.92e6,
              "residual_ffn": 156.96e6},
}


BATCH_BUDGET = 65536


def step_roofline(prof, pk, steps, world, ms):
    """The whole timed region against the tensor peak: algorithmic FLOPs of rank 0's forward (every
    GEMM's 2.N.K per row and the attention's 4.H.hd per visible query-key pair, as ge_profile
    counts them) times the forwards of all ranks, over the max-over-ranks time, against the
    per-GPU peak times the ranks.  A step runs seconds of back-to-back GEMMs under the power cap,
    so the sustained peak applies."""
    flops = sum(p["flops_per_launch"] * p["launches_per_forward"] for p in prof)
    ach = flops * steps * world / (ms / 1000.0) / 1e12
    peak = pk["bf16_tflops_sustained"] * world
    return {"flop_per_forward": flops, "achieved": ach, "unit": "TFLOP/s", "peak": peak,
            "peak_kind": "sustained bf16", "frac": ach / peak, "peak_source": pk["source"]}


def top_roofline(prof, pk):
    """The kernel class with the largest share of a forward (ge_profile: CUDA events on its
    stream), against the peak it runs closer to: tensor FLOP/s or HBM bytes/s."""
    fwd_ms = sum(p["ms_per_launch"] * p["launches_per_forward"] for p in prof)
    top = max(prof, key=lambda p: p["ms_per_launch"] * p["launches_per_forward"])
    sec = top["ms_per_launch"] / 1000.0
    tf = top["flops_per_launch"] / sec / 1e12
    gbs = top["bytes_per_launch"] / sec / 1e9
    tensor = tf / pk["bf16_tflops"] > gbs / pk["hbm_gbs"]
    ach, peak, unit = (tf, pk["bf16_tflops"], "TFLOP/s") if tensor else (gbs, pk["hbm_gbs"], "GB/s")
    return {"kernel": top["name"], "bound": "tensor" if tensor else "hbm", "achieved": ach, "peak": peak,
            "unit": unit, "frac": ach / peak, "traffic": None, "peak_source": pk["source"],
            "share_of_forward": top["ms_per_launch"] * top["launches_per_forward"] / fwd_ms,
            "launches_per_forward": top["launches_per_forward"], "forward_ms_sum_of_kernels": fwd_ms}


# Projection shapes of the measured model (N, K): the weight bytes each GEMM launch streams.
GEMM_SHAPES = {"gemm_qkv": (1280, 768), "gemm_o": (768, 768), "gemm_gate_up": (2304, 768), "gemm_down": (768, 1152)}


def q8_gemm_sweep(ge, synth, path, rows_list=(128, 256, 512, 1024, 2048, 4096), reps=5):
    """The two weight paths of the projection GEMMs by batch size: Q8_0 planes dequantised to
    fp16 in shared memory (int8 values + fp16 scales, 34/32 bytes per weight) against the
    fp16-resident copy (2 bytes per weight).  Per size, the four projection classes' mean time
    per launch (ge_profile, CUDA events), the Q8 path's weight bytes per second against HBM, and
    which path is faster.  The library reads the fp16 weights unless the model was loaded with
    only the Q8_0 planes (LoadOptions.q8_only)."""
    models = {"q8": ge.EmbeddingModel.load(path, ge.LoadOptions(q8_only=True, batch_token_budget=BATCH_BUDGET)),
              "fp16": ge.EmbeddingModel.load(path, ge.LoadOptions(batch_token_budget=BATCH_BUDGET))}
    pk = peaks()
    out = []
    try:
        for rows in rows_list:
            lens = [rows // 4] * 4  # four texts filling `rows` GEMM rows exactly
            toks, _, ranges = ge.pack(synth.random_sequences(lens, seed=rows))
            entry = {"rows": rows}
            for name, m in models.items():
                prof = {p["name"]: p for p in m.profile(toks, ranges, reps=reps)}
                us = {k: prof[k]["ms_per_launch"] * 1000.0 for k in GEMM_SHAPES}
                entry[name + "_us"] = {k: round(v, 2) for k, v in us.items()}
                entry[name + "_layer_us"] = round(sum(us.values()), 2)
                if name == "q8":
                    wbytes = sum(n * k * 34 / 32 for n, k in GEMM_SHAPES.values())
                    entry["q8_weight_gbs"] = wbytes / (sum(us.values()) * 1e-6) / 1e9
                    entry["q8_weight_frac_of_hbm"] = entry["q8_weight_gbs"] / pk["hbm_gbs"]
                    tflops = sum(2.0 * rows * n * k for n, k in GEMM_SHAPES.values()) / (sum(us.values()) * 1e-6) / 1e12
                    entry["q8_tflops"] = tflops
            entry["faster"] = "q8" if entry["q8_layer_us"] <= entry["fp16_layer_us"] else "fp16"
            out.append(entry)
    finally:
        for m in models.values():
            m.close()
    return {"sizes": out, "library_default": "fp16 weights at every size (Q8 only with LoadOptions.q8_only)",
            "crossover_rows": max([e["rows"] for e in out if e["faster"] == "q8"], default=None)}


def gemm_schedule_sweep(rows_list=(1024, 2432, 19584), reps=20):
    """Each projection GEMM of the measured model, per launch (ge_test_gemm_time: CUDA events
    over back-to-back launches on seeded operands), under its four schedules: whole 128 x 256
    tiles on persistent single CTAs (the library's default), the same with tiles split into
    narrower pieces where that would shorten the schedule, CTA pairs (256 x 256 tiles), and Q8_0
    weights dequantised in shared memory.  Rows: config 1 (1,024), a config-2 batch on 8 GPUs
    (about 2,400 per GPU) and config 2 on one (19,516, padded to 19,584)."""
    import ctypes
    lib = importlib.import_module(PKG + "._lib").lib()
    epi = {"gemm_qkv": 1, "gemm_o": 1, "gemm_gate_up": 2, "gemm_down": 1}
    paths = {"whole_tiles": 0, "split_tiles": 4, "cta_pairs": 2, "q8_smem": 1}
    pk = peaks()
    out = []
    for rows in rows_list:
        for name, (n, k) in GEMM_SHAPES.items():
            entry = {"gemm": name, "rows": rows, "n": n, "k": k, "tiles": (rows // 128) * (n // 256)}
            for pname, path in paths.items():
                us = ctypes.c_double(0.0)
                rc = lib.ge_test_gemm_time(rows, k, n, epi[name], path, reps, ctypes.byref(us))
                entry[pname + "_us"] = round(us.value, 2) if rc == 0 else None
            best = min((v for key, v in entry.items() if key.endswith("_us") and v), default=None)
            if best:
                entry["best_frac_of_bf16_burst"] = 2.0 * rows * n * k / (best * 1e-6) / 1e12 / pk["bf16_tflops"]
            out.append(entry)
    return out


def eg2_workload(ge, synth, seqs, reps):
    """The reference's own architecture (EmbeddingGemma 2: hidden 512, per-layer inputs, global
    layers with head dim 512, output projection) on the config-2 batch: one forward's kernel
    profile (ge_profile), rank 0 only."""
    path2 = synth.model_path("gemma-embedding2", seed=0)
    toks, _, ranges = ge.pack(seqs)
    with ge.EmbeddingModel.load(path2, ge.LoadOptions(batch_token_budget=BATCH_BUDGET)) as m2:
        for _ in range(3):
            m2.forward_packed(toks, None, ranges)
        prof = m2.profile(toks, ranges, reps=max(1, reps))
    fwd_ms = sum(p["ms_per_launch"] * p["launches_per_forward"] for p in prof)
    roof = top_roofline(prof, peaks())
    out = {"tokens": int(len(toks)), "forward_ms_sum_of_kernels": fwd_ms, "tokens_per_s_from_kernels": len(toks) / (fwd_ms / 1000.0),
           "roofline": roof,
           "kernels": [{k: (round(v, 5) if isinstance(v, float) else v) for k, v in p.items()} for p in prof]}
    for p in prof:
        if p["name"] == "attention_global":  # head dim 512
            sec = p["ms_per_launch"] / 1000.0
            out["attention_hd512"] = {"us_per_launch": p["ms_per_launch"] * 1000.0,
                                      "tflops": p["flops_per_launch"] / sec / 1e12,
                                      "launches_per_forward": p["launches_per_forward"]}
    return out


def strong_scaling(ge, path, texts, opts, n_devices, steps):
    """One config-2 batch embedded on devices 0..n-1 by one process through EmbeddingModel.embed
    (ge_embed_tokens): the library shards the sequences, runs each device's share on its own
    host thread and stream and gathers the vectors.  The call is synchronous, so each step is
    timed on the host around it (host-to-device ids and device-to-host vectors included)."""
    model = ge.EmbeddingModel.load(path, ge.LoadOptions(devices=tuple(range(n_devices)),
                                                        batch_token_budget=BATCH_BUDGET))
    try:
        for _ in range(3):
            model.embed(texts, opts)
        c0 = model.counters()
        ms = []
        t0 = time.perf_counter()
        for _ in range(steps):
            s0 = time.perf_counter()
            model.embed(texts, opts)
            ms.append((time.perf_counter() - s0) * 1000.0)
        dt = time.perf_counter() - t0
        c1 = model.counters()
    finally:
        model.close()
    ntok = sum(len(t) for t in texts)
    ms.sort()
    return {"value": ntok * steps / dt, "unit": "tokens/s", "devices": n_devices, "steps": steps,
            "tokens_per_step": ntok, "latency_ms_p50": pct(ms, 50), "latency_ms_p99": pct(ms, 99),
            "h2d_bytes_per_step": (c1["host_to_device_bytes"] - c0["host_to_device_bytes"]) // steps,
            "d2h_bytes_per_step": (c1["device_to_host_bytes"] - c0["device_to_host_bytes"]) // steps,
            "api": "ge_embed_tokens on a model loaded on every device (in-library dispatcher), 256-d normalised output"}


def text_batch(synth, tk, lengths, seed):
    """Seeded synthetic prose, one text per length, each cut so that with the document prefix
    and BOS/EOS it encodes to about that many tokens."""
    prefix = len(tk.encode("title: none | text: ", add_special_tokens=False))
    out = []
    for i, n in enumerate(lengths):
        body = tk.encode(synth.synthetic_text(seed * 1000 + i, n + 16), add_special_tokens=False)
        out.append(tk.decode(body[:max(1, n - prefix - 2)]))
    return out


def tokenizer_throughput(synth, tk, path, seconds=3.0):
    """Tokens/s of the library's tokenizer and of the oracle's Python restatement on one thread,
    over texts unseen by the warm-up (the library keeps a per-thread cache of word ids)."""
    from oracle.tokenizer import Tokenizer as OracleTokenizer
    warm = [synth.synthetic_text(7000 + i, 300) for i in range(20)]
    texts = [synth.synthetic_text(8000 + i, 300) for i in range(200)]
    for t in warm:
        tk.encode(t)
    n, t0 = 0, time.perf_counter()
    for t in texts:
        n += len(tk.encode(t))
    lib_tps = n / (time.perf_counter() - t0)
    orc = OracleTokenizer.from_gguf(path)
    n, done, t0 = 0, 0, time.perf_counter()
    for t in texts:
        n += len(orc.encode(t))
        done += 1
        if time.perf_counter() - t0 > seconds:
            break
    orc_tps = n / (time.perf_counter() - t0)
    return {"value": lib_tps, "unit": "tokens/s", "threads": 1, "api": "ge_tokenize",
            "cpu_baseline": {"value": orc_tps, "unit": "tokens/s", "cores": 1, "kind": "port",
                            "sample": f"{done} synthetic texts of 300 words"}}


IMAGES_PER_RANK = 32
IMAGE_SIDE = 768


def vision_oracle_step(vis, ref, tok, img):
    """One image through the oracle: preprocessing, the vision tower, the text tower."""
    patches, gx, gy = vis.prepare(img, max_image_tokens=256)
    rows = vis.forward(patches, gx, gy)
    begin = tok.encode("<|image>", False, True)[0]
    end = tok.encode("<image|>", False, True)[0]
    ids = [2, begin] + [-(r + 1) for r in range(rows.shape[0])] + [end, 1]
    import numpy as np
    ref.forward_rows(np.array(ids, np.int32), rows)


def images_cpu_baseline(synth, text_path, mmproj, img):
    from oracle import binding
    from oracle.tokenizer import Tokenizer as OracleTokenizer
    binding.set_threads(host_threads())
    vis, ref = binding.OracleVision(mmproj), binding.OracleModel(text_path)
    tok = OracleTokenizer.from_gguf(text_path)
    t0 = time.perf_counter()
    vision_oracle_step(vis, ref, tok, img)
    dt = time.perf_counter() - t0
    cores = binding.threads()
    vis.close()
    ref.close()
    return {"value": 1.0 / dt, "unit": "images/s", "cores": cores, "kind": "port",
            "sample": f"one 768x768 image of the batch (2304 patches, 256 image tokens), vision and text towers, {dt:.1f} s"}


def run_images(a, rank, world, local):
    """a batch of 32 synthetic 768 x 768 RGB images (pixels uniform in 0..255,
    2304 patches each, pooled to 256 rows and projected to 768) through the vision tower and the
    text tower, per rank; one step is the whole batch."""
    import numpy as np
    import torch
    ge = importlib.import_module(PKG)
    synth = importlib.import_module(PKG + ".synthetic")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier()

    if rank == 0:
        text_path, mmproj = synth.model_path(a.arch, seed=0), synth.mmproj_path(seed=0)
    barrier()
    if rank != 0:
        text_path, mmproj = synth.model_path(a.arch, seed=0), synth.mmproj_path(seed=0)
    model = ge.EmbeddingModel.load(text_path, ge.LoadOptions(devices=(local,), batch_token_budget=BATCH_BUDGET,
                                                            image_encoder=mmproj, image_patch_budget=1 << 20))
    images = synth.synthetic_images(IMAGES_PER_RANK, seed=100 + rank, width=IMAGE_SIDE, height=IMAGE_SIDE)
    n = len(images)
    od = model.info.output_dimensions
    d_rgb = torch.from_numpy(np.concatenate([im.reshape(-1) for im in images])).cuda()
    d_out = torch.empty((n, od), dtype=torch.float32, device="cuda")
    sizes = [(IMAGE_SIDE, IMAGE_SIDE)] * n
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    def step_device():
        model.image_forward_device(d_rgb.data_ptr(), sizes, d_out.data_ptr(), stream=stream.cuda_stream, device=local)

    for _ in range(max(a.warmup, 3)):
        step_device()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    time.sleep(0.3)
    launches0 = model_launches(model)
    barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.steps + 1)]
    ev[0].record(stream)
    for i in range(a.steps):
        step_device()
        ev[i + 1].record(stream)
    torch.cuda.synchronize()
    step_ms = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(a.steps))
    barrier()
    clock_info = clocks.stop()
    launches = model_launches(model) - launches0
    ms_max, img_sum = reduce_max_sum(dist, ev[0].elapsed_time(ev[-1]), n * a.steps)
    value = img_sum / (ms_max / 1000.0)
    patches = 2304 * n
    # ---- end to end: EmbeddingModel.embed(images:) on host pixels (resize check, upload, both towers,
    # 256-d normalised vectors back)
    opts = ge.ImageEmbedOptions(dimensions=256)
    for _ in range(2):
        model.embed_images(images, opts)
    barrier()
    torch.cuda.synchronize()
    info0 = model_info(model)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        model.embed_images(images, opts)
    t1 = time.perf_counter()
    barrier()
    info1 = model_info(model)
    e2e_ms, _ = reduce_max_sum(dist, (t1 - t0) * 1000.0, 0)
    e2e = img_sum / (e2e_ms / 1000.0)
    h2d = (info1.host_to_device_bytes - info0.host_to_device_bytes) // a.steps
    d2h = (info1.device_to_host_bytes - info0.device_to_host_bytes) // a.steps
    pk = peaks()
    roofline, prof = None, []
    if rank == 0:
        prof = model.profile_images(images, max_image_tokens=256, reps=3)
        kern = [p for p in prof if p["name"] not in ("image_forward", "vision_tower")]
        top = max(kern, key=lambda p: p["ms_per_launch"] * p["launches_per_forward"])
        sec = top["ms_per_launch"] / 1000.0
        tf = top["flops_per_launch"] / sec / 1e12
        gbs = top["bytes_per_launch"] / sec / 1e9
        tensor = tf / pk["bf16_tflops"] > gbs / pk["hbm_gbs"]
        ach, peak, unit = (tf, pk["bf16_tflops"], "TFLOP/s") if tensor else (gbs, pk["hbm_gbs"], "GB/s")
        tower_ms = sum(p["ms_per_launch"] * p["launches_per_forward"] for p in kern)
        roofline = {"kernel": "vision " + top["name"], "bound": "tensor" if tensor else "hbm", "achieved": ach,
                    "peak": peak, "unit": unit, "frac": ach / peak, "traffic": None, "peak_source": pk["source"],
                    "share_of_vision_tower": top["ms_per_launch"] * top["launches_per_forward"] / tower_ms,
                    "launches_per_forward": top["launches_per_forward"]}
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = images_cpu_baseline(synth, text_path, mmproj, images[0])
    if rank == 0:
        line = {"metric": "embedded images/sec (config 4: 32 images x 768x768, 2304 patches each)", "value": value,
                "unit": "images/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
                "ms_per_step": ms_max / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f16", "data": "synthetic",
                "config": {"workload": "config 4", "arch": a.arch + " + gemma4v (16 layers, 768, 12 heads, MLP 3072)",
                           "images_per_rank": n, "patches_per_rank": patches, "image_tokens_per_rank": 256 * n,
                           "text_rows_per_rank": 260 * n, "parallelism": f"dp{world}",
                           "l2": "working set larger than L2 (about 1.9 GB of activations per step)"},
                "patches_per_s": value * 2304, "latency_ms_p50": pct(step_ms, 50), "latency_ms_p99": pct(step_ms, 99),
                "e2e": {"value": e2e, "unit": "images/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "api": "ge_embed_images (EmbeddingModel.embed(images:)), 256-d normalised output"},
                "gpu_launches": int(launches), "clocks": clock_info, "roofline": roofline, "cpu_baseline": cpu,
                "kernels": [{k: (round(v, 5) if isinstance(v, float) else v) for k, v in p.items()} for p in prof]}
        print(json.dumps(line), flush=True)
    model.close()
    return 0


def run_images_reference(a, rank, world):
    """--impl reference --config 4: the oracle's image path (its restated CPUVisionReference and
    CPUReference) on the host cores, one image per step."""
    if rank != 0:
        return 0
    synth = importlib.import_module(PKG + ".synthetic")
    from oracle import binding
    from oracle.tokenizer import Tokenizer as OracleTokenizer
    text_path, mmproj = synth.model_path(a.arch, seed=0), synth.mmproj_path(seed=0)
    images = synth.synthetic_images(IMAGES_PER_RANK, seed=100, width=IMAGE_SIDE, height=IMAGE_SIDE)
    binding.set_threads(host_threads())
    vis, ref = binding.OracleVision(mmproj), binding.OracleModel(text_path)
    tok = OracleTokenizer.from_gguf(text_path)
    for i in range(a.warmup):
        vision_oracle_step(vis, ref, tok, images[i % len(images)])
    t0 = time.perf_counter()
    for i in range(a.steps):
        vision_oracle_step(vis, ref, tok, images[(a.warmup + i) % len(images)])
    dt = time.perf_counter() - t0
    value = a.steps / dt
    cores = binding.threads()
    line = {"impl": "reference", "metric": "embedded images/sec (config 4: 32 images x 768x768, 2304 patches each)",
            "value": value, "unit": "images/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": dt * 1000 / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config 4", "arch": a.arch + " + gemma4v", "step": "one image of the seeded batch"},
            "cpu_baseline": {"value": value, "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": f"{a.steps} images of the config-4 batch, vision and text towers"},
            "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    vis.close()
    ref.close()
    return 0


CLIPS_PER_RANK = 16
CLIP_SECONDS = 60.0


def audio_oracle_step(aud, ref, tok, clip):
    """One clip through the oracle: the log-mel front end, the audio tower chunk by chunk, the
    text tower over [bos, <|audio>, rows, <audio|>, eos]."""
    import numpy as np
    rows = aud.embed_rows(clip)
    begin = tok.encode("<|audio>", False, True)[0]
    end = tok.encode("<audio|>", False, True)[0]
    ids = [2, begin] + [-(r + 1) for r in range(rows.shape[0])] + [end, 1]
    ref.forward_rows(np.array(ids, np.int32), rows)


def audios_cpu_baseline(text_path, enc, clip):
    from oracle import binding
    from oracle.tokenizer import Tokenizer as OracleTokenizer
    binding.set_threads(host_threads())
    aud, ref = binding.OracleAudio(enc), binding.OracleModel(text_path)
    tok = OracleTokenizer.from_gguf(text_path)
    t0 = time.perf_counter()
    audio_oracle_step(aud, ref, tok, clip)
    dt = time.perf_counter() - t0
    cores = binding.threads()
    aud.close()
    ref.close()
    secs = len(clip) / 16000.0
    return {"value": secs / dt, "unit": "audio s/s", "cores": cores, "kind": "port",
            "sample": f"one {secs:.0f} s clip of the batch (2 chunks, 1500 rows), audio and text towers, {dt:.1f} s"}


def run_audios(a, rank, world, local):
    """16 clips x 60 s of Gaussian-noise PCM at 16 kHz per rank (two 30-second
    chunks and 1500 rows each) through the log-mel front end, the audio tower (12 Conformer layers,
    1024 wide) and the text tower; one step is the whole batch."""
    import numpy as np
    import torch
    ge = importlib.import_module(PKG)
    synth = importlib.import_module(PKG + ".synthetic")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier()

    if rank == 0:
        text_path, enc = synth.model_path(a.arch, seed=0), synth.audio_path(seed=0)
    barrier()
    if rank != 0:
        text_path, enc = synth.model_path(a.arch, seed=0), synth.audio_path(seed=0)
    model = ge.EmbeddingModel.load(text_path, ge.LoadOptions(devices=(local,), batch_token_budget=BATCH_BUDGET,
                                                            audio_encoder=enc, audio_frame_budget=1 << 22))
    clips = synth.synthetic_pcm(CLIPS_PER_RANK, CLIP_SECONDS, seed=300 + rank)
    n = len(clips)
    counts = [len(c) for c in clips]
    rows_per_clip = ge.audio_tokens(counts[0])
    od = model.info.output_dimensions
    d_pcm = torch.from_numpy(np.concatenate(clips)).cuda()
    d_out = torch.empty((n, od), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    def step_device():
        model.audio_forward_device(d_pcm.data_ptr(), counts, d_out.data_ptr(), stream=stream.cuda_stream, device=local)

    for _ in range(max(a.warmup, 3)):
        step_device()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    time.sleep(0.3)
    launches0 = model_launches(model)
    barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.steps + 1)]
    ev[0].record(stream)
    for i in range(a.steps):
        step_device()
        ev[i + 1].record(stream)
    torch.cuda.synchronize()
    step_ms = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(a.steps))
    barrier()
    clock_info = clocks.stop()
    launches = model_launches(model) - launches0
    audio_s = sum(counts) / 16000.0
    ms_max, s_sum = reduce_max_sum(dist, ev[0].elapsed_time(ev[-1]), audio_s * a.steps)
    value = s_sum / (ms_max / 1000.0)
    # ---- end to end: EmbeddingModel.embed(audios:) on host samples (upload, front end, both
    # towers, 256-d normalised vectors back)
    opts = ge.AudioEmbedOptions(dimensions=256)
    for _ in range(2):
        model.embed_audios(clips, opts)
    barrier()
    torch.cuda.synchronize()
    info0 = model_info(model)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        model.embed_audios(clips, opts)
    t1 = time.perf_counter()
    barrier()
    info1 = model_info(model)
    e2e_ms, _ = reduce_max_sum(dist, (t1 - t0) * 1000.0, 0)
    e2e = s_sum / (e2e_ms / 1000.0)
    h2d = (info1.host_to_device_bytes - info0.host_to_device_bytes) // a.steps
    d2h = (info1.device_to_host_bytes - info0.device_to_host_bytes) // a.steps
    pk = peaks()
    roofline, prof = None, []
    if rank == 0:
        prof = model.profile_audios(clips, reps=3)
        kern = [p for p in prof if p["name"] not in ("audio_forward", "audio_tower")]
        top = max(kern, key=lambda p: p["ms_per_launch"] * p["launches_per_forward"])
        sec = top["ms_per_launch"] / 1000.0
        tf = top["flops_per_launch"] / sec / 1e12
        gbs = top["bytes_per_launch"] / sec / 1e9
        tensor = tf / pk["bf16_tflops"] > gbs / pk["hbm_gbs"]
        ach, peak, unit = (tf, pk["bf16_tflops"], "TFLOP/s") if tensor else (gbs, pk["hbm_gbs"], "GB/s")
        tower_ms = sum(p["ms_per_launch"] * p["launches_per_forward"] for p in kern)
        roofline = {"kernel": "audio " + top["name"], "bound": "tensor" if tensor else "hbm", "achieved": ach,
                    "peak": peak, "unit": unit, "frac": ach / peak, "traffic": None, "peak_source": pk["source"],
                    "share_of_audio_tower": top["ms_per_launch"] * top["launches_per_forward"] / tower_ms,
                    "launches_per_forward": top["launches_per_forward"]}
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = audios_cpu_baseline(text_path, enc, clips[0])
    if rank == 0:
        metric = "embedded audio seconds/sec (config 5: 16 clips x 60 s, 1500 rows each)"
        line = {"metric": metric, "value": value, "unit": "audio s/s", "n_gpus": world, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": ms_max / a.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": {"workload": "config 5", "arch": a.arch + " + gemma4a (12 layers, 1024, 8 heads, FFN 4096)",
                           "clips_per_rank": n, "seconds_per_clip": CLIP_SECONDS, "rows_per_clip": rows_per_clip,
                           "text_rows_per_rank": (rows_per_clip + 4) * n, "parallelism": f"dp{world}",
                           "l2": "working set larger than L2 (about 4 GB of activations per step)"},
                "clips_per_s": value / CLIP_SECONDS, "latency_ms_p50": pct(step_ms, 50),
                "latency_ms_p99": pct(step_ms, 99),
                "e2e": {"value": e2e, "unit": "audio s/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "api": "ge_embed_audios (EmbeddingModel.embed(audios:)), 256-d normalised output"},
                "gpu_launches": int(launches), "clocks": clock_info, "roofline": roofline, "cpu_baseline": cpu,
                "kernels": [{k: (round(v, 5) if isinstance(v, float) else v) for k, v in p.items()} for p in prof]}
        print(json.dumps(line), flush=True)
    model.close()
    return 0


def run_audios_reference(a, rank, world):
    """--impl reference --config 5: the oracle's audio path (its restated AudioFrontEnd,
    CPUAudioReference and CPUReference) on the host cores, one 60-second clip per step."""
    if rank != 0:
        return 0
    synth = importlib.import_module(PKG + ".synthetic")
    from oracle import binding
    from oracle.tokenizer import Tokenizer as OracleTokenizer
    text_path, enc = synth.model_path(a.arch, seed=0), synth.audio_path(seed=0)
    clips = synth.synthetic_pcm(max(a.steps + a.warmup, 1), CLIP_SECONDS, seed=300)
    binding.set_threads(host_threads())
    aud, ref = binding.OracleAudio(enc), binding.OracleModel(text_path)
    tok = OracleTokenizer.from_gguf(text_path)
    for i in range(a.warmup):
        audio_oracle_step(aud, ref, tok, clips[i])
    t0 = time.perf_counter()
    for i in range(a.steps):
        audio_oracle_step(aud, ref, tok, clips[a.warmup + i])
    dt = time.perf_counter() - t0
    value = a.steps * CLIP_SECONDS / dt
    cores = binding.threads()
    line = {"impl": "reference", "metric": "embedded audio seconds/sec (config 5: 16 clips x 60 s, 1500 rows each)",
            "value": value, "unit": "audio s/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": dt * 1000 / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config 5", "arch": a.arch + " + gemma4a", "step": "one 60 s clip of the seeded batch"},
            "cpu_baseline": {"value": value, "unit": "audio s/s", "cores": cores, "kind": "port",
                             "sample": f"{a.steps} clips of 60 s, audio and text towers"},
            "e2e": {"value": value, "unit": "audio s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    aud.close()
    ref.close()
    return 0


def pct(sorted_values, q):
    """Nearest-rank percentile of an ascending list."""
    if not sorted_values:
        return None
    k = max(0, min(len(sorted_values) - 1, int(round(q / 100.0 * len(sorted_values) + 0.5)) - 1))
    return sorted_values[k]


def model_info(model):
    ctypes = importlib.import_module("ctypes")
    lib_mod = importlib.import_module(PKG + "._lib")
    info = lib_mod.GeInfo()
    lib_mod.lib().ge_info_get(model._h, ctypes.byref(info))
    return info


def model_launches(model) -> int:
    return int(model_info(model).kernel_launches)


def reduce_max_sum(dist, ms, tokens):
    """The job's time is the slowest rank's; its work is every rank's tokens."""
    if dist is None:
        return ms, tokens
    import torch
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    n = torch.tensor([tokens], dtype=torch.float64, device=dev)
    dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return float(t.item()), int(n.item())


if __name__ == "__main__":
    sys.exit(main())
