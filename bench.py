#!/usr/bin/env python3
"""Benchmark: batch-1 greedy decode of the SmolLM2-135M-shaped Q8_0 model
(30 layers, hidden 576, vocab 49152, 16-token prompt, 128
greedy tokens) on the device-resident CUDA engine, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one generation: prefill the 16-token prompt, then 128 decode steps.
`value` is decode tokens/s over the timed steps (device time from CUDA events
on the engine's stream; the GPU holds all weights, so no host copies).  `e2e`
is the same workload through the C ABI's cuq_generate with host prompt ids in
and host tokens out, timed by the host clock.  `roofline` measures the
dominant kernel (the Q8_0 quant-GEMV, here the 49152 x 576 lm_head, the
largest single launch) on its own with CUDA events, rotating weight copies
larger than L2.  The weights (142.9 MB) exceed the 126 MB L2, and L2 is also
flushed between timed steps.

N > 1 (torchrun): the path does not shard at this config, so each rank runs an
independent replica (weak scaling); value = all ranks' tokens / max rank time.
`--impl reference`: the reference CPU path (the C oracle restating
src/cpu.zig + main.zig refForward; the Zig reference cannot be built here) on
all host cores, rank 0 only.
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIG = "smollm2-135m"
N_PROMPT, N_DECODE = 16, 128


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", choices=["gemv"], default=None,
                    help="run only the roofline kernel (a few launches) for an ncu capture, print nothing")
    return ap.parse_args()


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region (the profiling recipe's clocks line)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(gpu_index), "--query-gpu=" + self.Q,
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = [l.split(", ") for l in open(self.f.name).read().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def prompt_ids(vocab, seed=0):
    return np.random.default_rng(seed).integers(0, vocab, size=N_PROMPT).astype(np.uint32)


def cpu_baseline(model, threads, n_prompt, n_decode):
    """The oracle (CPU restatement of the reference path) on a bounded sample."""
    from oracle import oracle as orc
    ref = orc.Model(model.cfg, threads=threads, max_seq=n_prompt + n_decode + 1)
    ref.load(model)
    ids = prompt_ids(model.cfg.vocab)[:n_prompt]
    for p, t in enumerate(ids):
        lg = ref.forward(int(t), p)
    tok = orc.argmax(lg)
    t0 = time.perf_counter()
    for s in range(n_decode):
        lg = ref.forward(tok, n_prompt + s)
        tok = orc.argmax(lg)
    dt = time.perf_counter() - t0
    return n_decode / dt


def run_reference(args, world, rank):
    if rank != 0:
        return
    from anedvd_b200 import synth
    model = synth.model(CONFIG)
    threads = os.cpu_count() or 1
    n_prompt, n_decode = 4, 4   # a bounded sample of the workload per step
    vals = []
    for i in range(args.warmup + args.steps):
        v = cpu_baseline(model, threads, n_prompt, n_decode)
        if i >= args.warmup:
            vals.append(v)
    value = float(np.mean(vals))
    print(json.dumps({
        "impl": "reference", "metric": "decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init weights, random prompt ids)",
        "config": {"workload": "c2: SmolLM2-135M-arch Q8_0, batch-1 greedy decode", "model": CONFIG,
                   "prompt": N_PROMPT, "decode": N_DECODE},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": "per step: %d-token prompt then %d greedy decode tokens, oracle refForward "
                                   "(rows split across %d threads, reference per-row order)"
                                   % (n_prompt, n_decode, threads)},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def gemv_roofline(model, stream_ptr, pk, reps=64):
    """Time the lm_head quant-GEMV alone: CUDA events around `reps` back-to-back
    launches on the engine's stream over 8 rotating weight copies (240 MB > L2),
    so every launch streams from HBM; the mean launch duration includes the
    short gap between consecutive launches."""
    import torch
    from anedvd_b200 import runtime as rt
    L = rt.load()
    t = model.tensor("token_embd.weight")
    raw = np.frombuffer(t.data, dtype=np.uint8)
    copies = [L.cuq_weight_create(t.ggml_type, raw.ctypes.data_as(ctypes.c_void_p), raw.size, t.rows, t.cols)
              for _ in range(8)]
    assert all(copies), rt.last_error()
    x = torch.randn(t.cols, device="cuda", dtype=torch.float32)
    xq = torch.empty(L.cuq_xq_halves(t.cols), dtype=torch.int16, device="cuda")
    y = torch.empty(t.rows, device="cuda", dtype=torch.float32)
    stream = torch.cuda.ExternalStream(stream_ptr)
    rt.check(L.cuq_prepare_x(ctypes.c_void_p(x.data_ptr()), t.cols, ctypes.c_void_p(xq.data_ptr()),
                             ctypes.c_void_p(stream_ptr)))
    for i in range(8 if reps > 0 else 6):  # warm-up (profile mode: these are the only launches)
        rt.check(L.cuq_gemv_prepared(copies[i % 8], ctypes.c_void_p(xq.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                     ctypes.c_void_p(stream_ptr)))
    if reps <= 0:
        torch.cuda.synchronize()
        for c in copies:
            L.cuq_weight_free(c)
        return None
    # back-to-back launches on the engine's stream; a spin kernel first lets the
    # host queue them all, so the events time the GPU, not the launch calls
    with torch.cuda.stream(stream):
        torch.cuda._sleep(4_000_000)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        L.cuq_gemv_prepared(copies[i % 8], ctypes.c_void_p(xq.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                            ctypes.c_void_p(stream_ptr))
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    for c in copies:
        L.cuq_weight_free(c)
    alg = t.rows * t.cols * 34 // 32 + 4 * t.cols + 4 * t.rows   # N*K*bpw + 4K + 4N (Q8_0 bpw 34/32)
    achieved = alg / (ms * 1e-3) / 1e9
    traffic = None
    try:
        prof = json.load(open(os.path.join(ROOT, "profiles", "gemv_q8_0_lm_head_traffic.json")))
        traffic = prof.get("dram_bytes_per_launch")
    except (OSError, ValueError):
        pass
    return {"kernel": "gemv_kernel<TQ8_0> (lm_head 49152x576 Q8_0)", "bound": "hbm", "achieved": achieved,
            "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
            "algorithmic_bytes": alg, "launch_us": ms * 1e3}


def run_ours(args, world, rank, local):
    import torch
    from anedvd_b200 import engine as E
    from anedvd_b200 import runtime as rt
    from anedvd_b200 import synth

    torch.cuda.set_device(local)
    pk, pk_kind = peaks()
    model = synth.model(CONFIG)
    max_seq = N_PROMPT + N_DECODE + 8
    eng = E.Engine.from_synth(model, max_seq=max_seq, device=local)
    stream_ptr = eng.stream
    stream = torch.cuda.ExternalStream(stream_ptr)
    ids = prompt_ids(model.cfg.vocab)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")

    def one_step():
        _, first = eng.prefill(ids, 0, want_logits=False)
        return eng.decode_greedy(first, N_PROMPT, N_DECODE)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    dec_ms, pre_ms = 0.0, 0.0
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        _, first = eng.prefill(ids, 0, want_logits=False)
        e1.record(stream)
        eng.decode_greedy(first, N_PROMPT, N_DECODE)
        e2.record(stream)
        torch.cuda.synchronize()
        pre_ms += e0.elapsed_time(e1)
        dec_ms += e1.elapsed_time(e2)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    dec_ms_max = max_over_ranks(dec_ms, world)
    pre_ms_max = max_over_ranks(pre_ms, world)
    tokens = N_DECODE * args.steps * world
    value = tokens / (dec_ms_max * 1e-3)
    prefill_tps = N_PROMPT * args.steps * world / (pre_ms_max * 1e-3)
    kps = eng.stats.kernels_per_step

    # end to end through the C ABI: host prompt ids in, host tokens out (cuq_generate)
    sess = E.Session(eng, max_seq)
    sess.generate(ids, N_DECODE)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sess.generate(ids, N_DECODE)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = N_DECODE * args.steps * world / e2e_s

    roof = gemv_roofline(model, stream_ptr, pk) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n_p, n_d = 16, 48
        cpu = {"value": cpu_baseline(model, 1, n_p, n_d), "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": "%d-token prompt, then %d greedy decode tokens timed; single thread (the reference "
                         "engine is single-threaded), oracle refForward in the reference's scalar order" % (n_p, n_d)}
    if rank == 0:
        line = {
            "metric": "decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": (dec_ms_max + pre_ms_max) / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 weights, fp16 tensor-core "
            "MMA with fp32 accumulate, fp32 activations",
            "data": "synthetic (seeded random-init weights, random prompt ids)",
            "config": {"workload": "c2: SmolLM2-135M-arch Q8_0 (30 layers, hidden 576, vocab 49152), batch-1 "
                                   "greedy decode of 128 tokens after a 16-token prompt",
                       "model": CONFIG, "prompt": N_PROMPT, "decode": N_DECODE,
                       "parallelism": "replicas" if world > 1 else "single GPU",
                       "l2": "flushed between steps; weights 142.9 MB > 126 MB L2"},
            "prefill_tok_per_s": prefill_tps,
            "weight_bytes_per_token": model.weight_bytes_per_token(),
            "weight_stream_gbs": model.weight_bytes_per_token() * value / world / 1e9,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 * N_PROMPT + 4,
                    "d2h_bytes_per_step": 4 * N_DECODE},
            "roofline": roof, "peak_kind": pk_kind, "cpu_baseline": cpu,
            "gpu_launches": int(kps * (N_PROMPT + N_DECODE) * args.steps),
            "kernels_per_token": int(kps),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    eng.close()


def profile_case(args):
    """A handful of launches of the roofline kernel alone (3 warm-up + 3), for
    `ncu -k regex:gemv_kernel -s 3 -c 3`; nothing printed."""
    import torch
    from anedvd_b200 import runtime as rt
    from anedvd_b200 import synth
    rt.load()
    rt.init(0)
    torch.cuda.set_device(0)
    if args.profile == "gemv":
        s = torch.cuda.Stream()
        gemv_roofline(synth.model(CONFIG), s.cuda_stream, peaks()[0], reps=0)  # 6 launches
    torch.cuda.synchronize()


def main():
    args = parse()
    if args.profile:
        profile_case(args)
        return
    world, rank, local = dist_init()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
