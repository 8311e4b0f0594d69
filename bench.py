#!/usr/bin/env python3
"""Benchmark of the quantized-weight decode/prefill path, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c3|c4|c5] [--profile gemv]

Workloads are the configs of the benchmark (random-init synthetic models of
the named architectures, seeded random prompt ids):
  c2  SmolLM2-135M-arch, Q8_0, 16-token prompt + 128 greedy tokens
  c3  Qwen2.5-0.5B-arch, Q8_0, 203 + 256
  c4  Qwen2.5-1.5B-arch, Q4_K_M mix, 2048 + 256
  c5  Llama-3-8B-arch, Q4_K_M mix, 4096 + 512  (the default: 1 GPU, or tensor
      parallel over the N ranks of a torchrun launch)

A step is one generation: prefill the prompt, then the decode tokens.  `value`
is decode tokens/s over the timed steps (device time from CUDA events on the
engine's stream, max over ranks); `prefill` reports the prompt pass the same
way.  `e2e` is the same workload through the public API (cuq_generate: host
prompt ids in, host tokens out) timed by the host clock, prefill included.
`kernels` is the per-node table of cuq_profile_decode (8 decode steps in the
timed window, one launch at a time with a CUDA event after each on the
engine's stream); `roofline` is that table's dominant node (algorithmic bytes
per launch / mean launch time) and `step_hbm` the whole decode step (weights +
the K/V rows read, per token, at the measured tok/s).  L2 (126 MB) is flushed
between timed steps; the weights (4.6 GB for c5) are far larger than L2.

N > 1 (torchrun): c5 runs tensor-parallel (one sequence, strong scaling: value
is that sequence's tokens/s); c2-c4 do not shard and run one replica per rank
(weak scaling: value = all ranks' tokens / max rank time).
`--impl reference`: the reference CPU path (the C oracle restating src/cpu.zig
+ main.zig refForward; the Zig reference cannot be built here) on all host
cores, rank 0 only (the other ranks exit at once), loaded once; each step
times decode tokens at positions inside the same decode window as this arm
(the attention walks the same number of cached positions; a CPU prefill of
the 4096-token prompt would take hours, and the work of a decode step does not
depend on the cached values).
`--profile gemv`: 6 launches of the config's lm_head GEMV only; `--profile
qgemm`: 4 prefill GEMMs of the config's first ffn_gate on 2048 tokens;
`--profile prefill` / `decode`: the model's prefill twice / 4 eager decode
steps (for ncu captures; nothing is printed).
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

CONFIGS = {
    "c2": dict(model="smollm2-135m", prompt=16, decode=128, payload="quantized", head="token_embd.weight",
               ref_tokens=8, cpu_tokens=48, cpu_threads=1,
               desc="c2: SmolLM2-135M-arch Q8_0 (30 layers, hidden 576, vocab 49152), batch-1 greedy decode of 128 "
                    "tokens after a 16-token prompt"),
    "c3": dict(model="qwen2.5-0.5b", prompt=203, decode=256, payload="tiled", head="token_embd.weight",
               ref_tokens=4, cpu_tokens=12, cpu_threads=1,
               desc="c3: Qwen2.5-0.5B-arch Q8_0 (24 layers, hidden 896, vocab 151936), 203-token prompt + 256 "
                    "greedy tokens"),
    "c4": dict(model="qwen2.5-1.5b", prompt=2048, decode=256, payload="tiled", head="token_embd.weight",
               ref_tokens=2, cpu_tokens=8, cpu_threads=0,
               desc="c4: Qwen2.5-1.5B-arch Q4_K_M mix (28 layers, hidden 1536, vocab 151936), 2048-token prompt + "
                    "256 greedy tokens"),
    "c5": dict(model="llama3-8b", prompt=4096, decode=512, payload="tiled", head="output.weight",
               ref_tokens=2, cpu_tokens=8, cpu_threads=0,
               desc="c5: Llama-3-8B-arch Q4_K_M mix (32 layers, hidden 4096, vocab 128256 untied), 4096-token "
                    "prompt + 512 greedy tokens"),
}
DATA = {"quantized": "synthetic: seeded N(0,0.02) weights quantized per tensor, seeded random prompt ids",
        "tiled": "synthetic: every block is one of 256 real quantized blocks of seeded N(0,0.02) weights per tensor "
                 "(valid blocks, same statistics; throughput does not depend on values), seeded random prompt ids"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=None, choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode-kernel", choices=["auto", "per_op", "persistent"], default="auto",
                    help="decode steps in one persistent kernel (auto: when the model allows) or one kernel per op")
    ap.add_argument("--persistent-ctas", type=int, default=0, help="CTAs per SM of the persistent kernel (0 = max)")
    ap.add_argument("--profile", choices=["gemv", "qgemm", "prefill", "decode"], default=None,
                    help="run only the roofline kernel (a few launches) for an ncu capture, print nothing")
    ap.add_argument("--layers", type=int, default=0,
                    help="--profile prefill/decode: a model of this many layers (same shapes; 0 = the config's)")
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


def prompt_ids(vocab, n, seed=0):
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.uint32)


class CpuReference:
    """The oracle (CPU restatement of the reference path, refForward in the
    reference's per-row order) for one config, loaded once.  Decode tokens are
    timed at positions inside the config's decode window: a decode step's work
    (every weight once, attention over pos + 1 cached rows) does not depend on
    the cached values, so no CPU prefill of the prompt is needed first."""

    def __init__(self, model, C, threads):
        from oracle import oracle as orc
        self.orc = orc
        self.C = C
        self.threads = threads
        self.ref = orc.Model(model.cfg, threads=threads, max_seq=C["prompt"] + C["decode"] + 1)
        self.ref.load(model)
        self.vocab = model.cfg.vocab
        self.k = 0

    def positions(self, n):
        """n positions spread over the decode window [prompt, prompt + decode)."""
        P, D = self.C["prompt"], self.C["decode"]
        out = []
        for _ in range(n):
            out.append(P + (self.k * 97) % D)
            self.k += 1
        return out

    def time_tokens(self, n):
        """Seconds for n decode tokens (greedy: each token is the previous argmax)."""
        tok = 1
        t0 = time.perf_counter()
        for pos in self.positions(n):
            tok = self.orc.argmax(self.ref.forward(tok, pos))
        return time.perf_counter() - t0

    def sample_desc(self, n, what):
        return ("%s: %d greedy decode tokens at positions spread over the decode window [%d, %d) of the same "
                "workload, oracle refForward (rows and query heads split across %d threads, reference per-row "
                "order)" % (what, n, self.C["prompt"], self.C["prompt"] + self.C["decode"], self.threads))


def pick_config(args, world):
    return args.config or "c5"


def line_config(C, name, world, tp):
    parallelism = ("tensor parallel x%d" % world) if tp else ("replicas x%d" % world if world > 1 else "single GPU")
    return {"workload": C["desc"], "model": C["model"], "prompt": C["prompt"], "decode": C["decode"],
            "parallelism": parallelism,
            "l2": "flushed between timed steps (256 MB write); the weights stream from HBM every token"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    from anedvd_b200 import synth
    name = pick_config(args, world)
    C = CONFIGS[name]
    tp = world > 1 and name == "c5"
    model = synth.model(C["model"], payload=C["payload"], cache=False)
    threads = os.cpu_count() or 1
    ref = CpuReference(model, C, threads)
    n_tok = C["ref_tokens"]
    dt = 0.0
    for i in range(args.warmup + args.steps):
        t = ref.time_tokens(n_tok)
        if i >= args.warmup:
            dt += t
    value = n_tok * args.steps / dt
    print(json.dumps({
        "impl": "reference", "metric": "decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "f32",
        "data": DATA[C["payload"]],
        "config": line_config(C, name, world, tp),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": ref.sample_desc(n_tok, "per step")},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def head_shard(model, C, rank, world):
    """The config's lm_head weight (this rank's vocab rows under tensor parallelism)."""
    t = model.tensor(C["head"])
    raw = np.frombuffer(t.data, dtype=np.uint8)
    rows = t.rows // world
    row_bytes = raw.size // t.rows
    return t.ggml_type, np.ascontiguousarray(raw[rank * rows * row_bytes:(rank + 1) * rows * row_bytes]), rows, t.cols


def gemv_roofline(ttype, raw, rows, cols, stream_ptr, pk, label, reps=64):
    """Time one quant-GEMV alone: CUDA events around `reps` back-to-back launches
    on the engine's stream over rotating weight copies (> 2 x L2 in total), so
    every launch streams from HBM; the mean launch duration includes the short
    gap between consecutive launches."""
    import torch
    from anedvd_b200 import gguf
    from anedvd_b200 import runtime as rt
    L = rt.load()
    ncopy = int(min(16, max(2, np.ceil(260e6 / raw.size))))
    copies = [L.cuq_weight_create(ttype, raw.ctypes.data_as(ctypes.c_void_p), raw.size, rows, cols)
              for _ in range(ncopy)]
    assert all(copies), rt.last_error()
    x = torch.randn(cols, device="cuda", dtype=torch.float32)
    xq = torch.empty(L.cuq_xq_halves(cols), dtype=torch.int16, device="cuda")
    y = torch.empty(rows, device="cuda", dtype=torch.float32)
    stream = torch.cuda.ExternalStream(stream_ptr)
    args = lambda i: (copies[i % ncopy], ctypes.c_void_p(xq.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                      ctypes.c_void_p(stream_ptr))
    rt.check(L.cuq_prepare_x(ctypes.c_void_p(x.data_ptr()), cols, ctypes.c_void_p(xq.data_ptr()),
                             ctypes.c_void_p(stream_ptr)))
    for i in range(8 if reps > 0 else 6):  # warm-up (profile mode: these are the only launches)
        rt.check(L.cuq_gemv_prepared(*args(i)))
    if reps <= 0:
        torch.cuda.synchronize()
        for c in copies:
            L.cuq_weight_free(c)
        return None
    # a spin kernel first lets the host queue every launch, so the events time the GPU
    with torch.cuda.stream(stream):
        torch.cuda._sleep(4_000_000)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        L.cuq_gemv_prepared(*args(i))
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    for c in copies:
        L.cuq_weight_free(c)
    alg = gguf.tensor_nbytes(ttype, rows * cols) + 4 * cols + 4 * rows   # N*K*bpw + 4K + 4N
    achieved = alg / (ms * 1e-3) / 1e9
    traffic = None
    try:
        prof = json.load(open(os.path.join(ROOT, "profiles", "roofline_traffic.json")))
        traffic = prof.get(label, {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        pass
    tname = {8: "TQ8_0", 12: "TQ4K", 14: "TQ6K"}.get(ttype, str(ttype))
    return {"kernel": "gemv_kernel<%s> (%s %dx%d)" % (tname, label, rows, cols), "bound": "hbm",
            "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
            "traffic": traffic, "algorithmic_bytes": alg, "launch_us": ms * 1e3}


# the kernel behind each node of the per-op decode step
NODE_KERNEL = {"embed": "embed_norm_kernel", "qkv": "%s, q||k||v (+ v when its type differs)",
               "attention": "attn_step_kernel", "o": "%s + residual",
               "gate_up": "%s, gate|up + SiLU*mul",
               "down": "%s + residual", "lm_head": "gemv_kernel + argmax",
               "norm": "rmsnorm_xq_kernel"}


def node_kernel(node, weight_bytes):
    """The kernel behind a decode node: the layer GEMVs are TMA-fed when a rank
    streams at least 2 GiB of weights per token, else register-prefetch; the
    lm_head always runs the register-prefetch kernel."""
    k = NODE_KERNEL.get(node, node)
    return k % ("gemv_tma_kernel" if weight_bytes >= (2 << 30) else "gemv_kernel") if "%s" in k else k


def tp_check(world, rank, local, exchange):
    """Correctness of the tensor-parallel path on this launch, outside the timed
    region: a 2-layer Llama-3-8B-shaped model (full width, vocab 4096) runs a
    12-token prompt and 4 decode steps across the ranks; rank 0 gathers the
    logit slices and compares them with the same model on one GPU, whose path
    the GPU test suite checks against the CPU oracle.  Returns the largest
    relative logits difference (max|a-b|/max|b|) and whether every greedy token
    agrees (rank 0; None elsewhere)."""
    import torch.distributed as dist
    from anedvd_b200 import engine as E
    from anedvd_b200 import synth
    m = synth.model("llama3-8b", layers=2, vocab=4096, payload="tiled", cache=False)
    ids = prompt_ids(m.cfg.vocab, 12, seed=3)
    n_dec = 4
    eng = E.Engine.from_synth(m, max_seq=32, device=local, max_chunk=64, tp_rank=rank, tp_size=world,
                              exchange=exchange)
    got = []
    barrier(world)
    lg, am = eng.prefill(ids, 0)
    got.append((lg, am))
    for s in range(n_dec):
        lg, am = eng.forward(got[-1][1], ids.size + s)
        got.append((lg, am))
    eng.close()
    parts = [None] * world
    dist.all_gather_object(parts, got)
    res = None
    if rank == 0:
        one = E.Engine.from_synth(m, max_seq=32, device=local, max_chunk=64)
        rel, same = 0.0, True
        want, wam = one.prefill(ids, 0)
        for s in range(n_dec + 1):
            if s:
                want, wam = one.forward(got[s - 1][1], ids.size + s - 1)
            full = np.concatenate([parts[r][s][0] for r in range(world)])
            rel = max(rel, float(np.max(np.abs(full - want)) / np.max(np.abs(want))))
            same = same and all(parts[r][s][1] == wam for r in range(world))
        one.close()
        res = {"model": "llama3-8b shape, 2 layers, vocab 4096", "prompt": int(ids.size), "decode_steps": n_dec,
               "reference": "the same model on one GPU", "max_rel_logits_diff": rel, "greedy_tokens_equal": same}
    barrier(world)
    return res


def run_ours(args, world, rank, local):
    import torch
    from anedvd_b200 import engine as E
    from anedvd_b200 import synth

    name = pick_config(args, world)
    C = CONFIGS[name]
    tp = world > 1 and name == "c5"
    torch.cuda.set_device(local)
    pk, pk_kind = peaks()
    model = synth.model(C["model"], payload=C["payload"], cache=False)
    n_prompt, n_decode = C["prompt"], C["decode"]
    max_seq = n_prompt + n_decode + 8

    def exchange(h):
        import torch.distributed as dist
        out = [None] * world
        dist.all_gather_object(out, h)
        return out

    dk = {"auto": 0, "per_op": 1, "persistent": 2}[args.decode_kernel]
    eng = E.Engine.from_synth(model, max_seq=max_seq, device=local, max_chunk=2048,
                              tp_rank=rank if tp else 0, tp_size=world if tp else 1, exchange=exchange,
                              decode_kernel=dk, persistent_ctas=args.persistent_ctas)
    persistent = eng.persistent_ctas > 0
    stream_ptr = eng.stream
    stream = torch.cuda.ExternalStream(stream_ptr)
    ids = prompt_ids(model.cfg.vocab, n_prompt)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")

    for _ in range(args.warmup):
        barrier(world)
        _, first = eng.prefill(ids, 0, want_logits=False)
        eng.decode_greedy(first, n_prompt, n_decode)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    launches0 = eng.stats.kernel_launches
    dec_ms, pre_ms = 0.0, 0.0
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        _, first = eng.prefill(ids, 0, want_logits=False)
        e1.record(stream)
        eng.decode_greedy(first, n_prompt, n_decode)
        e2.record(stream)
        torch.cuda.synchronize()
        pre_ms += e0.elapsed_time(e1)
        dec_ms += e1.elapsed_time(e2)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    launches = eng.stats.kernel_launches - launches0
    dec_ms_max = max_over_ranks(dec_ms, world)
    pre_ms_max = max_over_ranks(pre_ms, world)
    seqs = 1 if tp else world   # tensor parallel: the ranks share one sequence
    value = n_decode * args.steps * seqs / (dec_ms_max * 1e-3)
    prefill_tps = n_prompt * args.steps * seqs / (pre_ms_max * 1e-3)
    kps = eng.stats.kernels_per_step

    # end to end through the public API: host prompt ids in, host tokens out (cuq_generate)
    sess = E.Session(eng, max_seq)
    barrier(world)
    sess.generate(ids, n_decode)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sess.generate(ids, n_decode)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = n_decode * args.steps * seqs / e2e_s

    # per-node decode table (cuq_profile_decode) in the timed decode window;
    # the roofline is its dominant node, the step fraction the whole token
    _, first = eng.prefill(ids, 0, want_logits=False)
    n_prof = 8
    table = eng.profile_decode(first, n_prompt, n_prof)
    kernels = {k: {"launches": v[0], "ms": v[1], "bytes": v[2],
                   "us_per_launch": (1e3 * v[1] / v[0]) if v[0] else None,
                   "gbs": (v[2] / (v[1] * 1e-3) / 1e9) if v[1] > 0 else None} for k, v in table.items()}
    dom = max(kernels, key=lambda k: kernels[k]["ms"])
    dk_ = kernels[dom]
    per_launch_bytes = dk_["bytes"] / max(dk_["launches"], 1)
    achieved = dk_["gbs"]
    traffic = None
    try:
        prof = json.load(open(os.path.join(ROOT, "profiles", "roofline_traffic.json")))
        traffic = prof.get("%s %s" % (name, dom), {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        pass
    wlocal = sum(v["bytes"] for k, v in kernels.items() if k != "attention") / n_prof
    roof = {"kernel": "%s node of the %s decode step (%s)" % (dom, name, node_kernel(dom, wlocal)), "bound": "hbm",
            "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
            "traffic": traffic, "algorithmic_bytes": per_launch_bytes, "launch_us": dk_["us_per_launch"],
            "timing": "in-step, %d decode steps at positions %d..%d, CUDA events after every launch on the "
                      "engine's stream (no graph, no overlap between kernels)" % (n_prof, n_prompt,
                                                                                 n_prompt + n_prof - 1),
            "share_of_step": dk_["ms"] / sum(v["ms"] for v in kernels.values())}
    # whole step: this rank's weights once + the K/V rows over the decode window, per token
    cfg = model.cfg
    kvd_local = cfg.kv_heads * cfg.head_dim // (world if tp else 1)
    kv_avg = 2 * 2 * kvd_local * cfg.layers * (n_prompt + (n_decode + 1) / 2.0)
    step_bytes = wlocal + kv_avg
    step_gbs = step_bytes * value / seqs / 1e9
    step_hbm = {"bytes_per_token": step_bytes, "weight_bytes_per_token": wlocal, "kv_bytes_per_token": kv_avg,
                "achieved": step_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": step_gbs / pk["hbm_gbs"]}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = C["cpu_threads"] or (os.cpu_count() or 1)
        ref = CpuReference(model, C, threads)
        ref.time_tokens(1)  # warm-up
        n_tok = C["cpu_tokens"]
        cpu = {"value": n_tok / ref.time_tokens(n_tok), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": ref.sample_desc(n_tok, "bounded sample")}
        del ref
    wbytes = model.weight_bytes_per_token()
    tpc = tp_check(world, rank, local, exchange) if tp else None
    if rank == 0:
        line = {
            "metric": "decode_tok_per_s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": (dec_ms_max + pre_ms_max) / args.steps,
            "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "%s weights dequantized exactly to fp16, fp16 tensor-core MMA with fp32 accumulate, fp32 "
                     "activations (split hi+lo fp16)" % ("q8_0" if name in ("c2", "c3") else "q4_k/q6_k"),
            "data": DATA[C["payload"]],
            "config": line_config(C, name, world, tp),
            "decode_kernel": ("persistent, %d CTAs" % eng.persistent_ctas) if persistent else
                             "one kernel per op (CUDA graph per step)",
            "prefill": {"tok_per_s": prefill_tps, "ms": pre_ms_max / args.steps},
            "weight_bytes_per_token": wbytes,
            "weight_stream_gbs": wbytes * value / seqs / 1e9,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 * n_prompt + 4 * 1,
                    "d2h_bytes_per_step": 4 * n_decode},
            "kernels": kernels, "step_hbm": step_hbm,
            "roofline": roof, "peak_kind": pk_kind, "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "tp_check": tpc,
            "kernels_per_token": (1.0 / n_decode) if persistent else int(kps),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    barrier(world)
    eng.close()


def profile_case(args):
    """Small launch sets for ncu, nothing printed: gemv = the roofline kernel
    alone (6 launches, `ncu -k regex:gemv_kernel -s 3 -c 1`); qgemm = one
    prefill GEMM (4 launches); prefill / decode = the config's model end to end
    (launch lists)."""
    import torch
    from anedvd_b200 import runtime as rt
    from anedvd_b200 import synth
    rt.load()
    rt.init(0)
    torch.cuda.set_device(0)
    name = args.config or "c5"
    C = CONFIGS[name]
    extra = {"layers": args.layers} if args.layers else {}
    model = synth.model(C["model"], payload=C["payload"], cache=False, **extra)
    if args.profile == "gemv":
        s = torch.cuda.Stream()
        ttype, raw, rows, cols = head_shard(model, C, 0, 1)
        gemv_roofline(ttype, raw, rows, cols, s.cuda_stream, peaks()[0], name, reps=0)
    elif args.profile == "qgemm":
        # the prefill GEMM of the config's first ffn_gate on a 2048-token chunk, 4 launches
        L = rt.load()
        t = model.tensor("blk.0.ffn_gate.weight")
        raw = np.frombuffer(t.data, dtype=np.uint8)
        h = L.cuq_weight_create(t.ggml_type, raw.ctypes.data_as(ctypes.c_void_p), raw.size, t.rows, t.cols)
        assert h, rt.last_error()
        x = torch.randn(2048, t.cols, device="cuda")
        y = torch.empty(2048, t.rows, device="cuda")
        for _ in range(4):
            rt.check(L.cuq_gemm(h, ctypes.c_void_p(x.data_ptr()), 2048, ctypes.c_void_p(y.data_ptr()), None))
        L.cuq_weight_free(h)
    elif args.profile in ("prefill", "decode"):
        # prefill: the config's prompt prefilled twice (chunks of 2048).
        # decode: 4 tokens decoded at the first decode position with one kernel
        # per op and no graph, so every launch of a step shows in a launch list;
        # no prefill first (the KV cache is zeros: the same work per step)
        from anedvd_b200 import engine as E
        ids = prompt_ids(model.cfg.vocab, C["prompt"])
        eng = E.Engine.from_synth(model, max_seq=C["prompt"] + 16, max_chunk=2048,
                                  use_graphs=args.profile == "prefill")
        if args.profile == "prefill":
            eng.prefill(ids, 0, want_logits=False)
            eng.prefill(ids, 0, want_logits=False)
        else:
            eng.decode_greedy(1, C["prompt"], 4)
        eng.close()
    torch.cuda.synchronize()


def main():
    args = parse()
    if args.profile:
        profile_case(args)
        return
    if args.impl == "reference":
        # CPU only, rank 0 alone: no process group (the other ranks exit at once)
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_init()
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
