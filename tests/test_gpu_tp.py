"""Tensor parallelism on 2 GPUs (the Llama-3-8B Megatron split) against the CPU
oracle: one spawned process per GPU, each with its shard of the same synthetic
model; the ranks exchange IPC handles over a `gloo` group and the partial sums
inside the CUDA step kernels.  Rank 0 gathers the logit slices and checks them
against the oracle's full refForward (2e-3, main.zig:1920-1930), and every
rank's argmax against the oracle's.  Skipped with fewer than 2 GPUs.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
LOGIT_TOL = 2e-3

CASES = [("llama3-8b", dict(layers=2, vocab=1024, payload="tiled"), 512),   # Q4_K_M mix, untied, adjacent RoPE
         ("qwen2.5-0.5b", dict(layers=2, vocab=1024), 4)]                   # Q8_0, tied, biases, chunked prefill


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, name, kw, max_chunk):
    import torch
    import torch.distributed as dist
    from anedvd_b200 import engine as E
    from anedvd_b200 import synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        m = synth.model(name, **kw)
        n_prompt, n_dec = 9, 4

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        eng = E.Engine.from_synth(m, max_seq=32, device=rank, max_chunk=max_chunk, tp_rank=rank, tp_size=world,
                                  exchange=exchange)
        ids = np.random.default_rng(7).integers(0, m.cfg.vocab, n_prompt).astype(np.uint32)
        got, ams = [], []
        dist.barrier()
        lg, am = eng.prefill(ids, 0)
        got.append(lg)
        ams.append(am)
        toks = [am]
        for s in range(n_dec):
            dist.barrier()
            lg, am = eng.forward(toks[-1], n_prompt + s)
            got.append(lg)
            ams.append(am)
            toks.append(am)
        # generate() on the device: identical tokens on every rank
        dist.barrier()
        eng.reset()
        gen = E.Session(eng, 32).generate(ids, n_dec + 1)
        eng.close()
        parts = [None] * world
        dist.all_gather_object(parts, (got, ams, list(gen)))
        if rank == 0:
            from oracle import oracle as orc
            ref = orc.Model(m.cfg, threads=8, max_seq=32)
            ref.load(m)
            for r in range(world):
                assert parts[r][1] == ams, (r, parts[r][1], ams)       # same global argmax everywhere
                assert parts[r][2] == toks, (r, parts[r][2], toks)     # device generate == stepwise
            seq = list(ids) + toks[:-1]
            errs = []
            want = None
            for p, t in enumerate(seq[:n_prompt]):
                want = ref.forward(int(t), p)
            checks = [want]
            for s in range(n_dec):
                checks.append(ref.forward(int(toks[s]), n_prompt + s))
            for i, w in enumerate(checks):
                full = np.concatenate([parts[r][0][i] for r in range(world)])
                errs.append(float(np.max(np.abs(full - w)) / np.max(np.abs(w))))
                top = np.sort(w)[-2:]
                if top[1] - top[0] > LOGIT_TOL * np.max(np.abs(w)):
                    assert ams[i] == orc.argmax(w), (i, ams[i], orc.argmax(w))
            assert max(errs) < LOGIT_TOL, errs
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,kw,max_chunk", CASES, ids=[c[0] for c in CASES])
def test_tp2_matches_reference(name, kw, max_chunk):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_rank, args=(2, _free_port(), name, kw, max_chunk), nprocs=2, join=True)
