"""Tensor-parallel host logic on CPU (no GPU): the raw-tensor shard helpers of
the C ABI, and the Megatron split arithmetic of the Llama-3-8B shape checked with
two `gloo` ranks against the oracle's full-matrix results.

Column-parallel (q/k/v/gate/up/lm_head rows) must reassemble bit-exactly;
row-parallel (o/down whole-block columns) partial sums, all-reduced, must match
the full matvec to fp32 rounding; the cross-rank argmax packs (orderable value,
~index) into 64 bits so that a max-reduction keeps the reference's first-index
tie rule (cpu.zig:477-483).
"""
import ctypes
import os
import socket

import numpy as np
import pytest

from anedvd_b200 import quant, runtime as rt, synth
from oracle import oracle as orc

TYPES = [(8, "q8_0"), (12, "q4_k"), (14, "q6_k"), (2, "q4_0"), (1, "f16")]


def _raw(ttype, rows, cols, key):
    w = synth.seeded_normal(key, rows * cols)
    return np.ascontiguousarray(quant.quantize(ttype, w).view(np.uint8))


def _deq(ttype, raw, rows, cols):
    return orc.dequant(ttype, raw, rows * cols).reshape(rows, cols)


@pytest.mark.parametrize("ttype,name", TYPES, ids=[t[1] for t in TYPES])
def test_shard_rows_and_cols_are_exact(ttype, name):
    L = rt.load()
    rows, cols = 64, 1024
    raw = _raw(ttype, rows, cols, "tp/shard/" + name)
    full = _deq(ttype, raw, rows, cols)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    for r0, r1 in ((0, 16), (16, 48), (48, 64)):
        out = np.zeros(raw.size * (r1 - r0) // rows, dtype=np.uint8)
        rt.check(L.cuq_shard_rows(ttype, rows, cols, r0, r1, p(raw), p(out)))
        assert np.array_equal(_deq(ttype, out, r1 - r0, cols), full[r0:r1])
    for c0, c1 in ((0, 256), (256, 768), (768, 1024)):
        out = np.zeros(raw.size * (c1 - c0) // cols, dtype=np.uint8)
        rt.check(L.cuq_shard_cols(ttype, rows, cols, c0, c1, p(raw), p(out)))
        assert np.array_equal(_deq(ttype, out, rows, c1 - c0), full[:, c0:c1])


def test_shard_cols_rejects_partial_blocks():
    L = rt.load()
    raw = _raw(12, 16, 512, "tp/partial")
    out = np.zeros(raw.size, dtype=np.uint8)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    assert L.cuq_shard_cols(12, 16, 512, 0, 128, p(raw), p(out)) == rt.EINVAL
    assert "whole blocks" in rt.last_error()


def _pack(v, idx):
    u = np.float32(v).view(np.uint32)
    key = (~u) & 0xFFFFFFFF if u & 0x80000000 else u | 0x80000000
    return (int(key) << 32) | (0xFFFFFFFF - int(idx))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L = rt.load()
        p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
        hidden, inter = 512, 1024
        x = synth.seeded_normal("tp/x", hidden, std=1.0)
        # column-parallel gate rows: every rank's slice, gathered, is the full output
        raw_g = _raw(12, inter, hidden, "tp/gate")
        r0, r1 = rank * inter // world, (rank + 1) * inter // world
        sh = np.zeros(raw_g.size // world, dtype=np.uint8)
        rt.check(L.cuq_shard_rows(12, inter, hidden, r0, r1, p(raw_g), p(sh)))
        w16 = orc.f32_to_f16_bits(_deq(12, sh, r1 - r0, hidden))
        y_loc = orc.matvec_f16(w16, x)
        parts = [torch.zeros(r1 - r0) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(y_loc))
        y_full = orc.matvec_f16(orc.f32_to_f16_bits(_deq(12, raw_g, inter, hidden)), x)
        assert np.array_equal(torch.cat(parts).numpy(), y_full)
        # row-parallel down columns: partial sums all-reduced = full matvec (fp32 rounding)
        raw_d = _raw(12, hidden, inter, "tp/down")
        a = synth.seeded_normal("tp/a", inter, std=1.0)
        c0, c1 = rank * inter // world, (rank + 1) * inter // world
        sd = np.zeros(raw_d.size // world, dtype=np.uint8)
        rt.check(L.cuq_shard_cols(12, hidden, inter, c0, c1, p(raw_d), p(sd)))
        part = orc.matvec_f16(orc.f32_to_f16_bits(_deq(12, sd, hidden, c1 - c0)), a[c0:c1])
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        want = orc.matvec_f16(orc.f32_to_f16_bits(_deq(12, raw_d, hidden, inter)), a)
        assert np.max(np.abs(t.numpy() - want)) <= 1e-5 * np.max(np.abs(want))
        # cross-rank argmax with a tie planted across ranks: the smaller index wins
        logits = synth.seeded_normal("tp/logits", 64 * world).copy()
        logits[5] = logits[64 + 7] = np.float32(9.0)
        mine = logits[rank * 64:(rank + 1) * 64]
        li = int(np.argmax(mine))
        key = _pack(mine[li], rank * 64 + li)
        kt = torch.tensor([key - (1 << 63)], dtype=torch.int64)  # unsigned order as signed
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
        best = int(kt.item()) + (1 << 63)
        assert 0xFFFFFFFF - (best & 0xFFFFFFFF) == orc.argmax(logits) == 5
    finally:
        dist.destroy_process_group()


def test_megatron_split_two_gloo_ranks():
    import torch.multiprocessing as mp
    mp.spawn(_rank, args=(2, _free_port()), nprocs=2, join=True)
