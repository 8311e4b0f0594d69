"""Failure detection of the tensor-parallel exchange on one GPU, with the
failure made on the host: rank 0 of a 2-rank model is connected to a rank that
never joins (an all-zero handle, i.e. a dropped handshake message), so every
wait for that rank's partial sums runs out after the model's wait limit.  The
call must come back with CUQ_ETIMEOUT (the reference surfaces engine failures
as error unions, engine.zig:549,981) within a bounded time, cuq_reset must
leave a model that fails the same way again rather than hanging, and the GPU
context must stay usable: a single-GPU model in the same process afterwards
still matches the CPU oracle.  No GPU fault, trap or hang is involved: every
device wait is bounded and the kernels carry on after it."""
import time

import numpy as np
import pytest

from anedvd_b200 import engine as E
from anedvd_b200 import runtime as rt
from anedvd_b200 import synth
from oracle import oracle as orc

from .gpu_util import rel_err

pytestmark = pytest.mark.gpu


def test_rank_that_never_joins_times_out_and_the_context_survives():
    m = synth.model("llama3-8b", layers=1, vocab=1024, payload="tiled")
    limit_ms = 100
    eng = E.Engine.from_synth(m, max_seq=16, device=0, tp_rank=0, tp_size=2, wait_limit_ms=limit_ms,
                              exchange=lambda h: [h, bytes(rt.TP_HANDLE_BYTES)])
    for attempt in range(2):
        t0 = time.monotonic()
        with pytest.raises(rt.CuqError) as e:
            eng.forward(5, 0)
        dt = time.monotonic() - t0
        assert e.value.code == rt.ETIMEOUT, e.value
        assert "peer" in str(e.value)
        # o and down reductions and the argmax exchange: three waits of limit_ms each
        assert dt < 20 * limit_ms / 1000.0, dt
        eng.reset()
    eng.close()

    # the context is intact: an ordinary model still runs and matches the oracle
    m2 = synth.model("smollm2-135m", layers=2, vocab=1024)
    eng2 = E.Engine.from_synth(m2, max_seq=16, device=0)
    ref = orc.Model(m2.cfg, threads=4, max_seq=16)
    ref.load(m2)
    ids = np.array([3, 141, 59, 265], dtype=np.uint32)
    for p, t in enumerate(ids):
        want = ref.forward(int(t), p)
    got, am = eng2.prefill(ids)
    assert rel_err(got, want) < 2e-3
    eng2.close()
