"""Host-side mirror of the reference engine's interface over the C ABI.

`Engine` keeps the shape of ``src/engine.zig``'s Engine -- ``forward(token,
pos)`` (engine.zig:547), ``prefill(ids, start_pos)`` (engine.zig:975),
``reset()`` (engine.zig:1479), ``stats`` -- and `Session.generate` follows
``src/generate.zig:166-250`` for greedy decoding: truncate the prompt to the
context, prefill, then decode on the device with no per-token host round-trip.
Errors surface as `CuqError` with the library's status code (``ECONTEXT`` is
the reference's ``error.ContextOverflow``).
"""

import ctypes

import numpy as np

from . import runtime as rt


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class Engine:
    """A model resident on one GPU, built from a GGUF file or uploaded tensors."""

    def __init__(self, handle, cfg, tp_rank=0, tp_size=1):
        self._h = handle
        self.cfg = cfg  # CuqConfig
        self._tp = (tp_rank, tp_size)
        # logits returned by forward/prefill: this rank's vocab slice
        self.local_vocab = cfg.vocab // tp_size
        self.vocab_base = self.local_vocab * tp_rank

    @classmethod
    def from_gguf(cls, path, max_seq=2048, use_graphs=True, device=0, max_chunk=512, decode_kernel=rt.DECODE_AUTO,
                  persistent_ctas=0):
        L = rt.load()
        rt.init(device)
        opts = rt.CuqOptions(max_seq=max_seq, max_chunk=max_chunk, use_graphs=int(use_graphs), tp_rank=0, tp_size=1,
                             decode_kernel=decode_kernel, persistent_ctas=persistent_ctas)
        h = L.cuq_model_load_gguf(path.encode(), ctypes.byref(opts))
        if not h:
            raise rt.CuqError(rt.EINVAL, rt.last_error())
        cfg = rt.CuqConfig()
        rt.check(L.cuq_model_get_config(h, ctypes.byref(cfg)))
        return cls(h, cfg)

    @classmethod
    def from_hf(cls, path, max_seq=2048, use_graphs=True, device=0, max_chunk=512, decode_kernel=rt.DECODE_AUTO):
        """A HuggingFace model directory (config.json + safetensors), uploaded raw."""
        L = rt.load()
        rt.init(device)
        opts = rt.CuqOptions(max_seq=max_seq, max_chunk=max_chunk, use_graphs=int(use_graphs), tp_rank=0, tp_size=1,
                             decode_kernel=decode_kernel, persistent_ctas=0)
        h = L.cuq_model_load_hf(path.encode(), ctypes.byref(opts))
        if not h:
            raise rt.CuqError(rt.EFORMAT, rt.last_error())
        cfg = rt.CuqConfig()
        rt.check(L.cuq_model_get_config(h, ctypes.byref(cfg)))
        return cls(h, cfg)

    @classmethod
    def from_synth(cls, model, max_seq=None, use_graphs=True, device=0, max_chunk=512, tp_rank=0, tp_size=1,
                   exchange=None, decode_kernel=rt.DECODE_AUTO, persistent_ctas=0, wait_limit_ms=0):
        """Upload an anedvd_b200.synth.SynthModel tensor by tensor (raw GGUF payloads).

        Tensor parallel (tp_size > 1, one process per GPU): every rank uploads
        the full tensors and keeps its shard; `exchange(handle_bytes)` must
        return the list of every rank's handle in rank order (an all-gather
        over the caller's process group)."""
        L = rt.load()
        rt.init(device)
        c = model.cfg
        cfg = rt.CuqConfig(hidden=c.hidden, layers=c.layers, heads=c.heads, kv_heads=c.kv_heads,
                           head_dim=c.head_dim, inter=c.inter, vocab=c.vocab, eps=c.eps, rope_theta=c.rope_theta,
                           rope_adjacent=int(c.rope_adjacent), tie_embeddings=int(c.tie_embeddings))
        opts = rt.CuqOptions(max_seq=max_seq or c.max_seq, max_chunk=max_chunk, use_graphs=int(use_graphs),
                             tp_rank=tp_rank, tp_size=tp_size, decode_kernel=decode_kernel,
                             persistent_ctas=persistent_ctas, wait_limit_ms=wait_limit_ms)
        h = L.cuq_model_create(ctypes.byref(cfg), ctypes.byref(opts))
        if not h:
            raise rt.CuqError(rt.EINVAL, rt.last_error())
        eng = cls(h, cfg, tp_rank, tp_size)
        try:
            for t in model.tensors():
                buf = np.frombuffer(t.data, dtype=np.uint8)
                if t.role in ("attn_norm", "ffn_norm", "final_norm", "q_bias", "k_bias", "v_bias", "o_bias"):
                    v = np.frombuffer(t.data, dtype=np.float32)
                    rt.check(L.cuq_upload_f32(h, t.layer, rt.ROLE[t.role], _ptr(v), v.size))
                else:
                    rt.check(L.cuq_upload_tensor(h, t.layer, rt.ROLE[t.role], t.ggml_type, _ptr(buf), buf.size,
                                                 t.rows, t.cols))
            if tp_size > 1:
                eng.tp_connect(exchange)
            rt.check(L.cuq_model_finalize(h))
        except Exception:
            eng.close()
            raise
        return eng

    def tp_connect(self, exchange):
        """Publish this rank's communication buffer and map every peer's."""
        L = rt.load()
        mine = ctypes.create_string_buffer(rt.TP_HANDLE_BYTES)
        rt.check(L.cuq_tp_comm_handle(self._h, mine))
        handles = exchange(mine.raw)
        blob = ctypes.create_string_buffer(b"".join(handles), rt.TP_HANDLE_BYTES * len(handles))
        rt.check(L.cuq_tp_connect(self._h, blob))

    @property
    def tp_size(self):
        o = getattr(self, "_tp", (0, 1))
        return o[1]

    def close(self):
        if getattr(self, "_h", None):
            rt.load().cuq_model_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward(self, token, pos, want_logits=True):
        """Engine.forward: one decode step; returns (logits or None, argmax)."""
        logits = np.empty(self.local_vocab, dtype=np.float32) if want_logits else None
        am = ctypes.c_uint32(0)
        rt.check(rt.load().cuq_forward(self._h, token, pos, _ptr(logits) if want_logits else None,
                                       ctypes.byref(am)))
        return logits, am.value

    def prefill(self, ids, start_pos=0, want_logits=True):
        """Engine.prefill: logits (and argmax) of the last prompt token."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        logits = np.empty(self.local_vocab, dtype=np.float32) if want_logits else None
        am = ctypes.c_uint32(0)
        rt.check(rt.load().cuq_prefill(self._h, _ptr(ids), ids.size, start_pos,
                                       _ptr(logits) if want_logits else None, ctypes.byref(am)))
        return logits, am.value

    def decode_greedy(self, token, pos, n_steps):
        out = np.empty(n_steps, dtype=np.uint32)
        rt.check(rt.load().cuq_decode_greedy(self._h, token, pos, n_steps, _ptr(out)))
        return out

    def reset(self):
        rt.check(rt.load().cuq_reset(self._h))

    def kv_write(self, layer, pos0, k16, v16):
        """Replace cache rows [pos0, pos0 + n) of `layer` (fp16 bits [n][kv_heads*head_dim])."""
        k = np.ascontiguousarray(k16, dtype=np.uint16)
        v = np.ascontiguousarray(v16, dtype=np.uint16)
        n = k.size // (self.cfg.kv_heads * self.cfg.head_dim)
        rt.check(rt.load().cuq_kv_write(self._h, layer, pos0, n, _ptr(k), _ptr(v)))

    def kv_read(self, layer, pos0, n):
        """Cache rows [pos0, pos0 + n) of `layer` as fp16 bits ([n][kv_heads*head_dim] each for k, v)."""
        kvd = self.cfg.kv_heads * self.cfg.head_dim
        k = np.zeros((n, kvd), dtype=np.uint16)
        v = np.zeros((n, kvd), dtype=np.uint16)
        rt.check(rt.load().cuq_kv_read(self._h, layer, pos0, n, _ptr(k), _ptr(v)))
        return k, v

    def profile_decode(self, token, pos, n_steps):
        """Per-node decode timing (cuq_profile_decode, the `anedvd kernels` table):
        {node: (launches, ms, algorithmic bytes)} over n_steps eager steps."""
        tab = (rt.CuqNodeTime * len(rt.NODE_NAMES))()
        rt.check(rt.load().cuq_profile_decode(self._h, token, pos, n_steps, tab))
        return {name: (int(t.launches), float(t.ms), float(t.bytes)) for name, t in zip(rt.NODE_NAMES, tab)}

    @property
    def stats(self):
        s = rt.CuqStats()
        rt.check(rt.load().cuq_model_stats(self._h, ctypes.byref(s)))
        return s

    @property
    def persistent_ctas(self):
        """CTAs of the persistent decode kernel (0: decode runs one kernel per op)."""
        return int(self.stats.persistent_ctas)

    @property
    def stream(self):
        return rt.load().cuq_model_stream(self._h)


def reuse_length(cached, prompt):
    """generate.zig:456-460 reuseLength: how many leading prompt tokens may keep
    their KV rows.  Only a prompt that covers the WHOLE cached sequence may reuse
    it (a cache longer than the shared prefix would leave stale rows in front of
    the new tokens); otherwise nothing is reused."""
    n = min(len(cached), len(prompt))
    shared = 0
    while shared < n and int(cached[shared]) == int(prompt[shared]):
        shared += 1
    return shared if shared >= len(cached) else 0


class Session:
    """Session.generate (generate.zig:166-250): the decode loop runs on the device,
    greedy by default or with a sampler (cuq_sampler_params, drawn on the device).

    Like the reference's session it remembers which token ids the engine's KV
    cache holds, and a prompt that extends them (a multi-turn transcript) only
    prefills its new suffix (generate.zig:187-192)."""

    def __init__(self, engine, max_seq):
        self.engine = engine
        self.max_seq = max_seq
        self.cached = []      # token ids whose K/V rows the cache holds, in position order
        self.last = {}        # counters of the last call, as the reference's Stats

    def reset(self):
        self.engine.reset()
        self.cached = []

    def generate(self, ids, n_decode, sampler=None, seed=0x12345678, penalty_window=256):
        """`sampler`: None for greedy decoding, else rt.CuqSamplerParams (the
        reference's Params.sampler; seed and penalty_window as Params)."""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        sent = int(ids.size)
        # generate.zig:171-185: keep the newest tokens of a prompt that does not
        # leave room for the answer (and say how many were dropped)
        if ids.size + n_decode + 1 > self.max_seq:
            keep = self.max_seq - n_decode - 1
            if keep <= 0:
                raise rt.CuqError(rt.ECONTEXT, "PromptTooLong: %d prompt + %d decode > max_seq %d"
                                  % (ids.size, n_decode, self.max_seq))
            ids = ids[ids.size - keep:]
        reuse = reuse_length(self.cached, ids)
        # a prompt identical to the cache still needs its last position run for
        # the first token's logits: recompute that one row (same values)
        reuse = min(reuse, ids.size - 1)
        if reuse == 0:
            self.cached = []
        self.last = {"prompt_tokens_sent": sent, "prompt_tokens": int(ids.size),
                     "prompt_tokens_dropped": sent - int(ids.size), "prefill_reused": int(reuse)}
        out = np.empty(n_decode, dtype=np.uint32)
        L = rt.load()
        if sampler is not None:
            if n_decode > 0:
                rt.check(L.cuq_generate_sampled(self.engine._h, _ptr(ids), ids.size, reuse, n_decode,
                                                ctypes.byref(sampler), seed, penalty_window, _ptr(out)))
            else:
                tail = np.ascontiguousarray(ids[reuse:])
                rt.check(L.cuq_prefill(self.engine._h, _ptr(tail), tail.size, reuse, None, None))
        elif reuse == 0:
            # prefill from position 0 and decode on the device in one call
            rt.check(L.cuq_generate(self.engine._h, _ptr(ids), ids.size, n_decode, _ptr(out)))
        else:
            tail = np.ascontiguousarray(ids[reuse:])
            am = ctypes.c_uint32(0)
            rt.check(L.cuq_prefill(self.engine._h, _ptr(tail), tail.size, reuse, None, ctypes.byref(am)))
            out[0] = am.value
            if n_decode > 1:
                rest = np.empty(n_decode - 1, dtype=np.uint32)
                rt.check(L.cuq_decode_greedy(self.engine._h, am.value, ids.size, n_decode - 1, _ptr(rest)))
                out[1:] = rest
        # the cache now holds the prompt and every generated token but the last
        # (which was produced, not yet fed back)
        self.cached = [int(t) for t in ids] + [int(t) for t in out[:-1]]
        return out
