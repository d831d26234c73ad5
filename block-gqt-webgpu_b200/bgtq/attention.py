"""Attention over the key/value stores, mirroring the reference's attention classes.

    OptimizedAttention  src/attention/optimized.ts:5-45  (packed K, fused, no reconstruction)
    AttentionEngine / AttentionSession  src/attention/attention.ts:6-70 (FP16 K, or
                        CompressedKeys through materialised FP32 K)
    GroupedAttention    batched GQA decode: ``heads`` KV heads x ``rows`` query rows per
                        head over ``sequences`` independent sequences (the model path,
                        src/model/compressed-dot.wgsl + src/model/attention.wgsl)

``attend`` with NumPy inputs copies host <-> device inside the call and returns NumPy;
with CUDA tensors it is stream-ordered and returns a CUDA tensor.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib


class GroupedAttention:
    def __init__(self, keys, values, rows: int):
        keys, values = list(keys), list(values)
        if not keys or len(keys) != len(values):
            raise _lib.RangeError(_lib.EINVAL, "Incompatible attention storage")
        karr = (C.c_void_p * len(keys))(*[k._handle for k in keys])
        varr = (C.c_void_p * len(values))(*[v._handle for v in values])
        h = C.c_void_p()
        _lib.call("bgtq_attention_create", len(keys), karr, varr, int(rows), C.byref(h))
        self._handle = h
        self.keys, self.values, self.heads, self.rows = keys, values, len(keys), int(rows)
        self.dim = keys[0].dim
        self.device = keys[0].device

    def attend(self, q, positions=None, causal: bool = False, rows: int | None = None, seq_first: int = 0,
               seq_count: int | None = None, out=None, logits=None, probs=None, stream=None, wait: bool = True):
        """q: [seq_count, heads, rows, dim] (or [rows, dim] for one head / one sequence).
        Host (NumPy) inputs with wait=False: the output download is queued without waiting;
        `out` (page-locked) holds the result once the stream has been synchronised."""
        rows = self.rows if rows is None else int(rows)
        if isinstance(q, np.ndarray) or not hasattr(q, "data_ptr"):
            qa = np.ascontiguousarray(np.asarray(q, dtype=np.float32))
            if qa.size % (self.heads * rows * self.dim):
                raise _lib.RangeError(_lib.EINVAL, "Invalid Q/K/V shape or positions")
            n = qa.size // (self.heads * rows * self.dim)
            seq_count = n if seq_count is None else seq_count
            if n != seq_count:
                raise _lib.RangeError(_lib.EINVAL, "Invalid Q/K/V shape or positions")
            pos = None if positions is None else np.ascontiguousarray(np.asarray(positions, np.uint32))
            if pos is not None and pos.size != seq_count * rows:
                raise _lib.RangeError(_lib.EINVAL, "Invalid Q/K/V shape or positions")
            o = np.zeros(qa.shape[:-1] + (self.dim,), np.float32) if out is None else out
            _lib.call("bgtq_attend", self._handle, qa.ctypes.data, None if pos is None else pos.ctypes.data,
                      int(bool(causal)), rows, seq_first, seq_count, o.ctypes.data,
                      None if logits is None else logits.ctypes.data, None if probs is None else probs.ctypes.data,
                      1 if wait else 2, None)
            return o
        import torch
        seq_count = q.shape[0] if seq_count is None else seq_count
        o = torch.empty_like(q) if out is None else out
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        pp = None if positions is None else positions.data_ptr()
        _lib.call("bgtq_attend", self._handle, C.c_void_p(q.data_ptr()), C.c_void_p(pp) if pp else None,
                  int(bool(causal)), rows, seq_first, seq_count, C.c_void_p(o.data_ptr()),
                  None if logits is None else C.c_void_p(logits.data_ptr()),
                  None if probs is None else C.c_void_p(probs.data_ptr()), 0, C.c_void_p(int(st)))
        return o

    def prefill(self, q, pos_first: int = 0, seq_first: int = 0, out=None, stream=None):
        """Causal prefill (bgtq_attend_prefill): q [seq_count, n, heads * gqa, dim] holds the
        queries at positions pos_first .. pos_first + n - 1 of sequences seq_first ..;
        query head h * gqa + r uses KV head h and sees keys 0 .. its position.  NumPy in ->
        NumPy out (synchronous); a CUDA tensor in -> a CUDA tensor out (stream-ordered)."""
        if q.ndim != 4 or q.shape[2] % self.heads or q.shape[3] != self.dim:
            raise _lib.RangeError(_lib.EINVAL, "Invalid Q/K/V shape or positions")
        seq_count, n, gqa = int(q.shape[0]), int(q.shape[1]), q.shape[2] // self.heads
        if isinstance(q, np.ndarray) or not hasattr(q, "data_ptr"):
            qa = np.ascontiguousarray(np.asarray(q, dtype=np.float32))
            o = np.zeros(qa.shape, np.float32) if out is None else out
            _lib.call("bgtq_attend_prefill", self._handle, qa.ctypes.data, pos_first, n, gqa, seq_first, seq_count,
                      o.ctypes.data, 1, None)
            return o
        import torch
        if not q.is_contiguous() or q.dtype != torch.float32:
            raise _lib.RangeError(_lib.EINVAL, "Invalid Q/K/V shape or positions")
        o = torch.empty_like(q) if out is None else out
        st = stream if stream is not None else torch.cuda.current_stream(q.device).cuda_stream
        _lib.call("bgtq_attend_prefill", self._handle, C.c_void_p(q.data_ptr()), pos_first, n, gqa, seq_first,
                  seq_count, C.c_void_p(o.data_ptr()), 0, C.c_void_p(int(st)))
        return o

    def set_prefill_kernel(self, kernel: str) -> None:
        """"umma" (tcgen05 with TMEM accumulators, the default) or "mma" (mma.sync)."""
        _lib.call("bgtq_attention_set_prefill_kernel", self._handle, {"umma": 0, "mma": 1}[kernel])

    @property
    def last_splits(self) -> int:
        n = C.c_uint32()
        _lib.call("bgtq_attention_last_splits", self._handle, C.byref(n))
        return n.value

    @property
    def last_launches(self) -> int:
        n = C.c_uint32()
        _lib.call("bgtq_attention_last_launches", self._handle, C.byref(n))
        return n.value

    def set_splits(self, splits: int) -> None:
        _lib.call("bgtq_attention_set_splits", self._handle, int(splits))

    def set_schedule(self, mode: str) -> None:
        """'auto' (stream-K when estimated faster), 'split' (split-KV only) or 'stream_k'
        (whenever the kernel allows)."""
        modes = {"auto": 0, "split": 1, "stream_k": 2}
        if mode not in modes:
            raise ValueError(f"schedule must be one of {sorted(modes)}")
        _lib.call("bgtq_attention_set_schedule", self._handle, modes[mode])

    @property
    def last_stream_k(self) -> int:
        """CTAs of the last stream-K launch, 0 when the last launch used split-KV."""
        n = C.c_uint32()
        _lib.call("bgtq_attention_last_stream_k", self._handle, C.byref(n))
        return n.value

    def destroy(self) -> None:
        if getattr(self, "_handle", None):
            _lib.lib().bgtq_attention_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class _SingleHead(GroupedAttention):
    """One KV head, up to ``max_queries`` query rows with explicit positions."""

    def __init__(self, keys, values, max_queries: int = 3):
        if keys.dim != values.dim or keys.capacity != values.capacity:
            raise _lib.RangeError(_lib.EINVAL, "Incompatible attention storage")
        super().__init__([keys], [values], max_queries)
        self.max_queries = int(max_queries)
        self.queries = 0
        self._q = self._positions = None
        self._causal = False
        self._last = None

    def set_queries(self, q, positions, causal: bool = False) -> None:
        """setQueries (optimized.ts:29-31): validates before any state change."""
        self.keys[0].ready()
        q = np.asarray(q, np.float32).reshape(-1)
        positions = np.asarray(positions).reshape(-1)
        n = q.size / self.dim
        if (self.keys[0].length != self.values[0].length or n != int(n) or not 1 <= n <= self.max_queries
                or positions.size != n or np.any(positions < 0) or np.any(positions >= self.keys[0].length)):
            raise _lib.RangeError(_lib.EINVAL, "Invalid Q/K/V shape or positions")
        if not np.all(np.isfinite(q)):
            raise _lib.RangeError(_lib.ENONFINITE, "Q: finite inputs required")
        self.queries = int(n)
        self._q = q.reshape(self.queries, self.dim).copy()
        self._positions = positions.astype(np.uint32)
        self._causal = bool(causal)

    def record(self):
        """Run the attention pass for the current queries (the reference's record+submit)."""
        if not self.queries:
            raise _lib.StateError(_lib.EBUSY, "Attention not ready")
        tokens = self.keys[0].length
        logits = np.zeros((self.queries, tokens), np.float32)
        probs = np.zeros((self.queries, tokens), np.float32)
        out = super().attend(self._q[None, None], self._positions, self._causal, rows=self.queries,
                             logits=logits, probs=probs)
        self._last = dict(logits=logits, probabilities=probs, output=out.reshape(self.queries, self.dim),
                          queries=self.queries, tokens=tokens)
        return self._last["output"]

    def attend(self, q, positions, causal: bool = False):
        """attend (optimized.ts:42): fused pass only (no logits capture); returns [n, dim]."""
        self.set_queries(q, positions, causal)
        out = super().attend(self._q[None, None], self._positions, self._causal, rows=self.queries)
        self._last = None
        return out.reshape(self.queries, self.dim)

    def inspect(self):
        """inspect(): logits, probabilities and output of the current queries."""
        return self._last if self._last is not None else (self.record() and self._last)


class OptimizedAttention(_SingleHead):
    @classmethod
    def create(cls, keys, values, max_queries: int = 3):
        return cls(keys, values, max_queries)


class AttentionSession(_SingleHead):
    pass


class AttentionEngine:
    """AttentionEngine.create().session(keys, values, maxQueries) (attention.ts:6-17)."""

    @classmethod
    def create(cls, device: int = 0):
        return cls()

    def session(self, keys, values, max_queries: int = 3) -> AttentionSession:
        return AttentionSession(keys, values, max_queries)
