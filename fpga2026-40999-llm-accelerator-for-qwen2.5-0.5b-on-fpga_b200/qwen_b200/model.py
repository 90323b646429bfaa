"""Host-side mirror of the reference's behavioural-model interface,
legacy_100mhz_closed/src/PC/model_backend.py:14-115 (`Model(sd)`, `clear()`,
`forward(ids, position) -> token`, `last_logits`, `position`), backed by
libqwen_b200 on a B200. Same argument meaning and the same errors: a KV
position mismatch or an over-long request raises ValueError, non-finite
logits raise ValueError, greedy ties go to the highest token id.
"""
import ctypes
from pathlib import Path

import numpy as np

from . import _lib
from ._lib import c_uint32, c_uint16, check, lib, ptr


def bf16_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class Engine:
    """One libqwen_b200 handle (one GPU). Owns device memory until close()."""

    def __init__(self, device=0, max_seqs=1, max_context=256, max_rows=256, rms_eps=1e-6, flags=0):
        """flags: 0, or qwen_b200.FLAG_RTL_KV for the accelerator's own KV format."""
        cfg = _lib.Config()
        lib().qwen_b200_default_config(ctypes.byref(cfg))
        cfg.device, cfg.max_seqs, cfg.max_context, cfg.max_rows, cfg.rms_eps, cfg.flags = (
            device, max_seqs, max_context, max_rows, rms_eps, flags)
        handle = ctypes.c_void_p()
        check(lib().qwen_b200_open(ctypes.byref(cfg), ctypes.byref(handle)))
        self.h = handle
        self.cfg = cfg

    def load_assets(self, sd):
        check(lib().qwen_b200_load_assets(self.h, str(sd).encode()), self.h)
        return self

    def load_synthetic(self, seed):
        check(lib().qwen_b200_load_synthetic(self.h, seed), self.h)
        return self

    def close(self):
        if self.h:
            lib().qwen_b200_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def position(self, slot=0):
        p = c_uint32()
        check(lib().qwen_b200_position(self.h, slot, ctypes.byref(p)), self.h)
        return p.value

    def set_persistent(self, enable):
        """Single-row steps as one persistent launch: True / 1 up to 96 keys
        (the default), 2 up to 1024 keys, False / 0 never."""
        check(lib().qwen_b200_set_persistent_decode(self.h, int(enable)), self.h)
        return self

    def reset(self, slot=0):
        check(lib().qwen_b200_reset(self.h, slot), self.h)

    def forward(self, slot, ids, position, want_logits=False):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        tok = c_uint32()
        logits = np.empty(_lib.VOCAB, dtype=np.uint16) if want_logits else None
        status = lib().qwen_b200_forward(self.h, slot, ptr(ids, c_uint32), len(ids), position, ctypes.byref(tok),
                                         ptr(logits, c_uint16) if want_logits else None)
        check(status, self.h)
        return tok.value, logits

    def decode_step(self, slots, tokens):
        slots = np.ascontiguousarray(slots, dtype=np.uint32)
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(len(slots), dtype=np.uint32)
        check(lib().qwen_b200_decode_step(self.h, ptr(slots, c_uint32), ptr(tokens, c_uint32), len(slots),
                                          ptr(out, c_uint32)), self.h)
        return out

    def prefill(self, slots, prompts, want_tokens=True, want_hidden=False):
        """Batched prefill: prompts[i] appended to slot slots[i]. Returns
        (tokens [n] or None, last hidden rows [n][896] bf16 bits or None)."""
        slots = np.ascontiguousarray(slots, dtype=np.uint32)
        lens = np.array([len(p) for p in prompts], dtype=np.uint32)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.uint32) for p in prompts]))
        toks = np.empty(len(slots), dtype=np.uint32) if want_tokens else None
        hidden = np.empty((len(slots), _lib.HIDDEN), dtype=np.uint16) if want_hidden else None
        check(lib().qwen_b200_prefill(self.h, len(slots), ptr(slots, c_uint32), ptr(lens, c_uint32), ptr(ids, c_uint32),
                                      ptr(toks, c_uint32) if want_tokens else None,
                                      ptr(hidden, c_uint16) if want_hidden else None), self.h)
        return toks, hidden

    def lm_head_range(self, d_hidden, rows, begin, end, d_values, d_indices, stream=None):
        """Vocabulary rows [begin, end) of the LM head for device rows d_hidden
        (pointers as ctypes.c_void_p); per row best value and global index."""
        check(lib().qwen_b200_lm_head_range(self.h, d_hidden, rows, begin, end, d_values, d_indices, stream), self.h)

    def decode_step_logits(self, slots, tokens):
        """decode_step that also returns every row's logits [n][151936] (bf16 bits)."""
        slots = np.ascontiguousarray(slots, dtype=np.uint32)
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(len(slots), dtype=np.uint32)
        logits = np.empty((len(slots), _lib.VOCAB), dtype=np.uint16)
        check(lib().qwen_b200_decode_step_logits(self.h, ptr(slots, c_uint32), ptr(tokens, c_uint32), len(slots),
                                                 ptr(out, c_uint32), ptr(logits, c_uint16)), self.h)
        return out, logits

    def decode_step_device(self, tokens_in_ptr, n, tokens_out_ptr, stream=None):
        check(lib().qwen_b200_decode_step_device(self.h, tokens_in_ptr, n, tokens_out_ptr, stream), self.h)

    def fill_kv_synthetic(self, slot, length, seed):
        check(lib().qwen_b200_fill_kv_synthetic(self.h, slot, length, seed), self.h)

    def read_kv(self, slot, layer, n):
        kc = np.empty((2, n, 64), dtype=np.int8)
        vc = np.empty((2, n, 64), dtype=np.int8)
        ks = np.empty((2, n), dtype=np.float32)
        vs = np.empty((2, n), dtype=np.float32)
        i8 = ctypes.c_int8
        check(lib().qwen_b200_read_kv(self.h, slot, layer, n, ptr(kc, i8), ptr(ks, ctypes.c_float), ptr(vc, i8),
                                      ptr(vs, ctypes.c_float)), self.h)
        return kc, ks, vc, vs

    def read_kv_rtl(self, slot, layer, n):
        """FLAG_RTL_KV handles: (klo [2][n][64], K block locks [2][blocks], V locks [2])."""
        klo = np.empty((2, n, 64), dtype=np.int8)
        klock = np.empty((2, (self.cfg.max_context + 255) // 256), dtype=np.uint8)
        vlock = np.empty(2, dtype=np.uint8)
        u8 = ctypes.c_uint8
        check(lib().qwen_b200_read_kv_rtl(self.h, slot, layer, n, ptr(klo, ctypes.c_int8), ptr(klock, u8),
                                          ptr(vlock, u8)), self.h)
        return klo, klock, vlock

    def set_dump(self, layer, rows):
        """Arms the per-layer dump; returns the dict of host arrays it fills."""
        shapes = dict(q=896, k=128, v=128, context=896, h=896, m=4864, y=896)
        bufs = {k: np.zeros((rows, c), dtype=np.uint16) for k, c in shapes.items()}
        args = [ptr(bufs[k], c_uint16) for k in ['q', 'k', 'v', 'context', 'h', 'm', 'y']]
        check(lib().qwen_b200_set_dump(self.h, layer, *args), self.h)
        self._dump = bufs
        return bufs

    def disarm_dump(self):
        check(lib().qwen_b200_set_dump(self.h, -1, None, None, None, None, None, None, None), self.h)


class Scheduler:
    """Continuous batching over one Engine (qwen_b200_sched_*): submit
    prompts, step until done, read each request's tokens."""

    def __init__(self, engine, prefill_budget=256):
        handle = ctypes.c_void_p()
        check(lib().qwen_b200_sched_open(engine.h, prefill_budget, ctypes.byref(handle)), engine.h)
        self.s, self.engine = handle, engine

    def submit(self, ids, max_new):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        rid = c_uint32()
        check(lib().qwen_b200_sched_submit(self.s, ptr(ids, c_uint32), len(ids), max_new, ctypes.byref(rid)))
        return rid.value

    def step(self):
        """One scheduling step; returns the number of unfinished requests."""
        n = c_uint32()
        check(lib().qwen_b200_sched_step(self.s, ctypes.byref(n)), self.engine.h)
        return n.value

    def result(self, rid, cap=1024):
        toks = np.empty(cap, dtype=np.uint32)
        count, done = c_uint32(), ctypes.c_int()
        check(lib().qwen_b200_sched_result(self.s, rid, ptr(toks, c_uint32), cap, ctypes.byref(count),
                                           ctypes.byref(done)))
        return toks[:min(count.value, cap)].tolist(), bool(done.value)

    def close(self):
        if self.s:
            lib().qwen_b200_sched_close(self.s)
            self.s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    """model_backend.Model with the math on a B200 (one sequence, slot 0)."""

    def __init__(self, sd, threads=4, device=0, capacity=256, max_rows=256):
        del threads  # the reference's torch CPU thread count has no meaning here
        self.sd = Path(sd) / 'QWEN25'
        self.capacity = capacity
        self.engine = Engine(device=device, max_seqs=1, max_context=capacity, max_rows=max_rows)
        self.engine.load_assets(sd)
        self.last_logits = None
        self.clear()

    def clear(self):
        self.engine.reset(0)
        self.position = 0

    def forward(self, ids, position):
        ids = list(ids)
        if position != self.position or not ids or position + len(ids) > self.capacity:
            raise ValueError(f'KV position mismatch pos={position} cached={self.position} ids={len(ids)}')
        token, logits = self.engine.forward(0, ids, position, want_logits=True)
        self.last_logits = bf16_to_f32(logits)
        if not np.isfinite(self.last_logits).all():
            raise ValueError('Nonfinite B200 model logits')
        self.position = position + len(ids)
        return token

    def close(self):
        self.engine.close()
