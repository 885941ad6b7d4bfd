"""ctypes binding of the B200 decode engine (include/l3m.h), mirroring the reference's Python API
(fpedd/l3m python/l3m/__init__.py:1-157): the same Model constructor, encode/decode/generate,
logits and perf, with `cpus` read as a list of GPU ordinals. The library is the in-tree
l3m_b200/libl3m.so (override with L3M_LIB); there is no CPU fallback.
"""
import contextlib
import ctypes as C
import functools
import os
import threading
from pathlib import Path

import numpy as np

__all__ = ["Model", "Opts", "Perf", "lib", "kernels"]

_CB = C.CFUNCTYPE(C.c_int, C.c_int32, C.c_void_p)
HERE = Path(__file__).resolve().parent


class Opts(C.Structure):
    """l3m_opts: field order is ABI (reference src/l3m.h:10-19)."""
    _fields_ = [("cpus", C.POINTER(C.c_int)), ("n_cpus", C.c_int), ("ctx", C.c_int),
                ("reference", C.c_int), ("force", C.c_int), ("verbose", C.c_int), ("cold", C.c_int)]


class Perf(C.Structure):
    _fields_ = [(f, C.c_double) for f in ("tokens", "ns_token", "ns_compute", "ns_wait", "bytes_token", "l2_bytes",
                                           "l3_miss", "dram_bytes", "energy_j", "llc_occupancy")]


class Vec(C.Structure):
    """l3m_vec (reference src/kernels.h:24-30)."""
    _fields_ = [("f32", C.c_void_p), ("bf16", C.c_void_p), ("q8", C.c_void_p), ("scale", C.c_void_p), ("sum", C.c_void_p)]


GEMV = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(Vec))
ATTEND = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int)


class Kernels(C.Structure):
    _fields_ = [("name", C.c_char_p), ("gemv", GEMV * 5), ("attend", ATTEND)]


def _find_lib():
    p = os.environ.get("L3M_LIB")
    for cand in (p, HERE / "libl3m.so"):
        if cand and Path(cand).exists():
            return str(Path(cand).resolve())
    raise OSError("l3m_b200/libl3m.so not found: run `make -C l3m_b200` (or __graft_entry__.build()), or set L3M_LIB")


@functools.cache
def lib():
    """The loaded library with every l3m.h and l3m_kernels.h signature declared."""
    so = C.CDLL(_find_lib())
    vp, i, f, u64, sz = C.c_void_p, C.c_int, C.c_float, C.c_uint64, C.c_size_t
    sig = {
        "l3m_load": (vp, [C.c_char_p, C.POINTER(Opts)]),
        "l3m_free": (None, [vp]),
        "l3m_generate": (i, [vp, C.POINTER(C.c_int32), i, i, f, u64, _CB, vp]),
        "l3m_logits": (C.POINTER(C.c_float), [vp]),
        "l3m_vocab": (i, [vp]),
        "l3m_ctx": (i, [vp]),
        "l3m_describe": (C.c_char_p, [vp]),
        "l3m_encode": (i, [vp, C.c_char_p, i, C.POINTER(C.c_int32), i]),
        "l3m_decode": (vp, [vp, C.c_int32, C.POINTER(C.c_int)]),
        "l3m_bos": (i, [vp]),
        "l3m_eos": (i, [vp]),
        "l3m_chatml": (C.c_char_p, [vp, C.POINTER(C.c_int32)]),
        "l3m_perf_read": (i, [vp, C.POINTER(Perf)]),
        "l3m_device_ns": (C.c_double, [vp]),
        "l3m_parse_cpus": (i, [C.c_char_p, C.POINTER(C.c_int), i]),
        "l3m_row_bytes": (sz, [i, i]),
        "l3m_tile_bytes": (sz, [i, i]),
        "l3m_pack_tile": (None, [vp, i, C.POINTER(vp), i]),
        "l3m_dequant_row": (None, [vp, i, vp, i]),
        "l3m_vec_prepare": (None, [C.POINTER(Vec), i, vp, i, vp]),
        "l3m_kernels_pick": (C.POINTER(Kernels), []),
        "l3m_kernels_usable": (i, [C.POINTER(Kernels)]),
        "l3m_gemv_dev": (i, [i, i, vp, vp, i, i, C.POINTER(Vec), vp]),
        "l3m_gemv_splitk_dev": (i, [i, vp, vp, i, i, C.POINTER(Vec), vp]),
        "l3m_vec_prepare_dev": (i, [i, C.POINTER(Vec), vp, i, vp, vp]),
        "l3m_sample_dev": (i, [vp, i, f, vp, vp, vp, vp]),
        "l3m_block_dots_dev": (i, [i, vp, vp, i, i, C.POINTER(Vec), vp]),
        "l3m_unpack_dev": (i, [i, vp, vp, vp, i, i, vp]),
        "l3m_attend_dev": (i, [vp, vp, vp, vp, i, i, i, vp]),
        "l3m_expf_dev": (i, [vp, vp, i, vp]),
        "l3m_chain_cycles_dev": (i, [i, C.POINTER(C.c_double)]),
        "l3m_cuda_error": (C.c_char_p, []),
        "l3m_write_packed": (i, [C.c_char_p, C.c_char_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(so, name)
        fn.restype, fn.argtypes = res, args
    return so


def kernels(name="sm100a"):
    """The host-pointer kernel table `name` ("sm100a" exact, "sm100a-fast")."""
    sym = {"sm100a": "l3m_kernels_sm100a", "sm100a-fast": "l3m_kernels_sm100a_fast"}[name]
    return Kernels.in_dll(lib(), sym)


class _TokenSink:
    """The C on_token callback of one generate call: collects ids, forwards each to the user's
    callback, and turns its False (or an exception, kept for re-raising) into a stop request."""

    def __init__(self, user):
        self.ids, self.user, self.error = [], user, None
        self.cfunc = _CB(self._on_token)        # referenced until the call returns

    def _on_token(self, tok, _user):
        self.ids.append(tok)
        if self.user is None:
            return 1
        try:
            return 0 if self.user(tok) is False else 1
        except BaseException as e:              # noqa: BLE001 -- re-raised on the caller's thread
            self.error = e
            return 0


class Model:
    """A .l3m model loaded on GPUs (cpus: GPU ordinals, default GPU 0) with a KV cache of ctx entries
    (default min(model, 512)); the reference binding's interface (python/l3m/__init__.py:53-157).

    Calls on one model are serialised. Inside on_token the model can be read (logits, decode,
    describe, perf) but generate and close raise RuntimeError; every call on a closed model raises
    ValueError. A negative return from the library raises RuntimeError (its reason is on stderr)."""

    def __init__(self, path, cpus=None, ctx=0, reference=False, force=False, verbose=False, cold=False):
        if ctx and ctx < 2:
            raise ValueError(f"ctx {ctx}: needs room for a prompt token and one more")
        self._lib, self._lock, self._in_callback, self._ptr = lib(), threading.RLock(), False, None
        gpus = list(cpus or [])
        self._gpu_array = (C.c_int * max(1, len(gpus)))(*gpus)
        opts = Opts(cpus=self._gpu_array if gpus else None, n_cpus=len(gpus), ctx=ctx, reference=int(bool(reference)),
                    force=int(bool(force)), verbose=int(bool(verbose)), cold=int(bool(cold)))
        ptr = self._lib.l3m_load(os.fsencode(path), C.byref(opts))
        if not ptr:
            raise RuntimeError(f"l3m_load failed for {path} (the reason is on stderr)")
        self._ptr = ptr
        L = self._lib
        self.vocab, self.ctx, self.bos, self.eos = L.l3m_vocab(ptr), L.l3m_ctx(ptr), L.l3m_bos(ptr), L.l3m_eos(ptr)

    @contextlib.contextmanager
    def _using(self, mutates=False):
        """The model's pointer, with the lock held; refuses what the current state does not allow."""
        with self._lock:
            if mutates and self._in_callback:
                raise RuntimeError("l3m: on_token cannot call generate or close")
            if not self._ptr:
                raise ValueError("l3m: model is closed")
            yield self._ptr

    def close(self):
        with self._lock:
            if self._ptr is None:
                return
            with self._using(mutates=True) as ptr:
                self._ptr = None
                self._lib.l3m_free(ptr)

    def __del__(self):
        if getattr(self, "_ptr", None):
            self.close()

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()

    def describe(self):
        with self._using() as ptr:
            return self._lib.l3m_describe(ptr).decode()

    def encode(self, text, bos=True):
        if "\0" in text:
            raise ValueError("l3m: text contains a NUL")
        raw = text.encode()
        ids = (C.c_int32 * (len(raw) + 8))()          # one id per byte at most, plus BOS and the SentencePiece space
        with self._using() as ptr:
            n = self._lib.l3m_encode(ptr, raw, int(bool(bos)), ids, len(ids))
        return ids[:max(n, 0)]

    def decode_bytes(self, ids):
        bad = [t for t in ids if not 0 <= t < self.vocab]
        if bad:
            raise ValueError(f"token {bad[0]} is outside vocab {self.vocab}")
        size = C.c_int()
        with self._using() as ptr:
            return b"".join(C.string_at(self._lib.l3m_decode(ptr, t, C.byref(size)), size.value) for t in ids)

    def decode(self, ids):
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def generate(self, prompt, max_new, temperature=0.8, seed=0, on_token=None):
        """Up to max_new token ids after prompt, stopping at EOS or BOS; on_token(id) returning False stops."""
        prompt = list(prompt)
        if not (0 < len(prompt) < self.ctx and all(0 <= t < self.vocab for t in prompt)):
            raise ValueError(f"prompt of {len(prompt)} ids: needs 1 to {self.ctx - 1} ids, each below vocab {self.vocab}")
        sink = _TokenSink(on_token)
        ids = (C.c_int32 * len(prompt))(*prompt)
        with self._using(mutates=True) as ptr:
            self._in_callback = True
            try:
                rc = self._lib.l3m_generate(ptr, ids, len(ids), min(max_new, self.ctx), temperature, seed % 2**64, sink.cfunc, None)
            finally:
                self._in_callback = False
        if sink.error is not None:
            raise sink.error
        if rc < 0:
            raise RuntimeError("l3m_generate failed (the reason is on stderr)")
        return sink.ids

    @property
    def logits(self):
        """The logits of the last position run (during on_token: of the token just produced)."""
        with self._using() as ptr:
            return np.ctypeslib.as_array(self._lib.l3m_logits(ptr), shape=(self.vocab,)).copy()

    def device_ns(self):
        """Device time (ns) of the decode launches since the previous perf() call, cold flushes excluded."""
        with self._using() as ptr:
            return self._lib.l3m_device_ns(ptr)

    def perf(self):
        """Per-token counters since the previous call; NaN where unavailable."""
        counters = Perf()
        with self._using() as ptr:
            ok = self._lib.l3m_perf_read(ptr, C.byref(counters)) == 0
        return {name: getattr(counters, name) if ok else float("nan") for name, _ in Perf._fields_}
