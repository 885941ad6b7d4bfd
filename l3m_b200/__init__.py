"""ctypes binding of the B200 decode engine (include/l3m.h), mirroring the reference's Python API
(fpedd/l3m python/l3m/__init__.py:1-157): the same Model constructor, encode/decode/generate,
logits and perf, with `cpus` read as a list of GPU ordinals. The library is the in-tree
l3m_b200/libl3m.so (override with L3M_LIB); there is no CPU fallback.
"""
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


class Model:
    """A loaded .l3m file on one or more GPUs (cpus: GPU ordinals, default GPU 0) with a KV cache
    of ctx (default min(model, 512)). Thread-safe; on_token may read the model but not generate
    or close it."""
    _m = None

    def __init__(self, path, cpus=None, ctx=0, reference=False, force=False, verbose=False, cold=False):
        self._lock, self._generating = threading.RLock(), False
        if ctx and ctx < 2:
            raise ValueError(f"ctx {ctx}: needs room for a prompt token and one more")
        self._lib = lib()
        opts = Opts(ctx=ctx, reference=int(reference), force=int(force), verbose=int(verbose), cold=int(cold))
        if cpus:
            self._cpus = (C.c_int * len(cpus))(*cpus)
            opts.cpus, opts.n_cpus = self._cpus, len(cpus)
        self._m = self._lib.l3m_load(os.fsencode(path), C.byref(opts))
        if not self._m:
            raise RuntimeError(f"l3m_load failed for {path} (the reason is on stderr)")
        self.vocab, self.ctx = self._lib.l3m_vocab(self._m), self._lib.l3m_ctx(self._m)
        self.bos, self.eos = self._lib.l3m_bos(self._m), self._lib.l3m_eos(self._m)

    def _handle(self, writing=False):
        if writing and self._generating:
            raise RuntimeError("l3m: on_token cannot call generate or close")
        if not self._m:
            raise ValueError("l3m: model is closed")
        return self._m

    def close(self):
        with self._lock:
            if self._m:
                self._lib.l3m_free(self._handle(writing=True))
                self._m = None

    __del__ = close

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()

    def describe(self):
        with self._lock:
            return self._lib.l3m_describe(self._handle()).decode()

    def encode(self, text, bos=True):
        if "\0" in text:
            raise ValueError("l3m: text contains a NUL")
        data = text.encode()
        buf = (C.c_int32 * (len(data) + 8))()
        with self._lock:
            n = self._lib.l3m_encode(self._handle(), data, int(bos), buf, len(buf))
        return list(buf[:n])

    def decode_bytes(self, ids):
        out, n = bytearray(), C.c_int()
        with self._lock:
            for t in ids:
                if not 0 <= t < self.vocab:
                    raise ValueError(f"token {t} is outside vocab {self.vocab}")
                out += C.string_at(self._lib.l3m_decode(self._handle(), t, C.byref(n)), n.value)
        return bytes(out)

    def decode(self, ids):
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    def generate(self, prompt, max_new, temperature=0.8, seed=0, on_token=None):
        """Up to max_new token ids after prompt, stopping at EOS or BOS; on_token(id) returning False stops."""
        if not 0 < len(prompt) < self.ctx or not all(0 <= t < self.vocab for t in prompt):
            raise ValueError(f"prompt of {len(prompt)} ids: needs 1 to {self.ctx - 1} ids, each below vocab {self.vocab}")
        out, err = [], []

        def cb(tok, _):
            out.append(tok)
            try:
                return 0 if on_token is not None and on_token(tok) is False else 1
            except BaseException as e:
                err.append(e)
                return 0

        buf = (C.c_int32 * len(prompt))(*prompt)
        with self._lock:
            m = self._handle(writing=True)
            self._generating = True
            try:
                rc = self._lib.l3m_generate(m, buf, len(prompt), min(max_new, self.ctx), temperature, seed % 2**64, _CB(cb), None)
            finally:
                self._generating = False
        if err:
            raise err[0]
        if rc < 0:
            raise RuntimeError("l3m_generate failed (the reason is on stderr)")
        return out

    @property
    def logits(self):
        """The last position's logits."""
        with self._lock:
            return np.ctypeslib.as_array(self._lib.l3m_logits(self._handle()), shape=(self.vocab,)).copy()

    def perf(self):
        """Per-token counters since the previous call; NaN where unavailable."""
        p = Perf()
        with self._lock:
            if self._lib.l3m_perf_read(self._handle(), C.byref(p)):
                return {f: float("nan") for f, _ in Perf._fields_}
        return {f: getattr(p, f) for f, _ in Perf._fields_}
