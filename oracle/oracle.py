"""ctypes bindings for the parity checkers -- TEST INFRASTRUCTURE ONLY.

``Oracle``    wraps oracle/_build/liboracle.so (the C restatement in oracle.c).
``Reference`` wraps oracle/_ref/libeahmmf_ref.so (the reference engine compiled from its own sources by
              oracle/Makefile). On the GPU box it is the prebuilt copy that travelled with the repo.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may import this module.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libeahmmf_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def _ptr_array(arrs) -> C.Array:
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def _moe_args(T, D, FF, E, K, xn, logits, router_w, gate, up, down, types, row_bytes):
    tg, tu, td = types
    rg, ru, rd = row_bytes
    return (T, D, FF, E, K, np.ascontiguousarray(xn, np.float32),
            None if logits is None else np.ascontiguousarray(logits, np.float32).ctypes.data,
            None if router_w is None else np.ascontiguousarray(router_w, np.float32).ctypes.data,
            _ptr_array(gate), _ptr_array(up), _ptr_array(down), tg, tu, td, rg, ru, rd)


class _MoeLib:
    _prefix = ""

    def _bind_moe(self, lib, name):
        fn = getattr(lib, name)
        fn.restype = C.c_int
        fn.argtypes = [C.c_int] * 5 + [_f32p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_size_t, C.c_size_t, _f32p,
                                       C.c_void_p, C.c_void_p]
        return fn

    def moe_layer(self, x, xn, logits, gate, up, down, types, row_bytes, K, router_w=None):
        """x (T, D) residual, updated copy returned with the (T, K) routing ids and weights."""
        x = np.array(x, np.float32, copy=True, order="C")
        T, D = x.shape
        E = len(gate)
        FF = (gate[0].size // row_bytes[0])
        ids = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        args = _moe_args(T, D, FF, E, K, xn, logits, router_w, gate, up, down, types, row_bytes)
        keep = (args[5], logits, router_w)  # noqa: F841 keep buffers alive
        rc = self._moe(*args, x, ids.ctypes.data, w.ctypes.data)
        if rc:
            raise RuntimeError(f"{self._moe.__name__} failed: {rc}")
        return x, ids, w


class Oracle(_MoeLib):
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle oracle`")
        self.lib = lib = C.CDLL(path)
        lib.orc_matmul.restype = C.c_int
        lib.orc_matmul.argtypes = [_u8p, C.c_int, C.c_int64, C.c_int64, C.c_size_t, _f32p, C.c_int, C.c_int,
                                   _f32p, C.c_int]
        lib.orc_dequant_row.restype = C.c_int
        lib.orc_dequant_row.argtypes = [C.c_int, _u8p, C.c_int64, _f32p]
        lib.orc_route_token.restype = None
        lib.orc_route_token.argtypes = [_f32p, C.c_int, C.c_int, _i32p, _f32p]
        lib.orc_rmsnorm.restype = None
        lib.orc_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_float]
        self._moe = self._bind_moe(lib, "orc_moe_layer")

    def dequant(self, qtype: int, raw: np.ndarray, ne0: int, rows: int) -> np.ndarray:
        raw = np.ascontiguousarray(raw, np.uint8).reshape(rows, -1)
        out = np.zeros((rows, ne0), np.float32)
        for r in range(rows):
            row = np.ascontiguousarray(raw[r])
            tmp = np.zeros(ne0, np.float32)
            if self.lib.orc_dequant_row(qtype, row, ne0, tmp):
                raise ValueError("unsupported type/shape")
            out[r] = tmp
        return out

    def matmul(self, w: np.ndarray, qtype: int, ne0: int, ne1: int, row_bytes: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        nb = x.shape[0]
        out = np.zeros((nb, ne1), np.float32)
        rc = self.lib.orc_matmul(np.ascontiguousarray(w, np.uint8).reshape(-1), qtype, ne0, ne1, row_bytes, x, nb,
                                 x.shape[1], out, ne1)
        if rc:
            raise RuntimeError(f"orc_matmul failed: {rc}")
        return out

    def route(self, logits: np.ndarray, K: int):
        T, E = logits.shape
        ids = np.zeros((T, K), np.int32)
        w = np.zeros((T, K), np.float32)
        for t in range(T):
            r = np.array(logits[t], np.float32, copy=True)
            i1, w1 = np.zeros(K, np.int32), np.zeros(K, np.float32)
            self.lib.orc_route_token(r, E, K, i1, w1)
            ids[t], w[t] = i1, w1
        return ids, w


class Reference(_MoeLib):
    def __init__(self, path: str = REF_SO, threads: int = 0):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference tree exists")
        self.lib = lib = C.CDLL(path)
        lib.eref_init.restype = C.c_int
        lib.eref_init.argtypes = [C.c_int]
        lib.eref_matmul.restype = C.c_int
        lib.eref_matmul.argtypes = [_u8p, C.c_int, C.c_int64, C.c_int64, C.c_size_t, _f32p, C.c_int, C.c_int,
                                    _f32p, C.c_int]
        self._moe = self._bind_moe(lib, "eref_moe_layer")
        lib.eref_engine_load.restype = C.c_void_p
        lib.eref_engine_load.argtypes = [C.c_char_p, C.c_int]
        lib.eref_engine_free.argtypes = [C.c_void_p]
        lib.eref_engine_dims.argtypes = [C.c_void_p, _i32p]
        lib.eref_engine_eval.restype = C.c_int
        lib.eref_engine_eval.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        lib.eref_engine_trace.argtypes = [C.c_void_p, C.c_int]
        lib.eref_engine_trace_get.restype = C.c_int
        lib.eref_engine_trace_get.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        lib.eref_engine_greedy.restype = C.c_int
        lib.eref_engine_greedy.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int, _i32p, C.c_void_p]
        lib.eref_sample.restype = C.c_int
        lib.eref_sample.argtypes = [_f32p, C.c_int, C.c_void_p, C.c_int, C.c_float, C.c_float, C.c_float, C.c_float,
                                    C.c_int, C.c_int, C.c_uint64]
        lib.eref_hash64.restype = C.c_uint64
        lib.eref_hash64.argtypes = [C.c_void_p, C.c_size_t]
        lib.eref_uniform.restype = None
        lib.eref_uniform.argtypes = [C.c_uint64, C.c_int, _f32p]
        lib.eref_engine_generate.restype = C.c_int
        lib.eref_engine_generate.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float,
                                             C.c_float, C.c_float, C.c_int, C.c_int, C.c_uint64, _i32p]
        self.threads = lib.eref_init(threads)

    def sample(self, logits, hist, temp, top_p, min_p, rep, top_k, rep_n, seed):
        """Sampler::sample (qwen3moe.cpp:1095-1130) with a stream seeded by `seed`: (token, the penalised
        logits)."""
        lg = np.array(logits, np.float32, copy=True)
        h = np.ascontiguousarray(hist, np.int32)
        tok = self.lib.eref_sample(lg, len(lg), h.ctypes.data if len(h) else None, len(h), temp, top_p, min_p, rep,
                                   top_k, rep_n, seed)
        return int(tok), lg

    def hash64(self, data) -> int:
        a = np.ascontiguousarray(data, np.uint8)
        return int(self.lib.eref_hash64(a.ctypes.data if a.size else None, a.size))

    def uniform(self, seed: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        self.lib.eref_uniform(seed, n, out)
        return out

    def matmul(self, w, qtype, ne0, ne1, row_bytes, x):
        x = np.ascontiguousarray(x, np.float32)
        nb = x.shape[0]
        out = np.zeros((nb, ne1), np.float32)
        if self.lib.eref_matmul(np.ascontiguousarray(w, np.uint8).reshape(-1), qtype, ne0, ne1, row_bytes, x, nb,
                                x.shape[1], out, ne1):
            raise RuntimeError("eref_matmul failed")
        return out

    def engine(self, path: str, n_ctx: int) -> "RefEngine":
        return RefEngine(self, path, n_ctx)


class RefEngine:
    DIM_NAMES = ("n_layer", "D", "n_head", "n_kv", "hd", "n_expert", "n_used", "FF", "n_vocab", "n_ctx", "n_embd_rows")

    def __init__(self, ref: Reference, path: str, n_ctx: int):
        self.lib = ref.lib
        self.h = self.lib.eref_engine_load(path.encode(), n_ctx)
        d = np.zeros(11, np.int32)
        self.lib.eref_engine_dims(self.h, d)
        self.dims = dict(zip(self.DIM_NAMES, map(int, d)))

    def close(self):
        if self.h:
            self.lib.eref_engine_free(self.h)
            self.h = None

    def eval(self, toks, p0: int = 0, n_batch: int = 32, want_logits: bool = True):
        toks = np.ascontiguousarray(toks, np.int32)
        lg = np.zeros(self.dims["n_vocab"], np.float32) if want_logits else None
        rc = self.lib.eref_engine_eval(self.h, toks, len(toks), p0, n_batch, lg.ctypes.data if lg is not None else None)
        if rc:
            raise RuntimeError("eref_engine_eval failed")
        return lg

    def trace(self, enable: bool):
        self.lib.eref_engine_trace(self.h, int(enable))

    def trace_get(self):
        n = self.lib.eref_engine_trace_get(self.h, None, None, 0)
        ids, w = np.zeros(n, np.int32), np.zeros(n, np.float32)
        self.lib.eref_engine_trace_get(self.h, ids.ctypes.data, w.ctypes.data, n)
        return ids, w

    def generate(self, prompt, n_gen: int, params: dict, seed: int, n_batch: int = 32):
        """The reference generate loop with its Sampler (params: temp, top_p, min_p, rep, top_k, rep_n)."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        p = params
        if self.lib.eref_engine_generate(self.h, prompt, len(prompt), n_gen, n_batch, p["temp"], p["top_p"],
                                         p["min_p"], p["rep"], p["top_k"], p["rep_n"], seed, out):
            raise RuntimeError("eref_engine_generate failed")
        return out

    def greedy(self, prompt, n_gen: int, n_batch: int = 32):
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        lg = np.zeros(self.dims["n_vocab"], np.float32)
        if self.lib.eref_engine_greedy(self.h, prompt, len(prompt), n_gen, n_batch, out, lg.ctypes.data):
            raise RuntimeError("eref_engine_greedy failed")
        return out, lg
