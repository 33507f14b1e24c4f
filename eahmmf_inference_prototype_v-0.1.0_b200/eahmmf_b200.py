"""Python host glue over libeahmmf_b200.so (the C ABI in include/eahmmf_b200.h).

ctypes bindings with the reference's argument meaning and error behaviour: the legacy entry points
return False on bad arguments (the engine then uses its CPU kernel), the device-resident ones return
EAHMMF_ST_* bits. Device memory and streams come from torch (plumbing only). Importing this module
never falls back to a CPU implementation: it raises if the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libeahmmf_b200.so")

ST_OK, ST_BAD_ARG, ST_BAD_TYPE, ST_CUDA, ST_WAIT_TIMEOUT, ST_BAD_INDEX, ST_CAPACITY = 0, 1, 2, 4, 8, 16, 32

_lib = None


class EahmmfSamplerParams(C.Structure):
    _fields_ = [("temp", C.c_float), ("top_p", C.c_float), ("min_p", C.c_float), ("rep", C.c_float),
                ("top_k", C.c_int), ("rep_n", C.c_int)]


# the reference CLI's defaults (qwen3moe.cpp:1091-1092)
SAMPLER_DEFAULTS = dict(temp=0.7, top_p=0.8, min_p=0.0, rep=1.05, top_k=20, rep_n=64)


def sampler_params(**kw) -> EahmmfSamplerParams:
    p = dict(SAMPLER_DEFAULTS, **kw)
    return EahmmfSamplerParams(p["temp"], p["top_p"], p["min_p"], p["rep"], p["top_k"], p["rep_n"])


class EahmmfMoeLayer(C.Structure):
    _fields_ = [("n_expert", C.c_int), ("n_used", C.c_int), ("D", C.c_int), ("FF", C.c_int),
                ("gate_type", C.c_int), ("up_type", C.c_int), ("down_type", C.c_int),
                ("gate_row_bytes", C.c_size_t), ("up_row_bytes", C.c_size_t), ("down_row_bytes", C.c_size_t),
                ("d_gate", C.c_void_p), ("d_up", C.c_void_p), ("d_down", C.c_void_p), ("d_router", C.c_void_p)]


EXPORTS = {
    "eahmmf_cuda_matmul": (C.c_bool, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p, C.c_int,
                                      C.c_int, C.c_void_p, C.c_int]),
    "eahmmf_cuda_matmul_pair": (C.c_bool, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p, C.c_int,
                                           C.c_int, C.c_int, C.c_size_t, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                           C.c_int, C.c_void_p, C.c_int]),
    "eahmmf_cuda_moe_workspace_bytes": (C.c_size_t, [C.POINTER(EahmmfMoeLayer), C.c_int]),
    "eahmmf_cuda_moe_layer": (C.c_int, [C.POINTER(EahmmfMoeLayer), C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]),
    "eahmmf_cuda_moe_profile": (C.c_int, [C.c_int]),
    "eahmmf_cuda_moe_profile_read": (C.c_int, [C.c_void_p, C.c_int]),
    "eahmmf_cuda_gemv_workspace_bytes": (C.c_size_t, [C.c_int]),
    "eahmmf_cuda_gemv": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p, C.c_int, C.c_int,
                                   C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "eahmmf_cuda_gemv_static": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_size_t, C.c_void_p, C.c_int,
                                          C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "eahmmf_dev_create": (C.c_void_p, [C.c_size_t]),
    "eahmmf_dev_destroy": (None, [C.c_void_p]),
    "eahmmf_dev_alloc": (C.c_void_p, [C.c_void_p, C.c_size_t]),
    "eahmmf_dev_release": (None, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "eahmmf_dev_h2d": (C.c_bool, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "eahmmf_dev_d2h": (C.c_bool, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "eahmmf_dev_sync": (C.c_bool, [C.c_void_p]),
    "eahmmf_dev_total_memory": (C.c_size_t, [C.c_void_p]),
    "eahmmf_dev_free_memory": (C.c_size_t, [C.c_void_p]),
    "eahmmf_dev_stream": (C.c_void_p, [C.c_void_p]),
    "eahmmf_dev_inject_fault": (None, [C.c_void_p, C.c_int, C.c_int]),
    "eahmmf_cuda_route_topk": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p]),
    "eahmmf_cuda_moe_combine": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                          C.c_void_p]),
    "eahmmf_cuda_moe_experts_workspace_bytes": (C.c_size_t, [C.POINTER(EahmmfMoeLayer), C.c_int]),
    "eahmmf_cuda_moe_experts": (C.c_int, [C.POINTER(EahmmfMoeLayer), C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]),
    "eahmmf_cuda_ep_pack": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "eahmmf_cuda_ep_unpack": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p]),
    "eahmmf_cuda_ep_return": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "eahmmf_engine_step": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    "eahmmf_engine_sampler": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64]),
    "eahmmf_engine_generate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "eahmmf_cuda_sample_workspace_bytes": (C.c_size_t, [C.c_int]),
    "eahmmf_cuda_sample": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_float, C.c_void_p,
                                     C.c_void_p, C.c_size_t, C.c_void_p]),
    "eahmmf_engine_verify": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "eahmmf_engine_set_slots": (C.c_int, [C.c_void_p, C.c_int]),
    "eahmmf_engine_load_budget": (C.c_void_p, [C.c_char_p, C.c_int, C.c_size_t, C.c_char_p, C.c_size_t]),
    "eahmmf_engine_cache_stats": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "eahmmf_engine_prefill_slot": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "eahmmf_engine_step_slots": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "eahmmf_cuda_hash64": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "eahmmf_hash64": (C.c_uint64, [C.c_void_p, C.c_size_t]),
    "eahmmf_rng_create": (C.c_void_p, [C.c_uint64]),
    "eahmmf_rng_uniform": (C.c_float, [C.c_void_p]),
    "eahmmf_rng_free": (None, [C.c_void_p]),
    "eahmmf_engine_load": (C.c_void_p, [C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]),
    "eahmmf_engine_free": (None, [C.c_void_p]),
    "eahmmf_engine_dims": (C.c_int, [C.c_void_p, C.c_void_p]),
    "eahmmf_engine_eval": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "eahmmf_engine_greedy": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "eahmmf_engine_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "eahmmf_engine_trace": (None, [C.c_void_p, C.c_int]),
    "eahmmf_engine_trace_get": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]),
    "eahmmf_engine_graph_nodes": (C.c_int, [C.c_void_p]),
    "eahmmf_engine_profile": (C.c_int, [C.c_void_p, C.c_int]),
    "eahmmf_engine_profile_read": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "eahmmf_b200_version": (C.c_char_p, []),
    "eahmmf_b200_sm_count": (C.c_int, []),
}


def lib(path: str = LIB_PATH) -> C.CDLL:
    """Loads libeahmmf_b200.so (built by build.py). Raises when it is missing: there is no fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run `python {os.path.join(HERE, 'build.py')}` first")
        L = C.CDLL(path)
        for name, (res, args) in EXPORTS.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _ptr(a) -> int:
    """Device (torch tensor) or host (numpy array) address."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def _stream(stream) -> int | None:
    if stream is None:
        return None
    return getattr(stream, "cuda_stream", stream)


# ---- group 1: the reference's entry points (host activations) -----------------------------------
def cuda_matmul(d_w, qtype: int, ne0: int, ne1: int, row_bytes: int, x: np.ndarray, out: np.ndarray,
                nb: int | None = None, ldx: int | None = None, ldo: int | None = None) -> bool:
    nb = x.shape[0] if nb is None else nb
    ldx = x.shape[1] if ldx is None else ldx
    ldo = out.shape[1] if ldo is None else ldo
    return bool(lib().eahmmf_cuda_matmul(_ptr(d_w), qtype, ne0, ne1, row_bytes, _ptr(x), nb, ldx, _ptr(out), ldo))


def cuda_matmul_pair(d_g, gt, d_u, ut, ne0, ne1, grb, urb, x, g_out, u_out) -> bool:
    return bool(lib().eahmmf_cuda_matmul_pair(_ptr(d_g), gt, ne0, ne1, grb, _ptr(d_u), ut, ne0, ne1, urb, _ptr(x),
                                              x.shape[0], x.shape[1], _ptr(g_out), g_out.shape[1], _ptr(u_out),
                                              u_out.shape[1]))


# ---- group 2: device-resident ------------------------------------------------------------------
_gemv_ws = {}


def gemv_workspace(ne0: int):
    """A cached device workspace for gemv() (torch uint8 tensor)."""
    import torch
    n = int(lib().eahmmf_cuda_gemv_workspace_bytes(ne0))
    ws = _gemv_ws.get(torch.cuda.current_device())
    if ws is None or ws.numel() < n:
        ws = torch.empty(n, dtype=torch.uint8, device="cuda")
        _gemv_ws[torch.cuda.current_device()] = ws
    return ws


def gemv(d_w, qtype: int, ne0: int, ne1: int, row_bytes: int, d_x, d_out, accumulate: bool = False,
         stream=None, ws="auto") -> int:
    nb, ldx = d_x.shape
    if isinstance(ws, str):
        ws = gemv_workspace(ne0)
    return lib().eahmmf_cuda_gemv(_ptr(d_w), qtype, ne0, ne1, row_bytes, _ptr(d_x), nb, ldx, _ptr(d_out),
                                  d_out.shape[1], int(accumulate), _ptr(ws),
                                  0 if ws is None else ws.numel() * ws.element_size(), _stream(stream))


GEMV_STATIC_MAX_NE0 = 16384  # EAHMMF_GEMV_STATIC_MAX_NE0


def gemv_static(d_w, qtype: int, ne0: int, ne1: int, row_bytes: int, d_x, d_out, accumulate: bool = False,
                stream=None) -> int:
    """eahmmf_cuda_gemv_static: gemv() with the library's fixed device workspace (no allocation)."""
    nb, ldx = d_x.shape
    return lib().eahmmf_cuda_gemv_static(_ptr(d_w), qtype, ne0, ne1, row_bytes, _ptr(d_x), nb, ldx, _ptr(d_out),
                                         d_out.shape[1], int(accumulate), _stream(stream))


class MoeLayer:
    """One layer's experts on the device, in the form ExpertStore leases publish them: a device array
    of per-expert component pointers for gate, up and down."""

    def __init__(self, gate_ptrs, up_ptrs, down_ptrs, types, row_bytes, D: int, FF: int, n_used: int,
                 router=None):
        import torch
        self._keep = []
        E = len(gate_ptrs)
        tabs = []
        for ptrs in (gate_ptrs, up_ptrs, down_ptrs):
            t = torch.tensor(np.array(ptrs, dtype=np.uint64).view(np.int64), device="cuda")
            self._keep.append(t)
            tabs.append(t.data_ptr())
        if router is not None:
            self._keep.append(router)
        self.desc = EahmmfMoeLayer(E, n_used, D, FF, types[0], types[1], types[2], row_bytes[0], row_bytes[1],
                                   row_bytes[2], tabs[0], tabs[1], tabs[2], _ptr(router) if router is not None else None)
        self.E, self.K, self.D, self.FF = E, n_used, D, FF

    @classmethod
    def from_expert_set(cls, ex, n_used: int, router=None):
        """Uploads a synth.ExpertSet: one device buffer per component kind, experts back to back."""
        import torch
        bufs = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (ex.gate, ex.up, ex.down)]
        ptrs = [[b.data_ptr() + e * b.shape[1] for e in range(ex.n_expert)] for b in bufs]
        layer = cls(*ptrs, ex.types, ex.row_bytes, ex.D, ex.FF, n_used, router=router)
        layer._keep += bufs
        return layer

    def workspace_bytes(self, T: int) -> int:
        return int(lib().eahmmf_cuda_moe_workspace_bytes(C.byref(self.desc), T))

    def __call__(self, T: int, d_xn, d_logits, d_x, d_ws, stream=None, d_status=None) -> int:
        return lib().eahmmf_cuda_moe_layer(C.byref(self.desc), T, _ptr(d_xn), _ptr(d_logits), _ptr(d_x), _ptr(d_ws),
                                           d_ws.numel() * d_ws.element_size(), _stream(stream), _ptr(d_status))

    @staticmethod
    def profile(enable: bool) -> None:
        if lib().eahmmf_cuda_moe_profile(int(enable)):
            raise RuntimeError("eahmmf_cuda_moe_profile failed")

    @staticmethod
    def profile_read() -> np.ndarray:
        """Stage durations (us) of the last call: router GEMV, routing + activation prep, gate/up (+ h
        prep), down + combine."""
        us = np.zeros(4, np.float32)
        if lib().eahmmf_cuda_moe_profile_read(us.ctypes.data, 4):
            raise RuntimeError("eahmmf_cuda_moe_profile_read failed")
        return us

    def experts_workspace_bytes(self, R: int) -> int:
        return int(lib().eahmmf_cuda_moe_experts_workspace_bytes(C.byref(self.desc), R))

    def apply_experts(self, R: int, d_rows, d_eid, d_y, d_ws, stream=None, d_status=None) -> int:
        """eahmmf_cuda_moe_experts: d_y[r] += the output of expert d_eid[r] on d_rows[r] (rows with
        d_eid[r] < 0 are absent)."""
        return lib().eahmmf_cuda_moe_experts(C.byref(self.desc), R, _ptr(d_rows), _ptr(d_eid), _ptr(d_y), _ptr(d_ws),
                                             d_ws.numel() * d_ws.element_size(), _stream(stream), _ptr(d_status))

    def routing(self, d_ws, T: int):
        """(ids, weights) of the last call, read from the head of the workspace."""
        n = T * self.K
        ids = d_ws[: n * 4].view(dtype=__import__("torch").int32).cpu().numpy().reshape(T, self.K)
        off = ((n * 4 + 255) // 256) * 256
        w = d_ws[off: off + n * 4].view(dtype=__import__("torch").float32).cpu().numpy().reshape(T, self.K)
        return ids, w


class Engine:
    """The device-resident qwen3moe engine (eahmmf_engine_*): a GGUF model in HBM, with the reference
    harness's calls (load, dims, eval, greedy, routing trace). Raises on load failure; calls return the
    EAHMMF_ST_* status of the C ABI."""

    DIM_NAMES = ("n_layer", "D", "n_head", "n_kv", "hd", "n_expert", "n_used", "FF", "n_vocab", "n_ctx", "n_embd")

    CACHE_STATS = ("slots", "hits", "misses", "prefetched", "prefetch_hits", "evictions", "bytes_h2d", "dma")

    def __init__(self, path: str, n_ctx: int, expert_vram_bytes: int = 0):
        L = lib()
        err = C.create_string_buffer(256)
        if expert_vram_bytes:
            h = L.eahmmf_engine_load_budget(path.encode(), n_ctx, expert_vram_bytes, err, 256)
        else:
            h = L.eahmmf_engine_load(path.encode(), n_ctx, err, 256)
        if not h:
            raise RuntimeError(f"eahmmf_engine_load: {err.value.decode()}")
        self._h = h
        self._free = L.eahmmf_engine_free  # held here: module globals may be gone when __del__ runs at exit
        d = np.zeros(11, np.int32)
        L.eahmmf_engine_dims(h, d.ctypes.data)
        self.dims = dict(zip(self.DIM_NAMES, (int(v) for v in d)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library or the CUDA context may already be gone
            pass

    def eval(self, toks, p0: int = 0, n_batch: int = 32, want_logits: bool = True):
        t = np.ascontiguousarray(toks, np.int32)
        lg = np.zeros(self.dims["n_vocab"], np.float32) if want_logits else None
        rc = lib().eahmmf_engine_eval(self._h, t.ctypes.data, len(t), p0, n_batch,
                                      lg.ctypes.data if lg is not None else None)
        return rc, lg

    def greedy(self, prompt, n_gen: int, n_batch: int = 32, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        lg = np.zeros(self.dims["n_vocab"], np.float32) if want_logits else None
        rc = lib().eahmmf_engine_greedy(self._h, p.ctypes.data, len(p), n_gen, n_batch, out.ctypes.data,
                                        lg.ctypes.data if lg is not None else None)
        return rc, out, lg

    def decode(self, n_steps: int):
        """Continue greedy generation by n_steps tokens; returns (rc, tokens, device milliseconds)."""
        out = np.zeros(n_steps, np.int32)
        ms = C.c_float(0.0)
        rc = lib().eahmmf_engine_decode(self._h, n_steps, out.ctypes.data, C.byref(ms))
        return rc, out, float(ms.value)

    def step(self, token: int = -1):
        """One host-driven greedy step (eahmmf_engine_step): token in (negative: the engine's last
        argmax), next token out. Returns (rc, next)."""
        nxt = C.c_int(0)
        rc = lib().eahmmf_engine_step(self._h, int(token), C.byref(nxt))
        return rc, int(nxt.value)

    def sampler(self, seed: int = 0, **params) -> int:
        """Configure the reference's sampler (eahmmf_engine_sampler): no params = greedy selection; else
        sampler_params(**params) with its random stream seeded by `seed`."""
        p = C.byref(sampler_params(**params)) if params else None
        return lib().eahmmf_engine_sampler(self._h, p, C.c_uint64(seed))

    def generate(self, prompt, n_gen: int, n_batch: int = 32):
        """eahmmf_engine_generate with the configured selection: (rc, tokens)."""
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_gen, np.int32)
        rc = lib().eahmmf_engine_generate(self._h, p.ctypes.data, len(p), n_gen, n_batch, out.ctypes.data)
        return rc, out

    def cache_stats(self) -> dict:
        """eahmmf_engine_cache_stats of an oversubscribed engine."""
        v = np.zeros(len(self.CACHE_STATS), np.uint64)
        lib().eahmmf_engine_cache_stats(self._h, v.ctypes.data, len(v))
        return dict(zip(self.CACHE_STATS, (int(x) for x in v)))

    def set_slots(self, n: int) -> int:
        """eahmmf_engine_set_slots: KV caches for n sequences."""
        return lib().eahmmf_engine_set_slots(self._h, n)

    def prefill_slot(self, slot: int, prompt, n_batch: int = 64):
        """A new sequence in `slot`: (rc, first token)."""
        p = np.ascontiguousarray(prompt, np.int32)
        first = C.c_int(0)
        rc = lib().eahmmf_engine_prefill_slot(self._h, slot, p.ctypes.data, len(p), n_batch, C.byref(first))
        return rc, int(first.value)

    def step_slots(self, slots, pos, toks):
        """One greedy step of several sequences: (rc, next tokens)."""
        s_ = np.ascontiguousarray(slots, np.int32)
        p_ = np.ascontiguousarray(pos, np.int32)
        t_ = np.ascontiguousarray(toks, np.int32)
        out = np.zeros(len(s_), np.int32)
        rc = lib().eahmmf_engine_step_slots(self._h, len(s_), s_.ctypes.data, p_.ctypes.data, t_.ctypes.data,
                                            out.ctypes.data)
        return rc, out

    def verify(self):
        """eahmmf_engine_verify: (rc, components checked, components whose device hash64 differs from
        the file's)."""
        n, bad = C.c_int(0), C.c_int(0)
        rc = lib().eahmmf_engine_verify(self._h, C.byref(n), C.byref(bad))
        return rc, int(n.value), int(bad.value)

    def trace(self, enable: bool) -> None:
        lib().eahmmf_engine_trace(self._h, 1 if enable else 0)

    PROFILE_CLASSES = ("embed_rope", "attn_norm", "qkv_gemv", "qk_rope_kv", "attention", "o_gemv", "ffn_norm",
                       "moe", "output", "argmax")

    def graph_nodes(self) -> int:
        """Kernel launches in one captured decode step (0 before the first capture)."""
        return int(lib().eahmmf_engine_graph_nodes(self._h))

    def profile(self, enable: bool) -> None:
        lib().eahmmf_engine_profile(self._h, 1 if enable else 0)

    def profile_read(self) -> dict:
        us = np.zeros(len(self.PROFILE_CLASSES), np.float32)
        n = lib().eahmmf_engine_profile_read(self._h, us.ctypes.data, len(us))
        return dict(zip(self.PROFILE_CLASSES, map(float, us))) if n else {}

    def trace_get(self):
        L = lib()
        n = L.eahmmf_engine_trace_get(self._h, None, None, 0)
        ids = np.zeros(n, np.int32)
        w = np.zeros(n, np.float32)
        L.eahmmf_engine_trace_get(self._h, ids.ctypes.data, w.ctypes.data, n)
        return ids, w


def route_topk(d_logits, K: int, stream=None, d_status=None):
    """Top-k routing of device logits [T x E] (eahmmf_cuda_route_topk): (ids [T x K] int32, weights
    [T x K] fp32) on the same device, rank order."""
    import torch
    T, E = d_logits.shape
    ids = torch.empty((T, K), dtype=torch.int32, device=d_logits.device)
    w = torch.empty((T, K), dtype=torch.float32, device=d_logits.device)
    rc = lib().eahmmf_cuda_route_topk(_ptr(d_logits), T, E, K, _ptr(ids), _ptr(w), _stream(stream),
                                      _ptr(d_status) if d_status is not None else None)
    if rc:
        raise RuntimeError(f"eahmmf_cuda_route_topk returned {rc}")
    return ids, w


def moe_combine(d_token_slots, d_slot_w, d_y, d_x, stream=None) -> int:
    """d_x[t] += sum_k w[s] y[s] over token t's slots s (ascending expert order), eahmmf_cuda_moe_combine."""
    T, D = d_x.shape
    K = d_token_slots.numel() // T
    return lib().eahmmf_cuda_moe_combine(T, K, D, _ptr(d_token_slots), _ptr(d_slot_w), _ptr(d_y), _ptr(d_x),
                                         _stream(stream))


EP_HDR = 4  # EAHMMF_EP_HDR: header floats before each row of a dispatch buffer


def ep_pack(d_ids, d_w, d_xn, K: int, E_loc: int, world: int, cap: int, d_send, d_token_pos, d_pos_w, stream=None,
            d_status=None) -> int:
    """eahmmf_cuda_ep_pack: this rank's routed slots (d_ids/d_w [T x K]) into the world x cap dispatch
    blocks."""
    T, D = d_xn.shape
    return lib().eahmmf_cuda_ep_pack(_ptr(d_ids), _ptr(d_w), _ptr(d_xn), T, K, D, E_loc, world, cap, _ptr(d_send),
                                     _ptr(d_token_pos), _ptr(d_pos_w), _stream(stream), _ptr(d_status))


def ep_unpack(d_recv, D: int, world: int, cap: int, d_rows, d_eid, d_src, d_y=None, stream=None) -> int:
    """eahmmf_cuda_ep_unpack: the received blocks' valid rows compacted to the front by ascending local
    expert, stable in (source, row) order (expert -1 after)."""
    return lib().eahmmf_cuda_ep_unpack(_ptr(d_recv), D, world, cap, _ptr(d_rows), _ptr(d_eid), _ptr(d_src), _ptr(d_y),
                                       _stream(stream))


def ep_return(d_y, d_src, D: int, world: int, cap: int, d_ret, stream=None) -> int:
    """eahmmf_cuda_ep_return: the valid compact rows' outputs back to their received positions."""
    return lib().eahmmf_cuda_ep_return(_ptr(d_y), _ptr(d_src), D, world, cap, _ptr(d_ret), _stream(stream))


class Rng:
    """The reference sampler's random stream (eahmmf_rng_*): std::mt19937_64 seeded as the reference does,
    one canonical float draw per call."""

    def __init__(self, seed: int):
        self._h = lib().eahmmf_rng_create(C.c_uint64(seed))
        self._free = lib().eahmmf_rng_free

    def uniform(self) -> float:
        return float(lib().eahmmf_rng_uniform(self._h))

    def __del__(self):
        try:
            if self._h:
                self._free(self._h)
                self._h = None
        except Exception:
            pass


def sample(d_logits, d_hist, params: EahmmfSamplerParams, u: float, d_token, d_ws=None, stream=None) -> int:
    """eahmmf_cuda_sample on one device logits row (penalised in place); the token goes to d_token."""
    import torch
    n = d_logits.numel()
    if d_ws is None:
        d_ws = torch.empty(int(lib().eahmmf_cuda_sample_workspace_bytes(n)), dtype=torch.uint8, device=d_logits.device)
    nh = 0 if d_hist is None else d_hist.numel()
    return lib().eahmmf_cuda_sample(_ptr(d_logits), n, _ptr(d_hist) if nh else None, nh, C.byref(params),
                                    C.c_float(u), _ptr(d_token), _ptr(d_ws), d_ws.numel(), _stream(stream))


def hash64(data) -> int:
    """eahmmf_hash64 of a host byte buffer (numpy uint8)."""
    a = np.ascontiguousarray(data, np.uint8)
    return int(lib().eahmmf_hash64(a.ctypes.data if a.size else None, a.size))


def cuda_hash64(d_bufs, stream=None) -> list:
    """eahmmf_cuda_hash64 over device byte ranges: a list of (torch uint8 tensor, offset, size)."""
    import torch
    ptrs = torch.tensor([b.data_ptr() + o for b, o, _ in d_bufs], dtype=torch.int64, device="cuda")
    sizes = torch.tensor([n for _, _, n in d_bufs], dtype=torch.int64, device="cuda")
    out = torch.zeros(len(d_bufs), dtype=torch.int64, device="cuda")
    rc = lib().eahmmf_cuda_hash64(_ptr(ptrs), _ptr(sizes), len(d_bufs), _ptr(out), _stream(stream))
    if rc:
        raise RuntimeError(f"eahmmf_cuda_hash64 returned {rc}")
    return [int(v) & 0xFFFFFFFFFFFFFFFF for v in out.cpu().numpy().tolist()]
