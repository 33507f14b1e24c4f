"""CPU-only checks of the C ABI: the library loads, exports every function the public headers declare,
and the reference entry points reject bad arguments before touching the GPU (as expert_cuda.cu:263-267
and :353-357 do: return false, the engine falls back to its CPU kernel)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import eahmmf_b200 as eb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")


def declared_functions():
    names = set()
    for f in os.listdir(INCLUDE):
        if not f.endswith(".h"):
            continue
        text = open(os.path.join(INCLUDE, f)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(eahmmf_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_reference_entry_points():
    names = declared_functions()
    assert "eahmmf_cuda_matmul" in names and "eahmmf_cuda_matmul_pair" in names
    assert "eahmmf_cuda_moe_layer" in names


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(eb.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(eb.EXPORTS) <= set(declared_functions())


def test_version_string():
    assert b"sm_100a" in eb.lib().eahmmf_b200_version()


@pytest.mark.parametrize("bad", [
    dict(type=3),                      # unsupported ggml type
    dict(ne0=0), dict(ne1=0), dict(nb=0),
    dict(ldx=100), dict(ldo=10),       # ldx < ne0, ldo < ne1
    dict(row_bytes=143),               # inconsistent with ne0
    dict(w=None), dict(x=None),
])
def test_legacy_matmul_rejects_bad_arguments(bad):
    args = dict(w=0x1000, type=12, ne0=256, ne1=16, row_bytes=144, x=np.zeros((2, 256), np.float32), nb=2,
                ldx=256, out=np.zeros((2, 16), np.float32), ldo=16)
    args.update(bad)
    x, out = args["x"], args["out"]
    ok = eb.lib().eahmmf_cuda_matmul(args["w"], args["type"], args["ne0"], args["ne1"], args["row_bytes"],
                                     None if x is None else x.ctypes.data, args["nb"], args["ldx"],
                                     out.ctypes.data, args["ldo"])
    assert ok is False


def test_legacy_pair_rejects_mismatched_shapes():
    x = np.zeros((1, 256), np.float32)
    g = np.zeros((1, 16), np.float32)
    u = np.zeros((1, 16), np.float32)
    L = eb.lib()
    # up has a different row count than gate (expert_cuda.cu:355-356)
    assert L.eahmmf_cuda_matmul_pair(0x1000, 12, 256, 16, 144, 0x2000, 12, 256, 8, 144, x.ctypes.data, 1, 256,
                                     g.ctypes.data, 16, u.ctypes.data, 16) is False
    assert L.eahmmf_cuda_matmul_pair(0x1000, 12, 256, 16, 144, 0x2000, 2, 256, 16, 144, x.ctypes.data, 1, 256,
                                     g.ctypes.data, 16, u.ctypes.data, 16) is False


def test_moe_layer_validates_before_launch():
    L = eb.lib()
    desc = eb.EahmmfMoeLayer(128, 8, 2048, 768, 12, 12, 14, 1152, 1152, 630, 0x1000, 0x2000, 0x3000, None)
    assert L.eahmmf_cuda_moe_workspace_bytes(C.byref(desc), 8) > 0
    bad = eb.EahmmfMoeLayer(128, 8, 2048, 768, 12, 12, 3, 1152, 1152, 630, 0x1000, 0x2000, 0x3000, None)
    assert L.eahmmf_cuda_moe_workspace_bytes(C.byref(bad), 8) == 0
    xn, lg, x, ws = 0x10000, 0x20000, 0x30000, 0x40000
    assert L.eahmmf_cuda_moe_layer(C.byref(bad), 8, xn, lg, x, ws, 1 << 30, None, None) == eb.ST_BAD_TYPE
    # no logits and no router matrix
    assert L.eahmmf_cuda_moe_layer(C.byref(desc), 8, xn, None, x, ws, 1 << 30, None, None) == eb.ST_BAD_ARG
    # workspace too small
    assert L.eahmmf_cuda_moe_layer(C.byref(desc), 8, xn, lg, x, ws, 16, None, None) == eb.ST_CAPACITY
    # misaligned activations / workspace
    assert L.eahmmf_cuda_moe_layer(C.byref(desc), 8, xn + 4, lg, x, ws, 1 << 30, None, None) == eb.ST_BAD_ARG
    assert L.eahmmf_cuda_moe_layer(C.byref(desc), 8, xn, lg, x, ws + 64, 1 << 30, None, None) == eb.ST_BAD_ARG


@pytest.mark.parametrize("shape", [(128, 8, 2048, 768, 1152, 630), (128, 8, 4096, 1536, 2304, 1260),
                                   (16, 2, 512, 256, 288, 210)])
@pytest.mark.parametrize("router", [False, True])
def test_moe_workspace_bytes_follow_the_documented_formula(shape, router):
    """eahmmf_cuda_moe_workspace_bytes against the sizes the header states: 64-token passes below 256
    tokens (or below 16 slots per expert), the grouped tensor-core path's f16 expert copy and per-slot
    rows from there. The function's value may exceed the formula only by alignment padding and the
    per-expert arrays."""
    E, K, D, FF, rg, rd = shape
    L = eb.lib()
    desc = eb.EahmmfMoeLayer(E, K, D, FF, 12, 12, 14, rg, rg, rd, 0x1000, 0x2000, 0x3000, 0x5000 if router else None)
    prev = 0
    for T in (1, 8, 64, 65, 255, 256, 2048, 16193):
        ws = L.eahmmf_cuda_moe_workspace_bytes(C.byref(desc), T)
        S = T * K
        if T >= 256 and S >= 16 * E:
            f = (E * 3 * FF * D * 2 + E * (2 * FF + D) * 4 + S * (FF + D + 7) * 4
                 + (S // 128 + E + 1) * 128 * max(D, FF) * 2 + (T * E * 4 if router else 0) + T * 4)
            assert f <= ws <= f + 64 * 1024, (T, ws, f)
        else:
            # ids and weights of every token; per pass: slot maps, h and y rows, the XF digits, logits
            tc = min(T, 64)
            f = 8 * S + tc * K * (FF + D + 3) * 4 + tc * D * 3 + (tc * E * 4 if router else 0)
            assert f <= ws <= 1.03 * f + 64 * 1024, (T, ws, f)
        assert ws >= prev  # a workspace sized for T tokens serves every smaller call
        prev = ws
