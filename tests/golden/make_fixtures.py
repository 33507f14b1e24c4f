#!/usr/bin/env python3
"""Regenerates the golden fixtures in tests/golden/ from the reference itself.

Run in the build container, where the reference tree exists (default: the directory `reference` beside
the repository, or $EAHMMF_REF):

    make -C oracle ref && python tests/golden/make_fixtures.py

What it does:
  1. Runs the reference's own fixture generator (tests/test_tiny.py of the reference, seed 0) in a scratch
     directory to produce its tiny.gguf, and copies it here as ref_tiny.gguf.
  2. Checks the reference engine (oracle/_ref/libeahmmf_ref.so, compiled from the reference sources)
     against the reference's golden vectors: baseline/logits.txt (16 logits + argmax, tolerance 2e-6 as in
     check_baseline.sh) and baseline/gen_greedy.bin (24-token greedy bytes, byte-exact); refuses to write
     anything if either check fails.
  3. Records reference outputs as fixtures: ref_tiny.npz (full logits, greedy ids, routing trace),
     config1.npz (BASELINE config 1 model), moe_c2.npz (config-2 MoE layer, T = 1, 3, 8),
     moe_mixed.npz (Q5_K/Q4_K/Q6_K experts as in the reference's tiny model), matmul.npz (every type),
     kquant_small.npz (a small all-K-quant model: prompt logits and greedy ids).

`--only kquant_small` regenerates just that fixture (and its entry in fixtures.json).
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
GOLDEN = os.path.join(ROOT, "tests", "golden")
REF = os.environ.get("EAHMMF_REF", os.path.normpath(os.path.join(ROOT, "..", "reference")))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "eahmmf_inference_prototype_v-0.1.0_b200"))

import oracle  # noqa: E402
import synth  # noqa: E402

PROMPT_IDS = [5, 17, 200, 33, 99, 3, 150, 256, 42, 77, 8, 9, 10, 11, 12]  # check_baseline.sh:6


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 20), b""):
            h.update(b)
    return h.hexdigest()


def token_bytes(gguf_path):
    """id -> bytes for the byte-level vocabulary of a GGUF (byte tokens, merges, specials -> b'')."""
    import gguf
    rd = gguf.GGUFReader(gguf_path)
    f = rd.fields["tokenizer.ggml.tokens"]
    toks = [bytes(f.parts[i]).decode("utf-8") for i in f.data]
    inv = {c: b for b, c in enumerate(synth.byte_tokens())}
    out = []
    for t in toks:
        if t.startswith("<|"):
            out.append(b"")
        else:
            out.append(bytes(inv[ch] for ch in t))
    return out


def kquant_small(R, meta):
    """A small model with every projection K-quant (synth.config_kquant_small): the reference engine's
    logits and routing trace of a 40-token prompt (passes of 32) and its 16 greedy tokens after it."""
    cfg = synth.config_kquant_small()
    with tempfile.TemporaryDirectory() as td:
        p = synth.write_gguf(os.path.join(td, "ks.gguf"), cfg)
        meta["kquant_small_sha256"] = sha256(p)
        prompt = synth._rng(cfg.seed, 0x9E1).integers(0, cfg.n_vocab, 40).astype(np.int32)
        e = R.engine(p, 256)
        e.trace(True)
        lg = e.eval(prompt, 0, 32)
        tr_ids, tr_w = e.trace_get()
        e.close()
        e = R.engine(p, 256)
        gen, _ = e.greedy(prompt, 16, 32)
        e.close()
    np.savez_compressed(os.path.join(GOLDEN, "kquant_small.npz"), prompt=prompt, logits=lg, gen=gen.astype(np.int32),
                        trace_ids=tr_ids, trace_w=tr_w)


def main():
    R = oracle.Reference(threads=os.cpu_count() or 1)
    if sys.argv[1:] == ["--only", "kquant_small"]:
        with open(os.path.join(GOLDEN, "fixtures.json")) as f:
            meta = json.load(f)
        kquant_small(R, meta)
        with open(os.path.join(GOLDEN, "fixtures.json"), "w") as f:
            json.dump(meta, f, indent=1, sort_keys=True)
        return
    meta = {"reference": os.path.relpath(REF, ROOT)}

    # ---- 1. reference tiny.gguf -----------------------------------------------------------------
    with tempfile.TemporaryDirectory() as td:
        shutil.copy(os.path.join(ROOT, "oracle", "_ref", "qwen3moe"), os.path.join(td, "qwen3moe"))
        r = subprocess.run([sys.executable, os.path.join(REF, "tests", "test_tiny.py")], cwd=td, capture_output=True,
                           text=True)
        print(r.stdout[-400:])
        if r.returncode != 0:
            raise SystemExit(f"reference test_tiny.py failed:\n{r.stderr[-2000:]}")
        tiny = os.path.join(GOLDEN, "ref_tiny.gguf")
        shutil.copy(os.path.join(td, "tiny.gguf"), tiny)
        tok = subprocess.run([os.path.join(td, "qwen3moe"), "-m", tiny, "--tokenize", "hello world ab ab"],
                             capture_output=True, text=True)
        hello_ids = [int(v) for v in tok.stdout.split()]
    meta["ref_tiny_sha256"] = sha256(tiny)

    # ---- 2. golden-vector checks of the reference engine -------------------------------------------
    eng = R.engine(tiny, 128)
    lg = eng.eval(PROMPT_IDS, 0, 32)
    want = open(os.path.join(REF, "baseline", "logits.txt")).read().replace("argmax", "").split()
    want16, want_am = np.array(want[:16], np.float64), int(want[16])
    d = float(np.abs(lg[:16] - want16).max())
    if not (d < 2e-6 and int(lg.argmax()) == want_am):
        raise SystemExit(f"reference engine does not reproduce baseline/logits.txt ({d:.2e})")
    gen, _ = eng.greedy(hello_ids, 24, 32)
    pieces = token_bytes(tiny)
    text = b"".join(pieces[t] for t in gen) + b"\n"
    golden = open(os.path.join(REF, "baseline", "gen_greedy.bin"), "rb").read()
    if text != golden:
        raise SystemExit("reference engine does not reproduce baseline/gen_greedy.bin")
    meta["baseline_logits_maxdiff"] = d
    meta["baseline_gen_greedy"] = "byte-exact"
    # routing trace of the residency suite's inference (tests/test_eahmmf.cpp:36-54)
    eng.close()
    eng = R.engine(tiny, 128)
    eng.trace(True)
    lg4 = eng.eval(PROMPT_IDS, 0, 4)
    ids12, pos, cur = [], len(PROMPT_IDS), lg4
    for _ in range(12):
        t = int(cur.argmax())
        ids12.append(t)
        cur = eng.eval([t], pos, 1)
        pos += 1
    tr_ids, tr_w = eng.trace_get()
    eng.close()
    np.savez_compressed(os.path.join(GOLDEN, "ref_tiny.npz"), prompt=np.array(PROMPT_IDS, np.int32), logits=lg,
                        hello_ids=np.array(hello_ids, np.int32), hello_gen=gen.astype(np.int32),
                        hello_text=np.frombuffer(text, np.uint8),
                        logits_b4=lg4, gen12=np.array(ids12, np.int32), trace_ids=tr_ids, trace_w=tr_w)

    # ---- 3a. config 1 model ---------------------------------------------------------------------
    cfg1 = synth.config1_tiny()
    with tempfile.TemporaryDirectory() as td:
        p1 = synth.write_gguf(os.path.join(td, "c1.gguf"), cfg1)
        meta["config1_sha256"] = sha256(p1)
        prompt = synth._rng(cfg1.seed, 0x9E0).integers(0, cfg1.n_vocab, 16).astype(np.int32)
        e1 = R.engine(p1, 512)
        e1.trace(True)
        toks, lg1 = e1.greedy(prompt, 32, 16)
        tr_ids1, tr_w1 = e1.trace_get()
        e1.close()
    np.savez_compressed(os.path.join(GOLDEN, "config1.npz"), prompt=prompt, gen=toks, logits=lg1, trace_ids=tr_ids1,
                        trace_w=tr_w1)

    # ---- 3b. config-2 MoE layer (reference block restated around the reference matmul) ---------------
    ex = synth.expert_set()
    out = {}
    for T in (1, 3, 8):
        x = synth.activations(T, ex.D, seed=100 + T)
        xn = synth.activations(T, ex.D, seed=200 + T)
        lgt = synth.router_logits(T, ex.n_expert, seed=300 + T)
        y, ids, w = R.moe_layer(x, xn, lgt, list(ex.gate), list(ex.up), list(ex.down), ex.types, ex.row_bytes, 8)
        out[f"y{T}"], out[f"ids{T}"], out[f"w{T}"] = y, ids, w
    np.savez_compressed(os.path.join(GOLDEN, "moe_c2.npz"), **out)

    # ---- 3c. mixed-type experts with a router matrix (reference tiny model's expert types) ----------
    mx = synth.expert_set(D=256, FF=256, n_expert=8, types=(13, 12, 14), seed=7, d_sigma=0.002)
    T = 11
    x = synth.activations(T, 256, seed=17)
    xn = synth.activations(T, 256, seed=18)
    rw = (synth._rng(19).normal(0, 0.3, (8, 256))).astype(np.float32)
    y, ids, w = R.moe_layer(x, xn, None, list(mx.gate), list(mx.up), list(mx.down), mx.types, mx.row_bytes, 2,
                            router_w=rw)
    np.savez_compressed(os.path.join(GOLDEN, "moe_mixed.npz"), y=y, ids=ids, w=w)

    # ---- 3d. single matmuls of every type ---------------------------------------------------------
    mm = {}
    for qt, K in ((12, 1024), (13, 512), (14, 768), (8, 288), (0, 320)):
        rows = 40
        spec = synth.TensorSpec("m", qt, (K, rows), "quant" if qt else "normal", 0.01 if qt else 0.3)
        raw = synth.tensor_array(spec, 9, qt)
        rb = synth.row_bytes(qt, K)
        for nb in (1, 5):
            xx = synth.activations(nb, K, seed=qt * 10 + nb)
            mm[f"w{qt}"] = raw
            mm[f"x{qt}_{nb}"] = xx
            mm[f"y{qt}_{nb}"] = R.matmul(raw, qt, K, rows, rb, xx)
    np.savez_compressed(os.path.join(GOLDEN, "matmul.npz"), **mm)

    # ---- 3e. small all-K-quant model ----------------------------------------------------------------
    kquant_small(R, meta)

    with open(os.path.join(GOLDEN, "fixtures.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print(json.dumps(meta, indent=1))


if __name__ == "__main__":
    main()
