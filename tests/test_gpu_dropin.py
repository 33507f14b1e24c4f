"""Drop-in check of the reference's C ABI: the unmodified reference engine (qwen3moe.cpp, built by
oracle/Makefile with -DEAHMMF_CUDA -DEAHMMF_CUDA_COMPUTE) linked against libeahmmf_b200.so instead of
expert_cuda.o, run with every expert matmul on the GPU (--device cuda --expert-tier vram --cuda-compute).

Expected, as the reference's own check_baseline.sh states them for its tiny model: the 16 printed logits
within 2e-6 of the reference CPU run and the same argmax; the 24-token greedy text byte-exact; no CPU
fallback (cpu_fallbacks=0 in the engine's own counter, qwen3moe.cpp:463-469).
"""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "qwen3moe_b200")
TINY = os.path.join(ROOT, "tests", "golden", "ref_tiny.gguf")
GPU_FLAGS = ["--device", "cuda", "--expert-tier", "vram", "--cuda-compute"]


def run(args, env_extra=None):
    if not os.path.exists(BIN):
        pytest.fail(f"{BIN} missing: `make -C oracle dropin` in the build container")
    env = dict(os.environ, OMP_NUM_THREADS="4", **(env_extra or {}))
    r = subprocess.run([BIN, "-m", TINY, "-c", "128", *args], capture_output=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    return r.stdout, r.stderr.decode()


def counters(stderr):
    m = re.search(r"cuda-compute: gpu_calls=(\d+) cpu_fallbacks=(\d+) pair_calls=(\d+)", stderr)
    assert m, stderr[-1000:]
    return tuple(int(v) for v in m.groups())


@pytest.mark.parametrize("pair", [True, False])
def test_dropin_logits_match_reference(golden, pair):
    g = golden("ref_tiny.npz")
    ids = ",".join(str(int(t)) for t in g["prompt"])
    out, err = run(["-b", "32", *GPU_FLAGS, "--logits-test", ids], None if pair else {"EAHMMF_DISABLE_PAIR": "1"})
    lines = out.decode().strip().split("\n")
    got = np.array(lines[0].split(), np.float64)
    assert np.abs(got - g["logits"][:16]).max() < 2e-6
    assert int(lines[1].split()[1]) == int(np.argmax(g["logits"]))
    gpu_calls, fallbacks, pairs = counters(err)
    assert gpu_calls > 0 and fallbacks == 0
    assert (pairs > 0) == pair


def test_dropin_greedy_generation_byte_exact(golden):
    g = golden("ref_tiny.npz")
    out, err = run(["--raw", "-p", "hello world ab ab", "--temp", "0", "--repeat-penalty", "1.0", "-n", "24",
                    *GPU_FLAGS])
    assert out == g["hello_text"].tobytes()
    assert counters(err)[1] == 0


def test_dropin_shadow_agrees_with_cpu():
    # --cuda-shadow re-runs every GPU matmul on the CPU and counts results whose max-abs-normalised
    # error exceeds the reference's 1e-4 gate (qwen3moe.cpp:494-508)
    _, err = run(["-b", "8", *GPU_FLAGS, "--cuda-shadow", "--logits-test", "5,17,200,33"])
    m = re.search(r"cuda-shadow: calls=(\d+) bad=(\d+) skipped=(\d+) max_rel_err=([0-9.eE+-]+)", err)
    assert m, err[-1000:]
    calls, bad, skipped, rel = int(m.group(1)), int(m.group(2)), int(m.group(3)), float(m.group(4))
    assert calls > 0 and bad == 0 and rel < 1e-4
