"""The reference engine's ExpertStore on eahmmf::B200Device, and eahmmf_cuda_moe_layer fed from the
layer tables that eahmmf::B200LayerTable builds out of ExpertLeases (include/eahmmf_b200_device.hpp).

Runs oracle/_ref/b200_store_check (built with the reference engine compiled unmodified) on the
reference's tiny model:
  * the store places every expert in VRAM through B200Device with --verify checksums on, and the bytes
    read back through the backend equal the GGUF source;
  * decode with every expert matmul on the GPU gives the reference CPU logits within 2e-6 and the same
    12 greedy ids;
  * per layer, the table holds one pin per expert while it lives and none after clear(); the MoE layer
    on those tables routes bit-exactly and matches the reference MoE block within rel-L2 1e-5.
"""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "b200_store_check")
TINY = os.path.join(ROOT, "tests", "golden", "ref_tiny.gguf")


@pytest.fixture(scope="module")
def report(golden):
    if not os.path.exists(BIN):
        pytest.fail(f"{BIN} missing: `make -C oracle storecheck` in the build container")
    g = golden("ref_tiny.npz")
    ids = ",".join(str(int(t)) for t in g["prompt"])
    r = subprocess.run([BIN, TINY, ids, "12", "5"], capture_output=True, timeout=300,
                       env=dict(os.environ, OMP_NUM_THREADS="4"))
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    return r.stdout.decode(), g


def test_backend_decode_matches_reference(report):
    out, g = report
    assert re.search(r"^backend_name cuda$", out, re.M)
    lg = np.array(re.search(r"^logits (.*)$", out, re.M).group(1).split(), np.float64)
    assert np.abs(lg - g["logits"]).max() < 2e-6
    greedy = [int(v) for v in re.search(r"^greedy (.*)$", out, re.M).group(1).split()]
    assert greedy == [int(v) for v in g["gen12"]]
    assert re.search(r"^store_pinned_after_decode 0$", out, re.M)


def test_layer_tables_from_leases(report):
    out, _ = report
    n_layer = len(re.findall(r"^layer \d+ table", out, re.M))
    n_expert = int(re.search(r"^n_expert (\d+)$", out, re.M).group(1))
    assert n_layer >= 2
    for l in range(n_layer):
        m = re.search(rf"^layer {l} table (\d) pinned (\d+)$", out, re.M)
        assert m and m.group(1) == "1"
        assert int(m.group(2)) == n_expert  # one pin per expert while the table lives
        m = re.search(rf"^layer {l} bytes_equal (\d) status (-?\d+) ids_equal (\d) rel_l2 (\S+)$", out, re.M)
        assert m, out[-2000:]
        assert m.group(1) == "1" and m.group(2) == "0" and m.group(3) == "1"
        assert float(m.group(4)) < 1e-5
        assert re.search(rf"^layer {l} released pinned 0$", out, re.M)
    assert re.search(r"^done 1$", out, re.M)


# ---- the residency tiers on the device backend (oracle/b200_tier_check) ----------------------------
TIER_BIN = os.path.join(ROOT, "oracle", "_ref", "b200_tier_check")


@pytest.fixture(scope="module")
def tiers():
    if not os.path.exists(TIER_BIN):
        pytest.fail(f"{TIER_BIN} missing: `make -C oracle storecheck` in the build container")
    r = subprocess.run([TIER_BIN, TINY], capture_output=True, timeout=600, env=dict(os.environ, OMP_NUM_THREADS="4"))
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    return r.stdout.decode()


def test_tier_matrix_on_b200_device_is_bitwise_baseline(tiers):
    """Every tier / budget case of the reference suite's matrix (tests/test_eahmmf.cpp:184-219 of the
    reference) with B200Device as the store's backend: logits, greedy ids and routing trace bitwise equal
    to the SSD-tier run, invariants hold, no pins left."""
    cases = re.findall(r"^case (\S+) same (\d) invariants (\d) pinned (\d+) acq (\d+) rel (\d+) ssd_ram (\d+) "
                       r"ram_vram (\d+) vram_ram (\d+) ram_ssd (\d+) vram_ssd (\d+) fallbacks (\d+)", tiers, re.M)
    assert len(cases) == 9, tiers[-2000:]
    by = {c[0]: [int(v) for v in c[1:]] for c in cases}
    for name, v in by.items():
        assert v[0] == 1 and v[1] == 1 and v[2] == 0 and v[3] == v[4], (name, v)
    every = by["vram_2_ram_2_every_path"]
    assert every[5] > 0 and every[6] > 0 and every[7] > 0 and every[8] > 0  # all four pager paths
    drop = by["vram_2_ram_1_drop_path"]
    assert drop[9] > 0 and drop[7] == 0  # VRAM victims dropped to SSD when RAM cannot take them
    assert by["vram_unlimited"][6] > 0  # experts really went to the device


def test_residency_walk_and_faults_on_b200_device(tiers):
    for name in ("walk_ssd", "walk_ram", "walk_vram", "walk_back_ram", "walk_back_ssd", "walk_invariants"):
        assert re.search(rf"^check {name} 1$", tiers, re.M), (name, tiers[-1500:])
    faults = re.findall(r"^fault (\S+) same (\d) migration_failures (\d+) alloc_failures (\d+) fallbacks (\d+) "
                        r"invariants (\d) pinned (\d+)$", tiers, re.M)
    assert len(faults) == 3
    for f in faults:
        assert f[1] == "1" and f[5] == "1" and f[6] == "0", f
        assert int(f[2]) + int(f[3]) > 0, f  # the injected faults were seen by the store
    assert re.search(r"^done 1$", tiers, re.M)
