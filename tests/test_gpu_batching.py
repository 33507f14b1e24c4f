"""Several sequences decoded together (eahmmf_engine_set_slots / prefill_slot / step_slots and the
continuous-batching scheduler) against each sequence decoded alone by the single-sequence engine path:
greedy ids exact for every request, with requests of different prompt lengths joining and leaving the
batch as slots free up. The per-row arithmetic of a multi-sequence step is the single-sequence one (the
projections' per-token sums do not depend on the rows beside them; attention reads each row's own cache).
"""
import os

import numpy as np
import pytest

import batching
import eahmmf_b200 as eb
import synth

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = os.path.join(ROOT, "tests", "golden", "ref_tiny.gguf")


@pytest.fixture(scope="module")
def kquant_path(tmp_path_factory):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required")
    return synth.write_gguf(str(tmp_path_factory.mktemp("kb") / "ks.gguf"), synth.config_kquant_small())


@pytest.mark.parametrize("model", ["kquant", "tiny"])
def test_batched_requests_match_single_sequence_decode(kquant_path, model):
    path = kquant_path if model == "kquant" else TINY
    rng = np.random.default_rng(3)
    vocab = 1000 if model == "kquant" else 250
    reqs = [(rng.integers(0, vocab, int(rng.integers(3, 70))).astype(np.int32), int(rng.integers(2, 18)))
            for _ in range(9)]
    alone = eb.Engine(path, 128)
    want = []
    for prompt, n in reqs:
        rc, out, _ = alone.greedy(prompt, n, 64)
        assert rc == 0
        want.append(out)
    alone.close()
    e = eb.Engine(path, 128)
    try:
        b = batching.ContinuousBatcher(e, n_slots=4)
        rs = [b.submit(p, n) for p, n in reqs]
        b.run()
        assert b.steps > 0
        for r, w in zip(rs, want):
            np.testing.assert_array_equal(r.tokens, w)
        # the single-sequence calls still work on slot 0 afterwards
        rc, out, _ = e.greedy(reqs[0][0], reqs[0][1], 64)
        assert rc == 0
        np.testing.assert_array_equal(out, want[0])
    finally:
        e.close()


def test_step_slots_rejects_bad_rows(kquant_path):
    e = eb.Engine(kquant_path, 64)
    try:
        assert e.set_slots(2) == 0
        rc, first = e.prefill_slot(0, [1, 2, 3])
        assert rc == 0
        assert e.step_slots([0, 0], [3, 3], [first, first])[0] == eb.ST_BAD_ARG  # one row per sequence
        assert e.step_slots([2], [3], [first])[0] == eb.ST_BAD_ARG  # no such slot
        assert e.step_slots([1], [64], [first])[0] == eb.ST_BAD_ARG  # past the context
        assert e.step_slots([0], [3], [first])[0] == 0
    finally:
        e.close()
