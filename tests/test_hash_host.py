"""The residency layer's checksum on the host side of this library (eahmmf_hash64, the source side of
eahmmf_engine_verify) against the reference's own hash64 (eahmmf.h:64-76, compiled from its sources):
equal on buffers of every length modulo 8, empty included. No GPU needed."""
import numpy as np
import pytest

import eahmmf_b200 as eb


@pytest.mark.parametrize("n", [0, 1, 7, 8, 9, 63, 64, 65, 1000, 884736, 1290240 + 3])
def test_host_hash64_matches_reference(ref, n):
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8)
    assert eb.hash64(data) == ref.hash64(data)
