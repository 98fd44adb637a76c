"""The Python restatement of Philox4x32-10 used by the GPU noise tests,
pinned to the published known-answer vectors (Random123)."""
from test_philox_gpu import KAT, philox_py


def test_restatement_known_answers():
    for c, k, want in KAT:
        assert tuple(philox_py(c, k)) == want
