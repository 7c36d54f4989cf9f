"""The causal chunk planner against the reference's own tests
(src/util/causal.rs:165-271, restated). CPU only."""
import pytest

from burn_rocket_b200.causal import CausalChunk, causal_chunk_plan


def test_plan_chunk_zero_is_the_dense_run():
    assert causal_chunk_plan(5000, 5000, 0, None, 0) == [CausalChunk(0, 5000, 0, 5000)]
    p = causal_chunk_plan(64, 64, 0, None, 1024)
    assert len(p) == 1 and (p[0].q0, p[0].q1, p[0].k0, p[0].k1) == (0, 64, 0, 64)


def test_plan_pure_causal_prefixes():
    p = causal_chunk_plan(2500, 2500, 0, None, 1000)
    assert p == [CausalChunk(0, 1000, 0, 1000), CausalChunk(1000, 2000, 0, 2000), CausalChunk(2000, 2500, 0, 2500)]
    for c in p:
        assert c.k0 == 0 and c.k1 <= c.q1 and c.k1 == c.q1


def test_plan_sliding_window_bands():
    w, chunk = 256, 1024
    p = causal_chunk_plan(3000, 3000, 0, w, chunk)
    assert p[0].k0 == 0
    for c in p[1:]:
        assert c.k0 == max(c.q0 - (w - 1), 0)
        assert c.k1 == c.q1
        assert c.k1 - c.k0 <= chunk + w - 1
    assert p[-1].q1 == 3000 and p[-1].k0 == p[-1].q0 - (w - 1)


def test_plan_respects_a_shorter_key_axis():
    for c in causal_chunk_plan(1500, 2000, 0, None, 512):
        assert c.k1 == min(c.q1, 2000)
    p = causal_chunk_plan(600, 4000, 3000, 128, 256)
    assert all(c.k1 == 3000 + c.q1 for c in p)
    assert p[0].k0 == 3000 - 127 and p[1].k0 == 3000 + 256 - 127


@pytest.mark.parametrize("s", [1, 7, 1024, 1025, 3001])
@pytest.mark.parametrize("chunk", [1, 3, 64, 1024, 4096])
def test_plan_ragged_tail_counts_every_query_once(s, chunk):
    nxt = 0
    for c in causal_chunk_plan(s, s, 0, None, chunk):
        assert c.q0 == nxt and c.q1 > c.q0
        nxt = c.q1
    assert nxt == s


def test_plan_rejects_empty():
    with pytest.raises(ValueError):
        causal_chunk_plan(0, 5, 0, None, 0)
    with pytest.raises(ValueError):
        causal_chunk_plan(5, 0, 0, None, 0)
