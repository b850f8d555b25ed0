"""Host logic of the graph-replayed decode step (no GPU): the key bound its
fused layer plans are made for, a power of two of at least 256 covering the
longest stream, at most the window; the step moves to the next bound (a
second set of plans and a second graph) when the longest stream passes one."""
import pytest

torch = pytest.importorskip("torch")


def test_key_bound():
    from decode_step import key_bound
    assert key_bound(1, 8192) == 256
    assert key_bound(256, 8192) == 256
    assert key_bound(257, 8192) == 512
    assert key_bound(7301, 8192) == 8192
    assert key_bound(9000, 8192) == 8192          # lengths stop at the window
    assert key_bound(100, 64) == 64               # windows below 256
    assert key_bound(300, 384) == 384             # the window caps the power of two
    bounds = [key_bound(n, 8192) for n in range(1, 8193)]
    assert bounds == sorted(bounds) and all(b >= n for n, b in zip(range(1, 8193), bounds))
