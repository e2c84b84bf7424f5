"""Host-side rules of the FloatBackend operator set, checked without a GPU: AttentionLayout.validate's
shape and workspace rules (core/src/main/scala/scalatorch/AttentionLayout.scala:3-19) reject before any
native call, and the per-op path's scope releases in reverse order (BackendLlama.scala:9-24)."""
import pytest

from scalatorch import ffm
from scalatorch.models import _Scope


def test_attention_layout_accepts_grouped_heads():
    out, scores = ffm.attention_layout((2, 8, 3, 64), (2, 2, 5, 64), (2, 2, 5, 32), 2, 1 << 24)
    assert out == (2, 8, 3, 32) and scores == 2 * 8 * 3 * 5
    assert ffm.attention_layout((1, 4, 0, 16), (1, 2, 0, 16), (1, 2, 0, 16), 0, 0) == ((1, 4, 0, 16), 0)


@pytest.mark.parametrize("q,k,v,start,limit", [
    ((2, 8, 3, 64), (2, 2, 5, 64), (2, 2, 5), 0, 1 << 24),      # rank
    ((2, 8, 3, 64), (1, 2, 5, 64), (1, 2, 5, 64), 0, 1 << 24),  # batch
    ((2, 6, 3, 64), (2, 4, 5, 64), (2, 4, 5, 64), 0, 1 << 24),  # heads not a multiple of kv heads
    ((2, 8, 3, 64), (2, 2, 5, 32), (2, 2, 5, 64), 0, 1 << 24),  # key width
    ((2, 8, 3, 64), (2, 2, 5, 64), (2, 2, 4, 64), 0, 1 << 24),  # key / value tokens
    ((2, 8, 3, 64), (2, 2, 0, 64), (2, 2, 0, 64), 0, 1 << 24),  # queries without keys
    ((2, 8, 3, 64), (2, 2, 5, 64), (2, 2, 5, 64), -1, 1 << 24),  # offset
    ((2, 8, 3, 64), (2, 2, 5, 64), (2, 2, 5, 64), 0, 239),      # score workspace (240 needed)
])
def test_attention_layout_rejections(q, k, v, start, limit):
    with pytest.raises(ffm.IllegalArgumentException):
        ffm.attention_layout(q, k, v, start, limit)


class _Recorder:
    def __init__(self):
        self.released = []

    def release(self, t):
        self.released.append(t)


def test_scope_releases_in_reverse_and_hands_over_one_result():
    be = _Recorder()
    with _Scope(be) as scope:
        a, b, c = scope.keep("a"), scope.keep("b"), scope.keep("c")
        assert scope.take(b) == "b"
        scope.release(a)
    assert be.released == ["a", "c"]
    with pytest.raises(ffm.IllegalArgumentException):
        _Scope(be).take("x")
