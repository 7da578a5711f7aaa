"""CopyOverlap's ordering bookkeeping, without a GPU: a buffer is the element range it
covers in its owner; a copy or kernel waits for the recorded events of every range that
overlaps its own, and re-recording a range replaces its entry (the tables stay as large as
the set of distinct ranges)."""
from cormorant_b200.runtime import CopyOverlap, InferenceBuf


class _Buf:
    """Stand-in with the two things CopyOverlap reads: the device address and the count."""

    def __init__(self, dev, count, owner=None):
        self._dev, self._count, self._keep = dev, count, owner

    def phys(self):
        return self._dev

    def count(self):
        return self._count


def _view(owner, off, count):
    return _Buf(owner.phys() + off * InferenceBuf.BYTES_PER_ELEM, count, owner)


def test_ranges():
    own = _Buf(0x10000, 100)
    assert CopyOverlap._range(own) == (id(own), 0, 100)
    assert CopyOverlap._range(_view(own, 30, 20)) == (id(own), 30, 50)


def test_disjoint_views_independent_overlapping_ordered():
    own, other = _Buf(0x10000, 100), _Buf(0x90000, 100)
    t = {}
    CopyOverlap._record(t, CopyOverlap._range(_view(own, 0, 50)), "e0")
    CopyOverlap._record(t, CopyOverlap._range(_view(own, 50, 50)), "e1")
    assert CopyOverlap._overlapping(t, CopyOverlap._range(_view(own, 0, 50))) == ["e0"]
    assert CopyOverlap._overlapping(t, CopyOverlap._range(_view(own, 50, 50))) == ["e1"]
    assert CopyOverlap._overlapping(t, CopyOverlap._range(_view(own, 49, 2))) == ["e0", "e1"]
    assert sorted(CopyOverlap._overlapping(t, CopyOverlap._range(own))) == ["e0", "e1"]
    assert CopyOverlap._overlapping(t, CopyOverlap._range(other)) == []
    # empty and touching ranges do not overlap
    assert CopyOverlap._overlapping(t, CopyOverlap._range(_view(own, 100, 0))) == []


def test_rerecord_replaces():
    own = _Buf(0x10000, 64)
    t = {}
    for step in range(5):
        for i in range(4):
            CopyOverlap._record(t, CopyOverlap._range(_view(own, 16 * i, 16)), (step, i))
    assert len(t[id(own)]) == 4
    assert CopyOverlap._overlapping(t, CopyOverlap._range(_view(own, 16, 16))) == [(4, 1)]
    CopyOverlap._record(t, CopyOverlap._range(own), "whole")
    assert len(t[id(own)]) == 5
    assert "whole" in CopyOverlap._overlapping(t, CopyOverlap._range(_view(own, 0, 1)))
