"""Host-side behaviour of the sequence Session.call returns (no device work):
indexing, slicing and iteration wrap each entry once as a Buffer that then
owns it, and dropping the sequence releases the entries never read in one
sb_buffer_release_many call. Null handles stand in for device buffers, which
the release skips."""
import ctypes as C

import pytest

from sheaf_b200.runtime import Buffer, Outputs


def _outs(n: int, cap: int = 8) -> Outputs:
    return Outputs((C.c_void_p * cap)(), n)


def test_length_and_indexing():
    o = _outs(3)
    assert len(o) == 3
    b0 = o[0]
    assert isinstance(b0, Buffer)
    assert o[0] is b0  # wrapped once
    assert o[-1] is o[2]
    with pytest.raises(IndexError):
        o[3]
    with pytest.raises(IndexError):
        o[-4]


def test_slices_and_iteration():
    o = _outs(5)
    tail = o[1:]
    assert len(tail) == 4 and all(isinstance(b, Buffer) for b in tail)
    assert list(o)[1:] == tail
    assert o[::2] == [o[0], o[2], o[4]]


def test_read_entries_leave_the_batch_release():
    o = _outs(4)
    _ = o[1]
    arr = o._arr
    assert arr[1] is None  # owned by its Buffer now
    o.release()
    assert o._arr is None
    o.release()  # a second release does nothing
