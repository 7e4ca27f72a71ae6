"""Host-side logic of the cache's call path, without a GPU."""
import re

import numpy as np

from tests.conftest import ROOT


def test_int_list_accepts_only_python_ints():
    """Query positions take the numpy-free path only as a flat list or tuple of Python ints."""
    from apple_b200.cache import _int_list
    assert _int_list([3, 4]) == [3, 4]
    assert _int_list((7,)) == (7,)
    assert _int_list([]) == []
    for other in (None, [1, True], [np.int64(1)], np.array([1]), [1.0], [[1]]):
        assert _int_list(other) is None


def test_workspace_status_matches_header():
    """The wrapper retries a patched call on RFSN_ERR_WORKSPACE_TOO_SMALL: its value is the header's."""
    from apple_b200 import _lib
    header = (ROOT / "include" / "rfsn_b200.h").read_text()
    m = re.search(r"RFSN_ERR_WORKSPACE_TOO_SMALL\s*=\s*(-?\d+)", header)
    assert m and int(m.group(1)) == _lib.RFSN_ERR_WORKSPACE_TOO_SMALL
