"""Launch-overlap bookkeeping (no GPU needed): which reads a chain launch may issue before the
previous kernel on its stream has completed. gp_debug_pdl_flags runs the library's own decision
and record update for a set of byte ranges without launching anything.

Rules under test:
  - a stream without a record allows no early reads;
  - parameters (bit 1) or input rows (bit 2) that overlap what the stream's last chain launch
    writes must wait; ranges apart from those writes may be read early;
  - a launch whose writes are not listed leaves a record that allows nothing early;
  - streams are separate, except the legacy handle and NULL, which name the same stream;
  - the per-thread default stream is never tracked (it is a different stream per host thread).
"""
import os

import pytest

from gpu_pipes_b200 import _lib as L

PARAM, X, WRITE, UNKNOWN = 0, 1, 2, 3
LEGACY, PER_THREAD = 0x1, 0x2

pytestmark = pytest.mark.skipif(os.environ.get("GP_PDL", "1")[:1] in ("0", "2"),
                                reason="early reads are off in this environment")

_next = [0x5000]


def fresh_stream():
    """A stream handle no earlier test used (the library only compares handles)."""
    _next[0] += 0x10
    return _next[0]


def test_no_record_no_early_reads():
    s = fresh_stream()
    assert L.pdl_flags(s, [(0x100000, 4096, PARAM), (0x200000, 4096, X)]) == 0


def test_overlap_clears_its_bit():
    s = fresh_stream()
    L.pdl_flags(s, [(0x300000, 1 << 20, WRITE)])  # the stream's last launch writes [3 MB, 4 MB)
    # x inside that range waits; parameters elsewhere may go early
    assert L.pdl_flags(s, [(0x100000, 4096, PARAM), (0x300000 + 512, 64, X), (0x900000, 64, WRITE)]) == 1
    # the record is now [9 MB, 9 MB + 64): parameters overlapping it wait, x apart from it goes
    assert L.pdl_flags(s, [(0x900000 + 32, 64, PARAM), (0x100000, 4096, X)]) == 2
    # ranges that merely touch (end == start) do not overlap
    L.pdl_flags(s, [(0x400000, 4096, WRITE)])
    assert L.pdl_flags(s, [(0x400000 + 4096, 64, PARAM), (0x400000 - 64, 64, X)]) == 3


def test_unknown_writes_block_the_next_launch():
    s = fresh_stream()
    L.pdl_flags(s, [(0, 0, UNKNOWN)])
    assert L.pdl_flags(s, [(0x100000, 64, PARAM), (0x200000, 64, X)]) == 0
    # the launch that just probed recorded no writes, so the one after it may read early
    assert L.pdl_flags(s, [(0x100000, 64, PARAM), (0x200000, 64, X)]) == 3


def test_streams_are_separate():
    a, b = fresh_stream(), fresh_stream()
    L.pdl_flags(a, [(0x700000, 4096, WRITE)])
    L.pdl_flags(b, [(0x800000, 4096, WRITE)])
    assert L.pdl_flags(a, [(0x800000, 64, PARAM), (0x800000, 64, X)], record=False) == 3
    assert L.pdl_flags(b, [(0x800000, 64, PARAM)], record=False) == 2


def test_legacy_handle_and_null_share_a_record():
    L.pdl_flags(LEGACY, [(0xA00000, 4096, WRITE)])
    assert L.pdl_flags(0, [(0xA00000, 64, X), (0x100000, 64, PARAM)], record=False) == 1


def test_per_thread_stream_is_untracked():
    L.pdl_flags(PER_THREAD, [(0xB00000, 4096, WRITE)])
    assert L.pdl_flags(PER_THREAD, [(0x100000, 64, PARAM), (0x200000, 64, X)]) == 0


def test_bad_kind_is_rejected():
    assert L.lib().gp_debug_pdl_flags(None, 1, None, None, None, 0) == L.GP_ERR_ARG
    assert L.pdl_flags(fresh_stream(), [(0x100000, 64, 7)]) == L.GP_ERR_ARG
