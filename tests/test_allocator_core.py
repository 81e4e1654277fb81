"""The caching allocator's policy on a fake device (CPU only): rounding,
the 1.25x reuse window, stream-ordered reuse, out-of-memory retry and the
statistics the reference's tests read (tensorplay-mlu
tensorplay_mlu/csrc/MLUAllocator.cpp:37-128, tests/test_mlu.py:404-414)."""

from __future__ import annotations

import ctypes
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "native", "allocator_fake.cpp")
CSRC = os.path.join(ROOT, "tensorplay_mlu_b200", "csrc")


@pytest.fixture(scope="module")
def fake(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("alloc") / "libfake.so")
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", f"-I{CSRC}", SRC, "-o", out],
                   check=True)
    lib = ctypes.CDLL(out)
    lib.fake_alloc.restype = ctypes.c_void_p
    lib.fake_alloc.argtypes = [ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    lib.fake_free.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.fake_stats.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int64)]
    lib.fake_reset.argtypes = [ctypes.c_int64]
    lib.fake_capture_holding.argtypes = [ctypes.c_int]
    for name in ("fake_raw_allocs", "fake_cross_waits", "fake_device_syncs", "fake_used",
                 "fake_capture_allocations", "fake_capture_blocks"):
        getattr(lib, name).restype = ctypes.c_int64
    lib.fake_round.restype = ctypes.c_size_t
    lib.fake_round.argtypes = [ctypes.c_size_t]
    return lib


def stats(lib, dev=0):
    out = (ctypes.c_int64 * 4)()
    lib.fake_stats(dev, out)
    return list(out)


S1, S2 = ctypes.c_void_p(0x1000), ctypes.c_void_p(0x2000)  # two fake streams


def test_rounding(fake):
    MiB = 1 << 20
    assert fake.fake_round(1) == 512
    assert fake.fake_round(512) == 512
    assert fake.fake_round(513) == 1024
    assert fake.fake_round(MiB) == MiB
    assert fake.fake_round(MiB + 1) == 2 * MiB
    assert fake.fake_round(5 * MiB) == 6 * MiB


def test_reuse_window_and_stats(fake):
    fake.fake_reset(1 << 30)
    MiB = 1 << 20
    p = fake.fake_alloc(8 * MiB, 0, S1)
    assert stats(fake) == [8 * MiB, 8 * MiB, 8 * MiB, 8 * MiB]
    assert fake.fake_free(p, S1) == 0
    assert stats(fake)[0] == 0 and stats(fake)[1] == 8 * MiB
    # 8 MiB block serves a 7 MiB request (8 <= 1.25 * 7) ...
    q = fake.fake_alloc(7 * MiB, 0, S1)
    assert q == p and fake.fake_raw_allocs() == 1
    fake.fake_free(q, S1)
    # ... but not a 4 MiB one (8 > 1.25 * 4): a new block.
    r = fake.fake_alloc(4 * MiB, 0, S1)
    assert r != p and fake.fake_raw_allocs() == 2
    fake.fake_free(r, S1)
    fake.fake_reset_peak(0)
    assert stats(fake)[2] == 0
    fake.fake_empty_cache()
    assert stats(fake)[1] == 0 and fake.fake_used() == 0


def test_stream_ordered_reuse(fake):
    fake.fake_reset(1 << 30)
    MiB = 1 << 20
    p = fake.fake_alloc(2 * MiB, 0, S1)
    fake.fake_free(p, S1)
    # Same stream: reused with no cross-stream ordering.
    q = fake.fake_alloc(2 * MiB, 0, S1)
    assert q == p and fake.fake_cross_waits() == 0
    fake.fake_free(q, S1)
    # Another stream while the block's last use may still run: reused, but
    # ordered behind the event recorded at free time.
    r = fake.fake_alloc(2 * MiB, 0, S2)
    assert r == p and fake.fake_cross_waits() == 1
    fake.fake_free(r, S2)


def test_out_of_memory_releases_cache_and_retries(fake):
    MiB = 1 << 20
    fake.fake_reset(10 * MiB)
    p = fake.fake_alloc(8 * MiB, 0, S1)
    fake.fake_free(p, S1)  # cached, still reserved
    syncs = fake.fake_device_syncs()
    q = fake.fake_alloc(6 * MiB, 0, S1)  # 8 > 1.25 * 6: needs a new block; only fits after release
    assert q is not None and fake.fake_device_syncs() == syncs + 1
    assert stats(fake)[1] == 6 * MiB
    assert fake.fake_alloc(64 * MiB, 0, S1) is None  # beyond capacity even after release
    fake.fake_free(q, S1)


def test_foreign_pointer_rejected(fake):
    fake.fake_reset(1 << 30)
    assert fake.fake_free(ctypes.c_void_p(0xdead000), S1) == -1


def test_devices_are_separate(fake):
    fake.fake_reset(1 << 30)
    MiB = 1 << 20
    p = fake.fake_alloc(2 * MiB, 1, S1)
    assert stats(fake, 1)[0] == 2 * MiB and stats(fake, 0)[0] == 0
    fake.fake_free(p, S1)


def test_recording_holds_its_blocks_until_dropped(fake):
    """Stream capture (MLUAllocator.cpp:130-190): blocks handed out while
    recording are reused only inside the recording, are frozen when it ends,
    and go back to the driver only when it is dropped."""
    MiB = 1 << 20
    fake.fake_reset(1 << 30)
    before = fake.fake_alloc(2 * MiB, 0, S1)       # allocated before the recording
    fake.fake_free(before, S1)                      # cached; its event is pending
    fake.fake_capture_holding(1)
    a = fake.fake_alloc(2 * MiB, 0, S1)             # pending event: not taken while recording
    assert a != before
    fake.fake_free(a, S1)                           # given back inside the recording...
    b = fake.fake_alloc(2 * MiB, 0, S1)             # ...and reused by the recording itself
    assert b == a and fake.fake_cross_waits() == 0
    c = fake.fake_alloc(4 * MiB, 0, S1)
    assert fake.fake_capture_allocations() == 3
    fake.fake_free(c, S1)
    fake.fake_capture_holding(0)
    fake.fake_capture_freeze()                      # c's block is now held
    assert fake.fake_capture_blocks() == 1
    d = fake.fake_alloc(4 * MiB, 0, S1)             # the held block is not handed out again
    assert d != c
    fake.fake_free(d, S1)
    fake.fake_free(b, S1)                           # a block the recording uses, freed later: held
    assert fake.fake_capture_blocks() == 2
    reserved = stats(fake)[1]
    syncs = fake.fake_device_syncs()
    fake.fake_capture_drop()
    assert fake.fake_capture_blocks() == 0 and fake.fake_device_syncs() == syncs + 1
    assert stats(fake)[1] == reserved - 6 * MiB
    e = fake.fake_alloc(2 * MiB, 0, S1)             # the pre-recording block is back in use
    assert e == before
    fake.fake_free(e, S1)


def test_block_freed_during_recording_is_held(fake):
    """A block from before the recording that the recorded work frees may
    still be read by replays: it is held with the recording's blocks."""
    MiB = 1 << 20
    fake.fake_reset(1 << 30)
    p = fake.fake_alloc(2 * MiB, 0, S1)
    fake.fake_capture_holding(1)
    fake.fake_free(p, S1)
    fake.fake_capture_holding(0)
    fake.fake_capture_freeze()
    assert fake.fake_capture_blocks() == 1
    assert fake.fake_alloc(2 * MiB, 0, S1) != p
