"""Launch shapes of the NVLink kernels, checked on the CPU.

cail_dev_plan() returns the shape each path computes for a call (the same
functions the runtime uses), without a GPU.  Over many rank counts, element
sizes and message sizes (ragged tails, fewer elements than ranks, unaligned
buffers) every shape must keep each kernel inside its buffers and cover the
whole message:

* push two-shot: the slices partition [0, bytes) in order, start on 16-byte
  units in the vector path (and on elements otherwise), only the last slice
  holds the ragged tail, rounds x CTAs x piece covers the longest slice, and
  the slots of all CTAs fit the workspace area;
* one-shot: CTAs x rounds x piece covers the message, three slots per CTA
  and rank fit the area, and the slot layout depends on the call only
  through its piece (8 KiB for every message up to gmax x 8 KiB);
* NVLS: every CTA gets the same number of units, all units are covered,
  no CTA is idle, and the two slots per CTA fit the staging area.
"""
import ctypes
import os

import pytest

from conftest import LIB, ensure_build

SIZES = [1, 2, 3, 7, 15, 16, 17, 1000, 4099, 65536, 65537, 1000003, 4194304, 25 << 20, (256 << 20) + 12345,
         1 << 30]


@pytest.fixture(scope="module")
def lib():
    ensure_build()
    ctypes.CDLL(os.path.join(LIB, "libmpi.so"), mode=ctypes.RTLD_GLOBAL)
    c = ctypes.CDLL(os.path.join(LIB, "libcail.so"))
    c.cail_dev_plan.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int,
                                ctypes.c_int, ctypes.POINTER(ctypes.c_ulonglong), ctypes.c_int]
    return c


def plan(c, kind, P, count, esz, vec=1, gmax=296):
    out = (ctypes.c_ulonglong * 16)()
    n = c.cail_dev_plan(kind, P, count, esz, vec, gmax, out, 16)
    assert n > 0, (kind, P, count, esz)
    return list(out[:n])


@pytest.mark.parametrize("P", [2, 3, 4, 5, 7, 8])
@pytest.mark.parametrize("gmax", [296, 148, 37])
def test_push_two_shot_shapes(lib, P, gmax):
    for esz in (1, 2, 4, 8):
        for elems in SIZES:
            for vec in (1, 0):
                G, piece, rounds, max_slice, area, *off = plan(lib, 1, P, elems, esz, vec, gmax)
                nbytes = elems * esz
                assert off[0] == 0 and off[P] == nbytes and all(off[q] <= off[q + 1] for q in range(P))
                unit = 16 if vec else esz
                assert all(off[q] % unit == 0 for q in range(P))
                assert all(off[q + 1] - off[q] <= max_slice for q in range(P))
                assert max_slice == max(off[q + 1] - off[q] for q in range(P))
                # only the last slice may hold a partial unit (the ragged tail)
                assert all((off[q + 1] - off[q]) % unit == 0 for q in range(P - 1))
                assert 1 <= G <= gmax and piece % 16 == 0 and piece > 0
                assert rounds * G * piece >= max_slice
                assert (rounds - 1) * G * piece < max(max_slice, 1)  # no round without work
                assert 2 * G * P * piece <= area  # both parities of every CTA's slots


@pytest.mark.parametrize("P", [2, 3, 4, 8])
@pytest.mark.parametrize("gmax", [296, 148])
def test_one_shot_shapes(lib, P, gmax):
    layouts = set()
    for esz in (1, 4, 8):
        for elems in SIZES:
            G, piece, area, sg, piece_max = plan(lib, 0, P, elems, esz, 1, gmax)
            nbytes = elems * esz
            assert 1 <= G <= gmax and piece % 16 == 0 and 8192 <= piece <= piece_max
            # slot s of CTA b for source q at ((s * sg + b) * P + q) * piece:
            # the CTA stride is the communicator's, three rotating slots per
            # CTA and source fit the area
            assert sg == gmax and sg >= G
            assert 3 * sg * P * piece <= area
            if nbytes <= gmax * 8192:
                assert piece == 8192  # one layout for every message up to gmax x 8 KiB
            layouts.add((sg, piece, area))
            # CTA b handles offsets (k*G + b)*piece: every byte is covered
            rounds = -(-nbytes // (G * piece))
            assert rounds * G * piece >= nbytes
            assert G == 1 or (G - 1) * piece < nbytes  # no CTA without a piece
    # the layout depends on the call only through its piece (the host puts a
    # barrier between calls whose pieces differ): a CTA's slots sit at the
    # same place in every call of one piece, so a peer still folding the
    # previous call's last rounds never sees this call's pushes land in the
    # slots it reads
    assert len({(sg, area) for sg, _, area in layouts}) == 1


@pytest.mark.parametrize("gmax", [296, 148])
def test_nvls_shapes(lib, gmax):
    for elems in SIZES:
        blocks, unit, staging = plan(lib, 2, 8, elems, 4, 1, gmax)
        nbytes = elems * 4
        units = -(-nbytes // unit)
        assert 1 <= blocks <= gmax and unit % 65536 == 0 or unit == 16384
        per = -(-units // blocks)
        assert blocks * per >= units and (blocks - 1) * per < units  # covered, no idle CTA
        assert units % blocks == 0 or units < blocks * per  # the last CTAs get one unit less at most
        assert 2 * blocks * unit <= staging
    # 1 GiB of 1 MiB units on 296 CTAs: 256 CTAs of exactly 4 units
    assert plan(lib, 2, 8, 1 << 28, 4, 1, 296)[:2] == [256, 1 << 20]


def _os_slot_block(s, b, sg, P, piece):
    """Bytes of slot s of CTA b for all P sources: [start, end).  This is the
    one-shot kernel's slot_of(e, q) = ((e % 3 * sg + b) * P + q) * piece
    (oneshot_kernel in cail_dev_kernels.cu) taken over q = 0 .. P-1."""
    start = (s * sg + b) * P * piece
    return start, start + P * piece


@pytest.mark.parametrize("P", [2, 4, 8])
def test_one_shot_next_call_never_writes_slots_a_peer_may_still_fold(lib, P):
    """A rank starts pushing its next one-shot call as soon as its own kernel
    has finished, while a peer may still fold the last two rounds of every
    CTA of the previous call.  Over random sequences of message sizes (with
    the per-CTA round counters the kernel keeps), the first pushes of each
    call must land outside every slot the previous call may still read,
    unless the piece changed, in which case the host barrier separates the
    calls."""
    import random

    gmax = 296
    rng = random.Random(P)
    sizes = [1 << k for k in range(10, 25)] + [3000, 100003, 777777, 5 << 20]
    count = [0] * gmax  # completed rounds per CTA, the same on every rank
    prev = None  # (piece, {cta: [slots it may still fold]}, sg)
    checked = 0
    for _ in range(400):
        nbytes = rng.choice(sizes)
        G, piece, area, sg, _ = plan(lib, 0, P, nbytes, 1, 1, gmax)
        rounds = [len(range(b * piece, nbytes, G * piece)) for b in range(G)]
        if prev is not None and prev[0] == piece:
            busy = [_os_slot_block(s, b, prev[2], P, piece) for b, ss in prev[1].items() for s in ss]
            for b in range(G):
                if rounds[b] == 0:
                    continue
                lo, hi = _os_slot_block((count[b] + 1) % 3, b, sg, P, piece)  # round 0 of this call
                assert hi <= area
                for blo, bhi in busy:
                    assert hi <= blo or bhi <= lo, (nbytes, b, (lo, hi), (blo, bhi))
                    checked += 1
        last = {}
        for b in range(G):
            if rounds[b]:
                epochs = [count[b] + rounds[b] - i for i in range(min(2, rounds[b]))]  # last two rounds
                last[b] = [e % 3 for e in epochs]
                count[b] += rounds[b]
        prev = (piece, last, sg)
    assert checked > 1000
