"""The NVLS kernel's copier loop, compiled as host code (cail_copier_check).

The copier warps copy a unit out of a staging slot and then refill the slot
with the unit after next, with no barrier in between; that is correct only
if each slot byte is copied out and refilled by the same thread.  The check
runs the loop's threads one after another in several orders, for float and
double, whole and ragged units, and user buffers on or off a 16-byte
boundary.
"""
import os
import subprocess

from conftest import BIN, ensure_build


def test_copier_loop_gives_each_slot_chunk_one_thread():
    ensure_build()
    r = subprocess.run([os.path.join(BIN, "cail_copier_check")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "COPIER OK" in r.stdout, r.stdout
