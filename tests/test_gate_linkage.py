"""CPU: every reference gate built against librocketnpu.so calls OUR entry
points.  Gates that check against the reference's host references link the
reference's compiled sources (oracle/_ref/libref.so) after our library; this
test proves that the only functions left for that library to supply are the
*_ref_* host references (the checkers), so no entry under test can silently
resolve to the reference's own implementation.
"""
import glob
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "rocket-userspace_b200", "librocketnpu.so")
GATES = sorted(glob.glob(os.path.join(REPO, "oracle", "_ref", "gate_*")))


def _nm(args):
    return subprocess.run(["nm"] + args, capture_output=True, text=True, check=True).stdout.split("\n")


@pytest.mark.skipif(not GATES or shutil.which("nm") is None, reason="gates not built")
def test_gate_entries_resolve_to_librocketnpu():
    ours = {ln.split()[-1] for ln in _nm(["-D", "--defined-only", LIB]) if ln.strip()}
    refso = os.path.join(REPO, "oracle", "_ref", "libref.so")
    theirs = ({ln.split()[-1] for ln in _nm(["-D", "--defined-only", refso]) if ln.strip()}
              if os.path.exists(refso) else set())
    bad = {}
    for g in GATES:
        und = {ln.split()[-1] for ln in _nm(["-u", g]) if ln.strip()}
        # any library function the gate calls must be ours, except the reference's
        # host references (*_ref_*), which are the gates' checkers
        missing = sorted(s for s in und if (s.startswith("rocket_") or s in theirs)
                         and s not in ours and "_ref" not in s)
        if missing:
            bad[os.path.basename(g)] = missing
    assert not bad, bad
