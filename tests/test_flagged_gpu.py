"""GPU: decode launches of up to 8 tokens on one GPU hand data between CTAs as
tagged 64-bit words instead of meeting at grid barriers; BREAD_NO_FLAGGED=1
forces the grid-barrier path.  For one token both paths do the same arithmetic
in the same order, so the outputs must be bit-identical (for more tokens the
down sums may be grouped differently, see below) -- across a sequence of
launches of different sizes on one stack and back-to-back MoE block calls,
where a word left over from an earlier launch must never be taken for a
current one.  (The oracle parity of the flagged path itself is covered by the
MoE block and stack tests, which run it by default.)"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _run(tmp_path, name, flagged):
    path = str(tmp_path / f"{name}.npz")
    env = dict(os.environ)
    env.pop("BREAD_NO_FLAGGED", None)
    if not flagged:
        env["BREAD_NO_FLAGGED"] = "1"
    r = subprocess.run(["timeout", "-k", "20", "300", sys.executable, os.path.join(HERE, "_flagged_worker.py"), path],
                       capture_output=True, text=True, env=env, timeout=330)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return np.load(path)


def test_flagged_path_equals_barrier_path(cuda, tmp_path):
    a = _run(tmp_path, "flagged", True)
    b = _run(tmp_path, "barrier", False)
    assert int(a["device_error"][0]) == 0 and int(b["device_error"][0]) == 0
    assert sorted(a.files) == sorted(b.files)
    for k in a.files:
        T = int(k.rsplit("_T", 1)[1]) if "_T" in k else 0
        if T == 1 or "idx" in k or k == "device_error":
            assert np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)), k
        else:
            # several tokens: the barrier path keeps the intermediate in the
            # down-ring slots (a shallower ring), so its down rounds group the
            # chunks over the warps differently -- the same fp32 terms summed
            # in another order; each later layer re-quantises its input to
            # int16, where a last-bit difference can cross a rounding boundary
            # (one step = 1/32767 of the group maximum)
            assert np.linalg.norm(a[k] - b[k]) <= 1e-4 * np.linalg.norm(b[k]), k
    # the repeated launches reproduce the first ones (no stale word taken)
    assert np.array_equal(a["small_0_T1"], a["small_4_T1"])
    assert np.array_equal(a["small_1_T3"], a["small_5_T3"])
    assert np.array_equal(a["cfg_0_T1"], a["cfg_3_T1"])
    assert np.array_equal(a["ffn_0_T1"], a["ffn_3_T1"])
