"""The reference-side registration of INTEGRATION.md section 2, run on the reference's own engine
(``tests/reference_integration_check.py``, in a subprocess so that its accelerate stand-in and the
reference's modules stay out of this process).  Needs the reference's source tree; skipped where
it is absent."""
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import reference_harness  # noqa: E402


@pytest.mark.skipif(not reference_harness.reference_available(),
                    reason="the reference's source tree is not on this machine")
def test_reference_engine_places_rw4_through_the_registered_backend(tmp_path):
    r = subprocess.run([sys.executable, os.path.join(HERE, "reference_integration_check.py")],
                       cwd=str(tmp_path), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]
