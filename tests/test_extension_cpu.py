"""The compiled extension on the CPU host: load, link and error reporting (no kernel launches)."""
import subprocess
import sys

import pytest

from predicitivecoding_b200 import ops

pytestmark = pytest.mark.skipif(not ops.available(), reason="extension not built")


def test_status_error_raises_value_error_with_code():
    # A failing launcher status must surface as a Python exception whose message carries the numbers;
    # run in a child so a crash of the C++ runtime fails the test instead of the test session.
    code = ("from predicitivecoding_b200 import ops\n"
            "try:\n    ops.ext()._check_status(-3)\nexcept ValueError as e:\n    print('OK', e)\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "OK pcb kernel 'status probe' failed with code -3" in r.stdout


def test_status_zero_is_silent():
    ops.ext()._check_status(0)


def test_extension_links_shared_cxx_runtime():
    import re
    path = ops.ext().__file__
    out = subprocess.run(["readelf", "-d", path], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("readelf not available")
    assert re.search(r"NEEDED.*libstdc\+\+\.so", out.stdout), "extension must not embed a static libstdc++"
