"""The reference's own test suite, unmodified, against bin/cpde_server.

The reference's tests select the server executable through the environment
variable CPDE_TEST_EXECUTABLE (tests/test_interface.py:18-20 of the
reference) and drive it through the reference's unmodified Python front end
(package `cpde`). `make -C oracle suite` installs that package with pip into
baseline/_ref and copies the reference's tests and examples beside it; this
test runs them, as a child pytest process, with CPDE_TEST_EXECUTABLE pointing
at this repository's drop-in server. Every file below must pass: interface
and wire semantics (rejections with the reference's messages, session
recovery, stop and resume, snapshots), exact RPROP semantics, integrals,
multi-chunk cost reductions and gradient reports, and the examples' mathematics.

Not run: tests/test_cost_schedule.py and tests/test_reductions.py compile
and run the reference's own instrumented probes (a server with a forward
counter, the reduction kernels), not the server under test, and
tests/test_cpu_backend.py covers the front end's choice of a CPU executable.
B200 only (the server runs the CUDA engine).
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

from cpde_b200 import native

pytestmark = pytest.mark.gpu

SUITE = Path(__file__).resolve().parents[1] / 'baseline' / '_ref'
FILES = ['test_interface.py', 'test_rprop.py', 'test_integrals.py', 'test_audit_fixes.py',
         'test_examples.py', 'test_example_variants.py', 'test_circle_example.py', 'test_circle_projection.py']


@pytest.mark.skipif(not (SUITE / 'cpde' / 'api.py').exists(),
                    reason='reference front end not installed (make -C oracle suite)')
def test_reference_suite_against_drop_in_server():
    assert native.SERVER.exists(), 'bin/cpde_server is not built'
    env = dict(os.environ, CPDE_TEST_EXECUTABLE=str(native.SERVER),
               PYTHONPATH=os.pathsep.join([str(SUITE), str(SUITE / 'reference_tests')]))
    files = [str(SUITE / 'reference_tests' / f) for f in FILES]
    run = subprocess.run([sys.executable, '-m', 'pytest', '-q', '-p', 'no:cacheprovider', '--rootdir', str(SUITE),
                          *files], cwd=SUITE, env=env, capture_output=True, text=True, timeout=1500)
    assert run.returncode == 0, run.stdout[-6000:] + run.stderr[-2000:]
