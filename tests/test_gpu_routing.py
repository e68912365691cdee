"""The decode paths that the library selects by environment, against the golden outputs.

By default a bf16/fp16 unit of <= 32 query rows runs on the narrow tensor-core
kernel and a wider one on the wide kernel, and the decode kernels overlap through
programmatic dependent launch.  Three switches select the other paths:
``MENTAT_TC_MIN_ROWS=16`` sends units of fewer than 16 rows to the FFMA kernel
(the north star's literal routing rule), ``MENTAT_NARROW=0`` sends few-row units
to the wide kernel, and ``MENTAT_PDL=0`` launches the kernels one after another.
The library reads each switch once per process, so every setting runs the golden
attention cases and the sharing-invariance check in a child pytest.
"""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("env", [{"MENTAT_TC_MIN_ROWS": "16"}, {"MENTAT_NARROW": "0"}, {"MENTAT_PDL": "0"}],
                         ids=["ffma_below_16_rows", "no_narrow_kernel", "no_dependent_launch"])
def test_golden_attention_under_each_routing(env):
    e = dict(os.environ)
    e.update(env)
    r = subprocess.run([sys.executable, "-m", "pytest", "tests/test_gpu_attention.py", "-q", "-x", "-p",
                        "no:cacheprovider", "-k", "golden or invariance"],
                       cwd=ROOT, env=e, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
