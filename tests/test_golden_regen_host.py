"""The committed golden fixtures are what the committed generator makes from the reference:
``tests/golden/make_golden.py`` runs again here (in a subprocess, with its own environment) on
the single-rank blocks, the RMSNorm cases and one gloo EP case, and every array must equal the
committed ``tests/golden/*.npz`` bit for bit. Skipped where the reference source tree is absent
(the fixtures themselves are what travels)."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

REF = Path(os.environ.get("PRISM_REFERENCE", "/root/reference"))
GOLDEN = Path(__file__).resolve().parent / "golden"
pytestmark = pytest.mark.skipif(not (REF / "prism_infer" / "layers" / "moe.py").exists(),
                                reason="the reference's source tree is not available")

DRIVER = """
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
import make_golden as M
MoE, _ = M._import_reference()
torch.manual_seed(0)
out = sys.argv[2]
for case in M.NORM_CASES:
    np.savez(f"{out}/{case[0]}.npz", **M.run_rmsnorm(*case))
for case in M.SINGLE_CASES:
    np.savez(f"{out}/{case[0]}.npz", **M.run_single(MoE, *case))
for case in M.EP_CASES:
    if case[0] == "ep4_tiny":
        np.savez(f"{out}/{case[0]}.npz", **M.run_ep(case))
"""


def test_fixtures_regenerate_bit_for_bit(tmp_path):
    env = dict(os.environ, PRISM_REFERENCE=str(REF))
    r = subprocess.run([sys.executable, "-c", DRIVER, str(GOLDEN), str(tmp_path)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    made = sorted(tmp_path.glob("*.npz"))
    assert len(made) >= 14
    for f in made:
        new, old = np.load(f), np.load(GOLDEN / f.name)
        assert sorted(new.files) == sorted(old.files), f.name
        for key in new.files:
            a, b = new[key], old[key]
            assert a.dtype == b.dtype and a.shape == b.shape, (f.name, key)
            assert np.array_equal(a, b), (f.name, key)
