"""The reference M0 fixture (tests/golden/m0/m0_fp32.npz) decodes and covers the cases its
GPU test relies on: steps within the capacity, a step over it, and steps without change."""
import json
from pathlib import Path

import numpy as np

from golden_io import conv_specs, golden_weights, weights_digest

FIXTURE = Path(__file__).resolve().parent / "golden" / "m0" / "m0_fp32.npz"


def test_m0_fixture_decodes():
    z = np.load(FIXTURE)
    meta = json.loads(bytes(z["meta_json"]).decode())
    assert weights_digest(golden_weights(conv_specs(meta["nodes"]), meta["seed"])) == meta["weights_sha256"]
    overs = [s["over"] for s in meta["steps"]]
    assert True in overs and False in overs
    assert any(s["changed"] == 0 for s in meta["steps"])
    t14 = z["full_t14"]
    for i, s in enumerate(meta["steps"]):
        assert z[f"step{i}_frame"].dtype == np.uint8
        assert int(z[f"step{i}_changed"].sum()) == s["changed"]
        t14 = (t14.view(np.uint32) ^ z[f"step{i}_t14_x"]).view(np.float32)
        assert np.isfinite(t14).all()
