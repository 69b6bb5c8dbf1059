"""`sarbon_b200.stem_to_local` against the reference's own BatchNorm folding.

tests/golden/stem/stem_fold.npz was written by make_stem_golden.py from the reference's
`stem_to_local(build("s", 6, halo_zero=False).stem)` (sarbon/sparse/convert.py:14-44) with
deterministic parameters.  A stem of the same layout gets the same parameters here; the
folded weights and biases must be bit-identical (SHA-256 over their float32 bytes) and the
folded network's p4 / p8 equal the reference's on the stored input.
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import torch

from test_host_logic import _Stem

FIXTURE = Path(__file__).resolve().parent / "golden" / "stem" / "stem_fold.npz"


def stem_parameters(modules, seed):
    """The generator's deterministic parameters, in module order (make_stem_golden.py)."""
    rng = np.random.default_rng(seed)
    with torch.no_grad():
        for m in modules:
            if isinstance(m, torch.nn.Conv2d):
                fan = m.in_channels * m.kernel_size[0] * m.kernel_size[1]
                m.weight.copy_(torch.from_numpy(rng.standard_normal(m.weight.shape) * np.sqrt(2.0 / fan)))
                if m.bias is not None:
                    m.bias.copy_(torch.from_numpy(rng.standard_normal(m.bias.shape) * 0.01))
            elif isinstance(m, torch.nn.BatchNorm2d):
                c = m.num_features
                m.running_mean.copy_(torch.from_numpy(rng.uniform(-0.2, 0.2, c)))
                m.running_var.copy_(torch.from_numpy(rng.uniform(0.5, 2.0, c)))
                m.weight.copy_(torch.from_numpy(rng.uniform(0.5, 1.5, c)))
                m.bias.copy_(torch.from_numpy(rng.uniform(-0.2, 0.2, c)))


def test_stem_to_local_matches_reference_fold():
    from sarbon_b200 import stem_to_local
    z = np.load(FIXTURE)
    meta = json.loads(bytes(z["meta_json"]).decode())
    stem = _Stem().eval()
    stem_parameters(list(stem.modules()), meta["seed"])
    local = stem_to_local(stem)
    h = hashlib.sha256()
    for n in local.program()[0]:
        if n.kind == "conv":
            h.update(n.conv.weight.detach().float().contiguous().numpy().tobytes())
            h.update(n.conv.bias.detach().float().contiguous().numpy().tobytes())
    assert h.hexdigest() == meta["folded_sha256"]
    with torch.no_grad():
        p4, p8 = local(torch.from_numpy(z["x"]))
    for got, name in ((p4, "p4"), (p8, "p8")):
        ref = z[name]
        assert np.abs(got.numpy() - ref).max() / np.abs(ref).max() < 1e-6, name
    # and the folded network computes what the unfolded stem computes (fp32)
    assert np.abs(p8.numpy() - z["p8_stem"]).max() / np.abs(z["p8_stem"]).max() < 1e-5
