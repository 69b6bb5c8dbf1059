"""Golden values of the reference's BatchNorm folding (sarbon/sparse/convert.py, stem_to_local).

Run once with the reference checkout (its path is the first, required argument).  The
reference stem `build("s", 6, halo_zero=False).stem` gets deterministic parameters (numpy
PCG64: conv weights kaiming-scaled, BatchNorm statistics and affine parameters in the ranges
the reference's own pipeline test draws, tests/test_pipeline.py:20-27) in module order; the
reference's `stem_to_local` folds it.  Written: the SHA-256 of every folded weight and bias
(float32 bytes, in LocalBackbone program order) and the folded network's p4 / p8 for a small
seeded input.  The test gives the same parameters to a stem of the same layout and checks
`sarbon_b200.stem_to_local` against these, without the reference.

Usage: python tests/golden/make_stem_golden.py /path/to/reference
"""
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "stem"
if len(sys.argv) < 2:
    sys.exit("usage: make_stem_golden.py /path/to/reference")
sys.path.insert(0, sys.argv[1])
from sarbon.models.sarbon_det import build  # noqa: E402
from sarbon.sparse.convert import stem_to_local  # noqa: E402

SEED = 23


def stem_parameters(modules, seed=SEED):
    """Deterministic parameters for the convs and BatchNorms of a stem, in module order."""
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


def digest(net):
    h = hashlib.sha256()
    for n in net.program()[0]:
        if n.kind == "conv":
            h.update(n.conv.weight.detach().float().contiguous().numpy().tobytes())
            h.update(n.conv.bias.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def main():
    torch.manual_seed(0)
    stem = build("s", 6, halo_zero=False).stem.eval()
    stem_parameters(list(stem.modules()))
    local = stem_to_local(stem)
    x = torch.from_numpy(np.random.default_rng(SEED + 1).standard_normal((1, 3, 64, 96)).astype(np.float32))
    with torch.no_grad():
        p4, p8 = local(x)
        _, p8_stem = stem.forward_blocks(x)
    OUT.mkdir(exist_ok=True)
    np.savez_compressed(OUT / "stem_fold.npz", x=x.numpy(), p4=p4.numpy(), p8=p8.numpy(), p8_stem=p8_stem.numpy(),
                        meta_json=np.frombuffer(json.dumps({"seed": SEED, "folded_sha256": digest(local)}).encode(),
                                                np.uint8))
    print("wrote stem/stem_fold.npz", digest(local))


if __name__ == "__main__":
    main()
