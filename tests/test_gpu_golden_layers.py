"""Every tile-conv layer against the reference's own layer outputs, from the reference's
own inputs.

The ``norm_tau_fp16`` fixture holds every cache the reference ``FusedSparseEngine`` had
after its dense reset (cuDNN-path ``F.conv2d``) and after its last sparse step (the
interpreted Triton tile kernel for the active tiles) on normalised fp16 camera frames at
SarbonVideo's threshold.  Each layer of the B200 engine is run alone
(``FusedSparseEngine.dense_layers``) on the reference's input caches and compared,
element by element, with the reference's output cache: 1e-2 relative / 1e-3 absolute,
the fp16 tolerance, with no allowance for depth (one fp32 accumulation and one fp16
rounding on each side).
"""
import numpy as np
import pytest
import torch

from golden_io import load

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def _net(nodes):
    from sarbon_b200 import LocalBackbone
    net = LocalBackbone()
    convs = [n.conv for n in net.program()[0] if n.kind == "conv"]
    with torch.no_grad():
        for c, (w, b) in zip(convs, [(n["w"], n["b"]) for n in nodes if n["kind"] == "conv"]):
            c.weight.copy_(torch.from_numpy(w))
            c.bias.copy_(torch.from_numpy(b))
    return net.eval()


@pytest.mark.parametrize("when", ["reset", "final"])
def test_every_layer_from_reference_inputs(when):
    from sarbon_b200 import FusedSparseEngine
    case = load("norm_tau_fp16")
    m = case["meta"]
    ref = case[when + "_caches"]
    eng = FusedSparseEngine(_net(case["nodes"]).cuda(), m["n_cams"], m["h"], m["w"], block=m["block"],
                            dtype=torch.float16, tau=m["tau"], refresh=m["refresh"])
    assert set(ref) == set(eng.cache)
    for name, v in ref.items():
        eng.cache[name].copy_(torch.from_numpy(v).cuda())
    worst = {}
    for i, l in enumerate(eng.layers):
        eng.dense_layers(i)
        got = eng.cache[l.dst].float().cpu().numpy().astype(np.float64)
        exp = ref[l.dst].astype(np.float64)
        err = np.abs(got - exp)
        bound = 1e-3 + 1e-2 * np.abs(exp)
        worst[l.dst] = float((err / bound).max())
        assert (err <= bound).all(), (when, l.dst, int((err > bound).sum()), float(err.max()))
        # the next layer reads the reference's own output, not this one
        eng.cache[l.dst].copy_(torch.from_numpy(ref[l.dst]).cuda())
    print(f"\n{when}: worst err / (1e-3 + 1e-2|ref|) per layer {worst}")
