"""Every selectable tile-conv variant computes the same stem.

The engine runs each layer with its shape's default variant; the measurement switches
SARBON_NO_PAIR=1 (no CTA pairs) and SARBON_WINDOW_MODE=0|3 (per-tap im2col boxes, full
windows) select the other instantiations, which differ in how A tiles are loaded, how the
MMAs are split between CTAs and how the epilogue writes.  For each selection:

* every layer of a dense pass equals a PyTorch fp32 conv of the engine's own input cache
  within the fp16 tolerance (1e-2 rel / 1e-3 abs);
* a sparse step equals a dense pass of the same frames bit for bit (tau = 0: lossless).
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEFAULT_MODES = {}  # block -> layer variants without switches (filled by the first case)

SELECTIONS = [
    {},
    {"SARBON_NO_PAIR": "1"},
    {"SARBON_WINDOW_MODE": "0"},
    {"SARBON_WINDOW_MODE": "3"},
    {"SARBON_NO_PAIR": "1", "SARBON_WINDOW_MODE": "0"},
    {"SARBON_NO_PAIR": "1", "SARBON_WINDOW_MODE": "3"},
]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False


def _check_layers(eng):
    for l in eng.layers:
        x = eng.cache[l.src].float().permute(0, 3, 1, 2)
        w = l.w_tile.to(eng.dtype).float().permute(3, 2, 0, 1).contiguous().cuda()
        ref = F.conv2d(x, w, l.bias.cuda(), l.stride, 1)
        if l.res is not None:
            ref = ref + eng.cache[l.res].float().permute(0, 3, 1, 2)
        if l.act:
            ref = F.relu(ref)
        ref = ref.permute(0, 2, 3, 1)
        got = eng.cache[l.dst].float()
        bad = (got - ref).abs() > 1e-3 + 1e-2 * ref.abs()
        assert not bad.any(), (l.dst, bad.sum().item(), (got - ref).abs().max().item())


@pytest.mark.parametrize("block", [32, 64])
@pytest.mark.parametrize("env", SELECTIONS, ids=lambda e: ",".join(f"{k}={v}" for k, v in e.items()) or "default")
def test_variant_selection(env, block, monkeypatch):
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    for k, v in env.items():
        monkeypatch.setenv(k, v)  # read when an engine picks its layers' variants
    torch.manual_seed(5)
    n, h, w = 2, 384, 640
    net = LocalBackbone().cuda().eval()
    sparse = FusedSparseEngine(net, n, h, w, block=block, dtype=torch.float16)
    dense = FusedSparseEngine(net, n, h, w, block=block, dtype=torch.float16)
    modes = dense.layer_variants()
    default = DEFAULT_MODES.setdefault(block, modes if not env else None)
    if env.get("SARBON_NO_PAIR"):
        assert not any(m & 8 for m in modes), modes
    if env.get("SARBON_WINDOW_MODE"):
        want = int(env["SARBON_WINDOW_MODE"])
        assert any((m & 7) == want for m in modes), modes  # the switch reached some layers
    if env and default is not None and block == 32:  # at block 32 every switch changes some layer
        assert modes != default, (env, modes)
    f0 = (torch.rand(n, h, w, 3, device="cuda") * 4 - 2).half()
    dense.reset(f0)
    torch.cuda.synchronize()
    _check_layers(dense)
    # a sparse step over a few changed blocks equals a dense pass of the same frames
    sparse.reset(f0)
    sparse.fallback = sparse.n_blocks  # never fall back to dense: the sparse kernels must run
    f1 = f0.clone()
    f1[0, 40:90, 100:230] += 0.5
    f1[1, h - 50:, w - 70:] -= 0.25
    mode, k = sparse.step(f1)
    assert mode == "sparse" and k > 0
    dense.reset(f1)
    for name in sparse.cache:
        assert torch.equal(sparse.cache[name], dense.cache[name]), (name, env)
