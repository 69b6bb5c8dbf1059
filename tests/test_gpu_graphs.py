"""Step graphs: a step replayed from its captured CUDA graph computes exactly what the same
step launched kernel by kernel computes.

Two engines with the same weights run the same sequence, one with step graphs (the
default) and one launching every kernel from the host: sparse, skip and dense steps, the
hysteresis dense steps, a threshold change (which drops the captured graphs), and the
uint8 paths with and without the resize.  Modes, counts, masks and every cache must be
equal bit for bit after every step.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def _same(a, b, what):
    assert torch.equal(a.changed, b.changed), what
    for d in a.ds:
        assert torch.equal(a.masks[d], b.masks[d]), (what, d)
    for name in a.cache:
        assert torch.equal(a.cache[name], b.cache[name]), (what, name)


def test_graph_replay_equals_direct_launches():
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    torch.manual_seed(21)
    n, h, w = 3, 256, 384
    net = LocalBackbone().cuda().eval()
    tau = 8 / float(scenes.STD.mean())
    g = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=tau)
    d = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=tau)
    d.set_step_graphs(False)
    src = scenes.Streams(n, h, w, seed=22, n_rects=2, device="cuda")
    frames = [scenes.normalise(src.next()) for _ in range(6)]
    g.reset(frames[0])
    d.reset(frames[0])
    seen = set()
    # the same frame tensors come back: their captured graphs are replayed
    for i, f in enumerate(frames[1:] + frames[1:] + [frames[-1]]):
        mg, md = g.step(f), d.step(f)
        assert mg == md, (i, mg, md)
        seen.add(mg[0])
        _same(g, d, f"step {i}")
    assert "skip" in seen and "sparse" in seen
    # dense with hysteresis: fallback 0 forces dense, then dense_check_every - 1 steps without a gate
    for e in (g, d):
        e.fallback = 0
    for i, f in enumerate(frames[1:]):
        mg, md = g.step(f), d.step(f)
        assert mg == md, (i, mg, md)
        seen.add(mg[0])
        _same(g, d, f"dense {i}")
    assert "dense" in seen
    for e in (g, d):
        e.fallback = e.n_blocks
        e.set_tau(2 * tau)  # drops g's graphs: the threshold is a kernel argument
    for i, f in enumerate(frames[:3]):
        assert g.step(f) == d.step(f)
        _same(g, d, f"tau {i}")
    # uint8 frames at engine size and at a camera size that needs the resize
    for cam_h in (h, 240):
        s8 = scenes.Streams(n, cam_h, w, seed=23, n_rects=2, device="cuda")
        for i in range(3):
            bgr = s8.next().flip(-1).contiguous()
            assert g.step_u8(bgr, scenes.MEAN, scenes.STD) == d.step_u8(bgr, scenes.MEAN, scenes.STD)
            _same(g, d, f"u8 {cam_h} {i}")
    assert g.launch_count() == d.launch_count()
