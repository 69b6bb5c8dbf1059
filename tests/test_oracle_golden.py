"""Pin the CPU oracle against the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by running the reference ``FusedSparseEngine`` (its gate,
``nonzero_static`` lists, interpreted Triton tile kernel and dense ``F.conv2d`` path)
on CPU.  The oracle must reproduce, bit for bit, every change mask, dilated mask,
mode, active count and budget-padded block list, and the p4/p8 caches within the
dtype's tolerance.
"""
import numpy as np
import pytest

from golden_io import CASES, OUTPUT_ULPS, assert_close, load
from oracle import sparse_oracle as so


def _oracle_for(case):
    m = case["meta"]
    layers = so.fuse_program(case["nodes"])
    return so.OracleEngine(layers, m["n_cams"], m["h"], m["w"], block=m["block"], dtype=case["dtype"],
                           tau=m["tau"], refresh=m["refresh"], outputs=tuple(m["outputs"]))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference(name):
    case = _oracle_for_case = load(name)
    eng = _oracle_for(case)
    assert eng.ds == case["meta"]["ds"]
    assert eng.buckets == case["meta"]["buckets"]
    eng.reset(case["frames0"])
    assert_close(eng.cache["t7"], case["reset"]["t7"], case["dtype"], f"{name} reset t7", OUTPUT_ULPS["t7"])
    assert_close(eng.cache["t14"], case["reset"]["t14"], case["dtype"], f"{name} reset t14", OUTPUT_ULPS["t14"])
    for i, st in enumerate(_oracle_for_case["steps"]):
        eng.extra = st["extra"].astype(bool)
        mode, k = eng.step(st["frames"])
        assert (mode, k) == (st["mode"], st["k"]), f"{name} step {i}"
        np.testing.assert_array_equal(eng.changed, st["changed"], f"{name} step {i} changed")
        for d in eng.ds:
            np.testing.assert_array_equal(eng.masks[d], st["masks"][d], f"{name} step {i} mask d={d}")
        if mode == "sparse":
            assert eng.bucket(k) == st["cap"]
            for d in eng.ds:
                got = np.stack(eng.last_lists[d])
                np.testing.assert_array_equal(got, st["lists"][d], f"{name} step {i} list d={d}")
        assert_close(eng.cache["t7"], st["t7"], case["dtype"], f"{name} step {i} t7", OUTPUT_ULPS["t7"])
        assert_close(eng.cache["t14"], st["t14"], case["dtype"], f"{name} step {i} t14", OUTPUT_ULPS["t14"])


@pytest.mark.parametrize("name", CASES)
def test_exact_gate_sum_agrees_with_fp32_sum(name):
    """On the fixtures, the exact per-block sum and an fp32 sum give the same mask
    (the reference sums in fp32; exact and fp32 sums differ only in a rounding band)."""
    case = load(name)
    m = case["meta"]
    prev = case["frames0"]
    for st in case["steps"]:
        if "changed" not in st:
            continue
        a = so.block_change_sums(st["frames"], prev, m["block"])
        b = so.block_change_sums_fp32(st["frames"], prev, m["block"]).astype(np.float64)
        thr = np.float64(so.threshold(m["tau"], m["block"]))
        assert ((a > thr) == (b > thr)).all()
        # relative gap between the two sums stays inside the fp32 accumulation bound
        assert (np.abs(a - b) <= 3 * m["block"] ** 2 * np.finfo(np.float32).eps * np.abs(a) + 1e-30).all()
        break


def test_list_order_and_padding():
    """nonzero_static: ascending flat order, padded with index 0 (fused_engine.py:163)."""
    mask = np.zeros((2, 3, 4), bool)
    mask[0, 2, 3] = mask[1, 0, 0] = mask[1, 2, 1] = True
    cam, by, bx = so.block_lists(mask, cap=5)
    assert cam.tolist() == [0, 1, 1, 0, 0]
    assert by.tolist() == [2, 0, 2, 0, 0]
    assert bx.tolist() == [3, 0, 1, 0, 0]


def test_dilation_is_maxpool():
    import torch
    import torch.nn.functional as F
    rng = np.random.default_rng(0)
    m = rng.random((3, 7, 9)) < 0.1
    for d in (1, 2, 3):
        ref = F.max_pool2d(torch.from_numpy(m).float()[:, None], 2 * d + 1, 1, d)[:, 0] > 0
        np.testing.assert_array_equal(so.dilate(m, d), ref.numpy())


def test_threshold_is_fp32_of_double_product():
    import torch
    tau = 8 * 255 / float(np.float32(0.229 * 255 + 0.224 * 255 + 0.225 * 255) / 3)
    thr = so.threshold(tau, 32)
    s = torch.tensor([float(thr)], dtype=torch.float32)
    assert not (s > tau * 32 * 32 * 3).item()  # torch compares in fp32: equal, not greater
    assert (torch.nextafter(s, torch.tensor([1e9])) > tau * 32 * 32 * 3).item()


@pytest.mark.parametrize("when", ["reset", "final"])
def test_oracle_every_layer_from_reference_inputs(when):
    """Each oracle layer computed from the reference's own input caches equals the
    reference's output cache elementwise within 1e-2 rel / 1e-3 abs (fp16 fixture with
    every cache kept: dense reset and the last sparse step)."""
    case = load("norm_tau_fp16")
    ref = case[when + "_caches"]
    for l in _oracle_for(case).layers:
        res = None if l.res is None else ref[l.res]
        got = so.conv_dense(ref[l.src], l.w, l.bias, l.stride, l.act, res, np.float16).astype(np.float64)
        exp = ref[l.dst].astype(np.float64)
        bad = np.abs(got - exp) > 1e-3 + 1e-2 * np.abs(exp)
        assert not bad.any(), (when, l.dst, int(bad.sum()))
