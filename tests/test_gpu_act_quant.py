"""act_quant on the B200 against the reference: bit-exact values and scales (test_kernels.py:21-45,
BASELINE config 0 at full size)."""
import numpy as np
import pytest
import torch

import oracle as O
import deepseek_v32_gtx1650_b200 as D
from deepseek_v32_gtx1650_b200 import workloads
from tests.golden.make_golden import adversarial_groups
from tests.gpu_util import DEV, assert_no_device_error, bf16_from_bits, cuda, f32_of, npy

pytestmark = pytest.mark.gpu
DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@pytest.mark.parametrize("dn", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rs", [0, 1])
def test_act_quant_matches_reference_golden(golden, dn, rs):
    for si in range(int(golden["aq_nshapes"])):
        xg = golden[f"aq_{si}_{dn}_x"]
        x = bf16_from_bits(xg) if dn == "bf16" else cuda(xg)
        y, s = D.act_quant(x, bool(rs))
        assert y.dtype == torch.int8 and y.shape == x.shape and s.shape == (*x.shape[:-1], x.shape[-1] // 128)
        np.testing.assert_array_equal(npy(s), golden[f"aq_{si}_{dn}_r{rs}_s"])
        np.testing.assert_array_equal(npy(y), golden[f"aq_{si}_{dn}_r{rs}_y"])
    assert_no_device_error()


def test_act_quant_zero_and_tiny(golden):
    y, s = D.act_quant(cuda(golden["aq_zero_x"]))
    np.testing.assert_array_equal(npy(y), golden["aq_zero_y"])
    np.testing.assert_array_equal(npy(s), golden["aq_zero_s"])


@pytest.mark.parametrize("rs", [0, 1])
def test_act_quant_adversarial_ue8m0(golden, rs):
    x = cuda(adversarial_groups(golden["aq_adv_amax"]))
    y, s = D.act_quant(x, bool(rs))
    np.testing.assert_array_equal(npy(s), golden[f"aq_adv_r{rs}_s"])
    np.testing.assert_array_equal(npy(y), golden[f"aq_adv_r{rs}_y"])


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rs", [False, True])
def test_act_quant_baseline_config_full_size(dt, rs):
    """[2048, 7168] with outliers and a zero row, both scale formats, bit-exact."""
    x = workloads.act_quant_input(2048, 7168, seed=0).to(dt)
    y, s = D.act_quant(x.to(DEV), rs)
    yr, sr = O.act_quant_ref(f32_of(x), rs)
    np.testing.assert_array_equal(npy(s), sr)
    np.testing.assert_array_equal(npy(y), yr)
    assert_no_device_error()


@pytest.mark.parametrize("shape", [(3, 5, 7, 256), (1, 128), (777, 384), (64, 7168)])
@pytest.mark.parametrize("dt", [torch.float32, torch.float16, torch.bfloat16])
def test_act_quant_odd_shapes(shape, dt):
    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(shape, generator=g) * 3).to(dt)
    x.view(-1)[::97] *= 50
    for rs in (False, True):
        y, s = D.act_quant(x.to(DEV), rs)
        yr, sr = O.act_quant_ref(f32_of(x), rs)
        np.testing.assert_array_equal(npy(s), sr)
        np.testing.assert_array_equal(npy(y), yr)


def test_act_quant_roundtrip_error():
    x = torch.randn(64, 1024, generator=torch.Generator().manual_seed(1)).to(DEV)
    y, s = D.act_quant(x)
    deq = y.float().view(64, 8, 128) * s.unsqueeze(-1)
    assert (deq.view_as(x) - x).abs().max() <= s.max() / 2 + 1e-6  # error at most half a step


def test_act_quant_empty_and_nan():
    y, s = D.act_quant(torch.zeros(0, 256, device=DEV))
    assert y.shape == (0, 256) and s.shape == (0, 2)
    x = torch.randn(2, 256)
    x[1, 3] = float("nan")
    y, s = D.act_quant(x.to(DEV))
    _, sr = O.act_quant_ref(x.numpy())
    assert np.isnan(npy(s)[1, 0]) and np.isnan(sr[1, 0])  # NaN propagates to the group scale like torch.amax
    np.testing.assert_array_equal(npy(s)[0], sr[0])


@pytest.mark.parametrize("dt,n", [(torch.float32, 2048), (torch.bfloat16, 4096), (torch.float16, 4096)])
def test_act_quant_large_input_edge_cases(golden, dt, n):
    """A multi-wave input (every resident warp loops several times) with an odd row count (a ragged
    last iteration), the adversarial ue8m0 groups, outliers, a zero group, NaN and inf."""
    rows = 1031
    g = torch.Generator().manual_seed(n)
    x = torch.randn(rows, n, generator=g) * 2
    x.view(-1)[::97] *= 50
    adv = torch.from_numpy(adversarial_groups(golden["aq_adv_amax"])).float().reshape(-1)
    x.view(-1)[: adv.numel()] = adv[: x.numel()]
    x[5, :128] = 0
    x[7, 300] = float("nan")
    x[9, 1000] = float("inf")
    x[11, 129] = float("-inf")
    x = x.to(dt)
    for rs in (False, True):
        y, s = D.act_quant(x.to(DEV), rs)
        yr, sr = O.act_quant_ref(f32_of(x), rs)
        np.testing.assert_array_equal(npy(s), sr)
        np.testing.assert_array_equal(npy(y), yr)
    assert_no_device_error()


@pytest.mark.parametrize("rs", [True, False])
def test_act_quant_all_ties_large(rs):
    """Every value an exact (ue8m0) or near (fp32 scale) rounding tie, on a multi-wave input: every
    lane takes the exact path for more groups than it remembers, so the warp-wide redo runs too."""
    g = torch.Generator().manual_seed(12)
    n = torch.randint(-127, 127, (2048, 7168), generator=g).float()
    x = (n + 0.5) * 0.125
    x.view(-1, 128)[:, 0] = 127 * 0.125  # amax of every group: ue8m0 scale exactly 2^-3
    y, s = D.act_quant(x.to(DEV), rs)
    yr, sr = O.act_quant_ref(x.numpy(), rs)
    np.testing.assert_array_equal(npy(s), sr)
    np.testing.assert_array_equal(npy(y), yr)
    assert_no_device_error()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rs", [False, True])
def test_act_quant_16bit_ties_and_neighbours(dt, rs):
    """16-bit inputs whose quotients x / s are exact or near rounding ties: each group's values are
    amax * (2k + 1) / 254 rounded to the input type, then moved by -1, 0 or +1 unit in the last
    place, on a multi-wave input with a ragged last iteration (1031 rows)."""
    g = torch.Generator().manual_seed(21)
    rows, n = 1031, 4096
    amax = (torch.rand(rows, n // 128, 1, generator=g) * 8 + 0.01).to(dt).float()
    k = torch.randint(-127, 127, (rows, n // 128, 128), generator=g).float()
    x = (amax * (2 * k + 1) / 254).to(dt)
    nudge = torch.randint(-1, 2, x.shape, generator=g).to(torch.int16)
    x = (x.view(torch.int16) + nudge).view(dt).float()  # one ulp away in magnitude, sign kept
    x[..., 0] = amax[..., 0]
    x = x.to(dt).reshape(rows, n)
    y, s = D.act_quant(x.to(DEV), rs)
    yr, sr = O.act_quant_ref(f32_of(x), rs)
    np.testing.assert_array_equal(npy(s), sr)
    np.testing.assert_array_equal(npy(y), yr)
    assert_no_device_error()
