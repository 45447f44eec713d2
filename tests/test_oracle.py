"""Pin the CPU oracle to the reference: every oracle function against golden vectors produced by the
reference's own reference.py / hadamard_quant.py (tests/golden/make_golden.py). CPU only."""
import numpy as np
import pytest
import torch

import oracle as O
from deepseek_v32_gtx1650_b200 import workloads
from tests.golden.make_golden import adversarial_groups


def _x_f32(golden, key, dn):
    x = golden[key]
    if dn == "bf16":
        return O.bf16_bits_to_f32(x)
    return x.astype(np.float32)  # f32 as is, f16 exactly widened


@pytest.mark.parametrize("dn", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("rs", [0, 1])
def test_act_quant_oracle_matches_reference(golden, dn, rs):
    for si in range(int(golden["aq_nshapes"])):
        x = _x_f32(golden, f"aq_{si}_{dn}_x", dn)
        y, s = O.act_quant_ref(x, bool(rs))
        np.testing.assert_array_equal(s, golden[f"aq_{si}_{dn}_r{rs}_s"])
        np.testing.assert_array_equal(y, golden[f"aq_{si}_{dn}_r{rs}_y"])


def test_act_quant_oracle_zero_tiny(golden):
    y, s = O.act_quant_ref(golden["aq_zero_x"])
    np.testing.assert_array_equal(y, golden["aq_zero_y"])
    np.testing.assert_array_equal(s, golden["aq_zero_s"])
    assert (s[0] == np.float32(1e-4) * np.float32(1.0 / 127.0)).all()  # amax floor


@pytest.mark.parametrize("rs", [0, 1])
def test_act_quant_oracle_adversarial_ue8m0(golden, rs):
    x = adversarial_groups(golden["aq_adv_amax"])
    y, s = O.act_quant_ref(x, bool(rs))
    np.testing.assert_array_equal(s, golden[f"aq_adv_r{rs}_s"])
    np.testing.assert_array_equal(y, golden[f"aq_adv_r{rs}_y"])


def test_ue8m0_rule_differs_from_exact_bits(golden):
    """The adversarial set really exercises torch's log2 rounding: the naive exact-exponent rule
    (smallest power of two >= s) disagrees with the reference on some groups."""
    s0 = golden["aq_adv_r0_s"].astype(np.float64)
    exact = np.ldexp(1.0, np.ceil(np.log2(s0)).astype(np.int64))
    assert (exact != golden["aq_adv_r1_s"].astype(np.float64)).sum() > 0


def test_int8_gemm_oracle_matches_reference(golden):
    for gi in range(int(golden["gm_ncases"])):
        c = O.int8_gemm_ref(golden[f"gm_{gi}_a"], golden[f"gm_{gi}_as"], golden[f"gm_{gi}_b"], golden[f"gm_{gi}_bs"])
        np.testing.assert_allclose(c, golden[f"gm_{gi}_c"], rtol=1e-12, atol=1e-12)
    c = O.int8_gemm_ref(golden["gmb_a"], golden["gmb_as"], golden["gmb_b"], golden["gmb_bs"])
    assert c.shape == golden["gmb_c"].shape
    np.testing.assert_allclose(c, golden["gmb_c"], rtol=1e-12, atol=1e-12)


def test_int8_gemm_partials_sum_to_reference(golden):
    a, a_s, b, b_s = (golden[f"gm_3_{n}"] for n in ("a", "as", "b", "bs"))
    p = O.int8_gemm_partials_ref(a, b)
    KG = a.shape[1] // 128
    bs = np.repeat(b_s, 128, axis=0)
    c = sum(p[kb] * (a_s[:, kb:kb + 1].astype(np.float64) * bs[None, :, kb].astype(np.float64)) for kb in range(KG))
    assert O.rel_err(c, golden["gm_3_c"]) < 1e-13
    assert np.abs(p).max() <= 128 * 127 * 127


def test_int8_index_oracle_matches_reference(golden):
    for ii in range(int(golden["ix_ncases"])):
        B, M, N, H, D, causal, start = golden[f"ix_{ii}_meta"].tolist()
        o = O.int8_index_ref(golden[f"ix_{ii}_q"], golden[f"ix_{ii}_w"], golden[f"ix_{ii}_k"],
                             golden[f"ix_{ii}_ks"], causal=bool(causal), start=start)
        ref = golden[f"ix_{ii}_o"]
        np.testing.assert_array_equal(np.isinf(o), np.isinf(ref))
        assert O.rel_err(o, ref) < 1e-12


def test_int8_index_oracle_row_subset(golden):
    q, w, k, ks = (golden[f"ix_5_{n}"] for n in ("q", "w", "k", "ks"))
    B, M, N, H, D, causal, start = golden["ix_5_meta"].tolist()
    rows = np.array([0, 7, M - 1])
    o = O.int8_index_ref(q, w, k, ks, causal=True, start=start, rows=rows)
    ref = golden["ix_5_o"][:, rows]
    np.testing.assert_array_equal(np.isinf(o), np.isinf(ref))
    assert O.rel_err(o, ref) < 1e-12


def test_rotate_quant_oracle_matches_reference(golden):
    q, s = O.rotate_quant_ref(golden["rq_x"])
    np.testing.assert_array_equal(q, golden["rq_q"])
    np.testing.assert_array_equal(s, golden["rq_s"])
    qn, sn = O.rotate_quant_ref(golden["rq_x"], rotate=False)
    np.testing.assert_array_equal(qn, golden["rq_norot_q"])
    np.testing.assert_allclose(O.hadamard_matrix(128), golden["rq_h"], rtol=0, atol=1e-7)


def test_workload_rotation_matches_reference_producer(golden):
    """The bench/test input generator uses the reference's rotate+quantise semantics."""
    q, s = workloads.rotate_quant(torch.from_numpy(golden["rq_x"]))
    np.testing.assert_array_equal(q.numpy(), golden["rq_q"])
    np.testing.assert_array_equal(s.numpy(), golden["rq_s"])


def test_topk_oracle_is_a_valid_torch_topk(golden):
    sc, k = golden["tk_scores"], golden["tk_idx"].shape[-1]
    idx, vals = O.topk_ref(sc, k)
    assert O.topk_valid(idx, sc, k)
    assert O.topk_valid(golden["tk_idx"], sc, k)  # torch.topk's own choice passes the same check
    # Same multiset of values as torch.topk (ties may pick different positions).
    np.testing.assert_array_equal(np.sort(vals, -1), np.sort(golden["tk_vals"], -1))
    assert (np.diff(idx, axis=-1) > 0).all()  # increasing position order


def test_topk_valid_rejects_wrong_sets(golden):
    sc, k = golden["tk_scores"], 120
    idx, _ = O.topk_ref(sc, k)
    bad = idx.copy()
    row = 0
    worst = np.argmin(sc[row])  # swap in the smallest element of the row
    if worst not in bad[row]:
        bad[row, 0] = worst
        assert not O.topk_valid(bad, sc, k)
    dup = idx.copy()
    dup[1, 1] = dup[1, 0]
    assert not O.topk_valid(dup, sc, k)


def test_rel_err_definition():
    ref = np.array([1.0, -2.0, np.inf, 4.0])
    x = np.array([1.0, -2.0, 5.0, 4.004])
    assert abs(O.rel_err(x, ref) - 0.001) < 1e-12


def test_weight_quant_oracle_matches_reference_expressions(golden):
    """weight_quant_ref against the reference's own block-quantisation expressions
    (test_kernels.py:80-82, bench.py:43-44), evaluated in torch by make_golden.py."""
    for wi in range(int(golden["wq_ncases"])):
        q, s = O.weight_quant_ref(golden[f"wq_{wi}_w"])
        np.testing.assert_array_equal(s, golden[f"wq_{wi}_s"])
        np.testing.assert_array_equal(q, golden[f"wq_{wi}_q"])


# ---------------------------------------------------------------- torch-on-CPU baselines
def test_torch_baselines_match_reference(golden):
    """oracle/reference_torch.py restates the reference's eager CPU paths (reference.py:8-82) that
    bench.py times as the CPU baseline: act_quant_torch is bit-exact against the reference's golden
    vectors; gemm_dequant_fp32 and the two eager indexers agree with the float64 goldens to fp32
    accuracy; int_mm_unscaled is the exact unscaled integer product."""
    from oracle import reference_torch as RT
    for si in range(int(golden["aq_nshapes"])):
        for rs in (0, 1):
            x = torch.from_numpy(golden[f"aq_{si}_f32_x"])
            y, s = RT.act_quant_torch(x, bool(rs))
            np.testing.assert_array_equal(y.numpy(), golden[f"aq_{si}_f32_r{rs}_y"])
            np.testing.assert_array_equal(s.numpy(), golden[f"aq_{si}_f32_r{rs}_s"])
    for gi in range(int(golden["gm_ncases"])):
        a, a_s, b, b_s = (torch.from_numpy(golden[f"gm_{gi}_{n}"]) for n in ("a", "as", "b", "bs"))
        c = RT.gemm_dequant_fp32(a, a_s, RT.dequant_weight(b, b_s))
        assert O.rel_err(c.double().numpy(), golden[f"gm_{gi}_c"]) < 1e-5
    a, b = torch.from_numpy(golden["gm_3_a"]), torch.from_numpy(golden["gm_3_b"])
    if a.shape[0] > 16:  # torch._int_mm wants m > 16 on CPU
        p = RT.int_mm_unscaled(a, b.T.contiguous()).numpy().astype(np.int64)
        np.testing.assert_array_equal(p, O.int8_gemm_partials_ref(a.numpy(), b.numpy()).sum(0))
    for ii in range(int(golden["ix_ncases"])):
        B, M, N, H, D, causal, start = golden[f"ix_{ii}_meta"].tolist()
        if causal:
            continue  # the reference's eager baselines score every key
        q, w, k, ks = (torch.from_numpy(golden[f"ix_{ii}_{n}"]) for n in ("q", "w", "k", "ks"))
        ref = golden[f"ix_{ii}_o"]
        assert O.rel_err(RT.index_torch_fp32(q, w, k, ks).double().numpy(), ref) < 1e-5
        if M * H > 16:
            assert O.rel_err(RT.index_torch_int8(q, w, k, ks).double().numpy(), ref) < 1e-5
