"""Generate the golden vectors that pin the CPU oracle to the reference's own code.

Run once, in a container that has the reference checkout (read-only) at REFERENCE_DIR:

    python tests/golden/make_golden.py [/path/to/deepseek-v32-gtx1650]

It imports the reference's reference.py (act_quant_ref, int8_gemm_ref, int8_index_ref) and
hadamard_quant.py (rotate_quant_ref), evaluates them on CPU over the cases of the reference's
test suite (test_kernels.py:21-126, test_hadamard.py) plus adversarial ue8m0 scales, and writes
golden.npz next to this file. Inputs are stored with the outputs, so the fixtures do not depend
on any RNG. The GPU box never runs this script; tests read golden.npz.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "golden.npz")


def _t2n(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def adversarial_groups(amax: np.ndarray) -> np.ndarray:
    """One 128-group per amax: [amax, amax * linspace(-0.9, 0.9, 127)] in float32 (deterministic)."""
    pattern = np.linspace(-0.9, 0.9, 127, dtype=np.float32)
    return np.concatenate([amax[:, None], amax[:, None] * pattern[None, :]], axis=1).astype(np.float32)


def main(ref_dir: str) -> None:
    sys.path.insert(0, ref_dir)
    import reference as R  # noqa: E402  (the reference's own oracle)
    import hadamard_quant as HQ  # noqa: E402  (imports triton; only rotate_quant_ref is used, on CPU)

    torch.manual_seed(0)
    out: dict[str, np.ndarray] = {}
    dtypes = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}

    # ---- act_quant: test_kernels.py:21-31 cases (reduced largest shape) ---------------------
    shapes = [(1, 128), (7, 256), (33, 512), (4, 5, 384), (16, 1024)]
    for si, shape in enumerate(shapes):
        base = torch.randn(shape) * 3
        base.view(-1)[::97] *= 50
        for dn, dt in dtypes.items():
            x = base.to(dt)
            out[f"aq_{si}_{dn}_x"] = _t2n(x)
            for rs in (0, 1):
                y, s = R.act_quant_ref(x, bool(rs))
                out[f"aq_{si}_{dn}_r{rs}_y"] = y.numpy()
                out[f"aq_{si}_{dn}_r{rs}_s"] = s.numpy()
    out["aq_nshapes"] = np.array(len(shapes))
    # zero / tiny rows (test_kernels.py:34-38)
    x = torch.zeros(4, 256)
    x[1] = 1e-9
    x[2, :5] = -7.0
    y, s = R.act_quant_ref(x)
    out["aq_zero_x"], out["aq_zero_y"], out["aq_zero_s"] = x.numpy(), y.numpy(), s.numpy()
    # adversarial ue8m0: group amax placed so that s = amax/127 lands a few ulps around 2^e
    amaxes = []
    for e in range(-16, 17):
        a0 = np.float32(127.0 * 2.0 ** e)
        for d in range(-6, 34):
            a = np.float32(a0)
            step = np.float32(np.inf) if d > 0 else np.float32(-np.inf)
            for _ in range(abs(d)):
                a = np.nextafter(a, step, dtype=np.float32)
            amaxes.append(a)
    amax = np.array(amaxes, dtype=np.float32)
    xa = torch.from_numpy(adversarial_groups(amax))  # [G, 128]
    for rs in (0, 1):
        y, s = R.act_quant_ref(xa, bool(rs))
        out[f"aq_adv_r{rs}_y"], out[f"aq_adv_r{rs}_s"] = y.numpy(), s.numpy()
    out["aq_adv_amax"] = amax

    # ---- int8_gemm: make_gemm distribution (test_kernels.py:49-54) ----------------------------
    gemm_cases = [(1, 128, 128), (5, 256, 384), (37, 384, 256), (64, 256, 512)]
    for gi, (M, N, K) in enumerate(gemm_cases):
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8)
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8)
        a_s = torch.rand(M, K // 128) * 0.01 + 1e-4
        b_s = torch.rand(N // 128, K // 128) * 0.01 + 1e-4
        out.update({f"gm_{gi}_a": a.numpy(), f"gm_{gi}_as": a_s.numpy(), f"gm_{gi}_b": b.numpy(),
                    f"gm_{gi}_bs": b_s.numpy(), f"gm_{gi}_c": R.int8_gemm_ref(a, a_s, b, b_s).numpy()})
    out["gm_ncases"] = np.array(len(gemm_cases))
    # batched leading dims (test_kernels.py:67-73)
    a = torch.randint(-127, 128, (2, 3, 16, 256), dtype=torch.int8)
    a_s = torch.rand(2, 3, 16, 2) * 0.01 + 1e-4
    b = torch.randint(-127, 128, (256, 256), dtype=torch.int8)
    b_s = torch.rand(2, 2) * 0.01 + 1e-4
    out.update({"gmb_a": a.numpy(), "gmb_as": a_s.numpy(), "gmb_b": b.numpy(), "gmb_bs": b_s.numpy(),
                "gmb_c": R.int8_gemm_ref(a, a_s, b, b_s).numpy()})

    # ---- int8_index: make_index distribution (test_kernels.py:90-118) -----------------------
    idx_cases = [  # (B, M, N, H, D, causal, start)
        (1, 1, 128, 64, 128, 0, 0), (2, 3, 257, 64, 128, 0, 0), (1, 5, 300, 64, 128, 0, 0),
        (1, 24, 24, 64, 128, 1, 0), (1, 16, 200, 64, 128, 1, 84), (1, 17, 160, 64, 128, 1, 50),
        (1, 8, 256, 16, 64, 0, 0),
    ]
    for ii, (B, M, N, H, D, causal, start) in enumerate(idx_cases):
        q = torch.randint(-127, 128, (B, M, H, D), dtype=torch.int8)
        k = torch.randint(-127, 128, (B, N, D), dtype=torch.int8)
        w = torch.randn(B, M, H) * 1e-4
        k_s = torch.rand(B, N) * 0.01
        o = R.int8_index_ref(q, w, k, k_s, causal=bool(causal), start=start)
        out.update({f"ix_{ii}_q": q.numpy(), f"ix_{ii}_w": w.numpy(), f"ix_{ii}_k": k.numpy(),
                    f"ix_{ii}_ks": k_s.numpy(), f"ix_{ii}_o": o.numpy(),
                    f"ix_{ii}_meta": np.array([B, M, N, H, D, causal, start])})
    out["ix_ncases"] = np.array(len(idx_cases))

    # ---- rotate_quant_ref (hadamard_quant.py:106-110), the indexer's input producer -----------
    xr = torch.randn(2, 50, 128)
    xr[..., :4] *= 20
    qr, sr = HQ.rotate_quant_ref(xr)
    out["rq_x"], out["rq_q"], out["rq_s"] = xr.numpy(), qr.numpy(), sr.numpy()
    qn, sn = HQ.rotate_quant_ref(xr, rotate=False)
    out["rq_norot_q"], out["rq_norot_s"] = qn.numpy(), sn.numpy()
    out["rq_h"] = HQ.hadamard_matrix(device="cpu").numpy()

    # ---- top-k: torch.topk on scores with ties and -inf (test_kernels.py:121-126) -------------
    sc = torch.randint(0, 50, (6, 300)).float()  # many ties
    sc[3, 100:] = float("-inf")  # fewer finite values than k in this row
    vals, inds = torch.topk(sc, 120, dim=-1)
    out["tk_scores"], out["tk_vals"], out["tk_idx"] = sc.numpy(), vals.numpy(), inds.numpy()

    # ---- weight block quantiser: the expressions of test_kernels.py:80-82 / bench.py:43-44 ------
    g = torch.Generator().manual_seed(80)
    for wi, (N, K) in enumerate([(256, 384), (128, 1024)]):
        W = torch.randn(N, K, generator=g) * 0.02
        W[5, 7] = 3.0  # one outlier block
        W[:128, 128:256] = 0  # an all-zero block: the 1e-4 floor
        Wb = W.view(N // 128, 128, K // 128, 128)
        ws = (Wb.abs().amax((1, 3)).clamp_min(1e-4) / 127)
        Wq = torch.round(Wb / ws[:, None, :, None]).clamp(-127, 127).to(torch.int8).view(N, K)
        out[f"wq_{wi}_w"], out[f"wq_{wi}_q"], out[f"wq_{wi}_s"] = W.numpy(), Wq.numpy(), ws.numpy()
    out["wq_ncases"] = np.array(2)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({os.path.getsize(OUT) / 1e6:.2f} MB, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
