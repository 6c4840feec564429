"""The CPU oracle against the reference's own forward (golden fixtures), the
reference's own FP8 linear (golden vectors made on a B200) and the
reference's known-answer kernel tests.  CPU only."""
import functools
import hashlib
import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch

from laya_b200.config import LAYA, TINY
from laya_b200.weights import seeded_weights, weights_digest
from oracle import laya_oracle as O

GOLDEN = Path(__file__).parent / "golden"
CONFIGS = {"laya": LAYA, "tiny": TINY}


@functools.lru_cache(maxsize=2)
def oracle_for(name, precision="bf16", bf16_gemm=False):
    cfg = CONFIGS[name]
    w = seeded_weights(cfg, seed=0)
    return O.Oracle(w, cfg, precision, bf16_gemm=bf16_gemm), weights_digest(w)


def load_golden(path):
    z = np.load(path)
    keys = ("input_ids", "attention_mask", "marker_pos", "marker_mask", "qtype")
    return z, {k: z[k] for k in keys}


@pytest.mark.parametrize("bf16_gemm", [False, True], ids=["fp32-restatement", "bf16-gemm"])
@pytest.mark.parametrize("path", sorted(GOLDEN.glob("*.npz")), ids=lambda p: p.stem)
def test_oracle_matches_reference_forward(path, bf16_gemm):
    """Both oracle modes: the fp32-accumulating restatement the parity tests
    use, and the bf16-GEMM mode (the reference's CPU arithmetic) that the
    benchmark's CPU reference arm times."""
    z, inputs = load_golden(path)
    oracle, digest = oracle_for(str(z["config"]), "bf16", bf16_gemm)
    assert str(z["weights_sha256"]) == digest, "seeded weight generator drifted"
    logits, act = oracle.forward(**inputs)
    n = int(z["n_items"])
    ref_l, ref_a = z["ref_logits"][:n], z["ref_act"][:n]
    mm = inputs["marker_mask"][:n]
    # Padded option columns are exactly -1e4 in both.
    assert np.array_equal(logits[:n][~mm], ref_l[~mm])
    np.testing.assert_allclose(logits[:n][mm], ref_l[mm], rtol=0, atol=1e-2)
    np.testing.assert_allclose(act[:n], ref_a, rtol=0, atol=1e-2)
    margins = O.top2_margin(ref_l, mm)
    decided = margins > 2e-2
    assert O.decision_agreement(ref_l[decided], logits[:n][decided], mm[decided]) == 1.0


def _fp8_case_inputs():
    spec = importlib.util.spec_from_file_location("make_fp8_golden", GOLDEN / "make_fp8_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.fp8_case_inputs


@pytest.mark.parametrize("path", sorted((GOLDEN / "fp8_linear").glob("*.npz")), ids=lambda p: p.stem)
def test_fp8_oracle_matches_the_reference_fp8_linear(path):
    """The FP8 oracle against the reference's FP8Linear run on a B200
    (tests/golden/make_fp8_golden.py: Triton _quantize_rows + torch._scaled_mm,
    quantization.py:20-107): activation e4m3 codes and row scales bit-exact,
    weight row scales bit-exact and weight codes identical (digest), and the
    bf16 outputs within one bf16 rounding of the fp32 sums (the reference's
    GEMM accumulates in another order)."""
    z = np.load(path)
    m, n, k = int(z["m"]), int(z["n"]), int(z["k"])
    x, w = _fp8_case_inputs()(m, n, k, int(z["seed"]), str(z["kind"]))
    xq, xs = O.fp8_quantize_rows(x)
    codes = xq.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(codes, z["x_codes"])
    assert np.array_equal(xs[:, 0].numpy(), z["x_scale"])
    wq, ws = O.fp8_quantize_rows(w)
    assert np.array_equal(ws[:, 0].numpy(), z["w_scale"])
    wcodes = wq.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert hashlib.sha256(wcodes.tobytes()).hexdigest() == str(z["w_codes_sha256"])
    y = O.encoder_linear(x, w, "fp8", {}, "case").numpy()
    ref = (z["y"].astype(np.uint32) << 16).view(np.float32)
    exact = (((xq @ wq.T) * xs * ws.T)).numpy()           # fp32 sums before the bf16 rounding
    ulp = np.abs(exact) * 2.0 ** -7 + 1e-30                 # one bf16 step at the value
    assert np.all(np.abs(y - ref) <= ulp), float(np.abs(y - ref).max())
    assert (y == ref).mean() > 0.99


@pytest.mark.parametrize("fp32", [True])
def test_rope_known_answer(fp32):
    """tests/test_kernels.py:32-49: q,k rotate in fp32 then round; v untouched."""
    g = torch.Generator().manual_seed(6)
    x = torch.randn(2, 65, 16, 64, generator=g).bfloat16().float()
    angles = torch.randn(65, 32, generator=g)
    angles = torch.cat((angles, angles), -1)
    cos, sin = angles.cos(), angles.sin()
    got = O.rope(x, cos, sin)
    rotated = torch.cat((-x[..., 32:], x[..., :32]), -1)
    expected = (x * cos[None, :, None] + rotated * sin[None, :, None]).bfloat16().float()
    assert torch.equal(got, expected)


def test_fp8_row_quantizer_semantics():
    """quantization.py:20-29: scale=max(amax/448,1e-12), values clamp(x/scale)."""
    x = torch.tensor([[0.0, 1.0, -2.0, 448.0 * 3], [0.0, 0.0, 0.0, 0.0]])
    q, s = O.fp8_quantize_rows(x)
    assert s[0, 0] == pytest.approx(3.0) and s[1, 0] == pytest.approx(1e-12)
    assert q[0, 3] == 448.0 and torch.all(q[1] == 0)
    assert torch.equal(q, q.to(torch.float8_e4m3fn).float())


def test_e2m1_rounding_grid():
    """cvt.rn.satfinite.e2m1: nearest, ties to the even code, saturate at 6."""
    x = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.26, -100.0, 0.0, 6.0])
    want = torch.tensor([0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, -0.5, -6.0, 0.0, 6.0])
    assert torch.equal(O.e2m1(x), want)


def test_nvfp4_quantize_error_bound():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(64, 256, generator=g) * 0.02
    deq, outer = O.nvfp4_quantize(w, per_row=False)
    rec = deq * outer
    blocks = w.reshape(64, 16, 16).abs().amax(-1, keepdim=True)
    # Each element is within half the widest e2m1 step (1 scale unit ~ block_amax/6, +1/16 for
    # the e4m3 rounding of the scale) of its source value.
    err = (rec - w).reshape(64, 16, 16).abs()
    assert torch.all(err <= blocks / 6.0 * 1.0625 + 1e-7)


def test_fully_masked_query_gives_zero():
    q = torch.randn(1, 1, 3, 64)
    k = torch.randn(1, 1, 4, 64)
    v = torch.randn(1, 1, 4, 64)
    vis = torch.tensor([[True, False, False, False], [False] * 4, [True] * 4])[None, None]
    out = O.attention(q, k, v, vis)
    assert torch.all(out[0, 0, 1] == 0)
    assert torch.allclose(out[0, 0, 0], O.bf16(v[0, 0, 0]))
