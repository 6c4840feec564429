"""Golden vectors of the reference's own FP8 linear, for pinning the FP8 oracle.

Runs the reference's ``FP8Linear`` (``src/laya_blackwell/quantization.py:32-107``:
per-output-row e4m3 weight packing, the Triton ``_quantize_rows`` kernel for
the dynamic per-row activation scales, ``torch._scaled_mm`` with fp32
accumulation and bf16 output) on a Blackwell GPU, on seeded bf16 activations
and weights of Laya projection shapes (at least 64 rows, as FP8Linear
requires), and stores what it produced:

* ``x_codes`` / ``x_scale``: the activation e4m3 codes and row scales that
  ``_quantize_rows`` wrote (called exactly as ``FP8Linear.forward`` calls it);
* ``w_scale`` and ``w_codes_sha256``: the packed weight's row scales and a
  digest of its e4m3 bytes;
* ``y``: the layer's bf16 output (bit patterns).

Inputs are regenerated from ``seed`` by ``fp8_case_inputs`` (numpy PCG64, then
rounded to bf16), so the fixtures hold no inputs.  Needs CUDA, triton and the
reference package (``baseline/_ref`` or ``LAYA_REFERENCE_SRC``):

    python tests/golden/make_fp8_golden.py <output-dir>
"""
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

# name, rows M, features N, reduction K, seed, activation kind
CASES = [
    ("fp8_linear_qkv_m64", 64, 256, 1024, 11, "norm"),
    ("fp8_linear_wo2_m96", 96, 128, 2624, 12, "geglu"),
]


def fp8_case_inputs(m, n, k, seed, kind):
    """Seeded bf16 activations x [m][k] and weights w [n][k] (fp32 tensors of
    bf16 values).  `norm` activations look like LayerNorm outputs, `geglu` like
    GEGLU outputs (heavy tails); row 0 is all zero (scale floor) and row 1
    carries one large outlier (saturating scale)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if kind == "norm":
        x = rng.standard_normal((m, k)).astype(np.float32)
    else:
        a = rng.standard_normal((m, k)).astype(np.float32)
        g = rng.standard_normal((m, k)).astype(np.float32)
        x = a * 0.5 * (1.0 + np.tanh(0.7978845608 * (a + 0.044715 * a ** 3))) * g
    x[0] = 0.0
    x[1, 7] = 300.0
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    to_bf16 = lambda v: torch.from_numpy(v).bfloat16().float()  # noqa: E731
    return to_bf16(x), to_bf16(w)


def main():
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "fp8_linear"
    out.mkdir(parents=True, exist_ok=True)
    from baseline import laya_net
    quant = laya_net.import_reference("quantization")
    import triton
    dev = torch.device("cuda", 0)
    for name, m, n, k, seed, kind in CASES:
        x, w = fp8_case_inputs(m, n, k, seed, kind)
        lin = torch.nn.Linear(k, n, bias=False).to(dev).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(w.to(dev).bfloat16())
        layer = quant.FP8Linear.from_linear(lin)
        xb = x.to(dev).bfloat16()
        with torch.inference_mode():
            y = layer(xb)
            q = torch.empty_like(xb, dtype=torch.float8_e4m3fn)
            s = torch.empty((m, 1), device=dev, dtype=torch.float32)
            block = triton.next_power_of_2(k)
            quant._quantize_rows[(m,)](xb, q, s, k, block, num_warps=4 if block <= 2048 else 8)
        torch.cuda.synchronize()
        wcodes = layer.weight.view(torch.uint8).cpu().numpy()
        np.savez_compressed(
            out / f"{name}.npz", m=np.int64(m), n=np.int64(n), k=np.int64(k), seed=np.int64(seed),
            kind=np.str_(kind), y=y.view(torch.int16).cpu().numpy().view(np.uint16),
            x_codes=q.view(torch.uint8).cpu().numpy(), x_scale=s.cpu().numpy()[:, 0],
            w_scale=layer.weight_scale.float().cpu().numpy()[0],
            w_codes_sha256=np.str_(hashlib.sha256(wcodes.tobytes()).hexdigest()),
            device=np.str_(torch.cuda.get_device_name(dev)), torch_version=np.str_(torch.__version__),
            triton_version=np.str_(triton.__version__))
        print(f"{name}: y[0,:4]={y[2, :4].float().tolist()} x_scale[:3]={s[:3, 0].tolist()}")


if __name__ == "__main__":
    main()
