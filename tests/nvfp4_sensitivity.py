"""Measurement script (run by hand, not collected by pytest): how far the
NVFP4 oracle's C3 outputs move when the bf16 activations entering every
quantised projection are nudged by one bf16 ulp in a small fraction of their
nonzero elements -- the size of the rounding differences between two correct
implementations of the same forward (reduction orders in LayerNorm and
attention).  The e2m1 grid turns such differences into whole-step code flips,
which sets the scale of the NVFP4 parity tolerance.

    python tests/nvfp4_sensitivity.py
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "laya-inference-engine_b200"))
sys.path.insert(0, str(ROOT))

from laya_b200.config import LAYA  # noqa: E402
from laya_b200.weights import seeded_weights  # noqa: E402
from laya_b200.workload import synthetic_items, pack  # noqa: E402
from oracle import laya_oracle as O  # noqa: E402


def main():
    w = seeded_weights(LAYA, seed=0)
    items = synthetic_items([512], ["choice"], seed=40, vocab=LAYA.vocab)  # the C3 parity case
    inp = pack(items, 1, 512, 4, LAYA.pad_token_id)
    orc = O.Oracle(w, LAYA, "nvfp4")
    base_l, base_a = orc.forward(**inp)
    orig = O.encoder_linear
    mm = inp["marker_mask"]
    for frac, seed in ((0.01, 1), (0.01, 2), (0.05, 3)):
        g = torch.Generator().manual_seed(seed)

        def nudged(x, wt, precision, cache, key, _g=g, _f=frac):
            m = (torch.rand(x.shape, generator=_g) < _f) & (x != 0)
            bits = x.to(torch.bfloat16).view(torch.int16)
            step = torch.where(torch.rand(x.shape, generator=_g) < 0.5, 1, -1).to(torch.int16)
            bits = torch.where(m, bits + step, bits)
            return orig(bits.view(torch.bfloat16).to(torch.float32), wt, precision, cache, key)

        O.encoder_linear = nudged
        try:
            l, a = orc.forward(**inp)
        finally:
            O.encoder_linear = orig
        print(f"nudge {frac:.0%} (seed {seed}): logit max-abs {np.abs(l[mm] - base_l[mm]).max():.3e}, "
              f"act max-abs {np.abs(a - base_a).max():.3e}")


if __name__ == "__main__":
    main()
