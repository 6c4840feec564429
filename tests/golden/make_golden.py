"""Generate the golden fixtures by running the reference's own forward on CPU.

Run where ``transformers`` and the reference package are importable: the
offline install in ``baseline/_ref``, or the reference's ``src`` directory named
on the command line (or in ``LAYA_REFERENCE_SRC``):

    python tests/golden/make_golden.py [<reference-src-dir> [case names...]]

What it does, per case:
1. builds a Laya-shaped network from ``transformers.ModernBertModel`` and torch
   modules (encoder, 2-layer pre-norm ``nn.TransformerEncoder`` head,
   ``type_emb``, ``scorer``, ``act_head``), loads the seeded weights of
   ``laya_b200.weights`` into it;
2. wraps it in the reference's ``laya_blackwell.model.FastDecisionModel`` with
   the Triton ``rope_qkv`` replaced by its torch restatement from
   ``tests/test_kernels.py:42-49`` (fp32 rotate, bf16 round, V untouched);
3. runs the reference forward on seeded synthetic inputs and stores inputs and
   outputs in ``<name>.npz`` together with the weight digest and versions.

The fixtures hold no weights; tests regenerate them from the seed and check the
digest.  Only inputs and outputs are stored, so the files stay small.
"""
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "laya-inference-engine_b200"))
sys.path.insert(0, str(ROOT))

from laya_b200.config import LAYA, TINY  # noqa: E402
from laya_b200.weights import seeded_weights, weights_digest  # noqa: E402
from laya_b200.workload import synthetic_items, pack  # noqa: E402
from baseline import laya_net  # noqa: E402


# (name, cfg, lengths, kinds, batch, seq, options, seed)
CASES = [
    ("laya_c1_noul_full", LAYA, [64], ["noul"], 1, 64, 2, 0),
    ("laya_c1_noul_pad", LAYA, [37], ["noul"], 1, 64, 2, 1),
    ("laya_mixed_b4_s96", LAYA, [96, 70, 41], ["choice", "score", "noul"], 4, 96, 4, 2),
    ("laya_long_s512", LAYA, [300], ["choice"], 1, 512, 4, 3),
    ("laya_c3_s512_full", LAYA, [512], ["choice"], 1, 512, 4, 40),
    ("laya_c2_b16_s96", LAYA, [96] * 10 + [70, 41, 96, 88, 17, 64],
     ["choice", "noul", "score", "choice", "noul", "score", "choice", "choice", "noul", "score", "choice", "noul",
      "score", "choice", "noul", "score"], 16, 96, 4, 6),
    ("tiny_b3_s160", TINY, [160, 130, 12], ["choice", "noul", "score"], 3, 160, 4, 4),
    ("tiny_b2_s64_full", TINY, [64, 64], ["noul", "choice"], 2, 64, 4, 5),
]


def main():
    if len(sys.argv) > 1:
        os.environ["LAYA_REFERENCE_SRC"] = sys.argv[1]
    if laya_net.reference_src() is None:
        raise SystemExit("usage: make_golden.py [<reference-src-dir>] (or install the reference in baseline/_ref)")
    import transformers
    from oracle.laya_oracle import Oracle
    only = set(sys.argv[2:])

    torch.manual_seed(0)
    nets = {}
    for name, cfg, lengths, kinds, b, s, k, seed in CASES:
        if only and name not in only:
            continue
        key = id(cfg)
        if key not in nets:
            w = seeded_weights(cfg, seed=0)
            model = laya_net.build(cfg, w, "cpu", rope="shim")
            nets[key] = (model, w, weights_digest(w), Oracle(w, cfg))
        model, w, digest, oracle = nets[key]
        items = synthetic_items(lengths, kinds, seed=seed, vocab=cfg.vocab)
        inputs = pack(items, b, s, k, cfg.pad_token_id)
        unmasked = len(items) == b and all(len(it["ids"]) == s for it in items)
        with torch.inference_mode():
            logits, act = model(**{kk: torch.from_numpy(v) for kk, v in inputs.items()},
                                global_attention_unmasked=unmasked)
        logits, act = logits.float().numpy(), act.float().numpy()
        o_logits, o_act = oracle.forward(**inputs)
        n = len(items)
        err = float(np.abs(o_logits[:n] - logits[:n]).max())
        aerr = float(np.abs(o_act[:n] - act[:n]).max())
        print(f"{name}: ref logits {logits[:n].round(4).tolist()} oracle-vs-ref logit {err:.2e} act {aerr:.2e}")
        np.savez_compressed(
            HERE / f"{name}.npz", **inputs, n_items=np.int64(n), unmasked=np.bool_(unmasked),
            ref_logits=logits, ref_act=act, weights_seed=np.int64(0), weights_sha256=np.str_(digest),
            config=np.str_(name.split("_")[0]), torch_version=np.str_(torch.__version__),
            transformers_version=np.str_(transformers.__version__))


if __name__ == "__main__":
    main()
