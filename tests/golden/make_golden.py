"""Generate the golden fixtures by running the reference's own forward on CPU.

Run where the reference sources and ``transformers`` are importable, naming
the reference's ``src`` directory (the one holding ``laya_blackwell``):

    python tests/golden/make_golden.py <reference-src-dir>

(or set ``LAYA_REFERENCE_SRC`` to it).

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
from torch import nn

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "laya-inference-engine_b200"))
sys.path.insert(0, str(ROOT))

from laya_b200.config import LAYA, TINY  # noqa: E402
from laya_b200.weights import seeded_weights, as_float32, weights_digest  # noqa: E402
from laya_b200.workload import synthetic_items, pack  # noqa: E402


def torch_rope(qkv, cos, sin, *, fp32=False):
    """tests/test_kernels.py:42-49 restated: rotate-half on q,k; v passthrough."""
    length = qkv.shape[1]
    cos, sin = cos[:length], sin[:length]
    qk = qkv[:, :, :2]
    if fp32:
        qk = qk.float()
    else:
        cos, sin = cos.bfloat16(), sin.bfloat16()
    half = qk.shape[-1] // 2
    rotated = torch.cat((-qk[..., half:], qk[..., :half]), -1)
    out = qk * cos[None, :, None, None] + rotated * sin[None, :, None, None]
    return torch.cat((out.bfloat16(), qkv[:, :, 2:]), dim=2)


class LayaNet(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        from transformers import ModernBertConfig, ModernBertModel
        ec = ModernBertConfig(
            vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
            num_hidden_layers=cfg.layers, num_attention_heads=cfg.heads,
            local_attention=cfg.local_attention, global_attn_every_n_layers=cfg.global_every,
            norm_eps=cfg.norm_eps, norm_bias=False, mlp_bias=False, attention_bias=False,
            pad_token_id=cfg.pad_token_id, hidden_activation="gelu",
            max_position_embeddings=max(cfg.max_len, 512),
            rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": cfg.rope_theta_global},
                             "sliding_attention": {"rope_type": "default", "rope_theta": cfg.rope_theta_local}})
        self.encoder = ModernBertModel(ec)
        layer = nn.TransformerEncoderLayer(cfg.hidden, cfg.head_heads, cfg.head_ff, dropout=0.0,
                                           activation="relu", batch_first=True, norm_first=True)
        self.head = nn.TransformerEncoder(layer, cfg.head_layers, enable_nested_tensor=False)
        self.type_emb = nn.Embedding(cfg.num_qtypes, cfg.hidden)
        self.scorer = nn.Sequential(nn.LayerNorm(cfg.hidden), nn.Linear(cfg.hidden, cfg.hidden),
                                    nn.GELU(), nn.Linear(cfg.hidden, 1))
        self.act_head = nn.Sequential(nn.Linear(cfg.hidden + cfg.act_features, cfg.act_hidden),
                                      nn.GELU(), nn.Linear(cfg.act_hidden, 2))


def load(net, cfg, w):
    t = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in as_float32(w).items()}
    enc = net.encoder
    sets = [(enc.embeddings.tok_embeddings.weight, "embed.tok"), (enc.embeddings.norm.weight, "embed.norm.w"),
            (enc.final_norm.weight, "final_norm.w"), (net.type_emb.weight, "type_emb")]
    for i, layer in enumerate(enc.layers):
        p = f"enc.{i}."
        if i > 0:
            sets.append((layer.attn_norm.weight, p + "attn_norm.w"))
        sets += [(layer.attn.Wqkv.weight, p + "wqkv"), (layer.attn.Wo.weight, p + "wo"),
                 (layer.mlp_norm.weight, p + "mlp_norm.w"), (layer.mlp.Wi.weight, p + "wi"),
                 (layer.mlp.Wo.weight, p + "wo2")]
    for j, layer in enumerate(net.head.layers):
        p = f"head.{j}."
        sets += [(layer.norm1.weight, p + "norm1.w"), (layer.norm1.bias, p + "norm1.b"),
                 (layer.self_attn.in_proj_weight, p + "in_proj.w"), (layer.self_attn.in_proj_bias, p + "in_proj.b"),
                 (layer.self_attn.out_proj.weight, p + "out_proj.w"), (layer.self_attn.out_proj.bias, p + "out_proj.b"),
                 (layer.norm2.weight, p + "norm2.w"), (layer.norm2.bias, p + "norm2.b"),
                 (layer.linear1.weight, p + "linear1.w"), (layer.linear1.bias, p + "linear1.b"),
                 (layer.linear2.weight, p + "linear2.w"), (layer.linear2.bias, p + "linear2.b")]
    s, a = net.scorer, net.act_head
    sets += [(s[0].weight, "scorer.norm.w"), (s[0].bias, "scorer.norm.b"), (s[1].weight, "scorer.fc1.w"),
             (s[1].bias, "scorer.fc1.b"), (s[3].weight, "scorer.fc2.w"), (s[3].bias, "scorer.fc2.b"),
             (a[0].weight, "act.fc1.w"), (a[0].bias, "act.fc1.b"), (a[2].weight, "act.fc2.w"),
             (a[2].bias, "act.fc2.b")]
    seen = set()
    with torch.no_grad():
        for param, name in sets:
            param.copy_(t[name].reshape(param.shape))
            seen.add(name)
    missing = set(t) - seen
    if missing:
        raise RuntimeError(f"weights not mapped: {sorted(missing)}")


# (name, cfg, lengths, kinds, batch, seq, options, seed)
CASES = [
    ("laya_c1_noul_full", LAYA, [64], ["noul"], 1, 64, 2, 0),
    ("laya_c1_noul_pad", LAYA, [37], ["noul"], 1, 64, 2, 1),
    ("laya_mixed_b4_s96", LAYA, [96, 70, 41], ["choice", "score", "noul"], 4, 96, 4, 2),
    ("laya_long_s512", LAYA, [300], ["choice"], 1, 512, 4, 3),
    ("tiny_b3_s160", TINY, [160, 130, 12], ["choice", "noul", "score"], 3, 160, 4, 4),
    ("tiny_b2_s64_full", TINY, [64, 64], ["noul", "choice"], 2, 64, 4, 5),
]


def main():
    ref_src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LAYA_REFERENCE_SRC")
    if not ref_src:
        raise SystemExit("usage: make_golden.py <reference-src-dir> (or set LAYA_REFERENCE_SRC)")
    sys.path.insert(0, ref_src)
    import transformers
    import laya_blackwell.model as ref_model
    ref_model.rope_qkv = torch_rope
    from oracle.laya_oracle import Oracle

    torch.manual_seed(0)
    nets = {}
    for name, cfg, lengths, kinds, b, s, k, seed in CASES:
        key = id(cfg)
        if key not in nets:
            w = seeded_weights(cfg, seed=0)
            net = LayaNet(cfg).eval()
            load(net, cfg, w)
            model = ref_model.FastDecisionModel(net).eval()
            del net
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
