"""The reference's own forward on seeded weights, for the reference legs of
the benchmark and for the golden fixtures.  Not part of the b200 product.

It assembles a Laya-shaped network from ``transformers.ModernBertModel`` and
torch modules (encoder, two pre-norm ``nn.TransformerEncoderLayer`` head
layers, ``type_emb``, ``scorer``, ``act_head``), loads the seeded weights of
``laya_b200.weights`` into it and wraps it in the reference's
``laya_blackwell.model.FastDecisionModel`` (``src/laya_blackwell/model.py:22-56``),
exactly as the reference's engine wraps the SDK's network
(``src/laya_blackwell/engine.py:97-100``).  The reference package is imported
from ``baseline/_ref`` (the offline ``pip install --target`` of the reference,
which travels with the repository to a GPU box) or from the directory named by
``LAYA_REFERENCE_SRC``.

``rope="shim"`` replaces the reference's Triton ``rope_qkv`` by a torch
restatement of the same arithmetic (fp32 rotate-half, bf16 round, V untouched,
``tests/test_kernels.py:42-49`` of the reference), which the CPU needs;
``rope="native"`` keeps the reference's Triton kernel (GPU runs).
"""
import os
import sys
from pathlib import Path

import numpy as np
import torch
from torch import nn

HERE = Path(__file__).resolve().parent
REF_INSTALL = HERE / "_ref"


def reference_src():
    """Directory that holds the reference's ``laya_blackwell`` package, or None."""
    env = os.environ.get("LAYA_REFERENCE_SRC")
    for cand in ([Path(env)] if env else []) + [REF_INSTALL]:
        if (cand / "laya_blackwell" / "model.py").exists():
            return cand
    return None


def import_reference(module="model"):
    """Import ``laya_blackwell.<module>`` from the reference install; raises
    ImportError with the reason when it is absent."""
    src = reference_src()
    if src is None:
        raise ImportError("the reference package is not installed (baseline/_ref) and LAYA_REFERENCE_SRC is unset")
    if str(src) not in sys.path:
        sys.path.insert(0, str(src))
    import importlib
    return importlib.import_module(f"laya_blackwell.{module}")


def torch_rope(qkv, cos, sin, *, fp32=False):
    """The reference's RoPE known answer (tests/test_kernels.py:42-49):
    rotate-half on q, k; v passthrough."""
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
    """The network the Laya SDK builds (encoder + head + scorer + act_head)."""

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
    """Copy the parameter table of laya_b200.weights into the network."""
    from laya_b200.weights import as_float32
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


_NATIVE_ROPE = []


def use_rope(rope):
    """Select the RoPE the reference's forward calls (a module global it looks
    up at call time, so this applies to every model built from it): "native"
    (its Triton kernel) or "shim" (the torch restatement)."""
    ref_model = import_reference("model")
    if not _NATIVE_ROPE:
        _NATIVE_ROPE.append(ref_model.rope_qkv)
    if rope == "shim":
        ref_model.rope_qkv = torch_rope
    elif rope == "native":
        ref_model.rope_qkv = _NATIVE_ROPE[0]
    else:
        raise ValueError("rope must be shim or native")
    return ref_model


def build(cfg, weights, device="cpu", rope="shim"):
    """The reference's FastDecisionModel over the seeded network, on `device`
    (its Linears in bf16, embeddings and norms fp32, as model.py:28-35 casts)."""
    ref_model = use_rope(rope)
    net = LayaNet(cfg).eval()
    load(net, cfg, weights)
    net = net.to(device)
    model = ref_model.FastDecisionModel(net).eval()
    del net
    return model
