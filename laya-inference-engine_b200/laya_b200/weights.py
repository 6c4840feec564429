"""Parameter table of the Laya network and a seeded random initialiser.

The pinned checkpoint cannot be downloaded here, so every run uses seeded
random weights of the checkpoint's shapes.  Names follow the roles the
reference's forward gives them (``src/laya_blackwell/model.py:58-123``):

* ``embed.tok`` / ``embed.norm.w``      enc.embeddings (tok_embeddings + LayerNorm, no bias)
* ``enc.{i}.attn_norm.w``               layer.attn_norm (absent for layer 0: Identity)
* ``enc.{i}.wqkv|wo|mlp_norm.w|wi|wo2`` layer.attn.Wqkv, attn.Wo, mlp_norm, mlp.Wi, mlp.Wo
* ``final_norm.w`` / ``type_emb``       enc.final_norm, net.type_emb
* ``head.{j}.*``                        net.head.layers[j] (norm1, in_proj, out_proj, norm2, linear1, linear2)
* ``scorer.*`` / ``act.*``              net.scorer[0,1,3] and net.act_head[0,2]

Storage dtypes follow ``FastDecisionModel.__init__`` (``model.py:28-35``): every
Linear weight and bias (and the packed ``in_proj``) is bf16; embeddings and
LayerNorm parameters stay fp32.

Initialisation: N(0, 0.02) for matrices, embeddings and biases; LayerNorm
weights 1 + N(0, 0.02) and LayerNorm biases N(0, 0.02) so that every scale and
shift of the path is exercised.  One ``numpy.random.Generator(PCG64(seed))``
draws the tensors in table order, so any machine regenerates identical bits.
"""
import hashlib

import numpy as np

from .config import LayaConfig, LAYA

BF16, F32 = "bf16", "f32"


def param_table(cfg: LayaConfig = LAYA):
    """Ordered (name, shape, storage dtype, init kind) for every parameter."""
    d, I, V = cfg.hidden, cfg.intermediate, cfg.vocab
    t = [("embed.tok", (V, d), F32, "normal"), ("embed.norm.w", (d,), F32, "ln_w")]
    for i in range(cfg.layers):
        p = f"enc.{i}."
        if i > 0:
            t.append((p + "attn_norm.w", (d,), F32, "ln_w"))
        t += [(p + "wqkv", (3 * d, d), BF16, "normal"),
              (p + "wo", (d, d), BF16, "normal"),
              (p + "mlp_norm.w", (d,), F32, "ln_w"),
              (p + "wi", (2 * I, d), BF16, "normal"),
              (p + "wo2", (d, I), BF16, "normal")]
    t += [("final_norm.w", (d,), F32, "ln_w"),
          ("type_emb", (cfg.num_qtypes, d), F32, "normal")]
    F = cfg.head_ff
    for j in range(cfg.head_layers):
        p = f"head.{j}."
        t += [(p + "norm1.w", (d,), F32, "ln_w"), (p + "norm1.b", (d,), F32, "ln_b"),
              (p + "in_proj.w", (3 * d, d), BF16, "normal"), (p + "in_proj.b", (3 * d,), BF16, "normal"),
              (p + "out_proj.w", (d, d), BF16, "normal"), (p + "out_proj.b", (d,), BF16, "normal"),
              (p + "norm2.w", (d,), F32, "ln_w"), (p + "norm2.b", (d,), F32, "ln_b"),
              (p + "linear1.w", (F, d), BF16, "normal"), (p + "linear1.b", (F,), BF16, "normal"),
              (p + "linear2.w", (d, F), BF16, "normal"), (p + "linear2.b", (d,), BF16, "normal")]
    A = cfg.act_hidden
    t += [("scorer.norm.w", (d,), F32, "ln_w"), ("scorer.norm.b", (d,), F32, "ln_b"),
          ("scorer.fc1.w", (d, d), BF16, "normal"), ("scorer.fc1.b", (d,), BF16, "normal"),
          ("scorer.fc2.w", (1, d), BF16, "normal"), ("scorer.fc2.b", (1,), BF16, "normal"),
          ("act.fc1.w", (A, d + cfg.act_features), BF16, "normal"), ("act.fc1.b", (A,), BF16, "normal"),
          ("act.fc2.w", (2, A), BF16, "normal"), ("act.fc2.b", (2,), BF16, "normal")]
    return t


def f32_to_bf16_bits(x):
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def seeded_weights(cfg: LayaConfig = LAYA, seed: int = 0):
    """Dict name -> numpy array.  bf16 tensors are uint16 bit patterns."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for name, shape, dtype, kind in param_table(cfg):
        x = rng.standard_normal(size=shape, dtype=np.float32)
        x *= np.float32(0.02)
        if kind == "ln_w":
            x += np.float32(1.0)
        if name == "embed.tok":
            x[cfg.pad_token_id] = 0.0   # nn.Embedding(padding_idx=pad) zero row
        out[name] = f32_to_bf16_bits(x) if dtype == BF16 else x
    return out


def as_float32(weights):
    """Same dict with bf16 bit patterns widened to fp32 (exact)."""
    return {k: (bf16_bits_to_f32(v) if v.dtype == np.uint16 else v) for k, v in weights.items()}


def weights_digest(weights):
    h = hashlib.sha256()
    for k in sorted(weights):
        h.update(k.encode())
        h.update(np.ascontiguousarray(weights[k]).tobytes())
    return h.hexdigest()


def check_weights(weights, cfg: LayaConfig = LAYA):
    """Raise ValueError unless every table entry is present with its shape/dtype."""
    for name, shape, dtype, _ in param_table(cfg):
        if name not in weights:
            raise ValueError(f"missing weight {name!r}")
        w = weights[name]
        want = np.uint16 if dtype == BF16 else np.float32
        if tuple(w.shape) != tuple(shape) or w.dtype != want:
            raise ValueError(f"weight {name!r}: expected {shape} {np.dtype(want).name}, "
                             f"got {tuple(w.shape)} {w.dtype}")
        if dtype == F32 and not np.isfinite(w).all():
            raise ValueError(f"weight {name!r} contains NaN or infinity")
