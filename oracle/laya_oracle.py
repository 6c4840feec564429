"""CPU oracle for the Laya decision forward.  TEST INFRASTRUCTURE ONLY.

This module is the checker for the b200 CUDA path: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it.  The product path never calls it and has no CPU fallback.

It restates ``FastDecisionModel.forward`` (``src/laya_blackwell/model.py:72-123``)
in plain PyTorch fp32 arithmetic on the CPU, keeping every bf16 rounding point
of the reference:

* Linear layers: bf16 weights and inputs, fp32 accumulation, bias added in
  fp32, one rounding to bf16 (``model.py:28-35`` casts every ``nn.Linear``).
* ``add_norm``: fp32 residual add, LayerNorm in fp32, bf16 copy of the normed
  row (``model.py:15-19``).
* RoPE in fp32: ``y = bf16(a*cos + b*sin)`` with separate fp32 products (no
  FMA), V untouched (``kernels.py:62-93``, pinned bit-exactly by
  ``tests/test_kernels.py:32-49``).
* SDPA: fp32 softmax of ``q k^T / 8`` over visible keys, fp32 ``P V``, bf16
  output; a query with no visible key yields zeros (what PyTorch's SDPA
  returns for a fully masked row).
* Local layers see keys with ``|i - j| <= local_attention // 2``
  (``model.py:82-83``); global layers see every unpadded key.
* GEGLU: ``bf16(bf16(gelu(act)) * gate)`` (``model.py:98-101``).
* Head, scorer and act_head as ``model.py:58-70,105-123``.

FP8 follows ``src/laya_blackwell/quantization.py:20-101`` (per-row dynamic
activation scale amax/448, per-output-row weight scale, e4m3 values, fp32
accumulate, bf16 out) on the encoder linears only (``replace_encoder_linears``,
``quantization.py:110-129``).  NVFP4 follows ``experiments/frontier/nvfp4.py:29-92``
(e2m1 values, e4m3 scales per 16 elements, ``cvt.rn.satfinite`` rounding,
2^-9 scale floor) with the outer fp32 scale per tensor for weights and per row
for activations.
"""
import math

import numpy as np
import torch

E4M3_MAX = 448.0
FP8_MIN_SCALE = 1e-12


def bf16(x):
    return x.to(torch.bfloat16).to(torch.float32)


def _t(a):
    if isinstance(a, torch.Tensor):
        return a
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy((a.astype(np.uint32) << 16).view(np.float32).copy())
    return torch.from_numpy(np.ascontiguousarray(a))


# ---------------------------------------------------------------------------
# Quantisers (oracle restatements)

def e4m3(x):
    """fp32 -> e4m3fn -> fp32, round to nearest even (inputs already clamped)."""
    return x.to(torch.float8_e4m3fn).to(torch.float32)


# fp32 reciprocal of 448: the reference computes amax / 448 as amax * fl(1/448)
# (PyTorch's CUDA tensor-by-scalar division and Triton's division by a constant
# both lower to that product); pinned by tests/golden/fp8_linear.
INV_E4M3_MAX = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(E4M3_MAX, dtype=torch.float32)


def fp8_quantize_rows(x):
    """quantization.py:20-29 (_quantize_rows) and :69-73 (weights): per-row
    scale = max(amax * fl(1/448), 1e-12), values clamp(x/scale, +-448) -> e4m3."""
    amax = x.abs().amax(dim=-1, keepdim=True)
    scale = torch.clamp(amax * INV_E4M3_MAX, min=FP8_MIN_SCALE)
    q = e4m3(torch.clamp(x / scale, -E4M3_MAX, E4M3_MAX))
    return q, scale


E2M1_GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1(x):
    """fp32 -> e2m1 -> fp32: round to nearest, ties to even code, saturate at 6
    (cvt.rn.satfinite.e2m1x2.f32, nvfp4.py:17-26)."""
    a = x.abs().clamp(max=6.0)
    grid = E2M1_GRID
    idx = torch.searchsorted(grid, a.contiguous())          # first grid >= a
    idx = idx.clamp(max=7)
    lo = grid[(idx - 1).clamp(min=0)]
    hi = grid[idx]
    d_lo, d_hi = a - lo, hi - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((idx % 2) == 0))
    q = torch.where(pick_hi, hi, lo)
    q = torch.where(a >= hi, hi, q)
    return torch.where(x < 0, -q, q)


def nvfp4_quantize(x, per_row):
    """nvfp4.py:36-51: outer = max(amax/(6*448), 1e-20) (per row or per
    tensor), block scale = e4m3(max(block_amax/(6*outer), 2^-9)), values
    e2m1(x / (scale*outer)).  Returns the dequantised fp32 tensor and parts."""
    rows, k = x.shape
    amax = x.abs().amax(dim=1, keepdim=True) if per_row else x.abs().amax().reshape(1, 1)
    outer = torch.clamp(amax / (6.0 * E4M3_MAX), min=1e-20)
    outer3 = outer[:, :, None]
    blocks = x.reshape(rows, k // 16, 16)
    bmax = blocks.abs().amax(dim=2, keepdim=True)
    scale = e4m3(torch.clamp(bmax / (6.0 * outer3), min=2.0 ** -9))
    q = e2m1(blocks / (scale * outer3))
    deq = (q * scale).reshape(rows, k)
    return deq, outer


# ---------------------------------------------------------------------------
# Building blocks

def linear(x, w, b=None):
    y = x @ w.T
    if b is not None:
        y = y + b
    return bf16(y)


def linear_bf16(x, w, b=None):
    """The same Linear as the reference evaluates it on a CPU: bf16 operands
    through torch's bf16 GEMM (fp32 accumulation, one rounding of the output,
    the bias added before it), as ``nn.Linear`` after ``model.py:28-35``'s
    cast does.  ``w`` / ``b`` are bf16 tensors; returns bf16 values in fp32."""
    xb = x.to(torch.bfloat16)
    y = torch.addmm(b, xb.reshape(-1, xb.shape[-1]), w.T) if b is not None else xb.reshape(-1, xb.shape[-1]) @ w.T
    return y.reshape(*x.shape[:-1], w.shape[0]).float()


def encoder_linear(x, w, precision, cache, key, lin=None):
    """An encoder nn.Linear under the chosen precision (bias-free).  ``lin``
    (bf16 precision only) replaces the fp32-accumulating restatement."""
    if precision == "bf16":
        return lin(x, w) if lin is not None else linear(x, w)
    if precision == "fp8":
        if key not in cache:
            cache[key] = fp8_quantize_rows(w)
        wq, ws = cache[key]
        xq, xs = fp8_quantize_rows(x)
        return bf16((xq @ wq.T) * xs * ws.T)
    if precision == "nvfp4":
        if key not in cache:
            cache[key] = nvfp4_quantize(w, per_row=False)
        wq, wo = cache[key]
        k = x.shape[1]
        if k % 16:
            raise ValueError("NVFP4 needs K divisible by 16")
        xq, xo = nvfp4_quantize(x, per_row=True)
        return bf16((xq @ wq.T) * xo * wo)
    raise ValueError(f"unknown precision {precision!r}")


def layer_norm(x, w, b, eps):
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), w, b, eps)


def rope_tables(theta, max_len, dim):
    """transformers ModernBertRotaryEmbedding (default rope): inv_freq in fp32,
    freqs = inv_freq * pos (fp32), emb = cat(freqs, freqs); cos/sin fp32
    (model.py:50-56 registers them as [max_len, dim])."""
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    pos = torch.arange(max_len).float()
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def rope(x, cos, sin):
    """x: [b, s, heads, 64] (bf16 values in fp32); kernels.py:62-93 FP32 mode."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    c = cos[None, : x.shape[1], None, :]
    s = sin[None, : x.shape[1], None, :]
    return bf16(x * c + rot * s)


def attention(q, k, v, visible):
    """q: [b, h, sq, 64], k/v: [b, h, sk, 64], visible: bool broadcastable to
    [b, h, sq, sk].  fp32 softmax, bf16 output, zeros for rows with no key."""
    s = (q @ k.transpose(-1, -2)) * 0.125
    s = s.masked_fill(~visible, float("-inf"))
    any_visible = visible.any(dim=-1, keepdim=True)
    s = torch.where(any_visible, s, torch.zeros_like(s))
    p = torch.softmax(s, dim=-1)
    p = torch.where(visible, p, torch.zeros_like(p))
    return bf16(p @ v)


def gelu(x):
    return torch.nn.functional.gelu(x)


# ---------------------------------------------------------------------------
# The forward

class Oracle:
    """Holds fp32 copies of the weights; ``forward`` mirrors model.py:72-123.

    ``bf16_gemm=True`` evaluates every bf16 Linear with torch's bf16 GEMM, the
    reference's own CPU arithmetic (same rounding points, its accumulation
    order; several times faster on CPUs with bf16 matrix units).  It is pinned
    against the same golden fixtures and is what the benchmark's CPU
    reference arm times; the parity tests use the default fp32 restatement."""

    def __init__(self, weights, cfg, precision="bf16", bf16_gemm=False):
        self.cfg = cfg
        self.precision = precision
        self.w = {k: _t(v).float() for k, v in weights.items()}
        self.gcos, self.gsin = rope_tables(cfg.rope_theta_global, cfg.max_len, cfg.head_dim)
        self.lcos, self.lsin = rope_tables(cfg.rope_theta_local, cfg.max_len, cfg.head_dim)
        self.qcache = {}
        self.bf16_gemm = bf16_gemm
        self.wb = {}  # bf16 copies of the Linear weights and biases (bf16_gemm)

    def _lin(self, x, name, bias=None):
        """Linear `name` (+ bias `bias`) in the oracle's bf16 arithmetic."""
        w = self.w
        if not self.bf16_gemm:
            return linear(x, w[name], w[bias] if bias else None)
        for k in (name, bias):
            if k and k not in self.wb:
                self.wb[k] = w[k].to(torch.bfloat16)
        return linear_bf16(x, self.wb[name], self.wb[bias] if bias else None)

    def _enc(self, x, name):
        lin = (lambda xx, _w: self._lin(xx, name)) if self.bf16_gemm else None
        return encoder_linear(x, self.w[name], self.precision, self.qcache, name, lin)

    def _head_layer(self, h, j, key_visible, select=None):
        """model.py:58-70 (pre-norm nn.TransformerEncoderLayer, bf16 linears)."""
        w, cfg = self.w, self.cfg
        p = f"head.{j}."
        n = bf16(layer_norm(h, w[p + "norm1.w"], w[p + "norm1.b"], cfg.norm_eps))
        b, length, d = n.shape
        H = cfg.head_heads
        qkv = self._lin(n, p + "in_proj.w", p + "in_proj.b")
        qkv = qkv.view(b, length, 3, H, d // H).permute(0, 3, 2, 1, 4)
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        if select is not None:
            q = torch.gather(q, 2, select[:, None, :, None].expand(-1, H, -1, d // H))
            h = torch.gather(h, 1, select[:, :, None].expand(-1, -1, d))
        a = attention(q, k, v, key_visible)
        a = a.transpose(1, 2).reshape(b, -1, d)
        h = h + self._lin(a, p + "out_proj.w", p + "out_proj.b")
        n = bf16(layer_norm(h, w[p + "norm2.w"], w[p + "norm2.b"], cfg.norm_eps))
        f = torch.relu(self._lin(n, p + "linear1.w", p + "linear1.b"))
        return h + self._lin(f, p + "linear2.w", p + "linear2.b")

    @torch.inference_mode()
    def forward(self, input_ids, attention_mask, marker_pos, marker_mask, qtype, trace=None):
        cfg, w = self.cfg, self.w
        ids = torch.as_tensor(np.asarray(input_ids), dtype=torch.long)
        am = torch.as_tensor(np.asarray(attention_mask)).bool()
        mpos = torch.as_tensor(np.asarray(marker_pos), dtype=torch.long)
        mmask = torch.as_tensor(np.asarray(marker_mask)).bool()
        qt = torch.as_tensor(np.asarray(qtype), dtype=torch.long)
        b, length = ids.shape
        H, D = cfg.heads, cfg.head_dim
        key_visible = am[:, None, None, :]
        pos = torch.arange(length)
        local_visible = key_visible & ((pos[:, None] - pos[None, :]).abs() <= cfg.window)[None, None]
        # enc.embeddings: tok_embeddings gather + LayerNorm (no bias), model.py:84
        h = layer_norm(w["embed.tok"][ids], w["embed.norm.w"], None, cfg.norm_eps)
        pending = None
        for i in range(cfg.layers):
            p = f"enc.{i}."
            if i == 0:
                n = bf16(h)
            else:
                h = h + pending
                n = bf16(layer_norm(h, w[p + "attn_norm.w"], None, cfg.norm_eps))
            x = n.reshape(b * length, -1)
            qkv = self._enc(x, p + "wqkv")
            qkv = qkv.view(b, length, 3, H, D)
            glob = cfg.is_global(i)
            cos, sin = (self.gcos, self.gsin) if glob else (self.lcos, self.lsin)
            q = rope(qkv[:, :, 0], cos, sin).permute(0, 2, 1, 3)
            k = rope(qkv[:, :, 1], cos, sin).permute(0, 2, 1, 3)
            v = qkv[:, :, 2].permute(0, 2, 1, 3)
            a = attention(q, k, v, key_visible if glob else local_visible)
            a = a.transpose(1, 2).reshape(b * length, -1)
            h = h + self._enc(a, p + "wo").view(b, length, -1)
            n = bf16(layer_norm(h, w[p + "mlp_norm.w"], None, cfg.norm_eps)).reshape(b * length, -1)
            y = self._enc(n, p + "wi")
            act, gate = y.chunk(2, dim=-1)
            g = bf16(bf16(gelu(act)) * gate)
            pending = self._enc(g, p + "wo2").view(b, length, -1)
            if trace is not None:
                trace.append(h.clone())
        h = layer_norm(h + pending, w["final_norm.w"], None, cfg.norm_eps)
        h = h + w["type_emb"][qt][:, None, :]
        select = torch.cat((torch.zeros_like(mpos[:, :1]), mpos), dim=1)
        for j in range(cfg.head_layers):
            h = self._head_layer(h, j, key_visible, select if j == cfg.head_layers - 1 else None)
        if cfg.head_layers == 0:
            h = torch.gather(h, 1, select[:, :, None].expand(-1, -1, h.shape[-1]))
        m = bf16(layer_norm(h[:, 1:], w["scorer.norm.w"], w["scorer.norm.b"], cfg.norm_eps))
        z = bf16(gelu(self._lin(m, "scorer.fc1.w", "scorer.fc1.b")))
        logits = self._lin(z, "scorer.fc2.w", "scorer.fc2.b").squeeze(-1)
        logits = logits.masked_fill(~mmask, -1e4)
        p = logits.softmax(-1)
        count = mmask.sum(-1).clamp(min=2).float()
        ent = -(p * p.clamp_min(1e-9).log()).sum(-1) / count.log()
        top = p.topk(2, -1).values
        feats = torch.stack((top[:, 0], top[:, 0] - top[:, 1], ent, count / 255), -1)
        x = bf16(torch.cat((h[:, 0], feats), -1))
        a1 = bf16(gelu(self._lin(x, "act.fc1.w", "act.fc1.b")))
        act = self._lin(a1, "act.fc2.w", "act.fc2.b")
        return logits.numpy().astype(np.float32), act.numpy().astype(np.float32)


def decision_agreement(ref_logits, test_logits, marker_mask):
    """Fraction of rows whose argmax over the real options agrees."""
    agree = []
    for r, t, m in zip(ref_logits, test_logits, marker_mask):
        k = int(np.asarray(m).sum())
        agree.append(int(np.argmax(r[:k]) == np.argmax(t[:k])))
    return float(np.mean(agree)) if agree else 1.0


def top2_margin(logits, marker_mask):
    out = []
    for r, m in zip(logits, marker_mask):
        k = int(np.asarray(m).sum())
        s = np.sort(r[:k])
        out.append(float(s[-1] - s[-2]) if k > 1 else math.inf)
    return np.array(out)
