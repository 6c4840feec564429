"""The tcgen05 attention kernel against the oracle's attention, fed with the
GPU's own rotated q, k, v (read back from the engine after a forward), on the
shapes that exercise its tiling: 1 to 8 chunks of 64 keys per 128-query tile,
partial chunks and query tiles, key padding, fully masked query rows, the
radius-64 local window (keys [q0 - 64, q0 + 191]) and the head's selected
query rows.  One sequence of at most 64 tokens runs attention inside the
output projection instead, so every case here has more rows.

The reference is the oracle's attention (``oracle/laya_oracle.py``
``attention``: fp32 softmax and fp32 P.V, SDPA's semantics,
``model.py:92-96``): within 2e-2 max-abs (the bf16 tolerance of the forward),
and within one bf16 step of the oracle's value for at least 99.9% of the
outputs, since the kernel carries p to about 16 bits (hi + lo bf16 tiles)
and differs from fp32 only by exp2 and summation order."""
import numpy as np
import pytest
import torch

from laya_b200.config import LayaConfig
from laya_b200.weights import seeded_weights, bf16_bits_to_f32
from laya_b200.workload import synthetic_items, pack
from oracle import laya_oracle as O

pytestmark = pytest.mark.gpu

GLOBAL = LayaConfig(layers=1, hidden=256, heads=4, intermediate=384, vocab=1000, pad_token_id=999, max_len=512,
                    head_layers=0, head_heads=4, head_ff=512, act_hidden=64)
# layer 1 is a local (radius-64) layer
LOCAL = LayaConfig(layers=2, hidden=256, heads=4, intermediate=384, vocab=1000, pad_token_id=999, max_len=512,
                   head_layers=0, head_heads=4, head_ff=512, act_hidden=64)
# one head layer: its attention runs on the CLS and marker rows only
HEAD = LayaConfig(layers=1, hidden=256, heads=4, intermediate=384, vocab=1000, pad_token_id=999, max_len=512,
                  head_layers=1, head_heads=4, head_ff=512, act_hidden=64)


def bf16_of(u16):
    return torch.from_numpy(bf16_bits_to_f32(u16))


def run_forward(cfg, seed, lengths, s, options=4):
    from laya_b200.engine import NativeForward
    w = seeded_weights(cfg, seed=seed)
    b = len(lengths)
    kinds = ["choice", "score", "noul"]
    items = synthetic_items(lengths, [kinds[i % 3] for i in range(b)], seed=seed + s, vocab=cfg.vocab)
    inp = pack(items, b, s, options, cfg.pad_token_id)
    nf = NativeForward(0, cfg, w, "bf16", max_batch=4, max_options=8)
    try:
        slot = nf.capture(b, s, options, False)
        nf.run(slot, inp)
        T, d = b * s, cfg.hidden
        out = {"qkv": bf16_of(nf.read_buffer("qkv", (T, 3 * d), np.uint16)),
               "attn": bf16_of(nf.read_buffer("attn", (T, d), np.uint16)),
               "asel": bf16_of(nf.read_buffer("asel", (b * (1 + options), d), np.uint16))}
    finally:
        nf.close()
    return inp, out


def split_heads(qkv, b, s, heads):
    q5 = qkv.view(b, s, 3, heads, 64)
    return (q5[:, :, 0].permute(0, 2, 1, 3), q5[:, :, 1].permute(0, 2, 1, 3), q5[:, :, 2].permute(0, 2, 1, 3))


def bf16_step(x):
    """Spacing of bf16 values at |x| (8 significant bits)."""
    e = torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -126)))
    return torch.exp2(e - 7)


def check(got, q, k, v, visible, label):
    want = O.attention(q, k, v, visible)
    got = got.reshape(want.shape)
    diff = (got - want).abs()
    err = float(diff.max())
    far = float((diff > bf16_step(want) * 1.001).float().mean())
    print(label, "max-abs", err, "beyond one bf16 step", far)
    assert torch.isfinite(got).all(), label
    assert err < 2e-2, (label, err)
    assert far < 1e-3, (label, far)
    # rows that see no key are exact zeros
    blind = ~visible.any(dim=-1)
    if blind.any():
        assert float(got.abs().amax(dim=-1)[blind.expand(got.shape[:-1])].max()) == 0.0, label


@pytest.mark.parametrize("lengths, s", [
    ([64, 20], 64),             # one chunk, half a query tile
    ([65, 7], 65),              # a partial second chunk
    ([192, 100], 192),          # three chunks, two query tiles, key padding
    ([96, 50, 7, 96], 96),      # C2-shaped rows: one 128-query tile of 96
    ([448, 300], 448),          # seven chunks
    ([512], 512),               # eight chunks: the whole TMEM row
    ([512, 260, 33], 512),      # eight chunks with padding in every row
])
def test_global_attention_matches_oracle(lengths, s):
    cfg = GLOBAL
    b = len(lengths)
    inp, out = run_forward(cfg, 3, lengths, s)
    q, k, v = split_heads(out["qkv"], b, s, cfg.heads)
    visible = torch.from_numpy(inp["attention_mask"]).bool()[:, None, None, :].expand(b, cfg.heads, s, s)
    got = out["attn"].view(b, s, cfg.heads, 64).permute(0, 2, 1, 3)
    check(got, q, k, v, visible, (lengths, s))


@pytest.mark.parametrize("lengths, s", [
    ([64, 64], 64),
    ([130], 130),               # second query tile sees keys [64, 130)
    ([300, 40], 384),           # padded queries beyond the radius see no key
    ([512], 512),               # four chunks per query tile
    ([512, 500, 129, 7], 512),
])
def test_local_window_attention_matches_oracle(lengths, s):
    cfg = LOCAL
    b = len(lengths)
    inp, out = run_forward(cfg, 5, lengths, s)
    q, k, v = split_heads(out["qkv"], b, s, cfg.heads)
    keys = torch.from_numpy(inp["attention_mask"]).bool()[:, None, None, :]
    pos = torch.arange(s)
    band = (pos[:, None] - pos[None, :]).abs() <= cfg.window
    visible = (keys & band[None, None]).expand(b, cfg.heads, s, s)
    got = out["attn"].view(b, s, cfg.heads, 64).permute(0, 2, 1, 3)
    check(got, q, k, v, visible, (lengths, s))


@pytest.mark.parametrize("lengths, s, options", [
    ([40, 12], 64, 4),
    ([300, 512, 90], 512, 8),
])
def test_head_selected_rows_attention_matches_oracle(lengths, s, options):
    """The last head layer attends from the CLS row and the marker rows only
    (model.py:64-66); padded option slots select position 0."""
    cfg = HEAD
    b = len(lengths)
    inp, out = run_forward(cfg, 7, lengths, s, options)
    q, k, v = split_heads(out["qkv"], b, s, cfg.head_heads)
    sel = np.concatenate([np.zeros((b, 1), np.int64), inp["marker_pos"]], axis=1)   # [b, 1 + options]
    idx = torch.from_numpy(sel)
    qsel = torch.stack([q[i][:, idx[i]] for i in range(b)])                         # [b, h, 1+k, 64]
    keys = torch.from_numpy(inp["attention_mask"]).bool()[:, None, None, :]
    visible = keys.expand(b, cfg.head_heads, 1 + options, s)
    got = out["asel"].view(b, 1 + options, cfg.head_heads, 64).permute(0, 2, 1, 3)
    check(got, qsel, k, v, visible, (lengths, s, options))
