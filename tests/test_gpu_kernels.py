"""Kernel-level parity on a one-layer network: every stage of the CUDA forward
against the CPU oracle, each stage fed with the GPU's own previous stage so a
mismatch points at one kernel.  Calls the library through the C ABI."""
import numpy as np
import pytest
import torch

from laya_b200.config import LayaConfig
from laya_b200.weights import seeded_weights, as_float32, bf16_bits_to_f32
from laya_b200.workload import synthetic_items, pack
from oracle import laya_oracle as O

pytestmark = pytest.mark.gpu

MICRO = LayaConfig(layers=1, hidden=256, heads=4, intermediate=384, vocab=1000, pad_token_id=999, max_len=512,
                   head_layers=0, head_heads=4, head_ff=512, act_hidden=64)
MICRO_LOCAL = LayaConfig(layers=2, hidden=256, heads=4, intermediate=384, vocab=1000, pad_token_id=999,
                         max_len=512, head_layers=1, head_heads=4, head_ff=512, act_hidden=64)


def bf16_of(u16):
    return torch.from_numpy(bf16_bits_to_f32(u16))


def frac_mismatch(a, b, atol):
    return float((np.abs(a - b) > atol).mean())


@pytest.fixture(scope="module")
def micro():
    from laya_b200.engine import NativeForward
    w = seeded_weights(MICRO, seed=3)
    nf = NativeForward(0, MICRO, w, "bf16", max_batch=4, max_options=8)
    yield nf, w
    nf.close()


def test_stages_match_oracle(micro):
    nf, w = micro
    cfg = MICRO
    b, s, k = 2, 192, 4
    items = synthetic_items([192, 100], ["choice", "noul"], seed=11, vocab=cfg.vocab)
    inp = pack(items, b, s, k, cfg.pad_token_id)
    slot = nf.capture(b, s, k, False)
    logits, act = nf.run(slot, inp)
    T, d, I = b * s, cfg.hidden, cfg.intermediate
    wf = {kk: torch.from_numpy(v) for kk, v in as_float32(w).items()}
    qkv = bf16_of(nf.read_buffer("qkv", (T, 3 * d), np.uint16).view(np.uint16))
    attn = bf16_of(nf.read_buffer("attn", (T, d), np.uint16))
    g = bf16_of(nf.read_buffer("g", (T, I), np.uint16))
    h = torch.from_numpy(nf.read_buffer("h", (T, d), np.float32))
    report = {}
    ids = torch.from_numpy(inp["input_ids"]).reshape(-1)
    h0 = O.layer_norm(wf["embed.tok"][ids], wf["embed.norm.w"], None, cfg.norm_eps)
    n0 = O.bf16(h0)
    # The projection's epilogue applies the rotary embedding (layer 0 is
    # global) to q and k: compare with the rotated reference.
    gcos, gsin = O.rope_tables(cfg.rope_theta_global, cfg.max_len, 64)
    r5 = O.linear(n0, wf["enc.0.wqkv"]).view(b, s, 3, cfg.heads, 64)
    qkv_ref = torch.cat([O.rope(r5[:, :, 0], gcos, gsin)[:, :, None], O.rope(r5[:, :, 1], gcos, gsin)[:, :, None],
                         r5[:, :, 2:]], dim=2).reshape(T, 3 * d)
    report["qkv"] = (float((qkv - qkv_ref).abs().max()), frac_mismatch(qkv.numpy(), qkv_ref.numpy(), 1e-6))
    # attention from the GPU's own (rotated) qkv (global layer 0, key padding)
    q5 = qkv.view(b, s, 3, cfg.heads, 64)
    q = q5[:, :, 0].permute(0, 2, 1, 3)
    kk_ = q5[:, :, 1].permute(0, 2, 1, 3)
    v = q5[:, :, 2].permute(0, 2, 1, 3)
    vis = torch.from_numpy(inp["attention_mask"]).bool()[:, None, None, :]
    attn_ref = O.attention(q, kk_, v, vis).transpose(1, 2).reshape(T, d)
    report["attn"] = (float((attn - attn_ref).abs().max()), frac_mismatch(attn.numpy(), attn_ref.numpy(), 1e-6))
    h1 = h0 + O.linear(attn, wf["enc.0.wo"])
    n1 = O.bf16(O.layer_norm(h1, wf["enc.0.mlp_norm.w"], None, cfg.norm_eps))
    y = O.linear(n1, wf["enc.0.wi"])
    a_, gate = y.chunk(2, dim=-1)
    g_ref = O.bf16(O.bf16(O.gelu(a_)) * gate)
    report["geglu"] = (float((g - g_ref).abs().max()), frac_mismatch(g.numpy(), g_ref.numpy(), 1e-6))
    h2 = h1 + O.linear(g, wf["enc.0.wo2"])
    qt = torch.from_numpy(inp["qtype"])
    hf = O.layer_norm(h2, wf["final_norm.w"], None, cfg.norm_eps).view(b, s, d) + wf["type_emb"][qt][:, None, :]
    report["final_h"] = (float((h.view(b, s, d) - hf).abs().max()), 0.0)
    # whole forward against the oracle
    orc = O.Oracle(w, cfg)
    ol, oa = orc.forward(**inp)
    mm = inp["marker_mask"]
    report["logits"] = (float(np.abs(logits[mm] - ol[mm]).max()), 0.0)
    report["act"] = (float(np.abs(act - oa).max()), 0.0)
    print("stage max-abs / mismatch-fraction:", report)
    assert report["qkv"][0] < 2e-2 and report["qkv"][1] < 0.02, report
    # P is rounded to bf16 before P.V (as FlashAttention does) while the oracle
    # keeps fp32 probabilities, so many outputs differ by one bf16 ulp: only the
    # magnitude of the difference is checked.
    assert report["attn"][0] < 2e-2, report
    assert report["geglu"][0] < 2e-2 and report["geglu"][1] < 0.05, report
    assert report["final_h"][0] < 2e-2, report
    assert report["logits"][0] < 2e-2 and report["act"][0] < 2e-2, report
    assert np.array_equal(logits[~mm], np.full((~mm).sum(), -1e4, np.float32))


def test_local_window_and_head_select():
    from laya_b200.engine import NativeForward
    cfg = MICRO_LOCAL
    w = seeded_weights(cfg, seed=5)
    nf = NativeForward(0, cfg, w, "bf16", max_batch=4, max_options=8)
    try:
        orc = O.Oracle(w, cfg)
        # 300 valid tokens in a 384 bucket: padded queries beyond the radius see no key.
        for lengths, s in (([300, 40, 7], 384), ([64], 64), ([129, 130], 160)):
            b = 1 << (len(lengths) - 1).bit_length()
            kinds = ["choice", "score", "noul"][: len(lengths)]
            items = synthetic_items(lengths, kinds, seed=len(lengths) + s, vocab=cfg.vocab)
            inp = pack(items, b, s, 4, cfg.pad_token_id)
            slot = nf.capture(b, s, 4, False)
            logits, act = nf.run(slot, inp)
            ol, oa = orc.forward(**inp)
            mm = inp["marker_mask"]
            err = float(np.abs(logits[mm] - ol[mm]).max())
            aerr = float(np.abs(act - oa).max())
            assert err < 2e-2 and aerr < 2e-2, (lengths, s, err, aerr)
            assert np.isfinite(logits).all() and np.isfinite(act).all()
    finally:
        nf.close()


@pytest.mark.parametrize("precision", ["nvfp4", "fp8"])
def test_low_precision_qkv_stage_matches_oracle(precision):
    """Layer-0 QKV projection under FP8 / NVFP4 against the oracle's quantised
    linear on the same bf16 input (fp32 accumulation order differs, so a few
    outputs differ by one bf16 ulp)."""
    from laya_b200.engine import NativeForward
    cfg = MICRO
    w = seeded_weights(cfg, seed=3)
    nf = NativeForward(0, cfg, w, precision, max_batch=4, max_options=8)
    try:
        b, s, k = 2, 192, 4
        items = synthetic_items([192, 100], ["choice", "noul"], seed=11, vocab=cfg.vocab)
        inp = pack(items, b, s, k, cfg.pad_token_id)
        slot = nf.capture(b, s, k, False)
        logits, act = nf.run(slot, inp)
        T, d = b * s, cfg.hidden
        qkv = bf16_of(nf.read_buffer("qkv", (T, 3 * d), np.uint16))
    finally:
        nf.close()
    wf = {kk: torch.from_numpy(v) for kk, v in as_float32(w).items()}
    ids = torch.from_numpy(inp["input_ids"]).reshape(-1)
    n0 = O.bf16(O.layer_norm(wf["embed.tok"][ids], wf["embed.norm.w"], None, cfg.norm_eps))
    ref = O.encoder_linear(n0, wf["enc.0.wqkv"], precision, {}, "wqkv")
    # The projection's epilogue stores q and k rotated (layer 0 is global).
    gcos, gsin = O.rope_tables(cfg.rope_theta_global, cfg.max_len, 64)
    q5 = ref.view(b, s, 3, cfg.heads, 64)
    ref = torch.cat([O.rope(q5[:, :, 0], gcos, gsin)[:, :, None], O.rope(q5[:, :, 1], gcos, gsin)[:, :, None],
                     q5[:, :, 2:]], dim=2).reshape(T, 3 * d)
    err = float((qkv - ref).abs().max())
    rel = float(((qkv - ref).abs() / ref.abs().clamp_min(1e-2)).median())
    print(f"{precision} qkv: max-abs {err:.3e}, median rel {rel:.2e}")
    assert err < 3e-2, err
    orc = O.Oracle(w, cfg, precision)
    ol, oa = orc.forward(**inp)
    mm = inp["marker_mask"]
    tol = {"fp8": 6e-2, "nvfp4": 1.5e-1}[precision]
    assert np.abs(logits[mm] - ol[mm]).max() <= tol and np.abs(act - oa).max() <= tol


# (batch, seq, lengths): 256 rows run one CTA per row, 2,048 rows a warp per row
ROWS_SMALL = (2, 128, [128, 77])
ROWS_LARGE = (4, 512, [512, 300, 512, 77])


@pytest.mark.parametrize("intermediate, rows", [(384, ROWS_SMALL), (1920, ROWS_SMALL), (2624, ROWS_SMALL),
                                                (4096, ROWS_SMALL), (2624, ROWS_LARGE), (4096, ROWS_LARGE)])
def test_fp8_activation_quantiser_is_bit_exact(intermediate, rows):
    """The per-row e4m3 activation quantiser (quantization.py:20-29) on the
    attention output (k = hidden) and the GEGLU output (k = intermediate)
    against the oracle's torch restatement: scales and codes identical."""
    from laya_b200.engine import NativeForward
    cfg = LayaConfig(layers=1, hidden=256, heads=4, intermediate=intermediate, vocab=1000, pad_token_id=999,
                     max_len=512, head_layers=0, head_heads=4, head_ff=512, act_hidden=64)
    w = seeded_weights(cfg, seed=5)
    nf = NativeForward(0, cfg, w, "fp8", max_batch=4, max_options=8)
    try:
        b, s, lengths = rows
        k = 4
        items = synthetic_items(lengths, ["choice", "score", "noul", "choice"][:b], seed=12, vocab=cfg.vocab)
        nf.run(nf.capture(b, s, k, False), pack(items, b, s, k, cfg.pad_token_id))
        T = b * s
        for src, q, sc, width in (("attn", "a8", "a8s", cfg.hidden), ("g", "g8", "g8s", intermediate)):
            x = bf16_of(nf.read_buffer(src, (T, width), np.uint16))
            codes = torch.from_numpy(nf.read_buffer(q, (T, width), np.uint8))
            scale = torch.from_numpy(nf.read_buffer(sc, (T,), np.float32))
            ref_q, ref_scale = O.fp8_quantize_rows(x)
            assert torch.equal(scale, ref_scale[:, 0]), src
            got = codes.view(torch.float8_e4m3fn).to(torch.float32)
            assert torch.equal(got, ref_q), (src, int((got != ref_q).sum()))
    finally:
        nf.close()


def test_residual_tiles_with_a_partial_last_tile():
    """Unsplit 64-token residual tiles move their fp32 residual rows with one
    TMA load and one TMA store.  11 x 450 = 4,950 token rows at d = 256 give
    Wo and Wo2 156 such tiles, the last one 22 rows high: every row before the
    end must be updated (padded positions included) and none past it.  The
    final hidden rows are compared with the oracle fed with the GPU's own
    attention and GEGLU outputs, as in test_stages_match_oracle."""
    from laya_b200.engine import NativeForward
    cfg = MICRO
    w = seeded_weights(cfg, seed=5)
    b, s, k = 11, 450, 4
    kinds = ["choice", "score", "noul"]
    items = synthetic_items([450] * 9 + [300, 17], [kinds[i % 3] for i in range(b)], seed=13, vocab=cfg.vocab)
    inp = pack(items, b, s, k, cfg.pad_token_id)
    T, d, I = b * s, cfg.hidden, cfg.intermediate
    nf = NativeForward(0, cfg, w, "bf16", max_batch=b, max_options=8)
    try:
        slot = nf.capture(b, s, k, False)
        nf.run(slot, inp)
        attn = bf16_of(nf.read_buffer("attn", (T, d), np.uint16))
        g = bf16_of(nf.read_buffer("g", (T, I), np.uint16))
        h = torch.from_numpy(nf.read_buffer("h", (T, d), np.float32))
    finally:
        nf.close()
    wf = {kk: torch.from_numpy(v) for kk, v in as_float32(w).items()}
    ids = torch.from_numpy(inp["input_ids"]).reshape(-1)
    h0 = O.layer_norm(wf["embed.tok"][ids], wf["embed.norm.w"], None, cfg.norm_eps)
    h1 = h0 + O.linear(attn, wf["enc.0.wo"])
    h2 = h1 + O.linear(g, wf["enc.0.wo2"])
    qt = torch.from_numpy(inp["qtype"])
    hf = O.layer_norm(h2, wf["final_norm.w"], None, cfg.norm_eps).view(b, s, d) + wf["type_emb"][qt][:, None, :]
    err = (h.view(b, s, d) - hf).abs().amax(dim=-1)   # per token row
    print("final hidden rows: max-abs", float(err.max()), "in the last tile", float(err.view(-1)[-22:].max()))
    assert torch.isfinite(h).all()
    assert float(err.max()) < 2e-2, float(err.max())


@pytest.mark.parametrize("s,length", [(64, 64), (64, 37), (40, 40)])
def test_fused_attention_projection_matches_oracle(s, length):
    """One short sequence in bf16 runs attention inside the Wo projection and
    attn_norm / mlp_norm inside the QKV / Wi projections: whole forward
    against the oracle on a network with global and radius-64 local layers,
    full and key-padded."""
    from laya_b200.engine import NativeForward
    cfg = MICRO_LOCAL
    w = seeded_weights(cfg, seed=9)
    nf = NativeForward(0, cfg, w, "bf16", max_batch=4, max_options=8)
    try:
        items = synthetic_items([length], ["choice"], seed=21, vocab=cfg.vocab)
        inp = pack(items, 1, s, 4, cfg.pad_token_id)
        slot = nf.capture(1, s, 4, length == s)
        logits, act = nf.run(slot, inp)
        ol, oa = O.Oracle(w, cfg).forward(**inp)
        mm = inp["marker_mask"]
        assert np.abs(logits[mm] - ol[mm]).max() < 2e-2 and np.abs(act - oa).max() < 2e-2
        # the fused path is the one that ran: against the same sequence length
        # at batch 2, no attention launch per layer and no mlp_norm / attn_norm
        # launches inside the encoder
        two = nf.capture(2, s, 4, False)
        assert nf.kernel_count(slot) == nf.kernel_count(two) - cfg.layers - (2 * cfg.layers - 1)
    finally:
        nf.close()


def _sf_offset(row, g, rows_per_block, col_blocks):
    rb, r = row // rows_per_block, row % rows_per_block
    return (rb * col_blocks + (g >> 2)) * 512 + (r & 31) * 16 + (r >> 5) * 4 + (g & 3)


@pytest.mark.parametrize("intermediate, rows", [(384, ROWS_SMALL), (1920, ROWS_SMALL), (2624, ROWS_SMALL),
                                                (4096, ROWS_SMALL), (2624, ROWS_LARGE)])
def test_nvfp4_activation_quantiser_is_bit_exact(intermediate, rows):
    """The per-row NVFP4 activation quantiser (nvfp4.py:36-51 with a per-row
    outer scale) on the GEGLU output against the oracle's restatement: outer
    scales, e4m3 block scales and e2m1 codes identical."""
    from laya_b200.engine import NativeForward
    cfg = LayaConfig(layers=1, hidden=256, heads=4, intermediate=intermediate, vocab=1000, pad_token_id=999,
                     max_len=512, head_layers=0, head_heads=4, head_ff=512, act_hidden=64)
    w = seeded_weights(cfg, seed=6)
    nf = NativeForward(0, cfg, w, "nvfp4", max_batch=4, max_options=8)
    try:
        b, s, lengths = rows
        k = 4
        items = synthetic_items(lengths, ["choice", "noul", "score", "choice"][:b], seed=13, vocab=cfg.vocab)
        nf.run(nf.capture(b, s, k, False), pack(items, b, s, k, cfg.pad_token_id))
        T, K = b * s, intermediate
        col_blocks = 4 * ((K + 255) // 256)
        # token tile of the Wo2 projection at 384 tokens: 128, or 64 when the
        # 128-token grid would leave SMs idle (gemm_plan)
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        rows_per_block = 64 if (cfg.hidden // 128) * ((b * s + 127) // 128) < sms else 128
        x = bf16_of(nf.read_buffer("g", (T, K), np.uint16))
        nib = nf.read_buffer("x4", (T, K // 2), np.uint8)
        sf_bytes = ((T + rows_per_block - 1) // rows_per_block) * col_blocks * 512
        sf = nf.read_buffer("x4sf", (sf_bytes,), np.uint8)
        outer = torch.from_numpy(nf.read_buffer("x4o", (T,), np.float32))
    finally:
        nf.close()
    ref_deq, ref_outer = O.nvfp4_quantize(x, per_row=True)
    assert torch.equal(outer, ref_outer[:, 0])
    rows = np.arange(T)[:, None]
    groups = np.arange(K // 16)[None, :]
    idx = _sf_offset(rows, groups, rows_per_block, col_blocks)
    scale = torch.from_numpy(sf[idx].copy()).view(torch.float8_e4m3fn).to(torch.float32)  # [T, K/16]
    codes = np.stack([nib & 0xF, nib >> 4], axis=-1).reshape(T, K)
    grid = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)
    vals = grid[codes & 7] * np.where(codes & 8, -1.0, 1.0).astype(np.float32)
    deq = torch.from_numpy(vals).view(T, K // 16, 16) * scale[:, :, None]
    ref = ref_deq.view(T, K // 16, 16)
    assert torch.equal(deq, ref), int((deq != ref).sum())


@pytest.mark.parametrize("precision,b", [("bf16", 1), ("bf16", 2), ("fp8", 2), ("nvfp4", 2)])
def test_token_tables_match_the_computed_start(precision, b):
    """Token tables (embedding-norm and layer-0 QKV rows per id, token_tables.py
    of the reference's fast mode): the forward that starts from one gather
    matches the oracle and the forward without tables, with one launch fewer
    (gather in place of the embedding norm and the layer-0 QKV projection)."""
    from laya_b200.engine import NativeForward
    cfg = MICRO_LOCAL
    w = seeded_weights(cfg, seed=10)
    items = synthetic_items([64, 40][:b], ["choice", "noul"][:b], seed=23, vocab=cfg.vocab)
    inp = pack(items, b, 64, 4, cfg.pad_token_id)
    results = {}
    for tables in (False, True):
        nf = NativeForward(0, cfg, w, precision, max_batch=4, max_options=8)
        try:
            if tables:
                nf.build_token_tables()
            slot = nf.capture(b, 64, 4, b == 1)
            results[tables] = nf.run(slot, inp) + (nf.kernel_count(slot),)
        finally:
            nf.close()
    mm = inp["marker_mask"]
    tol = {"bf16": 2e-2, "fp8": 6e-2, "nvfp4": 1.5e-1}[precision]
    ol, oa = O.Oracle(w, cfg, precision).forward(**inp)
    (l0, a0, k0), (l1, a1, k1) = results[False], results[True]
    assert np.abs(l1[mm] - ol[mm]).max() <= tol and np.abs(a1 - oa).max() <= tol
    assert np.abs(l1[mm] - l0[mm]).max() <= tol
    assert k1 == k0 - 1


@pytest.mark.parametrize("precision", ["fp8", "nvfp4"])
@pytest.mark.parametrize("hidden, rows", [(256, (2, 192, [192, 100])), (768, (2, 192, [192, 100])),
                                          (256, (4, 512, [512, 200, 512, 64])), (768, (4, 512, [512, 511, 40, 512]))])
def test_layernorm_quantised_outputs_match_oracle(precision, hidden, rows):
    """LayerNorm rows with a quantised output (add_norm, model.py:15-19, then
    _quantize_rows / the NVFP4 quantiser) against the oracle.  Replaying only
    the row kernels leaves the MLP norm of the embedding-norm output as the
    last quantised operand.  The fp32 reduction order of the two LayerNorms
    differs from the oracle's, so a few elements round to the neighbouring
    bf16 value; everything else is identical."""
    from laya_b200.engine import NativeForward
    cfg = LayaConfig(layers=1, hidden=hidden, heads=hidden // 64, intermediate=384, vocab=1000, pad_token_id=999,
                     max_len=512, head_layers=0, head_heads=hidden // 64, head_ff=512, act_hidden=64)
    w = seeded_weights(cfg, seed=17)
    nf = NativeForward(0, cfg, w, precision, max_batch=4, max_options=8)
    try:
        b, s, lengths = rows
        k = 4
        items = synthetic_items(lengths, ["choice", "noul", "score", "choice"][:b], seed=29, vocab=cfg.vocab)
        inp = pack(items, b, s, k, cfg.pad_token_id)
        slot = nf.capture(b, s, k, False)
        nf.run(slot, inp)
        nf.replay_device(slot, 1, kernel_mask=4)
        T, d = b * s, hidden
        if precision == "fp8":
            q = torch.from_numpy(nf.read_buffer("n8", (T, d), np.uint8).copy()).view(torch.float8_e4m3fn)
            scale = torch.from_numpy(nf.read_buffer("n8s", (T,), np.float32))
        else:
            nib = nf.read_buffer("x4", (T, d // 2), np.uint8)
            outer = torch.from_numpy(nf.read_buffer("x4o", (T,), np.float32))
    finally:
        nf.close()
    wf = {kk: torch.from_numpy(v) for kk, v in as_float32(w).items()}
    ids = torch.from_numpy(inp["input_ids"]).reshape(-1)
    h0 = O.layer_norm(wf["embed.tok"][ids], wf["embed.norm.w"], None, cfg.norm_eps)
    n1 = O.bf16(O.layer_norm(h0, wf["enc.0.mlp_norm.w"], None, cfg.norm_eps))
    if precision == "fp8":
        q_ref, scale_ref = O.fp8_quantize_rows(n1)
        assert float(((scale - scale_ref[:, 0]).abs() / scale_ref[:, 0]).max()) < 1e-2
        assert float((scale != scale_ref[:, 0]).float().mean()) < 0.02
        assert float((q.to(torch.float32) != q_ref).float().mean()) < 2e-3
    else:
        _, outer_ref = O.nvfp4_quantize(n1, per_row=True)
        outer_ref = outer_ref[:, 0]
        assert float(((outer - outer_ref).abs() / outer_ref).max()) < 1e-2
        assert float((outer != outer_ref).float().mean()) < 0.02
        # e2m1 codes against the oracle's, from its block scales
        blocks = n1.reshape(T, d // 16, 16)
        sc = O.e4m3(torch.clamp(blocks.abs().amax(dim=2, keepdim=True) / (6.0 * outer_ref[:, None, None]),
                                min=2.0 ** -9))
        v_ref = O.e2m1(blocks / (sc * outer_ref[:, None, None])).reshape(T, d)
        codes = np.stack([nib & 0xF, nib >> 4], axis=-1).reshape(T, d)
        grid = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)
        v = torch.from_numpy(grid[codes & 7] * np.where(codes & 8, -1.0, 1.0).astype(np.float32))
        assert float((v != v_ref).float().mean()) < 2e-3
