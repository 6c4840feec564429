"""Seeded synthetic requests in the shape the reference's engine consumes.

The reference measures on no public dataset; its fixtures
(``src/laya_blackwell/workloads.py``) need the checkpoint's tokenizer, which is
absent.  These generators produce already-tokenised prepared items
(``{"ids", "markers", "qtype"}``, the item format of
``protocol.prepare_request``, ``src/laya_blackwell/protocol.py:96-99``):

* token ids uniform in ``[0, vocab)``;
* ``markers``: distinct positions in ``[1, len)``, sorted;
* question kinds: ``choice`` (4 options), ``noul`` (2), ``score`` (3 criteria),
  ``qtype`` ints ``choice=0, score=1, noul=2`` (the real ``QTYPES`` values live
  in the absent ``laya`` SDK; the forward only uses them to index ``type_emb``).
"""
import numpy as np

KINDS = {"choice": (0, 4), "score": (1, 3), "noul": (2, 2)}


def make_item(rng, length, kind, vocab):
    qtype, k = KINDS[kind]
    if length < k + 1:
        raise ValueError("sequence too short for its option markers")
    ids = rng.integers(0, vocab, size=length).tolist()
    markers = sorted(rng.choice(np.arange(1, length), size=k, replace=False).tolist())
    return {"ids": ids, "markers": markers, "qtype": qtype}


def synthetic_items(lengths, kinds, seed, vocab):
    rng = np.random.Generator(np.random.PCG64(seed))
    return [make_item(rng, n, kind, vocab) for n, kind in zip(lengths, kinds)]


def mixed_kinds(n, seed):
    rng = np.random.Generator(np.random.PCG64(seed + 7919))
    names = list(KINDS)
    return [names[i] for i in rng.integers(0, len(names), size=n)]


def pack(items, batch, length, options, pad_token_id):
    """Padded int64/bool arrays with ``BlackwellEngine._fill`` semantics
    (``src/laya_blackwell/engine.py:140-153``): pad ids, dummy batch rows keep
    one valid token and one valid option."""
    ids = np.full((batch, length), pad_token_id, dtype=np.int64)
    mask = np.zeros((batch, length), dtype=np.int64)
    mpos = np.zeros((batch, options), dtype=np.int64)
    mmask = np.zeros((batch, options), dtype=bool)
    qtype = np.zeros(batch, dtype=np.int64)
    mask[:, 0] = 1
    mmask[:, 0] = True
    for i, item in enumerate(items):
        n, k = len(item["ids"]), len(item["markers"])
        ids[i, :n] = item["ids"]
        mask[i, :n] = 1
        mpos[i, :k] = item["markers"]
        mmask[i, :k] = True
        qtype[i] = item["qtype"]
    return {"input_ids": ids, "attention_mask": mask, "marker_pos": mpos,
            "marker_mask": mmask, "qtype": qtype}
