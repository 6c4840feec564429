"""The serving paths on the GPU: one C4 step (64 questions, s ~ U[32, 512]
bucketed by 32, FP8) through the public engine API against the FP8 oracle;
the request-parallel dispatcher on one GPU against the engine it wraps; and a
bounded device wait that runs out (failure detection) without hanging or
poisoning the engine."""
import functools

import numpy as np
import pytest

from laya_b200.config import LAYA, TINY
from laya_b200.weights import seeded_weights
from laya_b200.workload import synthetic_items, pack
from oracle import laya_oracle as O

pytestmark = pytest.mark.gpu

BUCKETS = tuple(range(32, 513, 32))
TOL_FP8 = 6e-2


@functools.lru_cache(maxsize=1)
def laya_weights():
    return seeded_weights(LAYA, seed=0)


def c4_groups(seed):
    from laya_b200.dispatcher import c4_step, group_by_bucket
    from laya_b200.engine import request_from_items
    items = c4_step(seed, LAYA.vocab)
    groups = group_by_bucket(items, list(range(len(items))), BUCKETS, 64)
    return items, [(idx, request_from_items([items[i] for i in idx])) for _, idx in groups]


def test_c4_step_fp8_matches_the_fp8_oracle():
    """Every bucket group of one C4 step through B200Engine.run_prepared in
    FP8, against the FP8 oracle and the bf16 oracle on the same padded batch.
    Two FP8 forwards whose arithmetic differs only in fp32 summation order
    land a few 1e-2 apart (an activation on an e4m3 rounding boundary goes one
    way or the other and 28 layers carry it to the logits), about as far as
    the FP8 recipe itself is from bf16, and which group lands furthest is
    chance (one measured group: 0.062 from bf16 while the FP8 oracle was
    0.039, and 0.029 from the FP8 oracle).  So each group must take the FP8
    oracle's decision wherever the oracle's top-2 margin exceeds 6e-2 and lie
    within 2 x 6e-2 of the FP8 oracle, and over the whole step the GPU must be
    as accurate as the FP8 recipe: root-mean-square distance of its logits and
    act to the bf16 oracle at most 1.5 times the FP8 oracle's."""
    from laya_b200.engine import B200Engine
    items, groups = c4_groups(300)
    fp8 = O.Oracle(laya_weights(), LAYA, "fp8")
    ref = O.Oracle(laya_weights(), LAYA, "bf16")
    ours_err, oracle_err, worst = [], [], 0.0
    agree = []
    with B200Engine(config=LAYA, weights=laya_weights(), device=0, precision="fp8", max_questions=64,
                    max_options=4, max_graphs=64, sequence_buckets=BUCKETS) as eng:
        for idx, req in groups:
            logits, act, meta = eng.run_prepared(req)
            b, s, k = eng._shape(req)
            inp = pack(req.items, b, s, k, LAYA.pad_token_id)
            n = len(idx)
            ol, oa = (x[:n] for x in fp8.forward(**inp))
            bl, ba = (x[:n] for x in ref.forward(**inp))
            kk = logits.shape[1]
            mm = inp["marker_mask"][:n][:, :kk]
            ol, bl = ol[:, :kk], bl[:, :kk]
            to_oracle = max(float(np.abs(logits[mm] - ol[mm]).max()), float(np.abs(act - oa).max()))
            worst = max(worst, to_oracle)
            ours_err.append(np.concatenate([logits[mm] - bl[mm], (act - ba).ravel()]))
            oracle_err.append(np.concatenate([ol[mm] - bl[mm], (oa - ba).ravel()]))
            decided = O.top2_margin(ol, mm) > TOL_FP8
            if decided.any():
                assert O.decision_agreement(ol[decided], logits[decided], mm[decided]) == 1.0, (s, idx)
            agree.append(O.decision_agreement(ol, logits, mm))
            assert to_oracle <= 2 * TOL_FP8, (meta["shape"], to_oracle)
    rms_ours = float(np.sqrt(np.mean(np.concatenate(ours_err) ** 2)))
    rms_oracle = float(np.sqrt(np.mean(np.concatenate(oracle_err) ** 2)))
    print(f"C4 fp8 over {len(items)} questions in {len(groups)} bucket groups: worst max-abs to the fp8 oracle "
          f"{worst:.3e}; rms to the bf16 oracle {rms_ours:.3e} (fp8 oracle {rms_oracle:.3e}); "
          f"mean decision agreement with the fp8 oracle {np.mean(agree):.3f}")
    assert rms_ours <= 1.5 * rms_oracle, (rms_ours, rms_oracle)


def test_dispatcher_on_one_gpu_is_bit_identical_to_the_engine():
    """B200Dispatcher(devices=[0]) over a real engine returns exactly what a
    direct B200Engine returns for the same bucket groups of a C4 step."""
    from laya_b200.dispatcher import B200Dispatcher
    from laya_b200.engine import B200Engine
    items, groups = c4_groups(301)
    kw = dict(config=LAYA, weights=laya_weights(), precision="fp8", max_options=4, max_graphs=64)
    with B200Engine(device=0, max_questions=64, sequence_buckets=BUCKETS, **kw) as eng:
        want = {}
        for idx, req in groups:
            logits, act, _ = eng.run_prepared(req)
            for row, i in enumerate(idx):
                kq = len(items[i]["markers"])
                want[i] = (logits[row, :max(kq, 1)], act[row])
    with B200Dispatcher(devices=[0], sequence_buckets=BUCKETS, max_batch=64, **kw) as disp:
        got = disp.run_items(items)
    for i, (lg, a) in enumerate(got):
        assert np.array_equal(lg, want[i][0]) and np.array_equal(a, want[i][1]), i


def test_a_bounded_wait_that_runs_out_raises_and_the_engine_recovers():
    """Failure detection on the device: a projection whose first pipeline
    stage is never loaded (nothing completes its barrier) gives up after its
    wait limit, records the timeout and returns; the run raises RuntimeError,
    and the next run on the same engine is correct and bit-identical to the
    one before."""
    from laya_b200.engine import NativeForward
    w = seeded_weights(TINY, seed=0)
    items = synthetic_items([64, 40], ["choice", "noul"], seed=5, vocab=TINY.vocab)
    inp = pack(items, 2, 64, 4, TINY.pad_token_id)
    nf = NativeForward(0, TINY, w, "bf16", max_batch=2, max_options=4)
    try:
        slot = nf.capture(2, 64, 4, False)
        before = nf.run(slot, inp)
        nf.test_withhold_stage(wait_limit_us=2000)
        with pytest.raises(RuntimeError, match="timed out"):
            nf.run(slot, inp)
        after = nf.run(slot, inp)
        assert np.array_equal(before[0], after[0]) and np.array_equal(before[1], after[1])
        ol, oa = O.Oracle(w, TINY).forward(**inp)
        mm = inp["marker_mask"]
        assert np.abs(after[0][mm] - ol[mm]).max() <= 2e-2
    finally:
        nf.close()
