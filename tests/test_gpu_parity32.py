"""Parity of the full 32-layer backbone (the benchmarked geometry) against the
CPU F32 oracle, on a subset of the config-4 batch.

32 requests of 256-512 tokens (seed 3; ids drawn from a 4096-token vocabulary
so the oracle's embedding table stays small: the gather does not depend on the
vocabulary size) run through the 32-layer benchmark geometry (hidden 2560,
[3 DeltaNet + 1 attention] x 8) with the engine's seeded BF16 weights; the
oracle receives exactly those weights and runs the reference's F32 path.

Decisions follow answers() (crates/core/src/types.rs:728-802): softmax per
group, the choice winner is the first strict maximum, noul reports p[0]; the
noul decision compared here is its side of 1/2. A winner is required to match
wherever the oracle's top-two logit gap exceeds twice the largest logit error
measured on the batch (the reference qualifies winners only above its error
bound, docs/clef-flash-verification.md:24; specs/clef-serving-design.md:629).

Two checks per precision:
  * against the oracle's F32 path: the stated logits bound of the mode, and
    decisions. The split precision (split-BF16 GEMM operands, F32 projection
    outputs; only the attention's q, k, v and probabilities are single BF16
    operands) is held to the 2e-2 logits bound. The default BF16 precision
    rounds every GEMM operand and the projection outputs to BF16; those
    roundings alone move 32-layer logits by up to ~1e-1 from the F32 path on
    this geometry (the oracle with the same rounding points against the F32
    oracle, printed as the rounding floor), so its bound is 2e-1, and on the
    requests where the floor is measured the device may be at most twice as
    far from the F32 path as the floor;
  * against the oracle run with the precision's own BF16 rounding points
    (oracle.set_rounding), on 8 requests. With few roundings (split) the two
    runs stay close, which isolates the kernels' arithmetic: <= 5e-3. With a
    BF16 rounding at every GEMM operand, rounding decisions that flip on F32
    summation-order noise cascade through 32 layers, so the two runs are only
    as close as each is to the F32 path (<= 1.5e-1).
"""
import numpy as np
import pytest

import oracle
from clef_b200 import workloads
from clef_b200.config import benchmark_config

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

VOCAB = 4096
N_REQUESTS = 32
MATCHED_REQUESTS = 8

# BF16 rounding points of each precision mode, as oracle.set_rounding masks.
ROUNDING = {
    "bf16": oracle.ROUND_OPERAND | oracle.ROUND_PROJ | oracle.ROUND_ATTN_QKV | oracle.ROUND_P,
    "split": oracle.ROUND_ATTN_QKV | oracle.ROUND_P,
}
PRECISION = {"bf16": 0, "split": 1}
LOGITS_BOUND = {"bf16": 2e-1, "split": 2e-2}
MATCHED_BOUND = {"bf16": 2e-1, "split": 5e-3}


def softmax(x):
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


@pytest.fixture(scope="module")
def model32():
    import clef_b200 as cb
    cfg = benchmark_config(layers=32, head_outputs=7)
    cfg.vocab_size = VOCAB
    eng = cb.Engine(cfg, 0)
    eng.init_random(3, 0.02)
    eng.finalize()
    ref = oracle.Model(cfg)
    for name in ref.names():
        ref.set_weight(name, eng.get_weight(name))
    ref.check()
    head_w = eng.get_weight("clef.head.weight").reshape(7, cfg.hidden_size)
    reqs = workloads.backbone_requests(n=N_REQUESTS, lo=256, hi=512, seed=3, vocab=VOCAB)
    oracle.set_rounding(0)
    f32 = np.stack([oracle.head(ref.prefill(r)[0][-1], head_w) for r in reqs])
    yield eng, ref, head_w, reqs, f32
    oracle.set_rounding(0)
    eng.close()


def decision_report(lg, ref_lg, bound):
    """Winners compared where the oracle's gap exceeds 2 * bound; returns
    (compared, matched, lines)."""
    compared = matched = 0
    lines = []
    for i in range(ref_lg.shape[0]):
        for name, sl in (("noul", slice(0, 2)), ("choice", slice(2, 6))):
            r = ref_lg[i, sl]
            top = np.sort(r)[::-1]
            gap = float(top[0] - top[1])
            same = int(np.argmax(lg[i, sl])) == int(np.argmax(r))
            if gap > 2 * bound:
                compared += 1
                matched += same
                if not same:
                    lines.append(f"request {i} {name}: MISMATCH with oracle gap {gap:.3e}")
            elif not same:
                lines.append(f"request {i} {name}: differs inside the error band (gap {gap:.3e})")
    return compared, matched, lines


@pytest.mark.parametrize("mode", ["bf16", "split"])
def test_32_layer_logits_and_decisions(model32, mode):
    eng, ref, head_w, reqs, f32 = model32
    eng.set_precision(PRECISION[mode])
    try:
        lg, _, _ = eng.prefill(reqs)
    finally:
        eng.set_precision(0)
    assert np.isfinite(lg).all()
    err = np.abs(lg - f32)
    max_err = float(err.max())
    pe = np.concatenate([np.abs(softmax(lg[:, 0:2]) - softmax(f32[:, 0:2])),
                         np.abs(softmax(lg[:, 2:6]) - softmax(f32[:, 2:6]))], 1)
    # Same rounding points on the CPU: the kernels' own arithmetic error.
    oracle.set_rounding(ROUNDING[mode])
    matched_ref = np.stack([oracle.head(ref.prefill(r)[0][-1], head_w) for r in reqs[:MATCHED_REQUESTS]])
    oracle.set_rounding(0)
    err_matched = float(np.abs(lg[:MATCHED_REQUESTS] - matched_ref).max())
    floor = float(np.abs(matched_ref - f32[:MATCHED_REQUESTS]).max())
    compared, matched, lines = decision_report(lg, f32, max_err)
    print(f"\n32 layers, {mode}: logits max-abs vs F32 {max_err:.3e} (mean {err.mean():.3e}); "
          f"vs oracle with the same rounding {err_matched:.3e}; rounding floor (oracle vs oracle) "
          f"{floor:.3e}; probabilities max {pe.max():.3e} mean {pe.mean():.3e}; "
          f"decisions compared {compared}, matched {matched}")
    for line in lines:
        print("  " + line)
    assert err_matched <= MATCHED_BOUND[mode]
    assert max_err <= LOGITS_BOUND[mode]
    assert float(err[:MATCHED_REQUESTS].max()) <= max(2 * floor, 2e-2)
    assert matched == compared
