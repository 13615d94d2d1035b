"""End-to-end prefill on the B200 against the CPU F32 oracle.

The engine draws its seeded BF16 weights on the device; the oracle receives
exactly those values (exported through clef_engine_get_weight) and runs the
reference's F32 path. Geometry: the benchmark dimensions (hidden 2560,
16/32 DeltaNet heads of 128, 16/4 attention heads of 256, intermediate 9216)
with one [3 x DeltaNet + 1 x attention] block group; a reduced vocabulary
keeps the oracle's embedding table small (the gather does not depend on it).

Tolerances: final hidden states relative RMS <= 2e-2 and max-abs <= 1e-1
(BF16 projection inputs vs F32 everywhere); schema-head probabilities
max-abs <= 1e-2 and mean-abs <= 2e-3, the reference's stated gate for a BF16
CUDA profile (specs/clef-serving-design.md:627); raw logits max-abs is
reported. Packing requests together, capturing a prefix, and resuming from a
64-token-aligned prefix are bit-exact; resuming inside a chunk stays within
the BF16 bounds (hidden relative RMS <= 1e-2 against the uninterrupted run).
"""
import numpy as np
import pytest

import oracle
from clef_b200.config import benchmark_config

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def models():
    import clef_b200 as cb
    cfg = benchmark_config(layers=4, head_outputs=7)
    cfg.vocab_size = 4096
    eng = cb.Engine(cfg, 0)
    eng.init_random(2, 0.02)
    eng.finalize()
    ref = oracle.Model(cfg)
    for name in ref.names():
        ref.set_weight(name, eng.get_weight(name))
    ref.check()
    yield cfg, eng, ref
    eng.close()


def probs(lg):
    """Softmax over the noul (2) and choice (4) groups, as answers() does."""
    lg = np.asarray(lg, np.float64).reshape(-1, 7)
    out = []
    for a, b in ((0, 2), (2, 6)):
        x = lg[:, a:b] - lg[:, a:b].max(1, keepdims=True)
        e = np.exp(x)
        out.append(e / e.sum(1, keepdims=True))
    return np.concatenate(out, 1)


def ids(n, seed):
    return np.random.default_rng(seed).integers(0, 4096, n).astype(np.int32)


# BF16 rounding points of each engine precision, as oracle.set_rounding masks:
# the default rounds every GEMM operand and the projection outputs; the split
# precision keeps only the attention's q, k, v and probabilities in BF16.
ROUNDING = {0: oracle.ROUND_OPERAND | oracle.ROUND_PROJ | oracle.ROUND_ATTN_QKV | oracle.ROUND_P,
            1: oracle.ROUND_ATTN_QKV | oracle.ROUND_P}


@pytest.mark.parametrize("precision", [0, 1], ids=["bf16", "split"])
def test_block_group_matches_oracle(models, precision):
    """Against the F32 oracle: hidden rel-RMS and probabilities within the
    gates above; logits max-abs <= 2e-2 in both precisions at this depth.
    Against the oracle with the precision's own rounding points: logits
    max-abs <= 5e-3 in the split precision (the kernels' arithmetic alone);
    in the BF16 precision rounding decisions that flip on F32 summation-order
    noise cascade, so the two runs agree only to 2e-2."""
    cfg, eng, ref = models
    seq = ids(300, 1)
    eng.set_precision(precision)
    try:
        lg, hid, _ = eng.prefill([seq], hidden=True)
    finally:
        eng.set_precision(0)
    rh, _ = ref.prefill(seq)
    head_w = eng.get_weight("clef.head.weight").reshape(7, cfg.hidden_size)
    rl = oracle.head(rh[-1], head_w)
    oracle.set_rounding(ROUNDING[precision])
    try:
        rm, _ = ref.prefill(seq)
    finally:
        oracle.set_rounding(0)
    rml = oracle.head(rm[-1], head_w)
    err_h = np.abs(hid - rh).max()
    rel = np.sqrt(((hid - rh) ** 2).mean() / (rh ** 2).mean())
    err_l = np.abs(lg[0] - rl).max()
    err_m = np.abs(lg[0] - rml).max()
    rel_m = np.sqrt(((hid - rm) ** 2).mean() / (rm ** 2).mean())
    pe = np.abs(probs(lg) - probs(rl[None]))
    print(f"precision {precision}: hidden max-abs {err_h:.3e} rel-rms {rel:.3e} logits max-abs {err_l:.3e} "
          f"prob max {pe.max():.3e}; vs same-rounding oracle rel-rms {rel_m:.3e} logits {err_m:.3e}")
    assert np.isfinite(hid).all()
    assert rel <= (2e-2 if precision == 0 else 2e-3) and err_h <= 1e-1
    assert pe.max() <= 1e-2 and pe.mean() <= 2e-3
    assert err_l <= 2e-2
    assert err_m <= (2e-2 if precision == 0 else 5e-3)


def test_packed_batch_is_bit_exact(models):
    cfg, eng, _ = models
    seqs = [ids(n, 10 + n) for n in (1, 64, 65, 300, 129)]
    lg, _, _ = eng.prefill(seqs)
    for i, s in enumerate(seqs):
        single, _, _ = eng.prefill([s])
        assert np.array_equal(lg[i], single[0]), i


@pytest.mark.parametrize("boundary", [1, 3, 64, 100, 128, 200])
def test_prefix_capture_and_resume(models, boundary):
    cfg, eng, ref = models
    seq = ids(200 + 57, 3)
    full_lg, full_h, _ = eng.prefill([seq], hidden=True)
    cap_lg, cap_h, prefix = eng.prefill([seq], capture=boundary, hidden=True)
    assert np.array_equal(cap_h, full_h) and np.array_equal(cap_lg, full_lg)
    assert prefix.tokens == boundary
    lg, hid, _ = eng.prefill([seq[boundary:]], initial=prefix, hidden=True)
    assert hid.shape == full_h.shape
    assert np.array_equal(hid[:boundary], full_h[:boundary])
    err = np.abs(hid - full_h).max()
    print(f"resume at {boundary}: hidden max-abs vs full {err:.3e}")
    if boundary % 64 == 0:
        assert np.array_equal(hid, full_h) and np.array_equal(lg, full_lg)
    else:
        # A boundary inside a 64-token chunk changes the chunking of the
        # suffix, so the BF16 activations differ at rounding level.
        rel_full = np.sqrt(((hid - full_h) ** 2).mean() / (full_h ** 2).mean())
        assert err <= 5e-2 and rel_full <= 1e-2
        assert np.abs(probs(lg) - probs(full_lg)).max() <= 1e-2
    # The oracle's resume on the same weights agrees too.
    _, rstate = ref.prefill(seq, capture=boundary)
    rh, _ = ref.prefill(seq[boundary:], initial=rstate)
    rel = np.sqrt(((hid - rh) ** 2).mean() / (rh ** 2).mean())
    assert rel <= 2e-2
    # Many suffixes continue from one shared prefix.
    tails = [ids(n, 40 + n) for n in (5, 80)]
    lgs, _, _ = eng.prefill(tails, initial=prefix)
    for i, t in enumerate(tails):
        one, _, _ = eng.prefill([t], initial=prefix)
        assert np.array_equal(lgs[i], one[0])
    prefix.close()


@pytest.mark.parametrize("boundary", [3, 100])
def test_prefix_moves_through_a_device_copy(models, boundary):
    """clef_prefix_export / clef_prefix_create / clef_prefix_import (the path of
    the multi-GPU prefix broadcast): a prefix rebuilt from a copy of another's
    device allocation continues every suffix bit for bit like the original."""
    cfg, eng, ref = models
    seq = ids(200 + 57, 3)
    _, _, prefix = eng.prefill([seq], capture=boundary)
    span = prefix.span_bytes()
    assert span >= prefix.bytes() > 0
    buf = torch.empty(span, dtype=torch.uint8, device="cuda")
    prefix.export_to(buf)
    twin = eng.create_prefix(boundary)
    assert twin.tokens == boundary and twin.span_bytes() == span
    twin.import_from(buf)
    torch.cuda.synchronize()
    tails = [seq[boundary:], ids(80, 41)]
    a, ha, _ = eng.prefill(tails[:1], initial=prefix, hidden=True)
    b, hb, _ = eng.prefill(tails[:1], initial=twin, hidden=True)
    assert np.array_equal(a, b) and np.array_equal(ha, hb)
    a, _, _ = eng.prefill(tails, initial=prefix)
    b, _, _ = eng.prefill(tails, initial=twin)
    assert np.array_equal(a, b)
    import clef_b200 as cb
    with pytest.raises(cb.ClefError, match="span"):
        twin.import_from(buf[:-16])
    twin.close()
    prefix.close()


@pytest.mark.parametrize("boundary", [4160, 8192])
def test_prefix_beyond_4096_tokens(models, boundary):
    """Prefix state past the reference's 4096-token cap: capture after
    `boundary` tokens (64-aligned), resume a 300-token suffix. The resumed
    run equals the uninterrupted one bit for bit (the reference demands zero
    drift, docs/clef-flash-prefix-reuse.md:66), also after the prefix went
    through clef_prefix_export / clef_prefix_import; in the split precision
    the resumed hidden rows match the oracle's own capture and resume
    (Backbone::prefill, qwen.rs:337-364; models/mod.rs:116-171) within 2e-3
    relative RMS and its logits within 2e-2."""
    import clef_b200 as cb
    cfg, eng, ref = models
    seq = np.random.default_rng(boundary).integers(0, cfg.vocab_size, boundary + 300).astype(np.int32)
    full_lg, full_h, _ = eng.prefill([seq], hidden=True)
    _, _, prefix = eng.prefill([seq], capture=boundary)
    lg, hid, _ = eng.prefill([seq[boundary:]], initial=prefix, hidden=True)
    assert np.array_equal(hid, full_h) and np.array_equal(lg, full_lg)
    buf = torch.empty(prefix.span_bytes(), dtype=torch.uint8, device="cuda")
    prefix.export_to(buf)
    twin = eng.create_prefix(boundary)
    twin.import_from(buf)
    lg2, hid2, _ = eng.prefill([seq[boundary:]], initial=twin, hidden=True)
    assert np.array_equal(hid2, full_h) and np.array_equal(lg2, full_lg)
    twin.close()
    prefix.close()
    eng.set_precision(cb.PRECISION_SPLIT)
    try:
        _, _, prefix = eng.prefill([seq], capture=boundary)
        lg, hid, _ = eng.prefill([seq[boundary:]], initial=prefix, hidden=True)
        prefix.close()
    finally:
        eng.set_precision(cb.PRECISION_BF16)
    _, rstate = ref.prefill(seq, capture=boundary)
    rh, _ = ref.prefill(seq[boundary:], initial=rstate)
    head_w = eng.get_weight("clef.head.weight").reshape(7, cfg.hidden_size)
    rel = np.sqrt(((hid[boundary:] - rh[boundary:]) ** 2).mean() / (rh[boundary:] ** 2).mean())
    err_l = np.abs(lg[0] - oracle.head(rh[-1], head_w)).max()
    print(f"prefix {boundary}: resumed suffix vs oracle rel-rms {rel:.3e} logits {err_l:.3e}")
    assert rel <= 2e-3 and err_l <= 2e-2


def test_prefix_import_checks_the_layout(models):
    """A created prefix cannot seed a prefill before it is filled, and an
    import of a copy made for another layout (here: the same span, but the
    attention layer first instead of last) is refused and leaves it unfilled."""
    import clef_b200 as cb
    cfg, eng, _ = models
    seq = ids(257, 3)
    _, _, prefix = eng.prefill([seq], capture=100)
    empty = eng.create_prefix(100)
    with pytest.raises(cb.ClefError, match="no state"):
        eng.prefill([seq[100:]], initial=empty)
    other_cfg = benchmark_config(layers=4, head_outputs=7)
    other_cfg.vocab_size = 4096
    for i, kind in enumerate((1, 0, 0, 0)):
        other_cfg.layer_types[i] = kind
    other = cb.Engine(other_cfg, 0)
    other.init_random(2, 0.02)
    other.finalize()
    foreign = other.create_prefix(100)
    assert foreign.span_bytes() == prefix.span_bytes()
    buf = torch.empty(prefix.span_bytes(), dtype=torch.uint8, device="cuda")
    prefix.export_to(buf)
    with pytest.raises(cb.ClefError, match="another layout"):
        foreign.import_from(buf)
    with pytest.raises(cb.ClefError, match="no state"):
        other.prefill([seq[100:]], initial=foreign)
    empty.import_from(buf)
    a, _, _ = eng.prefill([seq[100:]], initial=empty)
    b, _, _ = eng.prefill([seq[100:]], initial=prefix)
    assert np.array_equal(a, b)
    for p in (foreign, empty, prefix):
        p.close()
    other.close()


def test_decisions_match_oracle(models):
    import clef_b200 as cb
    cfg, eng, ref = models
    head_w = eng.get_weight("clef.head.weight").reshape(7, cfg.hidden_size)
    seqs = [ids(n, 100 + n) for n in (40, 90, 150)]
    lg, _, _ = eng.prefill(seqs)
    ref_lg = np.stack([oracle.head(ref.prefill(s)[0][-1], head_w) for s in seqs])
    got, want = cb.decide(lg), cb.decide(ref_lg)
    for i, (a, b) in enumerate(zip(got, want)):
        margin = np.sort(ref_lg[i, 2:6])[-1] - np.sort(ref_lg[i, 2:6])[-2]
        if margin > 2 * 2e-2:
            assert a.choice == b.choice, (i, margin)
        assert abs(a.noul - b.noul) <= 1e-2
        assert abs(a.score - b.score) <= 5e-2


def test_sm_limit_changes_nothing_but_placement(models):
    """clef_engine_set_sm_limit: the persistent kernels on fewer SMs compute
    the same tiles and sequences, so the logits are bit-identical."""
    cfg, eng, _ = models
    seqs = [ids(n, 60 + n) for n in (300, 129, 64)]
    want, _, _ = eng.prefill(seqs)
    for sms in (74, 10):
        eng.set_sm_limit(sms)
        try:
            got, _, _ = eng.prefill(seqs)
        finally:
            eng.set_sm_limit(0)
        assert np.array_equal(got, want), sms


def test_cancel_between_layers(models):
    import clef_b200 as cb
    cfg, eng, _ = models
    eng.cancel(True)
    with pytest.raises(cb.ClefError) as e:
        eng.prefill([ids(10, 5)])
    assert e.value.code == 5
    eng.cancel(False)
    lg, _, _ = eng.prefill([ids(10, 5)])
    assert np.isfinite(lg).all()


def test_every_tensor_initialised_on_a_large_model():
    """A 3 GB weight blob (full vocabulary, two attention layers): every tensor
    holds its seeded values and the head reads them (regression: the zeroing
    of the blob must be ordered before the first weight write)."""
    import clef_b200 as cb
    from clef_b200.config import weight_shapes
    cfg = benchmark_config(layers=8, head_outputs=7)
    eng = cb.Engine(cfg, 0)
    eng.init_random(3, 0.02)
    eng.finalize()
    for name in weight_shapes(cfg):
        if "embed_tokens" in name:
            continue
        assert np.abs(eng.get_weight(name)).max() > 0, name
    seq = np.random.default_rng(0).integers(0, cfg.vocab_size, 300).astype(np.int32)
    lg, hid, _ = eng.prefill([seq], hidden=True)
    w = eng.get_weight("clef.head.weight").reshape(7, cfg.hidden_size)
    assert np.abs(lg[0] - w @ hid[-1]).max() <= 1e-4
    eng.close()


def test_flash_geometry_block_group_matches_oracle():
    """The released Flash geometry (hidden 4096, intermediate 12288; the dims of
    crates/core/fixtures/release/flash-config.json) through one block group on
    four records packed together. The released weights themselves are absent
    here; this checks that the engine and its kernels handle the geometry the
    reference's published numbers are quoted on.

    Gated: hidden relative RMS <= 2e-2 per record (as for the benchmark
    geometry) and the choice winner wherever the oracle's top-two probability
    gap exceeds 2e-2 (twice the BF16 maximum error, the reference's winner rule,
    specs/clef-serving-design.md:629). The reference's probability gates
    (max 1e-2, mean 2e-3) are defined against its matching BF16 profile over
    at least 100 records, which this F32 oracle on random weights is not; the
    probability errors are reported. The split precision is also run and held
    to hidden rel-RMS <= 2e-3 and logits max-abs <= 2e-2 per record."""
    import clef_b200 as cb
    from clef_b200.config import flash_config
    cfg = flash_config(layers=4, head_outputs=7)
    cfg.vocab_size = 4096
    eng = cb.Engine(cfg, 0)
    eng.init_random(5, 0.02)
    eng.finalize()
    ref = oracle.Model(cfg)
    for name in ref.names():
        ref.set_weight(name, eng.get_weight(name))
    ref.check()
    head_w = eng.get_weight("clef.head.weight").reshape(7, cfg.hidden_size)
    seqs = [ids(n, 7 + n) for n in (200, 64, 131, 90)]
    lg, hid, _ = eng.prefill(seqs, hidden=True)
    eng.set_precision(cb.PRECISION_SPLIT)
    lg_s, hid_s, _ = eng.prefill(seqs, hidden=True)
    eng.close()
    off = np.cumsum([0] + [len(q) for q in seqs])
    worst = 0.0
    for i, q in enumerate(seqs):
        rh, _ = ref.prefill(q)
        h = hid[off[i]:off[i + 1]]
        rel = np.sqrt(((h - rh) ** 2).mean() / (rh ** 2).mean())
        p_eng, p_ref = probs(lg[i]), probs(oracle.head(rh[-1], head_w)[None])
        pe = np.abs(p_eng - p_ref)
        worst = max(worst, float(pe.max()))
        top = np.sort(p_ref[0, 2:6])[::-1]
        print(f"flash geometry record {i}: hidden rel-rms {rel:.3e} prob max {pe.max():.3e} "
              f"mean {pe.mean():.3e} choice gap {top[0] - top[1]:.3e}")
        assert np.isfinite(h).all() and rel <= 2e-2
        if top[0] - top[1] > 2e-2:
            assert np.argmax(p_eng[0, 2:6]) == np.argmax(p_ref[0, 2:6])
        # Split precision at the released geometry: F32-class projections.
        hs = hid_s[off[i]:off[i + 1]]
        rel_s = np.sqrt(((hs - rh) ** 2).mean() / (rh ** 2).mean())
        err_s = np.abs(lg_s[i] - oracle.head(rh[-1], head_w)).max()
        print(f"flash geometry record {i}, split: hidden rel-rms {rel_s:.3e} logits max-abs {err_s:.3e}")
        assert rel_s <= 2e-3 and err_s <= 2e-2
    print(f"flash geometry: worst probability error {worst:.3e}")


def test_config3_block_group_full_size_matches_oracle():
    """Config 3 at its stated size: one random-init block group
    (3 DeltaNet + 1 attention layer, benchmark dims), a single 4096-token
    sequence with ids uniform over the full 248320-token vocabulary, weights
    N(0, 0.02) drawn by the engine with seed 2, against the F32 oracle on the
    same weights. Both precisions: hidden rel-RMS <= 2e-2 (BF16) / 2e-3
    (split), probabilities max <= 1e-2, logits max-abs <= 2e-2."""
    import clef_b200 as cb
    cfg = benchmark_config(layers=4, head_outputs=7)
    eng = cb.Engine(cfg, 0)
    eng.init_random(2, 0.02)
    eng.finalize()
    ref = oracle.Model(cfg)
    for name in ref.names():
        ref.set_weight(name, eng.get_weight(name))
    ref.check()
    seq = np.random.default_rng(2).integers(0, cfg.vocab_size, 4096).astype(np.int32)
    out = {}
    for precision in (cb.PRECISION_BF16, cb.PRECISION_SPLIT):
        eng.set_precision(precision)
        out[precision] = eng.prefill([seq], hidden=True)[:2]
    head_w = eng.get_weight("clef.head.weight").reshape(7, cfg.hidden_size)
    eng.close()
    rh, _ = ref.prefill(seq)
    rl = oracle.head(rh[-1], head_w)
    for precision, (lg, hid) in out.items():
        rel = np.sqrt(((hid - rh) ** 2).mean() / (rh ** 2).mean())
        pe = np.abs(probs(lg) - probs(rl[None]))
        err_l = np.abs(lg[0] - rl).max()
        print(f"config3 T=4096 precision {precision}: hidden rel-rms {rel:.3e} max-abs {np.abs(hid - rh).max():.3e} "
              f"logits max-abs {err_l:.3e} prob max {pe.max():.3e}")
        assert np.isfinite(hid).all() and rel <= (2e-2 if precision == cb.PRECISION_BF16 else 2e-3)
        assert pe.max() <= 1e-2 and err_l <= 2e-2
