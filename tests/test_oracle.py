"""Pins the CPU F32 oracle (oracle/oracle.cpp) to the reference's own tests.

- backbone parity against the reference's golden fixture
  (crates/core/src/models/mod.rs:87-111), tolerance 1e-5 + 1e-4|e| (:75-86);
- prefix capture/resume invariants at boundaries {1, 2, 3, 8, 19}
  (mod.rs:112-171), including the byte accounting and the rejected captures;
- tiled vs dense causal attention (ops.rs:237-263);
- the recurrence against an independent float64 restatement on the
  reference's deterministic sin/cos patterns (metal.rs:741-815) and the
  decay -1000 case (chunk.rs:213).
"""
import numpy as np
import pytest

import oracle
from clef_b200.config import from_text_config


def assert_close(actual, expected):
    a = np.asarray(actual, np.float32).reshape(-1)
    e = np.asarray(expected, np.float32).reshape(-1)
    assert a.shape == e.shape
    err = np.abs(a - e)
    tol = 1e-5 + 1e-4 * np.abs(e)
    bad = ~(np.isfinite(a) & (err <= tol))
    assert not bad.any(), f"{bad.sum()} elements out of tolerance, worst {err.max()}"


@pytest.fixture(scope="module")
def fixture_model(golden):
    cfg = from_text_config(golden["config"])
    m = oracle.Model(cfg)
    for name, w in golden["weights"].items():
        if name == "lm_head.weight":  # output embeddings: used only by the span head
            continue
        m.set_weight(name, w)
    m.check()
    return m


def test_backbone_matches_reference_golden(golden, fixture_model):
    hidden, _ = fixture_model.prefill(golden["ids"])
    assert_close(hidden, golden["expected"])


def test_prefix_resume_matches_full_prefill(golden, fixture_model):
    m = fixture_model
    cfg = m.cfg
    ids = np.arange(20, dtype=np.int32)
    expected, _ = m.prefill(ids)
    width = 2 * cfg.linear_num_key_heads * cfg.linear_key_head_dim + \
        cfg.linear_num_value_heads * cfg.linear_value_head_dim

    def prefix_bytes(tokens):  # Backbone::prefix_bytes (qwen.rs:278-310), F32
        n = tokens * cfg.hidden_size * 4
        for i in range(cfg.num_hidden_layers):
            if cfg.layer_types[i]:
                n += tokens * cfg.num_key_value_heads * cfg.head_dim * 2 * 4
            else:
                n += (cfg.linear_num_value_heads * cfg.linear_key_head_dim * cfg.linear_value_head_dim
                      + (cfg.linear_conv_kernel_dim - 1) * width) * 4
        return n

    for boundary in (1, 2, 3, 8, 19):
        captured, state = m.prefill(ids, capture=boundary)
        assert_close(captured, expected)
        short = (3 - boundary) * 3 * width * 4 if boundary < 3 else 0
        assert state.bytes() == prefix_bytes(boundary) - short
        with pytest.raises(ValueError):
            m.prefill(ids[boundary:], initial=state, capture=1)
        resumed, _ = m.prefill(ids[boundary:], initial=state)
        assert_close(resumed, expected)
        changed = ids.copy()
        changed[boundary:] += 20
        resumed, _ = m.prefill(changed[boundary:], initial=state)
        full_changed, _ = m.prefill(changed)
        assert_close(resumed, full_changed)
        # Resuming never mutates the shared state.
        again, _ = m.prefill(ids[boundary:], initial=state)
        assert_close(again, expected)
    with pytest.raises(ValueError):
        m.prefill(ids, capture=20)


def test_tiled_attention_matches_dense():
    q = np.sin(np.arange(300 * 4, dtype=np.float32) * np.float32(0.013)).reshape(1, 300, 4)
    tiled = oracle.attention(q, q, q, causal=True)
    qd = q.astype(np.float64)[0]
    s = qd @ qd.T / 2.0
    s[np.triu_indices(300, 1)] = -np.inf
    p = np.exp(s - s.max(axis=1, keepdims=True))
    dense = (p / p.sum(axis=1, keepdims=True)) @ qd
    assert np.abs(tiled[0] - dense).max() < 1e-5


def recurrence_f64(q, k, v, g, beta, state=None):
    """Independent float64 restatement of delta_recurrence_prefill."""
    t, hk, kd = q.shape
    hv, vd = v.shape[1], v.shape[2]
    rep = hv // hk
    qn = q / np.sqrt((q.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6) / np.sqrt(kd)
    kn = k / np.sqrt((k.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)
    S = np.zeros((hv, kd, vd)) if state is None else state.astype(np.float64).copy()
    out = np.zeros((t, hv, vd))
    for i in range(t):
        for h in range(hv):
            key, qry = kn[i, h // rep], qn[i, h // rep]
            S[h] *= np.exp(g[i, h])
            delta = (v[i, h] - S[h].T @ key) * beta[i, h]
            S[h] += np.outer(key, delta)
            out[i, h] = S[h].T @ qry
    return out, S


@pytest.mark.parametrize("t,h,kd,vd", [(1, 1, 1, 1), (33, 2, 4, 5), (33, 2, 32, 13), (17, 2, 128, 128)])
def test_recurrence_matches_float64_on_reference_patterns(t, h, kd, vd):
    q = np.sin(np.arange(t * h * kd, dtype=np.float32) * np.float32(0.017)).reshape(t, h, kd)
    k = q * np.float32(0.7) + np.float32(0.1)
    v = np.cos(np.arange(t * h * vd, dtype=np.float32) * np.float32(0.031)).reshape(t, h, vd)
    g = np.full((t, h), -0.03, np.float32)
    beta = np.full((t, h), 0.65, np.float32)
    out, st, _ = oracle.delta_recurrence(q, k, v, g, beta)
    ref, sref = recurrence_f64(q, k, v, g, beta)
    assert np.abs(out - ref).max() < 1e-5
    assert np.abs(st - sref).max() < 1e-5


def test_recurrence_extreme_decay_and_capture():
    t, h, kd, vd = 70, 2, 16, 8
    rng = np.random.default_rng(5)
    q = rng.standard_normal((t, 1, kd)).astype(np.float32)
    k = rng.standard_normal((t, 1, kd)).astype(np.float32)
    v = rng.standard_normal((t, h, vd)).astype(np.float32)
    g = np.full((t, h), -1000.0, np.float32)
    beta = np.full((t, h), 0.65, np.float32)
    out, st, cap = oracle.delta_recurrence(q, k, v, g, beta, capture=33)
    ref, sref = recurrence_f64(q, k, v, g, beta)
    assert np.abs(out - ref).max() < 1e-5
    # Resume from the captured state reproduces the tail exactly.
    tail, st2, _ = oracle.delta_recurrence(q[33:], k[33:], v[33:], g[33:], beta[33:], state=cap)
    assert np.array_equal(tail, out[33:])
    assert np.array_equal(st2, st)


def test_gemm_matches_float64():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((37, 96)).astype(np.float32)
    w = rng.standard_normal((50, 96)).astype(np.float32)
    y = oracle.linear(x, w)
    assert np.abs(y - x.astype(np.float64) @ w.astype(np.float64).T).max() < 1e-4


def _head_fixture():
    import json
    from pathlib import Path

    from oracle.joint_head import HeadConfig, Question
    z = np.load(Path(__file__).with_name("golden") / "head_fixture.npz")
    cfg = HeadConfig(**json.loads(bytes(z["config_json"]).decode()))
    w = {k[2:]: z[k] for k in z.files if k.startswith("w:")}
    qs = [Question(k, tuple(i), [tuple(o) for o in opts])
          for k, i, opts in json.loads(bytes(z["questions_json"]).decode())]
    return z, cfg, w, qs


def test_head_oracle_matches_reference_golden():
    """oracle/joint_head.py against the reference's pinned joint-head fixture
    (models/mod.rs:176-235), tolerance 1e-5 + 1e-4|e| (:75-86)."""
    from oracle.joint_head import head_forward
    z, cfg, w, qs = _head_fixture()
    out = head_forward(w, cfg, z["in:hidden"], z["in:output_embeddings"], list(z["ids"]), qs)
    assert len(out) == 3
    for i, o in enumerate(out):
        assert_close(o, z[f"in:logits.{i}"])


@pytest.mark.parametrize("T,H", [(1, 2), (31, 2), (64, 1), (65, 2), (139, 2)])
@pytest.mark.parametrize("decay", [-0.03, -1000.0])
def test_chunk_form_matches_recurrence(T, H, decay):
    """The chunked WY/UT algebra the GPU scan evaluates (oracle/chunk_form.py)
    equals the per-token recurrence on the reference's chunk-test patterns
    (chunk.rs:182-241 inputs at key = value = 128), decay -1000 included."""
    from oracle.chunk_form import chunked_scan
    kd = vd = 128
    q = (np.sin(np.arange(T * H * kd, dtype=np.float32) * np.float32(0.071)) * np.float32(0.02)).reshape(T, H, kd)
    k = np.cos(np.arange(T * H * kd, dtype=np.float32) * np.float32(0.037)).reshape(T, H, kd)
    v = np.sin(np.arange(T * H * vd, dtype=np.float32) * np.float32(0.033)).reshape(T, H, vd)
    g = np.full((T, H), decay, np.float32)
    beta = np.full((T, H), 0.65, np.float32)
    ref_o, ref_s, _ = oracle.delta_recurrence(q, k, v, g, beta)
    o, s, _ = chunked_scan(q, k, v, g, beta)
    # F32 recurrence against the float64 chunk form: rounding noise only
    # (outputs of magnitude ~0.03, observed differences ~3e-8).
    assert np.abs(o - ref_o).max() < 1e-6
    assert np.abs(s - ref_s).max() < 1e-6


@pytest.mark.parametrize("capture", [1, 16, 63, 64, 65, 128, 140])
def test_chunk_form_capture_and_gqa(capture):
    """Captured states inside and at the end of chunks, grouped heads (two value
    heads per key head), random gates and an initial state."""
    from oracle.chunk_form import chunked_scan
    T, hk, hv, kd, vd = 140, 1, 2, 32, 16
    rng = np.random.default_rng(capture)
    q = rng.standard_normal((T, hk, kd)).astype(np.float32)
    k = rng.standard_normal((T, hk, kd)).astype(np.float32)
    v = rng.standard_normal((T, hv, vd)).astype(np.float32)
    g = (-np.exp(rng.uniform(-4, 1, (T, hv)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, hv))))).astype(np.float32)
    s0 = (0.1 * rng.standard_normal((hv, kd, vd))).astype(np.float32)
    ref_o, ref_s, ref_c = oracle.delta_recurrence(q, k, v, g, beta, state=s0, capture=capture)
    o, s, c = chunked_scan(q, k, v, g, beta, state=s0, capture=capture)
    # Magnitudes ~0.2; observed differences below 2e-7.
    assert np.abs(o - ref_o).max() < 2e-6
    assert np.abs(s - ref_s).max() < 2e-6
    assert np.abs(c - ref_c).max() < 2e-6


def test_rounding_sites_partition_the_coarse_switches(golden, fixture_model):
    """The oracle's per-site BF16 rounding switches (a measuring aid for device
    precisions) split the two coarse ones exactly: the five GEMM-operand sites
    together reproduce ROUND_OPERAND and the four projection-output sites
    ROUND_PROJ, bit for bit; every site alone moves the result; 0 is the F32 path."""
    m, ids = fixture_model, golden["ids"]
    ops = [oracle.ROUND_OP_MIX_IN, oracle.ROUND_OP_MLP_IN, oracle.ROUND_OP_DOWN, oracle.ROUND_OP_DELTA_OUT,
           oracle.ROUND_OP_ATTN_OUT]
    projs = [oracle.ROUND_PROJ_DELTA_QKV, oracle.ROUND_PROJ_ATTN, oracle.ROUND_PROJ_DELTA_Z,
             oracle.ROUND_PROJ_DELTA_AB]
    base, _ = m.prefill(ids)

    def run(mask):
        oracle.set_rounding(mask)
        try:
            return m.prefill(ids)[0]
        finally:
            oracle.set_rounding(0)

    assert np.array_equal(run(oracle.ROUND_OPERAND), run(sum(ops)))
    assert np.array_equal(run(oracle.ROUND_PROJ), run(sum(projs)))
    for bit in ops + projs:
        assert not np.array_equal(run(bit), base), bit
    assert np.array_equal(m.prefill(ids)[0], base)
    assert_close(base, golden["expected"])
