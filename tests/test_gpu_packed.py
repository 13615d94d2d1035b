"""The DeltaKernel / CachedDelta / DeltaPrepareKernel boundary in the
reference's packed layout (crates/core/src/models/metal.rs:79-413,
pointwise.rs:195-279), checked against the oracle's per-token recurrence.

Cases are the reference's own (metal.rs:735-868): q_i = sin(0.017 i), k =
0.7 q + 0.1, v_i = cos(0.031 i), g = -0.03, beta = 0.65 with the dimension
tails (T, H, dk, dv) = (1,1,1,1), (33,2,4,5), (33,2,32,13), (257,2,64,13),
(257,2,128,13), (17,2,128,128), compared at 1e-5 max-abs as the reference
does; the capture/resume case with constant inputs must reproduce the
uninterrupted run exactly (the reference asserts an error of 0). Decay -1000
per token (chunk.rs:213) packs e^g = 0, a full state reset per token.
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TAILS = [(1, 1, 1, 1), (33, 2, 4, 5), (33, 2, 32, 13), (257, 2, 64, 13), (257, 2, 128, 13), (17, 2, 128, 128)]
# Beyond the reference's tails: the widest head count (two value columns per warp) and
# an odd value width at that head count.
WIDE = [(65, 32, 128, 128), (40, 32, 64, 127)]
# Every register layout of the kernel (lanes per value column x keys per lane, with the
# paired key loads used for an even dv and the single ones for an odd dv) not covered
# above.
LAYOUTS = [(37, 3, 2, 6), (37, 3, 2, 7), (37, 3, 4, 6), (37, 3, 8, 10), (37, 3, 8, 9), (37, 3, 16, 24),
           (37, 3, 16, 3), (37, 3, 32, 40), (37, 3, 64, 66)]


def l2(x):
    x = np.asarray(x, np.float32)
    return (x / np.sqrt((x * x).sum(-1, keepdims=True, dtype=np.float32) + np.float32(1e-6))).astype(np.float32)


def reference_inputs(T, H, dk, dv, g=-0.03):
    q = np.sin(np.arange(T * H * dk, dtype=np.float32) * np.float32(0.017)).reshape(T, H, dk).astype(np.float32)
    k = (q * np.float32(0.7) + np.float32(0.1)).astype(np.float32)
    v = np.cos(np.arange(T * H * dv, dtype=np.float32) * np.float32(0.031)).reshape(T, H, dv).astype(np.float32)
    gg = np.full((T, H), g, np.float32)
    beta = np.full((T, H), 0.65, np.float32)
    return q, k, v, gg, beta


def pack(q, k, v, g, beta):
    return np.ascontiguousarray(np.concatenate([q, k, v, np.exp(g)[..., None], beta[..., None]], -1),
                                dtype=np.float32)


@pytest.mark.parametrize("T,H,dk,dv", TAILS + WIDE + LAYOUTS)
def test_packed_recurrence_matches_oracle(T, H, dk, dv):
    import clef_b200 as cb
    q, k, v, g, beta = reference_inputs(T, H, dk, dv)
    # The caller normalises q and k before packing (qwen.rs:837-845).
    qn = (l2(q) * np.float32(1.0 / np.sqrt(dk))).astype(np.float32)
    kn = l2(k)
    o, _ = cb.delta_packed(torch.from_numpy(pack(qn, kn, v, g, beta)).cuda(), dk, dv)
    want, _, _ = oracle.delta_recurrence(q, k, v, g, beta)
    err = float(np.abs(o.cpu().numpy() - want).max())
    print(f"packed {T}/{H}/{dk}/{dv}: max-abs {err:.2e}")
    assert err < 1e-5


@pytest.mark.parametrize("dk,dv", [(4, 5), (128, 128), (128, 13), (64, 64), (8, 8)])
def test_packed_capture_and_resume_are_exact(dk, dv):
    import clef_b200 as cb
    T, H = 257, 2
    q = np.full((T, H, dk), 0.01, np.float32)
    k = np.full((T, H, dk), 0.088, np.float32)
    v = np.full((T, H, dv), 0.25, np.float32)
    g = np.full((T, H), -0.03, np.float32)
    beta = np.full((T, H), 0.65, np.float32)
    packed = torch.from_numpy(pack(q, k, v, g, beta)).cuda()
    full, _ = cb.delta_packed(packed, dk, dv)
    for boundary in (1, 16, 256):
        o, state = cb.delta_packed(packed, dk, dv, capture=boundary)
        assert torch.equal(o, full)
        tail, _ = cb.delta_packed(packed[boundary:].contiguous(), dk, dv, initial=state.contiguous())
        assert torch.equal(tail, full[boundary:])
    # The captured state is the state after 16 tokens of the same (raw,
    # unnormalised) inputs, evaluated in float64.
    _, state = cb.delta_packed(packed, dk, dv, capture=16)
    S = np.zeros((H, dk, dv), np.float64)
    for t in range(16):
        S *= np.exp(np.float64(-0.03))
        d = (0.25 - np.einsum("hkv,k->hv", S, np.full(dk, 0.088))) * 0.65
        S += 0.088 * d[:, None, :]
    assert np.abs(state.cpu().numpy() - S).max() < 1e-5


def test_packed_decay_minus_1000_resets_the_state():
    import clef_b200 as cb
    T, H, dk, dv = 300, 2, 128, 128
    q, k, v, _, beta = reference_inputs(T, H, dk, dv)
    g = np.full((T, H), -1000.0, np.float32)
    qn = (l2(q) * np.float32(1.0 / np.sqrt(dk))).astype(np.float32)
    o, _ = cb.delta_packed(torch.from_numpy(pack(qn, l2(k), v, g, beta)).cuda(), dk, dv)
    want, _, _ = oracle.delta_recurrence(q, k, v, g, beta)
    assert float(np.abs(o.cpu().numpy() - want).max()) < 1e-5


def test_packed_resume_from_an_initial_state_matches_oracle():
    import clef_b200 as cb
    T, H, dk, dv = 200, 3, 64, 40
    q, k, v, g, beta = reference_inputs(T, H, dk, dv)
    init = (0.1 * np.random.default_rng(0).standard_normal((H, dk, dv))).astype(np.float32)
    qn = (l2(q) * np.float32(1.0 / np.sqrt(dk))).astype(np.float32)
    o, _ = cb.delta_packed(torch.from_numpy(pack(qn, l2(k), v, g, beta)).cuda(), dk, dv,
                           initial=torch.from_numpy(init).cuda())
    want, _, _ = oracle.delta_recurrence(q, k, v, g, beta, state=init)
    assert float(np.abs(o.cpu().numpy() - want).max()) < 1e-5


def test_prepare_packed_layout():
    """DeltaPrepareKernel: L2 and scale of q and k, head repetition, e^g."""
    import clef_b200 as cb
    T, Hk, Hv = 70, 16, 32
    rng = np.random.default_rng(3)
    mixed = rng.standard_normal((T, (2 * Hk + Hv) * 128)).astype(np.float32)
    g = -np.abs(rng.standard_normal((T, Hv))).astype(np.float32)
    beta = rng.uniform(0, 1, (T, Hv)).astype(np.float32)
    out = cb.delta_prepare_packed(torch.from_numpy(mixed).cuda(), torch.from_numpy(g).cuda(),
                                  torch.from_numpy(beta).cuda(), Hk, Hv).cpu().numpy()
    q = mixed[:, :Hk * 128].reshape(T, Hk, 128)
    k = mixed[:, Hk * 128:2 * Hk * 128].reshape(T, Hk, 128)
    v = mixed[:, 2 * Hk * 128:].reshape(T, Hv, 128)
    rep = np.arange(Hv) // (Hv // Hk)
    want = np.concatenate([l2(q)[:, rep] / np.sqrt(128), l2(k)[:, rep], v, np.exp(g)[..., None],
                           beta[..., None]], -1)
    assert out.shape == (T, Hv, 386)
    assert np.abs(out - want).max() <= 1e-6
    # Prepared rows feed the packed recurrence directly (the reference's
    # prepared_prefill path, metal.rs:201-252).
    o, _ = cb.delta_packed(torch.from_numpy(out).cuda(), 128, 128)
    ref, _, _ = oracle.delta_recurrence(q, k, v, g, beta)
    assert float(np.abs(o.cpu().numpy() - ref).max()) < 1e-4
