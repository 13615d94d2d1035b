"""Chunked DeltaNet scan on the B200 against the oracle's per-token F32
recurrence (delta_recurrence_prefill, qwen.rs:826-882).

Tolerances: 1e-3 max-abs on config 1 (the per-op F32 bound of the north
star); 1e-4 on the reference's deterministic chunk-test patterns
(chunk.rs:177-238, which asserts 1e-5 on Apple hardware), including decay
-1000. Packing sequences and resuming from a captured state are bit-exact
where the chunking is identical.
"""
import numpy as np
import pytest

import oracle
from clef_b200 import workloads

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_scan(qs, ks, v, g, beta, **kw):
    import clef_b200 as cb
    out, cap, fin = cb.delta_scan(dev(qs), dev(ks), dev(v), dev(g), dev(beta), **kw)
    torch.cuda.synchronize()
    return (out.cpu().numpy(), None if cap is None else cap.cpu().numpy(),
            None if fin is None else fin.cpu().numpy())


def test_config1_operator_matches_recurrence():
    inp = workloads.delta_operator_inputs()
    ref_o, ref_s, _ = oracle.delta_recurrence(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"])
    qs, ks = workloads.scan_operands(inp)
    o, _, fin = run_scan(qs, ks, inp["v"], inp["g"], inp["beta"], final_state=True)
    err_o = np.abs(o - ref_o).max()
    err_s = np.abs(fin[0] - ref_s).max()
    print(f"config1 max-abs: o {err_o:.3e} state {err_s:.3e}")
    assert np.isfinite(o).all()
    assert err_o <= 1e-3 and err_s <= 1e-3


@pytest.mark.parametrize("T,H", [(1, 2), (31, 2), (32, 1), (33, 2), (64, 1), (65, 2), (139, 2),
                                 (512, 2), (1024, 1)])
@pytest.mark.parametrize("decay", [-0.03, -1000.0])
def test_reference_chunk_patterns(T, H, decay):
    """chunk.rs:182-241 inputs at key = value = 128."""
    kd = vd = 128
    q = (np.sin(np.arange(T * H * kd, dtype=np.float32) * np.float32(0.071)) * np.float32(0.02)).reshape(T, H, kd)
    k = np.cos(np.arange(T * H * kd, dtype=np.float32) * np.float32(0.037)).reshape(T, H, kd)
    k = workloads._l2(k)
    v = np.sin(np.arange(T * H * vd, dtype=np.float32) * np.float32(0.033)).reshape(T, H, vd)
    g = np.full((T, H), decay, np.float32)
    beta = np.full((T, H), 0.65, np.float32)
    ref_o, ref_s, _ = oracle.delta_recurrence(q, k, v, g, beta)
    qs, ks = workloads.scan_operands({"q": q, "k": k})
    o, _, fin = run_scan(qs, ks, v, g, beta, final_state=True)
    err = max(np.abs(o - ref_o).max(), np.abs(fin[0] - ref_s).max())
    print(f"T={T} H={H} decay={decay}: {err:.3e}")
    assert err <= 1e-4


def test_packed_sequences_equal_separate_runs():
    inp = workloads.delta_operator_inputs(T=700, seed=11)
    qs, ks = workloads.scan_operands(inp)
    cu = np.array([0, 1, 65, 200, 700], np.int64)
    o, _, fin = run_scan(qs, ks, inp["v"], inp["g"], inp["beta"], cu_seqlens=cu, final_state=True)
    for s in range(4):
        a, b = cu[s], cu[s + 1]
        os_, _, fs = run_scan(qs[a:b], ks[a:b], inp["v"][a:b], inp["g"][a:b], inp["beta"][a:b],
                              final_state=True)
        assert np.array_equal(o[a:b], os_)
        assert np.array_equal(fin[s], fs[0])


@pytest.mark.parametrize("boundary", [1, 16, 63, 64, 65, 128, 256, 257])
def test_capture_and_resume(boundary):
    T = 257
    inp = workloads.delta_operator_inputs(T=T, seed=12)
    qs, ks = workloads.scan_operands(inp)
    ref_o, ref_s, ref_cap = oracle.delta_recurrence(inp["q"], inp["k"], inp["v"], inp["g"],
                                                    inp["beta"], capture=boundary)
    plain, _, plain_fin = run_scan(qs, ks, inp["v"], inp["g"], inp["beta"], final_state=True)
    o, cap, fin = run_scan(qs, ks, inp["v"], inp["g"], inp["beta"], capture=boundary,
                           final_state=True)
    # Capturing never changes the computation.
    assert np.array_equal(o, plain) and np.array_equal(fin, plain_fin)
    assert np.abs(cap - ref_cap).max() <= 1e-4
    assert np.abs(o - ref_o).max() <= 1e-4
    if boundary == T:
        assert np.array_equal(cap, fin[0])
        return
    tail, _, fin2 = run_scan(qs[boundary:], ks[boundary:], inp["v"][boundary:], inp["g"][boundary:],
                             inp["beta"][boundary:], init_state=dev(cap[None]), final_state=True)
    if boundary % 64 == 0:
        # Same chunk boundaries as the uninterrupted run: bit-exact continuation.
        assert np.array_equal(tail, o[boundary:])
        assert np.array_equal(fin2[0], fin[0])
    else:
        assert np.abs(tail - o[boundary:]).max() <= 1e-4
        assert np.abs(fin2[0] - fin[0]).max() <= 1e-4


def test_shared_initial_state_for_many_sequences():
    inp = workloads.delta_operator_inputs(T=300, seed=13)
    qs, ks = workloads.scan_operands(inp)
    rng = np.random.default_rng(3)
    S0 = (0.1 * rng.standard_normal((32, 128, 128))).astype(np.float32)
    cu = np.array([0, 100, 300], np.int64)
    o, _, _ = run_scan(qs, ks, inp["v"], inp["g"], inp["beta"], cu_seqlens=cu,
                       init_state=dev(S0), init_shared=True)
    for s in range(2):
        a, b = cu[s], cu[s + 1]
        ref, _, _ = oracle.delta_recurrence(inp["q"][a:b], inp["k"][a:b], inp["v"][a:b],
                                            inp["g"][a:b], inp["beta"][a:b], state=S0)
        assert np.abs(o[a:b] - ref).max() <= 1e-4


def test_many_sequences_per_carry_cta():
    """12 ragged sequences x 32 value heads = 384 (sequence, head) pairs: more
    pairs than SMs, so each persistent carry CTA walks several pairs and its two
    shared-memory stages cross sequence boundaries. Each sequence starts from
    its own initial state and is checked against the per-token recurrence."""
    lens = [1, 63, 64, 65, 200, 17, 128, 300, 5, 129, 90, 250]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    T = int(cu[-1])
    inp = workloads.delta_operator_inputs(T=T, seed=17)
    rng = np.random.default_rng(17)
    S0 = (0.05 * rng.standard_normal((len(lens), 32, 128, 128))).astype(np.float32)
    qs, ks = workloads.scan_operands(inp)
    o, _, fin = run_scan(qs, ks, inp["v"], inp["g"], inp["beta"], cu_seqlens=cu, init_state=dev(S0),
                         final_state=True)
    worst = 0.0
    for s in range(len(lens)):
        a, b = cu[s], cu[s + 1]
        ref_o, ref_s, _ = oracle.delta_recurrence(inp["q"][a:b], inp["k"][a:b], inp["v"][a:b], inp["g"][a:b],
                                                  inp["beta"][a:b], state=S0[s])
        worst = max(worst, np.abs(o[a:b] - ref_o).max(), np.abs(fin[s] - ref_s).max())
    print(f"12 sequences x 32 heads: max-abs {worst:.3e}")
    assert np.isfinite(o).all() and worst <= 1e-4
