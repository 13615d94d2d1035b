"""The allocation-free scan entry point, checked against the workspace one.

clef_delta_scan_noalloc serves callers that cannot allocate device memory or
pass a workspace (an allocator that owns all device memory behind a fixed op
signature, or a latency-critical loop that must avoid cudaMalloc's implicit
synchronisation): the per-sequence offsets live in a fixed device array inside
the library instead. The allocation-free entry runs the fused single-pass scan
kernel, the workspace entry the two-kernel pipeline whose intra-chunk Gram
products run on the tcgen05 tensor core; the outputs therefore agree to F32
summation-order noise: max-abs 1e-5 on the outputs and 1e-4 on the final states
(the scan's tolerance against the oracle is 1e-3). Checked on two calls in a row
with different packings (the second call must not see the first call's offsets),
and directly against the oracle's per-token recurrence on config 1, with
initial states (per sequence and shared) and with a capture.

This file is collected last on purpose; it needs nothing from the others and
also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from clef_b200 import workloads

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def close(a, b, tol):
    return bool(np.isfinite(a).all()) and float(np.abs(a - b).max()) <= tol


def scan_both(inp, cu, final=True):
    import clef_b200 as cb
    qs, ks = workloads.scan_operands(inp)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda()
         for k, v in dict(q=qs, k=ks, v=inp["v"], g=inp["g"], b=inp["beta"]).items()}
    T, Hk, _ = qs.shape
    Hv = inp["v"].shape[1]
    nseq = len(cu) - 1
    cu = np.ascontiguousarray(cu, np.int64)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = []
    for fn in ("clef_delta_scan", "clef_delta_scan_noalloc"):
        out = torch.empty((T, Hv, 128), dtype=torch.float32, device="cuda")
        fin = torch.empty((nseq, Hv, 128, 128), dtype=torch.float32, device="cuda") if final else None
        args = [_p(t["q"]), _p(t["k"]), _p(t["v"]), _p(t["g"]), _p(t["b"]), T, Hk, Hv, 128, 128,
                cu.ctypes.data, nseq, None, 0, 0, None, _p(fin), _p(out)]
        if fn == "clef_delta_scan":
            size = cb.delta_scan_workspace_size(T, nseq, Hk, Hv)
            ws = torch.empty(size, dtype=torch.uint8, device="cuda")
            rc = cb.lib.clef_delta_scan(*args, _p(ws), size, stream)
        else:
            rc = cb.lib.clef_delta_scan_noalloc(*args, stream)
        assert rc == 0, cb.lib.clef_last_error().decode()
        torch.cuda.synchronize()
        outs.append((out.cpu().numpy(), None if fin is None else fin.cpu().numpy()))
    return outs


def test_noalloc_scan_matches_workspace_scan_on_two_calls_in_a_row():
    first = workloads.delta_operator_inputs(T=700, seed=21)
    (o_ws, f_ws), (o_na, f_na) = scan_both(first, [0, 1, 65, 200, 700])
    assert close(o_na, o_ws, 1e-5) and close(f_na, f_ws, 1e-4)
    # Second call, different packing and more sequences: the shared array is
    # rewritten for every entry the kernel reads.
    second = workloads.delta_operator_inputs(T=1000, seed=22)
    (o_ws, f_ws), (o_na, f_na) = scan_both(second, [0, 300, 301, 450, 640, 999, 1000])
    assert close(o_na, o_ws, 1e-5) and close(f_na, f_ws, 1e-4)


def _noalloc(inp, cu, init=None, init_shared=0, capture=0):
    import clef_b200 as cb
    qs, ks = workloads.scan_operands(inp)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda()
         for k, v in dict(q=qs, k=ks, v=inp["v"], g=inp["g"], b=inp["beta"]).items()}
    T, Hk, _ = qs.shape
    Hv = inp["v"].shape[1]
    nseq = len(cu) - 1
    cu = np.ascontiguousarray(cu, np.int64)
    out = torch.empty((T, Hv, 128), dtype=torch.float32, device="cuda")
    fin = torch.empty((nseq, Hv, 128, 128), dtype=torch.float32, device="cuda")
    cap = torch.empty((Hv, 128, 128), dtype=torch.float32, device="cuda") if capture else None
    init_t = None if init is None else torch.from_numpy(np.ascontiguousarray(init, np.float32)).cuda()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = cb.lib.clef_delta_scan_noalloc(_p(t["q"]), _p(t["k"]), _p(t["v"]), _p(t["g"]), _p(t["b"]), T, Hk, Hv,
                                        128, 128, cu.ctypes.data, nseq, _p(init_t), init_shared, capture,
                                        _p(cap), _p(fin), _p(out), stream)
    assert rc == 0, cb.lib.clef_last_error().decode()
    torch.cuda.synchronize()
    return out.cpu().numpy(), fin.cpu().numpy(), None if cap is None else cap.cpu().numpy()


def test_noalloc_scan_matches_the_oracle_recurrence():
    """Config 1 (T = 1024, 16 / 32 heads, seed 0) through the allocation-free
    entry against the oracle's per-token recurrence at the scan's 1e-3 bound."""
    import oracle
    inp = workloads.delta_operator_inputs(T=1024, seed=0)
    o, fin, _ = _noalloc(inp, [0, 1024])
    want, state, _ = oracle.delta_recurrence(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"])
    assert close(o, want, 1e-3) and close(fin[0], state, 1e-3)


def test_noalloc_scan_initial_states_and_capture_match_the_oracle():
    """Per-sequence initial states, one state shared by every sequence, and a
    capture inside a chunk: each against the oracle's recurrence (1e-3)."""
    import oracle
    inp = workloads.delta_operator_inputs(T=400, seed=24)
    cu = [0, 150, 400]
    rng = np.random.default_rng(5)
    init = (0.05 * rng.standard_normal((2, 32, 128, 128))).astype(np.float32)
    for shared in (0, 1):
        o, fin, _ = _noalloc(inp, cu, init=init[:1] if shared else init, init_shared=shared)
        for s in range(2):
            a, b = cu[s], cu[s + 1]
            start = init[0] if shared else init[s]
            want, state, _ = oracle.delta_recurrence(inp["q"][a:b], inp["k"][a:b], inp["v"][a:b], inp["g"][a:b],
                                                     inp["beta"][a:b], state=start)
            assert close(o[a:b], want, 1e-3) and close(fin[s], state, 1e-3), (shared, s)
    o, _, cap = _noalloc(inp, [0, 400], capture=100)
    want, _, wcap = oracle.delta_recurrence(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], capture=100)
    assert close(o, want, 1e-3) and close(cap, wcap, 1e-3)


def test_noalloc_scan_single_sequence_and_size_limit():
    import clef_b200 as cb
    inp = workloads.delta_operator_inputs(T=257, seed=23)
    (o_ws, f_ws), (o_na, f_na) = scan_both(inp, [0, 257])
    assert close(o_na, o_ws, 1e-5) and close(f_na, f_ws, 1e-4)
    # More sequences than the fixed array holds: rejected before any launch.
    cu = np.arange(0, 4098, dtype=np.int64)
    fake = ctypes.c_void_p(0x10000)
    rc = cb.lib.clef_delta_scan_noalloc(fake, fake, fake, fake, fake, 4097, 16, 32, 128, 128,
                                        cu.ctypes.data, 4097, None, 0, 0, None, None, fake, None)
    assert rc == 3 and "4096" in cb.lib.clef_last_error().decode()
