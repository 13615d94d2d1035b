"""Seeded synthetic inputs with the shapes and distributions of the benchmark
configurations (no dataset is involved; token ids and weights are synthetic).
"""
import numpy as np

VOCAB = 248320


def _l2(x: np.ndarray) -> np.ndarray:
    """x / sqrt(sum x^2 + 1e-6) over the last axis, in float32 (qwen.rs:837-840)."""
    x = x.astype(np.float32)
    n = np.sqrt((x * x).sum(-1, keepdims=True, dtype=np.float32) + np.float32(1e-6))
    return (x / n).astype(np.float32)


def softplus(a: np.ndarray) -> np.ndarray:
    a = a.astype(np.float32)
    return (np.maximum(a, 0) + np.log(np.exp(-np.abs(a)) + np.float32(1))).astype(np.float32)


def delta_operator_inputs(T=1024, Hk=16, Hv=32, dk=128, dv=128, seed=0):
    """Config 1: q, k ~ N(0,1) then L2-normalised per head; v ~ N(0,1);
    beta = sigmoid(N(0,1)); g = -exp(A_log) * softplus(N(0,1) + dt_bias) with
    A_log ~ U(0, ln 16), dt_bias ~ N(0, 0.1); zero initial state."""
    rng = np.random.default_rng(seed)
    q = _l2(rng.standard_normal((T, Hk, dk), dtype=np.float32))
    k = _l2(rng.standard_normal((T, Hk, dk), dtype=np.float32))
    v = rng.standard_normal((T, Hv, dv), dtype=np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal((T, Hv), dtype=np.float32)))).astype(np.float32)
    a_log = rng.uniform(0.0, np.log(16.0), Hv).astype(np.float32)
    dt_bias = (0.1 * rng.standard_normal(Hv)).astype(np.float32)
    a = rng.standard_normal((T, Hv), dtype=np.float32) + dt_bias
    g = (softplus(a) * -np.exp(a_log)).astype(np.float32)
    return {"q": q, "k": k, "v": v, "g": g, "beta": beta}


def scan_operands(inp):
    """The chunked-scan operands: the reference recurrence normalises q and k
    (again; idempotent up to eps) and scales q by 1/sqrt(dk) (qwen.rs:844)."""
    dk = inp["q"].shape[-1]
    qs = (_l2(inp["q"]) * np.float32(1.0 / np.sqrt(dk)) + np.float32(0)).astype(np.float32)
    ks = _l2(inp["k"])
    return qs, ks


def gemm_inputs(M, K=2560, seed=1):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K), dtype=np.float32)


GEMM_SHAPES = {  # config 2: name -> (N, K)
    "gate_up": (2 * 9216, 2560),
    "down": (2560, 9216),
    "qkv": (16 * 256 + 2 * 4 * 256, 2560),
    "qkv_gate": (2 * 16 * 256 + 2 * 4 * 256, 2560),
}


def gemm_weight(N, K, seed=1):
    rng = np.random.default_rng(seed + 1000 * N + K)
    return (0.02 * rng.standard_normal((N, K), dtype=np.float32)).astype(np.float32)


def backbone_requests(n=256, lo=256, hi=2048, seed=3, vocab=VOCAB):
    """Config 4: n requests, lengths U[lo, hi], ids U[0, vocab)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, n)
    return [rng.integers(0, vocab, int(L)).astype(np.int32) for L in lens]


def prefix_workload(prefix=16384, n=64, lo=512, hi=4096, seed=4, vocab=VOCAB):
    """Config 5: one shared prefix and n unique suffixes."""
    rng = np.random.default_rng(seed)
    pre = rng.integers(0, vocab, prefix).astype(np.int32)
    lens = rng.integers(lo, hi + 1, n)
    return pre, [rng.integers(0, vocab, int(L)).astype(np.int32) for L in lens]


def block_group_ids(T=4096, seed=2, vocab=VOCAB):
    """Config 3: one sequence of T uniform ids."""
    return np.random.default_rng(seed).integers(0, vocab, T).astype(np.int32)
