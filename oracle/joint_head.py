"""CPU F32 restatement of the reference's learned joint schema head.

TEST INFRASTRUCTURE ONLY: imported by tests/ (and nothing on the product path)
as the checker for the CUDA head in clef-rs_b200/csrc/head.cu.

Follows `Head::forward` (crates/core/src/models/head.rs:147-274) with the
reference's building blocks:
- `Norm::forward` LayerNorm with weight and bias (ops.rs:43-60), eps 1e-5;
- `normalize` x / max(|x|, eps) (ops.rs:33-42);
- `MultiAttention::forward` with PyTorch's packed in_proj rows q | k | v
  (ops.rs:190-225, weights.rs:167-188) and non-causal softmax attention,
  scale 1/sqrt(head width) (ops.rs:62-143);
- `Linear` y = x W^T + b; `gelu_erf` 0.5 x (1 + erf(x / sqrt 2));
- span means `mean_span` (head.rs:275-279) and the lexical means of the
  output-embedding rows of each option's token ids (head.rs:168-180).

Everything is float32 like the reference's F32 head; the erf of the GELU is
evaluated in float64 and rounded, as libm's erf is correctly rounded to
well below the comparison tolerance.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from math import erf, log, sqrt

import numpy as np

F32 = np.float32


@dataclass
class Question:
    kind: int                       # 0, 1, 2: row of type_embedding
    instruction: tuple[int, int]    # token span [start, end)
    options: list[tuple[int, int]] = field(default_factory=list)


@dataclass
class HeadConfig:
    hidden_size: int
    width: int
    routing_layers: int
    layers: int
    heads: int
    feedforward: int


def layer_norm(x, w, b, eps=1e-5):
    """ops.rs:43-60: (x - mean) / sqrt(var + eps) * w + b, biased variance."""
    f = x.astype(F32)
    mean = f.mean(-1, keepdims=True, dtype=F32)
    c = (f - mean).astype(F32)
    var = (c * c).mean(-1, keepdims=True, dtype=F32)
    n = c / np.sqrt(var + F32(eps)).astype(F32)
    return (n * w + b).astype(F32)


def normalize(x, eps):
    """ops.rs:33-42: x / clamp(|x|_2, eps)."""
    f = x.astype(F32)
    n = np.sqrt((f * f).sum(-1, keepdims=True, dtype=F32)).astype(F32)
    return (f / np.maximum(n, F32(eps))).astype(F32)


def linear(x, w, b=None):
    y = (x.astype(F32) @ w.T.astype(F32)).astype(F32)
    return y if b is None else (y + b).astype(F32)


try:  # scipy's erf is the same correctly rounded function, vectorised
    from scipy.special import erf as _erf
except ImportError:  # pragma: no cover
    _erf = np.vectorize(erf, otypes=[np.float64])


def gelu_erf(x):
    x = x.astype(F32)
    e = _erf(x.astype(np.float64) / sqrt(2.0)).astype(F32)
    return (F32(0.5) * x * (F32(1.0) + e)).astype(F32)


def softmax(x, axis):
    m = x.max(axis=axis, keepdims=True)
    e = np.exp((x - m).astype(F32)).astype(F32)
    return (e / e.sum(axis=axis, keepdims=True, dtype=F32)).astype(F32)


def mha(w, prefix, queries, memory, heads):
    """MultiAttention::forward (ops.rs:198-224) with weights.rs:167-188 packing."""
    width = queries.shape[1]
    inw, inb = w[f"{prefix}.in_proj_weight"], w[f"{prefix}.in_proj_bias"]
    hd = width // heads

    def proj(x, i):
        y = linear(x, inw[i * width:(i + 1) * width], inb[i * width:(i + 1) * width])
        return y.reshape(x.shape[0], heads, hd).transpose(1, 0, 2)

    q, k, v = proj(queries, 0), proj(memory, 1), proj(memory, 2)
    s = (q @ k.transpose(0, 2, 1)).astype(F32) / F32(sqrt(hd))
    p = softmax(s, -1)
    o = (p @ v).astype(F32).transpose(1, 0, 2).reshape(queries.shape[0], width)
    return linear(o, w[f"{prefix}.out_proj.weight"], w[f"{prefix}.out_proj.bias"])


def ln(w, name, x):
    return layer_norm(x, w[f"{name}.weight"], w[f"{name}.bias"])


def head_forward(w, cfg: HeadConfig, hidden, output_embeddings, ids, questions):
    """Head::forward (head.rs:147-274): one logit vector per question."""
    width = cfg.width
    hidden = hidden.astype(F32)
    normalized = ln(w, "hidden_norm", hidden)
    memory = linear(normalized, w["memory_projection.weight"])
    glob = normalized[len(ids) - 1:len(ids)]

    def mean_span(x, span):
        s, e = span
        return x[s:e].mean(0, keepdims=True, dtype=F32).astype(F32)

    qs = np.concatenate([mean_span(normalized, q.instruction) for q in questions], 0)
    lexical, queries, counts = [], [], []
    for i, q in enumerate(questions):
        contexts = np.concatenate([mean_span(normalized, sp) for sp in q.options], 0)
        lex = np.concatenate([output_embeddings[np.asarray(ids[s:e])].astype(F32).mean(
            0, keepdims=True, dtype=F32) for (s, e) in q.options], 0).astype(F32)
        query = (linear(contexts, w["option_context_projection.weight"])
                 + linear(lex, w["option_lexical_projection.weight"])).astype(F32)
        query = (query + linear(qs[i:i + 1], w["option_question_projection.weight"])).astype(F32)
        queries.append(query)
        lexical.append(lex)
        counts.append(len(q.options))
    routed = np.concatenate(queries, 0)
    for r in range(cfg.routing_layers):
        p = f"evidence_layers.{r}"
        nq = ln(w, f"{p}.query_norm", routed)
        nm = ln(w, f"{p}.memory_norm", memory)
        routed = (routed + mha(w, f"{p}.attention", nq, nm, cfg.heads)).astype(F32)
        ff = linear(gelu_erf(linear(ln(w, f"{p}.feedforward_norm", routed), w[f"{p}.feedforward.0.weight"],
                                    w[f"{p}.feedforward.0.bias"])),
                    w[f"{p}.feedforward.3.weight"], w[f"{p}.feedforward.3.bias"])
        routed = (routed + ff).astype(F32)
    base = linear(qs, w["question_projection.weight"])
    summaries, split, off = [], [], 0
    for i, n in enumerate(counts):
        options = routed[off:off + n]
        sc = ((options * base[i:i + 1]).sum(1, keepdims=True, dtype=F32) / F32(sqrt(width))).astype(F32)
        wts = softmax(sc, 0)
        summaries.append((options * wts).sum(0, keepdims=True, dtype=F32).astype(F32))
        split.append(options)
        off += n
    types = w["type_embedding.weight"][[q.kind for q in questions]]
    fields = (base + ln(w, "option_summary_norm", np.concatenate(summaries, 0))).astype(F32)
    fields = (fields + linear(glob, w["global_projection.weight"])).astype(F32)
    fields = (fields + types).astype(F32)
    for li in range(cfg.layers):
        p = f"layers.{li}"
        n1 = ln(w, f"{p}.norm1", fields)
        fields = (fields + mha(w, f"{p}.self_attn", n1, n1, cfg.heads)).astype(F32)
        n2 = ln(w, f"{p}.norm2", fields)
        fields = (fields + mha(w, f"{p}.multihead_attn", n2, memory, cfg.heads)).astype(F32)
        ff = linear(gelu_erf(linear(ln(w, f"{p}.norm3", fields), w[f"{p}.linear1.weight"], w[f"{p}.linear1.bias"])),
                    w[f"{p}.linear2.weight"], w[f"{p}.linear2.bias"])
        fields = (fields + ff).astype(F32)
    fields = ln(w, "field_norm", fields)
    prior_scale = F32(np.exp(min(float(w["prior_logit_scale"]), log(100.0))))
    joint_scale = F32(np.exp(min(float(w["joint_logit_scale"]), log(100.0))))
    gate = F32(1.0 / (1.0 + np.exp(-float(w["residual_gate"]))))
    out = []
    for i, (lex, options) in enumerate(zip(lexical, split)):
        anchor = normalize((qs[i:i + 1] + glob).astype(F32), 1e-12)
        prior = ((normalize(lex, 1e-12) * anchor).sum(1, dtype=F32) * prior_scale).astype(F32)
        opts = ln(w, "option_norm", options)
        fld = np.broadcast_to(fields[i:i + 1], opts.shape).astype(F32)
        cosine = (normalize(fld, 1e-8) * normalize(opts, 1e-8)).sum(1, dtype=F32).astype(F32)
        feats = np.concatenate([fld, opts, fld * opts, np.abs(fld - opts)], 1).astype(F32)
        resid = linear(gelu_erf(linear(feats, w["residual_scorer.0.weight"], w["residual_scorer.0.bias"])),
                       w["residual_scorer.3.weight"], w["residual_scorer.3.bias"])[:, 0]
        joint = (cosine * joint_scale + resid).astype(F32)
        out.append((prior + joint * gate).astype(F32))
    return out


def random_head_weights(cfg: HeadConfig, seed: int):
    """Seeded head weights of the reference's tensor names and shapes
    (head.rs:91-145), scaled like a trained checkpoint's fan-in init."""
    rng = np.random.default_rng(seed)
    h, wd, ff = cfg.hidden_size, cfg.width, cfg.feedforward
    w = {}

    def lin(name, o, i, bias):
        w[f"{name}.weight"] = (rng.standard_normal((o, i)) / np.sqrt(i)).astype(F32)
        if bias:
            w[f"{name}.bias"] = (0.02 * rng.standard_normal(o)).astype(F32)

    def norm(name, n):
        w[f"{name}.weight"] = (1.0 + 0.1 * rng.standard_normal(n)).astype(F32)
        w[f"{name}.bias"] = (0.05 * rng.standard_normal(n)).astype(F32)

    def attn(name):
        w[f"{name}.in_proj_weight"] = (rng.standard_normal((3 * wd, wd)) / np.sqrt(wd)).astype(F32)
        w[f"{name}.in_proj_bias"] = (0.02 * rng.standard_normal(3 * wd)).astype(F32)
        lin(f"{name}.out_proj", wd, wd, True)

    for r in range(cfg.routing_layers):
        p = f"evidence_layers.{r}"
        norm(f"{p}.query_norm", wd)
        norm(f"{p}.memory_norm", wd)
        attn(f"{p}.attention")
        norm(f"{p}.feedforward_norm", wd)
        lin(f"{p}.feedforward.0", ff, wd, True)
        lin(f"{p}.feedforward.3", wd, ff, True)
    for li in range(cfg.layers):
        p = f"layers.{li}"
        for n in ("norm1", "norm2", "norm3"):
            norm(f"{p}.{n}", wd)
        attn(f"{p}.self_attn")
        attn(f"{p}.multihead_attn")
        lin(f"{p}.linear1", ff, wd, True)
        lin(f"{p}.linear2", wd, ff, True)
    norm("hidden_norm", h)
    for n in ("memory_projection", "question_projection", "option_question_projection", "global_projection",
              "option_context_projection", "option_lexical_projection"):
        lin(n, wd, h, False)
    w["type_embedding.weight"] = (0.1 * rng.standard_normal((3, wd))).astype(F32)
    norm("option_summary_norm", wd)
    norm("field_norm", wd)
    norm("option_norm", wd)
    lin("residual_scorer.0", wd, 4 * wd, True)
    lin("residual_scorer.3", 1, wd, True)
    w["prior_logit_scale"] = np.asarray(np.log(10.0), F32)
    w["joint_logit_scale"] = np.asarray(np.log(20.0), F32)
    w["residual_gate"] = np.asarray(0.3, F32)
    return w
