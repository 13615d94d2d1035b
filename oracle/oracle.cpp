// oracle.cpp — TEST INFRASTRUCTURE ONLY: the CPU F32 restatement of the
// reference's CPU path for the hybrid-backbone prefill (tyrchen/clef-rs).
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
// this library, and only as the checker or as the timed CPU baseline. The
// product (libclef_b200.so) never links or calls it.
//
// The reference itself is Rust + Candle 0.11.0 (CPU matmul: the `gemm` 0.19.0
// crate); no Rust toolchain exists on the build host, so this file restates the
// reference equations in C++ F32, citing the file:line each function follows.
// It is pinned against the reference's own golden fixture
// crates/core/fixtures/synthetic/backbone{,-output}.safetensors (converted by
// tests/golden/make_golden.py) at the reference tolerance 1e-5 + 1e-4|e|
// (crates/core/src/models/mod.rs:75-86), and against the reference's
// prefix-resume invariants (mod.rs:116-171) and tiled-vs-dense attention test
// (ops.rs:238-263).
//
// Parallelism: OpenMP over rows / heads / output tiles. Within one output value
// the summation order is sequential, as in Candle's CPU reductions.

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include <immintrin.h>
#include <omp.h>

#include "../include/clef_b200.h"

namespace {

thread_local std::string g_err;
int fail(const std::string& m) {
  g_err = m;
  return 1;
}

// ---------------------------------------------------------------------------
// Optional BF16 rounding points (default off: the reference's F32 path). A
// mask set by oracle_set_rounding() rounds chosen intermediates to BF16
// (nearest, ties to even) so tests can measure how much of a BF16 device
// profile's distance from the F32 path each rounding point contributes, and
// can check a device path against the F32 path with exactly its own
// rounding points:
//   kRoundOperand  GEMM A operands: normed inputs, gated DeltaNet output,
//                  gated attention output, SwiGLU activation
//   kRoundProj     projection outputs (in_proj_qkv/z/a/b, q/k/v_proj)
//   kRoundAttnQKV  attention q, k (after norm and rotary) and v
//   kRoundP        attention probabilities as the P.V product reads them
//   kRoundFlow     the remaining model-dtype casts of the reference's
//                  mixed-precision path (qwen.rs:671-676, 463-524): DeltaNet
//                  o and norm output, q/k norm output, sigmoid(gate), attention
//                  output before the gate product
// ---------------------------------------------------------------------------
enum {
  kRoundOperand = 1,
  kRoundProj = 2,
  kRoundAttnQKV = 4,
  kRoundP = 8,
  kRoundFlow = 16,
  // Finer sites, each also covered by kRoundOperand / kRoundProj above.
  kRoundOpMixIn = 32,       // normed hidden into a mixer's projections
  kRoundOpMlpIn = 64,       // normed hidden into gate/up
  kRoundOpDown = 128,       // SwiGLU activation into down
  kRoundOpDeltaOut = 256,   // gated DeltaNet output into out_proj
  kRoundOpAttnOut = 512,    // gated attention output into o_proj
  kRoundProjDeltaQKV = 1024,  // DeltaNet in_proj_qkv output (conv input)
  kRoundProjAttn = 2048,      // attention q/gate, k, v projection outputs
  kRoundProjDeltaZ = 4096,    // DeltaNet in_proj_z output
  kRoundProjDeltaAB = 8192,   // DeltaNet in_proj_a / in_proj_b outputs
};
int g_round = 0;

inline float bf16r(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}
inline void round_if(int bit, float* x, size_t n) {
  if (!(g_round & bit)) return;
  for (size_t i = 0; i < n; ++i) x[i] = bf16r(x[i]);
}
inline void round_if(int bit, std::vector<float>& v) { round_if(bit, v.data(), v.size()); }

// ---------------------------------------------------------------------------
// Dense F32 GEMM: out[M,N] = x[M,K] * W[N,K]^T  (candle_nn::Linear without
// bias, projection.rs:82-95). W is packed once into 16-column panels
// [N/16][K][16] so the micro-kernel broadcasts x and streams W.
// ---------------------------------------------------------------------------
struct Packed {
  int64_t n = 0, k = 0, np = 0;  // np: N rounded up to 16
  std::vector<float> data;       // [np/16][k][16]
};

void pack_weight(const float* w, int64_t n, int64_t k, Packed& p) {
  p.n = n;
  p.k = k;
  p.np = (n + 15) / 16 * 16;
  p.data.assign((size_t)p.np * k, 0.f);
#pragma omp parallel for schedule(static)
  for (int64_t pn = 0; pn < p.np / 16; ++pn) {
    float* dst = p.data.data() + (size_t)pn * k * 16;
    for (int64_t j = 0; j < 16; ++j) {
      int64_t row = pn * 16 + j;
      if (row >= n) continue;
      const float* src = w + (size_t)row * k;
      for (int64_t kk = 0; kk < k; ++kk) dst[(size_t)kk * 16 + j] = src[kk];
    }
  }
}

// 6x16 register block: 12 AVX2 accumulators, fused multiply-add as in the
// `gemm` crate's F32 kernels.
inline void micro_6x16(const float* x, int64_t ldx, int rows, const float* panel, int64_t k,
                       float* out, int64_t ldo, int cols) {
  __m256 acc[6][2];
  for (int r = 0; r < 6; ++r) acc[r][0] = acc[r][1] = _mm256_setzero_ps();
  const float* xr[6];
  for (int r = 0; r < 6; ++r) xr[r] = x + (size_t)(r < rows ? r : 0) * ldx;
  for (int64_t kk = 0; kk < k; ++kk) {
    const __m256 b0 = _mm256_loadu_ps(panel + kk * 16);
    const __m256 b1 = _mm256_loadu_ps(panel + kk * 16 + 8);
    for (int r = 0; r < 6; ++r) {
      const __m256 av = _mm256_broadcast_ss(xr[r] + kk);
      acc[r][0] = _mm256_fmadd_ps(av, b0, acc[r][0]);
      acc[r][1] = _mm256_fmadd_ps(av, b1, acc[r][1]);
    }
  }
  for (int r = 0; r < rows; ++r) {
    float tmp[16];
    _mm256_storeu_ps(tmp, acc[r][0]);
    _mm256_storeu_ps(tmp + 8, acc[r][1]);
    for (int c = 0; c < cols; ++c) out[(size_t)r * ldo + c] = tmp[c];
  }
}

void gemm_packed(const float* x, int64_t m, const Packed& w, float* out) {
  const int64_t n = w.n, k = w.k;
  const int64_t mb = (m + 5) / 6, nb = w.np / 16;
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
  for (int64_t j = 0; j < nb; ++j) {
    for (int64_t i = 0; i < mb; ++i) {
      int rows = (int)std::min<int64_t>(6, m - i * 6);
      int cols = (int)std::min<int64_t>(16, n - j * 16);
      micro_6x16(x + (size_t)i * 6 * k, k, rows, w.data.data() + (size_t)j * k * 16, k,
                 out + (size_t)i * 6 * n + j * 16, n, cols);
    }
  }
}

void gemm_plain(const float* x, int64_t m, const float* w, int64_t n, int64_t k, float* out) {
  Packed p;
  pack_weight(w, n, k, p);
  gemm_packed(x, m, p, out);
}

// ---------------------------------------------------------------------------
// Elementwise pieces (Candle CPU semantics).
// ---------------------------------------------------------------------------
inline float sigmoidf_(float x) { return 1.f / (1.f + std::exp(-x)); }  // candle_nn::ops::sigmoid
inline float siluf_(float x) { return x / (1.f + std::exp(-x)); }       // candle_nn::ops::silu

// ops::rms_inner (ops.rs:24-32): x * recip(sqrt(mean(x^2) + eps)) * w, where
// w already carries the +1 offset (normalization.rs:44-45).
void rms_rows(const float* x, const float* w, int64_t rows, int64_t width, float eps,
              float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * width;
    float s = 0.f;
    for (int64_t i = 0; i < width; ++i) s += xr[i] * xr[i];
    float inv = 1.f / std::sqrt(s / (float)width + eps);
    for (int64_t i = 0; i < width; ++i) out[r * width + i] = xr[i] * inv * w[i];
  }
}

// causal_convolution (qwen.rs:765-796): taps accumulated oldest to newest,
// zero rows before the first input row.
void conv4(const float* x, int64_t t, int64_t width, const float* weight, int taps,
           float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < t; ++r) {
    for (int64_t c = 0; c < width; ++c) {
      float acc = 0.f;
      for (int tap = 0; tap < taps; ++tap) {
        int64_t delay = taps - 1 - tap;
        if (r >= delay) acc = acc + x[(r - delay) * width + c] * weight[c * taps + tap];
      }
      out[r * width + c] = acc;
    }
  }
}

// delta_recurrence_prefill (qwen.rs:826-882) after recur_portable's split and
// head repeat (qwen.rs:727-739). q, k: [t, hk, kd] (not yet normalised);
// v: [t, hv, vd]; g, beta: [t, hv]. state: [hv, kd, vd] in/out.
void delta_recurrence(const float* q_in, const float* k_in, const float* v, const float* g,
                      const float* beta, int64_t t, int hk, int hv, int kd, int vd,
                      float* state, int64_t capture, float* captured, float* out) {
  const int rep = hv / hk;
  // l2(x) = x / sqrt(sum x^2 + 1e-6) (qwen.rs:837-840); q also * 1/sqrt(kd)
  // (Candle's Tensor / f64 is affine(1/rhs, 0), qwen.rs:844).
  std::vector<float> qn((size_t)t * hk * kd), kn((size_t)t * hk * kd);
  const float qscale = (float)(1.0 / std::sqrt((double)kd));
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < t * hk; ++row) {
    const float* qr = q_in + row * kd;
    const float* kr = k_in + row * kd;
    float sq = 0.f, sk = 0.f;
    for (int i = 0; i < kd; ++i) sq += qr[i] * qr[i];
    for (int i = 0; i < kd; ++i) sk += kr[i] * kr[i];
    float nq = std::sqrt(sq + 1e-6f), nk = std::sqrt(sk + 1e-6f);
    for (int i = 0; i < kd; ++i) {
      qn[row * kd + i] = (qr[i] / nq) * qscale + 0.f;
      kn[row * kd + i] = kr[i] / nk;
    }
  }
#pragma omp parallel for schedule(static)
  for (int h = 0; h < hv; ++h) {
    float* s = state + (size_t)h * kd * vd;
    const int kh = h / rep;
    std::vector<float> mem(vd), delta(vd);
    for (int64_t i = 0; i < t; ++i) {
      const float* key = kn.data() + ((size_t)i * hk + kh) * kd;
      const float* qry = qn.data() + ((size_t)i * hk + kh) * kd;
      const float decay = std::exp(g[i * hv + h]);
      const float b = beta[i * hv + h];
      for (int a = 0; a < kd * vd; ++a) s[a] = s[a] * decay;
      for (int c = 0; c < vd; ++c) {
        float acc = 0.f;
        for (int a = 0; a < kd; ++a) acc += s[a * vd + c] * key[a];
        mem[c] = acc;
      }
      const float* vr = v + ((size_t)i * hv + h) * vd;
      for (int c = 0; c < vd; ++c) delta[c] = (vr[c] - mem[c]) * b;
      for (int a = 0; a < kd; ++a)
        for (int c = 0; c < vd; ++c) s[a * vd + c] = s[a * vd + c] + key[a] * delta[c];
      float* o = out + ((size_t)i * hv + h) * vd;
      for (int c = 0; c < vd; ++c) {
        float acc = 0.f;
        for (int a = 0; a < kd; ++a) acc += s[a * vd + c] * qry[a];
        o[c] = acc;
      }
      if (captured && capture == i + 1)
        memcpy(captured + (size_t)h * kd * vd, s, sizeof(float) * kd * vd);
    }
  }
}

// ops::attention (ops.rs:62-143): 128-query x 256-key tiles, online softmax in
// F32, lower-right causal offset kn - qn, scale 1/sqrt(width), GQA expanded
// by head index i / (heads / kv_heads).
void attention(const float* q, const float* k, const float* v, int heads, int kv_heads,
               int64_t qn, int64_t kn, int width, int vw, bool causal, float* out) {
  const int rep = heads / kv_heads;
  const float scale = (float)(1.0 / std::sqrt((double)width));
  const int64_t offset = causal ? kn - qn : 0;
  const int64_t qtiles = (qn + 127) / 128;
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int h = 0; h < heads; ++h) {
    for (int64_t qt = 0; qt < qtiles; ++qt) {
      const int kh = h / rep;
      const int64_t qs = qt * 128, count = std::min<int64_t>(128, qn - qs);
      std::vector<float> mx(count, -INFINITY), den(count, 0.f), acc((size_t)count * vw, 0.f);
      std::vector<float> sc((size_t)count * 256);
      for (int64_t ks = 0; ks < kn; ks += 256) {
        if (causal && ks >= offset + qs + count) break;
        const int64_t keys = std::min<int64_t>(256, kn - ks);
        for (int64_t i = 0; i < count; ++i) {
          const float* qr = q + ((size_t)h * qn + qs + i) * width;
          for (int64_t j = 0; j < keys; ++j) {
            const float* kr = k + ((size_t)kh * kn + ks + j) * width;
            float d = 0.f;
            for (int c = 0; c < width; ++c) d += qr[c] * kr[c];
            d = d * scale + 0.f;
            if (causal && ks + j > offset + qs + i) d = d + -INFINITY;
            sc[i * keys + j] = d;
          }
        }
        for (int64_t i = 0; i < count; ++i) {
          float rowmax = -INFINITY;
          for (int64_t j = 0; j < keys; ++j) rowmax = std::max(rowmax, sc[i * keys + j]);
          const float nm = std::max(mx[i], rowmax);
          const float rescale = std::exp(mx[i] - nm);
          float psum = 0.f;
          float* a = acc.data() + i * vw;
          for (int c = 0; c < vw; ++c) a[c] = a[c] * rescale;
          for (int64_t j = 0; j < keys; ++j) {
            float p = std::exp(sc[i * keys + j] - nm);
            if (g_round & kRoundP) p = bf16r(p);
            psum += p;
            const float* vr = v + ((size_t)kh * kn + ks + j) * vw;
            for (int c = 0; c < vw; ++c) a[c] += p * vr[c];
          }
          den[i] = den[i] * rescale + psum;
          mx[i] = nm;
        }
      }
      for (int64_t i = 0; i < count; ++i)
        for (int c = 0; c < vw; ++c)
          out[((size_t)h * qn + qs + i) * vw + c] = acc[i * vw + c] / den[i];
    }
  }
}

// rotary (ops.rs:144-188) for text positions (all three M-RoPE axes equal):
// NeoX rotate-half on the first `dim` features, angle = pos * theta^(-2i/dim).
void rotary(float* x, int64_t tokens, int heads, int width, const int64_t* positions, int dim,
            double theta) {
  const int half = dim / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = (float)std::pow(theta, -((double)(2 * i)) / dim);
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < tokens; ++t) {
    std::vector<float> cs(dim), sn(dim), rot(dim), orig(dim);
    for (int i = 0; i < half; ++i) {
      float a = (float)positions[t] * inv[i];
      cs[i] = cs[i + half] = std::cos(a);
      sn[i] = sn[i + half] = std::sin(a);
    }
    for (int h = 0; h < heads; ++h) {
      float* r = x + ((size_t)t * heads + h) * width;
      for (int i = 0; i < dim; ++i) orig[i] = r[i];
      for (int i = 0; i < half; ++i) {
        rot[i] = -orig[i + half];
        rot[i + half] = orig[i];
      }
      for (int i = 0; i < dim; ++i) r[i] = orig[i] * cs[i] + rot[i] * sn[i];
    }
  }
}

// ---------------------------------------------------------------------------
// Model (Backbone, qwen.rs:145-426).
// ---------------------------------------------------------------------------
struct Tensor {
  std::vector<int64_t> shape;
  std::vector<float> data;
  Packed packed;  // filled for projection matrices
  bool present = false;
  bool projection = false;
};

struct LayerState {  // MixerState (qwen.rs:159-163)
  bool full = false;
  std::vector<float> key, value;  // [kvh, c, d]
  int64_t kv_tokens = 0;
  std::vector<float> recurrent;   // [hv, kd, vd]
  std::vector<float> history;     // [rows, conv_width]
  int64_t history_rows = 0;
};

struct Prefix {  // PrefixState (qwen.rs:153-158)
  std::vector<float> hidden;  // [c, hidden]
  int64_t tokens = 0;
  std::vector<LayerState> layers;
};

struct Model {
  clef_config c;
  std::map<std::string, Tensor> w;
};

std::string L(int i) { return "model.language_model.layers." + std::to_string(i); }

void declare(Model& m, const std::string& name, std::vector<int64_t> shape, bool proj) {
  Tensor t;
  t.shape = shape;
  t.projection = proj;
  m.w[name] = std::move(t);
}

void declare_all(Model& m) {
  const clef_config& c = m.c;
  const int64_t h = c.hidden_size;
  declare(m, "model.language_model.embed_tokens.weight", {c.vocab_size, h}, false);
  declare(m, "model.language_model.norm.weight", {h}, false);
  if (c.head_outputs > 0) declare(m, "clef.head.weight", {c.head_outputs, h}, false);
  const int64_t key = (int64_t)c.linear_num_key_heads * c.linear_key_head_dim;
  const int64_t value = (int64_t)c.linear_num_value_heads * c.linear_value_head_dim;
  const int64_t n = (int64_t)c.num_attention_heads * c.head_dim;
  const int64_t kv = (int64_t)c.num_key_value_heads * c.head_dim;
  for (int i = 0; i < c.num_hidden_layers; ++i) {
    const std::string p = L(i);
    declare(m, p + ".input_layernorm.weight", {h}, false);
    declare(m, p + ".post_attention_layernorm.weight", {h}, false);
    declare(m, p + ".mlp.gate_proj.weight", {c.intermediate_size, h}, true);
    declare(m, p + ".mlp.up_proj.weight", {c.intermediate_size, h}, true);
    declare(m, p + ".mlp.down_proj.weight", {h, c.intermediate_size}, true);
    if (c.layer_types[i]) {
      declare(m, p + ".self_attn.q_proj.weight", {2 * n, h}, true);
      declare(m, p + ".self_attn.k_proj.weight", {kv, h}, true);
      declare(m, p + ".self_attn.v_proj.weight", {kv, h}, true);
      declare(m, p + ".self_attn.o_proj.weight", {h, n}, true);
      declare(m, p + ".self_attn.q_norm.weight", {c.head_dim}, false);
      declare(m, p + ".self_attn.k_norm.weight", {c.head_dim}, false);
    } else {
      declare(m, p + ".linear_attn.in_proj_qkv.weight", {2 * key + value, h}, true);
      declare(m, p + ".linear_attn.in_proj_z.weight", {value, h}, true);
      declare(m, p + ".linear_attn.in_proj_a.weight", {c.linear_num_value_heads, h}, true);
      declare(m, p + ".linear_attn.in_proj_b.weight", {c.linear_num_value_heads, h}, true);
      declare(m, p + ".linear_attn.out_proj.weight", {h, value}, true);
      declare(m, p + ".linear_attn.conv1d.weight", {2 * key + value, 1, c.linear_conv_kernel_dim},
              false);
      declare(m, p + ".linear_attn.dt_bias", {c.linear_num_value_heads}, false);
      declare(m, p + ".linear_attn.A_log", {c.linear_num_value_heads}, false);
      declare(m, p + ".linear_attn.norm.weight", {c.linear_value_head_dim}, false);
    }
  }
}

const Tensor& W(const Model& m, const std::string& name) { return m.w.at(name); }

void linear(const Model& m, const std::string& name, const float* x, int64_t rows,
            std::vector<float>& out) {
  const Tensor& t = W(m, name);
  out.resize((size_t)rows * t.shape[0]);
  gemm_packed(x, rows, t.packed, out.data());
}

// Offset norms store 1 + w, as Norms::load does (normalization.rs:44-45).
std::vector<float> norm_weight(const Model& m, const std::string& name, bool offset) {
  std::vector<float> w = W(m, name).data;
  if (offset)
    for (auto& x : w) x = x + 1.f;
  return w;
}

// Delta::forward (qwen.rs:589-688).
void delta_forward(const Model& m, int li, const float* x, int64_t t, const LayerState* init,
                   int64_t capture, LayerState* saved, std::vector<float>& mixed_out) {
  const clef_config& c = m.c;
  const std::string p = L(li) + ".linear_attn";
  const int hk = c.linear_num_key_heads, hv = c.linear_num_value_heads;
  const int kd = c.linear_key_head_dim, vd = c.linear_value_head_dim;
  const int64_t key = (int64_t)hk * kd, value = (int64_t)hv * vd, width = 2 * key + value;
  const int taps = c.linear_conv_kernel_dim;
  std::vector<float> proj;
  linear(m, p + ".in_proj_qkv.weight", x, t, proj);
  round_if(kRoundProj | kRoundProjDeltaQKV, proj);
  const int64_t hist = init ? init->history_rows : 0;
  std::vector<float> projected((size_t)(hist + t) * width);
  if (hist) memcpy(projected.data(), init->history.data(), sizeof(float) * hist * width);
  memcpy(projected.data() + hist * width, proj.data(), sizeof(float) * t * width);
  std::vector<float> conv((size_t)(hist + t) * width);
  conv4(projected.data(), hist + t, width, W(m, p + ".conv1d.weight").data.data(), taps,
        conv.data());
  std::vector<float> mixed((size_t)t * width);
  for (int64_t i = 0; i < t * width; ++i) mixed[i] = siluf_(conv[hist * width + i]);
  std::vector<float> a, b;
  linear(m, p + ".in_proj_a.weight", x, t, a);
  linear(m, p + ".in_proj_b.weight", x, t, b);
  round_if(kRoundProj | kRoundProjDeltaAB, a);
  round_if(kRoundProj | kRoundProjDeltaAB, b);
  const auto& dt = W(m, p + ".dt_bias").data;
  const auto& alog = W(m, p + ".A_log").data;
  std::vector<float> g((size_t)t * hv), beta((size_t)t * hv);
  for (int64_t i = 0; i < t; ++i)
    for (int h = 0; h < hv; ++h) {
      float av = a[i * hv + h] + dt[h];
      // Stable softplus (qwen.rs:624-626).
      float sp = std::max(av, 0.f) + std::log(std::exp(-std::fabs(av)) + 1.f);
      g[i * hv + h] = sp * -std::exp(alog[h]);
      beta[i * hv + h] = sigmoidf_(b[i * hv + h]);
    }
  // Split q|k|v (recur_portable, qwen.rs:731-739).
  std::vector<float> q((size_t)t * key), k((size_t)t * key), v((size_t)t * value);
  for (int64_t i = 0; i < t; ++i) {
    memcpy(&q[i * key], &mixed[i * width], sizeof(float) * key);
    memcpy(&k[i * key], &mixed[i * width + key], sizeof(float) * key);
    memcpy(&v[i * value], &mixed[i * width + 2 * key], sizeof(float) * value);
  }
  std::vector<float> state((size_t)hv * kd * vd, 0.f);
  if (init) state = init->recurrent;
  std::vector<float> captured;
  if (capture) captured.assign(state.size(), 0.f);
  std::vector<float> out((size_t)t * value);
  delta_recurrence(q.data(), k.data(), v.data(), g.data(), beta.data(), t, hk, hv, kd, vd,
                   state.data(), capture, capture ? captured.data() : nullptr, out.data());
  // norm(out) (no offset, qwen.rs:581-586) * silu(z) (qwen.rs:671-676).
  std::vector<float> z;
  linear(m, p + ".in_proj_z.weight", x, t, z);
  round_if(kRoundProj | kRoundProjDeltaZ, z);
  const std::vector<float> nw = norm_weight(m, p + ".norm.weight", false);
  std::vector<float> normed((size_t)t * value);
  round_if(kRoundFlow, out);
  rms_rows(out.data(), nw.data(), t * hv, vd, c.rms_norm_eps, normed.data());
  round_if(kRoundFlow, normed);
  std::vector<float> gated((size_t)t * value);
  for (int64_t i = 0; i < t * value; ++i) gated[i] = normed[i] * siluf_(z[i]);
  round_if(kRoundOperand | kRoundOpDeltaOut, gated);
  if (capture && saved) {
    saved->full = false;
    saved->recurrent = captured;
    const int64_t end = hist + capture;
    const int64_t count = std::min<int64_t>(end, taps - 1);
    saved->history_rows = count;
    saved->history.assign(projected.begin() + (end - count) * width,
                          projected.begin() + end * width);
  }
  linear(m, p + ".out_proj.weight", gated.data(), t, mixed_out);
}

// FullAttention::forward (qwen.rs:451-525).
void attention_forward(const Model& m, int li, const float* x, int64_t t,
                       const int64_t* positions, const LayerState* init, int64_t capture,
                       LayerState* saved, std::vector<float>& mixed_out) {
  const clef_config& c = m.c;
  const std::string p = L(li) + ".self_attn";
  const int d = c.head_dim, heads = c.num_attention_heads, kvh = c.num_key_value_heads;
  std::vector<float> proj, kp, vp;
  linear(m, p + ".q_proj.weight", x, t, proj);  // [t, heads, 2d]
  linear(m, p + ".k_proj.weight", x, t, kp);    // [t, kvh, d]
  linear(m, p + ".v_proj.weight", x, t, vp);    // [t, kvh, d]
  round_if(kRoundProj | kRoundProjAttn, proj);
  round_if(kRoundProj | kRoundProjAttn, kp);
  round_if(kRoundProj | kRoundProjAttn | kRoundAttnQKV, vp);
  std::vector<float> gate((size_t)t * heads * d), qraw((size_t)t * heads * d);
  for (int64_t i = 0; i < t; ++i)
    for (int h = 0; h < heads; ++h) {
      memcpy(&qraw[(i * heads + h) * d], &proj[(i * heads + h) * 2 * d], sizeof(float) * d);
      memcpy(&gate[(i * heads + h) * d], &proj[(i * heads + h) * 2 * d + d], sizeof(float) * d);
    }
  const std::vector<float> qw = norm_weight(m, p + ".q_norm.weight", true);
  const std::vector<float> kw = norm_weight(m, p + ".k_norm.weight", true);
  std::vector<float> qn(qraw.size()), kn(kp.size());
  rms_rows(qraw.data(), qw.data(), t * heads, d, c.rms_norm_eps, qn.data());
  rms_rows(kp.data(), kw.data(), t * kvh, d, c.rms_norm_eps, kn.data());
  round_if(kRoundFlow, qn);
  round_if(kRoundFlow, kn);
  rotary(qn.data(), t, heads, d, positions, c.rotary_dim, c.rope_theta);
  rotary(kn.data(), t, kvh, d, positions, c.rotary_dim, c.rope_theta);
  round_if(kRoundAttnQKV, qn);
  round_if(kRoundAttnQKV, kn);
  const int64_t pre = init ? init->kv_tokens : 0, kn_total = pre + t;
  // Transpose to [heads, tokens, d]; prefix K/V first (qwen.rs:497-503).
  std::vector<float> qt((size_t)heads * t * d), kt((size_t)kvh * kn_total * d),
      vt((size_t)kvh * kn_total * d);
  for (int h = 0; h < heads; ++h)
    for (int64_t i = 0; i < t; ++i)
      memcpy(&qt[((size_t)h * t + i) * d], &qn[(i * heads + h) * d], sizeof(float) * d);
  for (int h = 0; h < kvh; ++h) {
    if (pre) {
      memcpy(&kt[(size_t)h * kn_total * d], &init->key[(size_t)h * pre * d],
             sizeof(float) * pre * d);
      memcpy(&vt[(size_t)h * kn_total * d], &init->value[(size_t)h * pre * d],
             sizeof(float) * pre * d);
    }
    for (int64_t i = 0; i < t; ++i) {
      memcpy(&kt[((size_t)h * kn_total + pre + i) * d], &kn[(i * kvh + h) * d], sizeof(float) * d);
      memcpy(&vt[((size_t)h * kn_total + pre + i) * d], &vp[(i * kvh + h) * d], sizeof(float) * d);
    }
  }
  if (capture && saved) {
    saved->full = true;
    saved->kv_tokens = capture;
    saved->key.resize((size_t)kvh * capture * d);
    saved->value.resize((size_t)kvh * capture * d);
    for (int h = 0; h < kvh; ++h) {
      memcpy(&saved->key[(size_t)h * capture * d], &kt[(size_t)h * kn_total * d],
             sizeof(float) * capture * d);
      memcpy(&saved->value[(size_t)h * capture * d], &vt[(size_t)h * kn_total * d],
             sizeof(float) * capture * d);
    }
  }
  std::vector<float> att((size_t)heads * t * d);
  attention(qt.data(), kt.data(), vt.data(), heads, kvh, t, kn_total, d, d, true, att.data());
  std::vector<float> o((size_t)t * heads * d);
  for (int64_t i = 0; i < t; ++i)
    for (int h = 0; h < heads; ++h)
      for (int e = 0; e < d; ++e) {
        size_t idx = (i * heads + h) * d + e;
        float av = att[((size_t)h * t + i) * d + e], gv = sigmoidf_(gate[idx]);
        if (g_round & kRoundFlow) {
          av = bf16r(av);
          gv = bf16r(gv);
        }
        o[idx] = av * gv;
      }
  round_if(kRoundOperand | kRoundOpAttnOut, o);
  linear(m, p + ".o_proj.weight", o.data(), t, mixed_out);
}

// Backbone::prefill / prefill_embedded (qwen.rs:337-426).
int prefill(const Model& m, const int32_t* ids, int64_t t, const Prefix* init, int64_t capture,
            float* hidden_out, Prefix** captured) {
  const clef_config& c = m.c;
  const int64_t hsz = c.hidden_size;
  const int64_t offset = init ? init->tokens : 0;
  if (t <= 0) return fail("prefill: empty ids");
  for (int64_t i = 0; i < t; ++i)
    if (ids[i] < 0 || ids[i] >= c.vocab_size) return fail("prefill: token outside vocabulary");
  // Backbone::prefill (qwen.rs:349-358): 0 < capture < ids.len().
  if (capture < 0 || (capture > 0 && capture >= t)) return fail("prefill: capture boundary");
  if (init && capture) return fail("prefill: initial state and capture together");
  if (init && (int)init->layers.size() != c.num_hidden_layers)
    return fail("prefill: prefix layer count");
  const auto& emb = W(m, "model.language_model.embed_tokens.weight").data;
  std::vector<float> h((size_t)t * hsz);
  for (int64_t i = 0; i < t; ++i)
    memcpy(&h[i * hsz], &emb[(size_t)ids[i] * hsz], sizeof(float) * hsz);
  std::vector<int64_t> pos(t);
  for (int64_t i = 0; i < t; ++i) pos[i] = offset + i;
  std::unique_ptr<Prefix> saved;
  if (capture) {
    saved.reset(new Prefix());
    saved->layers.resize(c.num_hidden_layers);
    saved->tokens = capture;
  }
  std::vector<float> u((size_t)t * hsz), mixed, ff;
  for (int li = 0; li < c.num_hidden_layers; ++li) {
    const std::string p = L(li);
    const std::vector<float> wi = norm_weight(m, p + ".input_layernorm.weight", true);
    rms_rows(h.data(), wi.data(), t, hsz, c.rms_norm_eps, u.data());
    round_if(kRoundOperand | kRoundOpMixIn, u);
    const LayerState* st = init ? &init->layers[li] : nullptr;
    LayerState* sv = saved ? &saved->layers[li] : nullptr;
    if (c.layer_types[li])
      attention_forward(m, li, u.data(), t, pos.data(), st, capture, sv, mixed);
    else
      delta_forward(m, li, u.data(), t, st, capture, sv, mixed);
    for (int64_t i = 0; i < t * hsz; ++i) h[i] = h[i] + mixed[i];
    const std::vector<float> wp = norm_weight(m, p + ".post_attention_layernorm.weight", true);
    rms_rows(h.data(), wp.data(), t, hsz, c.rms_norm_eps, u.data());
    round_if(kRoundOperand | kRoundOpMlpIn, u);
    std::vector<float> gt, up;
    linear(m, p + ".mlp.gate_proj.weight", u.data(), t, gt);
    linear(m, p + ".mlp.up_proj.weight", u.data(), t, up);
    for (size_t i = 0; i < gt.size(); ++i) gt[i] = siluf_(gt[i]) * up[i];
    round_if(kRoundOperand | kRoundOpDown, gt);
    linear(m, p + ".mlp.down_proj.weight", gt.data(), t, ff);
    for (int64_t i = 0; i < t * hsz; ++i) h[i] = h[i] + ff[i];
  }
  const std::vector<float> wf = norm_weight(m, "model.language_model.norm.weight", true);
  std::vector<float> out((size_t)t * hsz);
  rms_rows(h.data(), wf.data(), t, hsz, c.rms_norm_eps, out.data());
  if (saved) saved->hidden.assign(out.begin(), out.begin() + capture * hsz);
  if (hidden_out) {
    int64_t pre = 0;
    if (init) {
      memcpy(hidden_out, init->hidden.data(), sizeof(float) * init->hidden.size());
      pre = (int64_t)init->hidden.size();
    }
    memcpy(hidden_out + pre, out.data(), sizeof(float) * out.size());
  }
  if (captured) *captured = saved.release();
  return 0;
}

}  // namespace

// ---------------------------------------------------------------------------
// C interface used by the Python test harness (ctypes).
// ---------------------------------------------------------------------------
extern "C" {

const char* oracle_last_error(void) { return g_err.c_str(); }
void oracle_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
int oracle_max_threads(void) { return omp_get_max_threads(); }
// BF16 rounding points (mask of kRound* bits); 0, the default, is the
// reference's F32 path. Process-wide: set it before a prefill.
void oracle_set_rounding(int mask) { g_round = mask; }
int oracle_rounding(void) { return g_round; }

void oracle_linear(const float* x, int64_t m, const float* w, int64_t n, int64_t k, float* out) {
  gemm_plain(x, m, w, n, k, out);
}
void oracle_rms(const float* x, const float* w, int64_t rows, int64_t width, float eps,
                float* out) {
  rms_rows(x, w, rows, width, eps, out);
}
void oracle_conv4(const float* x, int64_t t, int64_t width, const float* w, float* out) {
  conv4(x, t, width, w, 4, out);
}
// Public DeltaNet operator: q, k [t, hk, kd] raw (normalised inside, as the
// reference's delta_recurrence does); state [hv, kd, vd] in/out (zeros for a
// fresh sequence); captured [hv, kd, vd] at token `capture` (0 = none).
void oracle_delta_recurrence(const float* q, const float* k, const float* v, const float* g,
                             const float* beta, int64_t t, int hk, int hv, int kd, int vd,
                             float* state, int64_t capture, float* captured, float* out) {
  delta_recurrence(q, k, v, g, beta, t, hk, hv, kd, vd, state, capture, captured, out);
}
void oracle_attention(const float* q, const float* k, const float* v, int heads, int kv_heads,
                      int64_t qn, int64_t kn, int width, int causal, float* out) {
  attention(q, k, v, heads, kv_heads, qn, kn, width, width, causal != 0, out);
}
void oracle_rotary(float* x, int64_t tokens, int heads, int width, const int64_t* positions,
                   int dim, double theta) {
  rotary(x, tokens, heads, width, positions, dim, theta);
}

void* oracle_model_create(const clef_config* c) {
  Model* m = new Model();
  m->c = *c;
  declare_all(*m);
  return m;
}
void oracle_model_destroy(void* m) { delete (Model*)m; }
int oracle_model_set_weight(void* mp, const char* name, const float* data, int64_t count) {
  Model* m = (Model*)mp;
  auto it = m->w.find(name);
  if (it == m->w.end()) return fail(std::string("unknown tensor ") + name);
  int64_t n = 1;
  for (auto s : it->second.shape) n *= s;
  if (n != count) return fail(std::string("shape mismatch for ") + name);
  it->second.present = true;
  if (it->second.projection) {
    // Projections are only read through the packed panels; keep no second copy.
    pack_weight(data, it->second.shape[0], it->second.shape[1], it->second.packed);
    it->second.data.clear();
    it->second.data.shrink_to_fit();
  } else {
    it->second.data.assign(data, data + count);
  }
  return 0;
}
int64_t oracle_model_weight_count(void* mp, const char* name) {
  Model* m = (Model*)mp;
  auto it = m->w.find(name);
  if (it == m->w.end()) return 0;
  int64_t n = 1;
  for (auto s : it->second.shape) n *= s;
  return n;
}
// Number of declared tensors and their names (for iteration from Python).
int oracle_model_num_weights(void* mp) { return (int)((Model*)mp)->w.size(); }
const char* oracle_model_weight_name(void* mp, int i) {
  Model* m = (Model*)mp;
  auto it = m->w.begin();
  std::advance(it, i);
  return it->first.c_str();
}
int oracle_model_check(void* mp) {
  Model* m = (Model*)mp;
  for (auto& kv : m->w)
    if (!kv.second.present) return fail("missing tensor " + kv.first);
  return 0;
}
// hidden_out: [prefix tokens + t, hidden] (final-normed); captured: Prefix*.
int oracle_model_prefill(void* mp, const int32_t* ids, int64_t t, const void* init,
                         int64_t capture, float* hidden_out, void** captured) {
  Prefix* cap = nullptr;
  int rc = prefill(*(Model*)mp, ids, t, (const Prefix*)init, capture, hidden_out,
                   captured ? &cap : nullptr);
  if (captured) *captured = cap;
  return rc;
}
int64_t oracle_prefix_tokens(const void* p) { return ((const Prefix*)p)->tokens; }
// Byte count in the reference's accounting (PrefixState::bytes, qwen.rs:173-190):
// F32 elements of hidden, K/V, recurrent states and conv history.
int64_t oracle_prefix_bytes(const void* pp) {
  const Prefix* p = (const Prefix*)pp;
  int64_t n = (int64_t)p->hidden.size();
  for (auto& l : p->layers)
    n += l.full ? (int64_t)(l.key.size() + l.value.size())
                : (int64_t)(l.recurrent.size() + l.history.size());
  return n * 4;
}
void oracle_prefix_destroy(void* p) { delete (Prefix*)p; }

// Schema head (linear, F32): logits[n_out] = W[n_out, hidden] * h.
void oracle_head(const float* h, const float* w, int n_out, int hidden, float* logits) {
  for (int o = 0; o < n_out; ++o) {
    float acc = 0.f;
    for (int i = 0; i < hidden; ++i) acc += w[(size_t)o * hidden + i] * h[i];
    logits[o] = acc;
  }
}

}  // extern "C"
