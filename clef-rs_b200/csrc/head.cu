// head.cu — the reference's learned joint schema head on the GPU, in F32.
//
// Follows Head::forward (crates/core/src/models/head.rs:147-274) step by step:
// LayerNorm of the backbone's hidden rows, the memory projection, span means of
// the instruction and option spans, lexical means of the options' output
// embeddings, two evidence-routing layers (option queries cross-attend to the
// normalised memory, GELU feed-forward), the option summaries, four decoder
// layers over one field per question (self-attention, cross-attention to the
// memory, GELU feed-forward) and the joint scorer (lexical prior, cosine and
// residual MLP). Every tensor is F32 like the reference's head; products use
// F32 fused multiply-adds with F32 accumulation.
//
// The work of one record is a fixed sequence of small kernels on one stream:
// the T-row operations (LayerNorm, memory projection, the key/value
// projections of the memory for all six cross-attention layers) are the bulk;
// everything per option or per question has at most a few dozen rows.
#include <cmath>
#include <map>
#include <string>
#include <vector>

#include "kernels.cuh"

struct clef_head {
  clef_head_config cfg;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::map<std::string, std::vector<int64_t>> specs;  // expected name -> shape
  std::map<std::string, std::vector<float>> host;     // loaded, not yet uploaded
  std::map<std::string, int64_t> off;                 // name -> float offset in blob
  float* blob = nullptr;
  float* dec_kv_w = nullptr;  // [layers * 2 * width, width] decoder cross-attention K | V
  float* dec_kv_b = nullptr;  // [layers * 2 * width]
  bool finalized = false;
  float prior_scale = 0.f, joint_scale = 0.f, gate = 0.f;
  // workspace
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int32_t* meta_d = nullptr;
  size_t meta_cap = 0;
};

namespace clef {
namespace {

// ---- F32 GEMM on the CUDA cores --------------------------------------------
// out[m, n] = res[m, n] + act(X[m, :] . W[n, :] + bias[n]); 64 x 64 tiles,
// 16-wide K slabs through shared memory, 4 x 4 outputs per thread.
constexpr int FB_M = 64, FB_N = 64, FB_K = 16;

__device__ __forceinline__ float gelu_erf(float x) {
  // gelu_erf: 0.5 x (1 + erf(x / sqrt 2)).
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.f, erff(x * 0.70710678118654752f)));
}

__global__ void __launch_bounds__(256) f32_gemm_kernel(const float* __restrict__ X, int64_t ldx,
                                                       const float* __restrict__ W, int64_t ldw, int M,
                                                       int N, int K, const float* __restrict__ bias,
                                                       int gelu, const float* res, int64_t ldr, float* out,
                                                       int64_t ldo) {
  __shared__ __align__(16) float As[FB_K][FB_M + 4];
  __shared__ __align__(16) float Ws[FB_K][FB_N + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * FB_M, n0 = blockIdx.x * FB_N;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += FB_K) {
    for (int i = threadIdx.x; i < FB_M * FB_K; i += 256) {
      const int r = i / FB_K, kk = i % FB_K, k = k0 + kk;
      const int m = m0 + r, n = n0 + r;
      As[kk][r] = (m < M && k < K) ? X[(int64_t)m * ldx + k] : 0.f;
      Ws[kk][r] = (n < N && k < K) ? W[(int64_t)n * ldw + k] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < FB_K; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Ws[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (bias) v = __fadd_rn(v, bias[n]);
      if (gelu) v = gelu_erf(v);
      if (res) v = __fadd_rn(res[(int64_t)m * ldr + n], v);
      out[(int64_t)m * ldo + n] = v;
    }
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
  return t;
}

// Norm::forward (ops.rs:43-60): (x - mean) / sqrt(var + eps) * w + b per row.
__global__ void __launch_bounds__(256) layer_norm_kernel(const float* __restrict__ x, int64_t ldx, int n,
                                                         const float* __restrict__ w,
                                                         const float* __restrict__ b, float eps,
                                                         float* __restrict__ out, int64_t ldo) {
  __shared__ float red[32];
  const float* xr = x + (int64_t)blockIdx.x * ldx;
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += xr[i];
  const float mean = block_sum(s, red) / (float)n;
  float v = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float d = __fsub_rn(xr[i], mean);
    v = fmaf(d, d, v);
  }
  const float var = block_sum(v, red) / (float)n;
  const float den = sqrtf(__fadd_rn(var, eps));
  float* orow = out + (int64_t)blockIdx.x * ldo;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    orow[i] = __fadd_rn(__fmul_rn(__fdiv_rn(__fsub_rn(xr[i], mean), den), w[i]), b[i]);
}

// mean_span (head.rs:275-279) over spans [2s, 2s+1]; with `ids`, the rows are
// the output-embedding rows of those token ids (head.rs:168-180).
__global__ void span_mean_kernel(const float* __restrict__ x, int64_t ldx, int width,
                                 const int32_t* __restrict__ spans, const int32_t* __restrict__ ids,
                                 float* __restrict__ out, int64_t ldo) {
  const int s = blockIdx.x;
  const int start = spans[2 * s], end = spans[2 * s + 1];
  const float count = (float)(end - start);
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float acc = 0.f;
    for (int t = start; t < end; ++t) {
      const int64_t row = ids ? ids[t] : t;
      acc = __fadd_rn(acc, x[row * ldx + c]);
    }
    out[(int64_t)s * ldo + c] = __fdiv_rn(acc, count);
  }
}

// Non-causal softmax attention of one query row and one head over nk keys
// (attention, ops.rs:62-143): scores in shared memory, then the weighted sum
// of the value rows with (256 / hd) key groups per output feature.
__global__ void __launch_bounds__(256) attention_f32_kernel(const float* __restrict__ Q, int64_t ldq,
                                                            const float* __restrict__ K, int64_t ldk,
                                                            const float* __restrict__ V, int64_t ldv,
                                                            int nk, int hd, float scale,
                                                            float* __restrict__ out, int64_t ldo) {
  extern __shared__ float hsm[];
  float* qv = hsm;            // [hd]
  float* part = hsm + 256;    // [256]
  float* red = part + 256;    // [32]
  float* sc = red + 32;       // [nk]
  const int qi = blockIdx.x, h = blockIdx.y;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) qv[d] = Q[(int64_t)qi * ldq + (int64_t)h * hd + d];
  __syncthreads();
  float mx = -INFINITY;
  for (int t = threadIdx.x; t < nk; t += blockDim.x) {
    const float* kr = K + (int64_t)t * ldk + (int64_t)h * hd;
    float s = 0.f;
    for (int d = 0; d < hd; ++d) s = fmaf(qv[d], kr[d], s);
    s = __fmul_rn(s, scale);
    sc[t] = s;
    mx = fmaxf(mx, s);
  }
  mx = block_max(mx, red);
  float sum = 0.f;
  for (int t = threadIdx.x; t < nk; t += blockDim.x) {
    const float p = expf(__fsub_rn(sc[t], mx));
    sc[t] = p;
    sum += p;
  }
  sum = block_sum(sum, red);  // also orders the sc[] writes before the reads below
  const int groups = blockDim.x / hd;
  const int d = threadIdx.x % hd, g = threadIdx.x / hd;
  float acc = 0.f;
  if (g < groups)
    for (int t = g; t < nk; t += groups) acc = fmaf(sc[t], V[(int64_t)t * ldv + (int64_t)h * hd + d], acc);
  part[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x < hd) {
    float o = 0.f;
    for (int gi = 0; gi < groups; ++gi) o = __fadd_rn(o, part[gi * hd + threadIdx.x]);
    out[(int64_t)qi * ldo + (int64_t)h * hd + threadIdx.x] = __fdiv_rn(o, sum);
  }
}

// out[o, :] += src[idx[o], :] (the option-question projection, head.rs:181-183).
__global__ void add_rows_kernel(float* __restrict__ out, int64_t ldo, const float* __restrict__ src,
                                int64_t lds, const int32_t* __restrict__ idx, int width) {
  const int o = blockIdx.x;
  const float* s = src + (int64_t)idx[o] * lds;
  for (int c = threadIdx.x; c < width; c += blockDim.x)
    out[(int64_t)o * ldo + c] = __fadd_rn(out[(int64_t)o * ldo + c], s[c]);
}

// Option summaries (head.rs:208-220): softmax over a question's options of
// (option . base) / sqrt(width), then the weighted sum of the option rows.
__global__ void __launch_bounds__(256) summaries_kernel(const float* __restrict__ routed, int64_t ldr,
                                                        const float* __restrict__ base, int64_t ldb,
                                                        const int32_t* __restrict__ q_off, int width,
                                                        float inv_sqrt_w, float* __restrict__ out,
                                                        int64_t ldo) {
  __shared__ float red[32];
  __shared__ float wts[64];
  const int q = blockIdx.x;
  const int o0 = q_off[q], cnt = q_off[q + 1] - o0;
  for (int i = 0; i < cnt; ++i) {
    float s = 0.f;
    for (int c = threadIdx.x; c < width; c += blockDim.x)
      s = fmaf(routed[(int64_t)(o0 + i) * ldr + c], base[(int64_t)q * ldb + c], s);
    s = block_sum(s, red);
    if (threadIdx.x == 0) wts[i] = __fmul_rn(s, inv_sqrt_w);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mx = -INFINITY;
    for (int i = 0; i < cnt; ++i) mx = fmaxf(mx, wts[i]);
    float sum = 0.f;
    for (int i = 0; i < cnt; ++i) {
      wts[i] = expf(__fsub_rn(wts[i], mx));
      sum = __fadd_rn(sum, wts[i]);
    }
    for (int i = 0; i < cnt; ++i) wts[i] = __fdiv_rn(wts[i], sum);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < cnt; ++i) acc = __fadd_rn(acc, __fmul_rn(routed[(int64_t)(o0 + i) * ldr + c], wts[i]));
    out[(int64_t)q * ldo + c] = acc;
  }
}

// fields = base + LN(summaries) + global projection + type vector (head.rs:222-229).
__global__ void fields_kernel(const float* __restrict__ base, const float* __restrict__ summ,
                              const float* __restrict__ gproj, const float* __restrict__ types,
                              const int32_t* __restrict__ kinds, int width, float* __restrict__ out) {
  const int q = blockIdx.x;
  const float* ty = types + (int64_t)kinds[q] * width;
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    const int64_t i = (int64_t)q * width + c;
    out[i] = __fadd_rn(__fadd_rn(__fadd_rn(base[i], summ[i]), gproj[c]), ty[c]);
  }
}

// anchor_q = normalize(question_q + global, 1e-12) over the hidden width (head.rs:244).
__global__ void __launch_bounds__(256) anchor_kernel(const float* __restrict__ qs, const float* __restrict__ glob,
                                                     int h, float* __restrict__ out) {
  __shared__ float red[32];
  const int q = blockIdx.x;
  float s = 0.f;
  for (int c = threadIdx.x; c < h; c += blockDim.x) {
    const float v = __fadd_rn(qs[(int64_t)q * h + c], glob[c]);
    s = fmaf(v, v, s);
  }
  const float n = fmaxf(sqrtf(block_sum(s, red)), 1e-12f);
  for (int c = threadIdx.x; c < h; c += blockDim.x)
    out[(int64_t)q * h + c] = __fdiv_rn(__fadd_rn(qs[(int64_t)q * h + c], glob[c]), n);
}

// Per option: lexical prior, cosine of the normalised field and option, and
// the scorer features [field, option, field * option, |field - option|]
// (head.rs:243-258).
__global__ void __launch_bounds__(256) score_prep_kernel(
    const float* __restrict__ fields, const float* __restrict__ opts, const float* __restrict__ lex,
    const float* __restrict__ anchor, const int32_t* __restrict__ opt_q, int width, int h,
    float prior_scale, float* __restrict__ feats, float* __restrict__ prior, float* __restrict__ cosine) {
  __shared__ float red[32];
  const int o = blockIdx.x, q = opt_q[o];
  const float* f = fields + (int64_t)q * width;
  const float* p = opts + (int64_t)o * width;
  const float* l = lex + (int64_t)o * h;
  const float* a = anchor + (int64_t)q * h;
  float ll = 0.f;
  for (int c = threadIdx.x; c < h; c += blockDim.x) ll = fmaf(l[c], l[c], ll);
  const float ln = fmaxf(sqrtf(block_sum(ll, red)), 1e-12f);
  float dp = 0.f;
  for (int c = threadIdx.x; c < h; c += blockDim.x) dp = fmaf(__fdiv_rn(l[c], ln), a[c], dp);
  dp = block_sum(dp, red);
  float ff = 0.f, pp = 0.f;
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    ff = fmaf(f[c], f[c], ff);
    pp = fmaf(p[c], p[c], pp);
  }
  const float fn = fmaxf(sqrtf(block_sum(ff, red)), 1e-8f);
  const float pn = fmaxf(sqrtf(block_sum(pp, red)), 1e-8f);
  float cs = 0.f;
  float* ft = feats + (int64_t)o * 4 * width;
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    cs = fmaf(__fdiv_rn(f[c], fn), __fdiv_rn(p[c], pn), cs);
    ft[c] = f[c];
    ft[width + c] = p[c];
    ft[2 * width + c] = __fmul_rn(f[c], p[c]);
    ft[3 * width + c] = fabsf(__fsub_rn(f[c], p[c]));
  }
  cs = block_sum(cs, red);
  if (threadIdx.x == 0) {
    prior[o] = __fmul_rn(dp, prior_scale);
    cosine[o] = cs;
  }
}

// logit = prior + (cosine * joint_scale + residual) * gate (head.rs:259-263).
__global__ void logits_kernel(const float* __restrict__ prior, const float* __restrict__ cosine,
                              const float* __restrict__ resid, int n, float joint_scale, float gate,
                              float* __restrict__ out) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o < n)
    out[o] = __fadd_rn(prior[o], __fmul_rn(__fadd_rn(__fmul_rn(cosine[o], joint_scale), resid[o]), gate));
}

int gemm_f32(const float* X, int64_t ldx, const float* W, int64_t ldw, int M, int N, int K, const float* bias,
             bool gelu, const float* res, int64_t ldr, float* out, int64_t ldo, cudaStream_t s) {
  if (M == 0 || N == 0) return CLEF_OK;
  const dim3 grid((unsigned)ceil_div(N, FB_N), (unsigned)ceil_div(M, FB_M));
  CLEF_CHECK(grid.y <= 65535u, CLEF_ERR_UNSUPPORTED, "head: too many rows");
  f32_gemm_kernel<<<grid, 256, 0, s>>>(X, ldx, W, ldw, M, N, K, bias, gelu ? 1 : 0, res, ldr, out, ldo);
  return launch_status("head gemm");
}

int layer_norm(const float* x, int64_t ldx, int rows, int n, const float* w, const float* b, float* out,
               int64_t ldo, cudaStream_t s) {
  if (rows == 0) return CLEF_OK;
  layer_norm_kernel<<<rows, 256, 0, s>>>(x, ldx, n, w, b, 1e-5f, out, ldo);
  return launch_status("head layer_norm");
}

constexpr int kMaxKeys = 48 * 1024;

int attention_f32(const float* Q, int64_t ldq, const float* K, int64_t ldk, const float* V, int64_t ldv, int nq,
                  int nk, int heads, int hd, float* out, int64_t ldo, cudaStream_t s) {
  if (nq == 0) return CLEF_OK;
  CLEF_CHECK(nk <= kMaxKeys, CLEF_ERR_UNSUPPORTED, "head: more than 49152 memory rows");
  const size_t smem = sizeof(float) * (256 + 256 + 32 + (size_t)nk);
  static bool attr[64] = {false};
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    CLEF_CUDA(cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)(sizeof(float) * (256 + 256 + 32 + kMaxKeys))));
    attr[dev] = true;
  }
  attention_f32_kernel<<<dim3((unsigned)nq, (unsigned)heads), 256, smem, s>>>(
      Q, ldq, K, ldk, V, ldv, nk, hd, (float)(1.0 / std::sqrt((double)hd)), out, ldo);
  return launch_status("head attention");
}

// Tensor names and shapes of the head (head.rs:91-145, weights.rs:135-188).
std::map<std::string, std::vector<int64_t>> head_specs(const clef_head_config& c) {
  std::map<std::string, std::vector<int64_t>> m;
  const int64_t h = c.hidden_size, w = c.width, f = c.feedforward;
  auto lin = [&](const std::string& n, int64_t o, int64_t i, bool bias) {
    m[n + ".weight"] = {o, i};
    if (bias) m[n + ".bias"] = {o};
  };
  auto norm = [&](const std::string& n, int64_t k) {
    m[n + ".weight"] = {k};
    m[n + ".bias"] = {k};
  };
  auto attn = [&](const std::string& n) {
    m[n + ".in_proj_weight"] = {3 * w, w};
    m[n + ".in_proj_bias"] = {3 * w};
    lin(n + ".out_proj", w, w, true);
  };
  for (int r = 0; r < c.routing_layers; ++r) {
    const std::string p = "evidence_layers." + std::to_string(r);
    norm(p + ".query_norm", w);
    norm(p + ".memory_norm", w);
    attn(p + ".attention");
    norm(p + ".feedforward_norm", w);
    lin(p + ".feedforward.0", f, w, true);
    lin(p + ".feedforward.3", w, f, true);
  }
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l);
    norm(p + ".norm1", w);
    norm(p + ".norm2", w);
    norm(p + ".norm3", w);
    attn(p + ".self_attn");
    attn(p + ".multihead_attn");
    lin(p + ".linear1", f, w, true);
    lin(p + ".linear2", w, f, true);
  }
  norm("hidden_norm", h);
  for (const char* n : {"memory_projection", "question_projection", "option_question_projection",
                        "global_projection", "option_context_projection", "option_lexical_projection"})
    lin(n, w, h, false);
  m["type_embedding.weight"] = {3, w};
  norm("option_summary_norm", w);
  norm("field_norm", w);
  norm("option_norm", w);
  lin("residual_scorer.0", w, 4 * w, true);
  lin("residual_scorer.3", 1, w, true);
  m["prior_logit_scale"] = {};
  m["joint_logit_scale"] = {};
  m["residual_gate"] = {};
  return m;
}

int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}

struct DeviceGuardH {
  int prev = -1;
  explicit DeviceGuardH(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuardH() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace clef

using namespace clef;

namespace {

const float* W(const clef_head* hd, const std::string& name) { return hd->blob + hd->off.at(name); }

// Workspace layout for one record; every slot is a multiple of 64 floats.
struct HeadWs {
  float *normalized, *memory, *nm, *kv, *qs, *ctx, *lex, *routed, *tq, *q, *att, *ffh, *base, *oq, *summ,
      *summn, *fields, *gproj, *qkv, *anchor, *opts, *feats, *r1, *resid, *prior, *cosine, *logits;
};

size_t plan_ws(const clef_head_config& c, int64_t T, int nq, int no, float* base, HeadWs* w) {
  size_t off = 0;
  const int64_t h = c.hidden_size, wd = c.width, ff = c.feedforward;
  const int64_t rows = std::max(nq, no);
  const int64_t kvw = std::max<int64_t>(2 * wd, 2 * wd * c.layers);
  auto take = [&](float** p, int64_t n) {
    if (w) *p = base + off;
    off += (size_t)((n + 63) / 64 * 64);
  };
  HeadWs d;
  HeadWs* t = w ? w : &d;
  take(&t->normalized, T * h);
  take(&t->memory, T * wd);
  take(&t->nm, T * wd);
  take(&t->kv, T * kvw);
  take(&t->qs, nq * h);
  take(&t->ctx, no * h);
  take(&t->lex, no * h);
  take(&t->routed, no * wd);
  take(&t->tq, rows * wd);
  take(&t->q, rows * wd);
  take(&t->att, rows * wd);
  take(&t->ffh, rows * ff);
  take(&t->base, nq * wd);
  take(&t->oq, nq * wd);
  take(&t->summ, nq * wd);
  take(&t->summn, nq * wd);
  take(&t->fields, nq * wd);
  take(&t->gproj, wd);
  take(&t->qkv, nq * 3 * wd);
  take(&t->anchor, nq * h);
  take(&t->opts, no * wd);
  take(&t->feats, no * 4 * wd);
  take(&t->r1, no * wd);
  take(&t->resid, no);
  take(&t->prior, no);
  take(&t->cosine, no);
  take(&t->logits, no);
  return off * sizeof(float);
}

}  // namespace

extern "C" {

int clef_head_create(const clef_head_config* cfg, int32_t device, clef_head** out) {
  CLEF_CHECK(cfg && out, CLEF_ERR_INVALID, "head_create: null argument");
  *out = nullptr;
  const clef_head_config& c = *cfg;
  CLEF_CHECK(c.hidden_size > 0 && c.width > 0 && c.heads > 0 && c.feedforward > 0 && c.routing_layers >= 0 &&
                 c.layers >= 0 && c.layers <= 64 && c.routing_layers <= 64,
             CLEF_ERR_INVALID, "head_create: dimensions");
  CLEF_CHECK(c.width % c.heads == 0 && 256 % (c.width / c.heads) == 0, CLEF_ERR_UNSUPPORTED,
             "head_create: head width (width / heads) must divide 256");
  int n = 0;
  CLEF_CUDA(cudaGetDeviceCount(&n));
  CLEF_CHECK(device >= 0 && device < n, CLEF_ERR_INVALID, "head_create: device");
  auto* hd = new clef_head();
  hd->cfg = c;
  hd->device = device;
  hd->specs = head_specs(c);
  DeviceGuardH g(device);
  if (cudaStreamCreateWithFlags(&hd->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete hd;
    return fail(CLEF_ERR_CUDA, "head_create: stream");
  }
  *out = hd;
  return CLEF_OK;
}

int clef_head_set_weight(clef_head* hd, const char* name, const float* data, int64_t count) {
  CLEF_CHECK(hd && name && (data || count == 0), CLEF_ERR_INVALID, "head_set_weight: null argument");
  CLEF_CHECK(!hd->finalized, CLEF_ERR_INVALID, "head_set_weight: head already finalized");
  auto it = hd->specs.find(name);
  CLEF_CHECK(it != hd->specs.end(), CLEF_ERR_INVALID, std::string("head_set_weight: unknown tensor ") + name);
  CLEF_CHECK(count == numel(it->second), CLEF_ERR_INVALID, std::string("head_set_weight: tensor shape ") + name);
  hd->host[name].assign(data, data + count);
  return CLEF_OK;
}

int clef_head_finalize(clef_head* hd) {
  CLEF_CHECK(hd, CLEF_ERR_INVALID, "head_finalize: null handle");
  CLEF_CHECK(!hd->finalized, CLEF_ERR_INVALID, "head_finalize: already finalized");
  for (const auto& kv : hd->specs)
    CLEF_CHECK(hd->host.count(kv.first), CLEF_ERR_INVALID, "head_finalize: missing tensor " + kv.first);
  for (const char* s : {"prior_logit_scale", "joint_logit_scale", "residual_gate"})
    CLEF_CHECK(std::isfinite(hd->host[s][0]), CLEF_ERR_INVALID, "head_finalize: nonfinite scalar");
  const clef_head_config& c = hd->cfg;
  const int64_t w = c.width;
  int64_t total = 0;
  for (const auto& kv : hd->specs) {
    hd->off[kv.first] = total;
    total += (numel(kv.second) + 63) / 64 * 64;
  }
  const int64_t kvn = 2 * w * c.layers;  // fused decoder K | V rows
  const int64_t kvw_off = total;
  total += (kvn * w + 63) / 64 * 64;
  const int64_t kvb_off = total;
  total += (kvn + 63) / 64 * 64;
  DeviceGuardH g(hd->device);
  CLEF_CUDA(cudaMalloc(&hd->blob, sizeof(float) * (size_t)std::max<int64_t>(total, 64)));
  std::vector<float> staging((size_t)total, 0.f);
  for (const auto& kv : hd->host)
    std::copy(kv.second.begin(), kv.second.end(), staging.begin() + hd->off[kv.first]);
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".multihead_attn";
    const auto& iw = hd->host[p + ".in_proj_weight"];
    const auto& ib = hd->host[p + ".in_proj_bias"];
    std::copy(iw.begin() + w * w, iw.end(), staging.begin() + kvw_off + (int64_t)l * 2 * w * w);
    std::copy(ib.begin() + w, ib.end(), staging.begin() + kvb_off + (int64_t)l * 2 * w);
  }
  CLEF_CUDA(cudaMemcpy(hd->blob, staging.data(), sizeof(float) * (size_t)total, cudaMemcpyHostToDevice));
  hd->dec_kv_w = hd->blob + kvw_off;
  hd->dec_kv_b = hd->blob + kvb_off;
  // Scalars as Head::load derives them (head.rs:128-130).
  const double lim = std::log(100.0);
  hd->prior_scale = (float)std::exp(std::min((double)hd->host["prior_logit_scale"][0], lim));
  hd->joint_scale = (float)std::exp(std::min((double)hd->host["joint_logit_scale"][0], lim));
  hd->gate = (float)(1.0 / (1.0 + std::exp(-(double)hd->host["residual_gate"][0])));
  hd->host.clear();
  hd->finalized = true;
  return CLEF_OK;
}

int clef_head_forward(clef_head* hd, const float* hidden, int64_t T, const float* output_embeddings, int64_t vocab,
                      const int32_t* ids, const clef_head_question* questions, int32_t nq,
                      const int32_t* option_spans, float* logits) {
  CLEF_CHECK(hd && hidden && output_embeddings && ids && questions && option_spans && logits, CLEF_ERR_INVALID,
             "head_forward: null argument");
  CLEF_CHECK(hd->finalized, CLEF_ERR_INVALID, "head_forward: head not finalized");
  CLEF_CHECK(T > 0 && T <= kMaxKeys, CLEF_ERR_INVALID, "head_forward: T must be in [1, 49152]");
  CLEF_CHECK(nq > 0 && nq <= 4096, CLEF_ERR_INVALID, "head_forward: question count");
  CLEF_CHECK(vocab > 0, CLEF_ERR_INVALID, "head_forward: vocab");
  CLEF_CHECK((((uintptr_t)hidden | (uintptr_t)output_embeddings) & 3) == 0, CLEF_ERR_INVALID,
             "head_forward: tensors must be 4-byte aligned");
  const clef_head_config& c = hd->cfg;
  // Record validation (EncodedRecord spans, encoding.rs TokenSpan: start < end <= T).
  int no = 0;
  for (int i = 0; i < nq; ++i) {
    const clef_head_question& q = questions[i];
    CLEF_CHECK(q.kind >= 0 && q.kind < 3, CLEF_ERR_INVALID, "head_forward: question kind");
    CLEF_CHECK(q.instruction_start >= 0 && q.instruction_start < q.instruction_end && q.instruction_end <= T,
               CLEF_ERR_INVALID, "head_forward: instruction span");
    CLEF_CHECK(q.option_count > 0 && q.option_count <= 64 && q.option_offset == no, CLEF_ERR_INVALID,
               "head_forward: options must be 1..64 per question, listed in question order");
    no += q.option_count;
  }
  for (int o = 0; o < no; ++o) {
    const int s = option_spans[2 * o], e = option_spans[2 * o + 1];
    CLEF_CHECK(s >= 0 && s < e && e <= T, CLEF_ERR_INVALID, "head_forward: option span");
  }
  for (int64_t t = 0; t < T; ++t)
    CLEF_CHECK(ids[t] >= 0 && ids[t] < vocab, CLEF_ERR_INVALID, "head_forward: token id out of range");
  DeviceGuardH g(hd->device);
  cudaStream_t s = hd->stream;
  const int64_t h = c.hidden_size, wd = c.width, ff = c.feedforward;
  const int hdim = (int)(wd / c.heads);
  // Metadata: instruction spans | option spans | option -> question | kinds |
  // question option offsets | ids.
  std::vector<int32_t> meta;
  meta.reserve((size_t)(2 * nq + 2 * no + no + nq + nq + 1 + T));
  for (int i = 0; i < nq; ++i) {
    meta.push_back(questions[i].instruction_start);
    meta.push_back(questions[i].instruction_end);
  }
  const size_t m_ospan = meta.size();
  meta.insert(meta.end(), option_spans, option_spans + 2 * no);
  const size_t m_optq = meta.size();
  for (int i = 0; i < nq; ++i)
    for (int k = 0; k < questions[i].option_count; ++k) meta.push_back(i);
  const size_t m_kind = meta.size();
  for (int i = 0; i < nq; ++i) meta.push_back(questions[i].kind);
  const size_t m_qoff = meta.size();
  for (int i = 0; i < nq; ++i) meta.push_back(questions[i].option_offset);
  meta.push_back(no);
  const size_t m_ids = meta.size();
  meta.insert(meta.end(), ids, ids + T);
  if (meta.size() > hd->meta_cap) {
    if (hd->meta_d) cudaFree(hd->meta_d);
    hd->meta_d = nullptr;
    hd->meta_cap = meta.size() * 2;
    CLEF_CUDA(cudaMalloc(&hd->meta_d, sizeof(int32_t) * hd->meta_cap));
  }
  const size_t need = plan_ws(c, T, nq, no, nullptr, nullptr);
  if (need > hd->ws_bytes) {
    if (hd->ws) cudaFree(hd->ws);
    hd->ws = nullptr;
    hd->ws_bytes = 0;
    CLEF_CUDA(cudaMalloc(&hd->ws, need));
    hd->ws_bytes = need;
  }
  HeadWs b;
  plan_ws(c, T, nq, no, reinterpret_cast<float*>(hd->ws), &b);
  CLEF_CUDA(cudaMemcpyAsync(hd->meta_d, meta.data(), sizeof(int32_t) * meta.size(), cudaMemcpyHostToDevice, s));
  const int32_t* d_ispan = hd->meta_d;
  const int32_t* d_ospan = hd->meta_d + m_ospan;
  const int32_t* d_optq = hd->meta_d + m_optq;
  const int32_t* d_kind = hd->meta_d + m_kind;
  const int32_t* d_qoff = hd->meta_d + m_qoff;
  const int32_t* d_ids = hd->meta_d + m_ids;
#define RCH(x)                  \
  do {                          \
    int rc_ = (x);              \
    if (rc_) return rc_;        \
  } while (0)
  const int Ti = (int)T;
  // Memory side (head.rs:154-157).
  RCH(layer_norm(hidden, h, Ti, (int)h, W(hd, "hidden_norm.weight"), W(hd, "hidden_norm.bias"), b.normalized, h, s));
  RCH(gemm_f32(b.normalized, h, W(hd, "memory_projection.weight"), h, Ti, (int)wd, (int)h, nullptr, false, nullptr, 0,
               b.memory, wd, s));
  const float* glob = b.normalized + (T - 1) * h;
  // Questions, option contexts and lexical means (head.rs:158-186).
  span_mean_kernel<<<nq, 256, 0, s>>>(b.normalized, h, (int)h, d_ispan, nullptr, b.qs, h);
  RCH(launch_status("head span_mean"));
  span_mean_kernel<<<no, 256, 0, s>>>(b.normalized, h, (int)h, d_ospan, nullptr, b.ctx, h);
  RCH(launch_status("head span_mean"));
  span_mean_kernel<<<no, 256, 0, s>>>(output_embeddings, h, (int)h, d_ospan, d_ids, b.lex, h);
  RCH(launch_status("head lexical_mean"));
  RCH(gemm_f32(b.ctx, h, W(hd, "option_context_projection.weight"), h, no, (int)wd, (int)h, nullptr, false, nullptr,
               0, b.routed, wd, s));
  RCH(gemm_f32(b.lex, h, W(hd, "option_lexical_projection.weight"), h, no, (int)wd, (int)h, nullptr, false, b.routed,
               wd, b.routed, wd, s));
  RCH(gemm_f32(b.qs, h, W(hd, "option_question_projection.weight"), h, nq, (int)wd, (int)h, nullptr, false, nullptr,
               0, b.oq, wd, s));
  add_rows_kernel<<<no, 256, 0, s>>>(b.routed, wd, b.oq, wd, d_optq, (int)wd);
  RCH(launch_status("head add_rows"));
  // Evidence routing (head.rs:188-205).
  for (int r = 0; r < c.routing_layers; ++r) {
    const std::string p = "evidence_layers." + std::to_string(r);
    const std::string a = p + ".attention";
    RCH(layer_norm(b.routed, wd, no, (int)wd, W(hd, p + ".query_norm.weight"), W(hd, p + ".query_norm.bias"), b.tq,
                   wd, s));
    RCH(layer_norm(b.memory, wd, Ti, (int)wd, W(hd, p + ".memory_norm.weight"), W(hd, p + ".memory_norm.bias"), b.nm,
                   wd, s));
    const float* iw = W(hd, a + ".in_proj_weight");
    const float* ib = W(hd, a + ".in_proj_bias");
    RCH(gemm_f32(b.tq, wd, iw, wd, no, (int)wd, (int)wd, ib, false, nullptr, 0, b.q, wd, s));
    RCH(gemm_f32(b.nm, wd, iw + wd * wd, wd, Ti, (int)(2 * wd), (int)wd, ib + wd, false, nullptr, 0, b.kv, 2 * wd, s));
    RCH(attention_f32(b.q, wd, b.kv, 2 * wd, b.kv + wd, 2 * wd, no, Ti, c.heads, hdim, b.att, wd, s));
    RCH(gemm_f32(b.att, wd, W(hd, a + ".out_proj.weight"), wd, no, (int)wd, (int)wd, W(hd, a + ".out_proj.bias"),
                 false, b.routed, wd, b.routed, wd, s));
    RCH(layer_norm(b.routed, wd, no, (int)wd, W(hd, p + ".feedforward_norm.weight"),
                   W(hd, p + ".feedforward_norm.bias"), b.tq, wd, s));
    RCH(gemm_f32(b.tq, wd, W(hd, p + ".feedforward.0.weight"), wd, no, (int)ff, (int)wd,
                 W(hd, p + ".feedforward.0.bias"), true, nullptr, 0, b.ffh, ff, s));
    RCH(gemm_f32(b.ffh, ff, W(hd, p + ".feedforward.3.weight"), ff, no, (int)wd, (int)ff,
                 W(hd, p + ".feedforward.3.bias"), false, b.routed, wd, b.routed, wd, s));
  }
  // Summaries and fields (head.rs:206-229).
  RCH(gemm_f32(b.qs, h, W(hd, "question_projection.weight"), h, nq, (int)wd, (int)h, nullptr, false, nullptr, 0,
               b.base, wd, s));
  summaries_kernel<<<nq, 256, 0, s>>>(b.routed, wd, b.base, wd, d_qoff, (int)wd,
                                      (float)(1.0 / std::sqrt((double)wd)), b.summ, wd);
  RCH(launch_status("head summaries"));
  RCH(layer_norm(b.summ, wd, nq, (int)wd, W(hd, "option_summary_norm.weight"), W(hd, "option_summary_norm.bias"),
                 b.summn, wd, s));
  RCH(gemm_f32(glob, h, W(hd, "global_projection.weight"), h, 1, (int)wd, (int)h, nullptr, false, nullptr, 0, b.gproj,
               wd, s));
  fields_kernel<<<nq, 256, 0, s>>>(b.base, b.summn, b.gproj, W(hd, "type_embedding.weight"), d_kind, (int)wd,
                                   b.fields);
  RCH(launch_status("head fields"));
  // Decoder layers (head.rs:230-241); the memory's keys and values for all of
  // them come from one projection of the (un-normalised) memory.
  if (c.layers > 0)
    RCH(gemm_f32(b.memory, wd, hd->dec_kv_w, wd, Ti, (int)(2 * wd * c.layers), (int)wd, hd->dec_kv_b, false, nullptr,
                 0, b.kv, 2 * wd * c.layers, s));
  const int64_t ldkv = 2 * wd * c.layers;
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l);
    RCH(layer_norm(b.fields, wd, nq, (int)wd, W(hd, p + ".norm1.weight"), W(hd, p + ".norm1.bias"), b.tq, wd, s));
    RCH(gemm_f32(b.tq, wd, W(hd, p + ".self_attn.in_proj_weight"), wd, nq, (int)(3 * wd), (int)wd,
                 W(hd, p + ".self_attn.in_proj_bias"), false, nullptr, 0, b.qkv, 3 * wd, s));
    RCH(attention_f32(b.qkv, 3 * wd, b.qkv + wd, 3 * wd, b.qkv + 2 * wd, 3 * wd, nq, nq, c.heads, hdim, b.att, wd,
                      s));
    RCH(gemm_f32(b.att, wd, W(hd, p + ".self_attn.out_proj.weight"), wd, nq, (int)wd, (int)wd,
                 W(hd, p + ".self_attn.out_proj.bias"), false, b.fields, wd, b.fields, wd, s));
    RCH(layer_norm(b.fields, wd, nq, (int)wd, W(hd, p + ".norm2.weight"), W(hd, p + ".norm2.bias"), b.tq, wd, s));
    RCH(gemm_f32(b.tq, wd, W(hd, p + ".multihead_attn.in_proj_weight"), wd, nq, (int)wd, (int)wd,
                 W(hd, p + ".multihead_attn.in_proj_bias"), false, nullptr, 0, b.q, wd, s));
    const float* kl = b.kv + (int64_t)l * 2 * wd;
    RCH(attention_f32(b.q, wd, kl, ldkv, kl + wd, ldkv, nq, Ti, c.heads, hdim, b.att, wd, s));
    RCH(gemm_f32(b.att, wd, W(hd, p + ".multihead_attn.out_proj.weight"), wd, nq, (int)wd, (int)wd,
                 W(hd, p + ".multihead_attn.out_proj.bias"), false, b.fields, wd, b.fields, wd, s));
    RCH(layer_norm(b.fields, wd, nq, (int)wd, W(hd, p + ".norm3.weight"), W(hd, p + ".norm3.bias"), b.tq, wd, s));
    RCH(gemm_f32(b.tq, wd, W(hd, p + ".linear1.weight"), wd, nq, (int)ff, (int)wd, W(hd, p + ".linear1.bias"), true,
                 nullptr, 0, b.ffh, ff, s));
    RCH(gemm_f32(b.ffh, ff, W(hd, p + ".linear2.weight"), ff, nq, (int)wd, (int)ff, W(hd, p + ".linear2.bias"), false,
                 b.fields, wd, b.fields, wd, s));
  }
  RCH(layer_norm(b.fields, wd, nq, (int)wd, W(hd, "field_norm.weight"), W(hd, "field_norm.bias"), b.tq, wd, s));
  // Joint scorer (head.rs:242-270).
  anchor_kernel<<<nq, 256, 0, s>>>(b.qs, glob, (int)h, b.anchor);
  RCH(launch_status("head anchor"));
  RCH(layer_norm(b.routed, wd, no, (int)wd, W(hd, "option_norm.weight"), W(hd, "option_norm.bias"), b.opts, wd, s));
  score_prep_kernel<<<no, 256, 0, s>>>(b.tq, b.opts, b.lex, b.anchor, d_optq, (int)wd, (int)h, hd->prior_scale,
                                       b.feats, b.prior, b.cosine);
  RCH(launch_status("head score_prep"));
  RCH(gemm_f32(b.feats, 4 * wd, W(hd, "residual_scorer.0.weight"), 4 * wd, no, (int)wd, (int)(4 * wd),
               W(hd, "residual_scorer.0.bias"), true, nullptr, 0, b.r1, wd, s));
  RCH(gemm_f32(b.r1, wd, W(hd, "residual_scorer.3.weight"), wd, no, 1, (int)wd, W(hd, "residual_scorer.3.bias"),
               false, nullptr, 0, b.resid, 1, s));
  logits_kernel<<<(unsigned)ceil_div(no, 128), 128, 0, s>>>(b.prior, b.cosine, b.resid, no, hd->joint_scale, hd->gate,
                                                           b.logits);
  RCH(launch_status("head logits"));
#undef RCH
  CLEF_CUDA(cudaMemcpyAsync(logits, b.logits, sizeof(float) * no, cudaMemcpyDeviceToHost, s));
  CLEF_CUDA(cudaStreamSynchronize(s));
  for (int o = 0; o < no; ++o)
    CLEF_CHECK(std::isfinite(logits[o]), CLEF_ERR_CUDA, "head_forward: nonfinite head output");
  return CLEF_OK;
}

int clef_head_destroy(clef_head* hd) {
  if (!hd) return CLEF_OK;
  {
    DeviceGuardH g(hd->device);
    if (hd->blob) cudaFree(hd->blob);
    if (hd->ws) cudaFree(hd->ws);
    if (hd->meta_d) cudaFree(hd->meta_d);
    if (hd->stream) cudaStreamDestroy(hd->stream);
  }
  delete hd;
  return CLEF_OK;
}

}  // extern "C"
