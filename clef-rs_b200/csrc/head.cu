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
// The work of one record is a fixed sequence of small kernels on one stream.
// The T-row operations are the LayerNorms and the memory projection; the six
// cross-attention layers are reassociated (qk_fold_kernel) so the memory rows
// are only read, never projected to keys and values; everything per option or
// per question has at most a few dozen rows.
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
  // memory_projection as a three-term BF16 operand [W_hi | W_hi | W_lo]
  // [width, 3 hidden] for the tensor-core path (null when the shapes do not fit it).
  uint16_t* mem_w3 = nullptr;
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

// ---- F32-accurate products on the BF16 tensor cores -------------------------
// x = hi + lo with hi = bf16(x), lo = bf16(x - hi). A product of two such
// pairs keeps hi.hi + lo.hi + hi.lo (the dropped lo.lo term is below 2^-16 of
// it); laid out as X3 = [x_hi | x_lo | x_hi] and W3 = [w_hi | w_hi | w_lo]
// along K it is one BF16 GEMM with K' = 3K and F32 accumulation.
__global__ void split3_rows_kernel(const float* __restrict__ x, int64_t ldx, int64_t rows, int k, int w_side,
                                   uint16_t* __restrict__ out) {
  const int64_t n = rows * k;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / k;
    const int c = (int)(i - r * k);
    const float v = x[r * ldx + c];
    const uint16_t hi = f2bf(v), lo = f2bf(v - bf2f(hi));
    uint16_t* o = out + r * 3 * (int64_t)k;
    o[c] = hi;
    o[k + c] = w_side ? hi : lo;
    o[2 * k + c] = w_side ? lo : hi;
  }
}

int split3(const float* x, int64_t ldx, int64_t rows, int k, bool w_side, uint16_t* out, cudaStream_t s) {
  const int64_t n = rows * k;
  const unsigned blocks = (unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 32);
  split3_rows_kernel<<<blocks, 256, 0, s>>>(x, ldx, rows, k, w_side ? 1 : 0, out);
  return launch_status("head split3");
}

// ---- F32 GEMM on the CUDA cores --------------------------------------------
// out[m, n] = res[m, n] + act(sum_k X[m, k] W[n, k] + bias[n]) with W stored
// [N, K] (a Linear weight), or with W stored [K, N] when W_KN. 128 x 128
// tiles, 8-wide K slabs double-buffered through shared memory (the next slab
// is fetched into registers while the current one is consumed), 8 x 8 outputs
// per thread as four 4 x 4 blocks so every shared-memory read is a broadcast
// or a conflict-free 16-byte load.
constexpr int SG_M = 128, SG_N = 128, SG_K = 8, SG_PAD = 4;

__device__ __forceinline__ float gelu_erf(float x) {
  // gelu_erf: 0.5 x (1 + erf(x / sqrt 2)).
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.f, erff(x * 0.70710678118654752f)));
}

template <bool W_KN>
__global__ void __launch_bounds__(256) sgemm_kernel(const float* __restrict__ X, int64_t ldx,
                                                    const float* __restrict__ W, int64_t ldw, int M, int N,
                                                    int K, int kc, int vec, const float* __restrict__ bias,
                                                    int gelu, const float* res, int64_t ldr, float* out,
                                                    int64_t ldo) {
  // Split K: this CTA sums k in [kb, ke); with gridDim.z > 1 it writes plain
  // partial sums to slice z of `out` (the caller passes no epilogue).
  const int kb = blockIdx.z * kc, ke = min(K, kb + kc);
  if (gridDim.z > 1) out += (int64_t)blockIdx.z * M * ldo;
  __shared__ __align__(16) float As[2][SG_K][SG_M + SG_PAD];
  __shared__ __align__(16) float Bs[2][SG_K][SG_N + SG_PAD];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * SG_M, n0 = blockIdx.x * SG_N;
  // Loader coordinates: X rows (and [N, K] W rows) take 4 consecutive k per
  // thread; a [K, N] W slab takes 4 consecutive n per thread.
  const int lr = tid >> 1, lk = (tid & 1) * 4;
  const int wk = tid >> 5, wn = (tid & 31) * 4;
  float xa[4], wb[4];
  auto load = [&](int k0) {
    const int m = m0 + lr, k = k0 + lk;
    if (vec && m < M && k < ke) {
      const float4 v = *reinterpret_cast<const float4*>(X + (int64_t)m * ldx + k);
      xa[0] = v.x, xa[1] = v.y, xa[2] = v.z, xa[3] = v.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) xa[i] = (m < M && k + i < ke) ? X[(int64_t)m * ldx + k + i] : 0.f;
    }
    if (!W_KN) {
      const int n = n0 + lr;
      if (vec && n < N && k < ke) {
        const float4 v = *reinterpret_cast<const float4*>(W + (int64_t)n * ldw + k);
        wb[0] = v.x, wb[1] = v.y, wb[2] = v.z, wb[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) wb[i] = (n < N && k + i < ke) ? W[(int64_t)n * ldw + k + i] : 0.f;
      }
    } else {
      const int kk = k0 + wk, n = n0 + wn;
      if (vec && kk < ke && n < N) {
        const float4 v = *reinterpret_cast<const float4*>(W + (int64_t)kk * ldw + n);
        wb[0] = v.x, wb[1] = v.y, wb[2] = v.z, wb[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) wb[i] = (kk < ke && n + i < N) ? W[(int64_t)kk * ldw + n + i] : 0.f;
      }
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) As[buf][lk + i][lr] = xa[i];
    if (!W_KN) {
#pragma unroll
      for (int i = 0; i < 4; ++i) Bs[buf][lk + i][lr] = wb[i];
    } else {
      *reinterpret_cast<float4*>(&Bs[buf][wk][wn]) = make_float4(wb[0], wb[1], wb[2], wb[3]);
    }
  };
  const int tx = tid & 15, ty = tid >> 4;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  load(kb);
  store(0);
  __syncthreads();
  for (int k0 = kb, it = 0; k0 < ke; k0 += SG_K, ++it) {
    const int buf = it & 1;
    const bool more = k0 + SG_K < ke;
    if (more) load(k0 + SG_K);
#pragma unroll
    for (int kk = 0; kk < SG_K; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) store(buf ^ 1);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (n >= N) continue;
      float v = acc[i][j];
      if (bias) v = __fadd_rn(v, bias[n]);
      if (gelu) v = gelu_erf(v);
      if (res) v = __fadd_rn(res[(int64_t)m * ldr + n], v);
      out[(int64_t)m * ldo + n] = v;
    }
  }
}

// Skinny GEMM for M <= 16 rows (option and question rows): out[m, n] =
// res + act(X[m, :] . W[n, :] + bias[n]). A CTA covers 32 output columns
// (4 per warp) for all rows; X is staged in shared memory 512 columns of K at
// a time, W rows stream from global memory once, 16-byte loads along K.
constexpr int SK_M = 16, SK_KC = 512, SK_COLS = 4;

struct SkinnyBatch {
  int64_t x, w, out, bias;  // per-batch element offsets (blockIdx.z)
};

__global__ void __launch_bounds__(256) skinny_gemm_kernel(const float* __restrict__ X, int64_t ldx,
                                                          const float* __restrict__ W, int64_t ldw, int M, int N,
                                                          int K, int kc, SkinnyBatch bs,
                                                          const float* __restrict__ bias, int gelu,
                                                          const float* res, int64_t ldr, float* out, int64_t ldo) {
  __shared__ __align__(16) float xs[SK_M][SK_KC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nb = blockIdx.x * 8 * SK_COLS + warp * SK_COLS;
  // Batch element z = blockIdx.z; K slab [kb, ke) = blockIdx.y. With several
  // slabs the CTA writes plain partial sums to slice (y, z) of `out` (layout
  // [slabs][batch][M][N]) and the caller reduces them.
  const int z = blockIdx.z;
  X += z * bs.x;
  W += z * bs.w;
  const int kb = blockIdx.y * kc, ke = min(K, kb + kc);
  if (gridDim.y > 1) {
    out += ((int64_t)blockIdx.y * gridDim.z + z) * M * ldo;
  } else {
    out += z * bs.out;
    if (bias) bias += z * bs.bias;
  }
  float acc[SK_M][SK_COLS];
#pragma unroll
  for (int m = 0; m < SK_M; ++m)
#pragma unroll
    for (int j = 0; j < SK_COLS; ++j) acc[m][j] = 0.f;
  for (int k0 = kb; k0 < ke; k0 += SK_KC) {
    const int kn = min(SK_KC, ke - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < SK_M * (SK_KC / 4); i += blockDim.x) {
      const int m = i / (SK_KC / 4), k = (i % (SK_KC / 4)) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < M && k < kn) {
        const float* src = X + (int64_t)m * ldx + k0 + k;
        v.x = src[0];
        if (k + 1 < kn) v.y = src[1];
        if (k + 2 < kn) v.z = src[2];
        if (k + 3 < kn) v.w = src[3];
      }
      *reinterpret_cast<float4*>(&xs[m][k]) = v;
    }
    __syncthreads();
    for (int k = lane * 4; k < kn; k += 128) {
      float4 wv[SK_COLS];
#pragma unroll
      for (int j = 0; j < SK_COLS; ++j) {
        const int n = nb + j;
        wv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (n < N) {
          const float* src = W + (int64_t)n * ldw + k0 + k;
          wv[j].x = src[0];
          if (k + 1 < kn) wv[j].y = src[1];
          if (k + 2 < kn) wv[j].z = src[2];
          if (k + 3 < kn) wv[j].w = src[3];
        }
      }
#pragma unroll
      for (int m = 0; m < SK_M; ++m) {
        const float4 xv = *reinterpret_cast<const float4*>(&xs[m][k]);
#pragma unroll
        for (int j = 0; j < SK_COLS; ++j) {
          acc[m][j] = fmaf(xv.x, wv[j].x, acc[m][j]);
          acc[m][j] = fmaf(xv.y, wv[j].y, acc[m][j]);
          acc[m][j] = fmaf(xv.z, wv[j].z, acc[m][j]);
          acc[m][j] = fmaf(xv.w, wv[j].w, acc[m][j]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < SK_M; ++m)
#pragma unroll
    for (int j = 0; j < SK_COLS; ++j)
#pragma unroll
      for (int o = 16; o; o >>= 1) acc[m][j] += __shfl_xor_sync(0xffffffffu, acc[m][j], o);
  // Lane l writes entries l and l + 32 of the 16 x 4 block.
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int idx = lane + 32 * e, m = idx / SK_COLS, j = idx % SK_COLS, n = nb + j;
    float v = 0.f;
#pragma unroll
    for (int mm = 0; mm < SK_M; ++mm)
#pragma unroll
      for (int jj = 0; jj < SK_COLS; ++jj)
        if (mm * SK_COLS + jj == idx) v = acc[mm][jj];
    if (m < M && n < N) {
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

// Cross-attention of a few query rows over the T memory rows, reassociated
// so the memory is never projected to keys and values (MultiAttention::forward,
// ops.rs:198-224, with k_t = Wk m_t + bk and v_t = Wv m_t + bv):
//   score(o, h, t) = q_oh . (Wk_h m_t + bk_h) = (Wk_h^T q_oh) . m_t + q_oh . bk_h,
// and the last term is the same for every t, so it cancels in the softmax;
//   out(o, h) = sum_t p_t (Wv_h m_t + bv_h) = Wv_h (sum_t p_t m_t) + bv_h,
// as the probabilities sum to one. Rows of U, S and C are (o, h) pairs.

// U[(o, h), c] = sum_d q[o, h*hd + d] * Wk[h*hd + d, c]. CTA = (256 columns,
// head, 16 query rows): the rows' head slice of q sits in shared memory and
// each Wk element is read once per CTA.
__global__ void __launch_bounds__(256) qk_fold_kernel(const float* __restrict__ q, int64_t ldq,
                                                      const float* __restrict__ Wk, int width, int heads, int hd,
                                                      int R0, float* __restrict__ U) {
  __shared__ float qs[16][256];
  const int h = blockIdx.y, r0 = blockIdx.z * 16;
  const int nr = min(16, R0 - r0);
  for (int i = threadIdx.x; i < 16 * hd; i += blockDim.x) {
    const int r = i / hd, d = i % hd;
    qs[r][d] = r < nr ? q[(int64_t)(r0 + r) * ldq + (int64_t)h * hd + d] : 0.f;
  }
  __syncthreads();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= width) return;
  float acc[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) acc[r] = 0.f;
  const float* wk = Wk + (int64_t)h * hd * width + c;
  for (int d = 0; d < hd; ++d) {
    const float w = wk[(int64_t)d * width];
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = fmaf(qs[r][d], w, acc[r]);
  }
#pragma unroll
  for (int r = 0; r < 16; ++r)
    if (r < nr) U[((int64_t)(r0 + r) * heads + h) * width + c] = acc[r];
}

// In place: S[r, :] = softmax(S[r, :] * scale) over n columns.
__global__ void __launch_bounds__(256) softmax_rows_kernel(float* __restrict__ S, int64_t lds, int n,
                                                           float scale) {
  __shared__ float red[32];
  float* row = S + (int64_t)blockIdx.x * lds;
  float mx = -INFINITY;
  for (int t = threadIdx.x; t < n; t += blockDim.x) mx = fmaxf(mx, __fmul_rn(row[t], scale));
  mx = block_max(mx, red);
  float sum = 0.f;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float e = expf(__fsub_rn(__fmul_rn(row[t], scale), mx));
    row[t] = e;
    sum += e;
  }
  const float inv_sum = block_sum(sum, red);
  for (int t = threadIdx.x; t < n; t += blockDim.x) row[t] = __fdiv_rn(row[t], inv_sum);
}

// out[o, h*hd + d] = sum_c Wv[h*hd + d, c] * C[(o, h), c] + bv[h*hd + d]. One
// warp per output feature f: its Wv row is read once into registers and
// dotted with the C rows of all query rows o (head h = f / hd).
__global__ void __launch_bounds__(256) v_unfold_kernel(const float* __restrict__ C, const float* __restrict__ Wv,
                                                       const float* __restrict__ bv, int width, int heads, int hd,
                                                       int R0, float* __restrict__ out, int64_t ldo) {
  const int lane = threadIdx.x & 31;
  const int f = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (f >= width) return;
  const int h = f / hd;
  constexpr int MAXW = 64;  // elements per lane: width <= 2048
  float wr[MAXW];
#pragma unroll
  for (int i = 0; i < MAXW; ++i) {
    const int c = lane + 32 * i;
    wr[i] = c < width ? Wv[(int64_t)f * width + c] : 0.f;
  }
  for (int o = 0; o < R0; ++o) {
    const float* cr = C + ((int64_t)o * heads + h) * width;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < MAXW; ++i) {
      const int c = lane + 32 * i;
      if (c < width) acc = fmaf(wr[i], cr[c], acc);
    }
    for (int k = 16; k; k >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, k);
    if (lane == 0) out[(int64_t)o * ldo + f] = __fadd_rn(acc, bv[f]);
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

// out[m, n] = res[m, n] + act(sum_s P[s, b, m, n] + bias[n]) for batch element
// b = blockIdx.y, slabs summed in order.
__global__ void splitk_reduce_kernel(const float* __restrict__ P, int splits, int M, int N,
                                     const float* __restrict__ bias, int gelu, const float* res, int64_t ldr,
                                     float* out, int64_t ldo, SkinnyBatch bs) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * N) return;
  const int b = blockIdx.y, nb = gridDim.y;
  const int m = (int)(i / N), n = (int)(i % N);
  const int64_t mn = (int64_t)M * N;
  float v = P[(int64_t)b * mn + i];
  for (int z = 1; z < splits; ++z) v = __fadd_rn(v, P[((int64_t)z * nb + b) * mn + i]);
  if (bias) v = __fadd_rn(v, bias[b * bs.bias + n]);
  if (gelu) v = gelu_erf(v);
  out += b * bs.out;
  if (res) v = __fadd_rn(res[b * bs.out + (int64_t)m * ldr + n], v);
  out[(int64_t)m * ldo + n] = v;
}

// Split-K partial sums of the head's GEMMs live here (one buffer per device
// handle, sized at workspace planning).
struct SplitK {
  float* part = nullptr;
  size_t cap = 0;  // floats
  int sms = 148;
};
thread_local SplitK g_split;

// Skinny GEMM over `batch` independent problems (offsets in bs; `res`, when
// given, shares the output offsets), split along K when the column tiles
// alone would not fill the GPU.
int skinny_gemm(const float* X, int64_t ldx, const float* W, int64_t ldw, int M, int N, int K, const float* bias,
                bool gelu, const float* res, int64_t ldr, float* out, int64_t ldo, int batch, SkinnyBatch bs,
                cudaStream_t s) {
  const int64_t tiles = ceil_div(N, 8 * SK_COLS) * (int64_t)batch;
  int splits = 1, kc = K;
  if (tiles < 2 * g_split.sms && g_split.part) {
    int want = (int)std::min<int64_t>(32, ceil_div(2 * g_split.sms, tiles));
    want = (int)std::min<int64_t>(want, std::max<int64_t>(1, K / 256));
    want = (int)std::min<int64_t>(want, (int64_t)(g_split.cap / ((size_t)M * N * batch)));
    if (want > 1) {
      kc = (int)(ceil_div(ceil_div(K, want), 4) * 4);
      splits = (int)ceil_div(K, kc);
    }
  }
  const dim3 grid((unsigned)ceil_div(N, 8 * SK_COLS), (unsigned)splits, (unsigned)batch);
  if (splits == 1) {
    CLEF_CHECK(!res || batch == 1, CLEF_ERR_INVALID, "head: batched residual");
    skinny_gemm_kernel<<<grid, 256, 0, s>>>(X, ldx, W, ldw, M, N, K, kc, bs, bias, gelu ? 1 : 0, res, ldr, out,
                                            ldo);
    return launch_status("head skinny gemm");
  }
  skinny_gemm_kernel<<<grid, 256, 0, s>>>(X, ldx, W, ldw, M, N, K, kc, bs, nullptr, 0, nullptr, 0, g_split.part, N);
  int rc = launch_status("head skinny gemm");
  if (rc) return rc;
  splitk_reduce_kernel<<<dim3((unsigned)ceil_div((int64_t)M * N, 256), (unsigned)batch), 256, 0, s>>>(
      g_split.part, splits, M, N, bias, gelu ? 1 : 0, res, ldr, out, ldo, bs);
  return launch_status("head split-k reduce");
}

int gemm_f32(const float* X, int64_t ldx, const float* W, int64_t ldw, int M, int N, int K, const float* bias,
             bool gelu, const float* res, int64_t ldr, float* out, int64_t ldo, cudaStream_t s, bool w_kn = false) {
  if (M == 0 || N == 0) return CLEF_OK;
  if (M <= SK_M && !w_kn) return skinny_gemm(X, ldx, W, ldw, M, N, K, bias, gelu, res, ldr, out, ldo, 1,
                                              SkinnyBatch{0, 0, 0, 0}, s);
  dim3 grid((unsigned)ceil_div(N, SG_N), (unsigned)ceil_div(M, SG_M), 1);
  CLEF_CHECK(grid.y <= 65535u, CLEF_ERR_UNSUPPORTED, "head: too many rows");
  // 16-byte loads when every row start is 16-byte aligned and K (or N for a
  // [K, N] weight) is a multiple of 4.
  const bool vec = (((uintptr_t)X | (uintptr_t)W) & 15) == 0 && ldx % 4 == 0 && ldw % 4 == 0 &&
                   (w_kn ? (K % 4 == 0 && N % 4 == 0) : K % 4 == 0);
  // Too few output tiles to fill the GPU: split K into slabs of >= 64 that
  // sum in a second pass (deterministic order), up to 32 ways.
  const int64_t tiles = (int64_t)grid.x * grid.y;
  int splits = 1, kc = K;
  if (tiles < 2 * g_split.sms && g_split.part) {
    int want = (int)std::min<int64_t>(32, ceil_div(2 * g_split.sms, tiles));
    want = std::min<int64_t>(want, std::max<int64_t>(1, K / 64));
    want = (int)std::min<int64_t>(want, (int64_t)(g_split.cap / ((size_t)M * N)));
    if (want > 1) {
      kc = (int)(ceil_div(ceil_div(K, want), SG_K) * SG_K);
      splits = (int)ceil_div(K, kc);
    }
  }
  grid.z = (unsigned)splits;
  float* dst = splits > 1 ? g_split.part : out;
  const int64_t ldd = splits > 1 ? N : ldo;
  const float* eb = splits > 1 ? nullptr : bias;
  const float* er = splits > 1 ? nullptr : res;
  const int eg = splits > 1 ? 0 : (gelu ? 1 : 0);
  if (w_kn)
    sgemm_kernel<true><<<grid, 256, 0, s>>>(X, ldx, W, ldw, M, N, K, kc, vec, eb, eg, er, ldr, dst, ldd);
  else
    sgemm_kernel<false><<<grid, 256, 0, s>>>(X, ldx, W, ldw, M, N, K, kc, vec, eb, eg, er, ldr, dst, ldd);
  int rc = launch_status("head gemm");
  if (rc || splits == 1) return rc;
  const int64_t n = (int64_t)M * N;
  splitk_reduce_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(g_split.part, splits, M, N, bias, gelu ? 1 : 0, res,
                                                                  ldr, out, ldo, SkinnyBatch{0, 0, 0, 0});
  return launch_status("head split-k reduce");
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

// Reassociated cross-attention (see qk_fold_kernel): q [R0, width] already
// projected (Wq, bq); memory [T, width]; U, C [R0 * heads, width] and S
// [R0 * heads, T] are workspace; out [R0, width] before the output projection.
int cross_attention(const float* q, int R0, const float* mem, int T, const float* Wk, const float* Wv,
                    const float* bv, int width, int heads, float* U, float* S, float* C, float* out, cudaStream_t s) {
  if (R0 == 0) return CLEF_OK;
  const int hd = width / heads, R = R0 * heads;
  qk_fold_kernel<<<dim3((unsigned)ceil_div(width, 256), (unsigned)heads, (unsigned)ceil_div(R0, 16)), 256, 0, s>>>(
      q, width, Wk, width, heads, hd, R0, U);
  int rc = launch_status("head qk_fold");
  if (!rc) rc = gemm_f32(U, width, mem, width, R, T, width, nullptr, false, nullptr, 0, S, T, s);
  if (rc) return rc;
  softmax_rows_kernel<<<R, 256, 0, s>>>(S, T, T, (float)(1.0 / std::sqrt((double)hd)));
  rc = launch_status("head softmax");
  if (!rc) rc = gemm_f32(S, T, mem, width, R, width, T, nullptr, false, nullptr, 0, C, width, s, true);
  if (rc) return rc;
  if (R0 <= SK_M) {
    // Per head h: out[:, h*hd .. h*hd+hd) = C[(o, h), :] Wv[h*hd .. h*hd+hd, :]^T + bv.
    return skinny_gemm(C, (int64_t)heads * width, Wv, width, R0, hd, width, bv, false, nullptr, 0, out, width, heads,
                       SkinnyBatch{width, (int64_t)hd * width, hd, hd}, s);
  }
  v_unfold_kernel<<<(unsigned)ceil_div(width, 8), 256, 0, s>>>(C, Wv, bv, width, heads, hd, R0, out, width);
  return launch_status("head v_unfold");
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
  float *normalized, *x3, *memory, *nm, *U, *S, *C, *qs, *ctx, *lex, *routed, *tq, *q, *att, *ffh, *base, *oq, *summ,
      *summn, *fields, *gproj, *qkv, *anchor, *opts, *feats, *r1, *resid, *prior, *cosine, *logits, *part;
};

constexpr int64_t kSplitCap = 4 << 20;  // floats of split-K partial sums (16 MB)
constexpr int64_t kTensorRows = 64;     // records at least this long take the tensor-core memory projection

size_t plan_ws(const clef_head_config& c, int64_t T, int nq, int no, float* base, HeadWs* w) {
  size_t off = 0;
  const int64_t h = c.hidden_size, wd = c.width, ff = c.feedforward;
  const int64_t rows = std::max(nq, no);
  const int64_t R = rows * c.heads;
  auto take = [&](float** p, int64_t n) {
    if (w) *p = base + off;
    off += (size_t)((n + 63) / 64 * 64);
  };
  HeadWs d;
  HeadWs* t = w ? w : &d;
  take(&t->normalized, T * h);
  take(&t->x3, (T * 3 * h + 1) / 2);  // BF16 three-term operand of the memory projection
  take(&t->memory, T * wd);
  take(&t->nm, T * wd);
  take(&t->U, R * wd);
  take(&t->S, R * T);
  take(&t->C, R * wd);
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
  take(&t->part, kSplitCap);
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
  CLEF_CHECK(c.width % c.heads == 0 && 256 % (c.width / c.heads) == 0 && c.width <= 2048, CLEF_ERR_UNSUPPORTED,
             "head_create: width at most 2048 and head width (width / heads) dividing 256");
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
  DeviceGuardH g(hd->device);
  CLEF_CUDA(cudaMalloc(&hd->blob, sizeof(float) * (size_t)std::max<int64_t>(total, 64)));
  std::vector<float> staging((size_t)total, 0.f);
  for (const auto& kv : hd->host)
    std::copy(kv.second.begin(), kv.second.end(), staging.begin() + hd->off[kv.first]);
  CLEF_CUDA(cudaMemcpy(hd->blob, staging.data(), sizeof(float) * (size_t)total, cudaMemcpyHostToDevice));
  // Scalars as Head::load derives them (head.rs:128-130).
  const double lim = std::log(100.0);
  hd->prior_scale = (float)std::exp(std::min((double)hd->host["prior_logit_scale"][0], lim));
  hd->joint_scale = (float)std::exp(std::min((double)hd->host["joint_logit_scale"][0], lim));
  hd->gate = (float)(1.0 / (1.0 + std::exp(-(double)hd->host["residual_gate"][0])));
  hd->host.clear();
  // The memory projection (the head's one large product, T x hidden x width)
  // runs on the tcgen05 GEMM when its shapes fit the kernel's tiling.
  if (c.hidden_size % 64 == 0 && c.width % 16 == 0) {
    const int64_t h = c.hidden_size;
    CLEF_CUDA(cudaMalloc(&hd->mem_w3, sizeof(uint16_t) * (size_t)w * 3 * h));
    const int rc = split3(W(hd, "memory_projection.weight"), h, w, (int)h, true, hd->mem_w3, hd->stream);
    if (rc) return rc;
    CLEF_CUDA(cudaStreamSynchronize(hd->stream));
  }
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
  g_split.part = b.part;
  g_split.cap = (size_t)kSplitCap;
  g_split.sms = num_sms(hd->device);
  // Memory side (head.rs:154-157).
  RCH(layer_norm(hidden, h, Ti, (int)h, W(hd, "hidden_norm.weight"), W(hd, "hidden_norm.bias"), b.normalized, h, s));
  if (hd->mem_w3 && T >= kTensorRows) {
    // F32-accurate three-term product on the tensor cores (hi.hi + lo.hi + hi.lo).
    RCH(split3(b.normalized, h, T, (int)h, false, reinterpret_cast<uint16_t*>(b.x3), s));
    RCH(launch_gemm(reinterpret_cast<const uint16_t*>(b.x3), hd->mem_w3, nullptr, T, (int)wd, (int)(3 * h), kEpiF32,
                    b.memory, wd, s));
  } else {
    RCH(gemm_f32(b.normalized, h, W(hd, "memory_projection.weight"), h, Ti, (int)wd, (int)h, nullptr, false, nullptr,
                 0, b.memory, wd, s));
  }
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
    RCH(cross_attention(b.q, no, b.nm, Ti, iw + wd * wd, iw + 2 * wd * wd, ib + 2 * wd, (int)wd, c.heads, b.U, b.S,
                        b.C, b.att, s));
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
  // Decoder layers (head.rs:230-241); the cross-attention reads the
  // un-normalised memory.
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
    const float* mw = W(hd, p + ".multihead_attn.in_proj_weight");
    RCH(cross_attention(b.q, nq, b.memory, Ti, mw + wd * wd, mw + 2 * wd * wd,
                        W(hd, p + ".multihead_attn.in_proj_bias") + 2 * wd, (int)wd, c.heads, b.U, b.S, b.C, b.att,
                        s));
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
    if (hd->mem_w3) cudaFree(hd->mem_w3);
    if (hd->ws) cudaFree(hd->ws);
    if (hd->meta_d) cudaFree(hd->meta_d);
    if (hd->stream) cudaStreamDestroy(hd->stream);
  }
  delete hd;
  return CLEF_OK;
}

}  // extern "C"
