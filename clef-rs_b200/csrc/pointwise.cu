// pointwise.cu — HBM-bound kernels of the prefill: RMSNorm, causal conv,
// the DeltaNet prologue (conv + SiLU + L2 + gates) and epilogue
// (RMSNorm_128 * silu(z)), the attention prologue (q/k norm + partial RoPE),
// the embedding gather and the schema head.
//
// Every kernel reads and writes with 16-byte vectors where the layout allows
// and reduces with warp shuffles; one warp owns one normalisation row, so no
// shared-memory reduction or block barrier sits on the hot path.
#include <algorithm>
#include <cmath>

#include <type_traits>

#include "kernels.cuh"

namespace clef {

namespace {

__device__ __forceinline__ int64_t seq_of(const int64_t* cu, int nseq, int64_t t) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {  // largest s with cu[s] <= t
    int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// ---- RMSNorm (ops::rms_inner, ops.rs:24-32; clef_rms, pointwise.metal:7-43) --
// One warp per row: sum of squares, inverse = 1 / sqrt(sum / width + eps),
// out = (x * inverse) * w. With NV > 0 (width == 128 * NV) the row is read
// once into registers, all NV 16-byte loads of a lane in flight together.
// OUT_BF16: 0 = F32, 1 = BF16, 2 = split BF16 pair (hi in columns [0, width),
// lo in [width, 2 width) of a row of 2 width).
template <int OUT_BF16, int NV>
__global__ void rms_kernel(const float* __restrict__ x, const float* __restrict__ w, int64_t rows,
                           int width, float eps, void* __restrict__ out) {
  if constexpr (NV > 0) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float* xr = x + row * width;
    float4 a[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) a[j] = *reinterpret_cast<const float4*>(xr + lane * 4 + 128 * j);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) s += a[j].x * a[j].x + a[j].y * a[j].y + a[j].z * a[j].z + a[j].w * a[j].w;
    s = warp_sum(s);
    const float inv = 1.f / sqrtf(s / (float)width + eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane * 4 + 128 * j;
      const float4 b = *reinterpret_cast<const float4*>(w + i);
      const float r0 = __fmul_rn(__fmul_rn(a[j].x, inv), b.x), r1 = __fmul_rn(__fmul_rn(a[j].y, inv), b.y);
      const float r2 = __fmul_rn(__fmul_rn(a[j].z, inv), b.z), r3 = __fmul_rn(__fmul_rn(a[j].w, inv), b.w);
      if (OUT_BF16 == 2) {
        const uint2 hi = make_uint2(pack_bf16x2(r0, r1), pack_bf16x2(r2, r3));
        uint16_t* o = reinterpret_cast<uint16_t*>(out) + row * 2 * width + i;
        *reinterpret_cast<uint2*>(o) = hi;
        *reinterpret_cast<uint2*>(o + width) = make_uint2(split_lo_bf16x2(r0, r1, hi.x), split_lo_bf16x2(r2, r3, hi.y));
      } else if (OUT_BF16) {
        *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + row * width + i) =
            make_uint2(pack_bf16x2(r0, r1), pack_bf16x2(r2, r3));
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + row * width + i) = make_float4(r0, r1, r2, r3);
      }
    }
    return;
  }
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * width;
  float s = 0.f;
  const bool vec = (width & 3) == 0;
  if (vec) {
    for (int i = lane * 4; i < width; i += 128) {
      float4 a = *reinterpret_cast<const float4*>(xr + i);
      s += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    }
  } else {
    for (int i = lane; i < width; i += 32) s += xr[i] * xr[i];
  }
  s = warp_sum(s);
  const float inv = 1.f / sqrtf(s / (float)width + eps);
  if (vec) {
    for (int i = lane * 4; i < width; i += 128) {
      float4 a = *reinterpret_cast<const float4*>(xr + i);
      float4 b = *reinterpret_cast<const float4*>(w + i);
      float r0 = __fmul_rn(__fmul_rn(a.x, inv), b.x), r1 = __fmul_rn(__fmul_rn(a.y, inv), b.y);
      float r2 = __fmul_rn(__fmul_rn(a.z, inv), b.z), r3 = __fmul_rn(__fmul_rn(a.w, inv), b.w);
      if (OUT_BF16 == 2) {
        const uint2 hi = make_uint2(pack_bf16x2(r0, r1), pack_bf16x2(r2, r3));
        uint16_t* o = reinterpret_cast<uint16_t*>(out) + row * 2 * width + i;
        *reinterpret_cast<uint2*>(o) = hi;
        *reinterpret_cast<uint2*>(o + width) = make_uint2(split_lo_bf16x2(r0, r1, hi.x), split_lo_bf16x2(r2, r3, hi.y));
      } else if (OUT_BF16) {
        uint2 p = make_uint2(pack_bf16x2(r0, r1), pack_bf16x2(r2, r3));
        *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + row * width + i) = p;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + row * width + i) =
            make_float4(r0, r1, r2, r3);
      }
    }
  } else {
    for (int i = lane; i < width; i += 32) {
      float r = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
      if (OUT_BF16 == 2) {
        const uint16_t hi = f2bf(r);
        reinterpret_cast<uint16_t*>(out)[row * 2 * width + i] = hi;
        reinterpret_cast<uint16_t*>(out)[row * 2 * width + width + i] = f2bf(r - bf2f(hi));
      } else if (OUT_BF16) {
        reinterpret_cast<uint16_t*>(out)[row * width + i] = f2bf(r);
      } else {
        reinterpret_cast<float*>(out)[row * width + i] = r;
      }
    }
  }
}

// ---- causal conv (causal_convolution, qwen.rs:765-796) -----------------------
// value = ((((0 + x[t-3] w0) + x[t-2] w1) + x[t-1] w2) + x[t] w3), rows before
// the first input come from `hist` (right-aligned) or are zero.
__device__ __forceinline__ float conv_tap_row(const float* x, int64_t ldx, const float* hist,
                                              int hist_rows, int width, int64_t seq_start,
                                              int64_t pos, int delay, int c) {
  const int64_t r = pos - delay;
  if (r >= 0) return x[(seq_start + r) * ldx + c];
  const int64_t hr = hist_rows + r;
  if (hist && hr >= 0) return hist[hr * width + c];
  return 0.f;
}

__global__ void conv4_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ hist,
                             int hist_rows, const float* __restrict__ w, int64_t T, int width,
                             float* __restrict__ out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * width) return;
  const int64_t t = idx / width;
  const int c = (int)(idx % width);
  float acc = 0.f;
#pragma unroll
  for (int tap = 0; tap < 4; ++tap) {
    const int delay = 3 - tap;
    const int64_t r = t - delay;
    if (r < 0 && !(hist && hist_rows + r >= 0)) continue;
    const float xv = conv_tap_row(x, ldx, hist, hist_rows, width, 0, t, delay, c);
    acc = __fadd_rn(acc, __fmul_rn(xv, w[c * 4 + tap]));
  }
  out[t * width + c] = acc;
}

// ---- DeltaNet prologue -------------------------------------------------------
// CTA = 256 threads x 4 channels (1024 channels = 8 whole 128-wide heads) over a
// run of PRO_RUN consecutive tokens. Every thread issues the asynchronous
// copies of all PRO_RUN + 3 projection rows of its channels (3 rows of conv
// history) into shared memory up front, so the whole run is in flight at once
// without holding it in registers, then walks the tokens in one rolled loop.
// Four CTAs per SM (61 registers). A warp covers exactly one q/k head and
// reduces its L2 norm with shuffles (clef_delta_prepare, pointwise.metal:69-114;
// l2 and scaling, qwen.rs:837-845). The CTAs of channel block 0 also compute
// the gates (qwen.rs:619-627).
constexpr int PRO_RUN = 12;
constexpr int PRO_ROWS = PRO_RUN + 3;

// Staged element of one thread's 4 channels: F32 (16 bytes, the C-ABI
// operator) or BF16 (8 bytes, the engine's projection output, which the
// reference rounds to the model dtype before widening, qwen.rs:603).
template <typename In>
struct ProIn;
template <>
struct ProIn<float> {
  using V = float4;
  __device__ static float4 f4(const float4& v) { return v; }
  __device__ static float f(float x) { return x; }
};
template <>
struct ProIn<uint16_t> {
  using V = uint2;
  __device__ static float4 f4(const uint2& v) {
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                       __uint_as_float(v.y & 0xffff0000u));
  }
  __device__ static float f(uint16_t x) { return __uint_as_float((uint32_t)x << 16); }
};
template <typename In>
constexpr int pro_smem() {
  return PRO_ROWS * 256 * (int)sizeof(typename ProIn<In>::V);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_row(float4* dst, const float* src) { cp_async16(dst, src); }
__device__ __forceinline__ void cp_async_row(uint2* dst, const uint16_t* src) { cp_async8(dst, src); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// silu(x) = x / (1 + e^-x) with the MUFU exponential and divide (a few ulp of
// the correctly rounded quotient; e^-x overflowing gives -0 for very negative x).
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// Conv output of one token from its four input rows (oldest first), then
// SiLU, L2 normalisation of q/k heads and the store.
__device__ __forceinline__ void pro_finish(const float4 (&x)[4], const float (&tw)[4][4], int64_t t, int c, int key,
                                           int Hv, float qscale, float* __restrict__ q, float* __restrict__ k,
                                           float* __restrict__ v) {
  // Packed two-lane F32 multiplies and adds, each lane rounded on its own:
  // the same multiply-then-add per tap as the scalar form, half the issues.
  float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
#pragma unroll
  for (int tap = 0; tap < 4; ++tap) {
    a01 = __fadd2_rn(a01, __fmul2_rn(make_float2(x[tap].x, x[tap].y), make_float2(tw[tap][0], tw[tap][1])));
    a23 = __fadd2_rn(a23, __fmul2_rn(make_float2(x[tap].z, x[tap].w), make_float2(tw[tap][2], tw[tap][3])));
  }
  const float4 m = make_float4(silu_fast(a01.x), silu_fast(a01.y), silu_fast(a23.x), silu_fast(a23.y));
  if (c < 2 * key) {
    // The whole warp sits in one head (channel blocks of 1024, heads of 128).
    float ss = m.x * m.x + m.y * m.y + m.z * m.z + m.w * m.w;
    ss = warp_sum(ss);
    float inv = rsqrtf(ss + 1e-6f);  // the approximate reciprocal square root (a few ulp)
    if (c < key) inv = __fmul_rn(inv, qscale);
    const float2 i2 = make_float2(inv, inv);
    const float2 n01 = __fmul2_rn(make_float2(m.x, m.y), i2), n23 = __fmul2_rn(make_float2(m.z, m.w), i2);
    float* dst = c < key ? q + t * key + c : k + t * key + (c - key);
    *reinterpret_cast<float4*>(dst) = make_float4(n01.x, n01.y, n23.x, n23.y);
  } else {
    *reinterpret_cast<float4*>(v + t * (int64_t)(Hv * 128) + (c - 2 * key)) = m;
  }
}

// Input row of token t (this thread's 4 channels) for a sequence starting at
// `start`: the staged projection row, a conv-history row, or zeros.
template <typename V>
__device__ __forceinline__ float4 pro_row(const V* __restrict__ rows, int i, const float* __restrict__ hist,
                                          int hist_rows, int width, int64_t r, int64_t start, int c) {
  if (r >= start) return ProIn<std::conditional_t<sizeof(V) == 16, float, uint16_t>>::f4(rows[i * 256]);
  const int64_t hr = hist_rows + (r - start);
  if (!hist || hr < 0) return make_float4(0.f, 0.f, 0.f, 0.f);  // rows before the sequence are zero
  return *reinterpret_cast<const float4*>(hist + hr * width + c);
}

template <typename In>
__global__ void __launch_bounds__(256, 4) delta_prologue_kernel(
    const In* __restrict__ proj, int64_t ldp, int a_col, int b_col,
    const float* __restrict__ hist, int hist_rows, const float* __restrict__ conv_w,
    const float* __restrict__ dt_bias, const float* __restrict__ a_log,
    const int64_t* __restrict__ cu, int nseq, int64_t T, int Hk, int Hv, float qscale,
    float* __restrict__ q, float* __restrict__ k, float* __restrict__ v, float* __restrict__ g,
    float* __restrict__ beta) {
  using V = typename ProIn<In>::V;
  extern __shared__ __align__(16) uint8_t pro_raw[];
  V* pro_sm = reinterpret_cast<V*>(pro_raw);  // [PRO_ROWS][256]
  const int key = Hk * 128;
  const int width = 2 * key + Hv * 128;
  const int c = blockIdx.x * 1024 + threadIdx.x * 4;
  const int64_t t_begin = (int64_t)blockIdx.y * PRO_RUN;
  const int64_t t_end = min(T, t_begin + PRO_RUN);
  V* rows = pro_sm + threadIdx.x;
#pragma unroll
  for (int i = 0; i < PRO_ROWS; ++i) {
    const int64_t r = t_begin - 3 + i;
    if (r >= 0 && r < t_end) cp_async_row(rows + i * 256, proj + r * ldp + c);
  }
  cp_async_commit();
  // Sequence of the first token.
  int s = cu ? (int)seq_of(cu, nseq, t_begin) : 0;
  int64_t start = cu ? cu[s] : 0;
  int64_t next_start = cu ? cu[s + 1] : T;
  // Taps of the four channels: conv_w[c][0..3] for c .. c+3.
  const float4 w0 = *reinterpret_cast<const float4*>(conv_w + (c + 0) * 4);
  const float4 w1 = *reinterpret_cast<const float4*>(conv_w + (c + 1) * 4);
  const float4 w2 = *reinterpret_cast<const float4*>(conv_w + (c + 2) * 4);
  const float4 w3 = *reinterpret_cast<const float4*>(conv_w + (c + 3) * 4);
  const float tw[4][4] = {{w0.x, w1.x, w2.x, w3.x},
                          {w0.y, w1.y, w2.y, w3.y},
                          {w0.z, w1.z, w2.z, w3.z},
                          {w0.w, w1.w, w2.w, w3.w}};
  cp_async_wait<0>();
  // Sliding window of the four input rows (converted once each): staged row
  // i + j is token t_begin - 3 + i + j.
  float4 win[4];
#pragma unroll
  for (int j = 0; j < 3; ++j) win[j] = pro_row<V>(rows, j, hist, hist_rows, width, t_begin - 3 + j, start, c);
#pragma unroll 1
  for (int i = 0; i < PRO_RUN; ++i) {
    const int64_t t = t_begin + i;
    if (t >= t_end) break;
    if (t == next_start) {  // a new sequence starts: its window holds history or zeros
      ++s;
      start = t;
      next_start = cu[s + 1];
#pragma unroll
      for (int j = 0; j < 3; ++j) win[j] = pro_row<V>(rows, i + j, hist, hist_rows, width, t - 3 + j, start, c);
    }
    win[3] = pro_row<V>(rows, i + 3, hist, hist_rows, width, t, start, c);
    pro_finish(win, tw, t, c, key, Hv, qscale, q, k, v);
    win[0] = win[1];
    win[1] = win[2];
    win[2] = win[3];
  }
  if (blockIdx.x == 0) {
    for (int idx = threadIdx.x; idx < (t_end - t_begin) * Hv; idx += blockDim.x) {
      const int64_t t = t_begin + idx / Hv;
      const int h = idx % Hv;
      const float a = __fadd_rn(ProIn<In>::f(proj[t * ldp + a_col + h]), dt_bias[h]);
      const float sp = __fadd_rn(fmaxf(a, 0.f), logf(__fadd_rn(expf(-fabsf(a)), 1.f)));
      g[t * Hv + h] = __fmul_rn(sp, -expf(a_log[h]));
      beta[t * Hv + h] = sigmoid_f(ProIn<In>::f(proj[t * ldp + b_col + h]));
    }
  }
}

// ---- DeltaNet epilogue (qwen.rs:671-676) -------------------------------------
// y = RMSNorm_128(o) * w (no offset) * silu(z) in F32; the only rounding is
// the store of y, the out-projection's operand (BF16, or a split BF16 pair with
// hi in columns [0, Hv*128) and lo in [Hv*128, 2*Hv*128) when SPLIT). z is the
// in-projection output: BF16 in the engine's default precision, F32 in its
// split precision.
template <typename ZIn, bool SPLIT>
__global__ void __launch_bounds__(256) delta_epilogue_kernel(const float* __restrict__ o,
                                                             const ZIn* __restrict__ z, int64_t ldz,
                                                             const float* __restrict__ w, float eps,
                                                             int64_t T, int Hv, uint16_t* __restrict__ y) {
  // One warp per token; its Hv rows of 128 go four at a time with all eight
  // loads of a batch (o rows and z rows) issued before any is used.
  using ZV = std::conditional_t<std::is_same<ZIn, float>::value, float4, uint2>;
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const float4 wv = *reinterpret_cast<const float4*>(w + lane * 4);
  const int64_t V = (int64_t)Hv * 128;
  constexpr int HB = 4;  // heads per batch: 8 loads per lane in flight
  for (int h0 = 0; h0 < Hv; h0 += HB) {
    float4 a[HB];
    ZV zr[HB];
#pragma unroll
    for (int u = 0; u < HB; ++u) {
      if (h0 + u < Hv) {
        a[u] = *reinterpret_cast<const float4*>(o + (t * Hv + h0 + u) * 128 + lane * 4);
        zr[u] = *reinterpret_cast<const ZV*>(z + t * ldz + (h0 + u) * 128 + lane * 4);
      }
    }
    // Row sums of the HB = 4 heads by reduce-scatter: after the xor-16 and
    // xor-8 exchanges lane l holds the partial of head 2 ((l >> 4) & 1) +
    // ((l >> 3) & 1) over four lanes, the xor-4/2/1 tree completes it (the
    // same pairings as a full butterfly per head, so the same sums), and lane
    // 8u hands head u's normaliser to the warp.
    float ss[HB];
#pragma unroll
    for (int u = 0; u < HB; ++u)
      ss[u] = h0 + u < Hv ? a[u].x * a[u].x + a[u].y * a[u].y + a[u].z * a[u].z + a[u].w * a[u].w : 0.f;
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1;
    const float k0 = (b4 ? ss[2] : ss[0]) + __shfl_xor_sync(0xffffffffu, b4 ? ss[0] : ss[2], 16);
    const float k1 = (b4 ? ss[3] : ss[1]) + __shfl_xor_sync(0xffffffffu, b4 ? ss[1] : ss[3], 16);
    float part = (b3 ? k1 : k0) + __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const float inv_mine = 1.f / sqrtf(part / 128.f + eps);
#pragma unroll
    for (int u = 0; u < HB; ++u) {
      const float inv = __shfl_sync(0xffffffffu, inv_mine, 8 * u);
      if (h0 + u >= Hv) break;
      const float4 zv = ProIn<ZIn>::f4(zr[u]);
      const float4 b = a[u];
      const float y0 = __fmul_rn(__fmul_rn(__fmul_rn(b.x, inv), wv.x), silu_f(zv.x));
      const float y1 = __fmul_rn(__fmul_rn(__fmul_rn(b.y, inv), wv.y), silu_f(zv.y));
      const float y2 = __fmul_rn(__fmul_rn(__fmul_rn(b.z, inv), wv.z), silu_f(zv.z));
      const float y3 = __fmul_rn(__fmul_rn(__fmul_rn(b.w, inv), wv.w), silu_f(zv.w));
      const uint2 hi = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
      uint16_t* dst = y + t * (SPLIT ? 2 * V : V) + (h0 + u) * 128 + lane * 4;
      *reinterpret_cast<uint2*>(dst) = hi;
      if (SPLIT)
        *reinterpret_cast<uint2*>(dst + V) = make_uint2(split_lo_bf16x2(y0, y1, hi.x), split_lo_bf16x2(y2, y3, hi.y));
    }
  }
}

// ---- attention prologue (qwen.rs:463-490; rotary, ops.rs:144-188) ------------
// One warp per token: the token's position and its rotary cos/sin table
// (half = rot/2 frequencies, in shared memory) are computed once and used for
// all H + Hkv rows of 256 features, which go four at a time (8 features per
// lane, loads issued up front). Rows [0, H) are query heads (projection
// columns h*2d .. h*2d+d), rows [H, H+Hkv) key heads (columns 2*H*d + j*d).
// Each rotation pair (f, f + half), f < half, sits in one lane: lane l <
// half/4 holds features [4l, 4l + 4) and [half + 4l, half + 4l + 4), lane
// l >= half/4 the 8 features from rot + 8 (l - half/4); so a lane's norm
// weights and cos/sin are read once per token and no lane needs another's
// features. Norm and rotation run in F32; the rotated features are rounded
// once, to the BF16 operands of the tensor-core attention. The projection rows
// are BF16 (the engine's default precision) or F32 (its split precision).
constexpr int AP_WARPS = 8;

// Four consecutive projection features as F32.
__device__ __forceinline__ void load4(const uint16_t* src, float* x) {
  const uint2 r = *reinterpret_cast<const uint2*>(src);
  x[0] = __uint_as_float(r.x << 16), x[1] = __uint_as_float(r.x & 0xffff0000u);
  x[2] = __uint_as_float(r.y << 16), x[3] = __uint_as_float(r.y & 0xffff0000u);
}
__device__ __forceinline__ void load4(const float* src, float* x) {
  const float4 a = *reinterpret_cast<const float4*>(src);
  x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w;
}

template <typename In>
__global__ void __launch_bounds__(AP_WARPS * 32) attention_prologue_kernel(
    const In* __restrict__ proj, int64_t ldp, const float* __restrict__ qw,
    const float* __restrict__ kw, float eps, const int64_t* __restrict__ cu, int nseq, int64_t pos_offset,
    int H, int Hkv, int rot, const float* __restrict__ inv_freq, uint16_t* __restrict__ q_out,
    uint16_t* __restrict__ k_out, int64_t T) {
  __shared__ __align__(16) float cs_tab[AP_WARPS][2][128];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t = (int64_t)blockIdx.x * AP_WARPS + warp;
  if (t >= T) return;
  const int d = 256;
  const int half = rot / 2;
  const int64_t start = cu ? cu[seq_of(cu, nseq, t)] : 0;
  const float pos = (float)(pos_offset + (t - start));
  for (int f = lane; f < half; f += 32) {
    const float ang = __fmul_rn(pos, inv_freq[f]);
    cs_tab[warp][0][f] = cosf(ang);
    cs_tab[warp][1][f] = sinf(ang);
  }
  __syncwarp();
  const int per = H + Hkv;
  const bool rl = lane < half / 4;  // a rotation lane
  const int off0 = rl ? 4 * lane : rot + 8 * (lane - half / 4);
  const int off1 = rl ? half + 4 * lane : off0 + 4;
  // This lane's norm weights (q and k) and, on a rotation lane, cos/sin of
  // frequencies 4l .. 4l + 3.
  float wq[8], wk[8], cs[4], sn[4];
  load4(qw + off0, wq), load4(qw + off1, wq + 4);
  load4(kw + off0, wk), load4(kw + off1, wk + 4);
  if (rl) {
    load4(&cs_tab[warp][0][4 * lane], cs);
    load4(&cs_tab[warp][1][4 * lane], sn);
  }
  for (int h0 = 0; h0 < per; h0 += 4) {
    float xs[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int hh = h0 + u;
      if (hh < per) {
        const In* src = hh < H ? proj + t * ldp + (int64_t)hh * 2 * d
                               : proj + t * ldp + (int64_t)2 * H * d + (int64_t)(hh - H) * d;
        load4(src + off0, xs[u]);
        load4(src + off1, xs[u] + 4);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int hh = h0 + u;
      if (hh >= per) break;
      const bool isq = hh < H;
      float x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = xs[u][i];
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
      ss = warp_sum(ss);
      const float inv = 1.f / sqrtf(ss / (float)d + eps);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = __fmul_rn(__fmul_rn(x[i], inv), isq ? wq[i] : wk[i]);
      if (rl) {
        // Partial NeoX rotation: x cos + rotate_half(x) sin on the pairs
        // (x[j], x[4 + j]) = features (4l + j, half + 4l + j).
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = x[j], hi = x[4 + j];
          x[j] = __fadd_rn(__fmul_rn(lo, cs[j]), __fmul_rn(-hi, sn[j]));
          x[4 + j] = __fadd_rn(__fmul_rn(hi, cs[j]), __fmul_rn(lo, sn[j]));
        }
      }
      uint16_t* dst = isq ? q_out + (t * H + hh) * (int64_t)d : k_out + (t * Hkv + (hh - H)) * (int64_t)d;
      *reinterpret_cast<uint2*>(dst + off0) = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
      *reinterpret_cast<uint2*>(dst + off1) = make_uint2(pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7]));
    }
  }
}

// ---- embedding gather (Backbone::forward, qwen.rs:316-317; F32 cast :373) ----
__global__ void embed_kernel(const uint16_t* __restrict__ table, const int32_t* __restrict__ ids,
                             int hidden, float* __restrict__ h) {
  const int64_t t = blockIdx.x;
  const uint16_t* src = table + (int64_t)ids[t] * hidden;
  for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    uint4 raw = *reinterpret_cast<const uint4*>(src + i);
    const uint32_t r32[4] = {raw.x, raw.y, raw.z, raw.w};
    float4 a = make_float4(__uint_as_float(r32[0] << 16), __uint_as_float(r32[0] & 0xffff0000u),
                           __uint_as_float(r32[1] << 16), __uint_as_float(r32[1] & 0xffff0000u));
    float4 b = make_float4(__uint_as_float(r32[2] << 16), __uint_as_float(r32[2] & 0xffff0000u),
                           __uint_as_float(r32[3] << 16), __uint_as_float(r32[3] & 0xffff0000u));
    *reinterpret_cast<float4*>(h + t * hidden + i) = a;
    *reinterpret_cast<float4*>(h + t * hidden + i + 4) = b;
  }
}

// ---- final norm + linear schema head at each sequence's last token -----------
__global__ void head_kernel(const float* __restrict__ h, const float* __restrict__ nw, float eps,
                            const int64_t* __restrict__ cu, int hidden,
                            const float* __restrict__ hw, int n_out, float* __restrict__ logits) {
  extern __shared__ float hn[];  // [hidden]
  __shared__ float red[32];
  __shared__ float inv_s;
  const int s = blockIdx.x;
  const int64_t row = cu[s + 1] - 1;
  const float* x = h + row * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) ss += x[i] * x[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) inv_s = 1.f / sqrtf(v / (float)hidden + eps);
  }
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) hn[i] = __fmul_rn(__fmul_rn(x[i], inv), nw[i]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int o = warp; o < n_out; o += blockDim.x >> 5) {
    float acc = 0.f;
    for (int i = lane; i < hidden; i += 32) acc += hw[(int64_t)o * hidden + i] * hn[i];
    acc = warp_sum(acc);
    if (lane == 0) logits[(int64_t)s * n_out + o] = acc;
  }
}

__global__ void copy_rows_kernel(const uint8_t* __restrict__ src, int64_t ld_bytes,
                                 int64_t row_bytes, uint8_t* __restrict__ dst, int64_t ldd_bytes) {
  const int64_t r = blockIdx.x;
  for (int64_t i = threadIdx.x * 4; i < row_bytes; i += blockDim.x * 4)
    *reinterpret_cast<uint32_t*>(dst + r * ldd_bytes + i) =
        *reinterpret_cast<const uint32_t*>(src + r * ld_bytes + i);
}

// dst[r, i] = float(src[r, i]) for BF16 rows (conv history of a capture).
__global__ void rows_bf16_to_f32_kernel(const uint16_t* __restrict__ src, int64_t ld, int64_t ncols,
                                        float* __restrict__ dst, int64_t ldd) {
  const int64_t r = blockIdx.x;
  for (int64_t i = threadIdx.x; i < ncols; i += blockDim.x)
    dst[r * ldd + i] = __uint_as_float((uint32_t)src[r * ld + i] << 16);
}

template <typename T>
__global__ void compact_copy_kernel(const T* __restrict__ src, int64_t n, int64_t d1, int64_t d2,
                                    int64_t d3, int64_t s0, int64_t s1, int64_t s2, int64_t s3,
                                    T* __restrict__ dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int64_t r = i;
  const int64_t i3 = r % d3;
  r /= d3;
  const int64_t i2 = r % d2;
  r /= d2;
  const int64_t i1 = r % d1;
  const int64_t i0 = r / d1;
  dst[i] = src[i0 * s0 + i1 * s1 + i2 * s2 + i3 * s3];
}

}  // namespace

int launch_rmsnorm(const float* x, const float* w, int64_t rows, int width, float eps, int out_dtype,
                   void* out, cudaStream_t s) {
  if (rows == 0) return CLEF_OK;
  const int warps = 8;
  const dim3 grid((unsigned)ceil_div(rows, warps));
  // Register-resident rows for the backbone widths (hidden 2560 and 4096).
  const bool al = (((uintptr_t)x | (uintptr_t)w | (uintptr_t)out) & 15) == 0;
#define CLEF_RMS_LAUNCH(NV)                                                                  \
  do {                                                                                       \
    if (out_dtype == kOutBF16Split) rms_kernel<2, NV><<<grid, warps * 32, 0, s>>>(x, w, rows, width, eps, out); \
    else if (out_dtype == CLEF_BF16) rms_kernel<1, NV><<<grid, warps * 32, 0, s>>>(x, w, rows, width, eps, out); \
    else rms_kernel<0, NV><<<grid, warps * 32, 0, s>>>(x, w, rows, width, eps, out);       \
  } while (0)
  if (al && width == 2560) CLEF_RMS_LAUNCH(20);
  else if (al && width == 4096) CLEF_RMS_LAUNCH(32);
  else CLEF_RMS_LAUNCH(0);
#undef CLEF_RMS_LAUNCH
  return launch_status("rmsnorm");
}

int launch_conv4(const float* x, int64_t ldx, const float* hist, int hist_rows, const float* w,
                 int64_t T, int width, float* out, cudaStream_t s) {
  if (T == 0) return CLEF_OK;
  const int64_t n = T * width;
  conv4_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(x, ldx, hist, hist_rows, w, T, width, out);
  return launch_status("conv4");
}

template <typename In>
int launch_delta_prologue_t(const In* proj, int64_t ldp, int a_col, int b_col, const float* hist, int hist_rows,
                            const float* conv_w, const float* dt_bias, const float* a_log, const SeqPack& pack,
                            int Hk, int Hv, float* q, float* k, float* v, float* g, float* beta, cudaStream_t s) {
  if (pack.total == 0) return CLEF_OK;
  const float qscale = (float)(1.0 / std::sqrt(128.0));
  const int width = 2 * Hk * 128 + Hv * 128;
  const dim3 grid((unsigned)(width / 1024), (unsigned)ceil_div(pack.total, PRO_RUN));
  static bool attr[64] = {false};
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    CLEF_CUDA(cudaFuncSetAttribute(delta_prologue_kernel<In>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   pro_smem<In>()));
    attr[dev] = true;
  }
  delta_prologue_kernel<In><<<grid, 256, pro_smem<In>(), s>>>(proj, ldp, a_col, b_col, hist, hist_rows, conv_w,
                                                               dt_bias, a_log, pack.cu_seqlens, pack.nseq,
                                                               pack.total, Hk, Hv, qscale, q, k, v, g, beta);
  return launch_status("delta_prologue");
}

int launch_delta_prologue(const float* proj, int64_t ldp, int a_col, int b_col, const float* hist,
                          int hist_rows, const float* conv_w, const float* dt_bias,
                          const float* a_log, const SeqPack& pack, int Hk, int Hv, int dk, int dv,
                          float* q, float* k, float* v, float* g, float* beta, cudaStream_t s) {
  (void)dk;
  (void)dv;
  return launch_delta_prologue_t(proj, ldp, a_col, b_col, hist, hist_rows, conv_w, dt_bias, a_log, pack, Hk, Hv, q,
                                 k, v, g, beta, s);
}

int launch_delta_prologue(const uint16_t* proj, int64_t ldp, int a_col, int b_col, const float* hist,
                          int hist_rows, const float* conv_w, const float* dt_bias,
                          const float* a_log, const SeqPack& pack, int Hk, int Hv, int dk, int dv,
                          float* q, float* k, float* v, float* g, float* beta, cudaStream_t s) {
  (void)dk;
  (void)dv;
  return launch_delta_prologue_t(proj, ldp, a_col, b_col, hist, hist_rows, conv_w, dt_bias, a_log, pack, Hk, Hv, q,
                                 k, v, g, beta, s);
}

int launch_delta_epilogue(const float* o, const uint16_t* z, int64_t ldz, const float* w, float eps,
                          int64_t T, int Hv, int dv, uint16_t* y, cudaStream_t s) {
  (void)dv;
  const int64_t rows = T * Hv;
  if (rows == 0) return CLEF_OK;
  delta_epilogue_kernel<uint16_t, false><<<(unsigned)ceil_div(T, 8), 256, 0, s>>>(o, z, ldz, w, eps, T, Hv, y);
  return launch_status("delta_epilogue");
}

int launch_delta_epilogue_split(const float* o, const float* z, int64_t ldz, const float* w, float eps,
                                int64_t T, int Hv, uint16_t* y, cudaStream_t s) {
  if (T * Hv == 0) return CLEF_OK;
  CLEF_CHECK(ldz % 4 == 0 && ((uintptr_t)z & 15) == 0, CLEF_ERR_INVALID,
             "delta_epilogue: F32 z rows must be 16-byte aligned");
  delta_epilogue_kernel<float, true><<<(unsigned)ceil_div(T, 8), 256, 0, s>>>(o, z, ldz, w, eps, T, Hv, y);
  return launch_status("delta_epilogue");
}

template <typename In>
int launch_attention_prologue_t(const In* proj, int64_t ldp, const float* qw, const float* kw,
                                float eps, const SeqPack& pack, int64_t pos_offset, int H, int Hkv,
                                int rot, const float* inv_freq_dev, uint16_t* q_out, uint16_t* k_out,
                                cudaStream_t s) {
  const int64_t rows = pack.total * (H + Hkv);
  if (rows == 0) return CLEF_OK;
  CLEF_CHECK(rot % 16 == 0 && rot <= 256, CLEF_ERR_UNSUPPORTED,
             "attention_prologue: rotary_dim must be a multiple of 16, at most 256");
  attention_prologue_kernel<In><<<(unsigned)ceil_div(pack.total, AP_WARPS), AP_WARPS * 32, 0, s>>>(
      proj, ldp, qw, kw, eps, pack.cu_seqlens, pack.nseq, pos_offset, H, Hkv, rot, inv_freq_dev,
      q_out, k_out, pack.total);
  return launch_status("attention_prologue");
}

int launch_attention_prologue(const uint16_t* proj, int64_t ldp, const float* qw, const float* kw,
                              float eps, const SeqPack& pack, int64_t pos_offset, int H, int Hkv,
                              int d, int rot, const float* inv_freq_dev, uint16_t* q_out,
                              uint16_t* k_out, cudaStream_t s) {
  (void)d;
  return launch_attention_prologue_t(proj, ldp, qw, kw, eps, pack, pos_offset, H, Hkv, rot, inv_freq_dev, q_out,
                                     k_out, s);
}

int launch_attention_prologue(const float* proj, int64_t ldp, const float* qw, const float* kw,
                              float eps, const SeqPack& pack, int64_t pos_offset, int H, int Hkv,
                              int d, int rot, const float* inv_freq_dev, uint16_t* q_out,
                              uint16_t* k_out, cudaStream_t s) {
  (void)d;
  return launch_attention_prologue_t(proj, ldp, qw, kw, eps, pack, pos_offset, H, Hkv, rot, inv_freq_dev, q_out,
                                     k_out, s);
}

// ---- split precision: gated attention output ------------------------------
// y = o * sigmoid(gate) in F32 (qwen.rs:519-524), stored as the split BF16
// operand of o_proj: hi in columns [0, H*d), lo in [H*d, 2*H*d).
__global__ void gate_split_kernel(const float* __restrict__ o, const float* __restrict__ gate, int64_t g_ts,
                                  int64_t g_hs, int H, int d, int64_t T, uint16_t* __restrict__ y) {
  const int64_t width = (int64_t)H * d;
  const int64_t quads = T * width / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < quads; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = i * 4;
    const int64_t t = e0 / width;
    const int64_t c = e0 - t * width;
    const int64_t h = c / d, e = c - h * d;
    const float4 ov = *reinterpret_cast<const float4*>(o + e0);
    const float4 gv = *reinterpret_cast<const float4*>(gate + t * g_ts + h * g_hs + e);
    const float y0 = ov.x * sigmoid_f(gv.x), y1 = ov.y * sigmoid_f(gv.y);
    const float y2 = ov.z * sigmoid_f(gv.z), y3 = ov.w * sigmoid_f(gv.w);
    const uint2 hi = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
    uint16_t* dst = y + t * 2 * width + c;
    *reinterpret_cast<uint2*>(dst) = hi;
    *reinterpret_cast<uint2*>(dst + width) = make_uint2(split_lo_bf16x2(y0, y1, hi.x), split_lo_bf16x2(y2, y3, hi.y));
  }
}

int launch_gate_split(const float* o, const float* gate, int64_t g_ts, int64_t g_hs, int H, int d, int64_t T,
                      uint16_t* y, cudaStream_t s) {
  if (T == 0) return CLEF_OK;
  CLEF_CHECK(d % 4 == 0 && g_ts % 4 == 0 && g_hs % 4 == 0 && ((((uintptr_t)o) | (uintptr_t)gate) & 15) == 0,
             CLEF_ERR_INVALID, "gate_split: F32 rows must be 16-byte aligned");
  const int64_t quads = T * H * d / 4;
  const unsigned blocks = (unsigned)std::min<int64_t>(ceil_div(quads, 256), 148 * 16);
  gate_split_kernel<<<blocks, 256, 0, s>>>(o, gate, g_ts, g_hs, H, d, T, y);
  return launch_status("gate_split");
}

int launch_embed(const uint16_t* table, const int32_t* ids, int64_t T, int hidden, float* h,
                 cudaStream_t s) {
  if (T == 0) return CLEF_OK;
  embed_kernel<<<(unsigned)T, 128, 0, s>>>(table, ids, hidden, h);
  return launch_status("embed");
}

int launch_head(const float* h, const float* norm_w, float eps, const SeqPack& pack, int hidden,
                const float* head_w, int n_out, float* logits, cudaStream_t s) {
  head_kernel<<<pack.nseq, 256, hidden * sizeof(float), s>>>(h, norm_w, eps, pack.cu_seqlens, hidden,
                                                             head_w, n_out, logits);
  return launch_status("head");
}

int launch_rows_bf16_to_f32(const uint16_t* src, int64_t ld, int64_t r0, int64_t count, int64_t ncols, float* dst,
                            int64_t ldd, cudaStream_t s) {
  if (count == 0) return CLEF_OK;
  rows_bf16_to_f32_kernel<<<(unsigned)count, 256, 0, s>>>(src + r0 * ld, ld, ncols, dst, ldd);
  return launch_status("rows_bf16_to_f32");
}

int launch_copy_rows(const void* src, int64_t ld, int64_t r0, int64_t count, int64_t ncols, int elem,
                     void* dst, int64_t ldd, cudaStream_t s) {
  if (count == 0) return CLEF_OK;
  const uint8_t* sp = reinterpret_cast<const uint8_t*>(src) + r0 * ld * elem;
  copy_rows_kernel<<<(unsigned)count, 256, 0, s>>>(sp, ld * elem, ncols * elem,
                                                    reinterpret_cast<uint8_t*>(dst), ldd * elem);
  return launch_status("copy_rows");
}

}  // namespace clef

using namespace clef;

extern "C" {

int clef_rmsnorm(const float* x, const float* weight, int64_t rows, int32_t width, float eps,
                 int32_t out_dtype, void* out, void* stream) {
  CLEF_CHECK(x && weight && out, CLEF_ERR_INVALID, "rmsnorm: null pointer");
  CLEF_CHECK(rows >= 0 && width > 0 && width <= 65536, CLEF_ERR_INVALID, "rmsnorm: dimensions");
  CLEF_CHECK(out_dtype == CLEF_F32 || out_dtype == CLEF_BF16, CLEF_ERR_INVALID, "rmsnorm: dtype");
  CLEF_CHECK(eps > 0.f && eps <= 1.f, CLEF_ERR_INVALID, "rmsnorm: epsilon");
  CLEF_CHECK(((uintptr_t)x & 15) == 0 && ((uintptr_t)weight & 15) == 0 && ((uintptr_t)out & 15) == 0,
             CLEF_ERR_INVALID, "rmsnorm: pointers must be 16-byte aligned");
  return launch_rmsnorm(x, weight, rows, width, eps, out_dtype, out, as_stream(stream));
}

int clef_conv4(const float* x, int64_t ldx, const float* history, int32_t history_rows,
               const float* weight, int64_t T, int32_t width, float* out, void* stream) {
  CLEF_CHECK(x && weight && out, CLEF_ERR_INVALID, "conv4: null pointer");
  CLEF_CHECK(T >= 0 && width > 0 && ldx >= width, CLEF_ERR_INVALID, "conv4: dimensions");
  CLEF_CHECK(history_rows >= 0 && history_rows <= 3 && (history_rows == 0 || history),
             CLEF_ERR_INVALID, "conv4: history");
  return launch_conv4(x, ldx, history, history_rows, weight, T, width, out, as_stream(stream));
}

int clef_delta_prologue(const float* proj, int64_t ldp, int32_t a_col, int32_t b_col,
                        const float* history, int32_t history_rows, const float* conv_weight,
                        const float* dt_bias, const float* a_log, int64_t T, int32_t Hk, int32_t Hv,
                        int32_t dk, int32_t dv, float* q, float* k, float* v, float* g, float* beta,
                        void* stream) {
  CLEF_CHECK(proj && conv_weight && dt_bias && a_log && q && k && v && g && beta, CLEF_ERR_INVALID,
             "delta_prologue: null pointer");
  CLEF_CHECK(dk == 128 && dv == 128, CLEF_ERR_UNSUPPORTED, "delta_prologue: dk and dv must be 128");
  CLEF_CHECK(Hk > 0 && Hv > 0 && Hv % Hk == 0, CLEF_ERR_INVALID, "delta_prologue: head counts");
  const int64_t width = 2LL * Hk * dk + (int64_t)Hv * dv;
  CLEF_CHECK(width % 1024 == 0, CLEF_ERR_UNSUPPORTED,
             "delta_prologue: q|k|v width must be a multiple of 1024");
  CLEF_CHECK(T > 0 && T <= (1LL << 31), CLEF_ERR_INVALID, "delta_prologue: T");
  CLEF_CHECK(ldp >= width && ldp % 4 == 0, CLEF_ERR_INVALID, "delta_prologue: ldp");
  CLEF_CHECK(((uintptr_t)proj & 15) == 0 && ((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 &&
                 ((uintptr_t)v & 15) == 0 && ((uintptr_t)conv_weight & 15) == 0 &&
                 ((uintptr_t)history & 15) == 0,
             CLEF_ERR_INVALID, "delta_prologue: tensors must be 16-byte aligned");
  CLEF_CHECK(a_col >= width && a_col + Hv <= ldp && b_col >= width && b_col + Hv <= ldp,
             CLEF_ERR_INVALID, "delta_prologue: gate columns");
  CLEF_CHECK(history_rows >= 0 && history_rows <= 3 && (history_rows == 0 || history),
             CLEF_ERR_INVALID, "delta_prologue: history");
  SeqPack pack;  // one sequence: no offsets table
  pack.nseq = 1;
  pack.total = T;
  return launch_delta_prologue(proj, ldp, a_col, b_col, history, history_rows, conv_weight,
                               dt_bias, a_log, pack, Hk, Hv, dk, dv, q, k, v, g, beta,
                               as_stream(stream));
}

int clef_compact_copy(const void* src, int32_t ndim, const int64_t* dims, const int64_t* strides,
                      int32_t elem_size, void* dst, void* stream) {
  CLEF_CHECK(src && dst && dims && strides, CLEF_ERR_INVALID, "compact_copy: null pointer");
  CLEF_CHECK(ndim >= 1 && ndim <= 4, CLEF_ERR_INVALID, "compact_copy: ndim must be 1..4");
  CLEF_CHECK(elem_size == 2 || elem_size == 4, CLEF_ERR_INVALID, "compact_copy: element size");
  int64_t d[4] = {1, 1, 1, 1}, st[4] = {0, 0, 0, 0};
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) {
    CLEF_CHECK(dims[i] >= 0 && strides[i] >= 0, CLEF_ERR_INVALID, "compact_copy: dims/strides");
    d[4 - ndim + i] = dims[i];
    st[4 - ndim + i] = strides[i];
    n *= dims[i];
  }
  if (n == 0) return CLEF_OK;
  const unsigned grid = (unsigned)ceil_div(n, 256);
  cudaStream_t s = as_stream(stream);
  if (elem_size == 4)
    compact_copy_kernel<uint32_t><<<grid, 256, 0, s>>>(
        (const uint32_t*)src, n, d[1], d[2], d[3], st[0], st[1], st[2], st[3], (uint32_t*)dst);
  else
    compact_copy_kernel<uint16_t><<<grid, 256, 0, s>>>(
        (const uint16_t*)src, n, d[1], d[2], d[3], st[0], st[1], st[2], st[3], (uint16_t*)dst);
  return launch_status("compact_copy");
}

}  // extern "C"
