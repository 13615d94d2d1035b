// delta_packed.cu — the gated-DeltaNet operators in the reference's packed
// layout, for callers bound to its Candle custom ops:
//
//   clef_delta_packed          DeltaKernel / CachedDelta (models/metal.rs:79-413):
//                              packed [T, H, 2dk + dv + 2] = q | k | v | e^g | beta,
//                              output o [T, H, dv] followed, when a capture is
//                              asked, by the state after token `capture`
//                              [H, dk, dv]; optional initial state.
//   clef_delta_prepare_packed  DeltaPrepareKernel (models/pointwise.rs:195-279):
//                              post-conv rows [T, 2 Hk 128 + Hv 128], log-decay
//                              g and beta [T, Hv] -> the packed layout above with
//                              dk = dv = 128 (q L2-normalised and scaled by
//                              1/sqrt(128), k L2-normalised, both repeated per
//                              value head, decay = e^g).
//
// The recurrence kernel is the reference's per-token update in F32
// (delta_recurrence_prefill, qwen.rs:867-880; clef_delta, delta.metal:18-131):
//   S <- S * decay;  d = (v - S^T k) * beta;  S <- S + k d^T;  o = S^T q.
// One warp owns one value column of one head (two when H * dv > 2048), so
// many independent per-token chains share each SM; lane l holds the state
// rows (keys) l, l + 32, l + 64, l + 96 of its columns in registers, so a
// token costs two warp reductions. The inputs of the next four tokens are in
// flight while the current one is processed. The state never leaves registers
// between tokens, so capturing and resuming reproduce an uninterrupted run bit
// for bit. Any dk that is a power of two up to 128 and any dv up to 128 are
// accepted, as the reference's `dimensions` check allows (metal.rs:280-290).
#include <cmath>

#include "kernels.cuh"

namespace clef {

namespace {

constexpr int PK_WARPS = 4;  // 128-thread CTAs
constexpr int PK_AHEAD = 4;  // tokens whose inputs are in flight ahead of the one being processed

// KP: key rows per lane (1: dk <= 32, 2: dk = 64, 4: dk = 128); NV: value
// columns per warp (1, or 2 when H * dv warps of one column would not all be
// resident at once, which would run the token loop in two waves).
template <int KP, int NV>
__global__ void __launch_bounds__(PK_WARPS * 32)
    delta_packed_kernel(const float* __restrict__ in, int T, int H, int dk, int dv,
                        const float* __restrict__ init, int capture, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int groups = (dv + NV - 1) / NV;
  const int w = blockIdx.x * PK_WARPS + (threadIdx.x >> 5);
  if (w >= H * groups) return;  // whole warps
  const int head = w / groups;
  const int col0 = (w - head * groups) * NV;
  const int width = 2 * dk + dv + 2;
  float st[NV][KP];
#pragma unroll
  for (int c = 0; c < NV; ++c)
#pragma unroll
    for (int p = 0; p < KP; ++p) {
      const int key = lane + 32 * p, col = col0 + c;
      st[c][p] = (init && key < dk && col < dv) ? init[((int64_t)head * dk + key) * dv + col] : 0.f;
    }
  // Ring of the next PK_AHEAD tokens' inputs (slot s holds token t with t % PK_AHEAD == s).
  float rk[PK_AHEAD][KP], rq[PK_AHEAD][KP], rv[PK_AHEAD][NV], rd[PK_AHEAD], rb[PK_AHEAD];
  const float* base0 = in + (int64_t)head * width;
  const int64_t tstride = (int64_t)H * width;
#define CLEF_PK_LOAD(t, s)                                        \
  do {                                                            \
    const float* b_ = base0 + (int64_t)(t) * tstride;             \
    _Pragma("unroll") for (int p = 0; p < KP; ++p) {              \
      const int key = lane + 32 * p;                              \
      rq[s][p] = key < dk ? b_[key] : 0.f;                        \
      rk[s][p] = key < dk ? b_[dk + key] : 0.f;                   \
    }                                                             \
    _Pragma("unroll") for (int c = 0; c < NV; ++c)                \
      rv[s][c] = col0 + c < dv ? b_[2 * dk + col0 + c] : 0.f;     \
    rd[s] = b_[2 * dk + dv];                                      \
    rb[s] = b_[2 * dk + dv + 1];                                  \
  } while (0)
#pragma unroll
  for (int s = 0; s < PK_AHEAD; ++s)
    if (s < T) CLEF_PK_LOAD(s, s);
  const int64_t state_out = (int64_t)T * H * dv;
  for (int t0 = 0; t0 < T; t0 += PK_AHEAD) {
#pragma unroll
    for (int s = 0; s < PK_AHEAD; ++s) {
      const int t = t0 + s;
      if (t >= T) break;
      float k[KP], q[KP], v[NV];
#pragma unroll
      for (int p = 0; p < KP; ++p) {
        k[p] = rk[s][p];
        q[p] = rq[s][p];
      }
#pragma unroll
      for (int c = 0; c < NV; ++c) v[c] = rv[s][c];
      const float decay = rd[s], beta = rb[s];
      if (t + PK_AHEAD < T) CLEF_PK_LOAD(t + PK_AHEAD, s);
      float mem[NV];
#pragma unroll
      for (int c = 0; c < NV; ++c) {
        mem[c] = 0.f;
#pragma unroll
        for (int p = 0; p < KP; ++p) {
          st[c][p] = st[c][p] * decay;
          mem[c] = fmaf(st[c][p], k[p], mem[c]);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int c = 0; c < NV; ++c) mem[c] += __shfl_xor_sync(0xffffffffu, mem[c], o);
      float res[NV];
#pragma unroll
      for (int c = 0; c < NV; ++c) {
        const float d = (v[c] - mem[c]) * beta;
        res[c] = 0.f;
#pragma unroll
        for (int p = 0; p < KP; ++p) {
          st[c][p] = fmaf(k[p], d, st[c][p]);
          res[c] = fmaf(st[c][p], q[p], res[c]);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int c = 0; c < NV; ++c) res[c] += __shfl_xor_sync(0xffffffffu, res[c], o);
      if (lane < NV && col0 + lane < dv) {
        float r = res[0];
#pragma unroll
        for (int c = 1; c < NV; ++c)
          if (lane == c) r = res[c];
        out[((int64_t)t * H + head) * dv + col0 + lane] = r;
      }
      if (t + 1 == capture) {
#pragma unroll
        for (int c = 0; c < NV; ++c)
#pragma unroll
          for (int p = 0; p < KP; ++p) {
            const int key = lane + 32 * p, col = col0 + c;
            if (key < dk && col < dv) out[state_out + ((int64_t)head * dk + key) * dv + col] = st[c][p];
          }
      }
    }
  }
#undef CLEF_PK_LOAD
}

// One warp per (token, value head): the value head's query/key head is
// h / (Hv / Hk); q = q / sqrt(|q|^2 + 1e-6) / sqrt(128), k = k / sqrt(|k|^2 +
// 1e-6) (qwen.rs:837-845), v copied, decay = e^g, beta copied.
__global__ void __launch_bounds__(256)
    delta_prepare_packed_kernel(const float* __restrict__ mixed, int64_t ldm, const float* __restrict__ g,
                                const float* __restrict__ beta, int64_t T, int Hk, int Hv,
                                float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= T * Hv) return;
  const int64_t t = row / Hv;
  const int h = (int)(row - t * Hv);
  const int kh = h / (Hv / Hk);
  const float* src = mixed + t * ldm;
  const float4 q = *reinterpret_cast<const float4*>(src + kh * 128 + lane * 4);
  const float4 k = *reinterpret_cast<const float4*>(src + (int64_t)Hk * 128 + kh * 128 + lane * 4);
  const float4 v = *reinterpret_cast<const float4*>(src + (int64_t)2 * Hk * 128 + h * 128 + lane * 4);
  const float qs = warp_sum(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w);
  const float ks = warp_sum(k.x * k.x + k.y * k.y + k.z * k.z + k.w * k.w);
  const float qn = sqrtf(qs + 1e-6f), kn = sqrtf(ks + 1e-6f);
  const float scale = 0.08838834764831845f;  // 1 / sqrt(128)
  float* dst = out + row * 386;
  // Row pitch 386 floats: the 128-float blocks start at 8-byte boundaries only.
  reinterpret_cast<float2*>(dst + lane * 4)[0] = make_float2(q.x / qn * scale, q.y / qn * scale);
  reinterpret_cast<float2*>(dst + lane * 4)[1] = make_float2(q.z / qn * scale, q.w / qn * scale);
  reinterpret_cast<float2*>(dst + 128 + lane * 4)[0] = make_float2(k.x / kn, k.y / kn);
  reinterpret_cast<float2*>(dst + 128 + lane * 4)[1] = make_float2(k.z / kn, k.w / kn);
  reinterpret_cast<float2*>(dst + 256 + lane * 4)[0] = make_float2(v.x, v.y);
  reinterpret_cast<float2*>(dst + 256 + lane * 4)[1] = make_float2(v.z, v.w);
  if (lane == 0) {
    dst[384] = expf(g[row]);
    dst[385] = beta[row];
  }
}

}  // namespace

}  // namespace clef

using namespace clef;

extern "C" {

int clef_delta_packed(const float* packed, int64_t T, int32_t H, int32_t dk, int32_t dv,
                      const float* initial_state, int64_t capture, float* out, void* stream) {
  CLEF_CHECK(packed && out, CLEF_ERR_INVALID, "delta_packed: null pointer");
  // The reference's `dimensions` (metal.rs:280-290), checked before any launch.
  CLEF_CHECK(T >= 1 && T <= 4096 && H >= 1 && H <= 32 && dk >= 1 && dk <= 128 && (dk & (dk - 1)) == 0 &&
                 dv >= 1 && dv <= 128,
             CLEF_ERR_INVALID, "delta_packed: fused DeltaNet dimensions (T 1..4096, H 1..32, dk a power of two "
                               "up to 128, dv 1..128)");
  CLEF_CHECK(capture >= 0 && capture <= T, CLEF_ERR_INVALID, "delta_packed: capture boundary");
  cudaStream_t s = as_stream(stream);
  // One column per warp while all H * dv warps fit on the GPU at once
  // (<= 2048 here); two per warp beyond, so the token loop runs in one wave.
  const bool two = (int64_t)H * dv > 2048;
  const int nv = two ? 2 : 1;
  const unsigned blocks = (unsigned)ceil_div((int64_t)H * ((dv + nv - 1) / nv), PK_WARPS);
#define CLEF_PK_LAUNCH(KP)                                                                                 \
  do {                                                                                                   \
    if (two)                                                                                             \
      delta_packed_kernel<KP, 2><<<blocks, PK_WARPS * 32, 0, s>>>(packed, (int)T, H, dk, dv, initial_state, \
                                                                  (int)capture, out);                    \
    else                                                                                                 \
      delta_packed_kernel<KP, 1><<<blocks, PK_WARPS * 32, 0, s>>>(packed, (int)T, H, dk, dv, initial_state, \
                                                                  (int)capture, out);                    \
  } while (0)
  if (dk <= 32) CLEF_PK_LAUNCH(1);
  else if (dk == 64) CLEF_PK_LAUNCH(2);
  else CLEF_PK_LAUNCH(4);
#undef CLEF_PK_LAUNCH
  return launch_status("delta_packed");
}

int clef_delta_prepare_packed(const float* mixed, int64_t ldm, const float* g, const float* beta, int64_t T,
                              int32_t Hk, int32_t Hv, float* out, void* stream) {
  CLEF_CHECK(mixed && g && beta && out, CLEF_ERR_INVALID, "delta_prepare_packed: null pointer");
  CLEF_CHECK(T >= 1 && T <= 4096, CLEF_ERR_INVALID, "delta_prepare_packed: T must be 1..4096");
  CLEF_CHECK(Hk >= 1 && Hv >= Hk && Hv % Hk == 0 && Hv <= 128, CLEF_ERR_INVALID,
             "delta_prepare_packed: head counts");
  CLEF_CHECK(ldm >= (int64_t)(2 * Hk + Hv) * 128 && ldm % 4 == 0 && ((uintptr_t)mixed & 15) == 0,
             CLEF_ERR_INVALID, "delta_prepare_packed: mixed rows must be 16-byte aligned and hold q | k | v");
  CLEF_CHECK(((uintptr_t)out & 7) == 0, CLEF_ERR_INVALID, "delta_prepare_packed: out must be 8-byte aligned");
  const int64_t rows = T * Hv;
  delta_prepare_packed_kernel<<<(unsigned)ceil_div(rows, 8), 256, 0, as_stream(stream)>>>(mixed, ldm, g, beta, T,
                                                                                          Hk, Hv, out);
  return launch_status("delta_prepare_packed");
}

}  // extern "C"
