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
// Every (head, value column) is an independent chain through the tokens. A
// column is held by LPC lanes of a warp, each keeping KL = dk / LPC state rows
// (keys) in registers, so a warp carries 32 / LPC columns and a token costs
// two reductions of log2(LPC) shuffle levels. The per-token work is bound by
// the SM's load/store data path (shuffles and loads share it), so a lane's
// keys are interleaved in pairs (lane j of a group holds keys 2j + 2 LPC i +
// {0, 1}): the group's q and k loads of one pair index read one contiguous
// 8 LPC-byte run, and the arithmetic runs on packed two-lane F32 multiplies
// and FMAs (each lane rounded as the scalar form is). Each token's packed row
// is prefetched into L1 PK_PREFETCH tokens ahead and its q, k, v, decay and
// beta are loaded one token ahead into a second register set. The state never
// leaves registers between tokens, so capturing and resuming reproduce an
// uninterrupted run bit for bit. Any dk that is a power of two up to 128 and
// any dv up to 128 are accepted, as the reference's `dimensions` check allows
// (metal.rs:280-290).
#include <cmath>

#include "kernels.cuh"

namespace clef {

namespace {

constexpr int PK_WARPS = 4;      // 128-thread CTAs
constexpr int PK_PREFETCH = 16;  // tokens between a row's L1 prefetch and its use
constexpr int PK_LPC128 = 8;     // lanes per value column when dk = 128

__device__ __forceinline__ void prefetch_l1(const float* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// One token's inputs for one lane.
template <int KL>
struct PkTok {
  float q[KL], k[KL];
  float v, decay, beta;
};

// KL key rows per lane, LPC lanes per value column (KL * LPC = dk). PAIRS: KL
// is even and the lane's keys are read as float2 pairs (the packed row width
// 2 dk + dv + 2 is even and the input 8-byte aligned, so every row starts on
// 8 bytes); otherwise key p of lane j is j + LPC p, read as single floats.
template <int KL, int LPC, bool PAIRS>
__global__ void __launch_bounds__(PK_WARPS * 32)
    delta_packed_kernel(const float* __restrict__ in, int T, int H, int dk, int dv,
                        const float* __restrict__ init, int capture, float* __restrict__ out) {
  constexpr int CPW = 32 / LPC;  // value columns per warp
  constexpr bool EVEN = KL % 2 == 0;
  constexpr int NP = EVEN ? KL / 2 : 0;                // packed pairs per lane
  constexpr int NA = NP >= 4 ? 4 : (NP > 0 ? NP : 1);  // independent packed partial sums
  const int lane = threadIdx.x & 31;
  const int j = lane % LPC, cl = lane / LPC;
  const int groups = (dv + CPW - 1) / CPW;
  const int w = blockIdx.x * PK_WARPS + (threadIdx.x >> 5);
  if (w >= H * groups) return;  // whole warps
  const int head = w / groups;
  const int col = (w - head * groups) * CPW + cl;
  const bool live = col < dv;  // lanes past dv carry a zero chain and store nothing
  const int width = 2 * dk + dv + 2;
  auto key_of = [&](int p) { return PAIRS ? 2 * j + 2 * LPC * (p >> 1) + (p & 1) : j + LPC * p; };
  float st[KL];
#pragma unroll
  for (int p = 0; p < KL; ++p) st[p] = (init && live) ? init[((int64_t)head * dk + key_of(p)) * dv + col] : 0.f;
  const float* base0 = in + (int64_t)head * width;
  const int64_t tstride = (int64_t)H * width;
  auto load = [&](PkTok<KL>& x, int t) {
    const float* b = base0 + (int64_t)t * tstride;
    if (PAIRS) {
#pragma unroll
      for (int i = 0; i < KL / 2; ++i) {
        const float2 qq = *reinterpret_cast<const float2*>(b + 2 * j + 2 * LPC * i);
        const float2 kk = *reinterpret_cast<const float2*>(b + dk + 2 * j + 2 * LPC * i);
        x.q[2 * i] = qq.x, x.q[2 * i + 1] = qq.y;
        x.k[2 * i] = kk.x, x.k[2 * i + 1] = kk.y;
      }
    } else {
#pragma unroll
      for (int p = 0; p < KL; ++p) {
        x.q[p] = b[j + LPC * p];
        x.k[p] = b[dk + j + LPC * p];
      }
    }
    x.v = live ? b[2 * dk + col] : 0.f;
    x.decay = b[2 * dk + dv];
    x.beta = b[2 * dk + dv + 1];
  };
  // Every 128-byte line of token t's row (width <= 386 floats < 32 lanes x 32).
  auto prefetch = [&](int t) {
    if (t < T) {
      const float* b = base0 + (int64_t)t * tstride;
      if (lane * 32 < width) prefetch_l1(b + lane * 32);
      if (lane == 31) prefetch_l1(b + width - 1);
    }
  };
  const int64_t state_out = (int64_t)T * H * dv;
  // Group-of-LPC sum of per-lane packed partial sums (or of the scalar one).
  auto reduce = [&](const float2 (&a)[NA], float scalar) {
    float r = scalar;
    if (EVEN) {
      float2 s2 = a[0];
#pragma unroll
      for (int i = 1; i < NA; ++i) s2 = __fadd2_rn(s2, a[i]);
      r = s2.x + s2.y;
    }
#pragma unroll
    for (int o = LPC / 2; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
  };
  auto step = [&](const PkTok<KL>& x, int t) {
    float2 a[NA];
    float sa = 0.f;
#pragma unroll
    for (int i = 0; i < NA; ++i) a[i] = make_float2(0.f, 0.f);
    if (EVEN) {
      const float2 dd = make_float2(x.decay, x.decay);
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const float2 s2 = __fmul2_rn(make_float2(st[2 * i], st[2 * i + 1]), dd);
        st[2 * i] = s2.x, st[2 * i + 1] = s2.y;
        a[i % NA] = __ffma2_rn(s2, make_float2(x.k[2 * i], x.k[2 * i + 1]), a[i % NA]);
      }
    } else {
#pragma unroll
      for (int p = 0; p < KL; ++p) {
        st[p] = st[p] * x.decay;
        sa = fmaf(st[p], x.k[p], sa);
      }
    }
    const float mem = reduce(a, sa);
    const float d = (x.v - mem) * x.beta;
#pragma unroll
    for (int i = 0; i < NA; ++i) a[i] = make_float2(0.f, 0.f);
    sa = 0.f;
    if (EVEN) {
      const float2 d2 = make_float2(d, d);
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const float2 s2 =
            __ffma2_rn(make_float2(x.k[2 * i], x.k[2 * i + 1]), d2, make_float2(st[2 * i], st[2 * i + 1]));
        st[2 * i] = s2.x, st[2 * i + 1] = s2.y;
        a[i % NA] = __ffma2_rn(s2, make_float2(x.q[2 * i], x.q[2 * i + 1]), a[i % NA]);
      }
    } else {
#pragma unroll
      for (int p = 0; p < KL; ++p) {
        st[p] = fmaf(x.k[p], d, st[p]);
        sa = fmaf(st[p], x.q[p], sa);
      }
    }
    const float res = reduce(a, sa);
    if (j == 0 && live) out[((int64_t)t * H + head) * dv + col] = res;
    if (t + 1 == capture && live) {
#pragma unroll
      for (int p = 0; p < KL; ++p) out[state_out + ((int64_t)head * dk + key_of(p)) * dv + col] = st[p];
    }
  };
#pragma unroll 1
  for (int t = 0; t < PK_PREFETCH; ++t) prefetch(t);
  PkTok<KL> A, B;
  load(A, 0);
#pragma unroll 1
  for (int t = 0; t < T; t += 2) {
    if (t + 1 < T) load(B, t + 1);
    prefetch(t + PK_PREFETCH);
    step(A, t);
    if (t + 1 >= T) break;
    if (t + 2 < T) load(A, t + 2);
    prefetch(t + 1 + PK_PREFETCH);
    step(B, t + 1);
  }
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
  // LPC lanes per value column, 32 / LPC columns per warp.
  const int lpc = dk == 128 ? PK_LPC128 : dk < 4 ? dk : 4;
  const int groups = (dv + 32 / lpc - 1) / (32 / lpc);
  const unsigned blocks = (unsigned)ceil_div((int64_t)H * groups, PK_WARPS);
  const bool pairs = dv % 2 == 0 && ((uintptr_t)packed & 7) == 0;
#define CLEF_PK_LAUNCH(KL, LPC, PAIRS) \
  delta_packed_kernel<KL, LPC, PAIRS><<<blocks, PK_WARPS * 32, 0, s>>>(packed, (int)T, H, dk, dv, initial_state, \
                                                                       (int)capture, out)
#define CLEF_PK_LAUNCH2(KL, LPC)        \
  do {                                  \
    if (pairs)                          \
      CLEF_PK_LAUNCH(KL, LPC, true);    \
    else                                \
      CLEF_PK_LAUNCH(KL, LPC, false);   \
  } while (0)
  switch (dk) {
    case 128: CLEF_PK_LAUNCH2(128 / PK_LPC128, PK_LPC128); break;
    case 64: CLEF_PK_LAUNCH2(16, 4); break;
    case 32: CLEF_PK_LAUNCH2(8, 4); break;
    case 16: CLEF_PK_LAUNCH2(4, 4); break;
    case 8: CLEF_PK_LAUNCH2(2, 4); break;
    case 4: CLEF_PK_LAUNCH(1, 4, false); break;
    case 2: CLEF_PK_LAUNCH(1, 2, false); break;
    default: CLEF_PK_LAUNCH(1, 1, false); break;
  }
#undef CLEF_PK_LAUNCH2
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
