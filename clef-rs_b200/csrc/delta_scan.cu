// delta_scan.cu — chunked gated-DeltaNet scan on the tensor cores
// (chunk C = 64, dk = dv = 128).
//
// The reference recurrence, per v-head (delta_recurrence_prefill,
// crates/core/src/models/qwen.rs:867-880; clef_delta, delta.metal:62-130):
//   S <- S e^{g_t};  d_t = (v_t - S^T k_t) beta_t;  S <- S + k_t d_t^T;  o_t = S^T q_t
// is evaluated a chunk at a time in the WY / UT form that the reference states
// in its chunkwise candidate (chunk.rs:16-149, chunk.metal:10-164). With
//   G_i  = sum_{s<=i} g_s (chunk-relative, accumulated in FP64),
//   A_ij = beta_i e^{G_i-G_j} k_i.k_j (j < i),   T = (I + A)^{-1},
//   P_ij = e^{G_i-G_j} q_i.k_j (j <= i),
// and the state kept transposed (S^T, rows = value columns):
//   R^T  = V^T - (S^T K^T) diag(e^G)                 residual of the old state
//   D^T  = R^T (T diag(beta))^T                       the chunk's delta rows
//   O^T  = (S^T Q^T) diag(e^G) + D^T P^T
//   S^T <- e^{G_last} S^T + (D^T diag(e^{G_last-G})) K
// Every decay factor is the exponential of a non-positive difference of
// chunk-relative cumulative log-decays, so nothing divides by an underflowed
// prefix product (a per-token decay of -1000 is exact).
//
// Products use BF16 tensor-core MMAs with F32 accumulation and a two-term
// BF16 split of both operands (x = hi + lo; x*y ~ hi*hi + hi*lo + lo*hi), which
// keeps ~16 mantissa bits: the result tracks the F32 per-token recurrence to
// ~1e-5. The workspace path runs two kernels: delta_prep_kernel (chunk-
// parallel; Gram products on tcgen05) and delta_carry_tc_kernel (the state
// carry on tcgen05, S^T in TMEM). The allocation-free path runs one fused
// kernel, delta_scan_kernel (one CTA per (sequence, v-head), 8 warps; warp w
// keeps value rows [16w, 16w+16) of S^T as mma.sync accumulators in registers,
// re-packed in registers as the A operand of the next product).
// The triangular inverse T is computed by blocked forward substitution: the
// four 16 x 16 diagonal blocks in F32, then the off-diagonal blocks with the
// same split-BF16 tensor-core products.
// A capture point inside a chunk does not change the chunking: the state at
// the capture token is formed from the same chunk quantities, so a prefill with
// capture is bit-identical to one without.
#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "sm100.cuh"

#define RC_(x)           \
  do {                   \
    int rc_ = (x);       \
    if (rc_) return rc_; \
  } while (0)

namespace clef {

namespace {

constexpr int C = 64;    // chunk length
constexpr int DK = 128;  // key dim
constexpr int DV = 128;  // value dim
constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;

// ---- shared-memory layout (bytes) -------------------------------------------
constexpr int KQ_BYTES = C * DK * 2;   // one [64][128] BF16 tile (16 KB)
constexpr int SQ_BYTES = C * C * 2;    // one [64][64] BF16 tile (8 KB)
constexpr int OFF_KHI = 0;
constexpr int OFF_KLO = OFF_KHI + KQ_BYTES;
constexpr int OFF_QHI = OFF_KLO + KQ_BYTES;
constexpr int OFF_QLO = OFF_QHI + KQ_BYTES;
// THI, TLO, PHI, PLO: the order carry_step reads them in (ChunkOps::tp).
constexpr int OFF_THI = OFF_QLO + KQ_BYTES;
constexpr int OFF_TLO = OFF_THI + SQ_BYTES;
constexpr int OFF_PHI = OFF_TLO + SQ_BYTES;
constexpr int OFF_PLO = OFF_PHI + SQ_BYTES;
constexpr int AP = 68;                               // F32 pitch of A and T (16-byte row stores spread over all banks)
constexpr int OFF_A = OFF_PLO + SQ_BYTES;            // F32 [64][65]
constexpr int OFF_T = OFF_A + C * AP * 4;            // F32 [64][65]
constexpr int OFF_M = OFF_T + C * AP * 4;            // F32 [3][16][17] scratch
constexpr int OFF_G = OFF_M + 3 * 16 * 17 * 4;       // double [64]
constexpr int OFF_EG = OFF_G + C * 8;                // F32 [64] e^{G}
constexpr int OFF_EGD = OFF_EG + C * 4;              // F32 [64] e^{G_last - G}
constexpr int OFF_BETA = OFF_EGD + C * 4;            // F32 [64]
constexpr int OFF_ECAP = OFF_BETA + C * 4;           // F32 [64] e^{G_c - G} (capture)
constexpr int SMEM = OFF_ECAP + C * 4 + 16;

// Byte offset of element (row, col) in a BF16 tile whose rows hold `cpr`
// 16-byte chunks; the chunk index is XOR-swizzled with row & 7 so that the
// eight rows an ldmatrix phase reads hit distinct banks.
__device__ __forceinline__ uint32_t swz(int row, int col, int cpr) {
  return (uint32_t)(row * cpr * 16 + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1));
}

// Byte offset of element (row, k) of the prep kernel's tcgen05 Gram operand:
// the canonical K-major layout with the 128-byte swizzle, rows 0..63 = K and
// 64..127 = Q of the chunk, two 64-wide atoms along dk of [128 rows x 128 B]
// each (16-byte chunk index XOR row & 7 inside 1024-byte row groups).
constexpr int GRAM_TILE = 2 * 128 * 128;  // bytes of one (hi or lo) [128 x 128] BF16 operand
__device__ __forceinline__ uint32_t umma_off(int row, int k) {
  return (uint32_t)((k >> 6) * (128 * 128) + row * 128 + ((((k & 63) >> 3) ^ (row & 7)) << 4) + ((k & 7) << 1));
}

__device__ __forceinline__ void split(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  __nv_bfloat16 h0, l0, h1, l1;
  split(x0, h0, l0);
  split(x1, h1, l1);
  hi = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
  lo = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
}

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// c += a * b with both operands split: hi*hi + hi*lo + lo*hi.
__device__ __forceinline__ void mma3(float (&c)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                     uint32_t bh0, uint32_t bh1, uint32_t bl0, uint32_t bl1) {
  mma(c, al, bh0, bh1);
  mma(c, ah, bl0, bl1);
  mma(c, ah, bh0, bh1);
}

// A fragments (k-step of 16) from two accumulator n-tiles of a 16-row block.
__device__ __forceinline__ void acc_to_a(const float (&c0)[4], const float (&c1)[4], uint32_t (&ah)[4],
                                         uint32_t (&al)[4]) {
  split2(c0[0], c0[1], ah[0], al[0]);
  split2(c0[2], c0[3], ah[1], al[1]);
  split2(c1[0], c1[1], ah[2], al[2]);
  split2(c1[2], c1[3], ah[3], al[3]);
}

// B fragments for two n-tiles (rows n0..n0+15 of a row-major [n][k] tile) at
// k-step k0: out[0..1] = n-tile n0, out[2..3] = n-tile n0+8.
__device__ __forceinline__ void ldb_nk(uint32_t base, int n0, int k0, int cpr, int lane,
                                       uint32_t (&r)[4]) {
  const int row = n0 + (lane & 7) + ((lane >> 4) << 3);
  const int col = k0 + ((lane >> 3) & 1) * 8;
  ldsm4(base + swz(row, col, cpr), r);
}
// A fragments from a row-major [m][k] tile: rows m0..m0+15 at k-step k0.
__device__ __forceinline__ void lda(uint32_t base, int m0, int k0, int cpr, int lane, uint32_t (&r)[4]) {
  ldsm4(base + swz(m0 + (lane & 15), k0 + (lane >> 4) * 8, cpr), r);
}

// Byte offset of element (row, col) of K/Q tile t (0 = K hi, 1 = K lo, 2 = Q hi,
// 3 = Q lo) of a chunk's K/Q operand. UK: the tcgen05 layout of the workspace
// image and the prep kernel's Gram operand (hi tile [K; Q] then lo tile, in
// umma_off order); otherwise four [64][128] tiles in the ldmatrix swizzle (the
// fused kernel's shared-memory tiles).
template <bool UK>
__device__ __forceinline__ uint32_t kq_off(int t, int row, int col) {
  if (UK) return (uint32_t)((t & 1) * GRAM_TILE) + umma_off(row + (t >> 1) * 64, col);
  return (uint32_t)(t * KQ_BYTES) + swz(row, col, 16);
}
// B fragments of the fused kernel's K/Q tile t for two n-tiles at k-step k0:
// read as a row-major [n][k] tile (ldb_kq) or, transposed, as [k][n] (ldb_kq_t).
__device__ __forceinline__ void ldb_kq(uint32_t base, int t, int n0, int k0, int lane, uint32_t (&r)[4]) {
  const int row = n0 + (lane & 7) + ((lane >> 4) << 3);
  const int col = k0 + ((lane >> 3) & 1) * 8;
  ldsm4(base + kq_off<false>(t, row, col), r);
}
__device__ __forceinline__ void ldb_kq_t(uint32_t base, int t, int n0, int k0, int lane, uint32_t (&r)[4]) {
  const int row = k0 + (lane & 7) + (((lane >> 3) & 1) << 3);
  const int col = n0 + ((lane >> 4) << 3);
  ldsm4t(base + kq_off<false>(t, row, col), r);
}

// ---------------------------------------------------------------------------
// Building blocks shared by the fused kernel and the prep/carry pipeline, so
// both paths perform the same arithmetic in the same order.
// ---------------------------------------------------------------------------

// Stores one 32-bit word at byte offset `o` of a tile, in shared or global
// memory (the global "tile image" has the shared-memory layout byte for byte).
template <bool GLOBAL>
__device__ __forceinline__ void put32(uint8_t* base, uint32_t o, uint32_t v) {
  *reinterpret_cast<uint32_t*>(base + o) = v;
}

// K, Q rows [t0, t0 + n) of k-head kh, split into hi/lo BF16 tiles (zero rows
// past n). Writes the four tiles (KHI, KLO, QHI, QLO, 16 KB each) to `sm_kq`
// and, when `img` is set, the same bytes to a global tile image.
__device__ __forceinline__ void stage_kq(const float* __restrict__ q, const float* __restrict__ k,
                                         int64_t t0, int n, int Hk, int kh, uint8_t* sm_kq,
                                         uint8_t* img, int tid, int nthreads, bool umma_smem = false) {
  // Four rows' loads are issued before any is used, so a thread has eight
  // 16-byte loads in flight instead of two.
  constexpr int U = 4;
  for (int base = tid; base < C * (DK / 4); base += U * nthreads) {
    float4 kv[U], qv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * nthreads;
      const int i = idx >> 5, c4 = (idx & 31) * 4;
      kv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      qv[u] = kv[u];
      if (idx < C * (DK / 4) && i < n) {
        const int64_t off = ((t0 + i) * Hk + kh) * DK + c4;
        kv[u] = *reinterpret_cast<const float4*>(k + off);
        qv[u] = *reinterpret_cast<const float4*>(q + off);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * nthreads;
      if (idx >= C * (DK / 4)) break;
      const int i = idx >> 5, c4 = (idx & 31) * 4;
      uint32_t kh0, kl0, kh1, kl1, qh0, ql0, qh1, ql1;
      split2(kv[u].x, kv[u].y, kh0, kl0);
      split2(kv[u].z, kv[u].w, kh1, kl1);
      split2(qv[u].x, qv[u].y, qh0, ql0);
      split2(qv[u].z, qv[u].w, qh1, ql1);
      const uint32_t o = swz(i, c4, 16);
      const uint2 w[4] = {make_uint2(kh0, kh1), make_uint2(kl0, kl1), make_uint2(qh0, qh1),
                          make_uint2(ql0, ql1)};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if (umma_smem) {
          // [K; Q] rows of the tcgen05 operand (hi tile, then lo tile); the
          // workspace image has the same bytes.
          const uint32_t u = kq_off<true>(t, i, c4);
          *reinterpret_cast<uint2*>(sm_kq + u) = w[t];
          if (img) *reinterpret_cast<uint2*>(img + u) = w[t];
        } else {
          *reinterpret_cast<uint2*>(sm_kq + t * KQ_BYTES + o) = w[t];
        }
      }
    }
  }
}

// Chunk-relative inclusive cumsum of g in FP64 and the betas (one warp).
__device__ __forceinline__ void cumsum_gates(const float* __restrict__ g,
                                             const float* __restrict__ beta, int64_t t0, int n,
                                             int Hv, int h, int lane, double* Gs, float* bs) {
  const int i0 = 2 * lane, i1 = i0 + 1;
  const double g0 = i0 < n ? (double)g[(t0 + i0) * Hv + h] : 0.0;
  const double g1 = i1 < n ? (double)g[(t0 + i1) * Hv + h] : 0.0;
  const double pair = g0 + g1;
  double run = pair;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double up = __shfl_up_sync(0xffffffffu, run, o);
    if (lane >= o) run += up;
  }
  const double excl = run - pair;
  Gs[i0] = excl + g0;
  Gs[i1] = excl + g0 + g1;
  bs[i0] = i0 < n ? beta[(t0 + i0) * Hv + h] : 0.f;
  bs[i1] = i1 < n ? beta[(t0 + i1) * Hv + h] : 0.f;
}

// Raw Gram fragments of warp w: rows (w/2)*16.., columns (w%2)*32.. of K K^T
// and Q K^T (8 warps cover 64 x 64).
__device__ __forceinline__ void gram_mma(uint32_t kq_base, int warp, int lane, float (&kk)[4][4],
                                         float (&qk)[4][4]) {
  const int m0 = (warp >> 1) * 16, nb = (warp & 1) * 32;
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) kk[j][e] = qk[j][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < DK / 16; ++ks) {
    uint32_t akh[4], akl[4], aqh[4], aql[4];
    lda(kq_base + 0 * KQ_BYTES, m0, ks * 16, 16, lane, akh);
    lda(kq_base + 1 * KQ_BYTES, m0, ks * 16, 16, lane, akl);
    lda(kq_base + 2 * KQ_BYTES, m0, ks * 16, 16, lane, aqh);
    lda(kq_base + 3 * KQ_BYTES, m0, ks * 16, 16, lane, aql);
#pragma unroll
    for (int np = 0; np < 2; ++np) {
      uint32_t bh[4], bl[4];
      ldb_nk(kq_base + 0 * KQ_BYTES, nb + np * 16, ks * 16, 16, lane, bh);
      ldb_nk(kq_base + 1 * KQ_BYTES, nb + np * 16, ks * 16, 16, lane, bl);
      mma3(kk[2 * np], akh, akl, bh[0], bh[1], bl[0], bl[1]);
      mma3(kk[2 * np + 1], akh, akl, bh[2], bh[3], bl[2], bl[3]);
      mma3(qk[2 * np], aqh, aql, bh[0], bh[1], bl[0], bl[1]);
      mma3(qk[2 * np + 1], aqh, aql, bh[2], bh[3], bl[2], bl[3]);
    }
  }
}

// [K; Q] K^T (128 x 64, F32 in TMEM columns [tmem, tmem + 64)) on the tcgen05
// tensor core from the split-BF16 operand at `a_base` (umma_off layout):
// hi*hi + hi*lo + lo*hi, eight 16-wide K steps each. The B operand is rows
// 0..63 of the same tile (K). One thread issues; completion arrives on `bar`.
__device__ __forceinline__ void gram_tc_issue(uint32_t a_base, uint32_t tmem, uint64_t* bar) {
  constexpr uint32_t idesc = sm100::idesc_bf16_f32(128, 64);
  const uint32_t hi = a_base, lo = a_base + GRAM_TILE;
  uint32_t acc = 0;
#pragma unroll
  for (int term = 0; term < 3; ++term) {
    const uint32_t A = term == 2 ? lo : hi;
    const uint32_t B = term == 1 ? lo : hi;
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      const uint32_t off = (uint32_t)((kk >> 2) * (128 * 128) + (kk & 3) * 32);
      sm100::umma_f16(tmem, sm100::desc_k_sw128(A + off), sm100::desc_k_sw128(B + off), idesc, acc);
      acc = 1;
    }
  }
  sm100::umma_commit(bar);
}

// Row-per-thread form of gram_store for the tcgen05 Gram: `g` holds columns
// [32 half, 32 half + 32) of row `row` of [K K^T; Q K^T]. Rows < 64 give A
// (F32, strictly lower, beta_i e^{G_i-G_j} k_i.k_j) into As; rows >= 64 give
// P (lower incl. diagonal, e^{G_i-G_j} q_i.k_j) as hi/lo tiles at p_hi / p_lo.
template <bool GLOBAL>
__device__ __forceinline__ void gram_store_rows(const uint32_t (&g)[32], int row, int half, int n,
                                                const double* Gs, const float* bs, float* As, uint8_t* p_hi,
                                                uint8_t* p_lo) {
  const int i = row & 63, c0 = half * 32;
  const double gi = Gs[i];
  if (row < 64) {
    const float bi = bs[i];
#pragma unroll
    for (int c = 0; c < 32; c += 4) {
      float av[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int col = c0 + c + u;
        const bool lower = col < i && i < n;
        const float decay = lower ? expf((float)(gi - Gs[col])) : 0.f;
        av[u] = lower ? bi * (decay * __uint_as_float(g[c + u])) : 0.f;
      }
      *reinterpret_cast<float4*>(As + i * AP + c0 + c) = make_float4(av[0], av[1], av[2], av[3]);
    }
  } else {
    // One 16-byte chunk (8 columns) of the hi and lo tiles per store: the
    // swizzle puts the 8 rows of a store phase on 8 distinct chunks.
#pragma unroll
    for (int c = 0; c < 32; c += 8) {
      uint32_t ph[4], pl[4];
#pragma unroll
      for (int u = 0; u < 8; u += 2) {
        float pv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int col = c0 + c + u + e;
          const bool lower = col <= i && i < n;
          pv[e] = lower ? expf((float)(gi - Gs[col])) * __uint_as_float(g[c + u + e]) : 0.f;
        }
        split2(pv[0], pv[1], ph[u / 2], pl[u / 2]);
      }
      const uint32_t o = swz(i, c0 + c, 8);
      *reinterpret_cast<uint4*>(p_hi + o) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
      *reinterpret_cast<uint4*>(p_lo + o) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
    }
  }
}

// A (F32, strictly lower, beta_i e^{G_i-G_j} k_i.k_j) into As and
// P (lower incl. diagonal, e^{G_i-G_j} q_i.k_j) as hi/lo tiles at p_hi / p_lo.
template <bool GLOBAL>
__device__ __forceinline__ void gram_store(const float (&kk)[4][4], const float (&qk)[4][4],
                                           int warp, int lane, int n, const double* Gs,
                                           const float* bs, float* As, uint8_t* p_hi,
                                           uint8_t* p_lo) {
  const int m0 = (warp >> 1) * 16, nb = (warp & 1) * 32;
  const int r0 = lane >> 2, c0 = 2 * (lane & 3);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int i = m0 + r0 + (e >> 1) * 8;
      float pv[2], av[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int col = nb + j * 8 + c0 + u;
        const bool lower = col <= i && i < n;
        const float decay = lower ? expf((float)(Gs[i] - Gs[col])) : 0.f;
        av[u] = (lower && col < i) ? bs[i] * (decay * kk[j][e + u]) : 0.f;
        pv[u] = lower ? decay * qk[j][e + u] : 0.f;
      }
      *reinterpret_cast<float2*>(As + i * AP + nb + j * 8 + c0) = make_float2(av[0], av[1]);
      uint32_t ph, pl;
      split2(pv[0], pv[1], ph, pl);
      const uint32_t o = swz(i, nb + j * 8 + c0, 8);
      put32<GLOBAL>(p_hi, o, ph);
      put32<GLOBAL>(p_lo, o, pl);
    }
  }
}

// m16n8k16 fragments of F32 tiles in shared memory (leading dimension ld),
// split into hi/lo BF16: A (16 x 16, row-major) and B (16 x 8, element
// (k, n) at base[k * ld + n]); g = lane / 4, t = lane % 4.
__device__ __forceinline__ void frag_a_f32(const float* base, int ld, int lane, uint32_t (&ah)[4],
                                           uint32_t (&al)[4]) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 v = *reinterpret_cast<const float2*>(base + (g + (q & 1) * 8) * ld + 2 * t + (q >> 1) * 8);
    split2(v.x, v.y, ah[q], al[q]);
  }
}
__device__ __forceinline__ void frag_b_f32(const float* base, int ld, int lane, uint32_t (&bh)[2],
                                           uint32_t (&bl)[2]) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int q = 0; q < 2; ++q)
    split2(base[(2 * t + q * 8) * ld + g], base[(2 * t + 1 + q * 8) * ld + g], bh[q], bl[q]);
}
// One n8 accumulator tile (16 x 8) into a shared-memory tile, times `sign`.
__device__ __forceinline__ void store_c(const float (&c)[4], float* base, int ld, int lane, float sign) {
  const int g = lane >> 2, t = lane & 3;
  base[g * ld + 2 * t] = sign * c[0];
  base[g * ld + 2 * t + 1] = sign * c[1];
  base[(g + 8) * ld + 2 * t] = sign * c[2];
  base[(g + 8) * ld + 2 * t + 1] = sign * c[3];
}

// T = (I + A)^{-1} by blocked forward substitution (diagonal blocks in F32,
// off-diagonal blocks as split-BF16 mma.sync products), then
// T diag(beta) split into hi/lo tiles at t_hi / t_lo. Contains block barriers;
// every thread of the CTA calls it.
template <bool GLOBAL>
__device__ __forceinline__ void solve_t(const float* As, float* Ts, float* Ms, const float* bs,
                                        uint8_t* t_hi, uint8_t* t_lo, int tid, int warp, int lane,
                                        int nthreads) {
  // Diagonal 16 x 16 blocks: lane c of warp b solves column c of block b.
  if (warp < 4 && lane < 16) {
    const int b0 = warp * 16, c = lane;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float acc = r == c ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) acc -= As[(b0 + r) * AP + b0 + j] * x[j];
      x[r] = r < c ? 0.f : acc;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) Ts[(b0 + r) * AP + b0 + c] = x[r];
  }
  for (int idx = tid; idx < C * C; idx += nthreads) {  // upper blocks are zero
    const int i = idx >> 6, j = idx & 63;
    if ((j >> 4) > (i >> 4)) Ts[i * AP + j] = 0.f;
  }
  __syncthreads();
  // Off-diagonal blocks, block row by block row, on the tensor cores (split
  // BF16 operands, F32 accumulation): warp 2j + h forms columns [8h, 8h + 8) of
  //   M_bj = sum_{k=j}^{b-1} A_bk T_kj,   T_bj = -T_bb M_bj.
  for (int b = 1; b < 4; ++b) {
    if (warp < 2 * b) {
      const int j = warp >> 1, nt = warp & 1;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int kb = j; kb < b; ++kb) {
        uint32_t ah[4], al[4], bh[2], bl[2];
        frag_a_f32(As + (b * 16) * AP + kb * 16, AP, lane, ah, al);
        frag_b_f32(Ts + (kb * 16) * AP + j * 16 + nt * 8, AP, lane, bh, bl);
        mma3(acc, ah, al, bh[0], bh[1], bl[0], bl[1]);
      }
      // M_bj goes through this warp's scratch tile (C fragment -> B fragment).
      float* Mj = Ms + (j * 16) * 17 + nt * 8;
      store_c(acc, Mj, 17, lane, 1.f);
      __syncwarp();
      float t[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t ah[4], al[4], bh[2], bl[2];
      frag_a_f32(Ts + (b * 16) * AP + b * 16, AP, lane, ah, al);
      frag_b_f32(Mj, 17, lane, bh, bl);
      mma3(t, ah, al, bh[0], bh[1], bl[0], bl[1]);
      store_c(t, Ts + (b * 16) * AP + j * 16 + nt * 8, AP, lane, -1.f);
    }
    __syncthreads();
  }
  for (int idx = tid; idx < C * C / 2; idx += nthreads) {
    const int i = idx >> 5, j = (idx & 31) * 2;
    uint32_t th, tl;
    const float2 tv = *reinterpret_cast<const float2*>(Ts + i * AP + j);
    split2(tv.x * bs[j], tv.y * bs[j + 1], th, tl);
    const uint32_t o = swz(i, j, 8);
    put32<GLOBAL>(t_hi, o, th);
    put32<GLOBAL>(t_lo, o, tl);
  }
}

// Shared-memory addresses of one chunk's operands for the state products.
struct ChunkOps {
  uint32_t kq;  // KHI, KLO, QHI, QLO tiles (16 KB each)
  uint32_t tp;  // THI, TLO, PHI, PLO tiles (8 KB each)
  const float* eg;   // [64] e^{G}
  const float* egd;  // [64] e^{G_last - G}
  const double* G;   // [64] chunk-relative cumulative log-decay
  float el;          // e^{G_last}
};

// One warp's share of a chunk: value rows [16w, 16w+16) of S^T.
//   R^T = V^T - (S^T K^T) diag(e^G);  D^T = R^T (T diag(beta))^T
//   O^T = (S^T Q^T) diag(e^G) + D^T P^T;  S^T <- e^{G_last} S^T + (D^T diag(e^{G_last-G})) K
// Vr holds this thread's V^T fragment (token-major C layout) for the chunk.
__device__ __forceinline__ void carry_step(float (&S)[16][4], const float (&Vr)[8][4],
                                           const ChunkOps& c, int n, int64_t t0, int Hv, int h,
                                           int warp, int lane, float* __restrict__ out, int cap_row,
                                           float* __restrict__ capture_state) {
  const int r0 = lane >> 2, c0 = 2 * (lane & 3);
  const int dv0 = warp * 16;
  float R[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) R[nt][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < DK / 16; ++ks) {
    uint32_t ah[4], al[4];
    acc_to_a(S[2 * ks], S[2 * ks + 1], ah, al);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bh[4], bl[4];
      ldb_kq(c.kq, 0, np * 16, ks * 16, lane, bh);
      ldb_kq(c.kq, 1, np * 16, ks * 16, lane, bl);
      mma3(R[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
      mma3(R[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
    }
  }
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) R[nt][e] = Vr[nt][e] - c.eg[nt * 8 + c0 + (e & 1)] * R[nt][e];
  float D[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) D[nt][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < C / 16; ++ks) {
    uint32_t ah[4], al[4];
    acc_to_a(R[2 * ks], R[2 * ks + 1], ah, al);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bh[4], bl[4];
      ldb_nk(c.tp + 0 * SQ_BYTES, np * 16, ks * 16, 8, lane, bh);
      ldb_nk(c.tp + 1 * SQ_BYTES, np * 16, ks * 16, 8, lane, bl);
      mma3(D[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
      mma3(D[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
    }
  }
  // O^T (R's registers are reused).
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) R[nt][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < DK / 16; ++ks) {
    uint32_t ah[4], al[4];
    acc_to_a(S[2 * ks], S[2 * ks + 1], ah, al);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bh[4], bl[4];
      ldb_kq(c.kq, 2, np * 16, ks * 16, lane, bh);
      ldb_kq(c.kq, 3, np * 16, ks * 16, lane, bl);
      mma3(R[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
      mma3(R[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
    }
  }
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) R[nt][e] *= c.eg[nt * 8 + c0 + (e & 1)];
#pragma unroll
  for (int ks = 0; ks < C / 16; ++ks) {
    uint32_t ah[4], al[4];
    acc_to_a(D[2 * ks], D[2 * ks + 1], ah, al);
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t bh[4], bl[4];
      ldb_nk(c.tp + 2 * SQ_BYTES, np * 16, ks * 16, 8, lane, bh);
      ldb_nk(c.tp + 3 * SQ_BYTES, np * 16, ks * 16, 8, lane, bl);
      mma3(R[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
      mma3(R[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
    }
  }
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = nt * 8 + c0 + (e & 1);
      const int dv = dv0 + r0 + (e >> 1) * 8;
      if (tok < n) out[((t0 + tok) * Hv + h) * DV + dv] = R[nt][e];
    }
  }
  // Capture: S_c^T = e^{G_c} S^T + (D^T diag(e^{G_c - G} [j <= c])) K.
  if (cap_row >= 0) {
    const float ec = expf((float)c.G[cap_row]);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float X[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) X[nt][e] = ec * S[half * 8 + nt][e];
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        float d0[4], d1[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j0 = ks * 16 + c0 + (e & 1), j1 = j0 + 8;
          d0[e] = D[2 * ks][e] * (j0 <= cap_row ? expf((float)(c.G[cap_row] - c.G[j0])) : 0.f);
          d1[e] = D[2 * ks + 1][e] * (j1 <= cap_row ? expf((float)(c.G[cap_row] - c.G[j1])) : 0.f);
        }
        uint32_t ah[4], al[4];
        acc_to_a(d0, d1, ah, al);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t bh[4], bl[4];
          ldb_kq_t(c.kq, 0, half * 64 + np * 16, ks * 16, lane, bh);
          ldb_kq_t(c.kq, 1, half * 64 + np * 16, ks * 16, lane, bl);
          mma3(X[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
          mma3(X[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int dv = dv0 + r0 + (e >> 1) * 8;
          const int dk = (half * 8 + nt) * 8 + c0 + (e & 1);
          capture_state[((int64_t)h * DK + dk) * DV + dv] = X[nt][e];
        }
    }
  }
  // State update.
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) S[nt][e] *= c.el;
#pragma unroll
  for (int ks = 0; ks < C / 16; ++ks) {
    float d0[4], d1[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      d0[e] = D[2 * ks][e] * c.egd[ks * 16 + c0 + (e & 1)];
      d1[e] = D[2 * ks + 1][e] * c.egd[ks * 16 + 8 + c0 + (e & 1)];
    }
    uint32_t ah[4], al[4];
    acc_to_a(d0, d1, ah, al);
#pragma unroll
    for (int np = 0; np < 8; ++np) {
      uint32_t bh[4], bl[4];
      ldb_kq_t(c.kq, 0, np * 16, ks * 16, lane, bh);
      ldb_kq_t(c.kq, 1, np * 16, ks * 16, lane, bl);
      mma3(S[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
      mma3(S[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
    }
  }
}

// This thread's V^T fragment of a chunk (zero past n).
__device__ __forceinline__ void load_v(const float* __restrict__ v, int64_t t0, int n, int Hv, int h,
                                       int warp, int lane, float (&Vr)[8][4]) {
  const int r0 = lane >> 2, c0 = 2 * (lane & 3);
#pragma unroll
  for (int nt = 0; nt < 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = nt * 8 + c0 + (e & 1);
      const int dv = warp * 16 + r0 + (e >> 1) * 8;
      Vr[nt][e] = tok < n ? v[((t0 + tok) * Hv + h) * DV + dv] : 0.f;
    }
}

__device__ __forceinline__ void load_state(float (&S)[16][4], const float* init, int warp, int lane) {
  const int r0 = lane >> 2, c0 = 2 * (lane & 3);
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int dv = warp * 16 + r0 + (e >> 1) * 8;
      const int dk = nt * 8 + c0 + (e & 1);
      S[nt][e] = init ? init[(int64_t)dk * DV + dv] : 0.f;
    }
}

__device__ __forceinline__ void store_state(const float (&S)[16][4], float* dst, int warp, int lane) {
  const int r0 = lane >> 2, c0 = 2 * (lane & 3);
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int dv = warp * 16 + r0 + (e >> 1) * 8;
      const int dk = nt * 8 + c0 + (e & 1);
      dst[(int64_t)dk * DV + dv] = S[nt][e];
    }
}

struct ScanArgs {
  const float* q;  // [T, Hk, 128] normalised, scaled
  const float* k;  // [T, Hk, 128] normalised
  const float* v;  // [T, Hv, 128]
  const float* g;  // [T, Hv]
  const float* beta;
  const int64_t* cu;  // device [nseq + 1] or null (one sequence of T)
  int64_t T;
  int Hk, Hv;
  const float* init;  // [nseq or 1, Hv, 128, 128] or null
  int init_shared;
  int64_t capture;       // tokens before the captured state (0 = none); nseq == 1
  float* capture_state;  // [Hv, 128, 128]
  float* final_state;    // [nseq, Hv, 128, 128] or null
  float* out;            // [T, Hv, 128]
};

__device__ __forceinline__ const float* init_for(const ScanArgs& a, int s, int h) {
  return a.init ? a.init + (a.init_shared ? 0 : (int64_t)s * a.Hv * DK * DV) + (int64_t)h * DK * DV
                : nullptr;
}

// ---------------------------------------------------------------------------
// Fused single-pass kernel: one CTA per (sequence, v-head) does every stage of
// every chunk itself. Needs no workspace beyond the sequence offsets.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS, 1) delta_scan_kernel(ScanArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x % a.Hv;
  const int s = blockIdx.x / a.Hv;
  const int kh = h / (a.Hv / a.Hk);
  const int64_t start = a.cu ? a.cu[s] : 0;
  const int64_t len = a.cu ? a.cu[s + 1] - start : a.T;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(sm);
  float* As = reinterpret_cast<float*>(sm + OFF_A);
  float* Ts = reinterpret_cast<float*>(sm + OFF_T);
  float* Ms = reinterpret_cast<float*>(sm + OFF_M);
  double* Gs = reinterpret_cast<double*>(sm + OFF_G);
  float* eg = reinterpret_cast<float*>(sm + OFF_EG);
  float* egd = reinterpret_cast<float*>(sm + OFF_EGD);
  float* bs = reinterpret_cast<float*>(sm + OFF_BETA);

  float S[16][4];
  load_state(S, init_for(a, s, h), warp, lane);
  const int64_t nchunks = (len + C - 1) / C;
  for (int64_t ci = 0; ci < nchunks; ++ci) {
    const int64_t t0 = start + ci * C;
    const int n = (int)(len - ci * C < C ? len - ci * C : C);
    stage_kq(a.q, a.k, t0, n, a.Hk, kh, sm + OFF_KHI, nullptr, tid, THREADS);
    if (warp == 0) cumsum_gates(a.g, a.beta, t0, n, a.Hv, h, lane, Gs, bs);
    __syncthreads();
    const double Glast = Gs[C - 1];  // padded tokens carry g = 0
    if (tid < C) {
      eg[tid] = expf((float)Gs[tid]);
      egd[tid] = expf((float)(Glast - Gs[tid]));
    }
    {
      float kk[4][4], qk[4][4];
      gram_mma(sbase + OFF_KHI, warp, lane, kk, qk);
      gram_store<false>(kk, qk, warp, lane, n, Gs, bs, As, sm + OFF_PHI, sm + OFF_PLO);
    }
    __syncthreads();
    solve_t<false>(As, Ts, Ms, bs, sm + OFF_THI, sm + OFF_TLO, tid, warp, lane, THREADS);
    __syncthreads();
    int cap_row = -1;
    if (a.capture_state && a.capture > ci * C && a.capture <= ci * C + n)
      cap_row = (int)(a.capture - 1 - ci * C);
    ChunkOps ops;
    ops.kq = sbase + OFF_KHI;
    ops.tp = sbase + OFF_THI;
    ops.eg = eg;
    ops.egd = egd;
    ops.G = Gs;
    ops.el = expf((float)Glast);
    float Vr[8][4];
    load_v(a.v, t0, n, a.Hv, h, warp, lane, Vr);
    carry_step(S, Vr, ops, n, t0, a.Hv, h, warp, lane, a.out, cap_row, a.capture_state);
    __syncthreads();  // the next chunk overwrites the shared tiles
  }
  if (a.final_state) store_state(S, a.final_state + ((int64_t)s * a.Hv + h) * DK * DV, warp, lane);
}

// ---------------------------------------------------------------------------
// Pipelined pair. delta_prep_kernel: one CTA per (chunk, k-head), fully
// parallel: splits K, Q into hi/lo tiles (the [K; Q] tcgen05 operand, also
// written to the workspace as the chunk's K/Q image), forms the Gram products
// once, and for each v-head of the k-head writes T diag(beta), P and the decay
// vectors to the workspace as the chunk's T/P image. delta_carry_tc_kernel
// (below) walks the chunks of each (sequence, v-head); every chunk input is
// independent of the state, so the next chunk's images stream in while the
// tensor core works on the current one.
// ---------------------------------------------------------------------------
struct ScanSeq {
  int32_t chunk0;
  int32_t nchunks;
};
struct ScanChunk {
  int64_t t0;
  int32_t n;
  int32_t seq;
};

constexpr int TP_TILES = 4 * SQ_BYTES;                   // THI, TLO, PHI, PLO
constexpr int VEC_BYTES = 64 * 4 + 64 * 4 + 64 * 4 + 64 * 8;  // eg, egd, el, G
constexpr int TP_IMG = TP_TILES + VEC_BYTES;              // 34048 bytes
constexpr int KQ_IMG = 4 * KQ_BYTES;                      // 65536 bytes

// prep kernel shared layout
// A, T and the staged P tiles reuse the Gram operand's space once the Gram
// products have completed: 72 KB per CTA, three CTAs per SM.
constexpr int P_OFF_KQ = 0;
constexpr int P_OFF_A = 2 * SQ_BYTES;  // after the P hi/lo staging tiles
constexpr int P_OFF_T = P_OFF_A + C * AP * 4;
static_assert(P_OFF_T + C * AP * 4 <= KQ_IMG, "A and T inside the Gram operand's space");
constexpr int P_OFF_M = KQ_IMG;
constexpr int PREP_MAX_REP = 4;  // value heads per key head whose gates are staged at once
constexpr int P_OFF_G = P_OFF_M + 3 * 16 * 17 * 4;
constexpr int P_OFF_B = P_OFF_G + PREP_MAX_REP * C * 8;
constexpr int P_OFF_BAR = P_OFF_B + PREP_MAX_REP * C * 4;  // mbarrier + TMEM address
constexpr int PREP_SMEM = 1024 + P_OFF_BAR + 16;  // 1024: alignment of the swizzled operand

struct PipeArgs {
  ScanArgs a;
  const ScanSeq* seqs;
  const ScanChunk* chunks;
  uint8_t* kq_img;  // [chunks][Hk][KQ_IMG]
  uint8_t* tp_img;  // [chunks][Hv][TP_IMG]
  const int32_t* order;  // [nseq] carry order: longest sequences first
};

__global__ void __launch_bounds__(THREADS, 3) delta_prep_kernel(PipeArgs p) {
  extern __shared__ __align__(128) uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
  const ScanArgs& a = p.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kh = blockIdx.y;
  const int64_t gc = blockIdx.x;
  const ScanChunk ch = p.chunks[gc];
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(sm);
  uint64_t* gram_bar = reinterpret_cast<uint64_t*>(sm + P_OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + P_OFF_BAR + 8);
  if (tid == 0) {
    sm100::mbar_init(gram_bar, 1);
    sm100::fence_barrier_init();
  }
  if (warp == 0) {
    sm100::tmem_alloc(tmem_slot, 64);  // the 128 x 64 F32 Gram accumulator
    sm100::tmem_relinquish();
  }
  float* As = reinterpret_cast<float*>(sm + P_OFF_A);
  float* Ts = reinterpret_cast<float*>(sm + P_OFF_T);
  float* Ms = reinterpret_cast<float*>(sm + P_OFF_M);
  double* Gs0 = reinterpret_cast<double*>(sm + P_OFF_G);
  float* bs0 = reinterpret_cast<float*>(sm + P_OFF_B);
  double* Gs = Gs0;
  float* bs = bs0;
  uint8_t* kq = p.kq_img + (gc * a.Hk + kh) * (int64_t)KQ_IMG;
  const int rep = a.Hv / a.Hk;
  // The gates of up to PREP_MAX_REP value heads are summed by one warp each
  // while the other warps stage K and Q.
  const int staged = rep <= PREP_MAX_REP ? rep : 0;
  if (warp >= 8 - staged) {
    const int r = warp - (8 - staged);
    cumsum_gates(a.g, a.beta, ch.t0, ch.n, a.Hv, kh * rep + r, lane, Gs + r * C, bs + r * C);
  }
  stage_kq(a.q, a.k, ch.t0, ch.n, a.Hk, kh, sm + P_OFF_KQ, kq, tid, THREADS, true);
  // The operand written by st.shared is read by the tensor core (async proxy).
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) gram_tc_issue(sbase + P_OFF_KQ, tmem, gram_bar);
  // Warp w reads TMEM lanes 32 (w % 4) .. (rows of [K K^T; Q K^T]) and columns
  // 32 (w / 4) .. of the Gram; the wait ends warp-uniformly.
  const int grow = (warp & 3) * 32 + lane, ghalf = warp >> 2;
  uint32_t gr[32];
  const bool gram_ok = __all_sync(0xffffffffu, sm100::mbar_wait(gram_bar, 0));
  if (gram_ok) {
    sm100::tc_fence_after();
    sm100::tmem_ld_32x32b_x32(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(ghalf * 32), gr);
    sm100::tmem_ld_wait();
  } else {
    if (lane == 0) raise_device_error(kDevScanTimeout);
#pragma unroll
    for (int c = 0; c < 32; ++c) gr[c] = 0u;
  }
  for (int r = 0; r < rep; ++r) {
    const int h = kh * rep + r;
    uint8_t* tp = p.tp_img + (gc * a.Hv + h) * (int64_t)TP_IMG;
    double* Gs = Gs0 + (staged ? r * C : 0);
    float* bs = bs0 + (staged ? r * C : 0);
    if (!staged && warp == 0) cumsum_gates(a.g, a.beta, ch.t0, ch.n, a.Hv, h, lane, Gs, bs);
    __syncthreads();
    const double Glast = Gs[C - 1];
    if (tid < C) {
      float* vec = reinterpret_cast<float*>(tp + TP_TILES);
      vec[tid] = expf((float)Gs[tid]);                   // eg
      vec[64 + tid] = expf((float)(Glast - Gs[tid]));    // egd
      vec[128 + tid] = tid == 0 ? expf((float)Glast) : 0.f;  // el
      reinterpret_cast<double*>(vec + 192)[tid] = Gs[tid];   // G
    }
    // P goes through shared memory (the Gram operand's space, free once the
    // MMAs have completed) so that its image is written with coalesced stores.
    uint8_t* pst = sm + P_OFF_KQ;
    gram_store_rows<false>(gr, grow, ghalf, ch.n, Gs, bs, As, pst, pst + SQ_BYTES);
    __syncthreads();
    for (int o = tid * 16; o < 2 * SQ_BYTES; o += THREADS * 16)
      *reinterpret_cast<uint4*>(tp + 2 * SQ_BYTES + o) = *reinterpret_cast<const uint4*>(pst + o);
    solve_t<true>(As, Ts, Ms, bs, tp + 0 * SQ_BYTES, tp + 1 * SQ_BYTES, tid, warp, lane, THREADS);
    __syncthreads();  // Gs, bs, As, Ts are reused by the next v-head
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 64);
  }
}

}  // namespace

int scan_device_error(int* code) { return read_device_error(code); }

namespace {

// ---------------------------------------------------------------------------
// delta_carry_tc_kernel: the state carry on the tcgen05 tensor core.
//
// The chunk algebra of carry_step (three-term split-BF16 products with F32
// accumulation), with every product accumulated in TMEM and its BF16 A
// operands written back into TMEM, so no state tile goes through shared
// memory. The state S^T itself (row dv = TMEM lane) lives in TMEM in F32 and is
// the accumulator of the state update. Persistent: CTA b carries (sequence,
// v-head) pairs b, b + grid, ... of the longest-first order; each chunk's K/Q
// and T/P images stream into one of two shared-memory stages by bulk copies.
//
// Warps 0..7 are the epilogue: warp w reads TMEM lane quarter w % 4 and takes
// half hf = w / 4 of the columns, so thread (w, lane) owns value row
// dv = 32 (w % 4) + lane, dk columns [64 hf, 64 hf + 64) of S^T and tokens
// [32 hf, 32 hf + 32) of every chunk. Warp 8 lane 0 issues the MMAs, warp 9
// lane 0 the bulk copies.
//
// TMEM columns (512, one CTA per SM):
//   [0, 128)    S^T (F32)
//   [128, 256)  S^T split: hi [128, 192), lo [192, 256)
//   [256, 320)  R^T = S^T K^T, then X_R (R split in place), then X_D' (split
//               D^T diag(egd))
//   [320, 384)  O1 = S^T Q^T (one N = 128 product with R)
//   [384, 448)  D^T = X_R (T diag beta)^T, then X_D (D split in place)
//   [448, 512)  O2 = X_D P^T (a capture chunk first holds X_D'' there)
// Token-indexed operands (X_R, X_D, X_D', X_D''): warp half hf writes its 32
// tokens as 16 hi words then 16 lo words in columns [base + 32 hf, +32), so a
// warp only rewrites columns it has read; K step t (tokens 16t .. 16t + 15)
// starts at column base + 32 (t / 2) + 8 (t % 2), +16 for lo.
// Per chunk k (E = epilogue warps, M = MMA issuer):
//   E a   O1 of chunk k - 1 out; split S^T -> [128, 256);
//         S^T <- e^{G_last} S^T ahead of its update         -> a_bar
//   M     [R | O1] = S^T [K; Q]^T                           -> r_bar
//   E c   R <- V^T - R diag(e^G); split in place            -> c_bar
//   M     D = X_R (T diag beta)^T                           -> d_bar
//   E g   outputs of chunk k - 1 (O1 read in step a)       -> stage k - 1 free
//   E e   X_D' = split D diag(egd); split D in place        -> e_bar
//   M     S^T += X_D' K -> i_bar; O2 = X_D P^T -> f_bar, stage k free
// ---------------------------------------------------------------------------
constexpr int TC_STAGE = 100352;  // one chunk's K/Q and T/P images, 1024-aligned
constexpr int TC_THREADS = 320;
constexpr int TC_OFF_BAR = 2 * TC_STAGE;
constexpr int TC_SMEM = 1024 + TC_OFF_BAR + 17 * 8;
static_assert(KQ_IMG + TP_IMG <= TC_STAGE && TC_STAGE % 1024 == 0, "carry stage layout");
constexpr uint32_t TC_S = 0, TC_SA = 128, TC_R = 256, TC_O1 = 320, TC_D = 384, TC_O2 = 448;

// x = hi + lo with hi = bf16(x), lo = bf16(x - hi), two values per word (even
// index in the low half): the same values as split2.
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(x0, x1);
  lo = pack_bf16x2(x0 - __uint_as_float(hi << 16), x1 - __uint_as_float(hi & 0xffff0000u));
}

// Three-term product into TMEM: d (+)= A * B^T with A split in TMEM (column of
// K step t from a_col(lo, t), 8 columns per 16-wide step) and B split in
// shared memory (descriptor from b_desc(lo, t)); the small terms go first.
template <int KSTEPS, typename ACol, typename BDesc>
__device__ __forceinline__ void tc_mma3(uint32_t d, ACol a_col, uint32_t idesc, BDesc b_desc, bool accumulate) {
  uint32_t acc = accumulate ? 1u : 0u;
#pragma unroll
  for (int term = 0; term < 3; ++term) {
#pragma unroll
    for (int t = 0; t < KSTEPS; ++t) {
      // lo*hi, hi*lo, hi*hi
      sm100::umma_f16_ts(d, a_col(term == 0, t), b_desc(term == 1, t), idesc, acc);
      acc = 1;
    }
  }
}

// Column of K step t of a token-indexed operand at TMEM address `base`.
__device__ __forceinline__ uint32_t tok_col(uint32_t base, bool lo, int t) {
  return base + 32 * (t >> 1) + 8 * (t & 1) + (lo ? 16 : 0);
}

__global__ void __launch_bounds__(TC_THREADS, 1) delta_carry_tc_kernel(PipeArgs p, int npairs) {
  using namespace sm100;
  extern __shared__ __align__(128) uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)sm_raw + 1023) & ~(uintptr_t)1023);
  const ScanArgs& a = p.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + TC_OFF_BAR);
  uint64_t* full = bar + 0;    // [2] stage loaded
  uint64_t* empty = bar + 2;   // [2] stage consumed (MMA commit + 8 epilogue warps)
  uint64_t* a_bar = bar + 4;
  uint64_t* r_bar = bar + 5;
  uint64_t* c_bar = bar + 6;
  uint64_t* d_bar = bar + 7;
  uint64_t* e_bar = bar + 8;
  uint64_t* f_bar = bar + 9;
  uint64_t* i_bar = bar + 10;
  uint64_t* drain = bar + 11;     // error path: completion of this CTA's own MMAs
  uint64_t* cap_bar = bar + 12;   // capture chunk: captured-state product done
  uint64_t* capd_bar = bar + 13;  // capture chunk: captured state read by the 8 warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + 15);
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 9);
    }
    mbar_init(a_bar, 8);
    mbar_init(r_bar, 1);
    mbar_init(c_bar, 8);
    mbar_init(d_bar, 1);
    mbar_init(e_bar, 8);
    mbar_init(f_bar, 1);
    mbar_init(i_bar, 1);
    mbar_init(drain, 1);
    mbar_init(cap_bar, 1);
    mbar_init(capd_bar, 8);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);
  // A bounded wait; the first one to time out stops the whole CTA.
  auto wait = [&](uint64_t* b, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait(b, parity)) return true;
    *abort_flag = 1;
    raise_device_error(kDevScanTimeout);
    return false;
  };
  const int rep = a.Hv / a.Hk;
  // Capture inside chunk c (single sequence, so the chunk starts at token
  // c.t0 of it): the row of the last token before the capture, else -1.
  auto cap_row_of = [&](const ScanChunk& c) -> int {
    return (a.capture_state && a.capture > c.t0 && a.capture <= c.t0 + c.n) ? (int)(a.capture - 1 - c.t0) : -1;
  };

  if (warp == 9) {
    if (lane == 0) {
      int k = 0, last[2] = {-1, -1};
      bool ok = true;
      for (int item = blockIdx.x; item < npairs && ok; item += gridDim.x) {
        const int s = p.order[item / a.Hv], h = item % a.Hv;
        const ScanSeq sq = p.seqs[s];
        for (int ci = 0; ci < sq.nchunks; ++ci, ++k) {
          const int st = k & 1;
          if (k >= 2 && !(ok = wait(&empty[st], ((k >> 1) - 1) & 1))) break;
          const int64_t gc = sq.chunk0 + ci;
          uint8_t* dst = sm + st * TC_STAGE;
          mbar_expect_tx(&full[st], KQ_IMG + TP_IMG);
          bulk_load(dst, p.kq_img + (gc * a.Hk + h / rep) * (int64_t)KQ_IMG, KQ_IMG, &full[st]);
          bulk_load(dst + KQ_IMG, p.tp_img + (gc * a.Hv + h) * (int64_t)TP_IMG, TP_IMG, &full[st]);
          last[st] = k;
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA exits (bounded).
        for (int i = 0; i < 2; ++i)
          if (last[i] >= 0) mbar_wait(&full[i], (last[i] >> 1) & 1);
      }
    }
  } else if (warp == 8) {
    if (lane == 0) {
      constexpr uint32_t id64 = idesc_bf16_f32(128, 64);
      constexpr uint32_t id128 = idesc_bf16_f32(128, 128);
      constexpr uint32_t id128mn = idesc_bf16_f32_bmn(128, 128);
      auto sa = [&](bool lo, int t) { return tmem + TC_SA + (lo ? 64 : 0) + 8 * t; };
      int k = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < npairs && ok; item += gridDim.x) {
        const ScanSeq sq = p.seqs[p.order[item / a.Hv]];
        for (int ci = 0; ci < sq.nchunks; ++ci, ++k) {
          const int st = k & 1;
          const uint32_t kq = sbase + st * TC_STAGE, tp = kq + KQ_IMG;
          const int cap_row = cap_row_of(p.chunks[sq.chunk0 + ci]);
          // The [K; Q] image (128 rows) as the B operand of [R | O1] = S^T [K; Q]^T.
          auto kq_desc = [=](bool lo, int t) {
            return desc_k_sw128(kq + (lo ? GRAM_TILE : 0) + (t >> 2) * (128 * 128) + (t & 3) * 32);
          };
          // K read MN-major for the state update: rows are tokens, 64-wide dk atoms 16 KB apart.
          auto k_mn = [=](bool lo, int t) {
            return desc_mn_sw128(kq + (lo ? GRAM_TILE : 0) + t * (16 * 128), 128 * 128, 1024);
          };
          if (!(ok = wait(&full[st], (k >> 1) & 1) && wait(a_bar, k & 1))) break;
          tc_fence_after();
          tc_mma3<8>(tmem + TC_R, sa, id128, kq_desc, false);
          umma_commit(r_bar);
          // D overwrites the columns O2 of the previous chunk read (X_D).
          if (!(ok = wait(c_bar, k & 1) && (k == 0 || wait(f_bar, (k - 1) & 1)))) break;
          tc_fence_after();
          tc_mma3<4>(tmem + TC_D, [&](bool lo, int t) { return tok_col(tmem + TC_R, lo, t); }, id64,
                     [&](bool lo, int t) { return desc_k_sw128(tp + (lo ? SQ_BYTES : 0) + t * 32); }, false);
          umma_commit(d_bar);
          if (!(ok = wait(e_bar, k & 1))) break;
          tc_fence_after();
          if (cap_row >= 0) {
            // The captured state first (into S^T, which holds e^{G_c} S^T);
            // the carried update once the warps have read it and restored S^T.
            tc_mma3<4>(tmem + TC_S, [&](bool lo, int t) { return tok_col(tmem + TC_O2, lo, t); }, id128mn, k_mn,
                       true);
            umma_commit(cap_bar);
            if (!(ok = wait(capd_bar, 0))) break;
            tc_fence_after();
          }
          tc_mma3<4>(tmem + TC_S, [&](bool lo, int t) { return tok_col(tmem + TC_R, lo, t); }, id128mn, k_mn, true);
          umma_commit(i_bar);
          tc_mma3<4>(tmem + TC_O2, [&](bool lo, int t) { return tok_col(tmem + TC_D, lo, t); }, id64,
                     [&](bool lo, int t) { return desc_k_sw128(tp + (lo ? 3 : 2) * SQ_BYTES + t * 32); }, false);
          umma_commit(f_bar);
          umma_commit(&empty[st]);
        }
      }
      if (!ok) {
        // Wait (bounded) for the MMAs already issued before TMEM is released.
        umma_commit(drain);
        mbar_wait(drain, 0);
      }
    }
  } else {
    const int q = warp & 3, hf = warp >> 2;
    const int row = q * 32 + lane;  // dv
    const uint32_t lq = tmem + ((uint32_t)(q * 32) << 16);
    const int64_t tstride = (int64_t)a.Hv * DV;  // floats between tokens of v and out
    // Waits end warp-uniformly: the TMEM accesses after them are .sync.aligned.
    auto wait_all = [&](uint64_t* b, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, wait(b, parity));
    };
    auto arrive = [&](uint64_t* b) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(b);
    };
    // This thread's 32 token values val(0..31) of a token-indexed operand, split.
    auto put_tok = [&](uint32_t col, auto val) {
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) split_pair(val(2 * j), val(2 * j + 1), hi[j], lo[j]);
      tmem_st_32x32b_x16(lq + col + 32 * hf, hi);
      tmem_st_32x32b_x16(lq + col + 32 * hf + 16, lo);
    };
    // 32 dk columns of S^T (F32 bits) split into the state operand.
    auto put_sa = [&](int half, const uint32_t (&x)[32]) {
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        split_pair(__uint_as_float(x[2 * j]), __uint_as_float(x[2 * j + 1]), hi[j], lo[j]);
      tmem_st_32x32b_x16(lq + TC_SA + 32 * hf + 16 * half, hi);
      tmem_st_32x32b_x16(lq + TC_SA + 64 + 32 * hf + 16 * half, lo);
    };
    // This thread's O1 = S^T Q^T of the chunk in stage stc, times e^G.
    auto read_o1 = [&](int stc, float (&o1s)[32]) {
      uint32_t y[32];
      tmem_ld_32x32b_x32(lq + TC_O1 + 32 * hf, y);
      tmem_ld_wait();
      const float* eg = reinterpret_cast<const float*>(sm + stc * TC_STAGE + KQ_IMG + TP_TILES) + 32 * hf;
#pragma unroll
      for (int i = 0; i < 32; ++i) o1s[i] = eg[i] * __uint_as_float(y[i]);
    };
    // g: O^T = (S^T Q^T) diag(e^G) + D^T P^T of chunk c (CTA chunk kc, stage
    // stc), the first term read earlier into o1s.
    auto do_g = [&](const ScanChunk& c, int stc, int kc, int h, const float (&o1s)[32]) -> bool {
      if (!wait_all(f_bar, kc & 1)) return false;
      tc_fence_after();
      uint32_t o2[32];
      tmem_ld_32x32b_x32(lq + TC_O2 + 32 * hf, o2);
      tmem_ld_wait();
      const int nmine = c.n - 32 * hf;
      float* op = a.out + ((c.t0 + 32 * hf) * a.Hv + h) * DV + row;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nmine) op[i * tstride] = o1s[i] + __uint_as_float(o2[i]);
      arrive(&empty[stc]);
      return true;
    };
    int k = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < npairs && ok; item += gridDim.x) {
      const int s = p.order[item / a.Hv], h = item % a.Hv;
      const ScanSeq sq = p.seqs[s];
      ScanChunk prev;  // the chunk whose output step is still to do
      int st_prev = 0;
      for (int ci = 0; ci < sq.nchunks; ++ci, ++k) {
        const int st = k & 1;
        const ScanChunk ch = p.chunks[sq.chunk0 + ci];
        const int cap_row = cap_row_of(ch);
        // a: S^T of this chunk (the initial state at the first chunk), split,
        // and S^T <- e^{G_last} S^T ahead of its update (a capture chunk keeps
        // S^T unscaled until step e). Before it, O1 of the previous chunk is
        // taken out of its columns, which the next product overwrites.
        if (!(ok = wait_all(&full[st], (k >> 1) & 1))) break;
        const float* vec = reinterpret_cast<const float*>(sm + st * TC_STAGE + KQ_IMG + TP_TILES);
        float o1s[32];
        const float* init = ci == 0 ? init_for(a, s, h) : nullptr;
        if (ci > 0) {
          if (!(ok = wait_all(i_bar, (k - 1) & 1))) break;
          tc_fence_after();
          read_o1(st_prev, o1s);
        }
        const float f = cap_row < 0 ? vec[128] : 1.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t x[32];
          if (ci == 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              x[j] = init ? __float_as_uint(init[(int64_t)(64 * hf + 32 * half + j) * DV + row]) : 0u;
          } else {
            tmem_ld_32x32b_x32(lq + TC_S + 64 * hf + 32 * half, x);
            tmem_ld_wait();
          }
          put_sa(half, x);
          if (cap_row < 0 || ci == 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) x[j] = __float_as_uint(f * __uint_as_float(x[j]));
            tmem_st_32x32b_x32(lq + TC_S + 64 * hf + 32 * half, x);
          }
        }
        tmem_st_wait();
        arrive(a_bar);
        // This chunk's V^T row (tokens [32 hf, 32 hf + 32)), in flight during
        // the [R | O1] product.
        const int nmine = ch.n - 32 * hf;  // valid tokens of this half
        float vr[32];
        {
          const float* vp = a.v + ((ch.t0 + 32 * hf) * a.Hv + h) * DV + row;
#pragma unroll
          for (int i = 0; i < 32; ++i) vr[i] = i < nmine ? vp[i * tstride] : 0.f;
        }
        // c: R^T = V^T - (S^T K^T) diag(e^G), split in place.
        if (!(ok = wait_all(r_bar, k & 1))) break;
        tc_fence_after();
        {
          uint32_t x[32];
          tmem_ld_32x32b_x32(lq + TC_R + 32 * hf, x);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) vr[i] -= vec[32 * hf + i] * __uint_as_float(x[i]);
          put_tok(TC_R, [&](int i) { return vr[i]; });
          tmem_st_wait();
        }
        arrive(c_bar);
        // The previous chunk's outputs while the D product runs.
        if (ci > 0 && !(ok = do_g(prev, st_prev, k - 1, h, o1s))) break;
        // e: D^T diag(egd) split into the R columns (free since the D product
        // read X_R), then D^T split in place.
        if (!(ok = wait_all(d_bar, k & 1))) break;
        tc_fence_after();
        {
          uint32_t x[32];
          tmem_ld_32x32b_x32(lq + TC_D + 32 * hf, x);
          tmem_ld_wait();
          put_tok(TC_R, [&](int i) { return __uint_as_float(x[i]) * vec[64 + 32 * hf + i]; });
          if (cap_row >= 0) {
            // X_D'' = split D^T diag(e^{G_c - G_j} [j <= c]) into the O2
            // columns (the previous chunk's O2 is read, this chunk's not formed).
            const double* G = reinterpret_cast<const double*>(vec + 192);
            const double gc = G[cap_row];
            put_tok(TC_O2, [&](int i) {
              const int j = 32 * hf + i;
              return j <= cap_row ? __uint_as_float(x[i]) * expf((float)(gc - G[j])) : 0.f;
            });
          }
          put_tok(TC_D, [&](int i) { return __uint_as_float(x[i]); });
        }
        const float el = vec[128];
        if (cap_row < 0) {
          tmem_st_wait();
          arrive(e_bar);
        } else {
          // S_c = e^{G_c} S^T + X_D''^T K is formed in the S^T columns, read
          // out, and S^T <- e^{G_last} S^T restored for the carried update,
          // so the carried state does not depend on whether a capture was
          // asked for.
          // This thread's entries of S^T wait in its own entries of the
          // capture buffer meanwhile.
          const float ec = expf((float)reinterpret_cast<const double*>(vec + 192)[cap_row]);
          float* dst = a.capture_state + (int64_t)h * DK * DV;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t x[32];
            tmem_ld_32x32b_x32(lq + TC_S + 64 * hf + 32 * half, x);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              dst[(int64_t)(64 * hf + 32 * half + j) * DV + row] = __uint_as_float(x[j]);
              x[j] = __float_as_uint(ec * __uint_as_float(x[j]));
            }
            tmem_st_32x32b_x32(lq + TC_S + 64 * hf + 32 * half, x);
          }
          tmem_st_wait();
          arrive(e_bar);
          if (!(ok = wait_all(cap_bar, 0))) break;
          tc_fence_after();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t x[32], y[32];
            tmem_ld_32x32b_x32(lq + TC_S + 64 * hf + 32 * half, x);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float* e = dst + (int64_t)(64 * hf + 32 * half + j) * DV + row;
              y[j] = __float_as_uint(el * *e);
              *e = __uint_as_float(x[j]);
            }
            tmem_st_32x32b_x32(lq + TC_S + 64 * hf + 32 * half, y);
          }
          tmem_st_wait();
          arrive(capd_bar);
        }
        prev = ch;
        st_prev = st;
      }
      if (!ok) break;
      // Final state (S^T after the last chunk's update), then the last
      // chunk's output step.
      if (!(ok = wait_all(i_bar, (k - 1) & 1))) break;
      tc_fence_after();
      if (a.final_state) {
        float* dst = a.final_state + ((int64_t)s * a.Hv + h) * DK * DV;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t x[32];
          tmem_ld_32x32b_x32(lq + TC_S + 64 * hf + 32 * half, x);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) dst[(int64_t)(64 * hf + 32 * half + j) * DV + row] = __uint_as_float(x[j]);
        }
      }
      float o1s[32];
      read_o1(st_prev, o1s);
      if (!(ok = do_g(prev, st_prev, k - 1, h, o1s))) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// Fused-path workspace: the per-sequence token offsets (nseq + 1 int64).
size_t delta_scan_fused_workspace(int nseq) {
  return ((size_t)(nseq + 1) * sizeof(int64_t) + 255) & ~(size_t)255;
}

namespace {
size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }
struct PipeLayout {
  size_t seq_off, chunk_off, order_off, kq_off, tp_off, total;
  int64_t max_chunks;
};
PipeLayout pipe_layout(int64_t total_tokens, int nseq, int Hk, int Hv) {
  PipeLayout l;
  l.max_chunks = (total_tokens + C - 1) / C + nseq;
  l.seq_off = 0;
  l.chunk_off = al256(sizeof(ScanSeq) * (size_t)nseq);
  l.order_off = al256(l.chunk_off + sizeof(ScanChunk) * (size_t)l.max_chunks);
  l.kq_off = al256(l.order_off + sizeof(int32_t) * (size_t)nseq);
  l.tp_off = al256(l.kq_off + (size_t)KQ_IMG * l.max_chunks * Hk);
  l.total = al256(l.tp_off + (size_t)TP_IMG * l.max_chunks * Hv);
  return l;
}
bool g_attr_set[64] = {false};
int set_attrs() {
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !g_attr_set[dev]) {
    CLEF_CUDA(cudaFuncSetAttribute(delta_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    CLEF_CUDA(cudaFuncSetAttribute(delta_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   PREP_SMEM));
    CLEF_CUDA(cudaFuncSetAttribute(delta_carry_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   TC_SMEM));
    g_attr_set[dev] = true;
  }
  return CLEF_OK;
}
}  // namespace

size_t delta_scan_workspace(int64_t total_tokens, int nseq, int Hk, int Hv) {
  return pipe_layout(total_tokens, nseq, Hk, Hv).total;
}

int delta_scan_plan(const int64_t* cu_host, int nseq, int Hk, int Hv, void* ws, size_t ws_bytes,
                    cudaStream_t s, ScanPlan* plan) {
  const int64_t total = cu_host[nseq];
  const PipeLayout l = pipe_layout(total, nseq, Hk, Hv);
  CLEF_CHECK(ws && ws_bytes >= l.total, CLEF_ERR_INVALID, "delta_scan: workspace too small");
  CLEF_CHECK(((uintptr_t)ws & 255) == 0, CLEF_ERR_INVALID, "delta_scan: workspace alignment");
  std::vector<ScanSeq> seqs(nseq);
  std::vector<ScanChunk> chunks;
  chunks.reserve((size_t)l.max_chunks);
  for (int si = 0; si < nseq; ++si) {
    seqs[si].chunk0 = (int32_t)chunks.size();
    for (int64_t t = cu_host[si]; t < cu_host[si + 1]; t += C)
      chunks.push_back({t, (int32_t)std::min<int64_t>(C, cu_host[si + 1] - t), si});
    seqs[si].nchunks = (int32_t)chunks.size() - seqs[si].chunk0;
  }
  char* base = reinterpret_cast<char*>(ws);
  CLEF_CUDA(cudaMemcpyAsync(base + l.seq_off, seqs.data(), sizeof(ScanSeq) * seqs.size(),
                            cudaMemcpyHostToDevice, s));
  CLEF_CUDA(cudaMemcpyAsync(base + l.chunk_off, chunks.data(), sizeof(ScanChunk) * chunks.size(),
                            cudaMemcpyHostToDevice, s));
  std::vector<int32_t> order(nseq);
  for (int si = 0; si < nseq; ++si) order[si] = si;
  std::stable_sort(order.begin(), order.end(),
                   [&](int32_t x, int32_t y) { return seqs[x].nchunks > seqs[y].nchunks; });
  CLEF_CUDA(cudaMemcpyAsync(base + l.order_off, order.data(), sizeof(int32_t) * order.size(),
                            cudaMemcpyHostToDevice, s));
  plan->ws = ws;
  plan->nseq = nseq;
  plan->nchunks = (int64_t)chunks.size();
  plan->total = total;
  plan->Hk = Hk;
  plan->Hv = Hv;
  return CLEF_OK;
}

int launch_delta_scan_planned(const ScanPlan& plan, const float* q, const float* k, const float* v,
                              const float* g, const float* beta, const float* init, int init_shared,
                              int64_t capture, float* capture_state, float* final_state, float* out,
                              cudaStream_t s) {
  RC_(set_attrs());
  const PipeLayout l = pipe_layout(plan.total, plan.nseq, plan.Hk, plan.Hv);
  char* base = reinterpret_cast<char*>(plan.ws);
  PipeArgs p;
  p.a.q = q;
  p.a.k = k;
  p.a.v = v;
  p.a.g = g;
  p.a.beta = beta;
  p.a.cu = nullptr;
  p.a.T = plan.total;
  p.a.Hk = plan.Hk;
  p.a.Hv = plan.Hv;
  p.a.init = init;
  p.a.init_shared = init_shared;
  p.a.capture = capture;
  p.a.capture_state = capture_state;
  p.a.final_state = final_state;
  p.a.out = out;
  p.seqs = reinterpret_cast<const ScanSeq*>(base + l.seq_off);
  p.chunks = reinterpret_cast<const ScanChunk*>(base + l.chunk_off);
  p.kq_img = reinterpret_cast<uint8_t*>(base + l.kq_off);
  p.tp_img = reinterpret_cast<uint8_t*>(base + l.tp_off);
  p.order = reinterpret_cast<const int32_t*>(base + l.order_off);
  delta_prep_kernel<<<dim3((unsigned)plan.nchunks, (unsigned)plan.Hk), THREADS, PREP_SMEM, s>>>(p);
  RC_(launch_status("delta_prep"));
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  const int64_t pairs = (int64_t)plan.nseq * plan.Hv;
  // Persistent tcgen05 carry: one CTA per SM at most.
  const int grid = (int)std::min<int64_t>(pairs, persistent_ctas(dev));
  delta_carry_tc_kernel<<<grid, TC_THREADS, TC_SMEM, s>>>(p, (int)pairs);
  return launch_status("delta_carry_tc");
}

// Fused single-pass path with the offsets already on the device (null = one
// sequence of `total`).
int launch_delta_scan_dev(const float* q, const float* k, const float* v, const float* g,
                          const float* beta, const int64_t* cu_dev, int64_t total, int nseq, int Hk,
                          int Hv, const float* init, int init_shared, int64_t capture,
                          float* capture_state, float* final_state, float* out, cudaStream_t s) {
  RC_(set_attrs());
  ScanArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.g = g;
  a.beta = beta;
  a.cu = cu_dev;
  a.T = total;
  a.Hk = Hk;
  a.Hv = Hv;
  a.init = init;
  a.init_shared = init_shared;
  a.capture = capture;
  a.capture_state = capture_state;
  a.final_state = final_state;
  a.out = out;
  delta_scan_kernel<<<(unsigned)(nseq * Hv), THREADS, SMEM, s>>>(a);
  return launch_status("delta_scan");
}

int launch_delta_scan(const float* q, const float* k, const float* v, const float* g,
                      const float* beta, const int64_t* cu_host, int nseq, int Hk, int Hv, int dk,
                      int dv, const float* init, int init_shared, int64_t capture,
                      float* capture_state, float* final_state, float* out, void* ws,
                      size_t ws_bytes, cudaStream_t s) {
  CLEF_CHECK(dk == DK && dv == DV, CLEF_ERR_UNSUPPORTED, "delta_scan: dk and dv must be 128");
  ScanPlan plan;
  RC_(delta_scan_plan(cu_host, nseq, Hk, Hv, ws, ws_bytes, s, &plan));
  return launch_delta_scan_planned(plan, q, k, v, g, beta, init, init_shared, capture,
                                   capture_state, final_state, out, s);
}

// ---------------------------------------------------------------------------

// ---------------------------------------------------------------------------
// Allocation-free variant of clef_delta_scan.
//
// Some callers cannot call cudaMalloc or hand this library a workspace: hosts
// whose allocator owns every byte of device memory and whose op signature has
// no room for an extra buffer (a Candle/cudarc custom op gets its inputs and
// outputs and nothing else), and latency-critical serving loops that must not
// hit cudaMalloc's implicit device synchronisation. For them the per-sequence
// offsets table, the only scratch the scan needs, lives in a fixed
// device-resident array of this library instead of a caller workspace.
// ---------------------------------------------------------------------------
constexpr int kNoAllocMaxSeqs = 4096;  // 4097 int64 offsets = 32,776 bytes per device

// Loaded with the library on every device that uses it and kept until the
// process exits. In host code this name is only a stand-in for the device
// array: the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) int64_t g_noalloc_offsets[kNoAllocMaxSeqs + 1];

namespace {
// Device address of g_noalloc_offsets, resolved once per device with that
// device current (the first call on a device does this set-up). std::call_once
// makes concurrent first calls from several host threads on one device wait
// for a single lookup; a failed lookup is remembered and reported by every
// later call on that device.
constexpr int kNoAllocMaxDevices = 64;
int noalloc_offsets_ptr(int64_t** out) {
  static std::once_flag once[kNoAllocMaxDevices];
  static int64_t* ptrs[kNoAllocMaxDevices] = {nullptr};
  static cudaError_t errs[kNoAllocMaxDevices] = {};
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  CLEF_CHECK(dev >= 0 && dev < kNoAllocMaxDevices, CLEF_ERR_UNSUPPORTED,
             "delta_scan_noalloc: device index >= 64");
  std::call_once(once[dev], [dev] {
    void* p = nullptr;
    errs[dev] = cudaGetSymbolAddress(&p, g_noalloc_offsets);
    if (errs[dev] == cudaSuccess && !p) errs[dev] = cudaErrorInvalidSymbol;
    if (errs[dev] == cudaSuccess) ptrs[dev] = reinterpret_cast<int64_t*>(p);
  });
  if (errs[dev] != cudaSuccess)
    return fail(CLEF_ERR_CUDA, std::string("delta_scan_noalloc: cudaGetSymbolAddress: ") +
                                   cudaGetErrorString(errs[dev]));
  *out = ptrs[dev];
  return CLEF_OK;
}
}  // namespace

}  // namespace clef

using namespace clef;

extern "C" {

size_t clef_delta_scan_workspace_size(int64_t total_tokens, int32_t nseq, int32_t Hk, int32_t Hv,
                                      int32_t dk, int32_t dv) {
  if (total_tokens < 0 || nseq <= 0 || Hk <= 0 || Hv <= 0 || dk != 128 || dv != 128) return 0;
  return delta_scan_workspace(total_tokens, nseq, Hk, Hv);
}

int clef_delta_scan(const float* q, const float* k, const float* v, const float* g,
                    const float* beta, int64_t T, int32_t Hk, int32_t Hv, int32_t dk, int32_t dv,
                    const int64_t* cu_seqlens, int32_t nseq, const float* init_state,
                    int32_t init_shared, int64_t capture, float* capture_state, float* final_state,
                    float* out, void* workspace, size_t workspace_bytes, void* stream) {
  CLEF_CHECK(q && k && v && g && beta && out, CLEF_ERR_INVALID, "delta_scan: null pointer");
  CLEF_CHECK(dk == 128 && dv == 128, CLEF_ERR_UNSUPPORTED, "delta_scan: dk and dv must be 128");
  CLEF_CHECK(Hk > 0 && Hv > 0 && Hv % Hk == 0 && Hv <= 4096, CLEF_ERR_INVALID,
             "delta_scan: head counts");
  CLEF_CHECK(T > 0, CLEF_ERR_INVALID, "delta_scan: T must be positive");
  std::vector<int64_t> cu;
  if (cu_seqlens) {
    CLEF_CHECK(nseq > 0, CLEF_ERR_INVALID, "delta_scan: nseq");
    cu.assign(cu_seqlens, cu_seqlens + nseq + 1);
    CLEF_CHECK(cu[0] == 0 && cu[nseq] == T, CLEF_ERR_INVALID, "delta_scan: cu_seqlens range");
    for (int i = 0; i < nseq; ++i)
      CLEF_CHECK(cu[i + 1] > cu[i], CLEF_ERR_INVALID, "delta_scan: empty or unordered sequence");
  } else {
    CLEF_CHECK(nseq == 1 || nseq == 0, CLEF_ERR_INVALID, "delta_scan: nseq without cu_seqlens");
    nseq = 1;
    cu = {0, T};
  }
  CLEF_CHECK(capture >= 0, CLEF_ERR_INVALID, "delta_scan: capture");
  if (capture > 0) {
    CLEF_CHECK(nseq == 1, CLEF_ERR_INVALID, "delta_scan: capture needs a single sequence");
    CLEF_CHECK(capture <= T && capture_state, CLEF_ERR_INVALID,
               "delta_scan: capture boundary or capture_state");
  }
  CLEF_CHECK(((uintptr_t)q | (uintptr_t)k) % 16 == 0, CLEF_ERR_INVALID,
             "delta_scan: q and k must be 16-byte aligned");
  CLEF_CHECK(workspace && workspace_bytes >= delta_scan_workspace(T, nseq, Hk, Hv),
             CLEF_ERR_INVALID, "delta_scan: workspace too small");
  CLEF_CHECK(((uintptr_t)workspace & 255) == 0, CLEF_ERR_INVALID,
             "delta_scan: workspace must be 256-byte aligned");
  return launch_delta_scan(q, k, v, g, beta, cu.data(), nseq, Hk, Hv, dk, dv, init_state,
                           init_shared, capture, capture_state, final_state, out, workspace,
                           workspace_bytes, as_stream(stream));
}

// Same contract and results as clef_delta_scan, without a workspace: the
// sequence offsets are copied into the library's fixed device array (at most
// 4096 sequences). It allocates nothing. The first call on each device looks
// up the array's device address and should come before any stream capture.
// The offsets are copied from cu_seqlens by a copy ordered on `stream`; when
// cu_seqlens is page-locked that copy runs asynchronously, so the caller keeps
// the buffer unchanged until the stream has reached this call.
// Every call shares the one array per device, and each call rewrites the
// entries [0, nseq] it uses before its kernel reads them (nothing else needs
// to start at zero); calls whose work overlaps on the GPU (different streams,
// or host threads issuing concurrently on one device) race on it, so callers
// serialise them on one stream.
int clef_delta_scan_noalloc(const float* q, const float* k, const float* v, const float* g,
                            const float* beta, int64_t T, int32_t Hk, int32_t Hv, int32_t dk,
                            int32_t dv, const int64_t* cu_seqlens, int32_t nseq,
                            const float* init_state, int32_t init_shared, int64_t capture,
                            float* capture_state, float* final_state, float* out, void* stream) {
  CLEF_CHECK(q && k && v && g && beta && out, CLEF_ERR_INVALID, "delta_scan_noalloc: null pointer");
  CLEF_CHECK(dk == 128 && dv == 128, CLEF_ERR_UNSUPPORTED,
             "delta_scan_noalloc: dk and dv must be 128");
  CLEF_CHECK(Hk > 0 && Hv > 0 && Hv % Hk == 0 && Hv <= 4096, CLEF_ERR_INVALID,
             "delta_scan_noalloc: head counts");
  CLEF_CHECK(T > 0, CLEF_ERR_INVALID, "delta_scan_noalloc: T must be positive");
  if (cu_seqlens) {
    CLEF_CHECK(nseq > 0, CLEF_ERR_INVALID, "delta_scan_noalloc: nseq");
    CLEF_CHECK(nseq <= kNoAllocMaxSeqs, CLEF_ERR_UNSUPPORTED,
               "delta_scan_noalloc: at most 4096 sequences per call (fixed offsets array); "
               "use clef_delta_scan with a workspace for more");
    CLEF_CHECK(cu_seqlens[0] == 0 && cu_seqlens[nseq] == T, CLEF_ERR_INVALID,
               "delta_scan_noalloc: cu_seqlens range");
    for (int i = 0; i < nseq; ++i)
      CLEF_CHECK(cu_seqlens[i + 1] > cu_seqlens[i], CLEF_ERR_INVALID,
                 "delta_scan_noalloc: empty or unordered sequence");
  } else {
    CLEF_CHECK(nseq == 1 || nseq == 0, CLEF_ERR_INVALID,
               "delta_scan_noalloc: nseq without cu_seqlens");
    nseq = 1;
  }
  CLEF_CHECK(capture >= 0, CLEF_ERR_INVALID, "delta_scan_noalloc: capture");
  if (capture > 0) {
    CLEF_CHECK(nseq == 1, CLEF_ERR_INVALID, "delta_scan_noalloc: capture needs a single sequence");
    CLEF_CHECK(capture <= T && capture_state, CLEF_ERR_INVALID,
               "delta_scan_noalloc: capture boundary or capture_state");
  }
  CLEF_CHECK(((uintptr_t)q | (uintptr_t)k) % 16 == 0, CLEF_ERR_INVALID,
             "delta_scan_noalloc: q and k must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const int64_t* cu_dev = nullptr;
  if (nseq > 1) {
    int64_t* table = nullptr;
    int rc = noalloc_offsets_ptr(&table);
    if (rc) return rc;
    CLEF_CUDA(cudaMemcpyAsync(table, cu_seqlens, sizeof(int64_t) * (nseq + 1),
                              cudaMemcpyHostToDevice, s));
    cu_dev = table;
  }
  return launch_delta_scan_dev(q, k, v, g, beta, cu_dev, T, nseq, Hk, Hv, init_state, init_shared,
                               capture, capture_state, final_state, out, s);
}

}  // extern "C"
