// attention_tc.cu — causal grouped-query flash attention on the tcgen05
// tensor cores (head dim 256, BF16 operands, F32 accumulation in TMEM).
//
// Same result as ops::attention (crates/core/src/models/ops.rs:62-143):
// softmax(q k^T / 16 + lower-right causal mask) v per query head, kv head
// h / (H / Hkv), keys = [shared prefix keys] ++ [the sequence's own keys].
//
// CTA = 128 query rows of one (sequence, query head); 10 warps:
//   warp 0      TMA producer: the Q tile once, then K and V^T tiles of 64 keys
//               into a 4-slot ring in consumption order (no multicast);
//   warp 1      allocates 512 TMEM columns; one thread issues
//               S_j = Q K_j^T (128 x 64, double-buffered in TMEM) and
//               O += P_j V_j (128 x 256 accumulator in TMEM), with S_{j+2}
//               issued while the softmax of block j runs;
//   warps 2..9  one query row per thread, two warps per row quarter (each
//               exponentiates half of every 64-key block): tcgen05.ld of the S row, mask,
//               online softmax in the log2 domain, P row (BF16) stored back into
//               TMEM by tcgen05.st, where the PV product reads it as its A operand. The running maximum is
//               only raised (and O rescaled in TMEM) when a row's maximum grows
//               by more than 8 in log2 units, so O is rarely touched; the
//               epilogue normalises O by the row sum and applies the output
//               gate o * sigmoid(gate) (qwen.rs:519-524).
// V is consumed transposed (V^T rows = head dimension, keys contiguous) so both
// products use K-major shared-memory operands with the 128-byte swizzle.
// Entry points: the engine (token-major q/k, V^T per pack), clef_attention_gqa_vt
// (the same layouts from a caller) and clef_attention_gqa (the reference's
// head-major [H, T, 256] tensors of AttentionKernel, metal.rs:415-633, brought
// to those layouts in a caller-provided workspace first).
#include <cudaTypedefs.h>

#include "kernels.cuh"
#include "sm100.cuh"

#define RC_(x)           \
  do {                   \
    int rc_ = (x);       \
    if (rc_) return rc_; \
  } while (0)

namespace clef {

namespace {

using namespace sm100;

constexpr int D = 256;
constexpr int BQ = 128;
constexpr int BK = 64;
constexpr int Q_BYTES = BQ * D * 2;        // 64 KB: 4 atoms of [128 rows x 128 B]
constexpr int K_BYTES = BK * D * 2;        // 32 KB: 4 atoms of [64 rows x 128 B]
constexpr int VT_BYTES = D * BK * 2;       // 32 KB: [256 rows x 128 B]
constexpr int TILE_BYTES = 32 * 1024;      // one ring slot: a K tile or a V^T tile
static_assert(K_BYTES == TILE_BYTES && VT_BYTES == TILE_BYTES, "ring slots hold K or V^T tiles");
constexpr int NSLOT = 4;
constexpr int OFF_Q = 0;
constexpr int OFF_RING = OFF_Q + Q_BYTES;               // NSLOT slots
constexpr int OFF_BAR = OFF_RING + NSLOT * TILE_BYTES;
constexpr int OFF_LSUM = OFF_BAR + 256;                // [2][128] F32 partial row sums
constexpr int SMEM = 1024 + OFF_LSUM + 2 * BQ * 4;
constexpr int SOFTMAX_WARPS = 8;                        // two per TMEM lane quarter
constexpr int THREADS = 64 + SOFTMAX_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_O = 0, COL_S = 256;             // S buffers at 256 and 320
constexpr uint32_t COL_P = 384;                        // P buffers (BF16 pairs) at 384 and 416
constexpr float RESCALE_THRESHOLD = 8.f;               // log2 units

struct TcParams {
  int H, Hkv;
  int64_t prefix_len;
  float sl2;                 // scale * log2(e)
  const int64_t* cu;         // [nseq + 1] token offsets, or null (one sequence of `total`)
  const int64_t* cu_vt;      // [nseq + 1] padded key offsets of V^T, or null (= 0)
  const int32_t* cu_qb;      // [nseq + 1] query-block (128-row) offsets, or null
  int nseq;
  int64_t total;
  // output: F32 [t * o_ts + h * o_hs + e] if gate == null, else BF16 gated
  void* out;
  int64_t o_ts, o_hs;
  const uint16_t* gate;
  int64_t g_ts, g_hs;
};

// 2^x by the MUFU instruction (ex2.approx.ftz: relative error ~2^-22, far
// below the BF16 rounding applied to its result; -inf gives +0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ int find_seq(const int32_t* cu_qb, int nseq, int b) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_qb[mid] <= b) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                        const __grid_constant__ CUtensorMap map_vt, const __grid_constant__ CUtensorMap map_pk,
                        const __grid_constant__ CUtensorMap map_pvt, const __grid_constant__ CUtensorMap map_g,
                        TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bar + 0;
  uint64_t* s_full = bar + 1;    // [2]
  uint64_t* p_full = bar + 3;    // [2]
  uint64_t* pv_done = bar + 5;   // [2]
  uint64_t* o_final = bar + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 8);
  uint64_t* drain = bar + 9;     // error path: completion of this CTA's own MMAs
  uint64_t* q_free = bar + 10;   // the last S product has read Q
  uint64_t* g_full = bar + 11;   // gate tile landed in the Q buffer
  uint64_t* full = bar + 12;     // [NSLOT] ring slot loaded
  uint64_t* empty = bar + 12 + NSLOT;  // [NSLOT] ring slot consumed
  uint64_t* l_bar = bar + 12 + 2 * NSLOT;  // partial row sums exchanged
  float* l_part = reinterpret_cast<float*>(sm + OFF_LSUM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grid (heads, query blocks): the heads vary fastest, so the blocks of every
  // head go out in the order below, heaviest (last) query block first.
  const int h = blockIdx.x;
  const int bx = blockIdx.y;
  const int kvh = h / (p.H / p.Hkv);
  int s = 0;
  int64_t start = 0, len = p.total, vt0 = 0;
  int qb;
  if (p.cu) {
    s = find_seq(p.cu_qb, p.nseq, bx);
    start = p.cu[s];
    len = p.cu[s + 1] - start;
    vt0 = p.cu_vt ? p.cu_vt[s] : start;
    const int nqb = p.cu_qb[s + 1] - p.cu_qb[s];
    qb = nqb - 1 - (bx - p.cu_qb[s]);
  } else {
    qb = (int)((len + BQ - 1) / BQ) - 1 - bx;
  }
  const int64_t q0 = (int64_t)qb * BQ;
  const int64_t P = p.prefix_len;
  const int nbp = (int)((P + BK - 1) / BK);                         // prefix key blocks
  const int nbo = (int)((min(len, q0 + BQ) + BK - 1) / BK);          // own key blocks
  const int nblk = nbp + nbo;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], SOFTMAX_WARPS);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    mbar_init(l_bar, SOFTMAX_WARPS);
    mbar_init(q_free, 1);
    mbar_init(g_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      // The K and V^T tiles go through one ring in the order the MMA issuer
      // consumes them: K_0, K_1, then V_j, K_{j+2} for j = 0, 1, ...
      int t = 0;
      int last[NSLOT];
      for (int i = 0; i < NSLOT; ++i) last[i] = -1;
      mbar_expect_tx(q_full, Q_BYTES);
      for (int a = 0; a < 4; ++a)
        tma_load_2d(&map_q, q_full, sm + OFF_Q + a * (BQ * 128), h * D + a * 64, (int)(start + q0));
      auto load_tile = [&](bool is_k, int j) -> bool {
        const int slot = t % NSLOT;
        if (!mbar_wait(&empty[slot], ((t / NSLOT) & 1) ^ 1)) return false;
        mbar_expect_tx(&full[slot], TILE_BYTES);
        last[slot] = t++;
        uint8_t* dst = sm + OFF_RING + slot * TILE_BYTES;
        const bool pre = j < nbp;
        if (is_k) {
          const CUtensorMap* m = pre ? &map_pk : &map_k;
          const int row = pre ? j * BK : (int)(start + (int64_t)(j - nbp) * BK);
          for (int a = 0; a < 4; ++a) tma_load_2d(m, &full[slot], dst + a * (BK * 128), kvh * D + a * 64, row);
        } else if (pre) {
          tma_load_2d(&map_pvt, &full[slot], dst, j * BK, kvh * D);
        } else {
          tma_load_2d(&map_vt, &full[slot], dst, (int)(vt0 + (int64_t)(j - nbp) * BK), kvh * D);
        }
        return true;
      };
      for (int j = 0; j < 2 && j < nblk && ok; ++j) ok = load_tile(true, j);
      for (int j = 0; j < nblk && ok; ++j) {
        ok = load_tile(false, j);
        if (ok && j + 2 < nblk) ok = load_tile(true, j + 2);
      }
      // The gate tile of the output epilogue goes into the Q buffer once the
      // last S product has consumed Q: it is in shared memory before O is final.
      bool gate_issued = false;
      if (ok && p.gate) {
        ok = mbar_wait(q_free, 0);
        if (ok) {
          mbar_expect_tx(g_full, Q_BYTES);
          for (int a = 0; a < 4; ++a)
            tma_load_2d(&map_g, g_full, sm + OFF_Q + a * (BQ * 128), h * (int)p.g_hs + a * 64,
                        (int)(start + q0));
          gate_issued = true;
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA exits (bounded).
        raise_device_error(kDevAttentionTimeout);
        mbar_wait(q_full, 0);
        for (int i = 0; i < NSLOT; ++i)
          if (last[i] >= 0) mbar_wait(&full[i], (last[i] / NSLOT) & 1);
        if (gate_issued) mbar_wait(g_full, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(BQ, BK);
      constexpr uint32_t idesc_o = idesc_bf16_f32(BQ, D);
      bool ok = mbar_wait(q_full, 0);
      int t = 0;  // ring position, same order as the producer
      auto take = [&]() -> int {
        const int slot = t % NSLOT;
        if (!mbar_wait(&full[slot], (t / NSLOT) & 1)) return -1;
        ++t;
        tc_fence_after();
        return slot;
      };
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const int slot = take();
        if (slot < 0) return false;
        const uint32_t qa = sbase + OFF_Q, kb = sbase + OFF_RING + slot * TILE_BYTES;
        const uint32_t d = tmem + COL_S + st * BK;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2), in = (kk & 3) * 32;
          umma_f16(d, desc_k_sw128(qa + off * (BQ * 128) + in), desc_k_sw128(kb + off * (BK * 128) + in),
                   idesc_s, kk != 0);
        }
        umma_commit(&empty[slot]);
        umma_commit(&s_full[st]);
        if (j == nblk - 1) umma_commit(q_free);
        return true;
      };
      if (ok && nblk > 0) ok = issue_s(0);
      if (ok && nblk > 1) ok = issue_s(1);
      for (int j = 0; j < nblk && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&p_full[st], (j >> 1) & 1)) {
          ok = false;
          break;
        }
        const int slot = take();
        if (slot < 0) {
          ok = false;
          break;
        }
        const uint32_t vb = sbase + OFF_RING + slot * TILE_BYTES;
        // P_j from TMEM (16 keys = 8 columns per instruction) times V_j.
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_f16_ts(tmem + COL_O, tmem + COL_P + st * (BK / 2) + kk * 8, desc_k_sw128(vb + kk * 32), idesc_o,
                      (j | kk) != 0);
        umma_commit(&empty[slot]);
        umma_commit(&pv_done[st]);
        if (j + 2 < nblk) ok = issue_s(j + 2);
      }
      if (ok) {
        umma_commit(o_final);
      } else {
        // Wait (bounded) for the MMAs already issued before TMEM is released.
        raise_device_error(kDevAttentionTimeout);
        umma_commit(drain);
        mbar_wait(drain, 0);
      }
    }
  } else {
    // Softmax warps: row r of the query tile; TMEM lane quarter = warp % 4.
    // Two warps share each quarter: both read the whole S row (so both derive
    // the same row maximum without exchanging it), and warp half `hf`
    // exponentiates keys [32 hf, 32 hf + 32) of the block and owns O columns
    // [128 hf, 128 hf + 128).
    const int quarter = warp & 3;
    const int hf = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const int64_t qi = q0 + r;  // query index within the sequence
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int st = j & 1;
      // Waits end warp-uniformly so the .sync.aligned TMEM accesses below
      // always run with the full warp.
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[st], (j >> 1) & 1));
      if (!ok) break;
      tc_fence_after();
      // sr[0..32): this warp's 32 keys of the block; sr[32..64): the partner's.
      uint32_t sr[64];
      tmem_ld_32x32b_x32(tmem + lane_off + COL_S + st * BK + hf * 32, *reinterpret_cast<uint32_t(*)[32]>(sr));
      tmem_ld_32x32b_x32(tmem + lane_off + COL_S + st * BK + (1 - hf) * 32,
                         *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
      tmem_ld_wait();
      // Visible keys of this row in block j: columns c <= lim. A block every
      // row of the tile sees in full skips the mask (CTA-uniform branch).
      const bool pre = j < nbp;
      const int64_t kbase = pre ? (int64_t)j * BK : (int64_t)(j - nbp) * BK;
      const bool full = pre ? kbase + BK <= P : kbase + BK - 1 <= q0;
      if (!full) {
        const int64_t l64 = pre ? P - 1 - kbase : qi - kbase;
        const int lim = l64 < -1 ? -1 : (l64 > 63 ? 63 : (int)l64);
        const int mine = hf * 32, other = (1 - hf) * 32;  // block columns of sr[0], sr[32]
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (mine + c > lim) sr[c] = 0xff800000u;  // -inf
          if (other + c > lim) sr[32 + c] = 0xff800000u;
        }
      }
      // Row maximum of the raw scores (the scale is positive), four chains.
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 64; c += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) mx[u] = fmaxf(mx[u], __uint_as_float(sr[c + u]));
      }
      const float bmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * p.sl2;
      // Lazy maximum: raise it (and rescale O) only when it grows by > 8.
      const bool need = bmax > m_run + RESCALE_THRESHOLD;
      float alpha = 1.f;
      if (need) {
        alpha = exp2f(m_run - bmax);
        m_run = bmax;
        l_run *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O holds PV_0 .. PV_{j-1}: wait for the last one, rescale this row.
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1));
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = hf * 4; c < hf * 4 + 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tmem + lane_off + COL_O + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tmem + lane_off + COL_O + c * 32, o);
        }
        tmem_st_wait();
      }
      // P buffer st was last read by PV_{j-2}.
      if (j >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[st], ((j - 2) >> 1) & 1));
        if (!ok) break;
      }
      // p = 2^(s * scale * log2 e - m), rounded to BF16 as the PV product
      // consumes it; the row sum adds the rounded values. This warp's 32 keys
      // go into TMEM columns [COL_P + 32 st + 16 hf, +16) of its lanes, two
      // per column in key order.
      const float neg_m = -m_run;
      float ps[2] = {0.f, 0.f};
      uint32_t w[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(sr[2 * e]), p.sl2, neg_m));
        const float p1 = ex2_approx(fmaf(__uint_as_float(sr[2 * e + 1]), p.sl2, neg_m));
        w[e] = pack_bf16x2(p0, p1);
        ps[0] += __uint_as_float(w[e] << 16);
        ps[1] += __uint_as_float(w[e] & 0xffff0000u);
      }
      tmem_st_32x32b_x16(tmem + lane_off + COL_P + st * (BK / 2) + hf * 16, w);
      tmem_st_wait();
      l_run += ps[0] + ps[1];
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
    }
    if (ok && nblk > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_final, 0));
    if (ok && p.gate) ok = __all_sync(0xffffffffu, mbar_wait(g_full, 0));
    // Row sum = the two warps' partial sums, added in the same order by both.
    l_part[hf * BQ + r] = l_run;
    __syncwarp();
    if (lane == 0) mbar_arrive(l_bar);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(l_bar, 0));
    if (!ok) {
      raise_device_error(kDevAttentionTimeout);
    } else {
      tc_fence_after();
      const float inv = 1.f / (l_part[r] + l_part[BQ + r]);
      const bool valid = qi < len;
      const int64_t row = start + qi;
#pragma unroll 1
      for (int c = hf * 4; c < hf * 4 + 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem + lane_off + COL_O + c * 32, o);
        tmem_ld_wait();
        if (!valid) continue;
        if (p.gate) {
          // Gate columns c*32 .. c*32+31 of row r: atom c/2, 16-byte chunks
          // (c%2)*4 + e4, stored at chunk ^ (r % 8) by the 128-byte swizzle.
          const uint8_t* grow = sm + OFF_Q + (c >> 1) * (BQ * 128) + r * 128;
          uint16_t* op = reinterpret_cast<uint16_t*>(p.out) + row * p.o_ts + (int64_t)h * p.o_hs + c * 32;
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const uint4 graw =
                *reinterpret_cast<const uint4*>(grow + (((((c & 1) << 2) + e4) ^ (r & 7)) << 4));
            const uint32_t gw[4] = {graw.x, graw.y, graw.z, graw.w};
            uint32_t ow[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // o * sigmoid(gate) in F32, rounded once (the o_proj operand).
              const float g0 = sigmoid_f(__uint_as_float(gw[e] << 16));
              const float g1 = sigmoid_f(__uint_as_float(gw[e] & 0xffff0000u));
              const float v0 = __uint_as_float(o[e4 * 8 + 2 * e]) * inv;
              const float v1 = __uint_as_float(o[e4 * 8 + 2 * e + 1]) * inv;
              ow[e] = pack_bf16x2(v0 * g0, v1 * g1);
            }
            *reinterpret_cast<uint4*>(op + e4 * 8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
          }
        } else {
          float* op = reinterpret_cast<float*>(p.out) + row * p.o_ts + (int64_t)h * p.o_hs + c * 32;
#pragma unroll
          for (int e4 = 0; e4 < 8; ++e4)
            *reinterpret_cast<float4*>(op + e4 * 4) =
                make_float4(__uint_as_float(o[e4 * 4]) * inv, __uint_as_float(o[e4 * 4 + 1]) * inv,
                            __uint_as_float(o[e4 * 4 + 2]) * inv, __uint_as_float(o[e4 * 4 + 3]) * inv);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// V^T: vt[kvh * 256 + e][vt_off(s) + j] = v[(cu[s] + j) * v_ts + kvh * v_hs + e], one
// 64-key x 256-feature tile per CTA through shared memory. V is BF16, or F32
// (rounded to the BF16 operand here).
__device__ __forceinline__ uint4 load_v8(const uint16_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint4 load_v8(const float* p) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  return make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
}

template <typename In>
__global__ void transpose_v_kernel(const In* __restrict__ v, int64_t v_ts, int64_t v_hs,
                                   const int64_t* __restrict__ cu, const int64_t* __restrict__ cu_vt,
                                   const int32_t* __restrict__ cu_kb, int nseq, int64_t total,
                                   uint16_t* __restrict__ vt, int64_t vt_pitch) {
  // tileT[e][w]: feature e of keys (2w, 2w + 1) as one 32-bit word; the word
  // index is XOR-swizzled by (e & 7) << 2 so that both the column stores of
  // the first phase and the 16-byte row reads of the second are conflict-free.
  __shared__ __align__(16) uint32_t tileT[D][32];
  const int kvh = blockIdx.y;
  int s = 0;
  int64_t start = 0, len = total, off = 0;
  int kb = blockIdx.x;
  if (cu) {
    s = find_seq(cu_kb, nseq, blockIdx.x);
    start = cu[s];
    len = cu[s + 1] - start;
    off = cu_vt[s];
    kb = blockIdx.x - cu_kb[s];
  }
  const int64_t j0 = (int64_t)kb * 64;
  // Phase 1: lane = key pair, 8 features per thread from both keys' rows.
  for (int idx = threadIdx.x; idx < 32 * (D / 8); idx += blockDim.x) {
    const int jp = idx & 31, e8 = (idx >> 5) * 8;
    const int64_t r0 = j0 + 2 * jp;
    uint4 a = make_uint4(0, 0, 0, 0), b = a;
    if (r0 < len) a = load_v8(v + (start + r0) * v_ts + kvh * v_hs + e8);
    if (r0 + 1 < len) b = load_v8(v + (start + r0 + 1) * v_ts + kvh * v_hs + e8);
    const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int e = e8 + 2 * t;
      tileT[e][jp ^ ((e & 7) << 2)] = __byte_perm(wa[t], wb[t], 0x5410);
      tileT[e + 1][jp ^ (((e + 1) & 7) << 2)] = __byte_perm(wa[t], wb[t], 0x7632);
    }
  }
  __syncthreads();
  // Phase 2: V^T row e, keys [8q, 8q + 8) as one 16-byte read and store.
  for (int idx = threadIdx.x; idx < D * 8; idx += blockDim.x) {
    const int e = idx >> 3, q = idx & 7, j8 = q * 8;
    const uint4 w = *reinterpret_cast<const uint4*>(&tileT[e][(4 * q) ^ ((e & 7) << 2)]);
    *reinterpret_cast<uint4*>(vt + (int64_t)(kvh * D + e) * vt_pitch + off + j0 + j8) = w;
  }
}

// dst[(t * H + h) * 256 + e] = src[(h * T + t) * 256 + e]: head-major rows to
// the token-major layout the kernel's Q/K tensor maps read (one warp per
// 512-byte row, 16-byte accesses).
__global__ void head_to_token_major_kernel(const uint16_t* __restrict__ src, int H, int64_t T,
                                           uint16_t* __restrict__ dst) {
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= (int64_t)H * T) return;
  const int64_t h = r / T, t = r - h * T;
  const int lane = threadIdx.x & 31;
  reinterpret_cast<uint4*>(dst + (t * H + h) * D)[lane] = reinterpret_cast<const uint4*>(src + r * D)[lane];
}

PFN_cuTensorMapEncodeTiled_v12000 encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// BF16 matrix [rows, cols] with row pitch `pitch` elements; box = box_rows x 64.
int map2d(CUtensorMap* m, const void* ptr, uint64_t rows, uint64_t cols, uint64_t pitch,
          uint32_t box_rows) {
  auto fn = encode();
  if (!fn) return fail(CLEF_ERR_CUDA, "attention: cuTensorMapEncodeTiled unavailable");
  CLEF_CHECK(((uintptr_t)ptr & 15) == 0 && (pitch * 2) % 16 == 0, CLEF_ERR_INVALID,
             "attention: tensor base and row pitch must be 16-byte aligned");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CLEF_ERR_CUDA, "attention: cuTensorMapEncodeTiled failed");
  return CLEF_OK;
}

}  // namespace

template <typename In>
int launch_transpose_v_t(const In* v, int64_t v_ts, int64_t v_hs, const SeqPackVT& pk, int Hkv,
                         uint16_t* vt, int64_t vt_pitch, cudaStream_t s) {
  if (pk.total == 0) return CLEF_OK;
  const unsigned blocks = pk.cu ? (unsigned)pk.kblocks : (unsigned)ceil_div(pk.total, 64);
  transpose_v_kernel<In><<<dim3(blocks, (unsigned)Hkv), 256, 0, s>>>(v, v_ts, v_hs, pk.cu, pk.cu_vt, pk.cu_kb,
                                                                  pk.nseq, pk.total, vt, vt_pitch);
  return launch_status("transpose_v");
}

int launch_transpose_v(const uint16_t* v, int64_t v_ts, int64_t v_hs, const SeqPackVT& pk, int Hkv,
                       uint16_t* vt, int64_t vt_pitch, cudaStream_t s) {
  return launch_transpose_v_t(v, v_ts, v_hs, pk, Hkv, vt, vt_pitch, s);
}

int launch_transpose_v(const float* v, int64_t v_ts, int64_t v_hs, const SeqPackVT& pk, int Hkv,
                       uint16_t* vt, int64_t vt_pitch, cudaStream_t s) {
  return launch_transpose_v_t(v, v_ts, v_hs, pk, Hkv, vt, vt_pitch, s);
}

int launch_attention_tc(const AttnTcArgs& a, const SeqPackVT& pk, cudaStream_t s) {
  CLEF_CHECK(a.H > 0 && a.Hkv > 0 && a.H % a.Hkv == 0, CLEF_ERR_INVALID, "attention_tc: heads");
  if (pk.total == 0) return CLEF_OK;
  CLEF_CHECK(a.rows_q < (1LL << 31) && a.vt_cols < (1LL << 31), CLEF_ERR_UNSUPPORTED,
             "attention_tc: tensors too large for 32-bit TMA coordinates");
  CUtensorMap mq, mk, mvt, mpk, mpvt, mg;
  int rc = map2d(&mq, a.q, (uint64_t)a.rows_q, (uint64_t)a.H * D, (uint64_t)a.H * D, BQ);
  if (!rc) rc = map2d(&mk, a.k, (uint64_t)a.rows_k, (uint64_t)a.Hkv * D, (uint64_t)a.Hkv * D, BK);
  if (!rc) rc = map2d(&mvt, a.vt, (uint64_t)a.Hkv * D, (uint64_t)a.vt_cols, (uint64_t)a.vt_pitch, D);
  if (rc) return rc;
  if (a.prefix_len > 0) {
    rc = map2d(&mpk, a.pk, (uint64_t)a.prefix_len, (uint64_t)a.Hkv * D, (uint64_t)a.Hkv * D, BK);
    if (!rc)
      rc = map2d(&mpvt, a.pvt, (uint64_t)a.Hkv * D, (uint64_t)a.prefix_len, (uint64_t)a.pvt_pitch, D);
    if (rc) return rc;
  } else {
    mpk = mk;
    mpvt = mvt;
  }
  if (a.gate) {
    CLEF_CHECK(a.g_hs % 8 == 0, CLEF_ERR_INVALID, "attention_tc: gate head stride");
    rc = map2d(&mg, a.gate, (uint64_t)a.rows_q, (uint64_t)(a.H - 1) * a.g_hs + D, (uint64_t)a.g_ts, BQ);
    if (rc) return rc;
  } else {
    mg = mq;
  }
  TcParams p;
  p.H = a.H;
  p.Hkv = a.Hkv;
  p.prefix_len = a.prefix_len;
  p.sl2 = a.scale * 1.4426950408889634f;
  p.cu = pk.cu;
  p.cu_vt = pk.cu_vt;
  p.cu_qb = pk.cu_qb;
  p.nseq = pk.nseq;
  p.total = pk.total;
  p.out = a.out;
  p.o_ts = a.o_ts;
  p.o_hs = a.o_hs;
  p.gate = a.gate;
  p.g_ts = a.g_ts;
  p.g_hs = a.g_hs;
  static bool attr[64] = {false};
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    CLEF_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr[dev] = true;
  }
  const unsigned blocks = pk.cu ? (unsigned)pk.qblocks : (unsigned)ceil_div(pk.total, BQ);
  CLEF_CHECK(blocks <= 65535u, CLEF_ERR_UNSUPPORTED, "attention_tc: more than 65535 query blocks in one call");
  attention_tc_kernel<<<dim3((unsigned)a.H, blocks), THREADS, SMEM, s>>>(mq, mk, mvt, mpk, mpvt, mg, p);
  return launch_status("attention_tc");
}

int attention_tc_device_error(int* code) { return read_device_error(code); }

}  // namespace clef

using namespace clef;

extern "C" {

size_t clef_attention_gqa_workspace_size(int32_t Hq, int32_t Hkv, int64_t Tq, int64_t Tk) {
  if (Hq <= 0 || Hkv <= 0 || Tq <= 0 || Tk < Tq) return 0;
  auto a256 = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const int64_t pre = Tk - Tq;
  return a256((size_t)Tq * Hq * 256 * 2) + a256((size_t)Tk * Hkv * 256 * 2) +
         a256((size_t)Hkv * 256 * ((pre + 63) / 64 * 64) * 2) + a256((size_t)Hkv * 256 * ((Tq + 63) / 64 * 64) * 2);
}

int clef_attention_gqa(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t Hq,
                       int32_t Hkv, int64_t Tq, int64_t Tk, int32_t d, float* out, void* workspace,
                       size_t workspace_bytes, void* stream) {
  CLEF_CHECK(q && k && v && out, CLEF_ERR_INVALID, "attention_gqa: null pointer");
  CLEF_CHECK(d == 256, CLEF_ERR_UNSUPPORTED, "attention_gqa: d must be 256");
  CLEF_CHECK(Hq > 0 && Hkv > 0 && Hq % Hkv == 0, CLEF_ERR_INVALID, "attention_gqa: head counts");
  CLEF_CHECK(Tq > 0 && Tk >= Tq, CLEF_ERR_INVALID, "attention_gqa: need 0 < Tq <= Tk");
  CLEF_CHECK((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15) == 0,
             CLEF_ERR_INVALID, "attention_gqa: pointers must be 16-byte aligned");
  const size_t need = clef_attention_gqa_workspace_size(Hq, Hkv, Tq, Tk);
  CLEF_CHECK(workspace && workspace_bytes >= need && ((uintptr_t)workspace & 255) == 0, CLEF_ERR_INVALID,
             "attention_gqa: workspace must be 256-byte aligned and hold "
             "clef_attention_gqa_workspace_size() bytes");
  cudaStream_t s = as_stream(stream);
  auto a256 = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const int64_t pre = Tk - Tq;
  const int64_t pre_pitch = (pre + 63) / 64 * 64, own_pitch = (Tq + 63) / 64 * 64;
  uint8_t* w = reinterpret_cast<uint8_t*>(workspace);
  uint16_t* qt = reinterpret_cast<uint16_t*>(w);
  w += a256((size_t)Tq * Hq * 256 * 2);
  uint16_t* kt = reinterpret_cast<uint16_t*>(w);
  w += a256((size_t)Tk * Hkv * 256 * 2);
  uint16_t* pvt = reinterpret_cast<uint16_t*>(w);
  w += a256((size_t)Hkv * 256 * pre_pitch * 2);
  uint16_t* vt = reinterpret_cast<uint16_t*>(w);
  // Token-major q and k, transposed values (prefix keys and own keys in
  // separate V^T blocks so both start 64-key aligned).
  head_to_token_major_kernel<<<(unsigned)ceil_div((int64_t)Hq * Tq, 8), 256, 0, s>>>(q, Hq, Tq, qt);
  head_to_token_major_kernel<<<(unsigned)ceil_div((int64_t)Hkv * Tk, 8), 256, 0, s>>>(k, Hkv, Tk, kt);
  RC_(launch_status("attention_gqa: layout"));
  SeqPackVT one;
  one.nseq = 1;
  if (pre > 0) {
    one.total = pre;
    RC_(launch_transpose_v(v, 256, Tk * 256, one, Hkv, pvt, pre_pitch, s));
  }
  one.total = Tq;
  RC_(launch_transpose_v(v + pre * 256, 256, Tk * 256, one, Hkv, vt, own_pitch, s));
  AttnTcArgs a;
  a.H = Hq;
  a.Hkv = Hkv;
  a.scale = 1.f / 16.f;
  a.q = qt;
  a.rows_q = Tq;
  a.k = kt + pre * Hkv * 256;
  a.rows_k = Tq;
  a.vt = vt;
  a.vt_cols = Tq;
  a.vt_pitch = own_pitch;
  if (pre > 0) {
    a.prefix_len = pre;
    a.pk = kt;
    a.pvt = pvt;
    a.pvt_pitch = pre_pitch;
  }
  a.out = out;  // head-major F32 [Hq, Tq, 256]
  a.o_ts = 256;
  a.o_hs = Tq * 256;
  return launch_attention_tc(a, one, s);
}

int clef_attention_gqa_vt(const uint16_t* q, const uint16_t* k, const uint16_t* vt, int32_t Hq,
                          int32_t Hkv, int64_t Tq, int64_t Tk, int32_t d, int64_t vt_pitch,
                          float* out, void* stream) {
  CLEF_CHECK(q && k && vt && out, CLEF_ERR_INVALID, "attention_gqa_vt: null pointer");
  CLEF_CHECK(d == 256, CLEF_ERR_UNSUPPORTED, "attention_gqa_vt: d must be 256");
  CLEF_CHECK(Hq > 0 && Hkv > 0 && Hq % Hkv == 0, CLEF_ERR_INVALID, "attention_gqa_vt: head counts");
  CLEF_CHECK(Tq > 0 && Tk >= Tq, CLEF_ERR_INVALID, "attention_gqa_vt: need 0 < Tq <= Tk");
  const int64_t pre = Tk - Tq;
  CLEF_CHECK(pre % 8 == 0, CLEF_ERR_UNSUPPORTED,
             "attention_gqa_vt: Tk - Tq must be a multiple of 8 (16-byte aligned V^T columns)");
  CLEF_CHECK(vt_pitch >= Tk && vt_pitch % 8 == 0, CLEF_ERR_INVALID, "attention_gqa_vt: vt_pitch");
  CLEF_CHECK((((uintptr_t)q | (uintptr_t)k | (uintptr_t)vt | (uintptr_t)out) & 15) == 0,
             CLEF_ERR_INVALID, "attention_gqa_vt: pointers must be 16-byte aligned");
  AttnTcArgs a;
  a.H = Hq;
  a.Hkv = Hkv;
  a.scale = 1.f / 16.f;
  a.q = q;
  a.rows_q = Tq;
  a.k = k + pre * Hkv * 256;
  a.rows_k = Tq;
  a.vt = vt + pre;
  a.vt_cols = Tq;
  a.vt_pitch = vt_pitch;
  a.prefix_len = pre;
  a.pk = k;
  a.pvt = vt;
  a.pvt_pitch = vt_pitch;
  a.out = out;
  a.o_ts = (int64_t)Hq * 256;
  a.o_hs = 256;
  SeqPackVT pk;
  pk.nseq = 1;
  pk.total = Tq;
  return launch_attention_tc(a, pk, as_stream(stream));
}

}  // extern "C"
