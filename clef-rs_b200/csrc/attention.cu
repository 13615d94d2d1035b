// attention.cu — causal grouped-query flash attention, head dim 256.
//
// softmax(q k^T / sqrt(d) + lower-right causal mask) v with an online softmax
// in F32 (ops::attention, crates/core/src/models/ops.rs:62-143; the Metal
// AttentionKernel, metal.rs:415-633). Query head h reads kv head
// h / (H / Hkv) directly; K/V are never expanded.
//
// The key sequence of every query sequence is [shared prefix keys] followed by
// its own keys, so a request continuing from a captured prefix (PrefixState)
// attends to the prefix K/V in place. Query i of a sequence sees key j iff
// j <= i + prefix_len (the reference's lower-right offset kn - qn, ops.rs:107).
//
// CTA: 4 warps x 16 query rows of one (sequence, query head); K/V stream
// through a double-buffered shared-memory ring of 32-key tiles (cp.async,
// XOR-swizzled 16-byte chunks so ldmatrix is bank-conflict free). Q K^T and
// P V run on BF16 mma.sync with F32 accumulators; the 16 x 256 output tile of
// a warp stays in registers.
#include "kernels.cuh"

namespace clef {

namespace {

constexpr int D = 256;
constexpr int BQ = 64;   // query rows per CTA
constexpr int BKV = 32;  // keys per tile
constexpr int WARPS = 4;
constexpr int ROWB = D * 2;  // bytes per smem row
constexpr size_t SMEM = (size_t)BQ * ROWB + 2 * 2 * (size_t)BKV * ROWB;

__device__ __forceinline__ uint32_t swz(int row, int col) {  // byte offset in a tile
  return (uint32_t)(row * ROWB + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct Params {
  AttnArgs a;
  const int64_t* cu;      // device [nseq+1] or null (one sequence of `total` rows)
  const int32_t* cu_qb;   // device [nseq+1] q-block offsets or null
  int nseq;
  int64_t total;
};

__device__ __forceinline__ int find_seq(const int32_t* cu_qb, int nseq, int b) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_qb[mid] <= b) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(WARPS * 32, 2) attention_kernel(Params P) {
  extern __shared__ __align__(128) uint8_t sm[];
  const AttnArgs& a = P.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.y;
  const int kvh = h / (a.H / a.Hkv);

  // Sequence and query block (heaviest blocks of each sequence first).
  int s = 0;
  int64_t start = 0, len = P.total;
  int qb;
  if (P.cu) {
    s = find_seq(P.cu_qb, P.nseq, blockIdx.x);
    start = P.cu[s];
    len = P.cu[s + 1] - start;
    const int nqb = P.cu_qb[s + 1] - P.cu_qb[s];
    qb = nqb - 1 - (blockIdx.x - P.cu_qb[s]);
  } else {
    const int nqb = (int)((len + BQ - 1) / BQ);
    qb = nqb - 1 - blockIdx.x;
  }
  const int64_t q0 = (int64_t)qb * BQ;
  const int64_t pre = a.prefix_len;
  const int64_t kv_total = pre + len;
  const int64_t kv_end = min(kv_total, pre + q0 + BQ);  // last key any row of this block sees + 1
  const int nkv = (int)((kv_end + BKV - 1) / BKV);

  const uint32_t sQ = (uint32_t)__cvta_generic_to_shared(sm);
  const uint32_t sK0 = sQ + BQ * ROWB;
  const uint32_t sV0 = sK0 + 2 * BKV * ROWB;

  // Q tile.
  for (int c = tid; c < BQ * (D / 8); c += WARPS * 32) {
    const int r = c / (D / 8), col = (c % (D / 8)) * 8;
    const int64_t t = q0 + r;
    const bool valid = t < len;
    const uint16_t* src = a.q + (valid ? (start + t) * a.q_ts + (int64_t)h * a.q_hs + col : 0);
    cp_async16(sQ + swz(r, col), src, valid);
  }
  auto load_kv = [&](int blk, int buf) {
    const uint32_t sK = sK0 + buf * BKV * ROWB, sV = sV0 + buf * BKV * ROWB;
    for (int c = tid; c < BKV * (D / 8); c += WARPS * 32) {
      const int r = c / (D / 8), col = (c % (D / 8)) * 8;
      const int64_t j = (int64_t)blk * BKV + r;
      const bool valid = j < kv_total;
      const uint16_t* ks;
      const uint16_t* vs;
      if (j < pre) {
        ks = a.pk + j * a.p_ts + (int64_t)kvh * a.p_hs + col;
        vs = a.pv + j * a.p_ts + (int64_t)kvh * a.p_hs + col;
      } else {
        const int64_t o = valid ? start + (j - pre) : 0;
        ks = a.k + o * a.k_ts + (int64_t)kvh * a.k_hs + col;
        vs = a.v + o * a.v_ts + (int64_t)kvh * a.v_hs + col;
      }
      cp_async16(sK + swz(r, col), valid ? ks : a.q, valid);
      cp_async16(sV + swz(r, col), valid ? vs : a.q, valid);
    }
  };
  load_kv(0, 0);
  cp_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sl2 = a.scale * 1.4426950408889634f;  // log2(e)
  const int r_base = warp * 16 + (lane >> 2);        // rows r_base and r_base + 8 of the block

  for (int blk = 0; blk < nkv; ++blk) {
    const int buf = blk & 1;
    if (blk + 1 < nkv) {
      load_kv(blk + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + buf * BKV * ROWB, sV = sV0 + buf * BKV * ROWB;

    // S = Q K^T for 16 rows x 32 keys.
    float sacc[BKV / 8][4];
#pragma unroll
    for (int i = 0; i < BKV / 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(sQ + swz(warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8), a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < BKV / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int col = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(sK + swz(key, col), b0, b1, b2, b3);
        mma_bf16(sacc[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16(sacc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // Scale, mask, online softmax.
    const int64_t key0 = (int64_t)blk * BKV;
    const bool need_mask = key0 + BKV - 1 > pre + q0;  // the block crosses some row's diagonal
    float bmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < BKV / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = r_base + (e >> 1) * 8;
        const int64_t key = key0 + nt * 8 + 2 * (lane & 3) + (e & 1);
        float v = sacc[nt][e] * sl2;
        if (need_mask && key > pre + q0 + row) v = -INFINITY;
        sacc[nt][e] = v;
        bmax[e >> 1] = fmaxf(bmax[e >> 1], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      bmax[i] = fmaxf(bmax[i], __shfl_xor_sync(0xffffffffu, bmax[i], 1));
      bmax[i] = fmaxf(bmax[i], __shfl_xor_sync(0xffffffffu, bmax[i], 2));
      const float mn = fmaxf(mrow[i], bmax[i]);
      alpha[i] = exp2f(mrow[i] - mn);
      mrow[i] = mn;
      lrow[i] *= alpha[i];
    }
    uint32_t pa[BKV / 8][2];
#pragma unroll
    for (int nt = 0; nt < BKV / 8; ++nt) {
      const float p0 = exp2f(sacc[nt][0] - mrow[0]);
      const float p1 = exp2f(sacc[nt][1] - mrow[0]);
      const float p2 = exp2f(sacc[nt][2] - mrow[1]);
      const float p3 = exp2f(sacc[nt][3] - mrow[1]);
      lrow[0] += p0 + p1;
      lrow[1] += p2 + p3;
      pa[nt][0] = pack_bf16x2(p0, p1);
      pa[nt][1] = pack_bf16x2(p2, p3);
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // O += P V.
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk) {
      const uint32_t a0 = pa[2 * kk][0], a1 = pa[2 * kk][1], a2 = pa[2 * kk + 1][0],
                     a3 = pa[2 * kk + 1][1];
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        uint32_t b0, b1, b2, b3;
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int col = np * 16 + ((lane >> 4) << 3);
        ldsm_x4_t(sV + swz(key, col), b0, b1, b2, b3);
        mma_bf16(o[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // this buffer is refilled two iterations later
  }

  // Normalise and store.
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 1);
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 2);
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int64_t t = q0 + r_base + half * 8;
    if (t >= len) continue;
    const float inv = 1.f / lrow[half];
    const int64_t row = start + t;
#pragma unroll
    for (int nt = 0; nt < D / 8; ++nt) {
      const int col = nt * 8 + 2 * (lane & 3);
      const float v0 = o[nt][2 * half] * inv, v1 = o[nt][2 * half + 1] * inv;
      if (a.gate) {
        const uint32_t graw = *reinterpret_cast<const uint32_t*>(
            a.gate + row * a.g_ts + (int64_t)h * a.g_hs + col);
        const float g0 = bf16_round(sigmoid_f(__uint_as_float(graw << 16)));
        const float g1 = bf16_round(sigmoid_f(__uint_as_float(graw & 0xffff0000u)));
        *reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(a.out) + row * a.o_ts +
                                     (int64_t)h * a.o_hs + col) =
            pack_bf16x2(bf16_round(v0) * g0, bf16_round(v1) * g1);
      } else {
        *reinterpret_cast<float2*>(reinterpret_cast<float*>(a.out) + row * a.o_ts +
                                   (int64_t)h * a.o_hs + col) = make_float2(v0, v1);
      }
    }
  }
}

}  // namespace

int launch_attention(const AttnArgs& a, const SeqPack& pack, cudaStream_t s) {
  CLEF_CHECK(a.d == D, CLEF_ERR_UNSUPPORTED, "attention: head dim must be 256");
  CLEF_CHECK(a.H > 0 && a.Hkv > 0 && a.H % a.Hkv == 0, CLEF_ERR_INVALID, "attention: heads");
  if (pack.total == 0) return CLEF_OK;
  Params p;
  p.a = a;
  p.cu = pack.cu_seqlens;
  p.nseq = pack.nseq;
  p.total = pack.total;
  p.cu_qb = nullptr;
  unsigned blocks;
  if (pack.cu_seqlens) {
    // The engine supplies q-block offsets right after the sequence offsets:
    // cu_qb = (int32*)(cu_seqlens + nseq + 1).
    p.cu_qb = reinterpret_cast<const int32_t*>(pack.cu_seqlens + pack.nseq + 1);
    blocks = (unsigned)pack.qblocks;
  } else {
    blocks = (unsigned)ceil_div(pack.total, BQ);
  }
  static bool attr[64] = {false};
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    CLEF_CUDA(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)SMEM));
    attr[dev] = true;
  }
  attention_kernel<<<dim3(blocks, (unsigned)a.H), WARPS * 32, SMEM, s>>>(p);
  return launch_status("attention");
}

}  // namespace clef

using namespace clef;

extern "C" {

int clef_attention_gqa(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t Hq,
                       int32_t Hkv, int64_t Tq, int64_t Tk, int32_t d, float* out, void* stream) {
  CLEF_CHECK(q && k && v && out, CLEF_ERR_INVALID, "attention_gqa: null pointer");
  CLEF_CHECK(d == 256, CLEF_ERR_UNSUPPORTED, "attention_gqa: d must be 256");
  CLEF_CHECK(Hq > 0 && Hkv > 0 && Hq % Hkv == 0, CLEF_ERR_INVALID, "attention_gqa: head counts");
  CLEF_CHECK(Tq > 0 && Tk >= Tq, CLEF_ERR_INVALID, "attention_gqa: need 0 < Tq <= Tk");
  CLEF_CHECK((((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) & 15) == 0,
             CLEF_ERR_INVALID, "attention_gqa: pointers must be 16-byte aligned");
  AttnArgs a;
  a.H = Hq;
  a.Hkv = Hkv;
  a.d = d;
  a.scale = 1.f / 16.f;
  a.q = q;
  a.q_ts = d;
  a.q_hs = Tq * d;
  const int64_t pre = Tk - Tq;
  a.prefix_len = pre;
  a.pk = k;
  a.pv = v;
  a.p_ts = d;
  a.p_hs = Tk * d;
  a.k = k + pre * d;
  a.v = v + pre * d;
  a.k_ts = a.v_ts = d;
  a.k_hs = a.v_hs = Tk * d;
  a.out = out;
  a.o_ts = d;
  a.o_hs = Tq * d;
  SeqPack pack;
  pack.nseq = 1;
  pack.total = Tq;
  return launch_attention(a, pack, as_stream(stream));
}

}  // extern "C"
