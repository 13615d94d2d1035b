// delta_scan.cu — chunked gated-DeltaNet scan (chunk C = 64, dk = dv = 128).
//
// The reference recurrence, per v-head (delta_recurrence_prefill,
// crates/core/src/models/qwen.rs:867-880; clef_delta, delta.metal:62-130):
//   S <- S e^{g_t};  d_t = (v_t - S^T k_t) beta_t;  S <- S + k_t d_t^T;  o_t = S^T q_t
// is evaluated a chunk at a time in the WY / UT form that the reference states
// in its chunkwise candidate (chunk.rs:16-149, chunk.metal:10-164):
//   G_i   = sum_{s<=i} g_s (chunk-relative, accumulated in FP64)
//   A_ij  = beta_i e^{G_i-G_j} k_i.k_j           (j < i)
//   W     = (I + A)^{-1} diag(beta e^G) K,   U = (I + A)^{-1} diag(beta) V
//   D     = U - W S_prev                          (the chunk's delta rows)
//   O     = diag(e^G) Q S_prev + (M o Q K^T) D,   M_ij = e^{G_i-G_j} (j <= i)
//   S_new = e^{G_last} S_prev + (diag(e^{G_last-G}) K)^T D
// Every decay factor is the exponential of a non-positive difference of
// chunk-relative cumulative log-decays, so nothing is divided by an
// underflowed prefix product (a per-token decay of -1000 is exact).
//
// Phase 1 (delta_chunk_prep): one CTA per (chunk, v-head), all in parallel:
//   Gram matrices, the unit-lower-triangular solve by forward substitution
//   (each thread owns one of the 256 right-hand-side columns of [W | U] in
//   registers), and the decay vectors; results go to the workspace.
// Phase 2 (delta_chunk_carry): one CTA per (sequence, v-head, 16-column
//   slice of dv); walks the sequence's chunks in order carrying its
//   128 x 16 slice of S in shared memory.
#include <vector>

#include "kernels.cuh"

namespace clef {

namespace {

constexpr int C = 64;        // chunk length
constexpr int DK = 128;      // key dim
constexpr int DV = 128;      // value dim
constexpr int DVS = 16;      // value columns per carry CTA
constexpr int SLICES = DV / DVS;

struct ScanSeq {
  int32_t chunk0;
  int32_t nchunks;
  int32_t capture_chunk;  // relative index of the chunk that ends at the capture point, -1 none
  int32_t pad;
};
struct ScanChunk {
  int64_t t0;
  int32_t n;
  int32_t seq;
};

// Per (chunk, head) block in the workspace (floats).
constexpr int64_t kW = 0;                 // [C][DK]
constexpr int64_t kU = kW + C * DK;       // [C][DV]
constexpr int64_t kP = kU + C * DV;       // [C][C] lower (incl. diagonal) M o QK^T
constexpr int64_t kEG = kP + C * C;       // [C] e^{G_i}
constexpr int64_t kEGD = kEG + C;         // [C] e^{G_last - G_i}
constexpr int64_t kEGL = kEGD + C;        // [C] e^{G_last} in slot 0
constexpr int64_t kBlock = kEGL + C;

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct Layout {
  size_t seq_off, chunk_off, data_off, total;
  int64_t max_chunks;
};

Layout layout(int64_t total_tokens, int nseq, int Hv) {
  Layout l;
  l.max_chunks = ceil_div(total_tokens, C) + nseq + 1;
  l.seq_off = 0;
  l.chunk_off = align256(sizeof(ScanSeq) * (size_t)nseq);
  l.data_off = align256(l.chunk_off + sizeof(ScanChunk) * (size_t)l.max_chunks);
  l.total = l.data_off + sizeof(float) * (size_t)kBlock * (size_t)l.max_chunks * (size_t)Hv;
  return l;
}

// ---------------------------------------------------------------------------
// Phase 1.
// ---------------------------------------------------------------------------
constexpr int KP = 129;  // Gram-stage pitch (conflict-free row-strided reads)
constexpr int AP = 68;   // A pitch (16-byte aligned rows for float4 broadcasts)

__global__ void __launch_bounds__(256) delta_chunk_prep(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta,
    const ScanChunk* __restrict__ chunks, int Hk, int Hv, float* __restrict__ data) {
  extern __shared__ __align__(16) float sm[];
  float* Ks = sm;                       // [C][KP]
  float* Qs = Ks + C * KP;              // [C][KP]
  float* As = Qs + C * KP;              // [C][AP]
  float* bs = As + C * AP;              // [C] beta
  float* egs = bs + C;                  // [C] e^{G}
  double* Gs = reinterpret_cast<double*>(egs + C);  // [C]

  const int tid = threadIdx.x;
  const int h = blockIdx.y;
  const ScanChunk ch = chunks[blockIdx.x];
  const int n = ch.n;
  const int kh = h / (Hv / Hk);
  float* blk = data + ((int64_t)blockIdx.x * Hv + h) * kBlock;

  // Load K, Q rows of the chunk (zero rows past n).
  for (int idx = tid; idx < C * (DK / 4); idx += 256) {
    const int i = idx / (DK / 4), c4 = (idx % (DK / 4)) * 4;
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), qv = kv;
    if (i < n) {
      const int64_t off = ((ch.t0 + i) * Hk + kh) * DK + c4;
      kv = *reinterpret_cast<const float4*>(k + off);
      qv = *reinterpret_cast<const float4*>(q + off);
    }
    float* kr = Ks + i * KP + c4;
    float* qr = Qs + i * KP + c4;
    kr[0] = kv.x; kr[1] = kv.y; kr[2] = kv.z; kr[3] = kv.w;
    qr[0] = qv.x; qr[1] = qv.y; qr[2] = qv.z; qr[3] = qv.w;
  }
  // Chunk-relative inclusive cumsum of g in FP64 (warp 0, two tokens a lane).
  if (tid < 32) {
    const int i0 = 2 * tid, i1 = 2 * tid + 1;
    const double g0 = i0 < n ? (double)g[(ch.t0 + i0) * Hv + h] : 0.0;
    const double g1 = i1 < n ? (double)g[(ch.t0 + i1) * Hv + h] : 0.0;
    double pair = g0 + g1, run = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double up = __shfl_up_sync(0xffffffffu, run, o);
      if (tid >= o) run += up;
    }
    const double excl = run - pair;
    Gs[i0] = excl + g0;
    Gs[i1] = excl + g0 + g1;
    bs[i0] = i0 < n ? beta[(ch.t0 + i0) * Hv + h] : 0.f;
    bs[i1] = i1 < n ? beta[(ch.t0 + i1) * Hv + h] : 0.f;
  }
  __syncthreads();
  const double Glast = Gs[n - 1];
  if (tid < C) {
    const float eg = tid < n ? expf((float)Gs[tid]) : 0.f;
    egs[tid] = eg;
    blk[kEG + tid] = eg;
    blk[kEGD + tid] = tid < n ? expf((float)(Glast - Gs[tid])) : 0.f;
    blk[kEGL + tid] = tid == 0 ? expf((float)Glast) : 0.f;
  }

  // A (strictly lower) and P = M o QK^T (lower incl. diagonal): each thread a
  // 4 x 4 block, rows ti*4 + a, columns tj + 16 b.
  {
    const int ti = tid >> 4, tj = tid & 15;
    float akk[4][4], aqk[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) akk[a][b] = aqk[a][b] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < DK; ++kk) {
      float ki[4], qi[4], kj[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        ki[a] = Ks[(ti * 4 + a) * KP + kk];
        qi[a] = Qs[(ti * 4 + a) * KP + kk];
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) kj[b] = Ks[(tj + 16 * b) * KP + kk];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          akk[a][b] = fmaf(ki[a], kj[b], akk[a][b]);
          aqk[a][b] = fmaf(qi[a], kj[b], aqk[a][b]);
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int i = ti * 4 + a;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int j = tj + 16 * b;
        const bool valid = i < n && j <= i;
        const float decay = valid ? expf((float)(Gs[i] - Gs[j])) : 0.f;
        As[i * AP + j] = (valid && j < i) ? bs[i] * (decay * akk[a][b]) : 0.f;
        blk[kP + i * C + j] = valid ? decay * aqk[a][b] : 0.f;
      }
    }
  }
  __syncthreads();

  // Forward substitution (I + A) X = B for the 256 columns of [W | U].
  {
    const int c = tid;
    float x[C];
    if (c < DK) {
#pragma unroll
      for (int i = 0; i < C; ++i) x[i] = bs[i] * (egs[i] * Ks[i * KP + c]);
    } else {
      const int cv = c - DK;
#pragma unroll
      for (int i = 0; i < C; ++i)
        x[i] = i < n ? bs[i] * v[((ch.t0 + i) * Hv + h) * DV + cv] : 0.f;
    }
#pragma unroll
    for (int i = 1; i < C; ++i) {
      const float* arow = As + i * AP;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int j4 = 0; j4 < i; j4 += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(arow + j4);
        s0 = fmaf(a4.x, x[j4], s0);
        if (j4 + 1 < i) s1 = fmaf(a4.y, x[j4 + 1], s1);
        if (j4 + 2 < i) s2 = fmaf(a4.z, x[j4 + 2], s2);
        if (j4 + 3 < i) s3 = fmaf(a4.w, x[j4 + 3], s3);
      }
      x[i] = x[i] - ((s0 + s1) + (s2 + s3));
    }
    float* dst = blk + (c < DK ? kW + c : kU + (c - DK));
#pragma unroll
    for (int i = 0; i < C; ++i) dst[i * DK] = x[i];
  }
}

// ---------------------------------------------------------------------------
// Phase 2.
// ---------------------------------------------------------------------------
constexpr int WP = 132;  // row pitch of W / Q / K tiles (float4-aligned, conflict-free)
constexpr int PP = 68;

__global__ void __launch_bounds__(256) delta_chunk_carry(
    const float* __restrict__ q, const float* __restrict__ k, const ScanSeq* __restrict__ seqs,
    const ScanChunk* __restrict__ chunks, const float* __restrict__ data, int Hk, int Hv,
    const float* __restrict__ init, int init_shared, float* __restrict__ capture_state,
    float* __restrict__ final_state, float* __restrict__ out) {
  extern __shared__ __align__(16) float sm[];
  float* Ws = sm;                 // [C][WP]
  float* Qs = Ws + C * WP;        // [C][WP]
  float* Ks = Qs + C * WP;        // [C][WP]
  float* Ps = Ks + C * WP;        // [C][PP]
  float* Ss = Ps + C * PP;        // [DK][DVS]
  float* Ds = Ss + DK * DVS;      // [C][DVS]
  float* Us = Ds + C * DVS;       // [C][DVS]
  float* eg = Us + C * DVS;       // [C]
  float* egd = eg + C;            // [C]
  float* egl = egd + C;           // [4]

  const int tid = threadIdx.x;
  const int slice = blockIdx.x % SLICES;
  const int h = (blockIdx.x / SLICES) % Hv;
  const int s = blockIdx.x / (SLICES * Hv);
  const int kh = h / (Hv / Hk);
  const int c0 = slice * DVS;
  const ScanSeq sq = seqs[s];

  // Initial state slice.
  for (int idx = tid; idx < DK * DVS; idx += 256) {
    const int kk = idx / DVS, c = idx % DVS;
    float v0 = 0.f;
    if (init) {
      const int64_t base = init_shared ? 0 : (int64_t)s * Hv * DK * DV;
      v0 = init[base + ((int64_t)h * DK + kk) * DV + c0 + c];
    }
    Ss[idx] = v0;
  }

  for (int ci = 0; ci < sq.nchunks; ++ci) {
    const int64_t gc = sq.chunk0 + ci;
    const ScanChunk ch = chunks[gc];
    const int n = ch.n;
    const float* blk = data + (gc * Hv + h) * kBlock;
    // (a) stage the chunk.
    for (int idx = tid; idx < C * (DK / 4); idx += 256) {
      const int i = idx / (DK / 4), c4 = (idx % (DK / 4)) * 4;
      const float4 wv = *reinterpret_cast<const float4*>(blk + kW + i * DK + c4);
      float4 qv = make_float4(0.f, 0.f, 0.f, 0.f), kv = qv;
      if (i < n) {
        const int64_t off = ((ch.t0 + i) * Hk + kh) * DK + c4;
        qv = *reinterpret_cast<const float4*>(q + off);
        kv = *reinterpret_cast<const float4*>(k + off);
      }
      *reinterpret_cast<float4*>(Ws + i * WP + c4) = wv;
      *reinterpret_cast<float4*>(Qs + i * WP + c4) = qv;
      *reinterpret_cast<float4*>(Ks + i * WP + c4) = kv;
    }
    for (int idx = tid; idx < C * (C / 4); idx += 256) {
      const int i = idx / (C / 4), c4 = (idx % (C / 4)) * 4;
      *reinterpret_cast<float4*>(Ps + i * PP + c4) =
          *reinterpret_cast<const float4*>(blk + kP + i * C + c4);
    }
    {
      const int i = tid >> 2, c4 = (tid & 3) * 4;
      *reinterpret_cast<float4*>(Us + i * DVS + c4) =
          *reinterpret_cast<const float4*>(blk + kU + i * DV + c0 + c4);
    }
    if (tid < C) {
      eg[tid] = blk[kEG + tid];
      egd[tid] = blk[kEGD + tid];
    }
    if (tid == 0) egl[0] = blk[kEGL];
    __syncthreads();

    // (b) X = W S, Y = Q S; D = U - X.
    const int r = tid >> 2, cg = (tid & 3) * 4;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f), y = x;
#pragma unroll 8
    for (int kk = 0; kk < DK; ++kk) {
      const float4 sv = *reinterpret_cast<const float4*>(Ss + kk * DVS + cg);
      const float w = Ws[r * WP + kk], qq = Qs[r * WP + kk];
      x.x = fmaf(w, sv.x, x.x); x.y = fmaf(w, sv.y, x.y);
      x.z = fmaf(w, sv.z, x.z); x.w = fmaf(w, sv.w, x.w);
      y.x = fmaf(qq, sv.x, y.x); y.y = fmaf(qq, sv.y, y.y);
      y.z = fmaf(qq, sv.z, y.z); y.w = fmaf(qq, sv.w, y.w);
    }
    {
      const float4 u = *reinterpret_cast<const float4*>(Us + r * DVS + cg);
      *reinterpret_cast<float4*>(Ds + r * DVS + cg) =
          make_float4(u.x - x.x, u.y - x.y, u.z - x.z, u.w - x.w);
    }
    __syncthreads();

    // (c) O = e^G o Y + P D  (rows < n).
    {
      const float e = eg[r];
      float4 o = make_float4(e * y.x, e * y.y, e * y.z, e * y.w);
      const float* prow = Ps + r * PP;
      for (int j = 0; j <= r; ++j) {
        const float p = prow[j];
        const float4 dv = *reinterpret_cast<const float4*>(Ds + j * DVS + cg);
        o.x = fmaf(p, dv.x, o.x); o.y = fmaf(p, dv.y, o.y);
        o.z = fmaf(p, dv.z, o.z); o.w = fmaf(p, dv.w, o.w);
      }
      if (r < n)
        *reinterpret_cast<float4*>(out + ((ch.t0 + r) * Hv + h) * DV + c0 + cg) = o;
    }
    // (d) S = e^{G_last} S + (e^{G_last-G} o K)^T D.
    {
      const int kk = tid >> 1, hc = (tid & 1) * 8;
      const float el = egl[0];
      float4 s0 = *reinterpret_cast<const float4*>(Ss + kk * DVS + hc);
      float4 s1 = *reinterpret_cast<const float4*>(Ss + kk * DVS + hc + 4);
      float4 a0 = make_float4(el * s0.x, el * s0.y, el * s0.z, el * s0.w);
      float4 a1 = make_float4(el * s1.x, el * s1.y, el * s1.z, el * s1.w);
      for (int j = 0; j < n; ++j) {
        const float kd = egd[j] * Ks[j * WP + kk];
        const float4 d0 = *reinterpret_cast<const float4*>(Ds + j * DVS + hc);
        const float4 d1 = *reinterpret_cast<const float4*>(Ds + j * DVS + hc + 4);
        a0.x = fmaf(kd, d0.x, a0.x); a0.y = fmaf(kd, d0.y, a0.y);
        a0.z = fmaf(kd, d0.z, a0.z); a0.w = fmaf(kd, d0.w, a0.w);
        a1.x = fmaf(kd, d1.x, a1.x); a1.y = fmaf(kd, d1.y, a1.y);
        a1.z = fmaf(kd, d1.z, a1.z); a1.w = fmaf(kd, d1.w, a1.w);
      }
      __syncthreads();  // every reader of the old S (step b) is done
      *reinterpret_cast<float4*>(Ss + kk * DVS + hc) = a0;
      *reinterpret_cast<float4*>(Ss + kk * DVS + hc + 4) = a1;
      if (capture_state && ci == sq.capture_chunk) {
        float* dst = capture_state + ((int64_t)h * DK + kk) * DV + c0 + hc;
        *reinterpret_cast<float4*>(dst) = a0;
        *reinterpret_cast<float4*>(dst + 4) = a1;
      }
    }
    __syncthreads();
  }
  if (final_state) {
    for (int idx = tid; idx < DK * DVS; idx += 256) {
      const int kk = idx / DVS, c = idx % DVS;
      final_state[(((int64_t)s * Hv + h) * DK + kk) * DV + c0 + c] = Ss[idx];
    }
  }
}

constexpr size_t kPrepSmem = sizeof(float) * (2 * C * KP + C * AP + 2 * C) + sizeof(double) * C;
constexpr size_t kCarrySmem =
    sizeof(float) * (3 * C * WP + C * PP + DK * DVS + 2 * C * DVS + 2 * C + 4);

}  // namespace

size_t delta_scan_workspace(int64_t total_tokens, int nseq, int Hv, int dk, int dv) {
  (void)dk;
  (void)dv;
  return layout(total_tokens, nseq, Hv).total;
}

int launch_delta_scan(const float* q, const float* k, const float* v, const float* g,
                      const float* beta, const int64_t* cu_host, int nseq, int Hk, int Hv, int dk,
                      int dv, const float* init, int init_shared, int64_t capture,
                      float* capture_state, float* final_state, float* out, void* ws,
                      size_t ws_bytes, cudaStream_t s) {
  CLEF_CHECK(dk == DK && dv == DV, CLEF_ERR_UNSUPPORTED, "delta_scan: dk and dv must be 128");
  const int64_t total = cu_host[nseq];
  const Layout l = layout(total, nseq, Hv);
  CLEF_CHECK(ws_bytes >= l.total, CLEF_ERR_INVALID, "delta_scan: workspace too small");
  // Chunk plan: 64-token chunks per sequence; a capture point starts a new chunk.
  std::vector<ScanSeq> seqs(nseq);
  std::vector<ScanChunk> chunks;
  chunks.reserve((size_t)l.max_chunks);
  for (int si = 0; si < nseq; ++si) {
    const int64_t a = cu_host[si], b = cu_host[si + 1];
    seqs[si].chunk0 = (int32_t)chunks.size();
    seqs[si].capture_chunk = -1;
    seqs[si].pad = 0;
    const int64_t cut = (capture > 0 && capture < b - a) ? a + capture : b;
    for (int64_t t = a; t < cut; t += C)
      chunks.push_back({t, (int32_t)std::min<int64_t>(C, cut - t), si});
    if (capture > 0) seqs[si].capture_chunk = (int32_t)chunks.size() - 1 - seqs[si].chunk0;
    for (int64_t t = cut; t < b; t += C)
      chunks.push_back({t, (int32_t)std::min<int64_t>(C, b - t), si});
    seqs[si].nchunks = (int32_t)chunks.size() - seqs[si].chunk0;
  }
  CLEF_CHECK((int64_t)chunks.size() <= l.max_chunks, CLEF_ERR_INVALID, "delta_scan: chunk plan");
  char* base = reinterpret_cast<char*>(ws);
  ScanSeq* seqs_d = reinterpret_cast<ScanSeq*>(base + l.seq_off);
  ScanChunk* chunks_d = reinterpret_cast<ScanChunk*>(base + l.chunk_off);
  float* data = reinterpret_cast<float*>(base + l.data_off);
  CLEF_CUDA(cudaMemcpyAsync(seqs_d, seqs.data(), sizeof(ScanSeq) * seqs.size(),
                            cudaMemcpyHostToDevice, s));
  CLEF_CUDA(cudaMemcpyAsync(chunks_d, chunks.data(), sizeof(ScanChunk) * chunks.size(),
                            cudaMemcpyHostToDevice, s));
  static bool attr_set[64] = {false};
  int dev = 0;
  CLEF_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    CLEF_CUDA(cudaFuncSetAttribute(delta_chunk_prep, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kPrepSmem));
    CLEF_CUDA(cudaFuncSetAttribute(delta_chunk_carry, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kCarrySmem));
    attr_set[dev] = true;
  }
  const dim3 g1((unsigned)chunks.size(), (unsigned)Hv);
  delta_chunk_prep<<<g1, 256, kPrepSmem, s>>>(q, k, v, g, beta, chunks_d, Hk, Hv, data);
  int rc = launch_status("delta_chunk_prep");
  if (rc) return rc;
  const unsigned g2 = (unsigned)(nseq * Hv * SLICES);
  delta_chunk_carry<<<g2, 256, kCarrySmem, s>>>(q, k, seqs_d, chunks_d, data, Hk, Hv, init,
                                                init_shared, capture_state, final_state, out);
  return launch_status("delta_chunk_carry");
}

}  // namespace clef

using namespace clef;

extern "C" {

size_t clef_delta_scan_workspace_size(int64_t total_tokens, int32_t nseq, int32_t Hv, int32_t dk,
                                      int32_t dv) {
  if (total_tokens < 0 || nseq <= 0 || Hv <= 0) return 0;
  return delta_scan_workspace(total_tokens, nseq, Hv, dk, dv);
}

int clef_delta_scan(const float* q, const float* k, const float* v, const float* g,
                    const float* beta, int64_t T, int32_t Hk, int32_t Hv, int32_t dk, int32_t dv,
                    const int64_t* cu_seqlens, int32_t nseq, const float* init_state,
                    int32_t init_shared, int64_t capture, float* capture_state, float* final_state,
                    float* out, void* workspace, size_t workspace_bytes, void* stream) {
  CLEF_CHECK(q && k && v && g && beta && out && workspace, CLEF_ERR_INVALID,
             "delta_scan: null pointer");
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
  CLEF_CHECK(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out) % 16 == 0,
             CLEF_ERR_INVALID, "delta_scan: q, k, v, out must be 16-byte aligned");
  CLEF_CHECK(((uintptr_t)workspace & 255) == 0, CLEF_ERR_INVALID,
             "delta_scan: workspace must be 256-byte aligned");
  return launch_delta_scan(q, k, v, g, beta, cu.data(), nseq, Hk, Hv, dk, dv, init_state,
                           init_shared, capture, capture_state, final_state, out, workspace,
                           workspace_bytes, as_stream(stream));
}

}  // extern "C"
