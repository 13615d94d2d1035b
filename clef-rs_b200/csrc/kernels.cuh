// kernels.cuh — launchers shared between the operator entry points and the
// engine. All take device pointers and a stream and return a clef_status.
#pragma once

#include "common.cuh"

namespace clef {

// Packed-sequence description used by the varlen kernels: cu_seqlens holds
// nseq + 1 token offsets (device memory, int64).
// When cu_seqlens is set, the int32 query-block offsets (64-row blocks) of
// the attention kernel follow it in the same buffer:
// (const int32_t*)(cu_seqlens + nseq + 1), nseq + 1 entries, total `qblocks`.
struct SeqPack {
  const int64_t* cu_seqlens = nullptr;  // device, nseq + 1 entries; NULL = one sequence
  int32_t nseq = 1;
  int64_t total = 0;
  int64_t qblocks = 0;
};

// ---- pointwise.cu ----------------------------------------------------------
// out_dtype: CLEF_F32, CLEF_BF16, or kOutBF16Split (out [rows, 2 * width]
// BF16: hi = bf16(x) in columns [0, width), lo = bf16(x - hi) in [width, 2 width)).
constexpr int kOutBF16Split = 2;
int launch_rmsnorm(const float* x, const float* w, int64_t rows, int width, float eps,
                   int out_dtype, void* out, cudaStream_t s);
int launch_conv4(const float* x, int64_t ldx, const float* hist, int hist_rows, const float* w,
                 int64_t T, int width, float* out, cudaStream_t s);
// DeltaNet prologue over packed sequences; `hist` [hist_rows, qkv width] is
// the conv history every sequence continues from (NULL = zeros).
int launch_delta_prologue(const float* proj, int64_t ldp, int a_col, int b_col, const float* hist,
                          int hist_rows, const float* conv_w, const float* dt_bias,
                          const float* a_log, const SeqPack& pack, int Hk, int Hv, int dk, int dv,
                          float* q, float* k, float* v, float* g, float* beta, cudaStream_t s);
// Same with the BF16 projection rows of the engine (history rows stay F32).
int launch_delta_prologue(const uint16_t* proj, int64_t ldp, int a_col, int b_col, const float* hist,
                          int hist_rows, const float* conv_w, const float* dt_bias,
                          const float* a_log, const SeqPack& pack, int Hk, int Hv, int dk, int dv,
                          float* q, float* k, float* v, float* g, float* beta, cudaStream_t s);
// y[t, h*dv + i] = bf16(rms(o) * w * silu(z)) for each v-head (F32 math).
int launch_delta_epilogue(const float* o, const uint16_t* z, int64_t ldz, const float* w, float eps,
                          int64_t T, int Hv, int dv, uint16_t* y, cudaStream_t s);
// Same from F32 z rows, y stored as the split BF16 pair [T, 2 * Hv * 128].
int launch_delta_epilogue_split(const float* o, const float* z, int64_t ldz, const float* w, float eps,
                                int64_t T, int Hv, uint16_t* y, cudaStream_t s);
// Attention prologue: q/k RMSNorm (offset weights already +1) and partial
// RoPE from the fused BF16 projection; positions = offset + index in sequence.
int launch_attention_prologue(const uint16_t* proj, int64_t ldp, const float* qw, const float* kw,
                              float eps, const SeqPack& pack, int64_t pos_offset, int H, int Hkv,
                              int d, int rot, const float* inv_freq_dev, uint16_t* q_out,
                              uint16_t* k_out, cudaStream_t s);
// Same from the F32 projection rows of the engine's split precision.
int launch_attention_prologue(const float* proj, int64_t ldp, const float* qw, const float* kw,
                              float eps, const SeqPack& pack, int64_t pos_offset, int H, int Hkv,
                              int d, int rot, const float* inv_freq_dev, uint16_t* q_out,
                              uint16_t* k_out, cudaStream_t s);
// y [T, 2 * H * d] = split BF16 pair of o [T, H, d] * sigmoid(gate[t*g_ts + h*g_hs + e]).
int launch_gate_split(const float* o, const float* gate, int64_t g_ts, int64_t g_hs, int H, int d, int64_t T,
                      uint16_t* y, cudaStream_t s);
int launch_embed(const uint16_t* table, const int32_t* ids, int64_t T, int hidden, float* h,
                 cudaStream_t s);
// Final RMSNorm of each sequence's last row and the linear schema head.
int launch_head(const float* h, const float* norm_w, float eps, const SeqPack& pack, int hidden,
                const float* head_w, int n_out, float* logits, cudaStream_t s);
// Gathers rows [r0, r0+count) of a [T, ncols] BF16/F32 matrix (row stride ld)
// into dst [count, ncols].
int launch_copy_rows(const void* src, int64_t ld, int64_t r0, int64_t count, int64_t ncols,
                     int elem, void* dst, int64_t ldd, cudaStream_t s);
// dst rows (F32) = widened BF16 rows [r0, r0 + count) of src.
int launch_rows_bf16_to_f32(const uint16_t* src, int64_t ld, int64_t r0, int64_t count, int64_t ncols, float* dst,
                            int64_t ldd, cudaStream_t s);

// ---- delta_scan.cu ----------------------------------------------------------
// Pipelined scan (prep + carry kernels): workspace = offsets tables + the
// per-chunk tile images; a plan uploads the tables once and can be reused by
// every DeltaNet layer of a pack.
struct ScanPlan {
  void* ws = nullptr;
  int nseq = 0;
  int64_t nchunks = 0, total = 0;
  int Hk = 0, Hv = 0;
};
size_t delta_scan_workspace(int64_t total_tokens, int nseq, int Hk, int Hv);
int delta_scan_plan(const int64_t* cu_host, int nseq, int Hk, int Hv, void* ws, size_t ws_bytes,
                    cudaStream_t s, ScanPlan* plan);
int launch_delta_scan_planned(const ScanPlan& plan, const float* q, const float* k, const float* v,
                              const float* g, const float* beta, const float* init, int init_shared,
                              int64_t capture, float* capture_state, float* final_state, float* out,
                              cudaStream_t s);
// cu_host: host int64 [nseq+1]; builds a plan in `ws` and launches.
int launch_delta_scan(const float* q, const float* k, const float* v, const float* g,
                      const float* beta, const int64_t* cu_host, int nseq, int Hk, int Hv, int dk,
                      int dv, const float* init, int init_shared, int64_t capture,
                      float* capture_state, float* final_state, float* out, void* ws,
                      size_t ws_bytes, cudaStream_t s);
// Fused single-pass scan with the offsets already on the device (null = one
// sequence of `total`); needs no other workspace.
size_t delta_scan_fused_workspace(int nseq);
int launch_delta_scan_dev(const float* q, const float* k, const float* v, const float* g,
                          const float* beta, const int64_t* cu_dev, int64_t total, int nseq, int Hk,
                          int Hv, const float* init, int init_shared, int64_t capture,
                          float* capture_state, float* final_state, float* out, cudaStream_t s);

// ---- rng.cu -----------------------------------------------------------------
// Philox4x32-10 counter-based normal / uniform generator, deterministic in
// (seed, stream, element index) on host and device.
uint64_t name_stream(const char* name);
int launch_fill_normal_bf16(uint16_t* dst, int64_t n, uint64_t seed, uint64_t stream, float mean,
                            float std, cudaStream_t s);
void host_fill(float* dst, int64_t n, uint64_t seed, uint64_t stream, int kind, float a, float b);
enum HostFill { kFillNormal = 0, kFillUniform = 1 };

// ---- gemm.cu ----------------------------------------------------------------
// kEpiSwiGLUSplit stores the SwiGLU product as split BF16 halves: hi in
// columns [0, N), lo = bf16(y - hi) in [N, 2N) (ldo >= 2N).
enum GemmEpi { kEpiBF16 = 0, kEpiF32 = 1, kEpiAddF32 = 2, kEpiSwiGLU = 3, kEpiSwiGLUSplit = 4 };
// out[M, N] (ldo) = epilogue(X[M, K] * W[N, K]^T). For kEpiSwiGLU, W2 is the
// up matrix and W the gate matrix (both [N, K]); out is BF16. With x_split,
// X is [M, 2K]: the split BF16 pair of each activation (hi in columns [0, K),
// lo in [K, 2K)), and the result is (hi + lo) W^T.
int launch_gemm(const uint16_t* X, const uint16_t* W, const uint16_t* W2, int64_t M, int N, int K,
                int epi, void* out, int64_t ldo, cudaStream_t s, int x_split = 0);

// ---- attention_tc.cu --------------------------------------------------------
// Packed sequences for the tcgen05 attention: token offsets, padded V^T column
// offsets (each sequence starts at a multiple of 64 keys so every TMA
// coordinate is 16-byte aligned), 128-row query-block offsets and 64-key
// block offsets. All device arrays; cu == null means one sequence of `total`.
struct SeqPackVT {
  const int64_t* cu = nullptr;
  const int64_t* cu_vt = nullptr;
  const int32_t* cu_qb = nullptr;
  const int32_t* cu_kb = nullptr;
  int nseq = 1;
  int64_t total = 0, qblocks = 0, kblocks = 0;
};
struct AttnTcArgs {
  int H = 0, Hkv = 0;
  float scale = 0.0625f;
  const uint16_t* q = nullptr;   // [rows_q, H, 256]
  int64_t rows_q = 0;
  const uint16_t* k = nullptr;   // [rows_k, Hkv, 256] own keys
  int64_t rows_k = 0;
  const uint16_t* vt = nullptr;  // [Hkv * 256, vt_pitch] own values, transposed
  int64_t vt_cols = 0, vt_pitch = 0;
  int64_t prefix_len = 0;        // shared prefix keys every sequence sees first
  const uint16_t* pk = nullptr;  // [prefix_len, Hkv, 256]
  const uint16_t* pvt = nullptr; // [Hkv * 256, pvt_pitch]
  int64_t pvt_pitch = 0;
  void* out = nullptr;           // F32 (gate null) or BF16 o * sigmoid(gate)
  int64_t o_ts = 0, o_hs = 0;
  const uint16_t* gate = nullptr;
  int64_t g_ts = 0, g_hs = 0;
};
int launch_attention_tc(const AttnTcArgs& a, const SeqPackVT& pk, cudaStream_t s);
// vt[kvh * 256 + e][cu_vt[s] + j] = v[(cu[s] + j) * v_ts + kvh * v_hs + e].
int launch_transpose_v(const uint16_t* v, int64_t v_ts, int64_t v_hs, const SeqPackVT& pk, int Hkv,
                       uint16_t* vt, int64_t vt_pitch, cudaStream_t s);
int launch_transpose_v(const float* v, int64_t v_ts, int64_t v_hs, const SeqPackVT& pk, int Hkv,
                       uint16_t* vt, int64_t vt_pitch, cudaStream_t s);
int attention_tc_device_error(int* code);

}  // namespace clef
