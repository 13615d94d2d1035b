// engine.cu — the hybrid-backbone prefill engine behind clef_engine_*.
//
// Replaces Backbone::{load, forward, prefill, prefill_embedded}
// (crates/core/src/models/qwen.rs:193-426). Differences of design, not of
// result:
//   - Sequences are packed back to back ("varlen") so every projection GEMM
//     runs once per layer over all tokens of all requests in the pack
//     (M = total tokens), while the causal conv, the DeltaNet scan and the
//     attention respect sequence boundaries through offset tables.
//   - Projections that read the same input are fused into one weight matrix
//     whose named views are the checkpoint tensors: in_proj_qkv | in_proj_z |
//     in_proj_a | in_proj_b (one BF16-output GEMM feeding the DeltaNet
//     prologue and epilogue) and q_proj | k_proj | v_proj (one BF16-output GEMM).
//   - Residual adds are fused into the out_proj / o_proj / down_proj GEMM
//     epilogues; SwiGLU is fused into the gate/up GEMM epilogue.
//   - The prefix state (PrefixState, qwen.rs:153-190) lives on the device:
//     recurrent S and the last <= 3 conv rows per DeltaNet layer, K/V rows per
//     attention layer, and the captured final-normed hidden rows.
// The residual stream is F32 and projections are BF16 with F32 accumulation.
// Two precisions (clef_engine_set_precision):
//   CLEF_PRECISION_BF16   every GEMM operand is BF16, the fused in-projection
//                         and attention q/k/v projection outputs are BF16;
//   CLEF_PRECISION_SPLIT  every GEMM activation operand is a split BF16 pair
//                         (hi + lo, twice the tensor work) and the projection
//                         outputs are F32, so the projections match F32
//                         arithmetic to ~2^-17; only the attention's q, k, v
//                         and probabilities stay single BF16 operands.
// Everything between the GEMMs (norms, conv, gates, scan, gating) is F32 in both.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "kernels.cuh"

using namespace clef;

namespace {

std::string lp(int i) { return "model.language_model.layers." + std::to_string(i); }

enum InitKind { kInitNormal, kInitOnePlusNormal, kInitALog, kInitDtBias };

struct NamedTensor {
  std::vector<int64_t> shape;
  int64_t count = 0;
  bool bf16 = false;
  void* dev = nullptr;
  bool loaded = false;
  InitKind init = kInitNormal;
  bool offset = false;   // effective weight = 1 + w (offset RMSNorm)
  float* eff = nullptr;  // device effective weight for offset norms
};

struct LayerW {
  bool attention = false;
  uint16_t *w_in = nullptr, *w_out = nullptr;  // DeltaNet
  int n_in = 0;
  float *conv = nullptr, *dt = nullptr, *alog = nullptr, *dnorm = nullptr;
  uint16_t *w_att = nullptr, *w_o = nullptr;  // attention
  int n_att = 0;
  float *qn = nullptr, *kn = nullptr;
  float *in_eff = nullptr, *post_eff = nullptr;
  uint16_t *w_gate = nullptr, *w_up = nullptr, *w_down = nullptr;
};

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

constexpr int kStages = 9;
enum Stage { kStEmbed, kStNorm, kStGemm, kStDeltaPro, kStDeltaScan, kStDeltaEpi, kStAttnPro, kStAttn, kStHead };

}  // namespace

// Layout descriptor in the first 256 bytes of a prefix's device allocation:
// travels with every export, so an import can tell a copy made for another
// layout or token count from a matching one.
struct PrefixDescriptor {
  uint64_t magic = 0x3158464650464c43ull;  // "CLEFPFX1"
  int64_t tokens = 0;
  int64_t vt_pitch = 0;
  uint64_t span = 0;
  int32_t layers = 0, hidden = 0, value_heads = 0, kv_width = 0, qkv_width = 0, pad = 0;
  uint64_t attention_layers[2] = {0, 0};  // bit i: layer i is full attention
  bool operator==(const PrefixDescriptor& o) const { return memcmp(this, &o, sizeof(*this)) == 0; }
};
static_assert(sizeof(PrefixDescriptor) <= 256, "prefix descriptor exceeds its slot");

struct clef_prefix {
  int device = 0;
  int64_t tokens = 0;
  int hidden = 0;
  int64_t vt_pitch = 0;
  void* blob = nullptr;
  uint64_t bytes = 0;       // logical state bytes
  uint64_t span = 0;        // bytes of the device allocation (layout of the engine config)
  bool filled = false;      // set by a capture or a successful import
  PrefixDescriptor desc;    // host copy of the descriptor at the start of `blob`
  float* hidden_rows = nullptr;  // [tokens, hidden]
  struct Layer {
    bool full = false;
    uint16_t* k = nullptr;   // [tokens, Hkv, d] (post-RoPE keys)
    uint16_t* vt = nullptr;  // [Hkv * d, vt_pitch] values, transposed (keys contiguous)
    float* S = nullptr;     // [Hv, 128, 128]
    float* hist = nullptr;  // [hist_rows, qkv width]
    int hist_rows = 0;
  };
  std::vector<Layer> layers;
};

struct clef_engine {
  clef_config cfg;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::map<std::string, NamedTensor> tensors;
  std::vector<LayerW> layers;
  uint16_t* embed = nullptr;
  float* final_eff = nullptr;
  float* head_w = nullptr;
  void* wblob = nullptr;
  float* inv_freq = nullptr;
  bool finalized = false;
  int precision = CLEF_PRECISION_BF16;
  int sm_limit = 0;  // SMs the persistent kernels of a prefill may occupy (0 = all)
  int arena_precision = -1;  // precision the activation arena was sized for
  std::atomic<int> cancel{0};
  // geometry
  int key = 0, value = 0, qkv_w = 0, n_in = 0, att_n = 0, att_kv = 0, n_att = 0;
  int64_t max_pack = 65536;
  // activations
  void* arena = nullptr;
  size_t arena_bytes = 0;
  int64_t cap_tokens = 0, cap_seqs = 0;
  int32_t* ids_d = nullptr;
  int64_t* meta_d = nullptr;
  float *h = nullptr, *proj = nullptr, *dq = nullptr, *dk = nullptr, *dv = nullptr, *dg = nullptr,
        *db = nullptr, *dout = nullptr, *logits_d = nullptr;
  uint16_t *u = nullptr, *y = nullptr, *qatt = nullptr, *katt = nullptr, *act = nullptr;
  uint16_t* vt = nullptr;  // [Hkv * d, vt_pitch] transposed values of the pack
  int64_t vt_pitch = 0;
  void* scan_ws = nullptr;
  size_t scan_ws_bytes = 0;
  // profiling
  bool profiling = false;
  float stage_ms[kStages] = {0};
  std::vector<cudaEvent_t> ev_pool;
  std::vector<std::pair<int, int>> ev_used;  // (stage, first event index)
  int64_t launches = 0;  // kernels issued by prefill calls (cumulative)
};

namespace {

void declare(clef_engine* e, const std::string& name, std::vector<int64_t> shape, bool bf16,
             InitKind init = kInitNormal, bool offset = false) {
  NamedTensor t;
  t.shape = shape;
  t.count = 1;
  for (auto s : shape) t.count *= s;
  t.bf16 = bf16;
  t.init = init;
  t.offset = offset;
  e->tensors[name] = t;
}

int build_layout(clef_engine* e) {
  const clef_config& c = e->cfg;
  const int64_t h = c.hidden_size;
  e->key = c.linear_num_key_heads * c.linear_key_head_dim;
  e->value = c.linear_num_value_heads * c.linear_value_head_dim;
  e->qkv_w = 2 * e->key + e->value;
  e->n_in = e->qkv_w + e->value + 2 * c.linear_num_value_heads;
  e->n_in = (e->n_in + 63) / 64 * 64;
  e->att_n = c.num_attention_heads * c.head_dim;
  e->att_kv = c.num_key_value_heads * c.head_dim;
  e->n_att = 2 * e->att_n + 2 * e->att_kv;
  declare(e, "model.language_model.embed_tokens.weight", {c.vocab_size, h}, true);
  declare(e, "model.language_model.norm.weight", {h}, false, kInitNormal, true);
  if (c.head_outputs) declare(e, "clef.head.weight", {c.head_outputs, h}, false);
  for (int i = 0; i < c.num_hidden_layers; ++i) {
    const std::string p = lp(i);
    declare(e, p + ".input_layernorm.weight", {h}, false, kInitNormal, true);
    declare(e, p + ".post_attention_layernorm.weight", {h}, false, kInitNormal, true);
    declare(e, p + ".mlp.gate_proj.weight", {c.intermediate_size, h}, true);
    declare(e, p + ".mlp.up_proj.weight", {c.intermediate_size, h}, true);
    declare(e, p + ".mlp.down_proj.weight", {h, c.intermediate_size}, true);
    if (c.layer_types[i]) {
      declare(e, p + ".self_attn.q_proj.weight", {2LL * e->att_n, h}, true);
      declare(e, p + ".self_attn.k_proj.weight", {e->att_kv, h}, true);
      declare(e, p + ".self_attn.v_proj.weight", {e->att_kv, h}, true);
      declare(e, p + ".self_attn.o_proj.weight", {h, e->att_n}, true);
      declare(e, p + ".self_attn.q_norm.weight", {c.head_dim}, false, kInitNormal, true);
      declare(e, p + ".self_attn.k_norm.weight", {c.head_dim}, false, kInitNormal, true);
    } else {
      declare(e, p + ".linear_attn.in_proj_qkv.weight", {e->qkv_w, h}, true);
      declare(e, p + ".linear_attn.in_proj_z.weight", {e->value, h}, true);
      declare(e, p + ".linear_attn.in_proj_a.weight", {c.linear_num_value_heads, h}, true);
      declare(e, p + ".linear_attn.in_proj_b.weight", {c.linear_num_value_heads, h}, true);
      declare(e, p + ".linear_attn.out_proj.weight", {h, e->value}, true);
      declare(e, p + ".linear_attn.conv1d.weight", {e->qkv_w, 1, c.linear_conv_kernel_dim}, false);
      declare(e, p + ".linear_attn.dt_bias", {c.linear_num_value_heads}, false, kInitDtBias);
      declare(e, p + ".linear_attn.A_log", {c.linear_num_value_heads}, false, kInitALog);
      declare(e, p + ".linear_attn.norm.weight", {c.linear_value_head_dim}, false,
              kInitOnePlusNormal);
    }
  }
  // One device blob: fused BF16 matrices (with zero padding rows), then F32
  // tensors and the effective offset-norm weights.
  size_t bytes = 0;
  auto reserve = [&](size_t n) {
    const size_t off = bytes;
    bytes = a256(bytes + n);
    return off;
  };
  std::vector<size_t> in_off(c.num_hidden_layers), att_off(c.num_hidden_layers);
  for (int i = 0; i < c.num_hidden_layers; ++i) {
    if (c.layer_types[i]) att_off[i] = reserve((size_t)e->n_att * h * 2);
    else in_off[i] = reserve((size_t)e->n_in * h * 2);
  }
  std::map<std::string, size_t> off;
  for (auto& kv : e->tensors) {
    const std::string& n = kv.first;
    const bool fused = n.find("in_proj_") != std::string::npos ||
                       n.find(".q_proj.") != std::string::npos ||
                       n.find(".k_proj.") != std::string::npos ||
                       n.find(".v_proj.") != std::string::npos;
    if (!fused) off[n] = reserve((size_t)kv.second.count * (kv.second.bf16 ? 2 : 4));
    if (kv.second.offset) off[n + "#eff"] = reserve((size_t)kv.second.count * 4);
  }
  const size_t inv_off = reserve(sizeof(float) * 128);
  if (cudaMalloc(&e->wblob, bytes) != cudaSuccess)
    return fail(CLEF_ERR_NOMEM, "engine: weight allocation of " + std::to_string(bytes) + " bytes");
  // Zero padding rows. The memset is ordered on the engine's (non-blocking)
  // stream and completed here: a legacy-stream cudaMemset could still be
  // running when the first weights are written on the engine's stream.
  if (cudaMemsetAsync(e->wblob, 0, bytes, e->stream) != cudaSuccess ||
      cudaStreamSynchronize(e->stream) != cudaSuccess)
    return fail(CLEF_ERR_CUDA, "engine: memset");
  char* base = reinterpret_cast<char*>(e->wblob);
  for (auto& kv : e->tensors) {
    auto it = off.find(kv.first);
    if (it != off.end()) kv.second.dev = base + it->second;
    auto ie = off.find(kv.first + "#eff");
    if (ie != off.end()) kv.second.eff = reinterpret_cast<float*>(base + ie->second);
  }
  e->layers.resize(c.num_hidden_layers);
  for (int i = 0; i < c.num_hidden_layers; ++i) {
    const std::string p = lp(i);
    LayerW& L = e->layers[i];
    L.attention = c.layer_types[i] != 0;
    auto T = [&](const std::string& n) -> NamedTensor& { return e->tensors.at(p + n); };
    if (L.attention) {
      L.w_att = reinterpret_cast<uint16_t*>(base + att_off[i]);
      L.n_att = e->n_att;
      T(".self_attn.q_proj.weight").dev = L.w_att;
      T(".self_attn.k_proj.weight").dev = L.w_att + (size_t)2 * e->att_n * h;
      T(".self_attn.v_proj.weight").dev = L.w_att + (size_t)(2 * e->att_n + e->att_kv) * h;
      L.w_o = (uint16_t*)T(".self_attn.o_proj.weight").dev;
      L.qn = T(".self_attn.q_norm.weight").eff;
      L.kn = T(".self_attn.k_norm.weight").eff;
    } else {
      L.w_in = reinterpret_cast<uint16_t*>(base + in_off[i]);
      L.n_in = e->n_in;
      T(".linear_attn.in_proj_qkv.weight").dev = L.w_in;
      T(".linear_attn.in_proj_z.weight").dev = L.w_in + (size_t)e->qkv_w * h;
      T(".linear_attn.in_proj_a.weight").dev = L.w_in + (size_t)(e->qkv_w + e->value) * h;
      T(".linear_attn.in_proj_b.weight").dev =
          L.w_in + (size_t)(e->qkv_w + e->value + c.linear_num_value_heads) * h;
      L.w_out = (uint16_t*)T(".linear_attn.out_proj.weight").dev;
      L.conv = (float*)T(".linear_attn.conv1d.weight").dev;
      L.dt = (float*)T(".linear_attn.dt_bias").dev;
      L.alog = (float*)T(".linear_attn.A_log").dev;
      L.dnorm = (float*)T(".linear_attn.norm.weight").dev;
    }
    L.in_eff = T(".input_layernorm.weight").eff;
    L.post_eff = T(".post_attention_layernorm.weight").eff;
    L.w_gate = (uint16_t*)T(".mlp.gate_proj.weight").dev;
    L.w_up = (uint16_t*)T(".mlp.up_proj.weight").dev;
    L.w_down = (uint16_t*)T(".mlp.down_proj.weight").dev;
  }
  e->embed = (uint16_t*)e->tensors.at("model.language_model.embed_tokens.weight").dev;
  e->final_eff = e->tensors.at("model.language_model.norm.weight").eff;
  if (c.head_outputs) e->head_w = (float*)e->tensors.at("clef.head.weight").dev;
  e->inv_freq = reinterpret_cast<float*>(base + inv_off);
  return CLEF_OK;
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, int64_t n, uint16_t* __restrict__ dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = f2bf(src[i]);
}
__global__ void bf16_to_f32_kernel(const uint16_t* __restrict__ src, int64_t n, float* __restrict__ dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = bf2f(src[i]);
}
__global__ void one_plus_kernel(const float* __restrict__ src, int64_t n, float* __restrict__ dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i] + 1.f;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Per-pack device offsets for n1 = sequences + 1 entries: int64 cu | int32
// 64-row q-blocks | (8-byte aligned) int64 padded V^T offsets | int32 128-row
// q-blocks | int32 64-key blocks.
size_t meta_vt_offset(size_t n1) { return (n1 * (sizeof(int64_t) + sizeof(int32_t)) + 7) / 8 * 8; }
size_t meta_bytes(size_t n1) {
  return meta_vt_offset(n1) + n1 * (sizeof(int64_t) + 2 * sizeof(int32_t)) + 64;
}

int ensure_capacity(clef_engine* e, int64_t tokens, int64_t seqs) {
  if (tokens <= e->cap_tokens && seqs <= e->cap_seqs && e->arena && e->arena_precision == e->precision)
    return CLEF_OK;
  const int x2 = e->precision == CLEF_PRECISION_SPLIT ? 2 : 1;  // split operands: hi | lo
  const clef_config& c = e->cfg;
  tokens = std::max(tokens, e->cap_tokens);
  seqs = std::max(seqs, e->cap_seqs);
  const int64_t M = tokens;
  const int hid = c.hidden_size;
  const int hv = c.linear_num_value_heads;
  size_t b = 0;
  std::vector<size_t> o;
  auto take = [&](size_t n) {
    o.push_back(b);
    b = a256(b + n);
  };
  take(sizeof(int32_t) * M);                              // 0 ids
  take(meta_bytes((size_t)seqs + 1));                     // 1 meta
  take(sizeof(float) * M * hid);                          // 2 h
  take(sizeof(uint16_t) * x2 * M * std::max(e->n_in, e->n_att));  // 3 proj (BF16, or F32 when split)
  take(sizeof(float) * M * e->key);                       // 4 dq
  take(sizeof(float) * M * e->key);                       // 5 dk
  take(sizeof(float) * M * e->value);                     // 6 dv
  take(sizeof(float) * M * hv);                           // 7 dg
  take(sizeof(float) * M * hv);                           // 8 db
  take(sizeof(float) * M * std::max(e->value, e->att_n));  // 9 dout (scan out; F32 attention out when split)
  take(sizeof(uint16_t) * x2 * M * hid);                  // 10 u
  take(sizeof(uint16_t) * x2 * M * std::max(e->value, e->att_n));  // 11 y
  take(sizeof(uint16_t) * M * e->att_n);                  // 12 qatt
  take(sizeof(uint16_t) * M * e->att_kv);                 // 13 katt
  take(sizeof(uint16_t) * x2 * M * c.intermediate_size);  // 14 act
  take(sizeof(float) * seqs * std::max(1, c.head_outputs));  // 15 logits
  const size_t ws = delta_scan_workspace(M, (int)seqs, c.linear_num_key_heads, hv);
  take(ws);                                               // 16 scan ws
  const int64_t vt_pitch = (M + 64 * seqs + 63) / 64 * 64;
  take(sizeof(uint16_t) * (size_t)vt_pitch * e->att_kv);  // 17 V^T
  if (e->arena) cudaFree(e->arena);
  e->arena = nullptr;
  if (cudaMalloc(&e->arena, b) != cudaSuccess)
    return fail(CLEF_ERR_NOMEM, "engine: activation allocation of " + std::to_string(b) + " bytes");
  char* p = reinterpret_cast<char*>(e->arena);
  e->ids_d = (int32_t*)(p + o[0]);
  e->meta_d = (int64_t*)(p + o[1]);
  e->h = (float*)(p + o[2]);
  e->proj = (float*)(p + o[3]);
  e->dq = (float*)(p + o[4]);
  e->dk = (float*)(p + o[5]);
  e->dv = (float*)(p + o[6]);
  e->dg = (float*)(p + o[7]);
  e->db = (float*)(p + o[8]);
  e->dout = (float*)(p + o[9]);
  e->u = (uint16_t*)(p + o[10]);
  e->y = (uint16_t*)(p + o[11]);
  e->qatt = (uint16_t*)(p + o[12]);
  e->katt = (uint16_t*)(p + o[13]);
  e->act = (uint16_t*)(p + o[14]);
  e->logits_d = (float*)(p + o[15]);
  e->scan_ws = p + o[16];
  e->vt = (uint16_t*)(p + o[17]);
  e->vt_pitch = vt_pitch;
  e->scan_ws_bytes = ws;
  e->arena_bytes = b;
  e->arena_precision = e->precision;
  e->cap_tokens = tokens;
  e->cap_seqs = seqs;
  return CLEF_OK;
}

// Stage timing (only when profiling is enabled).
struct StageTimer {
  clef_engine* e;
  int stage;
  int idx = -1;
  StageTimer(clef_engine* e_, int s) : e(e_), stage(s) {
    if (!e->profiling) return;
    idx = (int)e->ev_used.size() * 2;
    while ((int)e->ev_pool.size() < idx + 2) {
      cudaEvent_t ev;
      cudaEventCreate(&ev);
      e->ev_pool.push_back(ev);
    }
    cudaEventRecord(e->ev_pool[idx], e->stream);
    e->ev_used.push_back({stage, idx});
  }
  ~StageTimer() {
    if (idx >= 0) cudaEventRecord(e->ev_pool[idx + 1], e->stream);
  }
};

#define STAGE(st) StageTimer timer_##__LINE__(e, st)
#define RC(x)            \
  do {                   \
    int rc_ = (x);       \
    if (rc_) return rc_; \
  } while (0)

int alloc_prefix(clef_engine* e, int64_t tokens, clef_prefix** out) {
  const clef_config& c = e->cfg;
  clef_prefix* p = new clef_prefix();
  p->device = e->device;
  p->tokens = tokens;
  p->hidden = c.hidden_size;
  size_t b = 0;
  std::vector<size_t> o;
  auto take = [&](size_t n) {
    o.push_back(b);
    b = a256(b + n);
  };
  take(sizeof(PrefixDescriptor));
  take(sizeof(float) * tokens * c.hidden_size);
  uint64_t logical = sizeof(float) * tokens * c.hidden_size;
  p->vt_pitch = (tokens + 63) / 64 * 64;
  p->layers.resize(c.num_hidden_layers);
  for (int i = 0; i < c.num_hidden_layers; ++i) {
    if (c.layer_types[i]) {
      take(sizeof(uint16_t) * tokens * e->att_kv);
      take(sizeof(uint16_t) * p->vt_pitch * e->att_kv);
      logical += 2 * sizeof(uint16_t) * tokens * e->att_kv;
    } else {
      const int64_t rows = std::min<int64_t>(tokens, 3);
      take(sizeof(float) * (size_t)c.linear_num_value_heads * 128 * 128);
      take(sizeof(float) * 3 * e->qkv_w);
      logical += sizeof(float) * ((size_t)c.linear_num_value_heads * 128 * 128 + rows * e->qkv_w);
    }
  }
  if (cudaMalloc(&p->blob, b) != cudaSuccess) {
    delete p;
    return fail(CLEF_ERR_NOMEM, "prefix: allocation of " + std::to_string(b) + " bytes");
  }
  p->span = b;
  char* base = reinterpret_cast<char*>(p->blob);
  int k = 1;  // o[0]: the descriptor
  p->hidden_rows = (float*)(base + o[k++]);
  for (int i = 0; i < c.num_hidden_layers; ++i) {
    auto& L = p->layers[i];
    L.full = c.layer_types[i] != 0;
    if (L.full) {
      L.k = (uint16_t*)(base + o[k++]);
      L.vt = (uint16_t*)(base + o[k++]);
    } else {
      L.S = (float*)(base + o[k++]);
      L.hist = (float*)(base + o[k++]);
      L.hist_rows = (int)std::min<int64_t>(tokens, 3);
    }
  }
  p->bytes = logical;
  PrefixDescriptor& d = p->desc;
  d.tokens = tokens;
  d.vt_pitch = p->vt_pitch;
  d.span = p->span;
  d.layers = c.num_hidden_layers;
  d.hidden = c.hidden_size;
  d.value_heads = c.linear_num_value_heads;
  d.kv_width = e->att_kv;
  d.qkv_width = e->qkv_w;
  for (int i = 0; i < c.num_hidden_layers; ++i)
    if (c.layer_types[i]) d.attention_layers[i / 64] |= 1ull << (i % 64);
  // Pageable source: the call returns once the bytes are staged, so the host
  // copy in `p` may change afterwards; the device copy is stream-ordered.
  if (cudaMemcpyAsync(p->blob, &d, sizeof(d), cudaMemcpyHostToDevice, e->stream) != cudaSuccess) {
    cudaFree(p->blob);
    delete p;
    return fail(CLEF_ERR_CUDA, "prefix: descriptor copy");
  }
  *out = p;
  return CLEF_OK;
}

// Adds the elapsed time of every recorded (start, end) event pair to its
// stage; the events must have completed (the caller synchronised).
void collect_stage_times(clef_engine* e) {
  for (auto& x : e->ev_used) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, e->ev_pool[x.second], e->ev_pool[x.second + 1]) == cudaSuccess)
      e->stage_ms[x.first] += ms;
  }
  e->ev_used.clear();
}

// One pack of whole sequences [s0, s1).
// ids_dev: when set, the token ids already sit in device memory (packed like
// `ids`) and logits_dev receives the logits on the device; nothing is copied
// to or from the host except the offsets table.
// Caps the persistent kernels launched from this thread for the scope.
struct PersistentCap {
  explicit PersistentCap(int n) { set_persistent_cap(n); }
  ~PersistentCap() { set_persistent_cap(0); }
};

int run_pack(clef_engine* e, const int32_t* ids, const int64_t* offsets, int s0, int s1,
             const clef_prefix* init, int64_t capture, clef_prefix* cap, float* logits,
             float* hidden, int64_t hidden_row0, const int32_t* ids_dev = nullptr,
             float* logits_dev = nullptr) {
  const clef_config& c = e->cfg;
  PersistentCap sm_cap(e->sm_limit);
  cudaStream_t s = e->stream;
  const int np = s1 - s0;
  const int64_t t0 = offsets[s0];
  const int64_t M = offsets[s1] - t0;
  RC(ensure_capacity(e, M, np));
  const int hid = c.hidden_size;
  const int hk = c.linear_num_key_heads, hv = c.linear_num_value_heads;
  const int H = c.num_attention_heads, Hkv = c.num_key_value_heads, d = c.head_dim;
  const float eps = c.rms_norm_eps;
  const int64_t P = init ? init->tokens : 0;
  // Offsets: int64 cu (rebased) then int32 q-block offsets.
  std::vector<int64_t> cu(np + 1);
  for (int i = 0; i <= np; ++i) cu[i] = offsets[s0 + i] - t0;
  // Device offsets: int64 cu | int32 64-row q-blocks | int64 padded V^T
  // offsets | int32 128-row q-blocks | int32 64-key blocks.
  const size_t n1 = (size_t)np + 1;
  std::vector<char> meta(meta_bytes(n1));
  int64_t* m_cu = reinterpret_cast<int64_t*>(meta.data());
  int32_t* qb = reinterpret_cast<int32_t*>(m_cu + n1);
  const size_t vt_off_bytes = meta_vt_offset(n1);
  int64_t* m_vt = reinterpret_cast<int64_t*>(meta.data() + vt_off_bytes);
  int32_t* qb128 = reinterpret_cast<int32_t*>(m_vt + n1);
  int32_t* kb64 = qb128 + n1;
  memcpy(m_cu, cu.data(), sizeof(int64_t) * n1);
  qb[0] = qb128[0] = kb64[0] = 0;
  m_vt[0] = 0;
  for (int i = 0; i < np; ++i) {
    const int64_t L = cu[i + 1] - cu[i];
    qb[i + 1] = qb[i] + (int32_t)ceil_div(L, 64);
    qb128[i + 1] = qb128[i] + (int32_t)ceil_div(L, 128);
    kb64[i + 1] = kb64[i] + (int32_t)ceil_div(L, 64);
    m_vt[i + 1] = m_vt[i] + ceil_div(L, 64) * 64;
  }
  CLEF_CHECK(m_vt[np] <= e->vt_pitch, CLEF_ERR_INVALID, "prefill: V^T buffer too small");
  CLEF_CUDA(cudaMemcpyAsync(e->meta_d, meta.data(), meta.size(), cudaMemcpyHostToDevice, s));
  SeqPackVT vpack;
  vpack.cu = e->meta_d;
  vpack.cu_vt = reinterpret_cast<const int64_t*>(reinterpret_cast<const char*>(e->meta_d) + vt_off_bytes);
  vpack.cu_qb = reinterpret_cast<const int32_t*>(vpack.cu_vt + n1);
  vpack.cu_kb = vpack.cu_qb + n1;
  vpack.nseq = np;
  vpack.total = M;
  vpack.qblocks = qb128[np];
  vpack.kblocks = kb64[np];
  const int32_t* ids_src = e->ids_d;
  if (ids_dev) ids_src = ids_dev + t0;
  else CLEF_CUDA(cudaMemcpyAsync(e->ids_d, ids + t0, sizeof(int32_t) * M, cudaMemcpyHostToDevice, s));
  {
    int64_t n = 2;  // embed + head
    for (int li = 0; li < c.num_hidden_layers; ++li) {
      n += 9;  // 2 norms, 4 GEMMs, 3 mixer kernels
      if (c.layer_types[li] && e->precision == CLEF_PRECISION_SPLIT) n += 1;  // gate split
    }
    if (hidden || cap) n += 1;
    e->launches += n;
  }
  SeqPack pack;
  pack.cu_seqlens = e->meta_d;
  pack.nseq = np;
  pack.total = M;
  pack.qblocks = qb[np];

  // Chunk tables of the DeltaNet scan, shared by every DeltaNet layer of the pack.
  ScanPlan plan;
  bool any_delta = false;
  for (int li = 0; li < c.num_hidden_layers; ++li) any_delta |= c.layer_types[li] == 0;
  if (any_delta) RC(delta_scan_plan(cu.data(), np, hk, hv, e->scan_ws, e->scan_ws_bytes, s, &plan));
  {
    STAGE(kStEmbed);
    RC(launch_embed(e->embed, ids_src, M, hid, e->h, s));
  }
  const bool split = e->precision == CLEF_PRECISION_SPLIT;
  const int x2 = split ? 2 : 1;
  const int norm_out = split ? kOutBF16Split : CLEF_BF16;
  for (int li = 0; li < c.num_hidden_layers; ++li) {
    if (e->cancel.load()) {
      cudaStreamSynchronize(s);
      return fail(CLEF_ERR_CANCELLED, "prefill: cancelled");
    }
    const LayerW& L = e->layers[li];
    {
      STAGE(kStNorm);
      RC(launch_rmsnorm(e->h, L.in_eff, M, hid, eps, norm_out, e->u, s));
    }
    if (!L.attention) {
      // in_proj_qkv | z | a | b: BF16 output in the default precision (the
      // model dtype of the reference's mixed-precision path, qwen.rs:603, 619,
      // 626, 669), F32 in the split precision.
      uint16_t* pin = reinterpret_cast<uint16_t*>(e->proj);
      float* pin32 = e->proj;
      {
        STAGE(kStGemm);
        if (split) RC(launch_gemm(e->u, L.w_in, nullptr, M, L.n_in, hid, kEpiF32, pin32, L.n_in, s, 1));
        else RC(launch_gemm(e->u, L.w_in, nullptr, M, L.n_in, hid, kEpiBF16, pin, L.n_in, s));
      }
      const clef_prefix::Layer* il = init ? &init->layers[li] : nullptr;
      {
        STAGE(kStDeltaPro);
        if (split)
          RC(launch_delta_prologue(pin32, L.n_in, e->qkv_w + e->value, e->qkv_w + e->value + hv,
                                   il ? il->hist : nullptr, il ? il->hist_rows : 0, L.conv, L.dt,
                                   L.alog, pack, hk, hv, 128, 128, e->dq, e->dk, e->dv, e->dg, e->db,
                                   s));
        else
          RC(launch_delta_prologue(pin, L.n_in, e->qkv_w + e->value, e->qkv_w + e->value + hv,
                                   il ? il->hist : nullptr, il ? il->hist_rows : 0, L.conv, L.dt,
                                   L.alog, pack, hk, hv, 128, 128, e->dq, e->dk, e->dv, e->dg, e->db,
                                   s));
      }
      {
        STAGE(kStDeltaScan);
        RC(launch_delta_scan_planned(plan, e->dq, e->dk, e->dv, e->dg, e->db,
                                     il ? il->S : nullptr, 1, capture,
                                     cap ? cap->layers[li].S : nullptr, nullptr, e->dout, s));
      }
      if (cap) {
        auto& cl = cap->layers[li];
        if (split)
          RC(launch_copy_rows(pin32, L.n_in, capture - cl.hist_rows, cl.hist_rows, e->qkv_w, 4, cl.hist,
                              e->qkv_w, s));
        else
          RC(launch_rows_bf16_to_f32(pin, L.n_in, capture - cl.hist_rows, cl.hist_rows, e->qkv_w, cl.hist,
                                     e->qkv_w, s));
      }
      {
        STAGE(kStDeltaEpi);
        if (split)
          RC(launch_delta_epilogue_split(e->dout, pin32 + e->qkv_w, L.n_in, L.dnorm, eps, M, hv, e->y, s));
        else
          RC(launch_delta_epilogue(e->dout, pin + e->qkv_w, L.n_in, L.dnorm, eps, M, hv, 128, e->y, s));
      }
      {
        STAGE(kStGemm);
        RC(launch_gemm(e->y, L.w_out, nullptr, M, hid, e->value, kEpiAddF32, e->h, hid, s, split));
      }
    } else {
      uint16_t* pb = reinterpret_cast<uint16_t*>(e->proj);
      float* pb32 = e->proj;
      {
        STAGE(kStGemm);
        if (split) RC(launch_gemm(e->u, L.w_att, nullptr, M, L.n_att, hid, kEpiF32, pb32, L.n_att, s, 1));
        else RC(launch_gemm(e->u, L.w_att, nullptr, M, L.n_att, hid, kEpiBF16, pb, L.n_att, s));
      }
      {
        STAGE(kStAttnPro);
        if (split)
          RC(launch_attention_prologue(pb32, L.n_att, L.qn, L.kn, eps, pack, P, H, Hkv, d, c.rotary_dim,
                                       e->inv_freq, e->qatt, e->katt, s));
        else
          RC(launch_attention_prologue(pb, L.n_att, L.qn, L.kn, eps, pack, P, H, Hkv, d, c.rotary_dim,
                                       e->inv_freq, e->qatt, e->katt, s));
      }
      const int v_col = 2 * e->att_n + e->att_kv;
      {
        STAGE(kStAttnPro);
        if (split) RC(launch_transpose_v(pb32 + v_col, L.n_att, d, vpack, Hkv, e->vt, e->vt_pitch, s));
        else RC(launch_transpose_v(pb + v_col, L.n_att, d, vpack, Hkv, e->vt, e->vt_pitch, s));
      }
      if (cap) {
        auto& cl = cap->layers[li];
        RC(launch_copy_rows(e->katt, e->att_kv, 0, capture, e->att_kv, 2, cl.k, e->att_kv, s));
        // V^T columns [0, capture) of the single captured sequence.
        CLEF_CUDA(cudaMemcpy2DAsync(cl.vt, sizeof(uint16_t) * cap->vt_pitch, e->vt,
                                    sizeof(uint16_t) * e->vt_pitch, sizeof(uint16_t) * capture,
                                    (size_t)e->att_kv, cudaMemcpyDeviceToDevice, s));
      }
      AttnTcArgs a;
      a.H = H;
      a.Hkv = Hkv;
      a.scale = (float)(1.0 / std::sqrt((double)d));
      a.q = e->qatt;
      a.rows_q = M;
      a.k = e->katt;
      a.rows_k = M;
      a.vt = e->vt;
      a.vt_cols = e->vt_pitch;
      a.vt_pitch = e->vt_pitch;
      if (init) {
        a.prefix_len = P;
        a.pk = init->layers[li].k;
        a.pvt = init->layers[li].vt;
        a.pvt_pitch = init->vt_pitch;
      }
      if (split) {
        // F32 attention output; the gate product and its split follow.
        a.out = e->dout;
        a.o_ts = e->att_n;
        a.o_hs = d;
      } else {
        a.gate = pb + d;
        a.g_ts = L.n_att;
        a.g_hs = 2 * d;
        a.out = e->y;
        a.o_ts = e->att_n;
        a.o_hs = d;
      }
      {
        STAGE(kStAttn);
        RC(launch_attention_tc(a, vpack, s));
      }
      if (split) {
        STAGE(kStAttnPro);
        RC(launch_gate_split(e->dout, pb32 + d, L.n_att, 2 * d, H, d, M, e->y, s));
      }
      {
        STAGE(kStGemm);
        RC(launch_gemm(e->y, L.w_o, nullptr, M, hid, e->att_n, kEpiAddF32, e->h, hid, s, split));
      }
    }
    {
      STAGE(kStNorm);
      RC(launch_rmsnorm(e->h, L.post_eff, M, hid, eps, norm_out, e->u, s));
    }
    {
      STAGE(kStGemm);
      RC(launch_gemm(e->u, L.w_gate, L.w_up, M, c.intermediate_size, hid, split ? kEpiSwiGLUSplit : kEpiSwiGLU,
                     e->act, (int64_t)x2 * c.intermediate_size, s, split));
      RC(launch_gemm(e->act, L.w_down, nullptr, M, hid, c.intermediate_size, kEpiAddF32, e->h, hid,
                     s, split));
    }
  }
  if ((logits || logits_dev) && c.head_outputs) {
    STAGE(kStHead);
    float* dst = logits_dev ? logits_dev + (size_t)s0 * c.head_outputs : e->logits_d;
    RC(launch_head(e->h, e->final_eff, eps, pack, hid, e->head_w, c.head_outputs, dst, s));
    if (logits)
      CLEF_CUDA(cudaMemcpyAsync(logits + (size_t)s0 * c.head_outputs, dst,
                                sizeof(float) * np * c.head_outputs, cudaMemcpyDeviceToHost, s));
  }
  if (hidden || cap) {
    float* hn = e->proj;  // [M, hidden] F32 scratch
    RC(launch_rmsnorm(e->h, e->final_eff, M, hid, eps, CLEF_F32, hn, s));
    if (cap)
      CLEF_CUDA(cudaMemcpyAsync(cap->hidden_rows, hn, sizeof(float) * capture * hid,
                                cudaMemcpyDeviceToDevice, s));
    if (hidden)
      CLEF_CUDA(cudaMemcpyAsync(hidden + hidden_row0 * hid, hn, sizeof(float) * M * hid,
                                cudaMemcpyDeviceToHost, s));
  }
  return CLEF_OK;
}

}  // namespace

extern "C" {

int clef_engine_create(const clef_config* cfg, int32_t device, clef_engine** out) {
  CLEF_CHECK(out, CLEF_ERR_INVALID, "engine_create: null output");
  *out = nullptr;
  RC(clef_config_validate(cfg));
  int n = 0;
  CLEF_CUDA(cudaGetDeviceCount(&n));
  CLEF_CHECK(device >= 0 && device < n, CLEF_ERR_INVALID, "engine_create: device index");
  DeviceGuard g(device);
  clef_engine* e = new clef_engine();
  e->cfg = *cfg;
  e->device = device;
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete e;
    return fail(CLEF_ERR_CUDA, "engine_create: stream");
  }
  int rc = build_layout(e);
  if (rc) {
    clef_engine_destroy(e);
    return rc;
  }
  *out = e;
  return CLEF_OK;
}

size_t clef_engine_weight_count(const clef_engine* e, const char* name) {
  if (!e || !name) return 0;
  auto it = e->tensors.find(name);
  return it == e->tensors.end() ? 0 : (size_t)it->second.count;
}

int clef_engine_set_weight(clef_engine* e, const char* name, const float* host, size_t count) {
  CLEF_CHECK(e && name && host, CLEF_ERR_INVALID, "set_weight: null argument");
  auto it = e->tensors.find(name);
  CLEF_CHECK(it != e->tensors.end(), CLEF_ERR_INVALID, std::string("set_weight: unknown tensor ") + name);
  NamedTensor& t = it->second;
  CLEF_CHECK((int64_t)count == t.count, CLEF_ERR_INVALID,
             std::string("set_weight: element count mismatch for ") + name);
  DeviceGuard g(e->device);
  if (t.bf16) {
    // Stage through a bounded F32 buffer and convert on the device.
    const int64_t chunk = 1 << 24;
    float* tmp = nullptr;
    CLEF_CUDA(cudaMalloc(&tmp, sizeof(float) * std::min<int64_t>(chunk, t.count)));
    for (int64_t o = 0; o < t.count; o += chunk) {
      const int64_t n = std::min<int64_t>(chunk, t.count - o);
      cudaError_t err = cudaMemcpyAsync(tmp, host + o, sizeof(float) * n, cudaMemcpyHostToDevice, e->stream);
      if (err == cudaSuccess) {
        f32_to_bf16_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, e->stream>>>(
            tmp, n, reinterpret_cast<uint16_t*>(t.dev) + o);
        err = cudaStreamSynchronize(e->stream);
      }
      if (err != cudaSuccess) {
        cudaFree(tmp);
        return fail(CLEF_ERR_CUDA, std::string("set_weight: ") + cudaGetErrorString(err));
      }
    }
    cudaFree(tmp);
  } else {
    CLEF_CUDA(cudaMemcpyAsync(t.dev, host, sizeof(float) * t.count, cudaMemcpyHostToDevice, e->stream));
    CLEF_CUDA(cudaStreamSynchronize(e->stream));
  }
  t.loaded = true;
  e->finalized = false;
  return CLEF_OK;
}

int clef_engine_init_random(clef_engine* e, uint64_t seed, float std_) {
  CLEF_CHECK(e, CLEF_ERR_INVALID, "init_random: null engine");
  CLEF_CHECK(std_ >= 0.f, CLEF_ERR_INVALID, "init_random: std");
  DeviceGuard g(e->device);
  for (auto& kv : e->tensors) {
    NamedTensor& t = kv.second;
    if (t.loaded) continue;
    const uint64_t stream = name_stream(kv.first.c_str());
    if (t.bf16) {
      RC(launch_fill_normal_bf16((uint16_t*)t.dev, t.count, seed, stream, 0.f, std_, e->stream));
    } else {
      std::vector<float> host(t.count);
      switch (t.init) {
        case kInitNormal: host_fill(host.data(), t.count, seed, stream, kFillNormal, 0.f, std_); break;
        case kInitOnePlusNormal:
          host_fill(host.data(), t.count, seed, stream, kFillNormal, 1.f, std_);
          break;
        case kInitALog:
          host_fill(host.data(), t.count, seed, stream, kFillUniform, 0.f, std::log(16.f));
          break;
        case kInitDtBias: host_fill(host.data(), t.count, seed, stream, kFillNormal, 0.f, 0.1f); break;
      }
      CLEF_CUDA(cudaMemcpyAsync(t.dev, host.data(), sizeof(float) * t.count, cudaMemcpyHostToDevice,
                                e->stream));
      CLEF_CUDA(cudaStreamSynchronize(e->stream));
    }
    t.loaded = true;
  }
  CLEF_CUDA(cudaStreamSynchronize(e->stream));
  e->finalized = false;
  return CLEF_OK;
}

int clef_engine_get_weight(clef_engine* e, const char* name, float* host, size_t count) {
  CLEF_CHECK(e && name && host, CLEF_ERR_INVALID, "get_weight: null argument");
  auto it = e->tensors.find(name);
  CLEF_CHECK(it != e->tensors.end(), CLEF_ERR_INVALID, std::string("get_weight: unknown tensor ") + name);
  NamedTensor& t = it->second;
  CLEF_CHECK((int64_t)count == t.count, CLEF_ERR_INVALID, "get_weight: element count mismatch");
  DeviceGuard g(e->device);
  if (t.bf16) {
    const int64_t chunk = 1 << 24;
    float* tmp = nullptr;
    CLEF_CUDA(cudaMalloc(&tmp, sizeof(float) * std::min<int64_t>(chunk, t.count)));
    for (int64_t o = 0; o < t.count; o += chunk) {
      const int64_t n = std::min<int64_t>(chunk, t.count - o);
      bf16_to_f32_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, e->stream>>>(
          reinterpret_cast<const uint16_t*>(t.dev) + o, n, tmp);
      cudaError_t err = cudaMemcpyAsync(host + o, tmp, sizeof(float) * n, cudaMemcpyDeviceToHost, e->stream);
      if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
      if (err != cudaSuccess) {
        cudaFree(tmp);
        return fail(CLEF_ERR_CUDA, std::string("get_weight: ") + cudaGetErrorString(err));
      }
    }
    cudaFree(tmp);
  } else {
    CLEF_CUDA(cudaMemcpyAsync(host, t.dev, sizeof(float) * t.count, cudaMemcpyDeviceToHost, e->stream));
    CLEF_CUDA(cudaStreamSynchronize(e->stream));
  }
  return CLEF_OK;
}

int clef_engine_finalize(clef_engine* e) {
  CLEF_CHECK(e, CLEF_ERR_INVALID, "finalize: null engine");
  DeviceGuard g(e->device);
  for (auto& kv : e->tensors)
    CLEF_CHECK(kv.second.loaded, CLEF_ERR_INVALID, "finalize: missing tensor " + kv.first);
  for (auto& kv : e->tensors) {
    NamedTensor& t = kv.second;
    if (t.offset)
      one_plus_kernel<<<(unsigned)ceil_div(t.count, 256), 256, 0, e->stream>>>((const float*)t.dev,
                                                                              t.count, t.eff);
  }
  RC(launch_status("finalize"));
  const clef_config& c = e->cfg;
  std::vector<float> inv(128, 0.f);
  for (int i = 0; i < c.rotary_dim / 2 && i < 128; ++i)
    inv[i] = (float)std::pow(c.rope_theta, -((double)(2 * i)) / c.rotary_dim);
  CLEF_CUDA(cudaMemcpyAsync(e->inv_freq, inv.data(), sizeof(float) * 128, cudaMemcpyHostToDevice,
                            e->stream));
  CLEF_CUDA(cudaStreamSynchronize(e->stream));
  e->finalized = true;
  return CLEF_OK;
}

int clef_engine_prefill(clef_engine* e, const int32_t* ids, const int64_t* offsets, int32_t nseq,
                        const clef_prefix* initial, int64_t capture, clef_prefix** captured,
                        float* logits, float* hidden) {
  CLEF_CHECK(e && ids && offsets, CLEF_ERR_INVALID, "prefill: null argument");
  CLEF_CHECK(e->finalized, CLEF_ERR_INVALID, "prefill: engine not finalized");
  CLEF_CHECK(nseq >= 1, CLEF_ERR_INVALID, "prefill: nseq must be positive");
  CLEF_CHECK(offsets[0] == 0, CLEF_ERR_INVALID, "prefill: offsets[0] must be 0");
  for (int i = 0; i < nseq; ++i)
    CLEF_CHECK(offsets[i + 1] > offsets[i], CLEF_ERR_INVALID, "prefill: empty or unordered sequence");
  const clef_config& c = e->cfg;
  const int64_t total = offsets[nseq];
  for (int64_t i = 0; i < total; ++i)
    CLEF_CHECK(ids[i] >= 0 && ids[i] < c.vocab_size, CLEF_ERR_INVALID,
               "prefill: token outside vocabulary");
  CLEF_CHECK(capture >= 0, CLEF_ERR_INVALID, "prefill: capture");
  if (capture) {
    CLEF_CHECK(captured, CLEF_ERR_INVALID, "prefill: capture needs an output handle");
    CLEF_CHECK(nseq == 1 && capture <= total, CLEF_ERR_INVALID, "prefill: capture boundary");
    CLEF_CHECK(!initial, CLEF_ERR_INVALID, "prefill: initial state and capture together");
  }
  if (initial) {
    CLEF_CHECK(initial->device == e->device && (int)initial->layers.size() == c.num_hidden_layers &&
                   initial->hidden == c.hidden_size,
               CLEF_ERR_INVALID, "prefill: prefix state does not match this engine");
    CLEF_CHECK(initial->filled, CLEF_ERR_INVALID,
               "prefill: the prefix holds no state (created but never imported)");
  }
  if (captured) *captured = nullptr;
  DeviceGuard g(e->device);
  clef_prefix* cap = nullptr;
  if (capture) RC(alloc_prefix(e, capture, &cap));
  int64_t row0 = 0;
  if (hidden && initial && nseq == 1) {
    CLEF_CUDA(cudaMemcpyAsync(hidden, initial->hidden_rows, sizeof(float) * initial->tokens * c.hidden_size,
                              cudaMemcpyDeviceToHost, e->stream));
    row0 = initial->tokens;
  }
  int rc = CLEF_OK;
  for (int s0 = 0; s0 < nseq && rc == CLEF_OK;) {
    int s1 = s0 + 1;
    while (s1 < nseq && offsets[s1 + 1] - offsets[s0] <= e->max_pack) ++s1;
    rc = run_pack(e, ids, offsets, s0, s1, initial, capture, cap, logits, hidden,
                  row0 + offsets[s0]);
    s0 = s1;
  }
  cudaError_t se = cudaStreamSynchronize(e->stream);
  if (rc == CLEF_OK && se != cudaSuccess)
    rc = fail(CLEF_ERR_CUDA, std::string("prefill: ") + cudaGetErrorString(se));
  if (rc == CLEF_OK) {
    int dev_err = 0;
    int derc = CLEF_OK;
    // The flag is read only when a kernel raised it (cheap symbol read).
    derc = device_errors(&dev_err);
    if (derc) rc = derc;
    else if (dev_err) rc = fail(CLEF_ERR_DEVICE_TIMEOUT, "prefill: a device-side wait timed out");
  }
  if (rc == CLEF_OK) collect_stage_times(e);
  if (rc != CLEF_OK) {
    if (cap) clef_prefix_destroy(cap);
    return rc;
  }
  if (cap) cap->filled = true;
  if (captured) *captured = cap;
  return CLEF_OK;
}

int clef_engine_prefill_device(clef_engine* e, const int32_t* ids_device, const int64_t* offsets,
                               int32_t nseq, const clef_prefix* initial, float* logits_device,
                               void* stream) {
  CLEF_CHECK(e && ids_device && offsets && logits_device, CLEF_ERR_INVALID,
             "prefill_device: null argument");
  CLEF_CHECK(e->finalized, CLEF_ERR_INVALID, "prefill_device: engine not finalized");
  CLEF_CHECK(nseq >= 1 && offsets[0] == 0, CLEF_ERR_INVALID, "prefill_device: offsets");
  for (int i = 0; i < nseq; ++i)
    CLEF_CHECK(offsets[i + 1] > offsets[i], CLEF_ERR_INVALID,
               "prefill_device: empty or unordered sequence");
  CLEF_CHECK(e->cfg.head_outputs > 0, CLEF_ERR_INVALID, "prefill_device: model has no head");
  if (initial) {
    CLEF_CHECK(initial->device == e->device &&
                   (int)initial->layers.size() == e->cfg.num_hidden_layers,
               CLEF_ERR_INVALID, "prefill_device: prefix state does not match this engine");
    CLEF_CHECK(initial->filled, CLEF_ERR_INVALID,
               "prefill_device: the prefix holds no state (created but never imported)");
  }
  DeviceGuard g(e->device);
  cudaStream_t user = as_stream(stream);
  cudaStream_t own = e->stream;
  e->stream = user ? user : own;
  int rc = CLEF_OK;
  for (int s0 = 0; s0 < nseq && rc == CLEF_OK;) {
    int s1 = s0 + 1;
    while (s1 < nseq && offsets[s1 + 1] - offsets[s0] <= e->max_pack) ++s1;
    rc = run_pack(e, nullptr, offsets, s0, s1, initial, 0, nullptr, nullptr, nullptr, 0, ids_device,
                  logits_device);
    s0 = s1;
  }
  e->stream = own;
  return rc;
}

int64_t clef_engine_launches(const clef_engine* e) { return e ? e->launches : 0; }

int clef_engine_set_precision(clef_engine* e, int32_t precision) {
  CLEF_CHECK(e, CLEF_ERR_INVALID, "set_precision: null engine");
  CLEF_CHECK(precision == CLEF_PRECISION_BF16 || precision == CLEF_PRECISION_SPLIT, CLEF_ERR_INVALID,
             "set_precision: unknown precision");
  if (precision != e->precision) {
    // The arena is resized on the next prefill; pending work must not use it.
    DeviceGuard g(e->device);
    CLEF_CUDA(cudaStreamSynchronize(e->stream));
    CLEF_CUDA(cudaDeviceSynchronize());
    e->precision = precision;
  }
  return CLEF_OK;
}

int32_t clef_engine_precision(const clef_engine* e) { return e ? e->precision : -1; }

int clef_engine_set_sm_limit(clef_engine* e, int32_t sms) {
  CLEF_CHECK(e, CLEF_ERR_INVALID, "set_sm_limit: null engine");
  CLEF_CHECK(sms >= 0, CLEF_ERR_INVALID, "set_sm_limit: negative SM count");
  CLEF_CHECK(sms == 0 || sms >= 2, CLEF_ERR_INVALID, "set_sm_limit: at least 2 SMs (one CTA pair)");
  e->sm_limit = sms;
  return CLEF_OK;
}

int clef_engine_cancel(clef_engine* e, int32_t cancel) {
  CLEF_CHECK(e, CLEF_ERR_INVALID, "cancel: null engine");
  e->cancel.store(cancel ? 1 : 0);
  return CLEF_OK;
}

int clef_engine_set_profiling(clef_engine* e, int32_t enabled) {
  CLEF_CHECK(e, CLEF_ERR_INVALID, "set_profiling: null engine");
  if (!e->ev_used.empty()) {
    DeviceGuard g(e->device);
    CLEF_CUDA(cudaDeviceSynchronize());
    e->ev_used.clear();
  }
  e->profiling = enabled != 0;
  for (auto& x : e->stage_ms) x = 0.f;
  return CLEF_OK;
}

int clef_engine_stage_times(clef_engine* e, float* ms, int32_t n) {
  if (!e || !ms) return 0;
  if (!e->ev_used.empty()) {
    DeviceGuard g(e->device);
    cudaDeviceSynchronize();
    collect_stage_times(e);
  }
  const int k = std::min<int>(n, kStages);
  for (int i = 0; i < k; ++i) ms[i] = e->stage_ms[i];
  return k;
}

int clef_engine_destroy(clef_engine* e) {
  if (!e) return CLEF_OK;
  DeviceGuard g(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto ev : e->ev_pool) cudaEventDestroy(ev);
  if (e->arena) cudaFree(e->arena);
  if (e->wblob) cudaFree(e->wblob);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
  return CLEF_OK;
}

int64_t clef_prefix_tokens(const clef_prefix* p) { return p ? p->tokens : 0; }
uint64_t clef_prefix_span_bytes(const clef_prefix* p) { return p ? p->span : 0; }

int clef_prefix_create(clef_engine* e, int64_t tokens, clef_prefix** out) {
  if (out) *out = nullptr;
  CLEF_CHECK(e && out, CLEF_ERR_INVALID, "prefix_create: null pointer");
  CLEF_CHECK(e->finalized, CLEF_ERR_INVALID, "prefix_create: engine not finalized");
  CLEF_CHECK(tokens > 0, CLEF_ERR_INVALID, "prefix_create: tokens must be positive");
  DeviceGuard g(e->device);
  RC(alloc_prefix(e, tokens, out));
  // The descriptor copy must land before an import on another stream reads it back.
  if (cudaStreamSynchronize(e->stream) != cudaSuccess) {
    clef_prefix_destroy(*out);
    *out = nullptr;
    return fail(CLEF_ERR_CUDA, "prefix_create: descriptor copy");
  }
  return CLEF_OK;
}

int clef_prefix_export(const clef_prefix* p, void* dst, uint64_t bytes, void* stream) {
  CLEF_CHECK(p && dst, CLEF_ERR_INVALID, "prefix_export: null pointer");
  CLEF_CHECK(p->filled, CLEF_ERR_INVALID, "prefix_export: the prefix holds no state");
  CLEF_CHECK(bytes == p->span, CLEF_ERR_INVALID,
             "prefix_export: bytes must equal the prefix span (" + std::to_string(p->span) + ")");
  DeviceGuard g(p->device);
  CLEF_CUDA(cudaMemcpyAsync(dst, p->blob, bytes, cudaMemcpyDeviceToDevice, as_stream(stream)));
  return CLEF_OK;
}

int clef_prefix_import(clef_prefix* p, const void* src, uint64_t bytes, void* stream) {
  CLEF_CHECK(p && src, CLEF_ERR_INVALID, "prefix_import: null pointer");
  CLEF_CHECK(bytes == p->span, CLEF_ERR_INVALID,
             "prefix_import: bytes must equal the prefix span (" + std::to_string(p->span) + ")");
  DeviceGuard g(p->device);
  p->filled = false;
  cudaStream_t s = as_stream(stream);
  CLEF_CUDA(cudaMemcpyAsync(p->blob, src, bytes, cudaMemcpyDeviceToDevice, s));
  PrefixDescriptor got;
  CLEF_CUDA(cudaMemcpyAsync(&got, p->blob, sizeof(got), cudaMemcpyDeviceToHost, s));
  CLEF_CUDA(cudaStreamSynchronize(s));
  if (!(got == p->desc)) {
    // Put this prefix's own descriptor back so a later import or export sees it.
    CLEF_CUDA(cudaMemcpy(p->blob, &p->desc, sizeof(p->desc), cudaMemcpyHostToDevice));
    return fail(CLEF_ERR_INVALID, "prefix_import: the copy was made for another layout or token count (" +
                                      std::to_string(got.tokens) + " tokens, " + std::to_string(got.layers) +
                                      " layers; this prefix: " + std::to_string(p->desc.tokens) + " tokens, " +
                                      std::to_string(p->desc.layers) + " layers)");
  }
  p->filled = true;
  return CLEF_OK;
}
uint64_t clef_prefix_bytes(const clef_prefix* p) { return p ? p->bytes : 0; }
int clef_prefix_destroy(clef_prefix* p) {
  if (!p) return CLEF_OK;
  DeviceGuard g(p->device);
  if (p->blob) cudaFree(p->blob);
  delete p;
  return CLEF_OK;
}

}  // extern "C"
