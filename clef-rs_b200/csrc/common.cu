// common.cu — error state, device error flag, configuration checks and the
// decision rule of the schema head.
#include <cmath>
#include <string>

#include "common.cuh"

namespace clef {

namespace {
thread_local std::string t_last_error;
}

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int device_errors(int* code) {
  *code = 0;
  CLEF_CUDA(cudaDeviceSynchronize());
  int v = 0, w = 0, x = 0;
  int rc = gemm_device_error(&v);
  if (!rc) rc = attention_tc_device_error(&w);
  if (!rc) rc = scan_device_error(&x);
  if (rc) return fail(rc, "device error flag read failed");
  *code = v ? v : (w ? w : x);
  return CLEF_OK;
}

thread_local int g_persistent_cap = 0;

void set_persistent_cap(int ctas) { g_persistent_cap = ctas > 0 ? ctas : 0; }

int persistent_ctas(int device) {
  const int n = num_sms(device);
  return g_persistent_cap > 0 && g_persistent_cap < n ? g_persistent_cap : n;
}

int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (!cached[device]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cached[device] = n;
  }
  return cached[device];
}

}  // namespace clef

extern "C" {

const char* clef_last_error(void) { return clef::t_last_error.c_str(); }

const char* clef_version(void) { return "clef_b200 0.1.0 (sm_100a)"; }

int clef_config_validate(const clef_config* c) {
  using clef::fail;
  if (!c) return fail(CLEF_ERR_INVALID, "config: null");
  if (c->hidden_size <= 0 || c->hidden_size % 64 != 0)
    return fail(CLEF_ERR_UNSUPPORTED, "config: hidden_size must be a positive multiple of 64");
  if (c->intermediate_size <= 0 || c->intermediate_size % 64 != 0)
    return fail(CLEF_ERR_UNSUPPORTED, "config: intermediate_size must be a multiple of 64");
  if (c->num_hidden_layers <= 0 || c->num_hidden_layers > CLEF_MAX_LAYERS)
    return fail(CLEF_ERR_INVALID, "config: num_hidden_layers");
  if (c->vocab_size <= 0) return fail(CLEF_ERR_INVALID, "config: vocab_size");
  if (c->linear_conv_kernel_dim != 4)
    return fail(CLEF_ERR_UNSUPPORTED, "config: linear_conv_kernel_dim must be 4");
  if (c->rms_norm_eps <= 0.f || !(c->rms_norm_eps <= 1.f))
    return fail(CLEF_ERR_INVALID, "config: rms_norm_eps");
  bool any_linear = false, any_full = false;
  for (int i = 0; i < c->num_hidden_layers; ++i) {
    if (c->layer_types[i] > 1) return fail(CLEF_ERR_INVALID, "config: layer_types");
    any_full |= c->layer_types[i] == 1;
    any_linear |= c->layer_types[i] == 0;
  }
  if (any_linear) {
    if (c->linear_key_head_dim != 128 || c->linear_value_head_dim != 128)
      return fail(CLEF_ERR_UNSUPPORTED, "config: DeltaNet head dims must be 128");
    if (c->linear_num_key_heads <= 0 || c->linear_num_value_heads <= 0 ||
        c->linear_num_value_heads % c->linear_num_key_heads != 0)
      return fail(CLEF_ERR_INVALID, "config: DeltaNet head counts");
  }
  if (any_full) {
    if (c->head_dim != 256) return fail(CLEF_ERR_UNSUPPORTED, "config: head_dim must be 256");
    if (c->num_attention_heads <= 0 || c->num_key_value_heads <= 0 ||
        c->num_attention_heads % c->num_key_value_heads != 0)
      return fail(CLEF_ERR_INVALID, "config: attention head counts");
    if (c->rotary_dim <= 0 || c->rotary_dim > c->head_dim || c->rotary_dim % 2)
      return fail(CLEF_ERR_INVALID, "config: rotary_dim");
  }
  if (c->head_outputs != 0 && c->head_outputs != 7)
    return fail(CLEF_ERR_UNSUPPORTED, "config: head_outputs must be 0 or 7");
  return CLEF_OK;
}

// answers (crates/core/src/types.rs:728-802) for the linear schema head:
// logits[0:2] noul (options true, false), logits[2:6] choice, logits[6] score.
// Softmax subtracts the maximum; the winner is the first strict maximum in
// option order; noul reports p[0]; a single-option softmax is 1.0, so the
// score is the raw logit.
int clef_decide(const float* logits, int32_t n, int32_t head_outputs, clef_decision* out) {
  using clef::fail;
  if (!logits || !out || n < 0) return fail(CLEF_ERR_INVALID, "decide: null pointer or count");
  if (head_outputs != 7) return fail(CLEF_ERR_UNSUPPORTED, "decide: head_outputs must be 7");
  for (int32_t r = 0; r < n; ++r) {
    const float* l = logits + (size_t)r * head_outputs;
    for (int i = 0; i < 7; ++i)
      if (!std::isfinite(l[i])) return fail(CLEF_ERR_INVALID, "decide: invalid logits");
    auto softmax = [](const float* x, int k, float* p) {
      float mx = -INFINITY;
      for (int i = 0; i < k; ++i) mx = std::fmax(mx, x[i]);
      float s = 0.f;
      for (int i = 0; i < k; ++i) {
        p[i] = std::exp(x[i] - mx);
        s += p[i];
      }
      for (int i = 0; i < k; ++i) p[i] /= s;
    };
    float pn[2], pc[4];
    softmax(l, 2, pn);
    softmax(l + 2, 4, pc);
    int win = -1;
    float best = -1.f;
    for (int i = 0; i < 4; ++i)
      if (pc[i] > best) {
        best = pc[i];
        win = i;
      }
    out[r].noul = pn[0];
    out[r].choice = win;
    out[r].confidence = best;
    out[r].score = l[6];
  }
  return CLEF_OK;
}

}  // extern "C"
