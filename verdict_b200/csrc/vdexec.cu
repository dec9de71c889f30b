// vdexec runtime: model load, workspaces, forward scheduling and the C ABI.
//
// One handle = one model replica pinned to one GPU (the reference never pins a
// replica to a device, src/main.rs:60-67; here vd_open selects it).  A batch
// arrives as the scheduler's right-padded CollatedBatch; the runtime computes the
// ragged layout (cu_seqlens, attention tile table) on the host, packs tokens on
// the device and runs the whole prefill forward as a fixed sequence of kernels
// on the handle's stream:
//   decoder: pack -> embed -> L x [RMSNorm, QKV GEMM (+q/k norm, RoPE),
//            attention, O GEMM (+residual), RMSNorm, gate/up GEMM (+act*up),
//            down GEMM (+residual)] -> slot readout (final norm, label rows,
//            restricted log-softmax)
//   encoder: pack -> embed+LN -> L x [QKV GEMM (+bias), attention, O GEMM
//            (+bias, residual), LN, FFN GEMM (+bias, GELU), FFN GEMM (+bias,
//            residual), LN] -> +type -> head layers (pre-LN, ReLU) -> marker
//            gather + scorer.
// Batches with more real tokens than the workspace holds are split by rows.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <type_traits>
#include <vector>

#include "vdexec.h"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "attention_tc_head.cuh"
#include "checkpoint.hpp"
#include "common.cuh"
#include "convert.cuh"
#include "elementwise.cuh"
#include "gemm.cuh"
#include "gemm2.cuh"
#include "gdn.cuh"
#include "json.hpp"
#include "synth.cuh"

namespace vd {

using bf16 = __nv_bfloat16;

struct VdError {
  int code;
  std::string msg;
};

[[noreturn]] static void fail(int code, const std::string& msg) { throw VdError{code, msg}; }

// Fused RMSNorm with fp16 activations: the 16-bit copy of the residual rows
// (times the norm's gains) is stored times 2^-6, so rows up to 4.2e6 in
// magnitude stay inside fp16's range while values down to 2^-8 remain normal
// numbers (the row factor undoes it exactly).  bf16 has fp32's exponent range
// and stores the rows as they are.
constexpr float kNormPrescale16 = 1.0f / 64.0f;

// Small batches (M <= kSplitMaxM rows) run their projections as 128-row tiles
// on one CTA each, with K split over work units when that fills the SMs better
// (a 515-token decision has 5 row tiles: 80 tiles for a 4096-wide output on 148
// SMs).  The partial tiles live in a workspace of kSplitPartElems floats.
constexpr int kSplitMaxM = 1024;
constexpr int64_t kSplitPartElems = int64_t(64) << 20;  // 256 MB

// Splits of K (k-blocks of 64) for `tiles` output tiles on `sms` SMs: the
// fewest rounds of the longest unit, a split costing about two k-blocks of
// partial-tile traffic; 1 = no split.
static int choose_splits(int tiles, int kblocks, int sms, int max_splits) {
  double best = std::ceil(static_cast<double>(tiles) / sms) * kblocks;
  int pick = 1;
  for (int S = 2; S <= max_splits && kblocks / S >= 4; ++S) {
    const double t = std::ceil(static_cast<double>(tiles) * S / sms) * std::ceil(static_cast<double>(kblocks) / S) + 2.0;
    if (t < 0.95 * best) {
      best = t;
      pick = S;
    }
  }
  return pick;
}

static void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(VD_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// Model spec
// ---------------------------------------------------------------------------
struct ModelSpec {
  std::string arch, style, family;
  int hidden = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, ffn = 0, vocab = 0;
  double rms_eps = 1e-6, rope_theta = 1e6, init_std = 0.02, ln_eps = 1e-12;
  bool qk_norm = false, qkv_bias = false, tied = false, embed_scale = false, norm_plus_one = false;
  int act = kActSilu;
  uint64_t seed = 0;
  std::string checkpoint;  // safetensors directory; empty = seeded synthetic weights
  std::vector<int> label_ids;
  int max_pos = 512, type_vocab = 2, pad_id = 0, head_layers = 2;
  // hybrid (Qwen3.5) stacks: per-layer token mixer and gated-delta-net sizes
  std::vector<char> linear_layer;  // 1: gated delta net, 0: full attention
  double partial_rotary = 1.0;
  // independent-options encoders (ModernBERT): sliding-window layers and RoPE thetas
  std::vector<char> sliding_layer;  // 1: sliding window, 0: full attention
  double global_theta = 160000.0, local_theta = 10000.0;
  int sliding_window = 64;
  bool von() const { return style == "modernbert"; }
  int lin_k_heads = 0, lin_v_heads = 0, lin_k_dim = 128, lin_v_dim = 128, conv_kernel = 4;

  bool decoder() const { return arch == "decoder"; }
  bool hybrid() const { return style == "qwen3_5"; }
  // fused full-attention projection: q, k, v (and the output gate of a hybrid)
  int qkv_width() const { return (heads + 2 * kv_heads + (hybrid() ? heads : 0)) * head_dim; }
  int rot_dim() const { return static_cast<int>(head_dim * partial_rotary); }
  int gdn_kd() const { return lin_k_heads * lin_k_dim; }
  int gdn_vd() const { return lin_v_heads * lin_v_dim; }
  int gdn_conv() const { return 2 * gdn_kd() + gdn_vd(); }
  // fused in_proj columns: conv input, z, a, b, padded to 256-wide GEMM tiles
  int gdn_proj() const { return (gdn_conv() + gdn_vd() + 2 * lin_v_heads + 255) / 256 * 256; }
  bool any_linear() const {
    for (char c : linear_layer)
      if (c) return true;
    return false;
  }
};

static ModelSpec parse_spec(const Json& j) {
  ModelSpec s;
  s.arch = j.string_or("arch", "decoder");
  s.style = j.string_or("style", s.arch == "decoder" ? "qwen3" : "bert");
  s.hidden = static_cast<int>(j.integer("hidden"));
  s.layers = static_cast<int>(j.integer("layers"));
  s.heads = static_cast<int>(j.integer("heads"));
  s.ffn = static_cast<int>(j.integer("ffn"));
  s.vocab = static_cast<int>(j.integer("vocab"));
  s.seed = static_cast<uint64_t>(j.integer_or("seed", 0));
  s.init_std = j.number_or("init_std", 0.02);
  s.checkpoint = j.string_or("checkpoint", "");
  if (s.decoder()) {
    s.family = j.string_or("family", "letter_branches");
    std::replace(s.family.begin(), s.family.end(), '-', '_');
    s.kv_heads = static_cast<int>(j.integer("kv_heads"));
    s.head_dim = static_cast<int>(j.integer("head_dim"));
    s.rms_eps = j.number_or("rms_eps", 1e-6);
    s.rope_theta = j.number_or("rope_theta", 1e6);
    s.qk_norm = j.boolean_or("qk_norm", s.style == "qwen3");
    s.qkv_bias = j.boolean_or("qkv_bias", s.style == "qwen2");
    s.tied = j.boolean_or("tied", false);
    s.embed_scale = j.boolean_or("embed_scale", false);
    s.norm_plus_one = j.boolean_or("norm_plus_one", s.style == "qwen3_5");
    if (s.hybrid()) {
      if (!j.has("layer_types") || j.at("layer_types").kind != Json::Array)
        fail(VD_ESPEC, "a qwen3_5 spec needs \"layer_types\"");
      for (const Json& v : j.at("layer_types").arr) {
        if (v.str == "linear_attention") s.linear_layer.push_back(1);
        else if (v.str == "full_attention") s.linear_layer.push_back(0);
        else fail(VD_ESPEC, "unknown layer type \"" + v.str + "\"");
      }
      s.partial_rotary = j.number_or("partial_rotary", 0.25);
      s.lin_k_heads = static_cast<int>(j.integer("lin_k_heads"));
      s.lin_v_heads = static_cast<int>(j.integer("lin_v_heads"));
      s.lin_k_dim = static_cast<int>(j.integer_or("lin_k_dim", 128));
      s.lin_v_dim = static_cast<int>(j.integer_or("lin_v_dim", 128));
      s.conv_kernel = static_cast<int>(j.integer_or("conv_kernel", 4));
    }
    const std::string act = j.string_or("act", "silu");
    if (act == "silu") s.act = kActSilu;
    else if (act == "gelu_tanh") s.act = kActGeluTanh;
    else fail(VD_ESPEC, "unsupported decoder activation " + act);
    if (!j.has("label_ids") || j.at("label_ids").kind != Json::Array)
      fail(VD_ESPEC, "decoder spec needs the option-label table \"label_ids\"");
    for (const Json& v : j.at("label_ids").arr) s.label_ids.push_back(static_cast<int>(v.num));
  } else {
    s.family = j.string_or("family", s.style == "modernbert" ? "independent_options" : "marker_head");
    std::replace(s.family.begin(), s.family.end(), '-', '_');
    s.kv_heads = s.heads;
    s.head_dim = s.hidden / s.heads;
    s.max_pos = static_cast<int>(j.integer_or("max_pos", 512));
    s.type_vocab = static_cast<int>(j.integer_or("type_vocab", 2));
    s.pad_id = static_cast<int>(j.integer_or("pad_id", 0));
    s.head_layers = static_cast<int>(j.integer_or("head_layers", 2));
    s.ln_eps = j.number_or("ln_eps", 1e-12);
    if (s.von()) {
      if (!j.has("layer_types") || j.at("layer_types").kind != Json::Array)
        fail(VD_ESPEC, "a modernbert spec needs \"layer_types\"");
      for (const Json& v : j.at("layer_types").arr) {
        if (v.str == "sliding_attention") s.sliding_layer.push_back(1);
        else if (v.str == "full_attention") s.sliding_layer.push_back(0);
        else fail(VD_ESPEC, "unknown layer type \"" + v.str + "\"");
      }
      s.global_theta = j.number_or("global_theta", 160000.0);
      s.local_theta = j.number_or("local_theta", 10000.0);
      s.sliding_window = static_cast<int>(j.integer_or("sliding_window", 64));
      s.head_layers = 0;
    }
  }
  return s;
}

// ---------------------------------------------------------------------------
// Specs that name a checkpoint and leave its shape out take the shape from the
// checkpoint's HF config: `config.json` of a Qwen3 / Qwen2 / Gemma CausalLM, or
// `encoder/config.json` (else `config.json`) of the BERT / XLM-R encoder of a
// marker-head DecisionModel.  Keys given in the spec win.  verdict_b200's
// checkpoint.spec_from_checkpoint applies the same mapping.
// ---------------------------------------------------------------------------
static Json jnum(double v) {
  Json j;
  j.kind = Json::Number;
  j.num = v;
  return j;
}
static Json jbool(bool v) {
  Json j;
  j.kind = Json::Bool;
  j.b = v;
  return j;
}
static Json jstr(const std::string& v) {
  Json j;
  j.kind = Json::String;
  j.str = v;
  return j;
}

static bool file_exists(const std::string& path) {
  std::ifstream f(path);
  return static_cast<bool>(f);
}

static Json read_json_file(const std::string& path) {
  std::ifstream f(path);
  if (!f) fail(VD_ESPEC, "cannot read " + path);
  std::stringstream ss;
  ss << f.rdbuf();
  return parse_json(ss.str());
}

static Json spec_from_hf_config(const Json& c) {
  Json o;
  o.kind = Json::Object;
  const std::string mt = c.string_or("model_type", "");
  auto need_num = [&](const char* k) {
    if (!c.has(k) || c.at(k).kind != Json::Number) fail(VD_ESPEC, std::string("HF config has no number \"") + k + "\"");
    return c.at(k).num;
  };
  if (mt == "modernbert") {
    const double layers = need_num("num_hidden_layers");
    o.obj["arch"] = jstr("encoder");
    o.obj["style"] = jstr("modernbert");
    o.obj["hidden"] = jnum(need_num("hidden_size"));
    o.obj["layers"] = jnum(layers);
    o.obj["heads"] = jnum(need_num("num_attention_heads"));
    o.obj["ffn"] = jnum(need_num("intermediate_size"));
    o.obj["vocab"] = jnum(need_num("vocab_size"));
    o.obj["max_pos"] = jnum(c.number_or("max_position_embeddings", 8192));
    o.obj["ln_eps"] = jnum(c.number_or("norm_eps", 1e-5));
    o.obj["pad_id"] = jnum(c.number_or("pad_token_id", 0));
    if (c.boolean_or("norm_bias", false) || c.boolean_or("attention_bias", false) || c.boolean_or("mlp_bias", false))
      fail(VD_ESPEC, "modernbert checkpoints with norm / attention / MLP biases are not supported");
    const std::string act = c.string_or("hidden_activation", "gelu");
    if (act != "gelu") fail(VD_ESPEC, "unsupported modernbert activation \"" + act + "\"");
    double g_theta = c.number_or("global_rope_theta", 160000.0), l_theta = c.number_or("local_rope_theta", 10000.0);
    if (c.has("rope_parameters") && c.at("rope_parameters").kind == Json::Object) {
      const Json& rp = c.at("rope_parameters");
      for (const char* kind : {"full_attention", "sliding_attention"}) {
        if (!rp.has(kind) || rp.at(kind).kind != Json::Object) continue;
        const Json& r = rp.at(kind);
        if (r.string_or("rope_type", "default") != "default") fail(VD_ESPEC, "rope scaling is not supported");
        if (std::string(kind) == "full_attention") g_theta = r.number_or("rope_theta", g_theta);
        else l_theta = r.number_or("rope_theta", l_theta);
      }
    }
    o.obj["global_theta"] = jnum(g_theta);
    o.obj["local_theta"] = jnum(l_theta);
    o.obj["sliding_window"] = jnum(c.number_or("local_attention", 128) / 2);
    Json types;
    types.kind = Json::Array;
    if (c.has("layer_types") && c.at("layer_types").kind == Json::Array) {
      types = c.at("layer_types");
    } else {
      const int every = static_cast<int>(c.number_or("global_attn_every_n_layers", 3));
      for (int i = 0; i < static_cast<int>(layers); ++i)
        types.arr.push_back(jstr(i % every ? "sliding_attention" : "full_attention"));
    }
    o.obj["layer_types"] = types;
    o.obj["family"] = jstr("independent_options");
    return o;
  }
  if (mt == "bert" || mt == "xlm-roberta") {
    const std::string pe = c.string_or("position_embedding_type", "absolute");
    if (pe != "absolute") fail(VD_ESPEC, "only absolute position embeddings are supported, not " + pe);
    const std::string act = c.string_or("hidden_act", "gelu");
    if (act != "gelu") fail(VD_ESPEC, "unsupported encoder activation " + act);
    o.obj["arch"] = jstr("encoder");
    o.obj["style"] = jstr(mt == "bert" ? "bert" : "xlmr");
    o.obj["hidden"] = jnum(need_num("hidden_size"));
    o.obj["layers"] = jnum(need_num("num_hidden_layers"));
    o.obj["heads"] = jnum(need_num("num_attention_heads"));
    o.obj["ffn"] = jnum(need_num("intermediate_size"));
    o.obj["vocab"] = jnum(need_num("vocab_size"));
    o.obj["max_pos"] = jnum(need_num("max_position_embeddings"));
    o.obj["type_vocab"] = jnum(c.number_or("type_vocab_size", 2));
    o.obj["ln_eps"] = jnum(c.number_or("layer_norm_eps", 1e-12));
    o.obj["pad_id"] = jnum(c.number_or("pad_token_id", 0));
    o.obj["family"] = jstr("marker_head");
    return o;
  }
  if (mt == "qwen3_5" || mt == "qwen3_5_text") {
    // A Qwen3.5 text stack (the text_config of a vision-language checkpoint).
    const Json& t = (mt == "qwen3_5" && c.has("text_config") && c.at("text_config").kind == Json::Object)
                        ? c.at("text_config")
                        : c;
    auto num = [&](const char* k) {
      if (!t.has(k) || t.at(k).kind != Json::Number) fail(VD_ESPEC, std::string("HF config has no number \"") + k + "\"");
      return t.at(k).num;
    };
    double theta = t.number_or("rope_theta", 0.0), partial = t.number_or("partial_rotary_factor", 0.25);
    std::string rope_type = "default";
    if (t.has("rope_parameters") && t.at("rope_parameters").kind == Json::Object) {
      const Json& rp = t.at("rope_parameters");
      if (theta == 0.0) theta = rp.number_or("rope_theta", 0.0);
      partial = rp.number_or("partial_rotary_factor", partial);
      rope_type = rp.string_or("rope_type", "default");
    }
    if ((t.has("rope_scaling") && t.at("rope_scaling").kind == Json::Object) || rope_type != "default")
      fail(VD_ESPEC, "rope scaling is not supported");
    if (t.boolean_or("attention_bias", false)) fail(VD_ESPEC, "qwen3_5 checkpoints with attention bias are not supported");
    const std::string act = t.string_or("hidden_act", "silu");
    if (act != "silu" && act != "swish") fail(VD_ESPEC, "unsupported qwen3_5 activation \"" + act + "\"");
    const double heads = num("num_attention_heads"), layers = num("num_hidden_layers");
    o.obj["arch"] = jstr("decoder");
    o.obj["style"] = jstr("qwen3_5");
    o.obj["hidden"] = jnum(num("hidden_size"));
    o.obj["layers"] = jnum(layers);
    o.obj["heads"] = jnum(heads);
    o.obj["kv_heads"] = jnum(t.number_or("num_key_value_heads", heads));
    o.obj["head_dim"] = jnum(t.number_or("head_dim", 256));
    o.obj["ffn"] = jnum(num("intermediate_size"));
    o.obj["vocab"] = jnum(num("vocab_size"));
    o.obj["rms_eps"] = jnum(t.number_or("rms_norm_eps", 1e-6));
    o.obj["rope_theta"] = jnum(theta == 0.0 ? 10000.0 : theta);
    o.obj["partial_rotary"] = jnum(partial);
    o.obj["tied"] = jbool(t.boolean_or("tie_word_embeddings", c.boolean_or("tie_word_embeddings", false)));
    o.obj["qk_norm"] = jbool(true);
    o.obj["qkv_bias"] = jbool(false);
    o.obj["act"] = jstr("silu");
    o.obj["embed_scale"] = jbool(false);
    o.obj["norm_plus_one"] = jbool(true);
    o.obj["lin_k_heads"] = jnum(num("linear_num_key_heads"));
    o.obj["lin_v_heads"] = jnum(num("linear_num_value_heads"));
    o.obj["lin_k_dim"] = jnum(t.number_or("linear_key_head_dim", 128));
    o.obj["lin_v_dim"] = jnum(t.number_or("linear_value_head_dim", 128));
    o.obj["conv_kernel"] = jnum(t.number_or("linear_conv_kernel_dim", 4));
    Json types;
    types.kind = Json::Array;
    if (t.has("layer_types") && t.at("layer_types").kind == Json::Array) {
      types = t.at("layer_types");
    } else {
      const int every = static_cast<int>(t.number_or("full_attention_interval", 4));
      for (int i = 0; i < static_cast<int>(layers); ++i)
        types.arr.push_back(jstr((i + 1) % every ? "linear_attention" : "full_attention"));
    }
    o.obj["layer_types"] = types;
    o.obj["family"] = jstr("letter_readout");
    return o;
  }
  if (mt != "qwen3" && mt != "qwen2" && mt != "gemma")
    fail(VD_ESPEC, "unsupported model_type \"" + mt +
                       "\" (qwen3, qwen2, gemma, qwen3_5, bert, xlm-roberta are supported)");
  const double heads = need_num("num_attention_heads"), hidden = need_num("hidden_size");
  o.obj["arch"] = jstr("decoder");
  o.obj["style"] = jstr(mt);
  o.obj["hidden"] = jnum(hidden);
  o.obj["layers"] = jnum(need_num("num_hidden_layers"));
  o.obj["heads"] = jnum(heads);
  o.obj["kv_heads"] = jnum(c.number_or("num_key_value_heads", heads));
  o.obj["head_dim"] = jnum(c.number_or("head_dim", hidden / heads));
  o.obj["ffn"] = jnum(need_num("intermediate_size"));
  o.obj["vocab"] = jnum(need_num("vocab_size"));
  o.obj["rms_eps"] = jnum(c.number_or("rms_norm_eps", 1e-6));
  double theta = c.number_or("rope_theta", 0.0);
  std::string rope_type = "default";
  if (c.has("rope_parameters") && c.at("rope_parameters").kind == Json::Object) {
    const Json& rp = c.at("rope_parameters");
    if (theta == 0.0) theta = rp.number_or("rope_theta", 0.0);
    rope_type = rp.string_or("rope_type", "default");
  }
  if ((c.has("rope_scaling") && c.at("rope_scaling").kind == Json::Object) || rope_type != "default")
    fail(VD_ESPEC, "rope scaling is not supported");
  o.obj["rope_theta"] = jnum(theta == 0.0 ? 10000.0 : theta);
  o.obj["tied"] = jbool(c.boolean_or("tie_word_embeddings", mt == "gemma"));
  if (c.boolean_or("use_sliding_window", false)) fail(VD_ESPEC, "sliding-window attention is not supported");
  const std::string act = c.string_or("hidden_activation", c.string_or("hidden_act", ""));
  const bool gemma = mt == "gemma";
  if (gemma ? (act != "gelu_pytorch_tanh" && act != "gelu_tanh") : (act != "silu" && act != "swish"))
    fail(VD_ESPEC, "unsupported " + mt + " activation \"" + act + "\"");
  if (mt == "qwen3" && c.boolean_or("attention_bias", false))
    fail(VD_ESPEC, "qwen3 checkpoints with attention_bias (o_proj bias) are not supported");
  o.obj["qk_norm"] = jbool(mt == "qwen3");
  o.obj["qkv_bias"] = jbool(mt == "qwen2");
  o.obj["act"] = jstr(gemma ? "gelu_tanh" : "silu");
  o.obj["embed_scale"] = jbool(gemma);
  o.obj["norm_plus_one"] = jbool(gemma);
  o.obj["family"] = jstr("letter_readout");  // the torch executor's default family
  return o;
}

// The effective spec JSON object: `j`, with "checkpoint" resolved against
// `spec_dir` and, when "hidden" is absent, the checkpoint's HF config beneath it.
static Json resolve_spec(const Json& j, const std::string& spec_dir) {
  if (j.kind != Json::Object) fail(VD_ESPEC, "the model spec must be a JSON object");
  Json out = j;
  if (!j.has("checkpoint")) return out;
  std::string ck = j.string_or("checkpoint", "");
  if (ck.empty()) fail(VD_ESPEC, "\"checkpoint\" must be a non-empty path");
  if (ck[0] != '/' && !spec_dir.empty()) ck = spec_dir + "/" + ck;
  out.obj["checkpoint"] = jstr(ck);
  if (j.has("hidden")) return out;
  const std::string enc = ck + "/encoder/config.json";
  Json merged = spec_from_hf_config(read_json_file(file_exists(enc) ? enc : ck + "/config.json"));
  for (const auto& kv : out.obj) merged.obj[kv.first] = kv.second;
  return merged;
}

static void json_write(std::string& o, const Json& v) {
  char buf[64];
  switch (v.kind) {
    case Json::Null: o += "null"; break;
    case Json::Bool: o += v.b ? "true" : "false"; break;
    case Json::Number:
      std::snprintf(buf, sizeof(buf), "%.17g", v.num);
      o += buf;
      break;
    case Json::String:
      o += '"';
      for (char c : v.str) {
        if (c == '"' || c == '\\') {
          o += '\\';
          o += c;
        } else if (static_cast<unsigned char>(c) < 0x20) {
          std::snprintf(buf, sizeof(buf), "\\u%04x", c);
          o += buf;
        } else {
          o += c;
        }
      }
      o += '"';
      break;
    case Json::Array:
      o += '[';
      for (size_t i = 0; i < v.arr.size(); ++i) {
        if (i) o += ',';
        json_write(o, v.arr[i]);
      }
      o += ']';
      break;
    case Json::Object: {
      o += '{';
      bool first = true;
      for (const auto& kv : v.obj) {
        if (!first) o += ',';
        first = false;
        json_write(o, jstr(kv.first));
        o += ':';
        json_write(o, kv.second);
      }
      o += '}';
      break;
    }
  }
}

static void validate_spec(const ModelSpec& s) {
  auto need = [](bool ok, const std::string& why) {
    if (!ok) fail(VD_ESPEC, why);
  };
  need(s.hidden > 0 && s.hidden % 128 == 0, "hidden must be a positive multiple of 128");
  need(s.layers > 0 && s.heads > 0, "layers and heads must be positive");
  need(s.ffn % 128 == 0, "ffn must be a multiple of 128");
  if (s.decoder()) {
    need(s.style == "qwen3" || s.style == "qwen2" || s.style == "gemma" || s.style == "qwen3_5",
         "decoder style must be qwen3/qwen2/gemma/qwen3_5");
    if (s.hybrid()) {
      need(static_cast<int>(s.linear_layer.size()) == s.layers, "layer_types must list every layer");
      need(s.rot_dim() % 64 == 0 && s.rot_dim() > 0 && s.rot_dim() <= s.head_dim,
           "the rotary width (head_dim * partial_rotary) must be a positive multiple of 64");
      need(s.lin_k_dim == 128 && s.lin_v_dim == 128, "gated-delta-net head dims must be 128");
      need(s.lin_k_heads > 0 && s.lin_v_heads % s.lin_k_heads == 0, "lin_v_heads must be a multiple of lin_k_heads");
      need(s.conv_kernel == 4, "the gated delta net's conv kernel must be 4 wide");
      need(!s.any_linear() || s.gdn_vd() == s.heads * s.head_dim,
           "the gated delta net's value width must equal heads * head_dim (shared output buffer)");
      need(s.qkv_bias == false, "qwen3_5 has no attention bias");
    }
    need(s.head_dim == 128 || s.head_dim == 256, "decoder head_dim must be 128 or 256");
    need(s.kv_heads > 0 && s.heads % s.kv_heads == 0, "heads must be a multiple of kv_heads");
    need((s.heads * s.head_dim) % 128 == 0, "heads*head_dim must be a multiple of 128");
    need(s.head_dim == 128 || (s.heads * s.head_dim) % 256 == 0, "head_dim 256 needs 256-aligned q/k/v blocks");
    need(!s.label_ids.empty(), "empty label table");
    for (int id : s.label_ids) need(id >= 0 && id < s.vocab, "label id outside the vocabulary");
  } else {
    need(s.style == "bert" || s.style == "xlmr" || s.style == "modernbert",
         "encoder style must be bert, xlmr or modernbert");
    if (s.von()) {
      need(static_cast<int>(s.sliding_layer.size()) == s.layers, "layer_types must list every layer");
      need(s.family == "independent_options", "a modernbert encoder serves the independent_options family");
      need(s.sliding_window > 0, "sliding_window must be positive");
      need((3 * s.hidden) % 128 == 0, "3 * hidden must be a multiple of 128");
    }
    need(s.hidden % s.heads == 0 && s.hidden / s.heads == 64, "encoder head size must be 64");
    need(s.hidden % 64 == 0, "encoder hidden must be a multiple of 64");
  }
}

// ---------------------------------------------------------------------------
// Synthetic checkpoint naming (matches verdict_b200/synth.py)
// ---------------------------------------------------------------------------
static uint64_t fnv1a64(const std::string& s) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (unsigned char c : s) {
    h ^= c;
    h *= 0x100000001B3ull;
  }
  return h;
}
static uint64_t tensor_base(uint64_t seed, const std::string& name) {
  return fnv1a64(name) ^ (seed * 0x9E3779B97F4A7C15ull);
}

// ---------------------------------------------------------------------------
// Tensor maps
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) fail(VD_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return fn;
}

// Row-major [rows, cols] 16-bit matrix, box = [box_rows, 64] with 128-byte swizzle.
static CUtensorMap make_map(const void* ptr, int64_t rows, int64_t cols, int box_rows, bool f16 = true) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(VD_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
  return m;
}

// Output map of a GEMM epilogue: 32x32 boxes; 16-bit data with the 64-byte
// swizzle (TMA store), fp32 with the 128-byte swizzle (TMA reduce-add).
static CUtensorMap make_out_map(const void* ptr, int64_t rows, int64_t cols, bool fp32, bool f16 = true) {
  CUtensorMap m;
  const int elem = fp32 ? 4 : 2;
  if ((cols * elem) % 16 != 0) fail(VD_EINVAL, "output row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * elem};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : (f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  CUresult r = encode_fn()(&m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           fp32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    fail(VD_ECUDA, "cuTensorMapEncodeTiled (output) failed (" + std::to_string(static_cast<int>(r)) + ")");
  return m;
}

// ---------------------------------------------------------------------------
// Weights
// ---------------------------------------------------------------------------
struct Linear {
  void* w = nullptr;    // [n, k] 16-bit (the handle's element type)
  float* b = nullptr;   // [n] or null
  int n = 0, k = 0, bn = 256;
  CUtensorMap map;
  CUtensorMap map_half;  // 128-row boxes: one CTA's half of a 256-row tile (two-CTA GEMM)
};

struct DecLayer {
  float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  Linear qkv, o, gu, down;
  // gated-delta-net layers (hybrid stacks): qkv = fused in_proj, o = out_proj
  bool linear = false;
  float *conv_w = nullptr, *A_log = nullptr, *dt_bias = nullptr, *gdn_norm = nullptr;
};

struct EncLayer {
  Linear qkv, o, f1, f2;
  float *ln1_w = nullptr, *ln1_b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
  bool pre_norm = false;
  int act = kActGeluErf;
  float eps = 1e-12f;
  bool sliding = false;  // ModernBERT local layer
};

struct Handle;

struct Options {
  int64_t max_tokens = 65536, max_rows = 512, max_seq = 8192, max_markers = 16384;
  bool logprobs = true;
  bool f16 = true;  // activations and projection weights in fp16 (else bf16)
  bool prune_last_layer = true;  // last layer's O projection and MLP on the slot rows only
  bool tc_attention = true;  // head_dim 128 causal attention on tcgen05 (else the mma.sync kernel)
  bool tc_head = true;       // head_dim 128 on the one-head-per-CTA tcgen05 kernel (else two heads per CTA)
  bool fork = true;          // shared-prefix rows: prefix computed once (host-memory decoder batches)
  bool gemm2 = true;         // 256-wide projections on CTA pairs (cta_group::2), else one CTA per tile
  int raster_group = 0;      // M tiles per GEMM raster group; 0 = the kernel's default
  bool gdn_chunk = true;     // gated delta nets in 64-token chunks on the tensor cores, else token by token
  bool fuse_norm = true;     // decoders: RMSNorm fused into the residual GEMMs and the projections that read it
  bool split_k = false;      // small batches: K split over CTAs where that fills the SMs better (measured slower)
  bool attn_persistent = true;  // one-head tcgen05 attention: CTAs loop over work items
  int attn_spr = 1;             // one-head tcgen05 attention: softmax threads per query row (1 or 2)
  bool l2_hints = false;        // pair GEMM: L2 eviction hints on its TMA loads
  bool pdl = true;           // GEMMs and attention start their set-up under the previous kernel's tail
  uint64_t wait_ns = 0;      // limit of the GEMM kernels' barrier waits (0: the compiled 2 s)
  int debug_stall = 0;       // failure-path tests: the first one-CTA GEMM of a call stalls after this many k-blocks
};

}  // namespace vd

struct vd_handle {
  std::mutex mu;
  int device = 0;
  vd::ModelSpec spec;
  vd::Options opt;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  int gemm2_pairs = 0;  // concurrent CTA pairs of the two-CTA GEMM
  std::atomic<bool> healthy{true};
  std::string dead_reason;
  std::vector<void*> allocations;
  // open checkpoint (during vd_open only) and its device staging buffer
  std::unique_ptr<vd::Checkpoint> ckpt;
  void* ckpt_stage = nullptr;
  size_t ckpt_stage_bytes = 0;
  // decoder weights
  __nv_bfloat16* embed = nullptr;
  float* final_norm = nullptr;
  float* head_rows = nullptr;
  int n_labels = 0;
  std::vector<vd::DecLayer> dec;
  // encoder weights
  __nv_bfloat16 *pos_emb = nullptr, *type_emb0 = nullptr, *qtype_emb = nullptr;
  float *emb_ln_w = nullptr, *emb_ln_b = nullptr;
  std::vector<vd::EncLayer> enc, head;
  float *sc_ln_w = nullptr, *sc_ln_b = nullptr, *sc_w3 = nullptr, *sc_b3 = nullptr;
  vd::Linear sc1;
  // workspace
  float* h = nullptr;
  void *xn = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr, *mrow = nullptr, *mhid = nullptr;  // 16-bit
  int *tokens = nullptr, *positions = nullptr, *seq_id = nullptr, *cu = nullptr, *midx = nullptr, *d_err = nullptr;
  vd::AttnTile* tiles = nullptr;
  int64_t max_tiles = 0;
  vd::PackSeg* segs = nullptr;  // packed sequences of a chunk (rows, shared prefixes, suffixes)
  vd::RowMap* rowmap = nullptr; // per decision: where its slot token is packed
  float2* rope = nullptr;
  CUtensorMap map_xn, map_attn, map_act, map_act2, map_mrow, map_qkv, map_qkv64;
  // fused RMSNorm: block sums of squares of the residual rows ([rows, d / 64]),
  // two for the main rows (attention / MLP input), one for the slot rows
  float *ss_a = nullptr, *ss_b = nullptr, *ss_s = nullptr;
  // split-K partial tiles and per-tile arrival counters (small batches)
  float* split_part = nullptr;
  int64_t split_part_elems = 0;
  int* split_cnt = nullptr;
  int64_t split_cnt_n = 0;
  // last-layer slot rows (one per decision of a chunk)
  float* h_s = nullptr;
  void *xn_s = nullptr, *attn_s = nullptr, *act_s = nullptr;
  CUtensorMap map_xn_s, map_attn_s, map_act_s;
  // GEMM output maps (epilogue TMA stores / reduce-adds)
  CUtensorMap out_qkv, out_act, out_act2, out_h, out_h_s, out_act_s, out_mhid;
  CUtensorMap out_xn, out_xn_s;  // 16-bit residual copies written by the fused-norm epilogue
  // gated-delta-net workspace (hybrid stacks)
  int ld_qkv = 0;        // row stride of qkv (elements)
  // independent-options encoders: per-token option and option-invariant
  // position, the local-layer RoPE table, a zero bias for bias-free LayerNorms
  int *von_opt = nullptr, *von_pos = nullptr;
  float2* rope_local = nullptr;
  float* zero_d = nullptr;
  void* proj = nullptr;  // 16-bit [T, gdn_proj]
  float *gdn_g = nullptr, *gdn_beta = nullptr;
  CUtensorMap out_proj;
  // device copies of host batches
  int64_t *in_ids = nullptr, *in_mpos = nullptr, *in_nopts = nullptr, *in_qtype = nullptr;
  uint8_t* in_mmask = nullptr;
  float* out_dev = nullptr;
  int64_t out_cap = 0, cap_ids = 0, cap_markers = 0, cap_markers_mask = 0, cap_rows = 0, cap_rows_q = 0;
  // pinned staging ring for per-chunk metadata
  static constexpr int kSlots = 4;
  char* pinned[kSlots] = {};
  cudaEvent_t slot_ev[kSlots] = {};
  int slot = 0;
  size_t pinned_bytes = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev_user = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;  // host-memory calls: before the uploads, after the download
  vd_stats stats{};
  int64_t launches = 0;
  bool stall_pending = false;  // opt.debug_stall: not yet applied in this call
  // per-kernel event timing (vd_set_profiling)
  bool profiling = false;
  struct ProfRec {
    int kind;
    cudaEvent_t a, b;
  };
  std::vector<cudaEvent_t> prof_pool;
  size_t prof_next = 0;
  std::vector<ProfRec> prof;
};

namespace vd {

template <class T>
static T* dalloc(vd_handle* H, size_t count) {
  void* p = nullptr;
  if (count == 0) count = 1;
  cudaError_t e = cudaMalloc(&p, count * sizeof(T));
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(VD_ENOMEM, "cudaMalloc of " + std::to_string(count * sizeof(T)) + " bytes failed: " + cudaGetErrorString(e));
  }
  H->allocations.push_back(p);
  return static_cast<T*>(p);
}

static cudaEvent_t prof_event(vd_handle* H) {
  if (H->prof_next == H->prof_pool.size()) {
    cudaEvent_t e;
    cuda_check(cudaEventCreate(&e), "profiling event");
    H->prof_pool.push_back(e);
  }
  return H->prof_pool[H->prof_next++];
}

// The GEMM and attention kernels: launched with programmatic stream
// serialization (option "pdl"), a kernel's CTAs may start on SMs the
// previous kernel has left while it finishes; each waits for the previous
// kernel's results (griddepcontrol.wait) before it touches global memory.
template <class... KArgs, class... Args>
static void launch_k(vd_handle* H, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
  if (!H->opt.pdl) {
    kernel<<<grid, block, smem, H->stream>>>(std::forward<Args>(args)...);
    return;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = H->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cuda_check(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), "kernel launch");
}

// Every forward kernel goes through here: counts launches and algorithmic FLOPs
// per kernel class and, with profiling on, brackets the launch with events.
template <class F>
static void launch(vd_handle* H, int kind, double flops, F&& f) {
  cudaEvent_t a = nullptr;
  if (H->profiling) {
    a = prof_event(H);
    cuda_check(cudaEventRecord(a, H->stream), "profiling event");
  }
  f();
  ++H->launches;
  H->stats.kernel_launches[kind] += 1;
  H->stats.kernel_flops[kind] += flops;
  if (H->profiling) {
    cudaEvent_t b = prof_event(H);
    cuda_check(cudaEventRecord(b, H->stream), "profiling event");
    H->prof.push_back(vd_handle::ProfRec{kind, a, b});
  }
}

// After a synchronize: fold the recorded event pairs into per-class times.
static void prof_collect(vd_handle* H) {
  for (const auto& r : H->prof) {
    float ms = 0;
    if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) H->stats.kernel_ms[r.kind] += ms;
  }
  H->prof.clear();
  H->prof_next = 0;
}

static int grid_for(int64_t n) { return static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16)); }

// Weights come from one of two sources, by state-dict name: the seeded
// synthetic generator, or the open safetensors checkpoint.  Either way a
// [rows, cols] tensor lands row r at destination row (r / group) * stride +
// (r % group) + off (group = rows, stride 0: a plain copy at row `off`).
static constexpr size_t kStageBytes = size_t(64) << 20;

static std::string shape_str(const std::vector<int64_t>& v) {
  std::string o = "[";
  for (size_t i = 0; i < v.size(); ++i) o += (i ? ", " : "") + std::to_string(v[i]);
  return o + "]";
}

// Tensors of a vision-language checkpoint's text stack live under
// "model.language_model." instead of "model."; both are accepted.
static const StTensor& ckpt_get(vd_handle* H, const std::string& name) {
  if (H->ckpt->has(name)) return H->ckpt->get(name);
  if (name.compare(0, 6, "model.") == 0) {
    const std::string vl = "model.language_model." + name.substr(6);
    if (H->ckpt->has(vl)) return H->ckpt->get(vl);
  }
  fail(VD_ESPEC, "checkpoint " + H->spec.checkpoint + " has no tensor " + name);
}

static const StTensor& ckpt_tensor(vd_handle* H, const std::string& name, const std::vector<int64_t>& shape) {
  const StTensor& t = ckpt_get(H, name);
  if (t.shape != shape)
    fail(VD_ESPEC, "checkpoint tensor " + name + " has shape " + shape_str(t.shape) + ", the spec needs " +
                       shape_str(shape));
  return t;
}

// Host bytes -> staging buffer (stream-ordered, so the next slice waits for the
// conversion kernel that reads the previous one).
static void* stage_bytes(vd_handle* H, const void* src, size_t bytes) {
  if (!H->ckpt_stage) {
    if (cudaMalloc(&H->ckpt_stage, kStageBytes) != cudaSuccess) {
      cudaGetLastError();
      H->ckpt_stage = nullptr;
      fail(VD_ENOMEM, "cannot allocate the checkpoint staging buffer");
    }
  }
  if (bytes > kStageBytes) fail(VD_ESPEC, "checkpoint row larger than the staging buffer");
  cuda_check(cudaMemcpyAsync(H->ckpt_stage, src, bytes, cudaMemcpyHostToDevice, H->stream), "checkpoint upload");
  return H->ckpt_stage;
}

// Called once the stream has finished with the staging buffer (after a synchronize).
static void release_checkpoint(vd_handle* H) {
  if (H->ckpt_stage) cudaFree(H->ckpt_stage);
  H->ckpt_stage = nullptr;
  H->ckpt.reset();
}

template <class T>
static void fill_rows_t(vd_handle* H, T* dst, const std::string& name, int64_t rows, int64_t cols, float scale,
                        float offset, const RowPlace& place) {
  if (!H->ckpt) {
    synth_rows_kernel<T><<<grid_for(rows * cols), 256, 0, H->stream>>>(
        dst, rows, cols, tensor_base(H->spec.seed, name), scale, offset, place);
    return;
  }
  const StTensor& t = ckpt_tensor(H, name, {rows, cols});
  const size_t row_bytes = static_cast<size_t>(cols) * (t.dtype == kStF32 ? 4 : 2);
  const int64_t slice = std::max<int64_t>(1, static_cast<int64_t>(kStageBytes / row_bytes));
  for (int64_t r0 = 0; r0 < rows; r0 += slice) {
    const int64_t n = std::min(slice, rows - r0);
    const void* src = stage_bytes(H, t.data + static_cast<size_t>(r0) * row_bytes, static_cast<size_t>(n) * row_bytes);
    convert_rows_kernel<T><<<grid_for(n * cols), 256, 0, H->stream>>>(dst, src, t.dtype, r0, n, cols, place);
  }
}

// A 16-bit tensor in the element type `f16` selects (embedding tables are always bf16).
static void fill_w(vd_handle* H, void* dst, bool f16, const std::string& name, int64_t rows, int64_t cols,
                   float scale, float offset, int64_t group = 0, int64_t stride = 0, int64_t off = 0,
                   int64_t alt_off = -1, int64_t part_rows = 0, int64_t part_off = 0) {
  RowPlace place;
  place.group = group == 0 ? rows : group;
  place.stride = stride;
  place.off = off;
  place.alt_off = alt_off;
  place.part_rows = part_rows;
  place.part_off = part_off;
  if (f16) fill_rows_t(H, static_cast<__half*>(dst), name, rows, cols, scale, offset, place);
  else fill_rows_t(H, static_cast<__nv_bfloat16*>(dst), name, rows, cols, scale, offset, place);
}
static void fill_bf16(vd_handle* H, bf16* dst, const std::string& name, int64_t rows, int64_t cols, float scale,
                      float offset) {
  fill_w(H, dst, false, name, rows, cols, scale, offset);
}
static void fill_lin(vd_handle* H, void* dst, const std::string& name, int64_t rows, int64_t cols, float scale,
                     float offset, int64_t group = 0, int64_t stride = 0, int64_t off = 0, int64_t alt_off = -1,
                     int64_t part_rows = 0, int64_t part_off = 0) {
  fill_w(H, dst, H->opt.f16, name, rows, cols, scale, offset, group, stride, off, alt_off, part_rows, part_off);
}
// An fp32 vector of n elements (gains, biases; a [1, n] Linear weight qualifies).
static void fill_f32(vd_handle* H, float* dst, const std::string& name, int64_t n, float scale, float offset) {
  if (!H->ckpt) {
    synth_f32_kernel<<<grid_for(n), 256, 0, H->stream>>>(dst, n, tensor_base(H->spec.seed, name), scale, offset);
    return;
  }
  const StTensor& t = ckpt_get(H, name);
  if (t.numel() != n)
    fail(VD_ESPEC, "checkpoint tensor " + name + " has shape " + shape_str(t.shape) + ", the spec needs " +
                       std::to_string(n) + " elements");
  const void* src = stage_bytes(H, t.data, t.nbytes);
  convert_f32_kernel<<<grid_for(n), 256, 0, H->stream>>>(dst, src, t.dtype, n);
}
// Rows `ids` of a [vocab, cols] tensor as fp32 (the option-label rows of the LM head).
static void fill_rows_gather_f32(vd_handle* H, float* dst, const std::string& name, const std::vector<int>& ids,
                                 int64_t vocab, int64_t cols, float scale, float offset) {
  const int n = static_cast<int>(ids.size());
  if (!H->ckpt) {
    int* rows = dalloc<int>(H, n);
    cuda_check(cudaMemcpyAsync(rows, ids.data(), sizeof(int) * n, cudaMemcpyHostToDevice, H->stream),
               "upload label ids");
    synth_rows_gather_f32_kernel<<<grid_for(static_cast<int64_t>(n) * cols), 256, 0, H->stream>>>(
        dst, rows, n, cols, tensor_base(H->spec.seed, name), scale, offset);
    return;
  }
  const StTensor& t = ckpt_tensor(H, name, {vocab, cols});
  const size_t row_bytes = static_cast<size_t>(cols) * (t.dtype == kStF32 ? 4 : 2);
  std::vector<uint8_t> host(row_bytes * n);
  for (int i = 0; i < n; ++i) std::memcpy(host.data() + i * row_bytes, t.data + ids[i] * row_bytes, row_bytes);
  const void* src = stage_bytes(H, host.data(), host.size());
  convert_f32_kernel<<<grid_for(static_cast<int64_t>(n) * cols), 256, 0, H->stream>>>(dst, src, t.dtype,
                                                                                     static_cast<int64_t>(n) * cols);
  // `host` is pageable: the copy above has left it before returning.
}

static int pick_bn(int n) { return n % 256 == 0 ? 256 : 128; }

static void init_linear(vd_handle* H, Linear& L, int n, int k, bool bias, int bn = 0) {
  if (n % 128 != 0 || k % 64 != 0) fail(VD_ESPEC, "GEMM shape not tileable: N % 128 and K % 64 must be 0");
  L.n = n;
  L.k = k;
  L.bn = bn ? bn : pick_bn(n);
  L.w = dalloc<uint16_t>(H, static_cast<size_t>(n) * k);
  L.b = bias ? dalloc<float>(H, n) : nullptr;
  L.map = make_map(L.w, n, k, L.bn, H->opt.f16);
  if (L.bn == 256) L.map_half = make_map(L.w, n, k, 128, H->opt.f16);
}

static float2* upload_rope(vd_handle* H, int rot, double theta);

static void load_decoder(vd_handle* H) {
  const ModelSpec& s = H->spec;
  const int d = s.hidden, hd = s.head_dim, nq = s.heads, nkv = s.kv_heads, f = s.ffn;
  const float lin = static_cast<float>(s.init_std * std::sqrt(3.0));
  const float n_scale = 0.1f, n_off = s.norm_plus_one ? 0.0f : 1.0f;
  H->embed = dalloc<bf16>(H, static_cast<size_t>(s.vocab) * d);
  fill_bf16(H, H->embed, "model.embed_tokens.weight", s.vocab, d, lin, 0.0f);
  const int qc = nq * hd, kc = nkv * hd;
  // QKV tiles must not straddle the q / k / v column blocks.
  int bn_qkv = 256;
  if (hd == 128 && (qc % 256 != 0 || kc % 256 != 0)) bn_qkv = 128;
  H->dec.resize(s.layers);
  for (int i = 0; i < s.layers; ++i) {
    DecLayer& L = H->dec[i];
    const std::string p = "model.layers." + std::to_string(i) + ".";
    L.in_norm = dalloc<float>(H, d);
    L.post_norm = dalloc<float>(H, d);
    fill_f32(H, L.in_norm, p + "input_layernorm.weight", d, n_scale, n_off);
    fill_f32(H, L.post_norm, p + "post_attention_layernorm.weight", d, n_scale, n_off);
    if (s.hybrid() && s.linear_layer[i]) {
      // Gated delta net: fused in_proj rows [conv input (C) | z | a | b | zero pad].
      const std::string a = p + "linear_attn.";
      const int C = s.gdn_conv(), vd = s.gdn_vd(), lv = s.lin_v_heads;
      L.linear = true;
      init_linear(H, L.qkv, s.gdn_proj(), d, false, 256);
      cuda_check(cudaMemsetAsync(L.qkv.w, 0, static_cast<size_t>(L.qkv.n) * d * 2, H->stream), "clear in_proj");
      fill_lin(H, L.qkv.w, a + "in_proj_qkv.weight", C, d, lin, 0.0f, C, 0, 0);
      fill_lin(H, L.qkv.w, a + "in_proj_z.weight", vd, d, lin, 0.0f, vd, 0, C);
      fill_lin(H, L.qkv.w, a + "in_proj_a.weight", lv, d, lin, 0.0f, lv, 0, C + vd);
      fill_lin(H, L.qkv.w, a + "in_proj_b.weight", lv, d, lin, 0.0f, lv, 0, C + vd + lv);
      L.conv_w = dalloc<float>(H, static_cast<size_t>(C) * s.conv_kernel);
      fill_f32(H, L.conv_w, a + "conv1d.weight", static_cast<int64_t>(C) * s.conv_kernel, 0.5f, 0.0f);
      L.A_log = dalloc<float>(H, lv);
      L.dt_bias = dalloc<float>(H, lv);
      L.gdn_norm = dalloc<float>(H, s.lin_v_dim);
      fill_f32(H, L.A_log, a + "A_log", lv, 1.0f, 1.0f);
      fill_f32(H, L.dt_bias, a + "dt_bias", lv, 0.1f, 1.0f);
      fill_f32(H, L.gdn_norm, a + "norm.weight", s.lin_v_dim, 0.1f, 1.0f);
      init_linear(H, L.o, d, vd, false);
      fill_lin(H, L.o.w, a + "out_proj.weight", d, vd, lin, 0.0f);
      init_linear(H, L.gu, 2 * f, d, false, 256);
      fill_lin(H, L.gu.w, p + "mlp.gate_proj.weight", f, d, lin, 0.0f, 128, 256, 0);
      fill_lin(H, L.gu.w, p + "mlp.up_proj.weight", f, d, lin, 0.0f, 128, 256, 128);
      init_linear(H, L.down, d, f, false);
      fill_lin(H, L.down.w, p + "mlp.down_proj.weight", d, f, lin, 0.0f);
      continue;
    }
    init_linear(H, L.qkv, s.qkv_width(), d, s.qkv_bias, bn_qkv);
    if (s.hybrid()) {
      // Gated attention: q_proj holds [query | gate] per head; queries go to the
      // q block, gates after v.
      fill_lin(H, L.qkv.w, p + "self_attn.q_proj.weight", 2 * qc, d, lin, 0.0f, hd, hd, 0, qc + 2 * kc);
    } else {
      fill_lin(H, L.qkv.w, p + "self_attn.q_proj.weight", qc, d, lin, 0.0f, qc, 0, 0);
    }
    fill_lin(H, L.qkv.w, p + "self_attn.k_proj.weight", kc, d, lin, 0.0f, kc, 0, qc);
    fill_lin(H, L.qkv.w, p + "self_attn.v_proj.weight", kc, d, lin, 0.0f, kc, 0, qc + kc);
    if (s.qkv_bias) {
      fill_f32(H, L.qkv.b, p + "self_attn.q_proj.bias", qc, lin, 0.0f);
      fill_f32(H, L.qkv.b + qc, p + "self_attn.k_proj.bias", kc, lin, 0.0f);
      fill_f32(H, L.qkv.b + qc + kc, p + "self_attn.v_proj.bias", kc, lin, 0.0f);
    }
    if (s.qk_norm) {
      L.q_norm = dalloc<float>(H, hd);
      L.k_norm = dalloc<float>(H, hd);
      fill_f32(H, L.q_norm, p + "self_attn.q_norm.weight", hd, n_scale, n_off);
      fill_f32(H, L.k_norm, p + "self_attn.k_norm.weight", hd, n_scale, n_off);
    }
    init_linear(H, L.o, d, qc, false);
    fill_lin(H, L.o.w, p + "self_attn.o_proj.weight", d, qc, lin, 0.0f);
    init_linear(H, L.gu, 2 * f, d, false, 256);
    fill_lin(H, L.gu.w, p + "mlp.gate_proj.weight", f, d, lin, 0.0f, 128, 256, 0);
    fill_lin(H, L.gu.w, p + "mlp.up_proj.weight", f, d, lin, 0.0f, 128, 256, 128);
    init_linear(H, L.down, d, f, false);
    fill_lin(H, L.down.w, p + "mlp.down_proj.weight", d, f, lin, 0.0f);
  }
  H->final_norm = dalloc<float>(H, d);
  fill_f32(H, H->final_norm, "model.norm.weight", d, n_scale, n_off);
  H->n_labels = static_cast<int>(s.label_ids.size());
  H->head_rows = dalloc<float>(H, static_cast<size_t>(H->n_labels) * d);
  const std::string head_name = s.tied ? "model.embed_tokens.weight" : "lm_head.weight";
  fill_rows_gather_f32(H, H->head_rows, head_name, s.label_ids, s.vocab, d, lin, 0.0f);
  // rotary width: head_dim, or its partial_rotary fraction in a hybrid's attention
  H->rope = upload_rope(H, s.hybrid() ? s.rot_dim() : hd, s.rope_theta);
}

// RoPE table [max_seq][rot/2] of (cos, sin)(pos * inv_freq_i), inv_freq_i =
// 1 / theta^(2i/rot) in fp32.
static float2* upload_rope(vd_handle* H, int rot, double theta) {
  const int half = rot / 2;
  std::vector<float2> tab(static_cast<size_t>(H->opt.max_seq) * half);
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i)
    inv[i] = 1.0f / std::pow(static_cast<float>(theta), static_cast<float>(2 * i) / static_cast<float>(rot));
  for (int64_t pos = 0; pos < H->opt.max_seq; ++pos)
    for (int i = 0; i < half; ++i) {
      const float a = static_cast<float>(pos) * inv[i];
      tab[pos * half + i] = make_float2(static_cast<float>(std::cos(static_cast<double>(a))),
                                        static_cast<float>(std::sin(static_cast<double>(a))));
    }
  float2* out = dalloc<float2>(H, tab.size());
  cuda_check(cudaMemcpy(out, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice), "upload rope");
  return out;
}

static void enc_linear(vd_handle* H, Linear& L, const std::string& wname, const std::string& bname, int n, int k,
                       float lin) {
  init_linear(H, L, n, k, true);
  fill_lin(H, L.w, wname, n, k, lin, 0.0f);
  fill_f32(H, L.b, bname, n, lin, 0.0f);
}

// ModernBERT encoder + per-marker scorer (independent-options family), HF
// `ModernBertModel` names under "encoder.", the scorer under "scorer.".
static void load_von(vd_handle* H) {
  const ModelSpec& s = H->spec;
  const int d = s.hidden, f = s.ffn;
  const float lin = static_cast<float>(s.init_std * std::sqrt(3.0));
  const float g_scale = 0.1f, g_off = 1.0f;
  // scales in double, rounded once, exactly as the host generator computes them
  const double unit_d = 1.0 / std::sqrt(static_cast<double>(d));
  const float unit = static_cast<float>(unit_d);
  const float unit_lin = static_cast<float>(unit_d * std::sqrt(3.0));
  const float unit_out = static_cast<float>(unit_d * std::sqrt(3.0) * 4.0);
  const std::string e = "encoder.";
  H->embed = dalloc<bf16>(H, static_cast<size_t>(s.vocab) * d);
  fill_bf16(H, H->embed, e + "embeddings.tok_embeddings.weight", s.vocab, d, lin, 0.0f);
  H->zero_d = dalloc<float>(H, d);
  cuda_check(cudaMemsetAsync(H->zero_d, 0, sizeof(float) * d, H->stream), "zero bias");
  H->emb_ln_w = dalloc<float>(H, d);
  fill_f32(H, H->emb_ln_w, e + "embeddings.norm.weight", d, g_scale, g_off);
  H->enc.resize(s.layers);
  for (int i = 0; i < s.layers; ++i) {
    EncLayer& L = H->enc[i];
    const std::string p = e + "layers." + std::to_string(i) + ".";
    init_linear(H, L.qkv, 3 * d, d, false);
    fill_lin(H, L.qkv.w, p + "attn.Wqkv.weight", 3 * d, d, lin, 0.0f);
    init_linear(H, L.o, d, d, false);
    fill_lin(H, L.o.w, p + "attn.Wo.weight", d, d, lin, 0.0f);
    // Wi = [input; gate]: gelu(input) * gate, interleaved into 128-row gate/up blocks
    init_linear(H, L.f1, 2 * f, d, false, 256);
    fill_lin(H, L.f1.w, p + "mlp.Wi.weight", 2 * f, d, lin, 0.0f, 128, 256, 0, -1, f, 128);
    init_linear(H, L.f2, d, f, false);
    fill_lin(H, L.f2.w, p + "mlp.Wo.weight", d, f, lin, 0.0f);
    if (i > 0) {
      L.ln1_w = dalloc<float>(H, d);
      fill_f32(H, L.ln1_w, p + "attn_norm.weight", d, g_scale, g_off);
    }
    L.ln1_b = H->zero_d;
    L.ln2_w = dalloc<float>(H, d);
    fill_f32(H, L.ln2_w, p + "mlp_norm.weight", d, g_scale, g_off);
    L.ln2_b = H->zero_d;
    L.pre_norm = true;
    L.act = kActGeluErf;
    L.eps = static_cast<float>(s.ln_eps);
    L.sliding = s.sliding_layer[i] != 0;
  }
  H->final_norm = dalloc<float>(H, d);
  fill_f32(H, H->final_norm, e + "final_norm.weight", d, g_scale, g_off);
  H->sc_ln_w = dalloc<float>(H, d);
  H->sc_ln_b = dalloc<float>(H, d);
  fill_f32(H, H->sc_ln_w, "scorer.0.weight", d, g_scale, g_off);
  fill_f32(H, H->sc_ln_b, "scorer.0.bias", d, lin, 0.0f);
  init_linear(H, H->sc1, d, d, true);
  fill_lin(H, H->sc1.w, "scorer.1.weight", d, d, unit_lin, 0.0f);
  fill_f32(H, H->sc1.b, "scorer.1.bias", d, unit, 0.0f);
  H->sc_w3 = dalloc<float>(H, d);
  H->sc_b3 = dalloc<float>(H, 1);
  fill_f32(H, H->sc_w3, "scorer.3.weight", d, unit_out, 0.0f);
  fill_f32(H, H->sc_b3, "scorer.3.bias", 1, unit, 0.0f);
  H->rope = upload_rope(H, s.head_dim, s.global_theta);
  H->rope_local = upload_rope(H, s.head_dim, s.local_theta);
}

static void load_encoder(vd_handle* H) {
  if (H->spec.von()) {
    load_von(H);
    return;
  }
  const ModelSpec& s = H->spec;
  const int d = s.hidden, f = s.ffn;
  const float lin = static_cast<float>(s.init_std * std::sqrt(3.0));
  const float g_scale = 0.1f, g_off = 1.0f;
  const std::string e = "encoder.embeddings.";
  H->embed = dalloc<bf16>(H, static_cast<size_t>(s.vocab) * d);
  fill_bf16(H, H->embed, e + "word_embeddings.weight", s.vocab, d, lin, 0.0f);
  H->pos_emb = dalloc<bf16>(H, static_cast<size_t>(s.max_pos) * d);
  fill_bf16(H, H->pos_emb, e + "position_embeddings.weight", s.max_pos, d, lin, 0.0f);
  H->type_emb0 = dalloc<bf16>(H, static_cast<size_t>(s.type_vocab) * d);
  fill_bf16(H, H->type_emb0, e + "token_type_embeddings.weight", s.type_vocab, d, lin, 0.0f);
  H->emb_ln_w = dalloc<float>(H, d);
  H->emb_ln_b = dalloc<float>(H, d);
  fill_f32(H, H->emb_ln_w, e + "LayerNorm.weight", d, g_scale, g_off);
  fill_f32(H, H->emb_ln_b, e + "LayerNorm.bias", d, lin, 0.0f);
  H->enc.resize(s.layers);
  for (int i = 0; i < s.layers; ++i) {
    EncLayer& L = H->enc[i];
    const std::string p = "encoder.encoder.layer." + std::to_string(i) + ".";
    init_linear(H, L.qkv, 3 * d, d, true);
    const char* parts[3] = {"query", "key", "value"};
    for (int j = 0; j < 3; ++j) {
      fill_lin(H, L.qkv.w, p + "attention.self." + parts[j] + ".weight", d, d, lin, 0.0f, d, 0,
                 static_cast<int64_t>(j) * d);
      fill_f32(H, L.qkv.b + j * d, p + "attention.self." + parts[j] + ".bias", d, lin, 0.0f);
    }
    enc_linear(H, L.o, p + "attention.output.dense.weight", p + "attention.output.dense.bias", d, d, lin);
    enc_linear(H, L.f1, p + "intermediate.dense.weight", p + "intermediate.dense.bias", f, d, lin);
    enc_linear(H, L.f2, p + "output.dense.weight", p + "output.dense.bias", d, f, lin);
    L.ln1_w = dalloc<float>(H, d);
    L.ln1_b = dalloc<float>(H, d);
    L.ln2_w = dalloc<float>(H, d);
    L.ln2_b = dalloc<float>(H, d);
    fill_f32(H, L.ln1_w, p + "attention.output.LayerNorm.weight", d, g_scale, g_off);
    fill_f32(H, L.ln1_b, p + "attention.output.LayerNorm.bias", d, lin, 0.0f);
    fill_f32(H, L.ln2_w, p + "output.LayerNorm.weight", d, g_scale, g_off);
    fill_f32(H, L.ln2_b, p + "output.LayerNorm.bias", d, lin, 0.0f);
    L.pre_norm = false;
    L.act = kActGeluErf;
    L.eps = static_cast<float>(s.ln_eps);
  }
  H->qtype_emb = dalloc<bf16>(H, 3 * static_cast<size_t>(d));
  fill_bf16(H, H->qtype_emb, "type_emb.weight", 3, d, lin, 0.0f);
  H->head.resize(s.head_layers);
  for (int i = 0; i < s.head_layers; ++i) {
    EncLayer& L = H->head[i];
    const std::string p = "head.layers." + std::to_string(i) + ".";
    enc_linear(H, L.qkv, p + "self_attn.in_proj_weight", p + "self_attn.in_proj_bias", 3 * d, d, lin);
    enc_linear(H, L.o, p + "self_attn.out_proj.weight", p + "self_attn.out_proj.bias", d, d, lin);
    enc_linear(H, L.f1, p + "linear1.weight", p + "linear1.bias", 4 * d, d, lin);
    enc_linear(H, L.f2, p + "linear2.weight", p + "linear2.bias", d, 4 * d, lin);
    L.ln1_w = dalloc<float>(H, d);
    L.ln1_b = dalloc<float>(H, d);
    L.ln2_w = dalloc<float>(H, d);
    L.ln2_b = dalloc<float>(H, d);
    fill_f32(H, L.ln1_w, p + "norm1.weight", d, g_scale, g_off);
    fill_f32(H, L.ln1_b, p + "norm1.bias", d, lin, 0.0f);
    fill_f32(H, L.ln2_w, p + "norm2.weight", d, g_scale, g_off);
    fill_f32(H, L.ln2_b, p + "norm2.bias", d, lin, 0.0f);
    L.pre_norm = true;
    L.act = kActRelu;
    L.eps = 1e-5f;  // nn.TransformerEncoderLayer default layer_norm_eps
  }
  H->sc_ln_w = dalloc<float>(H, d);
  H->sc_ln_b = dalloc<float>(H, d);
  fill_f32(H, H->sc_ln_w, "scorer.0.weight", d, g_scale, g_off);
  fill_f32(H, H->sc_ln_b, "scorer.0.bias", d, lin, 0.0f);
  enc_linear(H, H->sc1, "scorer.1.weight", "scorer.1.bias", d, d, lin);
  H->sc_w3 = dalloc<float>(H, d);
  H->sc_b3 = dalloc<float>(H, 1);
  fill_f32(H, H->sc_w3, "scorer.3.weight", d, lin, 0.0f);
  fill_f32(H, H->sc_b3, "scorer.3.bias", 1, lin, 0.0f);
}

// Device copies of host-memory batches; grown on demand (only when a batch is
// larger than any before it).
static void ensure_host_inputs(vd_handle* H, int64_t n_ids, int64_t n_markers, int64_t n_rows, int64_t n_out) {
  auto grow = [&](auto*& ptr, int64_t& cap, int64_t need, size_t elem) {
    if (need <= cap && ptr) return;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    cap = 0;
    void* p = nullptr;
    const int64_t n = std::max<int64_t>(need, 1);
    const cudaError_t e = cudaMalloc(&p, static_cast<size_t>(n) * elem);
    if (e != cudaSuccess) {
      cudaGetLastError();
      fail(VD_ENOMEM, std::string("input staging allocation failed: ") + cudaGetErrorString(e));
    }
    ptr = static_cast<std::remove_reference_t<decltype(ptr)>>(p);
    cap = n;
  };
  grow(H->in_ids, H->cap_ids, n_ids, sizeof(int64_t));
  grow(H->in_mpos, H->cap_markers, n_markers, sizeof(int64_t));
  int64_t cap_mask = H->cap_markers_mask;
  grow(H->in_mmask, cap_mask, n_markers, sizeof(uint8_t));
  H->cap_markers_mask = cap_mask;
  grow(H->in_nopts, H->cap_rows, n_rows, sizeof(int64_t));
  int64_t cap_q = H->cap_rows_q;
  grow(H->in_qtype, cap_q, n_rows, sizeof(int64_t));
  H->cap_rows_q = cap_q;
  grow(H->out_dev, H->out_cap, n_out, sizeof(float));
}

static void alloc_workspace(vd_handle* H) {
  const ModelSpec& s = H->spec;
  const Options& o = H->opt;
  const int64_t T = o.max_tokens;
  const int d = s.hidden;
  const int qkvw = s.decoder() ? std::max(s.qkv_width(), s.hybrid() ? s.gdn_conv() : 0) : 3 * d;
  const int attw = s.decoder() ? s.heads * s.head_dim : d;
  const int actw = s.decoder() ? s.ffn : std::max(s.ffn, 4 * d);
  H->h = dalloc<float>(H, T * d);
  H->xn = dalloc<uint16_t>(H, T * d);
  H->qkv = dalloc<uint16_t>(H, T * qkvw);
  H->ld_qkv = qkvw;
  // Attention tiles read whole 128-row K/V blocks, including rows past the
  // batch (masked to probability 0); zeroing once keeps those rows finite.
  cuda_check(cudaMemset(H->qkv, 0, static_cast<size_t>(T) * qkvw * 2), "clear qkv workspace");
  H->attn = dalloc<uint16_t>(H, T * attw);
  H->act = dalloc<uint16_t>(H, T * actw);
  // Rows past a batch's tokens are read as padding by the GEMMs (the last
  // tile) and attention (masked keys): start them at zero, never garbage.
  cuda_check(cudaMemset(H->h, 0, static_cast<size_t>(T) * d * 4), "clear residual workspace");
  cuda_check(cudaMemset(H->xn, 0, static_cast<size_t>(T) * d * 2), "clear normalised-input workspace");
  cuda_check(cudaMemset(H->attn, 0, static_cast<size_t>(T) * attw * 2), "clear attention workspace");
  cuda_check(cudaMemset(H->act, 0, static_cast<size_t>(T) * actw * 2), "clear activation workspace");
  H->tokens = dalloc<int>(H, T);
  H->positions = dalloc<int>(H, T);
  H->seq_id = dalloc<int>(H, T);
  H->cu = dalloc<int>(H, o.max_rows + 1);
  // A chunk packs at most 2 sequences per row (a shared prefix and a suffix).
  H->max_tiles = T / 64 + 2 * o.max_rows + 1;
  H->tiles = dalloc<AttnTile>(H, H->max_tiles);
  H->segs = dalloc<PackSeg>(H, 2 * o.max_rows);
  H->rowmap = dalloc<RowMap>(H, o.max_rows);
  H->d_err = dalloc<int>(H, 1);
  cuda_check(cudaMemset(H->d_err, 0, sizeof(int)), "clear error word");
  const bool f16 = o.f16;
  H->map_xn = make_map(H->xn, T, d, 128, f16);
  H->map_attn = make_map(H->attn, T, attw, 128, f16);
  H->map_qkv = make_map(H->qkv, T, qkvw, 128, f16);
  H->map_qkv64 = make_map(H->qkv, T, qkvw, 64, f16);
  H->out_qkv = make_out_map(H->qkv, T, qkvw, false, f16);
  H->out_h = make_out_map(H->h, T, d, true);
  if (s.decoder()) {
    const int64_t R = std::max<int64_t>(o.max_rows, 128);  // at least one 128-row TMA box
    H->h_s = dalloc<float>(H, R * d);
    H->xn_s = dalloc<uint16_t>(H, R * d);
    H->attn_s = dalloc<uint16_t>(H, R * attw);
    H->act_s = dalloc<uint16_t>(H, R * s.ffn);
    cuda_check(cudaMemset(H->h_s, 0, static_cast<size_t>(R) * d * 4), "clear slot-row workspace");
    cuda_check(cudaMemset(H->xn_s, 0, static_cast<size_t>(R) * d * 2), "clear slot-row workspace");
    cuda_check(cudaMemset(H->attn_s, 0, static_cast<size_t>(R) * attw * 2), "clear slot-row workspace");
    cuda_check(cudaMemset(H->act_s, 0, static_cast<size_t>(R) * s.ffn * 2), "clear slot-row workspace");
    H->map_xn_s = make_map(H->xn_s, R, d, 128, f16);
    H->map_attn_s = make_map(H->attn_s, R, attw, 128, f16);
    H->map_act_s = make_map(H->act_s, R, s.ffn, 128, f16);
    H->out_act_s = make_out_map(H->act_s, R, s.ffn, false, f16);
    H->out_h_s = make_out_map(H->h_s, R, d, true);
    H->out_xn = make_out_map(H->xn, T, d, false, f16);
    H->out_xn_s = make_out_map(H->xn_s, R, d, false, f16);
    if (d % kNormBlock != 0) fail(VD_ESPEC, "hidden size must be a multiple of 64");
    H->ss_a = dalloc<float>(H, T * (d / kNormBlock));
    H->ss_b = dalloc<float>(H, T * (d / kNormBlock));
    H->ss_s = dalloc<float>(H, R * (d / kNormBlock));
  }
  H->map_act = make_map(H->act, T, s.ffn, 128, f16);
  H->out_act = make_out_map(H->act, T, s.ffn, false, f16);
  if (o.split_k) {
    // Widest projection of the model: the fused gate/up (2 ffn), QKV, or hidden.
    const int64_t max_n = std::max<int64_t>({2 * static_cast<int64_t>(std::max(s.ffn, 4 * d)), qkvw, d,
                                              s.decoder() && s.any_linear() ? s.gdn_proj() : 0});
    H->split_part_elems = kSplitPartElems;
    H->split_part = dalloc<float>(H, H->split_part_elems);
    H->split_cnt_n = (kSplitMaxM / 128) * ((max_n + 127) / 128);
    H->split_cnt = dalloc<int>(H, H->split_cnt_n);
    cuda_check(cudaMemset(H->split_cnt, 0, sizeof(int) * H->split_cnt_n), "clear split-K counters");
  }
  if (s.decoder() && s.any_linear()) {
    // gated-delta-net in_proj output and per-(token, v head) gates
    H->proj = dalloc<uint16_t>(H, T * s.gdn_proj());
    H->out_proj = make_out_map(H->proj, T, s.gdn_proj(), false, f16);
    H->gdn_g = dalloc<float>(H, T * s.lin_v_heads);
    H->gdn_beta = dalloc<float>(H, T * s.lin_v_heads);
  }
  if (!s.decoder()) {
    H->map_act2 = make_map(H->act, T, 4 * d, 128, f16);
    H->out_act2 = make_out_map(H->act, T, 4 * d, false, f16);
    H->midx = dalloc<int>(H, o.max_markers);
    H->mrow = dalloc<uint16_t>(H, o.max_markers * d);
    H->mhid = dalloc<uint16_t>(H, o.max_markers * d);
    H->map_mrow = make_map(H->mrow, o.max_markers, d, 128, f16);
    H->out_mhid = make_out_map(H->mhid, o.max_markers, d, false, f16);
    if (s.von()) {
      H->von_opt = dalloc<int>(H, T);
      H->von_pos = dalloc<int>(H, T);
    }
  }
  ensure_host_inputs(H, o.max_rows * 1024, std::max(o.max_rows, o.max_markers), o.max_rows,
                     std::max<int64_t>(o.max_rows * 256, o.max_markers));
  H->pinned_bytes = sizeof(int) * (o.max_rows + 1) + sizeof(PackSeg) * 2 * o.max_rows +
                    sizeof(RowMap) * o.max_rows + sizeof(AttnTile) * H->max_tiles + 256;
  for (int i = 0; i < vd_handle::kSlots; ++i) {
    cuda_check(cudaHostAlloc(reinterpret_cast<void**>(&H->pinned[i]), H->pinned_bytes, cudaHostAllocDefault),
               "pinned staging");
    cuda_check(cudaEventCreateWithFlags(&H->slot_ev[i], cudaEventDisableTiming), "event");
  }
  cuda_check(cudaEventCreate(&H->ev0), "event");
  cuda_check(cudaEventCreate(&H->ev1), "event");
  cuda_check(cudaEventCreate(&H->ev_in), "event");
  cuda_check(cudaEventCreate(&H->ev_out), "event");
  cuda_check(cudaEventCreateWithFlags(&H->ev_user, cudaEventDisableTiming), "event");
}

// ---------------------------------------------------------------------------
// Kernel launch helpers
// ---------------------------------------------------------------------------
template <int BN, int EPI, class T>
static void set_gemm_attr() {
  cuda_check(cudaFuncSetAttribute(gemm_tcgen05_kernel<BN, EPI, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  GemmConfig<BN>::SMEM_BYTES),
             "gemm smem attribute");
}
template <int HD, bool C, class T>
static void set_attn_attr() {
  cuda_check(cudaFuncSetAttribute(attention_varlen_kernel<HD, C, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  AttnConfig<HD>::SMEM_BYTES),
             "attention smem attribute");
}

template <int HD, class T, bool C, int SPR>
static void set_attn_head_attr() {
  cuda_check(cudaFuncSetAttribute(attention_tc_head_kernel<HD, T, C, SPR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  AttnTcHeadConfig<HD, SPR>::SMEM_BYTES),
             "tcgen05 one-head attention smem attribute");
}

template <class T>
static void init_kernel_attrs_t() {
  set_gemm_attr<256, kEpiStore, T>();
  set_gemm_attr<128, kEpiStore, T>();
  set_gemm_attr<256, kEpiResidual, T>();
  set_gemm_attr<128, kEpiResidual, T>();
  set_gemm_attr<256, kEpiGated, T>();
  set_gemm_attr<256, kEpiQKRope, T>();
  set_gemm_attr<128, kEpiQKRope, T>();
  set_gemm_attr<256, kEpiResidualNorm, T>();
  set_gemm_attr<128, kEpiResidualNorm, T>();
  for (auto f : {gemm2_tcgen05_kernel<kEpiStore, T>, gemm2_tcgen05_kernel<kEpiResidual, T>,
                 gemm2_tcgen05_kernel<kEpiGated, T>, gemm2_tcgen05_kernel<kEpiQKRope, T>,
                 gemm2_tcgen05_kernel<kEpiResidualNorm, T>})
    cuda_check(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, Gemm2Config::SMEM_BYTES),
               "two-CTA gemm smem attribute");
  set_attn_attr<64, false, T>();
  set_attn_attr<128, true, T>();
  set_attn_attr<256, true, T>();
  cuda_check(cudaFuncSetAttribute(attention_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  AttnTcConfig::SMEM_BYTES),
             "tcgen05 attention smem attribute");
  set_attn_head_attr<128, T, true, 1>();
  set_attn_head_attr<256, T, true, 1>();
  set_attn_head_attr<64, T, false, 1>();
  set_attn_head_attr<128, T, true, 2>();
  set_attn_head_attr<256, T, true, 2>();
  set_attn_head_attr<64, T, false, 2>();
  cuda_check(cudaFuncSetAttribute(gdn_chunk_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  GdnChunkConfig::SMEM_BYTES),
             "chunked gated delta net smem attribute");
}

static void init_kernel_attrs() {
  init_kernel_attrs_t<__half>();
  init_kernel_attrs_t<__nv_bfloat16>();
}

// CTA pairs of the two-CTA GEMM that fit on the current device at once (0: none).
static int gemm2_max_pairs(int num_sms) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms & ~1), 1, 1);
  cfg.blockDim = dim3(Gemm2Config::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Gemm2Config::SMEM_BYTES;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm2_tcgen05_kernel<kEpiStore, __half>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// c: the output map; c2: the second output of kEpiResidualNorm (the 16-bit copy).
template <int EPI, class T>
static void gemm(vd_handle* H, int kind, const CUtensorMap& a, const Linear& L, int M, const EpiParams& ep,
                 const CUtensorMap& c, const CUtensorMap* c2 = nullptr) {
  if (M <= 0) return;
  if (EPI == kEpiResidualNorm && c2 == nullptr) fail(VD_EINVAL, "residual-norm GEMM needs the copy's map");
  const CUtensorMap& d = c2 ? *c2 : c;
  const int num_m = (M + 127) / 128;
  const int tiles = num_m * (L.n / L.bn);
  const int grid = std::min(tiles, H->num_sms);
  GemmShape shape{M, L.n, L.k, H->opt.raster_group > 0 ? H->opt.raster_group : GemmConfig<256>::GROUP_M,
                  H->opt.wait_ns, 0, 1, nullptr, nullptr, H->opt.l2_hints ? 1 : 0};
  const double flops = 2.0 * M * static_cast<double>(L.n) * L.k;
  // Failure-path tests: the first one-CTA GEMM of the call stalls its producer.
  auto stall_one_cta = [&] {
    if (H->stall_pending) {
      shape.stall_after = H->opt.debug_stall;
      H->stall_pending = false;
    }
  };
  if (H->split_part && M <= kSplitMaxM) {
    const int m_pad = num_m * 128;
    const int64_t plane = static_cast<int64_t>(m_pad) * L.n;
    const int max_s = static_cast<int>(std::min<int64_t>(8, H->split_part_elems / plane));
    const int S = tiles <= H->split_cnt_n ? choose_splits(tiles, L.k / 64, H->num_sms, max_s) : 1;
    if (S > 1) {
      shape.splits = S;
      shape.part = H->split_part;
      shape.counters = H->split_cnt;
      const int grid_s = std::min(tiles * S, H->num_sms);
      stall_one_cta();
      launch(H, kind, flops, [&] {
        if (L.bn == 256) {
          launch_k(H, gemm_tcgen05_kernel<256, EPI, T>, grid_s, GemmConfig<256>::THREADS,
                   GemmConfig<256>::SMEM_BYTES, a, L.map, c, d, shape, ep, H->d_err);
        } else {
          if constexpr (EPI == kEpiGated) fail(VD_ESPEC, "gated GEMM needs 256-wide tiles");
          else
            launch_k(H, gemm_tcgen05_kernel<128, EPI, T>, grid_s, GemmConfig<128>::THREADS,
                     GemmConfig<128>::SMEM_BYTES, a, L.map, c, d, shape, ep, H->d_err);
        }
      });
      return;
    }
  }
  if (L.bn == 256 && H->opt.gemm2 && H->gemm2_pairs > 0) {
    const int pair_tiles = ((M + 255) / 256) * (L.n / 256);
    // A GEMM of a wave or two of CTA pairs (short batches, the encoders' 768-
    // wide projections) leaves SMs idle; as 128 x 128 tiles on single CTAs
    // (the W map with 128-row boxes) it spreads over all SMs.  A 128 x 128
    // tile runs well below half a pair tile's rate, so this is taken only
    // when it needs at most half the pair kernel's per-SM tile rounds (a pair
    // tile is two 128 x 128 tiles per SM).
    if constexpr (EPI == kEpiStore || EPI == kEpiResidual || EPI == kEpiResidualNorm) {
      const int64_t t128 = static_cast<int64_t>(num_m) * (L.n / 128);
      const int64_t rounds2 = 2 * ((pair_tiles + H->gemm2_pairs - 1) / H->gemm2_pairs);
      const int64_t rounds1 = (t128 + H->num_sms - 1) / H->num_sms;
      if (2 * rounds1 <= rounds2) {
        const int grid1 = static_cast<int>(std::min<int64_t>(t128, H->num_sms));
        stall_one_cta();
        launch(H, kind, flops, [&] {
          launch_k(H, gemm_tcgen05_kernel<128, EPI, T>, grid1, GemmConfig<128>::THREADS,
                   GemmConfig<128>::SMEM_BYTES, a, L.map_half, c, d, shape, ep, H->d_err);
        });
        return;
      }
    }
    // One CTA per 128 x 256 tile does the same per-SM MMA work per round as a
    // CTA of a pair tile, over half the rows, but runs a tile ~10 % slower
    // (it loads all of W's tile instead of half).  Where that still takes
    // fewer rounds (a last pair row mostly padding, or pair tiles a fraction
    // of a round past a whole number: one decision's ~800 tokens, the last
    // layer's slot rows) the one-CTA kernel runs it.  Same bits either way.
    const int64_t rounds_pair = (pair_tiles + H->gemm2_pairs - 1) / H->gemm2_pairs;
    const int64_t rounds_one = (static_cast<int64_t>(num_m) * (L.n / 256) + H->num_sms - 1) / H->num_sms;
    if (10 * rounds_pair < 11 * rounds_one) {
      if (H->opt.raster_group <= 0) shape.group_m = Gemm2Config::GROUP_M;
      const int grid = 2 * std::min(pair_tiles, H->gemm2_pairs);
      launch(H, kind, flops, [&] {
        launch_k(H, gemm2_tcgen05_kernel<EPI, T>, grid, Gemm2Config::THREADS, Gemm2Config::SMEM_BYTES, a,
                 L.map_half, c, d, shape, ep, H->d_err);
      });
      return;
    }
  }
  stall_one_cta();
  launch(H, kind, flops, [&] {
    if (L.bn == 256) {
      launch_k(H, gemm_tcgen05_kernel<256, EPI, T>, grid, GemmConfig<256>::THREADS, GemmConfig<256>::SMEM_BYTES, a,
               L.map, c, d, shape, ep, H->d_err);
    } else {
      if constexpr (EPI == kEpiGated) fail(VD_ESPEC, "gated GEMM needs 256-wide tiles");
      else
        launch_k(H, gemm_tcgen05_kernel<128, EPI, T>, grid, GemmConfig<128>::THREADS, GemmConfig<128>::SMEM_BYTES, a,
                 L.map, c, d, shape, ep, H->d_err);
    }
  });
}

static EpiParams epi(const float* bias = nullptr, int act = kActNone) {
  EpiParams p{};
  p.bias = bias;
  p.act = act;
  return p;
}

static EpiParams epi_params_for(const float* bias, int act) { return epi(bias, act); }

// The tcgen05 kernels cover causal head_dim 128 and 256 with 128-row query
// tiles (gated head_dim 128 only on the one-head kernel); the warp-level kernel
// takes the rest with 64-row tiles.
static bool use_tc_attention(const vd_handle* H, int hd, bool causal, bool gated = false) {
  return H->opt.tc_attention && causal && (hd == 256 || (hd == 128 && (!gated || H->opt.tc_head)));
}

static int attn_tile_rows(const vd_handle* H, int hd, bool causal, bool gated = false) {
  return use_tc_attention(H, hd, causal, gated) ? 128 : 64;
}

// CTAs of the one-head tcgen05 attention for `items` work items: as many as
// run at once (persistent, each looping over items), or one per item.
static int attn_head_grid(const vd_handle* H, int items, int ctas_per_sm) {
  return H->opt.attn_persistent ? std::max(1, std::min(items, ctas_per_sm * H->num_sms)) : std::max(1, items);
}

template <int HD, class T, bool CAUSAL, int SPR>
static void launch_attn_head(vd_handle* H, const AttnTcHeadParams& tp, int items) {
  using C = AttnTcHeadConfig<HD, SPR>;
  launch_k(H, attention_tc_head_kernel<HD, T, CAUSAL, SPR>, attn_head_grid(H, items, C::MIN_CTAS), C::THREADS,
           C::SMEM_BYTES, H->map_qkv64, tp);
}

// gate_col0 >= 0: gated attention (the output is multiplied by the sigmoid of
// the gate columns of qkv), served by the warp-level kernel.
template <class T>
static void attention(vd_handle* H, double flops, int n_tiles, int heads, int hd, bool causal, int ld_qkv, int q0,
                      int k0, int v0, int group, int ld_out, int gate_col0 = -1, const int* opt_id = nullptr,
                      const int* opt_pos = nullptr, int window = 0) {
  AttnParams p{};
  p.gate_col0 = gate_col0;
  p.opt_id = opt_id;
  p.opt_pos = opt_pos;
  p.window = window;
  p.qkv = H->qkv;
  p.ld_qkv = ld_qkv;
  p.q_col0 = q0;
  p.k_col0 = k0;
  p.v_col0 = v0;
  p.out = H->attn;
  p.ld_out = ld_out;
  p.tiles = H->tiles;
  p.group = group;
  p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)) * 1.4426950408889634);
  dim3 grid(n_tiles, heads);
  if (!((hd == 64 && !causal) || (hd == 128 && causal) || (hd == 256 && causal)))
    fail(VD_ESPEC, "no attention kernel for this head size / mask");
  if (hd == 64 && !causal && opt_id == nullptr && window == 0 && gate_col0 < 0 && H->opt.tc_attention) {
    // Marker-head encoders: bidirectional head_dim 64 on the tensor cores
    // (128-row query tiles, planned by encoder_forward).  The option-masked
    // ModernBERT attention stays on the warp-level kernel.
    AttnTcHeadParams tp;
    tp.out = H->attn;
    tp.ld_out = ld_out;
    tp.qkv = H->qkv;
    tp.ld_qkv = ld_qkv;
    tp.q_col0 = q0;
    tp.k_col0 = k0;
    tp.v_col0 = v0;
    tp.gate_col0 = -1;
    tp.tiles = H->tiles;
    tp.n_tiles = n_tiles;
    tp.heads = heads;
    tp.group = group;
    tp.scale_log2 = p.scale_log2;
    tp.err = H->d_err;
    launch(H, VD_K_ATTN, flops, [&] {
      if (H->opt.attn_spr == 2) launch_attn_head<64, T, false, 2>(H, tp, n_tiles * heads);
      else launch_attn_head<64, T, false, 1>(H, tp, n_tiles * heads);
    });
    return;
  }
  if ((hd == 256 || H->opt.tc_head) && use_tc_attention(H, hd, causal, gate_col0 >= 0)) {
    AttnTcHeadParams tp;
    tp.out = H->attn;
    tp.ld_out = ld_out;
    tp.qkv = H->qkv;
    tp.ld_qkv = ld_qkv;
    tp.q_col0 = q0;
    tp.k_col0 = k0;
    tp.v_col0 = v0;
    tp.gate_col0 = gate_col0;
    tp.tiles = H->tiles;
    tp.n_tiles = n_tiles;
    tp.heads = heads;
    tp.group = group;
    tp.scale_log2 = p.scale_log2;
    tp.err = H->d_err;
    launch(H, VD_K_ATTN, flops, [&] {
      const int items = n_tiles * heads;
      if (hd == 256) {
        if (H->opt.attn_spr == 2) launch_attn_head<256, T, true, 2>(H, tp, items);
        else launch_attn_head<256, T, true, 1>(H, tp, items);
      } else {
        if (H->opt.attn_spr == 2) launch_attn_head<128, T, true, 2>(H, tp, items);
        else launch_attn_head<128, T, true, 1>(H, tp, items);
      }
    });
    return;
  }
  if (use_tc_attention(H, hd, causal, gate_col0 >= 0)) {
    AttnTcParams tp;
    tp.out = H->attn;
    tp.ld_out = ld_out;
    tp.q_col0 = q0;
    tp.k_col0 = k0;
    tp.v_col0 = v0;
    tp.tiles = H->tiles;
    tp.group = group;
    tp.pairs_per_kv = (group + 1) / 2;
    tp.scale_log2 = p.scale_log2;
    tp.err = H->d_err;
    const dim3 tgrid(n_tiles, (heads / group) * tp.pairs_per_kv);
    launch(H, VD_K_ATTN, flops, [&] {
      attention_tc_kernel<T><<<tgrid, AttnTcConfig::THREADS, AttnTcConfig::SMEM_BYTES, H->stream>>>(H->map_qkv, tp);
    });
    return;
  }
  launch(H, VD_K_ATTN, flops, [&] {
    if (hd == 64)
      attention_varlen_kernel<64, false, T><<<grid, 128, AttnConfig<64>::SMEM_BYTES, H->stream>>>(p);
    else if (hd == 128)
      attention_varlen_kernel<128, true, T><<<grid, 128, AttnConfig<128>::SMEM_BYTES, H->stream>>>(p);
    else
      attention_varlen_kernel<256, true, T><<<grid, 128, AttnConfig<256>::SMEM_BYTES, H->stream>>>(p);
  });
}

// ---------------------------------------------------------------------------
// Forward of one chunk of rows (device pointers already offset to the chunk).
// ---------------------------------------------------------------------------
struct Chunk {
  int nb = 0;
  int64_t l = 0, k = 0;
  const int64_t* ids = nullptr;      // device [nb*l]
  const int64_t* mpos = nullptr;     // device [nb*k]
  const uint8_t* mmask = nullptr;    // device [nb*k]
  const int64_t* nopts = nullptr;    // device [nb] or null
  const int64_t* qtype = nullptr;    // device [nb] or null
  const int64_t* real_len = nullptr; // host [nb]
  // host copies for the shared-prefix plan (null: rows run whole)
  const int64_t* ids_h = nullptr;    // host [nb*l]
  const int64_t* mpos_h = nullptr;   // host [nb*k]
  const int64_t* prefix_len = nullptr;  // host [nb] or null
  float* out = nullptr;              // device [nb*width]
  int64_t width = 0;
};

struct ChunkPlan {
  int ntok = 0;       // packed tokens
  int max_len = 0;    // longest packed sequence
  int n_seg = 0, n_tiles = 0;
  double pairs = 0;   // attention (query, key) pairs per head
  int fork_groups = 0, fork_rows = 0;
  int64_t shared_tokens = 0;  // prefix tokens not recomputed
};

// Shared-prefix groups of a chunk, the grouping of `_text_fork_forward`
// (executor/torch_exec.py:1935-1977): a row whose slot is its last token joins
// the group keyed by its declared prefix_len (>= 32 and < real_len) and those
// prefix tokens; otherwise a row longer than 32 tokens joins the group keyed by
// its first 32 tokens, whose prefix is then its members' longest common prefix.
// A group runs its prefix once; groups of one row, and groups whose prefix is
// under 32 tokens or leaves a member no suffix, run their rows whole (the
// result is the same, computing it whole is cheaper).
struct ForkGroup {
  int n = 0;                // prefix tokens
  std::vector<int> rows;
};

static constexpr int kForkFloor = 32;  // TEXT_FORK_MIN_PREFIX (GRAPH_PREFIX_STEP)

static std::vector<ForkGroup> plan_fork(const Chunk& c) {
  std::vector<ForkGroup> out;
  if (!c.ids_h || !c.mpos_h || c.nb < 2) return out;
  auto row_ids = [&](int i) { return c.ids_h + static_cast<int64_t>(i) * c.l; };
  auto hash = [&](int i, int n) {
    uint64_t h = 0xCBF29CE484222325ull;
    const int64_t* r = row_ids(i);
    for (int j = 0; j < n; ++j) {
      h ^= static_cast<uint64_t>(r[j]);
      h *= 0x100000001B3ull;
    }
    return h;
  };
  // key: (declared prefix length or 0 for the 32-token key, hash) -> groups whose keys compare equal
  std::map<std::pair<int, uint64_t>, std::vector<ForkGroup>> buckets;
  std::vector<std::pair<int, uint64_t>> order;
  for (int i = 0; i < c.nb; ++i) {
    const int len = static_cast<int>(c.real_len[i]);
    if (c.mpos_h[static_cast<int64_t>(i) * c.k] != len - 1) continue;
    const int declared = c.prefix_len ? static_cast<int>(c.prefix_len[i]) : 0;
    int key_len;
    if (declared >= kForkFloor && declared < len) key_len = declared;
    else if (len > kForkFloor) key_len = 0;
    else continue;
    const int cmp = key_len ? key_len : kForkFloor;
    const auto key = std::make_pair(key_len, hash(i, cmp));
    auto& groups = buckets[key];
    if (groups.empty()) order.push_back(key);
    ForkGroup* g = nullptr;
    for (ForkGroup& cand : groups)
      if (std::equal(row_ids(i), row_ids(i) + cmp, row_ids(cand.rows[0]))) g = &cand;
    if (!g) {
      groups.emplace_back();
      g = &groups.back();
      g->n = key_len;
    }
    g->rows.push_back(i);
  }
  for (const auto& key : order)
    for (ForkGroup& g : buckets[key]) {
      if (g.rows.size() < 2) continue;
      int min_len = INT32_MAX;
      for (int i : g.rows) min_len = std::min(min_len, static_cast<int>(c.real_len[i]));
      if (g.n == 0) {  // longest common prefix of the members
        const int64_t* r0 = row_ids(g.rows[0]);
        int n = kForkFloor;
        while (n < min_len) {
          bool same = true;
          for (size_t m = 1; m < g.rows.size() && same; ++m) same = row_ids(g.rows[m])[n] == r0[n];
          if (!same) break;
          ++n;
        }
        g.n = n;
      }
      if (g.n < kForkFloor || g.n >= min_len) continue;  // every member keeps a suffix
      out.push_back(std::move(g));
    }
  return out;
}

// Host plan of a chunk: the packed sequences (whole rows, or shared prefixes
// followed by their members' suffixes), each decision's slot location, and the
// attention tile table, staged through pinned memory.
static ChunkPlan plan_chunk(vd_handle* H, const Chunk& c, bool causal, int tile_rows) {
  ChunkPlan P;
  H->slot = (H->slot + 1) % vd_handle::kSlots;
  char* buf = H->pinned[H->slot];
  cuda_check(cudaEventSynchronize(H->slot_ev[H->slot]), "staging slot");
  auto align16 = [](size_t x) { return (x + 15) & ~size_t(15); };
  size_t off = 0;
  int* cu = reinterpret_cast<int*>(buf + off);
  off = align16(off + sizeof(int) * (c.nb + 1));
  PackSeg* segs = reinterpret_cast<PackSeg*>(buf + off);
  off = align16(off + sizeof(PackSeg) * 2 * c.nb);
  RowMap* rows = reinterpret_cast<RowMap*>(buf + off);
  off = align16(off + sizeof(RowMap) * c.nb);
  AttnTile* tiles = reinterpret_cast<AttnTile*>(buf + off);

  std::vector<ForkGroup> groups;
  // Gated-delta-net layers carry a recurrent state along the sequence; a
  // shared prefix would have to hand its state to every suffix, which this
  // executor does not do, so hybrid stacks run whole rows.
  if (causal && H->opt.fork && !H->spec.any_linear()) groups = plan_fork(c);
  std::vector<int> group_of(c.nb, -1);
  for (size_t g = 0; g < groups.size(); ++g)
    for (int i : groups[g].rows) group_of[i] = static_cast<int>(g);
  std::vector<char> emitted(groups.size(), 0);
  int n = 0;
  auto add_seq = [&](int src_row, int col0, int len, int pre_start, int pre_len) {
    const int start = P.ntok;
    segs[P.n_seg++] = PackSeg{start, len, col0, src_row};
    P.ntok += len;
    P.max_len = std::max(P.max_len, len);
    for (int q = 0; q < len; q += tile_rows) tiles[n++] = AttnTile{start, len, q, pre_start, pre_len, {0, 0, 0}};
    P.pairs += causal ? 0.5 * len * (len + 1.0) + static_cast<double>(len) * pre_len : static_cast<double>(len) * len;
    return start;
  };
  for (int i = 0; i < c.nb; ++i) {
    const int len = static_cast<int>(c.real_len[i]);
    const int g = group_of[i];
    if (g < 0) {
      const int start = add_seq(i, 0, len, 0, 0);
      rows[i] = RowMap{start, 0, len, 0};
      cu[i] = start;
      continue;
    }
    if (emitted[g]) continue;
    emitted[g] = 1;
    const ForkGroup& fg = groups[g];
    const int pre = add_seq(fg.rows[0], 0, fg.n, 0, 0);
    for (int m : fg.rows) {
      const int mlen = static_cast<int>(c.real_len[m]);
      const int start = add_seq(m, fg.n, mlen - fg.n, pre, fg.n);
      rows[m] = RowMap{start - fg.n, fg.n, mlen, 0};
      cu[m] = start - fg.n;
    }
    ++P.fork_groups;
    P.fork_rows += static_cast<int>(fg.rows.size());
    P.shared_tokens += static_cast<int64_t>(fg.n) * (fg.rows.size() - 1);
  }
  cu[c.nb] = P.ntok;
  P.n_tiles = n;
  // Gated-delta-net recurrences run one CTA per (sequence, head), as long as
  // the sequence: longest first, so the last wave is not one long sequence.
  // (Each entry carries its own start and source row; no kernel depends on
  // the order.)
  if (H->spec.any_linear())
    std::stable_sort(segs, segs + P.n_seg, [](const PackSeg& a, const PackSeg& b) { return a.len > b.len; });
  // Longest work first: a causal tile costs ~ its last query row's keys.
  std::stable_sort(tiles, tiles + n, [causal, tile_rows](const AttnTile& a, const AttnTile& b) {
    const int wa = (causal ? std::min(a.seq_len, a.q_start + tile_rows) : a.seq_len) + a.pre_len;
    const int wb = (causal ? std::min(b.seq_len, b.q_start + tile_rows) : b.seq_len) + b.pre_len;
    return wa > wb;
  });
  const size_t seg_off = reinterpret_cast<char*>(segs) - buf, row_off = reinterpret_cast<char*>(rows) - buf,
               tile_off = reinterpret_cast<char*>(tiles) - buf;
  cuda_check(cudaMemcpyAsync(H->cu, cu, sizeof(int) * (c.nb + 1), cudaMemcpyHostToDevice, H->stream), "upload cu");
  cuda_check(cudaMemcpyAsync(H->segs, buf + seg_off, sizeof(PackSeg) * P.n_seg, cudaMemcpyHostToDevice, H->stream),
             "upload segments");
  cuda_check(cudaMemcpyAsync(H->rowmap, buf + row_off, sizeof(RowMap) * c.nb, cudaMemcpyHostToDevice, H->stream),
             "upload row map");
  cuda_check(cudaMemcpyAsync(H->tiles, buf + tile_off, sizeof(AttnTile) * n, cudaMemcpyHostToDevice, H->stream),
             "upload tiles");
  cuda_check(cudaEventRecord(H->slot_ev[H->slot], H->stream), "staging event");
  H->stats.fork_groups += P.fork_groups;
  H->stats.fork_rows += P.fork_rows;
  H->stats.shared_tokens += P.shared_tokens;
  return P;
}

static void pack(vd_handle* H, const Chunk& c, const ChunkPlan& P, int pos_offset) {
  dim3 grid(std::max(1, std::min((P.max_len + 255) / 256, 64)), P.n_seg);
  launch(H, VD_K_OTHER, 0.0, [&] {
    pack_segments_kernel<<<grid, 256, 0, H->stream>>>(c.ids, c.l, H->segs, P.n_seg, H->spec.vocab, pos_offset,
                                                      H->tokens, H->positions, H->seq_id, H->d_err);
  });
}

// Full attention of one decoder layer: fused QKV GEMM (bias, q/k RMSNorm and
// RoPE in the epilogue; a hybrid's output-gate columns pass through), then
// varlen causal attention (gated in a hybrid) into H->attn.
template <class T>
static void full_attention_mixer(vd_handle* H, const DecLayer& L, int ntok, int n_tiles, double attn_flops,
                                 const EpiParams& norm_in) {
  const ModelSpec& s = H->spec;
  const int hd = s.head_dim, nq = s.heads, nkv = s.kv_heads, qc = nq * hd, kc = nkv * hd;
  EpiParams q = norm_in;
  q.bias = L.qkv.b;
  q.q_norm = L.q_norm;
  q.k_norm = L.k_norm;
  q.q_cols = qc;
  q.k_cols = kc;
  q.head_dim = hd;
  q.plus_one = s.norm_plus_one ? 1 : 0;
  q.eps = static_cast<float>(s.rms_eps);
  q.positions = H->positions;
  q.rope = H->rope;
  q.rot_dim = s.hybrid() ? s.rot_dim() : 0;
  gemm<kEpiQKRope, T>(H, VD_K_QKV, H->map_xn, L.qkv, ntok, q, H->out_qkv);
  attention<T>(H, attn_flops, n_tiles, nq, hd, true, H->ld_qkv, 0, qc, qc + kc, nq / nkv, qc,
               s.hybrid() ? qc + 2 * kc : -1);
}

// Gated delta net of one hybrid layer: fused in_proj GEMM into H->proj, conv +
// l2 norms + gates into H->qkv / gdn_g / gdn_beta, then the recurrence with the
// gated norm into H->attn (one CTA per sequence and value head).
template <class T>
static void gdn_mixer(vd_handle* H, const DecLayer& L, int ntok, const ChunkPlan& P, const EpiParams& norm_in) {
  const ModelSpec& s = H->spec;
  gemm<kEpiStore, T>(H, VD_K_QKV, H->map_xn, L.qkv, ntok, norm_in, H->out_proj);
  GdnParams g{};
  g.proj = H->proj;
  g.ld_proj = s.gdn_proj();
  g.conv_w = L.conv_w;
  g.A_log = L.A_log;
  g.dt_bias = L.dt_bias;
  g.norm_w = L.gdn_norm;
  g.positions = H->positions;
  g.ntok = ntok;
  g.kd = s.gdn_kd();
  g.vd = s.gdn_vd();
  g.lk = s.lin_k_heads;
  g.lv = s.lin_v_heads;
  g.col_z = s.gdn_conv();
  g.col_a = s.gdn_conv() + s.gdn_vd();
  g.col_b = g.col_a + s.lin_v_heads;
  g.qkv = H->qkv;
  g.ld_qkv = H->ld_qkv;
  g.g = H->gdn_g;
  g.beta = H->gdn_beta;
  g.out = H->attn;
  g.ld_out = s.heads * s.head_dim;
  g.q_scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(s.lin_k_dim)));
  g.eps = static_cast<float>(s.rms_eps);
  g.segs = reinterpret_cast<const int4*>(H->segs);
  const dim3 conv_grid((ntok + GDN_CONV_TOKENS - 1) / GDN_CONV_TOKENS, (2 * g.lk + g.lv + 7) / 8 + 1);
  launch(H, VD_K_GDN, 0.0, [&] { gdn_conv_prep_kernel<T, 4><<<conv_grid, 256, 0, H->stream>>>(g); });
  if (H->opt.gdn_chunk) {
    // per token and value head: K K^T and Q K^T rows (2 x 64 x 128), K S0 and
    // Q S0 (2 x 128 x 128), T R and P D (2 x 64 x 128), the state update (128 x 128)
    const double flops = 2.0 * ntok * s.lin_v_heads * (4.0 * 64 * 128 + 3.0 * 128 * 128);
    launch(H, VD_K_GDN, flops, [&] {
      gdn_chunk_kernel<T><<<dim3(s.lin_v_heads, P.n_seg), 256, GdnChunkConfig::SMEM_BYTES, H->stream>>>(g);
    });
    return;
  }
  // per token and value head: decay + two rank-1 passes over the 128 x 128 state
  const double flops = 4.0 * ntok * s.lin_v_heads * s.lin_k_dim * s.lin_v_dim;
  launch(H, VD_K_GDN, flops, [&] {
    gdn_scan_kernel<T><<<dim3(P.n_seg, s.lin_v_heads), 256, 0, H->stream>>>(g);
  });
}

template <class T>
static double decoder_forward(vd_handle* H, const Chunk& c) {
  const ModelSpec& s = H->spec;
  const int d = s.hidden, hd = s.head_dim, nq = s.heads;
  const ChunkPlan P = plan_chunk(H, c, true, attn_tile_rows(H, hd, true, s.hybrid()));
  const int ntok = P.ntok, n_tiles = P.n_tiles;
  pack(H, c, P, 0);
  const float escale = s.embed_scale ? static_cast<float>(std::pow(static_cast<double>(d), 0.5)) : 1.0f;
  const int qc = nq * hd;
  const float eps = static_cast<float>(s.rms_eps);
  const int pone = s.norm_plus_one ? 1 : 0;
  const double attn_flops = 4.0 * hd * nq * P.pairs;
  // Fused RMSNorm (default): every residual add that feeds a norm (embedding,
  // O / out_proj, down) also writes the 16-bit copy of the new rows and their
  // block sums of squares; the projection reading them (QKV / in_proj, gate/up)
  // applies the row factor.  ss_a feeds the attention input, ss_b the MLP input.
  const bool fused = H->opt.fuse_norm;
  const float pre = H->opt.f16 ? kNormPrescale16 : 1.0f;
  const int slots = d / kNormBlock;
  const float gadd = s.norm_plus_one ? 1.0f : 0.0f;
  auto produce = [&](float* ss, const float* next_gain) {
    EpiParams p = epi();
    p.prescale = pre;
    p.ss_out = ss;
    p.ss_slots = slots;
    p.norm_gain = next_gain;
    p.norm_add = gadd;
    return p;
  };
  auto consume = [&](EpiParams p, const float* ss) {
    if (!fused) return p;
    p.ss_in = ss;
    p.ss_slots = slots;
    p.ss_inv_n = 1.0f / static_cast<float>(d);
    p.ss_eps = eps;
    p.ss_post = 1.0f / pre;
    return p;
  };
  auto separate_norm = [&](const float* x, const float* g, void* out, int rows) {
    launch(H, VD_K_NORM, 0.0, [&] {
      rmsnorm_kernel<256, T><<<rows, 256, 0, H->stream>>>(x, d, g, pone, eps, static_cast<T*>(out), rows);
    });
  };
  launch(H, VD_K_OTHER, 0.0, [&] {
    if (fused)
      embed_norm_kernel<T><<<ntok, 128, 0, H->stream>>>(H->tokens, ntok, H->embed, d, escale, H->dec[0].in_norm,
                                                        gadd, pre, H->h, static_cast<T*>(H->xn), H->ss_a);
    else
      embed_kernel<<<ntok, 128, 0, H->stream>>>(H->tokens, ntok, H->embed, d, escale, H->h);
  });
  for (int i = 0; i < s.layers; ++i) {
    const DecLayer& L = H->dec[i];
    if (!fused) separate_norm(H->h, L.in_norm, H->xn, ntok);
    if (L.linear) {
      gdn_mixer<T>(H, L, ntok, P, consume(epi(), H->ss_a));
    } else {
      full_attention_mixer<T>(H, L, ntok, n_tiles, attn_flops, consume(epi(), H->ss_a));
    }
    const bool last = i + 1 == s.layers;
    if (last && H->opt.prune_last_layer) {
      // Only the slot rows feed the readout: gather them (attention output and
      // residual) and finish the layer on nb rows instead of ntok.
      launch(H, VD_K_OTHER, 0.0, [&] {
        gather_slot_rows_kernel<T><<<c.nb, 256, 0, H->stream>>>(H->rowmap, c.mpos, static_cast<int>(c.k),
                                                                 static_cast<const T*>(H->attn), qc, H->h, d,
                                                                 static_cast<T*>(H->attn_s), H->h_s, H->d_err);
      });
      if (fused) {
        gemm<kEpiResidualNorm, T>(H, VD_K_O, H->map_attn_s, L.o, c.nb, produce(H->ss_s, L.post_norm), H->out_h_s,
                                  &H->out_xn_s);
      } else {
        gemm<kEpiResidual, T>(H, VD_K_O, H->map_attn_s, L.o, c.nb, epi(), H->out_h_s);
        separate_norm(H->h_s, L.post_norm, H->xn_s, c.nb);
      }
      gemm<kEpiGated, T>(H, VD_K_GATEUP, H->map_xn_s, L.gu, c.nb, consume(epi(nullptr, s.act), H->ss_s),
                         H->out_act_s);
      gemm<kEpiResidual, T>(H, VD_K_DOWN, H->map_act_s, L.down, c.nb, epi(), H->out_h_s);
      continue;
    }
    if (fused) {
      gemm<kEpiResidualNorm, T>(H, VD_K_O, H->map_attn, L.o, ntok, produce(H->ss_b, L.post_norm), H->out_h,
                                &H->out_xn);
    } else {
      gemm<kEpiResidual, T>(H, VD_K_O, H->map_attn, L.o, ntok, epi(), H->out_h);
      separate_norm(H->h, L.post_norm, H->xn, ntok);
    }
    gemm<kEpiGated, T>(H, VD_K_GATEUP, H->map_xn, L.gu, ntok, consume(epi(nullptr, s.act), H->ss_b), H->out_act);
    // The last layer's down projection feeds only the readout's final norm.
    if (fused && !last)
      gemm<kEpiResidualNorm, T>(H, VD_K_DOWN, H->map_act, L.down, ntok, produce(H->ss_a, H->dec[i + 1].in_norm),
                                H->out_h, &H->out_xn);
    else
      gemm<kEpiResidual, T>(H, VD_K_DOWN, H->map_act, L.down, ntok, epi(), H->out_h);
  }
  const bool compact = H->opt.prune_last_layer;
  const size_t smem = sizeof(float) * (d + H->n_labels);
  launch(H, VD_K_OTHER, 0.0, [&] {
    readout_kernel<256><<<c.nb, 256, smem, H->stream>>>(compact ? H->h_s : H->h, d, H->rowmap, c.mpos,
                                                        static_cast<int>(c.k), c.nopts, H->final_norm, pone, eps,
                                                        H->head_rows, H->n_labels, c.out, static_cast<int>(c.width),
                                                        H->opt.logprobs ? 1 : 0, compact ? 1 : 0, H->d_err);
  });
  return ntok;
}

// LayerNorm of the ntok fp32 rows of h (16-bit copy to xn, fp32 in place when
// `inplace`): one warp per row for the widths that fit its registers.
template <class T>
static void layernorm_rows(vd_handle* H, int d, const float* w, const float* b, float eps, int inplace, int ntok) {
  launch(H, VD_K_NORM, 0.0, [&] {
    T* xn = static_cast<T*>(H->xn);
    const int blocks = (ntok + 7) / 8;
    switch (d % 128 == 0 ? d / 128 : 0) {
      case 4: layernorm_warp_kernel<4, T><<<blocks, 256, 0, H->stream>>>(H->h, d, w, b, eps, inplace, xn, ntok); break;
      case 6: layernorm_warp_kernel<6, T><<<blocks, 256, 0, H->stream>>>(H->h, d, w, b, eps, inplace, xn, ntok); break;
      case 8: layernorm_warp_kernel<8, T><<<blocks, 256, 0, H->stream>>>(H->h, d, w, b, eps, inplace, xn, ntok); break;
      default: layernorm_kernel<256, T><<<ntok, 256, 0, H->stream>>>(H->h, d, w, b, eps, inplace, xn, ntok);
    }
  });
}

template <class T>
static void enc_layer(vd_handle* H, const EncLayer& L, int ntok, int n_tiles, double attn_flops) {
  const int d = H->spec.hidden;
  const int nh = d / 64;
  auto ln = [&](const float* w, const float* b, int inplace) { layernorm_rows<T>(H, d, w, b, L.eps, inplace, ntok); };
  if (L.pre_norm) ln(L.ln1_w, L.ln1_b, 0);
  gemm<kEpiStore, T>(H, VD_K_QKV, H->map_xn, L.qkv, ntok, epi(L.qkv.b), H->out_qkv);
  attention<T>(H, attn_flops, n_tiles, nh, 64, false, 3 * d, 0, d, 2 * d, 1, d);
  gemm<kEpiResidual, T>(H, VD_K_O, H->map_attn, L.o, ntok, epi(L.o.b), H->out_h);
  if (L.pre_norm) ln(L.ln2_w, L.ln2_b, 0);
  else ln(L.ln1_w, L.ln1_b, 1);
  const CUtensorMap& amap = (L.f1.n == H->spec.ffn) ? H->map_act : H->map_act2;
  const CUtensorMap& omap = (L.f1.n == H->spec.ffn) ? H->out_act : H->out_act2;
  gemm<kEpiStore, T>(H, VD_K_GATEUP, H->map_xn, L.f1, ntok, epi(L.f1.b, L.act), omap);
  gemm<kEpiResidual, T>(H, VD_K_DOWN, amap, L.f2, ntok, epi(L.f2.b), H->out_h);
  if (!L.pre_norm) ln(L.ln2_w, L.ln2_b, 1);
}

// The independent-options forward: ModernBERT over packed rows with option
// masks and option-invariant positions, final norm, marker gather + scorer.
template <class T>
static double von_forward(vd_handle* H, const Chunk& c) {
  const ModelSpec& s = H->spec;
  const int d = s.hidden, nh = d / 64;
  const ChunkPlan P = plan_chunk(H, c, false, 64);
  const int ntok = P.ntok, n_tiles = P.n_tiles;
  pack(H, c, P, 0);
  launch(H, VD_K_OTHER, 0.0, [&] {
    dim3 grid(std::max(1, std::min((P.max_len + 255) / 256, 64)), P.n_seg);
    von_layout_kernel<<<grid, 256, 0, H->stream>>>(H->segs, P.n_seg, c.mpos, c.mmask, static_cast<int>(c.k),
                                                   H->von_opt, H->von_pos, H->d_err);
  });
  const float eps = static_cast<float>(s.ln_eps);
  auto ln = [&](const float* w, int inplace) { layernorm_rows<T>(H, d, w, H->zero_d, eps, inplace, ntok); };
  launch(H, VD_K_OTHER, 0.0,
         [&] { embed_kernel<<<ntok, 128, 0, H->stream>>>(H->tokens, ntok, H->embed, d, 1.0f, H->h); });
  ln(H->emb_ln_w, 1);  // the residual stream starts from the normalised embedding
  const double attn_flops = 4.0 * d * P.pairs;
  for (const EncLayer& L : H->enc) {
    if (L.ln1_w) ln(L.ln1_w, 0);  // layer 0 has no attention norm: xn already holds h
    EpiParams q = epi();
    q.q_cols = d;
    q.k_cols = d;
    q.head_dim = 64;
    q.eps = eps;
    q.positions = H->von_pos;
    q.rope = L.sliding ? H->rope_local : H->rope;
    gemm<kEpiQKRope, T>(H, VD_K_QKV, H->map_xn, L.qkv, ntok, q, H->out_qkv);
    attention<T>(H, attn_flops, n_tiles, nh, 64, false, 3 * d, 0, d, 2 * d, 1, d, -1, H->von_opt, H->von_pos,
                 L.sliding ? s.sliding_window : 0);
    gemm<kEpiResidual, T>(H, VD_K_O, H->map_attn, L.o, ntok, epi(), H->out_h);
    ln(L.ln2_w, 0);
    gemm<kEpiGated, T>(H, VD_K_GATEUP, H->map_xn, L.f1, ntok, epi(nullptr, L.act), H->out_act);
    gemm<kEpiResidual, T>(H, VD_K_DOWN, H->map_act, L.f2, ntok, epi(), H->out_h);
  }
  ln(H->final_norm, 1);
  const int nm = static_cast<int>(c.nb * c.k);
  if (nm > 0) {
    launch(H, VD_K_OTHER, 0.0, [&] {
      marker_index_kernel<<<(nm + 255) / 256, 256, 0, H->stream>>>(H->cu, c.mpos, c.mmask, c.nb,
                                                                   static_cast<int>(c.k), H->midx, H->d_err);
    });
    launch(H, VD_K_NORM, 0.0, [&] {
      gather_layernorm_kernel<256, T><<<nm, 256, 0, H->stream>>>(H->h, H->midx, nm, d, H->sc_ln_w, H->sc_ln_b,
                                                                 1e-5f, static_cast<T*>(H->mrow));
    });
    gemm<kEpiStore, T>(H, VD_K_OTHER, H->map_mrow, H->sc1, nm, epi(H->sc1.b, kActGeluErf), H->out_mhid);
  }
  launch(H, VD_K_OTHER, 0.0, [&] {
    marker_score_kernel<T><<<c.nb, 256, 0, H->stream>>>(static_cast<const T*>(H->mhid), d, H->sc_w3, H->sc_b3,
                                                        c.mmask, c.nb, static_cast<int>(c.k), c.out,
                                                        static_cast<int>(c.width), H->d_err);
  });
  return ntok;
}

template <class T>
static double encoder_forward(vd_handle* H, const Chunk& c) {
  const ModelSpec& s = H->spec;
  if (s.von()) return von_forward<T>(H, c);
  const int d = s.hidden;
  // Query tiles of 128 rows for the tcgen05 attention (head_dim 64, see
  // attention()), 64 for the warp-level kernel.
  const ChunkPlan P = plan_chunk(H, c, false, H->opt.tc_attention ? 128 : 64);
  const int ntok = P.ntok, n_tiles = P.n_tiles;
  const int pos_offset = s.style == "xlmr" ? s.pad_id + 1 : 0;
  if (P.max_len + pos_offset > s.max_pos) fail(VD_EINVAL, "a row is longer than the model's position table");
  pack(H, c, P, pos_offset);
  const int vpt = d % 128 == 0 ? d / 128 : 0;  // warp-per-token kernels for d = 512, 768, 1024
  launch(H, VD_K_OTHER, 0.0, [&] {
    const float eps = static_cast<float>(s.ln_eps);
    T* xn = static_cast<T*>(H->xn);
    const int blocks = (ntok + 7) / 8;
    switch (vpt) {
      case 4:
        embed_ln_warp_kernel<4, T><<<blocks, 256, 0, H->stream>>>(H->tokens, H->positions, ntok, H->embed,
                                                                  H->pos_emb, H->type_emb0, d, H->emb_ln_w,
                                                                  H->emb_ln_b, eps, H->h, xn);
        break;
      case 6:
        embed_ln_warp_kernel<6, T><<<blocks, 256, 0, H->stream>>>(H->tokens, H->positions, ntok, H->embed,
                                                                  H->pos_emb, H->type_emb0, d, H->emb_ln_w,
                                                                  H->emb_ln_b, eps, H->h, xn);
        break;
      case 8:
        embed_ln_warp_kernel<8, T><<<blocks, 256, 0, H->stream>>>(H->tokens, H->positions, ntok, H->embed,
                                                                  H->pos_emb, H->type_emb0, d, H->emb_ln_w,
                                                                  H->emb_ln_b, eps, H->h, xn);
        break;
      default:
        embed_ln_kernel<256, T><<<ntok, 256, 0, H->stream>>>(H->tokens, H->positions, ntok, H->embed, H->pos_emb,
                                                             H->type_emb0, d, H->emb_ln_w, H->emb_ln_b, eps, H->h,
                                                             xn);
    }
  });
  const double attn_flops = 4.0 * d * P.pairs;
  for (const EncLayer& L : H->enc) enc_layer<T>(H, L, ntok, n_tiles, attn_flops);
  launch(H, VD_K_OTHER, 0.0, [&] {
    const int blocks = (ntok + 7) / 8;
    if (vpt == 4)
      add_type_warp_kernel<4><<<blocks, 256, 0, H->stream>>>(H->h, ntok, d, H->seq_id, c.qtype, H->qtype_emb, 3,
                                                             H->d_err);
    else if (vpt == 6)
      add_type_warp_kernel<6><<<blocks, 256, 0, H->stream>>>(H->h, ntok, d, H->seq_id, c.qtype, H->qtype_emb, 3,
                                                             H->d_err);
    else if (vpt == 8)
      add_type_warp_kernel<8><<<blocks, 256, 0, H->stream>>>(H->h, ntok, d, H->seq_id, c.qtype, H->qtype_emb, 3,
                                                             H->d_err);
    else
      add_type_kernel<<<ntok, 256, 0, H->stream>>>(H->h, ntok, d, H->seq_id, c.qtype, H->qtype_emb, 3, H->d_err);
  });
  for (const EncLayer& L : H->head) enc_layer<T>(H, L, ntok, n_tiles, attn_flops);
  const int nm = static_cast<int>(c.nb * c.k);
  if (nm > 0) {
    launch(H, VD_K_OTHER, 0.0, [&] {
      marker_index_kernel<<<(nm + 255) / 256, 256, 0, H->stream>>>(H->cu, c.mpos, c.mmask, c.nb,
                                                                   static_cast<int>(c.k), H->midx, H->d_err);
    });
    launch(H, VD_K_NORM, 0.0, [&] {
      gather_layernorm_kernel<256, T><<<nm, 256, 0, H->stream>>>(H->h, H->midx, nm, d, H->sc_ln_w, H->sc_ln_b,
                                                                 1e-5f, static_cast<T*>(H->mrow));
    });
    gemm<kEpiStore, T>(H, VD_K_OTHER, H->map_mrow, H->sc1, nm, epi(H->sc1.b, kActGeluErf), H->out_mhid);
  }
  launch(H, VD_K_OTHER, 0.0, [&] {
    marker_score_kernel<T><<<c.nb, 256, 0, H->stream>>>(static_cast<const T*>(H->mhid), d, H->sc_w3, H->sc_b3,
                                                        c.mmask, c.nb,
                                                     static_cast<int>(c.k), c.out, static_cast<int>(c.width),
                                                     H->d_err);
  });
  return ntok;
}

// ---------------------------------------------------------------------------
// Batch validation and chunking
// ---------------------------------------------------------------------------
static void validate_batch(vd_handle* H, const vd_batch* b, int64_t width) {
  if (!b) fail(VD_EINVAL, "null batch");
  if (b->b < 0 || b->l < 0 || b->k < 0) fail(VD_EINVAL, "negative batch dimensions");
  if (b->b == 0) return;
  if (!b->input_ids || !b->real_len || !b->marker_pos) fail(VD_EINVAL, "missing input_ids / real_len / marker_pos");
  if (b->memory != VD_MEM_HOST && b->memory != VD_MEM_DEVICE) fail(VD_EINVAL, "unknown memory kind");
  const ModelSpec& s = H->spec;
  if (s.decoder()) {
    // TorchEngine::infer (src/torch_engine.rs:452-466)
    if (b->k != 1 || !b->nopts)
      fail(VD_EINVAL, "letter batches need exactly one slot per row (got k=" + std::to_string(b->k) +
                          ", nopts=" + std::string(b->nopts ? std::to_string(b->b) : "0") + ")");
    if (b->memory == VD_MEM_HOST && b->marker_mask)
      for (int64_t i = 0; i < b->b; ++i)
        if (!b->marker_mask[i]) fail(VD_EINVAL, "row " + std::to_string(i) + " has no slot marker");
    if (width < 1) fail(VD_EINVAL, "output width must be positive");
  } else {
    if (!b->marker_mask) fail(VD_EINVAL, "marker batches need marker_mask");
    if (width < b->k) fail(VD_EINVAL, "output width is smaller than k");
    if (b->b * b->k > H->opt.max_markers) fail(VD_EINVAL, "too many markers for this handle (max_markers)");
    if (s.von() && b->memory == VD_MEM_HOST)
      // independent_options_tensors (src/engine.rs:549-555)
      for (int64_t i = 0; i < b->b; ++i) {
        int64_t first = -1;
        for (int64_t j = 0; j < b->k; ++j)
          if (b->marker_mask[i * b->k + j]) {
            first = b->marker_pos[i * b->k + j];
            break;
          }
        if (first < 0 || first >= b->real_len[i])
          fail(VD_EINVAL, "row " + std::to_string(i) + ": no marker positions inside the real ids");
      }
  }
  for (int64_t i = 0; i < b->b; ++i) {
    const int64_t n = b->real_len[i];
    if (n < 1 || n > b->l) fail(VD_EINVAL, "row " + std::to_string(i) + " has real_len outside [1, l]");
    if (n > H->opt.max_seq) fail(VD_EINVAL, "row " + std::to_string(i) + " is longer than max_seq");
    if (n > H->opt.max_tokens) fail(VD_EINVAL, "row " + std::to_string(i) + " is longer than max_tokens");
  }
  if (b->memory == VD_MEM_HOST) {
    if (s.decoder())
      for (int64_t i = 0; i < b->b; ++i) {
        const int64_t slot = b->marker_pos[i];
        if (slot < 0 || slot >= b->real_len[i]) fail(VD_EINVAL, "row " + std::to_string(i) + " slot outside the row");
      }
  }
}

static void run_batch(vd_handle* H, const vd_batch* b, const int64_t* ids, const int64_t* mpos, const uint8_t* mmask,
                      const int64_t* nopts, const int64_t* qtype, float* out, int64_t width) {
  // Shared-prefix planning reads token ids and slots on the host.  A
  // device-memory batch is planned only when it declares prefix lengths: its
  // ids and slots are then copied back first (one synchronisation).
  const int64_t* ids_h = nullptr;
  const int64_t* mpos_h = nullptr;
  std::vector<int64_t> ids_copy, mpos_copy;
  if (H->spec.decoder() && H->opt.fork && b->b > 1) {
    if (b->memory == VD_MEM_HOST) {
      ids_h = b->input_ids;
      mpos_h = b->marker_pos;
    } else if (b->prefix_len) {
      ids_copy.resize(static_cast<size_t>(b->b * b->l));
      mpos_copy.resize(static_cast<size_t>(b->b * b->k));
      cuda_check(cudaMemcpyAsync(ids_copy.data(), b->input_ids, ids_copy.size() * 8, cudaMemcpyDeviceToHost,
                                 H->stream), "copy ids for the prefix plan");
      cuda_check(cudaMemcpyAsync(mpos_copy.data(), b->marker_pos, mpos_copy.size() * 8, cudaMemcpyDeviceToHost,
                                 H->stream), "copy slots for the prefix plan");
      cuda_check(cudaStreamSynchronize(H->stream), "prefix plan copies");
      ids_h = ids_copy.data();
      mpos_h = mpos_copy.data();
    }
  }
  const auto t_enqueue = std::chrono::steady_clock::now();
  H->stats = vd_stats{};
  H->launches = 0;
  H->stall_pending = H->opt.debug_stall > 0;
  cuda_check(cudaEventRecord(H->ev0, H->stream), "event");
  int64_t r0 = 0, chunks = 0, tokens = 0;
  while (r0 < b->b) {
    int64_t r1 = r0, t = 0;
    while (r1 < b->b && r1 - r0 < H->opt.max_rows && t + b->real_len[r1] <= H->opt.max_tokens) t += b->real_len[r1++];
    Chunk c;
    c.nb = static_cast<int>(r1 - r0);
    c.l = b->l;
    c.k = b->k;
    c.ids = ids + r0 * b->l;
    c.mpos = mpos + r0 * b->k;
    c.mmask = mmask ? mmask + r0 * b->k : nullptr;
    c.nopts = nopts ? nopts + r0 : nullptr;
    c.qtype = qtype ? qtype + r0 : nullptr;
    c.real_len = b->real_len + r0;
    if (ids_h) {
      c.ids_h = ids_h + r0 * b->l;
      c.mpos_h = mpos_h + r0 * b->k;
      c.prefix_len = b->prefix_len ? b->prefix_len + r0 : nullptr;
    }
    c.out = out + r0 * width;
    c.width = width;
    double nt = 0;
    if (H->spec.decoder())
      nt = H->opt.f16 ? decoder_forward<__half>(H, c) : decoder_forward<__nv_bfloat16>(H, c);
    else
      nt = H->opt.f16 ? encoder_forward<__half>(H, c) : encoder_forward<__nv_bfloat16>(H, c);
    tokens += static_cast<int64_t>(nt);
    ++chunks;
    r0 = r1;
  }
  cuda_check(cudaGetLastError(), "kernel launch");
  cuda_check(cudaEventRecord(H->ev1, H->stream), "event");
  // Algorithmic work actually launched, from the per-class counts of launch().
  H->stats.gemm_flops = H->stats.kernel_flops[VD_K_QKV] + H->stats.kernel_flops[VD_K_O] +
                        H->stats.kernel_flops[VD_K_GATEUP] + H->stats.kernel_flops[VD_K_DOWN];
  H->stats.attn_flops = H->stats.kernel_flops[VD_K_ATTN];
  H->stats.enqueue_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_enqueue).count();
  H->stats.rows = b->b;
  H->stats.tokens = tokens;
  H->stats.chunks = chunks;
  H->stats.launches = H->launches;
}

static void check_device_error(vd_handle* H) {
  int e = 0;
  cuda_check(cudaMemcpyAsync(&e, H->d_err, sizeof(int), cudaMemcpyDeviceToHost, H->stream), "read error word");
  cuda_check(cudaStreamSynchronize(H->stream), "synchronize");
  float ms = 0;
  if (cudaEventElapsedTime(&ms, H->ev0, H->ev1) == cudaSuccess) H->stats.forward_ms = ms;
  prof_collect(H);
  if (e != 0) {
    cuda_check(cudaMemsetAsync(H->d_err, 0, sizeof(int), H->stream), "clear error word");
    cuda_check(cudaStreamSynchronize(H->stream), "synchronize");
    if (e == kErrTokenRange) fail(VD_EDEVICE, "a token id or qtype is outside the model's range");
    if (e == kErrSlotRange) fail(VD_EDEVICE, "a slot / marker position lies outside its row");
    if (e == kErrNonFinite)
      fail(VD_EDEVICE, std::string("non-finite values (inf / NaN) reached a slot or marker hidden state: an "
                                   "activation overflowed its 16-bit range") +
                           (H->opt.f16 ? "; fp16 activations stop at 65504, reopen the model with "
                                         "\"act_dtype\": \"bf16\" (fp32's exponent range)"
                                       : ""));
    H->healthy = false;
    H->dead_reason = "a kernel pipeline timed out (device error " + std::to_string(e) + ")";
    fail(VD_ECUDA, H->dead_reason);
  }
}

}  // namespace vd

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using namespace vd;

static void put_err(char* err, size_t errlen, const std::string& msg) {
  if (!err || errlen == 0) return;
  const size_t n = std::min(errlen - 1, msg.size());
  std::memcpy(err, msg.data(), n);
  err[n] = '\0';
}

template <class F>
static int guarded(vd_handle* h, char* err, size_t errlen, F&& body) {
  try {
    body();
    return VD_OK;
  } catch (const VdError& e) {
    if (e.code == VD_ECUDA && h) {
      h->healthy = false;
      if (h->dead_reason.empty()) h->dead_reason = e.msg;
    }
    put_err(err, errlen, e.msg);
    return e.code;
  } catch (const std::exception& e) {
    put_err(err, errlen, e.what());
    return VD_EINVAL;
  }
}

extern "C" VD_API int vd_abi_version(void) { return VDEXEC_ABI_VERSION; }

// `model` as vd_open reads it: a JSON spec, or a directory holding vdexec.json.
static Json load_spec(const char* model) {
  if (!model) fail(VD_EINVAL, "null model");
  std::string text(model), spec_dir;
  if (text.empty() || text[0] != '{') {
    spec_dir = text;
    std::ifstream f(text + "/vdexec.json");
    if (!f) fail(VD_ESPEC, "no JSON spec given and no vdexec.json in " + text);
    std::stringstream ss;
    ss << f.rdbuf();
    text = ss.str();
  }
  return resolve_spec(parse_json(text), spec_dir);
}

extern "C" VD_API int vd_resolve_spec(const char* model, char* out, size_t outlen, char* err, size_t errlen) {
  return guarded(nullptr, err, errlen, [&] {
    Json j = load_spec(model);
    validate_spec(parse_spec(j));
    std::string text;
    json_write(text, j);
    if (!out || outlen < text.size() + 1)
      fail(VD_EINVAL, "the resolved spec needs " + std::to_string(text.size() + 1) + " bytes");
    std::memcpy(out, text.data(), text.size());
    out[text.size()] = '\0';
  });
}

extern "C" VD_API int vd_open(const char* model, int device, const char* opts_json, vd_handle** out, char* err,
                       size_t errlen) {
  if (!out) {
    put_err(err, errlen, "null output handle pointer");
    return VD_EINVAL;
  }
  *out = nullptr;
  vd_handle* H = new vd_handle();
  int rc = guarded(nullptr, err, errlen, [&] {
    H->spec = parse_spec(load_spec(model));
    validate_spec(H->spec);
    if (opts_json && *opts_json) {
      Json o = parse_json(opts_json);
      H->opt.max_tokens = o.integer_or("max_tokens", H->opt.max_tokens);
      H->opt.max_rows = o.integer_or("max_rows", H->opt.max_rows);
      H->opt.max_seq = o.integer_or("max_seq", H->opt.max_seq);
      H->opt.max_markers = o.integer_or("max_markers", H->opt.max_markers);
      H->opt.logprobs = o.string_or("output", "logprobs") != "logits";
      H->opt.prune_last_layer = o.boolean_or("prune_last_layer", true);
      H->opt.fork = o.boolean_or("fork", true);
      const std::string gm = o.string_or("gemm", "2sm");
      if (gm != "2sm" && gm != "1sm") fail(VD_EINVAL, "gemm must be \"2sm\" or \"1sm\"");
      H->opt.gemm2 = gm == "2sm";
      H->opt.raster_group = static_cast<int>(o.integer_or("raster_group", 0));
      const std::string gd = o.string_or("gdn", "chunk");
      if (gd != "chunk" && gd != "scan") fail(VD_EINVAL, "gdn must be \"chunk\" or \"scan\"");
      H->opt.gdn_chunk = gd == "chunk";
      if (H->opt.raster_group < 0 || H->opt.raster_group > 4096) fail(VD_EINVAL, "raster_group must be in [0, 4096]");
      const std::string at = o.string_or("attention", "tc");
      if (at != "tc" && at != "tc2" && at != "mma") fail(VD_EINVAL, "attention must be \"tc\", \"tc2\" or \"mma\"");
      H->opt.tc_attention = at != "mma";
      H->opt.tc_head = at == "tc";
      const std::string dt = o.string_or("act_dtype", "fp16");
      if (dt != "fp16" && dt != "bf16") fail(VD_EINVAL, "act_dtype must be \"fp16\" or \"bf16\"");
      H->opt.f16 = dt == "fp16";
      const std::string nm = o.string_or("norm", "fused");
      if (nm != "fused" && nm != "separate") fail(VD_EINVAL, "norm must be \"fused\" or \"separate\"");
      H->opt.fuse_norm = nm == "fused";
      H->opt.split_k = o.boolean_or("split_k", false);
      H->opt.attn_persistent = o.boolean_or("attention_persistent", true);
      H->opt.l2_hints = o.boolean_or("l2_hints", false);
      H->opt.pdl = o.boolean_or("pdl", true);
      H->opt.attn_spr = static_cast<int>(o.integer_or("attention_threads_per_row", 1));
      if (H->opt.attn_spr != 1 && H->opt.attn_spr != 2) fail(VD_EINVAL, "attention_threads_per_row must be 1 or 2");
      const long long wait_us = o.integer_or("wait_limit_us", 0);
      if (wait_us < 0 || wait_us > 60000000) fail(VD_EINVAL, "wait_limit_us must be in [0, 6e7]");
      H->opt.wait_ns = static_cast<uint64_t>(wait_us) * 1000ull;
      const long long stall = o.integer_or("debug_stall_gemm", 0);
      if (stall < 0 || stall > 1000000) fail(VD_EINVAL, "debug_stall_gemm must be in [0, 1e6]");
      H->opt.debug_stall = static_cast<int>(stall);
    }
    if (H->opt.max_tokens < 128 || H->opt.max_rows < 1 || H->opt.max_seq < 1)
      fail(VD_EINVAL, "max_tokens must be >= 128 and max_rows, max_seq >= 1");
    H->opt.max_tokens = (H->opt.max_tokens + 127) / 128 * 128;
    // Headers are parsed (and the files mapped) before any device work.
    if (!H->spec.checkpoint.empty()) {
      try {
        H->ckpt.reset(new Checkpoint(H->spec.checkpoint));
      } catch (const std::runtime_error& e) {
        fail(VD_ESPEC, e.what());
      }
    }
    H->device = device;
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop;
    cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10) fail(VD_ECUDA, std::string("this library targets sm_100a (B200); device is ") + prop.name);
    H->num_sms = prop.multiProcessorCount;
    cuda_check(cudaStreamCreateWithFlags(&H->stream, cudaStreamNonBlocking), "stream");
    init_kernel_attrs();
    H->gemm2_pairs = gemm2_max_pairs(H->num_sms);
    if (H->spec.decoder()) load_decoder(H);
    else load_encoder(H);
    alloc_workspace(H);
    cuda_check(cudaGetLastError(), "weight load launch");
    cuda_check(cudaStreamSynchronize(H->stream), "weight load");
    release_checkpoint(H);
  });
  if (rc != VD_OK) {
    vd_close(H);
    return rc;
  }
  *out = H;
  return VD_OK;
}

extern "C" VD_API int vd_infer(vd_handle* h, const vd_batch* batch, float* logits_out, int64_t out_width, char* err,
                        size_t errlen) {
  if (!h) {
    put_err(err, errlen, "null handle");
    return VD_EINVAL;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  if (!h->healthy) {
    put_err(err, errlen, "the executor is dead: " + h->dead_reason);
    return VD_EDEAD;
  }
  const auto t_call = std::chrono::steady_clock::now();
  return guarded(h, err, errlen, [&] {
    cuda_check(cudaSetDevice(h->device), "cudaSetDevice");
    validate_batch(h, batch, out_width);
    if (batch->b == 0) return;
    if (!logits_out) fail(VD_EINVAL, "null logits_out");
    struct HostTimer {
      vd_handle* h;
      std::chrono::steady_clock::time_point t0;
      ~HostTimer() {
        h->stats.host_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
      }
    } host_timer{h, t_call};
    if (batch->memory == VD_MEM_DEVICE) {
      run_batch(h, batch, batch->input_ids, batch->marker_pos, batch->marker_mask, batch->nopts, batch->qtype,
                logits_out, out_width);
      check_device_error(h);
      return;
    }
    const int64_t b = batch->b, n_ids = b * batch->l, n_m = b * batch->k;
    cudaStream_t s = h->stream;
    cuda_check(cudaStreamSynchronize(s), "synchronize");  // staging buffers may be regrown
    ensure_host_inputs(h, n_ids, n_m, b, b * out_width);
    cuda_check(cudaEventRecord(h->ev_in, s), "event");
    cuda_check(cudaMemcpyAsync(h->in_ids, batch->input_ids, n_ids * 8, cudaMemcpyHostToDevice, s), "upload ids");
    cuda_check(cudaMemcpyAsync(h->in_mpos, batch->marker_pos, n_m * 8, cudaMemcpyHostToDevice, s), "upload markers");
    if (batch->marker_mask)
      cuda_check(cudaMemcpyAsync(h->in_mmask, batch->marker_mask, n_m, cudaMemcpyHostToDevice, s), "upload mask");
    if (batch->nopts)
      cuda_check(cudaMemcpyAsync(h->in_nopts, batch->nopts, b * 8, cudaMemcpyHostToDevice, s), "upload nopts");
    if (batch->qtype)
      cuda_check(cudaMemcpyAsync(h->in_qtype, batch->qtype, b * 8, cudaMemcpyHostToDevice, s), "upload qtype");
    const double prep_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_call).count();
    run_batch(h, batch, h->in_ids, h->in_mpos, batch->marker_mask ? h->in_mmask : nullptr,
              batch->nopts ? h->in_nopts : nullptr, batch->qtype ? h->in_qtype : nullptr, h->out_dev, out_width);
    const auto t_launched = std::chrono::steady_clock::now();
    cuda_check(cudaMemcpyAsync(logits_out, h->out_dev, b * out_width * sizeof(float), cudaMemcpyDeviceToHost, s),
               "download logits");
    cuda_check(cudaEventRecord(h->ev_out, s), "event");
    check_device_error(h);
    float up = 0, down = 0;
    if (cudaEventElapsedTime(&up, h->ev_in, h->ev0) == cudaSuccess) h->stats.upload_ms = up;
    if (cudaEventElapsedTime(&down, h->ev1, h->ev_out) == cudaSuccess) h->stats.download_ms = down;
    h->stats.prep_ms = prep_ms;
    h->stats.finish_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_launched).count();
  });
}

extern "C" VD_API int vd_infer_async(vd_handle* h, const vd_batch* batch, float* logits_out_dev, int64_t out_width,
                              void* stream, char* err, size_t errlen) {
  if (!h) {
    put_err(err, errlen, "null handle");
    return VD_EINVAL;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  if (!h->healthy) {
    put_err(err, errlen, "the executor is dead: " + h->dead_reason);
    return VD_EDEAD;
  }
  return guarded(h, err, errlen, [&] {
    cuda_check(cudaSetDevice(h->device), "cudaSetDevice");
    validate_batch(h, batch, out_width);
    if (batch->memory != VD_MEM_DEVICE) fail(VD_EINVAL, "vd_infer_async takes device-resident batches");
    if (batch->b == 0) return;
    cudaStream_t user = static_cast<cudaStream_t>(stream);
    if (user && user != h->stream) {
      cuda_check(cudaEventRecord(h->ev_user, user), "event");
      cuda_check(cudaStreamWaitEvent(h->stream, h->ev_user, 0), "stream wait");
    }
    run_batch(h, batch, batch->input_ids, batch->marker_pos, batch->marker_mask, batch->nopts, batch->qtype,
              logits_out_dev, out_width);
    if (user && user != h->stream) cuda_check(cudaStreamWaitEvent(user, h->ev1, 0), "stream wait");
  });
}

extern "C" VD_API int vd_sync(vd_handle* h, char* err, size_t errlen) {
  if (!h) {
    put_err(err, errlen, "null handle");
    return VD_EINVAL;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  if (!h->healthy) {
    put_err(err, errlen, "the executor is dead: " + h->dead_reason);
    return VD_EDEAD;
  }
  return guarded(h, err, errlen, [&] {
    cuda_check(cudaSetDevice(h->device), "cudaSetDevice");
    check_device_error(h);
  });
}

extern "C" VD_API int vd_set_profiling(vd_handle* h, int on) {
  if (!h) return VD_EINVAL;
  std::lock_guard<std::mutex> lock(h->mu);
  h->profiling = on != 0;
  return VD_OK;
}

extern "C" VD_API void* vd_stream(vd_handle* h) { return h ? static_cast<void*>(h->stream) : nullptr; }

extern "C" VD_API int vd_shape_buckets(vd_handle* h, int64_t* out, int64_t cap) {
  (void)h;
  (void)out;
  (void)cap;
  return 0;
}

extern "C" VD_API int vd_media_capable(vd_handle* h) {
  (void)h;
  return 0;
}

extern "C" VD_API int vd_health(vd_handle* h) {
  if (!h || !h->healthy) return 0;
  std::lock_guard<std::mutex> lock(h->mu);
  if (cudaSetDevice(h->device) != cudaSuccess) return 0;
  const cudaError_t e = cudaStreamQuery(h->stream);
  if (e != cudaSuccess && e != cudaErrorNotReady) {
    h->healthy = false;
    h->dead_reason = cudaGetErrorString(e);
    return 0;
  }
  return 1;
}

extern "C" VD_API int64_t vd_label_width(vd_handle* h) { return h && h->spec.decoder() ? h->n_labels : 0; }

extern "C" VD_API int vd_last_stats(vd_handle* h, vd_stats* out) {
  if (!h || !out) return VD_EINVAL;
  std::lock_guard<std::mutex> lock(h->mu);
  *out = h->stats;
  return VD_OK;
}

extern "C" VD_API void vd_close(vd_handle* h) {
  if (!h) return;
  {
    std::lock_guard<std::mutex> lock(h->mu);
    if (cudaSetDevice(h->device) == cudaSuccess) {
      if (h->stream) cudaStreamSynchronize(h->stream);
      for (void* p : h->allocations) cudaFree(p);
      release_checkpoint(h);
      for (void* p : {static_cast<void*>(h->in_ids), static_cast<void*>(h->in_mpos), static_cast<void*>(h->in_mmask),
                      static_cast<void*>(h->in_nopts), static_cast<void*>(h->in_qtype), static_cast<void*>(h->out_dev)})
        if (p) cudaFree(p);
      for (int i = 0; i < vd_handle::kSlots; ++i) {
        if (h->pinned[i]) cudaFreeHost(h->pinned[i]);
        if (h->slot_ev[i]) cudaEventDestroy(h->slot_ev[i]);
      }
      if (h->ev0) cudaEventDestroy(h->ev0);
      if (h->ev1) cudaEventDestroy(h->ev1);
      if (h->ev_in) cudaEventDestroy(h->ev_in);
      if (h->ev_out) cudaEventDestroy(h->ev_out);
      if (h->ev_user) cudaEventDestroy(h->ev_user);
      for (cudaEvent_t e : h->prof_pool) cudaEventDestroy(e);
      if (h->stream) cudaStreamDestroy(h->stream);
    }
  }
  delete h;
}

// Kernel-level entry points share the helpers above.
#include "ops.cuh"

// ---------------------------------------------------------------------------
// vdk_attention_noalloc: the varlen attention kernel with its tile table in a
// fixed device array instead of memory allocated per call.
//
// The attention kernel needs one 32-byte work descriptor per 64-row query tile
// (AttnTile, eight ints).  vdk_attention allocates that table on every call; this variant
// keeps it in g_noalloc_tiles below, a file-scope device array that exists on
// every GPU that loads the library until the process exits.  The host side
// builds the table in a static host array and copies it over, so the call
// performs no device or host allocation of its own.
// ---------------------------------------------------------------------------
namespace vd {

// At most this many query tiles per call: sum over sequences of ceil(len / 64).
constexpr int kNoAllocMaxTiles = 16384;  // 512 KiB of device memory per GPU

static __device__ __align__(256) AttnTile g_noalloc_tiles[kNoAllocMaxTiles];

static std::mutex g_noalloc_mu;                         // guards the two arrays below
static AttnTile g_noalloc_host_tiles[kNoAllocMaxTiles];  // host staging, reused by every call
static AttnTile* g_noalloc_dev_tiles[64] = {};           // device address of g_noalloc_tiles, per GPU

// Device address of g_noalloc_tiles on the current GPU.  The name
// g_noalloc_tiles in host code is only a host-side stand-in, so the address is
// looked up once per device with that device current and kept.
static AttnTile* noalloc_tiles_on_current_device() {
  int dev = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 64) fail(VD_EINVAL, "device index out of range");
  if (!g_noalloc_dev_tiles[dev]) {
    void* p = nullptr;
    cuda_check(cudaGetSymbolAddress(&p, g_noalloc_tiles), "cudaGetSymbolAddress(g_noalloc_tiles)");
    g_noalloc_dev_tiles[dev] = static_cast<AttnTile*>(p);
  }
  return g_noalloc_dev_tiles[dev];
}

}  // namespace vd

extern "C" VD_API int vdk_attention_noalloc(const void* qkv, int64_t ld_qkv, int64_t q_col0, int64_t k_col0,
                                            int64_t v_col0, int heads, int kv_heads, int head_dim, int dtype,
                                            int causal, const int32_t* cu_seqlens_host, int64_t nseq, void* out,
                                            int64_t ld_out, void* stream, char* err, size_t errlen) {
  return guarded(nullptr, err, errlen, [&] {
    if (heads < 1 || kv_heads < 1 || heads % kv_heads != 0) fail(VD_EINVAL, "heads must be a multiple of kv_heads");
    if (nseq < 1 || !cu_seqlens_host) fail(VD_EINVAL, "need at least one sequence");
    if (!qkv || !out) fail(VD_EINVAL, "null buffer");
    if (!((head_dim == 64 && !causal) || (head_dim == 128 && causal) || (head_dim == 256 && causal)))
      fail(VD_EINVAL, "supported: head_dim 64 bidirectional, 128 / 256 causal");
    const bool f16 = ops_dtype(dtype);
    // Count the tiles before touching anything shared or the device.
    int64_t n = 0;
    for (int64_t i = 0; i < nseq; ++i) {
      const int64_t len = static_cast<int64_t>(cu_seqlens_host[i + 1]) - cu_seqlens_host[i];
      if (len < 0) fail(VD_EINVAL, "cu_seqlens must be non-decreasing");
      n += (len + 63) / 64;
    }
    if (n > kNoAllocMaxTiles)
      fail(VD_EINVAL, "vdk_attention_noalloc: the batch needs " + std::to_string(n) +
                          " query tiles of 64 rows; this entry point holds at most " +
                          std::to_string(kNoAllocMaxTiles) + " (use vdk_attention for larger batches)");
    if (n == 0) return;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    ops_attrs_once();
    AttnTile* d_tiles = noalloc_tiles_on_current_device();
    int t = 0;
    for (int64_t i = 0; i < nseq; ++i) {
      const int start = cu_seqlens_host[i], len = cu_seqlens_host[i + 1] - start;
      for (int q = 0; q < len; q += 64) g_noalloc_host_tiles[t++] = AttnTile{start, len, q, 0, 0, {0, 0, 0}};
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Every tile the kernel reads is written here, so nothing left over from an
    // earlier call is ever read.
    cuda_check(cudaMemcpyAsync(d_tiles, g_noalloc_host_tiles, sizeof(AttnTile) * t, cudaMemcpyHostToDevice, s),
               "upload tile table");
    AttnParams p{};
    p.gate_col0 = -1;
    p.qkv = qkv;
    p.ld_qkv = static_cast<int>(ld_qkv);
    p.q_col0 = static_cast<int>(q_col0);
    p.k_col0 = static_cast<int>(k_col0);
    p.v_col0 = static_cast<int>(v_col0);
    p.out = out;
    p.ld_out = static_cast<int>(ld_out);
    p.tiles = d_tiles;
    p.group = heads / kv_heads;
    p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)) * 1.4426950408889634);
    dim3 grid(static_cast<unsigned>(t), heads);
    auto run = [&](auto tag) {
      using T = decltype(tag);
      if (head_dim == 64)
        attention_varlen_kernel<64, false, T><<<grid, 128, AttnConfig<64>::SMEM_BYTES, s>>>(p);
      else if (head_dim == 128)
        attention_varlen_kernel<128, true, T><<<grid, 128, AttnConfig<128>::SMEM_BYTES, s>>>(p);
      else
        attention_varlen_kernel<256, true, T><<<grid, 128, AttnConfig<256>::SMEM_BYTES, s>>>(p);
    };
    if (f16) run(__half());
    else run(__nv_bfloat16());
    cuda_check(cudaGetLastError(), "attention launch");
    // The table stays in use until the kernel finishes; returning only then
    // keeps back-to-back calls from the same thread from overwriting it early.
    cuda_check(cudaStreamSynchronize(s), "synchronize");
  });
}
