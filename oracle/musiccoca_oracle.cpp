// TEST INFRASTRUCTURE ONLY.
//
// CPU oracle for the style-prompt path: the MusicCoCa text tower
// (token embedding, 12 pre-LN transformer layers with capped attention
// logits, exit LayerNorm, attention pooler with a per-dimension query scale)
// and the residual vector quantisation of its embedding into style tokens,
// restated in plain C++ float32 (the reference runs MusicCoCa in float32,
// system.cpp:116-117). Used by tests/ only; nothing in the engine links,
// loads or calls it. The SentencePiece tokenizer is not restated: the input
// is the token ids and padding mask that StyleModel::tokenize_text_ids
// (style_model.cpp) produces.
//
// Reference: rhymeswithlion/magenta-realtime-mlx-cpp (v0.1.0),
// src/magenta_realtime_mlx/{musiccoca.cpp, style_model.cpp, rvq.cpp,
// nn_ops.h}. Parity status: the reference ships no MusicCoCa test or golden
// vector and cannot be built here (MLX is absent): **parity unpinned**;
// tests/test_musiccoca_oracle.py checks this restatement against an
// independent torch formulation of the same code.

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "safetensors_reader.h"

namespace oracle {
namespace mc {

static thread_local std::string g_err;

// MusicCoCaConfig (musiccoca.h): text tower dimensions.
constexpr int kD = 768, kHeads = 12, kDHead = 64, kFF = 3072, kLayers = 12, kPoolDHead = 256;
constexpr float kCap = 50.0f;    // TransformerLayer::kAttenLogitCap
constexpr float kLnEps = 1e-5f;  // every LayerNorm (musiccoca.cpp TransformerLayer / pooler / exit)

typedef float v8f __attribute__((vector_size(32)));

static inline float dot(const float* a, const float* b, int K) {
  v8f acc = {0, 0, 0, 0, 0, 0, 0, 0};
  int k = 0;
  for (; k + 8 <= K; k += 8) {
    v8f x, y;
    std::memcpy(&x, a + k, 32);
    std::memcpy(&y, b + k, 32);
    acc += x * y;
  }
  float s = 0.f;
  for (int i = 0; i < 8; ++i) s += acc[i];
  for (; k < K; ++k) s += a[k] * b[k];
  return s;
}

// Linear with bias, weight stored (out, in) (Linear::operator():
// matmul(x, weight^T) + bias).
struct Lin {
  int out = 0, in = 0;
  std::vector<float> w, b;
};

static void linear(const float* x, int M, const Lin& l, float* y) {
#pragma omp parallel for schedule(static)
  for (int o = 0; o < l.out; ++o)
    for (int m = 0; m < M; ++m) y[(size_t)m * l.out + o] = dot(x + (size_t)m * l.in, l.w.data() + (size_t)o * l.in, l.in) + l.b[o];
}

struct LN {
  std::vector<float> w, b;
};

// LayerNorm::operator(): mean, centred, var = mean(centred^2),
// centred * rsqrt(var + eps), then * weight + bias.
static void layer_norm(const float* x, int M, const LN& ln, float* y) {
  for (int m = 0; m < M; ++m) {
    const float* r = x + (size_t)m * kD;
    float s = 0.f;
    for (int i = 0; i < kD; ++i) s += r[i];
    const float mean = s / kD;
    float v = 0.f;
    for (int i = 0; i < kD; ++i) v += (r[i] - mean) * (r[i] - mean);
    const float inv = 1.0f / std::sqrt(v / kD + kLnEps);
    for (int i = 0; i < kD; ++i) y[(size_t)m * kD + i] = (r[i] - mean) * inv * ln.w[i] + ln.b[i];
  }
}

// gelu, exact form (nn_ops.h:44-53)
static inline float gelu(float x) { return 0.5f * x * (1.0f + std::erf(x * 0.7071067811865475f)); }

// softplus, stable form (musiccoca.cpp softplus)
static inline float softplus(float x) { return std::max(x, 0.0f) + std::log1p(std::exp(-std::fabs(x))); }

struct MHA {
  Lin q, k, v, o;
  int H = kHeads, Dh = kDHead;
  std::vector<float> per_dim_scale;  // (Dh) or empty
  float cap = 0.f;
};

// CoCaMHA::operator(): projections, optional per-dimension query scale
// softplus(s) / ln 2, logits q.k / sqrt(Dh), optional cap * tanh(logits /
// cap), optional additive key mask, softmax, weighted values, o_proj.
static void mha(const MHA& a, const float* qin, int Sq, const float* kvin, int Sk, const float* key_mask,
                float* out) {
  const int HD = a.H * a.Dh;
  std::vector<float> q((size_t)Sq * HD), k((size_t)Sk * HD), v((size_t)Sk * HD), ctx((size_t)Sq * HD);
  linear(qin, Sq, a.q, q.data());
  linear(kvin, Sk, a.k, k.data());
  linear(kvin, Sk, a.v, v.data());
  if (!a.per_dim_scale.empty()) {
    std::vector<float> sc(a.Dh);
    for (int d = 0; d < a.Dh; ++d) sc[d] = softplus(a.per_dim_scale[d]) / std::log(2.0f);
    for (int i = 0; i < Sq; ++i)
      for (int h = 0; h < a.H; ++h)
        for (int d = 0; d < a.Dh; ++d) q[(size_t)i * HD + h * a.Dh + d] *= sc[d];
  }
  const float scale = 1.0f / std::sqrt(static_cast<float>(a.Dh));
#pragma omp parallel for collapse(2) schedule(static)
  for (int h = 0; h < a.H; ++h)
    for (int i = 0; i < Sq; ++i) {
      std::vector<float> p(Sk);
      float mx = -INFINITY;
      for (int j = 0; j < Sk; ++j) {
        float l = dot(q.data() + (size_t)i * HD + h * a.Dh, k.data() + (size_t)j * HD + h * a.Dh, a.Dh) * scale;
        if (a.cap > 0.f) l = a.cap * std::tanh(l / a.cap);
        if (key_mask) l += key_mask[j];
        p[j] = l;
        mx = std::max(mx, l);
      }
      float sum = 0.f;
      for (int j = 0; j < Sk; ++j) {
        p[j] = std::exp(p[j] - mx);
        sum += p[j];
      }
      float* c = ctx.data() + (size_t)i * HD + h * a.Dh;
      for (int d = 0; d < a.Dh; ++d) c[d] = 0.f;
      for (int j = 0; j < Sk; ++j) {
        const float w = p[j] / sum;
        const float* vr = v.data() + (size_t)j * HD + h * a.Dh;
        for (int d = 0; d < a.Dh; ++d) c[d] += w * vr[d];
      }
    }
  linear(ctx.data(), Sq, a.o, out);
}

struct Layer {
  LN attn_ln, ffn_ln;
  MHA attn;
  Lin w1, w2;
};

struct Model {
  std::vector<float> emb;  // (V, 768)
  int V = 0;
  std::vector<Layer> layers;
  LN exit_ln, pool_ln;
  std::vector<float> pool_query;  // (768)
  MHA pool;
  std::vector<float> codebooks;  // (K, C, 768)
  int K = 0, C = 0;
};

static Lin load_lin(const SafeTensors& st, const std::string& p, int out, int in) {
  Lin l;
  l.out = out;
  l.in = in;
  l.w = st.get(p + ".weight", (int64_t)out * in);
  l.b = st.get(p + ".bias", out);
  return l;
}

static LN load_ln(const SafeTensors& st, const std::string& p) {
  LN n;
  n.w = st.get(p + ".weight", kD);
  n.b = st.get(p + ".bias", kD);
  return n;
}

// Keys of the MusicCoCa encoder bundle read by the text tower
// (MusicCoCaEncoder / TransformerLayer / AttentionPooler constructors,
// musiccoca.cpp) and the "codebooks" tensor of its codebook bundle
// (StyleModel::StyleModel, style_model.cpp).
static Model* load(const char* enc_path, const char* cb_path) {
  std::unique_ptr<Model> m(new Model());
  {
    SafeTensors st(enc_path);
    auto it = st.info.find("token_embedding.weight");
    if (it == st.info.end()) throw std::out_of_range("missing key \"token_embedding.weight\"");
    m->V = (int)it->second.shape[0];
    m->emb = st.get("token_embedding.weight", (int64_t)m->V * kD);
    for (int i = 0; i < kLayers; ++i) {
      const std::string p = "text_layers." + std::to_string(i);
      Layer L;
      L.attn_ln = load_ln(st, p + ".attn_ln");
      L.ffn_ln = load_ln(st, p + ".ffn_ln");
      L.attn.q = load_lin(st, p + ".attn.q_proj", kHeads * kDHead, kD);
      L.attn.k = load_lin(st, p + ".attn.k_proj", kHeads * kDHead, kD);
      L.attn.v = load_lin(st, p + ".attn.v_proj", kHeads * kDHead, kD);
      L.attn.o = load_lin(st, p + ".attn.o_proj", kD, kHeads * kDHead);
      L.attn.cap = kCap;
      L.w1 = load_lin(st, p + ".ffn_w1", kFF, kD);
      L.w2 = load_lin(st, p + ".ffn_w2", kD, kFF);
      m->layers.push_back(std::move(L));
    }
    m->exit_ln = load_ln(st, "text_exit_ln");
    m->pool_ln = load_ln(st, "text_pooler.ln");
    m->pool_query = st.get("text_pooler.query", kD);
    m->pool.q = load_lin(st, "text_pooler.attn.q_proj", kHeads * kPoolDHead, kD);
    m->pool.k = load_lin(st, "text_pooler.attn.k_proj", kHeads * kPoolDHead, kD);
    m->pool.v = load_lin(st, "text_pooler.attn.v_proj", kHeads * kPoolDHead, kD);
    m->pool.o = load_lin(st, "text_pooler.attn.o_proj", kD, kHeads * kPoolDHead);
    m->pool.Dh = kPoolDHead;
    m->pool.per_dim_scale = st.get("text_pooler.attn._per_dim_scale", kPoolDHead);
  }
  {
    SafeTensors st(cb_path);
    auto it = st.info.find("codebooks");
    if (it == st.info.end()) throw std::out_of_range("missing key \"codebooks\"");
    if (it->second.shape.size() != 3 || it->second.shape[2] != kD) throw std::runtime_error("codebooks must be (K, C, 768)");
    m->K = (int)it->second.shape[0];
    m->C = (int)it->second.shape[1];
    m->codebooks = st.get("codebooks", (int64_t)m->K * m->C * kD);
  }
  return m.release();
}

// MusicCoCaEncoder::embed_text: ids (L) with padding (L, 1 = padded) ->
// the pooled (768) embedding.
static void embed_text(const Model& m, const int32_t* ids, const float* pad, int L, float* out) {
  std::vector<float> x((size_t)L * kD), h((size_t)L * kD), a((size_t)L * kD), f((size_t)L * kFF), mask(L);
  const float s = std::sqrt(static_cast<float>(kD));
  for (int l = 0; l < L; ++l) {
    if (ids[l] < 0 || ids[l] >= m.V) throw std::out_of_range("token id out of range");
    const float* e = m.emb.data() + (size_t)ids[l] * kD;
    for (int i = 0; i < kD; ++i) x[(size_t)l * kD + i] = e[i] * s;
    mask[l] = pad[l] * -1e9f;
  }
  for (const Layer& Ly : m.layers) {
    // TransformerLayer::operator(): x + attn(LN(x)); y + w2(gelu(w1(LN(y))))
    layer_norm(x.data(), L, Ly.attn_ln, h.data());
    mha(Ly.attn, h.data(), L, h.data(), L, mask.data(), a.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] += a[i];
    layer_norm(x.data(), L, Ly.ffn_ln, h.data());
    linear(h.data(), L, Ly.w1, f.data());
    for (auto& v : f) v = gelu(v);
    linear(f.data(), L, Ly.w2, a.data());
    for (size_t i = 0; i < x.size(); ++i) x[i] += a[i];
  }
  layer_norm(x.data(), L, m.exit_ln, h.data());
  // AttentionPooler::operator(): learned query over LN(encoder output), no mask
  layer_norm(h.data(), L, m.pool_ln, a.data());
  mha(m.pool, m.pool_query.data(), 1, a.data(), L, nullptr, out);
}

// rvq_quantization (rvq.cpp:24-66): per level, distances |r|^2 - 2 r.c +
// |c|^2 to every codeword, first argmin, residual -= codeword.
static void quantize(const Model& m, const float* emb, int levels, int32_t* tokens) {
  if (levels > m.K) throw std::runtime_error("more levels than codebooks");
  std::vector<float> r(emb, emb + kD);
  for (int k = 0; k < levels; ++k) {
    const float* cb = m.codebooks.data() + (size_t)k * m.C * kD;
    float r2 = 0.f;
    for (int i = 0; i < kD; ++i) r2 += r[i] * r[i];
    int best = 0;
    float bd = INFINITY;
    for (int c = 0; c < m.C; ++c) {
      const float* w = cb + (size_t)c * kD;
      float c2 = 0.f;
      for (int i = 0; i < kD; ++i) c2 += w[i] * w[i];
      const float d = (r2 - 2.0f * dot(r.data(), w, kD)) + c2;
      if (d < bd) {
        bd = d;
        best = c;
      }
    }
    tokens[k] = best;
    for (int i = 0; i < kD; ++i) r[i] -= cb[(size_t)best * kD + i];
  }
}

}  // namespace mc
}  // namespace oracle

using namespace oracle::mc;

extern "C" {

const char* orc_mc_last_error() { return g_err.c_str(); }

void* orc_mc_create(const char* encoder_path, const char* codebooks_path) {
  try {
    return load(encoder_path, codebooks_path);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void orc_mc_destroy(void* h) { delete static_cast<Model*>(h); }

// ids / pad (B, L) -> out (B, 768)
int orc_mc_embed_text(void* h, const int32_t* ids, const float* pad, int B, int L, float* out) {
  try {
    for (int b = 0; b < B; ++b) embed_text(*static_cast<Model*>(h), ids + (size_t)b * L, pad + (size_t)b * L, L, out + (size_t)b * kD);
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

// emb (N, 768) -> tokens (N, levels)
int orc_mc_quantize(void* h, const float* emb, int N, int levels, int32_t* tokens) {
  try {
    for (int n = 0; n < N; ++n) quantize(*static_cast<Model*>(h), emb + (size_t)n * kD, levels, tokens + (size_t)n * levels);
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}

}  // extern "C"
