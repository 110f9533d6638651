// TEST INFRASTRUCTURE ONLY.
//
// CPU oracle for the codec phase of a chunk: RVQ dequantisation, the
// SpectroStream decoder and the iSTFT post-processor, restated in plain C++
// float32 (the reference runs this decoder in float32, system.cpp:118-119).
// Used by tests/ (parity checks against the CUDA codec) and by bench.py's CPU
// baseline; the engine never links, loads or calls it.
//
// Reference: rhymeswithlion/magenta-realtime-mlx-cpp (v0.1.0),
// src/magenta_realtime_mlx/{spectrostream.cpp, rvq.cpp, nn_ops.h, system.cpp}.
// Parity status: the reference ships no SpectroStream test or golden vector
// and cannot be built here (MLX is absent), so the decoder numerics are
// **parity unpinned**; tests/test_codec_oracle.py checks this restatement
// against an independent torch formulation of the same layers.
//
// Layout: every activation is NHWC float32 (the reference's layout,
// spectrostream.h:22-25); conv weights are kept as (O, kh, kw, I), which is
// what WNConv2d / WNConvTranspose2d convert the file's canonical layouts to
// (spectrostream.cpp:110-116).

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "safetensors_reader.h"

namespace oracle {
namespace ss {

static thread_local std::string g_err;

struct T4 {
  int n = 0, h = 0, w = 0, c = 0;
  std::vector<float> v;
  T4() = default;
  T4(int n_, int h_, int w_, int c_) : n(n_), h(h_), w(w_), c(c_), v((size_t)n_ * h_ * w_ * c_, 0.f) {}
  float* px(int i, int y, int x) { return v.data() + (((size_t)i * h + y) * w + x) * c; }
  const float* px(int i, int y, int x) const { return v.data() + (((size_t)i * h + y) * w + x) * c; }
};

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

// A convolution: weight (O, kh, kw, I), bias (O) or empty.
struct Conv {
  int O = 0, kh = 1, kw = 1, I = 0;
  std::vector<float> w, b;
};

// conv2d weight: file layout (O, I, kh, kw) -> (O, kh, kw, I)
// (convert_conv2d_weight, spectrostream.cpp:110-112).
static Conv conv_from_canonical(const float* wc, const float* bias, int O, int I, int kh, int kw) {
  Conv cv;
  cv.O = O; cv.I = I; cv.kh = kh; cv.kw = kw;
  cv.w.resize((size_t)O * kh * kw * I);
  for (int o = 0; o < O; ++o)
    for (int i = 0; i < I; ++i)
      for (int y = 0; y < kh; ++y)
        for (int x = 0; x < kw; ++x)
          cv.w[(((size_t)o * kh + y) * kw + x) * I + i] = wc[(((size_t)o * I + i) * kh + y) * kw + x];
  if (bias) cv.b.assign(bias, bias + O);
  return cv;
}

// conv_transpose2d weight: file layout (I, O, kh, kw) -> (O, kh, kw, I)
// (convert_conv_transpose2d_weight, spectrostream.cpp:114-116).
static Conv convt_from_canonical(const float* wc, const float* bias, int I, int O, int kh, int kw) {
  Conv cv;
  cv.O = O; cv.I = I; cv.kh = kh; cv.kw = kw;
  cv.w.resize((size_t)O * kh * kw * I);
  for (int i = 0; i < I; ++i)
    for (int o = 0; o < O; ++o)
      for (int y = 0; y < kh; ++y)
        for (int x = 0; x < kw; ++x)
          cv.w[(((size_t)o * kh + y) * kw + x) * I + i] = wc[(((size_t)i * O + o) * kh + y) * kw + x];
  if (bias) cv.b.assign(bias, bias + O);
  return cv;
}

// mx::conv2d(x, w, stride, padding 0) + bias (WNConv2d::operator(),
// spectrostream.cpp:135-139): out[n, oy, ox, o] =
//   sum_{dy, dx, i} x[n, oy*sh + dy, ox*sw + dx, i] * w[o, dy, dx, i] (+ b[o]).
static T4 conv2d(const T4& x, const Conv& cv, int sh, int sw) {
  if (x.c != cv.I) throw std::runtime_error("conv2d: channel mismatch");
  const int Ho = (x.h - cv.kh) / sh + 1, Wo = (x.w - cv.kw) / sw + 1;
  if (Ho <= 0 || Wo <= 0) throw std::runtime_error("conv2d: input smaller than the kernel");
  T4 y(x.n, Ho, Wo, cv.O);
  const int seg = cv.kw * cv.I;  // one kernel row of an NHWC patch is contiguous
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int n = 0; n < x.n; ++n)
    for (int oy = 0; oy < Ho; ++oy)
      for (int ox = 0; ox < Wo; ++ox) {
        float* out = y.px(n, oy, ox);
        for (int o = 0; o < cv.O; ++o) {
          float acc = 0.f;
          for (int dy = 0; dy < cv.kh; ++dy)
            acc += dot(x.px(n, oy * sh + dy, ox * sw), cv.w.data() + ((size_t)o * cv.kh + dy) * seg, seg);
          out[o] = cv.b.empty() ? acc : acc + cv.b[o];
        }
      }
  return y;
}

// mx::conv_transpose2d(x, w, stride, padding 0) + bias
// (WNConvTranspose2d::operator(), spectrostream.cpp:153-157): the adjoint of
// conv2d, out[n, iy*sh + dy, ix*sw + dx, o] += x[n, iy, ix, :] . w[o, dy, dx, :],
// full size ((H - 1) sh + kh, (W - 1) sw + kw). Written as a gather per output.
static T4 conv_transpose2d(const T4& x, const Conv& cv, int sh, int sw) {
  if (x.c != cv.I) throw std::runtime_error("conv_transpose2d: channel mismatch");
  const int Ho = (x.h - 1) * sh + cv.kh, Wo = (x.w - 1) * sw + cv.kw;
  T4 y(x.n, Ho, Wo, cv.O);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int n = 0; n < x.n; ++n)
    for (int oy = 0; oy < Ho; ++oy)
      for (int ox = 0; ox < Wo; ++ox) {
        float* out = y.px(n, oy, ox);
        for (int o = 0; o < cv.O; ++o) {
          float acc = 0.f;
          for (int dy = 0; dy < cv.kh; ++dy) {
            const int ty = oy - dy;
            if (ty < 0 || ty % sh) continue;
            const int iy = ty / sh;
            if (iy >= x.h) continue;
            for (int dx = 0; dx < cv.kw; ++dx) {
              const int tx = ox - dx;
              if (tx < 0 || tx % sw) continue;
              const int ix = tx / sw;
              if (ix >= x.w) continue;
              acc += dot(x.px(n, iy, ix), cv.w.data() + (((size_t)o * cv.kh + dy) * cv.kw + dx) * cv.I, cv.I);
            }
          }
          out[o] = cv.b.empty() ? acc : acc + cv.b[o];
        }
      }
  return y;
}

// Zero padding of H (top, bottom) and W (left, right) (mx::pad).
static T4 pad(const T4& x, int top, int bottom, int left, int right) {
  T4 y(x.n, x.h + top + bottom, x.w + left + right, x.c);
  for (int n = 0; n < x.n; ++n)
    for (int r = 0; r < x.h; ++r)
      std::memcpy(y.px(n, r + top, left), x.px(n, r, 0), sizeof(float) * x.w * x.c);
  return y;
}

// causal_same_pad (spectrostream.cpp:41-62): H padded on top by kh - sh;
// W padded to the "same" output width ceil(W / sw), the total split
// left = total / 2, right = the rest.
static T4 causal_same_pad(const T4& x, int kh, int kw, int sh, int sw) {
  const int top = kh - sh;
  const int ow = (x.w + sw - 1) / sw;
  const int tot = std::max((ow - 1) * sw + kw - x.w, 0);
  if (top <= 0 && tot <= 0) return x;
  return pad(x, std::max(top, 0), 0, tot / 2, tot - tot / 2);
}

// elu with alpha 1 (nn_ops.h:31-39): x > 0 ? x : alpha * (exp(x) - 1).
static inline float elu1(float v) { return v > 0.f ? v : 1.0f * (std::exp(v) - 1.0f); }
static T4 elu(const T4& x) {
  T4 y = x;
  for (auto& v : y.v) v = elu1(v);
  return y;
}

static void add_inplace(T4& a, const T4& b) {
  if (a.v.size() != b.v.size()) throw std::runtime_error("residual shape mismatch");
  for (size_t i = 0; i < a.v.size(); ++i) a.v[i] += b.v[i];
}

// Decoder block table (dec_block_specs, spectrostream.cpp:328-338):
// in, out, stride (h, w), transposed kernel, post kernel.
struct DecSpec {
  int in, out, sh, sw, tkh, tkw, pkh, pkw;
};
static const DecSpec kDecSpecs[7] = {
    {512, 1024, 2, 1, 4, 3, 3, 3}, {512, 256, 2, 2, 4, 4, 3, 3}, {256, 256, 1, 2, 3, 4, 3, 3},
    {256, 256, 1, 2, 3, 4, 3, 3},  {256, 128, 1, 3, 3, 6, 3, 3}, {128, 128, 1, 2, 3, 4, 3, 3},
    {128, 64, 1, 2, 3, 4, 3, 3},
};
constexpr int kEmb = 256;          // SpectroStreamDecoder::kEmbeddingDim
constexpr int kProj = 2560;        // input_proj width (spectrostream.cpp:358-359)
constexpr int kUnfold = 5;         // unfold_width factor (spectrostream.cpp:380)
constexpr int kTemporalCrop = 4;   // spectrostream.h:223
constexpr int kFft = 960, kHop = 480;  // istft_postprocess (spectrostream.cpp:594-595)

struct Decoder {
  // input_proj (Res1x1Block 256 -> 2560 -> 2560, no pre-ELU), input_conv
  // (Res3x3Block 512, causal), 7 DecoderResBlocks, output_conv 7x7 64 -> 2.
  Conv ip_conv1, ip_conv2, ip_short, ic_conv1, ic_conv2;
  Conv ct[7], post[7], shortcut[7];
  bool has_short[7] = {};
  Conv out_conv;
  std::vector<float> codebooks;  // (K, C, D)
  int K = 0, C = 0, D = 0;
};

static Conv load_conv(const SafeTensors& st, const std::string& prefix, int O, int I, int kh, int kw) {
  std::vector<float> w = st.get(prefix + ".weight", (int64_t)O * I * kh * kw);
  std::vector<float> b = st.get(prefix + ".bias", O);
  return conv_from_canonical(w.data(), b.data(), O, I, kh, kw);
}

static Conv load_convt(const SafeTensors& st, const std::string& prefix, int I, int O, int kh, int kw) {
  std::vector<float> w = st.get(prefix + ".weight", (int64_t)I * O * kh * kw);
  std::vector<float> b = st.get(prefix + ".bias", O);
  return convt_from_canonical(w.data(), b.data(), I, O, kh, kw);
}

// Weight keys of spectrostream_decoder.safetensors (the constructors at
// spectrostream.cpp:163-172, 183-189, 202-222, 356-363) and the
// "codebooks" tensor (K, C, D) of the codebook bundle (system.cpp:372-373).
static Decoder* load_decoder(const char* dec_path, const char* cb_path) {
  std::unique_ptr<Decoder> d(new Decoder());
  {
    SafeTensors st(dec_path);
    d->ip_conv1 = load_conv(st, "input_proj.conv1", kProj, kEmb, 1, 1);
    d->ip_conv2 = load_conv(st, "input_proj.conv2", kProj, kProj, 1, 1);
    d->ip_short = load_conv(st, "input_proj.shortcut", kProj, kEmb, 1, 1);
    d->ic_conv1 = load_conv(st, "input_conv.conv1", 512, 512, 3, 3);
    d->ic_conv2 = load_conv(st, "input_conv.conv2", 512, 512, 3, 3);
    for (int i = 0; i < 7; ++i) {
      const DecSpec& s = kDecSpecs[i];
      const std::string p = "decoder_blocks." + std::to_string(i);
      d->ct[i] = load_convt(st, p + ".conv_transpose", s.in, s.out, s.tkh, s.tkw);
      d->post[i] = load_conv(st, p + ".conv", s.out, s.out, s.pkh, s.pkw);
      d->has_short[i] = s.in != s.out;
      if (d->has_short[i]) d->shortcut[i] = load_conv(st, p + ".shortcut", s.out, s.in, 1, 1);
    }
    d->out_conv = load_conv(st, "output_conv", 2, 64, 7, 7);
  }
  {
    SafeTensors st(cb_path);
    auto it = st.info.find("codebooks");
    if (it == st.info.end()) throw std::out_of_range("missing key \"codebooks\"");
    if (it->second.shape.size() != 3) throw std::runtime_error("codebooks must be (K, C, D)");
    d->K = (int)it->second.shape[0];
    d->C = (int)it->second.shape[1];
    d->D = (int)it->second.shape[2];
    d->codebooks = st.get("codebooks", (int64_t)d->K * d->C * d->D);
  }
  return d.release();
}

// Res1x1Block::operator() (spectrostream.cpp:174-181), pre_elu = false.
static T4 res1x1(const Decoder& d, const T4& x) {
  T4 skip = conv2d(x, d.ip_short, 1, 1);
  T4 m = conv2d(x, d.ip_conv1, 1, 1);
  m = elu(m);
  m = conv2d(m, d.ip_conv2, 1, 1);
  add_inplace(m, skip);
  return m;
}

// Res3x3Block::operator() with causal = true (spectrostream.cpp:191-199).
static T4 res3x3(const Decoder& d, const T4& x) {
  T4 y = elu(x);
  y = conv2d(causal_same_pad(y, 3, 3, 1, 1), d.ic_conv1, 1, 1);
  y = elu(y);
  y = conv2d(causal_same_pad(y, 3, 3, 1, 1), d.ic_conv2, 1, 1);
  add_inplace(y, x);
  return y;
}

// DecoderResBlock::operator() (spectrostream.cpp:224-267).
static T4 dec_block(const Decoder& d, int i, const T4& x) {
  const DecSpec& s = kDecSpecs[i];
  T4 y = conv_transpose2d(elu(x), d.ct[i], s.sh, s.sw);
  // crop: the last tkh - sh rows; (tkw - sw) / 2 columns at the start and
  // the rest at the end (spectrostream.cpp:210-213, 229-240)
  const int crop_h = s.tkh - s.sh;
  const int cws = (s.tkw - s.sw) / 2, cwe = (s.tkw - s.sw) - cws;
  T4 c(y.n, y.h - crop_h, y.w - cws - cwe, y.c);
  for (int n = 0; n < c.n; ++n)
    for (int r = 0; r < c.h; ++r) std::memcpy(c.px(n, r, 0), y.px(n, r, cws), sizeof(float) * c.w * c.c);
  y = elu(c);
  y = conv2d(causal_same_pad(y, s.pkh, s.pkw, 1, 1), d.post[i], 1, 1);
  // residual: repeat sh x along H and sw x along W (mx::repeat: each element
  // repeated consecutively), then the 1x1 shortcut when in != out
  T4 r(x.n, x.h * s.sh, x.w * s.sw, x.c);
  for (int n = 0; n < r.n; ++n)
    for (int yy = 0; yy < r.h; ++yy)
      for (int xx = 0; xx < r.w; ++xx) std::memcpy(r.px(n, yy, xx), x.px(n, yy / s.sh, xx / s.sw), sizeof(float) * x.c);
  if (d.has_short[i]) r = conv2d(r, d.shortcut[i], 1, 1);
  add_inplace(y, r);
  return y;
}

// SpectroStreamDecoder::operator() (spectrostream.cpp:365-419):
// embeddings (B, S, 256) -> (B, 4 S, 480, 4).
static T4 decode(const Decoder& d, const float* emb, int B, int S) {
  // zero frame appended along S, then (B, S + 1, 1, 256)
  T4 x(B, S + 1, 1, kEmb);
  for (int b = 0; b < B; ++b)
    for (int s = 0; s < S; ++s) std::memcpy(x.px(b, s, 0), emb + ((size_t)b * S + s) * kEmb, sizeof(float) * kEmb);
  x = res1x1(d, x);  // (B, S + 1, 1, 2560)
  // unfold_width(x, 5): a reshape (spectrostream.cpp:95-102)
  x.w = kUnfold;
  x.c = kProj / kUnfold;
  x = res3x3(d, x);
  x = dec_block(d, 0, x);
  // stereo split (B, H, W, 2 C') -> (2 B, H, W, C'): image s * B + b takes
  // channels [s C', (s + 1) C') (spectrostream.cpp:385-392)
  {
    const int Ch = x.c / 2;
    T4 y(2 * B, x.h, x.w, Ch);
    for (int s = 0; s < 2; ++s)
      for (int b = 0; b < B; ++b)
        for (int r = 0; r < x.h; ++r)
          for (int q = 0; q < x.w; ++q) std::memcpy(y.px(s * B + b, r, q), x.px(b, r, q) + s * Ch, sizeof(float) * Ch);
    x = std::move(y);
  }
  for (int i = 1; i < 7; ++i) x = dec_block(d, i, x);
  x = elu(x);
  x = conv2d(causal_same_pad(x, 7, 7, 1, 1), d.out_conv, 1, 1);  // (2B, H, 480, 2)
  // temporal crop of the first 4 rows, then stereo recombine
  // (2 B, H, W, 2) -> (B, H, W, 4) with channel s * 2 + c (spectrostream.cpp:400-417)
  const int Hc = x.h - kTemporalCrop;
  T4 out(B, Hc, x.w, 4);
  for (int s = 0; s < 2; ++s)
    for (int b = 0; b < B; ++b)
      for (int r = 0; r < Hc; ++r)
        for (int q = 0; q < x.w; ++q) {
          const float* src = x.px(s * B + b, r + kTemporalCrop, q);
          float* dst = out.px(b, r, q);
          dst[2 * s] = src[0];
          dst[2 * s + 1] = src[1];
        }
  return out;
}

// istft_postprocess (spectrostream.cpp:593-681): spec (B, H, 480, 4) with
// channels [s0 re, s0 im, s1 re, s1 im] -> audio (B, target, 2) interleaved.
// irfft with n = 960 over the 480 bins plus a zero Nyquist bin (imaginary
// parts of the DC and Nyquist bins do not contribute), evaluated as a direct
// sum in double precision; synthesis window = periodic Hann / (sum of the
// squared window over the two hops), computed in float like the reference;
// overlap-add with hop 480; trimmed to target.
static void istft(const float* spec, int B, int H, int target, float* out) {
  const int F = kHop;  // frequency bins given
  if (target > H * kHop + kHop) throw std::runtime_error("istft: target longer than the signal");
  std::vector<float> win(kFft), synth(kFft);
  const float two_pi_over_n = 2.0f * static_cast<float>(M_PI) / static_cast<float>(kFft);
  for (int t = 0; t < kFft; ++t) win[t] = 0.5f - 0.5f * std::cos(static_cast<float>(t) * two_pi_over_n);
  for (int j = 0; j < kHop; ++j) {
    const float p = win[j] * win[j] + win[j + kHop] * win[j + kHop];
    synth[j] = win[j] / p;
    synth[j + kHop] = win[j + kHop] / p;
  }
  std::vector<double> cosv(kFft), sinv(kFft);
  for (int m = 0; m < kFft; ++m) {
    cosv[m] = std::cos(2.0 * M_PI * m / kFft);
    sinv[m] = std::sin(2.0 * M_PI * m / kFft);
  }
  // frames (B * 2, H, 960), windowed
  std::vector<float> fr((size_t)B * 2 * H * kFft);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int bs = 0; bs < B * 2; ++bs)
    for (int i = 0; i < H; ++i) {
      const int b = bs / 2, s = bs % 2;
      const float* X = spec + ((size_t)b * H + i) * F * 4;
      float* o = fr.data() + ((size_t)bs * H + i) * kFft;
      for (int n = 0; n < kFft; ++n) {
        double acc = X[0 * 4 + 2 * s];
        for (int k = 1; k < F; ++k) {
          const int m = (int)(((long long)k * n) % kFft);
          acc += 2.0 * (X[k * 4 + 2 * s] * cosv[m] - X[k * 4 + 2 * s + 1] * sinv[m]);
        }
        o[n] = static_cast<float>(acc / kFft) * synth[n];
      }
    }
  for (int bs = 0; bs < B * 2; ++bs) {
    const int b = bs / 2, s = bs % 2;
    const float* f = fr.data() + (size_t)bs * H * kFft;
    for (int t = 0; t < target; ++t) {
      const int i = t / kHop, j = t % kHop;
      float v = 0.f;
      if (i < H) v = f[(size_t)i * kFft + j];
      if (i >= 1) v += f[(size_t)(i - 1) * kFft + j + kHop];
      out[((size_t)b * target + t) * 2 + s] = v;
    }
  }
}

// rvq_dequantization (rvq.cpp:68-87): (n, levels) codes -> (n, D) float32,
// sum over levels k = 0, 1, ... of codebooks[k][code].
static void dequantize(const Decoder& d, const int32_t* tokens, int n, int levels, float* out) {
  if (levels > d.K) throw std::runtime_error("more levels than codebooks");
  for (int r = 0; r < n; ++r) {
    float* o = out + (size_t)r * d.D;
    std::fill(o, o + d.D, 0.f);
    for (int k = 0; k < levels; ++k) {
      const int32_t t = tokens[(size_t)r * levels + k];
      if (t < 0 || t >= d.C) throw std::out_of_range("code out of range");
      const float* cb = d.codebooks.data() + ((size_t)k * d.C + t) * d.D;
      for (int j = 0; j < d.D; ++j) o[j] += cb[j];
    }
  }
}

}  // namespace ss
}  // namespace oracle

using namespace oracle::ss;

#define ORC_SS_TRY(body)              \
  try {                               \
    body;                             \
    return 0;                         \
  } catch (const std::exception& e) { \
    g_err = e.what();                 \
    return 1;                         \
  }

extern "C" {

const char* orc_ss_last_error() { return g_err.c_str(); }

void* orc_ss_create(const char* decoder_path, const char* codebooks_path) {
  try {
    return load_decoder(decoder_path, codebooks_path);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void orc_ss_destroy(void* h) { delete static_cast<Decoder*>(h); }

int orc_ss_dequantize(void* h, const int32_t* tokens, int n, int levels, float* out) {
  ORC_SS_TRY(dequantize(*static_cast<Decoder*>(h), tokens, n, levels, out));
}

// (B, S, 256) -> (B, 4 S, 480, 4)
int orc_ss_decode(void* h, const float* emb, int B, int S, float* out) {
  ORC_SS_TRY({
    T4 y = decode(*static_cast<Decoder*>(h), emb, B, S);
    std::memcpy(out, y.v.data(), y.v.size() * sizeof(float));
  });
}

int orc_ss_istft(const float* spec, int B, int H, int target, float* out) { ORC_SS_TRY(istft(spec, B, H, target, out)); }

// The codec phase of System::generate_chunk (system.cpp:372-390) for one
// stream: codes (S, levels) -> (S * 1920, 2) samples at 48 kHz.
int orc_ss_decode_tokens(void* h, const int32_t* tokens, int S, int levels, float* audio) {
  ORC_SS_TRY({
    const Decoder& d = *static_cast<Decoder*>(h);
    std::vector<float> emb((size_t)S * d.D);
    dequantize(d, tokens, S, levels, emb.data());
    T4 spec = decode(d, emb.data(), 1, S);
    istft(spec.v.data(), 1, spec.h, S * 4 * kHop, audio);
  });
}

// Single-layer hooks for tests against an independent formulation.
// x NHWC (N, H, W, C); weight in the file's canonical layout.
int orc_ss_conv2d(const float* x, int N, int H, int W, int C, const float* w, const float* b, int O, int kh, int kw,
                  int sh, int sw, int causal_pad, float* out) {
  ORC_SS_TRY({
    T4 t(N, H, W, C);
    std::memcpy(t.v.data(), x, t.v.size() * sizeof(float));
    if (causal_pad) t = causal_same_pad(t, kh, kw, sh, sw);
    T4 y = conv2d(t, conv_from_canonical(w, b, O, C, kh, kw), sh, sw);
    std::memcpy(out, y.v.data(), y.v.size() * sizeof(float));
  });
}

int orc_ss_conv_transpose2d(const float* x, int N, int H, int W, int C, const float* w, const float* b, int O, int kh,
                            int kw, int sh, int sw, float* out) {
  ORC_SS_TRY({
    T4 t(N, H, W, C);
    std::memcpy(t.v.data(), x, t.v.size() * sizeof(float));
    T4 y = conv_transpose2d(t, convt_from_canonical(w, b, C, O, kh, kw), sh, sw);
    std::memcpy(out, y.v.data(), y.v.size() * sizeof(float));
  });
}

void orc_ss_set_num_threads(int n) { omp_set_num_threads(n); }

}  // extern "C"
